// Backward tile engines of LUCID attention: two persistent, warp-specialised
// tcgen05 kernels per backward, a column pass and a row pass, with no
// atomics anywhere.
//
// Attention backward (of O = softmax(s Q K^T + causal) X, modeling_lucid.py:505-549)
//   column pass, key block i of kv head hk, tiles = (query head g, block j >= i):
//     S^T = K_i Q_j^T, P = exp2(S^T s log2e - lse_j) (causal),  dP^T = X_i dO_j^T,
//     dS = P (dP^T - delta_j);   dX_i += P dO_j,   dK_i += s dS Q_j
//   row pass, query block j of head hq, tiles = key blocks i <= j:
//     S = Q_j K_i^T, P = exp2(S s log2e - lse), dP = dO_j X_i^T,
//     dS = P (dP - delta);       dQ_j += s dS K_i
//
// Solve backward (of X = P^-1 V, modeling_lucid.py:314-382)
//   column pass = the transposed (back-substitution) solve, a wavefront over
//   column blocks i = NB-1 .. 0 that waits for every dV_j (j > i):
//     E = exp(s K^_i K^_j^T - 1/s),  D = X_i dV_j^T,  dG^T = -s E o D
//     acc_i += E dV_j,  dK^col_i += dG^T K^_j
//     then R = dX_i - acc_i,  dV_i = D_i^-1 (R + U_i^T R)  (published), and the
//     strictly-lower part of the diagonal block: dK^col_i += dG_ii^T K^_i + dG_ii K^_i
//   row pass (after all dV are final), row block j, tiles i < j:
//     E = exp(s K^_j K^_i^T - 1/s),  D = dV_j X_i^T,  dG = -s E o D,  dK^row_j += dG K^_i
//   The diagonal entries P_rr enter exactly in fp32 in the finalize kernel.
//
// Diagonal tiles of the attention (key block i = query block j): P and dS are split
// into bf16 hi + lo parts (lo = bf16(v - hi)) and both enter the GEMMs, so the rows
// whose softmax sits on a few keys (the first rows of a sequence, where P and dS are
// O(1)) do not lose bf16's half-ulp in dX, dK and dQ.  The attention column pass runs
// as two launches of one template: the off-diagonal tiles (j > i), then the diagonal
// tiles (DIAG), which add their hi + lo products to dX / dK; the main launch's code
// carries none of the residual work.  The row passes add the lo tile right after the
// hi tile of the diagonal in both schedules (same order, same results).
//
// Both passes: warps 0-7 are the epilogue (warp w reads TMEM lanes of
// sub-partition w%4 = tile rows 32(w%4).., column half w/4); in the control
// warpgroup warp 8 issues TMA and warp 9 issues tcgen05.mma (registers are
// shifted from the control warpgroup to the epilogue).  P and dS return to tensor memory as packed
// bf16 and feed the next GEMMs as the A operand (TS form); the next tile's
// S / dP GEMMs are issued while the epilogue of the current tile runs.
#include "lucid_common.cuh"

#include <algorithm>

namespace lb {

// Phase bookkeeping for one mbarrier as seen by one role.
struct Ph {
  uint32_t n = 0;
  __device__ __forceinline__ uint32_t full() { return (n++) & 1u; }          // k-th completion
  __device__ __forceinline__ uint32_t empty() { return ((n++) & 1u) ^ 1u; }  // (k-1)-th completion
};

// One arrival per warp, after every lane's preceding stores and fences: a barrier that
// counts warps completes after 16 arrivals instead of one per epilogue thread (the
// arrivals are shared-memory atomics and serialise).
__device__ __forceinline__ void warp_arrive(uint32_t bar) {
  __syncwarp();
  if (lane_id() == 0) mbar_arrive(bar);
}

__device__ __forceinline__ bool warp_wait_b(uint32_t bar, uint32_t parity, const Abort& ab) {
  const bool ok = mbar_wait(bar, parity, ab);
  return __all_sync(0xffffffffu, ok);
}

// bf16 residuals of a pair: (a - bf16(a), b - bf16(b)) packed as bf16.
__device__ __forceinline__ uint32_t pack_bf16_lo(float a, float b) {
  return pack_bf16(a - __bfloat162float(__float2bfloat16_rn(a)), b - __bfloat162float(__float2bfloat16_rn(b)));
}

// Packed bf16 operands written back into a 128-column TMEM region by the
// epilogue.  Warp half h owns columns [64h, 64h+64); its 32-column chunk q
// ([64h+32q, +32)) holds the packed values of tile columns [64h+32q, +32) in
// its first 16 columns and a second operand in the next 16.  Every warp
// writes only columns it has already read, so no cross-warp ordering is
// needed.  K-slice kk (16 tile columns) of the first operand:
__device__ __forceinline__ uint32_t packed_kslice(uint32_t region, int kk) {
  return region + 64u * (uint32_t)(kk >> 2) + 32u * (uint32_t)((kk >> 1) & 1) + 8u * (uint32_t)(kk & 1);
}

// Stored-tile layout (the stored-tile schedule): a packed bf16 dS^T / dG^T tile (rows =
// keys / column block, columns = queries / row block) is 16 "pieces" of 8 columns; piece
// p holds its 8 columns of all 128 rows as 16-byte rows, so element (r, c) sits at
// ((c / 8) * 128 + r) * 8 + c % 8.  The column pass writes it straight from registers:
// for one piece, the 32 threads of a warp (consecutive rows) store 512 contiguous bytes.
// The row pass copies a tile into shared memory unchanged (one bulk copy) and reads it
// as a non-swizzled MN-major operand: 8-row x 16-byte core matrices, 128 bytes apart
// along K (rows), 2048 bytes apart along M (pieces).
constexpr int kPieceElems = 128 * 8;
__device__ __forceinline__ void store_tile_pieces(bf16* tile, int r, int chunk, const uint32_t (&pk)[16]) {
#pragma unroll
  for (int c = 0; c < 4; ++c)
    __stcs(reinterpret_cast<uint4*>(tile + (4 * chunk + c) * kPieceElems + r * 8),
           make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]));
}
__device__ __forceinline__ uint64_t desc_pieces(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)(128u >> 4) << 16;   // leading byte offset: next 8 rows (K)
  d |= (uint64_t)(2048u >> 4) << 32;  // stride byte offset: next piece (M)
  d |= (uint64_t)1u << 46;            // descriptor version; no swizzle
  return d;
}
// D (+)= A B over a 128x128x128 product, A a stored tile in the piece layout (MN-major,
// K-slice kk = rows 16 kk .. 16 kk + 15) and B a swizzled MN-major tile.
__device__ __forceinline__ void umma_tile_pieces(uint32_t d_tmem, uint32_t a_tile, uint32_t b_tile,
                                                 uint32_t accumulate_first) {
  const uint32_t idesc = idesc_bf16(128, 128, true, true);
  const uint64_t a0 = desc_pieces(a_tile), b0 = desc_tile(b_tile, true);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
    umma_ss(d_tmem, a0 + (uint64_t)(kk * 16), desc_slice(b0, true, kk), idesc, (kk > 0) ? 1u : accumulate_first);
}

constexpr int kBwdEpiWarps = 8;
constexpr int kBwdEpiThreads = kBwdEpiWarps * 32;
constexpr int kBwdThreads = kBwdEpiThreads + 128;  // + control warpgroup (TMA, MMA, 2 idle warps)
constexpr int kBwdWarpTma = kBwdEpiWarps, kBwdWarpMma = kBwdEpiWarps + 1;
// register split: 384 x 168 at launch >= 256 x 192 + 128 x 120
constexpr int kBwdRegsEpi = 192, kBwdRegsCtl = 120;

// ===========================================================================
// column pass
// ===========================================================================
namespace bwdc {
constexpr uint32_t kOffA1 = 0, kOffA2 = 32768;
constexpr uint32_t kOffStage = 65536;        // stage s: B1 at +s*65536, B2 at +32768
constexpr uint32_t kOffDS = 196608;          // R / dV / dG^T tile of the diagonal steps
constexpr uint32_t kOffVec = 229376;         // stage s: lse[128], delta[128] at +s*1024
constexpr uint32_t kOffBar = kOffVec + 2048;
enum {
  A_FULL = 0, A_EMPTY, KV_FULL0, KV_FULL1, KV_EMPTY0, KV_EMPTY1, SD_FULL, DP_FULL, PD_FULL, DS_FREE,
  T_FULL, S_FREE, ACC_FULL, ACC2_FULL, ACC_FREE, EPI_DONE, DRAIN, DSP_FULL, NBAR
};
constexpr uint32_t kSmemBytes = kOffBar + NBAR * 8 + 16;
constexpr uint32_t kTmS = 0, kTmDP = 128, kTmAcc1 = 256, kTmAcc2 = 384;
// 16 epilogue warps (four per TMEM sub-partition, one 32-column chunk of the tile
// each) so that every scheduler has four epilogue warps to hide the latencies of the
// TMEM loads, exponentials and stores; warps 16-19: TMA, MMA, two idle.
constexpr int kColEpiWarps = 16, kColQ = 4 * 4 / kColEpiWarps;
constexpr int kColEpiThreads = kColEpiWarps * 32;
constexpr int kColThreads = kColEpiThreads + 128;
constexpr int kColWarpTma = kColEpiWarps, kColWarpMma = kColEpiWarps + 1;
// register split: 640 x 96 at launch >= 512 x 96 + 128 x 88
constexpr int kColRegsEpi = 96, kColRegsCtl = 88;
static_assert(kColEpiThreads * kColRegsEpi + 128 * kColRegsCtl <= kColThreads * (65536 / kColThreads / 8 * 8),
              "register split exceeds the launch allocation");
}  // namespace bwdc

template <bool SOLVE, bool DIAG>
__global__ void __launch_bounds__(bwdc::kColThreads, 1)
    lucid_bwd_col_kernel(const __grid_constant__ CUtensorMap tmA1, const __grid_constant__ CUtensorMap tmA2,
                         const __grid_constant__ CUtensorMap tmB1, const __grid_constant__ CUtensorMap tmB2,
                         const __grid_constant__ CUtensorMap tmU, BwdArgs p) {
  using namespace bwdc;
  static_assert(!(SOLVE && DIAG), "the diagonal launch is the attention's");
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + kOffBar;
  auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffBar + NBAR * 8);
  volatile int* abort_cta = reinterpret_cast<volatile int*>(smem + kOffBar + NBAR * 8 + 4);
  const Abort ab{abort_cta, p.status, SOLVE ? kTagBwdColSolve : kTagBwdColAttn};
  const uint32_t sA1 = sbase + kOffA1, sA2 = sbase + kOffA2, sDS = sbase + kOffDS;
  auto sB1 = [&](int st) { return sbase + kOffStage + (uint32_t)st * 65536u; };
  auto sB2 = [&](int st) { return sbase + kOffStage + (uint32_t)st * 65536u + 32768u; };

  const int warp = warp_id(), lane = lane_id();
  if ((sbase & 1023u) != 0) {  // the tile layout needs a 1024-byte aligned window
    if (threadIdx.x == 0) atomicCAS(p.status, 0, kStatusMisaligned | (ab.tag << 20));
    return;
  }
  if (threadIdx.x == kColWarpTma * 32) {
    mbar_init(bar(A_FULL), 1);
    mbar_init(bar(A_EMPTY), 1);
    for (int s2 = 0; s2 < 2; ++s2) {
      mbar_init(bar(KV_FULL0 + s2), 1);
      mbar_init(bar(KV_EMPTY0 + s2), 1);
    }
    mbar_init(bar(SD_FULL), 1);
    mbar_init(bar(DP_FULL), 1);
    mbar_init(bar(PD_FULL), kColEpiWarps);
    mbar_init(bar(DSP_FULL), kColEpiWarps);
    mbar_init(bar(DS_FREE), 1);
    mbar_init(bar(T_FULL), 1);
    mbar_init(bar(S_FREE), kColEpiWarps);
    mbar_init(bar(ACC_FULL), 1);
    mbar_init(bar(ACC2_FULL), 1);
    mbar_init(bar(ACC_FREE), kColEpiWarps);
    mbar_init(bar(EPI_DONE), kColEpiWarps);
    mbar_init(bar(DRAIN), 1);
    *abort_cta = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA1);
    tma_prefetch_desc(&tmA2);
    tma_prefetch_desc(&tmB1);
    tma_prefetch_desc(&tmB2);
    if (SOLVE) tma_prefetch_desc(&tmU);
  }
  if (warp == kColWarpMma) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int BHk = p.B * p.Hkv;
  const int G = p.Hq / p.Hkv;
  const int blk0 = p.blk0, blk1 = p.blk1 > 0 ? p.blk1 : p.NB, nblk = blk1 - blk0;
  const int total = nblk * BHk;
  // transposed solve: blocks blk1-1 .. blk0 across heads (wavefront order);
  // attention: head-major, longest columns first within a head, so the CTAs in
  // flight share one or two heads whose Q / dO tiles stay resident in L2
  auto decode = [&](int idx, int& i, int& b, int& hk) {
    i = SOLVE ? (blk1 - 1 - idx / BHk) : (blk0 + idx % nblk);
    const int bh = SOLVE ? idx % BHk : idx / nblk;
    b = bh / p.Hkv;
    hk = bh % p.Hkv;
  };
  // attention: the main launch takes the tiles j > i (query head g, block j), the
  // diagonal launch the tiles j = i of each query head of the group
  auto ntiles = [&](int i) { return SOLVE ? (p.NB - 1 - i) : (DIAG ? G : G * (p.NB - 1 - i)); };
  auto tile_at = [&](int i, int t, int& g, int& j) {
    if (SOLVE) {
      g = 0;
      j = p.NB - 1 - t;
    } else if (DIAG) {
      g = t;
      j = i;
    } else {
      const int per = p.NB - 1 - i;
      g = t / per;
      j = i + 1 + t % per;
    }
  };

  if (warp >= kColWarpTma) {
  regs_dec<kColRegsCtl>();
  if (warp == kColWarpTma) {
    // ======================= TMA producer =======================
    if (lane == 0) {
      Ph a_empty;
      uint32_t n_kv = 0, n_a = 0;
      int last_a = -1, last_kv[2] = {-1, -1};
      bool ok = true;
      for (int idx = blockIdx.x; idx < total && ok; idx += gridDim.x) {
        int i, b, hk;
        decode(idx, i, b, hk);
        if (!mbar_wait(bar(A_EMPTY), a_empty.empty(), ab)) break;
        last_a = n_a++ & 1;
        mbar_arrive_expect_tx(bar(A_FULL), 65536);
        tma_load_tile(sA1, &tmA1, bar(A_FULL), i * 128, hk, b);
        tma_load_tile(sA2, &tmA2, bar(A_FULL), i * 128, hk, b);
        const int T = ntiles(i);
        for (int t = 0; t < T + (SOLVE ? 1 : 0); ++t, ++n_kv) {
          const int st = n_kv & 1;
          const uint32_t use = n_kv >> 1;
          if (t < T) {
            int g, j;
            tile_at(i, t, g, j);
            if (SOLVE) {
              if (!wait_flag_geq(&p.flags[(b * p.Hkv + hk) * p.NB + j], 1, ab)) { ok = false; break; }
              fence_proxy_async_global();
            }
            if (!mbar_wait(bar(KV_EMPTY0 + st), (use & 1) ^ 1, ab)) { ok = false; break; }
            last_kv[st] = use & 1;
            if (SOLVE) {
              mbar_arrive_expect_tx(bar(KV_FULL0 + st), 65536);
              tma_load_tile(sB1(st), &tmB1, bar(KV_FULL0 + st), j * 128, hk, b);
              tma_load_tile(sB2(st), &tmB2, bar(KV_FULL0 + st), j * 128, hk, b);
            } else {
              const int hq = hk * G + g;
              const long long voff = ((long long)b * p.Hq + hq) * p.Npad + (long long)j * 128;
              mbar_arrive_expect_tx(bar(KV_FULL0 + st), 65536 + 1024);
              tma_load_tile(sB1(st), &tmB1, bar(KV_FULL0 + st), j * 128, hq, b);
              tma_load_tile(sB2(st), &tmB2, bar(KV_FULL0 + st), j * 128, hq, b);
              bulk_load(sbase + kOffVec + (uint32_t)st * 1024u, p.lse + voff, 512, bar(KV_FULL0 + st));
              bulk_load(sbase + kOffVec + (uint32_t)st * 1024u + 512u, p.delta + voff, 512,
                        bar(KV_FULL0 + st));
            }
          } else {
            // solve: diagonal-block inverse U_i into the stage's B1 slot
            if (!mbar_wait(bar(KV_EMPTY0 + st), (use & 1) ^ 1, ab)) { ok = false; break; }
            last_kv[st] = use & 1;
            mbar_arrive_expect_tx(bar(KV_FULL0 + st), 32768);
            tma_load_tile(sB1(st), &tmU, bar(KV_FULL0 + st), i * 128, hk, b);
          }
        }
      }
      if (last_a >= 0) mbar_wait_timed(bar(A_FULL), (uint32_t)last_a, kDrainNs);
      for (int s2 = 0; s2 < 2; ++s2)
        if (last_kv[s2] >= 0) mbar_wait_timed(bar(KV_FULL0 + s2), (uint32_t)last_kv[s2], kDrainNs);
    }
  } else if (warp == kColWarpMma) {
    // ======================= MMA issuer =======================
    if (lane == 0) {
      Ph a_full, pd_full, dsp_full, acc_free, s_free;
      uint32_t n_kv = 0;
      bool first_item = true;
      const uint32_t tS = tmem + kTmS, tDP = tmem + kTmDP;
      for (int idx = blockIdx.x; idx < total; idx += gridDim.x) {
        int i, b, hk;
        decode(idx, i, b, hk);
        const int T = ntiles(i);
        if (!mbar_wait(bar(A_FULL), a_full.full(), ab)) break;
        // solve: the previous item's diagonal steps read S / dP last
        // (S_FREE completes in D3 and D5 of every solve item; waits consume them in order)
        if (SOLVE && !first_item && !mbar_wait(bar(S_FREE), s_free.full(), ab)) break;
        first_item = false;
        bool ok = true;
        // tile t: S(t) = A1 B1^T (SD_FULL) and dP(t) = A2 B2^T (DP_FULL).  The epilogue
        // packs P(t) into the S region (PD_FULL), then dS(t) into the dP region
        // (DSP_FULL).  acc1 += P B2 and S(t+1) follow P(t); acc2 += dS B1 and dP(t+1)
        // follow dS(t), so the epilogue computes P(t+1) while the tensor core runs
        // acc2(t) and dP(t+1).  A region's next write is issued after the GEMM that
        // reads its packed operand (the MMAs of one issuer run in order) and after the
        // epilogue arrival that ends the epilogue's reads of it.
        if (T > 0) {
          const int st = n_kv & 1;
          if (!mbar_wait(bar(KV_FULL0 + st), (n_kv >> 1) & 1, ab)) break;
          tc_fence_after();
          umma_tile(tS, sA1, false, sB1(st), false, 0u);
          umma_commit(bar(SD_FULL));
          umma_tile(tDP, sA2, false, sB2(st), false, 0u);
          umma_commit(bar(DP_FULL));
        }
        for (int t = 0; t < T; ++t, ++n_kv) {
          const int st = n_kv & 1;
          const int st2 = (n_kv + 1) & 1;
          const bool has_next = t + 1 < T;
          if (!mbar_wait(bar(PD_FULL), pd_full.full(), ab)) { ok = false; break; }
          if (t == 0 && !mbar_wait(bar(ACC_FREE), acc_free.empty(), ab)) { ok = false; break; }
          tc_fence_after();
          const uint32_t acc = t > 0 ? 1u : 0u;
          // acc1 += P B2 (P packed in the S region; diagonal: its lo part too), then S(t+1) over it
          umma_tile_ts(tmem + kTmAcc1, [&](int kk) { return packed_kslice(tS, kk); }, sB2(st), true, acc);
          if constexpr (DIAG)
            umma_tile_ts(tmem + kTmAcc1, [&](int kk) { return packed_kslice(tS, kk) + 16u; }, sB2(st), true, 1u);
          if (has_next) {
            if (!mbar_wait(bar(KV_FULL0 + st2), ((n_kv + 1) >> 1) & 1, ab)) { ok = false; break; }
            tc_fence_after();
            umma_tile(tS, sA1, false, sB1(st2), false, 0u);    // S(t+1)
            umma_commit(bar(SD_FULL));
          }
          // acc2 += dS B1 (dS packed in the dP region), then dP(t+1) over it
          if (!mbar_wait(bar(DSP_FULL), dsp_full.full(), ab)) { ok = false; break; }
          tc_fence_after();
          umma_tile_ts(tmem + kTmAcc2, [&](int kk) { return packed_kslice(tDP, kk); }, sB1(st), true, acc);
          if constexpr (DIAG)
            umma_tile_ts(tmem + kTmAcc2, [&](int kk) { return packed_kslice(tDP, kk) + 16u; }, sB1(st), true, 1u);
          umma_commit(bar(KV_EMPTY0 + st));
          if (has_next) {
            umma_tile(tDP, sA2, false, sB2(st2), false, 0u);  // dP(t+1)
            umma_commit(bar(DP_FULL));
          }
        }
        if (!ok) break;
        // an item without tiles (the last key block of the off-diagonal launch) still
        // takes its turn on the accumulator barriers (the epilogue writes zeros)
        if (!SOLVE && T == 0 && !mbar_wait(bar(ACC_FREE), acc_free.empty(), ab)) break;
        umma_commit(bar(ACC_FULL));
        if (!SOLVE) {
          umma_commit(bar(A_EMPTY));
          continue;
        }
        // ---- diagonal block of the transposed solve ----
        const int st = n_kv & 1;
        const uint32_t use = n_kv >> 1;
        ++n_kv;
        // D2: T' = U^T R   (S region; its last readers were G3/G4 or the previous item)
        if (!mbar_wait(bar(KV_FULL0 + st), use & 1, ab) || !mbar_wait(bar(PD_FULL), pd_full.full(), ab)) break;
        tc_fence_after();
        umma_tile(tS, sB1(st), true, sDS, true, 0u);
        umma_commit(bar(T_FULL));
        umma_commit(bar(DS_FREE));
        umma_commit(bar(KV_EMPTY0 + st));
        // D4: S' = K^_i K^_i^T ; D' = X_i dV_i^T
        // (the last tile's readers of the dP region: the epilogue, done at its DSP_FULL,
        // and acc2, issued earlier)
        if (!mbar_wait(bar(PD_FULL), pd_full.full(), ab) || !mbar_wait(bar(S_FREE), s_free.full(), ab)) break;
        tc_fence_after();
        umma_tile(tS, sA1, false, sA1, false, 0u);
        umma_tile(tDP, sA2, false, sDS, false, 0u);
        umma_commit(bar(SD_FULL));
        umma_commit(bar(DS_FREE));
        // D6: acc2 += dG^T K^_i + dG K^_i
        if (!mbar_wait(bar(PD_FULL), pd_full.full(), ab)) break;
        if (T == 0 && !mbar_wait(bar(ACC_FREE), acc_free.empty(), ab)) break;
        tc_fence_after();
        umma_tile(tmem + kTmAcc2, sDS, false, sA1, true, T > 0 ? 1u : 0u);
        umma_tile(tmem + kTmAcc2, sDS, true, sA1, true, 1u);
        umma_commit(bar(DS_FREE));
        umma_commit(bar(A_EMPTY));
        umma_commit(bar(ACC2_FULL));
      }
      umma_commit(bar(DRAIN));
      mbar_wait_timed(bar(DRAIN), 0, kDrainNs);
    }
  }
  } else {
    regs_inc<kColRegsEpi>();
    // ======================= epilogue warps 0-7 =======================
    // warp w: TMEM lanes of sub-partition w % 4 (tile rows 32 (w % 4) ..) and the
    // kColQ 32-column chunks from chunk ch0 = (w / 4) kColQ
    const int sp = warp & 3, ch0 = (warp >> 2) * kColQ;
    const int r = sp * 32 + lane;
    const uint32_t lane_base = (uint32_t)(sp * 32) << 16;
    const uint32_t c0 = 32u * (uint32_t)ch0;
    const float kLog2e = 1.4426950408889634f;
    const float c1 = p.scale * kLog2e;
    const float c2 = kLog2e / p.scale;
    Ph sd_full, dp_full, ds_free, t_full, acc_full, acc2_full;
    uint32_t n_kv = 0, item = 0;
    // stored-tile schedule: every packed dS^T (attention) / dG^T (solve) tile also goes
    // to global memory, straight from the registers, in the piece layout: attention
    // tile (key block i, query block j >= i) of query head hq at pair j (j + 1) / 2 + i
    // of that head's NB (NB + 1) / 2 + NB tiles (the last NB: the diagonal blocks' lo
    // parts); solve tile (column block i, row block j > i) at j (j - 1) / 2 + i of the
    // head's NB (NB - 1) / 2
    const bool stage = p.store_tiles != 0;
    const long long tiles_per_head = SOLVE ? (long long)p.NB * (p.NB - 1) / 2
                                           : (long long)p.NB * (p.NB + 1) / 2 + p.NB;
    for (int idx = blockIdx.x; idx < total; idx += gridDim.x, ++item) {
      int i, b, hk;
      decode(idx, i, b, hk);
      const int T = ntiles(i);
      const long long bhk = (long long)b * p.Hkv + hk;
      const int row_i = i * 128 + r;
      bool ok = true;
      if (SOLVE) {
        // the diagonal step reads this row's dX (fp32, this warp's 32 columns) on the
        // wavefront's critical path: fetch it into L2 while the column's tiles run
        prefetch_l2(p.dx_in + (bhk * p.Npad + row_i) * kHeadDim + c0);
      }
      for (int t = 0; t < T; ++t, ++n_kv) {
        int g, j;
        tile_at(i, t, g, j);
        const int st = n_kv & 1;
        if (SOLVE && t == T - 1) {
          // the column's tiles ran long enough for other traffic to evict the row's dX
          // and 1 / P_rr from L2: fetch them again while the last tile waits for its dV
          prefetch_l2(p.dx_in + (bhk * p.Npad + row_i) * kHeadDim + c0);
          prefetch_l2(p.dinv + bhk * p.Npad + row_i);
        }
        if (!SOLVE && !warp_wait_b(bar(KV_FULL0 + st), (n_kv >> 1) & 1, ab)) { ok = false; break; }
        if (!warp_wait_b(bar(SD_FULL), sd_full.full(), ab)) { ok = false; break; }
        tc_fence_after();
        // phase 1: P (attention) / E (solve) from S alone, packed into the S region
        float pv[kColQ][32];
#pragma unroll
        for (int q = 0; q < kColQ; ++q) tmem_ld32(tmem + lane_base + kTmS + c0 + 32u * q, pv[q]);
        tmem_ld_wait();
        const float* vec = reinterpret_cast<const float*>(smem + kOffVec + st * 1024);
        const bool full = SOLVE ? ((j + 1) * 128 <= p.N)
                                : (!DIAG && (j + 1) * 128 <= p.N && (i + 1) * 128 <= p.N);
#pragma unroll
        for (int q = 0; q < kColQ; ++q) {
          const int cb = (int)c0 + 32 * q;
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            float4 ls4;
            if (!SOLVE) ls4 = *reinterpret_cast<const float4*>(vec + cb + e);
#pragma unroll
            for (int hh = 0; hh < 4; hh += 2) {
              const int c = cb + e + hh;
              float2 arg, pe;
              if (SOLVE) {
                arg = fma2(make_float2(pv[q][e + hh], pv[q][e + hh + 1]), make_float2(c1, c1), make_float2(-c2, -c2));
                pe = make_float2(fast_exp2(arg.x), fast_exp2(arg.y));
                if (!full) {
                  if (j * 128 + c >= p.N) pe.x = 0.f;
                  if (j * 128 + c + 1 >= p.N) pe.y = 0.f;
                }
              } else {
                const float2 ls = hh == 0 ? make_float2(ls4.x, ls4.y) : make_float2(ls4.z, ls4.w);
                arg = fma2(make_float2(pv[q][e + hh], pv[q][e + hh + 1]), make_float2(c1, c1), make_float2(-ls.x, -ls.y));
                pe = make_float2(fast_exp2(arg.x), fast_exp2(arg.y));
                if (!full) {
                  const int q0 = j * 128 + c;
                  if (!(q0 < p.N && row_i < p.N && q0 >= row_i)) pe.x = 0.f;
                  if (!(q0 + 1 < p.N && row_i < p.N && q0 + 1 >= row_i)) pe.y = 0.f;
                }
              }
              pv[q][e + hh] = pe.x;
              pv[q][e + hh + 1] = pe.y;
              pk[(e + hh) >> 1] = pack_bf16(pe.x, pe.y);
            }
          }
          tmem_st16(tmem + lane_base + kTmS + c0 + 32u * q, pk);
        }
        if constexpr (DIAG) {   // lo part of P into the second-operand columns
#pragma unroll
          for (int q = 0; q < kColQ; ++q) {
            uint32_t pl[16];
#pragma unroll
            for (int e = 0; e < 32; e += 2) pl[e >> 1] = pack_bf16_lo(pv[q][e], pv[q][e + 1]);
            tmem_st16(tmem + lane_base + kTmS + c0 + 32u * q + 16u, pl);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        warp_arrive(bar(PD_FULL));
        // phase 2: dS (attention) / dG^T (solve) from dP and the P kept in registers,
        // packed into the dP region (and staged for the tile store)
        if (!warp_wait_b(bar(DP_FULL), dp_full.full(), ab)) { ok = false; break; }
        tc_fence_after();
        float dv[kColQ][32];
#pragma unroll
        for (int q = 0; q < kColQ; ++q) tmem_ld32(tmem + lane_base + kTmDP + c0 + 32u * q, dv[q]);
        tmem_ld_wait();
        bf16* tile_out = nullptr;
        if (stage) {
          const long long head = SOLVE ? (long long)b * p.Hkv + hk : (long long)b * p.Hq + hk * G + g;
          const long long pair = SOLVE ? (long long)j * (j - 1) / 2 + i : (long long)j * (j + 1) / 2 + i;
          tile_out = p.tiles + (head * tiles_per_head + pair) * (long long)kTileBytes / 2;
        }
#pragma unroll
        for (int q = 0; q < kColQ; ++q) {
          const int cb = (int)c0 + 32 * q;
          uint32_t dk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            float4 dl4;
            if (!SOLVE) dl4 = *reinterpret_cast<const float4*>(vec + 128 + cb + e);
#pragma unroll
            for (int hh = 0; hh < 4; hh += 2) {
              const float2 pe = make_float2(pv[q][e + hh], pv[q][e + hh + 1]);
              float2 ds;
              if (SOLVE) {
                ds = mul2(pe, mul2(make_float2(dv[q][e + hh], dv[q][e + hh + 1]), make_float2(-p.scale, -p.scale)));
              } else {
                const float2 dl = hh == 0 ? make_float2(dl4.x, dl4.y) : make_float2(dl4.z, dl4.w);
                ds = mul2(pe, add2(make_float2(dv[q][e + hh], dv[q][e + hh + 1]), make_float2(-dl.x, -dl.y)));
              }
              dk[(e + hh) >> 1] = pack_bf16(ds.x, ds.y);
            }
          }
          tmem_st16(tmem + lane_base + kTmDP + c0 + 32u * q, dk);
          if (stage) store_tile_pieces(tile_out, r, ch0 + q, dk);
        }
        if constexpr (DIAG) {
          // lo part of dS: into the dP region's second-operand columns and, in the
          // stored-tile schedule, straight to its residual tile (row r of key block i)
          bf16* lo_tile = stage ? tile_out + ((long long)p.NB * (p.NB + 1) / 2 + i - ((long long)j * (j + 1) / 2 + i)) *
                                                (long long)kTileBytes / 2
                                : nullptr;
#pragma unroll
          for (int q = 0; q < kColQ; ++q) {
            const int cb = (int)c0 + 32 * q;
            uint32_t dl[16];
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              const float2 ds = mul2(make_float2(pv[q][e], pv[q][e + 1]),
                                     add2(make_float2(dv[q][e], dv[q][e + 1]),
                                          make_float2(-vec[128 + cb + e], -vec[128 + cb + e + 1])));
              dl[e >> 1] = pack_bf16_lo(ds.x, ds.y);
            }
            tmem_st16(tmem + lane_base + kTmDP + c0 + 32u * q + 16u, dl);
            if (stage) store_tile_pieces(lo_tile, r, ch0 + q, dl);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        warp_arrive(bar(DSP_FULL));
      }
      if (!ok) break;
      // solve: the diagonal step's dX row (this warp's columns) and 1 / P_rr, loaded while
      // the last tile's GEMMs finish (they sit on the wavefront's critical path)
      float dxv[kColQ][32];
      float di = 0.f;
      if constexpr (SOLVE) {
        const float4* dx4 = reinterpret_cast<const float4*>(p.dx_in + (bhk * p.Npad + row_i) * kHeadDim + c0);
#pragma unroll
        for (int q = 0; q < kColQ; ++q)
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const float4 x4 = dx4[q * 8 + c];
            dxv[q][4 * c] = x4.x;
            dxv[q][4 * c + 1] = x4.y;
            dxv[q][4 * c + 2] = x4.z;
            dxv[q][4 * c + 3] = x4.w;
          }
        di = p.dinv[bhk * p.Npad + row_i];
      }
      if (!warp_wait_b(bar(ACC_FULL), acc_full.full(), ab)) break;
      tc_fence_after();
      if (!SOLVE) {
        // dX_i, s dK_i: stored by the off-diagonal launch (zeros for an item without
        // tiles), added to by the diagonal launch, which runs after it
        float* dxr = p.dx + (bhk * p.Npad + row_i) * kHeadDim + c0;
        float* dkr = p.dk_col + (bhk * p.Npad + row_i) * kHeadDim + c0;
#pragma unroll
        for (int q = 0; q < kColQ; ++q) {
          float a1[32], a2[32];
          if (T > 0) {
            tmem_ld32(tmem + lane_base + kTmAcc1 + c0 + 32u * q, a1);
            tmem_ld32(tmem + lane_base + kTmAcc2 + c0 + 32u * q, a2);
            tmem_ld_wait();
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) a1[e] = a2[e] = 0.f;
          }
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            float4 x4 = make_float4(a1[4 * c], a1[4 * c + 1], a1[4 * c + 2], a1[4 * c + 3]);
            float4 k4 = make_float4(a2[4 * c] * p.scale, a2[4 * c + 1] * p.scale, a2[4 * c + 2] * p.scale,
                                    a2[4 * c + 3] * p.scale);
            if constexpr (DIAG) {
              const float4 ox = reinterpret_cast<const float4*>(dxr)[q * 8 + c];
              const float4 ok4 = reinterpret_cast<const float4*>(dkr)[q * 8 + c];
              x4 = make_float4(ox.x + x4.x, ox.y + x4.y, ox.z + x4.z, ox.w + x4.w);
              k4 = make_float4(ok4.x + k4.x, ok4.y + k4.y, ok4.z + k4.z, ok4.w + k4.w);
            }
            reinterpret_cast<float4*>(dxr)[q * 8 + c] = x4;
            reinterpret_cast<float4*>(dkr)[q * 8 + c] = k4;
          }
        }
        tc_fence_before();
        warp_arrive(bar(ACC_FREE));
        continue;
      }
      ++n_kv;  // the U_i load
      // ---------------- solve: diagonal block ----------------
      // D1: R = dX_i - acc1 (this warp's column half), staged as bf16 for U^T R
      float (&rr)[kColQ][32] = dxv;
#pragma unroll
      for (int q = 0; q < kColQ; ++q) {
        if (T > 0) {
          float a1[32];
          tmem_ld32(tmem + lane_base + kTmAcc1 + c0 + 32u * q, a1);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) rr[q][e] -= a1[e];
        }
      }
      if (!warp_wait_b(bar(DS_FREE), ds_free.empty(), ab)) break;
#pragma unroll
      for (int q = 0; q < kColQ; ++q) tile_store_row32(sDS, r, ch0 + q, rr[q]);
      fence_proxy_async_smem();
      tc_fence_before();
      warp_arrive(bar(PD_FULL));
      // D3: dV_i = D^-1 (R + U^T R) -> global bf16 and the smem tile; publish
      if (!warp_wait_b(bar(T_FULL), t_full.full(), ab) || !warp_wait_b(bar(DS_FREE), ds_free.empty(), ab))
        break;
      tc_fence_after();
      bf16* dvr = p.dv + (bhk * p.Npad + row_i) * kHeadDim + c0;
#pragma unroll
      for (int q = 0; q < kColQ; ++q) {
        float tv[32];
        tmem_ld32(tmem + lane_base + kTmS + c0 + 32u * q, tv);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) tv[e] = (rr[q][e] + tv[e]) * di;
#pragma unroll
        for (int c = 0; c < 4; ++c) st_bf16x8(dvr + q * 32 + c * 8, tv + c * 8);
        tile_store_row32(sDS, r, ch0 + q, tv);
      }
      tc_fence_before();
      warp_arrive(bar(S_FREE));
      fence_proxy_async_smem();
      warp_arrive(bar(PD_FULL));
      // (the readers fence the async proxy after acquiring the flag, before their TMA loads)
      warp_arrive(bar(EPI_DONE));
      if (threadIdx.x == 0) {   // publish: the CTA's dV rows, then the flag (one fence, cumulative)
        if (mbar_wait(bar(EPI_DONE), item & 1, ab)) {
          __threadfence();
          st_release_gpu(&p.flags[bhk * p.NB + i], 1);
        }
      }
      __syncwarp();
      // D5: dG^T of the strictly-lower part of P_ii -> smem tile
      if (!warp_wait_b(bar(SD_FULL), sd_full.full(), ab) || !warp_wait_b(bar(DS_FREE), ds_free.empty(), ab))
        break;
      tc_fence_after();
#pragma unroll
      for (int q = 0; q < kColQ; ++q) {
        float sv[32], dv[32];
        tmem_ld32(tmem + lane_base + kTmS + c0 + 32u * q, sv);
        tmem_ld32(tmem + lane_base + kTmDP + c0 + 32u * q, dv);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int c = (int)c0 + 32 * q + e;
          const bool valid = (c > r) && (i * 128 + c < p.N);
          sv[e] = valid ? -p.scale * fast_exp2(fmaf(sv[e], c1, -c2)) * dv[e] : 0.f;
        }
        tile_store_row32(sDS, r, ch0 + q, sv);
      }
      tc_fence_before();
      warp_arrive(bar(S_FREE));
      fence_proxy_async_smem();
      warp_arrive(bar(PD_FULL));
      // D7: column part of dK^_i
      if (!warp_wait_b(bar(ACC2_FULL), acc2_full.full(), ab)) break;
      tc_fence_after();
      float* dkr = p.dk_col + (bhk * p.Npad + row_i) * kHeadDim + c0;
#pragma unroll
      for (int q = 0; q < kColQ; ++q) {
        float a2[32];
        tmem_ld32(tmem + lane_base + kTmAcc2 + c0 + 32u * q, a2);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 8; ++c)
          reinterpret_cast<float4*>(dkr)[q * 8 + c] =
              make_float4(a2[4 * c], a2[4 * c + 1], a2[4 * c + 2], a2[4 * c + 3]);
      }
      tc_fence_before();
      warp_arrive(bar(ACC_FREE));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kColWarpMma) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ===========================================================================
// row pass
// ===========================================================================
namespace bwdr {
constexpr uint32_t kOffA1 = 0, kOffA2 = 32768;
constexpr uint32_t kOffK = 65536;             // 3-deep ring of B1 tiles (K / K^)
constexpr uint32_t kOffX = kOffK + 3 * 32768;  // 2-deep ring of B2 tiles (X)
constexpr uint32_t kOffBar = kOffX + 2 * 32768;
enum { A_FULL = 0, A_EMPTY, K_FULL0, K_EMPTY0 = K_FULL0 + 3, X_FULL0 = K_EMPTY0 + 3, X_EMPTY0 = X_FULL0 + 2,
       SD_FULL = X_EMPTY0 + 2, DP_READ, PD_FULL, ACC_FULL, ACC_FREE, DRAIN, NBAR };
constexpr uint32_t kSmemBytes = kOffBar + NBAR * 8 + 16;
constexpr uint32_t kTmS0 = 0, kTmS1 = 128, kTmDP = 256, kTmAcc = 384;
}  // namespace bwdr

template <bool SOLVE>
__global__ void __launch_bounds__(kBwdThreads, 1)
    lucid_bwd_row_kernel(const __grid_constant__ CUtensorMap tmA1, const __grid_constant__ CUtensorMap tmA2,
                         const __grid_constant__ CUtensorMap tmB1, const __grid_constant__ CUtensorMap tmB2,
                         BwdArgs p) {
  using namespace bwdr;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + kOffBar;
  auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffBar + NBAR * 8);
  volatile int* abort_cta = reinterpret_cast<volatile int*>(smem + kOffBar + NBAR * 8 + 4);
  const Abort ab{abort_cta, p.status, SOLVE ? kTagBwdRowSolve : kTagBwdRowAttn};
  const uint32_t sA1 = sbase + kOffA1, sA2 = sbase + kOffA2;
  auto sK = [&](uint32_t idx) { return sbase + kOffK + (idx % 3u) * 32768u; };
  auto sX = [&](uint32_t idx) { return sbase + kOffX + (idx & 1u) * 32768u; };

  const int warp = warp_id(), lane = lane_id();
  if ((sbase & 1023u) != 0) {
    if (threadIdx.x == 0) atomicCAS(p.status, 0, kStatusMisaligned | (ab.tag << 20));
    return;
  }
  if (threadIdx.x == kBwdWarpTma * 32) {
    mbar_init(bar(A_FULL), 1);
    mbar_init(bar(A_EMPTY), 1);
    for (int s2 = 0; s2 < 3; ++s2) {
      mbar_init(bar(K_FULL0 + s2), 1);
      mbar_init(bar(K_EMPTY0 + s2), 1);
    }
    for (int s2 = 0; s2 < 2; ++s2) {
      mbar_init(bar(X_FULL0 + s2), 1);
      mbar_init(bar(X_EMPTY0 + s2), 1);
    }
    mbar_init(bar(SD_FULL), 1);
    mbar_init(bar(DP_READ), kBwdEpiWarps);
    mbar_init(bar(PD_FULL), kBwdEpiWarps);
    mbar_init(bar(ACC_FULL), 1);
    mbar_init(bar(ACC_FREE), kBwdEpiWarps);
    mbar_init(bar(DRAIN), 1);
    *abort_cta = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA1);
    tma_prefetch_desc(&tmA2);
    tma_prefetch_desc(&tmB1);
    tma_prefetch_desc(&tmB2);
  }
  if (warp == kBwdWarpMma) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // items: (row block j, head)
  const int BH = SOLVE ? p.B * p.Hkv : p.B * p.Hq;
  const int G = p.Hq / p.Hkv;
  const int blk1 = p.blk1 > 0 ? p.blk1 : p.NB, nblk = blk1 - p.blk0;
  const int total = nblk * BH;
  auto decode = [&](int idx, int& j, int& b, int& ha, int& hk) {
    // head-major, longest rows first within a head (L2 residency of the head's tiles)
    j = blk1 - 1 - idx % nblk;
    const int bh = idx / nblk;
    if (SOLVE) {
      b = bh / p.Hkv;
      hk = bh % p.Hkv;
      ha = hk;
    } else {
      b = bh / p.Hq;
      ha = bh % p.Hq;
      hk = ha / G;
    }
  };
  auto ntiles = [&](int j) { return SOLVE ? j : j + 1; };  // key blocks i < j (solve) / i <= j

  if (warp >= kBwdWarpTma) {
  regs_dec<kBwdRegsCtl>();
  if (warp == kBwdWarpTma) {
    if (lane == 0) {
      Ph a_empty;
      uint32_t kidx = 0, xidx = 0, n_a = 0;
      int last_a = -1, last_k[3] = {-1, -1, -1}, last_x[2] = {-1, -1};
      bool ok = true;
      for (int idx = blockIdx.x; idx < total && ok; idx += gridDim.x) {
        int j, b, ha, hk;
        decode(idx, j, b, ha, hk);
        if (!mbar_wait(bar(A_EMPTY), a_empty.empty(), ab)) break;
        last_a = n_a++ & 1;
        mbar_arrive_expect_tx(bar(A_FULL), 65536);
        tma_load_tile(sA1, &tmA1, bar(A_FULL), j * 128, ha, b);
        tma_load_tile(sA2, &tmA2, bar(A_FULL), j * 128, ha, b);
        const int T = ntiles(j);
        for (int t = 0; t < T; ++t) {
          {
            const uint32_t st = kidx % 3u, use = kidx / 3u;
            if (!mbar_wait(bar(K_EMPTY0 + st), (use & 1) ^ 1, ab)) { ok = false; break; }
            last_k[st] = use & 1;
            mbar_arrive_expect_tx(bar(K_FULL0 + st), 32768);
            tma_load_tile(sK(kidx), &tmB1, bar(K_FULL0 + st), t * 128, hk, b);
            ++kidx;
          }
          {
            const uint32_t st = xidx & 1u, use = xidx >> 1;
            if (!mbar_wait(bar(X_EMPTY0 + st), (use & 1) ^ 1, ab)) { ok = false; break; }
            last_x[st] = use & 1;
            mbar_arrive_expect_tx(bar(X_FULL0 + st), 32768);
            tma_load_tile(sX(xidx), &tmB2, bar(X_FULL0 + st), t * 128, hk, b);
            ++xidx;
          }
        }
      }
      if (last_a >= 0) mbar_wait_timed(bar(A_FULL), (uint32_t)last_a, kDrainNs);
      for (int s2 = 0; s2 < 3; ++s2)
        if (last_k[s2] >= 0) mbar_wait_timed(bar(K_FULL0 + s2), (uint32_t)last_k[s2], kDrainNs);
      for (int s2 = 0; s2 < 2; ++s2)
        if (last_x[s2] >= 0) mbar_wait_timed(bar(X_FULL0 + s2), (uint32_t)last_x[s2], kDrainNs);
    }
  } else if (warp == kBwdWarpMma) {
    if (lane == 0) {
      Ph a_full, dp_read, pd_full, acc_free;
      uint32_t kidx = 0, xidx = 0, n_s = 0;
      bool pending_dp_read = false;
      const uint32_t tDP = tmem + kTmDP;
      auto tS = [&](uint32_t n) { return tmem + ((n & 1) ? kTmS1 : kTmS0); };
      for (int idx = blockIdx.x; idx < total; idx += gridDim.x) {
        int j, b, ha, hk;
        decode(idx, j, b, ha, hk);
        const int T = ntiles(j);
        if (!mbar_wait(bar(A_FULL), a_full.full(), ab)) break;
        bool ok = true;
        for (int t = 0; t <= T; ++t) {
          if (t < T) {
            // S(t) = A1 K_t^T into S[n_s % 2]; dP(t) = A2 X_t^T (after dP(t-1) was read)
            const uint32_t ki = kidx + t, xi = xidx + t;
            if (!mbar_wait(bar(K_FULL0 + ki % 3u), (ki / 3u) & 1, ab) ||
                !mbar_wait(bar(X_FULL0 + (xi & 1u)), (xi >> 1) & 1, ab)) { ok = false; break; }
            if (pending_dp_read && !mbar_wait(bar(DP_READ), dp_read.full(), ab)) { ok = false; break; }
            tc_fence_after();
            umma_tile(tS(n_s + t), sA1, false, sK(ki), false, 0u);
            umma_tile(tDP, sA2, false, sX(xi), false, 0u);
            umma_commit(bar(SD_FULL));
            umma_commit(bar(X_EMPTY0 + (xi & 1u)));
            pending_dp_read = true;
          }
          if (t >= 1) {
            // acc += dS(t-1) K_{t-1}, dS packed in S[(n_s + t - 1) % 2]
            const int tt = t - 1;
            const uint32_t ki = kidx + tt;
            if (!mbar_wait(bar(PD_FULL), pd_full.full(), ab)) { ok = false; break; }
            if (tt == 0 && !mbar_wait(bar(ACC_FREE), acc_free.empty(), ab)) { ok = false; break; }
            tc_fence_after();
            const uint32_t sreg = tS(n_s + tt);
            umma_tile_ts(tmem + kTmAcc, [&](int kk) { return packed_kslice(sreg, kk); }, sK(ki), true,
                         tt > 0 ? 1u : 0u);
            if (!SOLVE && tt == T - 1)   // diagonal tile: the lo part of dS
              umma_tile_ts(tmem + kTmAcc, [&](int kk) { return packed_kslice(sreg, kk) + 16u; }, sK(ki), true, 1u);
            umma_commit(bar(K_EMPTY0 + ki % 3u));
          }
        }
        if (!ok) break;
        kidx += T;
        xidx += T;
        n_s += T;
        if (T == 0 && !mbar_wait(bar(ACC_FREE), acc_free.empty(), ab)) break;
        umma_commit(bar(ACC_FULL));
        umma_commit(bar(A_EMPTY));
      }
      umma_commit(bar(DRAIN));
      mbar_wait_timed(bar(DRAIN), 0, kDrainNs);
    }
  }
  } else {
    regs_inc<kBwdRegsEpi>();
    const int sp = warp & 3, h = warp >> 2;
    const int r = sp * 32 + lane;
    const uint32_t lane_base = (uint32_t)(sp * 32) << 16;
    const uint32_t c0 = 64u * (uint32_t)h;
    const float kLog2e = 1.4426950408889634f;
    const float c1 = p.scale * kLog2e;
    const float c2 = kLog2e / p.scale;
    Ph sd_full, acc_full;
    uint32_t n_s = 0;
    for (int idx = blockIdx.x; idx < total; idx += gridDim.x) {
      int j, b, ha, hk;
      decode(idx, j, b, ha, hk);
      const int T = ntiles(j);
      const int row = j * 128 + r;
      const long long bha = (long long)b * (SOLVE ? p.Hkv : p.Hq) + ha;
      float lse_r = 0.f, dl_r = 0.f;
      if (!SOLVE) {
        lse_r = p.lse[bha * p.Npad + row];
        dl_r = p.delta[bha * p.Npad + row];
      }
      bool ok = true;
      for (int t = 0; t < T; ++t, ++n_s) {
        const int i = t;  // key block
        if (!warp_wait_b(bar(SD_FULL), sd_full.full(), ab)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sreg = tmem + lane_base + ((n_s & 1) ? kTmS1 : kTmS0);
        float dv[2][32], svv[2][32];
        tmem_ld32(tmem + lane_base + kTmDP + c0, dv[0]);
        tmem_ld32(tmem + lane_base + kTmDP + c0 + 32u, dv[1]);
        tmem_ld32(sreg + c0, svv[0]);
        tmem_ld32(sreg + c0 + 32u, svv[1]);
        tmem_ld_wait();
        tc_fence_before();
        warp_arrive(bar(DP_READ));
        const bool full = SOLVE ? true : (i < j && (j + 1) * 128 <= p.N);
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const float (&sv)[32] = svv[q];
          const int cb = (int)c0 + 32 * q;
          uint32_t dk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            float2 ds;
            if (SOLVE) {
              const float2 arg = fma2(make_float2(sv[e], sv[e + 1]), make_float2(c1, c1), make_float2(-c2, -c2));
              const float2 pe = make_float2(fast_exp2(arg.x), fast_exp2(arg.y));
              ds = mul2(pe, mul2(make_float2(dv[q][e], dv[q][e + 1]), make_float2(-p.scale, -p.scale)));
            } else {
              const float2 arg =
                  fma2(make_float2(sv[e], sv[e + 1]), make_float2(c1, c1), make_float2(-lse_r, -lse_r));
              float2 pe = make_float2(fast_exp2(arg.x), fast_exp2(arg.y));
              if (!full) {
                const int k0 = i * 128 + cb + e;  // key index
                if (!(k0 <= row && k0 < p.N && row < p.N)) pe.x = 0.f;
                if (!(k0 + 1 <= row && k0 + 1 < p.N && row < p.N)) pe.y = 0.f;
              }
              ds = mul2(pe, add2(make_float2(dv[q][e], dv[q][e + 1]), make_float2(-dl_r, -dl_r)));
            }
            dk[e >> 1] = pack_bf16(ds.x, ds.y);
          }
          tmem_st16(sreg + c0 + 32u * q, dk);
        }
        if (!SOLVE && i == j) {
          // diagonal tile: the lo part of dS into the second-operand columns
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const float (&sv)[32] = svv[q];
            const int cb = (int)c0 + 32 * q;
            uint32_t dl[16];
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              const float2 arg = fma2(make_float2(sv[e], sv[e + 1]), make_float2(c1, c1), make_float2(-lse_r, -lse_r));
              float2 pe = make_float2(fast_exp2(arg.x), fast_exp2(arg.y));
              const int k0 = i * 128 + cb + e;
              if (!(k0 <= row && k0 < p.N && row < p.N)) pe.x = 0.f;
              if (!(k0 + 1 <= row && k0 + 1 < p.N && row < p.N)) pe.y = 0.f;
              const float2 ds = mul2(pe, add2(make_float2(dv[q][e], dv[q][e + 1]), make_float2(-dl_r, -dl_r)));
              dl[e >> 1] = pack_bf16_lo(ds.x, ds.y);
            }
            tmem_st16(sreg + c0 + 32u * q + 16u, dl);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        warp_arrive(bar(PD_FULL));
      }
      if (!ok) break;
      if (!warp_wait_b(bar(ACC_FULL), acc_full.full(), ab)) break;
      tc_fence_after();
      float av[2][32];
      if (T > 0) {
        tmem_ld32(tmem + lane_base + kTmAcc + c0, av[0]);
        tmem_ld32(tmem + lane_base + kTmAcc + c0 + 32u, av[1]);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int q = 0; q < 2; ++q)
#pragma unroll
          for (int e = 0; e < 32; ++e) av[q][e] = 0.f;
      }
      tc_fence_before();
      warp_arrive(bar(ACC_FREE));
      if (SOLVE) {
        float* dst = p.dk_row + (bha * p.Npad + row) * kHeadDim + c0;
#pragma unroll
        for (int q = 0; q < 2; ++q)
#pragma unroll
          for (int c = 0; c < 8; ++c)
            reinterpret_cast<float4*>(dst)[q * 8 + c] =
                make_float4(av[q][4 * c], av[q][4 * c + 1], av[q][4 * c + 2], av[q][4 * c + 3]);
      } else if (row < p.N) {
        bf16* dst = p.dq + (long long)b * p.dq_sb + (long long)ha * p.dq_sh + (long long)row * p.dq_sn + c0;
#pragma unroll
        for (int q = 0; q < 2; ++q) {
#pragma unroll
          for (int e = 0; e < 32; ++e) av[q][e] *= p.scale;
#pragma unroll
          for (int c = 0; c < 4; ++c) st_bf16x8(dst + q * 32 + c * 8, av[q] + c * 8);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kBwdWarpMma) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ===========================================================================
// row pass, stored-tile schedule
// ===========================================================================
// The column pass stored every packed dS^T (attention) / dG^T (solve) tile, tile
// (key block i, row block j) at pair index j (j + 1) / 2 + i (attention, i <= j)
// or j (j - 1) / 2 + i (solve, i < j).  The row pass is then a streamed GEMM:
//   dQ_j = s sum_{i <= j} (dS^T_ij)^T K_i        dK^row_j = sum_{i < j} (dG^T_ij)^T K^_i
// with the stored tile as the MN-major A operand, in the same key-block order
// (and so with the same fp32 accumulation order) as the recomputing row pass.
// Warps 0-3 epilogue (TMEM lane = tile row), warp 4 TMA, warp 5 MMA; three
// stages of (stored tile, K tile), accumulator double-buffered in TMEM.
namespace bwds {
constexpr int kStages = 3;
constexpr int kThreads = 192;
constexpr uint32_t kOffBar = kStages * 65536u;
enum { FULL0 = 0, EMPTY0 = FULL0 + kStages, ACC_FULL0 = EMPTY0 + kStages, ACC_FREE0 = ACC_FULL0 + 2,
       DRAIN = ACC_FREE0 + 2, NBAR };
constexpr uint32_t kSmemBytes = kOffBar + NBAR * 8 + 16;
}  // namespace bwds

template <bool SOLVE>
__global__ void __launch_bounds__(bwds::kThreads, 1)
    lucid_bwd_row_stored_kernel(const __grid_constant__ CUtensorMap tmB, BwdArgs p) {
  using namespace bwds;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + kOffBar;
  auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffBar + NBAR * 8);
  volatile int* abort_cta = reinterpret_cast<volatile int*>(smem + kOffBar + NBAR * 8 + 4);
  const Abort ab{abort_cta, p.status, kTagBwdRowStored};
  auto sT = [&](uint32_t n) { return sbase + (n % kStages) * 65536u; };
  auto sB = [&](uint32_t n) { return sbase + (n % kStages) * 65536u + 32768u; };
  const int warp = warp_id(), lane = lane_id();
  if ((sbase & 1023u) != 0) {
    if (threadIdx.x == 0) atomicCAS(p.status, 0, kStatusMisaligned | (kTagBwdRowStored << 20));
    return;
  }
  if (threadIdx.x == 128) {
    for (int s2 = 0; s2 < kStages; ++s2) {
      mbar_init(bar(FULL0 + s2), 1);
      mbar_init(bar(EMPTY0 + s2), 1);
    }
    for (int a2 = 0; a2 < 2; ++a2) {
      mbar_init(bar(ACC_FULL0 + a2), 1);
      mbar_init(bar(ACC_FREE0 + a2), 4);  // one arrival per warp
    }
    mbar_init(bar(DRAIN), 1);
    *abort_cta = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmB);
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(tmem_slot), 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int BH = SOLVE ? p.B * p.Hkv : p.B * p.Hq;
  const int G = p.Hq / p.Hkv;
  const int blk1 = p.blk1 > 0 ? p.blk1 : p.NB, nblk = blk1 - p.blk0;
  const int total = nblk * BH;
  auto decode = [&](int idx, int& j, int& b, int& ha, int& hk) {
    j = blk1 - 1 - idx % nblk;   // head-major, longest rows first (as the recomputing row pass)
    const int bh = idx / nblk;
    b = bh / (SOLVE ? p.Hkv : p.Hq);
    ha = bh % (SOLVE ? p.Hkv : p.Hq);
    hk = SOLVE ? ha : ha / G;
  };
  // attention: the dS^T tiles of key blocks 0..j, then the residual (lo) tile of the
  // diagonal block j, stored after all pair tiles at index NB (NB + 1) / 2 + j
  auto ntiles = [&](int j) { return SOLVE ? j : j + 2; };
  auto pair0 = [&](int j) { return SOLVE ? j * (j - 1) / 2 : j * (j + 1) / 2; };
  auto tile_idx = [&](int j, int t) { return (SOLVE || t <= j) ? pair0(j) + t : p.NB * (p.NB + 1) / 2 + j; };
  auto key_blk = [&](int j, int t) { return (SOLVE || t <= j) ? t : j; };
  const long long tiles_per_head = SOLVE ? (long long)p.NB * (p.NB - 1) / 2 : (long long)p.NB * (p.NB + 1) / 2 + p.NB;
  auto bha_of = [&](int b, int ha) { return (long long)b * (SOLVE ? p.Hkv : p.Hq) + ha; };

  if (warp == 4) {
    // ======================= TMA producer =======================
    if (lane == 0) {
      uint32_t n = 0;
      int last[kStages];
      for (int s2 = 0; s2 < kStages; ++s2) last[s2] = -1;
      bool ok = true;
      for (int idx = blockIdx.x; idx < total && ok; idx += gridDim.x) {
        int j, b, ha, hk;
        decode(idx, j, b, ha, hk);
        const int T = ntiles(j);
        for (int t = 0; t < T; ++t, ++n) {
          const uint32_t st = n % kStages, use = n / kStages;
          if (!mbar_wait(bar(EMPTY0 + st), (use & 1) ^ 1, ab)) { ok = false; break; }
          last[st] = use & 1;
          mbar_arrive_expect_tx(bar(FULL0 + st), 65536);
          bulk_load(sT(n), p.tiles + (bha_of(b, ha) * tiles_per_head + tile_idx(j, t)) * (long long)kTileBytes / 2,
                    (uint32_t)kTileBytes, bar(FULL0 + st));
          tma_load_tile(sB(n), &tmB, bar(FULL0 + st), key_blk(j, t) * 128, hk, b);
        }
      }
      for (int s2 = 0; s2 < kStages; ++s2)
        if (last[s2] >= 0) mbar_wait_timed(bar(FULL0 + s2), (uint32_t)last[s2], kDrainNs);
    }
  } else if (warp == 5) {
    // ======================= MMA issuer =======================
    if (lane == 0) {
      uint32_t n = 0, item = 0;
      for (int idx = blockIdx.x; idx < total; idx += gridDim.x, ++item) {
        int j, b, ha, hk;
        decode(idx, j, b, ha, hk);
        const int T = ntiles(j);
        const uint32_t ab2 = item & 1u, use2 = item >> 1;
        if (!mbar_wait(bar(ACC_FREE0 + ab2), (use2 & 1) ^ 1, ab)) break;
        tc_fence_after();
        bool ok = true;
        for (int t = 0; t < T; ++t, ++n) {
          const uint32_t st = n % kStages;
          if (!mbar_wait(bar(FULL0 + st), (n / kStages) & 1, ab)) { ok = false; break; }
          tc_fence_after();
          umma_tile_pieces(tmem + 128u * ab2, sT(n), sB(n), t > 0 ? 1u : 0u);
          umma_commit(bar(EMPTY0 + st));
        }
        if (!ok) break;
        umma_commit(bar(ACC_FULL0 + ab2));
      }
      umma_commit(bar(DRAIN));
      mbar_wait_timed(bar(DRAIN), 0, kDrainNs);
    }
  } else {
    // ======================= epilogue warps 0-3 =======================
    const int r = warp * 32 + lane;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    uint32_t item = 0;
    for (int idx = blockIdx.x; idx < total; idx += gridDim.x, ++item) {
      int j, b, ha, hk;
      decode(idx, j, b, ha, hk);
      const int T = ntiles(j);
      const uint32_t ab2 = item & 1u, use2 = item >> 1;
      if (!warp_wait_b(bar(ACC_FULL0 + ab2), use2 & 1, ab)) break;
      tc_fence_after();
      const int row = j * 128 + r;
      const long long bha = (long long)b * (SOLVE ? p.Hkv : p.Hq) + ha;
#pragma unroll 1
      for (int q = 0; q < 4; ++q) {
        float av[32];
        if (T > 0) {
          tmem_ld32(tmem + 128u * ab2 + lane_base + 32u * (uint32_t)q, av);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) av[e] = 0.f;
        }
        if (SOLVE) {
          float* dst = p.dk_row + (bha * p.Npad + row) * kHeadDim + 32 * q;
#pragma unroll
          for (int c = 0; c < 8; ++c)
            reinterpret_cast<float4*>(dst)[c] = make_float4(av[4 * c], av[4 * c + 1], av[4 * c + 2], av[4 * c + 3]);
        } else if (row < p.N) {
          bf16* dst = p.dq + (long long)b * p.dq_sb + (long long)ha * p.dq_sh + (long long)row * p.dq_sn + 32 * q;
#pragma unroll
          for (int e = 0; e < 32; ++e) av[e] *= p.scale;
#pragma unroll
          for (int c = 0; c < 4; ++c) st_bf16x8(dst + c * 8, av + c * 8);
        }
      }
      tc_fence_before();
      warp_arrive(bar(ACC_FREE0 + ab2));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// --------------------------------------------------------------------------
// elementwise helpers of the backward
// --------------------------------------------------------------------------

// delta[bhq][row] = sum_d dO[row][d] * O[row][d]  (zero on padding rows); with the forward's
// rounding residual o_res (O's strides, nullable) O is taken as o + o_res
__global__ void lucid_delta_kernel(int B, int Hq, int N, int Npad, const bf16* o, long long o_sb,
                                   long long o_sh, long long o_sn, const bf16* dout, long long d_sb,
                                   long long d_sh, long long d_sn, const bf16* o_res, float* delta,
                                   int row0, int nrows) {
  const int warps = blockDim.x >> 5;
  const long long gw = (long long)blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const long long total = (long long)B * Hq * nrows;
  if (gw >= total) return;
  const int row = row0 + (int)(gw % nrows);
  const long long bh = gw / nrows;
  const int b = (int)(bh / Hq), h = (int)(bh % Hq);
  float acc = 0.f;
  if (row < N) {
    float a[4], c[4];
    const bf16* op = o + b * o_sb + h * o_sh + row * o_sn + lane * 4;
    const bf16* dp = dout + b * d_sb + h * d_sh + row * d_sn + lane * 4;
    const uint2 ua = *reinterpret_cast<const uint2*>(op);
    const uint2 uc = *reinterpret_cast<const uint2*>(dp);
    const __nv_bfloat162* ha = reinterpret_cast<const __nv_bfloat162*>(&ua);
    const __nv_bfloat162* hc = reinterpret_cast<const __nv_bfloat162*>(&uc);
    float2 f;
    f = __bfloat1622float2(ha[0]); a[0] = f.x; a[1] = f.y;
    f = __bfloat1622float2(ha[1]); a[2] = f.x; a[3] = f.y;
    f = __bfloat1622float2(hc[0]); c[0] = f.x; c[1] = f.y;
    f = __bfloat1622float2(hc[1]); c[2] = f.x; c[3] = f.y;
    if (o_res) {
      const uint2 ur = *reinterpret_cast<const uint2*>(o_res + (op - o));
      const __nv_bfloat162* hr = reinterpret_cast<const __nv_bfloat162*>(&ur);
      f = __bfloat1622float2(hr[0]); a[0] += f.x; a[1] += f.y;
      f = __bfloat1622float2(hr[1]); a[2] += f.x; a[3] += f.y;
    }
    acc = a[0] * c[0] + a[1] * c[1] + a[2] * c[2] + a[3] * c[3];
  }
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, s);
  if (lane == 0) delta[bh * Npad + row] = acc;
}

// Solve backward finalize, one warp per row (row < N):
//   dk^  = dk_col + dk_row + 2 dG_rr k^_r,  dG_rr = -s P_rr (dV_r . X_r)
//   dK   = rstd (dk^ - (k^.dk^ / D) k^) + dk_add        (RMSNorm backward; D the logical head dim)
//   dV   = copy of the internal bf16 dV
__global__ void lucid_solve_finalize_kernel(int B, int H, int N, int Npad, float s, const bf16* k,
                                            long long k_sb, long long k_sh, long long k_sn,
                                            const float* rstd, const float* dinv, const bf16* x,
                                            const bf16* dv_int, const float* dk_col,
                                            const float* dk_row, const float* dk_add, bf16* dk,
                                            long long dk_sb, long long dk_sh, long long dk_sn, bf16* dv,
                                            long long dv_sb, long long dv_sh, long long dv_sn, int row0,
                                            int nrows, float inv_d) {
  const int warps = blockDim.x >> 5;
  const long long gw = (long long)blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const long long total = (long long)B * H * nrows;
  if (gw >= total) return;
  const int row = row0 + (int)(gw % nrows);
  const long long bh = gw / nrows;
  const int b = (int)(bh / H), h = (int)(bh % H);
  const long long ir = bh * Npad + row;  // internal row
  const int d0 = lane * 4;
  auto ld4 = [](const bf16* ptr, float* out) {
    const uint2 u = *reinterpret_cast<const uint2*>(ptr);
    const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&u);
    const float2 f0 = __bfloat1622float2(hh[0]), f1 = __bfloat1622float2(hh[1]);
    out[0] = f0.x; out[1] = f0.y; out[2] = f1.x; out[3] = f1.y;
  };
  float kr[4], xv[4], dvv[4];
  ld4(k + b * k_sb + h * k_sh + row * k_sn + d0, kr);
  ld4(x + ir * kHeadDim + d0, xv);
  ld4(dv_int + ir * kHeadDim + d0, dvv);
  const float rs = rstd[ir];
  const float4 c4 = *reinterpret_cast<const float4*>(dk_col + ir * kHeadDim + d0);
  const float4 w4 = *reinterpret_cast<const float4*>(dk_row + ir * kHeadDim + d0);
  float dot = dvv[0] * xv[0] + dvv[1] * xv[1] + dvv[2] * xv[2] + dvv[3] * xv[3];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
  const float prr = 1.0f / dinv[ir];
  const float dgrr = -s * prr * dot;
  float kh[4], g[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) kh[e] = kr[e] * rs;
  g[0] = c4.x + w4.x + 2.f * dgrr * kh[0];
  g[1] = c4.y + w4.y + 2.f * dgrr * kh[1];
  g[2] = c4.z + w4.z + 2.f * dgrr * kh[2];
  g[3] = c4.w + w4.w + 2.f * dgrr * kh[3];
  float proj = kh[0] * g[0] + kh[1] * g[1] + kh[2] * g[2] + kh[3] * g[3];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) proj += __shfl_xor_sync(0xffffffffu, proj, o);
  proj *= inv_d;
  float outk[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) outk[e] = rs * (g[e] - proj * kh[e]);
  if (dk_add) {
    const float4 a4 = *reinterpret_cast<const float4*>(dk_add + ir * kHeadDim + d0);
    outk[0] += a4.x; outk[1] += a4.y; outk[2] += a4.z; outk[3] += a4.w;
  }
  uint2 ko;
  ko.x = pack_bf16(outk[0], outk[1]);
  ko.y = pack_bf16(outk[2], outk[3]);
  *reinterpret_cast<uint2*>(dk + b * dk_sb + h * dk_sh + row * dk_sn + d0) = ko;
  uint2 vo;
  vo.x = pack_bf16(dvv[0], dvv[1]);
  vo.y = pack_bf16(dvv[2], dvv[3]);
  *reinterpret_cast<uint2*>(dv + b * dv_sb + h * dv_sh + row * dv_sn + d0) = vo;
}

// --------------------------------------------------------------------------
// host launchers
// --------------------------------------------------------------------------
static int bwd_num_sms() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

template <typename K>
static cudaError_t set_smem(K kernel, uint32_t bytes) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

cudaError_t launch_bwd_col(bool solve, const CUtensorMap& tA1, const CUtensorMap& tA2, const CUtensorMap& tB1,
                           const CUtensorMap& tB2, const CUtensorMap& tU, const BwdArgs& a,
                           cudaStream_t st) {
  const int nblk = (a.blk1 > 0 ? a.blk1 : a.NB) - a.blk0;
  const int total = nblk * a.B * a.Hkv;
  if (total <= 0) return cudaSuccess;
  const int grid = std::min(total, a.max_ctas > 0 ? std::min(a.max_ctas, bwd_num_sms()) : bwd_num_sms());
  cudaError_t e;
  if (solve) {
    if ((e = set_smem(lucid_bwd_col_kernel<true, false>, bwdc::kSmemBytes)) != cudaSuccess) return e;
    // the transposed solve's CTAs wait on one another's flags: all of them must be resident
    return launch_cooperative(lucid_bwd_col_kernel<true, false>, grid, bwdc::kColThreads, bwdc::kSmemBytes, st, tA1,
                              tA2, tB1, tB2, tU, a);
  } else {
    // off-diagonal tiles, then the diagonal tiles (which add to dX, dK)
    if ((e = set_smem(lucid_bwd_col_kernel<false, false>, bwdc::kSmemBytes)) != cudaSuccess) return e;
    lucid_bwd_col_kernel<false, false><<<grid, bwdc::kColThreads, bwdc::kSmemBytes, st>>>(tA1, tA2, tB1, tB2, tU, a);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if ((e = set_smem(lucid_bwd_col_kernel<false, true>, bwdc::kSmemBytes)) != cudaSuccess) return e;
    lucid_bwd_col_kernel<false, true><<<grid, bwdc::kColThreads, bwdc::kSmemBytes, st>>>(tA1, tA2, tB1, tB2, tU, a);
  }
  return cudaGetLastError();
}

cudaError_t launch_bwd_row(bool solve, const CUtensorMap& tA1, const CUtensorMap& tA2, const CUtensorMap& tB1,
                           const CUtensorMap& tB2, const BwdArgs& a, cudaStream_t st) {
  const int nblk = (a.blk1 > 0 ? a.blk1 : a.NB) - a.blk0;
  const int total = nblk * a.B * (solve ? a.Hkv : a.Hq);
  if (total <= 0) return cudaSuccess;
  const int grid = std::min(total, a.max_ctas > 0 ? std::min(a.max_ctas, bwd_num_sms()) : bwd_num_sms());
  cudaError_t e;
  if (solve) {
    if ((e = set_smem(lucid_bwd_row_kernel<true>, bwdr::kSmemBytes)) != cudaSuccess) return e;
    lucid_bwd_row_kernel<true><<<grid, kBwdThreads, bwdr::kSmemBytes, st>>>(tA1, tA2, tB1, tB2, a);
  } else {
    if ((e = set_smem(lucid_bwd_row_kernel<false>, bwdr::kSmemBytes)) != cudaSuccess) return e;
    lucid_bwd_row_kernel<false><<<grid, kBwdThreads, bwdr::kSmemBytes, st>>>(tA1, tA2, tB1, tB2, a);
  }
  return cudaGetLastError();
}

// Row pass of the stored-tile schedule: tT = the stored tiles, tB = K (attention) / K^ (solve).
cudaError_t launch_bwd_row_stored(bool solve, const CUtensorMap& tB, const BwdArgs& a,
                                  cudaStream_t st) {
  const int nblk = (a.blk1 > 0 ? a.blk1 : a.NB) - a.blk0;
  const int total = nblk * a.B * (solve ? a.Hkv : a.Hq);
  if (total <= 0) return cudaSuccess;
  const int grid = std::min(total, a.max_ctas > 0 ? std::min(a.max_ctas, bwd_num_sms()) : bwd_num_sms());
  cudaError_t e;
  if (solve) {
    if ((e = set_smem(lucid_bwd_row_stored_kernel<true>, bwds::kSmemBytes)) != cudaSuccess) return e;
    lucid_bwd_row_stored_kernel<true><<<grid, bwds::kThreads, bwds::kSmemBytes, st>>>(tB, a);
  } else {
    if ((e = set_smem(lucid_bwd_row_stored_kernel<false>, bwds::kSmemBytes)) != cudaSuccess) return e;
    lucid_bwd_row_stored_kernel<false><<<grid, bwds::kThreads, bwds::kSmemBytes, st>>>(tB, a);
  }
  return cudaGetLastError();
}

cudaError_t launch_delta(int B, int Hq, int N, int Npad, const bf16* o, long long o_sb, long long o_sh,
                         long long o_sn, const bf16* dout, long long d_sb, long long d_sh,
                         long long d_sn, const bf16* o_res, float* delta, cudaStream_t st, int row0,
                         int row1) {
  if (row1 < 0) row1 = Npad;
  const long long warps = (long long)B * Hq * (row1 - row0);
  if (warps <= 0) return cudaSuccess;
  const int blocks = (int)((warps + 7) / 8);
  lucid_delta_kernel<<<blocks, 256, 0, st>>>(B, Hq, N, Npad, o, o_sb, o_sh, o_sn, dout, d_sb, d_sh,
                                             d_sn, o_res, delta, row0, row1 - row0);
  return cudaGetLastError();
}

cudaError_t launch_solve_finalize(int B, int H, int N, int Npad, float s, const bf16* k, long long k_sb,
                                  long long k_sh, long long k_sn, const float* rstd, const float* dinv,
                                  const bf16* x, const bf16* dv_int, const float* dk_col,
                                  const float* dk_row, const float* dk_add, bf16* dk, long long dk_sb,
                                  long long dk_sh, long long dk_sn, bf16* dv, long long dv_sb,
                                  long long dv_sh, long long dv_sn, cudaStream_t st, int row0, int row1,
                                  int D) {
  if (row1 < 0) row1 = N;
  const long long warps = (long long)B * H * (row1 - row0);
  if (warps <= 0) return cudaSuccess;
  const int blocks = (int)((warps + 7) / 8);
  lucid_solve_finalize_kernel<<<blocks, 256, 0, st>>>(B, H, N, Npad, s, k, k_sb, k_sh, k_sn, rstd, dinv,
                                                      x, dv_int, dk_col, dk_row, dk_add, dk, dk_sb,
                                                      dk_sh, dk_sn, dv, dv_sb, dv_sh, dv_sn, row0,
                                                      row1 - row0, 1.0f / (float)D);
  return cudaGetLastError();
}

}  // namespace lb
