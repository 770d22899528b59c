// Forward tile engine: one persistent, warp-specialised tcgen05 kernel
// template that runs the two causal row-block loops of the LUCID forward.
//
//   SOLVE  (modeling_lucid.py:566-570, and the blockwise form :285-302)
//     X = P^-1 V,  P = tril(exp(s K^K^T - 1/s))
//     Row block i:  R_i = V_i - sum_{j<i} exp(s K^_i K^_j^T - 1/s) X_j
//                   Y   = D_i^-1 R_i ;  X_i = Y + U_i Y
//     Blocks are processed as a wavefront: a work item waits on a global flag
//     for every X_j it consumes and publishes its own X_i.
//
//     Chain schedule (few heads per GPU): the chain X_0 -> X_1 -> ... of one head
//     is its critical path, and in the wavefront every step crosses CTAs (publish,
//     poll, reload X through L2).  Here CTA c < nchain owns the diagonal steps of
//     head c and keeps the X tiles it produces in shared memory (L = kChainLook):
//       X_i = Y + U_i Y,  Y = D_i^-1 (W_i - sum_{j=i-L}^{i-1} E_ij X_j)
//     while the other CTAs (workers) stream row-block pairs and publish, per row
//     block, the tiles E_{i,i-L} .. E_{i,i-1} first and the partial sum
//     W_i = V_i - sum_{j < i-L} E_ij X_j when its last X_j has arrived.  A chain
//     step is L + 1 GEMMs and two epilogues on one SM, and only one GEMM of it
//     waits for the previous step.
//
//   ATTN   (modeling_lucid.py:505-549)
//     O = softmax(scale Q K^T + causal) X   (raw K, X from SOLVE), keeping the
//     row log-sum-exp for the backward.  Grouped-query heads index kv head =
//     q head / (Hq / Hkv)  (repeat_kv, modeling_lucid.py:523-524).
//
//   FUSED  (the layer's forward, modeling_lucid.py:463 then :489): the chain
//     schedule's solve and the attention in one launch.  The workers take the
//     attention row-block pairs after their solve items, in increasing pair order,
//     and wait per tile for the X block's flag, so the attention of early rows runs
//     while the chains still produce later X blocks.
//
// A work item is a PAIR of consecutive row blocks (i0 = 2p, i1 = 2p+1) of one
// head: both rows share every K / X tile load, which halves the L2->SM
// traffic per FLOP.  Warp roles (320 threads): warpgroup 0 (warps 0-3) owns
// row block 0 and warpgroup 1 (warps 4-7) row block 1, one TMEM lane = one
// row per thread; in warpgroup 2, warp 8 issues TMA and warp 9 issues
// tcgen05.mma (registers are shifted to the epilogue warpgroups).  TMEM:
// S0 [0,128), S1 [128,256), O0 [256,384), O1 [384,512).  Per tile j:
//   S_k = A_k B_j^T  ->  P_k = f(S_k) written back over S_k as packed bf16
//   O_k += P_k C_j   (A operand from tensor memory)
// issued in the order PV0(j), S0(j+1), PV1(j), S1(j+1) so that each
// warpgroup's epilogue overlaps the other row's GEMMs.
#include "lucid_common.cuh"

#include <algorithm>
#include <cstdlib>
#include <cstring>

namespace lb {

namespace fwd {
constexpr int kEpiThreads = 256;
constexpr int kThreads = kEpiThreads + 128;  // + one warpgroup: TMA warp, MMA warp, 2 idle warps
constexpr int kWarpTma = 8, kWarpMma = 9;
// register split: 384 threads x 168 at launch >= 2 x 128 x 208 + 128 x 88
constexpr int kRegsEpi = 208, kRegsCtl = 88;
constexpr uint32_t kOffQ = 0;                 // row block k: A operand (Q / K^) or Y, at +k*32 KB
constexpr uint32_t kOffK = 65536;             // 3 stages of B tiles (K / K^ / U)
constexpr uint32_t kOffX = kOffK + 3 * 32768; // 2 stages of C tiles (X)
constexpr uint32_t kOffBar = kOffX + 2 * 32768;
enum {
  Q_FULL = 0, Q_EMPTY, K_FULL0, K_EMPTY0 = K_FULL0 + 3, X_FULL0 = K_EMPTY0 + 3, X_EMPTY0 = X_FULL0 + 2,
  S_FULL0 = X_EMPTY0 + 2, P_FULL0 = S_FULL0 + 2, O_DONE0 = P_FULL0 + 2, O_FREE0 = O_DONE0 + 2,
  Y_FULL0 = O_FREE0 + 2, EPI_DONE0 = Y_FULL0 + 2, DRAIN = EPI_DONE0 + 2, NBAR
};
constexpr uint32_t kSmemBytes = kOffBar + NBAR * 8 + 16;
constexpr uint32_t kTmS0 = 0, kTmO0 = 256;
}  // namespace fwd

// One arrival per warp, after every lane's preceding stores and fences: the epilogue
// barriers count warps (the arrivals are shared-memory atomics and serialise).
__device__ __forceinline__ void warp_arrive(uint32_t bar) {
  __syncwarp();
  if (lane_id() == 0) mbar_arrive(bar);
}

__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, const Abort& ab) {
  const bool ok = mbar_wait(bar, parity, ab);
  return __all_sync(0xffffffffu, ok);
}

// ---------------------------------------------------------------------------
// Chain CTA of the chain schedule: the diagonal steps of head blockIdx.x.
//   acc_i = sum_{e < kChainLook} E_{i,i-kChainLook+e} X_{i-kChainLook+e}
//   Y_i   = D_i^-1 (W_i - acc_i),  X_i = Y_i + U_i Y_i
// Shared memory: E ring (kChainLook tiles) | X ring (kChainLook tiles; Y_i is staged
// in the slot X_i will take, that of X_{i-kChainLook}) | U (one tile).  TMEM: two
// 128-column accumulators (step parity); the accumulator of step i holds acc_i,
// then T_i = U_i Y_i.  Warps 0-7: epilogue (warp w: rows 32 (w % 4).., columns
// 64 (w / 4)..), warp 8: E loads, warp 9: MMA, warp 10: publishes X flags, warp 11:
// U loads.
// ---------------------------------------------------------------------------
namespace chain {
constexpr uint32_t kOffE = 0, kOffX = kChainLook * 32768, kOffU = 2 * kChainLook * 32768;
static_assert(kOffU + 32768 <= fwd::kOffBar, "chain tiles exceed the engine's tile area");
constexpr int kEpiRing = kChainLook + 1;  // publisher barriers (see the publisher)
enum { EFULL0 = 0, EEMPTY0 = kChainLook, UFULL = 2 * kChainLook, UEMPTY, ACC, YF, TF, XR, EPI0,
       DRAIN = EPI0 + kEpiRing, NBAR };
static_assert((int)NBAR <= (int)fwd::NBAR, "chain barriers exceed the engine's barrier area");
constexpr int kEpiThreads = 256;
}  // namespace chain

__device__ __forceinline__ void solve_chain_cta(const CUtensorMap* tmU, const FwdArgs& p, uint8_t* smem) {
  using namespace chain;
  constexpr int L = kChainLook;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + fwd::kOffBar;
  auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + fwd::kOffBar + fwd::NBAR * 8);
  volatile int* abort_cta = reinterpret_cast<volatile int*>(smem + fwd::kOffBar + fwd::NBAR * 8 + 4);
  const Abort ab{abort_cta, p.status, kTagFwdSolve};
  auto sE = [&](uint32_t s) { return sbase + kOffE + s * 32768u; };
  auto sX = [&](int j) { return sbase + kOffX + (uint32_t)(j % L) * 32768u; };  // slot of block j
  const uint32_t sU = sbase + kOffU;
  const int warp = warp_id(), lane = lane_id();
  if (threadIdx.x == fwd::kWarpTma * 32) {
    for (int s = 0; s < L; ++s) {
      mbar_init(bar(EFULL0 + s), 1);
      mbar_init(bar(EEMPTY0 + s), 1);
    }
    mbar_init(bar(UFULL), 1);
    mbar_init(bar(UEMPTY), 1);
    mbar_init(bar(ACC), 1);
    mbar_init(bar(YF), kEpiThreads / 32);
    mbar_init(bar(TF), 1);
    mbar_init(bar(XR), kEpiThreads / 32);
    for (int s = 0; s < kEpiRing; ++s) mbar_init(bar(EPI0 + s), kEpiThreads / 32);
    mbar_init(bar(DRAIN), 1);
    *abort_cta = 0;
    fence_mbar_init();
    tma_prefetch_desc(tmU);
  }
  if (warp == fwd::kWarpMma) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int NB = p.NB;
  const long long bhk = blockIdx.x;
  const int b = (int)bhk / p.Hkv, hk = (int)bhk % p.Hkv;
  const int* cflag = p.cflags + bhk * NB;
  int* xflag = p.flags + bhk * NB;

  if (warp >= fwd::kWarpTma) {
    regs_dec<fwd::kRegsCtl>();
    if (warp == fwd::kWarpTma && lane == 0) {
      // ---- E loads: the tiles of row block i by bulk copy once the worker flagged them
      // (tile e of row i: key block i - L + e), each as soon as its slot is free
      const bf16* et = p.etiles + bhk * NB * L * (long long)(kTileBytes / 2);
      uint32_t e_idx = 0;
      int last_e[L];
      for (int s = 0; s < L; ++s) last_e[s] = -1;
      for (int i = 1; i < NB; ++i) {
        if (!wait_flag_geq(&cflag[i], 1, ab)) break;
        fence_proxy_async_global();
        bool ok = true;
        for (int e = (i >= L ? 0 : L - i); e < L; ++e) {
          const uint32_t se = e_idx % L, euse = e_idx / L;
          if (!mbar_wait(bar(EEMPTY0 + se), (euse & 1) ^ 1, ab)) { ok = false; break; }
          last_e[se] = (int)(euse & 1);
          mbar_arrive_expect_tx(bar(EFULL0 + se), 32768);
          bulk_load(sE(se), et + ((long long)i * L + e) * (kTileBytes / 2), 32768, bar(EFULL0 + se));
          ++e_idx;
        }
        if (!ok) break;
      }
      for (int s = 0; s < L; ++s)
        if (last_e[s] >= 0) mbar_wait_timed(bar(EFULL0 + s), (uint32_t)last_e[s], kDrainNs);
    } else if (warp == fwd::kWarpMma + 2 && lane == 0) {
      // ---- U loads (own thread, so that a U slot still in use never holds back an E load)
      int last_u = -1;
      for (int i = 0; i < NB; ++i) {
        if (!mbar_wait(bar(UEMPTY), ((uint32_t)i & 1) ^ 1, ab)) break;
        last_u = i & 1;
        mbar_arrive_expect_tx(bar(UFULL), 32768);
        tma_load_tile(sU, tmU, bar(UFULL), i * 128, hk, b);
      }
      if (last_u >= 0) mbar_wait_timed(bar(UFULL), (uint32_t)last_u, kDrainNs);
    } else if (warp == fwd::kWarpMma && lane == 0) {
      // ---- MMA.  Step i: acc_i = sum_e E_{i,j} X_j (j = i-L+e), then T_i = U_i Y_i over
      // it.  Only the last product (e = L-1, X_{i-1}) waits for the epilogue; the
      // lookahead products of step i+1 (e < L-1) are issued around T_i (one before it
      // when its tile is already loaded, the rest after), so that the tensor core runs
      // them while the epilogue works on step i.
      uint32_t e_idx = 0;  // next E tile (the loads run in the same order)
      auto e_first = [&](int i) { return i >= L ? 0 : L - i; };
      auto issue_e = [&](int i, int e) -> bool {
        const uint32_t se = e_idx % L;
        if (!mbar_wait(bar(EFULL0 + se), (e_idx / L) & 1, ab)) return false;
        if (e == L - 1 && !mbar_wait(bar(XR), (uint32_t)(i - 1) & 1, ab)) return false;
        tc_fence_after();
        umma_tile(tmem + 128u * (uint32_t)(i & 1), sE(se), false, sX(i - L + e), true, e > e_first(i) ? 1u : 0u);
        umma_commit(bar(EEMPTY0 + se));
        ++e_idx;
        return true;
      };
      int e_next = L - 1;  // first lookahead product of the current step still to issue
      for (int i = 0; i < NB; ++i) {
        bool ok = true;
        for (int e = e_next; e < L - 1 && ok; ++e) ok = issue_e(i, e);
        if (ok && i >= 1) ok = issue_e(i, L - 1);
        if (!ok) break;
        umma_commit(bar(ACC));
        e_next = i + 1 < NB ? e_first(i + 1) : L - 1;
        if (e_next < L - 1 && mbar_try_wait(bar(EFULL0 + e_idx % L), (e_idx / L) & 1)) {
          if (!issue_e(i + 1, e_next)) break;
          ++e_next;
        }
        if (!mbar_wait(bar(UFULL), (uint32_t)i & 1, ab) || !mbar_wait(bar(YF), (uint32_t)i & 1, ab)) break;
        tc_fence_after();
        umma_tile(tmem + 128u * (uint32_t)(i & 1), sU, false, sX(i), true, 0u);
        umma_commit(bar(TF));
        umma_commit(bar(UEMPTY));
      }
      umma_commit(bar(DRAIN));
      mbar_wait_timed(bar(DRAIN), 0, kDrainNs);
    } else if (warp == fwd::kWarpMma + 1 && lane == 0) {
      // ---- publisher: X_i rows are in global memory -> release the flag.  The
      // epilogue can finish steps i+1 .. i+L before this thread sees step i (W_{i+L+1}
      // waits for X_i), never step i+L+1: kEpiRing = L+1 barriers in rotation keep
      // every wait unambiguous.
      for (int i = 0; i < NB; ++i) {
        if (!mbar_wait(bar(EPI0 + i % kEpiRing), ((uint32_t)(i / kEpiRing)) & 1, ab)) break;
        __threadfence();
        st_release_gpu(&xflag[i], 1);
      }
    }
  } else {
    regs_inc<fwd::kRegsEpi>();
    // ---- epilogue: thread = (row r, column half h)
    const int sp = warp & 3, h = warp >> 2;
    const int r = sp * 32 + lane;
    const uint32_t lane_base = (uint32_t)(sp * 32) << 16;
    const float* wslots = p.wring + bhk * kChainWRing * (long long)(kBlock * kHeadDim);
    for (int i = 0; i < NB; ++i) {
      const int row = i * 128 + r;
      // W_i (fp32, this thread's 64 columns): chunk c4 of row r at (c4 * 128 + r) * 4,
      // read through L2 (the slot is rewritten every kChainWRing steps by other CTAs)
      bool ok = true;
      if (lane == 0) ok = wait_flag_geq(&cflag[i], 2, ab);
      if (!__all_sync(0xffffffffu, __shfl_sync(0xffffffffu, (int)ok, 0) != 0)) break;
      __syncwarp();  // the lanes' loads below are ordered after lane 0's acquire of the flag
      const float4* ws = reinterpret_cast<const float4*>(wslots + (long long)(i % kChainWRing) * (kBlock * kHeadDim));
      float y[2][32];
#pragma unroll
      for (int q = 0; q < 2; ++q)
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const float4 w4 = __ldcg(ws + (16 * h + 8 * q + m) * 128 + r);
          y[q][4 * m] = w4.x;
          y[q][4 * m + 1] = w4.y;
          y[q][4 * m + 2] = w4.z;
          y[q][4 * m + 3] = w4.w;
        }
      const float di = p.dinv[bhk * p.Npad + row];
      const uint32_t tacc = tmem + lane_base + 128u * (uint32_t)(i & 1) + 64u * (uint32_t)h;
      if (!warp_wait(bar(ACC), (uint32_t)i & 1, ab)) break;
      tc_fence_after();
      if (i > 0) {
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          float a[32];
          tmem_ld32(tacc + 32u * q, a);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) y[q][e] -= a[e];
        }
      }
#pragma unroll
      for (int q = 0; q < 2; ++q) {
#pragma unroll
        for (int e = 0; e < 32; ++e) y[q][e] *= di;
        tile_store_row32(sX(i), r, 2 * h + q, y[q]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      warp_arrive(bar(YF));
      // X_i = Y + U_i Y: into the slot (operand of steps i+1 .. i+L) and to global memory
      if (!warp_wait(bar(TF), (uint32_t)i & 1, ab)) break;
      tc_fence_after();
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        float t[32];
        tmem_ld32(tacc + 32u * q, t);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) y[q][e] += t[e];
        tile_store_row32(sX(i), r, 2 * h + q, y[q]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      warp_arrive(bar(XR));
      bf16* xrow = p.x + (bhk * p.Npad + row) * kHeadDim + 64 * h;
#pragma unroll
      for (int q = 0; q < 2; ++q)
#pragma unroll
        for (int c = 0; c < 4; ++c) st_bf16x8(xrow + q * 32 + c * 8, y[q] + c * 8);
      fence_proxy_async_global();
      warp_arrive(bar(EPI0 + i % kEpiRing));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == fwd::kWarpMma) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Tensor maps: solve items read their rows' normalised keys through tmA, the key tiles
// through tmB, X through tmC and the diagonal-block inverses through tmU; attention
// items read Q through tmQ, the raw keys through tmK and X through tmC.
template <int MODE>
__global__ void __launch_bounds__(fwd::kThreads, 1)
    lucid_fwd_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmU,
                     const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     FwdArgs p) {
  using namespace fwd;
  // MODE 0: attention; 1: solve, wavefront schedule; 2: solve, chain schedule;
  // 3: chain-schedule solve, then attention (fused)
  constexpr bool SOLVE = MODE != 0;              // the launch has solve items
  constexpr bool CHAIN = MODE == 2 || MODE == 3;
  constexpr bool FUSED = MODE == 3;
  constexpr bool ATTN = MODE == 0 || FUSED;      // the launch has attention items
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + kOffBar;
  auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffBar + NBAR * 8);
  volatile int* abort_cta = reinterpret_cast<volatile int*>(smem + kOffBar + NBAR * 8 + 4);
  const Abort ab{abort_cta, p.status, SOLVE ? kTagFwdSolve : kTagFwdAttn};
  auto sQ = [&](int k) { return sbase + kOffQ + (uint32_t)k * 32768u; };
  auto sK = [&](uint32_t idx) { return sbase + kOffK + (idx % 3u) * 32768u; };
  auto sX = [&](uint32_t idx) { return sbase + kOffX + (idx & 1u) * 32768u; };

  const int warp = warp_id(), lane = lane_id();
  if ((sbase & 1023u) != 0) {
    if (threadIdx.x == 0) atomicCAS(p.status, 0, kStatusMisaligned | (ab.tag << 20));
    return;
  }
  if constexpr (CHAIN) {
    if ((int)blockIdx.x < p.nchain) {
      solve_chain_cta(&tmU, p, smem);
      return;
    }
  }
  // this CTA's share of the work items (chain schedule: the CTAs after the chains)
  const int cta0 = CHAIN ? (int)blockIdx.x - p.nchain : (int)blockIdx.x;
  const int ncta = CHAIN ? (int)gridDim.x - p.nchain : (int)gridDim.x;
  if (threadIdx.x == kWarpTma * 32) {
    mbar_init(bar(Q_FULL), 1);
    mbar_init(bar(Q_EMPTY), 1);
    for (int s2 = 0; s2 < 3; ++s2) {
      mbar_init(bar(K_FULL0 + s2), 1);
      mbar_init(bar(K_EMPTY0 + s2), 1);
    }
    for (int s2 = 0; s2 < 2; ++s2) {
      mbar_init(bar(X_FULL0 + s2), 1);
      mbar_init(bar(X_EMPTY0 + s2), 1);
      mbar_init(bar(S_FULL0 + s2), 1);
      mbar_init(bar(P_FULL0 + s2), 4);  // one arrival per warp of the warpgroup
      mbar_init(bar(O_DONE0 + s2), 1);
      mbar_init(bar(O_FREE0 + s2), 4);  // one arrival per warp of the warpgroup
      mbar_init(bar(Y_FULL0 + s2), 4);  // one arrival per warp of the warpgroup
      mbar_init(bar(EPI_DONE0 + s2), 4);  // one arrival per warp of the warpgroup
    }
    mbar_init(bar(DRAIN), 1);
    *abort_cta = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
    if (SOLVE) tma_prefetch_desc(&tmU);
    if (ATTN) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
    }
  }
  if (warp == kWarpMma) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int BHk = p.B * p.Hkv, BHq = p.B * p.Hq;
  const int G = p.Hq / p.Hkv;
  const int NP = (p.NB + 1) / 2;
  const int NPe = p.pp1 > 0 ? p.pp1 : NP;  // one past the last pair processed
  const int n_solve = SOLVE ? (NPe - p.pp0) * BHk : 0;
  const int total = n_solve + (ATTN ? (NPe - p.pp0) * BHq : 0);
  // Fused item order: the solve items of pairs 0 .. lag-1, then per pair p >= lag the
  // solve items of pair p followed by the attention items of pair p - lag, then the
  // attention items of the last lag pairs.  Every item depends only on items before
  // it in this order (attention pair q reads X up to block 2q+1, which the chains
  // produce from the solve items of pairs <= q), and every CTA takes its items in
  // this order, so the earliest unfinished item can always progress.
  const int lag = FUSED ? (p.fuse_lag < NP ? p.fuse_lag : NP) : 0;
  const int mid = (NP - lag) * (BHk + BHq);
  // -> (solve item?, pair, (batch, head) index)
  auto locate = [&](int idx, bool& sv, int& pp, int& bh) {
    if (!FUSED) {
      sv = SOLVE;
      pp = SOLVE ? p.pp0 + idx / BHk : NPe - 1 - idx / BHq;  // solve: wavefront order; attention: longest first
      bh = SOLVE ? idx % BHk : idx % BHq;
      return;
    }
    int r = idx;
    if (r < lag * BHk) {
      sv = true; pp = r / BHk; bh = r % BHk;
      return;
    }
    r -= lag * BHk;
    if (r < mid) {
      const int blk = r / (BHk + BHq), off = r % (BHk + BHq);
      sv = off < BHk;
      pp = sv ? lag + blk : blk;
      bh = sv ? off : off - BHk;
      return;
    }
    r -= mid;
    sv = false; pp = NP - lag + r / BHq; bh = r % BHq;
  };
  auto is_solve = [&](int idx) {
    bool sv; int pp, bh;
    locate(idx, sv, pp, bh);
    return sv;
  };

  // Work item -> (pair pp, batch b, A-operand head ha, kv head hk).
  auto decode = [&](int idx, int& pp, int& b, int& ha, int& hk) {
    bool sv; int bh;
    locate(idx, sv, pp, bh);
    if (sv) {
      b = bh / p.Hkv;
      hk = bh % p.Hkv;
      ha = hk;
    } else {
      b = bh / p.Hq;
      ha = bh % p.Hq;
      hk = ha / G;
    }
  };
  // Streaming tiles of row k: attention row block i has tiles j = 0..i;
  // the solve streams the shared tiles j < 2pp (row 1's tile 2pp is part of
  // its tail).
  // Chain schedule: row block i = 2pp + k streams the tiles j < i - kChainLook (its
  // chain multiplies the blocks i - kChainLook .. i - 1).
  auto nrow = [&](int pp, int k, bool sv) -> int {
    const bool r1 = (2 * pp + 1) < p.NB;
    if (k == 1 && !r1) return 0;
    if (!sv) return 2 * pp + 1 + k;
    if (CHAIN) return 2 * pp - kChainLook + k > 0 ? 2 * pp - kChainLook + k : 0;
    return 2 * pp;
  };
  // Chain schedule: the E tiles of both rows come from the key blocks
  // j = 2pp - kChainLook + e (e = 0 .. kChainLook); row k uses them as its tile e - k.
  auto etile_used = [&](int pp, int e, int k) -> bool {
    const int j = 2 * pp - kChainLook + e, s2 = e - k;
    return j >= 0 && s2 >= 0 && s2 < kChainLook && (k == 0 || 2 * pp + 1 < p.NB);
  };

  if (warp >= kWarpTma) {
  regs_dec<kRegsCtl>();
  if (warp == kWarpTma) {
    // ======================= TMA producer =======================
    if (lane == 0) {
      uint32_t kidx = 0, xidx = 0, item = 0;
      int last_q = -1, last_k[3] = {-1, -1, -1}, last_x[2] = {-1, -1};
      bool ok = true;
      auto loadK = [&](const CUtensorMap* m, int row, int h2, int b2) -> bool {
        const uint32_t st = kidx % 3u, use = kidx / 3u;
        if (!mbar_wait(bar(K_EMPTY0 + st), (use & 1) ^ 1, ab)) return false;
        last_k[st] = use & 1;
        mbar_arrive_expect_tx(bar(K_FULL0 + st), 32768);
        tma_load_tile(sK(kidx), m, bar(K_FULL0 + st), row, h2, b2);
        ++kidx;
        return true;
      };
      auto loadX = [&](int row, int h2, int b2) -> bool {
        const uint32_t st = xidx & 1u, use = xidx >> 1;
        if (!mbar_wait(bar(X_EMPTY0 + st), (use & 1) ^ 1, ab)) return false;
        last_x[st] = use & 1;
        mbar_arrive_expect_tx(bar(X_FULL0 + st), 32768);
        tma_load_tile(sX(xidx), &tmC, bar(X_FULL0 + st), row, h2, b2);
        ++xidx;
        return true;
      };
      for (int idx = cta0; idx < total && ok; idx += ncta, ++item) {
        int pp, b, ha, hk;
        decode(idx, pp, b, ha, hk);
        const bool solve_item = is_solve(idx);
        const int i0 = 2 * pp;
        const bool r1 = i0 + 1 < p.NB;
        if (!mbar_wait(bar(Q_EMPTY), (item & 1) ^ 1, ab)) break;
        last_q = item & 1;
        mbar_arrive_expect_tx(bar(Q_FULL), r1 ? 65536 : 32768);
        const CUtensorMap* mA = solve_item ? &tmA : &tmQ;
        const CUtensorMap* mB = solve_item ? &tmB : &tmK;
        tma_load_tile(sQ(0), mA, bar(Q_FULL), i0 * 128, ha, b);
        if (r1) tma_load_tile(sQ(1), mA, bar(Q_FULL), (i0 + 1) * 128, ha, b);
        if (CHAIN && solve_item) {
          // the key blocks of the tiles handed to the chain (no X needed)
          for (int e = 0; e <= kChainLook && ok; ++e)
            if (etile_used(pp, e, 0) || etile_used(pp, e, 1))
              ok = loadK(&tmB, (2 * pp - kChainLook + e) * 128, hk, b);
          if (!ok) break;
        }
        const int nt = nrow(pp, 0, solve_item) > nrow(pp, 1, solve_item) ? nrow(pp, 0, solve_item) : nrow(pp, 1, solve_item);
        for (int j = 0; j < nt; ++j) {
          if (!loadK(mB, j * 128, hk, b)) { ok = false; break; }
          if (solve_item || FUSED) {  // X_j is still being produced
            if (!wait_flag_geq(&p.flags[(b * p.Hkv + hk) * p.NB + j], 1, ab)) { ok = false; break; }
            fence_proxy_async_global();
          }
          if (!loadX(j * 128, hk, b)) { ok = false; break; }
        }
        if (!ok || !solve_item || CHAIN) continue;
        // solve tail: K^_{2pp} for row 1, U_i0, U_i1, then X_{2pp} (made by row 0 of this item)
        if (r1 && !loadK(&tmB, i0 * 128, hk, b)) break;
        if (!loadK(&tmU, i0 * 128, hk, b)) break;
        if (r1 && !loadK(&tmU, (i0 + 1) * 128, hk, b)) break;
        if (r1) {
          if (!wait_flag_geq(&p.flags[(b * p.Hkv + hk) * p.NB + i0], 1, ab)) break;
          fence_proxy_async_global();
          if (!loadX(i0 * 128, hk, b)) break;
        }
      }
      if (last_q >= 0) mbar_wait_timed(bar(Q_FULL), (uint32_t)last_q, kDrainNs);
      for (int s2 = 0; s2 < 3; ++s2)
        if (last_k[s2] >= 0) mbar_wait_timed(bar(K_FULL0 + s2), (uint32_t)last_k[s2], kDrainNs);
      for (int s2 = 0; s2 < 2; ++s2)
        if (last_x[s2] >= 0) mbar_wait_timed(bar(X_FULL0 + s2), (uint32_t)last_x[s2], kDrainNs);
    }
  } else if (warp == kWarpMma) {
    // ======================= MMA issuer =======================
    if (lane == 0) {
      uint32_t kidx = 0, xidx = 0, item = 0;
      uint32_t n_pfull[2] = {0, 0}, n_ofree[2] = {0, 0}, n_yfull[2] = {0, 0};
      auto waitK = [&](uint32_t idx) { return mbar_wait(bar(K_FULL0 + idx % 3u), (idx / 3u) & 1, ab); };
      auto waitX = [&](uint32_t idx) { return mbar_wait(bar(X_FULL0 + (idx & 1u)), (idx >> 1) & 1, ab); };
      auto tS = [&](int k) { return tmem + kTmS0 + 128u * (uint32_t)k; };
      auto tO = [&](int k) { return tmem + kTmO0 + 128u * (uint32_t)k; };
      int cur_d = kHeadDim;  // attention items: K extent of S and N extent of PV (head dimension)
      auto issue_s = [&](int k, uint32_t kslot) {
        if (cur_d == kHeadDim)
          umma_tile(tS(k), sQ(k), false, sK(kslot), false, 0u);
        else
          umma_tile_part(tS(k), sQ(k), false, sK(kslot), false, 0u, cur_d / 16, 128);
        umma_commit(bar(S_FULL0 + k));
      };
      // PV_k of streaming tile t (x slot xs); first_pv: overwrite O_k
      auto issue_pv = [&](int k, uint32_t xs, bool first_pv) -> bool {
        if (!mbar_wait(bar(P_FULL0 + k), (n_pfull[k]++) & 1, ab)) return false;
        if (first_pv && !mbar_wait(bar(O_FREE0 + k), ((n_ofree[k]++) & 1) ^ 1, ab)) return false;
        tc_fence_after();
        const uint32_t sreg = tS(k);
        umma_tile_ts(tO(k), [&](int kk) { return sreg + 8u * (uint32_t)kk; }, sX(xs), true, first_pv ? 0u : 1u,
                     cur_d);
        umma_commit(bar(O_DONE0 + k));
        return true;
      };
      for (int idx = cta0; idx < total; idx += ncta, ++item) {
        int pp, b, ha, hk;
        decode(idx, pp, b, ha, hk);
        const bool solve_item = is_solve(idx);
        const int i0 = 2 * pp;
        const bool r1 = i0 + 1 < p.NB;
        const int n0 = nrow(pp, 0, solve_item), n1 = nrow(pp, 1, solve_item), nt = n0 > n1 ? n0 : n1;
        cur_d = solve_item ? kHeadDim : p.attn_d16;
        if (!mbar_wait(bar(Q_FULL), item & 1, ab)) break;
        tc_fence_after();
        bool ok = true;
        if (CHAIN && solve_item) {
          // S of the tiles handed to the chain; the epilogue reads each S_k before the
          // next GEMM into that region (P_FULL, with no PV in between)
          bool busy[2] = {false, false};
          for (int e = 0; e <= kChainLook && ok; ++e) {
            const bool u0 = etile_used(pp, e, 0), u1 = etile_used(pp, e, 1);
            if (!u0 && !u1) continue;
            if (!waitK(kidx)) { ok = false; break; }
            for (int k2 = 0; k2 < 2; ++k2) {
              if (!(k2 == 0 ? u0 : u1)) continue;
              if (busy[k2] && !mbar_wait(bar(P_FULL0 + k2), (n_pfull[k2]++) & 1, ab)) { ok = false; break; }
              tc_fence_after();
              issue_s(k2, kidx);
              busy[k2] = true;
            }
            umma_commit(bar(K_EMPTY0 + kidx % 3u));
            ++kidx;
          }
          for (int k2 = 0; k2 < 2 && ok; ++k2)
            if (busy[k2] && !mbar_wait(bar(P_FULL0 + k2), (n_pfull[k2]++) & 1, ab)) ok = false;
          if (!ok) break;
        }
        const uint32_t kb = kidx, xb = xidx;
        // S for the first tile of each row
        if (nt > 0) {
          if (!waitK(kb)) break;
          tc_fence_after();
          if (n0 > 0) issue_s(0, kb);
          if (n1 > 0) issue_s(1, kb);
          umma_commit(bar(K_EMPTY0 + kb % 3u));
        }
        for (int t = 0; t < nt && ok; ++t) {
          const uint32_t xs = xb + t;
          if (!waitX(xs)) { ok = false; break; }
          const bool has_next = t + 1 < nt;
          if (has_next && !waitK(kb + t + 1)) { ok = false; break; }
          if (t < n0) {
            if (!issue_pv(0, xs, t == 0)) { ok = false; break; }
            if (t + 1 < n0) issue_s(0, kb + t + 1);
          }
          if (t < n1) {
            if (!issue_pv(1, xs, t == 0)) { ok = false; break; }
            if (t + 1 < n1) issue_s(1, kb + t + 1);
          }
          umma_commit(bar(X_EMPTY0 + (xs & 1u)));
          if (has_next) umma_commit(bar(K_EMPTY0 + (kb + t + 1) % 3u));
        }
        if (!ok) break;
        kidx = kb + nt;
        xidx = xb + nt;
        if (solve_item && !CHAIN) {
          // tail: S1(2pp), DIAG0, PV1(2pp), DIAG1
          if (r1) {
            if (!waitK(kidx)) break;
            tc_fence_after();
            issue_s(1, kidx);
            umma_commit(bar(K_EMPTY0 + kidx % 3u));
            ++kidx;
          }
          // DIAG0: T0 = U_i0 Y0  (Y0 in row 0's A buffer)
          if (!waitK(kidx) || !mbar_wait(bar(Y_FULL0), (n_yfull[0]++) & 1, ab)) break;
          tc_fence_after();
          umma_tile(tS(0), sK(kidx), false, sQ(0), true, 0u);
          umma_commit(bar(S_FULL0));
          umma_commit(bar(K_EMPTY0 + kidx % 3u));
          ++kidx;
          if (r1) {
            if (!waitX(xidx) || !issue_pv(1, xidx, n1 == 0)) break;
            umma_commit(bar(X_EMPTY0 + (xidx & 1u)));
            ++xidx;
            if (!waitK(kidx) || !mbar_wait(bar(Y_FULL0 + 1), (n_yfull[1]++) & 1, ab)) break;
            tc_fence_after();
            umma_tile(tS(1), sK(kidx), false, sQ(1), true, 0u);
            umma_commit(bar(S_FULL0 + 1));
            umma_commit(bar(K_EMPTY0 + kidx % 3u));
            ++kidx;
          }
        }
        umma_commit(bar(Q_EMPTY));
      }
      umma_commit(bar(DRAIN));
      mbar_wait_timed(bar(DRAIN), 0, kDrainNs);
    }
  }
  } else {
    regs_inc<kRegsEpi>();
    // ======================= epilogue warpgroups =======================
    const int k = warp >> 2;            // row block of the pair owned by this warpgroup
    const int sp = warp & 3;            // TMEM sub-partition
    const int r = sp * 32 + lane;       // tile row == TMEM lane
    const uint32_t lane_base = (uint32_t)(sp * 32) << 16;
    const uint32_t tSk = tmem + lane_base + fwd::kTmS0 + 128u * (uint32_t)k;
    const uint32_t tOk = tmem + lane_base + fwd::kTmO0 + 128u * (uint32_t)k;
    const int wg_thread0 = k * 128;     // publishes this warpgroup's flags
    const float kLog2e = 1.4426950408889634f;
    const float ascale = FUSED ? p.attn_scale : p.scale;  // softmax scale of attention items
    uint32_t n_sfull = 0, n_p = 0, n_epi = 0, item = 0;
    for (int idx = cta0; idx < total; idx += ncta, ++item) {
      int pp, b, ha, hk;
      decode(idx, pp, b, ha, hk);
      const bool solve_item = is_solve(idx);
      const int i = 2 * pp + k;         // this warpgroup's row block
      if (i >= p.NB) continue;
      const float sc = solve_item ? p.scale : ascale;
      const float c1 = sc * kLog2e;
      const float c2 = kLog2e / sc;
      const int nk = nrow(pp, k, solve_item) + ((solve_item && !CHAIN && k == 1) ? 1 : 0);  // wavefront row 1 adds tile 2pp
      const int row = i * 128 + r;
      float m_run = -INFINITY, l_run = 0.f;
      bool ok = true;
      // chain schedule: make this row's writes visible, then release its chain flag
      auto publish = [&](int* flag, int value) {
        fence_proxy_async_global();
        warp_arrive(bar(EPI_DONE0 + k));
        if ((int)threadIdx.x == wg_thread0) {
          if (mbar_wait(bar(EPI_DONE0 + k), n_epi & 1, ab)) {
            __threadfence();
            st_release_gpu(flag, value);
          }
        }
        ++n_epi;
        __syncwarp();
      };
      if (CHAIN && solve_item) {
        // E_{i,i-kChainLook} .. E_{i,i-1} (row r) -> global, in the shared-memory image of
        // a K-major operand tile, which the chain copies unchanged
        const long long bhk = (long long)b * p.Hkv + hk;
        for (int s2 = 0; s2 < kChainLook && ok; ++s2) {
          if (i - kChainLook + s2 < 0) continue;
          if (!warp_wait(bar(S_FULL0 + k), (n_sfull++) & 1, ab)) { ok = false; break; }
          tc_fence_after();
          uint8_t* et = reinterpret_cast<uint8_t*>(p.etiles + ((bhk * p.NB + i) * kChainLook + s2) *
                                                                  (long long)(kTileBytes / 2));
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float sv[32];
            tmem_ld32(tSk + 32u * q, sv);
            tmem_ld_wait();
            uint32_t pk[16];
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              const float2 a = fma2(make_float2(sv[e], sv[e + 1]), make_float2(c1, c1), make_float2(-c2, -c2));
              pk[e >> 1] = pack_bf16(fast_exp2(a.x), fast_exp2(a.y));
            }
#pragma unroll
            for (int c = 0; c < 4; ++c)
              *reinterpret_cast<uint4*>(et + tile_chunk_off(r, 4 * q + c)) =
                  make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
          }
          tc_fence_before();
          warp_arrive(bar(P_FULL0 + k));
        }
        if (!ok) break;
        publish(&p.cflags[bhk * p.NB + i], 1);
      }
      if (solve_item && row < p.N) {
        // the diagonal step reads this row of V on the wavefront's critical path: fetch
        // it into L2 while the row's streaming tiles run
        const bf16* vrow = p.v + (long long)b * p.v_sb + (long long)hk * p.v_sh + (long long)row * p.v_sn;
        prefetch_l2(vrow);
        prefetch_l2(vrow + 64);
      }
      for (int t = 0; t < nk; ++t, ++n_p) {
        if (!warp_wait(bar(S_FULL0 + k), (n_sfull++) & 1, ab)) { ok = false; break; }
        tc_fence_after();
        float sv[4][32];
#pragma unroll
        for (int q = 0; q < 4; ++q) tmem_ld32(tSk + 32u * q, sv[q]);
        tmem_ld_wait();
        if (solve_item) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              const float2 a = fma2(make_float2(sv[q][e], sv[q][e + 1]), make_float2(c1, c1), make_float2(-c2, -c2));
              sv[q][e] = fast_exp2(a.x);
              sv[q][e + 1] = fast_exp2(a.y);
            }
        } else {
          // Few instructions per score (the epilogue of two warpgroups issues as many
          // instructions per tile as the tensor core needs cycles): the causal mask on the
          // diagonal tile only, the max on the raw scores (the scale c1 > 0 is monotone),
          // and the scale folded into one packed FMA ahead of the exponential.
          if (t == i) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
#pragma unroll
              for (int e = 0; e < 32; ++e)
                if ((q * 32 + e) > r) sv[q][e] = -INFINITY;
          }
          // four independent partial maxima, two scores per three-input max: 16-deep
          // dependency chains instead of one of 128
          float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
          for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              float& mj = m4[((q * 32 + e) >> 1) & 3];
              mj = fmax3(mj, sv[q][e], sv[q][e + 1]);
            }
          float mx = fmax3(m4[0], m4[1], fmaxf(m4[2], m4[3]));
          mx *= c1;
          // lazy rescale: keep the running reference unless it grows by > 8 (log2)
          bool need = false;
          float alpha = 1.f;
          if (t == 0) {
            m_run = mx;
          } else if (mx > m_run + 8.f) {
            need = true;
            alpha = fast_exp2(m_run - mx);
            m_run = mx;
          }
          if (__any_sync(0xffffffffu, need)) {
            // O_k must be stable: wait for the PV of the previous tile
            if (!warp_wait(bar(O_DONE0 + k), (n_p - 1) & 1, ab)) { ok = false; break; }
            tc_fence_after();
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              float av[32];
              tmem_ld32(tOk + 32u * q, av);
              tmem_ld_wait();
#pragma unroll
              for (int e = 0; e < 32; ++e) av[e] *= alpha;
              tmem_st32(tOk + 32u * q, av);
            }
            tmem_st_wait();
          }
          l_run *= alpha;
          const float2 cc = make_float2(c1, c1), nm = make_float2(-m_run, -m_run);
          float2 s4[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                          make_float2(0.f, 0.f)};
#pragma unroll
          for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              const float2 a = fma2(make_float2(sv[q][e], sv[q][e + 1]), cc, nm);
              const float2 ex = make_float2(fast_exp2(a.x), fast_exp2(a.y));
              sv[q][e] = ex.x;
              sv[q][e + 1] = ex.y;
              float2& sj = s4[((q * 32 + e) >> 1) & 3];
              sj = add2(sj, ex);
            }
          const float2 s01 = add2(s4[0], s4[1]), s23 = add2(s4[2], s4[3]);
          const float2 st = add2(s01, s23);
          l_run += st.x + st.y;
        }
        // P back into tensor memory over S_k (this lane's own columns)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) pk[e] = pack_bf16(sv[q][2 * e], sv[q][2 * e + 1]);
          tmem_st16(tSk + 16u * q, pk);
        }
        tmem_st_wait();
        tc_fence_before();
        warp_arrive(bar(P_FULL0 + k));
      }
      if (!ok) break;
      // O_k is final once the PV of the last tile of this row is done
      float acc[4][32];
      if (nk > 0) {
        if (!warp_wait(bar(O_DONE0 + k), (n_p - 1) & 1, ab)) break;
        tc_fence_after();
#pragma unroll
        for (int q = 0; q < 4; ++q) tmem_ld32(tOk + 32u * q, acc[q]);
        tmem_ld_wait();
        tc_fence_before();
        warp_arrive(bar(O_FREE0 + k));
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int e = 0; e < 32; ++e) acc[q][e] = 0.f;
      }
      if (!solve_item) {
        const float inv_l = 1.f / l_run;
        if (p.attn_d16 < kHeadDim) {  // columns the P X product did not write
#pragma unroll
          for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (q * 32 + e >= p.attn_d16) acc[q][e] = 0.f;
        }
        if (row < p.N) {
          bf16* orow = p.o + (long long)b * p.o_sb + (long long)ha * p.o_sh + (long long)row * p.o_sn;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
#pragma unroll
            for (int e = 0; e < 32; ++e) acc[q][e] *= inv_l;
#pragma unroll
            for (int c = 0; c < 4; ++c) st_bf16x8(orow + q * 32 + c * 8, acc[q] + c * 8);
          }
          if (p.o_res) {
            bf16* rrow = p.o_res + (orow - p.o);
#pragma unroll
            for (int q = 0; q < 4; ++q)
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                float res[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  const float v = acc[q][c * 8 + e];
                  res[e] = v - __bfloat162float(__float2bfloat16_rn(v));
                }
                st_bf16x8(rrow + q * 32 + c * 8, res);
              }
          }
        }
        p.lse[((long long)b * p.Hq + ha) * p.Npad + row] = m_run + __log2f(l_run);
        continue;
      }
      if (CHAIN) {
        // W_i = V_i - acc (fp32) into the head's ring slot: chunk c4 (4 columns) of row r
        // at (c4 * 128 + r) * 4 floats, so one warp store covers 512 contiguous bytes
        const long long bhk = (long long)b * p.Hkv + hk;
        const bf16* vrow = p.v + (long long)b * p.v_sb + (long long)hk * p.v_sh + (long long)row * p.v_sn;
        float4* ws = reinterpret_cast<float4*>(p.wring + (bhk * kChainWRing + i % kChainWRing) *
                                                             (long long)(kBlock * kHeadDim));
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float vv[8];
            if (row < p.N) {
              ld_bf16x8(vrow + q * 32 + c * 8, vv);
            } else {
#pragma unroll
              for (int e = 0; e < 8; ++e) vv[e] = 0.f;
            }
            const float* a = acc[q] + c * 8;
            ws[(8 * q + 2 * c) * 128 + r] = make_float4(vv[0] - a[0], vv[1] - a[1], vv[2] - a[2], vv[3] - a[3]);
            ws[(8 * q + 2 * c + 1) * 128 + r] = make_float4(vv[4] - a[4], vv[5] - a[5], vv[6] - a[6], vv[7] - a[7]);
          }
        publish(&p.cflags[bhk * p.NB + i], 2);
        continue;
      }
      // ---- solve: diagonal block.  Y = D^-1 (V - acc) -> A buffer of this row ----
      const long long bhk = (long long)b * p.Hkv + hk;
      const float di = p.dinv[bhk * p.Npad + row];
      const bf16* vrow = p.v + (long long)b * p.v_sb + (long long)hk * p.v_sh + (long long)row * p.v_sn;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float vv[8];
          if (row < p.N) {
            ld_bf16x8(vrow + q * 32 + c * 8, vv);
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) vv[e] = 0.f;
          }
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[q][c * 8 + e] = (vv[e] - acc[q][c * 8 + e]) * di;
        }
      }
      // the A buffer may still be in flight from TMA when this row had no tiles
      if (!warp_wait(bar(Q_FULL), item & 1, ab)) break;
#pragma unroll
      for (int q = 0; q < 4; ++q) tile_store_row32(sQ(k), r, q, acc[q]);
      fence_proxy_async_smem();
      warp_arrive(bar(Y_FULL0 + k));
      if (!warp_wait(bar(S_FULL0 + k), (n_sfull++) & 1, ab)) break;
      tc_fence_after();
      bf16* xrow = p.x + (bhk * p.Npad + row) * kHeadDim;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float tv[32];
        tmem_ld32(tSk + 32u * q, tv);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) tv[e] += acc[q][e];
#pragma unroll
        for (int c = 0; c < 4; ++c) st_bf16x8(xrow + q * 32 + c * 8, tv + c * 8);
      }
      tc_fence_before();
      fence_proxy_async_global();
      warp_arrive(bar(EPI_DONE0 + k));
      if ((int)threadIdx.x == wg_thread0) {   // publish: the rows of X, then the flag (one fence, cumulative)
        if (mbar_wait(bar(EPI_DONE0 + k), n_epi & 1, ab)) {
          __threadfence();
          st_release_gpu(&p.flags[bhk * p.NB + i], 1);
        }
      }
      ++n_epi;
      __syncwarp();
    }
  }

  // ---- teardown: every role is done (or aborted); release TMEM ----
  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// --------------------------------------------------------------------------
// host launchers
// --------------------------------------------------------------------------
static int num_sms() {
  int dev = 0;
  cudaGetDevice(&dev);
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

cudaError_t launch_fwd(bool solve, const CUtensorMap& tA, const CUtensorMap& tB, const CUtensorMap& tC,
                       const CUtensorMap& tU, const FwdArgs& a, cudaStream_t st) {
  // attention alone: Q and K come through tmQ / tmK (passed as tA / tB)
  const int pairs = (a.pp1 > 0 ? a.pp1 : (a.NB + 1) / 2) - a.pp0;
  const int total = solve ? pairs * a.B * a.Hkv : pairs * a.B * a.Hq;
  if (total <= 0) return cudaSuccess;
  const int cap = a.max_ctas > 0 ? std::min(a.max_ctas, num_sms()) : num_sms();
  cudaError_t e;
  if (solve && a.nchain > 0) {
    // chain schedule: the chains plus at least one worker CTA, all resident
    if (a.pp0 != 0 || a.pp1 != 0 || a.nchain != a.B * a.Hkv || a.nchain >= cap) return cudaErrorInvalidValue;
    const int grid = std::min(a.nchain + total, cap);
    e = cudaFuncSetAttribute(lucid_fwd_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)fwd::kSmemBytes);
    if (e != cudaSuccess) return e;
    return launch_cooperative(lucid_fwd_kernel<2>, grid, fwd::kThreads, fwd::kSmemBytes, st, tA, tB, tC, tU, tA, tB,
                              a);
  }
  const int grid = std::min(total, cap);
  if (solve) {
    e = cudaFuncSetAttribute(lucid_fwd_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)fwd::kSmemBytes);
    if (e != cudaSuccess) return e;
    // the wavefront's CTAs wait on one another's flags: all of them must be resident
    return launch_cooperative(lucid_fwd_kernel<1>, grid, fwd::kThreads, fwd::kSmemBytes, st, tA, tB, tC, tU, tA, tB,
                              a);
  } else {
    e = cudaFuncSetAttribute(lucid_fwd_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)fwd::kSmemBytes);
    if (e != cudaSuccess) return e;
    lucid_fwd_kernel<0><<<grid, fwd::kThreads, fwd::kSmemBytes, st>>>(tA, tB, tC, tU, tA, tB, a);
  }
  return cudaGetLastError();
}

// Fused forward (chain schedule, a.nchain = B*Hkv chains): the solve's items, then the
// attention's, in one cooperative launch.
cudaError_t launch_fwd_fused(const CUtensorMap& tKhat, const CUtensorMap& tX,
                             const CUtensorMap& tU, const CUtensorMap& tQ, const CUtensorMap& tK,
                             const FwdArgs& a, cudaStream_t st) {
  const int pairs = (a.NB + 1) / 2;
  const int total = pairs * a.B * (a.Hkv + a.Hq);
  const int cap = num_sms();
  if (a.pp0 != 0 || a.pp1 != 0 || a.nchain != a.B * a.Hkv || a.nchain >= cap) return cudaErrorInvalidValue;
  const int grid = std::min(a.nchain + total, cap);
  cudaError_t e = cudaFuncSetAttribute(lucid_fwd_kernel<3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)fwd::kSmemBytes);
  if (e != cudaSuccess) return e;
  return launch_cooperative(lucid_fwd_kernel<3>, grid, fwd::kThreads, fwd::kSmemBytes, st, tKhat, tKhat, tX, tU, tQ, tK,
                            a);
}

// Schedule of the solve forward for B*H heads of NB row blocks on this device: the
// number of chain CTAs (the chain schedule, one per head) or 0 (the wavefront).  Model
// (one B200, 32K rows): a tile of the row sums costs ~1.2 us of one SM; a diagonal step
// ~10 us in the wavefront (it crosses CTAs through L2) and ~4 us in a chain CTA, which
// waits for the workers' partial sums.  LUCID_B200_SOLVE_SCHEDULE=chain / wavefront
// overrides the choice.
int solve_chain_ctas(int BH, int NB) {
  const int sms = num_sms();
  if (BH <= 0 || NB <= 0 || BH + 4 > sms) return 0;
  const char* env = getenv("LUCID_B200_SOLVE_SCHEDULE");
  if (env && strcmp(env, "wavefront") == 0) return 0;
  if (env && strcmp(env, "chain") == 0) return BH;
  const double work = (double)BH * NB * (NB + 1) / 2.0 * 1.2;  // SM-microseconds
  const double t_wave = std::max(work / sms, NB * 10.0);
  const double t_chain = std::max(work / (sms - BH), NB * 4.0);
  return t_chain < 0.9 * t_wave ? BH : 0;
}

}  // namespace lb
