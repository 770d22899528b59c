// O(N^2) kernels of LUCID-Path (lucid_path/triton_code/), all persistent,
// warp-specialised tcgen05 kernels on [128 x 128] bf16 tiles (320 threads:
// warps 0-7 epilogue, warp 8 TMA producer, warp 9 MMA issuer; epilogue warp
// w reads TMEM lanes 32*(w%4).. and columns 64*(w/4)..).
//
//   path_scores_kernel  off-diagonal path scores (triangular_solve_fwd.py:177-209).
//       Row block i walks j = i-1 .. 0 carrying Q~ (fp32 in registers):
//         S = Q~ K_new_j^T -> L_ij = exp(s S - 1/s) (bf16 tile to HBM;
//             Q~ enters as bf16 hi + lo, so the score keeps ~16 mantissa bits)
//         Q~ <- Q~ - (Q~ W_j^T) W2_j               (two MMAs, -S2 staged in TMEM)
//       The bf16 operand copy of every Q~ is also stored (TMA) for the backward.
//   path_solve_kernel<false>  O = (I + L)^-1 V, block forward substitution as a
//       wavefront over flags (triangular_solve_fwd.py:160-221):
//         R_i = V_i - sum_{j<i} L_ij O_j,  O_i = R_i + U_i R_i,  U_i = (I + L_ii)^-1 - I
//   path_solve_kernel<true>   dV = (I + L)^-T dO, the transposed wavefront
//       (triangular_solve_bwd_dv_reuse.py:17-205):
//         R_j = dO_j - sum_{i>j} L_ij^T dV_i,  dV_j = R_j + U_j^T R_j
//   path_row_kernel     row pass of the backward, row block i, j = 0 .. i:
//         dA_ij = -s L_ij o (dV_i O_j^T)                  (stored for the column pass)
//         dQ~^{(j)} = dQ~^{(j-1)} - (dQ~^{(j-1)} W2_j^T) W_j + dA_ij K_new_j
//       giving dQ_new_i = dQ~^{(i-1)} and the snapshots dQ~_i^{(j-1)}
//       (the work of parallel_path_bwd_inter_dqh.py / parallel_path_bwd_intra.py).
//   path_col_kernel     column pass, column block j, i = j+1 .. NB-1:
//         dK_new_j = sum_i dA_ij^T Q~_i^{(j)},   Phi_j = sum_i Q~_i^{(j)T} dQ~_i^{(j-1)}
//         dW2_j = -W_j Phi_j,  dW_j = -W2_j Phi_j^T
//       (parallel_path_bwd_inter_dkv.py, cumprod_householder_bwd.py: Phi_j is
//       the gradient of the block transform G_j = I - W_j^T W2_j).
// Every spin wait is bounded (mbar_wait / wait_flag_geq); a timeout records
// the status word and unwinds.
#include "path_common.cuh"

#include <algorithm>

namespace lb {

namespace pk {
constexpr int kThreads = 320;
constexpr int kEpi = 256;
constexpr int kWarpTma = 8, kWarpMma = 9;
}  // namespace pk

__device__ __forceinline__ bool pwarp_wait(uint32_t bar, uint32_t parity, const Abort& ab) {
  const bool ok = mbar_wait(bar, parity, ab);
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
  tmem_ld32(taddr, *reinterpret_cast<float(*)[32]>(v));
  tmem_ld32(taddr + 32u, *reinterpret_cast<float(*)[32]>(v + 32));
  tmem_ld_wait();
}
// Rewrite 64 fp32 values (one thread's half row) as 32 packed bf16 columns
// starting at taddr (the first column of the half), optionally negated.
__device__ __forceinline__ void tmem_st_packed64(uint32_t taddr, const float (&v)[64], float sign) {
  uint32_t pk0[16], pk1[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    pk0[e] = pack_bf16(sign * v[2 * e], sign * v[2 * e + 1]);
    pk1[e] = pack_bf16(sign * v[32 + 2 * e], sign * v[32 + 2 * e + 1]);
  }
  tmem_st16(taddr, pk0);
  tmem_st16(taddr + 16u, pk1);
}
__device__ __forceinline__ void tile_store_row64(uint32_t tile, int r, int hf, const float (&v)[64]) {
  tile_store_row32(tile, r, 2 * hf, *reinterpret_cast<const float(*)[32]>(v));
  tile_store_row32(tile, r, 2 * hf + 1, *reinterpret_cast<const float(*)[32]>(v + 32));
}
__device__ __forceinline__ void st_f32x64(float* p, const float (&v)[64]) {
#pragma unroll
  for (int e = 0; e < 16; ++e)
    reinterpret_cast<float4*>(p)[e] = make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
}
__device__ __forceinline__ void st_bf16x64(bf16* p, const float (&v)[64]) {
#pragma unroll
  for (int e = 0; e < 8; ++e) st_bf16x8(p + 8 * e, v + 8 * e);
}
__device__ __forceinline__ void ld_bf16x64(const bf16* p, float (&v)[64]) {
#pragma unroll
  for (int e = 0; e < 8; ++e) ld_bf16x8(p + 8 * e, v + 8 * e);
}

// Producer-side ring of 32 KB tiles.
template <int R>
struct TileRing {
  uint32_t base, full0, empty0;
  uint32_t n = 0;
  int last[R];
  __device__ void init(uint32_t b, uint32_t f0, uint32_t e0) {
    base = b; full0 = f0; empty0 = e0; n = 0;
#pragma unroll
    for (int s = 0; s < R; ++s) last[s] = -1;
  }
  __device__ uint32_t slot(uint32_t idx) const { return base + (idx % R) * 32768u; }
  __device__ bool load(const CUtensorMap* m, int row, int c2, int c3, const Abort& ab) {
    const uint32_t st = n % R, use = n / R;
    if (!mbar_wait(empty0 + 8u * st, (use & 1) ^ 1, ab)) return false;
    last[st] = (int)(use & 1);
    mbar_arrive_expect_tx(full0 + 8u * st, 32768);
    tma_load_tile(slot(n), m, full0 + 8u * st, row, c2, c3);
    ++n;
    return true;
  }
  __device__ void drain() {
#pragma unroll
    for (int s = 0; s < R; ++s)
      if (last[s] >= 0) mbar_wait_timed(full0 + 8u * s, (uint32_t)last[s], kDrainNs);
  }
};

// ===========================================================================
// path_scores_kernel
// ===========================================================================
// Warps 4-7 carry the query chain, the critical path of the kernel: they write
// -S2 back into TMEM as the A operand of the chain GEMM, which accumulates
// Q~ += (-S2) W2_j in TMEM, then turn Q~ into the bf16 hi / lo operand tiles
// of the next step and store the snapshot.  Warps 0-3 turn each score tile
// into L_ij (exp, bf16, to HBM) off the critical path.  Per step the MMA warp
// issues the chain's S2 before the scores S.
namespace psc {
constexpr int kRing = 4;
constexpr uint32_t kOffQ = 0, kOffQlo = 32768, kOffRing = 65536, kOffBar = kOffRing + kRing * 32768;
enum { RF0 = 0, RE0 = RF0 + kRing, QOP_FULL = RE0 + kRing, QOP_FREE, QFREE, S_FULL, S_FREE, S2_FULL, NS2_FULL,
       QD_FULL, DRAIN, NBAR };
constexpr uint32_t kSmem = kOffBar + NBAR * 8 + 16;
constexpr uint32_t kTmS = 0, kTmS2 = 128, kTmQ = 256;
constexpr int kHalf = 128;
constexpr int kChainLead = 128;   // thread that stores the snapshots (first of warps 4-7)
}  // namespace psc

__global__ void __launch_bounds__(pk::kThreads, 1)
    path_scores_kernel(const __grid_constant__ CUtensorMap tmKn, const __grid_constant__ CUtensorMap tmW,
                       const __grid_constant__ CUtensorMap tmW2, const __grid_constant__ CUtensorMap tmQs,
                       PathScoresArgs p) {
  using namespace psc;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  auto bar = [&](int i) { return sbase + kOffBar + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffBar + NBAR * 8);
  volatile int* abort_cta = reinterpret_cast<volatile int*>(smem + kOffBar + NBAR * 8 + 4);
  const Abort ab{abort_cta, p.status, kTagPathScores};
  const uint32_t sQ = sbase + kOffQ, sQlo = sbase + kOffQlo;
  const int warp = warp_id(), lane = lane_id();
  if ((sbase & 1023u) != 0) {
    if (threadIdx.x == 0) atomicCAS(p.status, 0, kStatusMisaligned | (kTagPathScores << 20));
    return;
  }
  if (threadIdx.x == pk::kWarpTma * 32) {
    for (int s = 0; s < kRing; ++s) {
      mbar_init(bar(RF0 + s), 1);
      mbar_init(bar(RE0 + s), 1);
    }
    mbar_init(bar(QOP_FULL), kHalf);
    mbar_init(bar(QOP_FREE), 1);
    mbar_init(bar(QFREE), 1);
    mbar_init(bar(S_FULL), 1);
    mbar_init(bar(S_FREE), kHalf);
    mbar_init(bar(S2_FULL), 1);
    mbar_init(bar(NS2_FULL), kHalf);
    mbar_init(bar(QD_FULL), 1);
    mbar_init(bar(DRAIN), 1);
    *abort_cta = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmKn);
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmW2);
    tma_prefetch_desc(&tmQs);
  }
  if (warp == pk::kWarpMma) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int BHQ = p.B * p.HQ;
  const int total = (p.NB - 1) * BHQ;
  const long long Npad = (long long)p.NB * 128;
  auto decode = [&](int idx, int& i, int& bhq, int& b, int& h, int& bhk) {
    // longest rows first across all heads (the chain is latency-bound: balance
    // matters more here than L2 residency)
    i = p.NB - 1 - idx / BHQ;
    bhq = idx % BHQ;
    b = bhq / p.HQ;
    h = (bhq % p.HQ) / p.G;
    bhk = b * p.H + h;
  };

  if (warp == pk::kWarpTma) {
    if (lane == 0) {
      TileRing<kRing> ring;
      ring.init(sbase + kOffRing, bar(RF0), bar(RE0));
      bool ok = true;
      for (int idx = blockIdx.x; idx < total && ok; idx += gridDim.x) {
        int i, bhq, b, h, bhk;
        decode(idx, i, bhq, b, h, bhk);
        for (int j = i - 1; j >= 0 && ok; --j) {
          ok = ring.load(&tmKn, j * 128, bhk, 0, ab);
          if (ok && j > 0) ok = ring.load(&tmW, j * 128, h, b, ab) && ring.load(&tmW2, j * 128, bhk, 0, ab);
        }
      }
      ring.drain();
    }
  } else if (warp == pk::kWarpMma) {
    if (lane == 0) {
      uint32_t rc = 0, n_q = 0, n_ns2 = 0, n_sfree = 0;
      auto ring_slot = [&](uint32_t idx) { return sbase + kOffRing + (idx % kRing) * 32768u; };
      auto ring_wait = [&](uint32_t idx) { return mbar_wait(bar(RF0 + (int)(idx % kRing)), (idx / kRing) & 1, ab); };
      auto ring_free = [&](uint32_t idx) { umma_commit(bar(RE0 + (int)(idx % kRing))); };
      const uint32_t tS = tmem + kTmS, tS2 = tmem + kTmS2;
      bool ok = true;
      for (int idx = blockIdx.x; idx < total && ok; idx += gridDim.x) {
        int i, bhq, b, h, bhk;
        decode(idx, i, bhq, b, h, bhk);
        for (int j = i - 1; j >= 0; --j) {
          if (!mbar_wait(bar(QOP_FULL), (n_q++) & 1, ab)) { ok = false; break; }
          const uint32_t sK = rc++;
          if (!ring_wait(sK)) { ok = false; break; }
          uint32_t sW = 0;
          if (j > 0) {
            sW = rc++;
            if (!ring_wait(sW)) { ok = false; break; }
          }
          tc_fence_after();
          if (j > 0) {  // chain first
            umma_tile(tS2, sQ, false, ring_slot(sW), false, 0u);
            umma_commit(bar(S2_FULL));
          }
          // the previous score tile has been read by warps 0-3
          if (!mbar_wait(bar(S_FREE), ((n_sfree++) & 1) ^ 1, ab)) { ok = false; break; }
          tc_fence_after();
          umma_tile(tS, sQ, false, ring_slot(sK), false, 0u);
          umma_tile(tS, sQlo, false, ring_slot(sK), false, 1u);
          umma_commit(bar(S_FULL));
          ring_free(sK);
          if (j == 0) {
            umma_commit(bar(QOP_FREE));  // the operand tiles may be rewritten for the next item
            break;
          }
          ring_free(sW);
          if (!mbar_wait(bar(NS2_FULL), (n_ns2++) & 1, ab)) { ok = false; break; }
          const uint32_t sW2 = rc++;
          if (!ring_wait(sW2)) { ok = false; break; }
          tc_fence_after();
          // -S2 was packed by full rows: K-slice kk at column 8 kk; Q~ accumulates in TMEM
          umma_tile_ts(tmem + kTmQ, [&](int kk) { return tS2 + 8u * (uint32_t)kk; }, ring_slot(sW2), true, 1u);
          umma_commit(bar(QD_FULL));
          ring_free(sW2);
        }
      }
      umma_commit(bar(DRAIN));
      mbar_wait_timed(bar(DRAIN), 0, kDrainNs);
    }
  } else if (warp < 4) {
    // ---------------- score tiles -> L_ij ----------------
    const int r = warp * 32 + lane;
    const uint32_t tS = tmem + ((uint32_t)(warp * 32) << 16) + kTmS;
    const float c1 = p.s * 1.4426950408889634f, c2 = 1.4426950408889634f / p.s;
    uint32_t n_s = 0;
    bool ok = true;
    for (int idx = blockIdx.x; idx < total && ok; idx += gridDim.x) {
      int i, bhq, b, h, bhk;
      decode(idx, i, bhq, b, h, bhk);
      for (int j = i - 1; j >= 0; --j) {
        if (!pwarp_wait(bar(S_FULL), (n_s++) & 1, ab)) { ok = false; break; }
        tc_fence_after();
        bf16* dst = p.L + (((long long)bhq * p.NPAIR + path_pair(i, j)) * 128 + r) * 128;
        for (int c = 0; c < 4; ++c) {
          float v[32];
          tmem_ld32(tS + 32u * c, v);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const float2 a = fma2(make_float2(v[e], v[e + 1]), make_float2(c1, c1), make_float2(-c2, -c2));
            v[e] = fast_exp2(a.x);
            v[e + 1] = fast_exp2(a.y);
          }
#pragma unroll
          for (int e = 0; e < 4; ++e) st_bf16x8(dst + c * 32 + e * 8, v + e * 8);
        }
        tc_fence_before();
        mbar_arrive(bar(S_FREE));
      }
    }
  } else {
    // ---------------- query chain ----------------
    const int wq = warp - 4;
    const int r = wq * 32 + lane;
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    const uint32_t tS2 = tmem + lane_base + kTmS2, tQ = tmem + lane_base + kTmQ;
    uint32_t n_s2 = 0, n_qd = 0, n_qf = 0, n_free = 0, n_full = 0;
    bool first = true;
    auto write_op = [&](int c, const float (&v)[32]) {
      float hi[32], lo[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        hi[e] = __bfloat162float(__float2bfloat16(v[e]));
        lo[e] = v[e] - hi[e];
      }
      tile_store_row32(sQ, r, c, hi);
      tile_store_row32(sQlo, r, c, lo);
    };
    // the snapshot stores of the previous operand have finished reading it
    auto operand_free = [&]() -> bool {
      if ((int)threadIdx.x == kChainLead) {
        bulk_wait_read_all();
        mbar_arrive(bar(QFREE));
      }
      __syncwarp();
      return pwarp_wait(bar(QFREE), (n_qf++) & 1, ab);
    };
    // all 128 rows written: hand the operand to the MMA warp and store the snapshot
    auto publish = [&](long long pair, int bhq) {
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(bar(QOP_FULL));
      if ((int)threadIdx.x == kChainLead) {
        if (mbar_wait(bar(QOP_FULL), n_full & 1, ab)) {
          tma_store_tile(&tmQs, sQ, (int)(pair * 128), bhq, 0);
          bulk_commit();
        }
      }
      ++n_full;
      __syncwarp();
    };
    bool ok = true;
    for (int idx = blockIdx.x; idx < total && ok; idx += gridDim.x) {
      int i, bhq, b, h, bhk;
      decode(idx, i, bhq, b, h, bhk);
      // the previous item's last score GEMM has finished reading the operand tiles
      if (!first && !pwarp_wait(bar(QOP_FREE), (n_free++) & 1, ab)) break;
      first = false;
      if (!operand_free()) break;
      {
        const float* src = p.qn + (((long long)bhq * Npad) + i * 128 + r) * 128;
        for (int c = 0; c < 4; ++c) {
          float v[32];
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            const float4 f = *reinterpret_cast<const float4*>(src + c * 32 + e);
            v[e] = f.x; v[e + 1] = f.y; v[e + 2] = f.z; v[e + 3] = f.w;
          }
          tmem_st32(tQ + 32u * c, v);
          write_op(c, v);
        }
        tmem_st_wait();
        publish(path_pair(i, i - 1), bhq);
      }
      for (int j = i - 1; j >= 1; --j) {
        if (!pwarp_wait(bar(S2_FULL), (n_s2++) & 1, ab)) { ok = false; break; }
        tc_fence_after();
        for (int c = 0; c < 4; ++c) {
          float v[32];
          tmem_ld32(tS2 + 32u * c, v);
          tmem_ld_wait();
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) pk[e] = pack_bf16(-v[2 * e], -v[2 * e + 1]);
          // packed columns of chunk c go to [16c, 16c+16): inside chunks already read
          tmem_st16(tS2 + 16u * (uint32_t)c, pk);
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(bar(NS2_FULL));
        if (!pwarp_wait(bar(QD_FULL), (n_qd++) & 1, ab)) { ok = false; break; }
        tc_fence_after();
        if (!operand_free()) { ok = false; break; }
        for (int c = 0; c < 4; ++c) {
          float v[32];
          tmem_ld32(tQ + 32u * c, v);
          tmem_ld_wait();
          write_op(c, v);
        }
        publish(path_pair(i, j - 1), bhq);
      }
    }
    if ((int)threadIdx.x == kChainLead) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == pk::kWarpMma) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ===========================================================================
// path_solve_kernel<TR>
// ===========================================================================
namespace psv {
constexpr int kRing = 4;
constexpr uint32_t kOffY = 0, kOffY2 = 32768, kOffRing = 65536, kOffBar = kOffRing + kRing * 32768;
enum { RF0 = 0, RE0 = RF0 + kRing, ACC_FULL = RE0 + kRing, Y_FULL, T_FULL, ACC_FREE, EPI_DONE, DRAIN, NBAR };
constexpr uint32_t kSmem = kOffBar + NBAR * 8 + 16;
constexpr uint32_t kTmAcc = 0, kTmT = 128;
}  // namespace psv

template <bool TR>
__global__ void __launch_bounds__(pk::kThreads, 1)
    path_solve_kernel(const __grid_constant__ CUtensorMap tmL, const __grid_constant__ CUtensorMap tmX,
                      const __grid_constant__ CUtensorMap tmU, PathSolveArgs p) {
  using namespace psv;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  auto bar = [&](int i) { return sbase + kOffBar + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffBar + NBAR * 8);
  volatile int* abort_cta = reinterpret_cast<volatile int*>(smem + kOffBar + NBAR * 8 + 4);
  const Abort ab{abort_cta, p.status, TR ? kTagPathSolveT : kTagPathSolve};
  const uint32_t sY = sbase + kOffY, sY2 = sbase + kOffY2;
  const int warp = warp_id(), lane = lane_id();
  if ((sbase & 1023u) != 0) {
    if (threadIdx.x == 0) atomicCAS(p.status, 0, kStatusMisaligned | (ab.tag << 20));
    return;
  }
  if (threadIdx.x == pk::kWarpTma * 32) {
    for (int s = 0; s < kRing; ++s) {
      mbar_init(bar(RF0 + s), 1);
      mbar_init(bar(RE0 + s), 1);
    }
    mbar_init(bar(ACC_FULL), 1);
    mbar_init(bar(Y_FULL), pk::kEpi);
    mbar_init(bar(T_FULL), 1);
    mbar_init(bar(ACC_FREE), pk::kEpi);
    mbar_init(bar(EPI_DONE), pk::kEpi);
    mbar_init(bar(DRAIN), 1);
    *abort_cta = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmL);
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmU);
  }
  if (warp == pk::kWarpMma) {
    tmem_alloc(smem_u32(tmem_slot), 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int BHQ = p.B * p.HQ;
  const int total = p.NB * BHQ;
  const long long Npad = (long long)p.NB * 128;
  // item -> (block, head); the forward walks blocks upwards, the transposed solve downwards
  auto decode = [&](int idx, int& blk, int& bhq, int& ndeps) {
    blk = TR ? p.NB - 1 - idx / BHQ : idx / BHQ;
    bhq = idx % BHQ;
    ndeps = TR ? p.NB - 1 - blk : blk;
  };
  // dependencies in the order they were published (oldest first), so a block
  // stalls only on its last dependency
  auto dep_block = [&](int blk, int d) { (void)blk; return TR ? p.NB - 1 - d : d; };
  auto pair_of = [&](int blk, int db) { return TR ? path_pair(db, blk) : path_pair(blk, db); };

  if (warp == pk::kWarpTma) {
    if (lane == 0) {
      TileRing<kRing> ring;
      ring.init(sbase + kOffRing, bar(RF0), bar(RE0));
      bool ok = true;
      for (int idx = blockIdx.x; idx < total && ok; idx += gridDim.x) {
        int blk, bhq, nd;
        decode(idx, blk, bhq, nd);
        for (int d = 0; d < nd && ok; ++d) {
          const int db = dep_block(blk, d);
          if (!wait_flag_geq(&p.flags[(long long)bhq * p.NB + db], 1, ab)) { ok = false; break; }
          fence_proxy_async_global();
          ok = ring.load(&tmL, (int)(pair_of(blk, db) * 128), bhq, 0, ab) && ring.load(&tmX, db * 128, bhq, 0, ab);
        }
        if (ok) ok = ring.load(&tmU, blk * 128, bhq, 0, ab);
      }
      ring.drain();
    }
  } else if (warp == pk::kWarpMma) {
    if (lane == 0) {
      uint32_t rc = 0, n_free = 0, n_y = 0;
      auto ring_slot = [&](uint32_t idx) { return sbase + kOffRing + (idx % kRing) * 32768u; };
      auto ring_wait = [&](uint32_t idx) { return mbar_wait(bar(RF0 + (int)(idx % kRing)), (idx / kRing) & 1, ab); };
      auto ring_free = [&](uint32_t idx) { umma_commit(bar(RE0 + (int)(idx % kRing))); };
      for (int idx = blockIdx.x; idx < total; idx += gridDim.x) {
        int blk, bhq, nd;
        decode(idx, blk, bhq, nd);
        if (!mbar_wait(bar(ACC_FREE), ((n_free++) & 1) ^ 1, ab)) break;
        bool ok = true;
        for (int d = 0; d < nd; ++d) {
          const uint32_t sL = rc++, sX = rc++;
          if (!ring_wait(sL) || !ring_wait(sX)) { ok = false; break; }
          tc_fence_after();
          umma_tile(tmem + kTmAcc, ring_slot(sL), TR, ring_slot(sX), true, d > 0 ? 1u : 0u);
          ring_free(sL);
          ring_free(sX);
        }
        if (!ok) break;
        umma_commit(bar(ACC_FULL));
        const uint32_t sU = rc++;
        if (!ring_wait(sU) || !mbar_wait(bar(Y_FULL), (n_y++) & 1, ab)) break;
        tc_fence_after();
        umma_tile(tmem + kTmT, ring_slot(sU), TR, sY, true, 0u);
        umma_tile(tmem + kTmT, ring_slot(sU), TR, sY2, true, 1u);
        umma_commit(bar(T_FULL));
        ring_free(sU);
      }
      umma_commit(bar(DRAIN));
      mbar_wait_timed(bar(DRAIN), 0, kDrainNs);
    }
  } else {
    const int qd = warp & 3, hf = warp >> 2;
    const int r = qd * 32 + lane;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const uint32_t tAcc = tmem + lane_base + kTmAcc + 64u * hf;
    const uint32_t tT = tmem + lane_base + kTmT + 64u * hf;
    uint32_t n_acc = 0, n_t = 0, n_epi = 0;
    for (int idx = blockIdx.x; idx < total; idx += gridDim.x) {
      int blk, bhq, nd;
      decode(idx, blk, bhq, nd);
      const int b = bhq / p.HQ, hq = bhq % p.HQ, h = hq / p.G;
      if (!pwarp_wait(bar(ACC_FULL), (n_acc++) & 1, ab)) break;
      tc_fence_after();
      float R[64];
      if (nd > 0) {
        tmem_ld64(tAcc, R);
      } else {
#pragma unroll
        for (int e = 0; e < 64; ++e) R[e] = 0.f;
      }
      const long long t = (long long)blk * 128 + r;
      if (t < p.T) {
        float rhs[64];
        const bf16* src = p.rhs + (long long)b * p.r_sb + (long long)(TR ? hq : h) * p.r_sh + t * p.r_st + hf * 64;
        ld_bf16x64(src, rhs);
#pragma unroll
        for (int e = 0; e < 64; ++e) R[e] = rhs[e] - R[e];
      } else {
#pragma unroll
        for (int e = 0; e < 64; ++e) R[e] = -R[e];
      }
      {  // R = hi + lo, both bf16: the diagonal product U R keeps ~16 mantissa bits
        float hi[64], lo[64];
#pragma unroll
        for (int e = 0; e < 64; ++e) {
          hi[e] = __bfloat162float(__float2bfloat16(R[e]));
          lo[e] = R[e] - hi[e];
        }
        tile_store_row64(sY, r, hf, hi);
        tile_store_row64(sY2, r, hf, lo);
      }
      fence_proxy_async_smem();
      mbar_arrive(bar(Y_FULL));
      if (!pwarp_wait(bar(T_FULL), (n_t++) & 1, ab)) break;
      tc_fence_after();
      float X[64];
      tmem_ld64(tT, X);
#pragma unroll
      for (int e = 0; e < 64; ++e) X[e] += R[e];
      tc_fence_before();
      mbar_arrive(bar(ACC_FREE));
      st_bf16x64(p.xbuf + (((long long)bhq * Npad) + t) * 128 + hf * 64, X);
      if (!TR && p.out != nullptr && t < p.T)
        st_bf16x64(p.out + (long long)b * p.o_sb + (long long)hq * p.o_sh + t * p.o_st + hf * 64, X);
      fence_proxy_async_global();
      mbar_arrive(bar(EPI_DONE));
      if (threadIdx.x == 0) {   // publish: the block's rows, then the flag (one fence, cumulative)
        if (mbar_wait(bar(EPI_DONE), n_epi & 1, ab)) {
          __threadfence();
          st_release_gpu(&p.flags[(long long)bhq * p.NB + blk], 1);
        }
      }
      ++n_epi;
      __syncwarp();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == pk::kWarpMma) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ===========================================================================
// path_row_kernel
// ===========================================================================
// Warps 0-3 produce the dA tiles (P = dV_i O_j^T read from TMEM, the L tile from
// HBM, dA stored and packed back into TMEM as an A operand); warps 4-7 carry the
// dQ~ chain, the critical path: -S3 back into TMEM, then dQ~ -- accumulated in
// TMEM by the chain GEMM dQ~ += dA K_new_j + (-S3) W_j -- into the bf16 operand
// of the next step and the snapshot.  P is double-buffered in TMEM and issued
// one step ahead, so dA(j+1) is ready before the chain reaches step j+1.
namespace prw {
constexpr int kRing = 4;
constexpr uint32_t kOffDV = 0, kOffDOP = 32768, kOffRing = 65536, kOffBar = kOffRing + kRing * 32768;
enum { RF0 = 0, RE0 = RF0 + kRing, DV_FULL = RE0 + kRing, DV_EMPTY, P_FULL, PK_FULL, S3_FULL, NS3_FULL, DQ_FULL,
       DQ_FREE, DOP_FULL, QFREE, DRAIN, NBAR };
constexpr uint32_t kSmem = kOffBar + NBAR * 8 + 16;
constexpr uint32_t kTmP = 0, kTmS3 = 256, kTmDQ = 384;   // P: two 128-column buffers
constexpr int kHalf = 128;
constexpr int kChainLead = 128;
}  // namespace prw

__global__ void __launch_bounds__(pk::kThreads, 1)
    path_row_kernel(const __grid_constant__ CUtensorMap tmDV, const __grid_constant__ CUtensorMap tmO,
                    const __grid_constant__ CUtensorMap tmKn, const __grid_constant__ CUtensorMap tmW,
                    const __grid_constant__ CUtensorMap tmW2, const __grid_constant__ CUtensorMap tmDs,
                    PathRowArgs p) {
  using namespace prw;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  auto bar = [&](int i) { return sbase + kOffBar + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffBar + NBAR * 8);
  volatile int* abort_cta = reinterpret_cast<volatile int*>(smem + kOffBar + NBAR * 8 + 4);
  const Abort ab{abort_cta, p.status, kTagPathRow};
  const uint32_t sDV = sbase + kOffDV, sDOP = sbase + kOffDOP;
  const int warp = warp_id(), lane = lane_id();
  if ((sbase & 1023u) != 0) {
    if (threadIdx.x == 0) atomicCAS(p.status, 0, kStatusMisaligned | (kTagPathRow << 20));
    return;
  }
  if (threadIdx.x == pk::kWarpTma * 32) {
    for (int s = 0; s < kRing; ++s) {
      mbar_init(bar(RF0 + s), 1);
      mbar_init(bar(RE0 + s), 1);
    }
    mbar_init(bar(DV_FULL), 1);
    mbar_init(bar(DV_EMPTY), 1);
    mbar_init(bar(P_FULL), 1);
    mbar_init(bar(PK_FULL), kHalf);
    mbar_init(bar(S3_FULL), 1);
    mbar_init(bar(NS3_FULL), kHalf);
    mbar_init(bar(DQ_FULL), 1);
    mbar_init(bar(DQ_FREE), kHalf);
    mbar_init(bar(DOP_FULL), kHalf);
    mbar_init(bar(QFREE), 1);
    mbar_init(bar(DRAIN), 1);
    *abort_cta = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmDV);
    tma_prefetch_desc(&tmO);
    tma_prefetch_desc(&tmKn);
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmW2);
    tma_prefetch_desc(&tmDs);
  }
  if (warp == pk::kWarpMma) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int BHQ = p.B * p.HQ;
  const int total = p.NB * BHQ;
  const long long Npad = (long long)p.NB * 128;
  auto decode = [&](int idx, int& i, int& bhq, int& b, int& h, int& bhk) {
    // head-major, longest rows first within a head (L2 residency of the head's
    // O / K_new / W / W2 tiles across the CTAs in flight)
    i = p.NB - 1 - idx % p.NB;
    bhq = idx / p.NB;
    b = bhq / p.HQ;
    h = (bhq % p.HQ) / p.G;
    bhk = b * p.H + h;
  };

  if (warp == pk::kWarpTma) {
    if (lane == 0) {
      TileRing<kRing> ring;
      ring.init(sbase + kOffRing, bar(RF0), bar(RE0));
      bool ok = true;
      uint32_t it = 0;
      int last_dv = -1;
      for (int idx = blockIdx.x; idx < total && ok; idx += gridDim.x, ++it) {
        int i, bhq, b, h, bhk;
        decode(idx, i, bhq, b, h, bhk);
        if (!mbar_wait(bar(DV_EMPTY), (it & 1) ^ 1, ab)) break;
        last_dv = (int)(it & 1);
        mbar_arrive_expect_tx(bar(DV_FULL), 32768);
        tma_load_tile(sDV, &tmDV, bar(DV_FULL), i * 128, bhq, 0);
        // per step: O_j, W2_j, K_new_j, W_j.  The MMA warp takes O_{j+1} before it frees
        // W2_j, K_new_j and W_j, which is exactly the ring's four slots
        for (int j = 0; j <= i && ok; ++j) {
          ok = ring.load(&tmO, j * 128, bhq, 0, ab);
          if (ok && j >= 1 && j < i) ok = ring.load(&tmW2, j * 128, bhk, 0, ab);
          if (ok && j < i) ok = ring.load(&tmKn, j * 128, bhk, 0, ab);
          if (ok && j >= 1 && j < i) ok = ring.load(&tmW, j * 128, h, b, ab);
        }
      }
      if (last_dv >= 0) mbar_wait_timed(bar(DV_FULL), (uint32_t)last_dv, kDrainNs);
      ring.drain();
    }
  } else if (warp == pk::kWarpMma) {
    if (lane == 0) {
      uint32_t rc = 0, n_pk = 0, n_dop = 0, n_ns3 = 0, n_dqfree = 0, it = 0;
      auto ring_slot = [&](uint32_t idx) { return sbase + kOffRing + (idx % kRing) * 32768u; };
      auto ring_wait = [&](uint32_t idx) { return mbar_wait(bar(RF0 + (int)(idx % kRing)), (idx / kRing) & 1, ab); };
      auto ring_free = [&](uint32_t idx) { umma_commit(bar(RE0 + (int)(idx % kRing))); };
      const uint32_t tp = tmem + kTmP, ts3 = tmem + kTmS3;
      bool ok = true;
      for (int idx = blockIdx.x; idx < total && ok; idx += gridDim.x, ++it) {
        int i, bhq, b, h, bhk;
        decode(idx, i, bhq, b, h, bhk);
        if (!mbar_wait(bar(DV_FULL), it & 1, ab)) break;
        // slot index of O_j for step j; the other tiles of the step follow it
        auto tiles_of = [&](int j) { return 1 + ((j >= 1 && j < i) ? 1 : 0) + (j < i ? 1 : 0) + ((j >= 1 && j < i) ? 1 : 0); };
        auto issue_p = [&](int j, uint32_t sO) -> bool {  // P_j = dV_i O_j^T into buffer j & 1
          if (!ring_wait(sO)) return false;
          tc_fence_after();
          umma_tile(tp + 128u * (uint32_t)(j & 1), sDV, false, ring_slot(sO), false, 0u);
          umma_commit(bar(P_FULL));
          ring_free(sO);
          return true;
        };
        uint32_t base = rc;
        if (!issue_p(0, base)) break;
        for (int j = 0; j <= i; ++j) {
          const bool has_s3 = (j >= 1 && j < i);
          const uint32_t next = base + (uint32_t)tiles_of(j);
          // P of the next step goes out first: its buffer's previous dA was read by D(j-1)
          if (j + 1 <= i && !issue_p(j + 1, next)) { ok = false; break; }
          uint32_t k = base + 1;
          if (has_s3) {  // chain: S3 = dQ~^{(j-1)} W2_j^T
            if (!mbar_wait(bar(DOP_FULL), (n_dop++) & 1, ab)) { ok = false; break; }
            const uint32_t sW2 = k++;
            if (!ring_wait(sW2)) { ok = false; break; }
            tc_fence_after();
            umma_tile(ts3, sDOP, false, ring_slot(sW2), false, 0u);
            umma_commit(bar(S3_FULL));
            ring_free(sW2);
          }
          if (!mbar_wait(bar(PK_FULL), (n_pk++) & 1, ab)) { ok = false; break; }
          if (j == i) {
            base = next;
            break;
          }
          const uint32_t sK = k++;
          if (!ring_wait(sK)) { ok = false; break; }
          uint32_t sW = 0;
          if (j >= 1) {
            sW = k++;
            if (!ring_wait(sW) || !mbar_wait(bar(NS3_FULL), (n_ns3++) & 1, ab)) { ok = false; break; }
          } else if (!mbar_wait(bar(DQ_FREE), ((n_dqfree++) & 1) ^ 1, ab)) {
            ok = false;  // the previous item's dQ~ has been read out
            break;
          }
          tc_fence_after();
          // dQ~ (TMEM) = [dQ~ +] dA K_new_j [+ (-S3) W_j]; packed operands by full rows (slice kk at 8 kk)
          const uint32_t pj = tp + 128u * (uint32_t)(j & 1);
          umma_tile_ts(tmem + kTmDQ, [&](int kk) { return pj + 8u * (uint32_t)kk; }, ring_slot(sK), true,
                       j > 0 ? 1u : 0u);
          if (j >= 1)
            umma_tile_ts(tmem + kTmDQ, [&](int kk) { return ts3 + 8u * (uint32_t)kk; }, ring_slot(sW), true, 1u);
          umma_commit(bar(DQ_FULL));
          ring_free(sK);
          if (j >= 1) ring_free(sW);
          base = next;
        }
        rc = base;
        if (!ok) break;
        umma_commit(bar(DV_EMPTY));
      }
      umma_commit(bar(DRAIN));
      mbar_wait_timed(bar(DRAIN), 0, kDrainNs);
    }
  } else if (warp < 4) {
    // ---------------- dA tiles ----------------
    const int r = warp * 32 + lane;
    const uint32_t tP0 = tmem + ((uint32_t)(warp * 32) << 16) + kTmP;
    uint32_t n_p = 0;
    bool ok = true;
    for (int idx = blockIdx.x; idx < total && ok; idx += gridDim.x) {
      int i, bhq, b, h, bhk;
      decode(idx, i, bhq, b, h, bhk);
      for (int j = 0; j <= i; ++j) {
        if (!pwarp_wait(bar(P_FULL), (n_p++) & 1, ab)) { ok = false; break; }
        tc_fence_after();
        const uint32_t tP = tP0 + 128u * (uint32_t)(j & 1);
        const long long toff = (j < i) ? ((((long long)bhq * p.NPAIR + path_pair(i, j)) * 128 + r) * 128)
                                       : ((((long long)bhq * p.NB + i) * 128 + r) * 128);
        const bf16* lrow = (j < i ? p.L : p.Ld) + toff;
        bf16* drow = (j < i ? p.dA : p.dAd) + toff;
        for (int c = 0; c < 4; ++c) {
          float pv[32], lv[32];
          tmem_ld32(tP + 32u * c, pv);
#pragma unroll
          for (int e = 0; e < 4; ++e) ld_bf16x8(lrow + c * 32 + e * 8, lv + e * 8);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            float v = -p.s * lv[e] * pv[e];
            if (j == i && c * 32 + e >= r) v = 0.f;
            pv[e] = v;
          }
#pragma unroll
          for (int e = 0; e < 4; ++e) st_bf16x8(drow + c * 32 + e * 8, pv + e * 8);
          if (j < i) {
            uint32_t pk[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) pk[e] = pack_bf16(pv[2 * e], pv[2 * e + 1]);
            // packed columns of chunk c go to [16c, 16c+16): inside chunks already read
            tmem_st16(tP + 16u * (uint32_t)c, pk);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(bar(PK_FULL));
      }
    }
  } else {
    // ---------------- dQ~ chain ----------------
    const int wq = warp - 4;
    const int r = wq * 32 + lane;
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    const uint32_t tS3 = tmem + lane_base + kTmS3, tDQ = tmem + lane_base + kTmDQ;
    uint32_t n_s3 = 0, n_dq = 0, n_qf = 0, n_full = 0;
    auto operand_free = [&]() -> bool {
      if ((int)threadIdx.x == kChainLead) {
        bulk_wait_read_all();
        mbar_arrive(bar(QFREE));
      }
      __syncwarp();
      return pwarp_wait(bar(QFREE), (n_qf++) & 1, ab);
    };
    bool ok = true;
    for (int idx = blockIdx.x; idx < total && ok; idx += gridDim.x) {
      int i, bhq, b, h, bhk;
      decode(idx, i, bhq, b, h, bhk);
      float* dq_row = p.dqn + (((long long)bhq * Npad) + i * 128 + r) * 128;
      if (i == 0) {  // no off-diagonal block: dQ_new of the first row block is zero
        for (int e = 0; e < 128; e += 4) *reinterpret_cast<float4*>(dq_row + e) = make_float4(0.f, 0.f, 0.f, 0.f);
        continue;
      }
      for (int j = 0; j < i; ++j) {
        if (j >= 1) {
          if (!pwarp_wait(bar(S3_FULL), (n_s3++) & 1, ab)) { ok = false; break; }
          tc_fence_after();
          for (int c = 0; c < 4; ++c) {
            float v[32];
            tmem_ld32(tS3 + 32u * c, v);
            tmem_ld_wait();
            uint32_t pk[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) pk[e] = pack_bf16(-v[2 * e], -v[2 * e + 1]);
            tmem_st16(tS3 + 16u * (uint32_t)c, pk);
          }
          tmem_st_wait();
          tc_fence_before();
          mbar_arrive(bar(NS3_FULL));
        }
        if (!pwarp_wait(bar(DQ_FULL), (n_dq++) & 1, ab)) { ok = false; break; }
        tc_fence_after();
        if (j + 1 < i) {
          // dQ~^{(j)}: the operand of step j+1 and the snapshot of pair (i, j+1)
          if (!operand_free()) { ok = false; break; }
          for (int c = 0; c < 4; ++c) {
            float v[32];
            tmem_ld32(tDQ + 32u * c, v);
            tmem_ld_wait();
            tile_store_row32(sDOP, r, c, v);
          }
          fence_proxy_async_smem();
          tc_fence_before();
          mbar_arrive(bar(DOP_FULL));
          if ((int)threadIdx.x == kChainLead) {
            if (mbar_wait(bar(DOP_FULL), n_full & 1, ab)) {
              tma_store_tile(&tmDs, sDOP, (int)(path_pair(i, j + 1) * 128), bhq, 0);
              bulk_commit();
            }
          }
          ++n_full;
          __syncwarp();
        } else {
          for (int c = 0; c < 4; ++c) {
            float v[32];
            tmem_ld32(tDQ + 32u * c, v);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; e += 4)
              *reinterpret_cast<float4*>(dq_row + c * 32 + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
          }
          tc_fence_before();
          mbar_arrive(bar(DQ_FREE));
        }
      }
    }
    if ((int)threadIdx.x == kChainLead) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == pk::kWarpMma) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ===========================================================================
// path_col_kernel
// ===========================================================================
namespace pcl {
constexpr int kRing = 5;
constexpr uint32_t kOffHi = 0, kOffLo = 32768, kOffRing = 65536, kOffBar = kOffRing + kRing * 32768;
enum { RF0 = 0, RE0 = RF0 + kRing, ACC_FULL = RE0 + kRing, PHI_FULL, W_FULL, ACC_FREE, DRAIN, NBAR };
constexpr uint32_t kSmem = kOffBar + NBAR * 8 + 16;
constexpr uint32_t kTmA1 = 0, kTmA2 = 128, kTmW2 = 256, kTmW = 384;
}  // namespace pcl

__global__ void __launch_bounds__(pk::kThreads, 1)
    path_col_kernel(const __grid_constant__ CUtensorMap tmDA, const __grid_constant__ CUtensorMap tmQs,
                    const __grid_constant__ CUtensorMap tmDs, const __grid_constant__ CUtensorMap tmW,
                    const __grid_constant__ CUtensorMap tmW2, PathColArgs p) {
  using namespace pcl;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  auto bar = [&](int i) { return sbase + kOffBar + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffBar + NBAR * 8);
  volatile int* abort_cta = reinterpret_cast<volatile int*>(smem + kOffBar + NBAR * 8 + 4);
  const Abort ab{abort_cta, p.status, kTagPathCol};
  const uint32_t sHi = sbase + kOffHi, sLo = sbase + kOffLo;
  const int warp = warp_id(), lane = lane_id();
  if ((sbase & 1023u) != 0) {
    if (threadIdx.x == 0) atomicCAS(p.status, 0, kStatusMisaligned | (kTagPathCol << 20));
    return;
  }
  if (threadIdx.x == pk::kWarpTma * 32) {
    for (int s = 0; s < kRing; ++s) {
      mbar_init(bar(RF0 + s), 1);
      mbar_init(bar(RE0 + s), 1);
    }
    mbar_init(bar(ACC_FULL), 1);
    mbar_init(bar(PHI_FULL), pk::kEpi);
    mbar_init(bar(W_FULL), 1);
    mbar_init(bar(ACC_FREE), pk::kEpi);
    mbar_init(bar(DRAIN), 1);
    *abort_cta = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmDA);
    tma_prefetch_desc(&tmQs);
    tma_prefetch_desc(&tmDs);
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmW2);
  }
  if (warp == pk::kWarpMma) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int BHQ = p.B * p.HQ;
  const int total = p.NB * BHQ;
  const long long Npad = (long long)p.NB * 128;
  auto decode = [&](int idx, int& j, int& bhq, int& b, int& h, int& bhk, int& steps) {
    j = idx / BHQ;            // longest columns first across all heads
    bhq = idx % BHQ;
    b = bhq / p.HQ;
    h = (bhq % p.HQ) / p.G;
    bhk = b * p.H + h;
    steps = p.NB - 1 - j;
  };

  if (warp == pk::kWarpTma) {
    if (lane == 0) {
      TileRing<kRing> ring;
      ring.init(sbase + kOffRing, bar(RF0), bar(RE0));
      bool ok = true;
      for (int idx = blockIdx.x; idx < total && ok; idx += gridDim.x) {
        int j, bhq, b, h, bhk, steps;
        decode(idx, j, bhq, b, h, bhk, steps);
        if (steps == 0) continue;
        for (int i = j + 1; i < p.NB && ok; ++i) {
          const int row = (int)(path_pair(i, j) * 128);
          ok = ring.load(&tmDA, row, bhq, 0, ab) && ring.load(&tmQs, row, bhq, 0, ab);
          if (ok && j >= 1) ok = ring.load(&tmDs, row, bhq, 0, ab);
        }
        if (ok && j >= 1) ok = ring.load(&tmW, j * 128, h, b, ab) && ring.load(&tmW2, j * 128, bhk, 0, ab);
      }
      ring.drain();
    }
  } else if (warp == pk::kWarpMma) {
    if (lane == 0) {
      uint32_t rc = 0, n_act = 0, n_phi = 0;
      auto ring_slot = [&](uint32_t idx) { return sbase + kOffRing + (idx % kRing) * 32768u; };
      auto ring_wait = [&](uint32_t idx) { return mbar_wait(bar(RF0 + (int)(idx % kRing)), (idx / kRing) & 1, ab); };
      auto ring_free = [&](uint32_t idx) { umma_commit(bar(RE0 + (int)(idx % kRing))); };
      bool ok = true;
      for (int idx = blockIdx.x; idx < total && ok; idx += gridDim.x) {
        int j, bhq, b, h, bhk, steps;
        decode(idx, j, bhq, b, h, bhk, steps);
        if (steps == 0) continue;
        if (!mbar_wait(bar(ACC_FREE), ((n_act++) & 1) ^ 1, ab)) break;
        for (int s = 0; s < steps; ++s) {
          const uint32_t sA = rc++, sQ = rc++;
          if (!ring_wait(sA) || !ring_wait(sQ)) { ok = false; break; }
          uint32_t sD = 0;
          if (j >= 1) {
            sD = rc++;
            if (!ring_wait(sD)) { ok = false; break; }
          }
          tc_fence_after();
          umma_tile(tmem + kTmA1, ring_slot(sA), true, ring_slot(sQ), true, s > 0 ? 1u : 0u);
          if (j >= 1) umma_tile(tmem + kTmA2, ring_slot(sQ), true, ring_slot(sD), true, s > 0 ? 1u : 0u);
          ring_free(sA);
          ring_free(sQ);
          if (j >= 1) ring_free(sD);
        }
        if (!ok) break;
        umma_commit(bar(ACC_FULL));
        if (j >= 1) {
          const uint32_t sW = rc++, sW2 = rc++;
          if (!ring_wait(sW) || !ring_wait(sW2)) break;
          if (!mbar_wait(bar(PHI_FULL), (n_phi++) & 1, ab)) break;
          tc_fence_after();
          umma_tile(tmem + kTmW2, ring_slot(sW), false, sHi, true, 0u);
          umma_tile(tmem + kTmW2, ring_slot(sW), false, sLo, true, 1u);
          umma_tile(tmem + kTmW, ring_slot(sW2), false, sHi, false, 0u);
          umma_tile(tmem + kTmW, ring_slot(sW2), false, sLo, false, 1u);
          umma_commit(bar(W_FULL));
          ring_free(sW);
          ring_free(sW2);
        }
      }
      umma_commit(bar(DRAIN));
      mbar_wait_timed(bar(DRAIN), 0, kDrainNs);
    }
  } else {
    const int qd = warp & 3, hf = warp >> 2;
    const int r = qd * 32 + lane;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const uint32_t t1 = tmem + lane_base + kTmA1 + 64u * hf;
    const uint32_t t2 = tmem + lane_base + kTmA2 + 64u * hf;
    const uint32_t tw2 = tmem + lane_base + kTmW2 + 64u * hf;
    const uint32_t tw = tmem + lane_base + kTmW + 64u * hf;
    uint32_t n_acc = 0, n_w = 0;
    for (int idx = blockIdx.x; idx < total; idx += gridDim.x) {
      int j, bhq, b, h, bhk, steps;
      decode(idx, j, bhq, b, h, bhk, steps);
      const long long off = (((long long)bhq * Npad) + j * 128 + r) * 128 + hf * 64;
      float v[64];
      if (steps == 0 || j == 0) {
#pragma unroll
        for (int e = 0; e < 64; ++e) v[e] = 0.f;
        st_f32x64(p.dw2 + off, v);
        st_f32x64(p.dw + off, v);
        if (steps == 0) {
          st_f32x64(p.dkn + off, v);
          continue;
        }
      }
      if (!pwarp_wait(bar(ACC_FULL), (n_acc++) & 1, ab)) break;
      tc_fence_after();
      tmem_ld64(t1, v);
      st_f32x64(p.dkn + off, v);
      if (j >= 1) {
        float hi[64];
        tmem_ld64(t2, v);
#pragma unroll
        for (int e = 0; e < 64; ++e) {
          hi[e] = __bfloat162float(__float2bfloat16(v[e]));
          v[e] -= hi[e];
        }
        tile_store_row64(sHi, r, hf, hi);
        tile_store_row64(sLo, r, hf, v);
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(bar(PHI_FULL));
        if (!pwarp_wait(bar(W_FULL), (n_w++) & 1, ab)) break;
        tc_fence_after();
        tmem_ld64(tw2, v);
#pragma unroll
        for (int e = 0; e < 64; ++e) v[e] = -v[e];
        st_f32x64(p.dw2 + off, v);
        tmem_ld64(tw, v);
#pragma unroll
        for (int e = 0; e < 64; ++e) v[e] = -v[e];
        st_f32x64(p.dw + off, v);
      }
      tc_fence_before();
      mbar_arrive(bar(ACC_FREE));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == pk::kWarpMma) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------
static int path_num_sms() {
  int dev = 0;
  cudaGetDevice(&dev);
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// cooperative: the grid's CTAs wait on flags published by other CTAs of the grid (the
// wavefront solves), so the launch must place all of them at once
template <typename K, typename... Args>
static cudaError_t launch_persistent(K kernel, uint32_t smem, int total, cudaStream_t st, bool cooperative,
                                     Args... args) {
  if (total <= 0) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int grid = std::min(total, path_num_sms());
  if (cooperative) return launch_cooperative(kernel, grid, pk::kThreads, smem, st, args...);
  kernel<<<grid, pk::kThreads, smem, st>>>(args...);
  return cudaGetLastError();
}

cudaError_t launch_path_scores(const CUtensorMap& tmKn, const CUtensorMap& tmW, const CUtensorMap& tmW2,
                               const CUtensorMap& tmQs, const PathScoresArgs& a, cudaStream_t st) {
  return launch_persistent(path_scores_kernel, psc::kSmem, (a.NB - 1) * a.B * a.HQ, st, false, tmKn, tmW, tmW2, tmQs, a);
}

cudaError_t launch_path_solve(bool transposed, const CUtensorMap& tmL, const CUtensorMap& tmX, const CUtensorMap& tmU,
                              const PathSolveArgs& a, cudaStream_t st) {
  const int total = a.NB * a.B * a.HQ;
  if (transposed) return launch_persistent(path_solve_kernel<true>, psv::kSmem, total, st, true, tmL, tmX, tmU, a);
  return launch_persistent(path_solve_kernel<false>, psv::kSmem, total, st, true, tmL, tmX, tmU, a);
}

cudaError_t launch_path_row(const CUtensorMap& tmDV, const CUtensorMap& tmO, const CUtensorMap& tmKn,
                            const CUtensorMap& tmW, const CUtensorMap& tmW2, const CUtensorMap& tmDs,
                            const PathRowArgs& a, cudaStream_t st) {
  return launch_persistent(path_row_kernel, prw::kSmem, a.NB * a.B * a.HQ, st, false, tmDV, tmO, tmKn, tmW, tmW2, tmDs, a);
}

cudaError_t launch_path_col(const CUtensorMap& tmDA, const CUtensorMap& tmQs, const CUtensorMap& tmDs,
                            const CUtensorMap& tmW, const CUtensorMap& tmW2, const PathColArgs& a, cudaStream_t st) {
  return launch_persistent(path_col_kernel, pcl::kSmem, a.NB * a.B * a.HQ, st, false, tmDA, tmQs, tmDs, tmW, tmW2, a);
}

// ===========================================================================
// path_attn_kernel: PaTH softmax attention forward
// (parallel_path_fwd.py:13-124 + the diagonal blocks of intra_chunk_preprocess_fwd.py)
//   O_r = sum_{c<=r} softmax_c(s A_rc) v_c, lse_r = log2 sum_c exp2(s A_rc log2 e)
// Row block i: the diagonal block's scores come from the prep (raw A_ii, fp32);
// then j = i-1 .. 0 along the query chain:
//   S = Q~ K_new_j^T (Q~ as bf16 hi + lo), online softmax, O += P V_j,
//   Q~ += (-(Q~ W_j^T)) W2_j accumulated by the tensor core in TMEM.
// Warps 0-3 run the softmax (one row per thread), warps 4-7 the query chain.
// ===========================================================================
namespace pat {
constexpr int kRing = 4;
constexpr uint32_t kOffQ = 0, kOffQlo = 32768, kOffRing = 65536, kOffBar = kOffRing + kRing * 32768;
enum { RF0 = 0, RE0 = RF0 + kRing, QOP_FULL = RE0 + kRing, QOP_FREE, S_FULL, S2_FULL, NS2_FULL, QD_FULL, P_FULL,
       O_DONE, O_FREE, DRAIN, NBAR };
constexpr uint32_t kSmem = kOffBar + NBAR * 8 + 16;
constexpr uint32_t kTmS = 0, kTmS2 = 128, kTmQ = 256, kTmO = 384;
constexpr int kHalf = 128;  // threads per warpgroup
}  // namespace pat

__global__ void __launch_bounds__(pk::kThreads, 1)
    path_attn_kernel(const __grid_constant__ CUtensorMap tmKn, const __grid_constant__ CUtensorMap tmW,
                     const __grid_constant__ CUtensorMap tmW2, const __grid_constant__ CUtensorMap tmV,
                     PathAttnArgs p) {
  using namespace pat;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  auto bar = [&](int i) { return sbase + kOffBar + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffBar + NBAR * 8);
  volatile int* abort_cta = reinterpret_cast<volatile int*>(smem + kOffBar + NBAR * 8 + 4);
  const Abort ab{abort_cta, p.status, kTagPathAttn};
  const uint32_t sQ = sbase + kOffQ, sQlo = sbase + kOffQlo;
  const int warp = warp_id(), lane = lane_id();
  if ((sbase & 1023u) != 0) {
    if (threadIdx.x == 0) atomicCAS(p.status, 0, kStatusMisaligned | (kTagPathAttn << 20));
    return;
  }
  if (threadIdx.x == pk::kWarpTma * 32) {
    for (int s = 0; s < kRing; ++s) {
      mbar_init(bar(RF0 + s), 1);
      mbar_init(bar(RE0 + s), 1);
    }
    mbar_init(bar(QOP_FULL), kHalf);
    mbar_init(bar(QOP_FREE), 1);
    mbar_init(bar(S_FULL), 1);
    mbar_init(bar(S2_FULL), 1);
    mbar_init(bar(NS2_FULL), kHalf);
    mbar_init(bar(QD_FULL), 1);
    mbar_init(bar(P_FULL), kHalf);
    mbar_init(bar(O_DONE), 1);
    mbar_init(bar(O_FREE), kHalf);
    mbar_init(bar(DRAIN), 1);
    *abort_cta = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmKn);
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmW2);
    tma_prefetch_desc(&tmV);
  }
  if (warp == pk::kWarpMma) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int BHQ = p.B * p.HQ;
  const int total = p.NB * BHQ;
  const long long Npad = (long long)p.NB * 128;
  auto decode = [&](int idx, int& i, int& bhq, int& b, int& hq, int& h, int& bhk) {
    i = p.NB - 1 - idx % p.NB;  // head-major, longest rows first within a head
    bhq = idx / p.NB;
    b = bhq / p.HQ;
    hq = bhq % p.HQ;
    h = hq / p.G;
    bhk = b * p.H + h;
  };

  if (warp == pk::kWarpTma) {
    if (lane == 0) {
      TileRing<kRing> ring;
      ring.init(sbase + kOffRing, bar(RF0), bar(RE0));
      bool ok = true;
      for (int idx = blockIdx.x; idx < total && ok; idx += gridDim.x) {
        int i, bhq, b, hq, h, bhk;
        decode(idx, i, bhq, b, hq, h, bhk);
        ok = ring.load(&tmV, i * 128, h, b, ab);
        for (int j = i - 1; j >= 0 && ok; --j) {
          ok = ring.load(&tmKn, j * 128, bhk, 0, ab);
          if (ok && j > 0) ok = ring.load(&tmW, j * 128, h, b, ab);
          if (ok) ok = ring.load(&tmV, j * 128, h, b, ab);
          if (ok && j > 0) ok = ring.load(&tmW2, j * 128, bhk, 0, ab);
        }
      }
      ring.drain();
    }
  } else if (warp == pk::kWarpMma) {
    if (lane == 0) {
      uint32_t rc = 0, n_q = 0, n_ns2 = 0, n_p = 0, n_item = 0;
      auto ring_slot = [&](uint32_t idx) { return sbase + kOffRing + (idx % kRing) * 32768u; };
      auto ring_wait = [&](uint32_t idx) { return mbar_wait(bar(RF0 + (int)(idx % kRing)), (idx / kRing) & 1, ab); };
      auto ring_free = [&](uint32_t idx) { umma_commit(bar(RE0 + (int)(idx % kRing))); };
      const uint32_t tS = tmem + kTmS, tS2 = tmem + kTmS2;
      auto pv = [&](uint32_t sv, uint32_t acc) -> bool {
        if (!mbar_wait(bar(P_FULL), (n_p++) & 1, ab) || !ring_wait(sv)) return false;
        tc_fence_after();
        umma_tile_ts(tmem + kTmO, [&](int kk) { return tS + 8u * (uint32_t)kk; }, ring_slot(sv), true, acc);
        umma_commit(bar(O_DONE));
        ring_free(sv);
        return true;
      };
      bool ok = true;
      for (int idx = blockIdx.x; idx < total && ok; idx += gridDim.x, ++n_item) {
        int i, bhq, b, hq, h, bhk;
        decode(idx, i, bhq, b, hq, h, bhk);
        if (!mbar_wait(bar(O_FREE), (n_item & 1) ^ 1, ab)) break;
        if (!pv(rc++, 0u)) break;                        // diagonal block
        for (int j = i - 1; j >= 0; --j) {
          if (!mbar_wait(bar(QOP_FULL), (n_q++) & 1, ab)) { ok = false; break; }
          const uint32_t sK = rc++;
          if (!ring_wait(sK)) { ok = false; break; }
          uint32_t sW = 0;
          if (j > 0) {
            sW = rc++;
            if (!ring_wait(sW)) { ok = false; break; }
          }
          tc_fence_after();
          if (j > 0) {
            umma_tile(tS2, sQ, false, ring_slot(sW), false, 0u);
            umma_commit(bar(S2_FULL));
          }
          umma_tile(tS, sQ, false, ring_slot(sK), false, 0u);
          umma_tile(tS, sQlo, false, ring_slot(sK), false, 1u);
          umma_commit(bar(S_FULL));
          if (j == 0) umma_commit(bar(QOP_FREE));
          ring_free(sK);
          if (j > 0) ring_free(sW);
          const uint32_t sV = rc++;
          if (j > 0) {
            if (!mbar_wait(bar(NS2_FULL), (n_ns2++) & 1, ab)) { ok = false; break; }
            const uint32_t sW2 = rc++;
            if (!ring_wait(sW2)) { ok = false; break; }
            tc_fence_after();
            // -S2 was packed by full rows: K-slice kk at column 8 kk
            umma_tile_ts(tmem + kTmQ, [&](int kk) { return tS2 + 8u * (uint32_t)kk; }, ring_slot(sW2), true, 1u);
            umma_commit(bar(QD_FULL));
            ring_free(sW2);
          }
          if (!pv(sV, 1u)) { ok = false; break; }
        }
      }
      umma_commit(bar(DRAIN));
      mbar_wait_timed(bar(DRAIN), 0, kDrainNs);
    }
  } else if (warp < 4) {
    // ---------------- softmax warpgroup ----------------
    const int r = warp * 32 + lane;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const uint32_t tS = tmem + lane_base + kTmS, tO = tmem + lane_base + kTmO;
    const float sm = p.s * 1.4426950408889634f;
    uint32_t n_s = 0, n_pv = 0;
    auto store_p = [&](float (&v)[32], int c) {
      uint32_t pk[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) pk[e] = pack_bf16(v[2 * e], v[2 * e + 1]);
      tmem_st16(tS + 16u * (uint32_t)c, pk);
    };
    for (int idx = blockIdx.x; idx < total; idx += gridDim.x) {
      int i, bhq, b, hq, h, bhk;
      decode(idx, i, bhq, b, hq, h, bhk);
      float m_run, l_run = 0.f;
      bool ok = true;
      {  // diagonal block from the prep's raw scores (causal within the block)
        const float* arow = p.ad + (((long long)bhq * p.NB + i) * 128 + r) * 128;
        float mx = -INFINITY;
        for (int c = 0; c < 4; ++c) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (c * 32 + e <= r) mx = fmaxf(mx, arow[c * 32 + e] * sm);
        }
        m_run = mx;
        for (int c = 0; c < 4; ++c) {
          float v[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            v[e] = (c * 32 + e <= r) ? fast_exp2(arow[c * 32 + e] * sm - m_run) : 0.f;
            l_run += v[e];
          }
          store_p(v, c);
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(bar(P_FULL));
        ++n_pv;
      }
      for (int j = i - 1; j >= 0; --j) {
        if (!pwarp_wait(bar(S_FULL), (n_s++) & 1, ab)) { ok = false; break; }
        tc_fence_after();
        float mx = -INFINITY;
        for (int c = 0; c < 4; ++c) {
          float v[32];
          tmem_ld32(tS + 32u * c, v);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) mx = fmaxf(mx, v[e] * sm);
        }
        // lazy rescale: every P V issued so far has completed (S of this step was
        // issued after the last one), so O can be rescaled in place
        if (__any_sync(0xffffffffu, mx > m_run + 8.f)) {
          const float mn = fmaxf(m_run, mx);
          const float alpha = fast_exp2(m_run - mn);
          for (int c = 0; c < 4; ++c) {
            float ov[32];
            tmem_ld32(tO + 32u * c, ov);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) ov[e] *= alpha;
            tmem_st32(tO + 32u * c, ov);
          }
          tmem_st_wait();
          l_run *= alpha;
          m_run = mn;
        }
        for (int c = 0; c < 4; ++c) {
          float v[32];
          tmem_ld32(tS + 32u * c, v);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            v[e] = fast_exp2(fmaf(v[e], sm, -m_run));
            l_run += v[e];
          }
          store_p(v, c);
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(bar(P_FULL));
        ++n_pv;
      }
      if (!ok) break;
      if (!pwarp_wait(bar(O_DONE), (n_pv - 1) & 1, ab)) break;
      tc_fence_after();
      const long long t = (long long)i * 128 + r;
      const float inv_l = 1.f / l_run;
      for (int c = 0; c < 4; ++c) {
        float ov[32];
        tmem_ld32(tO + 32u * c, ov);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) ov[e] *= inv_l;
        if (t < p.T) {
          bf16* dst = p.o + (long long)b * p.o_sb + t * p.o_st + (long long)hq * p.o_sh + c * 32;
#pragma unroll
          for (int e = 0; e < 4; ++e) st_bf16x8(dst + 8 * e, ov + 8 * e);
        }
      }
      if (t < p.T) p.lse[(long long)b * p.l_sb + t * p.l_st + (long long)hq * p.l_sh] = m_run + __log2f(l_run);
      tc_fence_before();
      mbar_arrive(bar(O_FREE));
    }
  } else {
    // ---------------- query-chain warpgroup ----------------
    const int wq = warp - 4;
    const int r = wq * 32 + lane;
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    const uint32_t tS2 = tmem + lane_base + kTmS2, tQ = tmem + lane_base + kTmQ;
    uint32_t n_s2 = 0, n_qd = 0, n_free = 0;
    bool first = true;
    // bf16 hi / lo operand copies of Q~ (read from registers or TMEM in 32-column chunks)
    auto write_op = [&](int c, const float (&v)[32]) {
      float hi[32], lo[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        hi[e] = __bfloat162float(__float2bfloat16(v[e]));
        lo[e] = v[e] - hi[e];
      }
      tile_store_row32(sQ, r, c, hi);
      tile_store_row32(sQlo, r, c, lo);
    };
    for (int idx = blockIdx.x; idx < total; idx += gridDim.x) {
      int i, bhq, b, hq, h, bhk;
      decode(idx, i, bhq, b, hq, h, bhk);
      if (i == 0) continue;
      bool ok = true;
      // the previous item's last score GEMM has finished reading the operand tiles
      if (!first && !pwarp_wait(bar(QOP_FREE), (n_free++) & 1, ab)) break;
      first = false;
      {
        const float* src = p.qn + (((long long)bhq * Npad) + i * 128 + r) * 128;
        for (int c = 0; c < 4; ++c) {
          float v[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = src[c * 32 + e];
          tmem_st32(tQ + 32u * c, v);
          write_op(c, v);
        }
        tmem_st_wait();
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(bar(QOP_FULL));
      }
      for (int j = i - 1; j >= 1; --j) {
        if (!pwarp_wait(bar(S2_FULL), (n_s2++) & 1, ab)) { ok = false; break; }
        tc_fence_after();
        for (int c = 0; c < 4; ++c) {
          float v[32];
          tmem_ld32(tS2 + 32u * c, v);
          tmem_ld_wait();
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) pk[e] = pack_bf16(-v[2 * e], -v[2 * e + 1]);
          // packed columns of chunk c go to [16c, 16c+16): inside chunks already read
          tmem_st16(tS2 + 16u * (uint32_t)c, pk);
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(bar(NS2_FULL));
        if (!pwarp_wait(bar(QD_FULL), (n_qd++) & 1, ab)) { ok = false; break; }
        tc_fence_after();
        for (int c = 0; c < 4; ++c) {
          float v[32];
          tmem_ld32(tQ + 32u * c, v);
          tmem_ld_wait();
          write_op(c, v);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(bar(QOP_FULL));
      }
      if (!ok) break;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == pk::kWarpMma) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

cudaError_t launch_path_attn(const CUtensorMap& tmKn, const CUtensorMap& tmW, const CUtensorMap& tmW2,
                             const CUtensorMap& tmV, const PathAttnArgs& a, cudaStream_t st) {
  return launch_persistent(path_attn_kernel, pat::kSmem, a.NB * a.B * a.HQ, st, false, tmKn, tmW, tmW2, tmV, a);
}

}  // namespace lb
