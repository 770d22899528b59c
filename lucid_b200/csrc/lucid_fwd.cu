// Forward tile engine: one persistent, warp-specialised tcgen05 kernel
// template that runs the two causal row-block loops of the LUCID forward.
//
//   SOLVE  (modeling_lucid.py:566-570, and the blockwise form :285-302)
//     X = P^-1 V,  P = tril(exp(s K^K^T - 1/s))
//     Row block i:  R_i = V_i - sum_{j<i} exp(s K^_i K^_j^T - 1/s) X_j
//                   Y   = D_i^-1 R_i ;  X_i = Y + U_i Y
//     Blocks are processed as a wavefront: work item (i, head) waits on a
//     global flag for every X_j (j < i) it consumes and publishes X_i.
//
//   ATTN   (modeling_lucid.py:505-549)
//     O = softmax(scale Q K^T + causal) X   (raw K, X from SOLVE), with the
//     row log-sum-exp kept for the backward.  Grouped-query heads index
//     kv head = q head / (Hq / Hkv)  (repeat_kv, modeling_lucid.py:523-524).
//
// Warp roles (192 threads): warps 0-3 own one tile row each thread (the 128
// TMEM lanes), warp 4 issues TMA, warp 5 issues tcgen05.mma.  Per tile j:
//   S   = A_i B_j^T            (TMEM, double-buffered)
//   P   = f(S)   -> bf16 smem  (epilogue warps)
//   acc = acc + P C_j          (TMEM accumulator)
// with A = K^ (solve) or Q (attention), B = K^ or K, C = X.
#include "lucid_common.cuh"

#include <algorithm>

namespace lb {

namespace fwd {
constexpr int kThreads = 192;
// shared-memory map (bytes from the 1024-aligned base)
constexpr uint32_t kOffA = 0;
constexpr uint32_t kOffStage = 32768;        // stage s: B tile at +s*65536, C tile at +32768
constexpr uint32_t kOffP = 32768 + 2 * 65536;  // P / Y buffers: 2 x 32 KB
constexpr uint32_t kOffBar = kOffP + 2 * 32768;
enum {
  A_FULL = 0, A_EMPTY, KV_FULL0, KV_FULL1, KV_EMPTY0, KV_EMPTY1, S_FULL0, S_FULL1,
  S_FREE0, S_FREE1, P_FULL0, P_FULL1, P_FREE0, P_FREE1, ACC_FULL, ACC_FREE, EPI_DONE, DRAIN, NBAR
};
constexpr uint32_t kSmemBytes = kOffBar + NBAR * 8 + 16 + 1024;  // + alignment slack
// TMEM columns
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemS0 = 0, kTmemAcc = 256;
}  // namespace fwd

__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, const Abort& ab) {
  const bool ok = mbar_wait(bar, parity, ab);
  return __all_sync(0xffffffffu, ok);
}

template <bool SOLVE>
__global__ void __launch_bounds__(fwd::kThreads, 1)
    lucid_fwd_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmU,
                     FwdArgs p) {
  using namespace fwd;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (sbase - raw);
  const uint32_t bar0 = sbase + kOffBar;
  auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffBar + NBAR * 8);
  volatile int* abort_cta = reinterpret_cast<volatile int*>(smem + kOffBar + NBAR * 8 + 4);
  const Abort ab{abort_cta, p.status, SOLVE ? kTagFwdSolve : kTagFwdAttn};

  const int warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 128) {
    mbar_init(bar(A_FULL), 1);
    mbar_init(bar(A_EMPTY), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(KV_FULL0 + s), 1);
      mbar_init(bar(KV_EMPTY0 + s), 1);
      mbar_init(bar(S_FULL0 + s), 1);
      mbar_init(bar(S_FREE0 + s), 128);
      mbar_init(bar(P_FULL0 + s), 128);
      mbar_init(bar(P_FREE0 + s), 1);
    }
    mbar_init(bar(ACC_FULL), 1);
    mbar_init(bar(ACC_FREE), 128);
    mbar_init(bar(EPI_DONE), 128);
    mbar_init(bar(DRAIN), 1);
    *abort_cta = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
    if (SOLVE) tma_prefetch_desc(&tmU);
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int BHk = p.B * p.Hkv, BHq = p.B * p.Hq;
  const int G = p.Hq / p.Hkv;
  const int total = SOLVE ? p.NB * BHk : p.NB * BHq;

  // Decode a work item.  Solve: increasing block index (wavefront order).
  // Attention: longest rows first.
  auto decode = [&](int idx, int& i, int& b, int& ha, int& hk) {
    if (SOLVE) {
      i = idx / BHk;
      const int bh = idx % BHk;
      b = bh / p.Hkv;
      hk = bh % p.Hkv;
      ha = hk;
    } else {
      i = p.NB - 1 - idx / BHq;
      const int bh = idx % BHq;
      b = bh / p.Hq;
      ha = bh % p.Hq;
      hk = ha / G;
    }
  };

  if (warp == 4) {
    // ======================= TMA producer =======================
    if (lane == 0) {
      uint32_t g = 0, it = 0;
      int last_a = -1, last_kv[2] = {-1, -1};  // parity of the newest load per barrier
      for (int idx = blockIdx.x; idx < total; idx += gridDim.x, ++it) {
        int i, b, ha, hk;
        decode(idx, i, b, ha, hk);
        const int T = SOLVE ? i : i + 1;
        if (!mbar_wait(bar(A_EMPTY), (it & 1) ^ 1, ab)) break;
        last_a = it & 1;
        mbar_arrive_expect_tx(bar(A_FULL), 32768);
        tma_load_tile(sbase + kOffA, &tmA, bar(A_FULL), i * 128, ha, b);
        bool ok = true;
        for (int t = 0; t < T && ok; ++t, ++g) {
          const int st = g & 1;
          const uint32_t ph = (g >> 1) & 1;
          if (SOLVE) {
            if (!wait_flag_geq(&p.flags[(b * p.Hkv + hk) * p.NB + t], 1, ab)) { ok = false; break; }
            fence_proxy_async_global();
          }
          if (!mbar_wait(bar(KV_EMPTY0 + st), ph ^ 1, ab)) { ok = false; break; }
          last_kv[st] = (int)ph;
          mbar_arrive_expect_tx(bar(KV_FULL0 + st), 65536);
          const uint32_t dst = sbase + kOffStage + (uint32_t)st * 65536u;
          tma_load_tile(dst, &tmB, bar(KV_FULL0 + st), t * 128, hk, b);
          tma_load_tile(dst + 32768, &tmC, bar(KV_FULL0 + st), t * 128, hk, b);
        }
        if (!ok) break;
        if (SOLVE) {
          const int st = g & 1;
          const uint32_t ph = (g >> 1) & 1;
          if (!mbar_wait(bar(KV_EMPTY0 + st), ph ^ 1, ab)) break;
          last_kv[st] = (int)ph;
          mbar_arrive_expect_tx(bar(KV_FULL0 + st), 32768);
          tma_load_tile(sbase + kOffStage + (uint32_t)st * 65536u, &tmU, bar(KV_FULL0 + st),
                        i * 128, hk, b);
          ++g;
        }
      }
      // never leave with a TMA write into shared memory still in flight
      if (last_a >= 0) mbar_wait_timed(bar(A_FULL), (uint32_t)last_a, kDrainNs);
      for (int s2 = 0; s2 < 2; ++s2)
        if (last_kv[s2] >= 0) mbar_wait_timed(bar(KV_FULL0 + s2), (uint32_t)last_kv[s2], kDrainNs);
    }
  } else if (warp == 5) {
    // ======================= MMA issuer =======================
    if (lane == 0) {
      uint32_t g = 0, it = 0;
      bool ok = true;
      auto issue_pv = [&](uint32_t gg, int t) -> bool {
        const int st = gg & 1;
        const uint32_t ph = (gg >> 1) & 1;
        if (!mbar_wait(bar(P_FULL0 + st), ph, ab)) return false;
        if (t == 0 && !mbar_wait(bar(ACC_FREE), (it & 1) ^ 1, ab)) return false;
        tc_fence_after();
        umma_tile(tmem + kTmemAcc, sbase + kOffP + (uint32_t)st * 32768u, false,
                  sbase + kOffStage + (uint32_t)st * 65536u + 32768u, true, t > 0 ? 1u : 0u);
        umma_commit(bar(P_FREE0 + st));
        umma_commit(bar(KV_EMPTY0 + st));
        return true;
      };
      for (int idx = blockIdx.x; idx < total && ok; idx += gridDim.x, ++it) {
        int i, b, ha, hk;
        decode(idx, i, b, ha, hk);
        const int T = SOLVE ? i : i + 1;
        if (!mbar_wait(bar(A_FULL), it & 1, ab)) break;
        tc_fence_after();
        for (int t = 0; t < T; ++t) {
          const uint32_t gg = g + t;
          const int st = gg & 1;
          const uint32_t ph = (gg >> 1) & 1;
          if (!mbar_wait(bar(KV_FULL0 + st), ph, ab) || !mbar_wait(bar(S_FREE0 + st), ph ^ 1, ab)) {
            ok = false;
            break;
          }
          tc_fence_after();
          umma_tile(tmem + kTmemS0 + (uint32_t)st * 128u, sbase + kOffA, false,
                    sbase + kOffStage + (uint32_t)st * 65536u, false, 0u);
          umma_commit(bar(S_FULL0 + st));
          if (t == T - 1) umma_commit(bar(A_EMPTY));
          if (t >= 1 && !issue_pv(gg - 1, t - 1)) { ok = false; break; }
        }
        if (!ok) break;
        if (T >= 1) {
          if (!issue_pv(g + T - 1, T - 1)) break;
        } else {
          if (!mbar_wait(bar(ACC_FREE), (it & 1) ^ 1, ab)) break;
          umma_commit(bar(A_EMPTY));
        }
        umma_commit(bar(ACC_FULL));
        g += T;
        if (SOLVE) {
          // diagonal block: T = U_i * Y  (U from the stage's B slot, Y from the P buffer)
          const int st = g & 1;
          const uint32_t ph = (g >> 1) & 1;
          if (!mbar_wait(bar(KV_FULL0 + st), ph, ab) || !mbar_wait(bar(S_FREE0 + st), ph ^ 1, ab) ||
              !mbar_wait(bar(P_FULL0 + st), ph, ab))
            break;
          tc_fence_after();
          umma_tile(tmem + kTmemS0 + (uint32_t)st * 128u, sbase + kOffStage + (uint32_t)st * 65536u,
                    false, sbase + kOffP + (uint32_t)st * 32768u, true, 0u);
          umma_commit(bar(S_FULL0 + st));
          umma_commit(bar(KV_EMPTY0 + st));
          umma_commit(bar(P_FREE0 + st));
          ++g;
        }
      }
      // drain: no MMA may be in flight when TMEM is released
      umma_commit(bar(DRAIN));
      mbar_wait_timed(bar(DRAIN), 0, kDrainNs);
    }
  } else {
    // ======================= epilogue warps 0-3 =======================
    const int r = threadIdx.x;  // tile row == TMEM lane
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const float kLog2e = 1.4426950408889634f;
    const float c1 = p.scale * kLog2e;               // S -> log2 domain
    const float c2 = kLog2e / p.scale;               // 1/s in log2 domain (solve)
    uint32_t g = 0, it = 0;
    for (int idx = blockIdx.x; idx < total; idx += gridDim.x, ++it) {
      int i, b, ha, hk;
      decode(idx, i, b, ha, hk);
      const int T = SOLVE ? i : i + 1;
      float m_run = -INFINITY, l_run = 0.f;
      bool ok = true;
      for (int t = 0; t < T; ++t, ++g) {
        const int st = g & 1;
        const uint32_t ph = (g >> 1) & 1;
        if (!warp_wait(bar(S_FULL0 + st), ph, ab)) { ok = false; break; }
        tc_fence_after();
        float sv[4][32];
        const uint32_t ts = tmem + lane_base + kTmemS0 + (uint32_t)st * 128u;
#pragma unroll
        for (int q = 0; q < 4; ++q) tmem_ld32(ts + 32u * q, sv[q]);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(bar(S_FREE0 + st));
        if (SOLVE) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int e = 0; e < 32; ++e) sv[q][e] = fast_exp2(fmaf(sv[q][e], c1, -c2));
        } else {
          const bool diag = (t == i);
          float mx = -INFINITY;
#pragma unroll
          for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              float v = sv[q][e] * c1;
              if (diag && (q * 32 + e) > r) v = -INFINITY;
              sv[q][e] = v;
              mx = fmaxf(mx, v);
            }
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
            // acc must be stable: wait for the previous tile's P*C product
            const uint32_t gp = g - 1;
            if (!warp_wait(bar(P_FREE0 + (gp & 1)), (gp >> 1) & 1, ab)) { ok = false; break; }
            tc_fence_after();
            const uint32_t ta = tmem + lane_base + kTmemAcc;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              float av[32];
              tmem_ld32(ta + 32u * q, av);
              tmem_ld_wait();
#pragma unroll
              for (int e = 0; e < 32; ++e) av[e] *= alpha;
              tmem_st32(ta + 32u * q, av);
            }
            tmem_st_wait();
          }
          l_run *= alpha;
          float sum = 0.f;
#pragma unroll
          for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const float pe = fast_exp2(sv[q][e] - m_run);
              sv[q][e] = pe;
              sum += pe;
            }
          l_run += sum;
        }
        if (!warp_wait(bar(P_FREE0 + st), ph ^ 1, ab)) { ok = false; break; }
        const uint32_t pbuf = sbase + kOffP + (uint32_t)st * 32768u;
#pragma unroll
        for (int q = 0; q < 4; ++q) tile_store_row32(pbuf, r, q, sv[q]);
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(bar(P_FULL0 + st));
      }
      if (!ok) break;
      if (!warp_wait(bar(ACC_FULL), it & 1, ab)) break;
      tc_fence_after();
      float acc[4][32];
      const uint32_t ta = tmem + lane_base + kTmemAcc;
      if (T > 0) {
#pragma unroll
        for (int q = 0; q < 4; ++q) tmem_ld32(ta + 32u * q, acc[q]);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int e = 0; e < 32; ++e) acc[q][e] = 0.f;
      }
      tc_fence_before();
      mbar_arrive(bar(ACC_FREE));
      const int row = i * 128 + r;
      if (SOLVE) {
        // Y = D^-1 (V - acc), kept in fp32 registers and staged as bf16 for U*Y
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
        const int st = g & 1;
        const uint32_t ph = (g >> 1) & 1;
        if (!warp_wait(bar(P_FREE0 + st), ph ^ 1, ab)) break;
        const uint32_t pbuf = sbase + kOffP + (uint32_t)st * 32768u;
#pragma unroll
        for (int q = 0; q < 4; ++q) tile_store_row32(pbuf, r, q, acc[q]);
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(bar(P_FULL0 + st));
        if (!warp_wait(bar(S_FULL0 + st), ph, ab)) break;
        tc_fence_after();
        bf16* xrow = p.x + (bhk * p.Npad + row) * kHeadDim;
        const uint32_t ts = tmem + lane_base + kTmemS0 + (uint32_t)st * 128u;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float tv[32];
          tmem_ld32(ts + 32u * q, tv);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) tv[e] += acc[q][e];
#pragma unroll
          for (int c = 0; c < 4; ++c) st_bf16x8(xrow + q * 32 + c * 8, tv + c * 8);
        }
        tc_fence_before();
        mbar_arrive(bar(S_FREE0 + st));
        ++g;
        fence_proxy_async_global();
        __threadfence();
        mbar_arrive(bar(EPI_DONE));
        if (r == 0) {
          if (mbar_wait(bar(EPI_DONE), it & 1, ab)) st_release_gpu(&p.flags[bhk * p.NB + i], 1);
        }
        __syncwarp();
      } else {
        const float inv_l = 1.f / l_run;
        if (row < p.N) {
          bf16* orow = p.o + (long long)b * p.o_sb + (long long)ha * p.o_sh + (long long)row * p.o_sn;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
#pragma unroll
            for (int e = 0; e < 32; ++e) acc[q][e] *= inv_l;
#pragma unroll
            for (int c = 0; c < 4; ++c) st_bf16x8(orow + q * 32 + c * 8, acc[q] + c * 8);
          }
        }
        p.lse[((long long)b * p.Hq + ha) * p.Npad + row] = m_run + __log2f(l_run);
      }
    }
  }

  // ---- teardown: every role is done (or aborted); release TMEM ----
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
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
  const int total = solve ? a.NB * a.B * a.Hkv : a.NB * a.B * a.Hq;
  if (total == 0) return cudaSuccess;
  const int grid = std::min(total, num_sms());
  cudaError_t e;
  if (solve) {
    e = cudaFuncSetAttribute(lucid_fwd_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)fwd::kSmemBytes);
    if (e != cudaSuccess) return e;
    lucid_fwd_kernel<true><<<grid, fwd::kThreads, fwd::kSmemBytes, st>>>(tA, tB, tC, tU, a);
  } else {
    e = cudaFuncSetAttribute(lucid_fwd_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)fwd::kSmemBytes);
    if (e != cudaSuccess) return e;
    lucid_fwd_kernel<false><<<grid, fwd::kThreads, fwd::kSmemBytes, st>>>(tA, tB, tC, tU, a);
  }
  return cudaGetLastError();
}

}  // namespace lb
