// Backward tile engine: one persistent, warp-specialised tcgen05 kernel
// template for the two column-oriented loops of the LUCID backward.
//
//   ATTN  (backward of modeling_lucid.py:505-549, O = softmax(s Q K^T) X)
//     column = key block i of kv head hk; tiles = (query head g of the
//     group, query block j >= i).  With A1 = K_i, A2 = X_i, B1 = Q_j,
//     B2 = dO_j:
//       S^T = A1 B1^T, P = exp2(S^T s log2e - lse_j)      (causal mask)
//       dP^T = A2 B2^T, dS = P (dP^T - delta_j)
//       dX_i += P B2 ;  dK_i += dS B1 ;  dQ_j += dS^T A1 (fp32 atomics)
//
//   SOLVE (backward of X = P^-1 V, modeling_lucid.py:314-382)
//     column = block i; tiles j = NB-1 .. i+1 (waiting for dV_j); with
//     A1 = K^_i, A2 = X_i, B1 = K^_j, B2 = dV_j:
//       E = exp(s A1 B1^T - 1/s),  D = A2 B2^T,  dG^T = -s E o D
//       acc_i += E B2 ;  dK^_i += dG^T B1 ;  dK^_j += dG A1 (fp32 atomics)
//     then the diagonal block:
//       R = dX_i - acc_i ;  dV_i = D_i^-1 (R + U_i^T R)   (publish flag)
//       dG_ii (strictly lower) and  dK^_i += dG_ii^T K^_i + dG_ii K^_i.
//     The diagonal entries P_rr are handled exactly in fp32 by the
//     finalize kernel.
//
// Warp roles as in the forward: warps 0-3 epilogue (thread = tile row),
// warp 4 TMA producer, warp 5 MMA issuer.  TMEM: S/T 0, dP 128, acc1 256,
// acc2 384.
#include "lucid_common.cuh"

#include <algorithm>

namespace lb {

namespace bwd {
constexpr int kThreads = 192;
constexpr uint32_t kOffA1 = 0, kOffA2 = 32768, kOffB1 = 65536, kOffB2 = 98304;
constexpr uint32_t kOffP = 131072, kOffDS = 163840, kOffVec = 196608;  // vec: lse[128], delta[128]
constexpr uint32_t kOffBar = kOffVec + 1024;
enum {
  A_FULL = 0, A_EMPTY, KV_FULL, KV_EMPTY, SD_FULL, DP_FREE, PD_FULL, PD_FREE, T_FULL, T_FREE,
  ACC_FULL, ACC2_FULL, ACC_FREE, EPI_DONE, DRAIN, NBAR
};
constexpr uint32_t kSmemBytes = kOffBar + NBAR * 8 + 16 + 1024;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmS = 0, kTmDP = 128, kTmAcc1 = 256, kTmAcc2 = 384;
}  // namespace bwd

// Phase bookkeeping for one mbarrier as seen by one role.
struct Ph {
  uint32_t n = 0;
  __device__ __forceinline__ uint32_t full() { return (n++) & 1u; }          // k-th completion
  __device__ __forceinline__ uint32_t empty() { return ((n++) & 1u) ^ 1u; }  // (k-1)-th completion
};

__device__ __forceinline__ bool warp_wait_b(uint32_t bar, uint32_t parity, const Abort& ab) {
  const bool ok = mbar_wait(bar, parity, ab);
  return __all_sync(0xffffffffu, ok);
}

template <bool SOLVE>
__global__ void __launch_bounds__(bwd::kThreads, 1)
    lucid_bwd_kernel(const __grid_constant__ CUtensorMap tmA1, const __grid_constant__ CUtensorMap tmA2,
                     const __grid_constant__ CUtensorMap tmB1, const __grid_constant__ CUtensorMap tmB2,
                     const __grid_constant__ CUtensorMap tmU, BwdArgs p) {
  using namespace bwd;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (sbase - raw);
  const uint32_t bar0 = sbase + kOffBar;
  auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffBar + NBAR * 8);
  volatile int* abort_cta = reinterpret_cast<volatile int*>(smem + kOffBar + NBAR * 8 + 4);
  const float* svec = reinterpret_cast<const float*>(smem + kOffVec);
  const Abort ab{abort_cta, p.status};
  const uint32_t sA1 = sbase + kOffA1, sA2 = sbase + kOffA2, sB1 = sbase + kOffB1,
                 sB2 = sbase + kOffB2, sP = sbase + kOffP, sDS = sbase + kOffDS;

  const int warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 128) {
    mbar_init(bar(A_FULL), 1);
    mbar_init(bar(A_EMPTY), 1);
    mbar_init(bar(KV_FULL), 1);
    mbar_init(bar(KV_EMPTY), 1);
    mbar_init(bar(SD_FULL), 1);
    mbar_init(bar(DP_FREE), 128);
    mbar_init(bar(PD_FULL), 128);
    mbar_init(bar(PD_FREE), 1);
    mbar_init(bar(T_FULL), 1);
    mbar_init(bar(T_FREE), 128);
    mbar_init(bar(ACC_FULL), 1);
    mbar_init(bar(ACC2_FULL), 1);
    mbar_init(bar(ACC_FREE), 128);
    mbar_init(bar(EPI_DONE), 128);
    mbar_init(bar(DRAIN), 1);
    *abort_cta = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA1);
    tma_prefetch_desc(&tmA2);
    tma_prefetch_desc(&tmB1);
    tma_prefetch_desc(&tmB2);
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

  const int BHk = p.B * p.Hkv;
  const int G = p.Hq / p.Hkv;
  const int total = p.NB * BHk;
  auto decode = [&](int idx, int& i, int& b, int& hk) {
    i = SOLVE ? (p.NB - 1 - idx / BHk) : (idx / BHk);
    const int bh = idx % BHk;
    b = bh / p.Hkv;
    hk = bh % p.Hkv;
  };
  // number of off-diagonal (solve) / all (attention) tiles of column i
  auto ntiles = [&](int i) { return SOLVE ? (p.NB - 1 - i) : G * (p.NB - i); };
  // tile t of column i -> (query head offset g, row block j)
  auto tile_at = [&](int i, int t, int& g, int& j) {
    if (SOLVE) {
      g = 0;
      j = p.NB - 1 - t;
    } else {
      const int per = p.NB - i;
      g = t / per;
      j = i + t % per;
    }
  };

  if (warp == 4) {
    // ======================= TMA producer =======================
    if (lane == 0) {
      Ph a_empty, kv_empty;
      int last_a = -1, last_kv = -1;
      uint32_t n_a = 0, n_kv = 0;
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
        for (int t = 0; t < T; ++t) {
          int g, j;
          tile_at(i, t, g, j);
          if (SOLVE) {
            if (!wait_flag_geq(&p.flags[(b * p.Hkv + hk) * p.NB + j], 1, ab)) { ok = false; break; }
            fence_proxy_async_global();
          }
          if (!mbar_wait(bar(KV_EMPTY), kv_empty.empty(), ab)) { ok = false; break; }
          last_kv = n_kv++ & 1;
          if (SOLVE) {
            mbar_arrive_expect_tx(bar(KV_FULL), 65536);
            tma_load_tile(sB1, &tmB1, bar(KV_FULL), j * 128, hk, b);
            tma_load_tile(sB2, &tmB2, bar(KV_FULL), j * 128, hk, b);
          } else {
            const int hq = hk * G + g;
            const long long voff = ((long long)b * p.Hq + hq) * p.Npad + (long long)j * 128;
            mbar_arrive_expect_tx(bar(KV_FULL), 65536 + 1024);
            tma_load_tile(sB1, &tmB1, bar(KV_FULL), j * 128, hq, b);
            tma_load_tile(sB2, &tmB2, bar(KV_FULL), j * 128, hq, b);
            bulk_load(sbase + kOffVec, p.lse + voff, 512, bar(KV_FULL));
            bulk_load(sbase + kOffVec + 512, p.delta + voff, 512, bar(KV_FULL));
          }
        }
        if (!ok) break;
        if (SOLVE) {
          if (!mbar_wait(bar(KV_EMPTY), kv_empty.empty(), ab)) break;
          last_kv = n_kv++ & 1;
          mbar_arrive_expect_tx(bar(KV_FULL), 32768);
          tma_load_tile(sB1, &tmU, bar(KV_FULL), i * 128, hk, b);
        }
      }
      if (last_a >= 0) mbar_wait_timed(bar(A_FULL), (uint32_t)last_a, kDrainNs);
      if (last_kv >= 0) mbar_wait_timed(bar(KV_FULL), (uint32_t)last_kv, kDrainNs);
    }
  } else if (warp == 5) {
    // ======================= MMA issuer =======================
    if (lane == 0) {
      Ph a_full, kv_full, t_free, dp_free, pd_full, acc_free;
      for (int idx = blockIdx.x; idx < total; idx += gridDim.x) {
        int i, b, hk;
        decode(idx, i, b, hk);
        const int T = ntiles(i);
        if (!mbar_wait(bar(A_FULL), a_full.full(), ab)) break;
        bool ok = true;
        for (int t = 0; t < T; ++t) {
          if (!mbar_wait(bar(KV_FULL), kv_full.full(), ab) ||
              !mbar_wait(bar(T_FREE), t_free.empty(), ab) ||
              !mbar_wait(bar(DP_FREE), dp_free.empty(), ab)) { ok = false; break; }
          tc_fence_after();
          umma_tile(tmem + kTmS, sA1, false, sB1, false, 0u);   // S  = A1 B1^T
          umma_tile(tmem + kTmDP, sA2, false, sB2, false, 0u);  // dP = A2 B2^T
          umma_commit(bar(SD_FULL));
          if (!mbar_wait(bar(PD_FULL), pd_full.full(), ab)) { ok = false; break; }
          if (t == 0 && !mbar_wait(bar(ACC_FREE), acc_free.empty(), ab)) { ok = false; break; }
          tc_fence_after();
          const uint32_t acc = t > 0 ? 1u : 0u;
          umma_tile(tmem + kTmAcc1, sP, false, sB2, true, acc);   // acc1 += P B2
          umma_tile(tmem + kTmAcc2, sDS, false, sB1, true, acc);  // acc2 += dS B1
          umma_commit(bar(KV_EMPTY));
          umma_tile(tmem + kTmS, sDS, true, sA1, true, 0u);       // T = dS^T A1
          umma_commit(bar(T_FULL));
          umma_commit(bar(PD_FREE));
        }
        if (!ok) break;
        umma_commit(bar(ACC_FULL));
        if (!SOLVE) {
          umma_commit(bar(A_EMPTY));
          continue;
        }
        // ---- diagonal block of the transposed solve ----
        // D2: T' = U^T R
        if (!mbar_wait(bar(KV_FULL), kv_full.full(), ab) ||
            !mbar_wait(bar(PD_FULL), pd_full.full(), ab) ||
            !mbar_wait(bar(T_FREE), t_free.empty(), ab)) break;
        tc_fence_after();
        umma_tile(tmem + kTmS, sB1, true, sP, true, 0u);
        umma_commit(bar(T_FULL));
        umma_commit(bar(PD_FREE));
        umma_commit(bar(KV_EMPTY));
        // D4: S' = K^_i K^_i^T ; D' = X_i dV_i^T
        if (!mbar_wait(bar(PD_FULL), pd_full.full(), ab) ||
            !mbar_wait(bar(T_FREE), t_free.empty(), ab) ||
            !mbar_wait(bar(DP_FREE), dp_free.empty(), ab)) break;
        tc_fence_after();
        umma_tile(tmem + kTmS, sA1, false, sA1, false, 0u);
        umma_tile(tmem + kTmDP, sA2, false, sDS, false, 0u);
        umma_commit(bar(SD_FULL));
        umma_commit(bar(PD_FREE));
        // D6: acc2 += dG^T K^_i + dG K^_i
        if (!mbar_wait(bar(PD_FULL), pd_full.full(), ab)) break;
        if (T == 0 && !mbar_wait(bar(ACC_FREE), acc_free.empty(), ab)) break;
        tc_fence_after();
        umma_tile(tmem + kTmAcc2, sP, false, sA1, true, T > 0 ? 1u : 0u);
        umma_tile(tmem + kTmAcc2, sP, true, sA1, true, 1u);
        umma_commit(bar(PD_FREE));
        umma_commit(bar(A_EMPTY));
        umma_commit(bar(ACC2_FULL));
      }
      umma_commit(bar(DRAIN));
      mbar_wait_timed(bar(DRAIN), 0, kDrainNs);
    }
  } else {
    // ======================= epilogue warps 0-3 =======================
    const int r = threadIdx.x;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const float kLog2e = 1.4426950408889634f;
    const float c1 = p.scale * kLog2e;
    const float c2 = kLog2e / p.scale;
    Ph kv_full, sd_full, pd_free, t_full, acc_full, acc2_full;
    for (int idx = blockIdx.x; idx < total; idx += gridDim.x) {
      int i, b, hk;
      decode(idx, i, b, hk);
      const int T = ntiles(i);
      const long long bhk = (long long)b * p.Hkv + hk;
      const int row_i = i * 128 + r;  // this thread's row of column block i
      bool ok = true;
      for (int t = 0; t < T; ++t) {
        int g, j;
        tile_at(i, t, g, j);
        if (!SOLVE && !warp_wait_b(bar(KV_FULL), kv_full.full(), ab)) { ok = false; break; }
        if (!warp_wait_b(bar(SD_FULL), sd_full.full(), ab) ||
            !warp_wait_b(bar(PD_FREE), pd_free.empty(), ab)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float sv[32], dv[32];
          tmem_ld32(tmem + lane_base + kTmS + 32u * q, sv);
          tmem_ld32(tmem + lane_base + kTmDP + 32u * q, dv);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int c = q * 32 + e;      // column within the tile (query / key of block j)
            const int colg = j * 128 + c;  // global column
            float pe, ds;
            if (SOLVE) {
              pe = (colg < p.N) ? fast_exp2(fmaf(sv[e], c1, -c2)) : 0.f;
              ds = -p.scale * pe * dv[e];
            } else {
              const bool valid = (colg < p.N) && (row_i < p.N) && (colg >= row_i);
              pe = valid ? fast_exp2(fmaf(sv[e], c1, -svec[c])) : 0.f;
              ds = pe * (dv[e] - svec[128 + c]);
            }
            sv[e] = pe;
            dv[e] = ds;
          }
          tile_store_row32(sP, r, q, sv);
          tile_store_row32(sDS, r, q, dv);
        }
        tc_fence_before();
        mbar_arrive(bar(DP_FREE));
        fence_proxy_async_smem();
        mbar_arrive(bar(PD_FULL));
        // T rows -> fp32 atomics
        if (!warp_wait_b(bar(T_FULL), t_full.full(), ab)) { ok = false; break; }
        tc_fence_after();
        const long long drow =
            SOLVE ? (bhk * p.Npad + (long long)j * 128 + r)
                  : (((long long)b * p.Hq + hk * G + g) * p.Npad + (long long)j * 128 + r);
        float4* dst = reinterpret_cast<float4*>(p.d_row + drow * kHeadDim);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float tv[32];
          tmem_ld32(tmem + lane_base + kTmS + 32u * q, tv);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 8; ++c)
            atomicAdd(dst + q * 8 + c, make_float4(tv[4 * c], tv[4 * c + 1], tv[4 * c + 2], tv[4 * c + 3]));
        }
        tc_fence_before();
        mbar_arrive(bar(T_FREE));
      }
      if (!ok) break;
      if (!warp_wait_b(bar(ACC_FULL), acc_full.full(), ab)) break;
      tc_fence_after();
      if (!SOLVE) {
        float* dxr = p.dx + (bhk * p.Npad + row_i) * kHeadDim;
        float* dkr = p.dk_col + (bhk * p.Npad + row_i) * kHeadDim;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float a1[32], a2[32];
          tmem_ld32(tmem + lane_base + kTmAcc1 + 32u * q, a1);
          tmem_ld32(tmem + lane_base + kTmAcc2 + 32u * q, a2);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            reinterpret_cast<float4*>(dxr)[q * 8 + c] =
                make_float4(a1[4 * c], a1[4 * c + 1], a1[4 * c + 2], a1[4 * c + 3]);
            reinterpret_cast<float4*>(dkr)[q * 8 + c] =
                make_float4(a2[4 * c] * p.scale, a2[4 * c + 1] * p.scale, a2[4 * c + 2] * p.scale,
                            a2[4 * c + 3] * p.scale);
          }
        }
        tc_fence_before();
        mbar_arrive(bar(ACC_FREE));
        continue;
      }
      // ---------------- solve: diagonal block ----------------
      // D1: R = dX_i - acc1 -> P buffer (bf16), kept in fp32 registers
      float rr[4][32];
      const float* dxr = p.dx_in + (bhk * p.Npad + row_i) * kHeadDim;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float a1[32];
        if (T > 0) {
          tmem_ld32(tmem + lane_base + kTmAcc1 + 32u * q, a1);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) a1[e] = 0.f;
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float4 x4 = reinterpret_cast<const float4*>(dxr)[q * 8 + c];
          rr[q][4 * c + 0] = x4.x - a1[4 * c + 0];
          rr[q][4 * c + 1] = x4.y - a1[4 * c + 1];
          rr[q][4 * c + 2] = x4.z - a1[4 * c + 2];
          rr[q][4 * c + 3] = x4.w - a1[4 * c + 3];
        }
      }
      if (!warp_wait_b(bar(PD_FREE), pd_free.empty(), ab)) break;
#pragma unroll
      for (int q = 0; q < 4; ++q) tile_store_row32(sP, r, q, rr[q]);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(bar(PD_FULL));
      // D3: dV_i = D^-1 (R + U^T R) -> global bf16 + dS buffer; publish
      if (!warp_wait_b(bar(T_FULL), t_full.full(), ab) ||
          !warp_wait_b(bar(PD_FREE), pd_free.empty(), ab)) break;
      tc_fence_after();
      const float di = p.dinv[bhk * p.Npad + row_i];
      bf16* dvr = p.dv + (bhk * p.Npad + row_i) * kHeadDim;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float tv[32];
        tmem_ld32(tmem + lane_base + kTmS + 32u * q, tv);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) tv[e] = (rr[q][e] + tv[e]) * di;
#pragma unroll
        for (int c = 0; c < 4; ++c) st_bf16x8(dvr + q * 32 + c * 8, tv + c * 8);
        tile_store_row32(sDS, r, q, tv);
      }
      tc_fence_before();
      mbar_arrive(bar(T_FREE));
      fence_proxy_async_smem();
      mbar_arrive(bar(PD_FULL));
      fence_proxy_async_global();
      __threadfence();
      mbar_arrive(bar(EPI_DONE));
      if (r == 0) {
        const uint32_t ph = (uint32_t)((idx - (int)blockIdx.x) / (int)gridDim.x) & 1u;
        if (mbar_wait(bar(EPI_DONE), ph, ab)) st_release_gpu(&p.flags[bhk * p.NB + i], 1);
      }
      __syncwarp();
      // D5: dG^T of the strictly-lower part of P_ii -> P buffer
      if (!warp_wait_b(bar(SD_FULL), sd_full.full(), ab) ||
          !warp_wait_b(bar(PD_FREE), pd_free.empty(), ab)) break;
      tc_fence_after();
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float sv[32], dv[32];
        tmem_ld32(tmem + lane_base + kTmS + 32u * q, sv);
        tmem_ld32(tmem + lane_base + kTmDP + 32u * q, dv);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int c = q * 32 + e;
          const int colg = i * 128 + c;
          const bool valid = (c > r) && (colg < p.N);
          sv[e] = valid ? -p.scale * fast_exp2(fmaf(sv[e], c1, -c2)) * dv[e] : 0.f;
        }
        tile_store_row32(sP, r, q, sv);
      }
      tc_fence_before();
      mbar_arrive(bar(T_FREE));
      mbar_arrive(bar(DP_FREE));
      fence_proxy_async_smem();
      mbar_arrive(bar(PD_FULL));
      // D7: column part of dK^_i
      if (!warp_wait_b(bar(ACC2_FULL), acc2_full.full(), ab)) break;
      tc_fence_after();
      float* dkr = p.dk_col + (bhk * p.Npad + row_i) * kHeadDim;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float a2[32];
        tmem_ld32(tmem + lane_base + kTmAcc2 + 32u * q, a2);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 8; ++c)
          reinterpret_cast<float4*>(dkr)[q * 8 + c] =
              make_float4(a2[4 * c], a2[4 * c + 1], a2[4 * c + 2], a2[4 * c + 3]);
      }
      tc_fence_before();
      mbar_arrive(bar(ACC_FREE));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// --------------------------------------------------------------------------
// elementwise helpers of the backward
// --------------------------------------------------------------------------

// delta[bhq][row] = sum_d dO[row][d] * O[row][d]  (zero on padding rows)
__global__ void lucid_delta_kernel(int B, int Hq, int N, int Npad, const bf16* o, long long o_sb,
                                   long long o_sh, long long o_sn, const bf16* dout, long long d_sb,
                                   long long d_sh, long long d_sn, float* delta) {
  const int warps = blockDim.x >> 5;
  const long long gw = (long long)blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const long long total = (long long)B * Hq * Npad;
  if (gw >= total) return;
  const int row = (int)(gw % Npad);
  const long long bh = gw / Npad;
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
    acc = a[0] * c[0] + a[1] * c[1] + a[2] * c[2] + a[3] * c[3];
  }
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, s);
  if (lane == 0) delta[gw] = acc;
}

// dst (bf16, strided [B,H,N,128]) = scale * src (fp32 [B,H,Npad,128])
__global__ void lucid_f32_to_bf16_kernel(int B, int H, int N, int Npad, float scale, const float* src,
                                         bf16* dst, long long sb, long long sh, long long sn) {
  const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // one 8-element chunk
  const long long total = (long long)B * H * N * 16;
  if (t >= total) return;
  const int c8 = (int)(t & 15);
  const long long rowg = t >> 4;
  const int row = (int)(rowg % N);
  const long long bh = rowg / N;
  const int b = (int)(bh / H), h = (int)(bh % H);
  const float* s = src + ((bh * Npad + row) * kHeadDim) + c8 * 8;
  float v[8];
  const float4 x0 = reinterpret_cast<const float4*>(s)[0];
  const float4 x1 = reinterpret_cast<const float4*>(s)[1];
  v[0] = x0.x * scale; v[1] = x0.y * scale; v[2] = x0.z * scale; v[3] = x0.w * scale;
  v[4] = x1.x * scale; v[5] = x1.y * scale; v[6] = x1.z * scale; v[7] = x1.w * scale;
  st_bf16x8(dst + b * sb + h * sh + (long long)row * sn + c8 * 8, v);
}

// Solve backward finalize, one warp per row (row < N):
//   dk^  = dk_col + dk_row + 2 dG_rr k^_r,  dG_rr = -s P_rr (dV_r . X_r)
//   dK   = rstd (dk^ - (k^.dk^ / D) k^) + dk_add        (RMSNorm backward)
//   dV   = copy of the internal bf16 dV
__global__ void lucid_solve_finalize_kernel(int B, int H, int N, int Npad, float s, const bf16* k,
                                            long long k_sb, long long k_sh, long long k_sn,
                                            const float* rstd, const float* dinv, const bf16* x,
                                            const bf16* dv_int, const float* dk_col,
                                            const float* dk_row, const float* dk_add, bf16* dk,
                                            long long dk_sb, long long dk_sh, long long dk_sn, bf16* dv,
                                            long long dv_sb, long long dv_sh, long long dv_sn) {
  const int warps = blockDim.x >> 5;
  const long long gw = (long long)blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const long long total = (long long)B * H * N;
  if (gw >= total) return;
  const int row = (int)(gw % N);
  const long long bh = gw / N;
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
  proj *= (1.0f / kHeadDim);
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

cudaError_t launch_bwd(bool solve, const CUtensorMap& tA1, const CUtensorMap& tA2,
                       const CUtensorMap& tB1, const CUtensorMap& tB2, const CUtensorMap& tU,
                       const BwdArgs& a, cudaStream_t st) {
  const int total = a.NB * a.B * a.Hkv;
  if (total == 0) return cudaSuccess;
  const int grid = std::min(total, bwd_num_sms());
  cudaError_t e;
  if (solve) {
    e = cudaFuncSetAttribute(lucid_bwd_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)bwd::kSmemBytes);
    if (e != cudaSuccess) return e;
    lucid_bwd_kernel<true><<<grid, bwd::kThreads, bwd::kSmemBytes, st>>>(tA1, tA2, tB1, tB2, tU, a);
  } else {
    e = cudaFuncSetAttribute(lucid_bwd_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)bwd::kSmemBytes);
    if (e != cudaSuccess) return e;
    lucid_bwd_kernel<false><<<grid, bwd::kThreads, bwd::kSmemBytes, st>>>(tA1, tA2, tB1, tB2, tU, a);
  }
  return cudaGetLastError();
}

cudaError_t launch_delta(int B, int Hq, int N, int Npad, const bf16* o, long long o_sb, long long o_sh,
                         long long o_sn, const bf16* dout, long long d_sb, long long d_sh,
                         long long d_sn, float* delta, cudaStream_t st) {
  const long long warps = (long long)B * Hq * Npad;
  if (warps == 0) return cudaSuccess;
  const int blocks = (int)((warps + 7) / 8);
  lucid_delta_kernel<<<blocks, 256, 0, st>>>(B, Hq, N, Npad, o, o_sb, o_sh, o_sn, dout, d_sb, d_sh,
                                             d_sn, delta);
  return cudaGetLastError();
}

cudaError_t launch_f32_to_bf16(int B, int H, int N, int Npad, float scale, const float* src, bf16* dst,
                               long long sb, long long sh, long long sn, cudaStream_t st) {
  const long long total = (long long)B * H * N * 16;
  if (total == 0) return cudaSuccess;
  const int blocks = (int)((total + 255) / 256);
  lucid_f32_to_bf16_kernel<<<blocks, 256, 0, st>>>(B, H, N, Npad, scale, src, dst, sb, sh, sn);
  return cudaGetLastError();
}

cudaError_t launch_solve_finalize(int B, int H, int N, int Npad, float s, const bf16* k, long long k_sb,
                                  long long k_sh, long long k_sn, const float* rstd, const float* dinv,
                                  const bf16* x, const bf16* dv_int, const float* dk_col,
                                  const float* dk_row, const float* dk_add, bf16* dk, long long dk_sb,
                                  long long dk_sh, long long dk_sn, bf16* dv, long long dv_sb,
                                  long long dv_sh, long long dv_sn, cudaStream_t st) {
  const long long warps = (long long)B * H * N;
  if (warps == 0) return cudaSuccess;
  const int blocks = (int)((warps + 7) / 8);
  lucid_solve_finalize_kernel<<<blocks, 256, 0, st>>>(B, H, N, Npad, s, k, k_sb, k_sh, k_sn, rstd, dinv,
                                                      x, dv_int, dk_col, dk_row, dk_add, dk, dk_sb,
                                                      dk_sh, dk_sn, dv, dv_sb, dv_sh, dv_sn);
  return cudaGetLastError();
}

}  // namespace lb
