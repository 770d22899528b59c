// Per-block kernels of LUCID-Path: the O(N) part of the op (UT transform,
// q/k transforms, diagonal blocks, and their backward).
//
//   path_bgemm_kernel   one 128x128 output block per CTA:
//                       C = mask(epi(rsc .* sum_p op(A_p) op(B_p) + sum_c beta_c rsc_c .* C_c))
//                       operands fp32 or bf16 in global memory (any of the
//                       layouts PMat describes), staged as bf16 swizzled tiles,
//                       multiplied by tcgen05.mma into TMEM (fp32 accumulate).
//   path_triinv_kernel  (I + stril(M))^-1 by blocked forward substitution
//                       in fp32 shared memory (CUDA cores).
//   path_gsum_kernel / path_rowdot_kernel / path_pack_kernel
//                       elementwise reductions and the copies to the caller's
//                       strided gradient tensors.
//
// The host composes these into the forward prep (triangular_solve_fwd.py:118-148,
// parallel.py:39-51) and the per-block backward (intra_chunk_preprocess_bwd.py:10-110,
// intra_chunk_preprocess_bwd_prepare.py:8-140).
#include "path_common.cuh"

#include <algorithm>

namespace lb {

namespace pblk {
constexpr int kThreads = 256;
}

__device__ __forceinline__ float pvec_at(const PVec& v, int b, int h, long long t) {
  if (t >= v.rows) return 0.f;
  const long long off = (long long)b * v.s_b + (long long)(h / v.hdiv) * v.s_h + t * v.s_row;
  if (v.fp32) return reinterpret_cast<const float*>(v.ptr)[off];
  return __bfloat162float(reinterpret_cast<const bf16*>(v.ptr)[off]);
}

// W consecutive elements [c0, c0+W) of stored row r of matrix (b, h, blk), W = 32 or 64.
template <int W>
__device__ __forceinline__ bool pmat_load(const PMat& m, int b, int h, int blk, int r, int c0, float (&v)[W]) {
  const bool valid = (long long)blk * 128 + r < m.rows;
  if (!valid) {
#pragma unroll
    for (int e = 0; e < W; ++e) v[e] = 0.f;
    return false;
  }
  const long long off = (long long)b * m.s_b + (long long)(h / m.hdiv) * m.s_h + (long long)blk * m.s_blk +
                        (long long)r * m.s_row + c0;
  if (m.fp32) {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(m.ptr) + off);
#pragma unroll
    for (int e = 0; e < W / 4; ++e) {
      const float4 f = p[e];
      v[4 * e] = f.x; v[4 * e + 1] = f.y; v[4 * e + 2] = f.z; v[4 * e + 3] = f.w;
    }
  } else {
    const bf16* p = reinterpret_cast<const bf16*>(m.ptr) + off;
#pragma unroll
    for (int e = 0; e < W / 8; ++e) ld_bf16x8(p + 8 * e, v + 8 * e);
  }
  return true;
}

template <int W>
__device__ __forceinline__ void pmat_store(const PMat& m, int b, int h, int blk, int r, int c0, const float (&v)[W]) {
  if ((long long)blk * 128 + r >= m.rows) return;
  const long long off = (long long)b * m.s_b + (long long)(h / m.hdiv) * m.s_h + (long long)blk * m.s_blk +
                        (long long)r * m.s_row + c0;
  if (m.fp32) {
    float4* p = reinterpret_cast<float4*>(reinterpret_cast<float*>(m.ptr) + off);
#pragma unroll
    for (int e = 0; e < W / 4; ++e) p[e] = make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
  } else {
    bf16* p = reinterpret_cast<bf16*>(m.ptr) + off;
#pragma unroll
    for (int e = 0; e < W / 8; ++e) st_bf16x8(p + 8 * e, v + 8 * e);
  }
}

template <int W>
__device__ __forceinline__ void apply_mask(int mask, int r, int c0, float (&v)[W]) {
  if (mask == kMaskNone) return;
#pragma unroll
  for (int e = 0; e < W; ++e) {
    const int c = c0 + e;
    const bool keep = (mask == kMaskTril) ? (c <= r) : (c < r);
    if (!keep) v[e] = 0.f;
  }
}

__device__ __forceinline__ bool pmat_load64(const PMat& m, int b, int h, int blk, int r, int c0, float (&v)[64]) {
  return pmat_load<64>(m, b, h, blk, r, c0, v);
}
__device__ __forceinline__ void pmat_store64(const PMat& m, int b, int h, int blk, int r, int c0, const float (&v)[64]) {
  pmat_store<64>(m, b, h, blk, r, c0, v);
}
__device__ __forceinline__ void apply_mask64(int mask, int r, int c0, float (&v)[64]) { apply_mask<64>(mask, r, c0, v); }

// 32-column chunks keep the register footprint under 85 per thread, so that
// three CTAs (one output block each) share an SM: a CTA spends most of its
// life waiting on its operand loads, and the other two fill that time.
__global__ void __launch_bounds__(pblk::kThreads, 3) path_bgemm_kernel(const __grid_constant__ BGemmArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  // one (A, B) tile pair, reused by every product: 64 KB per CTA whatever nprod
  const uint32_t bar = sbase + 2u * 32768u;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 2 * 32768 + 8);
  volatile int* abort_cta = reinterpret_cast<volatile int*>(smem + 2 * 32768 + 12);
  const Abort ab{abort_cta, a.status, kTagPathGemm};
  const int warp = warp_id(), lane = lane_id();
  if ((sbase & 1023u) != 0) {
    if (threadIdx.x == 0) atomicCAS(a.status, 0, kStatusMisaligned | (kTagPathGemm << 20));
    return;
  }
  const int z = blockIdx.x;
  const int blk = z % a.NB;
  const int h = (z / a.NB) % a.Hx;
  const int b = z / (a.NB * a.Hx);
  const int qd = warp & 3, hf = warp >> 2;
  const int r = qd * 32 + lane;
  const int c0 = hf * 64;
  const long long t = (long long)blk * 128 + r;

  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    *abort_cta = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), 128);
    tmem_relinquish();
  }
  // ---- per product: stage (A_p, B_p) into the tile pair, then one MMA batch; the
  // next product overwrites the tiles once this MMA's commit has landed ----
  bool ok = true;
  uint32_t tmem = 0;
  for (int p = 0; p < a.nprod; ++p) {
    if (p > 0) {
      const bool w = mbar_wait(bar, (uint32_t)((p - 1) & 1), ab);
      if (!__syncthreads_and(w ? 1 : 0)) {
        ok = false;
        break;
      }
      tc_fence_after();
    }
    for (int side = 0; side < 2; ++side) {
      const POperand& op = side == 0 ? a.A[p] : a.B[p];
      float sc = op.scale;
      if (op.rsc.ptr != nullptr) sc *= pvec_at(op.rsc, b, h, t);
      const uint32_t tile = sbase + (uint32_t)side * 32768u;
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        float v[32];
        pmat_load<32>(op.m, b, h, blk, r, c0 + 32 * q, v);
        if (op.lo) {
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] -= __bfloat162float(__float2bfloat16(v[e]));
        }
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] *= sc;
        apply_mask<32>(op.mask, r, c0 + 32 * q, v);
        tile_store_row32(tile, r, 2 * hf + q, v);
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    tmem = *tmem_slot;
    if (threadIdx.x == 0) {
      umma_tile(tmem, sbase, a.A[p].trans != 0, sbase + 32768u, a.B[p].trans == 0, p > 0 ? 1u : 0u);
      umma_commit(bar);
    }
  }
  if (ok) ok = mbar_wait(bar, (uint32_t)((a.nprod - 1) & 1), ab);
  tc_fence_after();
  if (ok) {
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const float fo = a.orsc.ptr != nullptr ? pvec_at(a.orsc, b, h, t) : 1.f;
    float fc[2];
#pragma unroll
    for (int c = 0; c < 2; ++c)
      fc[c] = (c < a.nc && a.crsc[c].ptr != nullptr) ? a.cbeta[c] * pvec_at(a.crsc[c], b, h, t) : a.cbeta[c];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int cq = c0 + 32 * q;
      float acc[32];
      tmem_ld32(tmem + lane_base + (uint32_t)cq, acc);
      tmem_ld_wait();
#pragma unroll
      for (int e = 0; e < 32; ++e) acc[e] *= fo;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        if (c >= a.nc) break;
        float cv[32];
        pmat_load<32>(a.C[c], b, h, blk, r, cq, cv);
#pragma unroll
        for (int e = 0; e < 32; ++e) acc[e] = fmaf(fc[c], cv[e], acc[e]);
      }
      if (a.epi == kEpiPathExp) {
        const float c1 = a.s * 1.4426950408889634f, c2 = 1.4426950408889634f / a.s;
#pragma unroll
        for (int e = 0; e < 32; ++e) acc[e] = exp2f(fmaf(acc[e], c1, -c2));
      }
      apply_mask<32>(a.out_mask, r, cq, acc);
      pmat_store<32>(a.O, b, h, blk, r, cq, acc);
      if (a.O2.ptr != nullptr) pmat_store<32>(a.O2, b, h, blk, r, cq, acc);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

// ---------------------------------------------------------------------------
// (I + stril(M))^-1, fp32, in place in shared memory.
// ---------------------------------------------------------------------------
constexpr int kInvLD = 129;

__global__ void __launch_bounds__(256) path_triinv_kernel(const __grid_constant__ TriInvArgs a) {
  extern __shared__ float fsm[];
  float* z = fsm;                 // [128][kInvLD]
  float* tt = z + 128 * kInvLD;   // [8][16][16]
  const int zi = blockIdx.x;
  const int blk = zi % a.NB;
  const int h = (zi / a.NB) % a.Hx;
  const int b = zi / (a.NB * a.Hx);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  {
    const int r = tid >> 1, c0 = (tid & 1) * 64;
    float v[64];
    pmat_load64(a.M, b, h, blk, r, c0, v);
#pragma unroll
    for (int e = 0; e < 64; ++e) {
      const int c = c0 + e;
      z[r * kInvLD + c] = (c < r) ? v[e] : 0.f;
    }
    if (a.Mcopy.ptr != nullptr) {
      apply_mask64(kMaskStril, r, c0, v);
      pmat_store64(a.Mcopy, b, h, blk, r, c0, v);
    }
  }
  __syncthreads();
  // diagonal 16x16 blocks: warp I, lane c computes column c of Z_II
  if (lane < 16) {
    const int I = warp, c = lane;
    float zc[16];
#pragma unroll
    for (int rr = 0; rr < 16; ++rr) {
      float acc = (rr == c) ? 1.f : 0.f;
#pragma unroll
      for (int m = 0; m < rr; ++m) acc -= z[(I * 16 + rr) * kInvLD + I * 16 + m] * zc[m];
      zc[rr] = acc;
    }
    __syncwarp(0x0000ffffu);
#pragma unroll
    for (int rr = 0; rr < 16; ++rr) z[(I * 16 + rr) * kInvLD + I * 16 + c] = zc[rr];
  }
  __syncthreads();
  {
    const int rr = tid >> 4, c = tid & 15;
    for (int I = 1; I < 8; ++I) {
      // tt_J = L[I, J16:I16] Z[J16:I16, J]   (row block I still holds L): one pass over
      // the columns loads each L entry once for every J it feeds
      float acc[7];
#pragma unroll
      for (int J = 0; J < 7; ++J) acc[J] = 0.f;
#pragma unroll
      for (int K = 0; K < 7; ++K) {   // column block K of L's row block I feeds Z_IJ, J <= K
        if (K >= I) break;
        const float* lrow = z + (I * 16 + rr) * kInvLD + K * 16;
        const float* zrow = z + (K * 16) * kInvLD + c;
#pragma unroll 4
        for (int m = 0; m < 16; ++m) {
          const float l = lrow[m];
#pragma unroll
          for (int J = 0; J <= K; ++J) acc[J] = fmaf(l, zrow[m * kInvLD + J * 16], acc[J]);
        }
      }
#pragma unroll
      for (int J = 0; J < 7; ++J)
        if (J < I) tt[J * 256 + rr * 16 + c] = acc[J];
      __syncthreads();
      for (int J = 0; J < I; ++J) {
        float acc = 0.f;
#pragma unroll
        for (int m = 0; m < 16; ++m) acc = fmaf(z[(I * 16 + rr) * kInvLD + I * 16 + m], tt[J * 256 + m * 16 + c], acc);
        z[(I * 16 + rr) * kInvLD + J * 16 + c] = -acc;
      }
      __syncthreads();
    }
  }
  {
    const int r = tid >> 1, c0 = (tid & 1) * 64;
    float v[64];
#pragma unroll
    for (int e = 0; e < 64; ++e) {
      const int c = c0 + e;
      v[e] = (c > r) ? 0.f : z[r * kInvLD + c];
    }
    if (a.Z.ptr != nullptr) pmat_store64(a.Z, b, h, blk, r, c0, v);
    if (a.U.ptr != nullptr) {
#pragma unroll
      for (int e = 0; e < 64; ++e) v[e] -= (c0 + e == r) ? 1.f : 0.f;
      pmat_store64(a.U, b, h, blk, r, c0, v);
    }
  }
}

// out[bh_out][row][c] = sum_{g<G} (x0[bh_out*G+g][row][c] + x1[...])      (fp32)
__global__ void path_gsum_kernel(float* out, const float* x0, const float* x1, long long per_head, int G,
                                 long long total4) {
  const long long i4 = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i4 >= total4) return;
  const long long e = i4 * 4;
  const long long hb = e / per_head, w = e % per_head;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int g = 0; g < G; ++g) {
    const long long src = (hb * G + g) * per_head + w;
    float4 v = *reinterpret_cast<const float4*>(x0 + src);
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    if (x1 != nullptr) {
      v = *reinterpret_cast<const float4*>(x1 + src);
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
  }
  *reinterpret_cast<float4*>(out + e) = acc;
}

// dbeta[b, t, h] = sum_c X[bh][t][c] * W[b, t, h, c]   (X fp32 internal, W bf16 strided)
__global__ void path_rowdot_kernel(const float* X, int Npad, const bf16* w, long long w_sb, long long w_st,
                                   long long w_sh, void* out, int out_fp32, long long o_sb, long long o_st,
                                   long long o_sh, int B, int H, int T) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const long long rows = (long long)B * H * T;
  if (warp >= rows) return;
  const int t = warp % T;
  const int h = (warp / T) % H;
  const int b = warp / (T * H);
  const float* x = X + (((long long)b * H + h) * Npad + t) * 128 + lane * 4;
  const bf16* wp = w + (long long)b * w_sb + (long long)t * w_st + (long long)h * w_sh + lane * 4;
  const float4 xv = *reinterpret_cast<const float4*>(x);
  const uint2 u = *reinterpret_cast<const uint2*>(wp);
  const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&u);
  const float2 f0 = __bfloat1622float2(hh[0]), f1 = __bfloat1622float2(hh[1]);
  float acc = xv.x * f0.x + xv.y * f0.y + xv.z * f1.x + xv.w * f1.y;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) {
    const long long off = (long long)b * o_sb + (long long)t * o_st + (long long)h * o_sh;
    if (out_fp32) reinterpret_cast<float*>(out)[off] = acc;
    else reinterpret_cast<bf16*>(out)[off] = __float2bfloat16(acc);
  }
}

// out[b, t, h, :] (bf16 strided) = sum_{g<Ga} a[(b*H+h)*Ga+g][t] + sum_{g<Gb} bsrc[(b*H+h)*Gb+g][t]
// a / bsrc: [heads][Npad][128], fp32 or bf16.
__global__ void path_pack_kernel(bf16* out, long long o_sb, long long o_st, long long o_sh, const void* a,
                                 int a_fp32, int Ga, const void* bsrc, int b_fp32, int Gb, int B, int H, int T,
                                 int Npad) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // one thread per 8 elements
  const long long total = (long long)B * H * T * 16;
  if (i >= total) return;
  const int c8 = (int)(i & 15);
  const long long row = i >> 4;
  const int t = (int)(row % T);
  const int h = (int)((row / T) % H);
  const int b = (int)(row / ((long long)T * H));
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  auto add = [&](const void* src, int fp32, int G) {
    for (int g = 0; g < G; ++g) {
      const long long off = ((((long long)b * H + h) * G + g) * Npad + t) * 128 + c8 * 8;
      float v[8];
      if (fp32) {
        const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src) + off);
        const float4 x = p[0], y = p[1];
        v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w; v[4] = y.x; v[5] = y.y; v[6] = y.z; v[7] = y.w;
      } else {
        ld_bf16x8(reinterpret_cast<const bf16*>(src) + off, v);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += v[e];
    }
  };
  if (a != nullptr) add(a, a_fp32, Ga);
  if (bsrc != nullptr) add(bsrc, b_fp32, Gb);
  st_bf16x8(out + (long long)b * o_sb + (long long)t * o_st + (long long)h * o_sh + c8 * 8, acc);
}

// Identity matrices in an fp32 [heads][128][128] buffer (one 128x128 matrix per CTA).
__global__ void path_eye_kernel(float* out, long long head_stride) {
  float* m = out + (long long)blockIdx.x * head_stride;
  for (int e = threadIdx.x; e < 128 * 128; e += blockDim.x) m[e] = ((e >> 7) == (e & 127)) ? 1.f : 0.f;
}

// ---------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------
cudaError_t launch_path_bgemm(const BGemmArgs& a, cudaStream_t st) {
  const long long n = (long long)a.Bn * a.Hx * a.NB;
  if (n == 0) return cudaSuccess;
  const size_t smem = (size_t)2 * 32768 + 64;
  cudaError_t e = cudaFuncSetAttribute(path_bgemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  path_bgemm_kernel<<<(unsigned)n, pblk::kThreads, smem, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_path_eye(float* out, long long heads, long long head_stride, cudaStream_t st) {
  if (heads == 0) return cudaSuccess;
  path_eye_kernel<<<(unsigned)heads, 256, 0, st>>>(out, head_stride);
  return cudaGetLastError();
}

cudaError_t launch_path_triinv(const TriInvArgs& a, cudaStream_t st) {
  const long long n = (long long)a.Bn * a.Hx * a.NB;
  if (n == 0) return cudaSuccess;
  const size_t smem = (size_t)(128 * kInvLD + 8 * 256) * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute(path_triinv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  path_triinv_kernel<<<(unsigned)n, 256, smem, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_path_gsum(float* out, const float* x0, const float* x1, long long heads_out, long long per_head,
                             int G, cudaStream_t st) {
  const long long total4 = heads_out * per_head / 4;
  if (total4 == 0) return cudaSuccess;
  path_gsum_kernel<<<(unsigned)((total4 + 255) / 256), 256, 0, st>>>(out, x0, x1, per_head, G, total4);
  return cudaGetLastError();
}

cudaError_t launch_path_rowdot(const float* X, int Npad, const bf16* w, long long w_sb, long long w_st, long long w_sh,
                               void* out, int out_fp32, long long o_sb, long long o_st, long long o_sh, int B, int H,
                               int T, cudaStream_t st) {
  const long long rows = (long long)B * H * T;
  if (rows == 0) return cudaSuccess;
  path_rowdot_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, st>>>(X, Npad, w, w_sb, w_st, w_sh, out, out_fp32,
                                                                         o_sb, o_st, o_sh, B, H, T);
  return cudaGetLastError();
}

cudaError_t launch_path_pack(bf16* out, long long o_sb, long long o_st, long long o_sh, const void* a, int a_fp32,
                             int Ga, const void* bsrc, int b_fp32, int Gb, int B, int H, int T, int Npad,
                             cudaStream_t st) {
  const long long total = (long long)B * H * T * 16;
  if (total == 0) return cudaSuccess;
  path_pack_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(out, o_sb, o_st, o_sh, a, a_fp32, Ga, bsrc, b_fp32,
                                                                   Gb, B, H, T, Npad);
  return cudaGetLastError();
}

}  // namespace lb
