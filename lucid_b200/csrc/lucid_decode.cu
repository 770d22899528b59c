// Decode step of the LUCID solve: LucidAttention.get_new_v_prime
// (modeling_lucid.py:576-598).  For each (batch, kv head) and new token l:
//   x_new_l = v_new_l - sum_s exp(s k^_new_l . k^_s - 1/s) x_s
// over the cache of raw keys k_s and solved values x_s (modeling_lucid.py:479-481
// stores key_states and v_prime), k^ = RMSNorm(k) without affine.  As in the
// reference, the new tokens do not see one another and P's diagonal is not
// divided out.
//
// Memory-bound (one pass over K_cache and X_cache): the cache rows are split
// over CTAs (grid = splits x heads), each warp walks rows with one 8-byte
// load per lane per tensor, normalises the cached key on the fly and
// accumulates up to 8 new tokens at a time in registers; a second kernel sums
// the per-split partials and writes x_new.
#include "lucid_common.cuh"

#include <algorithm>

namespace lb {


constexpr int kDecTok = 8;  // new tokens per pass

__device__ __forceinline__ float4 ld_bf16x4(const bf16* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
  const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
  return make_float4(a.x, a.y, b.x, b.y);
}

// four elements of a row whose head dimension is D (a multiple of 4): lanes past
// D read nothing and return zeros
__device__ __forceinline__ float4 ld_bf16x4_d(const bf16* p, bool act) {
  return act ? ld_bf16x4(p) : make_float4(0.f, 0.f, 0.f, 0.f);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void __launch_bounds__(256) lucid_decode_partial_kernel(const DecodeArgs a) {
  __shared__ __align__(16) float khn[kDecTok][128];        // normalised new keys of this pass
  __shared__ __align__(16) float red[8][kDecTok][128];     // per-warp partials
  const int split = blockIdx.x, bh = blockIdx.y;
  const int b = bh / a.H, h = bh % a.H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float c1 = a.s * 1.4426950408889634f, c2 = 1.4426950408889634f / a.s;
  const int r0 = split * a.rows_per_split;
  const int r1 = min(a.Nc, r0 + a.rows_per_split);
  const bf16* kbase = a.kc + (long long)b * a.kc_sb + (long long)h * a.kc_sh + lane * 4;
  const bf16* xbase = a.xc + (long long)b * a.xc_sb + (long long)h * a.xc_sh + lane * 4;
  const bool act = lane * 4 < a.D;
  for (int t0 = 0; t0 < a.Ln; t0 += kDecTok) {
    const int nt = min(kDecTok, a.Ln - t0);
    __syncthreads();
    if (warp < nt) {  // RMSNorm of new token t0 + warp
      const float4 k4 = ld_bf16x4_d(a.kn + (long long)b * a.kn_sb + (long long)h * a.kn_sh +
                                    (long long)(t0 + warp) * a.kn_st + lane * 4, act);
      const float ss = warp_sum(k4.x * k4.x + k4.y * k4.y + k4.z * k4.z + k4.w * k4.w);
      const float r = rsqrtf(ss * (1.f / (float)a.D) + a.eps);
      khn[warp][lane * 4 + 0] = k4.x * r;
      khn[warp][lane * 4 + 1] = k4.y * r;
      khn[warp][lane * 4 + 2] = k4.z * r;
      khn[warp][lane * 4 + 3] = k4.w * r;
    }
    __syncthreads();
    float4 q[kDecTok];
#pragma unroll
    for (int t = 0; t < kDecTok; ++t)
      q[t] = t < nt ? make_float4(khn[t][lane * 4], khn[t][lane * 4 + 1], khn[t][lane * 4 + 2], khn[t][lane * 4 + 3])
                    : make_float4(0.f, 0.f, 0.f, 0.f);
    float4 acc[kDecTok];
#pragma unroll
    for (int t = 0; t < kDecTok; ++t) acc[t] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int row = r0 + warp; row < r1; row += 8) {
      const float4 k4 = ld_bf16x4_d(kbase + (long long)row * a.kc_st, act);
      const float4 x4 = ld_bf16x4_d(xbase + (long long)row * a.xc_st, act);
      const float rs = rsqrtf(warp_sum(k4.x * k4.x + k4.y * k4.y + k4.z * k4.z + k4.w * k4.w) * (1.f / (float)a.D) + a.eps);
#pragma unroll
      for (int t = 0; t < kDecTok; ++t) {
        if (t < nt) {
          const float d = warp_sum(q[t].x * k4.x + q[t].y * k4.y + q[t].z * k4.z + q[t].w * k4.w) * rs;
          const float e = exp2f(fmaf(d, c1, -c2));
          acc[t].x = fmaf(e, x4.x, acc[t].x);
          acc[t].y = fmaf(e, x4.y, acc[t].y);
          acc[t].z = fmaf(e, x4.z, acc[t].z);
          acc[t].w = fmaf(e, x4.w, acc[t].w);
        }
      }
    }
#pragma unroll
    for (int t = 0; t < kDecTok; ++t)
      if (t < nt) *reinterpret_cast<float4*>(&red[warp][t][lane * 4]) = acc[t];
    __syncthreads();
    for (int e = threadIdx.x; e < nt * 128; e += blockDim.x) {
      const int t = e >> 7, c = e & 127;
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) sum += red[w][t][c];
      a.part[(((long long)split * a.B * a.H + bh) * a.Ln + t0 + t) * 128 + c] = sum;
    }
  }
}

__global__ void lucid_decode_finish_kernel(const DecodeArgs a) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // one thread per element
  const long long total = (long long)a.B * a.H * a.Ln * 128;
  if (i >= total) return;
  const int c = (int)(i & 127);
  const long long row = i >> 7;
  const int l = (int)(row % a.Ln);
  const long long bh = row / a.Ln;
  const int b = (int)(bh / a.H), h = (int)(bh % a.H);
  if (c >= a.D) return;
  float sum = 0.f;
  for (int sp = 0; sp < a.nsplit; ++sp) sum += a.part[(((long long)sp * a.B * a.H + bh) * a.Ln + l) * 128 + c];
  const float v = __bfloat162float(a.vn[(long long)b * a.vn_sb + (long long)h * a.vn_sh + (long long)l * a.vn_st + c]);
  a.out[(long long)b * a.o_sb + (long long)h * a.o_sh + (long long)l * a.o_st + c] = __float2bfloat16(v - sum);
}

int decode_splits(int B, int H, int Nc) {
  // about 4 CTAs per SM over all heads, at least 256 cache rows per CTA
  const int bh = std::max(1, B * H);
  int n = (4 * 148 + bh - 1) / bh;
  n = std::min(n, std::max(1, (Nc + 255) / 256));
  return std::max(1, std::min(n, 1024));
}

cudaError_t launch_decode(DecodeArgs a, cudaStream_t st) {
  if (a.B == 0 || a.H == 0 || a.Ln == 0) return cudaSuccess;
  a.nsplit = decode_splits(a.B, a.H, a.Nc);
  a.rows_per_split = (a.Nc + a.nsplit - 1) / a.nsplit;
  lucid_decode_partial_kernel<<<dim3(a.nsplit, a.B * a.H), 256, 0, st>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const long long total = (long long)a.B * a.H * a.Ln * 128;
  lucid_decode_finish_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace lb

// ===========================================================================
// Decode attention: eager_lucid_attention_forward (modeling_lucid.py:505-549) for
// Ln new queries against the Nc cached keys / solved values (query l sits at
// position Nc - Ln + l and sees keys c <= Nc - Ln + l), grouped-query heads
// native.  Split over the cache like the update; each split keeps a running
// maximum, a denominator and the weighted sum, and the finish kernel merges them.
// part layout per (split, b, hq, l): [128 values][m][l]
// ===========================================================================
namespace lb {

__global__ void __launch_bounds__(256) lucid_decode_attn_partial_kernel(const DecodeArgs a) {
  // rows of 132 floats: 128 partial values, the running maximum and the
  // denominator, padded so that every row starts on a 16-byte boundary
  constexpr int kRow = 132;
  __shared__ __align__(16) float qs[kDecTok][128];
  __shared__ __align__(16) float red[8][kDecTok][kRow];
  const int split = blockIdx.x, bq = blockIdx.y;
  const int b = bq / a.Hq, hq = bq % a.Hq, h = hq / (a.Hq / a.H);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float sm = a.s * 1.4426950408889634f;
  const int r0 = split * a.rows_per_split;
  const int r1 = min(a.Nc, r0 + a.rows_per_split);
  const bf16* kbase = a.kc + (long long)b * a.kc_sb + (long long)h * a.kc_sh + lane * 4;
  const bf16* xbase = a.xc + (long long)b * a.xc_sb + (long long)h * a.xc_sh + lane * 4;
  const bool act = lane * 4 < a.D;
  for (int t0 = 0; t0 < a.Ln; t0 += kDecTok) {
    const int nt = min(kDecTok, a.Ln - t0);
    __syncthreads();
    for (int e = threadIdx.x; e < nt * 128; e += blockDim.x) {
      const int t = e >> 7, c = e & 127;
      qs[t][c] = c < a.D ? __bfloat162float(a.kn[(long long)b * a.kn_sb + (long long)hq * a.kn_sh +
                                                 (long long)(t0 + t) * a.kn_st + c]) * sm
                         : 0.f;
    }
    __syncthreads();
    float4 q[kDecTok], acc[kDecTok];
    float m[kDecTok], l[kDecTok];
#pragma unroll
    for (int t = 0; t < kDecTok; ++t) {
      q[t] = t < nt ? make_float4(qs[t][lane * 4], qs[t][lane * 4 + 1], qs[t][lane * 4 + 2], qs[t][lane * 4 + 3])
                    : make_float4(0.f, 0.f, 0.f, 0.f);
      acc[t] = make_float4(0.f, 0.f, 0.f, 0.f);
      m[t] = -INFINITY;
      l[t] = 0.f;
    }
    for (int row = r0 + warp; row < r1; row += 8) {
      const float4 k4 = ld_bf16x4_d(kbase + (long long)row * a.kc_st, act);
      const float4 x4 = ld_bf16x4_d(xbase + (long long)row * a.xc_st, act);
#pragma unroll
      for (int t = 0; t < kDecTok; ++t) {
        if (t < nt && row <= a.Nc - a.Ln + t0 + t) {
          const float z = warp_sum(q[t].x * k4.x + q[t].y * k4.y + q[t].z * k4.z + q[t].w * k4.w);
          const float mn = fmaxf(m[t], z);
          const float al = exp2f(m[t] - mn), p = exp2f(z - mn);
          l[t] = l[t] * al + p;
          acc[t].x = fmaf(p, x4.x, acc[t].x * al);
          acc[t].y = fmaf(p, x4.y, acc[t].y * al);
          acc[t].z = fmaf(p, x4.z, acc[t].z * al);
          acc[t].w = fmaf(p, x4.w, acc[t].w * al);
          m[t] = mn;
        }
      }
    }
#pragma unroll
    for (int t = 0; t < kDecTok; ++t) {
      if (t < nt) {
        *reinterpret_cast<float4*>(&red[warp][t][lane * 4]) = acc[t];
        if (lane == 0) {
          red[warp][t][128] = m[t];
          red[warp][t][129] = l[t];
        }
      }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < nt * 128; e += blockDim.x) {
      const int t = e >> 7, c = e & 127;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < 8; ++w) M = fmaxf(M, red[w][t][128]);
      float L = 0.f, S = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const float f = (red[w][t][128] == -INFINITY) ? 0.f : exp2f(red[w][t][128] - M);
        L += f * red[w][t][129];
        S += f * red[w][t][c];
      }
      float* dst = a.part + (((long long)split * a.B * a.Hq + bq) * a.Ln + t0 + t) * 130;
      dst[c] = S;
      if (c == 0) {
        dst[128] = M;
        dst[129] = L;
      }
    }
  }
}

__global__ void lucid_decode_attn_finish_kernel(const DecodeArgs a) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long total = (long long)a.B * a.Hq * a.Ln * 128;
  if (i >= total) return;
  const int c = (int)(i & 127);
  const long long row = i >> 7;
  const int l = (int)(row % a.Ln);
  const long long bq = row / a.Ln;
  const int b = (int)(bq / a.Hq), hq = (int)(bq % a.Hq);
  if (c >= a.D) return;
  float M = -INFINITY;
  for (int sp = 0; sp < a.nsplit; ++sp) M = fmaxf(M, a.part[(((long long)sp * a.B * a.Hq + bq) * a.Ln + l) * 130 + 128]);
  float L = 0.f, S = 0.f;
  for (int sp = 0; sp < a.nsplit; ++sp) {
    const float* pp = a.part + (((long long)sp * a.B * a.Hq + bq) * a.Ln + l) * 130;
    const float f = (pp[128] == -INFINITY) ? 0.f : exp2f(pp[128] - M);
    L += f * pp[129];
    S += f * pp[c];
  }
  a.out[(long long)b * a.o_sb + (long long)hq * a.o_sh + (long long)l * a.o_st + c] = __float2bfloat16(S / L);
}

cudaError_t launch_decode_attn(DecodeArgs a, cudaStream_t st) {
  if (a.B == 0 || a.Hq == 0 || a.Ln == 0) return cudaSuccess;
  a.nsplit = decode_splits(a.B, a.Hq, a.Nc);
  a.rows_per_split = (a.Nc + a.nsplit - 1) / a.nsplit;
  lucid_decode_attn_partial_kernel<<<dim3(a.nsplit, a.B * a.Hq), 256, 0, st>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const long long total = (long long)a.B * a.Hq * a.Ln * 128;
  lucid_decode_attn_finish_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace lb
