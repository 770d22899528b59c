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

// The cache passes give each cache row to a group of 8 lanes (4 rows per warp at a
// time, lane l holding elements [16 (l % 8), +16) of its group's row): the row's dot
// products need 3 shuffle levels, each shuffle instruction serving 4 rows, and each
// warp keeps kGrpRows rows in flight per group.
constexpr int kGrpTok = 2;   // new tokens per pass of the grouped kernels
constexpr int kGrpRows = 2;  // row iterations in flight per group

// 16 elements [e0, e0 + 16) of a row with head dimension D (a multiple of 4); the
// 4-element chunks at or past D read nothing and are zero
__device__ __forceinline__ void ld_row16(const bf16* row, int e0, int D, float (&v)[16]) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const float4 f = ld_bf16x4_d(row + e0 + 4 * c, e0 + 4 * c < D);
    v[4 * c] = f.x; v[4 * c + 1] = f.y; v[4 * c + 2] = f.z; v[4 * c + 3] = f.w;
  }
}

// sum over the 8 lanes of a lane group
__device__ __forceinline__ float grp_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  return v;
}

__device__ __forceinline__ float dot16_smem(const float* q, const float (&k)[16]) {
  float d = 0.f;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const float4 q4 = *reinterpret_cast<const float4*>(q + 4 * c);
    d = fmaf(q4.x, k[4 * c], d);
    d = fmaf(q4.y, k[4 * c + 1], d);
    d = fmaf(q4.z, k[4 * c + 2], d);
    d = fmaf(q4.w, k[4 * c + 3], d);
  }
  return d;
}

__global__ void __launch_bounds__(256, 2) lucid_decode_partial_kernel(const DecodeArgs a) {
  __shared__ __align__(16) float khn[kGrpTok][128];        // normalised new keys of this pass
  __shared__ __align__(16) float red[8][kGrpTok][128];     // per-warp partials
  const int split = blockIdx.x, bh = blockIdx.y;
  const int b = bh / a.H, h = bh % a.H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = lane >> 3, e0 = (lane & 7) * 16;
  const float c1 = a.s * 1.4426950408889634f, c2 = 1.4426950408889634f / a.s;
  const float inv_d = 1.f / (float)a.D;
  const int r0 = split * a.rows_per_split;
  const int r1 = min(a.Nc, r0 + a.rows_per_split);
  const bf16* kbase = a.kc + (long long)b * a.kc_sb + (long long)h * a.kc_sh;
  const bf16* xbase = a.xc + (long long)b * a.xc_sb + (long long)h * a.xc_sh;
  const bool act = lane * 4 < a.D;
  for (int t0 = 0; t0 < a.Ln; t0 += kGrpTok) {
    const int nt = min(kGrpTok, a.Ln - t0);
    __syncthreads();
    if (warp < nt) {  // RMSNorm of new token t0 + warp (a whole warp per token)
      const float4 k4 = ld_bf16x4_d(a.kn + (long long)b * a.kn_sb + (long long)h * a.kn_sh +
                                    (long long)(t0 + warp) * a.kn_st + lane * 4, act);
      const float ss = warp_sum(k4.x * k4.x + k4.y * k4.y + k4.z * k4.z + k4.w * k4.w);
      const float r = rsqrtf(ss * inv_d + a.eps);
      khn[warp][lane * 4 + 0] = k4.x * r;
      khn[warp][lane * 4 + 1] = k4.y * r;
      khn[warp][lane * 4 + 2] = k4.z * r;
      khn[warp][lane * 4 + 3] = k4.w * r;
    }
    __syncthreads();
    float acc[kGrpTok][16];
#pragma unroll
    for (int t = 0; t < kGrpTok; ++t)
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[t][i] = 0.f;
    // rows base + 32 u + 4 warp + grp; every lane runs every iteration (the shuffles
    // span the warp), rows past r1 load nothing and add nothing
    for (int base = r0; base < r1; base += 32 * kGrpRows) {
      float k[kGrpRows][16], x[kGrpRows][16];
#pragma unroll
      for (int u = 0; u < kGrpRows; ++u) {
        const int row = base + 32 * u + 4 * warp + grp;
        if (row < r1) {
          ld_row16(kbase + (long long)row * a.kc_st, e0, a.D, k[u]);
          ld_row16(xbase + (long long)row * a.xc_st, e0, a.D, x[u]);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) k[u][i] = x[u][i] = 0.f;
        }
      }
#pragma unroll
      for (int u = 0; u < kGrpRows; ++u) {
        const bool valid = base + 32 * u + 4 * warp + grp < r1;
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) ss = fmaf(k[u][i], k[u][i], ss);
        const float rs = rsqrtf(grp_sum(ss) * inv_d + a.eps);
#pragma unroll
        for (int t = 0; t < kGrpTok; ++t) {
          if (t < nt) {
            const float d = grp_sum(dot16_smem(&khn[t][e0], k[u])) * rs;
            const float e = valid ? exp2f(fmaf(d, c1, -c2)) : 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[t][i] = fmaf(e, x[u][i], acc[t][i]);
          }
        }
      }
    }
    // the 4 groups summed different rows into the same output elements
#pragma unroll
    for (int t = 0; t < kGrpTok; ++t)
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        acc[t][i] += __shfl_xor_sync(0xffffffffu, acc[t][i], 8);
        acc[t][i] += __shfl_xor_sync(0xffffffffu, acc[t][i], 16);
      }
    if (grp == 0) {
#pragma unroll
      for (int t = 0; t < kGrpTok; ++t)
        if (t < nt) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
            *reinterpret_cast<float4*>(&red[warp][t][e0 + 4 * c]) =
                make_float4(acc[t][4 * c], acc[t][4 * c + 1], acc[t][4 * c + 2], acc[t][4 * c + 3]);
        }
    }
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

__global__ void __launch_bounds__(256, 2) lucid_decode_attn_partial_kernel(const DecodeArgs a) {
  // rows of 132 floats: 128 partial values, the running maximum and the
  // denominator, padded so that every row starts on a 16-byte boundary
  constexpr int kRow = 132;
  __shared__ __align__(16) float qs[kGrpTok][128];
  __shared__ __align__(16) float red[8][kGrpTok][kRow];
  const int split = blockIdx.x, bq = blockIdx.y;
  const int b = bq / a.Hq, hq = bq % a.Hq, h = hq / (a.Hq / a.H);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = lane >> 3, e0 = (lane & 7) * 16;
  const float sm = a.s * 1.4426950408889634f;
  const int r0 = split * a.rows_per_split;
  const int r1 = min(a.Nc, r0 + a.rows_per_split);
  const bf16* kbase = a.kc + (long long)b * a.kc_sb + (long long)h * a.kc_sh;
  const bf16* xbase = a.xc + (long long)b * a.xc_sb + (long long)h * a.xc_sh;
  for (int t0 = 0; t0 < a.Ln; t0 += kGrpTok) {
    const int nt = min(kGrpTok, a.Ln - t0);
    __syncthreads();
    for (int e = threadIdx.x; e < nt * 128; e += blockDim.x) {
      const int t = e >> 7, c = e & 127;
      qs[t][c] = c < a.D ? __bfloat162float(a.kn[(long long)b * a.kn_sb + (long long)hq * a.kn_sh +
                                                 (long long)(t0 + t) * a.kn_st + c]) * sm
                         : 0.f;
    }
    __syncthreads();
    float acc[kGrpTok][16], m[kGrpTok], l[kGrpTok];
#pragma unroll
    for (int t = 0; t < kGrpTok; ++t) {
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[t][i] = 0.f;
      m[t] = -INFINITY;
      l[t] = 0.f;
    }
    for (int base = r0; base < r1; base += 32 * kGrpRows) {
      float k[kGrpRows][16], x[kGrpRows][16];
#pragma unroll
      for (int u = 0; u < kGrpRows; ++u) {
        const int row = base + 32 * u + 4 * warp + grp;
        if (row < r1) {
          ld_row16(kbase + (long long)row * a.kc_st, e0, a.D, k[u]);
          ld_row16(xbase + (long long)row * a.xc_st, e0, a.D, x[u]);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) k[u][i] = x[u][i] = 0.f;
        }
      }
#pragma unroll
      for (int u = 0; u < kGrpRows; ++u) {
        const int row = base + 32 * u + 4 * warp + grp;
#pragma unroll
        for (int t = 0; t < kGrpTok; ++t) {
          if (t < nt) {
            const float z = grp_sum(dot16_smem(&qs[t][e0], k[u]));
            // the new query t0 + t sits at cache position Nc - Ln + t0 + t (causal)
            if (row < r1 && row <= a.Nc - a.Ln + t0 + t) {   // uniform within the group
              const float mn = fmaxf(m[t], z);
              const float al = exp2f(m[t] - mn), p = exp2f(z - mn);
              l[t] = l[t] * al + p;
#pragma unroll
              for (int i = 0; i < 16; ++i) acc[t][i] = fmaf(p, x[u][i], acc[t][i] * al);
              m[t] = mn;
            }
          }
        }
      }
    }
    // merge the 4 groups' running (max, sum, weighted sum) of each token
#pragma unroll
    for (int t = 0; t < kGrpTok; ++t) {
      float M = fmaxf(m[t], __shfl_xor_sync(0xffffffffu, m[t], 8));
      M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 16));
      const float f = (m[t] == -INFINITY) ? 0.f : exp2f(m[t] - M);
      float L = l[t] * f;
      L += __shfl_xor_sync(0xffffffffu, L, 8);
      L += __shfl_xor_sync(0xffffffffu, L, 16);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float v = acc[t][i] * f;
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        acc[t][i] = v;
      }
      m[t] = M;
      l[t] = L;
    }
    if (grp == 0) {
#pragma unroll
      for (int t = 0; t < kGrpTok; ++t) {
        if (t < nt) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
            *reinterpret_cast<float4*>(&red[warp][t][e0 + 4 * c]) =
                make_float4(acc[t][4 * c], acc[t][4 * c + 1], acc[t][4 * c + 2], acc[t][4 * c + 3]);
          if (lane == 0) {
            red[warp][t][128] = m[t];
            red[warp][t][129] = l[t];
          }
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
