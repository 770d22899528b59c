// Decode step of the LUCID solve: LucidAttention.get_new_v_prime
// (modeling_lucid.py:576-598).  For each (batch, kv head) and new token l:
//   x_new_l = v_new_l - sum_s exp(s k^_new_l . k^_s - 1/s) x_s
// over the cache of raw keys k_s and solved values x_s (modeling_lucid.py:479-481
// stores key_states and v_prime), k^ = RMSNorm(k) without affine.  As in the
// reference, the new tokens do not see one another and P's diagonal is not
// divided out.
//
// Memory-bound (one pass over K_cache and X_cache): the cache rows are split
// over CTAs (grid = splits x heads), each cache row goes to a group of 8 lanes
// (16 elements per lane), the cached key is normalised on the fly and 2 new
// tokens at a time accumulate in registers; a second kernel sums the
// per-split partials and writes x_new.  The fused decode step at the end of
// the file computes the update and the new queries' attention in one pass.
#include "lucid_common.cuh"

#include <algorithm>
#include <climits>

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
  // Splits of each (batch, head)'s cache over CTAs for the partial kernels (two
  // resident CTAs per SM on 148 SMs): the count that minimises the modelled time,
  // waves x (cache rows per CTA + 64 rows' worth of fixed cost for the CTA's setup
  // and merges), with at least 128 cache rows per CTA.
  constexpr long long kSlots = 2 * 148, kFixedRows = 64;
  const long long bh = std::max(1, B * H);
  const int nmax = std::max(1, std::min(1024, (Nc + 127) / 128));
  int best = 1;
  long long best_t = LLONG_MAX;
  for (int n = 1; n <= nmax; ++n) {
    const long long waves = (bh * n + kSlots - 1) / kSlots;
    const long long t = waves * ((Nc + n - 1) / n + kFixedRows);
    if (t < best_t) {
      best_t = t;
      best = n;
    }
  }
  return best;
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


// ===========================================================================
// Fused decode step: the reference's decoding forward (modeling_lucid.py:467-481
// then :505-549) reads the cache twice, once in get_new_v_prime and once in the
// attention over the updated cache.  Here one pass over the Nc cached rows
// computes both: NU = Ln update slots (normalised new keys) and NA = (Hq/H) x Ln
// attention slots (scaled new queries; every cached row is visible to every new
// query).  The finish kernel forms x_new = v_new - sum, rounds it to bf16 as the
// cache stores it, and adds the Ln new rows (keys k_new, values x_new; query l
// sees new rows i <= l) to the attention.  Each slot keeps 16 accumulators per
// lane, so only small slot counts have an instance; decode_step_fused says which.
// ===========================================================================

// The cache rows stream through a per-thread ring of kStepStages stages in shared
// memory filled by cp.async: each lane copies exactly the 16 elements of K and of X
// it later reads, so a stage needs no synchronisation beyond the thread's own
// cp.async.wait_group, and kStepStages - 1 row iterations stay in flight while the
// current one computes.  Chunks are CB bytes (16 when every row start is 16-byte
// aligned, else 8) of CE = CB / 2 elements; lane j of a quarter-warp group holds
// chunks q at elements CE j + 8 CE q, so one copy instruction of the group covers
// 8 CB contiguous bytes of its row (whole sectors).  The bytes of a chunk at or past
// D, and whole chunks of rows past the split, are zero-filled (cp.async with a
// smaller source size) and read no memory.
constexpr int kStepStages = 5;
constexpr int kStepThreads = 256;
constexpr int kStepSmem = kStepStages * 2 * 32 * kStepThreads;  // bytes of the ring

template <int CB>
__device__ __forceinline__ void cp_async_zfill(uint32_t dst, const void* src, int bytes) {
  if constexpr (CB == 16)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void bf16x8_to_f32(const uint4 u, float* v) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// dot product of a lane's 16 elements (chunks of CE at ej + 8 CE q) with a row of
// 128 floats in shared memory
template <int CE>
__device__ __forceinline__ float dot_chunks(const float* row, int ej, const float (&k)[16]) {
  float d = 0.f;
#pragma unroll
  for (int q = 0; q < 16 / CE; ++q)
#pragma unroll
    for (int c = 0; c < CE / 4; ++c) {
      const float4 r4 = *reinterpret_cast<const float4*>(row + ej + 8 * CE * q + 4 * c);
      const float* kk = k + q * CE + 4 * c;
      d = fmaf(r4.x, kk[0], d);
      d = fmaf(r4.y, kk[1], d);
      d = fmaf(r4.z, kk[2], d);
      d = fmaf(r4.w, kk[3], d);
    }
  return d;
}

// dot product of two lanes' 16-element registers, four partial sums
__device__ __forceinline__ float dot16(const float (&a)[16], const float (&b)[16]) {
  float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll
  for (int i = 0; i < 16; i += 4) {
    d0 = fmaf(a[i], b[i], d0);
    d1 = fmaf(a[i + 1], b[i + 1], d1);
    d2 = fmaf(a[i + 2], b[i + 2], d2);
    d3 = fmaf(a[i + 3], b[i + 3], d3);
  }
  return (d0 + d1) + (d2 + d3);
}

template <int NU, int NA, int CB>
__global__ void __launch_bounds__(kStepThreads, 2) lucid_decode_step_partial_kernel(const DecodeStepArgs a) {
  constexpr int NS = NU + NA;
  constexpr int NQ = 32 / CB;    // chunks per lane per tensor row
  constexpr int CE = CB / 2;     // elements per chunk
  constexpr int kRow = 132;      // 128 values, the running maximum and the denominator, padded
  extern __shared__ __align__(16) unsigned char ring[];  // [stage][tensor][chunk][thread][CB]
  __shared__ __align__(16) float kq[NS][128];  // normalised new keys, then scaled queries
  __shared__ __align__(16) float red[8][NS][kRow];
  const int split = blockIdx.x, bh = blockIdx.y;
  const int b = bh / a.H, h = bh % a.H, gq = a.Hq / a.H;
  const long long BH = (long long)a.B * a.H;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int grp = lane >> 3, ej = (lane & 7) * CE;  // chunk q of this lane: elements ej + 8 CE q
  const float c1 = a.s * 1.4426950408889634f, c2 = 1.4426950408889634f / a.s;
  const float inv_d = 1.f / (float)a.D;
  const int r0 = split * a.rows_per_split;
  const int r1 = min(a.Nc, r0 + a.rows_per_split);
  const int nit = r1 > r0 ? (r1 - r0 + 31) / 32 : 0;  // row iterations (32 rows of the CTA each)
  const bf16* kbase = a.kc + (long long)b * a.kc_sb + (long long)h * a.kc_sh;
  const bf16* xbase = a.xc + (long long)b * a.xc_sb + (long long)h * a.xc_sh;
  const uint32_t ring0 = (uint32_t)__cvta_generic_to_shared(ring);
  // iteration `it` -> stage `st`: this thread's row r0 + 32 it + 4 warp + grp
  auto issue = [&](int it, int st) {
    const int row = r0 + 32 * it + 4 * warp + grp;
    const bool ok = row < r1;
    const bf16* kp = kbase + (long long)(ok ? row : r0) * a.kc_st;
    const bf16* xp = xbase + (long long)(ok ? row : r0) * a.xc_st;
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      const int el = ej + 8 * CE * q;
      const int bytes = ok ? max(0, min(CB, (a.D - el) * 2)) : 0;
      const uint32_t dk = ring0 + (uint32_t)((((st * 2 + 0) * NQ + q) * kStepThreads + tid) * CB);
      const uint32_t dx = ring0 + (uint32_t)((((st * 2 + 1) * NQ + q) * kStepThreads + tid) * CB);
      cp_async_zfill<CB>(dk, bytes ? (const void*)(kp + el) : (const void*)kbase, bytes);
      cp_async_zfill<CB>(dx, bytes ? (const void*)(xp + el) : (const void*)xbase, bytes);
    }
  };
#pragma unroll
  for (int i = 0; i < kStepStages - 1; ++i) {
    if (i < nit) issue(i, i);
    cp_async_commit();
  }
  if (warp < NU) {  // RMSNorm of new key `warp` (a whole warp per key)
    const bool act = lane * 4 < a.D;
    const float4 k4 = ld_bf16x4_d(a.kn + (long long)b * a.kn_sb + (long long)h * a.kn_sh +
                                  (long long)warp * a.kn_st + lane * 4, act);
    const float r = rsqrtf(warp_sum(k4.x * k4.x + k4.y * k4.y + k4.z * k4.z + k4.w * k4.w) * inv_d + a.eps);
    kq[warp][lane * 4 + 0] = k4.x * r;
    kq[warp][lane * 4 + 1] = k4.y * r;
    kq[warp][lane * 4 + 2] = k4.z * r;
    kq[warp][lane * 4 + 3] = k4.w * r;
  }
  for (int e = tid; e < NA * 128; e += blockDim.x) {
    const int sl = e >> 7, c = e & 127, j = sl / NU, l = sl % NU;  // query head h*gq + j, token l
    kq[NU + sl][c] = c < a.D ? __bfloat162float(a.q[(long long)b * a.q_sb + (long long)(h * gq + j) * a.q_sh +
                                                    (long long)l * a.q_st + c]) * c1
                             : 0.f;
  }
  __syncthreads();
  // this lane's 16 elements of every slot's vector (normalised new key / scaled query),
  // constant over the rows: held in registers instead of re-read from shared memory
  // for every row (the ring's writes and reads already keep the shared-memory pipe
  // busier than DRAM)
  float kr[NS][16];
#pragma unroll
  for (int t = 0; t < NS; ++t)
#pragma unroll
    for (int q = 0; q < 16 / CE; ++q)
#pragma unroll
      for (int c = 0; c < CE; ++c) kr[t][q * CE + c] = kq[t][ej + 8 * CE * q + c];
  float acc[NS][16], m[NA], l[NA];
#pragma unroll
  for (int t = 0; t < NS; ++t)
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[t][i] = 0.f;
#pragma unroll
  for (int t = 0; t < NA; ++t) {
    m[t] = -INFINITY;
    l[t] = 0.f;
  }
  int st = 0;
  for (int it = 0; it < nit; ++it) {
    {
      const int nx = it + kStepStages - 1;
      if (nx < nit) issue(nx, nx % kStepStages);
      cp_async_commit();
    }
    cp_async_wait<kStepStages - 1>();  // this thread's copies of iteration `it` have landed
    float k[16], x[16];
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      const unsigned char* pk = ring + (((st * 2 + 0) * NQ + q) * kStepThreads + tid) * CB;
      const unsigned char* px = ring + (((st * 2 + 1) * NQ + q) * kStepThreads + tid) * CB;
      if constexpr (CB == 16) {
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(pk), k + q * CE);
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(px), x + q * CE);
      } else {
        const uint2 uk = *reinterpret_cast<const uint2*>(pk), ux = *reinterpret_cast<const uint2*>(px);
        const __nv_bfloat162* hk = reinterpret_cast<const __nv_bfloat162*>(&uk);
        const __nv_bfloat162* hx = reinterpret_cast<const __nv_bfloat162*>(&ux);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const float2 fk = __bfloat1622float2(hk[i]), fx = __bfloat1622float2(hx[i]);
          k[q * CE + 2 * i] = fk.x;
          k[q * CE + 2 * i + 1] = fk.y;
          x[q * CE + 2 * i] = fx.x;
          x[q * CE + 2 * i + 1] = fx.y;
        }
      }
    }
    st = (st + 1 == kStepStages) ? 0 : st + 1;
    const bool valid = r0 + 32 * it + 4 * warp + grp < r1;  // uniform within the group
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) ss = fmaf(k[i], k[i], ss);
    const float rs = rsqrtf(grp_sum(ss) * inv_d + a.eps);
#pragma unroll
    for (int t = 0; t < NU; ++t) {
      const float d = grp_sum(dot16(kr[t], k)) * rs;
      const float e = valid ? exp2f(fmaf(d, c1, -c2)) : 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[t][i] = fmaf(e, x[i], acc[t][i]);
    }
#pragma unroll
    for (int t = 0; t < NA; ++t) {
      const float z = grp_sum(dot16(kr[NU + t], k));
      if (valid) {
        const float mn = fmaxf(m[t], z);
        const float al = exp2f(m[t] - mn), p = exp2f(z - mn);  // al = 0 while m is -inf
        l[t] = l[t] * al + p;
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[NU + t][i] = fmaf(p, x[i], acc[NU + t][i] * al);
        m[t] = mn;
      }
    }
  }
  cp_async_wait<0>();  // nothing of this thread's stays in flight past the loop
  // merge the 4 lane groups of the warp: sums for the update, (max, sum) for the attention
#pragma unroll
  for (int t = 0; t < NU; ++t)
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      acc[t][i] += __shfl_xor_sync(0xffffffffu, acc[t][i], 8);
      acc[t][i] += __shfl_xor_sync(0xffffffffu, acc[t][i], 16);
    }
#pragma unroll
  for (int t = 0; t < NA; ++t) {
    float M = fmaxf(m[t], __shfl_xor_sync(0xffffffffu, m[t], 8));
    M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 16));
    const float f = (m[t] == -INFINITY) ? 0.f : exp2f(m[t] - M);
    float L = l[t] * f;
    L += __shfl_xor_sync(0xffffffffu, L, 8);
    L += __shfl_xor_sync(0xffffffffu, L, 16);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float v = acc[NU + t][i] * f;
      v += __shfl_xor_sync(0xffffffffu, v, 8);
      v += __shfl_xor_sync(0xffffffffu, v, 16);
      acc[NU + t][i] = v;
    }
    m[t] = M;
    l[t] = L;
  }
  if (grp == 0) {
#pragma unroll
    for (int t = 0; t < NS; ++t)
#pragma unroll
      for (int c = 0; c < 4; ++c) {  // accumulators 4c..4c+3: chunk 4c / CE, offset 4c % CE
        const int col = ej + 8 * CE * (4 * c / CE) + (4 * c) % CE;
        *reinterpret_cast<float4*>(&red[warp][t][col]) =
            make_float4(acc[t][4 * c], acc[t][4 * c + 1], acc[t][4 * c + 2], acc[t][4 * c + 3]);
      }
    if (lane == 0) {
#pragma unroll
      for (int t = 0; t < NA; ++t) {
        red[warp][NU + t][128] = m[t];
        red[warp][NU + t][129] = l[t];
      }
    }
  }
  __syncthreads();
  // merge the 8 warps into this split's partials
  for (int e = tid; e < NS * 128; e += blockDim.x) {
    const int sl = e >> 7, c = e & 127;
    if (sl < NU) {
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) sum += red[w][sl][c];
      a.part_u[(((long long)split * BH + bh) * NU + sl) * 128 + c] = sum;
    } else {
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < 8; ++w) M = fmaxf(M, red[w][sl][128]);
      float L = 0.f, S = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const float f = (red[w][sl][128] == -INFINITY) ? 0.f : exp2f(red[w][sl][128] - M);
        L += f * red[w][sl][129];
        S += f * red[w][sl][c];
      }
      float* dst = a.part_a + (((long long)split * BH + bh) * NA + (sl - NU)) * 130;
      dst[c] = S;
      if (c == 0) {
        dst[128] = M;
        dst[129] = L;
      }
    }
  }
}

template <int NU, int NA>
__global__ void __launch_bounds__(256) lucid_decode_step_finish_kernel(const DecodeStepArgs a) {
  __shared__ __align__(16) float xs[NU][128];  // x_new as the cache holds it (bf16 values)
  __shared__ float zs[NA][NU];                 // new query x new key scores (log2 domain)
  const int bh = blockIdx.x, b = bh / a.H, h = bh % a.H, gq = a.Hq / a.H;
  const long long BH = (long long)a.B * a.H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float sm = a.s * 1.4426950408889634f;
  for (int e = threadIdx.x; e < NU * 128; e += blockDim.x) {
    const int l = e >> 7, c = e & 127;
    float xv = 0.f;
    if (c < a.D) {
      float sum = 0.f;
      for (int sp = 0; sp < a.nsplit; ++sp) sum += a.part_u[(((long long)sp * BH + bh) * NU + l) * 128 + c];
      const float v = __bfloat162float(a.vn[(long long)b * a.vn_sb + (long long)h * a.vn_sh +
                                            (long long)l * a.vn_st + c]);
      const bf16 xb = __float2bfloat16(v - sum);
      a.xo[(long long)b * a.xo_sb + (long long)h * a.xo_sh + (long long)l * a.xo_st + c] = xb;
      xv = __bfloat162float(xb);
    }
    xs[l][c] = xv;
  }
  for (int p = warp; p < NA * NU; p += 8) {  // one warp per (slot, new key) pair
    const int sl = p / NU, i = p % NU, j = sl / NU, l = sl % NU;
    float z = -INFINITY;
    if (i <= l) {  // causal among the new tokens (uniform within the warp)
      const bool act = lane * 4 < a.D;
      const float4 q4 = ld_bf16x4_d(a.q + (long long)b * a.q_sb + (long long)(h * gq + j) * a.q_sh +
                                    (long long)l * a.q_st + lane * 4, act);
      const float4 k4 = ld_bf16x4_d(a.kn + (long long)b * a.kn_sb + (long long)h * a.kn_sh +
                                    (long long)i * a.kn_st + lane * 4, act);
      z = warp_sum(q4.x * sm * k4.x + q4.y * sm * k4.y + q4.z * sm * k4.z + q4.w * sm * k4.w);
    }
    if (lane == 0) zs[sl][i] = z;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < NA * 128; e += blockDim.x) {
    const int sl = e >> 7, c = e & 127, j = sl / NU, l = sl % NU;
    if (c >= a.D) continue;
    float M = -INFINITY;
    for (int sp = 0; sp < a.nsplit; ++sp)
      M = fmaxf(M, a.part_a[(((long long)sp * BH + bh) * NA + sl) * 130 + 128]);
#pragma unroll
    for (int i = 0; i < NU; ++i) M = fmaxf(M, zs[sl][i]);
    float L = 0.f, S = 0.f;
    for (int sp = 0; sp < a.nsplit; ++sp) {
      const float* pp = a.part_a + (((long long)sp * BH + bh) * NA + sl) * 130;
      const float f = (pp[128] == -INFINITY) ? 0.f : exp2f(pp[128] - M);
      L += f * pp[129];
      S += f * pp[c];
    }
#pragma unroll
    for (int i = 0; i < NU; ++i) {
      if (i <= l) {
        const float p = exp2f(zs[sl][i] - M);
        L += p;
        S += p * xs[i][c];
      }
    }
    a.o[(long long)b * a.o_sb + (long long)(h * gq + j) * a.o_sh + (long long)l * a.o_st + c] =
        __float2bfloat16(S / L);
  }
}

template <int NU, int NA, int CB>
static cudaError_t launch_decode_step_cb(const DecodeStepArgs& a, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(lucid_decode_step_partial_kernel<NU, NA, CB>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, kStepSmem);
  if (e != cudaSuccess) return e;
  lucid_decode_step_partial_kernel<NU, NA, CB><<<dim3(a.nsplit, a.B * a.H), kStepThreads, kStepSmem, st>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  lucid_decode_step_finish_kernel<NU, NA><<<a.B * a.H, 256, 0, st>>>(a);
  return cudaGetLastError();
}

// 16-byte chunks when every row of both caches starts on a 16-byte boundary
template <int NU, int NA>
static cudaError_t launch_decode_step_t(const DecodeStepArgs& a, cudaStream_t st) {
  const bool a16 = ((reinterpret_cast<uintptr_t>(a.kc) | reinterpret_cast<uintptr_t>(a.xc)) & 15u) == 0 &&
                   ((a.kc_sb | a.kc_sh | a.kc_st | a.xc_sb | a.xc_sh | a.xc_st) & 7) == 0;
  return a16 ? launch_decode_step_cb<NU, NA, 16>(a, st) : launch_decode_step_cb<NU, NA, 8>(a, st);
}

bool decode_step_fused(int gq, int Ln) {
  return (Ln == 1 && (gq == 1 || gq == 2)) || (Ln == 2 && gq == 1);
}

cudaError_t launch_decode_step(DecodeStepArgs a, cudaStream_t st) {
  if (a.B == 0 || a.H == 0 || a.Ln == 0) return cudaSuccess;
  a.nsplit = decode_splits(a.B, a.H, a.Nc);
  a.rows_per_split = (a.Nc + a.nsplit - 1) / a.nsplit;
  const int gq = a.Hq / a.H;
  if (a.Ln == 1 && gq == 1) return launch_decode_step_t<1, 1>(a, st);
  if (a.Ln == 1 && gq == 2) return launch_decode_step_t<1, 2>(a, st);
  if (a.Ln == 2 && gq == 1) return launch_decode_step_t<2, 2>(a, st);
  return cudaErrorInvalidValue;
}

}  // namespace lb
