// Shared definitions of the LUCID-Path kernels (the Householder-path
// preconditioner of lucid_path/triton_code/).
//
// Per (batch, query head) and 128-row blocks i, j:
//   H_t      = I - beta_t w_t w_t^T
//   T_i      = (I + stril(diag(beta) W_i W_i^T))^-1        (UT transform)
//   W2_i     = T_i diag(beta) W_i,   G_i = I - W_i^T W2_i    (= H_last ... H_first of block i)
//   Q_new_i  = Q_i - tril(Q_i W_i^T) W2_i
//   K_new_i  = K_i - (T_i stril(diag(beta) W_i K_i^T))^T W_i
//   off-diagonal scores, i > j:  L_ij = exp(s Q~_i^{(j)} K_new_j^T - 1/s),
//       Q~_i^{(i-1)} = Q_new_i,  Q~_i^{(j-1)} = Q~_i^{(j)} G_j
//   diagonal block: L_ii = stril(exp(s A_ii - 1/s)),
//       A_ii = Q_i K_i^T - tril(Q_i W_i^T) T_i stril(diag(beta) W_i K_i^T)
//   O = (I + L)^-1 V
// (triangular_solve_fwd.py:118-221).
//
// Internal buffers are row-major with 128-column rows.  Per-block matrices
// are [heads][NB][128][128]; pair tiles (i > j) are [heads][NPAIR][128][128]
// with pair(i, j) = i (i - 1) / 2 + j.
#pragma once
#include "lucid_common.cuh"

namespace lb {

__host__ __device__ __forceinline__ long long path_pair(int i, int j) {
  return (long long)i * (i - 1) / 2 + j;
}

// A batch of 128 x 128 matrices addressed as
//   ptr + b*s_b + (h / hdiv)*s_h + blk*s_blk + r*s_row + c
// for batch index z = (b * Hx + h) * NB + blk.  Rows with blk*128 + r >= rows
// read as zero and are not written.
struct PMat {
  void* ptr = nullptr;
  int fp32 = 0;
  long long s_row = 128, s_blk = 128 * 128, s_h = 0, s_b = 0;
  int hdiv = 1;
  int rows = 1 << 30;
};

// A per-row vector (beta) addressed as ptr + b*s_b + (h / hdiv)*s_h + t*s_row.
struct PVec {
  const void* ptr = nullptr;
  int fp32 = 0;
  long long s_row = 1, s_h = 0, s_b = 0;
  int hdiv = 1;
  long long rows = 1LL << 40;   // entries t >= rows read as zero
};

enum : int { kMaskNone = 0, kMaskTril = 1, kMaskStril = 2 };
enum : int { kEpiIdentity = 0, kEpiPathExp = 1 };

struct POperand {
  PMat m;
  int trans = 0;        // use the stored matrix transposed
  int mask = kMaskNone; // mask of the stored matrix (row r, column c)
  float scale = 1.f;
  PVec rsc;             // optional scale of every stored row
  int lo = 0;           // use the bf16 rounding residual v - bf16(v) of the stored values
};

// C = out_mask(epi( rsc_out .* sum_p op(A_p) op(B_p)  +  sum_c beta_c rsc_c .* C_c ))
struct BGemmArgs {
  int nprod = 1;
  POperand A[3], B[3];
  int nc = 0;
  PMat C[2];
  float cbeta[2] = {1.f, 1.f};
  PVec crsc[2];
  PVec orsc;
  int epi = kEpiIdentity;
  float s = 1.f;
  int out_mask = kMaskNone;
  PMat O, O2;           // O2 optional second destination (e.g. bf16 and fp32 copies)
  int Bn = 0, Hx = 0, NB = 0;
  int* status = nullptr;
};

// Triangular inverse: Z = (I + stril(M))^-1 in fp32.
struct TriInvArgs {
  PMat M;               // input (strictly-lower part used)
  PMat Z;               // optional fp32 Z
  PMat U;               // optional Z - I (bf16 or fp32)
  PMat Mcopy;           // optional copy of stril(M) (e.g. bf16)
  int Bn = 0, Hx = 0, NB = 0;
};

struct PathScoresArgs {
  int B, HQ, H, G, NB, NPAIR;
  float s;
  const float* qn;      // [B*HQ][Npad][128] fp32 Q_new
  bf16* L;              // [B*HQ][NPAIR][128][128]
  int* status;
};

struct PathSolveArgs {
  int B, HQ, H, G, T, NB, NPAIR;
  const bf16* rhs;      // forward: v [B,T,H,V]; transposed: do [B,T,HQ,V]
  long long r_sb, r_sh, r_st;
  bf16* xbuf;           // [B*HQ][Npad][128] solution (MMA operand for later blocks)
  bf16* out;            // optional strided copy [B,T,HQ,V] (forward o)
  long long o_sb, o_sh, o_st;
  int* flags;           // [B*HQ][NB], zero before launch
  int* status;
};

struct PathRowArgs {
  int B, HQ, H, G, NB, NPAIR;
  float s;
  const bf16* L;        // [B*HQ][NPAIR][128][128]
  const bf16* Ld;       // [B*HQ][NB][128][128]
  bf16* dA;             // [B*HQ][NPAIR][128][128]
  bf16* dAd;            // [B*HQ][NB][128][128]
  float* dqn;           // [B*HQ][Npad][128]
  int* status;
};

struct PathColArgs {
  int B, HQ, H, G, NB, NPAIR;
  float* dkn;           // [B*HQ][Npad][128]  sum_i dA_ij^T Q~_i^{(j)}
  float* dw2;           // [B*HQ][Npad][128]  -W_j Phi_j
  float* dw;            // [B*HQ][Npad][128]  -W2_j Phi_j^T
  int* status;
};

struct PathAttnArgs {
  int B, HQ, H, G, T, NB;
  float s;
  const float* qn;      // [B*HQ][Npad][128] fp32 Q_new
  const float* ad;      // [B*HQ][NB][128][128] fp32 diagonal-block scores (tril, raw)
  bf16* o;              // caller's [B, T, HQ, V]
  long long o_sb, o_st, o_sh;
  float* lse;           // caller's [B, T, HQ] (log2 domain)
  long long l_sb, l_st, l_sh;
  int* status;
};

enum : int { kTagPathAttn = 14 };
enum : int { kTagPathGemm = 8, kTagPathScores = 9, kTagPathSolve = 10, kTagPathSolveT = 11,
             kTagPathRow = 12, kTagPathCol = 13 };



// Packed bf16 A-operand address in TMEM of K-slice kk when each 64-column
// half hf of a 128-column fp32 region was rewritten in place as 32 columns
// of bf16 pairs starting at region + 64*hf.
__device__ __forceinline__ uint32_t packed_half_kslice(uint32_t region, int kk) {
  return region + 64u * (uint32_t)(kk >> 2) + 8u * (uint32_t)(kk & 3);
}

}  // namespace lb
