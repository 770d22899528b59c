// Shared definitions of the LUCID kernels: problem geometry, argument
// structs, and the workspace layout contract between forward and backward.
#pragma once
#include "sm100.cuh"

namespace lb {

using bf16 = __nv_bfloat16;

constexpr int kBlock = 128;      // rows per block (queries / keys / solve rows)
constexpr int kHeadDim = 128;    // head dimension handled by the tensor-core kernels
constexpr int kTileBytes = kBlock * kHeadDim * 2;  // 32 KB bf16 tile

// Row statistics + diagonal-block inverse (CUDA cores).
struct PrepArgs {
  int B, H, N, NB, Npad;     // H = key/value heads
  float s, eps;              // s = D^-1/2, eps = RMSNorm epsilon
  const bf16* k;             // raw keys, element strides below
  long long k_sb, k_sh, k_sn;
  bf16* khat;                // [B][H][Npad][128]  RMS-normalised keys (bf16)
  float* rstd;               // [B*H][Npad]
  float* dinv;               // [B*H][Npad]        1 / P_rr
  bf16* u;                   // [B*H][NB][128][128] (I + L~)^-1 - I per diagonal block
  // block range [blk0, blk1) (blk1 == 0: NB); khat_only: row statistics and k^ only
  // (blocks whose solve runs elsewhere, e.g. another rank's chunk of the sequence)
  int blk0 = 0, blk1 = 0, khat_only = 0;
  // logical head dimension of the RMS mean (rows hold 128 elements; a smaller head
  // dimension is zero-padded to 128)
  int D = kHeadDim;
};

// Forward tile engine (solve or attention).
struct FwdArgs {
  int B, Hq, Hkv, N, NB, Npad;
  float scale;               // s (solve) or softmax scale (attention)
  // solve
  const float* dinv;
  const bf16* v;
  long long v_sb, v_sh, v_sn;
  bf16* x;                   // [B][Hkv][Npad][128]
  int* flags;                // [B*Hkv][NB], zero before launch, 1 = X block ready
  // attention
  bf16* o;
  long long o_sb, o_sh, o_sn;
  float* lse;                // [B*Hq][Npad], log2 domain
  bf16* o_res = nullptr;     // optional, O's strides: bf16(O_fp32 - bf16(O_fp32)), the rounding
                             // residual of O, so the backward's rowsum(dO * O) sees O to ~16 bits
  int* status;
  // row-block pairs [pp0, pp1) processed (pp1 == 0: all; earlier blocks are solved
  // elsewhere and their flags already set) and an optional cap on the persistent
  // grid (0: #SMs)
  int pp0 = 0, pp1 = 0, max_ctas = 0;
  // solve, chain schedule (nchain > 0): CTAs [0, nchain) each run the diagonal steps of
  // one (batch, kv head); the other CTAs stream row-block pairs and hand each row
  // block i to its chain as the partial sum W_i = V_i - sum_{j < i-kChainLook} E_ij X_j
  // (fp32, in a ring of kChainWRing slots per head) plus the kChainLook tiles
  // E_{i,i-kChainLook} .. E_{i,i-1} (bf16, in the shared-memory image of a K-major
  // operand tile)
  int nchain = 0;
  float attn_scale = 0.f;    // fused launch: the attention items' softmax scale
  int fuse_lag = 2;          // fused launch: attention pair p follows the solve items of pair p + fuse_lag
  // attention items: the head dimension rounded up to 16 (rows hold 128 elements, zero
  // from D on): the K extent of Q K^T and the N extent of P X, and O's columns from it
  // on are written as zeros
  int attn_d16 = kHeadDim;
  int* cflags = nullptr;     // [B*Hkv][NB]: 1 = E tiles of row block i written, 2 = W_i too
  float* wring = nullptr;    // [B*Hkv][kChainWRing][32][128][4] fp32
  bf16* etiles = nullptr;    // [B*Hkv][NB][kChainLook][128*128] bf16
};
// Chain schedule: key blocks i-kChainLook .. i-1 of row block i are multiplied by the
// chain CTA, the rest by the workers, so a worker has kChainLook + 1 chain steps to
// turn X_{i-kChainLook-1} into W_i.
constexpr int kChainLook = 3;
// W slots per head.  The worker writes W_i only after X_{i-kChainLook-1} is published,
// i.e. after the chain finished step i-kChainLook-1; a ring of kChainLook + 1 slots or
// more never overwrites a W that the chain has not read.
constexpr int kChainWRing = 8;
static_assert(kChainWRing >= kChainLook + 1, "W ring too small");

// Backward tile engines (column pass and row pass; attention or solve).
struct BwdArgs {
  int B, Hq, Hkv, N, NB, Npad;
  float scale;
  // attention backward
  const float* lse;          // [B*Hq][Npad] log2 domain
  const float* delta;        // [B*Hq][Npad]  rowsum(dO * O)
  float* dx;                 // column pass: dL/dX  [B][Hkv][Npad][128] fp32
  float* dk_col;             // column pass: dK (attention) or dK^ column part (solve), fp32
  bf16* dq;                  // row pass (attention): dQ, strided [B,Hq,N,128]
  long long dq_sb, dq_sh, dq_sn;
  float* dk_row;             // row pass (solve): dK^ row part [B][Hkv][Npad][128] fp32
  // solve backward
  const float* dinv;
  const float* dx_in;        // dX from the attention backward (fp32)
  bf16* dv;                  // [B][Hkv][Npad][128] bf16 (MMA operand + output source)
  int* flags;                // [B*Hkv][NB], zero before launch
  int* status;
  // output blocks [blk0, blk1) (blk1 == 0: NB): column blocks of the column pass, row
  // blocks of the row pass; the operand blocks on the other side span all of [0, NB)
  // (context parallel: the rest of the sequence is held as received from other ranks).
  // max_ctas caps the persistent grid (0: #SMs).
  int blk0 = 0, blk1 = 0, max_ctas = 0;
  // stored-tile schedule: the column pass also stores every packed dS^T (attention) /
  // dG^T (solve) tile it computes, and the row pass streams them instead of
  // recomputing S and dP (tensor map passed to both kernels)
  int store_tiles = 0;
  // attention, stored-tile schedule: the tiles' base address, [B*Hq][tile_rows][128] bf16
  // (tile_rows = (NB (NB + 1) / 2 + NB) * 128: the dS^T tiles, then one bf16 residual tile
  // per diagonal block, written by the column pass with plain stores)
  bf16* tiles = nullptr;
};

// Decode step (get_new_v_prime) and decode attention: one pass over the caches.
struct DecodeArgs {
  int B, H, Ln, Nc, nsplit, rows_per_split;
  float s, eps;
  const bf16* kn; long long kn_sb, kn_sh, kn_st;   // new keys    [B,H,Ln,D] (attention: queries [B,Hq,Ln,D])
  const bf16* vn; long long vn_sb, vn_sh, vn_st;   // new values  [B,H,Ln,D]
  const bf16* kc; long long kc_sb, kc_sh, kc_st;   // cached keys [B,H,Nc,D]
  const bf16* xc; long long xc_sb, xc_sh, xc_st;   // cached solved values [B,H,Nc,D]
  bf16* out; long long o_sb, o_sh, o_st;
  float* part;                                     // per-split partial sums
  int Hq;                                          // attention: query heads (H = kv heads)
  int D = kHeadDim;                                // logical head dimension of the RMS mean
};

// Fused decode step: get_new_v_prime and the new queries' attention in one pass
// over the cache (csrc/lucid_decode.cu)
struct DecodeStepArgs {
  int B, H, Hq, Ln, Nc, D, nsplit, rows_per_split;
  float s, eps;
  const bf16* q; long long q_sb, q_sh, q_st;       // new queries [B,Hq,Ln,D]
  const bf16* kn; long long kn_sb, kn_sh, kn_st;   // new keys [B,H,Ln,D]
  const bf16* vn; long long vn_sb, vn_sh, vn_st;   // new values [B,H,Ln,D]
  const bf16* kc; long long kc_sb, kc_sh, kc_st;   // cached keys [B,H,Nc,D]
  const bf16* xc; long long xc_sb, xc_sh, xc_st;   // cached solved values [B,H,Nc,D]
  bf16* xo; long long xo_sb, xo_sh, xo_st;         // solved new values [B,H,Ln,D]
  bf16* o; long long o_sb, o_sh, o_st;             // attention output [B,Hq,Ln,D]
  float* part_u;                                   // [nsplit][B*H][Ln][128] cache sums
  float* part_a;                                   // [nsplit][B*H][Hq/H*Ln][130] softmax partials
};

}  // namespace lb
