/*
 * lucid_b200 — C ABI of the B200 (sm_100a) LUCID attention kernels.
 *
 * LUCID attention computes  O = softmax(s Q K^T + causal) X,  X = P^-1 V,
 * P = tril(exp(s K^ K^T - 1/s)),  K^ = RMSNorm(K) (no affine),  s = D^-1/2.
 *
 * Conventions shared by every entry point
 *   - All tensors are device pointers to bf16 unless stated otherwise.
 *   - "Strided" tensors are 4-D [B, H, N, D] views given by element strides
 *     (sb, sh, sn); the innermost (D) stride is 1.  Strides and base
 *     addresses must be multiples of 8 elements (16 bytes).
 *   - "Internal" tensors are contiguous [B, H, Npad, D] (or [B, H, Npad])
 *     buffers with Npad = lucid_padded_len(N); the library owns their
 *     contents, the caller owns their memory.
 *   - D is the head dimension, 1 <= D <= 128.  lucid_solve_*, lucid_attn_*
 *     and lucid_cp_*: every row holds 128 elements (the tensor-core width of
 *     this build) and a smaller head dimension is zero-padded to 128 by the
 *     caller (columns D..127 zero); D enters only the RMS mean of K^ (the
 *     mean over D, not 128).  lucid_decode_*: rows hold D elements, D a
 *     multiple of 4 (no padding).  lucid_path_*: D = 128 (zero-pad smaller
 *     head dimensions: the Householder products act as the identity there).
 *   - Hq must be a multiple of Hkv (grouped-query attention).
 *   - Every call is asynchronous on `stream` (a cudaStream_t, 0 = legacy
 *     default stream), performs no host synchronisation and allocates no
 *     memory.  Scratch memory comes from the caller's `workspace`, whose
 *     size is given by the matching *_workspace_bytes function.
 *   - Return value: LUCID_OK, or one of the error codes below; nothing is
 *     launched when an error is returned.
 *   - The kernels record run-time failures (a bounded wait that timed out)
 *     in a status word inside the workspace; lucid_workspace_status_offset
 *     gives its byte offset for callers that want to read it back.
 */
#ifndef LUCID_B200_H_
#define LUCID_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LUCID_OK 0
#define LUCID_ERR_SHAPE 1       /* unsupported B/H/N/D combination */
#define LUCID_ERR_ALIGN 2       /* pointer or stride not 16-byte aligned */
#define LUCID_ERR_WORKSPACE 3   /* workspace missing or too small */
#define LUCID_ERR_TENSORMAP 4   /* TMA descriptor creation failed */
#define LUCID_ERR_LAUNCH 5      /* CUDA launch error */
#define LUCID_ERR_TOO_LARGE 6   /* problem exceeds a fixed-size internal buffer */

/* Library version, e.g. 100 for 0.1.0. */
int lucid_version(void);

/* Rows of the internal buffers: N rounded up to a multiple of 128. */
int lucid_padded_len(int N);

/* Byte offset of the int32 run-time status word inside every workspace. */
size_t lucid_workspace_status_offset(void);

/*
 * Solve forward: X = P^-1 V.
 * Replaces LucidAttention.get_v_prime (modeling_lucid.py:551-574: dense
 * branch, k_norm + einsum + exp + torch.linalg.solve_triangular) and the
 * blockwise Lucid_Tril_Solver.forward (modeling_lucid.py:285-312).
 * In : k, v strided [B,H,N,D]; scale = s; eps = RMSNorm epsilon.
 * Out: x    internal bf16 [B,H,Npad,D]   solved values
 *      khat internal bf16 [B,H,Npad,D]   RMS-normalised keys   (saved)
 *      u    bf16 [B,H,Npad/128,128,128]  diagonal-block inverses (saved)
 *      rstd, dinv internal fp32 [B,H,Npad]                         (saved)
 */
size_t lucid_solve_fwd_workspace_bytes(int B, int H, int N, int D);
/* Workspace of the chain schedule: with at least this many bytes (16-byte aligned) the
 * solve runs each head's diagonal steps in one CTA that keeps its X tiles in shared
 * memory, while the other CTAs publish the partial row sums, whenever that is faster
 * on this device (few heads per GPU: their dependency chains, not the GEMM work, set
 * the time).  Equals lucid_solve_fwd_workspace_bytes when the wavefront schedule is
 * faster.  Same results up to the fp32 summation order of the row sums.
 * LUCID_B200_SOLVE_SCHEDULE=chain or =wavefront in the environment forces a schedule
 * (the size follows). */
size_t lucid_solve_fwd_fast_workspace_bytes(int B, int H, int N, int D);
int lucid_solve_fwd(int B, int H, int N, int D, float scale, float eps,
                    const void* k, int64_t k_sb, int64_t k_sh, int64_t k_sn,
                    const void* v, int64_t v_sb, int64_t v_sh, int64_t v_sn,
                    void* x, void* khat, void* u, float* rstd, float* dinv,
                    void* workspace, size_t workspace_bytes, void* stream);

/*
 * Solve forward that allocates nothing and takes no workspace.
 * It has no counterpart in the reference: it exists for callers that cannot call
 * cudaMalloc, e.g. a plugin hosted by an engine that owns all device memory
 * and forbids allocations after start-up, or a code path that cannot afford
 * the implicit device synchronisation of an allocation.
 * Same arguments as lucid_solve_fwd minus the workspace, and the same x, khat, u,
 * rstd and dinv.  Its scratch (the per-block dependency flags and the run-time
 * status word) is a fixed static device array of LUCID_NOALLOC_SCRATCH_BYTES bytes
 * that every GPU loading the library holds until the process exits:
 *   - B * H * ceil(N / 128) must not exceed LUCID_NOALLOC_MAX_BLOCKS, else the
 *     call returns LUCID_ERR_TOO_LARGE and launches nothing;
 *   - the first call on each device looks up the array's device address, so
 *     make that first call before any stream capture;
 *   - every call clears and reuses the same array: calls whose execution
 *     overlaps on the GPU (e.g. on two streams) race, so serialise them;
 *   - the status word of the last call (0, or a bounded wait that ran out, as
 *     in every workspace) stays in the array until the next call clears it:
 *     lucid_solve_fwd_noalloc_status reads it.
 */
#define LUCID_NOALLOC_MAX_BLOCKS 16384
#define LUCID_NOALLOC_SCRATCH_BYTES (256 + 4 * LUCID_NOALLOC_MAX_BLOCKS)
int lucid_solve_fwd_noalloc(int B, int H, int N, int D, float scale, float eps,
                            const void* k, int64_t k_sb, int64_t k_sh, int64_t k_sn,
                            const void* v, int64_t v_sb, int64_t v_sh, int64_t v_sn,
                            void* x, void* khat, void* u, float* rstd, float* dinv, void* stream);
/* Copy the run-time status word of the last lucid_solve_fwd_noalloc call on the
 * current device into *status (host memory), ordered on `stream` after the work
 * queued there before it: with pinned memory the value is valid once the stream
 * has reached this point (synchronise it), with pageable memory when the call
 * returns.  No allocation; LUCID_ERR_LAUNCH if the copy cannot be queued. */
int lucid_solve_fwd_noalloc_status(int* status, void* stream);

/*
 * Decode step of the solve: x_new = v_new - exp(scale k^_new K^_cache^T - 1/scale) X_cache.
 * Replaces LucidAttention.get_new_v_prime (modeling_lucid.py:576-598) with the
 * reference's cache convention (raw keys and solved values, :479-481); as in the
 * reference the Ln new tokens do not see one another and the diagonal P_rr is not
 * divided out.  k^ = RMSNorm(k) without affine (eps), computed on the fly for the
 * cache.  All tensors bf16 [B, H, L, D] strided (sb, sh, sn), strides multiples of
 * 4 elements; k_new / v_new / x_new have L = Ln, k_cache / x_cache L = Nc.
 * The decode entry points take B x (query) heads <= 65535 (one grid row each).
 */
size_t lucid_decode_workspace_bytes(int B, int H, int Ln, int Nc, int D);
int lucid_decode_update(int B, int H, int Ln, int Nc, int D, float scale, float eps,
                        const void* k_new, int64_t kn_sb, int64_t kn_sh, int64_t kn_sn,
                        const void* v_new, int64_t vn_sb, int64_t vn_sh, int64_t vn_sn,
                        const void* k_cache, int64_t kc_sb, int64_t kc_sh, int64_t kc_sn,
                        const void* x_cache, int64_t xc_sb, int64_t xc_sh, int64_t xc_sn,
                        void* x_new, int64_t o_sb, int64_t o_sh, int64_t o_sn,
                        void* workspace, size_t workspace_bytes, void* stream);

/*
 * Decode attention: o = softmax(scale q K_cache^T + causal) X_cache for Ln new
 * queries at positions Nc - Ln .. Nc - 1 of a cache that already holds them
 * (eager_lucid_attention_forward, modeling_lucid.py:505-549, after the cache
 * update of :479-481).  q [B, Hq, Ln, D], caches [B, Hkv, Nc, D], o [B, Hq, Ln, D]
 * (pass the strides of a [B, Ln, Hq, D] tensor for the reference's layout).
 */
size_t lucid_decode_attn_workspace_bytes(int B, int Hq, int Ln, int Nc, int D);
int lucid_decode_attn(int B, int Hq, int Hkv, int Ln, int Nc, int D, float scale,
                      const void* q, int64_t q_sb, int64_t q_sh, int64_t q_sn,
                      const void* k_cache, int64_t kc_sb, int64_t kc_sh, int64_t kc_sn,
                      const void* x_cache, int64_t xc_sb, int64_t xc_sh, int64_t xc_sn,
                      void* o, int64_t o_sb, int64_t o_sh, int64_t o_sn,
                      void* workspace, size_t workspace_bytes, void* stream);

/*
 * Fused decode step: lucid_decode_update and the new queries' attention in one
 * pass over the cache (the reference's decoding forward, modeling_lucid.py:467-481
 * then :505-549, reads the cache in get_new_v_prime and again in the attention).
 * k_cache / x_cache [B, Hkv, Nc, D] hold the tokens BEFORE this step; the step
 * writes x_new [B, Hkv, Ln, D] (the solved values of the new tokens, as the cache
 * update of :479-481 stores them) and o [B, Hq, Ln, D] = softmax(scale q [K_cache;
 * k_new]^T + causal) [X_cache; x_new], query l at position Nc + l (pass the strides
 * of a [B, Ln, Hq, D] tensor for the reference's layout).  The caller appends
 * k_new / x_new to its cache.  lucid_decode_step_fused(Hq, Hkv, Ln) is 1 for the
 * shapes with a single-pass kernel (Ln 1 with Hq/Hkv 1 or 2, Ln 2 with Hq = Hkv);
 * any other shape returns LUCID_ERR_SHAPE (use lucid_decode_update, the cache
 * append and lucid_decode_attn).  Alignment as lucid_decode_update, q included.
 */
int lucid_decode_step_fused(int Hq, int Hkv, int Ln);
size_t lucid_decode_step_workspace_bytes(int B, int Hq, int Hkv, int Ln, int Nc, int D);
int lucid_decode_step(int B, int Hq, int Hkv, int Ln, int Nc, int D, float scale, float eps,
                      const void* q, int64_t q_sb, int64_t q_sh, int64_t q_sn,
                      const void* k_new, int64_t kn_sb, int64_t kn_sh, int64_t kn_sn,
                      const void* v_new, int64_t vn_sb, int64_t vn_sh, int64_t vn_sn,
                      const void* k_cache, int64_t kc_sb, int64_t kc_sh, int64_t kc_sn,
                      const void* x_cache, int64_t xc_sb, int64_t xc_sh, int64_t xc_sn,
                      void* x_new, int64_t xn_sb, int64_t xn_sh, int64_t xn_sn,
                      void* o, int64_t o_sb, int64_t o_sh, int64_t o_sn,
                      void* workspace, size_t workspace_bytes, void* stream);

/*
 * Attention forward: O = softmax(scale Q K^T + causal) X.
 * Replaces LucidAttention.eager_lucid_attention_forward
 * (modeling_lucid.py:505-549; SDPA with repeat_kv, is_causal=True).
 * In : q strided [B,Hq,N,D]; k strided [B,Hkv,N,D] (raw keys);
 *      x internal bf16 [B,Hkv,Npad,D].
 * Out: o strided [B,Hq,N,D] (pass the strides of the caller's output, e.g.
 *      the [B,N,Hq,D] layout the reference returns); lse internal fp32
 *      [B,Hq,Npad] (log2 domain, saved for the backward); o_res optional (NULL:
 *      not written), a bf16 buffer with o's strides that receives the rounding
 *      residual bf16(O - bf16(O)) of the fp32 output.  Passed on to lucid_attn_bwd
 *      it makes the backward's rowsum(dO o O) use O to about 16 significant bits
 *      instead of bf16's 8 (the dominant term of dQ's deviation from a float32
 *      reference when attention is spread over many keys).
 */
size_t lucid_attn_fwd_workspace_bytes(int B, int Hq, int Hkv, int N, int D);
int lucid_attn_fwd(int B, int Hq, int Hkv, int N, int D, float scale,
                   const void* q, int64_t q_sb, int64_t q_sh, int64_t q_sn,
                   const void* k, int64_t k_sb, int64_t k_sh, int64_t k_sn,
                   const void* x,
                   void* o, int64_t o_sb, int64_t o_sh, int64_t o_sn,
                   float* lse, void* o_res, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Layer forward: lucid_solve_fwd then lucid_attn_fwd in one call, with the same
 * arguments and outputs as the two (one scale for both, as LucidAttention uses
 * self.scaling for get_v_prime and for the attention).
 * Replaces LucidAttention.get_v_prime followed by eager_lucid_attention_forward
 * (modeling_lucid.py:463 and :489, the two halves of LucidAttention.forward).
 * With the chain schedule (workspace of lucid_fused_fwd_workspace_bytes, few heads per
 * GPU) the solve and the attention run as ONE launch: the attention's row-block pairs
 * start as soon as the X blocks they read are published.  Otherwise the two stages run
 * as two launches.  Same results either way.
 * In : q strided [B,Hq,N,D]; k, v strided [B,Hkv,N,D]; scale = s; eps.
 * Out: x, khat, u, rstd, dinv as lucid_solve_fwd; o, lse, o_res as lucid_attn_fwd.
 */
size_t lucid_fused_fwd_workspace_bytes(int B, int Hq, int Hkv, int N, int D);
int lucid_fused_fwd(int B, int Hq, int Hkv, int N, int D, float scale, float eps,
                    const void* q, int64_t q_sb, int64_t q_sh, int64_t q_sn,
                    const void* k, int64_t k_sb, int64_t k_sh, int64_t k_sn,
                    const void* v, int64_t v_sb, int64_t v_sh, int64_t v_sn,
                    void* x, void* khat, void* u, float* rstd, float* dinv,
                    void* o, int64_t o_sb, int64_t o_sh, int64_t o_sn,
                    float* lse, void* o_res, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Attention backward: what torch autograd derives for the SDPA call of
 * eager_lucid_attention_forward (modeling_lucid.py:505-549, causal, repeat_kv'd X),
 * with the grouped-query sums over the query heads of each kv head done in-kernel.
 * In : q, k, o, dout strided; x internal; lse and (optional, may be NULL) o_res from
 *      lucid_attn_fwd.
 * Out: dq strided bf16 [B,Hq,N,D];
 *      dk_f32 internal fp32 [B,Hkv,Npad,D]  (dL/dK through Q K^T)
 *      dx_f32 internal fp32 [B,Hkv,Npad,D]  (dL/dX)
 */
size_t lucid_attn_bwd_workspace_bytes(int B, int Hq, int Hkv, int N, int D);
/* Workspace of the stored-tile schedule: with at least this many bytes the column pass
 * also stores every bf16 dS^T tile (B*Hq*ceil(N/128)*(ceil(N/128)+1)/2 tiles of 32 KB,
 * plus B*Hq*ceil(N/128) tiles holding the bf16 residual of the diagonal blocks' dS^T)
 * and the row pass streams them instead of recomputing S and dP; same results. */
size_t lucid_attn_bwd_fast_workspace_bytes(int B, int Hq, int Hkv, int N, int D);
int lucid_attn_bwd(int B, int Hq, int Hkv, int N, int D, float scale,
                   const void* q, int64_t q_sb, int64_t q_sh, int64_t q_sn,
                   const void* k, int64_t k_sb, int64_t k_sh, int64_t k_sn,
                   const void* x,
                   const void* o, int64_t o_sb, int64_t o_sh, int64_t o_sn,
                   const void* dout, int64_t do_sb, int64_t do_sh, int64_t do_sn,
                   const float* lse, const void* o_res,
                   void* dq, int64_t dq_sb, int64_t dq_sh, int64_t dq_sn,
                   float* dk_f32, float* dx_f32,
                   void* workspace, size_t workspace_bytes, void* stream);

/*
 * Solve backward: dV = P^-T dX and dK through P and RMSNorm.
 * Replaces Lucid_Tril_Solver.backward (modeling_lucid.py:314-382) and the
 * autograd of the dense branch (modeling_lucid.py:566-570).
 * In : k strided (raw keys); x, khat, u, rstd, dinv from lucid_solve_fwd;
 *      dx_f32 internal fp32 [B,H,Npad,D]; dk_add optional internal fp32
 *      [B,H,Npad,D] added to dK (e.g. dk_f32 of lucid_attn_bwd), may be NULL.
 * Out: dk, dv strided bf16 [B,H,N,D].
 */
size_t lucid_solve_bwd_workspace_bytes(int B, int H, int N, int D);
/* Workspace of the stored-tile schedule: with at least this many bytes the transposed
 * solve also stores every bf16 dG^T tile (B*H*ceil(N/128)*(ceil(N/128)-1)/2 tiles of
 * 32 KB) and the row pass streams them instead of recomputing E and D; same results. */
size_t lucid_solve_bwd_fast_workspace_bytes(int B, int H, int N, int D);
int lucid_solve_bwd(int B, int H, int N, int D, float scale,
                    const void* k, int64_t k_sb, int64_t k_sh, int64_t k_sn,
                    const void* x, const void* khat, const void* u,
                    const float* rstd, const float* dinv,
                    const float* dx_f32, const float* dk_add,
                    void* dk, int64_t dk_sb, int64_t dk_sh, int64_t dk_sn,
                    void* dv, int64_t dv_sb, int64_t dv_sh, int64_t dv_sn,
                    void* workspace, size_t workspace_bytes, void* stream);

/*
 * LUCID-Path forward: O = (I + L)^-1 V with the Householder-path scores
 *   L = stril(exp(scale * A - 1/scale)),  A_rc = q_r^T (H_r ... H_{c+1}) k_c,
 *   H_t = I - beta_t w_t w_t^T.
 * Replaces parallel_lucid_path_attention / ParallelLUCIDPathAttentionFunction
 * .forward (lucid_path/triton_code/parallel.py:27-76, :180-241) together with
 * the kernels it launches: chunk_scaled_dot_kkt_fwd + solve_tril (:40-51),
 * triangular_solve_fwd_kernel (triangular_solve_fwd.py:14-225) and
 * mini_triangular_solve (mini_tril_solve.py:9-81).
 * Layout is the reference's BTHD: k, v, w are [B, T, H, D] and q, o are
 * [B, T, HQ, D], each given by element strides (sb, st, sh) with unit
 * innermost stride; beta is [B, T, H] (bf16, or fp32 when beta_fp32 != 0)
 * with strides (sb, st, sh).  q may be NULL, meaning q = k (then HQ == H).
 * The workspace (lucid_path_fwd_workspace_bytes) holds the state the
 * backward reads: keep it unchanged until lucid_path_bwd has run.
 * k_cache (may be NULL; [B, T, H, D] bf16 strided) receives the decode-time
 * keys of use_cache=True, k_cache_c = (H_{T-1} ... H_{c+1}) k_c
 * (prepare_k_cache.py:8-74).
 */
size_t lucid_path_fwd_workspace_bytes(int B, int T, int H, int HQ, int D);
int lucid_path_fwd(int B, int T, int H, int HQ, int D, float scale,
                   const void* q, int64_t q_sb, int64_t q_st, int64_t q_sh,
                   const void* k, int64_t k_sb, int64_t k_st, int64_t k_sh,
                   const void* v, int64_t v_sb, int64_t v_st, int64_t v_sh,
                   const void* w, int64_t w_sb, int64_t w_st, int64_t w_sh,
                   const void* beta, int beta_fp32, int64_t be_sb, int64_t be_st, int64_t be_sh,
                   void* o, int64_t o_sb, int64_t o_st, int64_t o_sh,
                   void* k_cache, int64_t kc_sb, int64_t kc_st, int64_t kc_sh,
                   void* workspace, size_t workspace_bytes, void* stream);

/*
 * LUCID-Path backward.  Replaces ParallelLUCIDPathAttentionFunction.backward
 * (parallel.py:78-177) and its kernels: triangular_solve_bwd_dv_kernel
 * (triangular_solve_bwd_dv_reuse.py:17-205), the prepare / cumprod / transform_q
 * / inter / intra / preprocess kernels and the GQA reduction (:165-171).
 * In : q, k, w, beta as for lucid_path_fwd (q NULL when the forward used q = k);
 *      dout [B, T, HQ, D]; fwd_workspace = the forward's workspace.
 * Out: dk, dv, dw [B, T, H, D] and dbeta [B, T, H] (bf16, fp32 when
 *      dbeta_fp32 != 0), dq [B, T, HQ, D] when q was given.  With q = k the
 *      query gradient is added into dk (the reference returns both and
 *      autograd sums them into k.grad).
 */
size_t lucid_path_bwd_workspace_bytes(int B, int T, int H, int HQ, int D);
int lucid_path_bwd(int B, int T, int H, int HQ, int D, float scale,
                   const void* q, int64_t q_sb, int64_t q_st, int64_t q_sh,
                   const void* k, int64_t k_sb, int64_t k_st, int64_t k_sh,
                   const void* w, int64_t w_sb, int64_t w_st, int64_t w_sh,
                   const void* beta, int beta_fp32, int64_t be_sb, int64_t be_st, int64_t be_sh,
                   const void* dout, int64_t do_sb, int64_t do_st, int64_t do_sh,
                   const void* fwd_workspace, size_t fwd_workspace_bytes,
                   void* dq, int64_t dq_sb, int64_t dq_st, int64_t dq_sh,
                   void* dk, int64_t dk_sb, int64_t dk_st, int64_t dk_sh,
                   void* dv, int64_t dv_sb, int64_t dv_st, int64_t dv_sh,
                   void* dw, int64_t dw_sb, int64_t dw_st, int64_t dw_sh,
                   void* dbeta, int dbeta_fp32, int64_t db_sb, int64_t db_st, int64_t db_sh,
                   void* workspace, size_t workspace_bytes, void* stream);

/*
 * PaTH softmax attention forward:
 *   o_r = sum_{c <= r} softmax_c(scale * A_rc) v_c,  A_rc = q_r^T (H_r ... H_{c+1}) k_c,
 *   lse_r = log2 sum_c exp2(scale * log2(e) * A_rc)   (log2 domain, as the reference's L).
 * Replaces the composition intra_chunk_preprocess_fwd_fn (intra_chunk_preprocess_fwd.py:124-168,
 * diagonal blocks) + parallel_path_fwd_fn (parallel_path_fwd.py:127-170, off-diagonal blocks
 * with online softmax), with the UT transform of parallel.py:40-51.  The reference has no
 * backward for this op.  Layout as lucid_path_fwd; lse is [B, T, HQ] fp32 with element
 * strides (sb, st, sh).
 */
size_t lucid_path_attn_fwd_workspace_bytes(int B, int T, int H, int HQ, int D);
int lucid_path_attn_fwd(int B, int T, int H, int HQ, int D, float scale,
                        const void* q, int64_t q_sb, int64_t q_st, int64_t q_sh,
                        const void* k, int64_t k_sb, int64_t k_st, int64_t k_sh,
                        const void* v, int64_t v_sb, int64_t v_st, int64_t v_sh,
                        const void* w, int64_t w_sb, int64_t w_st, int64_t w_sh,
                        const void* beta, int beta_fp32, int64_t be_sb, int64_t be_st, int64_t be_sh,
                        void* o, int64_t o_sb, int64_t o_st, int64_t o_sh,
                        float* lse, int64_t l_sb, int64_t l_st, int64_t l_sh,
                        void* workspace, size_t workspace_bytes, void* stream);

/*
 * Context-parallel building blocks (one process per GPU, each owning one or more
 * segments, i.e. contiguous row ranges, of the sequence; no counterpart in the
 * reference, which runs long sequences on one GPU).  They are block-range forms of
 * the prep and solve of get_v_prime (modeling_lucid.py:551-574; the blockwise
 * Lucid_Tril_Solver.forward, :285-312, runs the same recurrence over row blocks) and
 * of eager_lucid_attention_forward (:505-549).  Buffers are full-length ([B, H, N, D]
 * / internal [B, H, Npad, D]); a rank fills the rows it owns and the segments it
 * receives.
 *   lucid_cp_prep       prep of row blocks [blk_lo, blk_hi): khat_only = 1 computes
 *                       rstd and k^ only (received chunks), 0 also the diagonal
 *                       inverses (own chunk)
 *   lucid_cp_publish    mark row blocks [blk_lo, blk_hi) of BH (batch, head) rows of a
 *                       [BH][NB] flag array as solved (received chunks)
 *   lucid_cp_solve_fwd  the solve of row blocks [blk_lo, blk_hi) given every earlier
 *                       block published; flags / status are the caller's, zeroed
 *                       except for the published blocks
 *   lucid_cp_attn_fwd   the attention of query row blocks [blk_lo, blk_hi) over all
 *                       keys up to them
 * blk_lo must be even and blk_hi even or NB (whole pairs of 128-row blocks); the
 * kernels touch no row outside [0, 128 blk_hi) and write only rows of [blk_lo, blk_hi).
 * max_ctas caps the persistent grids (0 = one CTA per SM) so that NCCL kernels keep
 * SMs to run on.  The kernels never wait on anything another launch produces.
 */
int lucid_cp_prep(int B, int H, int N, int D, float scale, float eps, int blk_lo, int blk_hi, int khat_only,
                  const void* k, int64_t k_sb, int64_t k_sh, int64_t k_sn, void* khat, void* u, float* rstd,
                  float* dinv, void* stream);
int lucid_cp_publish(int* flags, int BH, int NB, int blk_lo, int blk_hi, void* stream);
int lucid_cp_solve_fwd(int B, int H, int N, int D, float scale, int blk_lo, int blk_hi, int max_ctas,
                       const void* v, int64_t v_sb, int64_t v_sh, int64_t v_sn, void* x,
                       const void* khat, const void* u, const float* dinv, int* flags, int* status, void* stream);
int lucid_cp_attn_fwd(int B, int Hq, int Hkv, int N, int D, float scale, int blk_lo, int blk_hi, int max_ctas,
                      const void* q, int64_t q_sb, int64_t q_sh, int64_t q_sn,
                      const void* k, int64_t k_sb, int64_t k_sh, int64_t k_sn, const void* x,
                      void* o, int64_t o_sb, int64_t o_sh, int64_t o_sn, float* lse, void* o_res, int* status,
                      void* stream);

/*
 * Context-parallel backward (same chunking; the backward of lucid_attn_fwd /
 * lucid_solve_fwd, replacing Lucid_Tril_Solver.backward, modeling_lucid.py:314-382,
 * and the autograd of eager_lucid_attention_forward, :505-549, for one chunk).
 * A rank computes every gradient of its own rows: the column passes cover its own
 * column blocks over all later rows (whose q, dO, lse, delta, k^ and dV it holds as
 * received), the row passes its own row blocks over all earlier columns.
 *   lucid_cp_delta      delta = rowsum(dO o O) of rows [row_lo, row_hi) into the
 *                       internal [B*Hq][Npad] fp32 layout (o / dout indexed by
 *                       global row; o_res, o's rounding residual from
 *                       lucid_cp_attn_fwd with o's strides, may be NULL)
 *   lucid_cp_attn_bwd   passes & 1: column pass of column blocks [blk_lo, blk_hi)
 *                       (dk_f32, dx_f32 internal fp32); passes & 2: row pass of
 *                       row blocks [blk_lo, blk_hi) (dq, indexed by global row)
 *   lucid_cp_solve_bwd  passes & 1: transposed solve of column blocks [blk_lo, blk_hi)
 *                       into dv_int (bf16 internal) and dk_col, publishing their flags;
 *                       every later block's flag must be set beforehand
 *                       (lucid_cp_publish after its dV arrived); passes & 2: row pass
 *                       of row blocks [blk_lo, blk_hi) into dk_row, then dK (= RMSNorm
 *                       backward of dk_col + dk_row + the diagonal term, + dk_add) and
 *                       dV of those rows (dk / dv indexed by global row)
 * Same block-range, max_ctas and no-cross-launch-wait rules as the forward blocks.
 */
int lucid_cp_delta(int B, int Hq, int N, int D, int row_lo, int row_hi, const void* o, int64_t o_sb, int64_t o_sh,
                   int64_t o_sn, const void* dout, int64_t do_sb, int64_t do_sh, int64_t do_sn,
                   const void* o_res, float* delta, void* stream);
int lucid_cp_attn_bwd(int B, int Hq, int Hkv, int N, int D, float scale, int blk_lo, int blk_hi, int max_ctas,
                      int passes, const void* q, int64_t q_sb, int64_t q_sh, int64_t q_sn,
                      const void* k, int64_t k_sb, int64_t k_sh, int64_t k_sn, const void* x,
                      const void* dout, int64_t do_sb, int64_t do_sh, int64_t do_sn, const float* lse,
                      const float* delta, void* dq, int64_t dq_sb, int64_t dq_sh, int64_t dq_sn,
                      float* dk_f32, float* dx_f32, int* status, void* stream);
int lucid_cp_solve_bwd(int B, int H, int N, int D, float scale, int blk_lo, int blk_hi, int max_ctas, int passes,
                       const void* k, int64_t k_sb, int64_t k_sh, int64_t k_sn, const void* x, const void* khat,
                       const void* u, const float* rstd, const float* dinv, const float* dx_f32,
                       const float* dk_add, void* dv_int, float* dk_col, float* dk_row, int* flags,
                       void* dk, int64_t dk_sb, int64_t dk_sh, int64_t dk_sn,
                       void* dv, int64_t dv_sb, int64_t dv_sh, int64_t dv_sn, int* status, void* stream);

/*
 * Kernel timing hook (benchmarks).  While enabled for one kernel family,
 * every launch of that family's main kernel is bracketed by a pair of CUDA
 * events recorded on the launch stream; lucid_profile_read waits for the
 * recorded events and returns the summed device time and the launch count.
 * lucid_profile_enable(0) disables recording.  Not thread-safe with
 * concurrent launches from several host threads.
 */
#define LUCID_KERNEL_PREP 1       /* row statistics + diagonal-block inverses */
#define LUCID_KERNEL_SOLVE_FWD 2  /* wavefront solve X = P^-1 V */
#define LUCID_KERNEL_ATTN_FWD 3   /* causal attention forward */
#define LUCID_KERNEL_ATTN_BWD 4       /* attention backward, column pass (dK, dX) */
#define LUCID_KERNEL_SOLVE_BWD 5      /* transposed-solve wavefront (dV, dK^ columns) */
#define LUCID_KERNEL_ATTN_BWD_ROW 6   /* attention backward, row pass (dQ) */
#define LUCID_KERNEL_SOLVE_BWD_ROW 7  /* solve backward, row pass (dK^ rows) */
#define LUCID_KERNEL_PATH_BLOCK 8     /* LUCID-Path per-block kernels (UT transform, diagonal blocks, their backward) */
#define LUCID_KERNEL_PATH_SCORES 9    /* LUCID-Path off-diagonal path scores */
#define LUCID_KERNEL_PATH_SOLVE 10    /* LUCID-Path wavefront solve O = (I + L)^-1 V */
#define LUCID_KERNEL_PATH_SOLVE_T 11  /* LUCID-Path transposed solve dV = (I + L)^-T dO */
#define LUCID_KERNEL_PATH_ROW 12      /* LUCID-Path backward row pass (dA, dQ~ chain) */
#define LUCID_KERNEL_PATH_COL 13      /* LUCID-Path backward column pass (dK_new, dW, dW2) */
#define LUCID_KERNEL_PATH_ATTN 14     /* PaTH softmax attention forward */
#define LUCID_KERNEL_DECODE 15        /* LUCID decode step (get_new_v_prime) */
#define LUCID_KERNEL_FWD_FUSED 16     /* chain-schedule solve + attention forward in one launch */
int lucid_profile_enable(int kernel);
int lucid_profile_read(float* total_ms, int* launches);

/*
 * Tensor-core self test: D = op(A) op(B) for one 128x128x128 bf16 tile,
 * A and B row-major [128][128] bf16, D row-major fp32 with room for one
 * extra int32 status word after the 128*128 results.  a_mn / b_mn select
 * the operand majorness (0: A is used as is / B^T; 1: A^T / B), i.e.
 *   (0,0) D = A B^T   (0,1) D = A B   (1,0) D = A^T B^T   (1,1) D = A^T B.
 * via_tma: 0 = operands written by threads, 1 = loaded with TMA,
 * 2 = as 1 but A is staged in tensor memory (the TS form of the MMA).
 */
int lucid_selftest_umma(const void* a, const void* b, float* d, int a_mn, int b_mn,
                        int via_tma, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LUCID_B200_H_ */
