// extern "C" entry points of liblucid_b200.so (declared in
// include/lucid_b200.h): argument checks, workspace carving, TMA descriptor
// creation and the launch sequence of each stage.
#include "lucid_b200.h"
#include "lucid_common.cuh"
#include "tmap.h"
#include "profile.h"

namespace lb {
cudaError_t launch_prep(const PrepArgs& a, cudaStream_t st);
cudaError_t launch_fwd(bool solve, const CUtensorMap& tA, const CUtensorMap& tB, const CUtensorMap& tC,
                       const CUtensorMap& tU, const FwdArgs& a, cudaStream_t st);
int solve_chain_ctas(int BH, int NB);
cudaError_t launch_fwd_fused(const CUtensorMap& tKhat, const CUtensorMap& tX, const CUtensorMap& tU,
                             const CUtensorMap& tQ, const CUtensorMap& tK, const FwdArgs& a, cudaStream_t st);
cudaError_t launch_bwd_col(bool solve, const CUtensorMap& tA1, const CUtensorMap& tA2, const CUtensorMap& tB1,
                           const CUtensorMap& tB2, const CUtensorMap& tU, const BwdArgs& a,
                           cudaStream_t st);
cudaError_t launch_bwd_row_stored(bool solve, const CUtensorMap& tB, const BwdArgs& a,
                                  cudaStream_t st);
cudaError_t launch_bwd_row(bool solve, const CUtensorMap& tA1, const CUtensorMap& tA2, const CUtensorMap& tB1,
                           const CUtensorMap& tB2, const BwdArgs& a, cudaStream_t st);
cudaError_t launch_delta(int B, int Hq, int N, int Npad, const bf16* o, long long o_sb, long long o_sh,
                         long long o_sn, const bf16* dout, long long d_sb, long long d_sh,
                         long long d_sn, const bf16* o_res, float* delta, cudaStream_t st, int row0 = 0,
                         int row1 = -1);
cudaError_t launch_solve_finalize(int B, int H, int N, int Npad, float s, const bf16* k, long long k_sb,
                                  long long k_sh, long long k_sn, const float* rstd, const float* dinv,
                                  const bf16* x, const bf16* dv_int, const float* dk_col,
                                  const float* dk_row, const float* dk_add, bf16* dk, long long dk_sb,
                                  long long dk_sh, long long dk_sn, bf16* dv, long long dv_sb,
                                  long long dv_sh, long long dv_sn, cudaStream_t st, int row0 = 0,
                                  int row1 = -1, int D = kHeadDim);
}  // namespace lb

using namespace lb;

#include <algorithm>
#include <mutex>
#include <vector>

namespace {

constexpr size_t kStatusRegion = 256;

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }
int npad_of(int N) { return ((N + 127) / 128) * 128; }
int nb_of(int N) { return (N + 127) / 128; }
// head dimension rounded up to the 16 columns of one MMA K-slice
int d16_of(int D) { return D >= kHeadDim ? kHeadDim : ((D + 15) / 16) * 16; }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool strides_ok(int64_t a, int64_t b, int64_t c) { return (a % 8 == 0) && (b % 8 == 0) && (c % 8 == 0); }

// D is the logical head dimension (1..128); rows always hold 128 elements, the
// columns from D on zero (a smaller head dimension is zero-padded by the caller).
bool shape_ok(int B, int Hq, int Hkv, int N, int D) {
  return B >= 0 && Hq >= 0 && Hkv >= 0 && N >= 0 && D >= 1 && D <= kHeadDim &&
         (Hkv == 0 || Hq % Hkv == 0) && (Hkv > 0 || Hq == 0) && N <= (1 << 30);
}
bool empty_problem(int B, int Hq, int Hkv, int N) { return B == 0 || Hq == 0 || Hkv == 0 || N == 0; }

int to_status(cudaError_t e) { return e == cudaSuccess ? LUCID_OK : LUCID_ERR_LAUNCH; }

// Internal contiguous [B][H][Npad][128] bf16 tensor map.
bool tmap_internal(CUtensorMap* m, const void* p, int B, int H, int Npad) {
  return make_tmap_bf16(m, p, kHeadDim, Npad, H, B, kHeadDim, (long long)Npad * kHeadDim,
                        (long long)H * Npad * kHeadDim);
}
// Caller's strided [B][H][N][128] bf16 tensor map.
bool tmap_strided(CUtensorMap* m, const void* p, int B, int H, int N, int64_t sb, int64_t sh, int64_t sn) {
  return make_tmap_bf16(m, p, kHeadDim, N, H, B, sn, sh, sb);
}

// The solve forward's chain-schedule workspace after the minimal one: chain flags, the
// W ring, the E tiles.
size_t chain_extra_bytes(int B, int H, int N) {
  const size_t bh = (size_t)B * H, nb = nb_of(N);
  return align256(bh * nb * sizeof(int)) + bh * kChainWRing * kBlock * kHeadDim * sizeof(float) +
         bh * nb * kChainLook * (size_t)kTileBytes;
}

}  // namespace

extern "C" {

int lucid_version(void) { return 100; }

int lucid_profile_enable(int kernel) {
  Profiler& p = profiler();
  std::lock_guard<std::mutex> g(p.mu);
  p.kernel = kernel;
  p.used = 0;
  return LUCID_OK;
}

int lucid_profile_read(float* total_ms, int* launches) {
  Profiler& p = profiler();
  std::lock_guard<std::mutex> g(p.mu);
  float tot = 0.f;
  for (int i = 0; i < p.used; ++i) {
    if (cudaEventSynchronize(p.ev[2 * i + 1]) != cudaSuccess) return LUCID_ERR_LAUNCH;
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, p.ev[2 * i], p.ev[2 * i + 1]) != cudaSuccess) return LUCID_ERR_LAUNCH;
    tot += ms;
  }
  if (total_ms) *total_ms = tot;
  if (launches) *launches = p.used;
  return LUCID_OK;
}
int lucid_padded_len(int N) { return npad_of(N); }
size_t lucid_workspace_status_offset(void) { return 0; }

// ---------------------------------------------------------------------------
// solve forward
// ---------------------------------------------------------------------------
size_t lucid_solve_fwd_workspace_bytes(int B, int H, int N, int D) {
  (void)D;
  return kStatusRegion + align256((size_t)B * H * nb_of(N) * sizeof(int));
}

size_t lucid_solve_fwd_fast_workspace_bytes(int B, int H, int N, int D) {
  const size_t base = lucid_solve_fwd_workspace_bytes(B, H, N, D);
  if (B <= 0 || H <= 0 || N <= 0 || solve_chain_ctas(B * H, nb_of(N)) == 0) return base;
  return base + chain_extra_bytes(B, H, N);
}

}  // extern "C"

namespace {
// The attention half of lucid_fused_fwd (q, o, lse, o_res of Hq query heads).
struct AttnPart {
  int Hq;
  const void* q;
  int64_t q_sb, q_sh, q_sn;
  void* o;
  int64_t o_sb, o_sh, o_sn;
  float* lse;
  void* o_res;
};

// lucid_solve_fwd, and with `at` the attention after it: fused into the chain
// schedule's launch when that schedule runs, else a second launch on the same
// status word.
int solve_fwd_impl(int B, int H, int N, int D, float scale, float eps, const void* k, int64_t k_sb, int64_t k_sh,
                   int64_t k_sn, const void* v, int64_t v_sb, int64_t v_sh, int64_t v_sn, void* x, void* khat,
                   void* u, float* rstd, float* dinv, void* workspace, size_t workspace_bytes, void* stream,
                   const AttnPart* at) {
  if (!aligned16(k) || !aligned16(v) || !aligned16(x) || !aligned16(khat) || !aligned16(u) ||
      !aligned16(rstd) || !aligned16(dinv) || !strides_ok(k_sb, k_sh, k_sn) ||
      !strides_ok(v_sb, v_sh, v_sn))
    return LUCID_ERR_ALIGN;
  if (!workspace || workspace_bytes < lucid_solve_fwd_workspace_bytes(B, H, N, D))
    return LUCID_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int NB = nb_of(N), Npad = npad_of(N);
  int* status = reinterpret_cast<int*>(workspace);
  int* flags = reinterpret_cast<int*>(static_cast<char*>(workspace) + kStatusRegion);
  // chain schedule when the model picks it and the (16-byte aligned) workspace holds its buffers
  const size_t base = lucid_solve_fwd_workspace_bytes(B, H, N, D);
  const int nchain = (workspace_bytes >= base + chain_extra_bytes(B, H, N) && aligned16(workspace))
                         ? solve_chain_ctas(B * H, NB) : 0;
  char* extra = static_cast<char*>(workspace) + base;
  const size_t cflag_bytes = align256((size_t)B * H * NB * sizeof(int));
  cudaError_t e = cudaMemsetAsync(workspace, 0, base + (nchain > 0 ? cflag_bytes : 0), st);
  if (e != cudaSuccess) return LUCID_ERR_LAUNCH;

  PrepArgs pa{};
  pa.B = B; pa.H = H; pa.N = N; pa.NB = NB; pa.Npad = Npad;
  pa.s = scale; pa.eps = eps; pa.D = D;
  pa.k = static_cast<const bf16*>(k); pa.k_sb = k_sb; pa.k_sh = k_sh; pa.k_sn = k_sn;
  pa.khat = static_cast<bf16*>(khat); pa.rstd = rstd; pa.dinv = dinv; pa.u = static_cast<bf16*>(u);
  {
    ProfileScope ps(LUCID_KERNEL_PREP, st);
    e = launch_prep(pa, st);
  }
  if (e != cudaSuccess) return LUCID_ERR_LAUNCH;

  CUtensorMap tK, tX, tU;
  if (!tmap_internal(&tK, khat, B, H, Npad) || !tmap_internal(&tX, x, B, H, Npad) ||
      !tmap_internal(&tU, u, B, H, Npad))
    return LUCID_ERR_TENSORMAP;
  FwdArgs fa{};
  fa.B = B; fa.Hq = H; fa.Hkv = H; fa.N = N; fa.NB = NB; fa.Npad = Npad;
  fa.scale = scale;
  fa.dinv = dinv;
  fa.v = static_cast<const bf16*>(v); fa.v_sb = v_sb; fa.v_sh = v_sh; fa.v_sn = v_sn;
  fa.x = static_cast<bf16*>(x);
  fa.flags = flags;
  fa.status = status;
  if (nchain > 0) {
    fa.nchain = nchain;
    fa.cflags = reinterpret_cast<int*>(extra);
    fa.wring = reinterpret_cast<float*>(extra + cflag_bytes);
    fa.etiles = reinterpret_cast<bf16*>(extra + cflag_bytes +
                                        (size_t)B * H * kChainWRing * kBlock * kHeadDim * sizeof(float));
  }
  if (!at) {
    ProfileScope ps(LUCID_KERNEL_SOLVE_FWD, st);
    return to_status(launch_fwd(true, tK, tK, tX, tU, fa, st));
  }
  CUtensorMap tQ, tKr;
  if (!tmap_strided(&tQ, at->q, B, at->Hq, N, at->q_sb, at->q_sh, at->q_sn) ||
      !tmap_strided(&tKr, k, B, H, N, k_sb, k_sh, k_sn))
    return LUCID_ERR_TENSORMAP;
  FwdArgs fb = fa;
  fb.Hq = at->Hq;
  fb.o = static_cast<bf16*>(at->o); fb.o_sb = at->o_sb; fb.o_sh = at->o_sh; fb.o_sn = at->o_sn;
  fb.lse = at->lse;
  fb.o_res = static_cast<bf16*>(at->o_res);
  fb.attn_d16 = d16_of(D);
  if (nchain > 0) {
    fb.attn_scale = scale;  // the layer uses one scale for both (modeling_lucid.py:204)
    ProfileScope ps(LUCID_KERNEL_FWD_FUSED, st);
    return to_status(launch_fwd_fused(tK, tX, tU, tQ, tKr, fb, st));
  }
  {
    ProfileScope ps(LUCID_KERNEL_SOLVE_FWD, st);
    e = launch_fwd(true, tK, tK, tX, tU, fa, st);
  }
  if (e != cudaSuccess) return LUCID_ERR_LAUNCH;
  FwdArgs fc{};
  fc.B = B; fc.Hq = at->Hq; fc.Hkv = H; fc.N = N; fc.NB = NB; fc.Npad = Npad;
  fc.scale = scale;
  fc.o = fb.o; fc.o_sb = fb.o_sb; fc.o_sh = fb.o_sh; fc.o_sn = fb.o_sn;
  fc.lse = fb.lse;
  fc.o_res = fb.o_res;
  fc.attn_d16 = fb.attn_d16;
  fc.status = status;
  ProfileScope ps(LUCID_KERNEL_ATTN_FWD, st);
  return to_status(launch_fwd(false, tQ, tKr, tX, tX, fc, st));
}
}  // namespace

extern "C" {

int lucid_solve_fwd(int B, int H, int N, int D, float scale, float eps, const void* k, int64_t k_sb,
                    int64_t k_sh, int64_t k_sn, const void* v, int64_t v_sb, int64_t v_sh, int64_t v_sn,
                    void* x, void* khat, void* u, float* rstd, float* dinv, void* workspace,
                    size_t workspace_bytes, void* stream) {
  if (!shape_ok(B, H, H, N, D)) return LUCID_ERR_SHAPE;
  if (empty_problem(B, H, H, N)) return LUCID_OK;
  return solve_fwd_impl(B, H, N, D, scale, eps, k, k_sb, k_sh, k_sn, v, v_sb, v_sh, v_sn, x, khat, u, rstd, dinv,
                        workspace, workspace_bytes, stream, nullptr);
}

size_t lucid_fused_fwd_workspace_bytes(int B, int Hq, int Hkv, int N, int D) {
  (void)Hq;
  return lucid_solve_fwd_fast_workspace_bytes(B, Hkv, N, D);
}

int lucid_fused_fwd(int B, int Hq, int Hkv, int N, int D, float scale, float eps, const void* q, int64_t q_sb,
                    int64_t q_sh, int64_t q_sn, const void* k, int64_t k_sb, int64_t k_sh, int64_t k_sn,
                    const void* v, int64_t v_sb, int64_t v_sh, int64_t v_sn, void* x, void* khat, void* u,
                    float* rstd, float* dinv, void* o, int64_t o_sb, int64_t o_sh, int64_t o_sn, float* lse,
                    void* o_res, void* workspace, size_t workspace_bytes, void* stream) {
  if (!shape_ok(B, Hq, Hkv, N, D)) return LUCID_ERR_SHAPE;
  if (empty_problem(B, Hq, Hkv, N)) return LUCID_OK;
  if (!aligned16(q) || !aligned16(o) || !aligned16(lse) || (o_res && !aligned16(o_res)) ||
      !strides_ok(q_sb, q_sh, q_sn) || !strides_ok(o_sb, o_sh, o_sn))
    return LUCID_ERR_ALIGN;
  const AttnPart at{Hq, q, q_sb, q_sh, q_sn, o, o_sb, o_sh, o_sn, lse, o_res};
  return solve_fwd_impl(B, Hkv, N, D, scale, eps, k, k_sb, k_sh, k_sn, v, v_sb, v_sh, v_sn, x, khat, u, rstd, dinv,
                        workspace, workspace_bytes, stream, &at);
}

// ---------------------------------------------------------------------------
// attention forward
// ---------------------------------------------------------------------------
size_t lucid_attn_fwd_workspace_bytes(int B, int Hq, int Hkv, int N, int D) {
  (void)B; (void)Hq; (void)Hkv; (void)N; (void)D;
  return kStatusRegion;
}

int lucid_attn_fwd(int B, int Hq, int Hkv, int N, int D, float scale, const void* q, int64_t q_sb,
                   int64_t q_sh, int64_t q_sn, const void* k, int64_t k_sb, int64_t k_sh, int64_t k_sn,
                   const void* x, void* o, int64_t o_sb, int64_t o_sh, int64_t o_sn, float* lse,
                   void* o_res, void* workspace, size_t workspace_bytes, void* stream) {
  if (!shape_ok(B, Hq, Hkv, N, D)) return LUCID_ERR_SHAPE;
  if (empty_problem(B, Hq, Hkv, N)) return LUCID_OK;
  if (!aligned16(q) || !aligned16(k) || !aligned16(x) || !aligned16(o) || !aligned16(lse) ||
      (o_res && !aligned16(o_res)) ||
      !strides_ok(q_sb, q_sh, q_sn) || !strides_ok(k_sb, k_sh, k_sn) || !strides_ok(o_sb, o_sh, o_sn))
    return LUCID_ERR_ALIGN;
  if (!workspace || workspace_bytes < lucid_attn_fwd_workspace_bytes(B, Hq, Hkv, N, D))
    return LUCID_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int NB = nb_of(N), Npad = npad_of(N);
  int* status = reinterpret_cast<int*>(workspace);
  if (cudaMemsetAsync(workspace, 0, kStatusRegion, st) != cudaSuccess) return LUCID_ERR_LAUNCH;
  CUtensorMap tQ, tK, tX;
  if (!tmap_strided(&tQ, q, B, Hq, N, q_sb, q_sh, q_sn) || !tmap_strided(&tK, k, B, Hkv, N, k_sb, k_sh, k_sn) ||
      !tmap_internal(&tX, x, B, Hkv, Npad))
    return LUCID_ERR_TENSORMAP;
  FwdArgs fa{};
  fa.B = B; fa.Hq = Hq; fa.Hkv = Hkv; fa.N = N; fa.NB = NB; fa.Npad = Npad;
  fa.scale = scale;
  fa.o = static_cast<bf16*>(o); fa.o_sb = o_sb; fa.o_sh = o_sh; fa.o_sn = o_sn;
  fa.lse = lse;
  fa.o_res = static_cast<bf16*>(o_res);
  fa.attn_d16 = d16_of(D);
  fa.status = status;
  ProfileScope ps(LUCID_KERNEL_ATTN_FWD, st);
  return to_status(launch_fwd(false, tQ, tK, tX, tX, fa, st));
}

// ---------------------------------------------------------------------------
// attention backward
// ---------------------------------------------------------------------------
size_t lucid_attn_bwd_workspace_bytes(int B, int Hq, int Hkv, int N, int D) {
  (void)Hkv; (void)D;
  const size_t rows = (size_t)B * Hq * npad_of(N);
  return kStatusRegion + align256(rows * sizeof(float));
}

// Stored-tile schedule: one bf16 dS^T tile per (batch, query head, key block i <= query block j),
// plus the bf16 residual (lo) tile of each diagonal block.
size_t lucid_attn_bwd_fast_workspace_bytes(int B, int Hq, int Hkv, int N, int D) {
  const size_t nb = (size_t)nb_of(N);
  return lucid_attn_bwd_workspace_bytes(B, Hq, Hkv, N, D) +
         align256((size_t)B * Hq * (nb * (nb + 1) / 2 + nb) * kTileBytes);
}

int lucid_attn_bwd(int B, int Hq, int Hkv, int N, int D, float scale, const void* q, int64_t q_sb,
                   int64_t q_sh, int64_t q_sn, const void* k, int64_t k_sb, int64_t k_sh, int64_t k_sn,
                   const void* x, const void* o, int64_t o_sb, int64_t o_sh, int64_t o_sn,
                   const void* dout, int64_t do_sb, int64_t do_sh, int64_t do_sn, const float* lse,
                   const void* o_res, void* dq, int64_t dq_sb, int64_t dq_sh, int64_t dq_sn, float* dk_f32,
                   float* dx_f32, void* workspace, size_t workspace_bytes, void* stream) {
  if (!shape_ok(B, Hq, Hkv, N, D)) return LUCID_ERR_SHAPE;
  if (empty_problem(B, Hq, Hkv, N)) return LUCID_OK;
  if (!aligned16(q) || !aligned16(k) || !aligned16(x) || !aligned16(o) || !aligned16(dout) ||
      (o_res && !aligned16(o_res)) ||
      !aligned16(lse) || !aligned16(dq) || !aligned16(dk_f32) || !aligned16(dx_f32) ||
      !strides_ok(q_sb, q_sh, q_sn) || !strides_ok(k_sb, k_sh, k_sn) || !strides_ok(o_sb, o_sh, o_sn) ||
      !strides_ok(do_sb, do_sh, do_sn) || !strides_ok(dq_sb, dq_sh, dq_sn))
    return LUCID_ERR_ALIGN;
  if (!workspace || workspace_bytes < lucid_attn_bwd_workspace_bytes(B, Hq, Hkv, N, D))
    return LUCID_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int NB = nb_of(N), Npad = npad_of(N);
  char* ws = static_cast<char*>(workspace);
  int* status = reinterpret_cast<int*>(ws);
  float* delta = reinterpret_cast<float*>(ws + kStatusRegion);
  if (cudaMemsetAsync(ws, 0, kStatusRegion, st) != cudaSuccess) return LUCID_ERR_LAUNCH;
  cudaError_t e = launch_delta(B, Hq, N, Npad, static_cast<const bf16*>(o), o_sb, o_sh, o_sn,
                               static_cast<const bf16*>(dout), do_sb, do_sh, do_sn,
                               static_cast<const bf16*>(o_res), delta, st);
  if (e != cudaSuccess) return LUCID_ERR_LAUNCH;
  CUtensorMap tK, tX, tQ, tDO;
  if (!tmap_strided(&tK, k, B, Hkv, N, k_sb, k_sh, k_sn) || !tmap_internal(&tX, x, B, Hkv, Npad) ||
      !tmap_strided(&tQ, q, B, Hq, N, q_sb, q_sh, q_sn) ||
      !tmap_strided(&tDO, dout, B, Hq, N, do_sb, do_sh, do_sn))
    return LUCID_ERR_TENSORMAP;
  // a workspace large enough for the dS^T tiles selects the stored-tile schedule
  const size_t ntile = (size_t)NB * (NB + 1) / 2 + NB;   // pair tiles + diagonal residual tiles
  const bool stored = workspace_bytes >= lucid_attn_bwd_fast_workspace_bytes(B, Hq, Hkv, N, D) &&
                      ntile * 128 < (size_t)1 << 31;
  bf16* tiles = stored ? reinterpret_cast<bf16*>(ws + lucid_attn_bwd_workspace_bytes(B, Hq, Hkv, N, D)) : nullptr;
  BwdArgs ba{};
  ba.B = B; ba.Hq = Hq; ba.Hkv = Hkv; ba.N = N; ba.NB = NB; ba.Npad = Npad;
  ba.scale = scale;
  ba.lse = lse; ba.delta = delta;
  ba.dx = dx_f32; ba.dk_col = dk_f32;
  ba.dq = static_cast<bf16*>(dq); ba.dq_sb = dq_sb; ba.dq_sh = dq_sh; ba.dq_sn = dq_sn;
  ba.status = status;
  ba.store_tiles = stored ? 1 : 0;
  ba.tiles = tiles;
  {
    ProfileScope ps(LUCID_KERNEL_ATTN_BWD, st);
    e = launch_bwd_col(false, tK, tX, tQ, tDO, tX, ba, st);
  }
  if (e != cudaSuccess) return LUCID_ERR_LAUNCH;
  ProfileScope ps(LUCID_KERNEL_ATTN_BWD_ROW, st);
  if (stored) return to_status(launch_bwd_row_stored(false, tK, ba, st));
  return to_status(launch_bwd_row(false, tQ, tDO, tK, tX, ba, st));
}

// ---------------------------------------------------------------------------
// solve backward
// ---------------------------------------------------------------------------
size_t lucid_solve_bwd_workspace_bytes(int B, int H, int N, int D) {
  (void)D;
  const size_t rows = (size_t)B * H * npad_of(N);
  return kStatusRegion + align256((size_t)B * H * nb_of(N) * sizeof(int)) +
         align256(rows * kHeadDim * sizeof(bf16)) + 2 * align256(rows * kHeadDim * sizeof(float));
}

// Stored-tile schedule: one bf16 dG^T tile per (batch, head, column block i < row block j).
size_t lucid_solve_bwd_fast_workspace_bytes(int B, int H, int N, int D) {
  const size_t nb = (size_t)nb_of(N);
  return lucid_solve_bwd_workspace_bytes(B, H, N, D) + align256((size_t)B * H * (nb * (nb - 1) / 2) * kTileBytes);
}

int lucid_solve_bwd(int B, int H, int N, int D, float scale, const void* k, int64_t k_sb, int64_t k_sh,
                    int64_t k_sn, const void* x, const void* khat, const void* u, const float* rstd,
                    const float* dinv, const float* dx_f32, const float* dk_add, void* dk, int64_t dk_sb,
                    int64_t dk_sh, int64_t dk_sn, void* dv, int64_t dv_sb, int64_t dv_sh, int64_t dv_sn,
                    void* workspace, size_t workspace_bytes, void* stream) {
  if (!shape_ok(B, H, H, N, D)) return LUCID_ERR_SHAPE;
  if (empty_problem(B, H, H, N)) return LUCID_OK;
  if (!aligned16(k) || !aligned16(x) || !aligned16(khat) || !aligned16(u) || !aligned16(rstd) ||
      !aligned16(dinv) || !aligned16(dx_f32) || (dk_add && !aligned16(dk_add)) || !aligned16(dk) ||
      !aligned16(dv) || !strides_ok(k_sb, k_sh, k_sn) || !strides_ok(dk_sb, dk_sh, dk_sn) ||
      !strides_ok(dv_sb, dv_sh, dv_sn))
    return LUCID_ERR_ALIGN;
  if (!workspace || workspace_bytes < lucid_solve_bwd_workspace_bytes(B, H, N, D))
    return LUCID_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int NB = nb_of(N), Npad = npad_of(N);
  const size_t rows = (size_t)B * H * Npad;
  char* ws = static_cast<char*>(workspace);
  int* status = reinterpret_cast<int*>(ws);
  size_t off = kStatusRegion;
  int* flags = reinterpret_cast<int*>(ws + off);
  off += align256((size_t)B * H * NB * sizeof(int));
  bf16* dv_int = reinterpret_cast<bf16*>(ws + off);
  off += align256(rows * kHeadDim * sizeof(bf16));
  float* dk_col = reinterpret_cast<float*>(ws + off);
  off += align256(rows * kHeadDim * sizeof(float));
  float* dk_row = reinterpret_cast<float*>(ws + off);
  // status word and the dependency flags start at zero
  if (cudaMemsetAsync(ws, 0, kStatusRegion + align256((size_t)B * H * NB * sizeof(int)), st) != cudaSuccess)
    return LUCID_ERR_LAUNCH;
  CUtensorMap tK, tX, tDV, tU;
  if (!tmap_internal(&tK, khat, B, H, Npad) || !tmap_internal(&tX, x, B, H, Npad) ||
      !tmap_internal(&tDV, dv_int, B, H, Npad) || !tmap_internal(&tU, u, B, H, Npad))
    return LUCID_ERR_TENSORMAP;
  // a workspace large enough for the dG^T tiles selects the stored-tile schedule
  const size_t npair = (size_t)NB * (NB - 1) / 2;
  const bool stored = npair > 0 && workspace_bytes >= lucid_solve_bwd_fast_workspace_bytes(B, H, N, D) &&
                      npair * 128 < (size_t)1 << 31;
  BwdArgs ba{};
  ba.B = B; ba.Hq = H; ba.Hkv = H; ba.N = N; ba.NB = NB; ba.Npad = Npad;
  ba.scale = scale;
  ba.dk_col = dk_col; ba.dk_row = dk_row;
  ba.dinv = dinv; ba.dx_in = dx_f32; ba.dv = dv_int;
  ba.flags = flags;
  ba.status = status;
  ba.store_tiles = stored ? 1 : 0;
  ba.tiles = stored ? reinterpret_cast<bf16*>(ws + lucid_solve_bwd_workspace_bytes(B, H, N, D)) : nullptr;
  cudaError_t e;
  {
    ProfileScope ps(LUCID_KERNEL_SOLVE_BWD, st);
    e = launch_bwd_col(true, tK, tX, tK, tDV, tU, ba, st);
  }
  if (e != cudaSuccess) return LUCID_ERR_LAUNCH;
  {
    ProfileScope ps(LUCID_KERNEL_SOLVE_BWD_ROW, st);
    e = stored ? launch_bwd_row_stored(true, tK, ba, st) : launch_bwd_row(true, tK, tDV, tK, tX, ba, st);
  }
  if (e != cudaSuccess) return LUCID_ERR_LAUNCH;
  return to_status(launch_solve_finalize(
      B, H, N, Npad, scale, static_cast<const bf16*>(k), k_sb, k_sh, k_sn, rstd, dinv,
      static_cast<const bf16*>(x), dv_int, dk_col, dk_row, dk_add, static_cast<bf16*>(dk), dk_sb, dk_sh,
      dk_sn, static_cast<bf16*>(dv), dv_sb, dv_sh, dv_sn, st, 0, -1, D));
}

}  // extern "C"

// ---------------------------------------------------------------------------
// solve forward without a workspace (static scratch)
// ---------------------------------------------------------------------------
// Scratch of lucid_solve_fwd_noalloc: status word region + dependency flags.
// Host code must not pass this symbol to a kernel (on the host it names a
// host-side stand-in); its device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[LUCID_NOALLOC_SCRATCH_BYTES];

namespace {
// Device address of g_noalloc_scratch for the current device, looked up once
// per device.  Returns nullptr if the lookup fails.
void* noalloc_scratch_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  static std::mutex mu;
  static void* ptrs[64] = {};
  std::lock_guard<std::mutex> g(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return nullptr;
    ptrs[dev] = p;
  }
  return ptrs[dev];
}
}  // namespace

// ---------------------------------------------------------------------------
// context-parallel building blocks
// ---------------------------------------------------------------------------
namespace {
__global__ void fill_flags_kernel(int* flags, int NB, int lo, int hi) {
  const int bh = blockIdx.x;
  for (int b = lo + threadIdx.x; b < hi; b += blockDim.x) flags[(long long)bh * NB + b] = 1;
}
}  // namespace

extern "C" int lucid_cp_publish(int* flags, int BH, int NB, int blk_lo, int blk_hi, void* stream) {
  if (BH < 0 || NB < 0 || blk_lo < 0 || blk_hi > NB || blk_lo > blk_hi) return LUCID_ERR_SHAPE;
  if (BH == 0 || blk_lo == blk_hi) return LUCID_OK;
  fill_flags_kernel<<<BH, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(flags, NB, blk_lo, blk_hi);
  return to_status(cudaGetLastError());
}

extern "C" int lucid_cp_prep(int B, int H, int N, int D, float scale, float eps, int blk_lo, int blk_hi,
                             int khat_only, const void* k, int64_t k_sb, int64_t k_sh, int64_t k_sn, void* khat,
                             void* u, float* rstd, float* dinv, void* stream) {
  if (!shape_ok(B, H, H, N, D)) return LUCID_ERR_SHAPE;
  const int NB = nb_of(N);
  if (blk_lo < 0 || blk_hi > NB || blk_lo > blk_hi) return LUCID_ERR_SHAPE;
  if (empty_problem(B, H, H, N) || blk_lo == blk_hi) return LUCID_OK;
  if (!aligned16(k) || !aligned16(khat) || !aligned16(u) || !aligned16(rstd) || !aligned16(dinv) ||
      !strides_ok(k_sb, k_sh, k_sn))
    return LUCID_ERR_ALIGN;
  PrepArgs pa{};
  pa.B = B; pa.H = H; pa.N = N; pa.NB = NB; pa.Npad = npad_of(N);
  pa.s = scale; pa.eps = eps; pa.D = D;
  pa.k = static_cast<const bf16*>(k); pa.k_sb = k_sb; pa.k_sh = k_sh; pa.k_sn = k_sn;
  pa.khat = static_cast<bf16*>(khat); pa.rstd = rstd; pa.dinv = dinv; pa.u = static_cast<bf16*>(u);
  pa.blk0 = blk_lo; pa.blk1 = blk_hi; pa.khat_only = khat_only;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  ProfileScope ps(LUCID_KERNEL_PREP, st);
  return to_status(launch_prep(pa, st));
}

// Row blocks [blk_lo, blk_hi) with blk_lo even and blk_hi even or NB: whole pairs.
bool cp_range_ok(int N, int blk_lo, int blk_hi) {
  const int NB = nb_of(N);
  return blk_lo >= 0 && !(blk_lo & 1) && blk_hi <= NB && blk_lo < blk_hi && (!(blk_hi & 1) || blk_hi == NB);
}

extern "C" int lucid_cp_solve_fwd(int B, int H, int N, int D, float scale, int blk_lo, int blk_hi, int max_ctas,
                                  const void* v, int64_t v_sb, int64_t v_sh, int64_t v_sn, void* x,
                                  const void* khat, const void* u, const float* dinv, int* flags, int* status,
                                  void* stream) {
  if (!shape_ok(B, H, H, N, D) || !cp_range_ok(N, blk_lo, blk_hi)) return LUCID_ERR_SHAPE;
  if (empty_problem(B, H, H, N)) return LUCID_OK;
  if (!aligned16(x) || !aligned16(khat) || !aligned16(u) || !aligned16(dinv) || !strides_ok(v_sb, v_sh, v_sn) ||
      flags == nullptr || status == nullptr)
    return LUCID_ERR_ALIGN;
  const int NB = nb_of(N), Npad = npad_of(N);
  CUtensorMap tK, tX, tU;
  if (!tmap_internal(&tK, khat, B, H, Npad) || !tmap_internal(&tX, x, B, H, Npad) ||
      !tmap_internal(&tU, u, B, H, Npad))
    return LUCID_ERR_TENSORMAP;
  FwdArgs fa{};
  fa.B = B; fa.Hq = H; fa.Hkv = H; fa.N = N; fa.NB = NB; fa.Npad = Npad;
  fa.scale = scale;
  fa.dinv = dinv;
  fa.v = static_cast<const bf16*>(v); fa.v_sb = v_sb; fa.v_sh = v_sh; fa.v_sn = v_sn;
  fa.x = static_cast<bf16*>(x);
  fa.flags = flags;
  fa.status = status;
  fa.pp0 = blk_lo / 2;
  fa.pp1 = (blk_hi + 1) / 2;
  fa.max_ctas = max_ctas;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  ProfileScope ps(LUCID_KERNEL_SOLVE_FWD, st);
  return to_status(launch_fwd(true, tK, tK, tX, tU, fa, st));
}

extern "C" int lucid_cp_attn_fwd(int B, int Hq, int Hkv, int N, int D, float scale, int blk_lo, int blk_hi,
                                 int max_ctas,
                                 const void* q, int64_t q_sb, int64_t q_sh, int64_t q_sn, const void* k,
                                 int64_t k_sb, int64_t k_sh, int64_t k_sn, const void* x, void* o, int64_t o_sb,
                                 int64_t o_sh, int64_t o_sn, float* lse, void* o_res, int* status, void* stream) {
  if (!shape_ok(B, Hq, Hkv, N, D) || !cp_range_ok(N, blk_lo, blk_hi)) return LUCID_ERR_SHAPE;
  if (empty_problem(B, Hq, Hkv, N)) return LUCID_OK;
  if (!aligned16(q) || !aligned16(k) || !aligned16(x) || !aligned16(lse) || (o_res && !aligned16(o_res)) ||
      !strides_ok(q_sb, q_sh, q_sn) ||
      !strides_ok(k_sb, k_sh, k_sn) || !strides_ok(o_sb, o_sh, o_sn) || status == nullptr)
    return LUCID_ERR_ALIGN;
  const int NB = nb_of(N), Npad = npad_of(N);
  CUtensorMap tQ, tK, tX;
  if (!tmap_strided(&tQ, q, B, Hq, N, q_sb, q_sh, q_sn) || !tmap_strided(&tK, k, B, Hkv, N, k_sb, k_sh, k_sn) ||
      !tmap_internal(&tX, x, B, Hkv, Npad))
    return LUCID_ERR_TENSORMAP;
  FwdArgs fa{};
  fa.B = B; fa.Hq = Hq; fa.Hkv = Hkv; fa.N = N; fa.NB = NB; fa.Npad = Npad;
  fa.scale = scale;
  fa.o = static_cast<bf16*>(o); fa.o_sb = o_sb; fa.o_sh = o_sh; fa.o_sn = o_sn;
  fa.lse = lse;
  fa.o_res = static_cast<bf16*>(o_res);
  fa.attn_d16 = d16_of(D);
  fa.status = status;
  fa.pp0 = blk_lo / 2;
  fa.pp1 = (blk_hi + 1) / 2;
  fa.max_ctas = max_ctas;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  ProfileScope ps(LUCID_KERNEL_ATTN_FWD, st);
  return to_status(launch_fwd(false, tQ, tK, tX, tX, fa, st));
}

extern "C" int lucid_cp_delta(int B, int Hq, int N, int D, int row_lo, int row_hi, const void* o, int64_t o_sb,
                              int64_t o_sh, int64_t o_sn, const void* dout, int64_t do_sb, int64_t do_sh,
                              int64_t do_sn, const void* o_res, float* delta, void* stream) {
  if (!shape_ok(B, Hq, Hq, N, D) || row_lo < 0 || row_hi > N || row_lo > row_hi) return LUCID_ERR_SHAPE;
  if (empty_problem(B, Hq, Hq, N) || row_lo == row_hi) return LUCID_OK;
  if (!aligned16(delta) || !strides_ok(o_sb, o_sh, o_sn) || !strides_ok(do_sb, do_sh, do_sn)) return LUCID_ERR_ALIGN;
  return to_status(launch_delta(B, Hq, N, npad_of(N), static_cast<const bf16*>(o), o_sb, o_sh, o_sn,
                                static_cast<const bf16*>(dout), do_sb, do_sh, do_sn,
                                static_cast<const bf16*>(o_res), delta, reinterpret_cast<cudaStream_t>(stream),
                                row_lo, row_hi));
}

extern "C" int lucid_cp_attn_bwd(int B, int Hq, int Hkv, int N, int D, float scale, int blk_lo, int blk_hi,
                                 int max_ctas, int passes, const void* q, int64_t q_sb, int64_t q_sh, int64_t q_sn,
                                 const void* k, int64_t k_sb, int64_t k_sh, int64_t k_sn, const void* x,
                                 const void* dout, int64_t do_sb, int64_t do_sh, int64_t do_sn, const float* lse,
                                 const float* delta, void* dq, int64_t dq_sb, int64_t dq_sh, int64_t dq_sn,
                                 float* dk_f32, float* dx_f32, int* status, void* stream) {
  if (!shape_ok(B, Hq, Hkv, N, D) || !cp_range_ok(N, blk_lo, blk_hi) || passes < 1 || passes > 3)
    return LUCID_ERR_SHAPE;
  if (empty_problem(B, Hq, Hkv, N)) return LUCID_OK;
  if (!aligned16(q) || !aligned16(k) || !aligned16(x) || !aligned16(dout) || !aligned16(lse) ||
      !aligned16(delta) || !aligned16(dk_f32) || !aligned16(dx_f32) || !strides_ok(q_sb, q_sh, q_sn) ||
      !strides_ok(k_sb, k_sh, k_sn) || !strides_ok(do_sb, do_sh, do_sn) || !strides_ok(dq_sb, dq_sh, dq_sn) ||
      status == nullptr)
    return LUCID_ERR_ALIGN;
  const int NB = nb_of(N), Npad = npad_of(N);
  CUtensorMap tK, tX, tQ, tDO;
  if (!tmap_strided(&tK, k, B, Hkv, N, k_sb, k_sh, k_sn) || !tmap_internal(&tX, x, B, Hkv, Npad) ||
      !tmap_strided(&tQ, q, B, Hq, N, q_sb, q_sh, q_sn) ||
      !tmap_strided(&tDO, dout, B, Hq, N, do_sb, do_sh, do_sn))
    return LUCID_ERR_TENSORMAP;
  BwdArgs ba{};
  ba.B = B; ba.Hq = Hq; ba.Hkv = Hkv; ba.N = N; ba.NB = NB; ba.Npad = Npad;
  ba.scale = scale;
  ba.lse = lse; ba.delta = delta;
  ba.dx = dx_f32; ba.dk_col = dk_f32;
  ba.dq = static_cast<bf16*>(dq); ba.dq_sb = dq_sb; ba.dq_sh = dq_sh; ba.dq_sn = dq_sn;
  ba.status = status;
  ba.blk0 = blk_lo; ba.blk1 = blk_hi; ba.max_ctas = max_ctas;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (passes & 1) {
    ProfileScope ps(LUCID_KERNEL_ATTN_BWD, st);
    if (launch_bwd_col(false, tK, tX, tQ, tDO, tX, ba, st) != cudaSuccess) return LUCID_ERR_LAUNCH;
  }
  if (passes & 2) {
    ProfileScope ps(LUCID_KERNEL_ATTN_BWD_ROW, st);
    if (launch_bwd_row(false, tQ, tDO, tK, tX, ba, st) != cudaSuccess) return LUCID_ERR_LAUNCH;
  }
  return LUCID_OK;
}

extern "C" int lucid_cp_solve_bwd(int B, int H, int N, int D, float scale, int blk_lo, int blk_hi, int max_ctas,
                                  int passes, const void* k, int64_t k_sb, int64_t k_sh, int64_t k_sn,
                                  const void* x, const void* khat, const void* u, const float* rstd,
                                  const float* dinv, const float* dx_f32, const float* dk_add, void* dv_int,
                                  float* dk_col, float* dk_row, int* flags, void* dk, int64_t dk_sb,
                                  int64_t dk_sh, int64_t dk_sn, void* dv, int64_t dv_sb, int64_t dv_sh,
                                  int64_t dv_sn, int* status, void* stream) {
  if (!shape_ok(B, H, H, N, D) || !cp_range_ok(N, blk_lo, blk_hi) || passes < 1 || passes > 3)
    return LUCID_ERR_SHAPE;
  if (empty_problem(B, H, H, N)) return LUCID_OK;
  if (!aligned16(x) || !aligned16(khat) || !aligned16(u) || !aligned16(rstd) || !aligned16(dinv) ||
      !aligned16(dx_f32) || (dk_add && !aligned16(dk_add)) || !aligned16(dv_int) || !aligned16(dk_col) ||
      !aligned16(dk_row) || !strides_ok(k_sb, k_sh, k_sn) || !strides_ok(dk_sb, dk_sh, dk_sn) ||
      !strides_ok(dv_sb, dv_sh, dv_sn) || flags == nullptr || status == nullptr)
    return LUCID_ERR_ALIGN;
  const int NB = nb_of(N), Npad = npad_of(N);
  CUtensorMap tK, tX, tDV, tU;
  if (!tmap_internal(&tK, khat, B, H, Npad) || !tmap_internal(&tX, x, B, H, Npad) ||
      !tmap_internal(&tDV, dv_int, B, H, Npad) || !tmap_internal(&tU, u, B, H, Npad))
    return LUCID_ERR_TENSORMAP;
  BwdArgs ba{};
  ba.B = B; ba.Hq = H; ba.Hkv = H; ba.N = N; ba.NB = NB; ba.Npad = Npad;
  ba.scale = scale;
  ba.dk_col = dk_col; ba.dk_row = dk_row;
  ba.dinv = dinv; ba.dx_in = dx_f32; ba.dv = static_cast<bf16*>(dv_int);
  ba.flags = flags;
  ba.status = status;
  ba.blk0 = blk_lo; ba.blk1 = blk_hi; ba.max_ctas = max_ctas;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (passes & 1) {
    ProfileScope ps(LUCID_KERNEL_SOLVE_BWD, st);
    if (launch_bwd_col(true, tK, tX, tK, tDV, tU, ba, st) != cudaSuccess) return LUCID_ERR_LAUNCH;
  }
  if (passes & 2) {
    {
      ProfileScope ps(LUCID_KERNEL_SOLVE_BWD_ROW, st);
      if (launch_bwd_row(true, tK, tDV, tK, tX, ba, st) != cudaSuccess) return LUCID_ERR_LAUNCH;
    }
    const int row_hi = std::min(N, blk_hi * 128);
    return to_status(launch_solve_finalize(
        B, H, N, Npad, scale, static_cast<const bf16*>(k), k_sb, k_sh, k_sn, rstd, dinv,
        static_cast<const bf16*>(x), static_cast<const bf16*>(dv_int), dk_col, dk_row, dk_add,
        static_cast<bf16*>(dk), dk_sb, dk_sh, dk_sn, static_cast<bf16*>(dv), dv_sb, dv_sh, dv_sn, st,
        blk_lo * 128, row_hi, D));
  }
  return LUCID_OK;
}

extern "C" int lucid_solve_fwd_noalloc(int B, int H, int N, int D, float scale, float eps, const void* k,
                                       int64_t k_sb, int64_t k_sh, int64_t k_sn, const void* v, int64_t v_sb,
                                       int64_t v_sh, int64_t v_sn, void* x, void* khat, void* u, float* rstd,
                                       float* dinv, void* stream) {
  if (!shape_ok(B, H, H, N, D)) return LUCID_ERR_SHAPE;
  if (empty_problem(B, H, H, N)) return LUCID_OK;
  if ((long long)B * H * nb_of(N) > LUCID_NOALLOC_MAX_BLOCKS) return LUCID_ERR_TOO_LARGE;
  void* ws = noalloc_scratch_ptr();
  if (!ws) return LUCID_ERR_LAUNCH;
  // lucid_solve_fwd clears the status word and the flags before its launches
  return lucid_solve_fwd(B, H, N, D, scale, eps, k, k_sb, k_sh, k_sn, v, v_sb, v_sh, v_sn, x, khat, u, rstd,
                         dinv, ws, LUCID_NOALLOC_SCRATCH_BYTES, stream);
}

extern "C" int lucid_solve_fwd_noalloc_status(int* status, void* stream) {
  if (!status) return LUCID_ERR_SHAPE;
  void* ws = noalloc_scratch_ptr();
  if (!ws) return LUCID_ERR_LAUNCH;
  // the status word sits at lucid_workspace_status_offset() of the scratch, as in every workspace
  const char* word = static_cast<const char*>(ws) + lucid_workspace_status_offset();
  return to_status(cudaMemcpyAsync(status, word, sizeof(int), cudaMemcpyDeviceToHost,
                                   reinterpret_cast<cudaStream_t>(stream)));
}

// ---------------------------------------------------------------------------
// tensor-core self test
// ---------------------------------------------------------------------------
namespace lb {

__global__ void __launch_bounds__(128, 1)
    umma_selftest_kernel(const __grid_constant__ CUtensorMap tA, const __grid_constant__ CUtensorMap tB,
                         const bf16* a, const bf16* b, float* d, int a_mn, int b_mn, int via_tma,
                         int* status) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (sbase - raw);
  const uint32_t sA = sbase, sB = sbase + 32768;
  const uint32_t bar_tma = sbase + 65536, bar_mma = bar_tma + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 65536 + 16);
  volatile int* abort_cta = reinterpret_cast<volatile int*>(smem + 65536 + 20);
  const Abort ab{abort_cta, status};
  const int r = threadIdx.x, warp = r >> 5;
  if (r == 0) {
    mbar_init(bar_tma, 1);
    mbar_init(bar_mma, 1);
    *abort_cta = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;
  if (via_tma == 1 || via_tma == 2) {
    if (r == 0) {
      mbar_arrive_expect_tx(bar_tma, 65536);
      tma_load_tile(sA, &tA, bar_tma, 0, 0, 0);
      tma_load_tile(sB, &tB, bar_tma, 0, 0, 0);
    }
    ok = mbar_wait(bar_tma, 0, ab);
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float va[32], vb[32];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        ld_bf16x8(a + r * 128 + q * 32 + c * 8, va + c * 8);
        ld_bf16x8(b + r * 128 + q * 32 + c * 8, vb + c * 8);
      }
      tile_store_row32(sA, r, q, va);
      tile_store_row32(sB, r, q, vb);
    }
    fence_proxy_async_smem();
  }
  // mode 2: A goes to TMEM columns [128, 256) in the split-half packed
  // layout (row elements [64h, 64h+64) packed into columns 128 + 64h + [0, 32))
  if (via_tma == 2) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        float va[32];
#pragma unroll
        for (int c = 0; c < 4; ++c) ld_bf16x8(a + r * 128 + h * 64 + q * 32 + c * 8, va + c * 8);
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) pk[e] = pack_bf16(va[2 * e], va[2 * e + 1]);
        tmem_st16(tmem + ((uint32_t)(warp * 32) << 16) + 128u + 64u * h + 16u * q, pk);
      }
    }
    tmem_st_wait();
    tc_fence_before();
  }
  __syncthreads();
  if (r == 0 && ok) {
    tc_fence_after();
    if (via_tma == 2) {
      umma_tile_ts(tmem, [&](int kk) { return tmem + 128u + 64u * (kk >> 2) + 8u * (kk & 3); }, sB,
                   b_mn != 0, 0u);
    } else {
      umma_tile(tmem, sA, a_mn != 0, sB, b_mn != 0, 0u);
    }
    umma_commit(bar_mma);
  }
  ok = ok && mbar_wait(bar_mma, 0, ab);
  ok = __all_sync(0xffffffffu, ok);
  if (ok) {
    tc_fence_after();
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float v[32];
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + 32u * q, v);
      tmem_ld_wait();
#pragma unroll
      for (int e = 0; e < 32; ++e) d[r * 128 + q * 32 + e] = v[e];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace lb

extern "C" int lucid_selftest_umma(const void* a, const void* b, float* d, int a_mn, int b_mn, int via_tma,
                                   void* stream) {
  if (!aligned16(a) || !aligned16(b) || !aligned16(d)) return LUCID_ERR_ALIGN;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  CUtensorMap tA, tB;
  if (!make_tmap_bf16(&tA, a, 128, 128, 1, 1, 128, 128 * 128, 128 * 128) ||
      !make_tmap_bf16(&tB, b, 128, 128, 1, 1, 128, 128 * 128, 128 * 128))
    return LUCID_ERR_TENSORMAP;
  // status word lives right after D (caller allocates 128*128 + 4 floats)
  int* status = reinterpret_cast<int*>(d + 128 * 128);
  const int smem = 65536 + 64 + 1024;
  if (cudaFuncSetAttribute(umma_selftest_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
      cudaSuccess)
    return LUCID_ERR_LAUNCH;
  umma_selftest_kernel<<<1, 128, smem, st>>>(tA, tB, static_cast<const bf16*>(a), static_cast<const bf16*>(b),
                                             d, a_mn, b_mn, via_tma, status);
  return cudaGetLastError() == cudaSuccess ? LUCID_OK : LUCID_ERR_LAUNCH;
}
