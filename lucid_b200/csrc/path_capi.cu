// extern "C" entry points of LUCID-Path (declared in include/lucid_b200.h):
// argument checks, workspace carving, tensor maps and the launch sequence of
// the forward (parallel.py:27-76) and backward (parallel.py:78-177).
#include "lucid_b200.h"
#include "path_common.cuh"
#include "profile.h"
#include "tmap.h"

namespace lb {
cudaError_t launch_path_bgemm(const BGemmArgs& a, cudaStream_t st);
cudaError_t launch_path_triinv(const TriInvArgs& a, cudaStream_t st);
cudaError_t launch_path_eye(float* out, long long heads, long long head_stride, cudaStream_t st);
cudaError_t launch_path_gsum(float* out, const float* x0, const float* x1, long long heads_out, long long per_head,
                             int G, cudaStream_t st);
cudaError_t launch_path_rowdot(const float* X, int Npad, const bf16* w, long long w_sb, long long w_st, long long w_sh,
                               void* out, int out_fp32, long long o_sb, long long o_st, long long o_sh, int B, int H,
                               int T, cudaStream_t st);
cudaError_t launch_path_pack(bf16* out, long long o_sb, long long o_st, long long o_sh, const void* a, int a_fp32,
                             int Ga, const void* bsrc, int b_fp32, int Gb, int B, int H, int T, int Npad,
                             cudaStream_t st);
cudaError_t launch_path_scores(const CUtensorMap& tmKn, const CUtensorMap& tmW, const CUtensorMap& tmW2,
                               const CUtensorMap& tmQs, const PathScoresArgs& a, cudaStream_t st);
cudaError_t launch_path_solve(bool transposed, const CUtensorMap& tmL, const CUtensorMap& tmX, const CUtensorMap& tmU,
                              const PathSolveArgs& a, cudaStream_t st);
cudaError_t launch_path_row(const CUtensorMap& tmDV, const CUtensorMap& tmO, const CUtensorMap& tmKn,
                            const CUtensorMap& tmW, const CUtensorMap& tmW2, const CUtensorMap& tmDs,
                            const PathRowArgs& a, cudaStream_t st);
cudaError_t launch_path_attn(const CUtensorMap& tmKn, const CUtensorMap& tmW, const CUtensorMap& tmW2,
                             const CUtensorMap& tmV, const PathAttnArgs& a, cudaStream_t st);
cudaError_t launch_path_col(const CUtensorMap& tmDA, const CUtensorMap& tmQs, const CUtensorMap& tmDs,
                            const CUtensorMap& tmW, const CUtensorMap& tmW2, const PathColArgs& a, cudaStream_t st);
}  // namespace lb

using namespace lb;

namespace {

constexpr size_t kTile = 128 * 128;  // elements of one per-block matrix

size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }

struct Dims {
  int B = 0, T = 0, H = 0, HQ = 0, G = 1, NB = 0;
  long long Np = 0, NPAIR = 0, BHK = 0, BHQ = 0;
  Dims(int B_, int T_, int H_, int HQ_) : B(B_), T(T_), H(H_), HQ(HQ_) {
    G = H > 0 ? HQ / H : 1;
    NB = (T + 127) / 128;
    Np = (long long)NB * 128;
    NPAIR = (long long)NB * (NB - 1) / 2;
    BHK = (long long)B * H;
    BHQ = (long long)B * HQ;
  }
  size_t blocks_k() const { return (size_t)BHK * NB * kTile; }   // elements of [BHK][NB][128][128]
  size_t blocks_q() const { return (size_t)BHQ * NB * kTile; }
  size_t pairs_q() const { return (size_t)BHQ * NPAIR * kTile; }
};

// Carves consecutive 256-byte aligned regions out of one workspace.
struct Carver {
  size_t off = 0;
  size_t take(size_t bytes) {
    const size_t o = off;
    off += al256(bytes);
    return o;
  }
};

struct FwdLayout {
  size_t status, flags, Tm, WbK, TB, Kn, W2, QW, Qn, Ld, U, Obuf, L, Qs, M, total;
  explicit FwdLayout(const Dims& d) {
    Carver c;
    status = c.take(256);
    flags = c.take((size_t)d.BHQ * d.NB * sizeof(int));
    Tm = c.take(d.blocks_k() * 4);
    WbK = c.take(d.blocks_k() * 2);
    TB = c.take(d.blocks_k() * 2);
    Kn = c.take(d.blocks_k() * 2);
    W2 = c.take(d.blocks_k() * 2);
    QW = c.take(d.blocks_q() * 2);
    Qn = c.take(d.blocks_q() * 4);
    Ld = c.take(d.blocks_q() * 2);
    U = c.take(d.blocks_q() * 2);
    Obuf = c.take(d.blocks_q() * 2);
    L = c.take(d.pairs_q() * 2);
    Qs = c.take(d.pairs_q() * 2);
    M = c.take((d.BHQ > d.BHK ? d.blocks_q() : d.blocks_k()) * 4);
    X = c.take((size_t)d.BHK * kTile * 4);
    total = c.off;
  }
  size_t X;
};

struct BwdLayout {
  size_t status, flags, dV, dA, D, dAd, dqn, dkn, dw2, dw, dQW, dQ, dKq, dTBq;
  size_t kKn, kW20, kW0, kK0, kTB0;  // kv-head sums (grouped heads only)
  size_t dTBb, dTb, dWbKb, Xb, dMb, dWb, dKfin, dWfin, total;
  explicit BwdLayout(const Dims& d) {
    Carver c;
    status = c.take(256);
    flags = c.take((size_t)d.BHQ * d.NB * sizeof(int));
    dV = c.take(d.blocks_q() * 2);
    dA = c.take(d.pairs_q() * 2);
    D = c.take(d.pairs_q() * 2);
    dAd = c.take(d.blocks_q() * 2);
    dqn = c.take(d.blocks_q() * 4);
    dkn = c.take(d.blocks_q() * 4);
    dw2 = c.take(d.blocks_q() * 4);
    dw = c.take(d.blocks_q() * 4);
    dQW = c.take(d.blocks_q() * 2);
    dQ = c.take(d.blocks_q() * 4);
    dKq = c.take(d.blocks_q() * 4);
    dTBq = c.take(d.blocks_q() * 4);
    const size_t kv = d.G > 1 ? d.blocks_k() * 4 : 0;
    kKn = c.take(kv);
    kW20 = c.take(kv);
    kW0 = c.take(kv);
    kK0 = c.take(kv);
    kTB0 = c.take(kv);
    dTBb = c.take(d.blocks_k() * 2);
    dTb = c.take(d.blocks_k() * 2);
    dWbKb = c.take(d.blocks_k() * 2);
    Xb = c.take(d.blocks_k() * 2);
    dMb = c.take(d.blocks_k() * 2);
    dWb = c.take(d.blocks_k() * 4);
    dKfin = c.take(d.blocks_k() * 4);
    dWfin = c.take(d.blocks_k() * 4);
    total = c.off;
  }
};

// PaTH attention forward: the per-block prep of the solve plus the raw diagonal scores.
struct AttnLayout {
  size_t status, Tm, WbK, TB, Kn, W2, QW, Qn, Ad, M, total;
  explicit AttnLayout(const Dims& d) {
    Carver c;
    status = c.take(256);
    Tm = c.take(d.blocks_k() * 4);
    WbK = c.take(d.blocks_k() * 2);
    TB = c.take(d.blocks_k() * 2);
    Kn = c.take(d.blocks_k() * 2);
    W2 = c.take(d.blocks_k() * 2);
    QW = c.take(d.blocks_q() * 2);
    Qn = c.take(d.blocks_q() * 4);
    Ad = c.take(d.blocks_q() * 4);
    M = c.take(d.blocks_k() * 4);
    total = c.off;
  }
};

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool st8(int64_t a, int64_t b, int64_t c) { return (a % 8 == 0) && (b % 8 == 0) && (c % 8 == 0); }

// Internal [heads][Np][128] (= [heads][NB][128][128]) buffer as PMat.
PMat ibuf(void* p, bool fp32, long long heads_per_batch, long long Np, int hdiv) {
  PMat m;
  m.ptr = p;
  m.fp32 = fp32 ? 1 : 0;
  m.s_row = 128;
  m.s_blk = (long long)kTile;
  m.s_h = Np * 128;
  m.s_b = heads_per_batch * Np * 128;
  m.hdiv = hdiv;
  return m;
}
// Caller's [B, T, heads, 128] tensor with element strides (sb, st, sh).
PMat ubuf(const void* p, int64_t sb, int64_t st, int64_t sh, int T, int hdiv) {
  PMat m;
  m.ptr = const_cast<void*>(p);
  m.fp32 = 0;
  m.s_row = st;
  m.s_blk = 128 * st;
  m.s_h = sh;
  m.s_b = sb;
  m.hdiv = hdiv;
  m.rows = T;
  return m;
}
PVec uvec(const void* p, int fp32, int64_t sb, int64_t st, int64_t sh, int T, int hdiv) {
  PVec v;
  v.ptr = p;
  v.fp32 = fp32;
  v.s_row = st;
  v.s_h = sh;
  v.s_b = sb;
  v.hdiv = hdiv;
  v.rows = T;
  return v;
}
POperand opnd(const PMat& m, int trans = 0, float scale = 1.f, int mask = kMaskNone) {
  POperand o;
  o.m = m;
  o.trans = trans;
  o.scale = scale;
  o.mask = mask;
  return o;
}
// The bf16 rounding residual of an fp32 operand (paired with opnd(m) it gives ~16 bits).
POperand opnd_lo(const PMat& m, int trans = 0, float scale = 1.f) {
  POperand o = opnd(m, trans, scale);
  o.lo = 1;
  return o;
}
POperand opnd_rs(const PMat& m, int trans, const PVec& rs) {
  POperand o = opnd(m, trans);
  o.rsc = rs;
  return o;
}

// bf16 tensor map over an internal [heads][rows][128] buffer.
bool tm_int(CUtensorMap* m, const void* p, long long heads, long long rows) {
  return make_tmap_bf16(m, p, 128, (int)rows, (int)heads, 1, 128, rows * 128, heads * rows * 128);
}
// bf16 tensor map over the caller's [B, T, heads, 128].
bool tm_user(CUtensorMap* m, const void* p, int B, int T, int heads, int64_t sb, int64_t st, int64_t sh) {
  return make_tmap_bf16(m, p, 128, T, heads, B, st, sh, sb);
}

struct PrepIn {
  const void *q, *k, *w, *beta;
  int64_t q_sb, q_st, q_sh, k_sb, k_st, k_sh, w_sb, w_st, w_sh, be_sb, be_st, be_sh;
  int beta_fp32;
};
struct PrepOut {
  void *M, *Tm, *WbK, *TB, *Kn, *W2, *QW, *Qn;
};

struct Launcher {
  cudaStream_t st;
  int* status;
  int B, NB;
  cudaError_t err = cudaSuccess;
  void gemm(BGemmArgs a, int Hx) {
    if (err != cudaSuccess) return;
    a.Bn = B;
    a.Hx = Hx;
    a.NB = NB;
    a.status = status;
    ProfileScope ps(LUCID_KERNEL_PATH_BLOCK, st);
    err = launch_path_bgemm(a, st);
  }
  void inv(TriInvArgs a, int Hx) {
    if (err != cudaSuccess) return;
    a.Bn = B;
    a.Hx = Hx;
    a.NB = NB;
    ProfileScope ps(LUCID_KERNEL_PATH_BLOCK, st);
    err = launch_path_triinv(a, st);
  }
};

// UT transform, W2, K_new, QW, Q_new of every 128-row block (triangular_solve_fwd.py:118-148).
void launch_prep_fwd(Launcher& Lc, const Dims& d, const PrepIn& in, const PrepOut& out) {
  const int H = d.H, HQ = d.HQ, G = d.G, T = d.T;
  const long long Np = d.Np;
  const PMat Wk = ubuf(in.w, in.w_sb, in.w_st, in.w_sh, T, 1), Wq = ubuf(in.w, in.w_sb, in.w_st, in.w_sh, T, G);
  const PMat Kk = ubuf(in.k, in.k_sb, in.k_st, in.k_sh, T, 1);
  const PMat Qq = ubuf(in.q, in.q_sb, in.q_st, in.q_sh, T, 1);
  const PVec bet = uvec(in.beta, in.beta_fp32, in.be_sb, in.be_st, in.be_sh, T, 1);
  const PMat Mk = ibuf(out.M, true, H, Np, 1);
  const PMat Tk = ibuf(out.Tm, true, H, Np, 1);
  const PMat WbKk = ibuf(out.WbK, false, H, Np, 1);
  const PMat TBk = ibuf(out.TB, false, H, Np, 1);
  const PMat W2k = ibuf(out.W2, false, H, Np, 1), W2q = ibuf(out.W2, false, H, Np, G);
  const PMat QWq = ibuf(out.QW, false, HQ, Np, 1);
  {  // M = stril(diag(beta) W W^T)
    BGemmArgs a;
    a.A[0] = opnd(Wk);
    a.B[0] = opnd(Wk, 1);
    a.orsc = bet;
    a.out_mask = kMaskStril;
    a.O = Mk;
    Lc.gemm(a, H);
  }
  {  // T = (I + M)^-1
    TriInvArgs a;
    a.M = Mk;
    a.Z = Tk;
    Lc.inv(a, H);
  }
  {  // W2 = T diag(beta) W
    BGemmArgs a;
    a.A[0] = opnd(Tk);
    a.B[0] = opnd_rs(Wk, 0, bet);
    a.O = W2k;
    Lc.gemm(a, H);
  }
  {  // WbK = stril(diag(beta) W K^T)
    BGemmArgs a;
    a.A[0] = opnd_rs(Wk, 0, bet);
    a.B[0] = opnd(Kk, 1);
    a.out_mask = kMaskStril;
    a.O = WbKk;
    Lc.gemm(a, H);
  }
  {  // TB = T WbK
    BGemmArgs a;
    a.A[0] = opnd(Tk);
    a.B[0] = opnd(WbKk);
    a.O = TBk;
    Lc.gemm(a, H);
  }
  {  // K_new = K - TB^T W
    BGemmArgs a;
    a.A[0] = opnd(TBk, 1, -1.f);
    a.B[0] = opnd(Wk);
    a.nc = 1;
    a.C[0] = Kk;
    a.O = ibuf(out.Kn, false, H, Np, 1);
    Lc.gemm(a, H);
  }
  {  // QW = tril(Q W^T)
    BGemmArgs a;
    a.A[0] = opnd(Qq);
    a.B[0] = opnd(Wq, 1);
    a.out_mask = kMaskTril;
    a.O = QWq;
    Lc.gemm(a, HQ);
  }
  {  // Q_new = Q - QW W2
    BGemmArgs a;
    a.A[0] = opnd(QWq, 0, -1.f);
    a.B[0] = opnd(W2q);
    a.nc = 1;
    a.C[0] = Qq;
    a.O = ibuf(out.Qn, true, HQ, Np, 1);
    Lc.gemm(a, HQ);
  }
}

bool path_shape_ok(int B, int T, int H, int HQ, int D) {
  return B >= 0 && T >= 0 && H >= 0 && HQ >= 0 && D == kHeadDim && (H == 0 ? HQ == 0 : HQ % H == 0) &&
         T <= (1 << 22);
}

}  // namespace

extern "C" {

size_t lucid_path_fwd_workspace_bytes(int B, int T, int H, int HQ, int D) {
  (void)D;
  return FwdLayout(Dims(B, T, H, HQ)).total;
}

size_t lucid_path_bwd_workspace_bytes(int B, int T, int H, int HQ, int D) {
  (void)D;
  return BwdLayout(Dims(B, T, H, HQ)).total;
}

int lucid_path_fwd(int B, int T, int H, int HQ, int D, float scale,
                   const void* q, int64_t q_sb, int64_t q_st, int64_t q_sh,
                   const void* k, int64_t k_sb, int64_t k_st, int64_t k_sh,
                   const void* v, int64_t v_sb, int64_t v_st, int64_t v_sh,
                   const void* w, int64_t w_sb, int64_t w_st, int64_t w_sh,
                   const void* beta, int beta_fp32, int64_t be_sb, int64_t be_st, int64_t be_sh,
                   void* o, int64_t o_sb, int64_t o_st, int64_t o_sh,
                   void* k_cache, int64_t kc_sb, int64_t kc_st, int64_t kc_sh,
                   void* workspace, size_t workspace_bytes, void* stream) {
  if (!path_shape_ok(B, T, H, HQ, D)) return LUCID_ERR_SHAPE;
  if (q == nullptr) {
    if (HQ != H) return LUCID_ERR_SHAPE;
    q = k; q_sb = k_sb; q_st = k_st; q_sh = k_sh;
  }
  if (B == 0 || T == 0 || H == 0) return LUCID_OK;
  if (!al16(q) || !al16(k) || !al16(v) || !al16(w) || !al16(o) || !st8(q_sb, q_st, q_sh) ||
      !st8(k_sb, k_st, k_sh) || !st8(v_sb, v_st, v_sh) || !st8(w_sb, w_st, w_sh) || !st8(o_sb, o_st, o_sh) ||
      (k_cache != nullptr && (!al16(k_cache) || !st8(kc_sb, kc_st, kc_sh))))
    return LUCID_ERR_ALIGN;
  const Dims d(B, T, H, HQ);
  if (d.NPAIR * 128 >= (1LL << 31)) return LUCID_ERR_TOO_LARGE;
  const FwdLayout lay(d);
  if (workspace == nullptr || workspace_bytes < lay.total || !al16(workspace)) return LUCID_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  int* status = reinterpret_cast<int*>(ws + lay.status);
  auto P = [&](size_t off) { return static_cast<void*>(ws + off); };
  const int G = d.G;
  const long long Np = d.Np;

  // ---- tensor maps ----
  CUtensorMap tmKn, tmW, tmW2, tmQs, tmL, tmO, tmU;
  const bool pairs = d.NPAIR > 0;
  bool ok = tm_int(&tmKn, P(lay.Kn), d.BHK, Np) && tm_user(&tmW, w, B, T, H, w_sb, w_st, w_sh) &&
            tm_int(&tmW2, P(lay.W2), d.BHK, Np) && tm_int(&tmO, P(lay.Obuf), d.BHQ, Np) &&
            tm_int(&tmU, P(lay.U), d.BHQ, Np);
  // pair maps (unused when there is a single block: point them at U)
  ok = ok && (pairs ? tm_int(&tmQs, P(lay.Qs), d.BHQ, d.NPAIR * 128) : tm_int(&tmQs, P(lay.U), d.BHQ, Np));
  ok = ok && (pairs ? tm_int(&tmL, P(lay.L), d.BHQ, d.NPAIR * 128) : tm_int(&tmL, P(lay.U), d.BHQ, Np));
  if (!ok) return LUCID_ERR_TENSORMAP;

  if (cudaMemsetAsync(ws, 0, lay.Tm, st) != cudaSuccess) return LUCID_ERR_LAUNCH;

  const PMat Kq = ubuf(k, k_sb, k_st, k_sh, T, G);
  const PMat Qq = ubuf(q, q_sb, q_st, q_sh, T, 1);
  const PMat Mq = ibuf(P(lay.M), true, HQ, Np, 1);
  const PMat TBq = ibuf(P(lay.TB), false, H, Np, G);
  const PMat QWq = ibuf(P(lay.QW), false, HQ, Np, 1);

  Launcher Lc{st, status, B, d.NB};
  launch_prep_fwd(Lc, d, PrepIn{q, k, w, beta, q_sb, q_st, q_sh, k_sb, k_st, k_sh, w_sb, w_st, w_sh, be_sb, be_st,
                                be_sh, beta_fp32},
                  PrepOut{P(lay.M), P(lay.Tm), P(lay.WbK), P(lay.TB), P(lay.Kn), P(lay.W2), P(lay.QW), P(lay.Qn)});
  {  // L_ii = stril(exp(s (Q K^T - QW TB) - 1/s))   (fp32 into M)
    BGemmArgs a;
    a.nprod = 2;
    a.A[0] = opnd(Qq);
    a.B[0] = opnd(Kq, 1);
    a.A[1] = opnd(QWq, 0, -1.f);
    a.B[1] = opnd(TBq);
    a.epi = kEpiPathExp;
    a.s = scale;
    a.out_mask = kMaskStril;
    a.O = Mq;
    Lc.gemm(a, HQ);
  }
  {  // U = (I + L_ii)^-1 - I, and the bf16 copy of L_ii
    TriInvArgs a;
    a.M = Mq;
    a.U = ibuf(P(lay.U), false, HQ, Np, 1);
    a.Mcopy = ibuf(P(lay.Ld), false, HQ, Np, 1);
    Lc.inv(a, HQ);
  }
  if (Lc.err != cudaSuccess) return LUCID_ERR_LAUNCH;

  if (pairs) {
    PathScoresArgs a{B, HQ, H, G, d.NB, (int)d.NPAIR, scale, reinterpret_cast<const float*>(P(lay.Qn)),
                     reinterpret_cast<bf16*>(P(lay.L)), status};
    ProfileScope ps(LUCID_KERNEL_PATH_SCORES, st);
    if (launch_path_scores(tmKn, tmW, tmW2, tmQs, a, st) != cudaSuccess) return LUCID_ERR_LAUNCH;
  }
  {
    PathSolveArgs a{B, HQ, H, G, T, d.NB, (int)d.NPAIR, reinterpret_cast<const bf16*>(v), v_sb, v_sh, v_st,
                    reinterpret_cast<bf16*>(P(lay.Obuf)), reinterpret_cast<bf16*>(o), o_sb, o_sh, o_st,
                    reinterpret_cast<int*>(P(lay.flags)), status};
    ProfileScope ps(LUCID_KERNEL_PATH_SOLVE, st);
    if (launch_path_solve(false, tmL, tmO, tmU, a, st) != cudaSuccess) return LUCID_ERR_LAUNCH;
  }
  if (k_cache != nullptr) {
    // Decode-time keys (prepare_k_cache.py:8-49): every key transformed by all later
    // Householders, k_cache_c = (H_{T-1} ... H_{c+1}) k_c.  Per block j:
    //   K_cache_j = K_new_j P_j,  P_{NB-1} = I,  P_j = G_{j+1}^T P_{j+1} = P_{j+1} - W2_{j+1}^T (W_{j+1} P_{j+1})
    // with the suffix products P_j (fp32, [B*H][NB][128][128]) in the M scratch.
    const int NB = d.NB;
    float* Pbuf = reinterpret_cast<float*>(P(lay.M));
    if (launch_path_eye(Pbuf + (size_t)(NB - 1) * kTile, d.BHK, (long long)NB * kTile, st) != cudaSuccess)
      return LUCID_ERR_LAUNCH;
    Launcher Lk{st, status, B, 1};
    for (int j = NB - 2; j >= 0; --j) {
      const PMat Pn = ibuf(Pbuf + (size_t)(j + 1) * kTile, true, H, Np, 1);
      const PMat Pj = ibuf(Pbuf + (size_t)j * kTile, true, H, Np, 1);
      PMat Wn = ubuf(static_cast<const bf16*>(w) + (int64_t)(j + 1) * 128 * w_st, w_sb, w_st, w_sh, T - (j + 1) * 128, 1);
      const PMat W2n = ibuf(static_cast<bf16*>(P(lay.W2)) + (size_t)(j + 1) * kTile, false, H, Np, 1);
      const PMat Xk = ibuf(P(lay.X), true, H, 128, 1);
      // fp32 products enter the tensor core as bf16 hi + lo, so the products keep
      // ~16 mantissa bits along the chain
      {  // X = W_{j+1} P_{j+1}
        BGemmArgs a;
        a.nprod = 2;
        a.A[0] = opnd(Wn);
        a.B[0] = opnd(Pn);
        a.A[1] = opnd(Wn);
        a.B[1] = opnd_lo(Pn);
        a.O = Xk;
        Lk.gemm(a, H);
      }
      {  // P_j = P_{j+1} - W2_{j+1}^T X
        BGemmArgs a;
        a.nprod = 2;
        a.A[0] = opnd(W2n, 1, -1.f);
        a.B[0] = opnd(Xk);
        a.A[1] = opnd(W2n, 1, -1.f);
        a.B[1] = opnd_lo(Xk);
        a.nc = 1;
        a.C[0] = Pn;
        a.O = Pj;
        Lk.gemm(a, H);
      }
    }
    {  // K_cache = K_new P   (all blocks)
      BGemmArgs a;
      a.nprod = 2;
      a.A[0] = opnd(ibuf(P(lay.Kn), false, H, Np, 1));
      a.B[0] = opnd(ibuf(Pbuf, true, H, Np, 1));
      a.A[1] = opnd(ibuf(P(lay.Kn), false, H, Np, 1));
      a.B[1] = opnd_lo(ibuf(Pbuf, true, H, Np, 1));
      PMat out = ubuf(k_cache, kc_sb, kc_st, kc_sh, T, 1);
      a.O = out;
      Lc.gemm(a, H);
    }
    if (Lk.err != cudaSuccess || Lc.err != cudaSuccess) return LUCID_ERR_LAUNCH;
  }
  return LUCID_OK;
}

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
                   void* workspace, size_t workspace_bytes, void* stream) {
  if (!path_shape_ok(B, T, H, HQ, D)) return LUCID_ERR_SHAPE;
  const bool q_is_k = (q == nullptr);
  if (q_is_k) {
    if (HQ != H) return LUCID_ERR_SHAPE;
    q = k; q_sb = k_sb; q_st = k_st; q_sh = k_sh;
  } else if (dq == nullptr) {
    return LUCID_ERR_SHAPE;
  }
  if (B == 0 || T == 0 || H == 0) return LUCID_OK;
  if (!al16(q) || !al16(k) || !al16(w) || !al16(dout) || !al16(dk) || !al16(dv) || !al16(dw) ||
      (!q_is_k && !al16(dq)) || !st8(q_sb, q_st, q_sh) || !st8(k_sb, k_st, k_sh) || !st8(w_sb, w_st, w_sh) ||
      !st8(do_sb, do_st, do_sh) || !st8(dk_sb, dk_st, dk_sh) || !st8(dv_sb, dv_st, dv_sh) ||
      !st8(dw_sb, dw_st, dw_sh) || (!q_is_k && !st8(dq_sb, dq_st, dq_sh)))
    return LUCID_ERR_ALIGN;
  const Dims d(B, T, H, HQ);
  if (d.NPAIR * 128 >= (1LL << 31)) return LUCID_ERR_TOO_LARGE;
  const FwdLayout fl(d);
  const BwdLayout bl(d);
  if (fwd_workspace == nullptr || fwd_workspace_bytes < fl.total) return LUCID_ERR_WORKSPACE;
  if (workspace == nullptr || workspace_bytes < bl.total || !al16(workspace)) return LUCID_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  char* fws = static_cast<char*>(const_cast<void*>(fwd_workspace));
  char* ws = static_cast<char*>(workspace);
  int* status = reinterpret_cast<int*>(ws + bl.status);
  auto F = [&](size_t off) { return static_cast<void*>(fws + off); };
  auto P = [&](size_t off) { return static_cast<void*>(ws + off); };
  const int G = d.G;
  const long long Np = d.Np;
  const bool pairs = d.NPAIR > 0;

  CUtensorMap tmL, tmDVb, tmU, tmO, tmKn, tmW, tmW2, tmDs, tmDA, tmQs;
  bool ok = tm_int(&tmDVb, P(bl.dV), d.BHQ, Np) && tm_int(&tmU, F(fl.U), d.BHQ, Np) &&
            tm_int(&tmO, F(fl.Obuf), d.BHQ, Np) && tm_int(&tmKn, F(fl.Kn), d.BHK, Np) &&
            tm_user(&tmW, w, B, T, H, w_sb, w_st, w_sh) && tm_int(&tmW2, F(fl.W2), d.BHK, Np);
  if (pairs) {
    ok = ok && tm_int(&tmL, F(fl.L), d.BHQ, d.NPAIR * 128) && tm_int(&tmDs, P(bl.D), d.BHQ, d.NPAIR * 128) &&
         tm_int(&tmDA, P(bl.dA), d.BHQ, d.NPAIR * 128) && tm_int(&tmQs, F(fl.Qs), d.BHQ, d.NPAIR * 128);
  } else {
    ok = ok && tm_int(&tmL, F(fl.U), d.BHQ, Np) && tm_int(&tmDs, F(fl.U), d.BHQ, Np) &&
         tm_int(&tmDA, F(fl.U), d.BHQ, Np) && tm_int(&tmQs, F(fl.U), d.BHQ, Np);
  }
  if (!ok) return LUCID_ERR_TENSORMAP;
  if (cudaMemsetAsync(ws, 0, bl.dV, st) != cudaSuccess) return LUCID_ERR_LAUNCH;

  // ---- dV = (I + L)^-T dO ----
  {
    PathSolveArgs a{B, HQ, H, G, T, d.NB, (int)d.NPAIR, reinterpret_cast<const bf16*>(dout), do_sb, do_sh, do_st,
                    reinterpret_cast<bf16*>(P(bl.dV)), nullptr, 0, 0, 0, reinterpret_cast<int*>(P(bl.flags)), status};
    ProfileScope ps(LUCID_KERNEL_PATH_SOLVE_T, st);
    if (launch_path_solve(true, tmL, tmDVb, tmU, a, st) != cudaSuccess) return LUCID_ERR_LAUNCH;
  }
  // ---- row pass: dA tiles, dQ~ chain ----
  {
    PathRowArgs a{B, HQ, H, G, d.NB, (int)d.NPAIR, scale, reinterpret_cast<const bf16*>(F(fl.L)),
                  reinterpret_cast<const bf16*>(F(fl.Ld)), reinterpret_cast<bf16*>(P(bl.dA)),
                  reinterpret_cast<bf16*>(P(bl.dAd)), reinterpret_cast<float*>(P(bl.dqn)), status};
    ProfileScope ps(LUCID_KERNEL_PATH_ROW, st);
    if (launch_path_row(tmDVb, tmO, tmKn, tmW, tmW2, tmDs, a, st) != cudaSuccess) return LUCID_ERR_LAUNCH;
  }
  // ---- column pass: dK_new, Phi -> dW2, dW ----
  {
    PathColArgs a{B, HQ, H, G, d.NB, (int)d.NPAIR, reinterpret_cast<float*>(P(bl.dkn)),
                  reinterpret_cast<float*>(P(bl.dw2)), reinterpret_cast<float*>(P(bl.dw)), status};
    ProfileScope ps(LUCID_KERNEL_PATH_COL, st);
    if (launch_path_col(tmDA, tmQs, tmDs, tmW, tmW2, a, st) != cudaSuccess) return LUCID_ERR_LAUNCH;
  }

  // ---- per-block backward ----
  const PMat Wk = ubuf(w, w_sb, w_st, w_sh, T, 1), Wq = ubuf(w, w_sb, w_st, w_sh, T, G);
  const PMat Kk = ubuf(k, k_sb, k_st, k_sh, T, 1), Kq = ubuf(k, k_sb, k_st, k_sh, T, G);
  const PMat Qq = ubuf(q, q_sb, q_st, q_sh, T, 1);
  const PVec bet = uvec(beta, beta_fp32, be_sb, be_st, be_sh, T, 1);
  const PMat Tk = ibuf(F(fl.Tm), true, H, Np, 1);
  const PMat WbKk = ibuf(F(fl.WbK), false, H, Np, 1);
  const PMat TBk = ibuf(F(fl.TB), false, H, Np, 1), TBq = ibuf(F(fl.TB), false, H, Np, G);
  const PMat W2q = ibuf(F(fl.W2), false, H, Np, G);
  const PMat QWq = ibuf(F(fl.QW), false, HQ, Np, 1);
  const PMat dAdq = ibuf(P(bl.dAd), false, HQ, Np, 1);
  const PMat dqnq = ibuf(P(bl.dqn), true, HQ, Np, 1);
  const PMat dQWq = ibuf(P(bl.dQW), false, HQ, Np, 1);
  const PMat dw2q = ibuf(P(bl.dw2), true, HQ, Np, 1), dwq = ibuf(P(bl.dw), true, HQ, Np, 1);

  Launcher Lc{st, status, B, d.NB};
  {  // dQW = tril(-dA TB^T - dQn W2^T)
    BGemmArgs a;
    a.nprod = 2;
    a.A[0] = opnd(dAdq, 0, -1.f);
    a.B[0] = opnd(TBq, 1);
    a.A[1] = opnd(dqnq, 0, -1.f);
    a.B[1] = opnd(W2q, 1);
    a.out_mask = kMaskTril;
    a.O = dQWq;
    Lc.gemm(a, HQ);
  }
  {  // dQ = dA K + dQW W + dQn
    BGemmArgs a;
    a.nprod = 2;
    a.A[0] = opnd(dAdq);
    a.B[0] = opnd(Kq);
    a.A[1] = opnd(dQWq);
    a.B[1] = opnd(Wq);
    a.nc = 1;
    a.C[0] = dqnq;
    a.O = ibuf(P(bl.dQ), true, HQ, Np, 1);
    Lc.gemm(a, HQ);
  }
  {  // dK (query-head part) = dA^T Q
    BGemmArgs a;
    a.A[0] = opnd(dAdq, 1);
    a.B[0] = opnd(Qq);
    a.O = ibuf(P(bl.dKq), true, HQ, Np, 1);
    Lc.gemm(a, HQ);
  }
  {  // dTB (query-head part) = -QW^T dA
    BGemmArgs a;
    a.A[0] = opnd(QWq, 1, -1.f);
    a.B[0] = opnd(dAdq);
    a.O = ibuf(P(bl.dTBq), true, HQ, Np, 1);
    Lc.gemm(a, HQ);
  }
  {  // dW2 (query-head part) = -QW^T dQn + column-pass dW2   (in place)
    BGemmArgs a;
    a.A[0] = opnd(QWq, 1, -1.f);
    a.B[0] = opnd(dqnq);
    a.nc = 1;
    a.C[0] = dw2q;
    a.O = dw2q;
    Lc.gemm(a, HQ);
  }
  {  // dW (query-head part) = dQW^T Q + column-pass dW   (in place)
    BGemmArgs a;
    a.A[0] = opnd(dQWq, 1);
    a.B[0] = opnd(Qq);
    a.nc = 1;
    a.C[0] = dwq;
    a.O = dwq;
    Lc.gemm(a, HQ);
  }
  if (Lc.err != cudaSuccess) return LUCID_ERR_LAUNCH;
  // sums over the query heads of each key head
  void *kKn = P(bl.dkn), *kW20 = P(bl.dw2), *kW0 = P(bl.dw), *kK0 = P(bl.dKq), *kTB0 = P(bl.dTBq);
  if (G > 1) {
    const long long per = Np * 128;
    kKn = P(bl.kKn); kW20 = P(bl.kW20); kW0 = P(bl.kW0); kK0 = P(bl.kK0); kTB0 = P(bl.kTB0);
    cudaError_t e = launch_path_gsum((float*)kKn, (const float*)P(bl.dkn), nullptr, d.BHK, per, G, st);
    if (e == cudaSuccess) e = launch_path_gsum((float*)kW20, (const float*)P(bl.dw2), nullptr, d.BHK, per, G, st);
    if (e == cudaSuccess) e = launch_path_gsum((float*)kW0, (const float*)P(bl.dw), nullptr, d.BHK, per, G, st);
    if (e == cudaSuccess) e = launch_path_gsum((float*)kK0, (const float*)P(bl.dKq), nullptr, d.BHK, per, G, st);
    if (e == cudaSuccess) e = launch_path_gsum((float*)kTB0, (const float*)P(bl.dTBq), nullptr, d.BHK, per, G, st);
    if (e != cudaSuccess) return LUCID_ERR_LAUNCH;
  }
  const PMat dKnk = ibuf(kKn, true, H, Np, 1), dW20k = ibuf(kW20, true, H, Np, 1), dW0k = ibuf(kW0, true, H, Np, 1);
  const PMat dK0k = ibuf(kK0, true, H, Np, 1), dTB0k = ibuf(kTB0, true, H, Np, 1);
  const PMat dTBb = ibuf(P(bl.dTBb), false, H, Np, 1), dTb = ibuf(P(bl.dTb), false, H, Np, 1);
  const PMat dWbKb = ibuf(P(bl.dWbKb), false, H, Np, 1), Xb = ibuf(P(bl.Xb), false, H, Np, 1);
  const PMat dMb = ibuf(P(bl.dMb), false, H, Np, 1), dWb = ibuf(P(bl.dWb), true, H, Np, 1);
  const PMat dKfin = ibuf(P(bl.dKfin), true, H, Np, 1), dWfin = ibuf(P(bl.dWfin), true, H, Np, 1);
  {  // dTB = dTB0 - W dK_new^T
    BGemmArgs a;
    a.A[0] = opnd(Wk, 0, -1.f);
    a.B[0] = opnd(dKnk, 1);
    a.nc = 1;
    a.C[0] = dTB0k;
    a.O = dTBb;
    Lc.gemm(a, H);
  }
  {  // dW0 -= TB dK_new   (in place)
    BGemmArgs a;
    a.A[0] = opnd(TBk, 0, -1.f);
    a.B[0] = opnd(dKnk);
    a.nc = 1;
    a.C[0] = dW0k;
    a.O = dW0k;
    Lc.gemm(a, H);
  }
  {  // dT = dTB WbK^T + dW2 (diag(beta) W)^T
    BGemmArgs a;
    a.nprod = 2;
    a.A[0] = opnd(dTBb);
    a.B[0] = opnd(WbKk, 1);
    a.A[1] = opnd(dW20k);
    a.B[1] = opnd_rs(Wk, 1, bet);
    a.O = dTb;
    Lc.gemm(a, H);
  }
  {  // dWbK = stril(T^T dTB)
    BGemmArgs a;
    a.A[0] = opnd(Tk, 1);
    a.B[0] = opnd(dTBb);
    a.out_mask = kMaskStril;
    a.O = dWbKb;
    Lc.gemm(a, H);
  }
  {  // X = T^T dT
    BGemmArgs a;
    a.A[0] = opnd(Tk, 1);
    a.B[0] = opnd(dTb);
    a.O = Xb;
    Lc.gemm(a, H);
  }
  {  // dM = stril(-X T^T)
    BGemmArgs a;
    a.A[0] = opnd(Xb, 0, -1.f);
    a.B[0] = opnd(Tk, 1);
    a.out_mask = kMaskStril;
    a.O = dMb;
    Lc.gemm(a, H);
  }
  {  // d(diag(beta) W) = dWbK K + T^T dW2 + dM W
    BGemmArgs a;
    a.nprod = 3;
    a.A[0] = opnd(dWbKb);
    a.B[0] = opnd(Kk);
    a.A[1] = opnd(Tk, 1);
    a.B[1] = opnd(dW20k);
    a.A[2] = opnd(dMb);
    a.B[2] = opnd(Wk);
    a.O = dWb;
    Lc.gemm(a, H);
  }
  {  // dK = dK0 + dK_new + dWbK^T diag(beta) W
    BGemmArgs a;
    a.A[0] = opnd(dWbKb, 1);
    a.B[0] = opnd_rs(Wk, 0, bet);
    a.nc = 2;
    a.C[0] = dK0k;
    a.C[1] = dKnk;
    a.O = dKfin;
    Lc.gemm(a, H);
  }
  {  // dW = dW0 + dM^T diag(beta) W + diag(beta) d(diag(beta) W)
    BGemmArgs a;
    a.A[0] = opnd(dMb, 1);
    a.B[0] = opnd_rs(Wk, 0, bet);
    a.nc = 2;
    a.C[0] = dW0k;
    a.C[1] = dWb;
    a.crsc[1] = bet;
    a.O = dWfin;
    Lc.gemm(a, H);
  }
  if (Lc.err != cudaSuccess) return LUCID_ERR_LAUNCH;
  {
    ProfileScope ps(LUCID_KERNEL_PATH_BLOCK, st);
    cudaError_t e = launch_path_rowdot((const float*)P(bl.dWb), (int)Np, (const bf16*)w, w_sb, w_st, w_sh, dbeta,
                                       dbeta_fp32, db_sb, db_st, db_sh, B, H, T, st);
    // outputs: dk (+ dq when q is k), dq, dv (sum over the query heads of a key head), dw
    if (e == cudaSuccess)
      e = launch_path_pack((bf16*)dk, dk_sb, dk_st, dk_sh, P(bl.dKfin), 1, 1, q_is_k ? P(bl.dQ) : nullptr, 1, 1, B, H,
                           T, (int)Np, st);
    if (e == cudaSuccess && !q_is_k)
      e = launch_path_pack((bf16*)dq, dq_sb, dq_st, dq_sh, P(bl.dQ), 1, 1, nullptr, 1, 1, B, HQ, T, (int)Np, st);
    if (e == cudaSuccess)
      e = launch_path_pack((bf16*)dv, dv_sb, dv_st, dv_sh, P(bl.dV), 0, G, nullptr, 1, 1, B, H, T, (int)Np, st);
    if (e == cudaSuccess)
      e = launch_path_pack((bf16*)dw, dw_sb, dw_st, dw_sh, P(bl.dWfin), 1, 1, nullptr, 1, 1, B, H, T, (int)Np, st);
    if (e != cudaSuccess) return LUCID_ERR_LAUNCH;
  }
  return LUCID_OK;
}

size_t lucid_path_attn_fwd_workspace_bytes(int B, int T, int H, int HQ, int D) {
  (void)D;
  return AttnLayout(Dims(B, T, H, HQ)).total;
}

int lucid_path_attn_fwd(int B, int T, int H, int HQ, int D, float scale,
                        const void* q, int64_t q_sb, int64_t q_st, int64_t q_sh,
                        const void* k, int64_t k_sb, int64_t k_st, int64_t k_sh,
                        const void* v, int64_t v_sb, int64_t v_st, int64_t v_sh,
                        const void* w, int64_t w_sb, int64_t w_st, int64_t w_sh,
                        const void* beta, int beta_fp32, int64_t be_sb, int64_t be_st, int64_t be_sh,
                        void* o, int64_t o_sb, int64_t o_st, int64_t o_sh,
                        float* lse, int64_t l_sb, int64_t l_st, int64_t l_sh,
                        void* workspace, size_t workspace_bytes, void* stream) {
  if (!path_shape_ok(B, T, H, HQ, D)) return LUCID_ERR_SHAPE;
  if (q == nullptr) {
    if (HQ != H) return LUCID_ERR_SHAPE;
    q = k; q_sb = k_sb; q_st = k_st; q_sh = k_sh;
  }
  if (B == 0 || T == 0 || H == 0) return LUCID_OK;
  if (!al16(q) || !al16(k) || !al16(v) || !al16(w) || !al16(o) || lse == nullptr || !st8(q_sb, q_st, q_sh) ||
      !st8(k_sb, k_st, k_sh) || !st8(v_sb, v_st, v_sh) || !st8(w_sb, w_st, w_sh) || !st8(o_sb, o_st, o_sh))
    return LUCID_ERR_ALIGN;
  const Dims d(B, T, H, HQ);
  const AttnLayout lay(d);
  if (workspace == nullptr || workspace_bytes < lay.total || !al16(workspace)) return LUCID_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  int* status = reinterpret_cast<int*>(ws + lay.status);
  auto P = [&](size_t off) { return static_cast<void*>(ws + off); };
  const long long Np = d.Np;
  CUtensorMap tmKn, tmW, tmW2, tmV;
  if (!(tm_int(&tmKn, P(lay.Kn), d.BHK, Np) && tm_user(&tmW, w, B, T, H, w_sb, w_st, w_sh) &&
        tm_int(&tmW2, P(lay.W2), d.BHK, Np) && tm_user(&tmV, v, B, T, H, v_sb, v_st, v_sh)))
    return LUCID_ERR_TENSORMAP;
  if (cudaMemsetAsync(ws, 0, 256, st) != cudaSuccess) return LUCID_ERR_LAUNCH;
  Launcher Lc{st, status, B, d.NB};
  launch_prep_fwd(Lc, d, PrepIn{q, k, w, beta, q_sb, q_st, q_sh, k_sb, k_st, k_sh, w_sb, w_st, w_sh, be_sb, be_st,
                                be_sh, beta_fp32},
                  PrepOut{P(lay.M), P(lay.Tm), P(lay.WbK), P(lay.TB), P(lay.Kn), P(lay.W2), P(lay.QW), P(lay.Qn)});
  {  // raw diagonal-block scores A_ii = tril(Q K^T - QW TB)
    BGemmArgs a;
    a.nprod = 2;
    a.A[0] = opnd(ubuf(q, q_sb, q_st, q_sh, T, 1));
    a.B[0] = opnd(ubuf(k, k_sb, k_st, k_sh, T, d.G), 1);
    a.A[1] = opnd(ibuf(P(lay.QW), false, HQ, Np, 1), 0, -1.f);
    a.B[1] = opnd(ibuf(P(lay.TB), false, H, Np, d.G));
    a.out_mask = kMaskTril;
    a.O = ibuf(P(lay.Ad), true, HQ, Np, 1);
    Lc.gemm(a, HQ);
  }
  if (Lc.err != cudaSuccess) return LUCID_ERR_LAUNCH;
  PathAttnArgs a{B, HQ, H, d.G, T, d.NB, scale, reinterpret_cast<const float*>(P(lay.Qn)),
                 reinterpret_cast<const float*>(P(lay.Ad)), reinterpret_cast<bf16*>(o), o_sb, o_st, o_sh, lse,
                 l_sb, l_st, l_sh, status};
  ProfileScope ps(LUCID_KERNEL_PATH_ATTN, st);
  if (launch_path_attn(tmKn, tmW, tmW2, tmV, a, st) != cudaSuccess) return LUCID_ERR_LAUNCH;
  return LUCID_OK;
}

}  // extern "C"
