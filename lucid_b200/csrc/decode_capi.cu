// extern "C" entry point of the LUCID decode step (include/lucid_b200.h).
#include "lucid_b200.h"
#include "lucid_common.cuh"
#include "profile.h"

namespace lb {
int decode_splits(int B, int H, int Nc);
cudaError_t launch_decode(DecodeArgs a, cudaStream_t st);
cudaError_t launch_decode_attn(DecodeArgs a, cudaStream_t st);
bool decode_step_fused(int gq, int Ln);
cudaError_t launch_decode_step(DecodeStepArgs a, cudaStream_t st);
}  // namespace lb

using namespace lb;

namespace {
bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool a8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; }
bool s4(int64_t a, int64_t b, int64_t c) { return (a % 4 == 0) && (b % 4 == 0) && (c % 4 == 0); }
}  // namespace

extern "C" {

size_t lucid_decode_workspace_bytes(int B, int H, int Ln, int Nc, int D) {
  (void)D;
  return (size_t)decode_splits(B, H, Nc) * B * H * Ln * 128 * sizeof(float) + 256;
}

int lucid_decode_update(int B, int H, int Ln, int Nc, int D, float scale, float eps,
                        const void* k_new, int64_t kn_sb, int64_t kn_sh, int64_t kn_sn,
                        const void* v_new, int64_t vn_sb, int64_t vn_sh, int64_t vn_sn,
                        const void* k_cache, int64_t kc_sb, int64_t kc_sh, int64_t kc_sn,
                        const void* x_cache, int64_t xc_sb, int64_t xc_sh, int64_t xc_sn,
                        void* x_new, int64_t o_sb, int64_t o_sh, int64_t o_sn,
                        void* workspace, size_t workspace_bytes, void* stream) {
  if (B < 0 || H < 0 || Ln < 0 || Nc < 0 || D < 4 || D > kHeadDim || D % 4 || (long long)B * H > 65535)
    return LUCID_ERR_SHAPE;
  if (B == 0 || H == 0 || Ln == 0) return LUCID_OK;
  if (!a8(k_new) || !a8(k_cache) || !a8(x_cache) || !s4(kn_sb, kn_sh, kn_sn) || !s4(kc_sb, kc_sh, kc_sn) ||
      !s4(xc_sb, xc_sh, xc_sn))
    return LUCID_ERR_ALIGN;
  if (workspace == nullptr || workspace_bytes < lucid_decode_workspace_bytes(B, H, Ln, Nc, D) || !a16(workspace))
    return LUCID_ERR_WORKSPACE;
  DecodeArgs a{B, H, Ln, Nc, 0, 0, scale, eps,
               static_cast<const bf16*>(k_new), kn_sb, kn_sh, kn_sn,
               static_cast<const bf16*>(v_new), vn_sb, vn_sh, vn_sn,
               static_cast<const bf16*>(k_cache), kc_sb, kc_sh, kc_sn,
               static_cast<const bf16*>(x_cache), xc_sb, xc_sh, xc_sn,
               static_cast<bf16*>(x_new), o_sb, o_sh, o_sn,
               reinterpret_cast<float*>(static_cast<char*>(workspace) + 256), H, D};
  ProfileScope ps(LUCID_KERNEL_DECODE, reinterpret_cast<cudaStream_t>(stream));
  return launch_decode(a, reinterpret_cast<cudaStream_t>(stream)) == cudaSuccess ? LUCID_OK : LUCID_ERR_LAUNCH;
}

size_t lucid_decode_attn_workspace_bytes(int B, int Hq, int Ln, int Nc, int D) {
  (void)D;
  return (size_t)decode_splits(B, Hq, Nc) * B * Hq * Ln * 130 * sizeof(float) + 256;
}

int lucid_decode_attn(int B, int Hq, int Hkv, int Ln, int Nc, int D, float scale,
                      const void* q, int64_t q_sb, int64_t q_sh, int64_t q_sn,
                      const void* k_cache, int64_t kc_sb, int64_t kc_sh, int64_t kc_sn,
                      const void* x_cache, int64_t xc_sb, int64_t xc_sh, int64_t xc_sn,
                      void* o, int64_t o_sb, int64_t o_sh, int64_t o_sn,
                      void* workspace, size_t workspace_bytes, void* stream) {
  if (B < 0 || Hq < 0 || Hkv <= 0 || Ln < 0 || Nc < Ln || D < 4 || D > kHeadDim || D % 4 || Hq % Hkv != 0 ||
      (long long)B * Hq > 65535)
    return LUCID_ERR_SHAPE;
  if (B == 0 || Hq == 0 || Ln == 0) return LUCID_OK;
  if (!a8(k_cache) || !a8(x_cache) || !s4(kc_sb, kc_sh, kc_sn) || !s4(xc_sb, xc_sh, xc_sn)) return LUCID_ERR_ALIGN;
  if (workspace == nullptr || workspace_bytes < lucid_decode_attn_workspace_bytes(B, Hq, Ln, Nc, D) ||
      !a16(workspace))
    return LUCID_ERR_WORKSPACE;
  DecodeArgs a{B, Hkv, Ln, Nc, 0, 0, scale, 0.f,
               static_cast<const bf16*>(q), q_sb, q_sh, q_sn,
               nullptr, 0, 0, 0,
               static_cast<const bf16*>(k_cache), kc_sb, kc_sh, kc_sn,
               static_cast<const bf16*>(x_cache), xc_sb, xc_sh, xc_sn,
               static_cast<bf16*>(o), o_sb, o_sh, o_sn,
               reinterpret_cast<float*>(static_cast<char*>(workspace) + 256), Hq, D};
  ProfileScope ps(LUCID_KERNEL_DECODE, reinterpret_cast<cudaStream_t>(stream));
  return launch_decode_attn(a, reinterpret_cast<cudaStream_t>(stream)) == cudaSuccess ? LUCID_OK : LUCID_ERR_LAUNCH;
}

int lucid_decode_step_fused(int Hq, int Hkv, int Ln) {
  return Hkv > 0 && Hq > 0 && Hq % Hkv == 0 && decode_step_fused(Hq / Hkv, Ln) ? 1 : 0;
}

size_t lucid_decode_step_workspace_bytes(int B, int Hq, int Hkv, int Ln, int Nc, int D) {
  (void)D;
  if (Hkv <= 0) return 256;
  const size_t rows = (size_t)decode_splits(B, Hkv, Nc) * B * Hkv;
  return rows * ((size_t)Ln * 128 + (size_t)(Hq / Hkv) * Ln * 130) * sizeof(float) + 256;
}

int lucid_decode_step(int B, int Hq, int Hkv, int Ln, int Nc, int D, float scale, float eps,
                      const void* q, int64_t q_sb, int64_t q_sh, int64_t q_sn,
                      const void* k_new, int64_t kn_sb, int64_t kn_sh, int64_t kn_sn,
                      const void* v_new, int64_t vn_sb, int64_t vn_sh, int64_t vn_sn,
                      const void* k_cache, int64_t kc_sb, int64_t kc_sh, int64_t kc_sn,
                      const void* x_cache, int64_t xc_sb, int64_t xc_sh, int64_t xc_sn,
                      void* x_new, int64_t xn_sb, int64_t xn_sh, int64_t xn_sn,
                      void* o, int64_t o_sb, int64_t o_sh, int64_t o_sn,
                      void* workspace, size_t workspace_bytes, void* stream) {
  if (B < 0 || Hq < 0 || Hkv <= 0 || Ln < 0 || Nc < 0 || D < 4 || D > kHeadDim || D % 4 || Hq % Hkv != 0 ||
      (long long)B * Hkv > 65535)
    return LUCID_ERR_SHAPE;
  if (B == 0 || Hq == 0 || Ln == 0) return LUCID_OK;
  if (!decode_step_fused(Hq / Hkv, Ln)) return LUCID_ERR_SHAPE;
  if (!a8(q) || !a8(k_new) || !a8(k_cache) || !a8(x_cache) || !s4(q_sb, q_sh, q_sn) ||
      !s4(kn_sb, kn_sh, kn_sn) || !s4(kc_sb, kc_sh, kc_sn) || !s4(xc_sb, xc_sh, xc_sn))
    return LUCID_ERR_ALIGN;
  if (workspace == nullptr || workspace_bytes < lucid_decode_step_workspace_bytes(B, Hq, Hkv, Ln, Nc, D) ||
      !a16(workspace))
    return LUCID_ERR_WORKSPACE;
  float* part = reinterpret_cast<float*>(static_cast<char*>(workspace) + 256);
  const size_t rows = (size_t)decode_splits(B, Hkv, Nc) * B * Hkv;
  DecodeStepArgs a{B, Hkv, Hq, Ln, Nc, D, 0, 0, scale, eps,
                   static_cast<const bf16*>(q), q_sb, q_sh, q_sn,
                   static_cast<const bf16*>(k_new), kn_sb, kn_sh, kn_sn,
                   static_cast<const bf16*>(v_new), vn_sb, vn_sh, vn_sn,
                   static_cast<const bf16*>(k_cache), kc_sb, kc_sh, kc_sn,
                   static_cast<const bf16*>(x_cache), xc_sb, xc_sh, xc_sn,
                   static_cast<bf16*>(x_new), xn_sb, xn_sh, xn_sn,
                   static_cast<bf16*>(o), o_sb, o_sh, o_sn,
                   part, part + rows * Ln * 128};
  ProfileScope ps(LUCID_KERNEL_DECODE, reinterpret_cast<cudaStream_t>(stream));
  return launch_decode_step(a, reinterpret_cast<cudaStream_t>(stream)) == cudaSuccess ? LUCID_OK : LUCID_ERR_LAUNCH;
}

}  // extern "C"
