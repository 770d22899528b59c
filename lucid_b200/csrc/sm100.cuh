// Blackwell (sm_100a) building blocks written as inline PTX: mbarriers with
// bounded waits, TMA tile loads, tcgen05 MMA / TMEM access, UMMA descriptors,
// and the 128B-swizzled shared-memory tile layout every kernel in this
// library uses.
//
// One tile format serves every GEMM operand: a [128 rows x 128 cols] bf16
// tile is stored as two 128B-swizzled "boxes" of [128 rows x 64 cols]
// (16 KB each, 1024-byte aligned).  The same bytes can be handed to the
// tensor core
//   * as a K-major operand whose rows are the M (or N) dimension and whose
//     columns are the K dimension, or
//   * as an MN-major operand whose rows are the K dimension and whose
//     columns are the M (or N) dimension,
// so a tile produced once (by TMA or by an epilogue) is reused transposed
// without any data movement.
#pragma once
#include <cstdint>
#include <utility>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

namespace lb {

// ---------------------------------------------------------------------------
// Status codes written to the per-launch status word.
// ---------------------------------------------------------------------------
// bits 0-7: code; bits 8-19: shared-memory offset of the barrier / 8 (mbarrier
// timeouts); bits 20-27: kernel tag.
enum : int {
  kStatusOk = 0,
  kStatusTimeoutMbar = 1,   // an mbarrier wait exceeded its time limit
  kStatusTimeoutFlag = 2,   // a cross-CTA dependency flag never arrived
  kStatusMisaligned = 3,    // dynamic shared memory window not 1024-byte aligned
};
// kernel tags
enum : int { kTagFwdSolve = 1, kTagFwdAttn = 2, kTagBwdColAttn = 3, kTagBwdColSolve = 4,
             kTagBwdRowAttn = 5, kTagBwdRowSolve = 6, kTagSelftest = 7, kTagBwdRowStored = 15 };

// Wall-clock bound for any spin wait inside a kernel.  A correct launch never
// comes close (the longest legitimate wait is one work item, milliseconds);
// the bound only keeps a broken launch from hanging the GPU.
constexpr uint64_t kWaitLimitNs = 2000ull * 1000ull * 1000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }

// Re-balance registers between warpgroups (all threads of a warpgroup execute it).
template <int N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
__device__ __forceinline__ int warp_id() { return threadIdx.x >> 5; }

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Per-CTA abort word (shared memory) plus the launch's global status word.
struct Abort {
  volatile int* cta;   // shared
  int* status;         // global
  int tag = 0;         // kernel tag recorded with a failure
};

__device__ __forceinline__ void raise_abort(const Abort& ab, int code, uint32_t where = 0) {
  *ab.cta = 1;
  atomicCAS(ab.status, 0, code | (int)((where & 0xFFFu) << 8) | (ab.tag << 20));
}

// Wait for phase `parity` of `bar`.  Returns false if the wait timed out or
// another thread of the CTA has already aborted; the caller must then unwind.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const Abort& ab) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*ab.cta) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_abort(ab, kStatusTimeoutMbar, (bar & 0x7FFFu) >> 3);
      return false;
    }
  }
}

// Time-bounded wait that ignores the CTA abort word: used while unwinding,
// to let copies / MMAs already issued finish before shared memory or TMEM
// is released.
constexpr uint64_t kDrainNs = 100ull * 1000ull * 1000ull;  // 100 ms
__device__ __forceinline__ bool mbar_wait_timed(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
  return true;
}

// ---------------------------------------------------------------------------
// Global flags used for cross-CTA dependencies (wavefront solves).
// ---------------------------------------------------------------------------
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Spin until *flag >= want (one polling thread per CTA; the wavefronts' critical path
// runs through these waits, so they poll without sleeping).  Returns false on timeout /
// abort.
__device__ __forceinline__ bool wait_flag_geq(const int* flag, int want, const Abort& ab) {
  if (ld_acquire_gpu(flag) >= want) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (ld_acquire_gpu(flag) >= want) return true;
    if (*ab.cta) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_abort(ab, kStatusTimeoutFlag);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// TMA (no multicast anywhere in this library)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// 4-D tiled load: coordinates (c0 innermost element index, c1 row, c2, c3).
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* m, uint32_t bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}

// Plain (untiled) bulk copy global -> shared; addresses 16-byte aligned,
// size a multiple of 16 bytes.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
      : "memory");
}

// Bulk tensor reduce-add (fp32) of a shared-memory box into global memory,
// tracked by the issuing thread's bulk async-group.
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* m, uint32_t src, int c0, int c1) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(m)),
      "r"(src), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// wait until the shared-memory sources of all committed bulk groups were read
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// wait until all committed bulk groups completed (global writes included)
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// TMA tile store (two 64-column boxes) from a swizzled shared-memory tile,
// tracked by the issuing thread's bulk async-group.
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* m, uint32_t src, int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(m)),
      "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void tma_store_tile(const CUtensorMap* m, uint32_t src, int row0, int c2, int c3) {
  tma_store_4d(m, src, 0, row0, c2, c3);
  tma_store_4d(m, src + 16384, 64, row0, c2, c3);
}

// L2 policy for data streamed once (written or read a single time): evicted first,
// so that it does not push the reused tiles of the current head out of L2.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void tma_store_4d_hint(const CUtensorMap* m, uint32_t src, int c0, int c1, int c2, int c3,
                                                  uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3, %4, %5}], [%1], %6;" ::"l"(
          reinterpret_cast<uint64_t>(m)),
      "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "l"(pol)
      : "memory");
}
__device__ __forceinline__ void tma_store_tile_hint(const CUtensorMap* m, uint32_t src, int row0, int c2, int c3,
                                                    uint64_t pol) {
  tma_store_4d_hint(m, src, 0, row0, c2, c3, pol);
  tma_store_4d_hint(m, src + 16384, 64, row0, c2, c3, pol);
}
__device__ __forceinline__ void tma_load_4d_hint(uint32_t dst, const CUtensorMap* m, uint32_t bar, int c0, int c1,
                                                 int c2, int c3, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar), "l"(pol)
      : "memory");
}
__device__ __forceinline__ void tma_load_tile_hint(uint32_t dst, const CUtensorMap* m, uint32_t bar, int row0, int c2,
                                                   int c3, uint64_t pol) {
  tma_load_4d_hint(dst, m, bar, 0, row0, c2, c3, pol);
  tma_load_4d_hint(dst + 16384, m, bar, 64, row0, c2, c3, pol);
}

// Load one [128 x 128] bf16 tile (two 64-column boxes) whose rows start at
// `row0` of matrix (c2, c3).  Box k of the tile lands at dst + k*16 KB.
__device__ __forceinline__ void tma_load_tile(uint32_t dst, const CUtensorMap* m, uint32_t bar,
                                              int row0, int c2, int c3) {
  tma_load_4d(dst, m, bar, 0, row0, c2, c3);
  tma_load_4d(dst + 16384, m, bar, 64, row0, c2, c3);
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, commit, TMEM <-> register moves
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]  (kind::f16, bf16 in, fp32 accum)
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]: A is M x K bf16 packed two per 32-bit
// TMEM column (element 2c in the low half of column c), lanes = rows.
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every tcgen05.mma issued so far by this thread is done.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

// 32 lanes x 32 columns of 32-bit: thread t of the warp receives columns
// [col, col+32) of TMEM lane (warp's lane base + t).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}
// 32 lanes x 16 columns store (packed bf16 pairs as 32-bit words).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------
// UMMA descriptors
// ---------------------------------------------------------------------------
// Shared-memory matrix descriptor, SWIZZLE_128B, sm_100 version field = 1.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;  // descriptor version (Blackwell)
  d |= (uint64_t)2u << 61;  // SWIZZLE_128B
  return d;
}

// Descriptor of the kk-th K=16 slice of a tile used as a K-major operand
// (tile rows = M/N dimension, tile columns = K dimension).
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t tile, int kk) {
  const uint32_t a = tile + (uint32_t)(kk >> 2) * 16384u + (uint32_t)(kk & 3) * 32u;
  return sdesc_sw128(a, 16, 1024);
}
// Descriptor of the kk-th K=16 slice of a tile used as an MN-major operand
// (tile rows = K dimension, tile columns = M/N dimension).
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t tile, int kk) {
  const uint32_t a = tile + (uint32_t)kk * 2048u;
  return sdesc_sw128(a, 16384, 1024);
}

// Instruction descriptor: bf16 x bf16 -> fp32, M x N, operand majorness.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4)                    // D format: f32
         | (1u << 7)                  // A format: bf16
         | (1u << 10)                 // B format: bf16
         | ((a_mn ? 1u : 0u) << 15)   // A major
         | ((b_mn ? 1u : 0u) << 16)   // B major
         | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Descriptor of K-slice kk from the slice-0 descriptor of the same tile: only the
// start-address field (bits 0-13, byte address >> 4) moves, by the slice's byte offset
// >> 4.  Tiles are 1024-byte aligned and shared memory ends below 256 KB, so the field
// never carries into the next one.  One add per slice keeps the single MMA-issuing
// thread's instruction count low (it shares its scheduler with epilogue warps).
__device__ __forceinline__ uint64_t desc_slice(uint64_t d0, bool mn, int kk) {
  return d0 + (uint64_t)(mn ? kk * 128 : (kk >> 2) * 1024 + (kk & 3) * 2);
}
__device__ __forceinline__ uint64_t desc_tile(uint32_t tile, bool mn) {
  return mn ? desc_mnmajor(tile, 0) : desc_kmajor(tile, 0);
}

// Issue the 8 K-slices of a 128x128x128 product.
__device__ __forceinline__ void umma_tile(uint32_t d_tmem, uint32_t a_tile, bool a_mn,
                                          uint32_t b_tile, bool b_mn, uint32_t accumulate_first) {
  const uint32_t idesc = idesc_bf16(128, 128, a_mn, b_mn);
  const uint64_t a0 = desc_tile(a_tile, a_mn), b0 = desc_tile(b_tile, b_mn);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
    umma_ss(d_tmem, desc_slice(a0, a_mn, kk), desc_slice(b0, b_mn, kk), idesc, (kk > 0) ? 1u : accumulate_first);
}

// The first nks K-slices (16 each) of a 128 x n product of two 128 x 128 tiles, n a
// multiple of 16 up to 128: the product of operands whose columns from 16 nks (K) and
// rows from n (B's N) on are zero, e.g. a head dimension below 128 zero-padded.
__device__ __forceinline__ void umma_tile_part(uint32_t d_tmem, uint32_t a_tile, bool a_mn, uint32_t b_tile,
                                               bool b_mn, uint32_t accumulate_first, int nks, int n) {
  const uint32_t idesc = idesc_bf16(128, n, a_mn, b_mn);
  const uint64_t a0 = desc_tile(a_tile, a_mn), b0 = desc_tile(b_tile, b_mn);
  for (int kk = 0; kk < nks; ++kk)
    umma_ss(d_tmem, desc_slice(a0, a_mn, kk), desc_slice(b0, b_mn, kk), idesc, (kk > 0) ? 1u : accumulate_first);
}

// The 8 K-slices of a 128x128x128 product whose A operand lives in TMEM (n < 128:
// only the first n columns of B and of the product).
// a_tmem(kk) gives the TMEM address of K-slice kk (8 columns of packed bf16).
template <typename AddrFn>
__device__ __forceinline__ void umma_tile_ts(uint32_t d_tmem, AddrFn a_tmem, uint32_t b_tile, bool b_mn,
                                             uint32_t accumulate_first, int n = 128) {
  const uint32_t idesc = idesc_bf16(128, n, false, b_mn);
  const uint64_t b0 = desc_tile(b_tile, b_mn);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
    umma_ts(d_tmem, a_tmem(kk), desc_slice(b0, b_mn, kk), idesc, (kk > 0) ? 1u : accumulate_first);
}

// ---------------------------------------------------------------------------
// Swizzled tile writes from registers (one thread owns one tile row)
// ---------------------------------------------------------------------------
// Byte offset of the 16-byte chunk `c16` (0..15, 8 bf16 each) of row `r`.
__device__ __forceinline__ uint32_t tile_chunk_off(int r, int c16) {
  const int box = c16 >> 3, c = c16 & 7;
  return (uint32_t)box * 16384u + (uint32_t)r * 128u + (uint32_t)((c ^ (r & 7)) << 4);
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

// Write 32 fp32 values (tile columns [32*q, 32*q+32) of row r) as bf16.
__device__ __forceinline__ void tile_store_row32(uint32_t tile, int r, int q, const float (&v)[32]) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int c16 = q * 4 + c;
    st_shared_v4(tile + tile_chunk_off(r, c16), pack_bf16(v[8 * c + 0], v[8 * c + 1]),
                 pack_bf16(v[8 * c + 2], v[8 * c + 3]), pack_bf16(v[8 * c + 4], v[8 * c + 5]),
                 pack_bf16(v[8 * c + 6], v[8 * c + 7]));
  }
}

// Fire-and-forget fp32 vector reduction into global memory (no return value,
// so the issuing thread never waits for the L2 round trip).
__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// Packed fp32 pair arithmetic (sm_100 f32x2 instructions).
union F2 {
  float2 f;
  unsigned long long u;
};
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  F2 x{a}, y{b}, z{c}, d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d.u) : "l"(x.u), "l"(y.u), "l"(z.u));
  return d.f;
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  F2 x{a}, y{b}, d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d.u) : "l"(x.u), "l"(y.u));
  return d.f;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  F2 x{a}, y{b}, d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d.u) : "l"(x.u), "l"(y.u));
  return d.f;
}

// Write 16 packed bf16 pairs (tile columns [32*q, 32*q+32) of row r).
__device__ __forceinline__ void tile_store_row32_packed(uint32_t tile, int r, int q, const uint32_t (&pk)[16]) {
#pragma unroll
  for (int c = 0; c < 4; ++c)
    st_shared_v4(tile + tile_chunk_off(r, q * 4 + c), pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
}

// max of three floats in one instruction (sm_100)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x for a pair, evaluated on the FMA pipe instead of the MUFU unit, so that an
// epilogue can split its exponentials between the two pipes.  x = n + f with
// n = round(x) (adding 1.5 * 2^23 leaves round(x) in the low mantissa bits) and
// f in [-1/2, 1/2]; 2^f is a polynomial of degree DEG whose coefficients minimise the
// maximum relative error on that interval (fitted by Lawson-weighted least squares on
// 4001 Chebyshev nodes; DEG 3: 7.5e-5, DEG 4: 2.7e-6, DEG 5: 2.3e-7 in fp32, against
// 1.2e-7 for MUFU ex2.approx); 2^n enters the exponent field by one integer add.
// x is clamped below at -126 (results >= 2^-126.5 instead of 0 there), above at 126.
template <int DEG>
__device__ __forceinline__ float2 exp2_fma2(float2 x) {
  static_assert(DEG >= 3 && DEG <= 5, "polynomial degree 3, 4 or 5");
  constexpr float C3[4] = {0.9999280571937561f, 0.6932609677314758f, 0.2426111400127411f, 0.0551716685295105f};
  constexpr float C4[5] = {0.9999992847442627f, 0.6931217908859253f, 0.240247443318367f, 0.05591786280274391f,
                           0.009570101276040077f};
  constexpr float C5[6] = {1.0000001192092896f, 0.6931469440460205f, 0.24022120237350464f, 0.05550713092088699f,
                           0.009675541892647743f, 0.001327647129073739f};
  const float* C = DEG == 3 ? C3 : (DEG == 4 ? C4 : C5);
  x.x = fminf(fmaxf(x.x, -126.f), 126.f);
  x.y = fminf(fmaxf(x.y, -126.f), 126.f);
  const float kShift = 12582912.f;  // 1.5 * 2^23
  const float2 t = add2(x, make_float2(kShift, kShift));
  const float2 n = add2(t, make_float2(-kShift, -kShift));
  const float2 f = fma2(n, make_float2(-1.f, -1.f), x);
  float2 p = make_float2(C[DEG], C[DEG]);
#pragma unroll
  for (int k = DEG - 1; k >= 0; --k) p = fma2(p, f, make_float2(C[k], C[k]));
  return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}

// Ask L2 to fetch a global line early (no data returned, no register written).
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Load 8 bf16 (16 bytes) from global and widen to fp32.
__device__ __forceinline__ void ld_bf16x8(const __nv_bfloat16* p, float* out) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    out[2 * i] = f.x;
    out[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void st_bf16x8(__nv_bfloat16* p, const float* in) {
  uint4 u;
  u.x = pack_bf16(in[0], in[1]);
  u.y = pack_bf16(in[2], in[3]);
  u.z = pack_bf16(in[4], in[5]);
  u.w = pack_bf16(in[6], in[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

// Host: launch `kernel` as a cooperative grid, for the wavefront kernels whose CTAs
// wait on flags other CTAs of the same grid publish.  A cooperative launch either
// places every CTA of the grid on the GPU at once or fails with an error
// (cudaErrorCooperativeLaunchTooLarge), so a CTA never waits on a CTA that cannot
// start while it occupies an SM (other streams or processes holding SMs included).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_cooperative(void (*kernel)(KArgs...), int grid, int threads, size_t smem, cudaStream_t st,
                                      Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3((unsigned)threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace lb
