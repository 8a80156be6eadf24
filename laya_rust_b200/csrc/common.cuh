// Device-side helpers shared by the sm_100a kernels: PTX wrappers for
// mbarriers, TMA tile loads and the tcgen05 (5th-generation tensor core)
// instructions, plus bounded waits.
//
// Every wait in these kernels is bounded: it polls with a wall-clock limit
// (%globaltimer), and on expiry records a code in the engine's device error
// word and reports failure so the kernel can unwind and return.  The host
// reads the error word after each forward and turns it into an error status.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

namespace laya {

// Error codes written to the device error word (first writer wins).
enum DeviceError : int {
  kErrNone = 0,
  kErrGemmProducerWait = 1,
  kErrGemmMmaWait = 2,
  kErrGemmEpilogueWait = 3,
  kErrGemmTeardownWait = 4,
  kErrAttnWait = 5,
};

// 2 s of wall clock: far above any legitimate wait in these kernels
// (microseconds), far below a watchdog.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that may suspend the thread in hardware for up to `hint_ns`
// (woken as soon as the phase completes), so a waiting warp issues no
// instructions while it waits instead of spinning on the barrier.
constexpr uint32_t kSuspendHintNs = 20000;
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete.  Returns false (and
// records `code` in *err) when the wall-clock limit passes (limit_ns, or
// kWaitLimitNs when 0) or when *abort (a shared-memory flag other roles
// raise on their own failure) is set.  Each try suspends the thread for at
// most kSuspendHintNs, so the limit and the abort flag are checked at least
// that often.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err,
                                                  int code, volatile int* abort_flag,
                                                  unsigned long long limit_ns = 0) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long limit = limit_ns ? limit_ns : kWaitLimitNs;
  const unsigned long long t0 = global_ns();
  for (;;) {
    if (mbar_try_wait_suspend(bar, parity)) return true;
    if (abort_flag && *abort_flag) return false;
    if (global_ns() - t0 > limit) {
      atomicCAS(err, 0, code);
      if (abort_flag) *abort_flag = 1;
      return false;
    }
  }
}

// ---- TMA ----------------------------------------------------------------
// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy reads (TMA stores, tcgen05.mma operands).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// 2-D tiled bulk-tensor load into this CTA's shared memory; completion is
// signalled on `bar` as transaction bytes.  x is the innermost coordinate.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* m, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// L2 eviction-priority policies for cache-hinted loads and stores.  Streams
// read once (GEMM A operands, attention's q/k/v tiles) are marked evict-first
// and the residual stream evict-last, so the residual stream stays in L2
// between the kernels that update and normalise it.
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// tma_load_2d with an L2 cache policy.
__device__ __forceinline__ void tma_load_2d_hint(void* smem_dst, const CUtensorMap* m, int x, int y,
                                                 uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// ---- tcgen05 ------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
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

// D[tmem] (+)= A[smem desc] x B[smem desc]^T, f16 inputs, f32 accumulate.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when every tcgen05.mma issued so far by this thread
// has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives
// lane (base_lane + i), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15,"
      " %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31},"
      " [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile written by TMA
// with 128-byte swizzle: rows of 64 f16 (128 B), 8-row atoms 1024 B apart.
// Fields: start address >> 4 [0,14), leading byte offset >> 4 [16,30) (unused
// for swizzled K-major, set to 1), stride byte offset >> 4 [32,46) = 1024 B,
// version 1 [46,48), layout type SWIZZLE_128B = 2 [61,64).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor for kind::f16: D = F32, A = B = F16, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int m, int n) {
  return (1u << 4)                                   // D format F32
         | (0u << 7) | (0u << 10)                    // A, B format F16
         | (0u << 15) | (0u << 16)                   // A, B K-major
         | (static_cast<uint32_t>(n >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);    // M / 16
}

// 2^x by the hardware's approximate exponential (one MUFU op).
__device__ __forceinline__ float exp2f_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// erf by Abramowitz & Stegun 7.1.26 (|error| <= 1.5e-7), the approximation
// the reference CPU backend uses (backend/cpu/mod.rs:59-74, there in f64):
//   erf(x) = 1 - t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) exp(-x^2),
//   t = 1 / (1 + p |x|), odd in x.
__device__ __forceinline__ float erf_as(float x) {
  const float ax = fabsf(x);
  const float t = __fdividef(1.0f, 1.0f + 0.3275911f * ax);
  const float poly =
      t * (0.254829592f + t * (-0.284496736f + t * (1.421413741f + t * (-1.453152027f + t * 1.061405429f))));
  return copysignf(1.0f - poly * __expf(-ax * ax), x);
}

__device__ __forceinline__ float gelu_erf(float v) {
  // exact-erf GELU (cpu/mod.rs:76-78): 0.5 v (1 + erf(v / sqrt 2))
  return 0.5f * v * (1.0f + erf_as(v * 0.70710678118654752f));
}

// ---- packed f32 pairs (sm_100 f32x2 arithmetic: two lanes per instruction, each
// rounded as the scalar f32 operation) --------------------------------------------
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_get(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_splat(float v) { return f2(v, v); }

// max(a, b, c) as one sm_100 three-input max (the same value as two fmaxf).
__device__ __forceinline__ float fmax3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// (gelu_erf(v0), gelu_erf(v1)) in packed pairs: the same A&S 7.1.26 formula,
// with the polynomial's coefficients negated so that erf(|x|) = 1 + p e is
// one fused step.  The divide and the exponential stay per lane (MUFU).
__device__ __forceinline__ uint64_t gelu_erf2(uint64_t v) {
  const uint64_t x = f2_mul(v, f2_splat(0.70710678118654752f));
  float x0, x1;
  f2_get(x, x0, x1);
  const uint64_t ax = f2(fabsf(x0), fabsf(x1));
  float d0, d1;
  f2_get(f2_fma(ax, f2_splat(0.3275911f), f2_splat(1.0f)), d0, d1);
  const uint64_t t = f2(__fdividef(1.0f, d0), __fdividef(1.0f, d1));
  uint64_t p = f2_fma(t, f2_splat(-1.061405429f), f2_splat(1.453152027f));
  p = f2_fma(t, p, f2_splat(-1.421413741f));
  p = f2_fma(t, p, f2_splat(0.284496736f));
  p = f2_fma(t, p, f2_splat(-0.254829592f));
  p = f2_mul(t, p);  // -t (a1 + t (a2 + t (a3 + t (a4 + t a5))))
  float e0, e1;
  f2_get(f2_mul(f2_mul(ax, ax), f2_splat(-1.4426950408889634f)), e0, e1);
  float r0, r1;
  f2_get(f2_fma(p, f2(exp2f_approx(e0), exp2f_approx(e1)), f2_splat(1.0f)), r0, r1);
  const uint64_t erf = f2(copysignf(r0, x0), copysignf(r1, x1));
  const uint64_t h = f2_mul(v, f2_splat(0.5f));
  return f2_fma(h, erf, h);
}

// ---- programmatic dependent launch ---------------------------------------------------
// Every kernel is launched with programmatic stream serialization allowed, so
// it may start while the kernel before it in the stream is still running.
// Each kernel therefore calls grid_dep_wait() before its first access to
// memory that a previous kernel writes or reads (everything except weights,
// tensor maps and its own shared memory) -- the wait returns once the previous
// grid has completed and its writes are visible, which by induction orders it
// after every earlier kernel too -- and grid_dep_trigger() right after, which
// lets the next kernel be scheduled into SM slots as they free up and run its
// own prologue.  Without a programmatic predecessor the wait returns at once.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Host: whether launches carry the programmatic-serialization attribute
// (LAYA_PDL=0 turns it off for the whole process).
bool pdl_enabled();

// cudaLaunchKernelEx with the programmatic-serialization attribute (when
// enabled) and optional extra attributes.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       const cudaLaunchAttribute* extra, int n_extra, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[4];
  int n = 0;
  for (int i = 0; i < n_extra && n < 3; ++i) attr[n++] = extra[i];
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace laya
