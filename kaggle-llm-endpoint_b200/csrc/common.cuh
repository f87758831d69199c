// Shared device helpers for the cbmoe kernels (sm_100a): status codes, bounded mbarrier waits, bulk copies,
// byte permutes and the bf16 tensor-core MMA used by the decode kernels.
#pragma once
#include <cstdint>
#include <mutex>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include "cbmoe.h"

namespace cbmoe {

// Device-side error word. Kernels OR a CBMOE_DEVERR_* bit into it instead of trapping; the host reads it with
// cbmoe_device_errors(). It is an error flag, not scratch: kernels never read it back.
extern __device__ int g_device_errors;

constexpr unsigned long long kWaitLimitNs = 4000000000ull;   // 4 s: every spin-wait gives up after this

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait until the phase with the given parity has completed. Returns false (and records CBMOE_DEVERR_TIMEOUT) if
// that takes longer than kWaitLimitNs; callers then stop issuing work and return.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++spins & 255u) == 0 && globaltimer_ns() - t0 > limit_ns) {
      atomicOr(&g_device_errors, CBMOE_DEVERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

// The same wait for a warp that is usually early (a producer waiting for consumers to free a stage): it sleeps
// between polls, so its spinning does not take issue slots from the consumer warps of the same scheduler.
__device__ __forceinline__ bool mbar_wait_sleepy(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  uint32_t ns = 32;
  while (!mbar_try_wait(bar, parity)) {
    __nanosleep(ns);
    if (ns < 256) ns <<= 1;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      atomicOr(&g_device_errors, CBMOE_DEVERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

// One contiguous global -> shared bulk copy completing on `bar` (addresses 16-byte aligned, size % 16 == 0).
// No multicast: the destination is this CTA's own shared memory.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// The MMA wrappers below are plain (not volatile) asm: pure functions of their register operands, so the compiler
// may schedule the next chunk's loads and table lookups around them. Shared-memory loads are ordinary C++ loads,
// which stay after the mbarrier waits (asm with a "memory" clobber) that make the data visible.

// D += A(16x16 bf16, row) * B(16x8 bf16, col), f32 accumulate.
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// D += A(16x32 int8, row) * B(32x8 int8, col), exact int32 accumulation: A signed (s8) or unsigned (u8), B s8.
template <bool kAUnsigned>
__device__ __forceinline__ void mma_i8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (kAUnsigned)
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 16-byte shared-memory load (p 16-byte aligned).
__device__ __forceinline__ uint4 lds128(const void* p) { return *reinterpret_cast<const uint4*>(p); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + __expf(-v)); }

// model.py:119-122: silu(min(g, L)) * clip(u, -L, L)
__device__ __forceinline__ float swiglu_clamped(float g, float u, float limit) {
  g = fminf(g, limit);
  u = fminf(fmaxf(u, -limit), limit);
  return silu_f(g) * u;
}

}  // namespace cbmoe

#define CBMOE_CUDA_TRY(expr)                          \
  do {                                                \
    cudaError_t e_ = (expr);                          \
    if (e_ != cudaSuccess) {                          \
      cbmoe::set_last_cuda_error(e_);                 \
      return CBMOE_ERR_CUDA;                          \
    }                                                 \
  } while (0)

namespace cbmoe {
void set_last_cuda_error(cudaError_t e);
int num_sms();

// Programmatic dependent launch: a kernel launched this way may start (launch, CTA placement, shared-memory set-up)
// while its predecessor on the stream is finishing; griddep_wait() then blocks until the predecessor has completed
// and its writes are visible, so every kernel of this library calls it before its first global-memory access.
// (In a kernel launched without the attribute it returns at once.) griddep_launch() lets the successor start being
// placed. CBMOE_PDL=0 in the environment launches everything plainly (a measurement switch).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
bool pdl_enabled();
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// One-time set-up per device (a kernel's shared-memory attribute, its resident grid): `init(value)` runs once for
// each device, with that device current, under a lock; on success (CBMOE_OK) the value it set is kept for that
// device. Kernel attributes are per device, so a process that drives several GPUs sets them on each.
struct PerDevice {
  std::mutex mu;
  long long val[64] = {};
  bool done[64] = {};
};
template <typename F>
int per_device(PerDevice& pd, F&& init, long long* out) {
  int dev = 0;
  CBMOE_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return CBMOE_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lk(pd.mu);
  if (!pd.done[dev]) {
    long long v = 0;
    const int rc = init(v);
    if (rc) return rc;
    pd.val[dev] = v;
    pd.done[dev] = true;
  }
  *out = pd.val[dev];
  return CBMOE_OK;
}
}  // namespace cbmoe
