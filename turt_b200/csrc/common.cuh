// common.cuh -- shared device/host helpers for libturt_cuda (sm_100a only).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <atomic>
#include <string>

#ifndef __CUDA_ARCH__
#define TURT_HOST_ONLY 1
#endif

namespace turt {

// ----------------------------------------------------------------- errors
// Status codes of the C ABI (include/turt_cuda.h).
enum Status : int {
  OK = 0,
  ERR_INVALID = 1,      // bad argument / shape mismatch (the reference throws Error)
  ERR_CUDA = 2,         // CUDA runtime failure
  ERR_RANGE = 3,        // token / target id out of range (reported by a device flag)
  ERR_TIMEOUT = 4,      // a bounded device wait gave up
  ERR_NCCL = 5,         // collective failure / abort
  ERR_NONFINITE = 6,    // non-finite loss or gradient norm
  ERR_UNSUPPORTED = 7,  // layout the kernels do not handle
};

void set_error(const std::string& msg);
const char* last_error();
// Process-wide count of kernel launches issued by this library (turt_launch_count).
void note_launch(int n = 1);

#define TURT_LAUNCH_CHECK()     \
  do {                          \
    turt::note_launch();        \
    TURT_CHECK_CUDA(cudaGetLastError()); \
  } while (0)

#define TURT_CHECK_CUDA(expr)                                                   \
  do {                                                                          \
    cudaError_t e__ = (expr);                                                   \
    if (e__ != cudaSuccess) {                                                   \
      turt::set_error(std::string(#expr) + ": " + cudaGetErrorString(e__));     \
      return turt::ERR_CUDA;                                                    \
    }                                                                           \
  } while (0)

// Propagates a non-zero status code.
#define RC(x)              \
  do {                     \
    int rc__ = (x);        \
    if (rc__) return rc__; \
  } while (0)

// Raises a kernel's dynamic shared-memory limit on the current device, once per device.
// Function attributes belong to each device's context, so a kernel launched from several
// device worker threads must be configured on every device; `done` is that kernel's own bit
// set of configured devices (a racing second set on the same device is harmless).
template <typename K>
int smem_attr_per_device(std::atomic<uint64_t>& done, K kfn, int bytes) {
  int dev = 0;
  TURT_CHECK_CUDA(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return OK;
  TURT_CHECK_CUDA(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  done.fetch_or(bit, std::memory_order_acq_rel);
  return OK;
}

#define TURT_REQUIRE(cond, msg)             \
  do {                                      \
    if (!(cond)) {                          \
      turt::set_error(std::string(msg));    \
      return turt::ERR_INVALID;             \
    }                                       \
  } while (0)

// Device-side error flags (one int array per context, see DeviceFlags).
enum FlagIndex : int {
  FLAG_RANGE = 0,    // bad token / target id seen
  FLAG_TIMEOUT = 1,  // bounded wait expired (value = site code)
  FLAG_NONFINITE = 2,
  FLAG_COUNT = 4,
};

// ------------------------------------------------------------- device utils
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Every spin-wait in this library gives up after this long and raises FLAG_TIMEOUT.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
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

// Bounded wait: returns false (and raises the timeout flag with `site`) after kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* flags, int site) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      if (flags) atomicExch(&flags[FLAG_TIMEOUT], site);
      return false;
    }
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// GELU tanh approximation and SiLU, the formulas of src/math/tensor.ts:607-635.
__device__ __forceinline__ float gelu_f(float x) {
  const float c = 0.7978845608028654f;
  return 0.5f * x * (1.0f + tanhf(c * (x + 0.044715f * x * x * x)));
}
__device__ __forceinline__ float gelu_grad_f(float x) {
  const float c = 0.7978845608028654f;
  float inner = c * (x + 0.044715f * x * x * x);
  float t = tanhf(inner);
  float dinner = c * (1.0f + 3.0f * 0.044715f * x * x);
  return 0.5f * (1.0f + t) + 0.5f * x * (1.0f - t * t) * dinner;
}
__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }

inline int ceil_div(long a, long b) { return (int)((a + b - 1) / b); }

// ------------------------------------------------ programmatic dependent launch
// The train step is a chain of ~175 kernels on one stream.  Launched with launch_pdl, a kernel
// may be scheduled while its predecessor is still draining, so its launch and set-up (barrier
// init, TMEM allocation) overlap the predecessor's tail.  Such a kernel calls pdl_wait() before
// its first global memory access, read or write: it returns once the predecessor has completed
// and its writes are visible.  pdl_trigger() lets the successor be scheduled; a grid triggers
// once every one of its CTAs has triggered or exited, i.e. no earlier than its last wave, so
// waiting successors only take resources the predecessor no longer asks for.  In a kernel not
// launched with launch_pdl both are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

}  // namespace turt
