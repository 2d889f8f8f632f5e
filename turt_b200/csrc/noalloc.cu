// noalloc.cu -- host-array matmul that performs no device allocation.
//
// turt_host_matmul copies the caller's host arrays into device memory it allocates per
// call, runs the tensor-core GEMM and copies the product back.  Some callers cannot let
// the library allocate device memory at call time: a process whose device memory is
// already reserved by another framework's caching allocator (a fresh cudaMalloc then fails
// or fragments the pool), or a latency-bound host that must not allocate after start-up
// (cudaMalloc can synchronize the device and its latency is unbounded).  For them,
// turt_host_matmul_noalloc stages A, B and C in one fixed, file-scope device array instead.
//
// The array is kNoAllocScratchFloats floats (8 MiB).  Each .cu file of the library is its
// own CUDA module, and under CUDA's default lazy module loading a module's device memory is
// reserved when the module is first used, not when the library is loaded.  So turt_init
// looks the array's address up for its device (noalloc_setup): from then on the device holds
// the array until the process exits, and no turt_host_matmul_noalloc call is the one that
// reserves it.  All calls share it and it keeps the last call's contents; each call
// overwrites every element it reads, so nothing needs clearing.  Calls that overlap on the
// GPU (from several host threads or streams) race on it.
#include <mutex>

#include "../../include/turt_cuda.h"
#include "ctx.cuh"
#include "gemm.cuh"

namespace turt {
namespace {

constexpr size_t kNoAllocScratchFloats = (size_t)2 << 20;  // 2 Mi floats = 8 MiB

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
float* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array for the current device (looked up once per device,
// with that device current: in host code the symbol itself is only a host-side stand-in).
int scratch_for_device(int dev, float** out) {
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("turt_host_matmul_noalloc: device index out of range");
    return ERR_INVALID;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    TURT_CHECK_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return OK;
}

inline size_t round64(size_t x) { return (x + 63) & ~size_t(63); }

}  // namespace

// Called by turt_init with `dev` current: loads this file's module and records the array's
// device address, so the 8 MiB are reserved at context creation.
int noalloc_setup(int dev) {
  float* p = nullptr;
  return scratch_for_device(dev, &p);
}

}  // namespace turt

using namespace turt;

extern "C" int turt_host_matmul_noalloc(turt_ctx* ctx, const float* a, int m, int k, const float* b, int n,
                                        float* out) {
  if (!ctx) {
    set_error("null context");
    return ERR_INVALID;
  }
  TURT_CHECK_CUDA(cudaSetDevice(ctx->device));
  TURT_REQUIRE(a && b && out, "matmul: null array");
  TURT_REQUIRE(m >= 0 && k >= 0 && n >= 0, "matmul: negative dimension");
  if ((size_t)m * n == 0) return OK;
  // Same staging as turt_host_bmm: the tensor-core path pitches rows to a multiple of 4 floats
  // (TMA needs 16-byte pitches); the FP32 CUDA-core path keeps dense rows.
  const bool simt = ctx->precision == 0;
  const size_t kp = simt ? (size_t)k : ((size_t)k + 3) & ~size_t(3);
  const size_t np = simt ? (size_t)n : ((size_t)n + 3) & ~size_t(3);
  const size_t need = round64((size_t)m * kp) + round64((size_t)k * np) + round64((size_t)m * np);
  if (need > kNoAllocScratchFloats) {
    set_error("turt_host_matmul_noalloc: [" + std::to_string(m) + "x" + std::to_string(k) + "] @ [" +
              std::to_string(k) + "x" + std::to_string(n) + "] needs " + std::to_string(need) +
              " floats of staging; the fixed scratch holds " + std::to_string(kNoAllocScratchFloats) +
              " (use turt_host_matmul for larger products)");
    return ERR_INVALID;
  }
  float* base = nullptr;
  int rc = scratch_for_device(ctx->device, &base);
  if (rc) return rc;
  float* da = base;
  float* db = da + round64((size_t)m * kp);
  float* dc = db + round64((size_t)k * np);
  cudaStream_t st = ctx->stream;
  if (k == 0) {
    TURT_CHECK_CUDA(cudaMemsetAsync(dc, 0, (size_t)m * np * 4, st));
  } else {
    TURT_CHECK_CUDA(cudaMemcpy2DAsync(da, kp * 4, a, (size_t)k * 4, (size_t)k * 4, m, cudaMemcpyHostToDevice, st));
    TURT_CHECK_CUDA(cudaMemcpy2DAsync(db, np * 4, b, (size_t)n * 4, (size_t)n * 4, k, cudaMemcpyHostToDevice, st));
    if (simt) {
      rc = gemm_simt(st, da, db, dc, m, k, n, 1, false, false, false);
    } else {
      GemmOperand A{da, (long)kp, (long)(m * kp), false};
      GemmOperand B{db, (long)np, (long)(k * np), true};
      GemmEpi epi;
      epi.kind = EPI_STORE;
      epi.C = dc;
      epi.ldc = (long)np;
      epi.strideC = (long)(m * np);
      // one pass over K: a split would stage partial sums in a workspace allocated on demand
      rc = gemm_tf32(st, m, n, k, 1, A, B, epi, ctx->flags, ctx->precision, /*force_splits=*/1);
    }
    if (rc) return rc;
  }
  TURT_CHECK_CUDA(cudaMemcpy2DAsync(out, (size_t)n * 4, dc, np * 4, (size_t)n * 4, m, cudaMemcpyDeviceToHost, st));
  TURT_CHECK_CUDA(cudaStreamSynchronize(st));
  return ctx_check_flags(ctx);
}
