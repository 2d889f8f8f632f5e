// diag.cu -- self-test of the bounded device wait.
//
// Every wait of the tcgen05 kernels (on an mbarrier that TMA, a tensor-core commit or another
// warp completes) gives up after a time limit, records a site code in the context's timeout
// flag and lets the kernel run to its end, so a lost arrival surfaces as TURT_ERR_TIMEOUT at
// the next synchronization instead of a hung GPU.  turt_wait_selftest exercises exactly that
// path: one thread waits on a shared-memory mbarrier that nothing ever arrives on, with a
// caller-chosen limit; the wait expires, the flag is raised and the kernel returns.
#include "../../include/turt_cuda.h"
#include "ctx.cuh"

namespace turt {
namespace {

constexpr int kSelftestSite = 900;

__global__ void k_wait_selftest(uint64_t limit_ns, int* flags) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  // The same loop as mbar_wait, with the limit as an argument: try_wait on phase 0, which
  // completes only if one thread arrives -- none does.
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(&bar, 0)) {
    if (global_timer_ns() - t0 > limit_ns) {
      atomicExch(&flags[FLAG_TIMEOUT], kSelftestSite);
      break;
    }
  }
  asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_u32(&bar)) : "memory");
}

}  // namespace
}  // namespace turt

using namespace turt;

extern "C" int turt_wait_selftest(turt_ctx* ctx, int limit_us) {
  if (!ctx) {
    set_error("null context");
    return ERR_INVALID;
  }
  TURT_REQUIRE(limit_us >= 1 && limit_us <= 1000000, "turt_wait_selftest: limit_us must be in [1, 1000000]");
  TURT_CHECK_CUDA(cudaSetDevice(ctx->device));
  k_wait_selftest<<<1, 32, 0, ctx->stream>>>((uint64_t)limit_us * 1000ull, ctx->flags);
  TURT_LAUNCH_CHECK();
  return ctx_check_flags(ctx);  // synchronizes; TURT_ERR_TIMEOUT with the site in the message
}
