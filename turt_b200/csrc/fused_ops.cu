// fused_ops.cu -- the train step's fused memory-bound kernels on raw device buffers.
//
// The model path (model.cu) calls these kernels on its own workspace; the entry points here
// expose the same kernels standalone, for validation against the oracle and for the
// standalone backward-op measurement.  SwiGLU backward, which the model fuses into the
// epilogue of the dact GEMM, has its own elementwise kernel here.
#include "../../include/turt_cuda.h"
#include "ctx.cuh"
#include "model_kernels.cuh"

namespace turt {
namespace {

// SwiGLU backward over separate gate / up arrays (act = silu(a) * u):
//   s = sigmoid(a); dup = dact * a * s; dgate = dact * u * (s + a*s*(1 - s))
// (the SILU_BWD formula d = s + silu*(1-s), autograd.ts:1044-1054, times the product rule).
__global__ void __launch_bounds__(256) k_swiglu_bwd(const float4* __restrict__ a, const float4* __restrict__ u,
                                                    const float4* __restrict__ d, float4* __restrict__ da,
                                                    float4* __restrict__ du, size_t n4) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    const float4 x = a[i], y = u[i], g = d[i];
    float4 rg, ru;
#define SWB(c)                                \
  {                                           \
    const float s = sigmoid_f(x.c);           \
    const float sl = x.c * s;                 \
    ru.c = g.c * sl;                          \
    rg.c = g.c * y.c * (s + sl * (1.0f - s)); \
  }
    SWB(x) SWB(y) SWB(z) SWB(w)
#undef SWB
    da[i] = rg;
    du[i] = ru;
  }
}

__global__ void k_swiglu_bwd_tail(const float* a, const float* u, const float* d, float* da, float* du, size_t i0,
                                  size_t n) {
  const size_t i = i0 + threadIdx.x;
  if (i >= n) return;
  const float s = sigmoid_f(a[i]), sl = a[i] * s;
  du[i] = d[i] * sl;
  da[i] = d[i] * u[i] * (s + sl * (1.0f - s));
}

// One block per window; threads stride over its t positions.
__global__ void k_sample_windows(const uint16_t* __restrict__ tokens, size_t n_tokens, const uint64_t* __restrict__ starts,
                                 int t, uint32_t* __restrict__ ids, uint32_t* __restrict__ tgt, int* flags) {
  const int i = blockIdx.x;
  const uint64_t s = starts[i];
  if (s + (uint64_t)t + 1 > n_tokens) {
    if (threadIdx.x == 0) atomicExch(&flags[FLAG_RANGE], 1);
    return;
  }
  for (int j = threadIdx.x; j < t; j += blockDim.x) {
    ids[(size_t)i * t + j] = tokens[s + j];
    tgt[(size_t)i * t + j] = tokens[s + j + 1];
  }
}

int scratch(turt_ctx* ctx, size_t bytes, void** out) {
  if (ctx->scratch_bytes < bytes) {
    if (ctx->scratch) {
      TURT_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
      cudaFree(ctx->scratch);
      ctx->scratch = nullptr;
      ctx->scratch_bytes = 0;
    }
    TURT_CHECK_CUDA(cudaMalloc(&ctx->scratch, bytes));
    ctx->scratch_bytes = bytes;
  }
  *out = ctx->scratch;
  return OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace turt

using namespace turt;

#define FCTX(ctx)                        \
  do {                                   \
    if (!(ctx)) {                        \
      set_error("null context");         \
      return ERR_INVALID;                \
    }                                    \
    TURT_CHECK_CUDA(cudaSetDevice((ctx)->device)); \
  } while (0)

extern "C" int turt_fused_rms_bwd(turt_ctx* ctx, const float* x, const float* dy, const float* g, const float* rstd,
                                  const float* dres, float* dx, float* dg, int rows, int E) {
  FCTX(ctx);
  TURT_REQUIRE(x && dy && g && rstd && dx && dg && rows > 0, "fused_rms_bwd: null buffer or empty problem");
  TURT_REQUIRE(aligned16(x) && aligned16(dy) && aligned16(g) && aligned16(dx) && (!dres || aligned16(dres)),
               "fused_rms_bwd: buffers must be 16-byte aligned");
  void* part = nullptr;
  RC(scratch(ctx, (size_t)norm_parts(rows) * E * 4, &part));
  return rms_bwd(ctx->stream, x, dy, g, rstd, dres, dx, dg, static_cast<float*>(part), rows, E);
}

extern "C" int turt_fused_swiglu_bwd(turt_ctx* ctx, const float* gate, const float* up, const float* dact,
                                     float* dgate, float* dup, size_t n) {
  FCTX(ctx);
  TURT_REQUIRE(gate && up && dact && dgate && dup, "fused_swiglu_bwd: null buffer");
  TURT_REQUIRE(aligned16(gate) && aligned16(up) && aligned16(dact) && aligned16(dgate) && aligned16(dup),
               "fused_swiglu_bwd: buffers must be 16-byte aligned");
  const size_t n4 = n / 4;
  if (n4) {
    size_t blocks = (n4 + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    k_swiglu_bwd<<<(unsigned)blocks, 256, 0, ctx->stream>>>(
        reinterpret_cast<const float4*>(gate), reinterpret_cast<const float4*>(up),
        reinterpret_cast<const float4*>(dact), reinterpret_cast<float4*>(dgate), reinterpret_cast<float4*>(dup), n4);
    TURT_LAUNCH_CHECK();
  }
  if (n % 4) {
    k_swiglu_bwd_tail<<<1, 32, 0, ctx->stream>>>(gate, up, dact, dgate, dup, n4 * 4, n);
    TURT_LAUNCH_CHECK();
  }
  return OK;
}

extern "C" int turt_fused_ce(turt_ctx* ctx, float* logits, const uint32_t* targets, float* loss_rows, int N, int V,
                             float gscale) {
  FCTX(ctx);
  TURT_REQUIRE(logits && targets && loss_rows && N > 0 && V > 0, "fused_ce: null buffer or empty problem");
  TURT_REQUIRE(V % 4 == 0 && aligned16(logits), "fused_ce: rows must be 16-byte aligned (V % 4 == 0)");
  return ce_fused(ctx->stream, logits, targets, loss_rows, N, V, gscale, ctx->flags);
}

extern "C" int turt_fused_adamw_clip(turt_ctx* ctx, float* p, const float* g, float* m, float* v, size_t n, float lr,
                                     float b1, float b2, float eps, float wd, float bc1, float bc2, float clip,
                                     double* norm_out) {
  FCTX(ctx);
  TURT_REQUIRE(p && g && m && v && n > 0, "fused_adamw_clip: null buffer or empty problem");
  TURT_REQUIRE(aligned16(p) && aligned16(g) && aligned16(m) && aligned16(v),
               "fused_adamw_clip: buffers must be 16-byte aligned");
  const float* coef = nullptr;
  if (clip > 0 || norm_out) {
    // scratch: [norm partials (doubles)] [norm (double)] [coef (float)]
    const size_t nd = norm_scratch_doubles();
    void* s = nullptr;
    RC(scratch(ctx, (nd + 2) * sizeof(double) + 16, &s));
    double* part = static_cast<double*>(s);
    double* nrm = part + nd;
    float* cf = reinterpret_cast<float*>(nrm + 2);
    RC(grad_norm(ctx->stream, g, n, 1.0f, clip > 0 ? clip : 0.0f, part, nrm, cf, ctx->flags));
    if (clip > 0) coef = cf;
    if (norm_out) {
      TURT_CHECK_CUDA(cudaMemcpyAsync(norm_out, nrm, 8, cudaMemcpyDeviceToHost, ctx->stream));
      TURT_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
    }
  }
  return adamw_flat(ctx->stream, p, g, m, v, n, lr, b1, b2, eps, wd, bc1, bc2, 1.0f, coef);
}

extern "C" int turt_sample_windows(turt_ctx* ctx, const uint16_t* tokens, size_t n_tokens, const uint64_t* starts,
                                   int b, int t, uint32_t* ids, uint32_t* targets) {
  FCTX(ctx);
  TURT_REQUIRE(tokens && starts && ids && targets, "sample_windows: null buffer");
  TURT_REQUIRE(b > 0 && t > 0 && n_tokens > (size_t)t + 1, "sample_windows: corpus shorter than one window");
  void* d_starts = nullptr;
  RC(scratch(ctx, (size_t)b * 8, &d_starts));
  TURT_CHECK_CUDA(cudaMemcpyAsync(d_starts, starts, (size_t)b * 8, cudaMemcpyHostToDevice, ctx->stream));
  k_sample_windows<<<b, 256, 0, ctx->stream>>>(tokens, n_tokens, static_cast<const uint64_t*>(d_starts), t, ids,
                                                targets, ctx->flags);
  TURT_LAUNCH_CHECK();
  return OK;
}
