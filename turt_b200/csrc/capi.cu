// capi.cu -- extern "C" context, buffer and op-level entry points of libturt_cuda.so.
#include <atomic>
#include <mutex>
#include <string>
#include <unordered_set>
#include <vector>

#include "../../include/turt_cuda.h"
#include "ctx.cuh"
#include "gemm.cuh"
#include "ops.cuh"

namespace turt {

static thread_local std::string g_last_error;
static std::atomic<uint64_t> g_launches{0};
void note_launch(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }
void set_error(const std::string& msg) { g_last_error = msg; }
int noalloc_setup(int dev);  // noalloc.cu
const char* last_error() { return g_last_error.c_str(); }

int ctx_check_flags(turt_ctx* ctx) {
  int h[FLAG_COUNT] = {0};
  TURT_CHECK_CUDA(cudaMemcpyAsync(h, ctx->flags, sizeof(h), cudaMemcpyDeviceToHost, ctx->stream));
  TURT_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
  if (h[FLAG_RANGE] || h[FLAG_TIMEOUT] || h[FLAG_NONFINITE]) {
    TURT_CHECK_CUDA(cudaMemsetAsync(ctx->flags, 0, sizeof(int) * FLAG_COUNT, ctx->stream));
    TURT_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
    if (h[FLAG_TIMEOUT]) {
      set_error("a device wait timed out (site " + std::to_string(h[FLAG_TIMEOUT]) + ")");
      return ERR_TIMEOUT;
    }
    if (h[FLAG_RANGE]) {
      set_error("token or target id out of range [0, vocab)");
      return ERR_RANGE;
    }
    set_error("non-finite loss or gradient norm");
    return ERR_NONFINITE;
  }
  return OK;
}

}  // namespace turt

using namespace turt;

#define CTX_GUARD(ctx)                                   \
  do {                                                   \
    if (!(ctx)) {                                        \
      set_error("null context");                         \
      return ERR_INVALID;                                \
    }                                                    \
    TURT_CHECK_CUDA(cudaSetDevice((ctx)->device));       \
  } while (0)

extern "C" {

const char* turt_last_error(void) { return last_error(); }
int turt_version(void) { return 1; }

int turt_launch_count(uint64_t* count) {
  if (!count) return ERR_INVALID;
  *count = g_launches.load();
  return OK;
}

int turt_init(int device, turt_ctx** out) {
  if (!out) {
    set_error("turt_init: null out");
    return ERR_INVALID;
  }
  int n = 0;
  TURT_CHECK_CUDA(cudaGetDeviceCount(&n));
  if (device < 0 || device >= n) {
    set_error("turt_init: no CUDA device " + std::to_string(device));
    return ERR_INVALID;
  }
  TURT_CHECK_CUDA(cudaSetDevice(device));
  cudaDeviceProp prop;
  TURT_CHECK_CUDA(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10) {
    set_error("libturt_cuda is built for sm_100a (B200); device is sm_" + std::to_string(prop.major * 10 + prop.minor));
    return ERR_UNSUPPORTED;
  }
  turt_ctx* c = new turt_ctx();
  c->device = device;
  TURT_CHECK_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
  c->own_stream = true;
  TURT_CHECK_CUDA(cudaMalloc(&c->flags, sizeof(int) * FLAG_COUNT));
  TURT_CHECK_CUDA(cudaMemset(c->flags, 0, sizeof(int) * FLAG_COUNT));
  // Reserve turt_host_matmul_noalloc's fixed staging array now.  Best effort: a failure here
  // is reported again by that entry point's first call, and is no reason to refuse a context.
  if (noalloc_setup(device) != OK) (void)cudaGetLastError();
  *out = c;
  return OK;
}

int turt_ctx_destroy(turt_ctx* ctx) {
  CTX_GUARD(ctx);
  cudaStreamSynchronize(ctx->stream);
  for (void* p : ctx->pending_free) cudaFree(p);
  for (void* p : ctx->live_set) cudaFree(p);
  cudaFree(ctx->flags);
  if (ctx->scratch) cudaFree(ctx->scratch);
  gemm_release_stream(ctx->stream);
  if (ctx->own_stream) cudaStreamDestroy(ctx->stream);
  delete ctx;
  return OK;
}

int turt_ctx_set_stream(turt_ctx* ctx, void* stream) {
  CTX_GUARD(ctx);
  TURT_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
  gemm_release_stream(ctx->stream);
  if (ctx->own_stream) cudaStreamDestroy(ctx->stream);
  ctx->stream = reinterpret_cast<cudaStream_t>(stream);
  ctx->own_stream = false;
  return OK;
}

void* turt_ctx_stream(turt_ctx* ctx) { return ctx ? reinterpret_cast<void*>(ctx->stream) : nullptr; }

int turt_set_precision(turt_ctx* ctx, int precision) {
  CTX_GUARD(ctx);
  TURT_REQUIRE(precision == 0 || precision == GEMM_TF32 || precision == GEMM_TF32X3,
               "precision must be 0 (FP32), 1 (TF32) or 3 (3xTF32)");
  ctx->precision = precision;
  return OK;
}

int turt_get_precision(turt_ctx* ctx, int* precision) {
  CTX_GUARD(ctx);
  TURT_REQUIRE(precision, "null precision");
  *precision = ctx->precision;
  return OK;
}

int turt_gemm_set_tile(int bn, int pair) {
  TURT_REQUIRE(bn == 0 || bn == 64 || bn == 128 || bn == 192 || bn == 256, "tile width must be 0, 64, 128, 192 or 256");
  TURT_REQUIRE(pair >= -1 && pair <= 2,
               "kernel must be -1 (automatic), 0 (single CTA), 1 (CTA pair) or 2 (two single CTAs per SM)");
  gemm_set_tile_override(bn, pair);
  return OK;
}

int turt_synchronize(turt_ctx* ctx) {
  CTX_GUARD(ctx);
  TURT_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
  return ctx_check_flags(ctx);
}

// ------------------------------------------------------------------ buffers
int turt_buffer(turt_ctx* ctx, size_t elems, float** out) {
  CTX_GUARD(ctx);
  size_t bytes = (elems < 1 ? 1 : elems) * 4;
  void* p = nullptr;
  TURT_CHECK_CUDA(cudaMalloc(&p, bytes));
  TURT_CHECK_CUDA(cudaMemsetAsync(p, 0, bytes, ctx->stream));
  ctx->live_set.insert(p);
  ctx->live++;
  if (ctx->live > ctx->peak) ctx->peak = ctx->live;
  *out = static_cast<float*>(p);
  return OK;
}

int turt_index_buffer(turt_ctx* ctx, const uint32_t* host, size_t n, uint32_t** out) {
  float* p = nullptr;
  int rc = turt_buffer(ctx, n, &p);
  if (rc) return rc;
  if (n) TURT_CHECK_CUDA(cudaMemcpyAsync(p, host, n * 4, cudaMemcpyHostToDevice, ctx->stream));
  TURT_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
  *out = reinterpret_cast<uint32_t*>(p);
  return OK;
}

int turt_free(turt_ctx* ctx, void* p) {
  CTX_GUARD(ctx);
  if (!p) return OK;
  if (ctx->live_set.erase(p)) ctx->pending_free.push_back(p);
  return OK;
}

int turt_reclaim(turt_ctx* ctx) {
  CTX_GUARD(ctx);
  TURT_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
  for (void* p : ctx->pending_free) {
    cudaFree(p);
    ctx->live--;
  }
  ctx->pending_free.clear();
  return ctx_check_flags(ctx);
}

int turt_upload(turt_ctx* ctx, void* dst, const void* src, size_t bytes) {
  CTX_GUARD(ctx);
  if (!bytes) return OK;
  TURT_CHECK_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
  TURT_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
  return OK;
}

int turt_download(turt_ctx* ctx, void* dst, const void* src, size_t bytes) {
  CTX_GUARD(ctx);
  if (!bytes) return OK;
  TURT_CHECK_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  TURT_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
  return ctx_check_flags(ctx);
}

int turt_fill(turt_ctx* ctx, float* buf, float value, size_t elems) {
  CTX_GUARD(ctx);
  return op_fill(ctx->stream, buf, value, elems);
}

int turt_live_buffers(turt_ctx* ctx, int* live, int* peak) {
  if (!ctx) return ERR_INVALID;
  if (live) *live = ctx->live;
  if (peak) *peak = ctx->peak;
  return OK;
}

// ------------------------------------------------------------------ ops
int turt_matmul_into(turt_ctx* ctx, const float* a, const float* b, float* out, int M, int K, int N, int batch,
                     int transA, int transB, int accum) {
  CTX_GUARD(ctx);
  TURT_REQUIRE(M >= 0 && K >= 0 && N >= 0 && batch >= 0, "matmul: negative dimension");
  if (M == 0 || N == 0 || batch == 0) return OK;
  if (K == 0) {
    if (!accum) TURT_CHECK_CUDA(cudaMemsetAsync(out, 0, (size_t)M * N * batch * 4, ctx->stream));
    return OK;
  }
  // A is [M,K] (transA = 0, K-major) or [K,M] (transA = 1, M-major);
  // B is [K,N] (transB = 0, N-major) or [N,K] (transB = 1, K-major).
  GemmOperand A{a, transA ? M : K, (long)M * K, transA != 0};
  GemmOperand B{b, transB ? K : N, (long)K * N, transB == 0};
  GemmEpi epi;
  epi.kind = accum ? EPI_ACCUM : EPI_STORE;
  epi.C = out;
  epi.ldc = N;
  epi.strideC = (long)M * N;
  if (ctx->precision != 0 && gemm_tf32_supported(A, B) && N % 4 == 0 && ((uintptr_t)out & 15) == 0)
    return gemm_tf32(ctx->stream, M, N, K, batch, A, B, epi, ctx->flags, ctx->precision);
  return gemm_simt(ctx->stream, a, b, out, M, K, N, batch, transA != 0, transB != 0, accum != 0);
}

int turt_ewise(turt_ctx* ctx, const float* a, const float* b, float* out, size_t n, size_t bLen, int op, int accum) {
  CTX_GUARD(ctx);
  TURT_REQUIRE(op >= 0 && op <= 2, "ewise: op must be 0 (add), 1 (sub) or 2 (mul)");
  return op_ewise(ctx->stream, a, b, out, n, bLen, op, accum);
}
int turt_scale(turt_ctx* ctx, const float* a, float* out, size_t n, float s, int accum) {
  CTX_GUARD(ctx);
  return op_scale(ctx->stream, a, out, n, s, accum);
}
int turt_bcast_acc(turt_ctx* ctx, const float* src, float* out, size_t n, size_t bLen, float s) {
  CTX_GUARD(ctx);
  return op_bcast_acc(ctx->stream, src, out, n, bLen, s);
}
int turt_segsum(turt_ctx* ctx, const float* g, float* out, size_t n, size_t bLen, float s, int accum) {
  CTX_GUARD(ctx);
  return op_segsum(ctx->stream, g, out, n, bLen, s, accum);
}
int turt_total(turt_ctx* ctx, const float* a, float* out, size_t n) {
  CTX_GUARD(ctx);
  return op_total(ctx->stream, a, out, n);
}
int turt_relu(turt_ctx* ctx, const float* x, float* out, size_t n) {
  CTX_GUARD(ctx);
  return op_relu(ctx->stream, x, out, n);
}
int turt_relu_bwd(turt_ctx* ctx, const float* x, const float* gOut, float* gIn, size_t n) {
  CTX_GUARD(ctx);
  return op_relu_bwd(ctx->stream, x, gOut, gIn, n);
}
int turt_sgd(turt_ctx* ctx, const float* grad, float* param, size_t n, float lr) {
  CTX_GUARD(ctx);
  return op_sgd(ctx->stream, grad, param, n, lr);
}
int turt_gelu(turt_ctx* ctx, const float* x, float* out, size_t n) {
  CTX_GUARD(ctx);
  return op_gelu(ctx->stream, x, out, n);
}
int turt_gelu_bwd(turt_ctx* ctx, const float* x, const float* gOut, float* gIn, size_t n) {
  CTX_GUARD(ctx);
  return op_gelu_bwd(ctx->stream, x, gOut, gIn, n);
}
int turt_silu(turt_ctx* ctx, const float* x, float* out, size_t n) {
  CTX_GUARD(ctx);
  return op_silu(ctx->stream, x, out, n);
}
int turt_silu_bwd(turt_ctx* ctx, const float* x, const float* gOut, float* gIn, size_t n) {
  CTX_GUARD(ctx);
  return op_silu_bwd(ctx->stream, x, gOut, gIn, n);
}
int turt_rms_fwd(turt_ctx* ctx, const float* x, const float* gamma, float* out, float* rstd, int rows, int d,
                 float eps) {
  CTX_GUARD(ctx);
  return op_rms_fwd(ctx->stream, x, gamma, out, rstd, rows, d, eps);
}
int turt_rms_dx(turt_ctx* ctx, const float* x, const float* gOut, const float* gamma, const float* rstd, float* gIn,
                int rows, int d, float eps) {
  CTX_GUARD(ctx);
  (void)eps;
  return op_rms_dx(ctx->stream, x, gOut, gamma, rstd, gIn, rows, d);
}
int turt_rms_dg(turt_ctx* ctx, const float* x, const float* gOut, const float* rstd, float* dgamma, int rows, int d) {
  CTX_GUARD(ctx);
  return op_rms_dg(ctx->stream, x, gOut, rstd, dgamma, rows, d);
}

static int rope_table_for(turt_ctx* ctx, int t, int hd, float base, const float2** out) {
  auto key = std::make_tuple(t, hd, base);
  auto it = ctx->rope_tables.find(key);
  if (it == ctx->rope_tables.end()) {
    float2* cs = nullptr;
    TURT_CHECK_CUDA(cudaMalloc(&cs, sizeof(float2) * (size_t)t * (hd / 2) + 16));
    int rc = op_rope_table(ctx->stream, cs, t, hd, (double)base);
    if (rc) return rc;
    it = ctx->rope_tables.emplace(key, cs).first;
  }
  *out = it->second;
  return OK;
}

int turt_rope(turt_ctx* ctx, const float* x, float* out, int groups, int t, int hd, float base) {
  CTX_GUARD(ctx);
  TURT_REQUIRE(hd % 2 == 0, "rope requires an even headDim");
  const float2* cs;
  int rc = rope_table_for(ctx, t, hd, base, &cs);
  if (rc) return rc;
  return op_rope(ctx->stream, x, out, cs, groups, t, hd, 0);
}
int turt_rope_bwd(turt_ctx* ctx, const float* gOut, float* gIn, int groups, int t, int hd, float base) {
  CTX_GUARD(ctx);
  TURT_REQUIRE(hd % 2 == 0, "rope requires an even headDim");
  const float2* cs;
  int rc = rope_table_for(ctx, t, hd, base, &cs);
  if (rc) return rc;
  return op_rope(ctx->stream, gOut, gIn, cs, groups, t, hd, 1);
}
int turt_softmax(turt_ctx* ctx, const float* x, float* out, int rows, int d) {
  CTX_GUARD(ctx);
  return op_softmax(ctx->stream, x, out, rows, d);
}
int turt_softmax_bwd(turt_ctx* ctx, const float* y, const float* gOut, float* gIn, int rows, int d) {
  CTX_GUARD(ctx);
  return op_softmax_bwd(ctx->stream, y, gOut, gIn, rows, d);
}
int turt_ln_fwd(turt_ctx* ctx, const float* x, const float* gamma, const float* beta, float* out, float* mean,
                float* rstd, int rows, int d, float eps) {
  CTX_GUARD(ctx);
  return op_ln_fwd(ctx->stream, x, gamma, beta, out, mean, rstd, rows, d, eps);
}
int turt_ln_dx(turt_ctx* ctx, const float* x, const float* gOut, const float* gamma, const float* mean,
               const float* rstd, float* gIn, int rows, int d, float eps) {
  CTX_GUARD(ctx);
  (void)eps;
  return op_ln_dx(ctx->stream, x, gOut, gamma, mean, rstd, gIn, rows, d);
}
int turt_ln_dgb(turt_ctx* ctx, const float* x, const float* gOut, const float* mean, const float* rstd, float* dgamma,
                float* dbeta, int rows, int d) {
  CTX_GUARD(ctx);
  return op_ln_dgb(ctx->stream, x, gOut, mean, rstd, dgamma, dbeta, rows, d);
}
int turt_gather(turt_ctx* ctx, const float* table, const uint32_t* idx, float* out, int n, int d, int vocab) {
  CTX_GUARD(ctx);
  return op_gather(ctx->stream, table, idx, out, n, d, vocab, ctx->flags);
}
int turt_gather_bwd(turt_ctx* ctx, const uint32_t* idx, const float* gOut, float* dTable, int n, int d, int vocab) {
  CTX_GUARD(ctx);
  return op_gather_bwd(ctx->stream, idx, gOut, dTable, n, d, vocab, ctx->flags);
}
int turt_ce_fwd(turt_ctx* ctx, const float* logits, const uint32_t* targets, float* perRow, int rows, int vocab) {
  CTX_GUARD(ctx);
  return op_ce_fwd(ctx->stream, logits, targets, perRow, rows, vocab, ctx->flags);
}
int turt_ce_bwd(turt_ctx* ctx, const float* logits, const uint32_t* targets, const float* gLoss, float* dLogits,
                int rows, int vocab) {
  CTX_GUARD(ctx);
  return op_ce_bwd(ctx->stream, logits, targets, gLoss, dLogits, rows, vocab, ctx->flags);
}
int turt_mask(turt_ctx* ctx, const float* x, float* out, int groups, int t) {
  CTX_GUARD(ctx);
  return op_mask(ctx->stream, x, out, groups, t, 0);
}
int turt_mask_bwd(turt_ctx* ctx, const float* gOut, float* gIn, int groups, int t) {
  CTX_GUARD(ctx);
  return op_mask(ctx->stream, gOut, gIn, groups, t, 1);
}
int turt_permute4(turt_ctx* ctx, const float* inp, float* out, const int* inShape4, const int* perm4, size_t n,
                  int accum) {
  CTX_GUARD(ctx);
  TURT_REQUIRE(inShape4 && perm4, "permute4: null shape/perm");
  int seen = 0;
  for (int a = 0; a < 4; a++) {
    TURT_REQUIRE(perm4[a] >= 0 && perm4[a] < 4, "permute4: perm entries must be 0..3");
    seen |= 1 << perm4[a];
  }
  TURT_REQUIRE(seen == 15, "permute4: perm is not a permutation");
  return op_permute4(ctx->stream, inp, out, inShape4, perm4, n, accum);
}
int turt_adamw(turt_ctx* ctx, const float* grad, float* param, float* m, float* v, size_t n, float lr, float b1,
               float b2, float eps, float wd, float bc1, float bc2) {
  CTX_GUARD(ctx);
  return op_adamw(ctx->stream, grad, param, m, v, n, lr, b1, b2, eps, wd, bc1, bc2);
}

// ----------------------------------------------------- host-array matmul
int turt_host_bmm(turt_ctx* ctx, const float* a, int batch, int m, int k, const float* b, int n, float* out) {
  CTX_GUARD(ctx);
  TURT_REQUIRE(a && b && out, "matmul: null array");
  TURT_REQUIRE(batch >= 0 && m >= 0 && k >= 0 && n >= 0, "matmul: negative dimension");
  const size_t na = (size_t)batch * m * k, nb = (size_t)batch * k * n, nc = (size_t)batch * m * n;
  if (nc == 0) return OK;
  // Pitch rows up to a multiple of 4 floats so every call takes the tensor-core path.
  // Tensor-core path: pitch rows up to a multiple of 4 floats (TMA needs 16-byte pitches).
  // CUDA-core (FP32) path: dense rows.
  const bool simt = ctx->precision == 0;
  const int kp = simt ? k : (k + 3) & ~3, np = simt ? n : (n + 3) & ~3;
  float *da = nullptr, *db = nullptr, *dc = nullptr;
  TURT_CHECK_CUDA(cudaMallocAsync(&da, (size_t)batch * m * kp * 4 + 16, ctx->stream));
  TURT_CHECK_CUDA(cudaMallocAsync(&db, (size_t)batch * k * np * 4 + 16, ctx->stream));
  TURT_CHECK_CUDA(cudaMallocAsync(&dc, (size_t)batch * m * np * 4 + 16, ctx->stream));
  (void)na;
  (void)nb;
  int rc = OK;
  if (k == 0) {
    TURT_CHECK_CUDA(cudaMemsetAsync(dc, 0, (size_t)batch * m * np * 4, ctx->stream));
  } else {
    TURT_CHECK_CUDA(cudaMemcpy2DAsync(da, kp * 4, a, k * 4, k * 4, (size_t)batch * m, cudaMemcpyHostToDevice,
                                      ctx->stream));
    TURT_CHECK_CUDA(cudaMemcpy2DAsync(db, np * 4, b, n * 4, n * 4, (size_t)batch * k, cudaMemcpyHostToDevice,
                                      ctx->stream));
    GemmOperand A{da, kp, (long)m * kp, false};
    GemmOperand B{db, np, (long)k * np, true};
    GemmEpi epi;
    epi.kind = EPI_STORE;
    epi.C = dc;
    epi.ldc = np;
    epi.strideC = (long)m * np;
    if (ctx->precision == 0)
      rc = gemm_simt(ctx->stream, da, db, dc, m, k, n, batch, false, false, false);
    else
      rc = gemm_tf32(ctx->stream, m, n, k, batch, A, B, epi, ctx->flags, ctx->precision);
  }
  if (rc == OK)
    TURT_CHECK_CUDA(cudaMemcpy2DAsync(out, n * 4, dc, np * 4, n * 4, (size_t)batch * m, cudaMemcpyDeviceToHost,
                                      ctx->stream));
  cudaFreeAsync(da, ctx->stream);
  cudaFreeAsync(db, ctx->stream);
  cudaFreeAsync(dc, ctx->stream);
  TURT_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
  if (rc) return rc;
  return ctx_check_flags(ctx);
}

int turt_host_matmul(turt_ctx* ctx, const float* a, int m, int k, const float* b, int n, float* out) {
  return turt_host_bmm(ctx, a, 1, m, k, b, n, out);
}

}  // extern "C"
