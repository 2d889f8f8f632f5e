// dp.cu -- data-parallel gradient reduction over NCCL (NVLink / NVSwitch).
//
// The reference reduces on the host: each worker returns its shard's mean gradient and the
// main thread forms the row-weighted mean (scripts/train-gpt.ts:200-219).  Here every rank
// owns one GPU and one replica; the flat gradient buffer is summed in place with
// ncclAllReduce, one call per layer issued on a communication stream as soon as that
// layer's backward has produced all of its gradients, so the reductions of layer l overlap
// the backward of layers l-1..0.  The head bucket (wte/wpe/lnf) follows the embedding
// backward.  The 1/world mean is folded into the AdamW pass (grad_scale).
//
// libnccl is opened at run time (the copy the process already has loaded, e.g. by
// torch.distributed, is reused), so libturt_cuda.so has no link-time NCCL dependency.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "model.cuh"

namespace turt {

namespace {
struct NcclApi {
  void* h = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) =
      nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

NcclApi& api() {
  static NcclApi a;
  return a;
}

int load_nccl() {
  static std::mutex mu;  // device worker threads may load it concurrently
  std::lock_guard<std::mutex> lock(mu);
  NcclApi& a = api();
  if (a.h) return OK;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
  if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
  if (!h) {
    set_error(std::string("cannot load libnccl.so.2: ") + dlerror());
    return ERR_NCCL;
  }
#define SYM(f, n)                                                   \
  a.f = reinterpret_cast<decltype(a.f)>(dlsym(h, n));               \
  if (!a.f) {                                                       \
    set_error(std::string("libnccl is missing ") + n);              \
    return ERR_NCCL;                                                \
  }
  SYM(GetUniqueId, "ncclGetUniqueId");
  SYM(CommInitRank, "ncclCommInitRank");
  SYM(AllReduce, "ncclAllReduce");
  SYM(CommDestroy, "ncclCommDestroy");
  SYM(CommAbort, "ncclCommAbort");
  SYM(CommGetAsyncError, "ncclCommGetAsyncError");
  SYM(GetErrorString, "ncclGetErrorString");
#undef SYM
  a.h = h;
  return OK;
}

#define NCCL_CHECK(expr)                                                                         \
  do {                                                                                           \
    ncclResult_t r__ = (expr);                                                                   \
    if (r__ != ncclSuccess) {                                                                    \
      set_error(std::string(#expr) + ": " + (api().GetErrorString ? api().GetErrorString(r__) : "nccl error")); \
      return ERR_NCCL;                                                                           \
    }                                                                                            \
  } while (0)
}  // namespace

struct DpState {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
  cudaStream_t comm_stream = nullptr;
  std::vector<cudaEvent_t> layer_ev;
  cudaEvent_t head_ev = nullptr, done_ev = nullptr;
};

bool dp_active(turt_model* m) { return m->dp && m->dp->world > 1; }

static int reduce_range(turt_model* m, size_t begin, size_t end, cudaEvent_t ev) {
  DpState* d = m->dp;
  cudaStream_t gs = nullptr;
  RC(grad_writes_stream(m, &gs));
  TURT_CHECK_CUDA(cudaEventRecord(ev, gs));
  TURT_CHECK_CUDA(cudaStreamWaitEvent(d->comm_stream, ev, 0));
  NCCL_CHECK(api().AllReduce(m->G + begin, m->G + begin, end - begin, ncclFloat32, ncclSum, d->comm, d->comm_stream));
  return OK;
}

int dp_after_layer(turt_model* m, int l) {
  return reduce_range(m, m->layers[l].begin, m->layers[l].end, m->dp->layer_ev[l]);
}
int dp_after_head(turt_model* m) { return reduce_range(m, 0, m->head_end, m->dp->head_ev); }
int dp_finish(turt_model* m) {
  DpState* d = m->dp;
  TURT_CHECK_CUDA(cudaEventRecord(d->done_ev, d->comm_stream));
  TURT_CHECK_CUDA(cudaStreamWaitEvent(m->ctx->stream, d->done_ev, 0));
  return OK;
}

}  // namespace turt

using namespace turt;

extern "C" {

int turt_dp_unique_id(char* id128) {
  TURT_REQUIRE(id128, "null id buffer");
  int rc = load_nccl();
  if (rc) return rc;
  ncclUniqueId id;
  NCCL_CHECK(api().GetUniqueId(&id));
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId must be 128 bytes");
  memcpy(id128, &id, 128);
  return OK;
}

int turt_dp_init(turt_model* m, int rank, int world, const char* id128) {
  TURT_REQUIRE(m && id128, "null argument");
  TURT_REQUIRE(world >= 1 && rank >= 0 && rank < world, "bad rank/world");
  TURT_CHECK_CUDA(cudaSetDevice(m->ctx->device));
  int rc = load_nccl();
  if (rc) return rc;
  if (m->dp) turt_dp_destroy(m);
  DpState* d = new DpState();
  d->rank = rank;
  d->world = world;
  ncclUniqueId id;
  memcpy(&id, id128, 128);
  NCCL_CHECK(api().CommInitRank(&d->comm, world, id, rank));
  TURT_CHECK_CUDA(cudaStreamCreateWithFlags(&d->comm_stream, cudaStreamNonBlocking));
  d->layer_ev.resize(m->cfg.n_layer);
  for (auto& e : d->layer_ev) TURT_CHECK_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  TURT_CHECK_CUDA(cudaEventCreateWithFlags(&d->head_ev, cudaEventDisableTiming));
  TURT_CHECK_CUDA(cudaEventCreateWithFlags(&d->done_ev, cudaEventDisableTiming));
  m->dp = d;
  return OK;
}

// Explicit (non-overlapped) reduction of the whole gradient buffer, for callers that
// accumulate micro-batches with the per-layer reduction deferred (turt_dp_defer).
int turt_dp_allreduce_grads(turt_model* m) {
  TURT_REQUIRE(m, "null model");
  if (!dp_active(m)) return OK;
  TURT_CHECK_CUDA(cudaSetDevice(m->ctx->device));
  int rc = reduce_range(m, 0, m->total, m->dp->head_ev);
  if (rc) return rc;
  return dp_finish(m);
}

int turt_dp_defer(turt_model* m, int defer) {
  TURT_REQUIRE(m, "null model");
  m->dp_defer = defer != 0;
  return OK;
}

// Waits for outstanding reductions with a wall-clock limit; on expiry or on an asynchronous
// NCCL error the communicator is aborted and TURT_ERR_NCCL returned (the process can then
// shut down cleanly instead of hanging in a collective).
int turt_dp_wait(turt_model* m, int timeout_ms) {
  TURT_REQUIRE(m, "null model");
  if (!m->dp) return OK;
  TURT_CHECK_CUDA(cudaSetDevice(m->ctx->device));
  DpState* d = m->dp;
  auto t0 = std::chrono::steady_clock::now();
  while (true) {
    cudaError_t q = cudaStreamQuery(d->comm_stream);
    if (q == cudaSuccess) return OK;
    if (q != cudaErrorNotReady) {
      set_error(std::string("comm stream: ") + cudaGetErrorString(q));
      return ERR_CUDA;
    }
    ncclResult_t ar = ncclSuccess;
    api().CommGetAsyncError(d->comm, &ar);
    const bool expired =
        std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count() > timeout_ms;
    if (ar != ncclSuccess || expired) {
      api().CommAbort(d->comm);
      d->comm = nullptr;
      set_error(expired ? "gradient all-reduce timed out; communicator aborted"
                        : std::string("NCCL async error: ") + api().GetErrorString(ar));
      return ERR_NCCL;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

int turt_dp_destroy(turt_model* m) {
  TURT_REQUIRE(m, "null model");
  DpState* d = m->dp;
  if (!d) return OK;
  cudaSetDevice(m->ctx->device);
  if (d->comm_stream) cudaStreamSynchronize(d->comm_stream);
  if (d->comm) api().CommDestroy(d->comm);
  for (auto& e : d->layer_ev) cudaEventDestroy(e);
  if (d->head_ev) cudaEventDestroy(d->head_ev);
  if (d->done_ev) cudaEventDestroy(d->done_ev);
  if (d->comm_stream) cudaStreamDestroy(d->comm_stream);
  delete d;
  m->dp = nullptr;
  return OK;
}

}  // extern "C"
