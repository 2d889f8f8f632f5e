// group.cu -- one host process driving several GPUs.
//
// The reference trains data-parallel inside one process: a pool of worker threads, one model
// replica each, the batch split into contiguous shards, and the main thread forming the
// row-weighted mean of the shard gradients (scripts/train-gpt.ts:66-101, 105-123, 200-219).
// A turt_group is that pool on GPUs: one replica (context + model) per device, each driven by
// its own host thread so that the devices' launches proceed in parallel, and the gradient
// mean formed by NCCL inside the backward pass (dp.cu: per-layer all-reduce on a
// communication stream, overlapped with the remaining backward).  Shard i of a b-sequence
// batch holds floor(b/n) sequences, plus one for i < b mod n (the reference's shard()); its
// mean-loss gradient is scaled by rows_i / b before the all-reduce sums the replicas, which is
// the reference's weighting exactly, so the optimizer step needs no further scaling.
#include <cstdio>
#include <cstdlib>
#include <condition_variable>
#include <deque>
#include <set>
#include <functional>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/turt_cuda.h"
#include "model.cuh"

namespace turt {
namespace {

// TURT_GROUP_TRACE=1 in the environment prints each phase of each replica's work to stderr.
bool trace_on() {
  static const bool on = [] {
    const char* v = getenv("TURT_GROUP_TRACE");
    return v && v[0] == '1';
  }();
  return on;
}
void trace(int dev, const char* what) {
  if (trace_on()) fprintf(stderr, "[turt group] device %d: %s\n", dev, what);
}

// One host thread per device, running posted jobs in order with that device current.
class DeviceWorker {
 public:
  explicit DeviceWorker(int dev) : dev_(dev), th_([this] { loop(); }) {}
  ~DeviceWorker() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    th_.join();
  }
  void post(std::function<int()> fn) {
    {
      std::lock_guard<std::mutex> lk(mu_);
      q_.push_back(std::move(fn));
      pending_++;
    }
    cv_.notify_all();
  }
  // Waits for every posted job; returns the first failure since the last wait (its message in *msg).
  int wait(std::string* msg) {
    std::unique_lock<std::mutex> lk(mu_);
    done_cv_.wait(lk, [this] { return pending_ == 0; });
    const int rc = rc_;
    if (rc && msg) *msg = msg_;
    rc_ = 0;
    msg_.clear();
    return rc;
  }

 private:
  void loop() {
    const bool dev_ok = cudaSetDevice(dev_) == cudaSuccess;
    for (;;) {
      std::function<int()> fn;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [this] { return stop_ || !q_.empty(); });
        if (q_.empty()) return;  // stop requested and nothing left
        fn = std::move(q_.front());
        q_.pop_front();
      }
      int rc = dev_ok ? fn() : ERR_CUDA;
      std::string m = rc ? (dev_ok ? std::string(last_error()) : std::string("cudaSetDevice failed")) : std::string();
      {
        std::lock_guard<std::mutex> lk(mu_);
        if (rc && !rc_) {
          rc_ = rc;
          msg_ = "device " + std::to_string(dev_) + ": " + m;
        }
        pending_--;
      }
      done_cv_.notify_all();
    }
  }
  int dev_;
  std::mutex mu_;
  std::condition_variable cv_, done_cv_;
  std::deque<std::function<int()>> q_;
  int pending_ = 0;
  int rc_ = 0;
  std::string msg_;
  bool stop_ = false;
  std::thread th_;  // last: started after every other member is constructed
};

}  // namespace
}  // namespace turt

struct turt_group {
  int n = 0;
  std::vector<int> devs;
  std::vector<turt_ctx*> ctx;
  std::vector<turt_model*> model;
  std::vector<turt::DeviceWorker*> workers;
  bool defer = false;
  std::set<std::pair<int, int>> shapes_seen;  // (b, t) of batches already run with reduction
};

using namespace turt;

namespace {

// Runs fn(i) for every replica on its own thread and waits for all of them; the first failure
// is returned with its message set on the calling thread.
int run_all(turt_group* g, const std::function<int(int)>& fn) {
  for (int i = 0; i < g->n; i++) g->workers[i]->post([fn, i] { return fn(i); });
  int rc = OK;
  std::string msg;
  for (int i = 0; i < g->n; i++) {
    std::string m;
    const int r = g->workers[i]->wait(&m);
    if (r && !rc) {
      rc = r;
      msg = m;
    }
  }
  if (rc) set_error(msg);
  return rc;
}

int run_one(turt_group* g, int i, const std::function<int()>& fn) {
  g->workers[i]->post(fn);
  std::string m;
  const int rc = g->workers[i]->wait(&m);
  if (rc) set_error(m);
  return rc;
}

void destroy_group(turt_group* g) {
  if (!g) return;
  if (!g->workers.empty()) {
    run_all(g, [g](int i) {
      if (g->model[i]) turt_model_destroy(g->model[i]);
      if (g->ctx[i]) turt_ctx_destroy(g->ctx[i]);
      g->model[i] = nullptr;
      g->ctx[i] = nullptr;
      return OK;
    });
  }
  for (auto* w : g->workers) delete w;
  delete g;
}

#define GROUP_GUARD(g)                    \
  do {                                    \
    if (!(g)) {                           \
      set_error("null group");            \
      return ERR_INVALID;                 \
    }                                     \
  } while (0)

}  // namespace

extern "C" {

int turt_group_create(int ndev, const int* devs, const turt_config* cfg, turt_group** out) {
  TURT_REQUIRE(out && cfg && devs, "turt_group_create: null argument");
  TURT_REQUIRE(ndev >= 1 && ndev <= 64, "turt_group_create: ndev must be in [1, 64]");
  int count = 0;
  TURT_CHECK_CUDA(cudaGetDeviceCount(&count));
  for (int i = 0; i < ndev; i++) {
    if (devs[i] < 0 || devs[i] >= count) {
      set_error("turt_group_create: no CUDA device " + std::to_string(devs[i]));
      return ERR_INVALID;
    }
    for (int j = 0; j < i; j++)
      if (devs[j] == devs[i]) {
        set_error("turt_group_create: device " + std::to_string(devs[i]) + " listed twice");
        return ERR_INVALID;
      }
  }
  turt_group* g = new turt_group();
  g->n = ndev;
  g->devs.assign(devs, devs + ndev);
  g->ctx.assign(ndev, nullptr);
  g->model.assign(ndev, nullptr);
  for (int i = 0; i < ndev; i++) g->workers.push_back(new DeviceWorker(devs[i]));
  int rc = run_all(g, [g, cfg](int i) -> int {
    trace(g->devs[i], "context");
    RC(turt_init(g->devs[i], &g->ctx[i]));
    trace(g->devs[i], "model");
    return turt_model_create(g->ctx[i], cfg, &g->model[i]);
  });
  if (rc == OK && ndev > 1) {
    char uid[128];
    rc = turt_dp_unique_id(uid);
    // every rank joins the communicator concurrently (ncclCommInitRank blocks until all have)
    if (rc == OK)
      rc = run_all(g, [g, &uid, ndev](int i) -> int {
        trace(g->devs[i], "communicator init");
        const int r = turt_dp_init(g->model[i], i, ndev, uid);
        trace(g->devs[i], "communicator ready");
        return r;
      });
  }
  if (rc) {
    const std::string msg = last_error();
    destroy_group(g);
    set_error(msg);
    return rc;
  }
  *out = g;
  return OK;
}

int turt_group_destroy(turt_group* g) {
  GROUP_GUARD(g);
  destroy_group(g);
  return OK;
}

int turt_group_size(turt_group* g, int* ndev) {
  GROUP_GUARD(g);
  TURT_REQUIRE(ndev, "null ndev");
  *ndev = g->n;
  return OK;
}

int turt_group_model(turt_group* g, int i, turt_model** out) {
  GROUP_GUARD(g);
  TURT_REQUIRE(out && i >= 0 && i < g->n, "turt_group_model: bad replica index");
  *out = g->model[i];
  return OK;
}

int turt_group_param_upload(turt_group* g, int index, const float* host, size_t n) {
  GROUP_GUARD(g);
  return run_all(g, [=](int i) { return turt_param_upload(g->model[i], index, host, n); });
}

int turt_group_param_download(turt_group* g, int index, float* host, size_t n) {
  GROUP_GUARD(g);
  return run_one(g, 0, [=] { return turt_param_download(g->model[0], index, host, n); });
}

int turt_group_grad_download(turt_group* g, int index, float* host, size_t n) {
  GROUP_GUARD(g);
  return run_one(g, 0, [=] { return turt_grad_download(g->model[0], index, host, n); });
}

int turt_group_model_init(turt_group* g, uint32_t seed) {
  GROUP_GUARD(g);
  return run_all(g, [=](int i) { return turt_model_init(g->model[i], seed); });
}

int turt_group_zero_grad(turt_group* g) {
  GROUP_GUARD(g);
  return run_all(g, [=](int i) { return turt_zero_grad(g->model[i]); });
}

int turt_group_defer(turt_group* g, int defer) {
  GROUP_GUARD(g);
  g->defer = defer != 0;
  return OK;
}

int turt_group_forward_backward(turt_group* g, const uint32_t* ids, const uint32_t* targets, int b, int t,
                                float loss_scale, float* loss_out) {
  GROUP_GUARD(g);
  TURT_REQUIRE(ids && targets, "null token array");
  if (b < g->n) {
    set_error("turt_group_forward_backward: batch of " + std::to_string(b) + " sequences is smaller than the " +
              std::to_string(g->n) + " devices of the group");
    return ERR_INVALID;
  }
  const int base = b / g->n, rem = b % g->n;
  std::vector<int> row0(g->n), rows(g->n);
  for (int i = 0, r = 0; i < g->n; i++) {
    rows[i] = base + (i < rem ? 1 : 0);
    row0[i] = r;
    r += rows[i];
  }
  std::vector<float> loss(g->n, 0.f);
  const bool defer = g->defer;
  const bool want = loss_out != nullptr;
  // The first call of a batch shape allocates (workspace, pinned staging, split-K partials) and
  // loads kernels on their first launch.  In one process with peer access enabled, an allocation
  // may wait for every device, including a peer whose collective already spins for this device's
  // part of it: so that call enqueues every replica's whole backward pass first (reductions
  // deferred) and only then, once all host threads are past their allocations, one all-reduce of
  // the gradient buffers.  Later calls of the shape allocate nothing and overlap the per-layer
  // reductions with the backward pass.
  const bool first = g->n > 1 && !defer && !g->shapes_seen.count({b, t});
  int rc = run_all(g, [&](int i) -> int {
    const int dev = g->devs[i];
    RC(turt_dp_defer(g->model[i], (defer || first) ? 1 : 0));
    const size_t off = (size_t)row0[i] * t;
    trace(dev, first ? "forward / backward (reduction after every replica's)" : "forward / backward");
    RC(turt_forward_backward(g->model[i], ids + off, targets + off, rows[i], t,
                             loss_scale * (float)rows[i] / (float)b, (want && !first) ? &loss[i] : nullptr));
    trace(dev, "forward / backward enqueued");
    return OK;
  });
  if (rc) return rc;
  if (first) {
    rc = run_all(g, [&](int i) -> int {
      const int dev = g->devs[i];
      RC(turt_dp_allreduce_grads(g->model[i]));
      trace(dev, "all-reduce enqueued");
      RC(turt_dp_defer(g->model[i], 0));
      const int r = want ? turt_read_loss(g->model[i], &loss[i]) : OK;
      trace(dev, "step done");
      return r;
    });
    if (rc) return rc;
  }
  if (first) g->shapes_seen.insert({b, t});
  if (want) {
    double l = 0;
    for (int i = 0; i < g->n; i++) l += (double)loss[i] * rows[i] / b;
    *loss_out = (float)l;
  }
  return OK;
}

int turt_group_adamw_step(turt_group* g, float lr, float b1, float b2, float eps, float wd, float bc1, float bc2,
                          float clip) {
  GROUP_GUARD(g);
  return run_all(g, [=](int i) { return turt_adamw_step(g->model[i], lr, b1, b2, eps, wd, bc1, bc2, clip, 1.0f); });
}

int turt_group_synchronize(turt_group* g) {
  GROUP_GUARD(g);
  return run_all(g, [=](int i) { return turt_synchronize(g->ctx[i]); });
}

}  // extern "C"
