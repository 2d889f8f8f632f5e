// model.cuh -- the GPT model object behind turt_model*.
#pragma once
#include <string>
#include <vector>

#include "../../include/turt_cuda.h"
#include "ctx.cuh"

namespace turt {

// Where one reference parameter (parameters() order) lives in the internal flat buffer:
// `rows` runs of `width` floats, `pitch` floats apart, starting at `off`.
struct ParamSlot {
  std::string name;
  int shape[2];
  int ndim;
  size_t off;
  int width;
  long rows;
  int pitch;
  size_t count() const { return (size_t)width * rows; }
};

struct LayerOff {
  size_t ln1g, ln1b, wqkv, bqkv, wproj, bproj, ln2g, ln2b, w1, b1, w2, b2;
  size_t begin, end;  // [begin, end) range of this layer in the flat buffer
};

struct LayerAct {
  float *x, *y1, *rs1, *mu1, *qkv, *att, *lse, *h, *y2, *rs2, *mu2, *pre, *act;
  float *P, *qr, *kr;  // tensor-core attention: probabilities, rotated q / k (kept for backward)
};

struct DpState;

}  // namespace turt

struct turt_model {
  turt_ctx* ctx = nullptr;
  turt_config cfg{};
  int hid = 0;
  bool modern = true;
  float eps = 1e-5f;
  // flat buffers (internal layout), 256-byte aligned tensors
  size_t total = 0;
  float *P = nullptr, *G = nullptr, *M = nullptr, *V = nullptr;
  size_t wte = 0, wpe = 0, lnfg = 0, lnfb = 0, head_end = 0;
  std::vector<turt::LayerOff> layers;
  std::vector<turt::ParamSlot> params;
  float2* rope_cs = nullptr;
  // workspace for the current token capacity
  int capN = 0, capB = 0;
  long capS = 0;       // B*H*T*pitch floats per layer of score storage in the workspace
  int attn_mode = 0;   // TURT_ATTN_*
  bool attn_tc = false;  // the current workspace uses tensor-core attention
  void* ws = nullptr;
  std::vector<turt::LayerAct> act;
  float *xL = nullptr, *yf = nullptr, *rsf = nullptr, *muf = nullptr, *logits = nullptr, *loss_rows = nullptr;
  float *dx = nullptr, *dy = nullptr, *datt = nullptr, *dqkv = nullptr, *dpre = nullptr, *Dsc = nullptr,
        *part = nullptr;
  float* dS = nullptr;    // tensor-core attention backward scratch
  float* dact = nullptr;  // d(SwiGLU output) [N][h] (modern arch)
  uint32_t *d_ids = nullptr, *d_tgt = nullptr;
  uint32_t *h_ids = nullptr, *h_tgt = nullptr;  // pinned staging
  float* loss_dev = nullptr;
  float* coef_dev = nullptr;
  double* norm_dev = nullptr;
  double* norm_scratch = nullptr;
  float* h_loss = nullptr;  // pinned
  turt::DpState* dp = nullptr;
  bool dp_defer = false;
  // Weight-gradient GEMMs of the backward pass run on their own stream, overlapping the
  // data-gradient chain; `wg_ring` events order the forks / joins, `wg_mark` ones are kept
  // until the main stream reuses a buffer that a pending weight-gradient GEMM reads.
  cudaStream_t wg = nullptr;
  cudaEvent_t wg_ring[16] = {};
  cudaEvent_t wg_mark[4] = {};
  int wg_next = 0;
  // Generation: KV cache [n_layer][n_head][block_size][head_dim] (k RoPE-rotated), the number of
  // positions it holds, and the decode-step vectors.
  float *kcache = nullptr, *vcache = nullptr, *dec = nullptr;
  size_t dec_floats = 0;
  int dec_len = 0;
  // The decode step is captured once into a CUDA graph that reads (token, position) from a
  // device cell; each step copies the pair there from pinned memory and replays the graph.
  int* dec_tok = nullptr;
  int* h_dec_tok = nullptr;  // pinned
  cudaStream_t dec_cap = nullptr;
  cudaGraphExec_t dec_graph = nullptr;
  int dec_graph_kernels = 0;
};

namespace turt {
// Logits-only forward of one sequence (b = 1) of t host token ids; logits land in m->logits and
// every layer's activations (qkv, rotated q / k copies) in the workspace.
int model_forward_logits(turt_model* m, const uint32_t* ids, int t);
// Makes stream `to` wait for everything issued so far on stream `from`.
int stream_join(turt_model* m, cudaStream_t from, cudaStream_t to);
// The stream whose completion implies every gradient write issued so far (joins the
// weight-gradient stream behind the main one).
int grad_writes_stream(turt_model* m, cudaStream_t* out);
// DP hooks called by the backward pass (dp.cu).
int dp_after_layer(turt_model* m, int layer);
int dp_after_head(turt_model* m);
int dp_finish(turt_model* m);  // compute stream waits for outstanding reductions
bool dp_active(turt_model* m);
}  // namespace turt
