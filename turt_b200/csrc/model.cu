// model.cu -- GPU-resident GPT train step (both architectures of src/models/gpt.ts).
//
// The reference builds the step as a tape of ~30 dispatches per block
// (src/models/gpu-gpt.ts:143-201 over src/infer/webgpu/autograd.ts).  Here one block is:
//   forward : norm1 -> GEMM(qkv) -> attention(+RoPE) -> GEMM(proj, +residual)
//             -> norm2 -> GEMM(gate|up, SwiGLU epilogue  |  fc, bias+GELU epilogue)
//             -> GEMM(down|mp, +residual)
//   backward: GEMM(dact, SwiGLU'/GELU' epilogue) + GEMM(dW) ... norm backward with the
//             residual gradient fused, attention backward, GEMM(dX) + GEMM(dW)
// on a flat parameter/gradient buffer so clip, AdamW and the DP all-reduce are single passes.
//
// Internal weight layout (the C ABI converts to/from the reference's [in,out] tensors):
//   Wqkv [E][3E]  = [qW | kW | vW] column blocks     bqkv [3E]
//   W1   [E][2h]  = gate/up interleaved in 32-column blocks (modern)   |  fcW [E][h] (gpt2)
//   W2   [h][E]   = downW (modern) | mpW (gpt2)
// Flat order: wte, wpe, lnf(g,b), then layers 0..L-1 (each contiguous), so the head bucket
// [0, head_end) and each layer are contiguous ranges for the gradient all-reduce.
#include <math.h>

#include <cmath>
#include <string>

#include "attention.cuh"
#include "gemm.cuh"
#include "model.cuh"
#include "model_kernels.cuh"
#include "ops.cuh"

using namespace turt;

namespace {

size_t align64(size_t x) { return (x + 63) & ~size_t(63); }

int mlp_hidden(const turt_config& c) {
  if (c.hidden > 0) return c.hidden;
  if (c.arch == TURT_ARCH_GPT2) return 4 * c.n_embd;
  // Math.max(64, Math.round((8 * nEmbd) / 3 / 64) * 64), src/models/gpt.ts:69-72
  double v = floor((8.0 * c.n_embd) / 3.0 / 64.0 + 0.5) * 64.0;
  return (int)(v < 64 ? 64 : v);
}

void build_layout(turt_model* m) {
  const int E = m->cfg.n_embd, V = m->cfg.vocab_size, T = m->cfg.block_size, h = m->hid;
  size_t p = 0;
  auto take = [&](size_t n) {
    size_t o = p;
    p = align64(p + n);
    return o;
  };
  m->wte = take((size_t)V * E);
  m->wpe = m->modern ? 0 : take((size_t)T * E);
  m->lnfg = take(E);
  m->lnfb = m->modern ? 0 : take(E);
  m->head_end = p;
  m->layers.resize(m->cfg.n_layer);
  for (auto& L : m->layers) {
    L.begin = p;
    L.ln1g = take(E);
    L.ln1b = m->modern ? 0 : take(E);
    L.wqkv = take((size_t)E * 3 * E);
    L.bqkv = m->modern ? 0 : take(3 * E);
    L.wproj = take((size_t)E * E);
    L.bproj = m->modern ? 0 : take(E);
    L.ln2g = take(E);
    L.ln2b = m->modern ? 0 : take(E);
    L.w1 = take((size_t)E * (m->modern ? 2 * h : h));
    L.b1 = m->modern ? 0 : take(h);
    L.w2 = take((size_t)h * E);
    L.b2 = m->modern ? 0 : take(E);
    L.end = p;
  }
  m->total = p;

  // parameters() order (src/models/gpu-gpt.ts:118-132) -> slots
  auto contig = [](const std::string& n, int r, int c, size_t off) {
    ParamSlot s;
    s.name = n;
    s.shape[0] = r;
    s.shape[1] = c;
    s.ndim = c ? 2 : 1;
    s.off = off;
    s.width = c ? r * c : r;
    s.rows = 1;
    s.pitch = s.width;
    return s;
  };
  auto block2d = [](const std::string& n, int r, int c, size_t off, int width, long rows, int pitch) {
    ParamSlot s;
    s.name = n;
    s.shape[0] = r;
    s.shape[1] = c;
    s.ndim = 2;
    s.off = off;
    s.width = width;
    s.rows = rows;
    s.pitch = pitch;
    return s;
  };
  auto& P = m->params;
  P.clear();
  P.push_back(contig("wte", V, E, m->wte));
  if (!m->modern) P.push_back(contig("wpe", T, E, m->wpe));
  for (int l = 0; l < m->cfg.n_layer; l++) {
    const LayerOff& L = m->layers[l];
    const std::string b = "blk" + std::to_string(l) + ".";
    P.push_back(contig(b + "ln1g", E, 0, L.ln1g));
    if (!m->modern) P.push_back(contig(b + "ln1b", E, 0, L.ln1b));
    P.push_back(block2d(b + "qW", E, E, L.wqkv, E, E, 3 * E));
    if (!m->modern) P.push_back(contig(b + "qb", E, 0, L.bqkv));
    P.push_back(block2d(b + "kW", E, E, L.wqkv + E, E, E, 3 * E));
    if (!m->modern) P.push_back(contig(b + "kb", E, 0, L.bqkv + E));
    P.push_back(block2d(b + "vW", E, E, L.wqkv + 2 * E, E, E, 3 * E));
    if (!m->modern) P.push_back(contig(b + "vb", E, 0, L.bqkv + 2 * E));
    P.push_back(contig(b + "projW", E, E, L.wproj));
    if (!m->modern) P.push_back(contig(b + "projb", E, 0, L.bproj));
    P.push_back(contig(b + "ln2g", E, 0, L.ln2g));
    if (!m->modern) P.push_back(contig(b + "ln2b", E, 0, L.ln2b));
    if (m->modern) {
      const long rows = (long)E * h / kGluBlock;
      P.push_back(block2d(b + "gateW", E, h, L.w1, kGluBlock, rows, 2 * kGluBlock));
      P.push_back(block2d(b + "upW", E, h, L.w1 + kGluBlock, kGluBlock, rows, 2 * kGluBlock));
      P.push_back(contig(b + "downW", h, E, L.w2));
    } else {
      P.push_back(contig(b + "fcW", E, h, L.w1));
      P.push_back(contig(b + "fcb", h, 0, L.b1));
      P.push_back(contig(b + "mpW", h, E, L.w2));
      P.push_back(contig(b + "mpb", E, 0, L.b2));
    }
  }
  P.push_back(contig("lnfg", E, 0, m->lnfg));
  if (!m->modern) P.push_back(contig("lnfb", E, 0, m->lnfb));
}

void free_workspace(turt_model* m) {
  if (m->ws) cudaFree(m->ws);
  m->ws = nullptr;
  m->capN = 0;
  m->capS = 0;
  m->act.clear();
}

// Attention path for B x T tokens: tensor-core (materialised scores) when allowed and the
// probabilities of every layer fit the budget, else the fused CUDA-core kernels.
constexpr size_t kAttnScoreBudget = (size_t)16 << 30;  // bytes

// Model GEMMs run on the tensor cores: FP32 (CUDA-core) precision applies to op-level calls only.
inline int mp(const turt_model* m) { return m->ctx->precision == 0 ? GEMM_TF32X3 : m->ctx->precision; }

// True when the tensor-core attention runs the online-softmax kernels (row log-sum-exp kept for
// the backward pass) instead of keeping [B*H][T][pitch] probabilities: on request, or by default
// for sequences longer than the single-pass fused kernels hold.
bool attention_online(const turt_model* m, int T) {
  const int hd = m->cfg.n_embd / m->cfg.n_head;
  if (m->attn_mode == TURT_ATTN_TENSOR_ONLINE) return true;
  return m->attn_mode != TURT_ATTN_FLASH && attention_tc_prefers_online(T, hd, mp(m));
}
bool attention_keeps_P(const turt_model* m, int T) { return !attention_online(m, T); }

bool use_tensor_attention(const turt_model* m, int B, int T) {
  const int hd = m->cfg.n_embd / m->cfg.n_head;
  if (m->attn_mode == TURT_ATTN_FLASH || !attention_tc_supported(hd)) return false;
  if (m->attn_mode == TURT_ATTN_TENSOR || m->attn_mode == TURT_ATTN_TENSOR_ONLINE || !attention_keeps_P(m, T))
    return true;
  const size_t bytes = (size_t)m->cfg.n_layer * B * m->cfg.n_head * T * attn_pitch(T) * 4;
  return bytes <= kAttnScoreBudget;
}

// Carves every activation / scratch buffer for N = B*T tokens out of one allocation.
int ensure_workspace(turt_model* m, int B, int T) {
  const int N = B * T;
  const bool tc = use_tensor_attention(m, B, T);
  const long S_need = tc && attention_keeps_P(m, T) ? (long)B * m->cfg.n_head * T * attn_pitch(T) : 0;
  if (N <= m->capN && B * m->cfg.n_head * T <= m->capB && tc == m->attn_tc && S_need <= m->capS) return OK;
  if (!tc && !attention_supported_hd(m->cfg.n_embd / m->cfg.n_head)) {
    set_error("fused CUDA-core attention supports head dim 16, 32 or 64; the tensor-core path is off or over budget");
    return ERR_UNSUPPORTED;
  }
  free_workspace(m);
  const int E = m->cfg.n_embd, H = m->cfg.n_head, V = m->cfg.vocab_size, h = m->hid, Lc = m->cfg.n_layer;
  const int W1 = m->modern ? 2 * h : h;
  size_t off = 0;
  std::vector<size_t*> dummy;
  auto take = [&](size_t n) {
    size_t o = off;
    off += (n * 4 + 255) & ~size_t(255);
    return o;
  };
  struct LA {
    size_t x, y1, rs1, mu1, qkv, att, lse, h, y2, rs2, mu2, pre, act, P, qr, kr;
  };
  const bool rope = m->modern;
  std::vector<LA> la(Lc);
  const size_t NE = (size_t)N * E, BHT = (size_t)B * H * T;
  for (int l = 0; l < Lc; l++) {
    LA& a = la[l];
    a.x = take(NE);
    a.y1 = take(NE);
    a.rs1 = take(N);
    a.mu1 = m->modern ? 0 : take(N);
    a.qkv = take(3 * NE);
    a.att = take(NE);
    a.lse = take(BHT);
    a.h = take(NE);
    a.y2 = take(NE);
    a.rs2 = take(N);
    a.mu2 = m->modern ? 0 : take(N);
    a.pre = take((size_t)N * W1);
    a.act = take((size_t)N * h);
    a.P = S_need ? take((size_t)S_need) : 0;
    a.qr = tc && rope ? take(NE) : 0;
    a.kr = tc && rope ? take(NE) : 0;
  }
  size_t xL = take(NE), yf = take(NE), rsf = take(N), muf = take(N);
  size_t logits = take((size_t)N * V), loss_rows = take(N);
  size_t dx = take(NE), dy = take(NE), datt = take(NE), dqkv = take(3 * NE), dpre = take((size_t)N * W1);
  size_t Dsc = take(BHT);
  size_t dS = S_need ? take((size_t)S_need) : 0;
  size_t dact = rope ? take((size_t)N * h) : 0;
  const int C = 3 * E > W1 ? 3 * E : W1;
  size_t part = take((size_t)2 * norm_parts(N) * (C > E ? C : E));
  size_t ids = take(N), tgt = take(N);
  void* ws = nullptr;
  TURT_CHECK_CUDA(cudaMalloc(&ws, off));
  m->ws = ws;
  char* base = static_cast<char*>(ws);
  auto F = [&](size_t o) { return reinterpret_cast<float*>(base + o); };
  m->act.resize(Lc);
  for (int l = 0; l < Lc; l++) {
    LA& a = la[l];
    LayerAct& A = m->act[l];
    A.x = F(a.x);
    A.y1 = F(a.y1);
    A.rs1 = F(a.rs1);
    A.mu1 = m->modern ? nullptr : F(a.mu1);
    A.qkv = F(a.qkv);
    A.att = F(a.att);
    A.lse = F(a.lse);
    A.h = F(a.h);
    A.y2 = F(a.y2);
    A.rs2 = F(a.rs2);
    A.mu2 = m->modern ? nullptr : F(a.mu2);
    A.pre = F(a.pre);
    A.act = F(a.act);
    A.P = S_need ? F(a.P) : nullptr;
    A.qr = tc && rope ? F(a.qr) : nullptr;
    A.kr = tc && rope ? F(a.kr) : nullptr;
  }
  m->xL = F(xL);
  m->yf = F(yf);
  m->rsf = F(rsf);
  m->muf = F(muf);
  m->logits = F(logits);
  m->loss_rows = F(loss_rows);
  m->dx = F(dx);
  m->dy = F(dy);
  m->datt = F(datt);
  m->dqkv = F(dqkv);
  m->dpre = F(dpre);
  m->Dsc = F(Dsc);
  m->dS = S_need ? F(dS) : nullptr;
  m->dact = rope ? F(dact) : nullptr;
  m->part = F(part);
  m->d_ids = reinterpret_cast<uint32_t*>(base + ids);
  m->d_tgt = reinterpret_cast<uint32_t*>(base + tgt);
  if (m->h_ids) cudaFreeHost(m->h_ids);
  if (m->h_tgt) cudaFreeHost(m->h_tgt);
  TURT_CHECK_CUDA(cudaMallocHost(&m->h_ids, (size_t)N * 4));
  TURT_CHECK_CUDA(cudaMallocHost(&m->h_tgt, (size_t)N * 4));
  m->capN = N;
  m->capB = B * H * T;
  m->capS = S_need;
  m->attn_tc = tc;
  return OK;
}

// ---------------------------------------------------------------- GEMM helpers
inline GemmOperand opK(const float* p, long ld) { return GemmOperand{p, ld, 0, false}; }   // stored [rows][K]
inline GemmOperand opMN(const float* p, long ld) { return GemmOperand{p, ld, 0, true}; }  // stored [K][rows]
inline GemmEpi epi(int kind, float* C, long ldc) {
  GemmEpi e;
  e.kind = kind;
  e.C = C;
  e.ldc = ldc;
  return e;
}

int stage_tokens(turt_model* m, const uint32_t* ids, const uint32_t* tgt, int N) {
  cudaStream_t st = m->ctx->stream;
  // Copy through pinned staging so the H2D transfer is a true async DMA on the stream.
  TURT_CHECK_CUDA(cudaStreamSynchronize(st));
  memcpy(m->h_ids, ids, (size_t)N * 4);
  memcpy(m->h_tgt, tgt, (size_t)N * 4);
  TURT_CHECK_CUDA(cudaMemcpyAsync(m->d_ids, m->h_ids, (size_t)N * 4, cudaMemcpyHostToDevice, st));
  TURT_CHECK_CUDA(cudaMemcpyAsync(m->d_tgt, m->h_tgt, (size_t)N * 4, cudaMemcpyHostToDevice, st));
  return OK;
}

int forward(turt_model* m, int B, int T, bool train, float loss_scale, bool logits_only = false) {
  cudaStream_t st = m->ctx->stream;
  int* flags = m->ctx->flags;
  const int N = B * T, E = m->cfg.n_embd, H = m->cfg.n_head, hd = E / H, V = m->cfg.vocab_size, h = m->hid;
  const float* P = m->P;
  RC(embed_fwd(st, P + m->wte, m->modern ? nullptr : P + m->wpe, m->d_ids, m->act.empty() ? m->xL : m->act[0].x, N, T,
               E, V, flags));
  for (int l = 0; l < m->cfg.n_layer; l++) {
    const LayerOff& L = m->layers[l];
    LayerAct& a = m->act[l];
    float* xnext = (l + 1 < m->cfg.n_layer) ? m->act[l + 1].x : m->xL;
    if (m->modern)
      RC(rms_fwd(st, a.x, P + L.ln1g, a.y1, a.rs1, N, E, m->eps));
    else
      RC(ln_fwd(st, a.x, P + L.ln1g, P + L.ln1b, a.y1, a.mu1, a.rs1, N, E, m->eps));
    GemmEpi e = epi(m->modern ? EPI_STORE : EPI_BIAS, a.qkv, 3 * E);
    if (!m->modern) e.bias = P + L.bqkv;
    const bool rope_epi = m->modern && m->attn_tc;  // q, k rotated straight into the head-major copies
    if (rope_epi) {
      e.kind = EPI_QKV_ROPE;
      e.rope = m->rope_cs;
      e.rope_T = T;
      e.rope_H = H;
      e.rope_hd = hd;
      e.qr = a.qr;
      e.kr = a.kr;
    }
    RC(gemm_tf32(st, N, 3 * E, E, 1, opK(a.y1, E), opMN(P + L.wqkv, 3 * E), e, flags, mp(m)));
    if (m->attn_tc) {
      AttnTensors at{a.P, a.qr, a.kr, a.lse, attention_online(m, T)};
      RC(attention_tc_fwd(st, a.qkv, m->rope_cs, a.att, at, B, T, H, hd, m->modern ? 1 : 0, rope_epi ? 1 : 0, flags,
                          mp(m)));
    } else {
      RC(attention_fwd(st, a.qkv, m->rope_cs, a.att, a.lse, B, T, H, hd, m->modern ? 1 : 0));
    }
    e = epi(EPI_ADD_RES, a.h, E);
    e.R = a.x;
    e.ldr = E;
    if (!m->modern) e.bias = P + L.bproj;
    RC(gemm_tf32(st, N, E, E, 1, opK(a.att, E), opMN(P + L.wproj, E), e, flags, mp(m)));
    if (m->modern)
      RC(rms_fwd(st, a.h, P + L.ln2g, a.y2, a.rs2, N, E, m->eps));
    else
      RC(ln_fwd(st, a.h, P + L.ln2g, P + L.ln2b, a.y2, a.mu2, a.rs2, N, E, m->eps));
    if (m->modern) {
      e = epi(EPI_SWIGLU_FWD, a.pre, 2 * h);
      e.C2 = a.act;
      e.ldc2 = h;
      RC(gemm_tf32(st, N, 2 * h, E, 1, opK(a.y2, E), opMN(P + L.w1, 2 * h), e, flags, mp(m)));
    } else {
      e = epi(EPI_BIAS_GELU, a.pre, h);
      e.bias = P + L.b1;
      e.C2 = a.act;
      e.ldc2 = h;
      RC(gemm_tf32(st, N, h, E, 1, opK(a.y2, E), opMN(P + L.w1, h), e, flags, mp(m)));
    }
    e = epi(EPI_ADD_RES, xnext, E);
    e.R = a.h;
    e.ldr = E;
    if (!m->modern) e.bias = P + L.b2;
    RC(gemm_tf32(st, N, E, h, 1, opK(a.act, h), opMN(P + L.w2, E), e, flags, mp(m)));
  }
  if (m->modern)
    RC(rms_fwd(st, m->xL, P + m->lnfg, m->yf, m->rsf, N, E, m->eps));
  else
    RC(ln_fwd(st, m->xL, P + m->lnfg, P + m->lnfb, m->yf, m->muf, m->rsf, N, E, m->eps));
  // tied head: logits = yf * wte^T (wte [V][E] is the K-major B operand)
  RC(gemm_tf32(st, N, V, E, 1, opK(m->yf, E), opK(P + m->wte, E), epi(EPI_STORE, m->logits, V), flags, mp(m)));
  if (logits_only) return OK;
  if (train)
    RC(ce_fused(st, m->logits, m->d_tgt, m->loss_rows, N, V, loss_scale / (float)N, flags));
  else
    RC(ce_loss(st, m->logits, m->d_tgt, m->loss_rows, N, V, flags));
  RC(loss_mean(st, m->loss_rows, N, m->loss_dev, flags));
  return OK;
}

}  // namespace

int turt::stream_join(turt_model* m, cudaStream_t from, cudaStream_t to) {
  cudaEvent_t e = m->wg_ring[m->wg_next++ % 16];
  TURT_CHECK_CUDA(cudaEventRecord(e, from));
  TURT_CHECK_CUDA(cudaStreamWaitEvent(to, e, 0));
  return OK;
}

int turt::grad_writes_stream(turt_model* m, cudaStream_t* out) {
  RC(stream_join(m, m->ctx->stream, m->wg));
  *out = m->wg;
  return OK;
}

namespace {

int backward(turt_model* m, int B, int T) {
  cudaStream_t st = m->ctx->stream, wg = m->wg;
  int* flags = m->ctx->flags;
  const int N = B * T, E = m->cfg.n_embd, H = m->cfg.n_head, hd = E / H, V = m->cfg.vocab_size, h = m->hid;
  const float* P = m->P;
  float* G = m->G;
  // Weight-gradient GEMMs (dW = X^T dY) are forked onto `wg` as soon as dY exists.  The main
  // stream waits for them only where it overwrites a buffer they read: dx (updated in place by
  // the norm backward), dpre and dqkv (reused by the next layer), and the wte gradient (the
  // embedding backward accumulates into it).  mark[0]: after dW2 (reads dx), mark[1]: after
  // dW1 (reads dpre), mark[2]: after dWproj (reads dx), mark[3]: after dWqkv (reads dqkv).
  cudaEvent_t* mark = m->wg_mark;
  bool pending[4] = {false, false, false, false};
  auto fork = [&]() { return stream_join(m, st, wg); };
  auto set_mark = [&](int i) -> int {
    TURT_CHECK_CUDA(cudaEventRecord(mark[i], wg));
    pending[i] = true;
    return OK;
  };
  auto wait_mark = [&](int i) -> int {
    if (pending[i]) TURT_CHECK_CUDA(cudaStreamWaitEvent(st, mark[i], 0));
    pending[i] = false;
    return OK;
  };
  // head: dyf = dlogits * wte ; dwte += dlogits^T * yf
  RC(gemm_tf32(st, N, E, V, 1, opK(m->logits, V), opMN(P + m->wte, E), epi(EPI_STORE, m->dy, E), flags, mp(m)));
  RC(fork());
  RC(gemm_tf32(wg, V, E, N, 1, opMN(m->logits, V), opMN(m->yf, E), epi(EPI_ACCUM, G + m->wte, E), flags, mp(m)));
  if (m->modern)
    RC(rms_bwd(st, m->xL, m->dy, P + m->lnfg, m->rsf, nullptr, m->dx, G + m->lnfg, m->part, N, E));
  else
    RC(ln_bwd(st, m->xL, m->dy, P + m->lnfg, m->muf, m->rsf, nullptr, m->dx, G + m->lnfg, G + m->lnfb, m->part, N, E));
  for (int l = m->cfg.n_layer - 1; l >= 0; l--) {
    const LayerOff& L = m->layers[l];
    LayerAct& a = m->act[l];
    // ---- MLP
    RC(wait_mark(1));  // dpre is rewritten below; the previous layer's dW1 reads it
    if (m->modern) {
      // d(act) = dx W2^T, then the coalesced elementwise SwiGLU backward into dpre (a fused
      // epilogue reads and writes the gate|up rows one row per lane and measured slower)
      RC(gemm_tf32(st, N, h, E, 1, opK(m->dx, E), opK(P + L.w2, E), epi(EPI_STORE, m->dact, h), flags, mp(m)));
      RC(swiglu_bwd_interleaved(st, m->dact, a.pre, m->dpre, N, h));
      RC(fork());
      RC(gemm_tf32(wg, h, E, N, 1, opMN(a.act, h), opMN(m->dx, E), epi(EPI_ACCUM, G + L.w2, E), flags, mp(m)));
      RC(set_mark(0));
      RC(gemm_tf32(st, N, E, 2 * h, 1, opK(m->dpre, 2 * h), opK(P + L.w1, 2 * h), epi(EPI_STORE, m->dy, E), flags, mp(m)));
      RC(fork());
      RC(gemm_tf32(wg, E, 2 * h, N, 1, opMN(a.y2, E), opMN(m->dpre, 2 * h), epi(EPI_ACCUM, G + L.w1, 2 * h), flags,
                   mp(m)));
      RC(set_mark(1));
    } else {
      GemmEpi e = epi(EPI_GELU_BWD, m->dpre, h);
      e.R = a.pre;
      e.ldr = h;
      RC(gemm_tf32(st, N, h, E, 1, opK(m->dx, E), opK(P + L.w2, E), e, flags, mp(m)));
      RC(fork());
      RC(gemm_tf32(wg, h, E, N, 1, opMN(a.act, h), opMN(m->dx, E), epi(EPI_ACCUM, G + L.w2, E), flags, mp(m)));
      RC(set_mark(0));
      RC(colsum_accum(st, m->dx, N, E, G + L.b2, m->part));
      RC(gemm_tf32(st, N, E, h, 1, opK(m->dpre, h), opK(P + L.w1, h), epi(EPI_STORE, m->dy, E), flags, mp(m)));
      RC(fork());
      RC(gemm_tf32(wg, E, h, N, 1, opMN(a.y2, E), opMN(m->dpre, h), epi(EPI_ACCUM, G + L.w1, h), flags, mp(m)));
      RC(set_mark(1));
      RC(colsum_accum(st, m->dpre, N, h, G + L.b1, m->part));
    }
    RC(wait_mark(0));  // dx is rewritten in place below; dW2 reads it
    if (m->modern)
      RC(rms_bwd(st, a.h, m->dy, P + L.ln2g, a.rs2, m->dx, m->dx, G + L.ln2g, m->part, N, E));
    else
      RC(ln_bwd(st, a.h, m->dy, P + L.ln2g, a.mu2, a.rs2, m->dx, m->dx, G + L.ln2g, G + L.ln2b, m->part, N, E));
    // ---- attention
    RC(gemm_tf32(st, N, E, E, 1, opK(m->dx, E), opK(P + L.wproj, E), epi(EPI_STORE, m->datt, E), flags, mp(m)));
    RC(fork());
    RC(gemm_tf32(wg, E, E, N, 1, opMN(a.att, E), opMN(m->dx, E), epi(EPI_ACCUM, G + L.wproj, E), flags, mp(m)));
    RC(set_mark(2));
    if (!m->modern) RC(colsum_accum(st, m->dx, N, E, G + L.bproj, m->part));
    RC(wait_mark(3));  // dqkv is rewritten below; the previous layer's dWqkv reads it
    if (m->attn_tc) {
      AttnTensors at{a.P, a.qr, a.kr, a.lse, attention_online(m, T)};
      AttnScratch sc{m->dS, m->Dsc};
      RC(attention_tc_bwd(st, a.qkv, m->rope_cs, a.att, m->datt, at, sc, m->dqkv, B, T, H, hd, m->modern ? 1 : 0, flags,
                          mp(m)));
    } else {
      RC(attention_bwd(st, a.qkv, m->rope_cs, a.att, m->datt, a.lse, m->Dsc, m->dqkv, B, T, H, hd,
                       m->modern ? 1 : 0));
    }
    if (!m->modern) RC(colsum_accum(st, m->dqkv, N, 3 * E, G + L.bqkv, m->part));
    RC(gemm_tf32(st, N, E, 3 * E, 1, opK(m->dqkv, 3 * E), opK(P + L.wqkv, 3 * E), epi(EPI_STORE, m->dy, E), flags, mp(m)));
    RC(fork());
    RC(gemm_tf32(wg, E, 3 * E, N, 1, opMN(a.y1, E), opMN(m->dqkv, 3 * E), epi(EPI_ACCUM, G + L.wqkv, 3 * E), flags,
                 mp(m)));
    RC(set_mark(3));
    RC(wait_mark(2));  // dx is rewritten in place below; dWproj reads it
    if (m->modern)
      RC(rms_bwd(st, a.x, m->dy, P + L.ln1g, a.rs1, m->dx, m->dx, G + L.ln1g, m->part, N, E));
    else
      RC(ln_bwd(st, a.x, m->dy, P + L.ln1g, a.mu1, a.rs1, m->dx, m->dx, G + L.ln1g, G + L.ln1b, m->part, N, E));
    if (dp_active(m) && !m->dp_defer) RC(dp_after_layer(m, l));
  }
  // the embedding backward accumulates into the wte gradient that the head's dW GEMM (on wg)
  // writes, and the next forward rewrites the activations the weight-gradient GEMMs read
  RC(stream_join(m, wg, st));
  RC(embed_bwd(st, m->dx, m->d_ids, G + m->wte, m->modern ? nullptr : G + m->wpe, N, T, E, V));
  if (dp_active(m) && !m->dp_defer) {
    RC(dp_after_head(m));
    RC(dp_finish(m));
  }
  return OK;
}

int read_loss(turt_model* m, float* loss_out) {
  if (!loss_out) return OK;
  TURT_CHECK_CUDA(cudaMemcpyAsync(m->h_loss, m->loss_dev, 4, cudaMemcpyDeviceToHost, m->ctx->stream));
  int rc = ctx_check_flags(m->ctx);  // synchronizes
  *loss_out = *m->h_loss;
  return rc;
}

int check_batch(turt_model* m, const uint32_t* ids, const uint32_t* tgt, int b, int t) {
  TURT_REQUIRE(m && ids && tgt, "null model or token array");
  TURT_REQUIRE(b > 0 && t > 0, "batch and time must be positive");
  if (t > m->cfg.block_size) {
    set_error("Sequence length " + std::to_string(t) + " exceeds block size " + std::to_string(m->cfg.block_size));
    return ERR_INVALID;
  }
  return OK;
}

}  // namespace

int turt::model_forward_logits(turt_model* m, const uint32_t* ids, int t) {
  RC(check_batch(m, ids, ids, 1, t));
  RC(ensure_workspace(m, 1, t));
  RC(stage_tokens(m, ids, ids, t));
  return forward(m, 1, t, false, 1.0f, true);
}

#define MODEL_GUARD(m)                                   \
  do {                                                   \
    if (!(m)) {                                          \
      set_error("null model");                           \
      return ERR_INVALID;                                \
    }                                                    \
    TURT_CHECK_CUDA(cudaSetDevice((m)->ctx->device));    \
  } while (0)

extern "C" {

int turt_model_create(turt_ctx* ctx, const turt_config* cfg, turt_model** out) {
  TURT_REQUIRE(ctx && cfg && out, "turt_model_create: null argument");
  TURT_REQUIRE(cfg->vocab_size > 0 && cfg->block_size > 0 && cfg->n_layer > 0 && cfg->n_head > 0 && cfg->n_embd > 0,
               "turt_model_create: non-positive dimension");
  if (cfg->n_embd % cfg->n_head != 0) {
    set_error("nEmbd (" + std::to_string(cfg->n_embd) + ") must be divisible by nHead (" +
              std::to_string(cfg->n_head) + ")");
    return ERR_INVALID;
  }
  TURT_REQUIRE(cfg->arch == TURT_ARCH_GPT2 || cfg->arch == TURT_ARCH_MODERN, "arch must be gpt2 (0) or modern (1)");
  const int hd = cfg->n_embd / cfg->n_head;
  if (!attention_supported_hd(hd) && !attention_tc_supported(hd)) {
    set_error("head dim " + std::to_string(hd) + " not supported (a multiple of 16 up to 256)");
    return ERR_UNSUPPORTED;
  }
  TURT_REQUIRE(cfg->n_embd % 32 == 0 && cfg->n_embd <= 1024, "nEmbd must be a multiple of 32, at most 1024");
  TURT_REQUIRE(cfg->vocab_size % 4 == 0, "vocab size must be a multiple of 4");
  TURT_CHECK_CUDA(cudaSetDevice(ctx->device));
  turt_model* m = new turt_model();
  m->ctx = ctx;
  m->cfg = *cfg;
  m->modern = cfg->arch == TURT_ARCH_MODERN;
  m->hid = mlp_hidden(*cfg);
  if (m->hid % kGluBlock != 0) {
    delete m;
    set_error("MLP hidden width must be a multiple of 32");
    return ERR_UNSUPPORTED;
  }
  build_layout(m);
  const size_t bytes = m->total * 4;
  TURT_CHECK_CUDA(cudaMalloc(&m->P, bytes));
  TURT_CHECK_CUDA(cudaMalloc(&m->G, bytes));
  TURT_CHECK_CUDA(cudaMalloc(&m->M, bytes));
  TURT_CHECK_CUDA(cudaMalloc(&m->V, bytes));
  cudaStream_t st = ctx->stream;
  TURT_CHECK_CUDA(cudaMemsetAsync(m->P, 0, bytes, st));
  TURT_CHECK_CUDA(cudaMemsetAsync(m->G, 0, bytes, st));
  TURT_CHECK_CUDA(cudaMemsetAsync(m->M, 0, bytes, st));
  TURT_CHECK_CUDA(cudaMemsetAsync(m->V, 0, bytes, st));
  // gains start at 1 (src/nn/rmsnorm.ts:21, layernorm.ts:22); weights arrive via turt_param_upload
  const int E = cfg->n_embd;
  op_fill(st, m->P + m->lnfg, 1.0f, E);
  for (auto& L : m->layers) {
    op_fill(st, m->P + L.ln1g, 1.0f, E);
    op_fill(st, m->P + L.ln2g, 1.0f, E);
  }
  const int hdim = E / cfg->n_head;
  TURT_CHECK_CUDA(cudaMalloc(&m->rope_cs, sizeof(float2) * (size_t)cfg->block_size * (hdim / 2) + 16));
  RC(op_rope_table(st, m->rope_cs, cfg->block_size, hdim, 10000.0));
  TURT_CHECK_CUDA(cudaMalloc(&m->loss_dev, 16));
  TURT_CHECK_CUDA(cudaMalloc(&m->coef_dev, 16));
  TURT_CHECK_CUDA(cudaMalloc(&m->norm_dev, 16));
  TURT_CHECK_CUDA(cudaMalloc(&m->norm_scratch, sizeof(double) * norm_scratch_doubles()));
  TURT_CHECK_CUDA(cudaMallocHost(&m->h_loss, 16));
  TURT_CHECK_CUDA(cudaStreamCreateWithFlags(&m->wg, cudaStreamNonBlocking));
  for (auto& e : m->wg_ring) TURT_CHECK_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  for (auto& e : m->wg_mark) TURT_CHECK_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  TURT_CHECK_CUDA(cudaStreamSynchronize(st));
  *out = m;
  return OK;
}

int turt_model_set_attention(turt_model* m, int mode) {
  TURT_REQUIRE(m, "null model");
  TURT_REQUIRE(mode >= TURT_ATTN_AUTO && mode <= TURT_ATTN_TENSOR_ONLINE,
               "attention mode must be 0 (auto), 1 (tensor), 2 (flash) or 3 (tensor online)");
  const int hd = m->cfg.n_embd / m->cfg.n_head;
  if (mode == TURT_ATTN_TENSOR) TURT_REQUIRE(attention_tc_supported(hd), "tensor-core attention needs hd % 16 == 0");
  if (mode == TURT_ATTN_TENSOR_ONLINE)
    TURT_REQUIRE(attention_flash_supported(1, hd), "online-softmax tensor-core attention needs hd of 32 or 64");
  if (mode == TURT_ATTN_FLASH) TURT_REQUIRE(attention_supported_hd(hd), "flash attention needs hd of 16, 32 or 64");
  m->attn_mode = mode;
  return OK;
}

int turt_model_destroy(turt_model* m) {
  MODEL_GUARD(m);
  cudaStreamSynchronize(m->ctx->stream);
  if (m->wg) {
    cudaStreamSynchronize(m->wg);
    gemm_release_stream(m->wg);
    cudaStreamDestroy(m->wg);
  }
  for (auto& e : m->wg_ring)
    if (e) cudaEventDestroy(e);
  for (auto& e : m->wg_mark)
    if (e) cudaEventDestroy(e);
  if (m->dp) turt_dp_destroy(m);
  free_workspace(m);
  cudaFree(m->P);
  cudaFree(m->G);
  cudaFree(m->M);
  cudaFree(m->V);
  cudaFree(m->rope_cs);
  cudaFree(m->loss_dev);
  cudaFree(m->coef_dev);
  cudaFree(m->norm_dev);
  cudaFree(m->norm_scratch);
  if (m->kcache) cudaFree(m->kcache);
  if (m->vcache) cudaFree(m->vcache);
  if (m->dec) cudaFree(m->dec);
  if (m->dec_tok) cudaFree(m->dec_tok);
  if (m->h_dec_tok) cudaFreeHost(m->h_dec_tok);
  if (m->dec_graph) cudaGraphExecDestroy(m->dec_graph);
  if (m->dec_cap) cudaStreamDestroy(m->dec_cap);
  cudaFreeHost(m->h_loss);
  if (m->h_ids) cudaFreeHost(m->h_ids);
  if (m->h_tgt) cudaFreeHost(m->h_tgt);
  delete m;
  return OK;
}

int turt_param_count(turt_model* m, int* count) {
  MODEL_GUARD(m);
  *count = (int)m->params.size();
  return OK;
}

int turt_num_params(turt_model* m, size_t* total) {
  MODEL_GUARD(m);
  size_t s = 0;
  for (auto& p : m->params) s += p.count();
  *total = s;
  return OK;
}

int turt_param_info(turt_model* m, int i, char* name, int cap, int* shape2, int* ndim) {
  MODEL_GUARD(m);
  TURT_REQUIRE(i >= 0 && i < (int)m->params.size(), "param index out of range");
  const ParamSlot& s = m->params[i];
  if (name && cap > 0) {
    snprintf(name, cap, "%s", s.name.c_str());
  }
  if (shape2) {
    shape2[0] = s.shape[0];
    shape2[1] = s.shape[1];
  }
  if (ndim) *ndim = s.ndim;
  return OK;
}

// Which flat buffer a per-parameter copy addresses.
enum ParamBuf { BUF_PARAM = 0, BUF_GRAD = 1, BUF_ADAM_M = 2, BUF_ADAM_V = 3 };

static int copy_param(turt_model* m, int i, float* host, size_t n, bool up, int which) {
  MODEL_GUARD(m);
  TURT_REQUIRE(i >= 0 && i < (int)m->params.size(), "param index out of range");
  TURT_REQUIRE(host, "null host array");
  const ParamSlot& s = m->params[i];
  if (n != s.count()) {
    set_error("param " + std::to_string(i) + " size mismatch: expected " + std::to_string(s.count()) + ", got " +
              std::to_string(n));
    return ERR_INVALID;
  }
  float* base = which == BUF_GRAD ? m->G : which == BUF_ADAM_M ? m->M : which == BUF_ADAM_V ? m->V : m->P;
  float* dev = base + s.off;
  cudaStream_t st = m->ctx->stream;
  if (up)
    TURT_CHECK_CUDA(cudaMemcpy2DAsync(dev, (size_t)s.pitch * 4, host, (size_t)s.width * 4, (size_t)s.width * 4, s.rows,
                                      cudaMemcpyHostToDevice, st));
  else
    TURT_CHECK_CUDA(cudaMemcpy2DAsync(host, (size_t)s.width * 4, dev, (size_t)s.pitch * 4, (size_t)s.width * 4, s.rows,
                                      cudaMemcpyDeviceToHost, st));
  TURT_CHECK_CUDA(cudaStreamSynchronize(st));
  return OK;
}

int turt_param_upload(turt_model* m, int i, const float* host, size_t n) {
  return copy_param(m, i, const_cast<float*>(host), n, true, BUF_PARAM);
}
int turt_param_download(turt_model* m, int i, float* host, size_t n) {
  return copy_param(m, i, host, n, false, BUF_PARAM);
}
int turt_grad_download(turt_model* m, int i, float* host, size_t n) { return copy_param(m, i, host, n, false, BUF_GRAD); }
int turt_adam_state_download(turt_model* m, int i, float* mom1, float* mom2, size_t n) {
  RC(copy_param(m, i, mom1, n, false, BUF_ADAM_M));
  return copy_param(m, i, mom2, n, false, BUF_ADAM_V);
}
int turt_adam_state_upload(turt_model* m, int i, const float* mom1, const float* mom2, size_t n) {
  RC(copy_param(m, i, const_cast<float*>(mom1), n, true, BUF_ADAM_M));
  return copy_param(m, i, const_cast<float*>(mom2), n, true, BUF_ADAM_V);
}

// mulberry32 (src/math/random.ts:8-17): the uint32 state advances by 0x6d2b79f5 and is
// mixed by two wrapping multiplies; the draw is the mixed word / 2^32.
static double mulberry32_next(uint32_t* state) {
  *state += 0x6d2b79f5u;
  uint32_t t = *state;
  t = (t ^ (t >> 15)) * (t | 1u);
  t ^= t + (t ^ (t >> 7)) * (t | 61u);
  return (double)(t ^ (t >> 14)) / 4294967296.0;
}

// Box-Muller over mulberry32, redrawing u while it is 0 (src/math/random.ts:20-25).
static double gaussian_next(uint32_t* state) {
  double u = 0.0;
  while (u == 0.0) u = mulberry32_next(state);
  const double v = mulberry32_next(state);
  return std::sqrt(-2.0 * std::log(u)) * std::cos(2.0 * M_PI * v);
}

// The reference's CPU constructor GPT(config, rng) draws, in parameters() order, every weight
// matrix as Float32(gaussian(rng) * std) (Tensor.randn, src/math/tensor.ts:83-88): std 0.02
// (INIT_STD) for wte, wpe, q, k, v, gate, up, fc and 0.02 / sqrt(2 nLayer) for the residual
// projections proj, down, mp (src/models/gpt.ts:97-102,154-155,182-184,225-239); norm gains
// are 1 and biases 0 (no draws).  The draws run on the host, then each tensor is uploaded.
int turt_model_init(turt_model* m, uint32_t seed) {
  MODEL_GUARD(m);
  uint32_t state = seed;
  const double std0 = 0.02, std_res = 0.02 / std::sqrt(2.0 * m->cfg.n_layer);
  std::vector<float> buf;
  for (int i = 0; i < (int)m->params.size(); i++) {
    const ParamSlot& s = m->params[i];
    const std::string& n = s.name;
    const std::string leaf = n.substr(n.rfind('.') + 1);
    buf.assign(s.count(), 0.0f);
    if (s.ndim == 2) {
      const bool residual = leaf == "projW" || leaf == "downW" || leaf == "mpW";
      const double sd = residual ? std_res : std0;
      for (size_t j = 0; j < buf.size(); j++) buf[j] = (float)(gaussian_next(&state) * sd);
    } else if (leaf.back() == 'g') {
      std::fill(buf.begin(), buf.end(), 1.0f);  // norm gain
    }
    RC(copy_param(m, i, buf.data(), buf.size(), true, BUF_PARAM));
  }
  return OK;
}

int turt_zero_grad(turt_model* m) {
  MODEL_GUARD(m);
  TURT_CHECK_CUDA(cudaMemsetAsync(m->G, 0, m->total * 4, m->ctx->stream));
  return OK;
}

int turt_forward_backward(turt_model* m, const uint32_t* ids, const uint32_t* tgt, int b, int t, float loss_scale,
                          float* loss_out) {
  MODEL_GUARD(m);
  RC(check_batch(m, ids, tgt, b, t));
  RC(ensure_workspace(m, b, t));
  RC(stage_tokens(m, ids, tgt, b * t));
  RC(forward(m, b, t, true, loss_scale));
  RC(backward(m, b, t));
  return read_loss(m, loss_out);
}

int turt_forward_backward_device(turt_model* m, const uint32_t* d_ids, const uint32_t* d_tgt, int b, int t,
                                 float loss_scale) {
  MODEL_GUARD(m);
  RC(check_batch(m, d_ids, d_tgt, b, t));
  RC(ensure_workspace(m, b, t));
  cudaStream_t st = m->ctx->stream;
  TURT_CHECK_CUDA(cudaMemcpyAsync(m->d_ids, d_ids, (size_t)b * t * 4, cudaMemcpyDeviceToDevice, st));
  TURT_CHECK_CUDA(cudaMemcpyAsync(m->d_tgt, d_tgt, (size_t)b * t * 4, cudaMemcpyDeviceToDevice, st));
  RC(forward(m, b, t, true, loss_scale));
  return backward(m, b, t);
}

int turt_read_loss(turt_model* m, float* loss_out) {
  MODEL_GUARD(m);
  TURT_REQUIRE(loss_out, "null loss_out");
  return read_loss(m, loss_out);
}

int turt_forward(turt_model* m, const uint32_t* ids, const uint32_t* tgt, int b, int t, float* loss_out) {
  MODEL_GUARD(m);
  RC(check_batch(m, ids, tgt, b, t));
  RC(ensure_workspace(m, b, t));
  RC(stage_tokens(m, ids, tgt, b * t));
  RC(forward(m, b, t, false, 1.0f));
  return read_loss(m, loss_out);
}

int turt_forward_device(turt_model* m, const uint32_t* d_ids, const uint32_t* d_tgt, int b, int t, float* loss_out) {
  MODEL_GUARD(m);
  RC(check_batch(m, d_ids, d_tgt, b, t));
  TURT_REQUIRE(loss_out, "null loss_out");
  RC(ensure_workspace(m, b, t));
  cudaStream_t st = m->ctx->stream;
  TURT_CHECK_CUDA(cudaMemcpyAsync(m->d_ids, d_ids, (size_t)b * t * 4, cudaMemcpyDeviceToDevice, st));
  TURT_CHECK_CUDA(cudaMemcpyAsync(m->d_tgt, d_tgt, (size_t)b * t * 4, cudaMemcpyDeviceToDevice, st));
  RC(forward(m, b, t, false, 1.0f));
  return read_loss(m, loss_out);
}

int turt_clip_grad_norm(turt_model* m, double max_norm, double* norm_out) {
  MODEL_GUARD(m);
  cudaStream_t st = m->ctx->stream;
  RC(grad_norm(st, m->G, m->total, 1.0f, (float)max_norm, m->norm_scratch, m->norm_dev, m->coef_dev, m->ctx->flags));
  RC(scale_by(st, m->G, m->total, m->coef_dev, 1.0f));
  if (norm_out) {
    TURT_CHECK_CUDA(cudaMemcpyAsync(norm_out, m->norm_dev, 8, cudaMemcpyDeviceToHost, st));
    TURT_CHECK_CUDA(cudaStreamSynchronize(st));
  }
  return OK;
}

int turt_adamw_step(turt_model* m, float lr, float b1, float b2, float eps, float wd, float bc1, float bc2, float clip,
                    float grad_scale) {
  MODEL_GUARD(m);
  cudaStream_t st = m->ctx->stream;
  const float* coef = nullptr;
  if (clip > 0.f) {
    RC(grad_norm(st, m->G, m->total, grad_scale, clip, m->norm_scratch, m->norm_dev, m->coef_dev, m->ctx->flags));
    coef = m->coef_dev;
  }
  return adamw_flat(st, m->P, m->G, m->M, m->V, m->total, lr, b1, b2, eps, wd, bc1, bc2, grad_scale, coef);
}

}  // extern "C"
