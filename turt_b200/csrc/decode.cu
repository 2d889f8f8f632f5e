// decode.cu -- autoregressive generation on the GPU with a KV cache.
//
// The reference samples continuations with GPT.generate (src/models/gpt.ts:291-321): every new
// token re-runs the full forward over the last blockSize tokens and samples from the final
// position's logits.  While the context still fits the block, positions never shift, so the
// keys and values of earlier positions do not change: they are cached per layer and each new
// token costs one decode step (M = 1: fp32 GEMVs on the CUDA cores, the weights being L2
// resident).  turt_generate_prefill runs the ordinary forward over a prompt (or, once the window
// slides, over the cropped window) and refills the cache; turt_generate_step appends one token.
// Both hand back that position's logits; sampling (temperature, top-k, sampleFromLogits) stays
// on the host with the reference's RNG.
#include "../../include/turt_cuda.h"
#include "gemm.cuh"
#include "model.cuh"
#include "model_kernels.cuh"

using namespace turt;

namespace {

// Decode-step vectors carved from turt_model::dec.
struct DecBufs {
  float *x, *y, *qkv, *att, *h, *pre, *act, *logits, *rstd, *mean, *part, *apart;
  size_t part_floats;
};

constexpr int kGemvCols = 128;  // columns per block (32 lanes x float4)
constexpr int kGemvRows = 64;   // K rows per block (8 warps x 8)
constexpr int kAttnWarps = 8;   // decode attention: warps per block
constexpr int kAttnSplits = 8;  // decode attention: position slices per head

DecBufs dec_bufs(turt_model* m) {
  const int E = m->cfg.n_embd, h = m->hid, V = m->cfg.vocab_size;
  const int W1 = m->modern ? 2 * h : h;
  const int maxN = std::max(std::max(3 * E, W1), E), maxK = std::max(E, h);
  DecBufs d;
  float* p = m->dec;
  auto take = [&](size_t n) {
    float* r = p;
    p += (n + 63) & ~size_t(63);
    return r;
  };
  d.x = take(E);
  d.y = take(E);
  d.qkv = take(3 * E);
  d.att = take(E);
  d.h = take(E);
  d.pre = take(W1);
  d.act = take(h);
  d.logits = take(V);
  d.rstd = take(16);
  d.mean = take(16);
  d.apart = take((size_t)kAttnSplits * (E + 2 * m->cfg.n_head));
  d.part_floats = (size_t)((maxK + kGemvRows - 1) / kGemvRows) * maxN;
  d.part = take(d.part_floats);
  return d;
}

size_t dec_floats_needed(turt_model* m) {
  const int E = m->cfg.n_embd, h = m->hid, V = m->cfg.vocab_size;
  const int W1 = m->modern ? 2 * h : h;
  const int maxN = std::max(std::max(3 * E, W1), E), maxK = std::max(E, h);
  size_t n = 0;
  for (size_t k : {(size_t)E, (size_t)E, (size_t)3 * E, (size_t)E, (size_t)E, (size_t)W1, (size_t)h, (size_t)V,
                   (size_t)16, (size_t)16, (size_t)kAttnSplits * (E + 2 * m->cfg.n_head),
                   (size_t)((maxK + kGemvRows - 1) / kGemvRows) * maxN})
    n += (k + 63) & ~size_t(63);
  return n;
}

// x = wte[id] (+ wpe[pos]) of the token in the device cell tok = {id, pos}.
__global__ void k_dec_embed(const float* __restrict__ wte, const float* __restrict__ wpe, const int* __restrict__ tok,
                            float* __restrict__ x, int E) {
  const size_t id = (uint32_t)tok[0], pos = tok[1];
  for (int c = threadIdx.x; c < E; c += blockDim.x) x[c] = wte[id * E + c] + (wpe ? wpe[pos * E + c] : 0.0f);
}

// GEMV, first stage: part[ks][n] = sum over K rows [64 ks, 64 ks + 64) of a[k] W[k][n].  A block
// covers 128 columns; its 8 warps take 8 rows each, lanes 4 consecutive columns (one float4 when
// the row pitch and N allow it, else guarded scalar loads).
template <bool VEC>
__global__ void __launch_bounds__(256) k_gemv_part(const float* __restrict__ a, const float* __restrict__ W, int ldw,
                                                   int K, int N, float* __restrict__ part) {
  __shared__ float4 red[8][32];
  const int w = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int n = blockIdx.x * kGemvCols + lane * 4;
  const int k0 = blockIdx.y * kGemvRows + w * 8;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (n < N) {
#pragma unroll
    for (int r = 0; r < 8; r++) {
      const int k = k0 + r;
      if (k < K) {
        const float av = a[k];
        const float* row = W + (size_t)k * ldw + n;
        float4 wv;
        if (VEC) {
          wv = *reinterpret_cast<const float4*>(row);
        } else {
          wv.x = row[0];
          wv.y = n + 1 < N ? row[1] : 0.f;
          wv.z = n + 2 < N ? row[2] : 0.f;
          wv.w = n + 3 < N ? row[3] : 0.f;
        }
        acc.x += av * wv.x;
        acc.y += av * wv.y;
        acc.z += av * wv.z;
        acc.w += av * wv.w;
      }
    }
  }
  red[w][lane] = acc;
  __syncthreads();
  if (w == 0 && n < N) {
    float4 s = red[0][lane];
#pragma unroll
    for (int q = 1; q < 8; q++) {
      s.x += red[q][lane].x;
      s.y += red[q][lane].y;
      s.z += red[q][lane].z;
      s.w += red[q][lane].w;
    }
    float* dst = part + (size_t)blockIdx.y * N + n;
    if (VEC) {
      *reinterpret_cast<float4*>(dst) = s;
    } else {
      dst[0] = s.x;
      if (n + 1 < N) dst[1] = s.y;
      if (n + 2 < N) dst[2] = s.z;
      if (n + 3 < N) dst[3] = s.w;
    }
  }
}

// GEMV, second stage: y[n] = sum_ks part[ks][n] (fixed order) + bias[n] + res[n].
__global__ void k_gemv_sum(const float* __restrict__ part, int KS, int N, const float* __restrict__ bias,
                           const float* res, float* y) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  float s = 0.f;
  for (int q = 0; q < KS; q++) s += part[(size_t)q * N + n];
  if (bias) s += bias[n];
  if (res) s += res[n];
  y[n] = s;
}

int gemv(cudaStream_t st, const DecBufs& d, const float* a, const float* W, int ldw, int K, int N, const float* bias,
         const float* res, float* y) {
  const int KS = (K + kGemvRows - 1) / kGemvRows;
  TURT_REQUIRE((size_t)KS * N <= d.part_floats, "decode: GEMV scratch too small");
  const dim3 grid((N + kGemvCols - 1) / kGemvCols, KS);
  // float4 path: 16-byte aligned rows (W is 256-byte aligned) and whole float4 groups
  if (ldw % 4 == 0 && N % 4 == 0 && ((uintptr_t)W & 15) == 0)
    k_gemv_part<true><<<grid, 256, 0, st>>>(a, W, ldw, K, N, d.part);
  else
    k_gemv_part<false><<<grid, 256, 0, st>>>(a, W, ldw, K, N, d.part);
  TURT_LAUNCH_CHECK();
  k_gemv_sum<<<(N + 255) / 256, 256, 0, st>>>(d.part, KS, N, bias, res, y);
  TURT_LAUNCH_CHECK();
  return OK;
}

// q, k of the new token rotated at `pos` (RoPE, interleaved pairs); k and v appended to the cache.
__global__ void k_dec_qkv_post(float* __restrict__ qkv, const float2* __restrict__ cs, const int* __restrict__ tok,
                               int H, int hd, int rope, float* __restrict__ kc, float* __restrict__ vc, int Tc) {
  const int E = H * hd, pos = tok[1];
  for (int i = threadIdx.x; i < E / 2; i += blockDim.x) {
    const int c = 2 * i, hh = c / hd, d = c % hd;
    float q0 = qkv[c], q1 = qkv[c + 1], k0 = qkv[E + c], k1 = qkv[E + c + 1];
    if (rope) {
      const float2 r = cs[(size_t)pos * (hd / 2) + d / 2];
      const float a0 = q0 * r.x - q1 * r.y, a1 = q0 * r.y + q1 * r.x;
      const float b0 = k0 * r.x - k1 * r.y, b1 = k0 * r.y + k1 * r.x;
      q0 = a0, q1 = a1, k0 = b0, k1 = b1;
    }
    qkv[c] = q0;
    qkv[c + 1] = q1;
    const size_t o = ((size_t)hh * Tc + pos) * hd + d;
    kc[o] = k0;
    kc[o + 1] = k1;
    vc[o] = qkv[2 * E + c];
    vc[o + 1] = qkv[2 * E + c + 1];
  }
}

// Attention of the new token, split over positions (flash-decoding): block (head, s) takes the
// s-th of kAttnSplits slices of the cached positions j <= pos and writes its running max m,
// sum l = sum_j exp(score_j - m) and unnormalised output o = sum_j exp(score_j - m) v_j;
// k_dec_attn_merge combines the slices in a fixed order.  Inside a block each warp takes every
// 8th position, lanes across the head dim, so every key / value row is one coalesced read.
__global__ void __launch_bounds__(kAttnWarps * 32) k_dec_attn(const float* __restrict__ qkv, const float* __restrict__ kc,
                                                              const float* __restrict__ vc, const int* __restrict__ tok,
                                                              int hd, int Tc, float scale, float* __restrict__ part) {
  extern __shared__ float sh[];  // [slice] probabilities, [hd] q, [kAttnWarps][hd] partial outputs
  __shared__ float red[kAttnWarps];
  const int hh = blockIdx.x, sp = blockIdx.y, n = tok[1] + 1, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per = (n + kAttnSplits - 1) / kAttnSplits, j0 = sp * per, j1 = min(n, j0 + per);
  const int cap = (Tc + kAttnSplits - 1) / kAttnSplits;
  float* pr = sh;
  float* q = sh + cap;
  float* po = q + hd;
  float* out = part + ((size_t)hh * kAttnSplits + sp) * (hd + 2);  // [m, l, o[hd]]
  const float* K = kc + (size_t)hh * Tc * hd;
  const float* V = vc + (size_t)hh * Tc * hd;
  for (int d = threadIdx.x; d < hd; d += blockDim.x) q[d] = qkv[hh * hd + d];
  __syncthreads();
  float mx = -INFINITY;
  for (int j = j0 + w; j < j1; j += kAttnWarps) {
    float s = 0.f;
    for (int d = lane; d < hd; d += 32) s += q[d] * K[(size_t)j * hd + d];
    s = warp_sum(s) * scale;
    if (lane == 0) pr[j - j0] = s;
    mx = fmaxf(mx, s);
  }
  if (lane == 0) red[w] = mx;
  __syncthreads();
  mx = red[0];
  for (int i = 1; i < kAttnWarps; i++) mx = fmaxf(mx, red[i]);
  __syncthreads();
  float sum = 0.f;
  for (int j = j0 + threadIdx.x; j < j1; j += blockDim.x) {
    const float e = expf(pr[j - j0] - mx);
    pr[j - j0] = e;
    sum += e;
  }
  sum = warp_sum(sum);
  if (lane == 0) red[w] = sum;
  __syncthreads();
  for (int d0 = 0; d0 < hd; d0 += 32) {
    const int d = d0 + lane;
    if (d < hd) {
      float o = 0.f;
      for (int j = j0 + w; j < j1; j += kAttnWarps) o += pr[j - j0] * V[(size_t)j * hd + d];
      po[w * hd + d] = o;
    }
  }
  __syncthreads();
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float o = 0.f;
    for (int i = 0; i < kAttnWarps; i++) o += po[i * hd + d];
    out[2 + d] = o;
  }
  if (threadIdx.x == 0) {
    float l = 0.f;
    for (int i = 0; i < kAttnWarps; i++) l += red[i];
    out[0] = mx;  // -inf for an empty slice (l = 0, o = 0)
    out[1] = l;
  }
}

// out[h][d] = sum_s exp(m_s - M) o_s[d] / sum_s exp(m_s - M) l_s, slices in order.
__global__ void k_dec_attn_merge(const float* __restrict__ part, int hd, float* __restrict__ out) {
  const int hh = blockIdx.x;
  const float* p = part + (size_t)hh * kAttnSplits * (hd + 2);
  float M = -INFINITY;
  for (int i = 0; i < kAttnSplits; i++) M = fmaxf(M, p[i * (hd + 2)]);
  float L = 0.f;
  for (int i = 0; i < kAttnSplits; i++) {
    const float m = p[i * (hd + 2)];
    if (m > -INFINITY) L += expf(m - M) * p[i * (hd + 2) + 1];
  }
  const float inv = 1.0f / L;
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float o = 0.f;
    for (int i = 0; i < kAttnSplits; i++) {
      const float m = p[i * (hd + 2)];
      if (m > -INFINITY) o += expf(m - M) * p[i * (hd + 2) + 2 + d];
    }
    out[hh * hd + d] = o * inv;
  }
}

// MLP activation of one token: SwiGLU over the interleaved gate|up pre-activations, or GELU.
__global__ void k_dec_act(const float* __restrict__ pre, float* __restrict__ act, int h, int modern) {
  for (int u = blockIdx.x * blockDim.x + threadIdx.x; u < h; u += gridDim.x * blockDim.x) {
    if (modern) {
      const int c = (u / kGluBlock) * 2 * kGluBlock + u % kGluBlock;
      const float g = pre[c], v = pre[c + kGluBlock];
      act[u] = g * sigmoid_f(g) * v;
    } else {
      act[u] = gelu_f(pre[u]);
    }
  }
}

// logits[v] = y . wte[v] (tied head), one warp per vocabulary row.
__global__ void k_dec_logits(const float* __restrict__ y, const float* __restrict__ wte, int V, int E,
                             float* __restrict__ logits) {
  const int v = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (v >= V) return;
  float s = 0.f;
  for (int k = lane; k < E; k += 32) s += y[k] * wte[(size_t)v * E + k];
  s = warp_sum(s);
  if (lane == 0) logits[v] = s;
}

// Cache rows [0, t) of one layer from a full forward: k from the rotated head-major copy when the
// tensor-core attention made one, else from qkv (rotated here for RoPE models); v from qkv.
__global__ void k_cache_fill(const float* __restrict__ qkv, const float* __restrict__ kr,
                             const float2* __restrict__ cs, int t, int H, int hd, int rope, float* __restrict__ kc,
                             float* __restrict__ vc, int Tc) {
  const int E = H * hd;
  const long total = (long)t * E / 2;
  for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (long)gridDim.x * blockDim.x) {
    const int pos = (int)(e / (E / 2)), c = (int)(e % (E / 2)) * 2, hh = c / hd, d = c % hd;
    const size_t o = ((size_t)hh * Tc + pos) * hd + d;
    float k0, k1;
    if (kr) {
      k0 = kr[((size_t)hh * t + pos) * hd + d];
      k1 = kr[((size_t)hh * t + pos) * hd + d + 1];
    } else {
      k0 = qkv[(size_t)pos * 3 * E + E + c];
      k1 = qkv[(size_t)pos * 3 * E + E + c + 1];
      if (rope) {
        const float2 r = cs[(size_t)pos * (hd / 2) + d / 2];
        const float b0 = k0 * r.x - k1 * r.y, b1 = k0 * r.y + k1 * r.x;
        k0 = b0, k1 = b1;
      }
    }
    kc[o] = k0;
    kc[o + 1] = k1;
    vc[o] = qkv[(size_t)pos * 3 * E + 2 * E + c];
    vc[o + 1] = qkv[(size_t)pos * 3 * E + 2 * E + c + 1];
  }
}

size_t attn_smem(int Tc, int hd) {
  return (size_t)((Tc + kAttnSplits - 1) / kAttnSplits + hd + kAttnWarps * hd) * 4;
}

int ensure_decode(turt_model* m) {
  if (m->kcache) return OK;
  const size_t cache = (size_t)m->cfg.n_layer * m->cfg.block_size * m->cfg.n_embd;
  TURT_CHECK_CUDA(cudaMalloc(&m->kcache, cache * 4));
  TURT_CHECK_CUDA(cudaMalloc(&m->vcache, cache * 4));
  m->dec_floats = dec_floats_needed(m);
  TURT_CHECK_CUDA(cudaMalloc(&m->dec, m->dec_floats * 4));
  TURT_CHECK_CUDA(cudaMalloc(&m->dec_tok, 2 * sizeof(int)));
  TURT_CHECK_CUDA(cudaMallocHost(&m->h_dec_tok, 2 * sizeof(int)));
  TURT_CHECK_CUDA(cudaStreamCreateWithFlags(&m->dec_cap, cudaStreamNonBlocking));
  return OK;
}

// Every kernel of one decode step on stream `st`; the token and its position come from
// m->dec_tok.  Returns the number of kernels enqueued in *launches.
int enqueue_step(turt_model* m, cudaStream_t st, int* launches) {
  const int E = m->cfg.n_embd, H = m->cfg.n_head, hd = E / H, h = m->hid, V = m->cfg.vocab_size;
  const int Tc = m->cfg.block_size, W1 = m->modern ? 2 * h : h;
  const float* P = m->P;
  const DecBufs d = dec_bufs(m);
  const size_t per_layer = (size_t)Tc * E;
  const float scale = 1.0f / sqrtf((float)hd);
  int n = 0;
  k_dec_embed<<<1, 256, 0, st>>>(P + m->wte, m->modern ? nullptr : P + m->wpe, m->dec_tok, d.x, E);
  TURT_LAUNCH_CHECK();
  n++;
  for (int l = 0; l < m->cfg.n_layer; l++) {
    const LayerOff& L = m->layers[l];
    if (m->modern)
      RC(rms_fwd(st, d.x, P + L.ln1g, d.y, d.rstd, 1, E, m->eps));
    else
      RC(ln_fwd(st, d.x, P + L.ln1g, P + L.ln1b, d.y, d.mean, d.rstd, 1, E, m->eps));
    RC(gemv(st, d, d.y, P + L.wqkv, 3 * E, E, 3 * E, m->modern ? nullptr : P + L.bqkv, nullptr, d.qkv));
    k_dec_qkv_post<<<1, 256, 0, st>>>(d.qkv, m->rope_cs, m->dec_tok, H, hd, m->modern ? 1 : 0,
                                      m->kcache + l * per_layer, m->vcache + l * per_layer, Tc);
    TURT_LAUNCH_CHECK();
    k_dec_attn<<<dim3(H, kAttnSplits), kAttnWarps * 32, attn_smem(Tc, hd), st>>>(
        d.qkv, m->kcache + l * per_layer, m->vcache + l * per_layer, m->dec_tok, hd, Tc, scale, d.apart);
    TURT_LAUNCH_CHECK();
    k_dec_attn_merge<<<H, 64, 0, st>>>(d.apart, hd, d.att);
    TURT_LAUNCH_CHECK();
    RC(gemv(st, d, d.att, P + L.wproj, E, E, E, m->modern ? nullptr : P + L.bproj, d.x, d.h));
    if (m->modern)
      RC(rms_fwd(st, d.h, P + L.ln2g, d.y, d.rstd, 1, E, m->eps));
    else
      RC(ln_fwd(st, d.h, P + L.ln2g, P + L.ln2b, d.y, d.mean, d.rstd, 1, E, m->eps));
    RC(gemv(st, d, d.y, P + L.w1, W1, E, W1, m->modern ? nullptr : P + L.b1, nullptr, d.pre));
    k_dec_act<<<(h + 255) / 256, 256, 0, st>>>(d.pre, d.act, h, m->modern ? 1 : 0);
    TURT_LAUNCH_CHECK();
    RC(gemv(st, d, d.act, P + L.w2, E, h, E, m->modern ? nullptr : P + L.b2, d.h, d.x));
    n += 14;
  }
  if (m->modern)
    RC(rms_fwd(st, d.x, P + m->lnfg, d.y, d.rstd, 1, E, m->eps));
  else
    RC(ln_fwd(st, d.x, P + m->lnfg, P + m->lnfb, d.y, d.mean, d.rstd, 1, E, m->eps));
  k_dec_logits<<<(V + 7) / 8, 256, 0, st>>>(d.y, P + m->wte, V, E, d.logits);
  TURT_LAUNCH_CHECK();
  *launches = n + 2;
  return OK;
}

// Captures enqueue_step into m->dec_graph (on a private stream: capture needs one that is not
// the legacy default stream).
int capture_step(turt_model* m) {
  cudaGraph_t g = nullptr;
  int n = 0;
  TURT_CHECK_CUDA(cudaStreamBeginCapture(m->dec_cap, cudaStreamCaptureModeThreadLocal));
  const int rc = enqueue_step(m, m->dec_cap, &n);
  const cudaError_t ce = cudaStreamEndCapture(m->dec_cap, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  TURT_CHECK_CUDA(ce);
  const cudaError_t ie = cudaGraphInstantiate(&m->dec_graph, g, 0);
  cudaGraphDestroy(g);
  TURT_CHECK_CUDA(ie);
  note_launch(-n);  // captured, not run: replays are counted when they are launched
  m->dec_graph_kernels = n;
  return OK;
}

int copy_logits_out(turt_model* m, const float* dev, float* host) {
  cudaStream_t st = m->ctx->stream;
  TURT_CHECK_CUDA(cudaMemcpyAsync(host, dev, (size_t)m->cfg.vocab_size * 4, cudaMemcpyDeviceToHost, st));
  TURT_CHECK_CUDA(cudaStreamSynchronize(st));
  return ctx_check_flags(m->ctx);
}

}  // namespace

extern "C" int turt_generate_prefill(turt_model* m, const uint32_t* ids, int t, float* logits_out) {
  TURT_REQUIRE(m && ids && logits_out, "generate_prefill: null argument");
  TURT_CHECK_CUDA(cudaSetDevice(m->ctx->device));
  TURT_REQUIRE(t > 0 && t <= m->cfg.block_size, "generate_prefill: context must hold 1 .. block_size tokens");
  for (int i = 0; i < t; i++)
    TURT_REQUIRE(ids[i] < (uint32_t)m->cfg.vocab_size, "generate_prefill: token id out of range");
  TURT_REQUIRE(attn_smem(m->cfg.block_size, m->cfg.n_embd / m->cfg.n_head) <= 48 * 1024,
               "generate_prefill: the decode attention keeps block_size / 8 + 9 * head_dim floats in 48 KB of shared memory");
  RC(ensure_decode(m));
  RC(model_forward_logits(m, ids, t));
  cudaStream_t st = m->ctx->stream;
  const int E = m->cfg.n_embd, H = m->cfg.n_head, hd = E / H, Tc = m->cfg.block_size;
  const size_t per_layer = (size_t)Tc * E;
  for (int l = 0; l < m->cfg.n_layer; l++) {
    const LayerAct& a = m->act[l];
    const float* kr = (m->attn_tc && m->modern) ? a.kr : nullptr;
    const long total = (long)t * E / 2;
    k_cache_fill<<<(int)std::min<long>((total + 255) / 256, 148 * 8), 256, 0, st>>>(
        a.qkv, kr, m->rope_cs, t, H, hd, m->modern ? 1 : 0, m->kcache + l * per_layer, m->vcache + l * per_layer, Tc);
    TURT_LAUNCH_CHECK();
  }
  m->dec_len = t;
  return copy_logits_out(m, m->logits + (size_t)(t - 1) * m->cfg.vocab_size, logits_out);
}

extern "C" int turt_generate_step(turt_model* m, uint32_t id, int pos, float* logits_out) {
  TURT_REQUIRE(m && logits_out, "generate_step: null argument");
  TURT_CHECK_CUDA(cudaSetDevice(m->ctx->device));
  TURT_REQUIRE(m->kcache && pos == m->dec_len, "generate_step: position must follow the cached context");
  TURT_REQUIRE(pos < m->cfg.block_size, "generate_step: the context is full (prefill the cropped window instead)");
  TURT_REQUIRE(id < (uint32_t)m->cfg.vocab_size, "generate_step: token id out of range");
  cudaStream_t st = m->ctx->stream;
  if (!m->dec_graph) RC(capture_step(m));
  m->h_dec_tok[0] = (int)id;
  m->h_dec_tok[1] = pos;
  TURT_CHECK_CUDA(cudaMemcpyAsync(m->dec_tok, m->h_dec_tok, 2 * sizeof(int), cudaMemcpyHostToDevice, st));
  TURT_CHECK_CUDA(cudaGraphLaunch(m->dec_graph, st));
  note_launch(m->dec_graph_kernels);
  m->dec_len = pos + 1;
  return copy_logits_out(m, dec_bufs(m).logits, logits_out);
}
