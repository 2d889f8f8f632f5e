// ops.cu -- op-level kernels behind the GpuEngine mirror (one per reference WGSL kernel,
// src/infer/webgpu/autograd.ts:78-531).  These serve the op-by-op autograd tape; the
// fused model path (model.cu) uses its own fused kernels.
#include "ops.cuh"

namespace turt {
namespace {

constexpr int TPB = 256;

inline int grid_for(size_t n) {
  size_t g = (n + TPB - 1) / TPB;
  if (g > 148 * 64) g = 148 * 64;
  if (g < 1) g = 1;
  return (int)g;
}

#define GRID_STRIDE(i, n) for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < (n); i += (size_t)gridDim.x * blockDim.x)

__global__ void k_ewise(const float* a, const float* b, float* out, size_t n, size_t bLen, int op, int accum) {
  GRID_STRIDE(i, n) {
    float bv = b[i % bLen];
    float r = op == 1 ? a[i] - bv : (op == 2 ? a[i] * bv : a[i] + bv);
    out[i] = accum ? out[i] + r : r;
  }
}
__global__ void k_scale(const float* a, float* out, size_t n, float s, int accum) {
  GRID_STRIDE(i, n) {
    float r = a[i] * s;
    out[i] = accum ? out[i] + r : r;
  }
}
__global__ void k_bcast_acc(const float* src, float* out, size_t n, size_t bLen, float s) {
  GRID_STRIDE(i, n) out[i] += src[i % bLen] * s;
}
// out[j] (+)= s * sum_{i % bLen == j} g[i]; one thread per column, rows in ascending order.
__global__ void k_segsum(const float* g, float* out, size_t n, size_t bLen, float s, int accum) {
  GRID_STRIDE(j, bLen) {
    float acc = 0.f;
    for (size_t i = j; i < n; i += bLen) acc += g[i];
    float r = acc * s;
    out[j] = accum ? out[j] + r : r;
  }
}
// Single-block deterministic sum (the reference's TOTAL is a 1-thread loop).
__global__ void k_total(const float* a, float* out, size_t n) {
  __shared__ double part[32];
  double s = 0;
  for (size_t i = threadIdx.x; i < n; i += blockDim.x) s += a[i];
  s = warp_sum_d(s);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    double v = threadIdx.x < blockDim.x / 32 ? part[threadIdx.x] : 0.0;
    v = warp_sum_d(v);
    if (threadIdx.x == 0) out[0] = (float)v;
  }
}
__global__ void k_relu(const float* x, float* out, size_t n) { GRID_STRIDE(i, n) out[i] = fmaxf(x[i], 0.f); }
__global__ void k_relu_bwd(const float* x, const float* go, float* gi, size_t n) {
  GRID_STRIDE(i, n) if (x[i] > 0.f) gi[i] += go[i];
}
__global__ void k_sgd(const float* g, float* p, size_t n, float lr) { GRID_STRIDE(i, n) p[i] -= lr * g[i]; }
__global__ void k_gelu(const float* x, float* out, size_t n) { GRID_STRIDE(i, n) out[i] = gelu_f(x[i]); }
__global__ void k_gelu_bwd(const float* x, const float* go, float* gi, size_t n) {
  GRID_STRIDE(i, n) gi[i] += go[i] * gelu_grad_f(x[i]);
}
__global__ void k_silu(const float* x, float* out, size_t n) {
  GRID_STRIDE(i, n) out[i] = x[i] / (1.0f + expf(-x[i]));
}
__global__ void k_silu_bwd(const float* x, const float* go, float* gi, size_t n) {
  GRID_STRIDE(i, n) {
    float s = sigmoid_f(x[i]);
    float y = x[i] * s;
    gi[i] += go[i] * (s + y * (1.0f - s));
  }
}

// Row kernels: one warp per row.
__global__ void k_rms_fwd(const float* x, const float* gamma, float* out, float* rstd, int rows, int d, float eps) {
  int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* xr = x + (size_t)row * d;
  float s = 0;
  for (int j = lane; j < d; j += 32) s += xr[j] * xr[j];
  s = warp_sum(s);
  float rs = rsqrtf(s / d + eps);
  if (lane == 0) rstd[row] = rs;
  for (int j = lane; j < d; j += 32) out[(size_t)row * d + j] = xr[j] * rs * gamma[j];
}
__global__ void k_rms_dx(const float* x, const float* go, const float* gamma, const float* rstd, float* gi, int rows,
                         int d) {
  int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* xr = x + (size_t)row * d;
  const float* gr = go + (size_t)row * d;
  float s = 0;
  for (int j = lane; j < d; j += 32) s += gr[j] * gamma[j] * xr[j];
  s = warp_sum(s);
  float rs = rstd[row];
  float k = rs * rs * rs * s / d;
  for (int j = lane; j < d; j += 32) gi[(size_t)row * d + j] += rs * gr[j] * gamma[j] - k * xr[j];
}
// Column reductions: one thread per column, rows ascending (as RMS_DG / LN_DGB).
__global__ void k_rms_dg(const float* x, const float* go, const float* rstd, float* dg, int rows, int d) {
  GRID_STRIDE(j, (size_t)d) {
    float acc = 0;
    for (int r = 0; r < rows; r++) acc += go[(size_t)r * d + j] * x[(size_t)r * d + j] * rstd[r];
    dg[j] += acc;
  }
}
__global__ void k_ln_fwd(const float* x, const float* gamma, const float* beta, float* out, float* mean, float* rstd,
                         int rows, int d, float eps) {
  int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* xr = x + (size_t)row * d;
  float s = 0;
  for (int j = lane; j < d; j += 32) s += xr[j];
  float mu = warp_sum(s) / d;
  float v = 0;
  for (int j = lane; j < d; j += 32) v += (xr[j] - mu) * (xr[j] - mu);
  v = warp_sum(v) / d;
  float rs = rsqrtf(v + eps);
  if (lane == 0) {
    mean[row] = mu;
    rstd[row] = rs;
  }
  for (int j = lane; j < d; j += 32) out[(size_t)row * d + j] = (xr[j] - mu) * rs * gamma[j] + beta[j];
}
__global__ void k_ln_dx(const float* x, const float* go, const float* gamma, const float* mean, const float* rstd,
                        float* gi, int rows, int d) {
  int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* xr = x + (size_t)row * d;
  const float* gr = go + (size_t)row * d;
  float mu = mean[row], rs = rstd[row];
  float sdy = 0, sdyx = 0;
  for (int j = lane; j < d; j += 32) {
    float dy = gr[j] * gamma[j];
    sdy += dy;
    sdyx += dy * (xr[j] - mu) * rs;
  }
  sdy = warp_sum(sdy);
  sdyx = warp_sum(sdyx);
  for (int j = lane; j < d; j += 32) {
    float dy = gr[j] * gamma[j], xh = (xr[j] - mu) * rs;
    gi[(size_t)row * d + j] += rs * (dy - sdy / d - xh * sdyx / d);
  }
}
__global__ void k_ln_dgb(const float* x, const float* go, const float* mean, const float* rstd, float* dg, float* db,
                         int rows, int d) {
  GRID_STRIDE(j, (size_t)d) {
    float a = 0, b = 0;
    for (int r = 0; r < rows; r++) {
      float g = go[(size_t)r * d + j];
      a += g * (x[(size_t)r * d + j] - mean[r]) * rstd[r];
      b += g;
    }
    dg[j] += a;
    db[j] += b;
  }
}
// RoPE: one thread per (group, pos, pair); the angle table is precomputed in double.
__global__ void k_rope(const float* x, float* out, const float2* cs, int groups, int t, int hd, int bwd) {
  int half = hd / 2;
  size_t n = (size_t)groups * t * half;
  GRID_STRIDE(i, n) {
    int pair = (int)(i % half);
    int pos = (int)((i / half) % t);
    size_t off = (i / half) * hd + 2 * pair;
    float2 c = cs[pos * half + pair];
    float x0 = x[off], x1 = x[off + 1];
    if (!bwd) {
      out[off] = x0 * c.x - x1 * c.y;
      out[off + 1] = x0 * c.y + x1 * c.x;
    } else {
      out[off] += x0 * c.x + x1 * c.y;
      out[off + 1] += -x0 * c.y + x1 * c.x;
    }
  }
}
__global__ void k_softmax(const float* x, float* out, int rows, int d) {
  int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* xr = x + (size_t)row * d;
  float m = -INFINITY;
  for (int j = lane; j < d; j += 32) m = fmaxf(m, xr[j]);
  m = warp_max(m);
  float s = 0;
  for (int j = lane; j < d; j += 32) s += expf(xr[j] - m);
  s = warp_sum(s);
  for (int j = lane; j < d; j += 32) out[(size_t)row * d + j] = expf(xr[j] - m) / s;
}
__global__ void k_softmax_bwd(const float* y, const float* go, float* gi, int rows, int d) {
  int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* yr = y + (size_t)row * d;
  const float* gr = go + (size_t)row * d;
  float dot = 0;
  for (int j = lane; j < d; j += 32) dot += gr[j] * yr[j];
  dot = warp_sum(dot);
  for (int j = lane; j < d; j += 32) gi[(size_t)row * d + j] += yr[j] * (gr[j] - dot);
}
__global__ void k_gather(const float* table, const uint32_t* idx, float* out, int n, int d, int vocab, int* flags) {
  size_t total = (size_t)n * d;
  GRID_STRIDE(i, total) {
    size_t row = i / d, col = i % d;
    uint32_t r = idx[row];
    if (r >= (uint32_t)vocab) {
      atomicExch(&flags[FLAG_RANGE], 1);
      r = 0;
    }
    out[i] = table[(size_t)r * d + col];
  }
}
// GATHER_BWD (autograd.ts:428-438): dTable[v,:] = dTable[v,:] + gOut[i,:] for each position i
// with idx[i] == v, in increasing i -- the reference's order, so the result is deterministic and
// matches its arithmetic.  One warp per vocab row: lanes compare 32 ids at a time and a ballot
// lists the matching positions; each match is added in place, lane-strided over the columns.
// Ids >= vocab raise the range flag (block 0 checks them) and match no row.
__global__ void k_gather_bwd(const uint32_t* idx, const float* go, float* dt, int n, int d, int vocab, int* flags) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < n; i += blockDim.x)
      if (idx[i] >= (uint32_t)vocab) atomicExch(&flags[FLAG_RANGE], 1);
  const uint32_t v = (uint32_t)(blockIdx.x * (blockDim.x >> 5) + warp);
  if (v >= (uint32_t)vocab) return;
  float* row = dt + (size_t)v * d;
  for (int base = 0; base < n; base += 32) {
    const int i = base + lane;
    uint32_t m = __ballot_sync(0xffffffffu, i < n && idx[i] == v);
    while (m) {
      const int k = __ffs(m) - 1;
      m &= m - 1;
      const float* g = go + (size_t)(base + k) * d;
      for (int c = lane; c < d; c += 32) row[c] = row[c] + g[c];
    }
  }
}
// Cross-entropy: one block per row (logsumexp - logit[target]).
__device__ __forceinline__ void row_max_sum(const float* x, int vocab, float* out_m, float* out_s) {
  __shared__ float red[32];
  __shared__ float bc[2];
  float m = -INFINITY;
  for (int j = threadIdx.x; j < vocab; j += blockDim.x) m = fmaxf(m, x[j]);
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : -INFINITY;
    v = warp_max(v);
    if (threadIdx.x == 0) bc[0] = v;
  }
  __syncthreads();
  m = bc[0];
  float s = 0;
  for (int j = threadIdx.x; j < vocab; j += blockDim.x) s += expf(x[j] - m);
  s = warp_sum(s);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) bc[1] = v;
  }
  __syncthreads();
  *out_m = m;
  *out_s = bc[1];
}
__global__ void k_ce_fwd(const float* logits, const uint32_t* tgt, float* per_row, int rows, int vocab, int* flags) {
  int row = blockIdx.x;
  const float* x = logits + (size_t)row * vocab;
  float m, s;
  row_max_sum(x, vocab, &m, &s);
  if (threadIdx.x == 0) {
    uint32_t t = tgt[row];
    if (t >= (uint32_t)vocab) {
      atomicExch(&flags[FLAG_RANGE], 1);
      t = 0;
    }
    per_row[row] = m + logf(s) - x[t];
  }
}
__global__ void k_ce_bwd(const float* logits, const uint32_t* tgt, const float* gloss, float* dl, int rows, int vocab,
                         int* flags) {
  int row = blockIdx.x;
  const float* x = logits + (size_t)row * vocab;
  float m, s;
  row_max_sum(x, vocab, &m, &s);
  float scale = gloss[0] / rows;
  for (int j = threadIdx.x; j < vocab; j += blockDim.x) dl[(size_t)row * vocab + j] += scale * expf(x[j] - m) / s;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t t = tgt[row];
    if (t >= (uint32_t)vocab) {
      atomicExch(&flags[FLAG_RANGE], 1);
    } else {
      dl[(size_t)row * vocab + t] -= scale;
    }
  }
}
__global__ void k_mask(const float* x, float* out, int groups, int t, int bwd) {
  size_t n = (size_t)groups * t * t;
  GRID_STRIDE(i, n) {
    size_t w = i % ((size_t)t * t);
    int r = (int)(w / t), c = (int)(w % t);
    if (!bwd)
      out[i] = c > r ? -1e9f : x[i];
    else if (c <= r)
      out[i] += x[i];
  }
}
struct Perm4 {
  int s[4], p[4];
};
__global__ void k_permute4(const float* inp, float* out, Perm4 pm, size_t n, int accum) {
  GRID_STRIDE(o, n) {
    int os[4] = {pm.s[pm.p[0]], pm.s[pm.p[1]], pm.s[pm.p[2]], pm.s[pm.p[3]]};
    size_t istr[4] = {(size_t)pm.s[1] * pm.s[2] * pm.s[3], (size_t)pm.s[2] * pm.s[3], (size_t)pm.s[3], 1};
    size_t ostr[4] = {(size_t)os[1] * os[2] * os[3], (size_t)os[2] * os[3], (size_t)os[3], 1};
    size_t rem = o, in = 0;
    for (int a = 0; a < 4; a++) {
      size_t c = rem / ostr[a];
      rem -= c * ostr[a];
      in += c * istr[pm.p[a]];
    }
    if (!accum)
      out[o] = inp[in];
    else
      out[in] += inp[o];
  }
}
__global__ void k_adamw(const float* g, float* p, float* m, float* v, size_t n, float lr, float b1, float b2,
                        float eps, float wd, float bc1, float bc2) {
  GRID_STRIDE(i, n) {
    float gr = g[i];
    float mi = b1 * m[i] + (1.f - b1) * gr;
    float vi = b2 * v[i] + (1.f - b2) * gr * gr;
    m[i] = mi;
    v[i] = vi;
    float mh = mi / bc1, vh = vi / bc2;
    p[i] = p[i] - lr * (mh / (sqrtf(vh) + eps) + wd * p[i]);
  }
}
__global__ void k_fill(float* p, float v, size_t n) { GRID_STRIDE(i, n) p[i] = v; }

__global__ void k_rope_table(float2* cs, int t, int hd, double base) {
  int half = hd / 2;
  GRID_STRIDE(i, (size_t)t * half) {
    int p = (int)(i / half), k = (int)(i % half);
    double theta = (double)p / pow(base, (double)(2 * k) / (double)hd);
    cs[i] = make_float2((float)cos(theta), (float)sin(theta));
  }
}

}  // namespace

#define LAUNCH_1D(kern, n, ...)                                   \
  do {                                                            \
    if ((n) == 0) return OK;                                      \
    kern<<<grid_for(n), TPB, 0, st>>>(__VA_ARGS__);               \
    TURT_LAUNCH_CHECK();                          \
    return OK;                                                    \
  } while (0)

#define LAUNCH_ROWS(kern, rows, ...)                               \
  do {                                                             \
    if ((rows) == 0) return OK;                                    \
    kern<<<ceil_div(rows, 8), 256, 0, st>>>(__VA_ARGS__);          \
    TURT_LAUNCH_CHECK();                           \
    return OK;                                                     \
  } while (0)

int op_ewise(cudaStream_t st, const float* a, const float* b, float* out, size_t n, size_t bLen, int op, int accum) {
  TURT_REQUIRE(bLen > 0 || n == 0, "ewise: bLen must be > 0");
  LAUNCH_1D(k_ewise, n, a, b, out, n, bLen, op, accum);
}
int op_scale(cudaStream_t st, const float* a, float* out, size_t n, float s, int accum) {
  LAUNCH_1D(k_scale, n, a, out, n, s, accum);
}
int op_bcast_acc(cudaStream_t st, const float* src, float* out, size_t n, size_t bLen, float s) {
  TURT_REQUIRE(bLen > 0 || n == 0, "bcastAcc: bLen must be > 0");
  LAUNCH_1D(k_bcast_acc, n, src, out, n, bLen, s);
}
int op_segsum(cudaStream_t st, const float* g, float* out, size_t n, size_t bLen, float s, int accum) {
  LAUNCH_1D(k_segsum, bLen, g, out, n, bLen, s, accum);
}
int op_total(cudaStream_t st, const float* a, float* out, size_t n) {
  k_total<<<1, 1024, 0, st>>>(a, out, n);
  TURT_LAUNCH_CHECK();
  return OK;
}
int op_relu(cudaStream_t st, const float* x, float* out, size_t n) { LAUNCH_1D(k_relu, n, x, out, n); }
int op_relu_bwd(cudaStream_t st, const float* x, const float* go, float* gi, size_t n) {
  LAUNCH_1D(k_relu_bwd, n, x, go, gi, n);
}
int op_sgd(cudaStream_t st, const float* g, float* p, size_t n, float lr) { LAUNCH_1D(k_sgd, n, g, p, n, lr); }
int op_gelu(cudaStream_t st, const float* x, float* out, size_t n) { LAUNCH_1D(k_gelu, n, x, out, n); }
int op_gelu_bwd(cudaStream_t st, const float* x, const float* go, float* gi, size_t n) {
  LAUNCH_1D(k_gelu_bwd, n, x, go, gi, n);
}
int op_silu(cudaStream_t st, const float* x, float* out, size_t n) { LAUNCH_1D(k_silu, n, x, out, n); }
int op_silu_bwd(cudaStream_t st, const float* x, const float* go, float* gi, size_t n) {
  LAUNCH_1D(k_silu_bwd, n, x, go, gi, n);
}
int op_rms_fwd(cudaStream_t st, const float* x, const float* g, float* out, float* rstd, int rows, int d, float eps) {
  LAUNCH_ROWS(k_rms_fwd, rows, x, g, out, rstd, rows, d, eps);
}
int op_rms_dx(cudaStream_t st, const float* x, const float* go, const float* g, const float* rstd, float* gi, int rows,
              int d) {
  LAUNCH_ROWS(k_rms_dx, rows, x, go, g, rstd, gi, rows, d);
}
int op_rms_dg(cudaStream_t st, const float* x, const float* go, const float* rstd, float* dg, int rows, int d) {
  LAUNCH_1D(k_rms_dg, (size_t)d, x, go, rstd, dg, rows, d);
}
int op_ln_fwd(cudaStream_t st, const float* x, const float* g, const float* b, float* out, float* mean, float* rstd,
              int rows, int d, float eps) {
  LAUNCH_ROWS(k_ln_fwd, rows, x, g, b, out, mean, rstd, rows, d, eps);
}
int op_ln_dx(cudaStream_t st, const float* x, const float* go, const float* g, const float* mean, const float* rstd,
             float* gi, int rows, int d) {
  LAUNCH_ROWS(k_ln_dx, rows, x, go, g, mean, rstd, gi, rows, d);
}
int op_ln_dgb(cudaStream_t st, const float* x, const float* go, const float* mean, const float* rstd, float* dg,
              float* db, int rows, int d) {
  LAUNCH_1D(k_ln_dgb, (size_t)d, x, go, mean, rstd, dg, db, rows, d);
}
int op_rope_table(cudaStream_t st, float2* cs, int t, int hd, double base) {
  LAUNCH_1D(k_rope_table, (size_t)t * (hd / 2), cs, t, hd, base);
}
int op_rope(cudaStream_t st, const float* x, float* out, const float2* cs, int groups, int t, int hd, int bwd) {
  LAUNCH_1D(k_rope, (size_t)groups * t * (hd / 2), x, out, cs, groups, t, hd, bwd);
}
int op_softmax(cudaStream_t st, const float* x, float* out, int rows, int d) {
  LAUNCH_ROWS(k_softmax, rows, x, out, rows, d);
}
int op_softmax_bwd(cudaStream_t st, const float* y, const float* go, float* gi, int rows, int d) {
  LAUNCH_ROWS(k_softmax_bwd, rows, y, go, gi, rows, d);
}
int op_gather(cudaStream_t st, const float* table, const uint32_t* idx, float* out, int n, int d, int vocab, int* flags) {
  LAUNCH_1D(k_gather, (size_t)n * d, table, idx, out, n, d, vocab, flags);
}
int op_gather_bwd(cudaStream_t st, const uint32_t* idx, const float* go, float* dt, int n, int d, int vocab,
                  int* flags) {
  if (n <= 0 || d <= 0 || vocab <= 0) return OK;
  k_gather_bwd<<<ceil_div(vocab, 8), 256, 0, st>>>(idx, go, dt, n, d, vocab, flags);
  TURT_LAUNCH_CHECK();
  return OK;
}
int op_ce_fwd(cudaStream_t st, const float* logits, const uint32_t* tgt, float* per_row, int rows, int vocab,
              int* flags) {
  if (rows == 0) return OK;
  k_ce_fwd<<<rows, 256, 0, st>>>(logits, tgt, per_row, rows, vocab, flags);
  TURT_LAUNCH_CHECK();
  return OK;
}
int op_ce_bwd(cudaStream_t st, const float* logits, const uint32_t* tgt, const float* gloss, float* dl, int rows,
              int vocab, int* flags) {
  if (rows == 0) return OK;
  k_ce_bwd<<<rows, 256, 0, st>>>(logits, tgt, gloss, dl, rows, vocab, flags);
  TURT_LAUNCH_CHECK();
  return OK;
}
int op_mask(cudaStream_t st, const float* x, float* out, int groups, int t, int bwd) {
  LAUNCH_1D(k_mask, (size_t)groups * t * t, x, out, groups, t, bwd);
}
int op_permute4(cudaStream_t st, const float* inp, float* out, const int* shape, const int* perm, size_t n, int accum) {
  Perm4 pm;
  for (int a = 0; a < 4; a++) {
    pm.s[a] = shape[a];
    pm.p[a] = perm[a];
  }
  LAUNCH_1D(k_permute4, n, inp, out, pm, n, accum);
}
int op_adamw(cudaStream_t st, const float* g, float* p, float* m, float* v, size_t n, float lr, float b1, float b2,
             float eps, float wd, float bc1, float bc2) {
  LAUNCH_1D(k_adamw, n, g, p, m, v, n, lr, b1, b2, eps, wd, bc1, bc2);
}
int op_fill(cudaStream_t st, float* p, float v, size_t n) { LAUNCH_1D(k_fill, n, p, v, n); }

}  // namespace turt
