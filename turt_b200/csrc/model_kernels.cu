// model_kernels.cu -- fused memory-bound kernels of the train step (model path).
// Each kernel replaces a run of reference dispatches (src/infer/webgpu/autograd.ts) with
// one coalesced pass: 128-bit loads where rows allow, one warp per row, warp-shuffle
// reductions, and deterministic two-stage column reductions for parameter gradients.
#include "model_kernels.cuh"

namespace turt {
namespace {

#define GRID_STRIDE(i, n) \
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < (n); i += (size_t)gridDim.x * blockDim.x)

// ------------------------------------------------------------- embedding
// x[n,:] = wte[ids[n],:] (+ wpe[n % T,:]); GATHER (+EWISE add), autograd.ts:416-425.
__global__ void k_embed(const float* __restrict__ wte, const float* __restrict__ wpe, const uint32_t* __restrict__ ids,
                        float* __restrict__ x, int N, int T, int E, int V, int* flags) {
  pdl_trigger();
  pdl_wait();
  const int e4 = E / 4;
  GRID_STRIDE(i, (size_t)N * e4) {
    const int n = (int)(i / e4), c = (int)(i % e4);
    uint32_t id = ids[n];
    if (id >= (uint32_t)V) {
      atomicExch(&flags[FLAG_RANGE], 1);
      id = 0;
    }
    float4 v = reinterpret_cast<const float4*>(wte + (size_t)id * E)[c];
    if (wpe) {
      const float4 p = reinterpret_cast<const float4*>(wpe + (size_t)(n % T) * E)[c];
      v.x += p.x;
      v.y += p.y;
      v.z += p.z;
      v.w += p.w;
    }
    reinterpret_cast<float4*>(x + (size_t)n * E)[c] = v;
  }
}

// dwte[v,:] += sum of dx[i,:] over the positions i with ids[i] == v, added one position at a
// time in increasing i onto the running value, exactly the order of GATHER_BWD (one thread per
// vocab row scanning all positions, autograd.ts:428-438), so the result is deterministic.
// One warp per vocab row; the block stages the ids in shared memory (kIdTile at a time) and
// each warp finds its row's positions 128 ids per step: every lane compares four ids, a ballot
// marks the lanes with a match and each match's 4-bit mask is read from its lane in turn.
// Rows no position uses are not touched.  Ids >= V match no row (the forward flags them).
constexpr int kIdTile = 8192;        // ids staged per pass (32 KB)
constexpr int kEmbedRowsPerBlock = 16;

template <int NJ>
__global__ void __launch_bounds__(32 * kEmbedRowsPerBlock)
    k_embed_bwd_rows(const float* __restrict__ dx, const uint32_t* __restrict__ ids, float* __restrict__ dwte, int N,
                     int E, int V) {
  __shared__ __align__(16) uint32_t sid[kIdTile];
  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t v = (uint32_t)(blockIdx.x * kEmbedRowsPerBlock + warp);
  const int E4 = E / 4;
  float4 acc[NJ];
  bool any = false;  // warp-uniform: every lane sees the same matches
  for (int base = 0; base < N; base += kIdTile) {
    const int cnt = min(kIdTile, N - base);
    const int padded = (cnt + 127) & ~127;
    __syncthreads();  // the previous tile has been scanned
    for (int k = threadIdx.x; k < padded; k += blockDim.x) sid[k] = k < cnt ? ids[base + k] : 0xFFFFFFFFu;
    __syncthreads();
    if (v >= (uint32_t)V) continue;
    const uint4* sid4 = reinterpret_cast<const uint4*>(sid);
    for (int c = 0; c < padded / 128; c++) {
      const uint4 q = sid4[c * 32 + lane];  // ids base + 128c + 4 lane .. + 3
      const uint32_t nib = (q.x == v ? 1u : 0u) | (q.y == v ? 2u : 0u) | (q.z == v ? 4u : 0u) | (q.w == v ? 8u : 0u);
      uint32_t m = __ballot_sync(0xffffffffu, nib != 0);
      while (m) {
        const int src = __ffs(m) - 1;
        m &= m - 1;
        uint32_t bits = __shfl_sync(0xffffffffu, nib, src);
        while (bits) {
          const int k = __ffs(bits) - 1;
          bits &= bits - 1;
          const float4* g = reinterpret_cast<const float4*>(dx + (size_t)(base + 128 * c + 4 * src + k) * E);
          if (!any) {
            const float4* w = reinterpret_cast<const float4*>(dwte + (size_t)v * E);
#pragma unroll
            for (int j = 0; j < NJ; j++)
              if (lane + 32 * j < E4) acc[j] = w[lane + 32 * j];
            any = true;
          }
#pragma unroll
          for (int j = 0; j < NJ; j++)
            if (lane + 32 * j < E4) {
              const float4 t = g[lane + 32 * j];
              acc[j].x += t.x, acc[j].y += t.y, acc[j].z += t.z, acc[j].w += t.w;
            }
        }
      }
    }
  }
  if (any) {
    float4* w = reinterpret_cast<float4*>(dwte + (size_t)v * E);
#pragma unroll
    for (int j = 0; j < NJ; j++)
      if (lane + 32 * j < E4) w[lane + 32 * j] = acc[j];
  }
}

// dwpe[t,:] += dx[b*T + t,:] for b = 0, 1, ... in order (the learned positions' share of the
// gpt2 embedding backward, deterministic): one warp per position.
template <int NJ>
__global__ void __launch_bounds__(256) k_pos_bwd(const float* __restrict__ dx, float* __restrict__ dwpe, int N, int T,
                                                 int E) {
  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= T || t >= N) return;
  const int E4 = E / 4;
  float4* w = reinterpret_cast<float4*>(dwpe + (size_t)t * E);
  float4 acc[NJ];
#pragma unroll
  for (int j = 0; j < NJ; j++)
    if (lane + 32 * j < E4) acc[j] = w[lane + 32 * j];
#pragma unroll 4
  for (int n = t; n < N; n += T) {
    const float4* g = reinterpret_cast<const float4*>(dx + (size_t)n * E);
#pragma unroll
    for (int j = 0; j < NJ; j++)
      if (lane + 32 * j < E4) {
        const float4 x = g[lane + 32 * j];
        acc[j].x += x.x, acc[j].y += x.y, acc[j].z += x.z, acc[j].w += x.w;
      }
  }
#pragma unroll
  for (int j = 0; j < NJ; j++)
    if (lane + 32 * j < E4) w[lane + 32 * j] = acc[j];
}

// ------------------------------------------------------------------ norms
// One warp per row.  Lane `lane` owns the float4 chunks lane + 32j (j < NJ = ceil(E/128)) of
// the row, so every load and store is a coalesced 16-byte access.  E is a multiple of 32 and at
// most 1024 (NJ <= 8).
constexpr int MAXV = 32;  // E <= 32 * MAXV
constexpr int kNormWarps = 8;

__device__ __forceinline__ float4 ld4(const float* p, int i) { return reinterpret_cast<const float4*>(p)[i]; }
__device__ __forceinline__ void st4(float* p, int i, float4 v) { reinterpret_cast<float4*>(p)[i] = v; }
__device__ __forceinline__ float dot4(float4 a, float4 b) { return a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w; }

// RMSNorm forward: y = x * rs * g, rs = (mean(x^2) + eps)^-1/2 (autograd.ts:315-330).
template <int NJ>
__global__ void __launch_bounds__(256) k_rms_fwd(const float* __restrict__ x, const float* __restrict__ g,
                                                 float* __restrict__ y, float* __restrict__ rstd, int rows, int E,
                                                 float eps) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x * kNormWarps + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int n4 = E / 4;
  const float* xr = x + (size_t)row * E;
  float4 v[NJ];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NJ; j++) {
    const int i = lane + 32 * j;
    v[j] = i < n4 ? ld4(xr, i) : make_float4(0.f, 0.f, 0.f, 0.f);
    ss += dot4(v[j], v[j]);
  }
  ss = warp_sum(ss);
  const float rs = rsqrtf(ss / E + eps);
  if (lane == 0) rstd[row] = rs;
  float* yr = y + (size_t)row * E;
#pragma unroll
  for (int j = 0; j < NJ; j++) {
    const int i = lane + 32 * j;
    if (i < n4) {
      const float4 gg = ld4(g, i);
      st4(yr, i, make_float4(v[j].x * rs * gg.x, v[j].y * rs * gg.y, v[j].z * rs * gg.z, v[j].w * rs * gg.w));
    }
  }
}

// Block partial of a per-column sum: the 8 warps' register partials (lane chunks) are combined
// in shared memory in fixed order and written column-major as part[c][blockIdx.x] (nparts =
// gridDim.x entries per column), so that the final reduction reads each column contiguously.
template <int NJ>
__device__ __forceinline__ void block_partial(const float4 (&acc)[NJ], float* sm, float* __restrict__ part, int E) {
  const int w = threadIdx.x / 32, lane = threadIdx.x & 31, n4 = E / 4;
#pragma unroll
  for (int j = 0; j < NJ; j++) {
    const int i = lane + 32 * j;
    if (i < n4) st4(sm + (size_t)w * E, i, acc[j]);
  }
  __syncthreads();
  for (int c = threadIdx.x; c < E; c += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int q = 0; q < kNormWarps; q++) t += sm[q * E + c];
    part[(size_t)c * gridDim.x + blockIdx.x] = t;
  }
}

// Register budget of the norm backwards: two 256-thread blocks per SM up to E = 512, one block
// per SM (more registers per thread) for the wider rows.
template <int NJ>
struct NormBwdCfg {
  static constexpr int kMinBlocks = NJ <= 4 ? 2 : 1;
  static constexpr int kRows = NJ <= 3 ? 2 : 1;  // RMSNorm rows per warp iteration
};

// RMSNorm backward with the residual gradient fused in:
//   dx = dres + rs*g*dy - (rs^3/E) * (sum_j dy_j g_j x_j) * x      (RMS_DX, autograd.ts:331-351)
// and per-block partial dgamma = sum_rows dy * x * rs              (RMS_DG, :352-365).
// dx may alias dres.  Rows are dealt to warps grid-stride, R rows per iteration (two for rows of
// up to 384 floats, so that each warp keeps 6*NJ independent 16-byte loads in flight; one for
// wider rows, whose registers would spill otherwise).
template <int NJ>
__global__ void __launch_bounds__(256, NormBwdCfg<NJ>::kMinBlocks)
    k_rms_bwd(const float* __restrict__ x, const float* __restrict__ dy, const float* __restrict__ g,
              const float* __restrict__ rstd, const float* dres, float* dx, float* __restrict__ dg_part, int rows,
              int E) {
  constexpr int R = NormBwdCfg<NJ>::kRows;
  pdl_trigger();
  pdl_wait();
  extern __shared__ float sm[];
  const int lane = threadIdx.x & 31, n4 = E / 4;
  const int stride = gridDim.x * kNormWarps;
  float4 gv[NJ], dgl[NJ];
#pragma unroll
  for (int j = 0; j < NJ; j++) {
    const int i = lane + 32 * j;
    gv[j] = i < n4 ? ld4(g, i) : make_float4(0.f, 0.f, 0.f, 0.f);
    dgl[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int r0 = blockIdx.x * kNormWarps + threadIdx.x / 32; r0 < rows; r0 += R * stride) {
    int rr[R];
    float4 xv[R][NJ], dv[R][NJ];
    float s[R], rs[R];
#pragma unroll
    for (int q = 0; q < R; q++) {
      rr[q] = r0 + q * stride;
      const bool ok = rr[q] < rows;
      s[q] = 0.f;
      rs[q] = ok ? rstd[rr[q]] : 0.f;
#pragma unroll
      for (int j = 0; j < NJ; j++) {
        const int i = lane + 32 * j;
        const bool in = ok && i < n4;
        xv[q][j] = in ? ld4(x + (size_t)rr[q] * E, i) : make_float4(0.f, 0.f, 0.f, 0.f);
        dv[q][j] = in ? ld4(dy + (size_t)rr[q] * E, i) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int q = 0; q < R; q++)
#pragma unroll
      for (int j = 0; j < NJ; j++) {
        const float4 a = xv[q][j], d = dv[q][j], gg = gv[j];
        s[q] += d.x * gg.x * a.x + d.y * gg.y * a.y + d.z * gg.z * a.z + d.w * gg.w * a.w;
        dgl[j].x += d.x * a.x * rs[q];
        dgl[j].y += d.y * a.y * rs[q];
        dgl[j].z += d.z * a.z * rs[q];
        dgl[j].w += d.w * a.w * rs[q];
      }
#pragma unroll
    for (int q = 0; q < R; q++) {
      if (rr[q] >= rows) continue;  // warp-uniform
      const float sum = warp_sum(s[q]);
      const float kf = rs[q] * rs[q] * rs[q] * sum / E;
      const float* dr = dres ? dres + (size_t)rr[q] * E : nullptr;
      float* dxr = dx + (size_t)rr[q] * E;
#pragma unroll
      for (int j = 0; j < NJ; j++) {
        const int i = lane + 32 * j;
        if (i >= n4) continue;
        const float4 a = xv[q][j], d = dv[q][j], gg = gv[j];
        float4 o = make_float4(rs[q] * d.x * gg.x - kf * a.x, rs[q] * d.y * gg.y - kf * a.y,
                               rs[q] * d.z * gg.z - kf * a.z, rs[q] * d.w * gg.w - kf * a.w);
        if (dr) {
          const float4 t = ld4(dr, i);
          o.x += t.x;
          o.y += t.y;
          o.z += t.z;
          o.w += t.w;
        }
        st4(dxr, i, o);
      }
    }
  }
  block_partial<NJ>(dgl, sm, dg_part, E);
}

// LayerNorm forward (biased variance), autograd.ts:256-274.
template <int NJ>
__global__ void __launch_bounds__(256) k_ln_fwd(const float* __restrict__ x, const float* __restrict__ g,
                                                const float* __restrict__ b, float* __restrict__ y,
                                                float* __restrict__ mean, float* __restrict__ rstd, int rows, int E,
                                                float eps) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x * kNormWarps + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int n4 = E / 4;
  const float* xr = x + (size_t)row * E;
  float4 v[NJ];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < NJ; j++) {
    const int i = lane + 32 * j;
    v[j] = i < n4 ? ld4(xr, i) : make_float4(0.f, 0.f, 0.f, 0.f);
    s += v[j].x + v[j].y + v[j].z + v[j].w;
  }
  const float mu = warp_sum(s) / E;
  float qv = 0.f;
#pragma unroll
  for (int j = 0; j < NJ; j++) {
    const int i = lane + 32 * j;
    if (i < n4) {
      const float4 d = make_float4(v[j].x - mu, v[j].y - mu, v[j].z - mu, v[j].w - mu);
      qv += dot4(d, d);
    }
  }
  const float rs = rsqrtf(warp_sum(qv) / E + eps);
  if (lane == 0) {
    mean[row] = mu;
    rstd[row] = rs;
  }
  float* yr = y + (size_t)row * E;
#pragma unroll
  for (int j = 0; j < NJ; j++) {
    const int i = lane + 32 * j;
    if (i < n4) {
      const float4 gg = ld4(g, i), bb = ld4(b, i);
      st4(yr, i,
          make_float4((v[j].x - mu) * rs * gg.x + bb.x, (v[j].y - mu) * rs * gg.y + bb.y,
                      (v[j].z - mu) * rs * gg.z + bb.z, (v[j].w - mu) * rs * gg.w + bb.w));
    }
  }
}

// LayerNorm backward (LN_DX + LN_DGB, autograd.ts:275-308) with the residual gradient fused;
// partial dgamma / dbeta per block.  One row per warp iteration, grid-stride.
template <int NJ>
__global__ void __launch_bounds__(256, NormBwdCfg<NJ>::kMinBlocks) k_ln_bwd(const float* __restrict__ x, const float* __restrict__ dy,
                                                const float* __restrict__ g, const float* __restrict__ mean,
                                                const float* __restrict__ rstd, const float* dres, float* dx,
                                                float* __restrict__ dg_part, float* __restrict__ db_part, int rows,
                                                int E) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float sm[];
  const int lane = threadIdx.x & 31, n4 = E / 4;
  const int stride = gridDim.x * kNormWarps;
  float4 gv[NJ], dgl[NJ], dbl[NJ];
#pragma unroll
  for (int j = 0; j < NJ; j++) {
    const int i = lane + 32 * j;
    gv[j] = i < n4 ? ld4(g, i) : make_float4(0.f, 0.f, 0.f, 0.f);
    dgl[j] = dbl[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int r = blockIdx.x * kNormWarps + threadIdx.x / 32; r < rows; r += stride) {
    const float mu = mean[r], rs = rstd[r];
    float4 xh[NJ], dv[NJ];
    float sdy = 0.f, sdyx = 0.f;
#pragma unroll
    for (int j = 0; j < NJ; j++) {
      const int i = lane + 32 * j;
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f), gy = a;
      if (i < n4) {
        a = ld4(x + (size_t)r * E, i);
        gy = ld4(dy + (size_t)r * E, i);
      }
      xh[j] = make_float4((a.x - mu) * rs, (a.y - mu) * rs, (a.z - mu) * rs, (a.w - mu) * rs);
      if (i >= n4) xh[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      dgl[j].x += gy.x * xh[j].x;
      dgl[j].y += gy.y * xh[j].y;
      dgl[j].z += gy.z * xh[j].z;
      dgl[j].w += gy.w * xh[j].w;
      dbl[j].x += gy.x;
      dbl[j].y += gy.y;
      dbl[j].z += gy.z;
      dbl[j].w += gy.w;
      dv[j] = make_float4(gy.x * gv[j].x, gy.y * gv[j].y, gy.z * gv[j].z, gy.w * gv[j].w);
      sdy += dv[j].x + dv[j].y + dv[j].z + dv[j].w;
      sdyx += dot4(dv[j], xh[j]);
    }
    sdy = warp_sum(sdy) / E;
    sdyx = warp_sum(sdyx) / E;
    const float* dr = dres ? dres + (size_t)r * E : nullptr;
    float* dxr = dx + (size_t)r * E;
#pragma unroll
    for (int j = 0; j < NJ; j++) {
      const int i = lane + 32 * j;
      if (i >= n4) continue;
      float4 o = make_float4(rs * (dv[j].x - sdy - xh[j].x * sdyx), rs * (dv[j].y - sdy - xh[j].y * sdyx),
                             rs * (dv[j].z - sdy - xh[j].z * sdyx), rs * (dv[j].w - sdy - xh[j].w * sdyx));
      if (dr) {
        const float4 t = ld4(dr, i);
        o.x += t.x;
        o.y += t.y;
        o.z += t.z;
        o.w += t.w;
      }
      st4(dxr, i, o);
    }
  }
  block_partial<NJ>(dgl, sm, dg_part, E);
  __syncthreads();
  block_partial<NJ>(dbl, sm, db_part, E);
}

// out[c] += sum_b part[c][b] (column-major partials, fixed order: deterministic).  One warp per
// column: the lanes' strided loads are all independent (one memory round trip for up to a few
// hundred partials), then a butterfly sum.
__global__ void k_reduce_parts(const float* __restrict__ part, int nparts, int C, float* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int c = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (c >= C) return;
  const float* col = part + (size_t)c * nparts;
  float s = 0.f;
  for (int b = lane; b < nparts; b += 32) s += col[b];
  s = warp_sum(s);
  if (lane == 0) out[c] += s;
}

// Column sums of g[rows][C] into column-major partials part[c][p] (bias gradients; SEGSUM,
// autograd.ts:122-135): partial p sums rows p, p + P, p + 2P, ... (P = gridDim.y).
__global__ void k_colsum_parts(const float* __restrict__ g, int rows, int C, float* __restrict__ part) {
  pdl_trigger();
  pdl_wait();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  float s = 0.f;
  for (int r = blockIdx.y; r < rows; r += gridDim.y) s += g[(size_t)r * C + c];
  part[(size_t)c * gridDim.y + blockIdx.y] = s;
}

// SwiGLU backward over the interleaved gate|up layout (kGluBlock = 32: columns [64j, 64j+32)
// gate units [32j, 32j+32), [64j+32, 64j+64) the matching up units): from d(act) [N][h] and the
// pre-activations [N][2h], s = sigmoid(gate): d(up) = dact * gate * s,
// d(gate) = dact * up * (s + gate*s*(1 - s)) (SILU_BWD, autograd.ts:1044-1054, and the product
// rule).  One thread per float4 of d(act); consecutive threads read consecutive 16-byte pieces.
__global__ void __launch_bounds__(256) k_swiglu_bwd_il(const float* __restrict__ dact, const float* __restrict__ pre,
                                                       float* __restrict__ dpre, long N, int h) {
  pdl_trigger();
  pdl_wait();
  const int h4 = h / 4;
  const long total = N * h4;
  for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (long)gridDim.x * blockDim.x) {
    const long n = e / h4;
    const int u = (int)(e % h4) * 4;                // hidden unit
    const long gi = n * 2L * h + (u / 32) * 64 + u % 32;  // gate column; up is 32 further
    const float4 d = reinterpret_cast<const float4*>(dact)[e];
    const float4 g = *reinterpret_cast<const float4*>(pre + gi);
    const float4 v = *reinterpret_cast<const float4*>(pre + gi + 32);
    float4 dg, du;
#define SWIL(c)                                  \
  {                                              \
    const float sg = sigmoid_f(g.c);             \
    const float sl = g.c * sg;                   \
    du.c = d.c * sl;                             \
    dg.c = d.c * v.c * (sg + sl * (1.0f - sg));  \
  }
    SWIL(x) SWIL(y) SWIL(z) SWIL(w)
#undef SWIL
    *reinterpret_cast<float4*>(dpre + gi) = dg;
    *reinterpret_cast<float4*>(dpre + gi + 32) = du;
  }
}

// -------------------------------------------------- fused softmax + cross-entropy
// One block per row of logits[N][V]: per-row loss (CE_FWD, autograd.ts:441-454) and the
// gradient (CE_BWD, :455-471) written in place over the logits: one HBM read, one write.
__global__ void __launch_bounds__(512) k_ce_fused(float* __restrict__ logits, const uint32_t* __restrict__ tgt,
                                                  float* __restrict__ loss_rows, int V, float gscale, int* flags) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  float* x = logits + (size_t)row * V;
  __shared__ float red_m[32], red_s[32];
  __shared__ float bc[2];
  // online (max, sum) over this thread's elements
  float m = -INFINITY, s = 0.f;
  const int V4 = V / 4;
  const bool vec = (V % 4) == 0;
  if (vec) {
    for (int j = threadIdx.x; j < V4; j += blockDim.x) {
      const float4 v = reinterpret_cast<const float4*>(x)[j];
      const float mx = fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
      if (mx > m) {
        s *= __expf(m - mx);
        m = mx;
      }
      s += __expf(v.x - m) + __expf(v.y - m) + __expf(v.z - m) + __expf(v.w - m);
    }
  } else {
    for (int j = threadIdx.x; j < V; j += blockDim.x) {
      const float v = x[j];
      if (v > m) {
        s *= __expf(m - v);
        m = v;
      }
      s += __expf(v - m);
    }
  }
  // warp combine
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const float mm = fmaxf(m, m2);
    s = (m == -INFINITY ? 0.f : s * __expf(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mm));
    m = mm;
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    red_m[w] = m;
    red_s[w] = s;
  }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x / 32;
    m = lane < nw ? red_m[lane] : -INFINITY;
    s = lane < nw ? red_s[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      const float mm = fmaxf(m, m2);
      s = (m == -INFINITY ? 0.f : s * __expf(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mm));
      m = mm;
    }
    if (lane == 0) {
      bc[0] = m;
      bc[1] = s;
    }
  }
  __syncthreads();
  m = bc[0];
  s = bc[1];
  uint32_t t = tgt[row];
  const bool bad = t >= (uint32_t)V;
  if (threadIdx.x == 0) {
    if (bad) atomicExch(&flags[FLAG_RANGE], 1);
    loss_rows[row] = bad ? 0.f : m + logf(s) - x[t];
  }
  __syncthreads();  // the target logit is read before it is overwritten
  const float inv = 1.0f / s;
  if (vec) {
    for (int j = threadIdx.x; j < V4; j += blockDim.x) {
      float4 v = reinterpret_cast<float4*>(x)[j];
      v.x = gscale * __expf(v.x - m) * inv;
      v.y = gscale * __expf(v.y - m) * inv;
      v.z = gscale * __expf(v.z - m) * inv;
      v.w = gscale * __expf(v.w - m) * inv;
      const int base = 4 * j;
      if (!bad && (uint32_t)(t - base) < 4u) {
        const int q = (int)(t - base);
        if (q == 0) v.x -= gscale;
        if (q == 1) v.y -= gscale;
        if (q == 2) v.z -= gscale;
        if (q == 3) v.w -= gscale;
      }
      reinterpret_cast<float4*>(x)[j] = v;
    }
  } else {
    for (int j = threadIdx.x; j < V; j += blockDim.x) {
      float v = gscale * __expf(x[j] - m) * inv;
      if (!bad && (uint32_t)j == t) v -= gscale;
      x[j] = v;
    }
  }
}

// Forward-only variant: per-row loss, logits untouched.
__global__ void __launch_bounds__(512) k_ce_loss(const float* __restrict__ logits, const uint32_t* __restrict__ tgt,
                                                 float* __restrict__ loss_rows, int V, int* flags) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  const float* x = logits + (size_t)row * V;
  __shared__ float red_m[32], red_s[32];
  float m = -INFINITY, s = 0.f;
  for (int j = threadIdx.x; j < V; j += blockDim.x) {
    const float v = x[j];
    if (v > m) {
      s *= __expf(m - v);
      m = v;
    }
    s += __expf(v - m);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const float mm = fmaxf(m, m2);
    s = (m == -INFINITY ? 0.f : s * __expf(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mm));
    m = mm;
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    red_m[w] = m;
    red_s[w] = s;
  }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x / 32;
    m = lane < nw ? red_m[lane] : -INFINITY;
    s = lane < nw ? red_s[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      const float mm = fmaxf(m, m2);
      s = (m == -INFINITY ? 0.f : s * __expf(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mm));
      m = mm;
    }
    if (lane == 0) {
      const uint32_t t = tgt[row];
      if (t >= (uint32_t)V) {
        atomicExch(&flags[FLAG_RANGE], 1);
        loss_rows[row] = 0.f;
      } else {
        loss_rows[row] = m + logf(s) - x[t];
      }
    }
  }
}

// loss = (sum of per-row losses, in double) / n; one block, fixed order.
__global__ void k_loss_mean(const float* __restrict__ rows, int n, float* __restrict__ out, int* flags) {
  pdl_trigger();
  pdl_wait();
  __shared__ double part[32];
  double s = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += rows[i];
  s = warp_sum_d(s);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    double v = threadIdx.x < blockDim.x / 32 ? part[threadIdx.x] : 0.0;
    v = warp_sum_d(v);
    if (threadIdx.x == 0) {
      const float l = (float)(v / n);
      out[0] = l;
      if (!isfinite(l)) atomicExch(&flags[FLAG_NONFINITE], 1);
    }
  }
}

// ---------------------------------------------------------- optimizer
// Sum of squares of scale*g in double: per-block partials, then a fixed-order final pass.
constexpr int NORM_BLOCKS = 592;  // 4 x 148 SMs
__global__ void k_sumsq_parts(const float* __restrict__ g, size_t n, float scale, double* __restrict__ part) {
  pdl_trigger();
  pdl_wait();
  __shared__ double red[32];
  double s = 0;
  const size_t n4 = n / 4;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(g)[i];
    const double a = (double)(v.x * scale), b = (double)(v.y * scale), c = (double)(v.z * scale),
                 d = (double)(v.w * scale);
    s += a * a + b * b + c * c + d * d;
  }
  if (blockIdx.x == 0)
    for (size_t i = n4 * 4 + threadIdx.x; i < n; i += blockDim.x) {
      const double a = (double)(g[i] * scale);
      s += a * a;
    }
  s = warp_sum_d(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    double v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.0;
    v = warp_sum_d(v);
    if (threadIdx.x == 0) part[blockIdx.x] = v;
  }
}
// norm = sqrt(sum); coef = clip > 0 && norm > clip ? clip / norm : 1 (src/optim/clip.ts:7-24).
__global__ void k_norm_final(const double* __restrict__ part, int nparts, float clip, double* __restrict__ norm_out,
                             float* __restrict__ coef_out, int* flags) {
  pdl_trigger();
  pdl_wait();
  __shared__ double red[32];
  double s = 0;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) s += part[i];
  s = warp_sum_d(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    double v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.0;
    v = warp_sum_d(v);
    if (threadIdx.x == 0) {
      const double norm = sqrt(v);
      norm_out[0] = norm;
      float coef = 1.0f;
      if (clip > 0.f && norm > (double)clip && norm > 0) coef = (float)((double)clip / norm);
      if (!isfinite(norm)) {
        atomicExch(&flags[FLAG_NONFINITE], 1);
        coef = 0.0f;  // a non-finite step is skipped rather than applied
      }
      coef_out[0] = coef;
    }
  }
}
// g *= coef (standalone clipGradNorm).
__global__ void k_scale_by(float* __restrict__ g, size_t n, const float* __restrict__ coef, float pre) {
  pdl_trigger();
  pdl_wait();
  const float c = coef[0] * pre;
  GRID_STRIDE(i, n) g[i] *= c;
}

// AdamW over the flat parameter buffer (ADAMW, autograd.ts:516-531 / src/optim/adam.ts:50-55)
// with the gradient pre-scaled by gscale * coef (DP mean and global-norm clip).
__global__ void k_adamw_flat(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, size_t n, float lr, float b1, float b2, float eps, float wd,
                             float bc1, float bc2, float gscale, const float* __restrict__ coef) {
  pdl_trigger();
  pdl_wait();
  const float cs = gscale * (coef ? coef[0] : 1.0f);
  const float rbc1 = 1.0f / bc1, rbc2 = 1.0f / bc2;
  const size_t n4 = n / 4;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    float4 pp = reinterpret_cast<float4*>(p)[i];
    const float4 gg = reinterpret_cast<const float4*>(g)[i];
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
#define ADAM1(c)                                                      \
  {                                                                   \
    const float gr = gg.c * cs;                                       \
    mm.c = b1 * mm.c + (1.f - b1) * gr;                               \
    vv.c = b2 * vv.c + (1.f - b2) * gr * gr;                          \
    const float mh = mm.c * rbc1, vh = vv.c * rbc2;                   \
    pp.c = pp.c - lr * (mh / (sqrtf(vh) + eps) + wd * pp.c);          \
  }
    ADAM1(x) ADAM1(y) ADAM1(z) ADAM1(w)
#undef ADAM1
    reinterpret_cast<float4*>(p)[i] = pp;
    reinterpret_cast<float4*>(m)[i] = mm;
    reinterpret_cast<float4*>(v)[i] = vv;
  }
  if (blockIdx.x == 0)
    for (size_t i = n4 * 4 + threadIdx.x; i < n; i += blockDim.x) {
      const float gr = g[i] * cs;
      m[i] = b1 * m[i] + (1.f - b1) * gr;
      v[i] = b2 * v[i] + (1.f - b2) * gr * gr;
      p[i] = p[i] - lr * ((m[i] * rbc1) / (sqrtf(v[i] * rbc2) + eps) + wd * p[i]);
    }
}

}  // namespace

int embed_fwd(cudaStream_t st, const float* wte, const float* wpe, const uint32_t* ids, float* x, int N, int T, int E,
              int V, int* flags) {
  TURT_REQUIRE(E % 4 == 0, "embedding width must be a multiple of 4");
  const size_t n = (size_t)N * (E / 4);
  TURT_CHECK_CUDA((launch_pdl(k_embed, dim3((int)std::min<size_t>((n + 255) / 256, 148 * 32)), dim3(256), 0, st, wte, wpe, ids, x, N, T, E, V, flags)));
  TURT_LAUNCH_CHECK();
  return OK;
}

namespace {
int sm_count() {
  static std::atomic<int> cached{0};  // every device of one node has the same SM count
  int n = cached.load(std::memory_order_relaxed);
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
    cached.store(n, std::memory_order_relaxed);
  }
  return n;
}
// Dispatch on NJ = ceil(E / 128) float4 chunks per lane.
#define TURT_NJ_SWITCH(E, CALL) \
  switch (((E) + 127) / 128) {  \
    case 1: CALL(1); break;     \
    case 2: CALL(2); break;     \
    case 3: CALL(3); break;     \
    case 4: CALL(4); break;     \
    case 5: CALL(5); break;     \
    case 6: CALL(6); break;     \
    case 7: CALL(7); break;     \
    default: CALL(8); break;    \
  }
}  // namespace

int embed_bwd(cudaStream_t st, const float* dx, const uint32_t* ids, float* dwte, float* dwpe, int N, int T, int E,
              int V) {
  TURT_REQUIRE(E % 4 == 0 && E <= 1024, "embedding width must be a multiple of 4, at most 1024");
  const dim3 grid_rows((V + kEmbedRowsPerBlock - 1) / kEmbedRowsPerBlock);
#define TURT_EMBED_BWD(NJV)                                                                                     \
  TURT_CHECK_CUDA((launch_pdl(k_embed_bwd_rows<NJV>, grid_rows, dim3(32 * kEmbedRowsPerBlock), 0, st, dx, ids, \
                              dwte, N, E, V)));
  TURT_NJ_SWITCH(E, TURT_EMBED_BWD)
#undef TURT_EMBED_BWD
  TURT_LAUNCH_CHECK();
  if (dwpe) {
#define TURT_POS_BWD(NJV) \
  TURT_CHECK_CUDA((launch_pdl(k_pos_bwd<NJV>, dim3((T + 7) / 8), dim3(256), 0, st, dx, dwpe, N, T, E)));
    TURT_NJ_SWITCH(E, TURT_POS_BWD)
#undef TURT_POS_BWD
    TURT_LAUNCH_CHECK();
  }
  return OK;
}

int rms_fwd(cudaStream_t st, const float* x, const float* g, float* y, float* rstd, int rows, int E, float eps) {
  TURT_REQUIRE(E % 32 == 0 && E <= 32 * MAXV, "norm width must be a multiple of 32, at most 1024");
#define CALL(NJ) TURT_CHECK_CUDA((launch_pdl(k_rms_fwd<NJ>, dim3(ceil_div(rows, kNormWarps)), dim3(256), 0, st, x, g, y, rstd, rows, E, eps)))
  TURT_NJ_SWITCH(E, CALL)
#undef CALL
  TURT_LAUNCH_CHECK();
  return OK;
}
// Partial-sum rows a norm backward writes: one per block, at most two blocks per SM.
int norm_parts(int rows) {
  const int b = ceil_div(rows, kNormWarps);
  return b < 2 * sm_count() ? b : 2 * sm_count();
}
int rms_bwd(cudaStream_t st, const float* x, const float* dy, const float* g, const float* rstd, const float* dres,
            float* dx, float* dg_accum, float* part, int rows, int E) {
  TURT_REQUIRE(E % 32 == 0 && E <= 32 * MAXV, "norm width must be a multiple of 32, at most 1024");
  const int nb = norm_parts(rows);
  const size_t smem = (size_t)kNormWarps * E * 4;
#define CALL(NJ) TURT_CHECK_CUDA((launch_pdl(k_rms_bwd<NJ>, dim3(nb), dim3(256), smem, st, x, dy, g, rstd, dres, dx, part, rows, E)))
  TURT_NJ_SWITCH(E, CALL)
#undef CALL
  TURT_LAUNCH_CHECK();
  TURT_CHECK_CUDA((launch_pdl(k_reduce_parts, dim3(ceil_div(E, 8)), dim3(256), 0, st, part, nb, E, dg_accum)));
  TURT_LAUNCH_CHECK();
  return OK;
}
int ln_fwd(cudaStream_t st, const float* x, const float* g, const float* b, float* y, float* mean, float* rstd, int rows,
           int E, float eps) {
  TURT_REQUIRE(E % 32 == 0 && E <= 32 * MAXV, "norm width must be a multiple of 32, at most 1024");
#define CALL(NJ) TURT_CHECK_CUDA((launch_pdl(k_ln_fwd<NJ>, dim3(ceil_div(rows, kNormWarps)), dim3(256), 0, st, x, g, b, y, mean, rstd, rows, E, eps)))
  TURT_NJ_SWITCH(E, CALL)
#undef CALL
  TURT_LAUNCH_CHECK();
  return OK;
}
int ln_bwd(cudaStream_t st, const float* x, const float* dy, const float* g, const float* mean, const float* rstd,
           const float* dres, float* dx, float* dg_accum, float* db_accum, float* part, int rows, int E) {
  TURT_REQUIRE(E % 32 == 0 && E <= 32 * MAXV, "norm width must be a multiple of 32, at most 1024");
  const int nb = norm_parts(rows);
  const size_t smem = (size_t)kNormWarps * E * 4;
#define CALL(NJ) \
  TURT_CHECK_CUDA((launch_pdl(k_ln_bwd<NJ>, dim3(nb), dim3(256), smem, st, x, dy, g, mean, rstd, dres, dx, part, part + (size_t)nb * E, rows, E)))
  TURT_NJ_SWITCH(E, CALL)
#undef CALL
  TURT_LAUNCH_CHECK();
  TURT_CHECK_CUDA((launch_pdl(k_reduce_parts, dim3(ceil_div(E, 8)), dim3(256), 0, st, part, nb, E, dg_accum)));
  TURT_LAUNCH_CHECK();
  TURT_CHECK_CUDA((launch_pdl(k_reduce_parts, dim3(ceil_div(E, 8)), dim3(256), 0, st, part + (size_t)nb * E, nb, E, db_accum)));
  TURT_LAUNCH_CHECK();
  return OK;
}
int colsum_accum(cudaStream_t st, const float* g, int rows, int C, float* out_accum, float* part) {
  const int nb = norm_parts(rows);
  dim3 grid(ceil_div(C, 128), nb);
  TURT_CHECK_CUDA((launch_pdl(k_colsum_parts, dim3(grid), dim3(128), 0, st, g, rows, C, part)));
  TURT_LAUNCH_CHECK();
  TURT_CHECK_CUDA((launch_pdl(k_reduce_parts, dim3(ceil_div(C, 8)), dim3(256), 0, st, part, nb, C, out_accum)));
  TURT_LAUNCH_CHECK();
  return OK;
}
int swiglu_bwd_interleaved(cudaStream_t st, const float* dact, const float* pre, float* dpre, int N, int h) {
  TURT_REQUIRE(h % 32 == 0, "swiglu backward: hidden width must be a multiple of 32");
  const long total = (long)N * (h / 4);
  long blocks = (total + 255) / 256;
  if (blocks > 148L * 16) blocks = 148L * 16;
  TURT_CHECK_CUDA((launch_pdl(k_swiglu_bwd_il, dim3((int)blocks), dim3(256), 0, st, dact, pre, dpre, N, h)));
  TURT_LAUNCH_CHECK();
  return OK;
}
int ce_fused(cudaStream_t st, float* logits, const uint32_t* tgt, float* loss_rows, int N, int V, float gscale,
             int* flags) {
  TURT_CHECK_CUDA((launch_pdl(k_ce_fused, dim3(N), dim3(512), 0, st, logits, tgt, loss_rows, V, gscale, flags)));
  TURT_LAUNCH_CHECK();
  return OK;
}
int ce_loss(cudaStream_t st, const float* logits, const uint32_t* tgt, float* loss_rows, int N, int V, int* flags) {
  TURT_CHECK_CUDA((launch_pdl(k_ce_loss, dim3(N), dim3(512), 0, st, logits, tgt, loss_rows, V, flags)));
  TURT_LAUNCH_CHECK();
  return OK;
}
int loss_mean(cudaStream_t st, const float* rows, int n, float* out, int* flags) {
  TURT_CHECK_CUDA((launch_pdl(k_loss_mean, dim3(1), dim3(1024), 0, st, rows, n, out, flags)));
  TURT_LAUNCH_CHECK();
  return OK;
}
size_t norm_scratch_doubles() { return NORM_BLOCKS + 1; }
int grad_norm(cudaStream_t st, const float* g, size_t n, float gscale, float clip, double* scratch, double* norm_out,
              float* coef_out, int* flags) {
  TURT_CHECK_CUDA((launch_pdl(k_sumsq_parts, dim3(NORM_BLOCKS), dim3(512), 0, st, g, n, gscale, scratch)));
  TURT_LAUNCH_CHECK();
  TURT_CHECK_CUDA((launch_pdl(k_norm_final, dim3(1), dim3(1024), 0, st, scratch, NORM_BLOCKS, clip, norm_out, coef_out, flags)));
  TURT_LAUNCH_CHECK();
  return OK;
}
int scale_by(cudaStream_t st, float* g, size_t n, const float* coef, float pre) {
  TURT_CHECK_CUDA((launch_pdl(k_scale_by, dim3(148 * 8), dim3(256), 0, st, g, n, coef, pre)));
  TURT_LAUNCH_CHECK();
  return OK;
}
int adamw_flat(cudaStream_t st, float* p, const float* g, float* m, float* v, size_t n, float lr, float b1, float b2,
               float eps, float wd, float bc1, float bc2, float gscale, const float* coef) {
  TURT_REQUIRE(((uintptr_t)p & 15) == 0 && ((uintptr_t)g & 15) == 0 && ((uintptr_t)m & 15) == 0 &&
                   ((uintptr_t)v & 15) == 0,
               "adamw: buffers must be 16-byte aligned");
  TURT_CHECK_CUDA((launch_pdl(k_adamw_flat, dim3(148 * 8), dim3(256), 0, st, p, g, m, v, n, lr, b1, b2, eps, wd, bc1, bc2, gscale, coef)));
  TURT_LAUNCH_CHECK();
  return OK;
}

}  // namespace turt
