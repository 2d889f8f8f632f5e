// attention.cu -- fused causal self-attention with RoPE for the model path.
//
// Replaces the reference's per-layer chain (src/models/gpu-gpt.ts:143-168):
//   split heads (PERMUTE4) -> ROPE q,k -> bmmBT -> scale -> maskedFillCausal(-1e9) -> softmax
//   -> bmm(v) -> merge heads
// with one forward kernel (online softmax, no [T,T] scores in HBM) and two backward
// kernels (dK/dV per key tile, dQ per query tile; deterministic, no atomics).
// q/k/v are read in place from the fused projection output qkv[N][3E] (token n = b*T + t,
// head h at columns h*hd); RoPE (interleaved pairs, src/math/tensor.ts:650-700) is applied
// on load and its inverse rotation is applied to dQ/dK before they are written to dqkv.
#include "attention.cuh"

namespace turt {
namespace {

constexpr int BQ = 64;
constexpr int BKV = 64;
constexpr int PAD = 4;  // keeps float4 alignment of rows, breaks bank regularity

struct AttnShape {
  int B, T, H, hd, E;  // E = H * hd
  float scale;
  int rope;  // apply rotary embedding to q and k
};

// Loads rows [r0, r0+64) of q (col_off 0), k (E) or v (2E) for head h into a transposed
// smem tile dst[d][64+PAD] (and optionally a row-major copy rm[64][hd+PAD]), rotating pairs.
template <int HD>
__device__ __forceinline__ void load_tile(const float* __restrict__ qkv, const float2* __restrict__ rope_cs,
                                          const AttnShape& s, int b, int h, int r0, int col_off, bool rotate,
                                          float* dstT, float* rm) {
  const int ld = 3 * s.E;
  for (int e = threadIdx.x; e < 64 * (HD / 2); e += blockDim.x) {
    const int r = e / (HD / 2), pr = e % (HD / 2);
    const int t = r0 + r;
    float x0 = 0.f, x1 = 0.f;
    if (t < s.T) {
      const float* src = qkv + ((long)b * s.T + t) * ld + col_off + h * HD + 2 * pr;
      x0 = src[0];
      x1 = src[1];
      if (rotate) {
        const float2 c = rope_cs[t * (HD / 2) + pr];
        const float y0 = x0 * c.x - x1 * c.y;
        const float y1 = x0 * c.y + x1 * c.x;
        x0 = y0;
        x1 = y1;
      }
    }
    dstT[(2 * pr) * (64 + PAD) + r] = x0;
    dstT[(2 * pr + 1) * (64 + PAD) + r] = x1;
    if (rm) {
      rm[r * (HD + PAD) + 2 * pr] = x0;
      rm[r * (HD + PAD) + 2 * pr + 1] = x1;
    }
  }
}

// Same for a [N][E] tensor (attention output O or its gradient dO).
template <int HD>
__device__ __forceinline__ void load_tile_ne(const float* __restrict__ x, const AttnShape& s, int b, int h, int r0,
                                             float* dstT, float* rm) {
  for (int e = threadIdx.x; e < 64 * HD; e += blockDim.x) {
    const int r = e / HD, d = e % HD;
    const int t = r0 + r;
    const float v = t < s.T ? x[((long)b * s.T + t) * s.E + h * HD + d] : 0.f;
    if (dstT) dstT[d * (64 + PAD) + r] = v;
    if (rm) rm[r * (HD + PAD) + d] = v;
  }
}

// acc[i][j] = sum_d A[d][ra+i] * B[d][cb+j] over transposed smem tiles (4x4 micro-tile).
template <int HD>
__device__ __forceinline__ void mm_tt(const float* AT, const float* BT, int ra, int cb, float acc[4][4]) {
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) acc[i][j] = 0.f;
#pragma unroll 8
  for (int d = 0; d < HD; d++) {
    const float4 a = *reinterpret_cast<const float4*>(AT + d * (64 + PAD) + ra);
    const float4 bb = *reinterpret_cast<const float4*>(BT + d * (64 + PAD) + cb);
    const float av[4] = {a.x, a.y, a.z, a.w};
    const float bv[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int j = 0; j < 4; j++) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
  }
}

// --------------------------------------------------------------- forward
template <int HD>
__global__ void __launch_bounds__(256) k_attn_fwd(const float* __restrict__ qkv, const float2* __restrict__ rope_cs,
                                                  float* __restrict__ out, float* __restrict__ lse, AttnShape s) {
  constexpr int DPT = HD / 16;
  extern __shared__ __align__(16) float sm[];
  float* QT = sm;                       // [HD][64+PAD]
  float* KT = QT + HD * (64 + PAD);     // [HD][64+PAD]
  float* V = KT + HD * (64 + PAD);      // [64][HD+PAD]
  float* P = V + 64 * (HD + PAD);       // [64][64+PAD]
  float* VT_unused = nullptr;
  (void)VT_unused;
  const int qt = blockIdx.x, bh = blockIdx.y, b = bh / s.H, h = bh % s.H;
  const int tid = threadIdx.x, ty = tid / 16, tx = tid % 16;
  const int q0 = qt * BQ;
  load_tile<HD>(qkv, rope_cs, s, b, h, q0, 0, s.rope, QT, nullptr);
  float o[4][DPT];
  float m[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int j = 0; j < DPT; j++) o[i][j] = 0.f;
  }
  const int nkv = min((q0 + BQ + BKV - 1) / BKV, (s.T + BKV - 1) / BKV);
  for (int kt = 0; kt < nkv; kt++) {
    const int k0 = kt * BKV;
    __syncthreads();
    load_tile<HD>(qkv, rope_cs, s, b, h, k0, s.E, s.rope, KT, nullptr);
    for (int e = tid; e < 64 * HD; e += 256) {
      const int r = e / HD, d = e % HD, t = k0 + r;
      V[r * (HD + PAD) + d] = t < s.T ? qkv[((long)b * s.T + t) * 3 * s.E + 2 * s.E + h * HD + d] : 0.f;
    }
    __syncthreads();
    float sc[4][4];
    mm_tt<HD>(QT, KT, ty * 4, tx * 4, sc);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int qi = q0 + ty * 4 + i;
      float rmax = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int kj = k0 + tx * 4 + j;
        const bool valid = kj <= qi && kj < s.T;
        sc[i][j] = valid ? sc[i][j] * s.scale : -INFINITY;
        rmax = fmaxf(rmax, sc[i][j]);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, off));
      const float mnew = fmaxf(m[i], rmax);
      const float alpha = (m[i] == -INFINITY) ? 0.f : __expf(m[i] - mnew);
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float p = (sc[i][j] == -INFINITY) ? 0.f : __expf(sc[i][j] - mnew);
        sc[i][j] = p;
        rs += p;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
      l[i] = l[i] * alpha + rs;
      m[i] = mnew;
#pragma unroll
      for (int j = 0; j < DPT; j++) o[i][j] *= alpha;
      *reinterpret_cast<float4*>(P + (ty * 4 + i) * (64 + PAD) + tx * 4) =
          make_float4(sc[i][0], sc[i][1], sc[i][2], sc[i][3]);
    }
    __syncthreads();
    const int jmax = min(BKV, s.T - k0);
    for (int j = 0; j < jmax; j++) {
      float pv[4];
#pragma unroll
      for (int i = 0; i < 4; i++) pv[i] = P[(ty * 4 + i) * (64 + PAD) + j];
      const float* vr = V + j * (HD + PAD) + tx * DPT;
#pragma unroll
      for (int d = 0; d < DPT; d++) {
        const float vv = vr[d];
#pragma unroll
        for (int i = 0; i < 4; i++) o[i][d] = fmaf(pv[i], vv, o[i][d]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int qi = q0 + ty * 4 + i;
    if (qi >= s.T) continue;
    const float inv = 1.f / l[i];
    float* dst = out + ((long)b * s.T + qi) * s.E + h * HD + tx * DPT;
#pragma unroll
    for (int d = 0; d < DPT; d++) dst[d] = o[i][d] * inv;
    if (tx == 0) lse[(long)bh * s.T + qi] = m[i] + logf(l[i]);
  }
}

// D[b,h,t] = sum_d dO * O  (softmax backward row term)
__global__ void k_attn_dot(const float* __restrict__ o, const float* __restrict__ dout, float* __restrict__ D,
                           AttnShape s) {
  const int warps = blockDim.x / 32;
  const long row = (long)blockIdx.x * warps + threadIdx.x / 32;  // over B*T*H
  const int lane = threadIdx.x & 31;
  if (row >= (long)s.B * s.T * s.H) return;
  const int h = (int)(row % s.H);
  const long n = row / s.H;  // token
  const int b = (int)(n / s.T), t = (int)(n % s.T);
  const float* a = o + n * s.E + h * s.hd;
  const float* g = dout + n * s.E + h * s.hd;
  float acc = 0.f;
  for (int d = lane; d < s.hd; d += 32) acc += a[d] * g[d];
  acc = warp_sum(acc);
  if (lane == 0) D[((long)b * s.H + h) * s.T + t] = acc;
}

// Writes a [64][HD] register tile (rows r0+ty*4+i, cols tx*DPT+d) into dqkv, applying the
// inverse RoPE rotation (rotate by -theta) when `rotate`.
template <int HD, int DPT>
__device__ __forceinline__ void store_grad(float (&acc)[4][DPT], float* __restrict__ dqkv,
                                           const float2* __restrict__ rope_cs, const AttnShape& s, int b, int h,
                                           int r0, int col_off, bool rotate) {
  const int tid = threadIdx.x, ty = tid / 16, tx = tid % 16;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int t = r0 + ty * 4 + i;
    float v[DPT];
#pragma unroll
    for (int d = 0; d < DPT; d++) v[d] = acc[i][d];
    if (rotate) {
      if (DPT >= 2) {
#pragma unroll
        for (int d = 0; d < DPT; d += 2) {
          const int pr = (tx * DPT + d) / 2;
          const float2 c = (t < s.T) ? rope_cs[t * (HD / 2) + pr] : make_float2(1.f, 0.f);
          const float g0 = v[d], g1 = v[d + 1];
          v[d] = g0 * c.x + g1 * c.y;
          v[d + 1] = -g0 * c.y + g1 * c.x;
        }
      } else {
        // HD == 16: the pair partner lives in the neighbouring lane (tx ^ 1).
        const float other = __shfl_xor_sync(0xffffffffu, v[0], 1);
        const int pr = tx / 2;
        const float2 c = (t < s.T) ? rope_cs[t * (HD / 2) + pr] : make_float2(1.f, 0.f);
        if ((tx & 1) == 0)
          v[0] = v[0] * c.x + other * c.y;
        else
          v[0] = -other * c.y + v[0] * c.x;
      }
    }
    if (t < s.T) {
      float* dst = dqkv + ((long)b * s.T + t) * 3 * s.E + col_off + h * HD + tx * DPT;
#pragma unroll
      for (int d = 0; d < DPT; d++) dst[d] = v[d];
    }
  }
}

// --------------------------------------------------------- backward dK, dV
template <int HD>
__global__ void __launch_bounds__(256) k_attn_bwd_kv(const float* __restrict__ qkv, const float2* __restrict__ rope_cs,
                                                     const float* __restrict__ dout, const float* __restrict__ lse,
                                                     const float* __restrict__ D, float* __restrict__ dqkv,
                                                     AttnShape s) {
  constexpr int DPT = HD / 16;
  extern __shared__ __align__(16) float sm[];
  float* KT = sm;                       // [HD][64+PAD]
  float* VT = KT + HD * (64 + PAD);     // [HD][64+PAD]
  float* QT = VT + HD * (64 + PAD);     // [HD][64+PAD]
  float* Qr = QT + HD * (64 + PAD);     // [64][HD+PAD]
  float* dOT = Qr + 64 * (HD + PAD);    // [HD][64+PAD]
  float* dOr = dOT + HD * (64 + PAD);   // [64][HD+PAD]
  float* Pt = dOr + 64 * (HD + PAD);    // [64 keys][64+PAD queries]
  float* dSt = Pt + 64 * (64 + PAD);    // [64 keys][64+PAD queries]
  float* lq = dSt + 64 * (64 + PAD);    // [64]
  float* Dq = lq + 64;                  // [64]
  const int kt = blockIdx.x, bh = blockIdx.y, b = bh / s.H, h = bh % s.H;
  const int tid = threadIdx.x, ty = tid / 16, tx = tid % 16;
  const int k0 = kt * BKV;
  load_tile<HD>(qkv, rope_cs, s, b, h, k0, s.E, s.rope, KT, nullptr);
  load_tile<HD>(qkv, rope_cs, s, b, h, k0, 2 * s.E, false, VT, nullptr);
  float dk[4][DPT], dv[4][DPT];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int d = 0; d < DPT; d++) dk[i][d] = dv[i][d] = 0.f;
  const int nq = (s.T + BQ - 1) / BQ;
  for (int qt = kt; qt < nq; qt++) {
    const int q0 = qt * BQ;
    __syncthreads();
    load_tile<HD>(qkv, rope_cs, s, b, h, q0, 0, s.rope, QT, Qr);
    load_tile_ne<HD>(dout, s, b, h, q0, dOT, dOr);
    for (int e = tid; e < 64; e += 256) {
      const int t = q0 + e;
      lq[e] = t < s.T ? lse[(long)bh * s.T + t] : 0.f;
      Dq[e] = t < s.T ? D[(long)bh * s.T + t] : 0.f;
    }
    __syncthreads();
    // St[key][query] and dPt[key][query]
    float st[4][4], dpt[4][4];
    mm_tt<HD>(KT, QT, ty * 4, tx * 4, st);
    mm_tt<HD>(VT, dOT, ty * 4, tx * 4, dpt);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int kj = k0 + ty * 4 + i;
      float p4[4], ds4[4];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int qi = q0 + tx * 4 + j;
        const bool valid = kj <= qi && qi < s.T && kj < s.T;
        const float p = valid ? __expf(st[i][j] * s.scale - lq[tx * 4 + j]) : 0.f;
        p4[j] = p;
        ds4[j] = p * (dpt[i][j] - Dq[tx * 4 + j]);
      }
      *reinterpret_cast<float4*>(Pt + (ty * 4 + i) * (64 + PAD) + tx * 4) = make_float4(p4[0], p4[1], p4[2], p4[3]);
      *reinterpret_cast<float4*>(dSt + (ty * 4 + i) * (64 + PAD) + tx * 4) =
          make_float4(ds4[0], ds4[1], ds4[2], ds4[3]);
    }
    __syncthreads();
    const int jmax = min(BQ, s.T - q0);
    for (int j = 0; j < jmax; j++) {
      float pv[4], dsv[4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        pv[i] = Pt[(ty * 4 + i) * (64 + PAD) + j];
        dsv[i] = dSt[(ty * 4 + i) * (64 + PAD) + j];
      }
      const float* gor = dOr + j * (HD + PAD) + tx * DPT;
      const float* qr = Qr + j * (HD + PAD) + tx * DPT;
#pragma unroll
      for (int d = 0; d < DPT; d++) {
        const float g = gor[d], q = qr[d];
#pragma unroll
        for (int i = 0; i < 4; i++) {
          dv[i][d] = fmaf(pv[i], g, dv[i][d]);
          dk[i][d] = fmaf(dsv[i], q, dk[i][d]);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int d = 0; d < DPT; d++) dk[i][d] *= s.scale;
  store_grad<HD, DPT>(dk, dqkv, rope_cs, s, b, h, k0, s.E, s.rope);
  store_grad<HD, DPT>(dv, dqkv, rope_cs, s, b, h, k0, 2 * s.E, false);
}

// --------------------------------------------------------------- backward dQ
template <int HD>
__global__ void __launch_bounds__(256) k_attn_bwd_q(const float* __restrict__ qkv, const float2* __restrict__ rope_cs,
                                                    const float* __restrict__ dout, const float* __restrict__ lse,
                                                    const float* __restrict__ D, float* __restrict__ dqkv,
                                                    AttnShape s) {
  constexpr int DPT = HD / 16;
  extern __shared__ __align__(16) float sm[];
  float* QT = sm;                       // [HD][64+PAD]
  float* dOT = QT + HD * (64 + PAD);    // [HD][64+PAD]
  float* KT = dOT + HD * (64 + PAD);    // [HD][64+PAD]
  float* VT = KT + HD * (64 + PAD);     // [HD][64+PAD]
  float* Kr = VT + HD * (64 + PAD);     // [64][HD+PAD]
  float* dS = Kr + 64 * (HD + PAD);     // [64 q][64+PAD k]
  const int qt = blockIdx.x, bh = blockIdx.y, b = bh / s.H, h = bh % s.H;
  const int tid = threadIdx.x, ty = tid / 16, tx = tid % 16;
  const int q0 = qt * BQ;
  load_tile<HD>(qkv, rope_cs, s, b, h, q0, 0, s.rope, QT, nullptr);
  load_tile_ne<HD>(dout, s, b, h, q0, dOT, nullptr);
  float lrow[4], drow[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int t = q0 + ty * 4 + i;
    lrow[i] = t < s.T ? lse[(long)bh * s.T + t] : 0.f;
    drow[i] = t < s.T ? D[(long)bh * s.T + t] : 0.f;
  }
  float dq[4][DPT];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int d = 0; d < DPT; d++) dq[i][d] = 0.f;
  const int nkv = min((q0 + BQ + BKV - 1) / BKV, (s.T + BKV - 1) / BKV);
  for (int kt = 0; kt < nkv; kt++) {
    const int k0 = kt * BKV;
    __syncthreads();
    load_tile<HD>(qkv, rope_cs, s, b, h, k0, s.E, s.rope, KT, Kr);
    load_tile<HD>(qkv, rope_cs, s, b, h, k0, 2 * s.E, false, VT, nullptr);
    __syncthreads();
    float sc[4][4], dp[4][4];
    mm_tt<HD>(QT, KT, ty * 4, tx * 4, sc);
    mm_tt<HD>(dOT, VT, ty * 4, tx * 4, dp);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int qi = q0 + ty * 4 + i;
      float ds4[4];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int kj = k0 + tx * 4 + j;
        const bool valid = kj <= qi && kj < s.T && qi < s.T;
        const float p = valid ? __expf(sc[i][j] * s.scale - lrow[i]) : 0.f;
        ds4[j] = p * (dp[i][j] - drow[i]);
      }
      *reinterpret_cast<float4*>(dS + (ty * 4 + i) * (64 + PAD) + tx * 4) =
          make_float4(ds4[0], ds4[1], ds4[2], ds4[3]);
    }
    __syncthreads();
    const int jmax = min(BKV, s.T - k0);
    for (int j = 0; j < jmax; j++) {
      float dsv[4];
#pragma unroll
      for (int i = 0; i < 4; i++) dsv[i] = dS[(ty * 4 + i) * (64 + PAD) + j];
      const float* kr = Kr + j * (HD + PAD) + tx * DPT;
#pragma unroll
      for (int d = 0; d < DPT; d++) {
        const float kv = kr[d];
#pragma unroll
        for (int i = 0; i < 4; i++) dq[i][d] = fmaf(dsv[i], kv, dq[i][d]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int d = 0; d < DPT; d++) dq[i][d] *= s.scale;
  store_grad<HD, DPT>(dq, dqkv, rope_cs, s, b, h, q0, 0, s.rope);
}

template <int HD>
int launch_fwd(cudaStream_t st, const float* qkv, const float2* cs, float* out, float* lse, const AttnShape& s) {
  const int smem = (2 * HD * (64 + PAD) + 64 * (HD + PAD) + 64 * (64 + PAD)) * 4;
  static std::atomic<uint64_t> cfg{0};
  RC(smem_attr_per_device(cfg, k_attn_fwd<HD>, smem));
  dim3 grid(ceil_div(s.T, BQ), s.B * s.H);
  k_attn_fwd<HD><<<grid, 256, smem, st>>>(qkv, cs, out, lse, s);
  TURT_LAUNCH_CHECK();
  return OK;
}

template <int HD>
int launch_bwd(cudaStream_t st, const float* qkv, const float2* cs, const float* out, const float* dout,
               const float* lse, float* D, float* dqkv, const AttnShape& s) {
  const long rows = (long)s.B * s.T * s.H;
  k_attn_dot<<<(int)((rows + 7) / 8), 256, 0, st>>>(out, dout, D, s);
  TURT_LAUNCH_CHECK();
  const int smem_kv = (4 * HD * (64 + PAD) + 2 * 64 * (HD + PAD) + 2 * 64 * (64 + PAD) + 128) * 4;
  const int smem_q = (4 * HD * (64 + PAD) + 64 * (HD + PAD) + 64 * (64 + PAD)) * 4;
  static std::atomic<uint64_t> cfg_kv{0}, cfg_q{0};
  RC(smem_attr_per_device(cfg_kv, k_attn_bwd_kv<HD>, smem_kv));
  RC(smem_attr_per_device(cfg_q, k_attn_bwd_q<HD>, smem_q));
  dim3 grid(ceil_div(s.T, 64), s.B * s.H);
  k_attn_bwd_kv<HD><<<grid, 256, smem_kv, st>>>(qkv, cs, dout, lse, D, dqkv, s);
  TURT_LAUNCH_CHECK();
  k_attn_bwd_q<HD><<<grid, 256, smem_q, st>>>(qkv, cs, dout, lse, D, dqkv, s);
  TURT_LAUNCH_CHECK();
  return OK;
}

}  // namespace

bool attention_supported_hd(int hd) { return hd == 16 || hd == 32 || hd == 64; }

int attention_fwd(cudaStream_t st, const float* qkv, const float2* rope_cs, float* out, float* lse, int B, int T, int H,
                  int hd, int rope) {
  AttnShape s{B, T, H, hd, H * hd, 1.0f / sqrtf((float)hd), rope};
  switch (hd) {
    case 16: return launch_fwd<16>(st, qkv, rope_cs, out, lse, s);
    case 32: return launch_fwd<32>(st, qkv, rope_cs, out, lse, s);
    case 64: return launch_fwd<64>(st, qkv, rope_cs, out, lse, s);
  }
  set_error("attention: head dim must be 16, 32 or 64");
  return ERR_UNSUPPORTED;
}

int attention_bwd(cudaStream_t st, const float* qkv, const float2* rope_cs, const float* out, const float* dout,
                  const float* lse, float* D, float* dqkv, int B, int T, int H, int hd, int rope) {
  AttnShape s{B, T, H, hd, H * hd, 1.0f / sqrtf((float)hd), rope};
  switch (hd) {
    case 16: return launch_bwd<16>(st, qkv, rope_cs, out, dout, lse, D, dqkv, s);
    case 32: return launch_bwd<32>(st, qkv, rope_cs, out, dout, lse, D, dqkv, s);
    case 64: return launch_bwd<64>(st, qkv, rope_cs, out, dout, lse, D, dqkv, s);
  }
  set_error("attention: head dim must be 16, 32 or 64");
  return ERR_UNSUPPORTED;
}

}  // namespace turt
