// attention_tc.cu -- causal self-attention on the tensor cores, materialised per head.
//
// The reference computes attention per layer as (src/models/gpu-gpt.ts:143-168)
//   split heads -> ROPE(q), ROPE(k) -> S = bmmBT(q, k) -> S *= 1/sqrt(hd)
//   -> maskedFillCausal(S, -1e9) -> P = softmax(S) -> O = bmm(P, v) -> merge heads
// and its autograd tape runs the matching backward ops.  This file keeps that dataflow and
// puts every contraction on the batched tcgen05 GEMM (3xTF32) with the B*H heads as a
// two-level (sequence, head) batch, so q, k, v, dO and the merged outputs are addressed in
// place inside the fused [N][3E] / [N][E] activations:
//   forward : [RoPE q,k -> head-major copies, normally done by the qkv projection's epilogue]
//             S = q k^T (upper tiles skipped)
//             softmax rows (scale, causal mask, P kept)  O = P v (K-range cut at the diagonal)
//   backward: dP = dO v^T  dS = P (dP - rowsum(P dP)) * scale  dV = P^T dO  dQ = dS k
//             dK = dS^T q  (inverse RoPE in the dQ / dK epilogues)
// Masked probabilities are exact zeros, so the causal tile / K-range skips change no result.
// For T <= 256 with head dims 32 / 64 in 3xTF32 the same steps run as three fused kernels
// (attention_fused.cu: forward; dP + dS + dQ; dV + dK), for longer sequences with those head
// dims as online-softmax kernels without [T][T] buffers (attention_flash.cu); this chain covers
// the other shapes.
#include "attention.cuh"
#include "gemm.cuh"

namespace turt {
namespace {

// q, k of [N][3E] (token n = b*T + t, head h at columns h*hd) -> rotated head-major
// copies [B*H][T][hd].  RoPE rotates interleaved pairs (src/math/tensor.ts:650-700):
// (x0, x1) -> (x0 c - x1 s, x0 s + x1 c) with (c, s) = rope_cs[t][pair].
__global__ void k_rope_heads(const float* __restrict__ qkv, const float2* __restrict__ cs, float* __restrict__ qr,
                             float* __restrict__ kr, int B, int T, int H, int hd) {
  pdl_trigger();
  pdl_wait();
  const int E = H * hd, q4 = hd / 4;
  const long total = (long)B * T * H * q4;
  const int which = blockIdx.y;  // 0 = q, 1 = k
  const float* src = qkv + which * E;
  float* dst = which ? kr : qr;
  for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (long)gridDim.x * blockDim.x) {
    const int f = (int)(e % q4);
    const long r = e / q4;  // (n, h)
    const int h = (int)(r % H);
    const long n = r / H;
    const int t = (int)(n % T), b = (int)(n / T);
    const float4 x = *reinterpret_cast<const float4*>(src + n * 3 * E + h * hd + 4 * f);
    const float2 c0 = cs[(long)t * (hd / 2) + 2 * f], c1 = cs[(long)t * (hd / 2) + 2 * f + 1];
    float4 y;
    y.x = x.x * c0.x - x.y * c0.y;
    y.y = x.x * c0.y + x.y * c0.x;
    y.z = x.z * c1.x - x.w * c1.y;
    y.w = x.z * c1.y + x.w * c1.x;
    *reinterpret_cast<float4*>(dst + (((long)b * H + h) * T + t) * hd + 4 * f) = y;
  }
}

constexpr int kRowWarps = 8;       // warps per 256-thread block

// Causal softmax of score rows in place: P[j] = exp(s_j*scale - max) / sum for j <= i, 0 for
// i < j < pitch.  A warp handles R consecutive rows at once (more loads in flight); lane `lane`
// owns the float4 chunks starting at 4*(32c + lane), c < C = ceil(pitch / 128).  Entries
// right of the diagonal may be unwritten (skipped score tiles): they are read only into
// masked lanes.
template <int C, int R>
__global__ void __launch_bounds__(256) k_softmax_causal(float* __restrict__ S, long rows, int T, long pitch,
                                                        float scale) {
  pdl_trigger();
  pdl_wait();
  const long row0 = ((long)blockIdx.x * kRowWarps + threadIdx.x / 32) * R;
  const int lane = threadIdx.x & 31;
  if (row0 >= rows) return;
  float v[R][C * 4];
  float mx[R];
#pragma unroll
  for (int r = 0; r < R; r++) {
    const long row = row0 + r;
    const int n = row < rows ? (int)(row % T) + 1 : 0;  // valid keys
    const float* p = S + (row / T) * T * pitch + (row % T) * pitch;
    mx[r] = -INFINITY;
#pragma unroll
    for (int c = 0; c < C; c++) {
      const int j0 = (c * 32 + lane) * 4;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (j0 < n) x = *reinterpret_cast<const float4*>(p + j0);
      v[r][c * 4 + 0] = j0 + 0 < n ? x.x * scale : -INFINITY;
      v[r][c * 4 + 1] = j0 + 1 < n ? x.y * scale : -INFINITY;
      v[r][c * 4 + 2] = j0 + 2 < n ? x.z * scale : -INFINITY;
      v[r][c * 4 + 3] = j0 + 3 < n ? x.w * scale : -INFINITY;
    }
  }
#pragma unroll
  for (int r = 0; r < R; r++) {
#pragma unroll
    for (int c = 0; c < C * 4; c++) mx[r] = fmaxf(mx[r], v[r][c]);
    mx[r] = warp_max(mx[r]);
  }
#pragma unroll
  for (int r = 0; r < R; r++) {
    const long row = row0 + r;
    if (row >= rows) break;
    float sum = 0.f;
#pragma unroll
    for (int c = 0; c < C * 4; c++) {
      v[r][c] = expf(v[r][c] - mx[r]);  // exp(-inf) = 0 for masked keys
      sum += v[r][c];
    }
    sum = warp_sum(sum);
    const float inv = 1.0f / sum;
    float* p = S + (row / T) * T * pitch + (row % T) * pitch;
#pragma unroll
    for (int c = 0; c < C; c++) {
      const int j0 = (c * 32 + lane) * 4;
      if (j0 < pitch)
        *reinterpret_cast<float4*>(p + j0) =
            make_float4(v[r][c * 4] * inv, v[r][c * 4 + 1] * inv, v[r][c * 4 + 2] * inv, v[r][c * 4 + 3] * inv);
    }
  }
}

// Rows longer than the register budget: three passes over memory, one warp per row.
__global__ void __launch_bounds__(256) k_softmax_causal_long(float* __restrict__ S, long rows, int T, long pitch,
                                                             float scale) {
  pdl_trigger();
  pdl_wait();
  const long row = (long)blockIdx.x * kRowWarps + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float* p = S + (row / T) * T * pitch + (row % T) * pitch;
  const int n = (int)(row % T) + 1;
  float mx = -INFINITY;
  for (int j = lane; j < n; j += 32) mx = fmaxf(mx, p[j] * scale);
  mx = warp_max(mx);
  float sum = 0.f;
  for (int j = lane; j < n; j += 32) sum += expf(p[j] * scale - mx);
  sum = warp_sum(sum);
  const float inv = 1.0f / sum;
  for (int j = lane; j < pitch; j += 32) p[j] = j < n ? expf(p[j] * scale - mx) * inv : 0.f;
}

// Softmax + scale backward, in place over dP: dS_j = P_j (dP_j - sum_k P_k dP_k) * scale for
// j <= i, 0 right of the diagonal (masked scores get no gradient).  Same row mapping as above.
template <int C, int R>
__global__ void __launch_bounds__(256) k_softmax_causal_bwd(const float* __restrict__ P, float* __restrict__ dP,
                                                            long rows, int T, long pitch, float scale) {
  pdl_trigger();
  pdl_wait();
  const long row0 = ((long)blockIdx.x * kRowWarps + threadIdx.x / 32) * R;
  const int lane = threadIdx.x & 31;
  if (row0 >= rows) return;
  float pv[R][C * 4], gv[R][C * 4], dot[R];
#pragma unroll
  for (int r = 0; r < R; r++) {
    const long row = row0 + r;
    const int n = row < rows ? (int)(row % T) + 1 : 0;
    const long off = (row / T) * T * pitch + (row % T) * pitch;
    dot[r] = 0.f;
#pragma unroll
    for (int c = 0; c < C; c++) {
      const int j0 = (c * 32 + lane) * 4;
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f), d = a;
      if (j0 < n) {
        a = *reinterpret_cast<const float4*>(P + off + j0);
        d = *reinterpret_cast<const float4*>(dP + off + j0);
      }
      pv[r][c * 4 + 0] = j0 + 0 < n ? a.x : 0.f;
      pv[r][c * 4 + 1] = j0 + 1 < n ? a.y : 0.f;
      pv[r][c * 4 + 2] = j0 + 2 < n ? a.z : 0.f;
      pv[r][c * 4 + 3] = j0 + 3 < n ? a.w : 0.f;
      gv[r][c * 4 + 0] = j0 + 0 < n ? d.x : 0.f;
      gv[r][c * 4 + 1] = j0 + 1 < n ? d.y : 0.f;
      gv[r][c * 4 + 2] = j0 + 2 < n ? d.z : 0.f;
      gv[r][c * 4 + 3] = j0 + 3 < n ? d.w : 0.f;
    }
  }
#pragma unroll
  for (int r = 0; r < R; r++) {
#pragma unroll
    for (int c = 0; c < C * 4; c++) dot[r] += pv[r][c] * gv[r][c];
    dot[r] = warp_sum(dot[r]);
  }
#pragma unroll
  for (int r = 0; r < R; r++) {
    const long row = row0 + r;
    if (row >= rows) break;
    float* g = dP + (row / T) * T * pitch + (row % T) * pitch;
#pragma unroll
    for (int c = 0; c < C; c++) {
      const int j0 = (c * 32 + lane) * 4;
      if (j0 < pitch) {
        float4 o;
        o.x = pv[r][c * 4 + 0] * (gv[r][c * 4 + 0] - dot[r]) * scale;
        o.y = pv[r][c * 4 + 1] * (gv[r][c * 4 + 1] - dot[r]) * scale;
        o.z = pv[r][c * 4 + 2] * (gv[r][c * 4 + 2] - dot[r]) * scale;
        o.w = pv[r][c * 4 + 3] * (gv[r][c * 4 + 3] - dot[r]) * scale;
        *reinterpret_cast<float4*>(g + j0) = o;
      }
    }
  }
}

__global__ void __launch_bounds__(256) k_softmax_causal_bwd_long(const float* __restrict__ P, float* __restrict__ dP,
                                                                 long rows, int T, long pitch, float scale) {
  pdl_trigger();
  pdl_wait();
  const long row = (long)blockIdx.x * kRowWarps + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const long off = (row / T) * T * pitch + (row % T) * pitch;
  const float* p = P + off;
  float* g = dP + off;
  const int n = (int)(row % T) + 1;
  float dot = 0.f;
  for (int j = lane; j < n; j += 32) dot += p[j] * g[j];
  dot = warp_sum(dot);
  for (int j = lane; j < pitch; j += 32) g[j] = j < n ? p[j] * (g[j] - dot) * scale : 0.f;
}

template <int C>
int rows_launch_c(cudaStream_t st, long rows, int T, long pitch, float scale, float* S, const float* P, bool bwd) {
  constexpr int R = C <= 2 ? 4 : (C <= 4 ? 2 : 1);  // rows per warp: ~8 float4 loads in flight per array
  const int blocks = (int)((rows + kRowWarps * R - 1) / (kRowWarps * R));
  if (!bwd)
    TURT_CHECK_CUDA((launch_pdl(k_softmax_causal<C, R>, dim3(blocks), dim3(256), 0, st, S, rows, T, pitch, scale)));
  else
    TURT_CHECK_CUDA((launch_pdl(k_softmax_causal_bwd<C, R>, dim3(blocks), dim3(256), 0, st, P, S, rows, T, pitch, scale)));
  TURT_LAUNCH_CHECK();
  return OK;
}

int rows_launch(cudaStream_t st, long rows, int T, long pitch, float scale, float* S, const float* P, bool bwd) {
  switch ((pitch + 127) / 128) {
    case 1: return rows_launch_c<1>(st, rows, T, pitch, scale, S, P, bwd);
    case 2: return rows_launch_c<2>(st, rows, T, pitch, scale, S, P, bwd);
    case 3: return rows_launch_c<3>(st, rows, T, pitch, scale, S, P, bwd);
    case 4: return rows_launch_c<4>(st, rows, T, pitch, scale, S, P, bwd);
    case 5: case 6: return rows_launch_c<6>(st, rows, T, pitch, scale, S, P, bwd);
    case 7: case 8: return rows_launch_c<8>(st, rows, T, pitch, scale, S, P, bwd);
    default: break;
  }
  const int blocks = (int)((rows + kRowWarps - 1) / kRowWarps);
  if (!bwd)
    TURT_CHECK_CUDA((launch_pdl(k_softmax_causal_long, dim3(blocks), dim3(256), 0, st, S, rows, T, pitch, scale)));
  else
    TURT_CHECK_CUDA((launch_pdl(k_softmax_causal_bwd_long, dim3(blocks), dim3(256), 0, st, P, S, rows, T, pitch, scale)));
  TURT_LAUNCH_CHECK();
  return OK;
}

int grid_for(long total) {
  long b = (total + 255) / 256;
  if (b > 148 * 16) b = 148 * 16;
  return (int)(b < 1 ? 1 : b);
}

// Operand views.  Batch index = b * H + h (inner level = head).
struct Views {
  GemmOperand q, k, v, dout, P, PT;
  long pitch;
};

Views views(const float* qkv, const float* dout, const AttnTensors& at, const float* P, int T, int H, int hd,
            bool rope) {
  const int E = H * hd;
  Views w;
  w.pitch = attn_pitch(T);
  auto inplace = [&](const float* base, long ld, long rows_stride) {
    GemmOperand o;
    o.ptr = base;
    o.ld = ld;
    o.stride = hd;
    o.stride_hi = rows_stride;
    return o;
  };
  auto headmajor = [&](const float* base) {
    GemmOperand o;
    o.ptr = base;
    o.ld = hd;
    o.stride = (long)T * hd;
    o.stride_hi = (long)H * T * hd;
    return o;
  };
  w.q = rope ? headmajor(at.qr) : inplace(qkv, 3L * E, (long)T * 3 * E);
  w.k = rope ? headmajor(at.kr) : inplace(qkv + E, 3L * E, (long)T * 3 * E);
  w.v = inplace(qkv + 2 * E, 3L * E, (long)T * 3 * E);
  if (dout) w.dout = inplace(dout, E, (long)T * E);
  w.P.ptr = P;
  w.P.ld = w.pitch;
  w.P.stride = (long)T * w.pitch;
  w.P.stride_hi = (long)H * T * w.pitch;
  w.PT = w.P;
  w.PT.mn_major = true;
  return w;
}

GemmOperand mn(GemmOperand o) {
  o.mn_major = true;
  return o;
}

GemmEpi scores_epi(float* S, int T, int H, long pitch) {
  GemmEpi e;
  e.kind = EPI_STORE;
  e.C = S;
  e.ldc = pitch;
  e.strideC = (long)T * pitch;
  e.strideC_hi = (long)H * T * pitch;
  e.bdiv = H;
  e.causal = CAUSAL_SKIP_UPPER;
  return e;
}

// [T][hd] per-head output written into a merged [N][ld] activation at column `col`.
GemmEpi merged_epi(float* base, long ld, int T, int hd, int causal) {
  GemmEpi e;
  e.kind = EPI_STORE;
  e.C = base;
  e.ldc = ld;
  e.strideC = hd;
  e.strideC_hi = (long)T * ld;
  e.causal = causal;
  return e;
}

}  // namespace

bool attention_tc_supported(int hd) { return hd >= 16 && hd <= 256 && hd % 16 == 0; }

bool attention_tc_prefers_online(int T, int hd, int precision) {
  return precision == GEMM_TF32X3 && !attention_fused_supported(T, hd) && attention_flash_supported(T, hd);
}

int attention_tc_fwd(cudaStream_t st, const float* qkv, const float2* rope_cs, float* out, const AttnTensors& at, int B,
                     int T, int H, int hd, int rope, int rotated, int* flags, int precision) {
  TURT_REQUIRE(attention_tc_supported(hd), "attention: head dim must be a multiple of 16 in [16, 256]");
  const bool flash = at.online;
  if (flash)
    TURT_REQUIRE(precision == GEMM_TF32X3 && attention_flash_supported(T, hd),
                 "online-softmax attention: needs 3xTF32 and a head dim of 32 or 64");
  TURT_REQUIRE((flash ? at.lse != nullptr : at.P != nullptr) && (!rope || (at.qr && at.kr)), "attention: buffers missing");
  const int E = H * hd, BH = B * H;
  const float scale = 1.0f / sqrtf((float)hd);
  if (rope && !rotated) {
    TURT_CHECK_CUDA((launch_pdl(k_rope_heads, dim3(dim3(grid_for((long)B * T * H * hd / 4), 2)), dim3(256), 0, st, qkv, rope_cs, at.qr, at.kr, B, T, H, hd)));
    TURT_LAUNCH_CHECK();
  }
  const Views w = views(qkv, nullptr, at, at.P, T, H, hd, rope != 0);
  if (flash) return attention_flash_fwd(st, w.q, w.k, w.v, out, E, at.lse, B, T, H, hd, scale, flags);
  if (precision == GEMM_TF32X3 && attention_fused_supported(T, hd))
    return attention_fused_fwd(st, w.q, w.k, w.v, at.P, w.pitch, out, E, B, T, H, hd, scale, flags);
  // S = q k^T  (k [T][hd] is the K-major B operand)
  RC(gemm_tf32(st, T, T, hd, BH, w.q, w.k, scores_epi(at.P, T, H, w.pitch), flags, precision));
  RC(rows_launch(st, (long)BH * T, T, w.pitch, scale, at.P, nullptr, false));
  // O = P v  (v [T][hd] is the MN-major B operand), merged into out[N][E]
  GemmEpi e = merged_epi(out, E, T, hd, CAUSAL_K_LOWER);
  e.bdiv = H;
  RC(gemm_tf32(st, T, hd, T, BH, w.P, mn(w.v), e, flags, precision));
  return OK;
}

int attention_tc_bwd(cudaStream_t st, const float* qkv, const float2* rope_cs, const float* out, const float* dout,
                     const AttnTensors& at, const AttnScratch& sc, float* dqkv, int B, int T, int H, int hd, int rope,
                     int* flags, int precision) {
  TURT_REQUIRE(attention_tc_supported(hd), "attention: head dim must be a multiple of 16 in [16, 256]");
  const int E = H * hd, BH = B * H;
  const float scale = 1.0f / sqrtf((float)hd);
  if (at.online) {
    TURT_REQUIRE(precision == GEMM_TF32X3 && attention_flash_supported(T, hd),
                 "online-softmax attention: needs 3xTF32 and a head dim of 32 or 64");
    TURT_REQUIRE(at.lse && sc.D && out && (!rope || (at.qr && at.kr)), "attention: buffers missing");
    const Views w = views(qkv, dout, at, nullptr, T, H, hd, rope != 0);
    GemmOperand o;  // the forward's merged output [N][E], head h at columns h * hd
    o.ptr = out;
    o.ld = E;
    o.stride = hd;
    o.stride_hi = (long)T * E;
    return attention_flash_bwd(st, w.q, w.k, w.v, w.dout, o, at.lse, sc.D, dqkv, 3L * E, rope ? rope_cs : nullptr, B,
                               T, H, hd, scale, flags);
  }
  TURT_REQUIRE(at.P && sc.dS && (!rope || (at.qr && at.kr)), "attention: buffers missing");
  const Views w = views(qkv, dout, at, at.P, T, H, hd, rope != 0);
  const bool fused = precision == GEMM_TF32X3 && attention_fused_supported(T, hd);
  if (fused) {
    // dS and dQ (-> dqkv[:, 0:E), rotated back for RoPE) in one kernel
    RC(attention_fused_dsoftmax(st, w.dout, w.v, w.k, at.P, sc.dS, w.pitch, dqkv, 3L * E, rope ? rope_cs : nullptr, B,
                                T, H, hd, scale, flags));
  } else {
    // dP = dO v^T
    RC(gemm_tf32(st, T, T, hd, BH, w.dout, w.v, scores_epi(sc.dS, T, H, w.pitch), flags, precision));
    // dS = P (dP - rowsum(P dP)) * scale, in place
    RC(rows_launch(st, (long)BH * T, T, w.pitch, scale, sc.dS, at.P, true));
  }
  if (fused)  // dV and dK in one kernel as well
    return attention_fused_dkv(st, at.P, sc.dS, w.pitch, w.dout, w.q, dqkv, 3L * E, rope ? rope_cs : nullptr, B, T, H,
                               hd, flags);
  GemmOperand dS = w.P, dST = w.PT;
  dS.ptr = sc.dS;
  dST.ptr = sc.dS;
  // dV = P^T dO  -> dqkv[:, 2E:3E)
  GemmEpi e = merged_epi(dqkv + 2 * E, 3L * E, T, hd, CAUSAL_K_UPPER);
  e.bdiv = H;
  RC(gemm_tf32(st, T, hd, T, BH, w.PT, mn(w.dout), e, flags, precision));
  // dQ = dS k, dK = dS^T q, written into dqkv; with RoPE they are computed in the rotated frame
  // and rotated back (by -theta) in the epilogue.
  e = merged_epi(dqkv, 3L * E, T, hd, CAUSAL_K_LOWER);
  e.bdiv = H;
  if (rope) {
    e.kind = EPI_STORE_UNROPE;
    e.rope = rope_cs;
    e.rope_hd = hd;
  }
  if (!fused) RC(gemm_tf32(st, T, hd, T, BH, dS, mn(w.k), e, flags, precision));
  e.C = dqkv + E;
  e.causal = CAUSAL_K_UPPER;
  RC(gemm_tf32(st, T, hd, T, BH, dST, mn(w.q), e, flags, precision));
  return OK;
}

}  // namespace turt
