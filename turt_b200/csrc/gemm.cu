// gemm.cu -- TF32 tensor-core GEMM for sm_100a: TMA -> 128B-swizzled smem ring ->
// tcgen05.mma (kind::tf32, fp32 accumulate in TMEM) -> tcgen05.ld epilogue.
//
// One CTA computes a 128 x BN output tile.  Warp roles (192 threads):
//   warp 0      TMA producer (one elected lane)
//   warp 1      TMEM allocator + MMA issuer (one elected lane)
//   warps 2..5  epilogue; warp w reads TMEM lanes 32*(w%4) .. 32*(w%4)+31
// Operands may be K-major ([rows][K]) or MN-major ([K][rows]); both are legal for
// tf32 in the tcgen05 instruction descriptor, so no transposed copies are ever made:
// forward (X*W), data-gradient (dY*W^T) and weight-gradient (X^T*dY) GEMMs all read
// the tensors where they lie.
#include <cuda.h>

#include <algorithm>
#include <atomic>
#include <map>
#include <mutex>
#include <vector>

#include "gemm.cuh"
#include "tcgen05.cuh"

namespace turt {

namespace {

constexpr int BM = 128;

// ------------------------------------------------------------ epilogue
// tcgen05.ld gives one epilogue lane one accumulator row (32 consecutive columns per load).
// Stored lane by lane, every warp store would touch 32 rows with 16 bytes each; instead each
// warp turns its 32 x 32 chunk around in a private shared-memory tile, 16 columns at a time,
// so that a warp access covers 8 rows x 64 contiguous bytes.  The tile pitch of 20 floats
// keeps both the row-wise float4 writes and the column-group float4 reads free of bank
// conflicts (each 8-lane phase hits 8 distinct 4-bank groups).
constexpr int kEpiPitch = 20;
constexpr int kEpiTileFloats = 32 * kEpiPitch;
constexpr int kEpiStageBytes = 4 * kEpiTileFloats * 4;  // four epilogue warps

struct EpiVec {
  bool C, R, C2;
};

__device__ __forceinline__ void st4(float* p, float4 x, int nv, bool vec) {
  if (vec && nv == 4) {
    *reinterpret_cast<float4*>(p) = x;
  } else {
    p[0] = x.x;
    if (nv > 1) p[1] = x.y;
    if (nv > 2) p[2] = x.z;
    if (nv > 3) p[3] = x.w;
  }
}

__device__ __forceinline__ float4 ld4(const float* p, int nv, bool vec) {
  if (vec && nv == 4) return *reinterpret_cast<const float4*>(p);
  return make_float4(p[0], nv > 1 ? p[1] : 0.f, nv > 2 ? p[2] : 0.f, nv > 3 ? p[3] : 0.f);
}

__device__ __forceinline__ float4 add4(float4 a, float4 b) {
  return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}

__device__ __forceinline__ float4 bias4(const float* bias, int col, int nv) {
  return make_float4(bias[col], nv > 1 ? bias[col + 1] : 0.f, nv > 2 ? bias[col + 2] : 0.f,
                     nv > 3 ? bias[col + 3] : 0.f);
}

// One epilogue lane owns one accumulator row; `v` holds 32 consecutive columns of it.
__device__ __forceinline__ void st32(float* dst, const float* v, int n, bool vec) {
  if (vec && n >= 32) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < 32; j++)
      if (j < n) dst[j] = v[j];
  }
}

__device__ __forceinline__ void ld32(const float* src, float* v, int n, bool vec) {
  if (vec && n >= 32) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      const float4 t = *reinterpret_cast<const float4*>(src + j);
      v[j] = t.x;
      v[j + 1] = t.y;
      v[j + 2] = t.z;
      v[j + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; j++) v[j] = j < n ? src[j] : 0.0f;
  }
}

// Columns [col0, col0 + 32) of one output row (every kind except the fused SwiGLU forward).
__device__ __forceinline__ void epi_chunk(const GemmEpi& epi, const EpiVec& vec, float* v, float* Cb, long row,
                                          int col0, int n, long cboff) {
  float* dst = Cb + row * epi.ldc + col0;
  switch (epi.kind) {
    case EPI_STORE:
      st32(dst, v, n, vec.C);
      break;
    case EPI_ACCUM: {
      float o[32];
      ld32(dst, o, n, vec.C);
#pragma unroll
      for (int j = 0; j < 32; j++) v[j] += o[j];
      st32(dst, v, n, vec.C);
    } break;
    case EPI_ADD_RES: {
      float o[32];
      ld32(epi.R + cboff + row * epi.ldr + col0, o, n, vec.R);
#pragma unroll
      for (int j = 0; j < 32; j++) v[j] += o[j];
      if (epi.bias) {
#pragma unroll
        for (int j = 0; j < 32; j++) v[j] += j < n ? epi.bias[col0 + j] : 0.0f;
      }
      st32(dst, v, n, vec.C);
    } break;
    case EPI_BIAS:
    case EPI_BIAS_GELU:
#pragma unroll
      for (int j = 0; j < 32; j++) v[j] += j < n ? epi.bias[col0 + j] : 0.0f;
      st32(dst, v, n, vec.C);
      if (epi.kind == EPI_BIAS_GELU) {
#pragma unroll
        for (int j = 0; j < 32; j++) v[j] = gelu_f(v[j]);
        st32(epi.C2 + row * epi.ldc2 + col0, v, n, vec.C2);
      }
      break;
    case EPI_GELU_BWD: {
      float z[32];
      ld32(epi.R + row * epi.ldr + col0, z, n, vec.R);
#pragma unroll
      for (int j = 0; j < 32; j++) v[j] *= gelu_grad_f(z[j]);
      st32(dst, v, n, vec.C);
    } break;
    case EPI_QKV_ROPE: {
      const int hd = epi.rope_hd, H = epi.rope_H, T = epi.rope_T, E = H * hd;
      const int sec = col0 / E;  // 0 q, 1 k, 2 v (E is a multiple of 32: a chunk never straddles)
      if (sec == 2) {
        st32(dst, v, n, vec.C);
        break;
      }
      float* base = sec == 0 ? epi.qr : epi.kr;
      const int t = (int)(row % T);
      const long b = row / T;
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        if (j >= n) break;
        const int c = col0 - sec * E + j, h = c / hd, d = c % hd;
        const float2 c0 = epi.rope[(long)t * (hd / 2) + d / 2], c1 = epi.rope[(long)t * (hd / 2) + d / 2 + 1];
        const float4 y = make_float4(v[j] * c0.x - v[j + 1] * c0.y, v[j] * c0.y + v[j + 1] * c0.x,
                                     v[j + 2] * c1.x - v[j + 3] * c1.y, v[j + 2] * c1.y + v[j + 3] * c1.x);
        *reinterpret_cast<float4*>(base + ((b * H + h) * T + t) * hd + d) = y;
      }
    } break;
    case EPI_STORE_UNROPE: {
      const int hd = epi.rope_hd;
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        if (j < n) {
          const float2 cs = epi.rope[row * (hd / 2) + (col0 + j) / 2];
          const float g0 = v[j], g1 = v[j + 1];
          v[j] = g0 * cs.x + g1 * cs.y;
          v[j + 1] = -g0 * cs.y + g1 * cs.x;
        }
      }
      st32(dst, v, n, vec.C);
    } break;
    default:
      break;
  }
}

// Hands the lane's row v[0..n) of a 16-column group to fn(x, row, col, nv) as float4 groups in
// the coalesced order: fn sees columns [col, col + nv) of `row` (nv <= 4), rows < M only.
template <typename F>
__device__ __forceinline__ void half_t(float* tile, int lane, const float* v, long rowbase, int M, int col0, int n,
                                       F&& fn) {
  __syncwarp();
  float4* tr = reinterpret_cast<float4*>(tile + lane * kEpiPitch);
#pragma unroll
  for (int j = 0; j < 4; j++) tr[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  __syncwarp();
#pragma unroll
  for (int p = 0; p < 4; p++) {
    const int r = 8 * p + (lane & 7), c = 4 * (lane >> 3);
    const float4 x = *reinterpret_cast<const float4*>(tile + r * kEpiPitch + c);
    const long row = rowbase + r;
    const int nv = min(4, n - c);
    if (row < M && nv > 0) fn(x, row, col0 + c, nv);
  }
}

// The same for a 32-column chunk (two 16-column groups).
template <typename F>
__device__ __forceinline__ void chunk_t(float* tile, int lane, const float* v, long rowbase, int M, int col0, int n,
                                        F&& fn) {
  half_t(tile, lane, v, rowbase, M, col0, n, fn);
  if (n > 16) half_t(tile, lane, v + 16, rowbase, M, col0 + 16, n - 16, fn);
}

// Columns [col, col + nv) of one output row, every kind except the fused SwiGLU forward.
__device__ __forceinline__ void epi_quad(const GemmEpi& epi, const EpiVec& vec, float4 x, float* Cb, long row, int col,
                                         int nv, long cboff) {
  float* dst = Cb + row * epi.ldc + col;
  switch (epi.kind) {
    case EPI_STORE:
      st4(dst, x, nv, vec.C);
      break;
    case EPI_ACCUM:
      st4(dst, add4(x, ld4(dst, nv, vec.C)), nv, vec.C);
      break;
    case EPI_ADD_RES:
      x = add4(x, ld4(epi.R + cboff + row * epi.ldr + col, nv, vec.R));
      if (epi.bias) x = add4(x, bias4(epi.bias, col, nv));
      st4(dst, x, nv, vec.C);
      break;
    case EPI_BIAS:
    case EPI_BIAS_GELU:
      x = add4(x, bias4(epi.bias, col, nv));
      st4(dst, x, nv, vec.C);
      if (epi.kind == EPI_BIAS_GELU)
        st4(epi.C2 + row * epi.ldc2 + col, make_float4(gelu_f(x.x), gelu_f(x.y), gelu_f(x.z), gelu_f(x.w)), nv,
            vec.C2);
      break;
    case EPI_GELU_BWD: {
      const float4 z = ld4(epi.R + row * epi.ldr + col, nv, vec.R);
      x = make_float4(x.x * gelu_grad_f(z.x), x.y * gelu_grad_f(z.y), x.z * gelu_grad_f(z.z), x.w * gelu_grad_f(z.w));
      st4(dst, x, nv, vec.C);
    } break;
    case EPI_QKV_ROPE: {
      // E and the head dim are multiples of 16: a group of 4 never straddles q / k / v or heads
      const int hd = epi.rope_hd, H = epi.rope_H, T = epi.rope_T, E = H * hd;
      const int sec = col / E;  // 0 q, 1 k, 2 v
      if (sec == 2) {
        st4(dst, x, nv, vec.C);
        break;
      }
      float* base = sec == 0 ? epi.qr : epi.kr;
      const int t = (int)(row % T);
      const long b = row / T;
      const int c = col - sec * E, h = c / hd, d = c % hd;
      const float2 c0 = epi.rope[(long)t * (hd / 2) + d / 2], c1 = epi.rope[(long)t * (hd / 2) + d / 2 + 1];
      *reinterpret_cast<float4*>(base + ((b * H + h) * T + t) * hd + d) =
          make_float4(x.x * c0.x - x.y * c0.y, x.x * c0.y + x.y * c0.x, x.z * c1.x - x.w * c1.y,
                      x.z * c1.y + x.w * c1.x);
    } break;
    case EPI_STORE_UNROPE: {
      // rows are positions (one head per batch entry); (col, col + 1), (col + 2, col + 3) are pairs
      const int hd = epi.rope_hd;
      const float2 c0 = epi.rope[row * (hd / 2) + col / 2], c1 = epi.rope[row * (hd / 2) + col / 2 + 1];
      x = make_float4(x.x * c0.x + x.y * c0.y, -x.x * c0.y + x.y * c0.x, x.z * c1.x + x.w * c1.y,
                      -x.z * c1.y + x.w * c1.x);
      st4(dst, x, nv, vec.C);
    } break;
    default:
      break;
  }
}

// One accumulator tile of an epilogue warp: 32 rows from `rowbase`, columns [n0, n0 + BN).
// `tile` != nullptr selects the shared-memory-transposed stores (8 rows x 64 B per warp
// access); otherwise each lane stores its own row.  Measured on B200: the transposed stores
// win when the epilogue overlaps a long mainloop (they disturb it less), the row stores when
// the epilogue itself is the critical path (short K).
template <int BN, bool T>
__device__ __forceinline__ void epi_tile(const GemmEpi& epi, const EpiVec& vec, float* tile, int lane,
                                         uint32_t tbase, long rowbase, int M, int N, int n0, float* Cb, long cboff) {
  const long row = rowbase + lane;
  if (!T) tile = nullptr;
  if (epi.kind == EPI_SWIGLU_FWD) {
    // Chunk pairs (gate, up): C keeps both pre-activations, C2 gets silu(gate) * up.
#pragma unroll 1
    for (int c = 0; c < BN / 32; c += 2) {
      const int col0 = n0 + c * 32;
      if (col0 >= N) break;  // warp-uniform
      const int nu = min(32, N - col0 - 32);
      if (!tile) {
        float g[32], v[32];
        tmem_ld32(tbase + c * 32, g);
        tmem_ld32(tbase + (c + 1) * 32, v);
        if (row < M) {
          st32(Cb + row * epi.ldc + col0, g, min(32, N - col0), vec.C);
          st32(Cb + row * epi.ldc + col0 + 32, v, nu, vec.C);
#pragma unroll
          for (int j = 0; j < 32; j++) v[j] *= g[j] * sigmoid_f(g[j]);
          st32(epi.C2 + row * epi.ldc2 + col0 / 2, v, nu, vec.C2);
        }
        continue;
      }
      const bool vc = vec.C, vc2 = vec.C2;
      const long ldc = epi.ldc, ldc2 = epi.ldc2;
      float* C2 = epi.C2;
      auto to_c = [&](float4 x, long r, int col, int nv) { st4(Cb + r * ldc + col, x, nv, vc); };
      {
        float g[32];
        tmem_ld32(tbase + c * 32, g);
        chunk_t(tile, lane, g, rowbase, M, col0, min(32, N - col0), to_c);
      }
      {
        float v[32];
        tmem_ld32(tbase + (c + 1) * 32, v);
        chunk_t(tile, lane, v, rowbase, M, col0 + 32, nu, to_c);
      }
      // silu(gate) * up, 16 columns at a time (TMEM is re-read: it is cheaper than registers)
#pragma unroll 1
      for (int h = 0; h < 32 && h < nu; h += 16) {
        float g[16], v[16];
        tmem_ld16(tbase + c * 32 + h, g);
        tmem_ld16(tbase + (c + 1) * 32 + h, v);
#pragma unroll
        for (int j = 0; j < 16; j++) v[j] *= g[j] * sigmoid_f(g[j]);
        half_t(tile, lane, v, rowbase, M, col0 / 2 + h, nu - h,
               [&](float4 x, long r, int col, int nv) { st4(C2 + r * ldc2 + col, x, nv, vc2); });
      }
    }
  } else {
    // Causal scores: a 32-column chunk wholly right of this warp's last row is never read
    // (the row kernels mask it), so it is not stored either.
    const long last_col = epi.causal == CAUSAL_SKIP_UPPER ? rowbase + 31 : (long)N;
#pragma unroll 1
    for (int c = 0; c < BN / 32; c++) {
      const int col0 = n0 + c * 32;
      if (col0 >= N || col0 > last_col) break;  // warp-uniform; later chunks lie further right
      float v[32];
      tmem_ld32(tbase + c * 32, v);
      if (tile)
        chunk_t(tile, lane, v, rowbase, M, col0, min(32, N - col0),
                [&](float4 x, long r, int col, int nv) { epi_quad(epi, vec, x, Cb, r, col, nv, cboff); });
      else if (row < M)
        epi_chunk(epi, vec, v, Cb, row, col0, min(32, N - col0), cboff);
    }
  }
}

// ------------------------------------------------------------ split-K
// A split's partial of one 32-row x BN piece (rows rowbase.., columns n0..) goes to its own
// dense plane of the workspace, [batch][split][M][N], through L2 (st.global.cg).
template <int BN>
__device__ __forceinline__ void split_store(const GemmEpi& epi, int lane, uint32_t tbase, long rowbase, int M, int N,
                                            int n0, int b, int split, int ksplits) {
  const long row = rowbase + lane;
  const bool vw = (N & 3) == 0;
  float* W = epi.split_ws + ((size_t)b * ksplits + split) * ((size_t)M * N) + (size_t)(row < M ? row : 0) * N;
#pragma unroll 1
  for (int c = 0; c < BN / 32; c++) {
    const int col0 = n0 + c * 32;
    if (col0 >= N) break;  // warp-uniform
    float v[32];
    tmem_ld32(tbase + c * 32, v);
    if (row >= M) continue;
    const int n = min(32, N - col0);
    if (vw && n == 32) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        __stcg(reinterpret_cast<float4*>(W + col0 + j), make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
    } else {
      for (int j = 0; j < n; j++) __stcg(W + col0 + j, v[j]);
    }
  }
}

// Fixed-order reduction of the split-K partial planes, launched right after the GEMM on the
// same stream: C (=|+=) W[0] + W[1] + ... + W[ks-1], element by element, so the sum does not
// depend on which split finished first.  Planes are [batch][ks][M][N]; C of batch b is
// C + (b % bdiv) * strideC + (b / bdiv) * strideC_hi with row pitch ldc.
__global__ void __launch_bounds__(256) k_splitk_reduce(const float* __restrict__ W, int ks, int M, int N, int batch,
                                                       float* __restrict__ C, long ldc, long strideC, long strideC_hi,
                                                       int bdiv, int accumulate, int vec) {
  pdl_trigger();
  pdl_wait();
  const size_t plane = (size_t)M * N;
  if (vec) {  // N % 4 == 0 and C rows 16-byte aligned
    const int n4 = N / 4;
    const size_t total = (size_t)batch * M * n4;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
      const int c4 = (int)(e % n4);
      const size_t r = e / n4;
      const int row = (int)(r % M), b = (int)(r / M);
      const float4* w = reinterpret_cast<const float4*>(W + (size_t)b * ks * plane + (size_t)row * N) + c4;
      float4 acc = __ldcg(w);
      for (int sp = 1; sp < ks; sp++) {
        const float4 t = __ldcg(w + sp * (plane / 4));
        acc.x += t.x, acc.y += t.y, acc.z += t.z, acc.w += t.w;
      }
      float4* dst = reinterpret_cast<float4*>(C + (long)(b % bdiv) * strideC + (long)(b / bdiv) * strideC_hi +
                                              (long)row * ldc) + c4;
      if (accumulate) {
        const float4 o = *dst;
        acc.x += o.x, acc.y += o.y, acc.z += o.z, acc.w += o.w;
      }
      *dst = acc;
    }
  } else {
    const size_t total = (size_t)batch * plane;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
      const int col = (int)(e % N);
      const size_t r = e / N;
      const int row = (int)(r % M), b = (int)(r / M);
      const float* w = W + (size_t)b * ks * plane + (size_t)row * N + col;
      float acc = __ldcg(w);
      for (int sp = 1; sp < ks; sp++) acc += __ldcg(w + sp * plane);
      float* dst = C + (long)(b % bdiv) * strideC + (long)(b / bdiv) * strideC_hi + (long)row * ldc + col;
      if (accumulate) acc += *dst;
      *dst = acc;
    }
  }
}

// ------------------------------------------------------------ kernel
// Persistent: one CTA per SM walks the (batch, k-split, n-tile, m-tile) work units
// blockIdx.x, blockIdx.x + gridDim.x, ...  The producer and the MMA issuer run ahead
// across unit boundaries; the accumulator is double-buffered in TMEM (2 x BN columns), so
// the epilogue of one unit overlaps the mainloop of the next.
//
// Warp roles:
//   warp 0        TMA producer (one elected lane)
//   warp 1        TMEM allocator + MMA issuer (one elected lane)
//   warps 2..5    epilogue; warp w reads TMEM lanes 32*(w%4) .. 32*(w%4)+31
//   warps 6..9    (X3 only) lo-part converters
//
// X3 = error-compensated 3xTF32 (Ootomo & Yokota, 2022): every operand x is split as
// x = hi + lo with hi = x truncated to tf32 (what the tensor core reads from the raw fp32
// bits) and lo = x - hi (exact in fp32); the product is accumulated as
// lo*hi + hi*lo + hi*hi, which keeps ~21 mantissa bits instead of tf32's 10.  The lo tiles
// are written to shared memory by the converter warps in the same swizzled layout as the
// TMA-written hi tiles.
//
// Shared-memory layouts (per stage: [A hi | B hi | A lo | B lo]):
//   K-major, BK = 32: rows of 128 B, 128-byte swizzle (8-row atoms of 1 KB)
//   K-major, BK = 16: rows of 64 B, 64-byte swizzle (8-row atoms of 512 B)
//   MN-major: 32 (MN) x BK (K) TMA boxes of 128-byte K-rows, 128-byte swizzle with 32-byte
//             atomicity (4-row atoms of 512 B); the only MN-major layout tf32 accepts.
// MINB = CTAs resident per SM: 2 halves the stage ring so that two independent pipelines
// share an SM (latency hiding for skinny tiles whose stages hold little MMA work).
template <int BN, int BK, bool X3, int MINB = 1>
struct GemmShape {
  static constexpr int A_BYTES = BM * BK * 4;
  static constexpr int B_BYTES = BN * BK * 4;
  static constexpr int HI_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGE_BYTES = HI_BYTES * (X3 ? 2 : 1);
  static constexpr int MN_BOX = 32 * BK * 4;
  static constexpr int THREADS = X3 ? 320 : 192;
  static constexpr uint32_t TMEM_COLS = 2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512);
  static constexpr int SMEM_CAP = MINB == 1 ? 232448 : 233472 / MINB - 1024;  // per-CTA share of the SM
  static constexpr int STAGES_FIT = (SMEM_CAP - 1024 - 256) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
};

template <int BN, int BK, bool A_MN, bool B_MN, bool X3, int MINB = 1>
__global__ void __launch_bounds__(GemmShape<BN, BK, X3, MINB>::THREADS, MINB)
    k_gemm_tf32(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmEpi epi,
                int M, int N, int K, int batches, int bdiv, int causal, int ksplits, int kt_per_split, int* flags) {
  using S = GemmShape<BN, BK, X3, MINB>;
  constexpr int STAGES = S::STAGES;
  static_assert(BK == 16 || BK == 32, "BK");
  static_assert(BN % 64 == 0 && BN <= 256, "BN");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * S::STAGE_BYTES);
  uint64_t* conv = full + STAGES;
  uint64_t* empty = conv + STAGES;
  uint64_t* tfull = empty + STAGES;  // [2] accumulator ready (MMA -> epilogue)
  uint64_t* tempty = tfull + 2;      // [2] accumulator drained (epilogue -> MMA)
  uint64_t* done = tempty + 2;       // every MMA of this CTA retired
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = (M + BM - 1) / BM, nt = (N + BN - 1) / BN;
  const int units = mt * nt * ksplits * batches;
  const int kt_total = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 4);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(S::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  // set-up done: from here on global memory is touched (PDL; no-ops under a plain launch)
  pdl_trigger();
  pdl_wait();

  // unit -> (m0, n0, batch, first k-tile, k-tile count); false = nothing to compute (causal skip)
  auto decode = [&](int u, int& m0, int& n0, int& b, int& kt0, int& nkt) {
    m0 = (u % mt) * BM;
    u /= mt;
    n0 = (u % nt) * BN;
    u /= nt;
    const int split = u % ksplits;
    b = u / ksplits;
    kt0 = split * kt_per_split;
    int kt1 = min(kt_total, kt0 + kt_per_split);
    if (causal == CAUSAL_SKIP_UPPER && n0 >= m0 + BM) return false;
    if (causal == CAUSAL_K_LOWER) kt1 = min(kt1, (m0 + BM + BK - 1) / BK);
    if (causal == CAUSAL_K_UPPER) kt0 = max(kt0, m0 / BK);
    nkt = kt1 - kt0;
    return nkt > 0;
  };

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      uint32_t it = 0;
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
        int m0, n0, b, kt0, nkt;
        if (!decode(u, m0, n0, b, kt0, nkt)) continue;
        // Boxes that start beyond M (or N) only feed output rows (columns) that are never
        // written, so they are skipped and not counted.
        int na = 1, nb = 1;
        if (A_MN) {
          na = 0;
          for (int j = 0; j < BM / 32; j++) na += (m0 + 32 * j < M);
        }
        if (B_MN) {
          nb = 0;
          for (int j = 0; j < BN / 32; j++) nb += (n0 + 32 * j < N);
        }
        const uint32_t bytes = (A_MN ? na * S::MN_BOX : S::A_BYTES) + (B_MN ? nb * S::MN_BOX : S::B_BYTES);
        const int bi = b % bdiv, bo = b / bdiv;
        for (int i = 0; i < nkt; i++, it++) {
          const int s = it % STAGES;
          if (!mbar_wait(&empty[s], ((it / STAGES) + 1) & 1, flags, 101)) {
            *abort_flag = 1;
            break;
          }
          const int kc = (kt0 + i) * BK;
          const uint32_t sa = smem_u32(smem + s * S::STAGE_BYTES);
          const uint32_t sb = sa + S::A_BYTES;
          mbar_arrive_expect_tx(&full[s], bytes);
          if (!A_MN) {
            tma_load_4d(sa, &tmA, kc, m0, bi, bo, &full[s]);
          } else {
            for (int j = 0; j < BM / 32; j++)
              if (m0 + 32 * j < M) tma_load_4d(sa + j * S::MN_BOX, &tmA, m0 + 32 * j, kc, bi, bo, &full[s]);
          }
          if (!B_MN) {
            tma_load_4d(sb, &tmB, kc, n0, bi, bo, &full[s]);
          } else {
            for (int j = 0; j < BN / 32; j++)
              if (n0 + 32 * j < N) tma_load_4d(sb + j * S::MN_BOX, &tmB, n0 + 32 * j, kc, bi, bo, &full[s]);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      constexpr uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((A_MN ? 1u : 0u) << 15) |
                                 ((B_MN ? 1u : 0u) << 16) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
      constexpr uint32_t kKLayout = BK == 32 ? kLayoutSW128 : kLayoutSW64;
      constexpr uint32_t kKSbo = BK == 32 ? 1024 : 512;
      uint32_t it = 0;
      int t = 0;
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
        int m0, n0, b, kt0, nkt;
        if (!decode(u, m0, n0, b, kt0, nkt)) continue;
        const int acc = t & 1, use = t >> 1;
        t++;  // counts computed units only (causal skips do not use an accumulator)
        if (!mbar_wait(&tempty[acc], (use + 1) & 1, flags, 105)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * BN);
        bool ok = true;
        for (int i = 0; i < nkt; i++, it++) {
          const int s = it % STAGES;
          if (!mbar_wait(X3 ? &conv[s] : &full[s], (it / STAGES) & 1, flags, 102)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * S::STAGE_BYTES);
          const uint32_t sb = sa + S::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 8; kk++) {
            // K-major: advance 8 tf32 (32 bytes) inside the swizzle row.  MN-major: advance 8
            // K-rows (two 4-row atoms, 1 KB); TMA boxes (32-element MN blocks) MN_BOX apart.
            const uint32_t oa = A_MN ? kk * 1024 : kk * 32, ob = B_MN ? kk * 1024 : kk * 32;
            const uint64_t da = A_MN ? smem_desc(sa + oa, S::MN_BOX, 512, kLayoutSW128Atom32)
                                     : smem_desc(sa + oa, 16, kKSbo, kKLayout);
            const uint64_t db = B_MN ? smem_desc(sb + ob, S::MN_BOX, 512, kLayoutSW128Atom32)
                                     : smem_desc(sb + ob, 16, kKSbo, kKLayout);
            const uint32_t first = (i > 0 || kk > 0) ? 1u : 0u;
            if (X3) {
              // lo tiles sit HI_BYTES after the hi tiles with the same layout: bump the start address.
              const uint64_t lo = (uint64_t)(S::HI_BYTES >> 4);
              mma_tf32(d, da + lo, db, idesc, first);
              mma_tf32(d, da, db + lo, idesc, 1u);
              mma_tf32(d, da, db, idesc, 1u);
            } else {
              mma_tf32(d, da, db, idesc, first);
            }
          }
          mma_commit(&empty[s]);
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        mma_commit(&tfull[acc]);
      }
      // TMEM is released only after every MMA this thread issued has retired.
      mma_commit(done);
      if (!mbar_wait(done, 0, flags, 106)) *abort_flag = 1;
    }
  } else if (warp >= 6) {
    // -------------------------------------------------- lo-part converters (X3)
    const int ct = threadIdx.x - 192;
    uint32_t it = 0;
    for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
      int m0, n0, b, kt0, nkt;
      if (!decode(u, m0, n0, b, kt0, nkt)) continue;
      bool ok = true;
      for (int i = 0; i < nkt; i++, it++) {
        const int s = it % STAGES;
        if (!mbar_wait(&full[s], (it / STAGES) & 1, flags, 104)) {
          ok = false;
          break;
        }
        const float4* hi = reinterpret_cast<const float4*>(smem + s * S::STAGE_BYTES);
        float4* lo = reinterpret_cast<float4*>(smem + s * S::STAGE_BYTES + S::HI_BYTES);
#pragma unroll 4
        for (int e = ct; e < S::HI_BYTES / 16; e += 128) {
          const float4 v = hi[e];
          float4 r;
          r.x = v.x - __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
          r.y = v.y - __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
          r.z = v.z - __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
          r.w = v.w - __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
          lo[e] = r;
        }
        // make the generic-proxy smem writes visible to the tensor core (async proxy)
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[s]);
      }
      if (!ok) {
        *abort_flag = 1;
        break;
      }
    }
  } else {
    // -------------------------------------------------- epilogue warps (2..5)
    const int q = warp & 3;
    const EpiVec vec{(epi.ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(epi.C) & 15) == 0) && (epi.strideC % 4 == 0) &&
                         (epi.strideC_hi % 4 == 0),
                     epi.R && (epi.ldr % 4 == 0) && ((reinterpret_cast<uintptr_t>(epi.R) & 15) == 0),
                     epi.C2 && (epi.ldc2 % 4 == 0) && ((reinterpret_cast<uintptr_t>(epi.C2) & 15) == 0)};
    int t = 0;
    for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
      int m0, n0, b, kt0, nkt;
      if (!decode(u, m0, n0, b, kt0, nkt)) continue;
      const int acc = t & 1, use = t >> 1;
      t++;
      if (!mbar_wait(&tfull[acc], use & 1, flags, 103)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      const long cboff = (long)(b % bdiv) * epi.strideC + (long)(b / bdiv) * epi.strideC_hi;
      const long rowbase = m0 + q * 32;
      const bool split_piece = ksplits > 1 && rowbase < M;  // warp-uniform
      if (split_piece)
        split_store<BN>(epi, lane, tbase, rowbase, M, N, n0, b, (u / (mt * nt)) % ksplits, ksplits);
      else if (ksplits == 1)
        epi_tile<BN, false>(epi, vec, nullptr, lane, tbase, rowbase, M, N, n0, epi.C + cboff, cboff);
      // hand the accumulator back to the MMA issuer
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(S::TMEM_COLS) : "memory");
  }
}

// ------------------------------------------------------------ CTA-pair kernel (3xTF32)
// Two CTAs of a cluster compute one 256 x BN tile with tcgen05.mma.cta_group::2: each CTA
// stages its own 128 rows of A and its own BN/2 rows of B (plus their lo parts), and the MMA
// issued by the even CTA reads both CTAs' tiles.  Per SM this halves the B operand traffic
// (shared-memory reads, TMA writes and lo-part conversion), which is what bounds the
// single-CTA kernel.  Both accumulators (128 lanes x BN columns, double-buffered) live in each
// CTA's own TMEM, so each CTA drains its own rows.
//
// Cross-CTA signalling, every arrive and commit aimed at one barrier of one CTA:
//   full[s]    (each CTA)  its own TMA bytes landed              -> its converter warps
//   conv[s]    (each CTA)  its 4 converter warps done            -> MMA issuer / odd relay
//   pconv[s]   (even CTA)  odd CTA's conv[s] completed (relayed) -> MMA issuer
//   empty[s]   (each CTA)  MMA retired (two commits, one per CTA) -> its producer
//   tfull[a]   (each CTA)  accumulator a ready (two commits)      -> its epilogue warps
//   tempty[a]  (each CTA)  its 4 epilogue warps drained a         -> MMA issuer / odd relay
//   ptempty[a] (even CTA)  odd CTA's tempty[a] completed (relayed) -> MMA issuer
// Workers arrive on their own CTA's barriers (CTA-scope release, no wait on their earlier
// stores); two otherwise idle threads of the odd CTA (warp 1 for conv, warp 10 for tempty)
// forward each completed phase with one cluster-scope arrive.
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t peer_addr(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Bounded wait with cluster-scope acquire, for barriers that the other CTA arrives on.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* flags, int site) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      if (flags) atomicExch(&flags[FLAG_TIMEOUT], site);
      return false;
    }
  }
}
// Arrive on an mbarrier given by its shared::cluster address (this CTA's or the peer's).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr) : "memory");
}
__device__ __forceinline__ void mma_tf32_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit_pair(uint32_t bar_cluster_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster_addr)
               : "memory");
}

template <int BN>
struct PairShape {
  static constexpr int BK = 32;  // 32-deep stages halve the cross-CTA handshakes per FLOP (measured 1.3x)
  static constexpr int BH = BN / 2;  // B rows staged by each CTA
  static constexpr int A_BYTES = BM * BK * 4;
  static constexpr int B_BYTES = BH * BK * 4;
  static constexpr int HI_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGE_BYTES = HI_BYTES * 2;
  static constexpr int MN_BOX = 32 * BK * 4;
  static constexpr int THREADS = 352;
  static constexpr uint32_t TMEM_COLS = 2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512);
  // Transposed-store tiles only where they cost no pipeline stage (BN = 256: 3 stages either way).
  static constexpr int EPI_BYTES = BN == 256 ? kEpiStageBytes : 0;
  static constexpr int STAGES_FIT = (232448 - 1024 - 512 - EPI_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  // stages | barriers (512 B) | epilogue tiles, plus 1 KB of alignment slack
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 512 + EPI_BYTES;
};

template <int BN, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(352, 1)
    k_gemm_tf32_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmEpi epi,
                     int M, int N, int K, int batches, int bdiv, int causal, int ksplits, int kt_per_split,
                     int* flags) {
  using S = PairShape<BN>;
  constexpr int STAGES = S::STAGES, BK = S::BK;
  static_assert(BN % 64 == 0 && BN <= 256, "BN");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * S::STAGE_BYTES);
  uint64_t* conv = full + STAGES;
  uint64_t* pconv = conv + STAGES;
  uint64_t* empty = pconv + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* ptempty = tempty + 2;
  uint64_t* done = ptempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int mt = (M + 2 * BM - 1) / (2 * BM), nt = (N + BN - 1) / BN;
  const int units = mt * nt * ksplits * batches;
  const int kt_total = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 4);
      mbar_init(&pconv[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
      mbar_init(&ptempty[b], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(S::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated before any cross-CTA use
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  pdl_trigger();
  pdl_wait();
  // shared::cluster addresses of the even CTA's relay targets
  const uint32_t lead_pconv = peer_addr(smem_u32(pconv), 0);
  const uint32_t lead_ptempty = peer_addr(smem_u32(ptempty), 0);

  // unit -> (m0 of the 256-row pair tile, n0, batch, k-tile range); false = causal skip
  auto decode = [&](int u, int& m0, int& n0, int& b, int& kt0, int& nkt) {
    m0 = (u % mt) * 2 * BM;
    u /= mt;
    n0 = (u % nt) * BN;
    u /= nt;
    const int split = u % ksplits;
    b = u / ksplits;
    kt0 = split * kt_per_split;
    int kt1 = min(kt_total, kt0 + kt_per_split);
    if (causal == CAUSAL_SKIP_UPPER && n0 >= m0 + 2 * BM) return false;
    if (causal == CAUSAL_K_LOWER) kt1 = min(kt1, (m0 + 2 * BM + BK - 1) / BK);
    if (causal == CAUSAL_K_UPPER) kt0 = max(kt0, m0 / BK);
    nkt = kt1 - kt0;
    return nkt > 0;
  };

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer (both CTAs)
      uint32_t it = 0;
      for (int u = pair; u < units && !*abort_flag; u += npairs) {
        int m0, n0, b, kt0, nkt;
        if (!decode(u, m0, n0, b, kt0, nkt)) continue;
        const int ma0 = m0 + (int)rank * BM;       // this CTA's A rows
        const int nb0 = n0 + (int)rank * S::BH;    // this CTA's B rows (output columns)
        // Rows beyond M (columns beyond N) only feed accumulator rows (columns) that are
        // never written: their boxes are not loaded and their stale tiles are harmless.
        int na = 0, nbx = 0;
        if (A_MN) {
          for (int j = 0; j < BM / 32; j++) na += (ma0 + 32 * j < M);
        } else {
          na = ma0 < M;
        }
        if (B_MN) {
          for (int j = 0; j < S::BH / 32; j++) nbx += (nb0 + 32 * j < N);
        } else {
          nbx = nb0 < N;
        }
        const uint32_t bytes =
            (A_MN ? na * S::MN_BOX : na * S::A_BYTES) + (B_MN ? nbx * S::MN_BOX : nbx * S::B_BYTES);
        const int bi = b % bdiv, bo = b / bdiv;
        for (int i = 0; i < nkt; i++, it++) {
          const int s = it % STAGES;
          if (!mbar_wait(&empty[s], ((it / STAGES) + 1) & 1, flags, 111)) {
            *abort_flag = 1;
            break;
          }
          const int kc = (kt0 + i) * BK;
          const uint32_t sa = smem_u32(smem + s * S::STAGE_BYTES);
          const uint32_t sb = sa + S::A_BYTES;
          mbar_arrive_expect_tx(&full[s], bytes);
          if (!A_MN) {
            if (na) tma_load_4d(sa, &tmA, kc, ma0, bi, bo, &full[s]);
          } else {
            for (int j = 0; j < BM / 32; j++)
              if (ma0 + 32 * j < M) tma_load_4d(sa + j * S::MN_BOX, &tmA, ma0 + 32 * j, kc, bi, bo, &full[s]);
          }
          if (!B_MN) {
            if (nbx) tma_load_4d(sb, &tmB, kc, nb0, bi, bo, &full[s]);
          } else {
            for (int j = 0; j < S::BH / 32; j++)
              if (nb0 + 32 * j < N) tma_load_4d(sb + j * S::MN_BOX, &tmB, nb0 + 32 * j, kc, bi, bo, &full[s]);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ------------------------------------------------ MMA issuer (even CTA)
      constexpr uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((A_MN ? 1u : 0u) << 15) |
                                 ((B_MN ? 1u : 0u) << 16) | ((uint32_t)(BN >> 3) << 17) |
                                 ((uint32_t)((2 * BM) >> 4) << 24);
      const uint32_t empty_peer = peer_addr(smem_u32(empty), 1);
      const uint32_t tfull_peer = peer_addr(smem_u32(tfull), 1);
      uint32_t it = 0;
      int t = 0;
      for (int u = pair; u < units && !*abort_flag; u += npairs) {
        int m0, n0, b, kt0, nkt;
        if (!decode(u, m0, n0, b, kt0, nkt)) continue;
        const int acc = t & 1, use = t >> 1;
        t++;
        if (!mbar_wait(&tempty[acc], (use + 1) & 1, flags, 115) ||
            !mbar_wait_cluster(&ptempty[acc], (use + 1) & 1, flags, 117)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * BN);
        bool ok = true;
        for (int i = 0; i < nkt; i++, it++) {
          const int s = it % STAGES;
          if (!mbar_wait(&conv[s], (it / STAGES) & 1, flags, 112) ||
              !mbar_wait_cluster(&pconv[s], (it / STAGES) & 1, flags, 118)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * S::STAGE_BYTES);
          const uint32_t sb = sa + S::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 8; kk++) {
            const uint32_t oa = A_MN ? kk * 1024 : kk * 32, ob = B_MN ? kk * 1024 : kk * 32;
            const uint64_t da = A_MN ? smem_desc(sa + oa, S::MN_BOX, 512, kLayoutSW128Atom32)
                                     : smem_desc(sa + oa, 16, 1024, kLayoutSW128);
            const uint64_t db = B_MN ? smem_desc(sb + ob, S::MN_BOX, 512, kLayoutSW128Atom32)
                                     : smem_desc(sb + ob, 16, 1024, kLayoutSW128);
            const uint32_t first = (i > 0 || kk > 0) ? 1u : 0u;
            const uint64_t lo = (uint64_t)(S::HI_BYTES >> 4);
            mma_tf32_pair(d, da + lo, db, idesc, first);
            mma_tf32_pair(d, da, db + lo, idesc, 1u);
            mma_tf32_pair(d, da, db, idesc, 1u);
          }
          mma_commit_pair(smem_u32(&empty[s]));
          mma_commit_pair(empty_peer + (uint32_t)(s * 8));
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        mma_commit_pair(smem_u32(&tfull[acc]));
        mma_commit_pair(tfull_peer + (uint32_t)(acc * 8));
      }
      mma_commit_pair(smem_u32(done));
      if (!mbar_wait(done, 0, flags, 116)) *abort_flag = 1;
    } else if (lane == 0 && rank == 1) {
      // ------------------------------------------------ conv relay (odd CTA)
      uint32_t it = 0;
      for (int u = pair; u < units && !*abort_flag; u += npairs) {
        int m0, n0, b, kt0, nkt;
        if (!decode(u, m0, n0, b, kt0, nkt)) continue;
        bool ok = true;
        for (int i = 0; i < nkt; i++, it++) {
          const int s = it % STAGES;
          if (!mbar_wait(&conv[s], (it / STAGES) & 1, flags, 119)) {
            ok = false;
            break;
          }
          mbar_arrive_cluster(lead_pconv + (uint32_t)(s * 8));
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
      }
    }
  } else if (warp == 10) {
    if (lane == 0 && rank == 1) {
      // ------------------------------------------------ tempty relay (odd CTA)
      int t = 0;
      for (int u = pair; u < units && !*abort_flag; u += npairs) {
        int m0, n0, b, kt0, nkt;
        if (!decode(u, m0, n0, b, kt0, nkt)) continue;
        const int acc = t & 1, use = t >> 1;
        t++;
        if (!mbar_wait(&tempty[acc], use & 1, flags, 120)) {
          *abort_flag = 1;
          break;
        }
        mbar_arrive_cluster(lead_ptempty + (uint32_t)(acc * 8));
      }
    }
  } else if (warp >= 6) {
    // -------------------------------------------------- lo-part converters (both CTAs)
    const int ct = threadIdx.x - 192;
    uint32_t it = 0;
    for (int u = pair; u < units && !*abort_flag; u += npairs) {
      int m0, n0, b, kt0, nkt;
      if (!decode(u, m0, n0, b, kt0, nkt)) continue;
      bool ok = true;
      for (int i = 0; i < nkt; i++, it++) {
        const int s = it % STAGES;
        if (!mbar_wait(&full[s], (it / STAGES) & 1, flags, 114)) {
          ok = false;
          break;
        }
        const float4* hi = reinterpret_cast<const float4*>(smem + s * S::STAGE_BYTES);
        float4* lo = reinterpret_cast<float4*>(smem + s * S::STAGE_BYTES + S::HI_BYTES);
#pragma unroll 4
        for (int e = ct; e < S::HI_BYTES / 16; e += 128) {
          const float4 v = hi[e];
          float4 r;
          r.x = v.x - __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
          r.y = v.y - __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
          r.z = v.z - __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
          r.w = v.w - __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
          lo[e] = r;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[s]);
      }
      if (!ok) {
        *abort_flag = 1;
        break;
      }
    }
  } else {
    // -------------------------------------------------- epilogue warps (2..5, both CTAs)
    const int q = warp & 3;
    // transposed stores when the tiles exist and the mainloop is long (>= 8 k-steps per unit)
    float* tile = (S::EPI_BYTES && kt_per_split >= 8)
                      ? reinterpret_cast<float*>(smem + STAGES * S::STAGE_BYTES + 512) + q * kEpiTileFloats
                      : nullptr;
    const EpiVec vec{(epi.ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(epi.C) & 15) == 0) && (epi.strideC % 4 == 0) &&
                         (epi.strideC_hi % 4 == 0),
                     epi.R && (epi.ldr % 4 == 0) && ((reinterpret_cast<uintptr_t>(epi.R) & 15) == 0),
                     epi.C2 && (epi.ldc2 % 4 == 0) && ((reinterpret_cast<uintptr_t>(epi.C2) & 15) == 0)};
    int t = 0;
    for (int u = pair; u < units && !*abort_flag; u += npairs) {
      int m0, n0, b, kt0, nkt;
      if (!decode(u, m0, n0, b, kt0, nkt)) continue;
      const int acc = t & 1, use = t >> 1;
      t++;
      if (!mbar_wait(&tfull[acc], use & 1, flags, 113)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      const long cboff = (long)(b % bdiv) * epi.strideC + (long)(b / bdiv) * epi.strideC_hi;
      const long rowbase = m0 + (int)rank * BM + q * 32;
      const bool split_piece = ksplits > 1 && rowbase < M;  // warp-uniform
      if (split_piece)
        split_store<BN>(epi, lane, tbase, rowbase, M, N, n0, b, (u / (mt * nt)) % ksplits, ksplits);
      else if (ksplits == 1)
        epi_tile<BN, (S::EPI_BYTES > 0)>(epi, vec, tile, lane, tbase, rowbase, M, N, n0, epi.C + cboff, cboff);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // every MMA retired (the even CTA waited on `done`) before TMEM is released
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(S::TMEM_COLS) : "memory");
  }
}

// ------------------------------------------------------------ SIMT fallback
// 64x64 tiles, 16x16 threads, 4x4 outputs per thread; transpose flags only change indexing.
__global__ void k_gemm_simt(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C, int M,
                            int K, int N, bool transA, bool transB, bool accum) {
  __shared__ float As[16][65];
  __shared__ float Bs[16][65];
  const int bz = blockIdx.z;
  A += (long)bz * M * K;
  B += (long)bz * K * N;
  C += (long)bz * M * N;
  const int tx = threadIdx.x, ty = threadIdx.y, tid = ty * 16 + tx;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int e = tid; e < 64 * 16; e += 256) {
      int mm = e / 16, kk = e % 16;
      int m = m0 + mm, k = k0 + kk;
      As[kk][mm] = (m < M && k < K) ? (transA ? A[(long)k * M + m] : A[(long)m * K + k]) : 0.0f;
      int nn = e % 64, kb = e / 64;
      int n = n0 + nn, k2 = k0 + kb;
      Bs[kb][nn] = (n < N && k2 < K) ? (transB ? B[(long)n * K + k2] : B[(long)k2 * N + n]) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; kk++) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; i++) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; j++) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
  for (int i = 0; i < 4; i++)
    for (int j = 0; j < 4; j++) {
      int m = m0 + ty * 4 + i, n = n0 + tx * 4 + j;
      if (m < M && n < N) {
        float* c = C + (long)m * N + n;
        *c = accum ? *c + acc[i][j] : acc[i][j];
      }
    }
}

// ------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 4-D tensor map over a row-major [outer][inner batch][rows][inner] view with `ld` elements per
// row, `s_in` / `s_out` elements between inner / outer batch entries (one level: n_out = 1).
// K-major operands take a box_inner-float-wide swizzle (128 B for 32 floats, 64 B for 16);
// MN-major ones the 128-byte swizzle with 32-byte atomicity.
int make_map(CUtensorMap* map, const float* base, long inner, long rows, long n_in, long n_out, long ld, long s_in,
             long s_out, int box_inner, int box_rows, bool mn_major) {
  EncodeTiledFn enc = get_encode();
  if (!enc) {
    set_error("cuTensorMapEncodeTiled entry point unavailable");
    return ERR_CUDA;
  }
  // Strides of size-1 dimensions are never used; give them a legal value.
  if (n_in <= 1) s_in = ld * rows;
  if (n_out <= 1) s_out = s_in * n_in;
  if (s_in % 4 != 0) s_in = ((s_in + 3) / 4) * 4;
  if (s_out % 4 != 0) s_out = ((s_out + 3) / 4) * 4;
  cuuint64_t dims[4] = {(cuuint64_t)inner, (cuuint64_t)rows, (cuuint64_t)n_in, (cuuint64_t)n_out};
  cuuint64_t strides[3] = {(cuuint64_t)ld * 4, (cuuint64_t)s_in * 4, (cuuint64_t)s_out * 4};
  cuuint32_t box[4] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapSwizzle sw = mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                         : (box_inner == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (code " + std::to_string((int)r) + ")");
    return ERR_CUDA;
  }
  return OK;
}

int num_sms() {
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

struct LaunchArgs {
  cudaStream_t st;
  CUtensorMap ma, mb;
  GemmEpi epi;
  int M, N, K, batch, bdiv, causal, ks, kt_per;
  int* flags;
};

template <int BN, int BK, bool A_MN, bool B_MN, bool X3, int MINB = 1>
int launch(const LaunchArgs& a) {
  using S = GemmShape<BN, BK, X3, MINB>;
  static_assert(S::SMEM <= S::SMEM_CAP, "gemm: shared memory budget exceeded");
  static_assert(S::STAGES >= 2, "gemm: fewer than two pipeline stages fit");
  static std::atomic<uint64_t> configured{0};
  auto kfn = k_gemm_tf32<BN, BK, A_MN, B_MN, X3, MINB>;
  RC(smem_attr_per_device(configured, kfn, S::SMEM));
  const long units = (long)ceil_div(a.M, BM) * ceil_div(a.N, BN) * a.batch * a.ks;
  const long slots = (long)MINB * num_sms();
  const int grid = (int)(units < slots ? units : slots);
  TURT_CHECK_CUDA((launch_pdl(kfn, dim3(grid), dim3(S::THREADS), S::SMEM, a.st, a.ma, a.mb, a.epi, a.M, a.N, a.K, a.batch, a.bdiv, a.causal, a.ks, a.kt_per,
                                           a.flags)));
  TURT_LAUNCH_CHECK();
  return OK;
}

template <int BN, int BK, bool X3>
int dispatch_major(bool amn, bool bmn, const LaunchArgs& a) {
  if (!amn && !bmn) return launch<BN, BK, false, false, X3>(a);
  if (!amn && bmn) return launch<BN, BK, false, true, X3>(a);
  if (amn && !bmn) return launch<BN, BK, true, false, X3>(a);
  return launch<BN, BK, true, true, X3>(a);
}

template <bool X3>
int dispatch_bn(int bn, bool amn, bool bmn, const LaunchArgs& a) {
  constexpr int BK = X3 ? 16 : 32;
  switch (bn) {
    case 64:
      return dispatch_major<64, BK, X3>(amn, bmn, a);
    case 128:
      return dispatch_major<128, BK, X3>(amn, bmn, a);
    case 192:
      return dispatch_major<192, BK, X3>(amn, bmn, a);
    default:
      return dispatch_major<256, BK, X3>(amn, bmn, a);
  }
}

template <int BN, bool A_MN, bool B_MN>
int launch_pair(const LaunchArgs& a) {
  using S = PairShape<BN>;
  static_assert(S::SMEM <= 232448, "gemm: shared memory budget exceeded");
  static_assert(S::STAGES >= 3, "gemm: fewer than three pipeline stages fit");
  auto kfn = k_gemm_tf32_pair<BN, A_MN, B_MN>;
  // Per device: the attribute and the co-resident pair count belong to each device's context.
  static std::atomic<uint64_t> configured{0};
  static std::atomic<int> max_pairs_dev[64];
  int dev = 0;
  TURT_CHECK_CUDA(cudaGetDevice(&dev));
  std::atomic<int>& max_pairs_slot = max_pairs_dev[dev & 63];
  int max_pairs = max_pairs_slot.load(std::memory_order_acquire);
  if (!max_pairs) {
    RC(smem_attr_per_device(configured, kfn, S::SMEM));
    cudaLaunchConfig_t q = {};
    cudaLaunchAttribute qa[1];
    qa[0].id = cudaLaunchAttributeClusterDimension;
    qa[0].val.clusterDim.x = 2;
    qa[0].val.clusterDim.y = 1;
    qa[0].val.clusterDim.z = 1;
    q.gridDim = dim3(2 * 74);
    q.blockDim = dim3(S::THREADS);
    q.dynamicSmemBytes = S::SMEM;
    q.attrs = qa;
    q.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kfn, &q) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = num_sms() / 2;
    }
    max_pairs = n;
    max_pairs_slot.store(n, std::memory_order_release);
  }
  const long units = (long)ceil_div(a.M, 2 * BM) * ceil_div(a.N, BN) * a.batch * a.ks;
  const int pairs = (int)(units < max_pairs ? units : max_pairs);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see launch_pdl
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(S::THREADS);
  cfg.dynamicSmemBytes = S::SMEM;
  cfg.stream = a.st;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  TURT_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kfn, a.ma, a.mb, a.epi, a.M, a.N, a.K, a.batch, a.bdiv, a.causal, a.ks,
                                     a.kt_per, a.flags));
  note_launch();
  return OK;
}

int dispatch_pair(int bn, bool amn, bool bmn, const LaunchArgs& a) {
#define TURT_PAIR_BN(BNV)                                            \
  if (!amn && !bmn) return launch_pair<BNV, false, false>(a);        \
  if (!amn && bmn) return launch_pair<BNV, false, true>(a);          \
  if (amn && !bmn) return launch_pair<BNV, true, false>(a);          \
  return launch_pair<BNV, true, true>(a);
  switch (bn) {
    case 64: {
      TURT_PAIR_BN(64)
    }
    case 128: {
      TURT_PAIR_BN(128)
    }
    case 192: {
      TURT_PAIR_BN(192)
    }
    default: {
      TURT_PAIR_BN(256)
    }
  }
#undef TURT_PAIR_BN
}

// Two single-CTA pipelines per SM (3xTF32, BN 64 or 128).
int dispatch_dual(int bn, bool amn, bool bmn, const LaunchArgs& a) {
#define TURT_DUAL_BN(BNV)                                                  \
  if (!amn && !bmn) return launch<BNV, 16, false, false, true, 2>(a);     \
  if (!amn && bmn) return launch<BNV, 16, false, true, true, 2>(a);       \
  if (amn && !bmn) return launch<BNV, 16, true, false, true, 2>(a);       \
  return launch<BNV, 16, true, true, true, 2>(a);
  if (bn == 64) {
    TURT_DUAL_BN(64)
  }
  TURT_DUAL_BN(128)
#undef TURT_DUAL_BN
}

// Per-SM cycles of one 32-deep k-step for a 128-row slice of a BN-wide tile: the larger of
// the tensor-pipe time (3 or 1 MMAs of 128 x BN x 8 per 8 of K at ~1890 MAC/cycle) and the
// shared-memory time at 128 B/cycle (TMA writes, operand reads by the MMAs, 3xTF32 lo-part
// conversion).  A CTA pair stages and converts only half of B per SM.
long kstep_cycles(int bn, bool x3, bool pair) {
  const long mma = (x3 ? 13L : 13L / 3) * bn / 2;
  const long smem = x3 ? (pair ? 768 + 3L * bn : 768 + 6L * bn) : 256 + 2L * bn;
  return mma > smem ? mma : smem;
}

struct TilePlan {
  int bn = 256;
  int ks = 1;
  bool pair = false;
};

// Tile width, K-split count and single-CTA / CTA-pair kernel with the shortest modelled
// makespan: ceil(units / concurrent units) x (k-steps per unit x step cost) + pipeline fill
// + one epilogue drain, plus, per extra split, the atomic reduction of the M x N output.
// `max_ks` is 1 when the epilogue cannot accumulate partial sums.  Pairs run 3xTF32 only.
TilePlan plan_tiles(int M, int N, int K, int batch, bool x3, int max_ks, int force_bn, int force_pair) {
  const int sms = num_sms();
  const long k32 = (K + 31) / 32;
  TilePlan best;
  double best_cost = -1;
  const int widths[4] = {256, 192, 128, 64};
  for (int pair = 0; pair <= (x3 ? 1 : 0); pair++) {
    if (force_pair >= 0 && pair != force_pair) continue;
    for (int bn : widths) {
      if (force_bn && bn != force_bn) continue;
      if (!force_bn && bn > 64 && N <= bn / 2) continue;  // most of the tile would be empty
      const int rows = pair ? 2 * BM : BM;
      const long tiles = (long)ceil_div(M, rows) * ceil_div(N, bn) * batch;
      const long slots = pair ? sms / 2 : sms;
      for (int ks = 1; ks <= max_ks; ks++) {
        if (ks > 1 && tiles * (ks - 1) >= slots) break;  // already a full wave without this split
        const long units = tiles * ks;
        const long rounds = (units + slots - 1) / slots;
        const double steps = (double)((k32 + ks - 1) / ks);
        double cost = rounds * steps * kstep_cycles(bn, x3, pair) + 2000.0 + 16.0 * bn;
        // split partials: stored by the epilogues, summed by one more launch in a fixed order
        if (ks > 1) cost += (double)M * N * batch * (ks + 1) / (sms * 8.0) + 3000.0;
        if (best_cost < 0 || cost < best_cost) {
          best_cost = cost;
          best.bn = bn;
          best.ks = ks;
          best.pair = pair != 0;
        }
      }
    }
  }
  return best;
}

std::atomic<int> g_tile_override{0};
std::atomic<int> g_pair_override{-1};

// Split-K workspaces, one per (device, stream): GEMMs on one stream run one after another, so
// they can share partial planes; GEMMs on different streams may overlap.
struct SplitWorkspace {
  float* ws = nullptr;
  size_t floats = 0;
  std::vector<float*> retired;  // outgrown buffers, freed with the stream's workspace
};
std::mutex g_split_mu;
std::map<std::pair<int, cudaStream_t>, SplitWorkspace> g_split_ws;
constexpr size_t kSplitWsMaxFloats = (size_t)64 << 20;  // 256 MB of partial planes at most

// Grows the stream's workspace to `floats` partial floats.  While the stream is being captured
// nothing can be allocated: ERR_UNSUPPORTED, and the caller does not split.
int split_workspace(cudaStream_t st, size_t floats, float** ws) {
  int dev = 0;
  TURT_CHECK_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(g_split_mu);
  SplitWorkspace& w = g_split_ws[{dev, st}];
  if (w.floats < floats) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    TURT_CHECK_CUDA(cudaStreamIsCapturing(st, &cs));
    if (cs != cudaStreamCaptureStatusNone) return ERR_UNSUPPORTED;
    // The outgrown buffer is kept, not freed: cudaFree waits for the whole device (and its peers),
    // which could stall behind a collective of the backward pass that waits for another device.
    if (w.ws) w.retired.push_back(w.ws);
    w.ws = nullptr;
    w.floats = 0;
    const size_t nf = std::max(floats, (size_t)1 << 20);
    TURT_CHECK_CUDA(cudaMalloc(&w.ws, nf * 4));
    w.floats = nf;
  }
  *ws = w.ws;
  return OK;
}

}  // namespace

void gemm_release_stream(cudaStream_t st) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return;
  std::lock_guard<std::mutex> lock(g_split_mu);
  auto it = g_split_ws.find({dev, st});
  if (it == g_split_ws.end()) return;
  cudaStreamSynchronize(st);
  if (it->second.ws) cudaFree(it->second.ws);
  for (float* p : it->second.retired) cudaFree(p);
  g_split_ws.erase(it);
}

void gemm_set_tile_override(int bn, int pair) {
  g_tile_override.store(bn);
  g_pair_override.store(pair);
}

int tensor_map_f32(CUtensorMap* map, const GemmOperand& op, long inner, long rows, int bdiv, int batch,
                   int box_inner, int box_rows, bool mn_major) {
  return make_map(map, op.ptr, inner, rows, bdiv, batch / bdiv, op.ld, op.stride, op.stride_hi, box_inner, box_rows,
                  mn_major);
}

bool gemm_tf32_supported(const GemmOperand& A, const GemmOperand& B) {
  auto ok = [](const GemmOperand& o) {
    return (reinterpret_cast<uintptr_t>(o.ptr) & 15) == 0 && o.ld % 4 == 0 && o.stride % 4 == 0 &&
           o.stride_hi % 4 == 0;
  };
  return ok(A) && ok(B);
}

int gemm_tf32(cudaStream_t stream, int M, int N, int K, int batch, const GemmOperand& A, const GemmOperand& B,
              const GemmEpi& epi_in, int* flags, int precision, int force_splits) {
  TURT_REQUIRE(M > 0 && N > 0 && batch > 0, "gemm: empty problem");
  TURT_REQUIRE(gemm_tf32_supported(A, B), "gemm: operand pitch/base not 16-byte aligned");
  if (K == 0) {
    set_error("gemm: K == 0");
    return ERR_INVALID;
  }
  const bool x3 = precision == GEMM_TF32X3;
  const int BK = x3 ? 16 : 32;
  int force_bn = g_tile_override.load();
  if (force_bn != 64 && force_bn != 128 && force_bn != 192 && force_bn != 256) force_bn = 0;
  LaunchArgs la;
  la.st = stream;
  la.epi = epi_in;
  la.M = M;
  la.N = N;
  la.K = K;
  la.batch = batch;
  la.flags = flags;
  const int bdiv = epi_in.bdiv > 0 ? epi_in.bdiv : batch;
  TURT_REQUIRE(batch % bdiv == 0, "gemm: batch is not a multiple of the inner batch count");
  la.bdiv = bdiv;
  la.causal = epi_in.causal;
  if (la.causal != CAUSAL_NONE) TURT_REQUIRE(M == N || la.causal != CAUSAL_SKIP_UPPER, "gemm: causal skip needs M == N");
  // K is split (partial sums reduced with atomics) only when the output alone gives too few
  // units to fill the GPU (weight gradients), with at least 256 of K per split.
  const bool can_split = (la.epi.kind == EPI_ACCUM || la.epi.kind == EPI_STORE || la.epi.kind == EPI_RED) &&
                         la.causal == CAUSAL_NONE;
  const int max_ks = force_splits > 0 ? 1 : (can_split ? std::max(1, K / 256) : 1);
  const int kernel_ov = x3 ? g_pair_override.load() : 0;
  const bool dual_forced = kernel_ov == 2;  // two single-CTA pipelines per SM (BN 64 / 128)
  const int force_pair = dual_forced ? 0 : kernel_ov;
  if (dual_forced && force_bn != 64) force_bn = 128 < N ? 128 : 64;
  TilePlan plan = plan_tiles(M, N, K, batch, x3, std::min(max_ks, 64), force_bn, force_splits > 0 ? 0 : force_pair);
  // 64-wide 3xTF32 tiles hold little MMA work per k-stage, so one pipeline cannot hide its
  // handshake latency: run two single-CTA pipelines per SM (measured 8 % faster than one CTA or
  // a CTA pair on the per-head attention products, N = 64).
  bool dual = dual_forced;
  if (kernel_ov == -1 && x3 && plan.bn == 64) {
    dual = true;
    plan.pair = false;
  }
  const int BN = plan.bn;
  const int kt_total = ceil_div(K, plan.pair ? PairShape<64>::BK : BK);
  int ks = force_splits > 0 ? force_splits : plan.ks;
  const size_t plane = (size_t)batch * M * N;
  if (ks > 1 && plane * ks > kSplitWsMaxFloats) ks = (int)std::max<size_t>(1, kSplitWsMaxFloats / plane);
  la.kt_per = ceil_div(kt_total, ks);
  la.ks = ceil_div(kt_total, la.kt_per);
  float* split_ws = nullptr;
  if (la.ks > 1) {
    GemmEpi& epi = la.epi;
    TURT_REQUIRE(can_split, "gemm: split-K needs a store or accumulate epilogue");
    const int wrc = split_workspace(stream, plane * la.ks, &split_ws);
    if (wrc == OK) {
      epi.split_final = epi.kind == EPI_STORE ? EPI_STORE : EPI_ACCUM;
      epi.kind = EPI_RED;
      epi.split_ws = split_ws;
    } else if (wrc == ERR_UNSUPPORTED) {  // capturing: one pass over K
      la.kt_per = kt_total;
      la.ks = 1;
    } else {
      return wrc;
    }
  }
  int rc;
  const int BKm = plan.pair ? PairShape<64>::BK : BK;  // k-tile depth of the chosen kernel
  if (!A.mn_major)
    rc = make_map(&la.ma, A.ptr, K, M, bdiv, batch / bdiv, A.ld, A.stride, A.stride_hi, BKm, BM, false);
  else
    rc = make_map(&la.ma, A.ptr, M, K, bdiv, batch / bdiv, A.ld, A.stride, A.stride_hi, 32, BKm, true);
  if (rc) return rc;
  if (!B.mn_major)
    rc = make_map(&la.mb, B.ptr, K, N, bdiv, batch / bdiv, B.ld, B.stride, B.stride_hi, BKm, plan.pair ? BN / 2 : BN,
                  false);
  else
    rc = make_map(&la.mb, B.ptr, N, K, bdiv, batch / bdiv, B.ld, B.stride, B.stride_hi, 32, BKm, true);
  if (rc) return rc;
  if (plan.pair)
    rc = dispatch_pair(BN, A.mn_major, B.mn_major, la);
  else if (dual)
    rc = dispatch_dual(BN, A.mn_major, B.mn_major, la);
  else
    rc = x3 ? dispatch_bn<true>(BN, A.mn_major, B.mn_major, la) : dispatch_bn<false>(BN, A.mn_major, B.mn_major, la);
  if (rc || la.ks == 1) return rc;
  const GemmEpi& e = la.epi;
  const bool vec = N % 4 == 0 && e.ldc % 4 == 0 && e.strideC % 4 == 0 && e.strideC_hi % 4 == 0 &&
                   (reinterpret_cast<uintptr_t>(e.C) & 15) == 0;
  const size_t work = vec ? plane / 4 : plane;
  const int blocks = (int)std::min<size_t>((work + 255) / 256, (size_t)num_sms() * 8);
  TURT_CHECK_CUDA((launch_pdl(k_splitk_reduce, dim3(blocks), dim3(256), 0, stream, (const float*)split_ws, la.ks, M, N,
                              batch, e.C, e.ldc, e.strideC, e.strideC_hi, bdiv, e.split_final == EPI_ACCUM ? 1 : 0,
                              vec ? 1 : 0)));
  TURT_LAUNCH_CHECK();
  return OK;
}

int gemm_simt(cudaStream_t stream, const float* A, const float* B, float* C, int M, int K, int N, int batch,
              bool transA, bool transB, bool accum) {
  if (M <= 0 || N <= 0 || batch <= 0) return OK;
  dim3 grid(ceil_div(N, 64), ceil_div(M, 64), batch);
  k_gemm_simt<<<grid, dim3(16, 16), 0, stream>>>(A, B, C, M, K, N, transA, transB, accum);
  TURT_LAUNCH_CHECK();
  return OK;
}

}  // namespace turt
