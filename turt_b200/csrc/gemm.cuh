// gemm.cuh -- TF32 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM, TMA-fed).
#pragma once
#include "common.cuh"

namespace turt {

// Epilogue variants.  The accumulator tile (fp32, TMEM) is combined with these before
// it is written; each variant exists to remove one memory-bound pass of the train step.
enum EpiKind : int {
  EPI_STORE = 0,       // C = acc
  EPI_ACCUM = 1,       // C += acc
  EPI_RED = 2,         // split-K partial sums (set by gemm_tf32): each split stores its partial
                       // plane; a reduction kernel adds them in split order and applies split_final
  EPI_ADD_RES = 3,     // C = acc + R            (residual add)
  EPI_BIAS = 4,        // C = acc + bias[n]
  EPI_BIAS_GELU = 5,   // C = acc + bias[n] (pre-activation), C2 = gelu(C)
  EPI_SWIGLU_FWD = 6,  // C = acc (interleaved gate|up pre-activations), C2 = silu(gate) * up
  EPI_GELU_BWD = 8,    // C = acc * gelu'(R)
  EPI_QKV_ROPE = 9,    // acc = fused q|k|v projection of token `row`: q, k rotated (RoPE) into the
                       // head-major qr / kr [B*H][T][hd]; v stored into C (columns [2E, 3E))
  EPI_STORE_UNROPE = 10,  // C = acc rotated back by -theta (row = position t, columns = head dims)
};

// Interleave granularity of the fused gate|up weight and activations: columns
// [64j, 64j+32) hold gate units [32j, 32j+32), columns [64j+32, 64j+64) the matching up units.
constexpr int kGluBlock = 32;

// Causal structure of a batched attention GEMM over [T x T] score / probability tiles
// (row index = query, column index = key, lower triangle kept).  Work that only touches the
// masked upper triangle is skipped; the skipped products are exact zeros.
enum GemmCausal : int {
  CAUSAL_NONE = 0,
  CAUSAL_SKIP_UPPER = 1,  // output [T x T] scores: tiles (32-column chunks) wholly above the diagonal are not computed (stored)
  CAUSAL_K_LOWER = 2,     // A = lower-triangular [rows x K]: K-range of a row tile ends at its last row
  CAUSAL_K_UPPER = 3,     // A = upper-triangular (a transposed lower one): K-range starts at the first row
};

struct GemmEpi {
  int kind = EPI_STORE;
  float* C = nullptr;
  long ldc = 0;
  long strideC = 0;  // per batch (per inner batch index when bdiv > 0)
  const float* R = nullptr;
  long ldr = 0;
  const float* bias = nullptr;
  float* C2 = nullptr;
  long ldc2 = 0;
  // Two-level batch: batch index b = outer * bdiv + inner addresses C + inner * strideC +
  // outer * strideC_hi (bdiv = 0: one level).  Operands use GemmOperand::stride_hi likewise.
  int bdiv = 0;
  long strideC_hi = 0;
  int causal = CAUSAL_NONE;
  // RoPE epilogues: cos/sin table [T][hd/2] and the head geometry; qr / kr for EPI_QKV_ROPE.
  const float2* rope = nullptr;
  int rope_T = 0, rope_H = 0, rope_hd = 0;
  float* qr = nullptr;
  float* kr = nullptr;
  // Split-K (kind EPI_RED, filled in by gemm_tf32): partial planes [batch][ksplits][M][N] and the
  // epilogue the summed result takes (EPI_STORE or EPI_ACCUM).
  float* split_ws = nullptr;
  int split_final = EPI_STORE;
};

// Operand description.  `mn_major` = the operand's contiguous dimension is M (for A) or N
// (for B), i.e. it is stored [K][M] / [K][N]; otherwise it is stored [M][K] / [N][K].
struct GemmOperand {
  const float* ptr = nullptr;
  long ld = 0;      // row pitch in elements
  long stride = 0;  // batch stride in elements (inner batch index when GemmEpi::bdiv > 0)
  bool mn_major = false;
  long stride_hi = 0;  // outer batch stride (GemmEpi::bdiv > 0)
};

// Tensor-core precision: plain TF32 (10 mantissa bits per operand) or error-compensated
// 3xTF32 (three MMAs per k-step on hi/lo operand splits, ~fp32 accuracy).
enum GemmPrecision : int { GEMM_TF32 = 1, GEMM_TF32X3 = 3 };

// C[M,N] (per batch) = A[M,K] * B[K,N] with the epilogue applied.  K-splits > 1 are chosen
// automatically for store / accumulate epilogues when the tile count is below the SM count;
// their partial sums are added in a fixed order (the result does not depend on scheduling),
// through a workspace held per (device, stream) and grown on first need.  force_splits = 1
// disables splitting (no workspace is touched).
int gemm_tf32(cudaStream_t stream, int M, int N, int K, int batch, const GemmOperand& A,
              const GemmOperand& B, const GemmEpi& epi, int* dev_flags, int precision = GEMM_TF32X3,
              int force_splits = 0);

// 4-D TMA tensor map over operand `op` viewed as [batch / bdiv][bdiv][rows][inner] (the same
// view gemm_tf32 uses), with a box of box_inner x box_rows floats: K-major boxes 32 floats wide
// take the 128-byte swizzle, MN-major ones the 128-byte swizzle with 32-byte atoms.
int tensor_map_f32(CUtensorMap* map, const GemmOperand& op, long inner, long rows, int bdiv, int batch,
                   int box_inner, int box_rows, bool mn_major);

// True when gemm_tf32 can take these operands (TMA needs 16-byte pitches and bases).
bool gemm_tf32_supported(const GemmOperand& A, const GemmOperand& B);

// Frees the split-K workspace held for `st` on the current device (call before destroying a
// stream that ran GEMMs).
void gemm_release_stream(cudaStream_t st);

// Forces the output-tile width (64/128/192/256; 0 = automatic) and the kernel (pair = 1: CTA
// pair, 0: single CTA, -1: automatic) of every later gemm_tf32 call.
void gemm_set_tile_override(int bn, int pair);

// CUDA-core fp32 GEMM for shapes the TMA path cannot address (odd pitches): same
// flags as the reference's MATMUL kernel (src/infer/webgpu/autograd.ts:33-75).
int gemm_simt(cudaStream_t stream, const float* A, const float* B, float* C, int M, int K, int N, int batch,
              bool transA, bool transB, bool accum);

}  // namespace turt
