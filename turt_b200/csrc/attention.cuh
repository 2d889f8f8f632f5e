// attention.cuh -- fused causal attention with RoPE (attention.cu).
#pragma once
#include "common.cuh"

namespace turt {
bool attention_supported_hd(int hd);
// out[N][E] (merged heads) and lse[B*H][T] from qkv[N][3E]; rope_cs = [T][hd/2] (cos, sin).
int attention_fwd(cudaStream_t st, const float* qkv, const float2* rope_cs, float* out, float* lse, int B, int T, int H,
                  int hd, int rope);
// dqkv[N][3E] (overwritten) from dout[N][E]; D is scratch of B*H*T floats.
int attention_bwd(cudaStream_t st, const float* qkv, const float2* rope_cs, const float* out, const float* dout,
                  const float* lse, float* D, float* dqkv, int B, int T, int H, int hd, int rope);
}  // namespace turt

// ------------------------------------------------------------------------------------------
// Tensor-core attention: the reference's materialised chain (scores -> scale -> causal mask
// -> softmax -> P*V) as batched 3xTF32 tcgen05 GEMMs over the B*H heads plus row kernels.
// P stays resident from the forward to the backward pass.  Score rows have pitch
// attn_pitch(T) (T rounded up to 4 floats, the TMA row-pitch granule).
namespace turt {
struct AttnTensors {
  float* P = nullptr;   // [B*H][T][pitch] scores, then probabilities (kept for backward)
  float* qr = nullptr;  // [B*H][T][hd] rotated q (RoPE models; null otherwise)
  float* kr = nullptr;  // [B*H][T][hd] rotated k
  float* lse = nullptr;  // [B*H][T] row log-sum-exp (online-softmax kernels, instead of P)
  bool online = false;   // run the online-softmax kernels (attention_flash.cu) instead of keeping P
};
struct AttnScratch {
  float* dS = nullptr;  // [B*H][T][pitch]
  float* D = nullptr;   // [B*H][T] rowsum(dO * O) (long-sequence kernels)
};
inline long attn_pitch(int T) { return ((long)T + 3) & ~3L; }
bool attention_tc_supported(int hd);
// rotated != 0: the RoPE-rotated head-major q / k copies in `at` were already written (by the
// projection GEMM's EPI_QKV_ROPE epilogue); otherwise they are made here from qkv.
int attention_tc_fwd(cudaStream_t st, const float* qkv, const float2* rope_cs, float* out, const AttnTensors& at, int B,
                     int T, int H, int hd, int rope, int rotated, int* flags, int precision);
// Single-kernel forward for T <= 256 and head dims 32 / 64 (attention_fused.cu): the same P
// (pitch `pitch`, zeros right of the diagonal) and merged output as the three-launch chain.
struct GemmOperand;
bool attention_fused_supported(int T, int hd);
int attention_fused_fwd(cudaStream_t st, const GemmOperand& q, const GemmOperand& k, const GemmOperand& v, float* P,
                        long pitch, float* out, long ld_out, int B, int T, int H, int hd, float scale, int* flags);
// dS = P (dP - rowsum(P dP)) * scale with dP = dout v^T, and dQ = dS k written into dq (row
// pitch ld_dq, head columns h * hd; rotated back with `rope` when it is not null), in one
// kernel (same limits).
int attention_fused_dsoftmax(cudaStream_t st, const GemmOperand& dout, const GemmOperand& v, const GemmOperand& k,
                             const float* P, float* dS, long pitch, float* dq, long ld_dq, const float2* rope, int B,
                             int T, int H, int hd, float scale, int* flags);
// dV = P^T dout -> dqkv[:, 2E:3E) and dK = dS^T q -> dqkv[:, E:2E) (rotated back with `rope`
// when it is not null), in one kernel (same limits).
int attention_fused_dkv(cudaStream_t st, const float* P, const float* dS, long pitch, const GemmOperand& dout,
                        const GemmOperand& q, float* dqkv, long ld, const float2* rope, int B, int T, int H, int hd,
                        int* flags);
// Online-softmax kernels (head dims 32 / 64, 3xTF32, any T; the default above 256 tokens) that
// keep no [T][T] buffer (attention_flash.cu).  The forward writes the merged output and the row
// log-sum-exp; the backward recomputes the probabilities, writes D = rowsum(dO * O) and dQ, dK,
// dV into dqkv (rotated back with `rope` when it is not null).
bool attention_flash_supported(int T, int hd);
// The default choice: the online-softmax kernels for sequences the single-pass fused kernels
// cannot hold (T > 256), in 3xTF32, at head dims 32 / 64.
bool attention_tc_prefers_online(int T, int hd, int precision);
int attention_flash_fwd(cudaStream_t st, const GemmOperand& q, const GemmOperand& k, const GemmOperand& v, float* out,
                        long ld_out, float* lse, int B, int T, int H, int hd, float scale, int* flags);
int attention_flash_bwd(cudaStream_t st, const GemmOperand& q, const GemmOperand& k, const GemmOperand& v,
                        const GemmOperand& dout, const GemmOperand& o, const float* lse, float* D, float* dqkv,
                        long ld, const float2* rope, int B, int T, int H, int hd, float scale, int* flags);
// `out` is the forward's merged output (read by the long-sequence backward for D).
int attention_tc_bwd(cudaStream_t st, const float* qkv, const float2* rope_cs, const float* out, const float* dout,
                     const AttnTensors& at, const AttnScratch& sc, float* dqkv, int B, int T, int H, int hd, int rope,
                     int* flags, int precision);
}  // namespace turt
