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
