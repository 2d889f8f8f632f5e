// model_kernels.cuh -- fused memory-bound kernels of the model path (model_kernels.cu).
#pragma once
#include <algorithm>

#include "common.cuh"

namespace turt {
int embed_fwd(cudaStream_t st, const float* wte, const float* wpe, const uint32_t* ids, float* x, int N, int T, int E,
              int V, int* flags);
int embed_bwd(cudaStream_t st, const float* dx, const uint32_t* ids, float* dwte, float* dwpe, int N, int T, int E,
              int V);
int rms_fwd(cudaStream_t st, const float* x, const float* g, float* y, float* rstd, int rows, int E, float eps);
int norm_parts(int rows);  // rows of partial sums a norm backward writes (each E wide)
int rms_bwd(cudaStream_t st, const float* x, const float* dy, const float* g, const float* rstd, const float* dres,
            float* dx, float* dg_accum, float* part, int rows, int E);
int ln_fwd(cudaStream_t st, const float* x, const float* g, const float* b, float* y, float* mean, float* rstd, int rows,
           int E, float eps);
int ln_bwd(cudaStream_t st, const float* x, const float* dy, const float* g, const float* mean, const float* rstd,
           const float* dres, float* dx, float* dg_accum, float* db_accum, float* part, int rows, int E);
int colsum_accum(cudaStream_t st, const float* g, int rows, int C, float* out_accum, float* part);
// SwiGLU backward: d(act) [N][h] and interleaved gate|up pre-activations [N][2h] -> interleaved grads.
int swiglu_bwd_interleaved(cudaStream_t st, const float* dact, const float* pre, float* dpre, int N, int h);
int ce_fused(cudaStream_t st, float* logits, const uint32_t* tgt, float* loss_rows, int N, int V, float gscale,
             int* flags);
int ce_loss(cudaStream_t st, const float* logits, const uint32_t* tgt, float* loss_rows, int N, int V, int* flags);
int loss_mean(cudaStream_t st, const float* rows, int n, float* out, int* flags);
size_t norm_scratch_doubles();
int grad_norm(cudaStream_t st, const float* g, size_t n, float gscale, float clip, double* scratch, double* norm_out,
              float* coef_out, int* flags);
int scale_by(cudaStream_t st, float* g, size_t n, const float* coef, float pre);
int adamw_flat(cudaStream_t st, float* p, const float* g, float* m, float* v, size_t n, float lr, float b1, float b2,
               float eps, float wd, float bc1, float bc2, float gscale, const float* coef);
}  // namespace turt
