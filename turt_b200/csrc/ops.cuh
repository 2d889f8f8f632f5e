// ops.cuh -- launchers for the op-level kernels (ops.cu).
#pragma once
#include "common.cuh"

namespace turt {
int op_ewise(cudaStream_t st, const float* a, const float* b, float* out, size_t n, size_t bLen, int op, int accum);
int op_scale(cudaStream_t st, const float* a, float* out, size_t n, float s, int accum);
int op_bcast_acc(cudaStream_t st, const float* src, float* out, size_t n, size_t bLen, float s);
int op_segsum(cudaStream_t st, const float* g, float* out, size_t n, size_t bLen, float s, int accum);
int op_total(cudaStream_t st, const float* a, float* out, size_t n);
int op_relu(cudaStream_t st, const float* x, float* out, size_t n);
int op_relu_bwd(cudaStream_t st, const float* x, const float* go, float* gi, size_t n);
int op_sgd(cudaStream_t st, const float* g, float* p, size_t n, float lr);
int op_gelu(cudaStream_t st, const float* x, float* out, size_t n);
int op_gelu_bwd(cudaStream_t st, const float* x, const float* go, float* gi, size_t n);
int op_silu(cudaStream_t st, const float* x, float* out, size_t n);
int op_silu_bwd(cudaStream_t st, const float* x, const float* go, float* gi, size_t n);
int op_rms_fwd(cudaStream_t st, const float* x, const float* g, float* out, float* rstd, int rows, int d, float eps);
int op_rms_dx(cudaStream_t st, const float* x, const float* go, const float* g, const float* rstd, float* gi, int rows,
              int d);
int op_rms_dg(cudaStream_t st, const float* x, const float* go, const float* rstd, float* dg, int rows, int d);
int op_ln_fwd(cudaStream_t st, const float* x, const float* g, const float* b, float* out, float* mean, float* rstd,
              int rows, int d, float eps);
int op_ln_dx(cudaStream_t st, const float* x, const float* go, const float* g, const float* mean, const float* rstd,
             float* gi, int rows, int d);
int op_ln_dgb(cudaStream_t st, const float* x, const float* go, const float* mean, const float* rstd, float* dg,
              float* db, int rows, int d);
int op_rope_table(cudaStream_t st, float2* cs, int t, int hd, double base);
int op_rope(cudaStream_t st, const float* x, float* out, const float2* cs, int groups, int t, int hd, int bwd);
int op_softmax(cudaStream_t st, const float* x, float* out, int rows, int d);
int op_softmax_bwd(cudaStream_t st, const float* y, const float* go, float* gi, int rows, int d);
int op_gather(cudaStream_t st, const float* table, const uint32_t* idx, float* out, int n, int d, int vocab, int* flags);
int op_gather_bwd(cudaStream_t st, const uint32_t* idx, const float* go, float* dt, int n, int d, int vocab, int* flags);
int op_ce_fwd(cudaStream_t st, const float* logits, const uint32_t* tgt, float* per_row, int rows, int vocab,
              int* flags);
int op_ce_bwd(cudaStream_t st, const float* logits, const uint32_t* tgt, const float* gloss, float* dl, int rows,
              int vocab, int* flags);
int op_mask(cudaStream_t st, const float* x, float* out, int groups, int t, int bwd);
int op_permute4(cudaStream_t st, const float* inp, float* out, const int* shape, const int* perm, size_t n, int accum);
int op_adamw(cudaStream_t st, const float* g, float* p, float* m, float* v, size_t n, float lr, float b1, float b2,
             float eps, float wd, float bc1, float bc2);
int op_fill(cudaStream_t st, float* p, float v, size_t n);
}  // namespace turt
