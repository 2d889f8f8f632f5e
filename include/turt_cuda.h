/*
 * turt_cuda.h -- C ABI of libturt_cuda.so, the B200 (sm_100a) backend for turt's
 * GPU-resident GPT training step.
 *
 * Every entry point returns an int status (0 = TURT_OK); the message of the last failure
 * on the calling thread is turt_last_error().  Pointers named `d_*` or documented as
 * "device" are CUDA device pointers owned by the library (turt_buffer) or by the caller;
 * everything else is host memory.  No C++ or torch types cross this boundary.
 *
 * The reference interfaces each group replaces are cited as path:line inside the turt
 * project (TypeScript).  A TypeScript host binds each symbol with Deno.dlopen (or a Node
 * N-API shim) using the C types declared here: pointers as "buffer" / "pointer", int as "i32",
 * size_t as "usize", float / double as "f32" / "f64".
 */
#ifndef TURT_CUDA_H
#define TURT_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define TURT_OK 0
#define TURT_ERR_INVALID 1     /* bad argument or shape mismatch (reference: throws Error) */
#define TURT_ERR_CUDA 2        /* CUDA runtime / driver failure */
#define TURT_ERR_RANGE 3       /* token or target id out of range */
#define TURT_ERR_TIMEOUT 4     /* a bounded device wait expired */
#define TURT_ERR_NCCL 5        /* collective failed or was aborted */
#define TURT_ERR_NONFINITE 6   /* non-finite loss / gradient norm */
#define TURT_ERR_UNSUPPORTED 7 /* layout not handled */

#define TURT_ARCH_GPT2 0
#define TURT_ARCH_MODERN 1

typedef struct turt_ctx turt_ctx;
typedef struct turt_model turt_model;

/* ------------------------------------------------------------------ context
 * GpuEngine.create / device handling, src/infer/webgpu/autograd.ts:554-577. */
const char* turt_last_error(void);
int turt_version(void);
int turt_init(int device, turt_ctx** out);
int turt_ctx_destroy(turt_ctx* ctx);
/* Run all of this context's work on an external CUDA stream (cudaStream_t as void*). */
int turt_ctx_set_stream(turt_ctx* ctx, void* stream);
void* turt_ctx_stream(turt_ctx* ctx);
/* Waits for the context's stream and reports device-side error flags (range, timeout). */
int turt_synchronize(turt_ctx* ctx);
/* Self-test of the bounded device wait that every tcgen05 kernel of this library uses: one
 * thread waits on a shared-memory mbarrier that nothing completes, gives up after limit_us
 * microseconds (1 .. 1,000,000), raises the context's timeout flag and returns, so the call
 * returns TURT_ERR_TIMEOUT and the context stays usable.  No reference counterpart: the
 * reference can only notice a failed GPU step through a loss of exactly 0
 * (scripts/gpu-pretrain.ts:232-238). */
int turt_wait_selftest(turt_ctx* ctx, int limit_us);
/* Precision of every GEMM issued through this context:
 * TURT_PRECISION_TF32X3 (default) = error-compensated 3xTF32 on the tensor cores (~2^-20
 * relative per product), meets the reference's gradient tolerance;
 * TURT_PRECISION_TF32 = one TF32 tensor-core pass (10-bit mantissa);
 * TURT_PRECISION_FP32 = fp32 FMA on the CUDA cores, the arithmetic of the reference's WGSL
 * matmul (op-level and host-array matmuls only; model GEMMs then use 3xTF32). */
#define TURT_PRECISION_FP32 0
#define TURT_PRECISION_TF32 1
#define TURT_PRECISION_TF32X3 3
int turt_set_precision(turt_ctx* ctx, int precision);
int turt_get_precision(turt_ctx* ctx, int* precision);
/* Process-wide tuning override of the tensor-core GEMM: output-tile width `bn` (64, 128, 192
 * or 256 columns; 0 = chosen per problem shape, the default) and kernel `pair` (1 = two-CTA
 * cluster kernel with 256-row tiles, 3xTF32 only; 0 = single-CTA kernel; 2 = single-CTA
 * kernel with two CTAs resident per SM, 3xTF32, tile width 64 or 128; -1 = chosen per shape,
 * the default).  No reference counterpart: the reference's WGSL matmul has one fixed
 * 16x16 workgroup tile. */
int turt_gemm_set_tile(int bn, int pair);

/* ------------------------------------------------------------------ fused kernels
 * The memory-bound kernels of the fused train step, on raw device buffers, so that each can
 * be validated and timed on its own (standalone backward-op workload).  No reference
 * counterpart: the reference runs these as chains of GpuEngine ops (rmsDx + rmsDg; siluBwd +
 * ewise; ceFwd + ceBwd; adamw per tensor after a CPU-side clip).
 * turt_fused_rms_bwd: dx = dres + RMS_DX(x, dy, g, rstd) (dres may be NULL), dg += RMS_DG.
 * turt_fused_swiglu_bwd: with s = sigmoid(a): dgate = dact*u*(s + a*s*(1-s)), dup = dact*a*s.
 * turt_fused_ce: per-row CE loss of logits[N][V] and, in place, gscale*(softmax - onehot).
 * turt_fused_adamw_clip: global-norm clip of g to `clip` (<= 0: none; norm_out, host, may be
 * NULL) fused into one AdamW update of p, m, v (adam.ts:31-54 algebra, bias corrections given). */
int turt_fused_rms_bwd(turt_ctx* ctx, const float* x, const float* dy, const float* g, const float* rstd,
                       const float* dres, float* dx, float* dg, int rows, int E);
int turt_fused_swiglu_bwd(turt_ctx* ctx, const float* gate, const float* up, const float* dact, float* dgate,
                          float* dup, size_t n);
int turt_fused_ce(turt_ctx* ctx, float* logits, const uint32_t* targets, float* loss_rows, int N, int V,
                  float gscale);
int turt_fused_adamw_clip(turt_ctx* ctx, float* p, const float* g, float* m, float* v, size_t n, float lr, float b1,
                          float b2, float eps, float wd, float bc1, float bc2, float clip, double* norm_out);
/* Corpus window gather of the pretraining data feed (sampleBatch, scripts/gpu-pretrain.ts:57-68):
 * for i < b, j < t: ids[i*t + j] = tokens[starts[i] + j], targets[i*t + j] = tokens[starts[i] +
 * j + 1].  tokens: device uint16 corpus of n_tokens; starts: HOST uint64[b] (copied in order on
 * the context's stream), each at most n_tokens - t - 1 (a start beyond that raises
 * TURT_ERR_RANGE at the next synchronization and its window is left unwritten); ids / targets:
 * device uint32[b*t]. */
int turt_sample_windows(turt_ctx* ctx, const uint16_t* tokens, size_t n_tokens, const uint64_t* starts, int b, int t,
                        uint32_t* ids, uint32_t* targets);

/* ------------------------------------------------------------------ buffers
 * GpuEngine.buffer / free / reclaim / read / fill / tensor / indexBuffer,
 * src/infer/webgpu/autograd.ts:589-595, 641-662, 701-709, 790-814.  Buffers are
 * zero-filled; free is deferred to turt_reclaim (mirrors the reference's deferred destroy). */
int turt_buffer(turt_ctx* ctx, size_t elems, float** d_out);
int turt_index_buffer(turt_ctx* ctx, const uint32_t* host, size_t n, uint32_t** d_out);
int turt_free(turt_ctx* ctx, void* d_ptr);
int turt_reclaim(turt_ctx* ctx);
int turt_upload(turt_ctx* ctx, void* d_dst, const void* host_src, size_t bytes);
int turt_download(turt_ctx* ctx, void* host_dst, const void* d_src, size_t bytes);
int turt_fill(turt_ctx* ctx, float* d_buf, float value, size_t elems);
int turt_live_buffers(turt_ctx* ctx, int* live, int* peak);

/* ----------------------------------------------------------------- op level
 * One entry per GpuEngine kernel wrapper, same argument order and accumulate flags,
 * src/infer/webgpu/autograd.ts:664-788.  All float / uint32 pointers are device pointers. */
/* matmulInto :664-671 -- C (+)= op(A) op(B), batched; TF32 tensor cores when every pitch is a
 * multiple of 4 elements, else an fp32 CUDA-core kernel. */
int turt_matmul_into(turt_ctx* ctx, const float* a, const float* b, float* out, int M, int K, int N, int batch,
                     int transA, int transB, int accum);
/* ewise :672-674 -- out (+)= a op b[i % bLen]; op 0 add, 1 sub, 2 mul. */
int turt_ewise(turt_ctx* ctx, const float* a, const float* b, float* out, size_t n, size_t bLen, int op, int accum);
int turt_scale(turt_ctx* ctx, const float* a, float* out, size_t n, float s, int accum);            /* :675-678 */
int turt_bcast_acc(turt_ctx* ctx, const float* src, float* out, size_t n, size_t bLen, float s);    /* :679-682 */
int turt_segsum(turt_ctx* ctx, const float* g, float* out, size_t n, size_t bLen, float s, int accum); /* :683-686 */
int turt_total(turt_ctx* ctx, const float* a, float* out, size_t n);                                /* :687-689 */
int turt_relu(turt_ctx* ctx, const float* x, float* out, size_t n);                                 /* :690-692 */
int turt_relu_bwd(turt_ctx* ctx, const float* x, const float* gOut, float* gIn, size_t n);          /* :693-695 */
int turt_sgd(turt_ctx* ctx, const float* grad, float* param, size_t n, float lr);                   /* :696-699 */
int turt_gelu(turt_ctx* ctx, const float* x, float* out, size_t n);                                 /* :711-713 */
int turt_gelu_bwd(turt_ctx* ctx, const float* x, const float* gOut, float* gIn, size_t n);          /* :714-716 */
int turt_silu(turt_ctx* ctx, const float* x, float* out, size_t n);                                 /* :717-719 */
int turt_silu_bwd(turt_ctx* ctx, const float* x, const float* gOut, float* gIn, size_t n);          /* :720-722 */
int turt_rms_fwd(turt_ctx* ctx, const float* x, const float* gamma, float* out, float* rstd, int rows, int d,
                 float eps);                                                                         /* :723-726 */
int turt_rms_dx(turt_ctx* ctx, const float* x, const float* gOut, const float* gamma, const float* rstd,
                float* gIn, int rows, int d, float eps);                                             /* :727-730 */
int turt_rms_dg(turt_ctx* ctx, const float* x, const float* gOut, const float* rstd, float* dgamma, int rows,
                int d);                                                                              /* :731-734 */
int turt_rope(turt_ctx* ctx, const float* x, float* out, int groups, int t, int hd, float base);    /* :735-738 */
int turt_rope_bwd(turt_ctx* ctx, const float* gOut, float* gIn, int groups, int t, int hd, float base); /* :739-742 */
int turt_softmax(turt_ctx* ctx, const float* x, float* out, int rows, int d);                       /* :743-745 */
int turt_softmax_bwd(turt_ctx* ctx, const float* y, const float* gOut, float* gIn, int rows, int d); /* :746-748 */
int turt_ln_fwd(turt_ctx* ctx, const float* x, const float* gamma, const float* beta, float* out, float* mean,
                float* rstd, int rows, int d, float eps);                                           /* :749-752 */
int turt_ln_dx(turt_ctx* ctx, const float* x, const float* gOut, const float* gamma, const float* mean,
               const float* rstd, float* gIn, int rows, int d, float eps);                           /* :753-756 */
int turt_ln_dgb(turt_ctx* ctx, const float* x, const float* gOut, const float* mean, const float* rstd,
                float* dgamma, float* dbeta, int rows, int d);                                       /* :757-760 */
/* gatherInto / gatherBwd :761-766 -- out-of-range ids raise TURT_ERR_RANGE at the next sync. */
int turt_gather(turt_ctx* ctx, const float* table, const uint32_t* idx, float* out, int n, int d, int vocab);
int turt_gather_bwd(turt_ctx* ctx, const uint32_t* idx, const float* gOut, float* dTable, int n, int d, int vocab);
int turt_ce_fwd(turt_ctx* ctx, const float* logits, const uint32_t* targets, float* perRow, int rows,
                int vocab);                                                                          /* :767-769 */
int turt_ce_bwd(turt_ctx* ctx, const float* logits, const uint32_t* targets, const float* gLoss, float* dLogits,
                int rows, int vocab);                                                                /* :770-772 */
int turt_mask(turt_ctx* ctx, const float* x, float* out, int groups, int t);                        /* :773-775 */
int turt_mask_bwd(turt_ctx* ctx, const float* gOut, float* gIn, int groups, int t);                 /* :776-778 */
int turt_permute4(turt_ctx* ctx, const float* inp, float* out, const int* inShape4, const int* perm4, size_t n,
                  int accum);                                                                        /* :779-782 */
int turt_adamw(turt_ctx* ctx, const float* grad, float* param, float* m, float* v, size_t n, float lr, float b1,
               float b2, float eps, float wd, float bc1, float bc2);                                 /* :783-788 */

/* ----------------------------------------------------- host-array matmul
 * GpuCompute.matmul / bmm, src/infer/webgpu/gpu.ts:66-141, and Backend.matmul,
 * src/infer/backend.ts:11-16 / gpu-backend.ts:45-55: host arrays in, host array out. */
int turt_host_matmul(turt_ctx* ctx, const float* a, int m, int k, const float* b, int n, float* out);
int turt_host_bmm(turt_ctx* ctx, const float* a, int batch, int m, int k, const float* b, int n, float* out);
/* No counterpart in the reference.  Same product as turt_host_matmul (at the context's
 * precision), for callers that cannot let the library allocate device memory during the call
 * (a process whose device memory is held by another framework's caching allocator, or a
 * latency-bound host that must not allocate after start-up): A, B and C are staged in one
 * fixed 8 MiB device array owned by the library instead of per-call buffers.  turt_init
 * reserves the array on its device and looks up its address, so no call of this entry point
 * allocates; the device holds the array until the process exits.  Products whose staged
 * A + B + C (rows padded to 4 floats on the tensor-core paths, each part rounded up to 64
 * floats) exceed 2 Mi floats are rejected with TURT_ERR_INVALID.  All calls share the array;
 * calls that overlap on the GPU race on it. */
int turt_host_matmul_noalloc(turt_ctx* ctx, const float* a, int m, int k, const float* b, int n, float* out);

/* -------------------------------------------------------------- model level
 * GpuGPT, src/models/gpu-gpt.ts:54-202 (+ GPTConfig, src/models/gpt.ts:40-51) with the
 * AdamW / clipGradNorm step of scripts/gpu-pretrain.ts:204-224 and scripts/train-gpt.ts:241-242. */
typedef struct turt_config {
  int vocab_size;
  int block_size;
  int n_layer;
  int n_head;
  int n_embd;
  int arch;   /* TURT_ARCH_GPT2 or TURT_ARCH_MODERN */
  int hidden; /* MLP width; 0 = mlpHidden(config) (gpt.ts:69-72) */
} turt_config;

int turt_model_create(turt_ctx* ctx, const turt_config* cfg, turt_model** out);
int turt_model_destroy(turt_model* model);
/* Attention implementation of the model's fused train step.  No reference counterpart (the
 * reference always materialises scores per head):
 * TURT_ATTN_AUTO (default) = TURT_ATTN_TENSOR_ONLINE for sequences longer than 256 tokens at
 * head dims 32 / 64 (3xTF32), else TURT_ATTN_TENSOR when the per-layer [B*H][T][T]
 * probabilities of all layers fit a 16 GiB budget and the head dim is a multiple of 16, else
 * TURT_ATTN_FLASH;
 * TURT_ATTN_TENSOR = probabilities computed on the tensor cores (one fused kernel per pass for
 * T <= 256 at head dims 32 / 64, score / probability GEMMs otherwise) and kept for the backward
 * pass; TURT_ATTN_FLASH = fused online-softmax kernels on the CUDA cores, no [T][T] buffers
 * (head dim 16, 32 or 64); TURT_ATTN_TENSOR_ONLINE = online-softmax kernels on the tensor cores
 * at any T (head dim 32 or 64, 3xTF32 GEMMs), no [T][T] buffers, the probabilities recomputed in
 * the backward pass from the row log-sum-exp. */
#define TURT_ATTN_AUTO 0
#define TURT_ATTN_TENSOR 1
#define TURT_ATTN_FLASH 2
#define TURT_ATTN_TENSOR_ONLINE 3
int turt_model_set_attention(turt_model* model, int mode);
/* parameters() order, gpu-gpt.ts:118-132: count, total scalars, per-tensor name and shape. */
int turt_param_count(turt_model* model, int* count);
int turt_num_params(turt_model* model, size_t* total);
int turt_param_info(turt_model* model, int index, char* name, int name_cap, int* shape2, int* ndim);
/* Host <-> device copies of one parameter (or its gradient) in the reference's [in,out] layout. */
int turt_param_upload(turt_model* model, int index, const float* host, size_t n);
int turt_param_download(turt_model* model, int index, float* host, size_t n);
int turt_grad_download(turt_model* model, int index, float* host, size_t n);
/* Sets every parameter as the reference's CPU constructor GPT(config, mulberry32(seed)) does
 * (src/models/gpt.ts:225-239 with nn/linear.ts:20-22, math/tensor.ts:83-88,
 * math/random.ts:8-25): N(0, 0.02) weights drawn in parameters() order, residual projections
 * scaled by 1/sqrt(2 nLayer), unit gains, zero biases.  scripts/gpu-pretrain.ts seeds its GPU
 * model this way (seed 1337).  The draws run on the host. */
int turt_model_init(turt_model* model, uint32_t seed);
/* AdamW first / second moments of one parameter, same layout and sizes as the parameter.  No
 * reference counterpart: scripts/gpu-pretrain.ts keeps m and v in device buffers only and
 * restarts them at zero on --resume (:171-173); these let a checkpoint carry them. */
int turt_adam_state_download(turt_model* model, int index, float* m, float* v, size_t n);
int turt_adam_state_upload(turt_model* model, int index, const float* m, const float* v, size_t n);
/* zeroGrad on every parameter (gpu-gpt usage: scripts/gpu-pretrain.ts:205). */
int turt_zero_grad(turt_model* model);
/* GpuGPT.loss + backward (gpu-gpt.ts:185-201, autograd.ts:1196-1209): accumulates
 * loss_scale * d(mean CE)/d(theta) into the gradients.  ids/targets are host arrays of b*t
 * uint32.  loss_out (host, may be NULL) receives the mean loss; passing it synchronizes. */
int turt_forward_backward(turt_model* model, const uint32_t* ids, const uint32_t* targets, int b, int t,
                          float loss_scale, float* loss_out);
/* Same step with ids/targets already in device memory (uint32[b*t] each): no host copies and
 * no synchronization; the loss stays on the device (turt_read_loss fetches it). */
int turt_forward_backward_device(turt_model* model, const uint32_t* d_ids, const uint32_t* d_targets, int b, int t,
                                 float loss_scale);
/* Synchronizes and returns the last step's mean loss (device flags are checked too). */
int turt_read_loss(turt_model* model, float* loss_out);
/* Number of kernels this library has launched in the process (all contexts). */
int turt_launch_count(uint64_t* count);
/* Forward only (evaluation loss), gpu-pretrain.ts:188-200. */
int turt_forward(turt_model* model, const uint32_t* ids, const uint32_t* targets, int b, int t, float* loss_out);
/* turt_forward with ids / targets already in device memory (uint32[b*t] each); synchronizes
 * to return the mean loss.  The pretraining eval loss (scripts/gpu-pretrain.ts:188-200) runs it
 * on device-sampled validation windows. */
int turt_forward_device(turt_model* model, const uint32_t* ids, const uint32_t* targets, int b, int t,
                        float* loss_out);
/* Generation with a KV cache, the forward half of GPT.generate (src/models/gpt.ts:291-321).
 * prefill runs the forward over t <= block_size host token ids (one sequence), refills the
 * per-layer key / value cache and writes the last position's logits (V floats, host).  step
 * appends token `id` at position `pos` (which must equal the number of cached positions, and
 * be < block_size) and writes its logits.  When the context outgrows the block, the caller
 * prefills the cropped window again, as the reference's per-token forward over
 * ids.slice(-blockSize) does.  Both synchronize. */
int turt_generate_prefill(turt_model* model, const uint32_t* ids, int t, float* logits_out);
int turt_generate_step(turt_model* model, uint32_t id, int pos, float* logits_out);
/* clipGradNorm (src/optim/clip.ts:7-24) over all gradients; norm_out may be NULL. */
int turt_clip_grad_norm(turt_model* model, double max_norm, double* norm_out);
/* AdamW over every parameter (one fused pass over the flat buffers), autograd.ts:516-531 with
 * bias corrections from the host; clip > 0 folds the global-norm clip of clip.ts into the
 * same pass (no host round trip); grad_scale multiplies the gradients first (1/world for DP). */
int turt_adamw_step(turt_model* model, float lr, float b1, float b2, float eps, float wd, float bc1, float bc2,
                    float clip, float grad_scale);

/* ----------------------------------------------------------- data parallel
 * The reference's worker-pool reduction (scripts/train-gpt.ts:200-219) as an NCCL all-reduce
 * of the flat gradient buffer, issued per layer bucket during the backward pass. */
int turt_dp_unique_id(char* id128);
int turt_dp_init(turt_model* model, int rank, int world, const char* id128);
int turt_dp_allreduce_grads(turt_model* model);
/* defer = 1 skips the per-layer reduction (micro-batches before the last of a step). */
int turt_dp_defer(turt_model* model, int defer);
/* Waits for outstanding reductions; aborts the communicator after timeout_ms or on an
 * asynchronous NCCL error and returns TURT_ERR_NCCL. */
int turt_dp_wait(turt_model* model, int timeout_ms);
int turt_dp_destroy(turt_model* model);

/* ------------------------------------------------------ one process, several GPUs
 * The reference's data-parallel worker pool inside one process (scripts/train-gpt.ts:66-101:
 * one replica per worker; :105-123 contiguous shards; :200-219 row-weighted gradient mean), on
 * GPUs: a group holds one context + model replica per device, each driven by its own host
 * thread, joined by one NCCL communicator (the per-layer all-reduce of turt_dp_init, issued
 * during the backward pass).  Calls come from one host thread.
 * turt_group_forward_backward splits the b sequences contiguously as the reference's shard()
 * does (floor(b / ndev) each, one more for the first b mod ndev devices; b >= ndev), scales each
 * shard's mean-loss gradient by loss_scale * rows_i / b and sums the replicas, so every replica
 * then holds loss_scale times the full-batch mean gradient; loss_out (may be NULL, else the call
 * synchronizes) receives the row-weighted mean loss.  Gradients accumulate across calls like
 * turt_forward_backward's, but the all-reduce sums whole gradient buffers: for micro-batch
 * accumulation set turt_group_defer(g, 1) for every micro-batch but the last, and start each
 * step with turt_group_zero_grad.  turt_group_adamw_step runs the fused clip + AdamW on every
 * replica (identical gradients, so the replicas stay identical).  Parameter uploads go to every
 * replica; downloads come from replica 0. */
typedef struct turt_group turt_group;
int turt_group_create(int ndev, const int* devs, const turt_config* cfg, turt_group** out);
int turt_group_destroy(turt_group* g);
int turt_group_size(turt_group* g, int* ndev);
int turt_group_model(turt_group* g, int replica, turt_model** out);
int turt_group_param_upload(turt_group* g, int index, const float* host, size_t n);
int turt_group_param_download(turt_group* g, int index, float* host, size_t n);
int turt_group_grad_download(turt_group* g, int index, float* host, size_t n);
int turt_group_model_init(turt_group* g, uint32_t seed);
int turt_group_zero_grad(turt_group* g);
int turt_group_defer(turt_group* g, int defer);
int turt_group_forward_backward(turt_group* g, const uint32_t* ids, const uint32_t* targets, int b, int t,
                                float loss_scale, float* loss_out);
int turt_group_adamw_step(turt_group* g, float lr, float b1, float b2, float eps, float wd, float bc1, float bc2,
                          float clip);
int turt_group_synchronize(turt_group* g);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif
#endif /* TURT_CUDA_H */
