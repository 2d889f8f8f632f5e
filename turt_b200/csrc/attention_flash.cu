// attention_flash.cu -- causal attention for long sequences without [T][T] storage.
//
// The reference computes attention per head as S = q k^T, scale, causal mask, softmax, O = P v
// and runs the matching backward ops (src/models/gpu-gpt.ts:143-168 over
// src/infer/webgpu/autograd.ts).  For T <= 256 the fused kernels of attention_fused.cu keep a
// tile's whole score row in tensor memory and store P once for the backward pass.  Longer
// sequences take the kernels here, which never write scores or probabilities to memory:
//   forward : per 128-query tile, 64-key blocks with an online softmax (running row maximum
//             and sum, O rescaled in tensor memory when the maximum grows), O and the row
//             log-sum-exp L = m + log(l) written out;
//   backward: dQ kernel per 128-query tile and dK / dV kernel per 128-key tile, each
//             recomputing P = exp(scale s - L) block by block (FlashAttention-2's split, with
//             D = rowsum(dO * O) formed once by the dQ kernel), so every result is a sum in a
//             fixed order: deterministic, no atomics.
// Arithmetic: 3xTF32 products (hi / lo splits, fp32 accumulation in TMEM), softmax in fp32.
//
// Shared memory cannot hold the hi and lo copies of every operand at head dim 64, so every A
// operand lives in tensor memory and the MMAs read it from there (tcgen05.mma with A in TMEM):
// Q (forward, dQ), dO (dQ), V (dK / dV) are split and stored into TMEM by the row warps at the
// start; P and dS are written back over the scores they come from.  Only B operands (K, V, Q,
// dO tiles) stream through shared memory, by TMA, with the lo parts made by converter warps.
#include "attention.cuh"
#include "gemm.cuh"
#include "tcgen05.cuh"

namespace turt {
namespace {

// tcgen05.mma with the A operand in tensor memory (128 lanes = M rows, K along the columns).
__device__ __forceinline__ void mma_tf32_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ float tf32_lo(float x) { return x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

// lo = x - tf32(x) for `bytes` of fp32 at `hi`, written `lo_off` bytes further (128 converter threads).
__device__ __forceinline__ void split_lo(uint8_t* hi_base, int bytes, int lo_off, int ct) {
  const float4* hi = reinterpret_cast<const float4*>(hi_base);
  float4* lo = reinterpret_cast<float4*>(hi_base + lo_off);
#pragma unroll 4
  for (int e = ct; e < bytes / 16; e += 128) {
    const float4 v = hi[e];
    lo[e] = make_float4(tf32_lo(v.x), tf32_lo(v.y), tf32_lo(v.z), tf32_lo(v.w));
  }
}

// Stores 32 consecutive floats of this thread's row into TMEM columns [col, col + 32) twice:
// the value (the MMA reads its tf32 part) at `hi`, its remainder x - tf32(x) at `lo`.
__device__ __forceinline__ void tmem_st_split(uint32_t hi, uint32_t lo, float* v) {
  tmem_st32(hi, v);
#pragma unroll
  for (int j = 0; j < 32; j++) v[j] = tf32_lo(v[j]);
  tmem_st32(lo, v);
}

// Loads 32 floats of a global row (16-byte aligned) or zeros.
__device__ __forceinline__ void ld_row32(const float* src, bool valid, float* v) {
#pragma unroll
  for (int g = 0; g < 8; g++) {
    const float4 x = valid ? __ldg(reinterpret_cast<const float4*>(src) + g) : make_float4(0.f, 0.f, 0.f, 0.f);
    v[4 * g] = x.x, v[4 * g + 1] = x.y, v[4 * g + 2] = x.z, v[4 * g + 3] = x.w;
  }
}

constexpr uint32_t kFlashCols = 512;
constexpr float kRescaleThreshold = 8.0f;  // keep a stale row maximum until it is 8 (e^8) behind

__device__ __forceinline__ void tmem_alloc_all(uint32_t* slot) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(kFlashCols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_free_all(uint32_t tmem) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kFlashCols) : "memory");
}

// Instruction descriptor, kind::tf32, fp32 accumulate, M = 128: N, and whether B is MN-major.
__host__ __device__ constexpr uint32_t idesc_tf32(int n, bool b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(128 >> 4) << 24);
}

// ============================================================================ forward
// One CTA per (128-query tile, head); 320 threads:
//   warp 0      TMA producer: K and V blocks of 64 keys (three-stage rings)
//   warp 1      TMEM allocator + MMA issuer: S_j = Q K_j^T into one of two score buffers,
//               then O += P_{j-1} V_{j-1}, so the scores of block j + 1 are on the tensor cores
//               while the row warps work on block j
//   warps 2..5  lo-part converters for the K and V stages
//   warps 6..9  row warps: warp w owns TMEM lanes (query rows) 32 (w % 4) .. + 31; they load Q
//               into TMEM, run the online softmax and write O and L
// TMEM columns: Q hi | Q lo [0, 2 HD), S / P-hi [2 HD, 2 HD + 128), P-lo [2 HD + 128,
// 2 HD + 256), O [2 HD + 256, 3 HD + 256).
template <int HD>
struct FlashFwd {
  static constexpr int KB = 64;                   // keys per block
  static constexpr int SLABS = HD / 32;
  static constexpr int K_SLAB = KB * 128;         // one 32-float slab of the K block (K-major rows)
  static constexpr int K_HI = SLABS * K_SLAB;
  static constexpr int V_BOX = 32 * 32 * 4;       // MN-major box: 32 head-dim values x 32 keys
  static constexpr int V_SLAB = SLABS * V_BOX;    // 32 keys
  static constexpr int V_HI = 2 * V_SLAB;         // 64 keys
  static constexpr int STAGE = 2 * K_HI + 2 * V_HI;  // K hi | K lo | V hi | V lo
  static constexpr int STAGES = 3;
  static constexpr int SMEM = STAGES * STAGE + 1024 + 512;
  static constexpr uint32_t C_Q = 0, C_S = 2 * HD, C_PLO = 2 * HD + 2 * KB, C_O = 2 * HD + 4 * KB;
  static_assert(C_O + HD <= kFlashCols, "flash forward: TMEM columns");
};

template <int HD>
__global__ void __launch_bounds__(320, 1)
    k_flash_fwd(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV, GemmOperand q,
                float* __restrict__ out, long ld_out, float* __restrict__ lse, int T, int H, float scale, int* flags) {
  using S = FlashFwd<HD>;
  constexpr int KB = S::KB, ST = S::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + ST * S::STAGE);
  uint64_t* k_full = bars;           // [ST]
  uint64_t* k_conv = bars + 3;       // [ST]
  uint64_t* k_empty = bars + 6;      // [ST]
  uint64_t* v_full = bars + 9;       // [ST]
  uint64_t* v_conv = bars + 12;      // [ST]
  uint64_t* v_empty = bars + 15;     // [ST]
  uint64_t* s_full = bars + 18;      // [2]
  uint64_t* p_ready = bars + 20;     // [2]
  uint64_t* pv_done = bars + 22;     // [2]
  uint64_t* q_ready = bars + 24;
  uint64_t* o_full = bars + 25;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 26);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x, b = bh / H, h = bh % H;
  const int q0 = (gridDim.y - 1 - blockIdx.y) * 128;  // longest tiles first
  const int nk = min(T, q0 + 128);                     // keys any row of the tile sees
  const int nkb = (nk + KB - 1) / KB;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; s++) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_conv[s], 4);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_conv[s], 4);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < 2; s++) {
      mbar_init(&s_full[s], 1);
      mbar_init(&p_ready[s], 4);
      mbar_init(&pv_done[s], 1);
    }
    mbar_init(q_ready, 4);
    mbar_init(o_full, 1);
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc_all(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer
      for (int j = 0; j < nkb; j++) {
        const int s = j % ST;
        if (j >= ST && !mbar_wait(&k_empty[s], ((j / ST) - 1) & 1, flags, 301)) break;
        const uint32_t sk = smem_u32(smem + s * S::STAGE);
        mbar_arrive_expect_tx(&k_full[s], S::K_HI);
        for (int sl = 0; sl < S::SLABS; sl++) tma_load_4d(sk + sl * S::K_SLAB, &tmK, 32 * sl, j * KB, h, b, &k_full[s]);
        if (j >= ST && !mbar_wait(&v_empty[s], ((j / ST) - 1) & 1, flags, 302)) break;
        const uint32_t sv = sk + 2 * S::K_HI;
        mbar_arrive_expect_tx(&v_full[s], S::V_HI);
        for (int hf = 0; hf < 2; hf++)
          for (int sl = 0; sl < S::SLABS; sl++)
            tma_load_4d(sv + hf * S::V_SLAB + sl * S::V_BOX, &tmV, 32 * sl, j * KB + 32 * hf, h, b, &v_full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t idesc_s = idesc_tf32(KB, false);
      constexpr uint32_t idesc_o = idesc_tf32(HD, true);
      bool ok = mbar_wait(q_ready, 0, flags, 303);
      auto issue_pv = [&](int c) -> bool {
        const int s = c % ST;
        if (!mbar_wait(&p_ready[c & 1], (c >> 1) & 1, flags, 304) || !mbar_wait(&v_conv[s], (c / ST) & 1, flags, 305))
          return false;
        tc_fence_after();
        const uint32_t sv = smem_u32(smem + s * S::STAGE + 2 * S::K_HI);
        const uint64_t lov = (uint64_t)(S::V_HI >> 4);
        const uint32_t a_hi = tmem + S::C_S + (c & 1) * KB, a_lo = tmem + S::C_PLO + (c & 1) * KB;
#pragma unroll
        for (int kk = 0; kk < KB / 8; kk++) {
          const uint64_t db = smem_desc(sv + (kk >> 2) * S::V_SLAB + (kk & 3) * 1024, S::V_BOX, 512, kLayoutSW128Atom32);
          mma_tf32_ts(tmem + S::C_O, a_lo + 8 * kk, db, idesc_o, (c > 0 || kk > 0) ? 1u : 0u);
          mma_tf32_ts(tmem + S::C_O, a_hi + 8 * kk, db + lov, idesc_o, 1u);
          mma_tf32_ts(tmem + S::C_O, a_hi + 8 * kk, db, idesc_o, 1u);
        }
        mma_commit(&pv_done[c & 1]);
        mma_commit(&v_empty[s]);
        return true;
      };
      for (int j = 0; j < nkb && ok; j++) {
        const int s = j % ST;
        // score buffer j & 1 holds P-hi of block j - 2 until its P.V product has run
        if (j >= 2 && !mbar_wait(&pv_done[j & 1], ((j - 2) >> 1) & 1, flags, 306)) {
          ok = false;
          break;
        }
        if (!mbar_wait(&k_conv[s], (j / ST) & 1, flags, 307)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sk = smem_u32(smem + s * S::STAGE);
        const uint64_t lok = (uint64_t)(S::K_HI >> 4);
        const uint32_t d = tmem + S::C_S + (j & 1) * KB;
#pragma unroll
        for (int kk = 0; kk < HD / 8; kk++) {
          const uint64_t db = smem_desc(sk + (kk >> 2) * S::K_SLAB + (kk & 3) * 32, 16, 1024, kLayoutSW128);
          mma_tf32_ts(d, tmem + S::C_Q + HD + 8 * kk, db, idesc_s, kk > 0 ? 1u : 0u);
          mma_tf32_ts(d, tmem + S::C_Q + 8 * kk, db + lok, idesc_s, 1u);
          mma_tf32_ts(d, tmem + S::C_Q + 8 * kk, db, idesc_s, 1u);
        }
        mma_commit(&s_full[j & 1]);
        mma_commit(&k_empty[s]);
        if (j >= 1 && !issue_pv(j - 1)) ok = false;
      }
      if (ok && issue_pv(nkb - 1)) mma_commit(o_full);
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------ lo-part converters
    const int ct = threadIdx.x - 64;
    for (int j = 0; j < nkb; j++) {
      const int s = j % ST;
      uint8_t* st = smem + s * S::STAGE;
      if (!mbar_wait(&k_full[s], (j / ST) & 1, flags, 308)) break;
      split_lo(st, S::K_HI, S::K_HI, ct);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&k_conv[s]);
      if (!mbar_wait(&v_full[s], (j / ST) & 1, flags, 309)) break;
      split_lo(st + 2 * S::K_HI, S::V_HI, S::V_HI, ct);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&v_conv[s]);
    }
  } else {
    // ------------------------------------------------------------ row warps
    const int qd = warp & 3;
    const int row = qd * 32 + lane, i = q0 + row;
    const int n = min(i + 1, T);  // keys this row sees
    const uint32_t lrow = (uint32_t)(qd * 32) << 16;
    // Q row -> TMEM (hi | lo); rows past T are zero
    {
      const float* src = q.ptr + (long)b * q.stride_hi + (long)h * q.stride + (long)(i < T ? i : 0) * q.ld;
#pragma unroll 1
      for (int c = 0; c < HD; c += 32) {
        float v[32];
        ld_row32(src + c, i < T, v);
        tmem_st_split(tmem + lrow + S::C_Q + c, tmem + lrow + S::C_Q + HD + c, v);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_ready);
    }
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkb; j++) {
      if (!mbar_wait(&s_full[j & 1], (j >> 1) & 1, flags, 310)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t cs = tmem + lrow + S::C_S + (j & 1) * KB;
      float v[64];
      tmem_ld32(cs, v);
      tmem_ld32(cs + 32, v + 32);
      const int k0 = j * KB;
      float mb = -INFINITY;
#pragma unroll
      for (int c = 0; c < 64; c++) {
        v[c] *= scale;
        if (k0 + c < n) mb = fmaxf(mb, v[c]);
      }
      // Online softmax: the running maximum m moves only when the block's maximum exceeds it by
      // more than the threshold (then O and l are rescaled); otherwise p may exceed 1, by e^8
      // at most, which the final O / l cancels exactly.
      float alpha = 1.f;
      if (j == 0) {
        m = mb;
      } else if (mb > m + kRescaleThreshold) {
        alpha = __expf(m - mb);
        m = mb;
      }
      if (__any_sync(0xffffffffu, alpha != 1.f)) {
        // O holds the products of blocks < j - 1 for sure; wait for block j - 1's too
        if (!mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, flags, 311)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < HD; c += 32) {
          float o[32];
          tmem_ld32(tmem + lrow + S::C_O + c, o);
#pragma unroll
          for (int e = 0; e < 32; e++) o[e] *= alpha;
          tmem_st32(tmem + lrow + S::C_O + c, o);
        }
      }
      l *= alpha;
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < 64; c++) {
        v[c] = k0 + c < n ? __expf(v[c] - m) : 0.f;
        sum += v[c];
      }
      l += sum;
      tmem_st_split(cs, tmem + lrow + S::C_PLO + (j & 1) * KB, v);
      tmem_st_split(cs + 32, tmem + lrow + S::C_PLO + (j & 1) * KB + 32, v + 32);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_ready[j & 1]);
    }
    if (ok && mbar_wait(o_full, 0, flags, 312)) {
      tc_fence_after();
      const float inv = 1.0f / l;
      const bool store = i < T;
      float* orow = out + ((long)b * T + (store ? i : 0)) * ld_out + (long)h * HD;
#pragma unroll 1
      for (int c = 0; c < HD; c += 32) {
        float o[32];
        tmem_ld32(tmem + lrow + S::C_O + c, o);
        if (store) {
#pragma unroll
          for (int g = 0; g < 8; g++)
            *reinterpret_cast<float4*>(orow + c + 4 * g) =
                make_float4(o[4 * g] * inv, o[4 * g + 1] * inv, o[4 * g + 2] * inv, o[4 * g + 3] * inv);
        }
      }
      if (store) lse[(long)bh * T + i] = m + __logf(l);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_free_all(tmem);
  }
}

// ============================================================================ backward: dQ
// One CTA per (128-query tile, head); 320 threads in the forward's roles:
//   warp 0      producer: per 32-key block K (K-major: B of S = Q K^T), V (K-major: B of
//               dP = dO V^T) and K again MN-major (B of dQ += dS K); four-stage ring
//   warp 1      MMA issuer: S_j and dP_j into buffer j & 1, then dQ += dS_{j-1} K_{j-1}
//   warps 2..5  lo-part converters
//   warps 6..9  row warps: Q and dO into TMEM, D = rowsum(dO * O) (also written out for the
//               dK / dV kernel), P = exp(scale s - L), dS = P (dP - D) scale written over S,
//               and at the end dQ (rotated back by -theta for RoPE) into dqkv
// TMEM columns: Q hi | lo, dO hi | lo, S / dS-hi 2 x 32, dP 2 x 32, dS-lo 2 x 32, dQ.
template <int HD>
struct FlashDq {
  static constexpr int KB = 32;
  static constexpr int SLABS = HD / 32;
  static constexpr int K_SLAB = KB * 128;      // 32 keys x 32 floats, K-major
  static constexpr int K_HI = SLABS * K_SLAB;
  static constexpr int MN_BOX = 32 * 32 * 4;   // 32 head-dim values x 32 keys, MN-major
  static constexpr int KM_HI = SLABS * MN_BOX;
  static constexpr int HI = 2 * K_HI + KM_HI;  // K | V | K (MN-major)
  static constexpr int STAGE = 2 * HI;
  static constexpr int STAGES = 4;
  static constexpr int SMEM = STAGES * STAGE + 1024 + 512;
  static constexpr uint32_t C_Q = 0, C_DO = 2 * HD, C_S = 4 * HD, C_DP = 4 * HD + 2 * KB, C_DSLO = 4 * HD + 4 * KB,
                            C_DQ = 4 * HD + 6 * KB;
  static_assert(C_DQ + HD <= kFlashCols, "flash dQ: TMEM columns");
};

template <int HD>
__global__ void __launch_bounds__(320, 1)
    k_flash_dq(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
               const __grid_constant__ CUtensorMap tmKm, GemmOperand q, GemmOperand dout, GemmOperand o,
               const float* __restrict__ lse, float* __restrict__ Dout, float* __restrict__ dq, long ld_dq,
               const float2* __restrict__ rope, int T, int H, float scale, int* flags) {
  using S = FlashDq<HD>;
  constexpr int KB = S::KB, ST = S::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + ST * S::STAGE);
  uint64_t* full = bars;            // [ST]
  uint64_t* conv = bars + 4;        // [ST]
  uint64_t* empty = bars + 8;       // [ST]
  uint64_t* sd_full = bars + 12;    // [2] S and dP of a block ready
  uint64_t* ds_ready = bars + 14;   // [2] dS written
  uint64_t* dq_done = bars + 16;    // [2] dQ product of a block ran
  uint64_t* qd_ready = bars + 18;
  uint64_t* dq_full = bars + 19;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 20);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x, b = bh / H, h = bh % H;
  const int q0 = (gridDim.y - 1 - blockIdx.y) * 128;
  const int nk = min(T, q0 + 128);
  const int nkb = (nk + KB - 1) / KB;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 4);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < 2; s++) {
      mbar_init(&sd_full[s], 1);
      mbar_init(&ds_ready[s], 4);
      mbar_init(&dq_done[s], 1);
    }
    mbar_init(qd_ready, 4);
    mbar_init(dq_full, 1);
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc_all(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      for (int j = 0; j < nkb; j++) {
        const int s = j % ST;
        if (j >= ST && !mbar_wait(&empty[s], ((j / ST) - 1) & 1, flags, 321)) break;
        const uint32_t base = smem_u32(smem + s * S::STAGE);
        mbar_arrive_expect_tx(&full[s], S::HI);
        for (int sl = 0; sl < S::SLABS; sl++) {
          tma_load_4d(base + sl * S::K_SLAB, &tmK, 32 * sl, j * KB, h, b, &full[s]);
          tma_load_4d(base + S::K_HI + sl * S::K_SLAB, &tmV, 32 * sl, j * KB, h, b, &full[s]);
          tma_load_4d(base + 2 * S::K_HI + sl * S::MN_BOX, &tmKm, 32 * sl, j * KB, h, b, &full[s]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_tf32(KB, false);
      constexpr uint32_t idesc_q = idesc_tf32(HD, true);
      constexpr uint64_t lo = (uint64_t)(S::HI >> 4);
      bool ok = mbar_wait(qd_ready, 0, flags, 322);
      auto issue_dq = [&](int c) -> bool {
        if (!mbar_wait(&ds_ready[c & 1], (c >> 1) & 1, flags, 323)) return false;
        tc_fence_after();
        const uint32_t skm = smem_u32(smem + (c % ST) * S::STAGE + 2 * S::K_HI);
        const uint32_t a_hi = tmem + S::C_S + (c & 1) * KB, a_lo = tmem + S::C_DSLO + (c & 1) * KB;
#pragma unroll
        for (int kk = 0; kk < KB / 8; kk++) {
          const uint64_t db = smem_desc(skm + kk * 1024, S::MN_BOX, 512, kLayoutSW128Atom32);
          mma_tf32_ts(tmem + S::C_DQ, a_lo + 8 * kk, db, idesc_q, (c > 0 || kk > 0) ? 1u : 0u);
          mma_tf32_ts(tmem + S::C_DQ, a_hi + 8 * kk, db + lo, idesc_q, 1u);
          mma_tf32_ts(tmem + S::C_DQ, a_hi + 8 * kk, db, idesc_q, 1u);
        }
        mma_commit(&dq_done[c & 1]);
        mma_commit(&empty[c % ST]);
        return true;
      };
      for (int j = 0; j < nkb && ok; j++) {
        const int s = j % ST;
        if (j >= 2 && !mbar_wait(&dq_done[j & 1], ((j - 2) >> 1) & 1, flags, 324)) {
          ok = false;
          break;
        }
        if (!mbar_wait(&conv[s], (j / ST) & 1, flags, 325)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sk = smem_u32(smem + s * S::STAGE), sv = sk + S::K_HI;
        const uint32_t ds = tmem + S::C_S + (j & 1) * KB, dp = tmem + S::C_DP + (j & 1) * KB;
#pragma unroll
        for (int kk = 0; kk < HD / 8; kk++) {
          const uint32_t off = (kk >> 2) * S::K_SLAB + (kk & 3) * 32;
          const uint64_t dk = smem_desc(sk + off, 16, 1024, kLayoutSW128);
          const uint64_t dv = smem_desc(sv + off, 16, 1024, kLayoutSW128);
          mma_tf32_ts(ds, tmem + S::C_Q + HD + 8 * kk, dk, idesc_s, kk > 0 ? 1u : 0u);
          mma_tf32_ts(ds, tmem + S::C_Q + 8 * kk, dk + lo, idesc_s, 1u);
          mma_tf32_ts(ds, tmem + S::C_Q + 8 * kk, dk, idesc_s, 1u);
          mma_tf32_ts(dp, tmem + S::C_DO + HD + 8 * kk, dv, idesc_s, kk > 0 ? 1u : 0u);
          mma_tf32_ts(dp, tmem + S::C_DO + 8 * kk, dv + lo, idesc_s, 1u);
          mma_tf32_ts(dp, tmem + S::C_DO + 8 * kk, dv, idesc_s, 1u);
        }
        mma_commit(&sd_full[j & 1]);
        if (j >= 1 && !issue_dq(j - 1)) ok = false;
      }
      if (ok && issue_dq(nkb - 1)) mma_commit(dq_full);
    }
  } else if (warp < 6) {
    const int ct = threadIdx.x - 64;
    for (int j = 0; j < nkb; j++) {
      const int s = j % ST;
      if (!mbar_wait(&full[s], (j / ST) & 1, flags, 326)) break;
      split_lo(smem + s * S::STAGE, S::HI, S::HI, ct);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&conv[s]);
    }
  } else {
    const int qd = warp & 3;
    const int row = qd * 32 + lane, i = q0 + row;
    const bool in = i < T;
    const int n = min(i + 1, T);
    const uint32_t lrow = (uint32_t)(qd * 32) << 16;
    float Drow = 0.f;
    {
      const int ii = in ? i : 0;
      const float* qs = q.ptr + (long)b * q.stride_hi + (long)h * q.stride + (long)ii * q.ld;
      const float* gs = dout.ptr + (long)b * dout.stride_hi + (long)h * dout.stride + (long)ii * dout.ld;
      const float* os = o.ptr + (long)b * o.stride_hi + (long)h * o.stride + (long)ii * o.ld;
#pragma unroll 1
      for (int c = 0; c < HD; c += 32) {
        float v[32], w[32];
        ld_row32(qs + c, in, v);
        tmem_st_split(tmem + lrow + S::C_Q + c, tmem + lrow + S::C_Q + HD + c, v);
        ld_row32(gs + c, in, v);
        ld_row32(os + c, in, w);
#pragma unroll
        for (int e = 0; e < 32; e++) Drow += v[e] * w[e];
        tmem_st_split(tmem + lrow + S::C_DO + c, tmem + lrow + S::C_DO + HD + c, v);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(qd_ready);
    }
    if (in) Dout[(long)bh * T + i] = Drow;
    const float L = in ? lse[(long)bh * T + i] : 0.f;
    bool ok = true;
    for (int j = 0; j < nkb; j++) {
      if (!mbar_wait(&sd_full[j & 1], (j >> 1) & 1, flags, 327)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t cs = tmem + lrow + S::C_S + (j & 1) * KB;
      float sv[32], gv[32];
      tmem_ld32(cs, sv);
      tmem_ld32(tmem + lrow + S::C_DP + (j & 1) * KB, gv);
      const int k0 = j * KB;
#pragma unroll
      for (int c = 0; c < 32; c++) {
        const float p = k0 + c < n ? __expf(sv[c] * scale - L) : 0.f;
        sv[c] = p * (gv[c] - Drow) * scale;
      }
      tmem_st_split(cs, tmem + lrow + S::C_DSLO + (j & 1) * KB, sv);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ds_ready[j & 1]);
    }
    if (ok && mbar_wait(dq_full, 0, flags, 328)) {
      tc_fence_after();
      float* orow = dq + ((long)b * T + (in ? i : 0)) * ld_dq + (long)h * HD;
#pragma unroll 1
      for (int d0 = 0; d0 < HD; d0 += 32) {
        float v[32];
        tmem_ld32(tmem + lrow + S::C_DQ + d0, v);
        if (rope && in) {  // rotate back by -theta (pairs (2p, 2p + 1), theta of position i)
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const float2 cs2 = rope[(long)i * (HD / 2) + (d0 + e) / 2];
            const float g0 = v[e], g1 = v[e + 1];
            v[e] = g0 * cs2.x + g1 * cs2.y;
            v[e + 1] = -g0 * cs2.y + g1 * cs2.x;
          }
        }
        if (in) {
#pragma unroll
          for (int g = 0; g < 8; g++)
            *reinterpret_cast<float4*>(orow + d0 + 4 * g) = make_float4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_free_all(tmem);
  }
}

// ============================================================================ backward: dK, dV
// One CTA per (128-key tile, head); 320 threads:
//   warp 0      producer: the K tile once (K-major: A of S^T = K Q^T), then per 32-query block
//               Q and dO K-major (B of S^T and dP^T = V dO^T) and MN-major (B of dK, dV);
//               two-stage ring
//   warp 1      MMA issuer: S^T_i and dP^T_i into buffer i & 1, then dV += P^T_{i-1} dO_{i-1}
//               and dK += dS^T_{i-1} Q_{i-1}
//   warps 2..5  lo-part converters (the K tile, then each stage)
//   warps 6..9  row warps (row = key): V into TMEM; P^T = exp(scale s - L_q) and
//               dS^T = P^T (dP^T - D_q) scale written over S^T and dP^T; at the end dV and dK
//               (rotated back for RoPE) into dqkv
// TMEM columns: V hi | lo, S^T / P^T-hi 2 x 32, dP^T / dS^T-hi 2 x 32, P^T-lo 2 x 32,
// dS^T-lo 2 x 32, dV, dK.
template <int HD>
struct FlashDkv {
  static constexpr int QB = 32;
  static constexpr int SLABS = HD / 32;
  static constexpr int K_SLAB = 128 * 128;     // 128 keys x 32 floats, K-major
  static constexpr int K_HI = SLABS * K_SLAB;
  static constexpr int QK_SLAB = QB * 128;     // 32 queries x 32 floats, K-major
  static constexpr int QK_HI = SLABS * QK_SLAB;
  static constexpr int MN_BOX = 32 * 32 * 4;
  static constexpr int QM_HI = SLABS * MN_BOX;
  static constexpr int HI = 2 * QK_HI + 2 * QM_HI;  // Q | dO (K-major) | Q | dO (MN-major)
  static constexpr int STAGE = 2 * HI;
  static constexpr int STAGES = 2;
  static constexpr int KREG = 2 * K_HI;
  static constexpr int SMEM = KREG + STAGES * STAGE + 1024 + 512;
  static constexpr uint32_t C_V = 0, C_S = 2 * HD, C_DP = 2 * HD + 2 * QB, C_PLO = 2 * HD + 4 * QB,
                            C_DSLO = 2 * HD + 6 * QB, C_DV = 2 * HD + 8 * QB, C_DK = 3 * HD + 8 * QB;
  static_assert(C_DK + HD <= kFlashCols, "flash dK/dV: TMEM columns");
};

template <int HD>
__global__ void __launch_bounds__(320, 1)
    k_flash_dkv(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmQk,
                const __grid_constant__ CUtensorMap tmOk, const __grid_constant__ CUtensorMap tmQm,
                const __grid_constant__ CUtensorMap tmOm, GemmOperand v, const float* __restrict__ lse,
                const float* __restrict__ Dq, float* __restrict__ dqkv, long ld, const float2* __restrict__ rope,
                int T, int H, float scale, int* flags) {
  using S = FlashDkv<HD>;
  constexpr int QB = S::QB, ST = S::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem + S::KREG;
  uint64_t* bars = reinterpret_cast<uint64_t*>(stages + ST * S::STAGE);
  uint64_t* full = bars;           // [ST]
  uint64_t* conv = bars + 2;       // [ST]
  uint64_t* empty = bars + 4;      // [ST]
  uint64_t* sd_full = bars + 6;    // [2]
  uint64_t* p_ready = bars + 8;    // [2]
  uint64_t* kv_done = bars + 10;   // [2]
  uint64_t* k_full = bars + 12;
  uint64_t* k_conv = bars + 13;
  uint64_t* v_ready = bars + 14;
  uint64_t* acc_full = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x, b = bh / H, h = bh % H, E = H * HD;
  const int j0 = blockIdx.y * 128;           // first key of the tile (the first tiles see the most queries)
  const int nqb = (T - j0 + QB - 1) / QB;    // query blocks from query j0 on

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 4);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < 2; s++) {
      mbar_init(&sd_full[s], 1);
      mbar_init(&p_ready[s], 4);
      mbar_init(&kv_done[s], 1);
    }
    mbar_init(k_full, 1);
    mbar_init(k_conv, 4);
    mbar_init(v_ready, 4);
    mbar_init(acc_full, 1);
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc_all(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t sk = smem_u32(smem);
      mbar_arrive_expect_tx(k_full, S::K_HI);
      for (int sl = 0; sl < S::SLABS; sl++) tma_load_4d(sk + sl * S::K_SLAB, &tmK, 32 * sl, j0, h, b, k_full);
      for (int i = 0; i < nqb; i++) {
        const int s = i % ST, qb0 = j0 + i * QB;
        if (i >= ST && !mbar_wait(&empty[s], ((i / ST) - 1) & 1, flags, 341)) break;
        const uint32_t base = smem_u32(stages + s * S::STAGE);
        mbar_arrive_expect_tx(&full[s], S::HI);
        for (int sl = 0; sl < S::SLABS; sl++) {
          tma_load_4d(base + sl * S::QK_SLAB, &tmQk, 32 * sl, qb0, h, b, &full[s]);
          tma_load_4d(base + S::QK_HI + sl * S::QK_SLAB, &tmOk, 32 * sl, qb0, h, b, &full[s]);
          tma_load_4d(base + 2 * S::QK_HI + sl * S::MN_BOX, &tmQm, 32 * sl, qb0, h, b, &full[s]);
          tma_load_4d(base + 2 * S::QK_HI + S::QM_HI + sl * S::MN_BOX, &tmOm, 32 * sl, qb0, h, b, &full[s]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_tf32(QB, false);
      constexpr uint32_t idesc_a = idesc_tf32(HD, true);
      constexpr uint64_t lo = (uint64_t)(S::HI >> 4), lok = (uint64_t)(S::K_HI >> 4);
      bool ok = mbar_wait(k_conv, 0, flags, 342) && mbar_wait(v_ready, 0, flags, 343);
      auto issue_kv = [&](int c) -> bool {
        if (!mbar_wait(&p_ready[c & 1], (c >> 1) & 1, flags, 344)) return false;
        tc_fence_after();
        const uint32_t base = smem_u32(stages + (c % ST) * S::STAGE);
        const uint32_t sqm = base + 2 * S::QK_HI, som = sqm + S::QM_HI;
        const uint32_t p_hi = tmem + S::C_S + (c & 1) * QB, p_lo = tmem + S::C_PLO + (c & 1) * QB;
        const uint32_t g_hi = tmem + S::C_DP + (c & 1) * QB, g_lo = tmem + S::C_DSLO + (c & 1) * QB;
#pragma unroll
        for (int kk = 0; kk < QB / 8; kk++) {
          const uint64_t dO = smem_desc(som + kk * 1024, S::MN_BOX, 512, kLayoutSW128Atom32);
          const uint64_t dQ = smem_desc(sqm + kk * 1024, S::MN_BOX, 512, kLayoutSW128Atom32);
          const uint32_t first = (c > 0 || kk > 0) ? 1u : 0u;
          mma_tf32_ts(tmem + S::C_DV, p_lo + 8 * kk, dO, idesc_a, first);
          mma_tf32_ts(tmem + S::C_DV, p_hi + 8 * kk, dO + lo, idesc_a, 1u);
          mma_tf32_ts(tmem + S::C_DV, p_hi + 8 * kk, dO, idesc_a, 1u);
          mma_tf32_ts(tmem + S::C_DK, g_lo + 8 * kk, dQ, idesc_a, first);
          mma_tf32_ts(tmem + S::C_DK, g_hi + 8 * kk, dQ + lo, idesc_a, 1u);
          mma_tf32_ts(tmem + S::C_DK, g_hi + 8 * kk, dQ, idesc_a, 1u);
        }
        mma_commit(&kv_done[c & 1]);
        mma_commit(&empty[c % ST]);
        return true;
      };
      const uint32_t sk = smem_u32(smem);
      for (int i = 0; i < nqb && ok; i++) {
        const int s = i % ST;
        if (i >= 2 && !mbar_wait(&kv_done[i & 1], ((i - 2) >> 1) & 1, flags, 345)) {
          ok = false;
          break;
        }
        if (!mbar_wait(&conv[s], (i / ST) & 1, flags, 346)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t base = smem_u32(stages + s * S::STAGE);
        const uint32_t ds = tmem + S::C_S + (i & 1) * QB, dp = tmem + S::C_DP + (i & 1) * QB;
#pragma unroll
        for (int kk = 0; kk < HD / 8; kk++) {
          const uint64_t da = smem_desc(sk + (kk >> 2) * S::K_SLAB + (kk & 3) * 32, 16, 1024, kLayoutSW128);
          const uint64_t dq = smem_desc(base + (kk >> 2) * S::QK_SLAB + (kk & 3) * 32, 16, 1024, kLayoutSW128);
          const uint64_t dd = smem_desc(base + S::QK_HI + (kk >> 2) * S::QK_SLAB + (kk & 3) * 32, 16, 1024,
                                        kLayoutSW128);
          mma_tf32(ds, da + lok, dq, idesc_s, kk > 0 ? 1u : 0u);
          mma_tf32(ds, da, dq + lo, idesc_s, 1u);
          mma_tf32(ds, da, dq, idesc_s, 1u);
          mma_tf32_ts(dp, tmem + S::C_V + HD + 8 * kk, dd, idesc_s, kk > 0 ? 1u : 0u);
          mma_tf32_ts(dp, tmem + S::C_V + 8 * kk, dd + lo, idesc_s, 1u);
          mma_tf32_ts(dp, tmem + S::C_V + 8 * kk, dd, idesc_s, 1u);
        }
        mma_commit(&sd_full[i & 1]);
        if (i >= 1 && !issue_kv(i - 1)) ok = false;
      }
      if (ok && issue_kv(nqb - 1)) mma_commit(acc_full);
    }
  } else if (warp < 6) {
    const int ct = threadIdx.x - 64;
    if (mbar_wait(k_full, 0, flags, 347)) {
      split_lo(smem, S::K_HI, S::K_HI, ct);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(k_conv);
      for (int i = 0; i < nqb; i++) {
        const int s = i % ST;
        if (!mbar_wait(&full[s], (i / ST) & 1, flags, 348)) break;
        split_lo(stages + s * S::STAGE, S::HI, S::HI, ct);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[s]);
      }
    }
  } else {
    const int qd = warp & 3;
    const int j = j0 + qd * 32 + lane;  // this thread's key
    const bool in = j < T;
    const uint32_t lrow = (uint32_t)(qd * 32) << 16;
    {
      const float* vs = v.ptr + (long)b * v.stride_hi + (long)h * v.stride + (long)(in ? j : 0) * v.ld;
#pragma unroll 1
      for (int c = 0; c < HD; c += 32) {
        float x[32];
        ld_row32(vs + c, in, x);
        tmem_st_split(tmem + lrow + S::C_V + c, tmem + lrow + S::C_V + HD + c, x);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(v_ready);
    }
    bool ok = true;
    for (int i = 0; i < nqb; i++) {
      const int qb0 = j0 + i * QB;
      // lane c holds L and D of query qb0 + c (broadcast below by shuffles)
      const int qc = qb0 + lane;
      const float Lc = qc < T ? lse[(long)bh * T + qc] : 0.f;
      const float Dc = qc < T ? Dq[(long)bh * T + qc] : 0.f;
      if (!mbar_wait(&sd_full[i & 1], (i >> 1) & 1, flags, 349)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t cs = tmem + lrow + S::C_S + (i & 1) * QB, cd = tmem + lrow + S::C_DP + (i & 1) * QB;
      float sv[32], gv[32];
      tmem_ld32(cs, sv);
      tmem_ld32(cd, gv);
#pragma unroll
      for (int c = 0; c < 32; c++) {
        const float Lq = __shfl_sync(0xffffffffu, Lc, c), Dqv = __shfl_sync(0xffffffffu, Dc, c);
        const int qq = qb0 + c;
        const float p = (in && qq >= j && qq < T) ? __expf(sv[c] * scale - Lq) : 0.f;
        sv[c] = p;
        gv[c] = p * (gv[c] - Dqv) * scale;
      }
      tmem_st_split(cs, tmem + lrow + S::C_PLO + (i & 1) * QB, sv);
      tmem_st_split(cd, tmem + lrow + S::C_DSLO + (i & 1) * QB, gv);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_ready[i & 1]);
    }
    if (ok && mbar_wait(acc_full, 0, flags, 350)) {
      tc_fence_after();
      float* row = dqkv + ((long)b * T + (in ? j : 0)) * ld;
#pragma unroll 1
      for (int which = 0; which < 2; which++) {  // 0: dV -> [2E, 3E), 1: dK -> [E, 2E)
#pragma unroll 1
        for (int d0 = 0; d0 < HD; d0 += 32) {
          float x[32];
          tmem_ld32(tmem + lrow + (which ? S::C_DK : S::C_DV) + d0, x);
          if (which == 1 && rope && in) {  // rotate back by -theta of key position j
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              const float2 cs2 = rope[(long)j * (HD / 2) + (d0 + e) / 2];
              const float g0 = x[e], g1 = x[e + 1];
              x[e] = g0 * cs2.x + g1 * cs2.y;
              x[e + 1] = -g0 * cs2.y + g1 * cs2.x;
            }
          }
          if (in) {
            float* dst = row + (which == 0 ? 2 * E : E) + h * HD + d0;
#pragma unroll
            for (int g = 0; g < 8; g++)
              *reinterpret_cast<float4*>(dst + 4 * g) = make_float4(x[4 * g], x[4 * g + 1], x[4 * g + 2], x[4 * g + 3]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_free_all(tmem);
  }
}

template <int HD>
int flash_fwd(cudaStream_t st, const GemmOperand& q, const GemmOperand& k, const GemmOperand& v, float* out,
              long ld_out, float* lse, int B, int T, int H, float scale, int* flags) {
  using S = FlashFwd<HD>;
  static_assert(S::SMEM <= 232448, "flash forward: shared memory budget exceeded");
  static std::atomic<uint64_t> attr{0};
  RC(smem_attr_per_device(attr, k_flash_fwd<HD>, S::SMEM));
  CUtensorMap mk, mv;
  RC(tensor_map_f32(&mk, k, HD, T, H, B * H, 32, S::KB, false));
  RC(tensor_map_f32(&mv, v, HD, T, H, B * H, 32, 32, true));
  TURT_CHECK_CUDA((launch_pdl(k_flash_fwd<HD>, dim3(B * H, ceil_div(T, 128)), dim3(320), S::SMEM, st, mk, mv, q, out,
                              ld_out, lse, T, H, scale, flags)));
  TURT_LAUNCH_CHECK();
  return OK;
}

template <int HD>
int flash_bwd(cudaStream_t st, const GemmOperand& q, const GemmOperand& k, const GemmOperand& v,
              const GemmOperand& dout, const GemmOperand& o, const float* lse, float* D, float* dqkv, long ld,
              const float2* rope, int B, int T, int H, float scale, int* flags) {
  using SQ = FlashDq<HD>;
  using SK = FlashDkv<HD>;
  static_assert(SQ::SMEM <= 232448 && SK::SMEM <= 232448, "flash backward: shared memory budget exceeded");
  static std::atomic<uint64_t> attr_q{0}, attr_kv{0};
  RC(smem_attr_per_device(attr_q, k_flash_dq<HD>, SQ::SMEM));
  RC(smem_attr_per_device(attr_kv, k_flash_dkv<HD>, SK::SMEM));
  CUtensorMap mk, mv, mkm;
  RC(tensor_map_f32(&mk, k, HD, T, H, B * H, 32, SQ::KB, false));
  RC(tensor_map_f32(&mv, v, HD, T, H, B * H, 32, SQ::KB, false));
  RC(tensor_map_f32(&mkm, k, HD, T, H, B * H, 32, 32, true));
  TURT_CHECK_CUDA((launch_pdl(k_flash_dq<HD>, dim3(B * H, ceil_div(T, 128)), dim3(320), SQ::SMEM, st, mk, mv, mkm, q,
                              dout, o, lse, D, dqkv, ld, rope, T, H, scale, flags)));
  TURT_LAUNCH_CHECK();
  CUtensorMap mk128, mqk, mok, mqm, mom;
  RC(tensor_map_f32(&mk128, k, HD, T, H, B * H, 32, 128, false));
  RC(tensor_map_f32(&mqk, q, HD, T, H, B * H, 32, SK::QB, false));
  RC(tensor_map_f32(&mok, dout, HD, T, H, B * H, 32, SK::QB, false));
  RC(tensor_map_f32(&mqm, q, HD, T, H, B * H, 32, 32, true));
  RC(tensor_map_f32(&mom, dout, HD, T, H, B * H, 32, 32, true));
  TURT_CHECK_CUDA((launch_pdl(k_flash_dkv<HD>, dim3(B * H, ceil_div(T, 128)), dim3(320), SK::SMEM, st, mk128, mqk, mok,
                              mqm, mom, v, lse, (const float*)D, dqkv, ld, rope, T, H, scale, flags)));
  TURT_LAUNCH_CHECK();
  return OK;
}

}  // namespace

bool attention_flash_supported(int T, int hd) { return T >= 1 && (hd == 32 || hd == 64); }

int attention_flash_fwd(cudaStream_t st, const GemmOperand& q, const GemmOperand& k, const GemmOperand& v, float* out,
                        long ld_out, float* lse, int B, int T, int H, int hd, float scale, int* flags) {
  TURT_REQUIRE(attention_flash_supported(T, hd), "flash attention: head dim must be 32 or 64");
  TURT_REQUIRE(lse, "flash attention: log-sum-exp buffer missing");
  if (hd == 64) return flash_fwd<64>(st, q, k, v, out, ld_out, lse, B, T, H, scale, flags);
  return flash_fwd<32>(st, q, k, v, out, ld_out, lse, B, T, H, scale, flags);
}

int attention_flash_bwd(cudaStream_t st, const GemmOperand& q, const GemmOperand& k, const GemmOperand& v,
                        const GemmOperand& dout, const GemmOperand& o, const float* lse, float* D, float* dqkv,
                        long ld, const float2* rope, int B, int T, int H, int hd, float scale, int* flags) {
  TURT_REQUIRE(attention_flash_supported(T, hd), "flash attention: head dim must be 32 or 64");
  TURT_REQUIRE(lse && D, "flash attention: log-sum-exp / row-dot buffers missing");
  if (hd == 64) return flash_bwd<64>(st, q, k, v, dout, o, lse, D, dqkv, ld, rope, B, T, H, scale, flags);
  return flash_bwd<32>(st, q, k, v, dout, o, lse, D, dqkv, ld, rope, B, T, H, scale, flags);
}

}  // namespace turt
