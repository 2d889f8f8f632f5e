// attention_fused.cu -- causal attention forward for sequences of up to 256 tokens in one kernel.
//
// The tensor-core path materialises the reference's chain (src/models/gpt.ts:126-141: scores,
// scale, causal mask, softmax, P.V) as three launches: S = Q K^T written out, the softmax in
// place, O = P V reading P back.  With T <= 256 a tile of 128 query rows meets at most 256 keys,
// so its whole score block fits the tensor memory (256 fp32 columns of the 512): this kernel
// computes S there, takes the row softmax in registers, writes P once (the backward pass keeps
// using it) and multiplies P by V from shared memory, 64 keys at a time.  The arithmetic is the
// unfused path's: 3xTF32 products with fp32 accumulation, softmax of scale * s minus the row
// maximum, P = exp(.) / sum, zeros right of the diagonal.
//
// One CTA per (query tile of 128 rows, batch entry, head); 448 threads:
//   warp 0       TMA producer: Q and K tiles, then V in 64-key chunks (two buffers)
//   warp 1       TMEM allocator + MMA issuer: S = Q K^T, then O += P_c V_c per chunk
//   warps 2..9   softmax and output: warp w owns TMEM lanes (query rows) 32*(w%4) .. +31 and
//                the 32-key column blocks of parity (w - 2) / 4 (two warps per row, so the
//                exponentials of a 128-row tile run on 256 threads)
//   warps 10..13 lo-part converters for Q, K and each V chunk (3xTF32 splits)
// Shared memory holds Q|K (hi and lo) during the score product, then the same bytes hold two
// P chunks and two V chunks (hi and lo): 192 KB for a head dim of 64.
#include "attention.cuh"
#include "gemm.cuh"
#include "tcgen05.cuh"

namespace turt {
namespace {

constexpr int kFQ = 128;        // query rows per CTA (TMEM lanes)
constexpr int kFKeys = 256;     // keys one CTA can hold in TMEM
constexpr int kFThreads = 448;  // see the file comment
constexpr uint32_t kFTmemCols = 512;
constexpr uint32_t kFTmemO = 256;  // O accumulator columns [256, 256 + HD)

template <int HD>
struct FShape {
  static constexpr int SLABS = HD / 32;           // 32-float k slabs of the Q / K rows
  static constexpr int Q_SLAB = kFQ * 128;        // bytes of one slab of the Q tile
  static constexpr int K_SLAB = kFKeys * 128;     // bytes of one slab of the K tile
  static constexpr int Q_BYTES = SLABS * Q_SLAB;  // one copy (hi or lo)
  static constexpr int K_BYTES = SLABS * K_SLAB;
  static constexpr int Q_HI = 0, K_HI = 2 * Q_BYTES;
  static constexpr int PH1 = 2 * Q_BYTES + 2 * K_BYTES;
  static constexpr int P_SLAB = kFQ * 128;   // 32 keys of P, K-major A operand
  static constexpr int P_BYTES = 2 * P_SLAB; // one 64-key chunk, one copy
  static constexpr int V_BOX = 32 * 32 * 4;  // MN-major box: 32 head-dim values x 32 keys
  static constexpr int V_SLAB = SLABS * V_BOX;
  static constexpr int V_BYTES = 2 * V_SLAB;  // one 64-key chunk, one copy
  static constexpr int PH2 = 4 * P_BYTES + 4 * V_BYTES;
  static constexpr int REGION = PH1 > PH2 ? PH1 : PH2;
  static constexpr int SMEM = REGION + 256 + 2048 + 1024;  // + barriers, row max / sum halves, alignment
  __host__ __device__ static constexpr int p_hi(int s) { return s * 2 * P_BYTES; }
  __host__ __device__ static constexpr int v_hi(int s) { return 4 * P_BYTES + s * 2 * V_BYTES; }
};

// lo = x - tf32(x) for `bytes` of fp32 at `hi`, written `lo_off` bytes further (converter threads).
__device__ __forceinline__ void lo_split(uint8_t* hi_base, int bytes, int lo_off, int ct) {
  const float4* hi = reinterpret_cast<const float4*>(hi_base);
  float4* lo = reinterpret_cast<float4*>(hi_base + lo_off);
#pragma unroll 4
  for (int e = ct; e < bytes / 16; e += 128) {
    const float4 v = hi[e];
    float4 r;
    r.x = v.x - __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
    r.y = v.y - __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
    r.z = v.z - __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
    r.w = v.w - __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
    lo[e] = r;
  }
}

__device__ __forceinline__ float4 lo4(float4 v) {
  return make_float4(v.x - __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u),
                     v.y - __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u),
                     v.z - __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u),
                     v.w - __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u));
}

// Bulk tensor store of one 128-row x 32-float box from shared memory (same swizzled layout as
// the loads), tracked as a bulk-async group of the issuing thread.
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, uint32_t src, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until at most N committed groups still read their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// The eight softmax warps (256 threads) meet at named barrier 1.
__device__ __forceinline__ void softmax_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

template <int HD>
__global__ void __launch_bounds__(kFThreads, 1)
    k_attn_fwd_fused(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmP, long pitch,
                     float* __restrict__ out, long ld_out, int T, int H, float scale, int* flags) {
  using S = FShape<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::REGION);
  uint64_t* qk_full = bars + 0;
  uint64_t* qk_conv = bars + 1;
  uint64_t* s_full = bars + 2;
  uint64_t* o_full = bars + 3;
  uint64_t* v_full = bars + 4;   // [2]
  uint64_t* v_conv = bars + 6;   // [2]
  uint64_t* v_empty = bars + 8;  // [2]
  uint64_t* p_ready = bars + 10; // [2]
  uint64_t* p_free = bars + 12;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  volatile int* sm_ok = reinterpret_cast<volatile int*>(tmem_slot + 1);  // softmax group's shared verdict
  float* red = reinterpret_cast<float*>(smem + S::REGION + 256);          // [2 halves][128 rows]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // grid (heads, query tiles), the last (longest: most keys) query tiles first: CTAs dispatch
  // x-fastest, so the short tiles fill the tail of the last wave
  const int bh = blockIdx.x, b = bh / H, h = bh % H;
  const int q0 = (gridDim.y - 1 - blockIdx.y) * kFQ;
  const int nk = min(T, q0 + kFQ);          // keys any row of this tile can see
  const int nkr = (nk + 63) & ~63;          // rounded up to whole 64-key chunks (<= 256)
  const int nch = nkr / 64;
  const int nbox = (nkr + 127) / 128;       // 128-row TMA boxes of K per slab

  if (threadIdx.x == 0) {
    mbar_init(qk_full, 1);
    mbar_init(qk_conv, 4);
    mbar_init(s_full, 1);
    mbar_init(o_full, 1);
    for (int s = 0; s < 2; s++) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_conv[s], 4);
      mbar_init(&v_empty[s], 1);
      mbar_init(&p_ready[s], 1);
      mbar_init(&p_free[s], 1);
    }
    mbar_fence_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kFTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- TMA producer
      const uint32_t sq = smem_u32(smem + S::Q_HI), sk = smem_u32(smem + S::K_HI);
      mbar_arrive_expect_tx(qk_full, S::SLABS * (S::Q_SLAB + nbox * 16384));
      for (int sl = 0; sl < S::SLABS; sl++) {
        tma_load_4d(sq + sl * S::Q_SLAB, &tmQ, sl * 32, q0, h, b, qk_full);
        for (int bx = 0; bx < nbox; bx++) tma_load_4d(sk + sl * S::K_SLAB + bx * 16384, &tmK, sl * 32, bx * 128, h, b, qk_full);
      }
      // V chunks reuse the Q / K bytes: wait until the score product has read them
      bool ok = mbar_wait(s_full, 0, flags, 131);
      for (int c = 0; c < nch && ok; c++) {
        const int s = c & 1;
        if (c >= 2 && !mbar_wait(&v_empty[s], ((c >> 1) - 1) & 1, flags, 132)) break;
        const uint32_t sv = smem_u32(smem + S::v_hi(s));
        mbar_arrive_expect_tx(&v_full[s], S::V_BYTES);
        for (int sl = 0; sl < 2; sl++)
          for (int j = 0; j < S::SLABS; j++)
            tma_load_4d(sv + sl * S::V_SLAB + j * S::V_BOX, &tmV, 32 * j, c * 64 + sl * 32, h, b, &v_full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      bool ok = mbar_wait(qk_conv, 0, flags, 133);
      if (ok) {
        tc_fence_after();
        const uint32_t idesc_s = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(nkr >> 3) << 17) |
                                 ((uint32_t)(kFQ >> 4) << 24);
        const uint32_t sq = smem_u32(smem + S::Q_HI), sk = smem_u32(smem + S::K_HI);
        const uint64_t loq = (uint64_t)(S::Q_BYTES >> 4), lok = (uint64_t)(S::K_BYTES >> 4);
#pragma unroll
        for (int kk = 0; kk < HD / 8; kk++) {
          const uint64_t da = smem_desc(sq + (kk >> 2) * S::Q_SLAB + (kk & 3) * 32, 16, 1024, kLayoutSW128);
          const uint64_t db = smem_desc(sk + (kk >> 2) * S::K_SLAB + (kk & 3) * 32, 16, 1024, kLayoutSW128);
          mma_tf32(tmem, da + loq, db, idesc_s, kk > 0 ? 1u : 0u);
          mma_tf32(tmem, da, db + lok, idesc_s, 1u);
          mma_tf32(tmem, da, db, idesc_s, 1u);
        }
        mma_commit(s_full);
      }
      constexpr uint32_t idesc_o = (1u << 4) | (2u << 7) | (2u << 10) | (1u << 16) | ((uint32_t)(HD >> 3) << 17) |
                                   ((uint32_t)(kFQ >> 4) << 24);
      const uint64_t lop = (uint64_t)(S::P_BYTES >> 4), lov = (uint64_t)(S::V_BYTES >> 4);
      for (int c = 0; c < nch && ok; c++) {
        const int s = c & 1;
        if (!mbar_wait(&p_ready[s], (c >> 1) & 1, flags, 134) || !mbar_wait(&v_conv[s], (c >> 1) & 1, flags, 135)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sp = smem_u32(smem + S::p_hi(s)), sv = smem_u32(smem + S::v_hi(s));
#pragma unroll
        for (int kk = 0; kk < 8; kk++) {
          const uint64_t da = smem_desc(sp + (kk >> 2) * S::P_SLAB + (kk & 3) * 32, 16, 1024, kLayoutSW128);
          const uint64_t db = smem_desc(sv + (kk >> 2) * S::V_SLAB + (kk & 3) * 1024, S::V_BOX, 512, kLayoutSW128Atom32);
          const uint32_t first = (c > 0 || kk > 0) ? 1u : 0u;
          mma_tf32(tmem + kFTmemO, da + lop, db, idesc_o, first);
          mma_tf32(tmem + kFTmemO, da, db + lov, idesc_o, 1u);
          mma_tf32(tmem + kFTmemO, da, db, idesc_o, 1u);
        }
        mma_commit(&v_empty[s]);
        mma_commit(&p_free[s]);
      }
      if (ok) mma_commit(o_full);
    }
  } else if (warp >= 10) {
    // ---------------------------------------------------------------- lo-part converters
    const int ct = threadIdx.x - 320;
    bool ok = mbar_wait(qk_full, 0, flags, 136);
    if (ok) {
      lo_split(smem + S::Q_HI, S::Q_BYTES, S::Q_BYTES, ct);
      for (int sl = 0; sl < S::SLABS; sl++) lo_split(smem + S::K_HI + sl * S::K_SLAB, nbox * 16384, S::K_BYTES, ct);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(qk_conv);
    }
    for (int c = 0; c < nch && ok; c++) {
      const int s = c & 1;
      if (!mbar_wait(&v_full[s], (c >> 1) & 1, flags, 137)) break;
      lo_split(smem + S::v_hi(s), S::V_BYTES, S::V_BYTES, ct);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&v_conv[s]);
    }
  } else {
    // ---------------------------------------------------------------- softmax + output
    // P leaves through bulk tensor stores issued by thread 64 (warp 2, lane 0) from the same
    // swizzled chunk buffers the P.V products read, so the global writes are whole lines.
    const int q = warp & 3, half = (warp - 2) >> 2;
    const int row = q * 32 + lane, i = q0 + row;  // query index
    const int n = min(i + 1, T);                  // keys this row sees
    const int warp_last = q0 + q * 32 + 31;       // last query row of this warp
    const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
    const bool issuer = threadIdx.x == 64;
    // Every wait of this group is done by the issuer alone and its verdict shared through
    // sm_ok at a named barrier, so all 256 threads take the same path through every barrier.
    if (issuer) *sm_ok = mbar_wait(s_full, 0, flags, 138) ? 1 : 0;
    softmax_sync();
    bool ok = *sm_ok != 0;
    if (ok) {
      tc_fence_after();
      // this warp's column blocks: cc = half, half + 2, ... while left of its last row
      float mx = -INFINITY;
      for (int cc = half; cc < nkr / 32 && cc * 32 <= warp_last; cc += 2) {
        float v[32];
        tmem_ld32(trow + cc * 32, v);
#pragma unroll
        for (int j = 0; j < 32; j++)
          if (cc * 32 + j < n) mx = fmaxf(mx, v[j] * scale);
      }
      red[half * 128 + row] = mx;
      softmax_sync();
      mx = fmaxf(red[row], red[128 + row]);
      softmax_sync();  // both halves read the maxima before the sums overwrite them
      // e = exp(scale * s - max), kept in TMEM over the scores for the normalising pass
      float sum = 0.f;
      for (int cc = half; cc < nkr / 32 && cc * 32 <= warp_last; cc += 2) {
        float v[32];
        tmem_ld32(trow + cc * 32, v);
#pragma unroll
        for (int j = 0; j < 32; j++) {
          v[j] = cc * 32 + j < n ? __expf(v[j] * scale - mx) : 0.f;
          sum += v[j];
        }
        tmem_st32(trow + cc * 32, v);
      }
      red[half * 128 + row] = sum;
      softmax_sync();
      const float inv = 1.0f / (red[row] + red[128 + row]);
      for (int c = 0; c < nch; c++) {
        const int s = c & 1;
        if (c >= 2) {
          // buffer s is free once the products of chunk c - 2 ran and its store has read it
          if (issuer) {
            *sm_ok = mbar_wait(&p_free[s], ((c >> 1) - 1) & 1, flags, 139) ? 1 : 0;
            bulk_wait_read<1>();
          }
          softmax_sync();
          ok = *sm_ok != 0;
          if (!ok) break;
        }
        const int cc = 2 * c + half;
        float v[32];
        if (cc * 32 <= warp_last) {  // warp-uniform
          tmem_ld32(trow + cc * 32, v);
#pragma unroll
          for (int j = 0; j < 32; j++) v[j] *= inv;
        } else {
#pragma unroll
          for (int j = 0; j < 32; j++) v[j] = 0.f;
        }
        // K-major rows of 128 B with 16-byte chunks XOR (row % 8): the A operand of O += P V
        // and the source of the bulk store
        uint8_t* slab = smem + S::p_hi(s) + half * S::P_SLAB + row * 128;
#pragma unroll
        for (int g = 0; g < 8; g++) {
          const float4 x = make_float4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
          const int off = ((g ^ (row & 7)) * 16);
          *reinterpret_cast<float4*>(slab + off) = x;
          *reinterpret_cast<float4*>(slab + S::P_BYTES + off) = lo4(x);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        softmax_sync();
        if (issuer) {
          const uint32_t sp = smem_u32(smem + S::p_hi(s));
          for (int hh = 0; hh < 2; hh++)
            if ((2 * c + hh) * 32 < pitch) tma_store_4d(&tmP, sp + hh * S::P_SLAB, (2 * c + hh) * 32, q0, h, b);
          bulk_commit();
          mbar_arrive(&p_ready[s]);
        }
      }
    }
    if (ok) {
      if (issuer) *sm_ok = mbar_wait(o_full, 0, flags, 140) ? 1 : 0;
      softmax_sync();
      ok = *sm_ok != 0;
    }
    if (ok) {
      tc_fence_after();
      const bool store = i < T;
      float* orow = out + ((long)b * T + (store ? i : 0)) * ld_out + (long)h * HD;
      for (int d0 = half * 32; d0 < HD; d0 += 64) {  // warp-uniform: halves take alternate 32 columns
        float v[32];
        tmem_ld32(trow + kFTmemO + d0, v);
        if (store) {
#pragma unroll
          for (int g = 0; g < 8; g++)
            *reinterpret_cast<float4*>(orow + d0 + 4 * g) = make_float4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
        }
      }
      // columns [nkr, pitch) of P: zeros, stored from a zeroed 32-column slab of buffer 0 (every
      // product has run, so the buffers are free once the pending stores have read them)
      if (nkr < pitch) {
        if (issuer) bulk_wait_read<0>();
        softmax_sync();
        uint8_t* zslab = smem + S::p_hi(0) + row * 128 + half * 64;
#pragma unroll
        for (int g = 0; g < 4; g++) *reinterpret_cast<float4*>(zslab + 16 * g) = make_float4(0.f, 0.f, 0.f, 0.f);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        softmax_sync();
        if (issuer) {
          for (long col = nkr; col < pitch; col += 32) tma_store_4d(&tmP, smem_u32(smem + S::p_hi(0)), (int)col, q0, h, b);
          bulk_commit();
        }
      }
    }
    if (issuer) bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kFTmemCols) : "memory");
  }
}


// Backward of the softmax and dQ for T <= 256 in one kernel: dP = dO v^T into TMEM (the
// score-product machinery above with dO for q and v for k), P of the tile loaded into shared
// memory by TMA, per row D = sum_j P_j dP_j and dS_j = P_j (dP_j - D) * scale (j <= i; 0 right
// of the diagonal), written over P in place 64 keys at a time and stored by bulk tensor stores;
// each dS chunk also feeds dQ += dS_c k_c on the tensor cores (k chunks MN-major from TMA), so
// dQ leaves the kernel finished (rotated back by -theta for RoPE models).  Replaces the dP GEMM,
// the softmax-backward row kernel and the dQ GEMM; same warp roles as the forward.
template <int HD>
struct DShape {
  using F = FShape<HD>;
  static constexpr int DL = 8 * F::P_SLAB;           // dS lo of one 64-key chunk (2 slabs)
  static constexpr int KC = DL + 2 * F::P_SLAB;      // k chunk, MN-major, hi then lo
  static constexpr int PH2 = KC + 2 * F::V_BYTES;
  static constexpr int REGION = F::PH1 > PH2 ? F::PH1 : PH2;
  static constexpr int SMEM = REGION + 256 + 4096 + 1024;
};

template <int HD>
__global__ void __launch_bounds__(kFThreads, 1)
    k_attn_dsoftmax_fused(const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmV,
                          const __grid_constant__ CUtensorMap tmP, const __grid_constant__ CUtensorMap tmS,
                          const __grid_constant__ CUtensorMap tmK, long pitch, float* __restrict__ dq, long ld_dq,
                          const float2* __restrict__ rope, int T, int H, float scale, int* flags) {
  using S = FShape<HD>;
  using D = DShape<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + D::REGION);
  uint64_t* qk_full = bars + 0;
  uint64_t* qk_conv = bars + 1;
  uint64_t* s_full = bars + 2;
  uint64_t* p_full = bars + 3;
  uint64_t* ds_ready = bars + 4;
  uint64_t* dsl_free = bars + 5;
  uint64_t* k_full = bars + 6;
  uint64_t* k_conv = bars + 7;
  uint64_t* k_empty = bars + 8;
  uint64_t* dq_full = bars + 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
  volatile int* sm_ok = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(smem + D::REGION + 256);  // [2 halves][128 rows]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // grid (heads, query tiles), the last (longest: most keys) query tiles first: CTAs dispatch
  // x-fastest, so the short tiles fill the tail of the last wave
  const int bh = blockIdx.x, b = bh / H, h = bh % H;
  const int q0 = (gridDim.y - 1 - blockIdx.y) * kFQ;
  const int nk = min(T, q0 + kFQ);
  const int nkr = (nk + 63) & ~63;
  const int nch = nkr / 64;
  const int nbox = (nkr + 127) / 128;

  if (threadIdx.x == 0) {
    mbar_init(qk_full, 1);
    mbar_init(qk_conv, 4);
    mbar_init(s_full, 1);
    mbar_init(p_full, 1);
    mbar_init(ds_ready, 1);
    mbar_init(dsl_free, 1);
    mbar_init(k_full, 1);
    mbar_init(k_conv, 4);
    mbar_init(k_empty, 1);
    mbar_init(dq_full, 1);
    mbar_fence_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kFTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- TMA producer
      const uint32_t sq = smem_u32(smem + S::Q_HI), sk = smem_u32(smem + S::K_HI);
      mbar_arrive_expect_tx(qk_full, S::SLABS * (S::Q_SLAB + nbox * 16384));
      for (int sl = 0; sl < S::SLABS; sl++) {
        tma_load_4d(sq + sl * S::Q_SLAB, &tmO, sl * 32, q0, h, b, qk_full);
        for (int bx = 0; bx < nbox; bx++)
          tma_load_4d(sk + sl * S::K_SLAB + bx * 16384, &tmV, sl * 32, bx * 128, h, b, qk_full);
      }
      // P and the k chunks reuse the dO / v bytes once the product has read them
      bool ok = mbar_wait(s_full, 0, flags, 151);
      if (ok) {
        mbar_arrive_expect_tx(p_full, (nkr / 32) * S::P_SLAB);
        for (int sl = 0; sl < nkr / 32; sl++)
          tma_load_4d(smem_u32(smem) + sl * S::P_SLAB, &tmP, sl * 32, q0, h, b, p_full);
      }
      for (int c = 0; c < nch && ok; c++) {
        if (c >= 1 && !mbar_wait(k_empty, (c - 1) & 1, flags, 157)) break;
        const uint32_t kc = smem_u32(smem + D::KC);
        mbar_arrive_expect_tx(k_full, S::V_BYTES);
        for (int sl = 0; sl < 2; sl++)
          for (int j = 0; j < S::SLABS; j++)
            tma_load_4d(kc + sl * S::V_SLAB + j * S::V_BOX, &tmK, 32 * j, c * 64 + sl * 32, h, b, k_full);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      bool ok = mbar_wait(qk_conv, 0, flags, 152);
      if (ok) {
        tc_fence_after();
        const uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(nkr >> 3) << 17) |
                               ((uint32_t)(kFQ >> 4) << 24);
        const uint32_t sq = smem_u32(smem + S::Q_HI), sk = smem_u32(smem + S::K_HI);
        const uint64_t loq = (uint64_t)(S::Q_BYTES >> 4), lok = (uint64_t)(S::K_BYTES >> 4);
#pragma unroll
        for (int kk = 0; kk < HD / 8; kk++) {
          const uint64_t da = smem_desc(sq + (kk >> 2) * S::Q_SLAB + (kk & 3) * 32, 16, 1024, kLayoutSW128);
          const uint64_t db = smem_desc(sk + (kk >> 2) * S::K_SLAB + (kk & 3) * 32, 16, 1024, kLayoutSW128);
          mma_tf32(tmem, da + loq, db, idesc, kk > 0 ? 1u : 0u);
          mma_tf32(tmem, da, db + lok, idesc, 1u);
          mma_tf32(tmem, da, db, idesc, 1u);
        }
        mma_commit(s_full);
      }
      constexpr uint32_t idesc_q = (1u << 4) | (2u << 7) | (2u << 10) | (1u << 16) | ((uint32_t)(HD >> 3) << 17) |
                                   ((uint32_t)(kFQ >> 4) << 24);
      const uint64_t lok = (uint64_t)(S::V_BYTES >> 4);
      for (int c = 0; c < nch && ok; c++) {
        if (!mbar_wait(ds_ready, c & 1, flags, 158) || !mbar_wait(k_conv, c & 1, flags, 159)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // dS chunk c: hi in slabs 2c, 2c+1 of the P tile, lo in the DL buffer
        const uint32_t sd = smem_u32(smem) + 2 * c * S::P_SLAB, sk = smem_u32(smem + D::KC);
        const uint64_t lod = (uint64_t)((D::DL - 2 * c * S::P_SLAB) >> 4);
#pragma unroll
        for (int kk = 0; kk < 8; kk++) {
          const uint64_t da = smem_desc(sd + (kk >> 2) * S::P_SLAB + (kk & 3) * 32, 16, 1024, kLayoutSW128);
          const uint64_t db = smem_desc(sk + (kk >> 2) * S::V_SLAB + (kk & 3) * 1024, S::V_BOX, 512, kLayoutSW128Atom32);
          const uint32_t first = (c > 0 || kk > 0) ? 1u : 0u;
          mma_tf32(tmem + kFTmemO, da + lod, db, idesc_q, first);
          mma_tf32(tmem + kFTmemO, da, db + lok, idesc_q, 1u);
          mma_tf32(tmem + kFTmemO, da, db, idesc_q, 1u);
        }
        mma_commit(dsl_free);
        mma_commit(k_empty);
      }
      if (ok) mma_commit(dq_full);
    }
  } else if (warp >= 10) {
    // ---------------------------------------------------------------- lo-part converters
    const int ct = threadIdx.x - 320;
    bool ok = mbar_wait(qk_full, 0, flags, 153);
    if (ok) {
      lo_split(smem + S::Q_HI, S::Q_BYTES, S::Q_BYTES, ct);
      for (int sl = 0; sl < S::SLABS; sl++) lo_split(smem + S::K_HI + sl * S::K_SLAB, nbox * 16384, S::K_BYTES, ct);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(qk_conv);
    }
    for (int c = 0; c < nch && ok; c++) {
      if (!mbar_wait(k_full, c & 1, flags, 160)) break;
      lo_split(smem + D::KC, S::V_BYTES, S::V_BYTES, ct);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(k_conv);
    }
  } else {
    // ---------------------------------------------------------------- row arithmetic + dQ out
    const int q = warp & 3, half = (warp - 2) >> 2;
    const int row = q * 32 + lane, i = q0 + row;
    const int n = min(i + 1, T);
    const int warp_last = q0 + q * 32 + 31;
    const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
    const bool issuer = threadIdx.x == 64;
    if (issuer) *sm_ok = (mbar_wait(s_full, 0, flags, 154) && mbar_wait(p_full, 0, flags, 155)) ? 1 : 0;
    softmax_sync();
    bool ok = *sm_ok != 0;
    if (ok) {
      mbar_wait(p_full, 0, flags, 156);  // complete already: orders the TMA-written P before the reads below
      tc_fence_after();
      float Dsum = 0.f;
      for (int cc = half; cc < nkr / 32 && cc * 32 <= warp_last; cc += 2) {
        float g[32];
        tmem_ld32(trow + cc * 32, g);
        const uint8_t* prow = smem + cc * S::P_SLAB + row * 128;
#pragma unroll
        for (int k = 0; k < 8; k++) {
          const float4 p = *reinterpret_cast<const float4*>(prow + ((k ^ (row & 7)) * 16));
          const int j = cc * 32 + 4 * k;
          Dsum += (j + 0 < n ? p.x * g[4 * k + 0] : 0.f) + (j + 1 < n ? p.y * g[4 * k + 1] : 0.f) +
                  (j + 2 < n ? p.z * g[4 * k + 2] : 0.f) + (j + 3 < n ? p.w * g[4 * k + 3] : 0.f);
        }
      }
      red[half * 128 + row] = Dsum;
      softmax_sync();
      Dsum = red[row] + red[128 + row];
      for (int c = 0; c < nch; c++) {
        if (c >= 1) {  // the dS lo buffer is free once the dQ products of chunk c - 1 ran
          if (issuer) *sm_ok = mbar_wait(dsl_free, (c - 1) & 1, flags, 161) ? 1 : 0;
          softmax_sync();
          ok = *sm_ok != 0;
          if (!ok) break;
        }
        const int cc = 2 * c + half;
        uint8_t* prow = smem + cc * S::P_SLAB + row * 128;
        uint8_t* lrow = smem + D::DL + half * S::P_SLAB + row * 128;
        if (cc * 32 <= warp_last) {  // warp-uniform
          float g[32];
          tmem_ld32(trow + cc * 32, g);
#pragma unroll
          for (int k = 0; k < 8; k++) {
            const int off = (k ^ (row & 7)) * 16;
            float4* pp = reinterpret_cast<float4*>(prow + off);
            const float4 p = *pp;
            const int j = cc * 32 + 4 * k;
            const float4 x = make_float4(j + 0 < n ? p.x * (g[4 * k + 0] - Dsum) * scale : 0.f,
                                         j + 1 < n ? p.y * (g[4 * k + 1] - Dsum) * scale : 0.f,
                                         j + 2 < n ? p.z * (g[4 * k + 2] - Dsum) * scale : 0.f,
                                         j + 3 < n ? p.w * (g[4 * k + 3] - Dsum) * scale : 0.f);
            *pp = x;
            *reinterpret_cast<float4*>(lrow + off) = lo4(x);
          }
        } else {
#pragma unroll
          for (int k = 0; k < 8; k++) {
            *reinterpret_cast<float4*>(prow + 16 * k) = make_float4(0.f, 0.f, 0.f, 0.f);
            *reinterpret_cast<float4*>(lrow + 16 * k) = make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        softmax_sync();
        if (issuer) {
          for (int hh = 0; hh < 2; hh++)
            if ((2 * c + hh) * 32 < pitch)
              tma_store_4d(&tmS, smem_u32(smem) + (2 * c + hh) * S::P_SLAB, (2 * c + hh) * 32, q0, h, b);
          bulk_commit();
          mbar_arrive(ds_ready);
        }
      }
      // columns [nkr, pitch) of dS: zeros from a zeroed slab past the tile's chunks
      if (ok && nkr < pitch) {
        uint8_t* z = smem + (nkr / 32) * S::P_SLAB + row * 128 + half * 64;
#pragma unroll
        for (int k = 0; k < 4; k++) *reinterpret_cast<float4*>(z + 16 * k) = make_float4(0.f, 0.f, 0.f, 0.f);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        softmax_sync();
        if (issuer) {
          for (long col = nkr; col < pitch; col += 32)
            tma_store_4d(&tmS, smem_u32(smem) + (nkr / 32) * S::P_SLAB, (int)col, q0, h, b);
          bulk_commit();
        }
      }
    }
    if (ok) {
      if (issuer) *sm_ok = mbar_wait(dq_full, 0, flags, 162) ? 1 : 0;
      softmax_sync();
      ok = *sm_ok != 0;
    }
    if (ok) {
      tc_fence_after();
      const bool store = i < T;
      float* orow = dq + ((long)b * T + (store ? i : 0)) * ld_dq + (long)h * HD;
      for (int d0 = half * 32; d0 < HD; d0 += 64) {  // warp-uniform
        float v[32];
        tmem_ld32(trow + kFTmemO + d0, v);
        if (rope && store) {  // rotate back by -theta (pairs (2p, 2p + 1), theta of position i)
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const float2 cs = rope[(long)i * (HD / 2) + (d0 + j) / 2];
            const float g0 = v[j], g1 = v[j + 1];
            v[j] = g0 * cs.x + g1 * cs.y;
            v[j + 1] = -g0 * cs.y + g1 * cs.x;
          }
        }
        if (store) {
#pragma unroll
          for (int g = 0; g < 8; g++)
            *reinterpret_cast<float4*>(orow + d0 + 4 * g) = make_float4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
        }
      }
    }
    if (issuer) bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kFTmemCols) : "memory");
  }
}

template <int HD>
int launch_fused(cudaStream_t st, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                 const CUtensorMap& mp, long pitch, float* out, long ld_out, int B, int T, int H, float scale,
                 int* flags) {
  using S = FShape<HD>;
  static_assert(S::SMEM <= 232448, "fused attention: shared memory budget exceeded");
  auto kfn = k_attn_fwd_fused<HD>;
  static std::atomic<uint64_t> attr{0};
  RC(smem_attr_per_device(attr, kfn, S::SMEM));
  TURT_CHECK_CUDA((launch_pdl(kfn, dim3(B * H, ceil_div(T, kFQ)), dim3(kFThreads), S::SMEM, st, mq, mk, mv, mp, pitch,
                              out, ld_out, T, H, scale, flags)));
  TURT_LAUNCH_CHECK();
  return OK;
}

template <int HD>
int launch_dsoftmax(cudaStream_t st, const CUtensorMap& mo, const CUtensorMap& mv, const CUtensorMap& mp,
                    const CUtensorMap& ms, const CUtensorMap& mk, long pitch, float* dq, long ld_dq,
                    const float2* rope, int B, int T, int H, float scale, int* flags) {
  using Dsh = DShape<HD>;
  static_assert(Dsh::SMEM <= 232448, "fused softmax backward: shared memory budget exceeded");
  auto kfn = k_attn_dsoftmax_fused<HD>;
  static std::atomic<uint64_t> attr{0};
  RC(smem_attr_per_device(attr, kfn, Dsh::SMEM));
  TURT_CHECK_CUDA((launch_pdl(kfn, dim3(B * H, ceil_div(T, kFQ)), dim3(kFThreads), Dsh::SMEM, st, mo, mv, mp, ms, mk,
                              pitch, dq, ld_dq, rope, T, H, scale, flags)));
  TURT_LAUNCH_CHECK();
  return OK;
}

// P / dS view [B*H][T][pitch] as a GemmOperand (rows of `pitch` floats, heads T * pitch apart).
GemmOperand score_operand(const float* base, int T, int H, long pitch) {
  GemmOperand o;
  o.ptr = base;
  o.ld = pitch;
  o.stride = (long)T * pitch;
  o.stride_hi = (long)H * T * pitch;
  return o;
}


// dV = P^T dO and dK = dS^T q for T <= 256 in one kernel: one CTA per (key tile of 128, batch
// entry, head) runs both products over the query slabs from the tile's first key on (the
// causal blocks; P and dS are zero right of the diagonal), two TMEM accumulators, one k-loop:
// per 32-query slab P^T and dS^T arrive as MN-major A tiles and dO, q as MN-major B tiles by
// TMA, the converters split lo parts, and the issuer runs 2 x 3 MMAs per 8 queries.  The
// epilogue writes dV and dK (rotated back by -theta for RoPE) into dqkv.  Replaces the two
// batched per-head GEMMs.
template <int HD>
struct KVShape {
  static constexpr int A_BYTES = 4 * 32 * 32 * 4;        // 128 keys x 32 queries (4 MN boxes)
  static constexpr int B_BYTES = (HD / 32) * 32 * 32 * 4;  // 32 queries x HD
  static constexpr int HI = 2 * A_BYTES + 2 * B_BYTES;      // P^T, dS^T, dO, q
  static constexpr int STAGE = 2 * HI;                      // + lo parts
  static constexpr int STAGES = 2;
  static constexpr int SMEM = STAGES * STAGE + 256 + 1024;
};

template <int HD>
__global__ void __launch_bounds__(320, 1)
    k_attn_dkv_fused(const __grid_constant__ CUtensorMap tmP, const __grid_constant__ CUtensorMap tmS,
                     const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmQ,
                     float* __restrict__ dqkv, long ld, const float2* __restrict__ rope, int T, int H, int* flags) {
  using S = KVShape<HD>;
  constexpr int MN_BOX = 32 * 32 * 4;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::STAGES * S::STAGE);
  uint64_t* full = bars;        // [2]
  uint64_t* conv = bars + 2;    // [2]
  uint64_t* empty = bars + 4;   // [2]
  uint64_t* acc_full = bars + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 7);
  constexpr uint32_t kCols = 256;  // dV at [0, HD), dK at [128, 128 + HD)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // grid (heads, key tiles): the first key tiles (the most query slabs) dispatch first
  const int bh = blockIdx.x, b = bh / H, h = bh % H, E = H * HD;
  const int j0 = blockIdx.y * 128;         // first key of the tile
  const int nsl = (T - j0 + 31) / 32;      // query slabs from query j0 on

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 4);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_fence_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      for (int sl = 0; sl < nsl; sl++) {
        const int s = sl & 1;
        if (sl >= 2 && !mbar_wait(&empty[s], ((sl >> 1) - 1) & 1, flags, 171)) break;
        const uint32_t base = smem_u32(smem + s * S::STAGE);
        const int i0 = j0 + sl * 32;  // first query of the slab
        mbar_arrive_expect_tx(&full[s], S::HI);
        for (int jb = 0; jb < 4; jb++) {
          tma_load_4d(base + jb * MN_BOX, &tmP, j0 + 32 * jb, i0, h, b, &full[s]);
          tma_load_4d(base + S::A_BYTES + jb * MN_BOX, &tmS, j0 + 32 * jb, i0, h, b, &full[s]);
        }
        for (int db = 0; db < HD / 32; db++) {
          tma_load_4d(base + 2 * S::A_BYTES + db * MN_BOX, &tmO, 32 * db, i0, h, b, &full[s]);
          tma_load_4d(base + 2 * S::A_BYTES + S::B_BYTES + db * MN_BOX, &tmQ, 32 * db, i0, h, b, &full[s]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | (1u << 15) | (1u << 16) |
                                 ((uint32_t)(HD >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
      bool ok = true;
      for (int sl = 0; sl < nsl; sl++) {
        const int s = sl & 1;
        if (!mbar_wait(&conv[s], (sl >> 1) & 1, flags, 172)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t base = smem_u32(smem + s * S::STAGE);
        const uint64_t lo = (uint64_t)(S::HI >> 4);
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
          const uint32_t first = (sl > 0 || kk > 0) ? 1u : 0u;
          const uint64_t dp = smem_desc(base + kk * 1024, MN_BOX, 512, kLayoutSW128Atom32);
          const uint64_t ds = smem_desc(base + S::A_BYTES + kk * 1024, MN_BOX, 512, kLayoutSW128Atom32);
          const uint64_t dO = smem_desc(base + 2 * S::A_BYTES + kk * 1024, MN_BOX, 512, kLayoutSW128Atom32);
          const uint64_t dq = smem_desc(base + 2 * S::A_BYTES + S::B_BYTES + kk * 1024, MN_BOX, 512, kLayoutSW128Atom32);
          mma_tf32(tmem, dp + lo, dO, idesc, first);
          mma_tf32(tmem, dp, dO + lo, idesc, 1u);
          mma_tf32(tmem, dp, dO, idesc, 1u);
          mma_tf32(tmem + 128, ds + lo, dq, idesc, first);
          mma_tf32(tmem + 128, ds, dq + lo, idesc, 1u);
          mma_tf32(tmem + 128, ds, dq, idesc, 1u);
        }
        mma_commit(&empty[s]);
      }
      if (ok) mma_commit(acc_full);
    }
  } else if (warp >= 6) {
    const int ct = threadIdx.x - 192;
    for (int sl = 0; sl < nsl; sl++) {
      const int s = sl & 1;
      if (!mbar_wait(&full[s], (sl >> 1) & 1, flags, 173)) break;
      lo_split(smem + s * S::STAGE, S::HI, S::HI, ct);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&conv[s]);
    }
  } else {
    // epilogue: warp w holds keys j0 + 32*(w%4) + lane
    const int q = warp & 3;
    const int j = j0 + q * 32 + lane;
    if (mbar_wait(acc_full, 0, flags, 174)) {
      tc_fence_after();
      const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
      const bool store = j < T;
      float* row = dqkv + ((long)b * T + (store ? j : 0)) * ld;
#pragma unroll 1
      for (int which = 0; which < 2; which++) {  // 0: dV -> [2E, 3E), 1: dK -> [E, 2E)
#pragma unroll 1
        for (int d0 = 0; d0 < HD; d0 += 32) {
          float v[32];
          tmem_ld32(trow + which * 128 + d0, v);
          if (which == 1 && rope && store) {  // rotate back by -theta of key position j
#pragma unroll
            for (int t = 0; t < 32; t += 2) {
              const float2 cs = rope[(long)j * (HD / 2) + (d0 + t) / 2];
              const float g0 = v[t], g1 = v[t + 1];
              v[t] = g0 * cs.x + g1 * cs.y;
              v[t + 1] = -g0 * cs.y + g1 * cs.x;
            }
          }
          if (store) {
            float* dst = row + (which == 0 ? 2 * E : E) + h * HD + d0;
#pragma unroll
            for (int g = 0; g < 8; g++)
              *reinterpret_cast<float4*>(dst + 4 * g) = make_float4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
  }
}

template <int HD>
int launch_dkv(cudaStream_t st, const CUtensorMap& mp, const CUtensorMap& ms, const CUtensorMap& mo,
               const CUtensorMap& mq, float* dqkv, long ld, const float2* rope, int B, int T, int H, int* flags) {
  using Sh = KVShape<HD>;
  static_assert(Sh::SMEM <= 232448, "fused dK/dV: shared memory budget exceeded");
  auto kfn = k_attn_dkv_fused<HD>;
  static std::atomic<uint64_t> attr{0};
  RC(smem_attr_per_device(attr, kfn, Sh::SMEM));
  TURT_CHECK_CUDA((launch_pdl(kfn, dim3(B * H, ceil_div(T, 128)), dim3(320), Sh::SMEM, st, mp, ms, mo, mq, dqkv, ld,
                              rope, T, H, flags)));
  TURT_LAUNCH_CHECK();
  return OK;
}

}  // namespace

int attention_fused_dsoftmax(cudaStream_t st, const GemmOperand& dout, const GemmOperand& v, const GemmOperand& k,
                             const float* P, float* dS, long pitch, float* dq, long ld_dq, const float2* rope, int B,
                             int T, int H, int hd, float scale, int* flags) {
  TURT_REQUIRE(attention_fused_supported(T, hd), "fused attention: needs T <= 256 and a head dim of 32 or 64");
  TURT_REQUIRE(pitch % 4 == 0 && pitch >= T, "fused attention: bad probability row pitch");
  CUtensorMap mo, mv, mp, ms, mk;
  RC(tensor_map_f32(&mo, dout, hd, T, H, B * H, 32, kFQ, false));
  RC(tensor_map_f32(&mv, v, hd, T, H, B * H, 32, 128, false));
  RC(tensor_map_f32(&mp, score_operand(P, T, H, pitch), pitch, T, H, B * H, 32, kFQ, false));
  RC(tensor_map_f32(&ms, score_operand(dS, T, H, pitch), pitch, T, H, B * H, 32, kFQ, false));
  RC(tensor_map_f32(&mk, k, hd, T, H, B * H, 32, 32, true));
  if (hd == 64) return launch_dsoftmax<64>(st, mo, mv, mp, ms, mk, pitch, dq, ld_dq, rope, B, T, H, scale, flags);
  return launch_dsoftmax<32>(st, mo, mv, mp, ms, mk, pitch, dq, ld_dq, rope, B, T, H, scale, flags);
}

int attention_fused_dkv(cudaStream_t st, const float* P, const float* dS, long pitch, const GemmOperand& dout,
                        const GemmOperand& q, float* dqkv, long ld, const float2* rope, int B, int T, int H, int hd,
                        int* flags) {
  TURT_REQUIRE(attention_fused_supported(T, hd), "fused attention: needs T <= 256 and a head dim of 32 or 64");
  TURT_REQUIRE(pitch % 4 == 0 && pitch >= T, "fused attention: bad probability row pitch");
  CUtensorMap mp, ms, mo, mq;
  // P^T / dS^T: MN-major A tiles (keys contiguous within a query row)
  RC(tensor_map_f32(&mp, score_operand(P, T, H, pitch), pitch, T, H, B * H, 32, 32, true));
  RC(tensor_map_f32(&ms, score_operand(dS, T, H, pitch), pitch, T, H, B * H, 32, 32, true));
  RC(tensor_map_f32(&mo, dout, hd, T, H, B * H, 32, 32, true));
  RC(tensor_map_f32(&mq, q, hd, T, H, B * H, 32, 32, true));
  if (hd == 64) return launch_dkv<64>(st, mp, ms, mo, mq, dqkv, ld, rope, B, T, H, flags);
  return launch_dkv<32>(st, mp, ms, mo, mq, dqkv, ld, rope, B, T, H, flags);
}

bool attention_fused_supported(int T, int hd) { return T >= 1 && T <= kFKeys && (hd == 32 || hd == 64); }

int attention_fused_fwd(cudaStream_t st, const GemmOperand& q, const GemmOperand& k, const GemmOperand& v, float* P,
                        long pitch, float* out, long ld_out, int B, int T, int H, int hd, float scale, int* flags) {
  TURT_REQUIRE(attention_fused_supported(T, hd), "fused attention: needs T <= 256 and a head dim of 32 or 64");
  TURT_REQUIRE(pitch % 4 == 0 && pitch >= T, "fused attention: bad probability row pitch");
  CUtensorMap mq, mk, mv, mp;
  RC(tensor_map_f32(&mq, q, hd, T, H, B * H, 32, kFQ, false));
  RC(tensor_map_f32(&mk, k, hd, T, H, B * H, 32, 128, false));
  RC(tensor_map_f32(&mv, v, hd, T, H, B * H, 32, 32, true));
  GemmOperand po;  // P [B*H][T][pitch]: rows of `pitch` floats, heads T * pitch apart
  po.ptr = P;
  po.ld = pitch;
  po.stride = (long)T * pitch;
  po.stride_hi = (long)H * T * pitch;
  RC(tensor_map_f32(&mp, po, pitch, T, H, B * H, 32, kFQ, false));
  if (hd == 64) return launch_fused<64>(st, mq, mk, mv, mp, pitch, out, ld_out, B, T, H, scale, flags);
  return launch_fused<32>(st, mq, mk, mv, mp, pitch, out, ld_out, B, T, H, scale, flags);
}

}  // namespace turt
