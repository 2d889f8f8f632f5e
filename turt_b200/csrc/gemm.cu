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

#include <mutex>

#include "gemm.cuh"

namespace turt {

namespace {

constexpr int BM = 128;
constexpr int BK = 32;  // fp32 elements per k-tile = one 128-byte swizzle row
constexpr int A_TILE_BYTES = BM * BK * 4;
constexpr int MN_BOX_BYTES = 32 * BK * 4;  // one 32(MN) x 32(K) box of an MN-major operand

// ------------------------------------------------------------ PTX wrappers
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor (tcgen05 format): start>>4 [0,14), LBO>>4 [16,30),
// SBO>>4 [32,46), version 1 [46,48), layout type [61,64).
// K-major operands use the 128-byte swizzle (type 2: 16-byte chunks XOR row%8, 8-row atoms).
// MN-major tf32 operands must use the 128-byte swizzle with 32-byte atomicity (type 1:
// 32-byte chunks XOR row%4, 4-row atoms); it is the only MN-major layout tf32 accepts.
constexpr uint32_t kLayoutSW128 = 2;
constexpr uint32_t kLayoutSW128Atom32 = 1;
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)layout << 61;
  return d;
}

// Instruction descriptor for kind::tf32: D fp32 [4,6)=1, A tf32 [7,10)=2, B tf32 [10,13)=2,
// A major [15], B major [16], N>>3 [17,23), M>>4 [24,29).
template <int BN, bool A_MN, bool B_MN>
__device__ __forceinline__ uint32_t instr_desc() {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((A_MN ? 1u : 0u) << 15) | ((B_MN ? 1u : 0u) << 16) |
         ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// ------------------------------------------------------------ epilogue
// Applies the epilogue to 32 consecutive accumulator columns [col0, col0+32) of `row`.
__device__ __forceinline__ void store32(float* dst, const float* v, int ncols, bool vec) {
  if (vec && ncols >= 32) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
  } else {
    for (int j = 0; j < ncols && j < 32; j++) dst[j] = v[j];
  }
}

__device__ __forceinline__ void load32(const float* src, float* v, int ncols, bool vec) {
  if (vec && ncols >= 32) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      float4 t = *reinterpret_cast<const float4*>(src + j);
      v[j] = t.x;
      v[j + 1] = t.y;
      v[j + 2] = t.z;
      v[j + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; j++) v[j] = j < ncols ? src[j] : 0.0f;
  }
}

// X3 = error-compensated 3xTF32 (Ootomo & Yokota, 2022): every operand x is split as
// x = hi + lo with hi = x truncated to tf32 (what the tensor core reads from the raw fp32
// bits) and lo = x - hi (exact in fp32); the product is accumulated as
// hi*hi + hi*lo + lo*hi, which keeps ~21 mantissa bits instead of tf32's 10.  The lo
// tiles are produced in shared memory by the (otherwise idle) epilogue warps while the
// mainloop runs, in the same swizzled layout as the TMA-written tiles.
template <int BN, bool A_MN, bool B_MN, int STAGES, bool X3>
__global__ void __launch_bounds__(192, 1)
    k_gemm_tf32(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmEpi epi,
                int M, int N, int K, int ksplits, int kt_per_split, int* flags) {
  constexpr int B_TILE_BYTES = BN * BK * 4;
  constexpr int HI_BYTES = A_TILE_BYTES + B_TILE_BYTES;
  constexpr int STAGE_BYTES = HI_BYTES * (X3 ? 2 : 1);
  constexpr uint32_t TMEM_COLS = BN < 32 ? 32 : BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* conv = full + STAGES;
  uint64_t* empty = conv + STAGES;
  uint64_t* accum_bar = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
  const int batch = blockIdx.z / ksplits, split = blockIdx.z % ksplits;
  const int kt_total = (K + BK - 1) / BK;
  const int kt0 = split * kt_per_split;
  const int kt1 = min(kt_total, kt0 + kt_per_split);
  const int nkt = kt1 - kt0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 4);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum_bar, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && nkt > 0) {
      // ------------------------------------------------ TMA producer
      for (int i = 0; i < nkt; i++) {
        const int s = i % STAGES;
        if (i >= STAGES) {
          if (!mbar_wait(&empty[s], ((i / STAGES) + 1) & 1, flags, 101)) {
            *abort_flag = 1;
            break;
          }
        }
        if (*abort_flag) break;
        const int kc = (kt0 + i) * BK;
        const uint32_t sa = smem_u32(smem + s * STAGE_BYTES);
        const uint32_t sb = sa + A_TILE_BYTES;
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
        const uint32_t bytes = (A_MN ? na * MN_BOX_BYTES : A_TILE_BYTES) + (B_MN ? nb * MN_BOX_BYTES : B_TILE_BYTES);
        mbar_arrive_expect_tx(&full[s], bytes);
        if (!A_MN) {
          tma_load_3d(sa, &tmA, kc, m0, batch, &full[s]);
        } else {
          for (int j = 0; j < BM / 32; j++)
            if (m0 + 32 * j < M) tma_load_3d(sa + j * MN_BOX_BYTES, &tmA, m0 + 32 * j, kc, batch, &full[s]);
        }
        if (!B_MN) {
          tma_load_3d(sb, &tmB, kc, n0, batch, &full[s]);
        } else {
          for (int j = 0; j < BN / 32; j++)
            if (n0 + 32 * j < N) tma_load_3d(sb + j * MN_BOX_BYTES, &tmB, n0 + 32 * j, kc, batch, &full[s]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && nkt > 0) {
      // ------------------------------------------------ MMA issuer
      const uint32_t idesc = instr_desc<BN, A_MN, B_MN>();
      for (int i = 0; i < nkt; i++) {
        const int s = i % STAGES;
        if (!mbar_wait(X3 ? &conv[s] : &full[s], (i / STAGES) & 1, flags, 102)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + s * STAGE_BYTES);
        const uint32_t sb = sa + A_TILE_BYTES;
#pragma unroll
        for (int kk = 0; kk < BK / 8; kk++) {
          // K-major: advance 8 tf32 (32 bytes) inside the 128-byte swizzle row; 8-row atoms 1 KB apart.
          // MN-major: advance 8 K-rows (two 4-row atoms, 1 KB); atoms along K are 512 B apart,
          // 32-element MN column blocks (one TMA box each) 4 KB apart.
          const uint32_t oa = A_MN ? kk * 1024 : kk * 32, ob = B_MN ? kk * 1024 : kk * 32;
          const uint64_t da = A_MN ? smem_desc(sa + oa, MN_BOX_BYTES, 512, kLayoutSW128Atom32)
                                   : smem_desc(sa + oa, 16, 1024, kLayoutSW128);
          const uint64_t db = B_MN ? smem_desc(sb + ob, MN_BOX_BYTES, 512, kLayoutSW128Atom32)
                                   : smem_desc(sb + ob, 16, 1024, kLayoutSW128);
          if (X3) {
            // lo tiles sit HI_BYTES after the hi tiles with the same layout: bump the start address.
            const uint64_t lo = (uint64_t)(HI_BYTES >> 4);
            mma_tf32(tmem, da + lo, db, idesc, (i > 0 || kk > 0) ? 1u : 0u);
            mma_tf32(tmem, da, db + lo, idesc, 1u);
            mma_tf32(tmem, da, db, idesc, 1u);
          } else {
            mma_tf32(tmem, da, db, idesc, (i > 0 || kk > 0) ? 1u : 0u);
          }
        }
        mma_commit(&empty[s]);
      }
      mma_commit(accum_bar);
    }
  } else {
    if (X3) {
      // ------------------------------------------ lo-part converters (warps 2..5)
      const int ct = threadIdx.x - 64;
      for (int i = 0; i < nkt; i++) {
        const int s = i % STAGES;
        if (!mbar_wait(&full[s], (i / STAGES) & 1, flags, 104)) {
          *abort_flag = 1;
          break;
        }
        const float4* hi = reinterpret_cast<const float4*>(smem + s * STAGE_BYTES);
        float4* lo = reinterpret_cast<float4*>(smem + s * STAGE_BYTES + HI_BYTES);
#pragma unroll 4
        for (int e = ct; e < HI_BYTES / 16; e += 128) {
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
    }
    // -------------------------------------------------- epilogue warps
    const bool ok = nkt > 0 && mbar_wait(accum_bar, 0, flags, 103);
    tc_fence_after();
    if (ok && !*abort_flag) {
      const int q = warp & 3;
      const int row = m0 + q * 32 + lane;
      const bool row_ok = row < M;
      float* Cb = epi.C + (long)batch * epi.strideC;
      const bool vecC = (epi.ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(epi.C) & 15) == 0) &&
                        ((epi.strideC % 4) == 0);
      if (epi.kind == EPI_SWIGLU_FWD) {
        // Chunk pairs (gate, up) -> C keeps the pre-activations, C2 gets silu(gate) * up.
        for (int c = 0; c < BN / 32; c += 2) {
          float g[32], u[32];
          tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + c * 32, g);
          tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (c + 1) * 32, u);
          const int col = n0 + c * 32;
          if (row_ok && col < N) {
            float* dst = Cb + (long)row * epi.ldc + col;
            store32(dst, g, N - col, vecC);
            store32(dst + 32, u, N - col - 32, vecC);
            float a[32];
#pragma unroll
            for (int j = 0; j < 32; j++) a[j] = g[j] * sigmoid_f(g[j]) * u[j];
            store32(epi.C2 + (long)row * epi.ldc2 + col / 2, a, (N - col) / 2, vecC && (epi.ldc2 % 4 == 0));
          }
        }
      } else {
        for (int c = 0; c < BN / 32; c++) {
          float v[32];
          tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + c * 32, v);
          const int col = n0 + c * 32;
          if (!row_ok || col >= N) continue;
          const int ncols = min(32, N - col);
          float* dst = Cb + (long)row * epi.ldc + col;
          switch (epi.kind) {
            case EPI_STORE:
              store32(dst, v, ncols, vecC);
              break;
            case EPI_ACCUM: {
              float o[32];
              load32(dst, o, ncols, vecC);
#pragma unroll
              for (int j = 0; j < 32; j++) v[j] += o[j];
              store32(dst, v, ncols, vecC);
            } break;
            case EPI_RED:
              if (vecC && ncols == 32) {
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                  atomicAdd(reinterpret_cast<float4*>(dst + j), make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
              } else {
                for (int j = 0; j < ncols; j++) atomicAdd(dst + j, v[j]);
              }
              break;
            case EPI_ADD_RES: {
              float o[32];
              const bool vecR = vecC && (epi.ldr % 4 == 0) && ((reinterpret_cast<uintptr_t>(epi.R) & 15) == 0);
              load32(epi.R + (long)batch * epi.strideC + (long)row * epi.ldr + col, o, ncols, vecR);
#pragma unroll
              for (int j = 0; j < 32; j++) v[j] += o[j];
              if (epi.bias)
                for (int j = 0; j < ncols; j++) v[j] += epi.bias[col + j];
              store32(dst, v, ncols, vecC);
            } break;
            case EPI_BIAS:
            case EPI_BIAS_GELU: {
              for (int j = 0; j < 32; j++) v[j] += (j < ncols) ? epi.bias[col + j] : 0.0f;
              store32(dst, v, ncols, vecC);
              if (epi.kind == EPI_BIAS_GELU) {
#pragma unroll
                for (int j = 0; j < 32; j++) v[j] = gelu_f(v[j]);
                store32(epi.C2 + (long)row * epi.ldc2 + col, v, ncols, vecC && (epi.ldc2 % 4 == 0));
              }
            } break;
            case EPI_GELU_BWD: {
              float x[32];
              load32(epi.R + (long)row * epi.ldr + col, x, ncols, vecC && (epi.ldr % 4 == 0));
#pragma unroll
              for (int j = 0; j < 32; j++) v[j] *= gelu_grad_f(x[j]);
              store32(dst, v, ncols, vecC);
            } break;
            case EPI_SWIGLU_BWD: {
              // v = d(act) for hidden units [col, col+32); pre-activations and outputs are interleaved.
              const long ic = (long)(col / kGluBlock) * (2 * kGluBlock);
              const float* pg = epi.R + (long)row * epi.ldr + ic;
              float g[32], u[32];
              load32(pg, g, 32, vecC && (epi.ldr % 4 == 0));
              load32(pg + kGluBlock, u, 32, vecC && (epi.ldr % 4 == 0));
              float dg[32], du[32];
#pragma unroll
              for (int j = 0; j < 32; j++) {
                const float s = sigmoid_f(g[j]);
                const float sl = g[j] * s;
                du[j] = v[j] * sl;
                dg[j] = v[j] * u[j] * (s + sl * (1.0f - s));
              }
              float* o = epi.C + (long)row * epi.ldc + ic;
              store32(o, dg, ncols, vecC);
              store32(o + kGluBlock, du, ncols, vecC);
            } break;
            default:
              break;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
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

// 3-D tensor map over a row-major [batch][rows][inner] view with `ld` elements per row.
int make_map(CUtensorMap* map, const float* base, long inner, long rows, long batch, long ld, long bstride,
             int box_inner, int box_rows, bool mn_major) {
  EncodeTiledFn enc = get_encode();
  if (!enc) {
    set_error("cuTensorMapEncodeTiled entry point unavailable");
    return ERR_CUDA;
  }
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)rows, (cuuint64_t)batch};
  long bs = batch > 1 ? bstride : ld * rows;
  if (bs % 4 != 0) bs = ((bs + 3) / 4) * 4;  // unused for batch == 1
  cuuint64_t strides[2] = {(cuuint64_t)ld * 4, (cuuint64_t)bs * 4};
  cuuint32_t box[3] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                   mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (code " + std::to_string((int)r) + ")");
    return ERR_CUDA;
  }
  return OK;
}

template <int BN, bool A_MN, bool B_MN, int STAGES, bool X3>
int launch(cudaStream_t st, const CUtensorMap& ma, const CUtensorMap& mb, const GemmEpi& epi, int M, int N, int K,
           int batch, int ksplits, int kt_per, int* flags) {
  constexpr int smem = STAGES * (A_TILE_BYTES + BN * BK * 4) * (X3 ? 2 : 1) + 1024 + 256;
  static_assert(smem <= 232448, "gemm: shared memory budget exceeded");
  static bool configured = false;
  auto kfn = k_gemm_tf32<BN, A_MN, B_MN, STAGES, X3>;
  if (!configured) {
    TURT_CHECK_CUDA(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured = true;
  }
  dim3 grid(ceil_div(M, BM), ceil_div(N, BN), batch * ksplits);
  kfn<<<grid, 192, smem, st>>>(ma, mb, epi, M, N, K, ksplits, kt_per, flags);
  TURT_LAUNCH_CHECK();
  return OK;
}

template <int BN, int STAGES, bool X3>
int dispatch_major(cudaStream_t st, bool amn, bool bmn, const CUtensorMap& ma, const CUtensorMap& mb,
                   const GemmEpi& epi, int M, int N, int K, int batch, int ks, int kt, int* flags) {
  if (!amn && !bmn) return launch<BN, false, false, STAGES, X3>(st, ma, mb, epi, M, N, K, batch, ks, kt, flags);
  if (!amn && bmn) return launch<BN, false, true, STAGES, X3>(st, ma, mb, epi, M, N, K, batch, ks, kt, flags);
  if (amn && !bmn) return launch<BN, true, false, STAGES, X3>(st, ma, mb, epi, M, N, K, batch, ks, kt, flags);
  return launch<BN, true, true, STAGES, X3>(st, ma, mb, epi, M, N, K, batch, ks, kt, flags);
}

int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

}  // namespace

bool gemm_tf32_supported(const GemmOperand& A, const GemmOperand& B) {
  auto ok = [](const GemmOperand& o) {
    return (reinterpret_cast<uintptr_t>(o.ptr) & 15) == 0 && o.ld % 4 == 0 && o.stride % 4 == 0;
  };
  return ok(A) && ok(B);
}

int gemm_tf32(cudaStream_t stream, int M, int N, int K, int batch, const GemmOperand& A, const GemmOperand& B,
              const GemmEpi& epi_in, int* flags, int precision, int force_splits) {
  TURT_REQUIRE(M > 0 && N > 0 && batch > 0, "gemm: empty problem");
  TURT_REQUIRE(gemm_tf32_supported(A, B), "gemm: operand pitch/base not 16-byte aligned");
  GemmEpi epi = epi_in;
  if (K == 0) {
    set_error("gemm: K == 0");
    return ERR_INVALID;
  }
  // Tile width: the fused gate|up epilogue needs whole (gate, up) chunk pairs.
  int BN = 128;
  if (N <= 64) BN = 64;
  const int tiles = ceil_div(M, BM) * ceil_div(N, BN) * batch;
  const int kt_total = ceil_div(K, BK);
  int ks = 1;
  if (force_splits > 0) {
    ks = force_splits;
  } else if ((epi.kind == EPI_ACCUM || epi.kind == EPI_STORE || epi.kind == EPI_RED) && tiles < num_sms() &&
             kt_total >= 16) {
    ks = num_sms() / tiles;
    if (ks > kt_total / 8) ks = kt_total / 8;
    if (ks < 1) ks = 1;
  }
  int kt_per = ceil_div(kt_total, ks);
  ks = ceil_div(kt_total, kt_per);
  if (ks > 1) {
    if (epi.kind == EPI_STORE) {
      TURT_CHECK_CUDA(cudaMemset2DAsync(epi.C, epi.ldc * 4, 0, (size_t)N * 4, (size_t)M, stream));
      for (int b = 1; b < batch; b++)
        TURT_CHECK_CUDA(
            cudaMemset2DAsync(epi.C + (long)b * epi.strideC, epi.ldc * 4, 0, (size_t)N * 4, (size_t)M, stream));
    }
    TURT_REQUIRE(epi.kind == EPI_STORE || epi.kind == EPI_ACCUM || epi.kind == EPI_RED,
                 "gemm: split-K needs an accumulating epilogue");
    epi.kind = EPI_RED;
  }
  CUtensorMap ma, mb;
  int rc;
  if (!A.mn_major)
    rc = make_map(&ma, A.ptr, K, M, batch, A.ld, A.stride, 32, BM, false);
  else
    rc = make_map(&ma, A.ptr, M, K, batch, A.ld, A.stride, 32, 32, true);
  if (rc) return rc;
  if (!B.mn_major)
    rc = make_map(&mb, B.ptr, K, N, batch, B.ld, B.stride, 32, BN, false);
  else
    rc = make_map(&mb, B.ptr, N, K, batch, B.ld, B.stride, 32, 32, true);
  if (rc) return rc;
  if (precision == GEMM_TF32X3) {
    if (BN == 64)
      return dispatch_major<64, 4, true>(stream, A.mn_major, B.mn_major, ma, mb, epi, M, N, K, batch, ks, kt_per, flags);
    return dispatch_major<128, 3, true>(stream, A.mn_major, B.mn_major, ma, mb, epi, M, N, K, batch, ks, kt_per, flags);
  }
  if (BN == 64)
    return dispatch_major<64, 8, false>(stream, A.mn_major, B.mn_major, ma, mb, epi, M, N, K, batch, ks, kt_per, flags);
  return dispatch_major<128, 6, false>(stream, A.mn_major, B.mn_major, ma, mb, epi, M, N, K, batch, ks, kt_per, flags);
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
