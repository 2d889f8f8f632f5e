// ctx.cuh -- the context object behind turt_ctx*.
#pragma once
#include <map>
#include <tuple>
#include <unordered_set>
#include <vector>

#include "common.cuh"

struct turt_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  int* flags = nullptr;  // FLAG_COUNT device ints raised by kernels
  std::unordered_set<void*> live_set;
  std::vector<void*> pending_free;
  int live = 0, peak = 0;
  int precision = 3;  // GEMM_TF32X3 (validated default) or GEMM_TF32
  std::map<std::tuple<int, int, float>, float2*> rope_tables;
  void* scratch = nullptr;  // grow-only device scratch of the standalone fused kernels
  size_t scratch_bytes = 0;
};

namespace turt {
// Reads and clears the device flags; returns the matching status.
int ctx_check_flags(turt_ctx* ctx);
}  // namespace turt
