// Shared definitions of the swiftlet_b200 CUDA runtime (host + device).
#pragma once

#include <cuda_runtime.h>
#ifdef __CUDACC__
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#endif
#include <stdint.h>

#include <stdexcept>
#include <string>

namespace swl {

// Status codes of the C ABI (mirrored in include/swiftlet_cuda.h).
enum Status : int {
  OK = 0,
  ERR_INVALID = -1,
  ERR_IO = -2,
  ERR_FORMAT = -3,
  ERR_CUDA = -4,
  ERR_OOM = -5,
  ERR_UNSUPPORTED = -6,
  ERR_CAPACITY = -7,
};

struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

// Message returned by swl_last_error() on the calling thread.
void set_last_error(const std::string& message);

#define SWL_CUDA(x)                                                                              \
  do {                                                                                           \
    cudaError_t e_ = (x);                                                                        \
    if (e_ != cudaSuccess)                                                                       \
      throw ::swl::Error(e_ == cudaErrorMemoryAllocation ? ::swl::ERR_OOM : ::swl::ERR_CUDA,     \
                         std::string(#x) + ": " + cudaGetErrorString(e_));                       \
  } while (0)

// Element dtypes of weight payloads.
enum DType : int { DT_F32 = 0, DT_BF16 = 1, DT_F16 = 2 };

// One linear module resident in HBM, in the checkpoint's own MLX layout:
// quantised weights are uint32 words packed low-bits-first along the input
// dim with one scale and one bias per `gs` consecutive inputs
// (w = scale * q + bias); plain weights are row-major f32/bf16/f16.
struct QLin {
  const uint8_t* w = nullptr;
  const uint8_t* s = nullptr;
  const uint8_t* b = nullptr;
  int32_t out = 0, in = 0;
  int32_t bits = 0;      // 4 or 8; 0 = plain (unquantised)
  int32_t gs = 0;        // group size (quantised)
  int32_t dt = DT_F32;   // scale/bias dtype (quantised) or weight dtype (plain)
  int32_t pad = 0;
  int64_t row_bytes = 0; // bytes of one weight row
  int64_t srow = 0;      // scale entries per row
};

// A stack of same-shaped expert matrices: expert e lives at w + e*wstride
// (bytes), scales at s + e*sstride, biases at b + e*bstride. Both the
// .qpack fixed-stride blob layout and mlx's stacked switch_mlp tensors are
// expressed this way.
struct ExpertProj {
  QLin lin;
  int64_t wstride = 0, sstride = 0, bstride = 0;
  int count = 0;  // experts in the pool (0: unknown)
};

__host__ __device__ inline int dtype_bytes(int dt) { return dt == DT_F32 ? 4 : 2; }

#ifdef __CUDACC__
__device__ __forceinline__ float bf16_to_f32(uint16_t u) { return __uint_as_float(uint32_t(u) << 16); }
__device__ __forceinline__ float f16_bits_to_f32(uint16_t u) {
  __half_raw r; r.x = u; return __half2float(__half(r));
}
__device__ __forceinline__ float load_scalar(const uint8_t* p, int dt, int64_t i) {
  if (dt == DT_F32) return __ldg(reinterpret_cast<const float*>(p) + i);
  uint16_t u = __ldg(reinterpret_cast<const unsigned short*>(p) + i);
  return dt == DT_BF16 ? bf16_to_f32(u) : f16_bits_to_f32(u);
}
#endif

}  // namespace swl
