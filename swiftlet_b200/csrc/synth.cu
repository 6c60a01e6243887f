// Device-side synthetic checkpoint generator "swl-synth-v1".
//
// A synthetic checkpoint is a config.json with a "synthetic" block instead of
// weight files. Element i of the tensor named `name` is drawn from
// h = mix64(key + (i + 1) * GAMMA), key = fnv1a64(name) ^ (seed * GAMMA),
// where mix64 is the splitmix64 finaliser (Steele, Lea & Flood, OOPSLA 2014).
// All float arithmetic uses explicitly rounded single operations
// (__fmul_rn / __fadd_rn), so any IEEE host implementation of the same
// definition reproduces the bytes exactly. Packed weights are uniform
// words; scales are bf16(std_w / std_q * (0.75 + u/2)); biases are
// bf16(-mid * scale + 0.1 * std_w * n) with n ~ Irwin-Hall(4) standardised,
// which centres each dequantised group near zero with std ~ std_w.
#include "synth.h"

#include "launch.h"

namespace swl {

namespace {
constexpr uint64_t GAMMA = 0x9E3779B97F4A7C15ull;

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__device__ __forceinline__ uint64_t hash_at(uint64_t key, uint64_t i) { return mix64(key + (i + 1) * GAMMA); }
__device__ __forceinline__ float unif(uint64_t h) { return __fmul_rn(float(h >> 40), 5.9604644775390625e-08f); }
__device__ __forceinline__ float gauss(uint64_t h) {
  const int s = int(h & 0xFFFF) + int((h >> 16) & 0xFFFF) + int((h >> 32) & 0xFFFF) + int((h >> 48) & 0xFFFF);
  return __fmul_rn(float(s - 131070), 2.6429039e-05f);
}
__device__ __forceinline__ uint16_t to_bf16(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) return 0x7FC0;
  u += 0x7FFFu + ((u >> 16) & 1u);
  return uint16_t(u >> 16);
}
__device__ __forceinline__ float from_bf16(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }

// Destination of element i: dense (per_expert == 0) or one section of
// fixed-stride expert blobs.
__device__ __forceinline__ uint8_t* place(uint8_t* base, int64_t i, int64_t per_expert, int64_t stride, int eb) {
  if (per_expert == 0) return base + i * eb;
  return base + (i / per_expert) * stride + (i % per_expert) * eb;
}

__global__ void k_gen_words(uint8_t* dst, uint64_t key, int64_t n, int64_t pe, int64_t stride) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    *reinterpret_cast<uint32_t*>(place(dst, i, pe, stride, 4)) = uint32_t(hash_at(key, i));
}

__global__ void k_gen_affine(uint8_t* ds, uint8_t* db, uint64_t skey, uint64_t bkey, float s0, float mid, float nb,
                             int bf16, int64_t n, int64_t pe, int64_t stride) {
  const int eb = bf16 ? 2 : 4;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const float t = __fadd_rn(__fmul_rn(unif(hash_at(skey, i)), 0.5f), 0.75f);
    const float s = __fmul_rn(t, s0);
    const float sq = bf16 ? from_bf16(to_bf16(s)) : s;
    const float b = __fadd_rn(__fmul_rn(sq, -mid), __fmul_rn(gauss(hash_at(bkey, i)), nb));
    uint8_t* ps = place(ds, i, pe, stride, eb);
    uint8_t* pb = place(db, i, pe, stride, eb);
    if (bf16) {
      *reinterpret_cast<uint16_t*>(ps) = to_bf16(s);
      *reinterpret_cast<uint16_t*>(pb) = to_bf16(b);
    } else {
      *reinterpret_cast<float*>(ps) = s;
      *reinterpret_cast<float*>(pb) = b;
    }
  }
}

// Plain tensors are stored as f32 on the device; `bf16` rounds them through
// the bf16 value the synthetic checkpoint defines.
__global__ void k_gen_plain(float* dst, uint64_t key, int role, float wstd, int bf16, int64_t n) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const uint64_t h = hash_at(key, i);
    float v;
    switch (role) {
      case SYN_NORM: v = __fadd_rn(1.0f, __fmul_rn(gauss(h), 0.05f)); break;
      case SYN_ALOG: v = unif(h); break;
      case SYN_DTBIAS: v = __fmul_rn(gauss(h), 0.5f); break;
      case SYN_CONV: v = __fmul_rn(gauss(h), 0.3f); break;
      default: v = __fmul_rn(gauss(h), wstd);
    }
    dst[i] = bf16 ? from_bf16(to_bf16(v)) : v;
  }
}

int grid_for(int64_t n) { return int(std::min<int64_t>((n + 255) / 256, 65536)); }
}  // namespace

uint64_t synth_key(const std::string& name, uint64_t seed) {
  uint64_t h = 0xcbf29ce484222325ull;
  for (unsigned char c : name) { h ^= c; h *= 0x100000001b3ull; }
  return h ^ (seed * GAMMA);
}

void synth_words(uint8_t* dst, const std::string& name, uint64_t seed, int64_t n, int64_t pe, int64_t stride, cudaStream_t st) {
  if (n <= 0) return;
  launch(k_gen_words, dim3(grid_for(n)), dim3(256), 0, st, false, dst, synth_key(name, seed), n, pe, stride);
}

void synth_affine(uint8_t* ds, uint8_t* db, const std::string& module, uint64_t seed, int bits, float wstd, bool bf16,
                  int64_t n, int64_t pe, int64_t stride, cudaStream_t st) {
  if (n <= 0) return;
  const double qstd = bits == 4 ? 4.6097722286464435 : 73.90027063549903;
  const float s0 = float(double(wstd) / qstd);
  const float mid = bits == 4 ? 7.5f : 127.5f;
  const float nb = float(0.1 * double(wstd));
  launch(k_gen_affine, dim3(grid_for(n)), dim3(256), 0, st, false, ds, db, synth_key(module + ".scales", seed),
         synth_key(module + ".biases", seed), s0, mid, nb, bf16 ? 1 : 0, n, pe, stride);
}

void synth_plain(float* dst, const std::string& name, uint64_t seed, int role, float wstd, bool bf16, int64_t n, cudaStream_t st) {
  if (n <= 0) return;
  launch(k_gen_plain, dim3(grid_for(n)), dim3(256), 0, st, false, dst, synth_key(name, seed), role, wstd, bf16 ? 1 : 0, n);
}

}  // namespace swl
