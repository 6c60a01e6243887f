// Integer tensor-core weight streaming for 4- and 8-bit MLX-affine weights
// (B = 1 decode): mma.sync m16n8k32 with unsigned 8-bit weight codes (A) and
// signed 8-bit activation digits (B), int32 accumulation per quantisation
// group, then the group's scale and bias in f32.
//
// Activations: per quantisation group g, with inv = 127 / max_g|x| and
// xs = x * inv, three base-254 digits d0 = rint(xs), d1 = rint((xs - d0) *
// 254), d2 = rint(((xs - d0) * 254 - d1) * 254) (each in [-127, 127]) give
// x = (d0 + d1/254 + d2/254^2) / inv to within 0.5 / 254^2 / inv =
// 6.1e-8 * max_g|x|, i.e. f32-level accuracy. Digit n is column n of B (columns 3..7 are zero), so one MMA
// yields sum(q * d_n) for n = 0, 1, 2 of 16 rows at once. A group (>= 32
// weights) fits an int32 exactly (64 * 255 * 127 < 2^24), so it is converted
// once per group: acc_n += scale_g / inv_g * float(D_n). Finally
//   y = acc_0 + (acc_1 + acc_2 / 254) / 254 + sum_g bias_g * sum(x_g).
//
// Fragment mapping (m16n8k32, A row-major, B column-major): lane T holds
// A rows T/4 and T/4 + 8, k-slots 4t..4t+3 (a0/a1) and 16+4t..16+4t+3 (a2/a3)
// with t = T % 4. For 4-bit weights lane t reads word t (8 codes) of the
// 16-byte block: low nibbles (codes 0, 2, 4, 6) go to the first slot set, high
// nibbles (1, 3, 5, 7) to the second; for 8-bit weights words t and 4 + t of
// the 32-byte block. The B table stores each lane's digits in the same k
// order, so the permutation cancels in the dot product.
#pragma once

#include "slice_impl.cuh"

namespace swl {

constexpr int IW = 8;               // consumer warps of the tensor-core kernels
constexpr int IM_NT = IW * 32;      // consumer threads
constexpr int IM_T = IM_NT + 32;    // + one producer warp

// D += A * B on the integer tensor cores (16x8x32, u8 x s8 -> s32).
__device__ __forceinline__ void mma_u8s8(int (&d)[4], const uint32_t (&a)[4], uint2 b) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y));
}

__device__ __forceinline__ int clamp127(float v) { return max(-127, min(127, int(v))); }

// Exact int -> float for |d| < 2^22 on the full-rate pipes: the bits of
// 1.5 * 2^23 + d read as a float are 12582912 + d (one group's MMA sum is at
// most 128 * 255 * 127 < 2^22 in magnitude).
__device__ __forceinline__ float i2f_small(int d) { return __int_as_float(d + 0x4B400000) - 12582912.f; }

// The three digits of xs (|xs| <= 127) packed as signed bytes at byte `pos`.
// Adding 1.5 * 2^23 rounds to an integer (round to nearest even, as rintf)
// whose low byte, read from the float's bits, is the digit's two's-complement
// byte (|digit| <= 127 by construction).
__device__ __forceinline__ void put_digits(float xs, int pos, uint32_t (&b)[3]) {
  constexpr float M = 12582912.f;
  const float a0 = xs + M;
  const float r1 = (xs - (a0 - M)) * 254.f;
  const float a1 = r1 + M;
  const float r2 = (r1 - (a1 - M)) * 254.f;
  const float a2 = r2 + M;
  const int sh = 8 * pos;
  b[0] |= (__float_as_uint(a0) & 0xFFu) << sh;
  b[1] |= (__float_as_uint(a1) & 0xFFu) << sh;
  b[2] |= (__float_as_uint(a2) & 0xFFu) << sh;
}

__device__ __forceinline__ float absmax4(const float4 v) {
  return fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
}
__device__ __forceinline__ bool finite4(const float4 v) {
  return isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w);
}

// Digit scale of a group from its largest magnitude m (infinite when a value
// is not finite): inv = 127 / m; rs = 1 / inv, or NaN so that non-finite
// inputs give non-finite outputs, or 0 for an all-zero group.
__device__ __forceinline__ void digit_scale(float m, float& inv, float& rs) {
  inv = (m > 0.f && m < INFINITY) ? 127.f / m : 0.f;
  rs = inv > 0.f ? 1.f / inv : (m == INFINITY ? __int_as_float(0x7fc00000) : 0.f);
}

// The 8 values of B-table entry (kb, t) in k order of the fragment: 4-bit
// weights pair codes 8t..8t+7 of the block (even codes -> first slot set),
// 8-bit weights words t and 4 + t.
template <int BITS>
__device__ __forceinline__ void entry_values(const float* x, int kb, int t, float (&v)[8]) {
  const float4* p4 = reinterpret_cast<const float4*>(x);
  float4 lo, hi;
  if constexpr (BITS == 4) {
    lo = p4[(32 * kb + 8 * t) >> 2];
    hi = p4[((32 * kb + 8 * t) >> 2) + 1];
  } else {
    lo = p4[(32 * kb + 4 * t) >> 2];
    hi = p4[(32 * kb + 16 + 4 * t) >> 2];
  }
  v[0] = lo.x; v[1] = lo.y; v[2] = lo.z; v[3] = lo.w;
  v[4] = hi.x; v[5] = hi.y; v[6] = hi.z; v[7] = hi.w;
}
template <int BITS>
__device__ __forceinline__ void entry_store(const float (&v)[8], float inv, uint2* slot_t) {
  uint32_t b0[3] = {0u, 0u, 0u}, b1[3] = {0u, 0u, 0u};
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if constexpr (BITS == 4) {
      if (j & 1) put_digits(v[j] * inv, j >> 1, b1);
      else put_digits(v[j] * inv, j >> 1, b0);
    } else {
      if (j < 4) put_digits(v[j] * inv, j, b0);
      else put_digits(v[j] * inv, j - 4, b1);
    }
  }
#pragma unroll
  for (int n = 0; n < 3; ++n) slot_t[4 * n] = make_uint2(b0[n], b1[n]);
}

// Digit staging of `nvec` vectors of n values each (vector v at x + v *
// stride, shared memory) by the consumer threads: quad (g, t) of four
// consecutive threads covers group g (KPG 32-value blocks): its largest
// magnitude and sum (two shuffle rounds), the group's reconstruction scale
// grs[g] and sum gsum[g], and B-table entries (kb, t) of its blocks. The
// vectors' groups, tables and sums are laid out back to back.
template <int BITS, int KPG>
__device__ __forceinline__ void stage_digits(const float* x, int stride, int nvec, int n, uint2* bt, float* gsum,
                                             float* grs) {
  const int tid = threadIdx.x, t = tid & 3;
  const int gpv = n / (32 * KPG), items = nvec * gpv * 4;
  for (int base = 0; base < items; base += IM_NT) {
    const int it = base + tid;
    const bool ok = it < items;
    const int G = ok ? it >> 2 : 0, vec = G / gpv, g = G - vec * gpv;
    const float* xv = x + vec * stride;
    float v[KPG][8];
    float m = 0.f, sum = 0.f;
    bool fin = true;
#pragma unroll
    for (int kk = 0; kk < KPG; ++kk) {
      entry_values<BITS>(xv, g * KPG + kk, t, v[kk]);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        m = fmaxf(m, fabsf(v[kk][j]));
        fin = fin && isfinite(v[kk][j]);
        sum += v[kk][j];
      }
    }
    if (!fin) m = INFINITY;
#pragma unroll
    for (int o = 1; o < 4; o <<= 1) {
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      sum += __shfl_xor_sync(0xffffffffu, sum, o);
    }
    float inv, rs;
    digit_scale(m, inv, rs);
    if (ok) {
      uint2* btv = bt + size_t(vec) * (n >> 5) * 12;
#pragma unroll
      for (int kk = 0; kk < KPG; ++kk) entry_store<BITS>(v[kk], inv, btv + (g * KPG + kk) * 12 + t);
      if (t == 0) {
        gsum[G] = sum;
        grs[G] = rs;
      }
    }
  }
}
// Order-preserving unsigned key of a float (larger float, larger key).
__device__ __forceinline__ unsigned f_key(float f) {
  const unsigned u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_f(unsigned k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Routing by one warp from the router's E + 1 logits (E <= 512, K <= 32):
// softmax weights over E, top-K, combine weights renormalised when norm_topk,
// and sigmoid of the shared-expert gate logit (QwenCPUModel.swift:506-521,
// 546-550; routerPicks QwenMetalModel.swift:875-892). The top-K is taken on
// the logits, whose order the softmax preserves, with ties to the lower
// expert id (the reference's insertion scan with a strict `>`): each round is
// one warp max of order-preserving keys and one warp min over the ids that
// hold it. Lane l holds experts l, l + 32, ... and keeps its own three best
// (key, slot) pairs, so a round costs the winning lane a shift; only a lane
// picked a third time rescans its unpicked slots. Only the K picked
// probabilities are divided out. ids / w / sh are shared memory.
template <int PL>
__device__ __forceinline__ void warp_route_pl(const float* lg, int E, int K, int norm_topk, int* ids, float* w,
                                              float* sh) {
  const int lane = threadIdx.x & 31;
  float lv[PL];
  unsigned key[PL];
#pragma unroll
  for (int i = 0; i < PL; ++i) {
    const int e = i * 32 + lane;
    lv[i] = e < E ? __ldcg(lg + e) : 0.f;
    key[i] = e < E ? f_key(lv[i]) : 0u;
  }
  const float shared_logit = __ldcg(lg + E);
  // this lane's three best (ascending slots and a strict `>`: the lower
  // expert id first among equal keys); slot PL = none
  unsigned k1 = 0u, k2 = 0u, k3 = 0u;
  int s1 = PL, s2 = PL, s3 = PL;
  unsigned picked = 0u;
  auto best3 = [&]() {
    k1 = k2 = k3 = 0u;
    s1 = s2 = s3 = PL;
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      const unsigned kk = (picked >> i) & 1u ? 0u : key[i];
      if (kk > k1) { k3 = k2; s3 = s2; k2 = k1; s2 = s1; k1 = kk; s1 = i; }
      else if (kk > k2) { k3 = k2; s3 = s2; k2 = kk; s2 = i; }
      else if (kk > k3) { k3 = kk; s3 = i; }
    }
  };
  best3();
  float mine = 0.f;  // lane k: the logit of pick k
  float top = 0.f;   // the largest logit (softmax shift)
  for (int k = 0; k < K; ++k) {
    const unsigned mx = __reduce_max_sync(0xffffffffu, k1);
    const unsigned bi = k1 ? unsigned(s1 * 32 + lane) : 0x7fffffffu;
    int id = int(__reduce_min_sync(0xffffffffu, k1 == mx ? bi : 0x7fffffffu));
    if (mx && (id & 31) == lane) {
      picked |= 1u << s1;
      k1 = k2; s1 = s2; k2 = k3; s2 = s3; k3 = 0u; s3 = PL;
      if (!k1) best3();  // all three consumed: rescan the unpicked slots
    }
    if (id >= E) id = 0;  // fewer valid logits than K: keep indices in range
    const float val = key_f(mx);
    if (k == 0) top = val;
    if (lane == k) mine = val;
    if (lane == 0) ids[k] = id;
  }
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < PL; ++i)
    if (i * 32 + lane < E) sum += expf(lv[i] - top);
  sum = warp_sum(sum);
  const float p = lane < K ? expf(mine - top) / sum : 0.f;
  // renormalisation: the picks' sum in pick order (as the reference adds
  // them), gathered by shuffles rather than through shared memory
  float score_sum = 0.f;
  for (int k = 0; k < K; ++k) score_sum += __shfl_sync(0xffffffffu, p, k);
  if (lane < K) w[lane] = norm_topk ? p / score_sum : p;
  if (lane == 0) *sh = sigmoid_ref(shared_logit);
  __syncwarp();
}
__device__ __forceinline__ void warp_route(const float* lg, int E, int K, int norm_topk, int* ids, float* w,
                                           float* sh) {
  if (E <= 256) warp_route_pl<8>(lg, E, K, norm_topk, ids, w, sh);
  else warp_route_pl<16>(lg, E, K, norm_topk, ids, w, sh);
}

// Four consecutive scale (or bias) entries g..g+3 of a row in shared memory
// (g % 4 == 0; the row is 8-byte aligned for 16-bit and 16-byte aligned for
// f32 entries).
template <int DT>
__device__ __forceinline__ float4 sm_scalar4(const uint8_t* p, int g) {
  if constexpr (DT == DT_F32) {
    return *reinterpret_cast<const float4*>(p + 4 * g);
  } else {
    const uint2 u = *reinterpret_cast<const uint2*>(p + 2 * g);
    if constexpr (DT == DT_BF16)
      return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u), __uint_as_float(u.y << 16),
                         __uint_as_float(u.y & 0xFFFF0000u));
    else
      return make_float4(f16_bits_to_f32(uint16_t(u.x & 0xFFFF)), f16_bits_to_f32(uint16_t(u.x >> 16)),
                         f16_bits_to_f32(uint16_t(u.y & 0xFFFF)), f16_bits_to_f32(uint16_t(u.y >> 16)));
  }
}
__device__ __forceinline__ float f4_at(const float4 v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }

// Weight tiles arrive by tensor TMA with the 128-byte swizzle, laid out
// [row segment of 128 bytes][row][128 bytes] (segb = rows per box * 128 bytes
// per segment) with 16-byte chunk c of row r stored at chunk c ^ (r & 7): the
// 8 rows a warp reads at once then fall on distinct shared-memory banks.
__device__ __forceinline__ int swz_off(int k16, int rx, int segb) {
  return (k16 >> 3) * segb + (((k16 & 7) << 4) ^ rx);
}

// One 16-row tile against staged digits over quantisation groups
// [g_begin, g_end) ((g_end - g_begin) % 4 == 0, KPG 32-weight blocks per
// group): rows r0 (of the box at W0) and r1 (of the box at W1), with
// r0 & 7 == r1 & 7, held by lane quad T/4; their scale / bias rows start at
// s0, s1 / b0, b1. Four groups run per step with independent accumulators
// (all their fragment loads issued first), so the MMA chains overlap. Lane
// t == 0 of each quad returns the two rows' partial results (others return
// garbage); partials over disjoint group ranges add up to the full result.
template <int BITS, int DT, int KPG>
__device__ __forceinline__ void imma_rows(const uint8_t* W0, const uint8_t* W1, int r0, int r1, int segb,
                                          const uint8_t* s0, const uint8_t* s1, const uint8_t* b0, const uint8_t* b1,
                                          const uint2* bt, const float* gsum, const float* grs, int g_begin,
                                          int g_end, float& y0, float& y1) {
  constexpr int NB = 4 * KPG;                        // 32-weight blocks per step
  constexpr int CPB = BITS == 4 ? 1 : 2;              // 16-byte chunks per block
  constexpr bool ALIGNED = (NB * CPB) % 8 == 0;       // every step starts on a 128-byte segment
  const int lane = threadIdx.x & 31, t = lane & 3, rx = (r0 & 7) << 4;
  const uint8_t* p0 = W0 + r0 * 128 + 4 * t;
  const uint8_t* p1 = W1 + r1 * 128 + 4 * t;
  int xo[8];  // swizzled offset of chunk c inside a segment (lane constant)
#pragma unroll
  for (int c = 0; c < 8; ++c) xo[c] = (c << 4) ^ rx;
  const bool blane = lane < 12;
  float f[4] = {0.f, 0.f, 0.f, 0.f};
  float ba0 = 0.f, ba1 = 0.f;
  for (int g = g_begin; g < g_end; g += 4) {
    const int kb0 = g * KPG;
    const int sbase = ((kb0 * CPB) >> 3) * segb;  // segment of the step's first chunk
    uint2 b[NB];
    uint32_t u0[NB], u1[NB], v0[NB], v1[NB];
#pragma unroll
    for (int j = 0; j < NB; ++j) {
      const int kb = kb0 + j;
      b[j] = blane ? bt[kb * 12 + lane] : make_uint2(0u, 0u);
#pragma unroll
      for (int h = 0; h < CPB; ++h) {
        // chunk CPB * kb + h; with aligned steps its segment and slot are
        // compile-time offsets from the step's first segment
        const int o = ALIGNED ? sbase + ((CPB * j + h) >> 3) * segb + xo[(CPB * j + h) & 7]
                              : swz_off(CPB * kb + h, rx, segb);
        const uint32_t w0 = *reinterpret_cast<const uint32_t*>(p0 + o);
        const uint32_t w1 = *reinterpret_cast<const uint32_t*>(p1 + o);
        if (h == 0) { u0[j] = w0; u1[j] = w1; }
        else { v0[j] = w0; v1[j] = w1; }
      }
    }
    int d[4][4];
#pragma unroll
    for (int q = 0; q < 4; ++q) d[q][0] = d[q][1] = d[q][2] = d[q][3] = 0;
#pragma unroll
    for (int kk = 0; kk < KPG; ++kk)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int j = q * KPG + kk;
        uint32_t a[4];
        if constexpr (BITS == 4) {
          a[0] = u0[j] & 0x0F0F0F0Fu;
          a[2] = (u0[j] >> 4) & 0x0F0F0F0Fu;
          a[1] = u1[j] & 0x0F0F0F0Fu;
          a[3] = (u1[j] >> 4) & 0x0F0F0F0Fu;
        } else {
          a[0] = u0[j];
          a[2] = v0[j];
          a[1] = u1[j];
          a[3] = v1[j];
        }
        mma_u8s8(d[q], a, b[j]);
      }
    const float4 sc0 = sm_scalar4<DT>(s0, g), sc1 = sm_scalar4<DT>(s1, g);
    const float4 bb0 = sm_scalar4<DT>(b0, g), bb1 = sm_scalar4<DT>(b1, g);
    const float4 xg = *reinterpret_cast<const float4*>(gsum + g);
    const float4 rg = *reinterpret_cast<const float4*>(grs + g);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float c0 = f4_at(sc0, q) * f4_at(rg, q), c1 = f4_at(sc1, q) * f4_at(rg, q);
      f[0] = fmaf(c0, i2f_small(d[q][0]), f[0]);
      f[1] = fmaf(c0, i2f_small(d[q][1]), f[1]);
      f[2] = fmaf(c1, i2f_small(d[q][2]), f[2]);
      f[3] = fmaf(c1, i2f_small(d[q][3]), f[3]);
      ba0 = fmaf(f4_at(bb0, q), f4_at(xg, q), ba0);
      ba1 = fmaf(f4_at(bb1, q), f4_at(xg, q), ba1);
    }
  }
  // lane t == 1 holds digit 2 (column 2) of the same rows
  const float e0 = __shfl_down_sync(0xffffffffu, f[0], 1);
  const float e1 = __shfl_down_sync(0xffffffffu, f[2], 1);
  y0 = (f[0] + (f[1] + e0 * (1.f / 254.f)) * (1.f / 254.f)) + ba0;
  y1 = (f[2] + (f[3] + e1 * (1.f / 254.f)) * (1.f / 254.f)) + ba1;
}

// Tensor maps of the matrices a launch streams (see TileMaps in slice.h).
__device__ __forceinline__ void tma_rows(uint8_t* dst, const CUtensorMap* m, int row, int expert, uint64_t* bar,
                                         uint64_t pol) {
  if (expert < 0)
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
        "l"(m), "r"(0), "r"(row), "r"(0), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
  else
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(dst)),
        "l"(m), "r"(0), "r"(row), "r"(0), "r"(expert), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}
// One matrix block of a slot: [box rows of weights, swizzled][box scale rows]
// [box bias rows]. The weights box is always copied whole (rows past the
// matrix end read as zeros); scales and biases for the n rows in use.
__device__ __forceinline__ unsigned tile_bytes(const SliceTab& T, int sb, int box, int n) {
  return unsigned(box * T.rb) + 2u * unsigned(n * T.srow * sb);
}
__device__ __forceinline__ void tile_copy(const SliceTab& T, int sb, int box, uint8_t* d, uint64_t* bar,
                                          const CUtensorMap* m, int expert, const uint8_t* s, const uint8_t* b,
                                          int row, int n, uint64_t pol) {
  const int ss = T.srow * sb;
  tma_rows(d, m, row, expert, bar, pol);
  bulk_g2s(d + box * T.rb, s + int64_t(row) * ss, unsigned(n * ss), bar, pol);
  bulk_g2s(d + box * T.rb + box * ss, b + int64_t(row) * ss, unsigned(n * ss), bar, pol);
}

__device__ __forceinline__ void imma_init_barriers(uint64_t* full, uint64_t* empty, int S) {
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, 1);  // one consumer warp per tile
    }
    mbar_init_fence();
  }
  __syncthreads();
}

// Tiles are reduced by groups of KS = T.W consumer warps (KS in {1, 2, 4, 8}):
// tile i goes to warp group i % (IW / KS), whose warp kw covers the
// quantisation groups [kw * ng / KS, (kw + 1) * ng / KS). With KS > 1 the
// partials meet in `kp` (two buffers of IW * 16 floats, alternating per
// round so that the next round's writes cannot overtake the reads), behind
// named barrier 2 + group.
struct KSplit {
  int ks, ng_warps, grp, kw;
  __device__ __forceinline__ KSplit(int ks_, int warp) : ks(ks_), ng_warps(IW / ks_), grp(warp / ks_), kw(warp % ks_) {}
  __device__ __forceinline__ bool mine(int tile) const { return tile % ng_warps == grp; }
  __device__ __forceinline__ int round(int tile) const { return tile / ng_warps; }
  __device__ __forceinline__ void range(int ngroups, int& g0, int& g1) const {
    g0 = kw * ngroups / ks;
    g1 = (kw + 1) * ngroups / ks;
  }
  // Sums the KS partials of rows gi / gi + 8 into warp kw == 0 (t == 0 lanes).
  __device__ __forceinline__ void combine(float* kp, int rnd, int gi, int t, float& y0, float& y1) const {
    if (ks == 1) return;
    float* buf = kp + (rnd & 1) * IW * 16;
    const int warp = threadIdx.x >> 5;
    if (t == 0) { buf[warp * 16 + gi] = y0; buf[warp * 16 + gi + 8] = y1; }
    asm volatile("bar.sync %0, %1;" ::"r"(2 + grp), "r"(ks * 32) : "memory");
    if (kw == 0 && t == 0) {
      y0 = 0.f;
      y1 = 0.f;
      for (int q = 0; q < ks; ++q) {
        y0 += buf[(grp * ks + q) * 16 + gi];
        y1 += buf[(grp * ks + q) * 16 + gi + 8];
      }
    }
  }
};

// ------------------------------------------------------------ dense GEMV --
// As k_sgemv (same tiles of 16 rows, producer, prologues and epilogues); tile
// i is reduced by consumer warp i % IW on the tensor cores.
template <int BITS, int DT, int KPG>
__global__ void __launch_bounds__(IM_T, 2) k_igemv(const GemvArgs a, const SliceTab T, const __grid_constant__ TileMaps M,
                                                 const RouterTail rt) {
  constexpr int SB = DT == DT_F32 ? 4 : 2;
  extern __shared__ __align__(1024) uint8_t sm_raw[];
  // the swizzled tensor copies need 1024-byte aligned slots
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = sm;
  float* plain = reinterpret_cast<float*>(sm + T.off_raw);
  float* red = reinterpret_cast<float*>(sm + T.off_red);
  float* gsum = reinterpret_cast<float*>(sm + T.off_cs);
  uint2* bt = reinterpret_cast<uint2*>(sm + T.off_xs);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + T.off_bar);
  uint64_t* empty = full + T.S;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r0 = blockIdx.x * T.rpc, r1 = min(T.total, r0 + T.rpc);
  const int ss = T.srow * SB, segb = 16 * 128;
  auto tiles = [&](auto&& f) {
    int idx = 0;
    for (int sg = 0; sg < T.nseg; ++sg) {
      const int a0 = max(r0, T.cum[sg]), a1 = min(r1, T.cum[sg + 1]);
      for (int r = a0; r < a1; r += 16) f(idx++, sg, r - T.cum[sg], min(16, a1 - r));
    }
  };
  imma_init_barriers(full, empty, T.S);
  if (warp == IW) {  // producer
    if (lane == 0) {
      const uint64_t pol = l2_evict_first();
      int issued = 0;
      bool ok = true;
      tiles([&](int i, int sg, int row, int n) {
        if (!ok) return;
        const int s = i % T.S;
        if (i >= T.S && !mbar_wait(empty + s, unsigned(i / T.S - 1) & 1u)) { ok = false; return; }
        mbar_expect_tx(full + s, tile_bytes(T, SB, 16, n));
        tile_copy(T, SB, 16, ring + size_t(s) * T.slot, full + s, &M.m[sg], -1, seg_pick(T.s, sg), seg_pick(T.b, sg),
                  row, n, pol);
        issued = i + 1;
      });
      if (!ok) sl_fail(T);
      pdl_launch();
      sl_drain(full, T.S, issued);
    }
    return;
  }
  TraceRec trc;
  trc.start(a.trace);
  pdl_wait();
  trc.waited(a.trace);
  sl_stage_plain<IM_NT>(a, red, plain);
  const int ngroups = a.in >> T.gs_shift, gi = lane >> 2, t = lane & 3;
  float* grs = gsum + ((ngroups + 3) & ~3);
  stage_digits<BITS, KPG>(plain, 0, 1, a.in, bt, gsum, grs);
  bar_sync_n(IM_NT);
  pdl_launch();
  trc.staged(a.trace);
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  auto epi = [&](int sg, int row, float v) {
    float* y = seg_pick(T.y, sg);
    if (a.epilogue == EPI_RESIDUAL) y[row] += v;
    else y[row] = v;
    if (sg == 0 && (v > bv || (v == bv && row < bi))) { bv = v; bi = row; }
  };
  const KSplit ksp(T.W, warp);
  float* kp = reinterpret_cast<float*>(sm + T.off_part);
  int g0, g1;
  ksp.range(ngroups, g0, g1);
  bool dead = false;
  // A warp whose bounded wait gave up keeps taking part in its group's
  // combine barriers (with zeros), so no partner waits on it forever.
  tiles([&](int i, int sg, int row, int n) {
    if (!ksp.mine(i)) return;
    const int s = i % T.S;
    const bool ok = !dead && __all_sync(0xffffffffu, mbar_wait(full + s, unsigned(i / T.S) & 1u));
    dead = !ok;
    float y0 = 0.f, y1 = 0.f;
    if (ok) {
      const uint8_t* wt = ring + size_t(s) * T.slot;
      const uint8_t* st = wt + 16 * T.rb;
      const uint8_t* btt = st + 16 * ss;
      imma_rows<BITS, DT, KPG>(wt, wt, gi, gi + 8, segb, st + gi * ss, st + (gi + 8) * ss, btt + gi * ss,
                               btt + (gi + 8) * ss, bt, gsum, grs, g0, g1, y0, y1);
    }
    ksp.combine(kp, ksp.round(i), gi, t, y0, y1);
    __syncwarp();
    if (ksp.kw == 0 && ok) {
      if (lane == 0) mbar_arrive(empty + s);
      if (t == 0) {
        if (gi < n) epi(sg, row + gi, y0);
        if (gi + 8 < n) epi(sg, row + gi + 8, y1);
      }
    }
  });
  trc.looped(a.trace);
  if (dead) sl_fail(T);
  if (a.argmax_out) sl_argmax_tail<IM_NT>(a, bv, bi, red);
  if (rt.logits) sl_router_done<IM_NT>(rt, plain, red);
  trc.end(a.trace);
}

// ---------------------------------------------------------------- MoE ----
// Gate/up of the shared and routed experts with SiLU * up fused. CTA b owns
// one item of up to BR = T.TR rows of one gate/up pair: items [0, nsh) cover
// the shared expert's rows, item nsh + q routed expert slot k = q / ipe, rows
// ((q % ipe) * BR, ...) (ipe items per expert). An item's gate rows and its up
// rows arrive as one tensor-TMA box each plus their scale and bias rows, so a
// CTA issues six copies: the shared items at kernel entry, the routed ones as
// soon as the producer warp has routed from the router's logits (while the
// consumers stage the input). The 16-row MMA tile is 8 gate rows over the
// same 8 up rows, so the lane holding gate row p also holds up row p; the
// item's BR / 8 tiles are split over warp groups as in the dense kernel.
template <int BITS, int DT, int KPG>
__global__ void __launch_bounds__(IM_T, 2) k_igateup(const MoeArgs m, const SliceTab T,
                                                   const __grid_constant__ TileMaps M) {
  constexpr int SB = DT == DT_F32 ? 4 : 2;
  extern __shared__ __align__(1024) uint8_t sm_raw[];
  // the swizzled tensor copies need 1024-byte aligned slots
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = sm;
  float* plain = reinterpret_cast<float*>(sm + T.off_raw);
  float* red = reinterpret_cast<float*>(sm + T.off_red);
  float* gsum = reinterpret_cast<float*>(sm + T.off_cs);
  uint2* bt = reinterpret_cast<uint2*>(sm + T.off_xs);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + T.off_bar);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = m.topk, inter = m.g.lin.out, sh = m.sg.out, BR = T.TR;
  const int nsh = (sh + BR - 1) / BR, ipe = (inter + BR - 1) / BR, b = blockIdx.x;
  const bool shared_item = b < nsh;
  const int k = shared_item ? K : (b - nsh) / ipe;
  const int row0 = shared_item ? b * BR : (b - nsh - k * ipe) * BR;
  const int n = min(BR, (shared_item ? sh : inter) - row0);
  const int ss = T.srow * SB, half = T.slot / 2, segb = BR * 128;
  const bool route_here = !shared_item && m.logits != nullptr;
  __shared__ int r_ids[16];
  __shared__ float r_w[16], r_sh;
  if (tid == 0) {
    mbar_init(full, 1);
    mbar_init_fence();
  }
  __syncthreads();
  if (warp == IW) {  // producer
    if (route_here) {
      // the routing comes from the previous (router) grid; the consumers
      // stage the input meanwhile and never need it (the item's slot k is
      // known), so it costs only the copies' start
      pdl_wait();
      warp_route(m.logits, m.experts, K, m.norm_topk, r_ids, r_w, &r_sh);
      // the first routed item also stores the routing for observers
      if (b == nsh) {
        if (lane < K) {
          m.pick_ids[lane] = r_ids[lane];
          m.pick_w[lane] = r_w[lane];
        }
        if (lane == 0) *m.shared_scale = r_sh;
      }
    }
    if (lane == 0) {
      const uint64_t pol = l2_evict_first();
      bool issued = false;
      auto issue = [&](int id) {
        QLin G = m.sg, U = m.su;
        if (!shared_item) {
          G = expert_lin(m.g, id);
          U = expert_lin(m.u, id);
        }
        mbar_expect_tx(full, 2u * tile_bytes(T, SB, BR, n));
        tile_copy(T, SB, BR, ring, full, &M.m[shared_item ? 0 : 2], shared_item ? -1 : id, G.s, G.b, row0, n, pol);
        tile_copy(T, SB, BR, ring + half, full, &M.m[shared_item ? 1 : 3], shared_item ? -1 : id, U.s, U.b, row0, n,
                  pol);
        issued = true;
      };
      // the shared expert's weights do not depend on the routing
      if (shared_item) issue(0);
      pdl_wait();  // the routing comes from the previous (router) grid
      if (!shared_item) issue(route_here ? r_ids[k] : __ldcg(m.pick_ids + k));
      // Dependents are released only after the router grid is complete: the
      // down kernel reads the router's output before its own dependency wait.
      pdl_launch();
      sl_drain(full, 1, issued ? 1 : 0);
    }
    return;
  }
  TraceRec trc;
  trc.start(m.trace);
  pdl_wait();
  trc.waited(m.trace);
  GemvArgs a;
  a.in = m.g.lin.in; a.prologue = PRO_COPY; a.x = m.x;
  sl_stage_plain<IM_NT>(a, red, plain);
  const int ngroups = a.in >> T.gs_shift, gi = lane >> 2, t = lane & 3;
  float* grs = gsum + ((ngroups + 3) & ~3);
  stage_digits<BITS, KPG>(plain, 0, 1, a.in, bt, gsum, grs);
  bar_sync_n(IM_NT);
  pdl_launch();
  trc.staged(m.trace);
  const KSplit ksp(T.W, warp);
  float* kp = reinterpret_cast<float*>(sm + T.off_part);
  int g0, g1;
  ksp.range(ngroups, g0, g1);
  const int so = BR * T.rb, bo = BR * T.rb + BR * ss;  // scale and bias rows after each weight box
  bool dead = false;
  for (int j = 0; j < (n + 7) / 8; ++j) {
    if (!ksp.mine(j)) continue;
    const bool ok = !dead && __all_sync(0xffffffffu, mbar_wait(full, 0u));
    dead = !ok;
    float gv = 0.f, uv = 0.f;
    const int r = 8 * j + gi;
    if (ok) {
      const uint8_t* gt = ring;
      const uint8_t* ut = ring + half;
      imma_rows<BITS, DT, KPG>(gt, ut, r, r, segb, gt + so + r * ss, ut + so + r * ss, gt + bo + r * ss,
                               ut + bo + r * ss, bt, gsum, grs, g0, g1, gv, uv);
    }
    ksp.combine(kp, ksp.round(j), gi, t, gv, uv);
    __syncwarp();
    if (ksp.kw == 0 && ok && t == 0 && r < n) m.hmid[k * m.hmid_stride + row0 + r] = silu_ref(gv) * uv;
  }
  trc.looped(m.trace);
  if (dead) sl_fail(T);
  trc.end(m.trace);
}

// Down projections, combine and residual (as k_sdown): tile e holds expert
// slot e's rows of the CTA (at most 16); warp e % IW stages that slot's
// digits and reduces the tile into part[e][row]; the consumers then combine
// part over the experts with the routing weights.
template <int BITS, int DT, int KPG>
__global__ void __launch_bounds__(IM_T, 2) k_idown(const MoeArgs m, const SliceTab T,
                                                 const __grid_constant__ TileMaps M) {
  constexpr int SB = DT == DT_F32 ? 4 : 2;
  extern __shared__ __align__(1024) uint8_t sm_raw[];
  // the swizzled tensor copies need 1024-byte aligned slots
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = sm;
  float* raw = reinterpret_cast<float*>(sm + T.off_raw);
  float* part = reinterpret_cast<float*>(sm + T.off_part);
  float* gsum = reinterpret_cast<float*>(sm + T.off_cs);
  uint2* bt = reinterpret_cast<uint2*>(sm + T.off_xs);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + T.off_bar);
  uint64_t* empty = full + T.S;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = m.topk, D = m.d.lin.out, inter = m.d.lin.in;
  const int o0 = int(blockIdx.x) * T.rpc, o1 = min(D, o0 + T.rpc), nrow = o1 - o0;
  const int ss = T.srow * SB, segb = 16 * 128;
  __shared__ int r_ids[16];
  __shared__ float r_w[16], r_sh;
  imma_init_barriers(full, empty, T.S);
  if (warp == IW) {  // producer
    // The router grid completed before this grid was launched, so its output
    // (logits, or the routing it stored) can be read before the dependency wait.
    if (m.logits) warp_route(m.logits, m.experts, K, m.norm_topk, r_ids, r_w, &r_sh);
    if (lane == 0) {
      const uint64_t pol = l2_evict_first();
      int issued = 0;
      bool ok = true;
      for (int e = 0; e <= K && ok; ++e) {
        const int s = e % T.S;
        if (e >= T.S && !mbar_wait(empty + s, unsigned(e / T.S - 1) & 1u)) { ok = false; break; }
        const int id = e < K ? (m.logits ? r_ids[e] : __ldcg(m.pick_ids + e)) : -1;
        const QLin L = e < K ? expert_lin(m.d, id) : m.sd;
        mbar_expect_tx(full + s, tile_bytes(T, SB, 16, nrow));
        tile_copy(T, SB, 16, ring + size_t(s) * T.slot, full + s, &M.m[e < K ? 2 : 0], id, L.s, L.b, o0, nrow, pol);
        issued = e + 1;
      }
      if (!ok) sl_fail(T);
      pdl_launch();
      sl_drain(full, T.S, issued);
    }
    return;
  }
  TraceRec trc;
  trc.start(m.trace);
  pdl_wait();
  trc.waited(m.trace);
  const int nfl = (K + 1) * m.hmid_stride;
  for (int i = tid; i < (nfl >> 2); i += IM_NT) cp_async16(raw + 4 * i, m.hmid + 4 * i);
  cp_async_wait_all();
  bar_sync_n(IM_NT);
  const int nkb = inter >> 5, ngroups = inter >> T.gs_shift;
  float* grs = gsum + (((K + 1) * ngroups + 3) & ~3);
  stage_digits<BITS, KPG>(raw, m.hmid_stride, K + 1, inter, bt, gsum, grs);
  bar_sync_n(IM_NT);
  pdl_launch();
  trc.staged(m.trace);
  const int gi = lane >> 2, t = lane & 3;
  bool dead = false;
  for (int e = warp; e <= K && !dead; e += IW) {
    const int s = e % T.S;
    if (!__all_sync(0xffffffffu, mbar_wait(full + s, unsigned(e / T.S) & 1u))) { dead = true; break; }
    const uint8_t* dt = ring + size_t(s) * T.slot;
    const uint8_t* st = dt + 16 * T.rb;
    const uint8_t* btt = st + 16 * ss;
    float y0, y1;
    imma_rows<BITS, DT, KPG>(dt, dt, gi, gi + 8, segb, st + gi * ss, st + (gi + 8) * ss, btt + gi * ss,
                             btt + (gi + 8) * ss, bt + e * nkb * 12, gsum + e * ngroups, grs + e * ngroups, 0, ngroups,
                             y0, y1);
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + s);
    if (t == 0) {
      if (gi < nrow) part[e * T.rpc + gi] = y0;
      if (gi + 8 < nrow) part[e * T.rpc + gi + 8] = y1;
    }
  }
  trc.looped(m.trace);
  if (dead) sl_fail(T);
  bar_sync_n(IM_NT);
  // combine weights: computed by this CTA's producer (released to the
  // consumers by the arrivals that completed the tiles' barriers) or stored
  // by the router grid
  for (int rl = tid; rl < nrow; rl += IM_NT) {
    float acc = 0.f;
    for (int e = 0; e <= K; ++e) {
      const float we = m.logits ? (e < K ? r_w[e] : r_sh) : (e < K ? __ldcg(m.pick_w + e) : __ldcg(m.shared_scale));
      acc = fmaf(we, part[e * T.rpc + rl], acc);
    }
    m.h[o0 + rl] += acc;
  }
  if (m.advance_sd && blockIdx.x == 0 && tid == 0) {
    // Advance the sequence position and the token cursor once the last
    // layer of the step is done (no other CTA of this grid reads them;
    // dependents read them only after this grid completes).
    *m.advance_sd->pos += 1;
    *m.advance_cursor += 1;
  }
  trc.end(m.trace);
}

// ------------------------------------------------- per-format launchers --
// kpg: 32-weight blocks per quantisation group (group size 32, 64 or 128).
#define SWL_KPG_LAUNCH(KERNEL, ...)                                                                 \
  do {                                                                                              \
    if (kpg == 2) launch(KERNEL<B, D, 2>, dim3(grid), dim3(IM_T), smem, st, pdl, __VA_ARGS__);      \
    else if (kpg == 4) launch(KERNEL<B, D, 4>, dim3(grid), dim3(IM_T), smem, st, pdl, __VA_ARGS__); \
    else launch(KERNEL<B, D, 1>, dim3(grid), dim3(IM_T), smem, st, pdl, __VA_ARGS__);               \
  } while (0)
template <int B, int D>
void igemv_fmt(const GemvArgs& a, const SliceTab& T, const TileMaps& M, const RouterTail& rt, int kpg, int grid,
               size_t smem, cudaStream_t st, bool pdl) {
  SWL_KPG_LAUNCH(k_igemv, a, T, M, rt);
}
template <int B, int D>
void igateup_fmt(const MoeArgs& m, const SliceTab& T, const TileMaps& M, int kpg, int grid, size_t smem,
                 cudaStream_t st, bool pdl) {
  SWL_KPG_LAUNCH(k_igateup, m, T, M);
}
template <int B, int D>
void idown_fmt(const MoeArgs& m, const SliceTab& T, const TileMaps& M, int kpg, int grid, size_t smem, cudaStream_t st,
               bool pdl) {
  SWL_KPG_LAUNCH(k_idown, m, T, M);
}
#undef SWL_KPG_LAUNCH

#define SWL_INSTANTIATE_IMMA(B, D)                                                                                 \
  template void igemv_fmt<B, D>(const GemvArgs&, const SliceTab&, const TileMaps&, const RouterTail&, int, int,     \
                                size_t, cudaStream_t, bool);                                                       \
  template void igateup_fmt<B, D>(const MoeArgs&, const SliceTab&, const TileMaps&, int, int, size_t, cudaStream_t, \
                                  bool);                                                                           \
  template void idown_fmt<B, D>(const MoeArgs&, const SliceTab&, const TileMaps&, int, int, size_t, cudaStream_t,   \
                                bool);

}  // namespace swl
