// Decode-path kernels for B200 (sm_100a).
//
// Every weight-streaming kernel follows one pattern:
//   1. (before the programmatic-dependency wait) nothing that depends on the
//      previous kernel: address math only;
//   2. griddepcontrol.wait, then stage the input vector x in shared memory,
//      pre-scaled for the dequantisation trick below, with per-chunk sums;
//   3. griddepcontrol.launch_dependents so the next kernel's CTAs launch
//      while this one streams;
//   4. warps stream 16-byte chunks of packed weights (ld.global.nc, no L1
//      allocation) for R rows at a time, reduce with shuffles, and run a
//      fused epilogue.
//
// Dequantisation without integer->float conversions: for a 4-bit nibble at
// bit 4j of a word w, (w & (0xF << 4j)) | 0x4B000000 is the float
// 2^23 + q * 2^(4j) exactly (j <= 4; nibbles 5..7 use w >> 12). One packed
// f32x2 subtract removes 2^23 and one packed f32x2 FMA multiplies by
// x * 2^-(4j), which the prologue stored pre-scaled (exact: powers of two).
// Per group, y += scale * sum(q*x) + bias * sum(x): the MLX affine form
// w = scale*q + bias (Checkpoint.swift:168-209) folded out of the inner loop.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "kernels.h"
#include "launch.h"

namespace swl {

// ------------------------------------------------------------ primitives --
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ uint4 ld_stream(const uint8_t* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p));
  return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// Block-wide sum; `red` is >= 32 floats of shared memory. All threads get it.
__device__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  v = l < nw ? red[l] : 0.f;
  return warp_sum(v);
}

__device__ __forceinline__ float sigmoid_ref(float v) { return 1.f / (1.f + expf(-v)); }  // QwenCPUModel.swift:61
__device__ __forceinline__ float silu_ref(float v) { return v * sigmoid_ref(v); }        // :62
__device__ __forceinline__ float softplus_ref(float v) { return v > 20.f ? v : log1pf(expf(v)); }  // :63

// Weights per 16-byte chunk.
template <int BITS, int DT>
struct ChunkInfo {
  static constexpr int WPC = BITS == 4 ? 32 : BITS == 8 ? 16 : (DT == DT_F32 ? 4 : 8);
};

// Power-of-two pre-scale for element k (its position inside a packed word).
template <int BITS>
__device__ __forceinline__ float prescale(int k) {
  if (BITS == 4) {
    const int j = k & 7;
    const int e = j < 5 ? 4 * j : 4 * j - 12;
    return __int_as_float((127 - e) << 23);
  }
  if (BITS == 8) return (k & 1) ? 0.00390625f : 1.f;
  return 1.f;
}

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

// sum over one 16-byte chunk of q * x' (quantised) or w * x (plain).
template <int BITS, int DT>
__device__ __forceinline__ float chunk_dot(const uint4 w, const float* __restrict__ xs) {
  const float4* x4 = reinterpret_cast<const float4*>(xs);
  const uint32_t word[4] = {w.x, w.y, w.z, w.w};
  if constexpr (BITS == 4) {
    const float2 M = f2(-8388608.f, -8388608.f);
    float2 acc = f2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t lo = word[i], hi = lo >> 12;
      const float4 xa = x4[2 * i], xb = x4[2 * i + 1];
      const float2 p01 = __fadd2_rn(f2(__uint_as_float((lo & 0xFu) | 0x4B000000u), __uint_as_float((lo & 0xF0u) | 0x4B000000u)), M);
      const float2 p23 = __fadd2_rn(f2(__uint_as_float((lo & 0xF00u) | 0x4B000000u), __uint_as_float((lo & 0xF000u) | 0x4B000000u)), M);
      const float2 p45 = __fadd2_rn(f2(__uint_as_float((lo & 0xF0000u) | 0x4B000000u), __uint_as_float((hi & 0xF00u) | 0x4B000000u)), M);
      const float2 p67 = __fadd2_rn(f2(__uint_as_float((hi & 0xF000u) | 0x4B000000u), __uint_as_float((hi & 0xF0000u) | 0x4B000000u)), M);
      acc = __ffma2_rn(p01, f2(xa.x, xa.y), acc);
      acc = __ffma2_rn(p23, f2(xa.z, xa.w), acc);
      acc = __ffma2_rn(p45, f2(xb.x, xb.y), acc);
      acc = __ffma2_rn(p67, f2(xb.z, xb.w), acc);
    }
    return acc.x + acc.y;
  } else if constexpr (BITS == 8) {
    const float2 M = f2(-8388608.f, -8388608.f);
    float2 acc = f2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t lo = word[i], hi = lo >> 16;
      const float4 xa = x4[i];
      const float2 p01 = __fadd2_rn(f2(__uint_as_float((lo & 0xFFu) | 0x4B000000u), __uint_as_float((lo & 0xFF00u) | 0x4B000000u)), M);
      const float2 p23 = __fadd2_rn(f2(__uint_as_float((hi & 0xFFu) | 0x4B000000u), __uint_as_float((hi & 0xFF00u) | 0x4B000000u)), M);
      acc = __ffma2_rn(p01, f2(xa.x, xa.y), acc);
      acc = __ffma2_rn(p23, f2(xa.z, xa.w), acc);
    }
    return acc.x + acc.y;
  } else if constexpr (DT == DT_F32) {
    const float4 xa = x4[0];
    return __uint_as_float(w.x) * xa.x + __uint_as_float(w.y) * xa.y + __uint_as_float(w.z) * xa.z + __uint_as_float(w.w) * xa.w;
  } else {
    float2 acc = f2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 xa = x4[i >> 1];
      const float xl = (i & 1) ? xa.z : xa.x, xh = (i & 1) ? xa.w : xa.y;
      float lo, hi;
      if constexpr (DT == DT_BF16) {
        lo = __uint_as_float(word[i] << 16);
        hi = __uint_as_float(word[i] & 0xFFFF0000u);
      } else {
        __half2_raw r; r.x = (unsigned short)(word[i] & 0xFFFF); r.y = (unsigned short)(word[i] >> 16);
        const float2 v = __half22float2(__half2(r));
        lo = v.x; hi = v.y;
      }
      acc = __ffma2_rn(f2(lo, hi), f2(xl, xh), acc);
    }
    return acc.x + acc.y;
  }
}

// Dot products of rows [row0, row0+nr) of L with the staged x, accumulated
// over this lane's chunks (lane sl of LPR lanes per row).
template <int BITS, int DT, int R>
__device__ __forceinline__ void rows_dot(const QLin& L, int row0, int nr, const float* __restrict__ xs,
                                         const float* __restrict__ cs, int sl, int LPR, float (&acc)[R]) {
  constexpr int WPC = ChunkInfo<BITS, DT>::WPC;
  if (nr <= 0) return;
  const int nch = int(L.row_bytes >> 4);
  const uint8_t* wb = L.w + int64_t(row0) * L.row_bytes;
#pragma unroll 2
  for (int c = sl; c < nch; c += LPR) {
    uint4 w[R];
#pragma unroll
    for (int r = 0; r < R; ++r) w[r] = r < nr ? ld_stream(wb + int64_t(r) * L.row_bytes + (int64_t(c) << 4)) : make_uint4(0, 0, 0, 0);
    float sc[R], bi[R];
    if constexpr (BITS != 0) {
      const int64_t g = int64_t(c) * WPC / L.gs;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int64_t idx = int64_t(row0 + (r < nr ? r : 0)) * L.srow + g;
        sc[r] = load_scalar(L.s, DT, idx);
        bi[r] = load_scalar(L.b, DT, idx);
      }
    }
    const float* xc = xs + c * WPC;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float d = chunk_dot<BITS, DT>(w[r], xc);
      if constexpr (BITS != 0) acc[r] = fmaf(sc[r], d, fmaf(bi[r], cs[c], acc[r]));
      else acc[r] += d;
    }
  }
}

// Same as rows_dot over two matrices of identical shape sharing x (gate/up).
template <int BITS, int DT, int R>
__device__ __forceinline__ void rows_dot_pair(const QLin& A, const QLin& B, int row0, int nr, const float* __restrict__ xs,
                                              const float* __restrict__ cs, int sl, int LPR, float (&aa)[R], float (&ab)[R]) {
  constexpr int WPC = ChunkInfo<BITS, DT>::WPC;
  if (nr <= 0) return;
  const int nch = int(A.row_bytes >> 4);
  const uint8_t* wa = A.w + int64_t(row0) * A.row_bytes;
  const uint8_t* wb = B.w + int64_t(row0) * B.row_bytes;
#pragma unroll 2
  for (int c = sl; c < nch; c += LPR) {
    uint4 va[R], vb[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      va[r] = r < nr ? ld_stream(wa + int64_t(r) * A.row_bytes + (int64_t(c) << 4)) : make_uint4(0, 0, 0, 0);
      vb[r] = r < nr ? ld_stream(wb + int64_t(r) * B.row_bytes + (int64_t(c) << 4)) : make_uint4(0, 0, 0, 0);
    }
    float sa[R], ba[R], sb[R], bb[R];
    if constexpr (BITS != 0) {
      const int64_t g = int64_t(c) * WPC / A.gs;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int64_t idx = int64_t(row0 + (r < nr ? r : 0)) * A.srow + g;
        sa[r] = load_scalar(A.s, DT, idx); ba[r] = load_scalar(A.b, DT, idx);
        sb[r] = load_scalar(B.s, DT, idx); bb[r] = load_scalar(B.b, DT, idx);
      }
    }
    const float* xc = xs + c * WPC;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float da = chunk_dot<BITS, DT>(va[r], xc), db = chunk_dot<BITS, DT>(vb[r], xc);
      if constexpr (BITS != 0) {
        aa[r] = fmaf(sa[r], da, fmaf(ba[r], cs[c], aa[r]));
        ab[r] = fmaf(sb[r], db, fmaf(bb[r], cs[c], ab[r]));
      } else {
        aa[r] += da; ab[r] += db;
      }
    }
  }
}

template <int R>
__device__ __forceinline__ void sub_reduce(float (&acc)[R], int LPR) {
#pragma unroll
  for (int r = 0; r < R; ++r)
    for (int o = LPR >> 1; o; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
}

// Stage x[in] into xs (pre-scaled) and per-chunk sums into cs.
template <int BITS, int DT>
__device__ void stage_x(const GemvArgs& a, float* xs, float* cs, float* red) {
  constexpr int WPC = ChunkInfo<BITS, DT>::WPC;
  const int in = a.in, tid = threadIdx.x, nt = blockDim.x;
  if (a.prologue == PRO_RMSNORM) {
    float ss = 0.f;
    for (int k = tid; k < in; k += nt) { const float v = a.x[k]; ss += v * v; }
    ss = block_sum(ss, red);
    const float scale = 1.f / sqrtf(ss / float(in) + a.eps);  // QwenCPUModel.rmsNorm :47-59
    for (int k = tid; k < in; k += nt) xs[k] = a.x[k] * (scale * a.aux[k]);
  } else if (a.prologue == PRO_GATEDNORM) {
    // DeltaNet output gate (QwenCPUModel.swift:490-493): per v-head RMSNorm with
    // weight, then * silu(z). One warp per head.
    const int hd = a.head_dim, nh = in / hd, w = tid >> 5, l = tid & 31, nw = nt >> 5;
    for (int h = w; h < nh; h += nw) {
      float ss = 0.f;
      for (int i = l; i < hd; i += 32) { const float v = a.x[h * hd + i]; ss += v * v; }
      ss = warp_sum(ss);
      const float scale = 1.f / sqrtf(ss / float(hd) + a.eps);
      for (int i = l; i < hd; i += 32) {
        const int k = h * hd + i;
        xs[k] = (a.x[k] * (scale * a.aux2[i])) * silu_ref(a.aux[k]);
      }
    }
  } else {
    for (int k = tid; k < in; k += nt) xs[k] = a.x[k];
  }
  __syncthreads();
  if (a.x_out && blockIdx.x == 0)
    for (int k = tid; k < in; k += nt) a.x_out[k] = xs[k];
  if constexpr (BITS != 0) {
    for (int c = tid; c < in / WPC; c += nt) {
      float s = 0.f;
      for (int j = 0; j < WPC; ++j) s += xs[c * WPC + j];
      cs[c] = s;
    }
    __syncthreads();
    for (int k = tid; k < in; k += nt) xs[k] *= prescale<BITS>(k);
  }
  __syncthreads();
}

// Generic multi-segment GEMV: tasks of R rows, block b owns a contiguous
// task range, each warp runs 32/LPR tasks at a time.
template <int BITS, int DT, int R>
__device__ void gemv_tasks(const GemvArgs& a, const float* xs, const float* cs, int LPR, int t0, int t1) {
  const int spw = 32 / LPR, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31, subw = lane / LPR, sl = lane % LPR;
  for (int tw = t0 + warp * spw; tw < t1; tw += nwarps * spw) {
    const int t = tw + subw;
    int s = 0, tb = t;
    int ntask0 = (a.seg[0].lin.out + R - 1) / R;
    QLin L = a.seg[0].lin;
    float* y = a.seg[0].y;
    if (a.nseg > 1 && tb >= ntask0) {
      tb -= ntask0; s = 1;
      const int n1 = (a.seg[1].lin.out + R - 1) / R;
      if (a.nseg > 2 && tb >= n1) {
        tb -= n1; s = 2;
        const int n2 = (a.seg[2].lin.out + R - 1) / R;
        if (a.nseg > 3 && tb >= n2) { tb -= n2; s = 3; }
      }
    }
    if (s == 1) { L = a.seg[1].lin; y = a.seg[1].y; }
    else if (s == 2) { L = a.seg[2].lin; y = a.seg[2].y; }
    else if (s == 3) { L = a.seg[3].lin; y = a.seg[3].y; }
    const int row0 = tb * R;
    const int nr = t < t1 ? min(R, L.out - row0) : 0;
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.f;
    rows_dot<BITS, DT, R>(L, row0, nr, xs, cs, sl, LPR, acc);
    sub_reduce<R>(acc, LPR);
    if (sl == 0) {
#pragma unroll
      for (int r = 0; r < R; ++r)
        if (r < nr) {
          if (a.epilogue == EPI_RESIDUAL) y[row0 + r] += acc[r];
          else y[row0 + r] = acc[r];
        }
    }
  }
}

constexpr int GEMV_R = 4;
constexpr int GEMV_THREADS = 256;

template <int BITS, int DT>
__global__ void __launch_bounds__(GEMV_THREADS) k_gemv(const GemvArgs a, int LPR, int total, int tpb) {
  extern __shared__ __align__(16) float smem[];
  constexpr int WPC = ChunkInfo<BITS, DT>::WPC;
  float* xs = smem;
  float* cs = smem + a.in;
  float* red = cs + (a.in / WPC + 4);
  pdl_wait();
  stage_x<BITS, DT>(a, xs, cs, red);
  pdl_launch();
  const int t0 = blockIdx.x * tpb, t1 = min(total, t0 + tpb);
  gemv_tasks<BITS, DT, GEMV_R>(a, xs, cs, LPR, t0, t1);
  if (a.argmax_out) {
    // Fused greedy argmax over segment 0 (first index wins on ties, as the
    // reference's `logits[v] > logits[best]` scan).
    __syncthreads();
    const float* y = a.seg[0].y;
    const int n = a.seg[0].lin.out;
    const int r0 = t0 * GEMV_R, r1 = min(n, t1 * GEMV_R);
    float bv = -INFINITY; int bi = 0x7fffffff;
    for (int r = r0 + threadIdx.x; r < r1; r += blockDim.x) {
      const float v = y[r];
      if (v > bv || (v == bv && r < bi)) { bv = v; bi = r; }
    }
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    __shared__ float wv[32];
    __shared__ int wi[32];
    __shared__ bool last;
    if ((threadIdx.x & 31) == 0) { wv[threadIdx.x >> 5] = bv; wi[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
        if (wv[w] > bv || (wv[w] == bv && wi[w] < bi)) { bv = wv[w]; bi = wi[w]; }
      a.argmax_val[blockIdx.x] = bv;
      a.argmax_idx[blockIdx.x] = bi;
      __threadfence();
      last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
      __threadfence();
      float gv = -INFINITY; int gi = 0x7fffffff;
      for (int b = 0; b < (int)gridDim.x; ++b) {
        const float v = __ldcg(a.argmax_val + b);
        const int i = __ldcg(a.argmax_idx + b);
        if (v > gv || (v == gv && i < gi)) { gv = v; gi = i; }
      }
      *a.argmax_out = gi;
      *a.counter = 0u;
    }
  }
}

// ------------------------------------------------------------- router ----
// Post-attention RMSNorm + router GEMV + shared-expert gate logit, then the
// last CTA to finish computes softmax, top-k and the combine weights
// (QwenCPUModel.swift:506-521, 546-550; routerPicks QwenMetalModel.swift:875-892).
template <int BITS, int DT>
__global__ void __launch_bounds__(GEMV_THREADS) k_router(const RouterArgs ra, int E, int LPR, int total, int tpb) {
  extern __shared__ __align__(16) float smem[];
  constexpr int WPC = ChunkInfo<BITS, DT>::WPC;
  const int D = ra.gate.in;
  float* xs = smem;
  float* cs = smem + D;
  float* red = cs + (D / WPC + 4);
  GemvArgs a;
  a.seg[0].lin = ra.gate; a.seg[0].y = ra.logits;
  a.seg[1].lin = ra.sgate; a.seg[1].y = ra.logits + E;
  a.nseg = 2; a.in = D; a.prologue = PRO_RMSNORM; a.epilogue = EPI_STORE;
  a.x = ra.h; a.aux = ra.norm_w; a.eps = ra.eps; a.x_out = ra.x_out;
  pdl_wait();
  stage_x<BITS, DT>(a, xs, cs, red);
  pdl_launch();
  const int t0 = blockIdx.x * tpb, t1 = min(total, t0 + tpb);
  gemv_tasks<BITS, DT, GEMV_R>(a, xs, cs, LPR, t0, t1);
  __shared__ bool last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(ra.counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  // softmax over E (max-subtracted, QwenCPUModel.softmaxRow :65-71)
  float* p = smem;  // reuse: E floats
  float m = -INFINITY;
  for (int e = threadIdx.x; e < E; e += blockDim.x) { p[e] = __ldcg(ra.logits + e); m = fmaxf(m, p[e]); }
  m = warp_max(m);
  __shared__ float wm[32];
  if ((threadIdx.x & 31) == 0) wm[threadIdx.x >> 5] = m;
  __syncthreads();
  m = -INFINITY;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, wm[w]);
  float sum = 0.f;
  for (int e = threadIdx.x; e < E; e += blockDim.x) { p[e] = expf(p[e] - m); sum += p[e]; }
  __shared__ float red2[32];
  sum = block_sum(sum, red2);
  for (int e = threadIdx.x; e < E; e += blockDim.x) p[e] = p[e] / sum;
  __syncthreads();
  // top-k: repeated warp argmax; ties keep the lower expert id, which is the
  // outcome of the reference's insertion scan with a strict `>` (:516).
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    float score_sum = 0.f;
    __shared__ float kp[64];
    __shared__ int ki[64];
    for (int k = 0; k < ra.topk; ++k) {
      float bv = -1.f; int bi = 0x7fffffff;
      for (int e = lane; e < E; e += 32) {
        const float v = p[e];
        if (v > bv || (v == bv && e < bi)) { bv = v; bi = e; }
      }
      for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      if (bi >= E) bi = 0;  // non-finite logits: keep indices in range
      if (lane == 0) { kp[k] = bv; ki[k] = bi; p[bi] = -2.f; }
      __syncwarp();
    }
    if (lane == 0) {
      for (int k = 0; k < ra.topk; ++k) score_sum += kp[k];
      for (int k = 0; k < ra.topk; ++k) {
        ra.pick_ids[k] = ki[k];
        ra.pick_w[k] = ra.norm_topk ? kp[k] / score_sum : kp[k];
      }
      *ra.shared_scale = sigmoid_ref(__ldcg(ra.logits + E));
      *ra.counter = 0u;
    }
  }
}

// ---------------------------------------------------------------- MoE ----
__device__ __forceinline__ QLin expert_lin(const ExpertProj& p, int id) {
  QLin l = p.lin;
  l.w += int64_t(id) * p.wstride;
  l.s += int64_t(id) * p.sstride;
  l.b += int64_t(id) * p.bstride;
  return l;
}

constexpr int MOE_RG = 2;  // gate/up rows per task (each paired with its up row)

// Gate/up of the K routed experts and the shared expert, SiLU * up fused
// (encodePendingMoE QwenMetalModel.swift:806-841; QwenCPUModel.swift:552-561).
template <int BITS, int DT>
__global__ void __launch_bounds__(GEMV_THREADS) k_moe_gateup(const MoeArgs m, int LPR, int tasks_routed, int tasks_shared, int tpb) {
  extern __shared__ __align__(16) float smem[];
  constexpr int WPC = ChunkInfo<BITS, DT>::WPC;
  const int D = m.g.lin.in;
  float* xs = smem;
  float* cs = smem + D;
  float* red = cs + (D / WPC + 4);
  GemvArgs a;
  a.in = D; a.prologue = PRO_COPY; a.x = m.x;
  pdl_wait();
  stage_x<BITS, DT>(a, xs, cs, red);
  pdl_launch();
  const int total = tasks_routed * m.topk + tasks_shared;
  const int t0 = blockIdx.x * tpb, t1 = min(total, t0 + tpb);
  const int spw = 32 / LPR, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31, subw = lane / LPR, sl = lane % LPR;
  for (int tw = t0 + warp * spw; tw < t1; tw += nwarps * spw) {
    const int t = tw + subw;
    const int slot = t < tasks_routed * m.topk ? t / tasks_routed : m.topk;
    const int tb = slot < m.topk ? t - slot * tasks_routed : t - tasks_routed * m.topk;
    QLin G, U;
    if (slot < m.topk) {
      const int id = t < t1 ? m.pick_ids[slot] : 0;
      G = expert_lin(m.g, id); U = expert_lin(m.u, id);
    } else {
      G = m.sg; U = m.su;
    }
    const int row0 = tb * MOE_RG;
    const int nr = t < t1 ? min(MOE_RG, G.out - row0) : 0;
    float ag[MOE_RG], au[MOE_RG];
#pragma unroll
    for (int r = 0; r < MOE_RG; ++r) { ag[r] = 0.f; au[r] = 0.f; }
    rows_dot_pair<BITS, DT, MOE_RG>(G, U, row0, nr, xs, cs, sl, LPR, ag, au);
    sub_reduce<MOE_RG>(ag, LPR);
    sub_reduce<MOE_RG>(au, LPR);
    if (sl == 0)
      for (int r = 0; r < nr; ++r) m.hmid[slot * m.hmid_stride + row0 + r] = silu_ref(ag[r]) * au[r];
  }
}

// Down projections of the K routed experts + shared expert, router-weighted
// combine and the residual add, one output row per sub-warp task
// (weighted_accum Kernels.metal.txt:463-478; QwenCPUModel.swift:555-566).
template <int BITS, int DT>
__global__ void __launch_bounds__(128) k_moe_down(const MoeArgs m, int LPR, int tpb) {
  extern __shared__ __align__(16) float smem[];
  constexpr int WPC = ChunkInfo<BITS, DT>::WPC;
  const int K = m.topk, D = m.d.lin.out;
  const int I = m.d.lin.in, SI = m.sd.in;
  const int xstride = m.hmid_stride, cstride = m.hmid_stride / WPC + 4;
  float* xs = smem;                       // [(K+1) * xstride]
  float* cs = xs + (K + 1) * xstride;     // [(K+1) * cstride]
  __shared__ float wts[65];
  pdl_wait();
  for (int e = 0; e <= K; ++e) {
    const int in = e < K ? I : SI;
    for (int k = threadIdx.x; k < in; k += blockDim.x) xs[e * xstride + k] = m.hmid[e * m.hmid_stride + k];
  }
  if (threadIdx.x < K) wts[threadIdx.x] = m.pick_w[threadIdx.x];
  if (threadIdx.x == 0) wts[K] = *m.shared_scale;
  __syncthreads();
  if constexpr (BITS != 0) {
    for (int e = 0; e <= K; ++e) {
      const int in = e < K ? I : SI;
      for (int c = threadIdx.x; c < in / WPC; c += blockDim.x) {
        float s = 0.f;
        for (int j = 0; j < WPC; ++j) s += xs[e * xstride + c * WPC + j];
        cs[e * cstride + c] = s;
      }
    }
    __syncthreads();
    for (int e = 0; e <= K; ++e) {
      const int in = e < K ? I : SI;
      for (int k = threadIdx.x; k < in; k += blockDim.x) xs[e * xstride + k] *= prescale<BITS>(k);
    }
  }
  __syncthreads();
  pdl_launch();
  const int t0 = blockIdx.x * tpb, t1 = min(D, t0 + tpb);
  const int spw = 32 / LPR, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31, subw = lane / LPR, sl = lane % LPR;
  for (int tw = t0 + warp * spw; tw < t1; tw += nwarps * spw) {
    const int row = tw + subw;
    const int nr = row < t1 ? 1 : 0;
    float out = 0.f;
    for (int e = 0; e <= K; ++e) {
      const QLin L = e < K ? expert_lin(m.d, m.pick_ids[e]) : m.sd;
      float acc[1] = {0.f};
      rows_dot<BITS, DT, 1>(L, nr ? row : 0, nr, xs + e * xstride, cs + e * cstride, sl, LPR, acc);
      sub_reduce<1>(acc, LPR);
      out += wts[e] * acc[0];
    }
    if (sl == 0 && nr) m.h[row] += out;
  }
  if (m.advance_sd && blockIdx.x == 0 && threadIdx.x == 0) {
    // Advance the sequence position and the token cursor once the last
    // layer of the step is done (no other CTA of this grid reads them).
    *m.advance_sd->pos += 1;
    *m.advance_cursor += 1;
  }
}

// ------------------------------------------------------------ DeltaNet ----
// One decode step of a gated-DeltaNet layer after its in-projections:
// causal conv (ring of conv_k rows) + SiLU, q/k RMSNorm scaled 1/dk and
// 1/sqrt(dk), gating g = exp(-exp(A_log) * softplus(a + dt_bias)),
// beta = sigmoid(b), and the recurrence S <- gS; d = (v - S k) beta;
// S <- S + k d^T; y = S q (QwenCPUModel.swift:423-488). Block = (v-head,
// slice of dv rows); each warp owns rows, lanes stride over dk.
__device__ __forceinline__ int delta_src(const DeltaArgs& a, int c) {
  // Index into `proj` of mixed-qkv channel c.
  if (a.split) return c;
  const int keyDim = a.nk * a.dk, rep = a.nv / a.nk, chunk = 2 * a.dk + 2 * rep * a.dv;
  if (c < keyDim) { const int hk = c / a.dk; return hk * chunk + (c - hk * a.dk); }
  if (c < 2 * keyDim) { const int cc = c - keyDim, hk = cc / a.dk; return hk * chunk + a.dk + (cc - hk * a.dk); }
  const int cv = c - 2 * keyDim, hv = cv / a.dv, i = cv - hv * a.dv, hk = hv / rep, ri = hv - hk * rep;
  return hk * chunk + 2 * a.dk + ri * a.dv + i;
}
__device__ __forceinline__ int delta_z(const DeltaArgs& a, int hv, int i) {
  const int valueDim = a.nv * a.dv;
  if (a.split) return a.conv_dim + hv * a.dv + i;
  const int rep = a.nv / a.nk, chunk = 2 * a.dk + 2 * rep * a.dv, hk = hv / rep, ri = hv - hk * rep;
  (void)valueDim;
  return hk * chunk + 2 * a.dk + rep * a.dv + ri * a.dv + i;
}
__device__ __forceinline__ void delta_ba(const DeltaArgs& a, int hv, int& bi, int& ai) {
  const int valueDim = a.nv * a.dv;
  if (a.split) { bi = a.conv_dim + valueDim + hv; ai = a.conv_dim + valueDim + a.nv + hv; return; }
  const int keyDim = a.nk * a.dk, rep = a.nv / a.nk, hk = hv / rep, ri = hv - hk * rep;
  const int base = 2 * keyDim + 2 * valueDim + hk * 2 * rep;
  bi = base + ri; ai = base + rep + ri;
}

__global__ void __launch_bounds__(128) k_delta(const DeltaArgs a) {
  extern __shared__ __align__(16) float sm[];
  const int dk = a.dk, dv = a.dv, K = a.conv_k, RB = a.rows_per_block;
  const int hv = blockIdx.x, slice = blockIdx.y, rep = a.nv / a.nk, hk = hv / rep;
  const int keyDim = a.nk * dk;
  float* q = sm;            // [dk]
  float* k = q + dk;        // [dk]
  float* v = k + dk;        // [RB]
  float* red = v + RB;      // [32]
  __shared__ float gb[2];
  pdl_wait();
  const StateDev* sd = a.sd;
  const int pos = *sd->pos;
  float* ring = sd->conv[a.layer];
  float* S = sd->dstate[a.layer];
  const int slot = pos % K;
  // conv + silu for q (dk), k (dk) and this block's v rows
  const int nch = 2 * dk + RB;
  const bool own_qk = (hv % rep) == 0 && slice == 0;
  for (int t = threadIdx.x; t < nch; t += blockDim.x) {
    int c;
    if (t < dk) c = hk * dk + t;
    else if (t < 2 * dk) c = keyDim + hk * dk + (t - dk);
    else c = 2 * keyDim + hv * dv + slice * RB + (t - 2 * dk);
    const float xn = a.proj[delta_src(a, c)];
    float acc = 0.f;
    for (int j = 0; j < K - 1; ++j) {
      const int rs = ((pos - (K - 1) + j) % K + K) % K;
      acc += a.conv_w[c * K + j] * ring[int64_t(rs) * a.conv_dim + c];
    }
    acc += a.conv_w[c * K + K - 1] * xn;
    const float o = silu_ref(acc);
    if (t < dk) q[t] = o; else if (t < 2 * dk) k[t - dk] = o; else v[t - 2 * dk] = o;
    if (t >= 2 * dk || own_qk) ring[int64_t(slot) * a.conv_dim + c] = xn;
  }
  if (threadIdx.x == 0) {
    int bi, ai;
    delta_ba(a, hv, bi, ai);
    gb[0] = expf(-expf(a.a_log[hv]) * softplus_ref(a.proj[ai] + a.dt_bias[hv]));
    gb[1] = sigmoid_ref(a.proj[bi]);
  }
  // z rows of this slice, de-interleaved for the out-projection prologue
  for (int i = threadIdx.x; i < RB; i += blockDim.x) {
    const int d = slice * RB + i;
    a.z[hv * dv + d] = a.proj[delta_z(a, hv, d)];
  }
  __syncthreads();
  pdl_launch();
  // q/k RMSNorm (no weight, eps 1e-6) then 1/dk and 1/sqrt(dk)
  float sq = 0.f, sk = 0.f;
  for (int i = threadIdx.x; i < dk; i += blockDim.x) { sq += q[i] * q[i]; sk += k[i] * k[i]; }
  sq = block_sum(sq, red);
  sk = block_sum(sk, red);
  const float inv = 1.f / sqrtf(float(dk));
  const float scq = 1.f / sqrtf(sq / float(dk) + 1e-6f), sck = 1.f / sqrtf(sk / float(dk) + 1e-6f);
  __syncthreads();
  for (int i = threadIdx.x; i < dk; i += blockDim.x) { q[i] = (q[i] * scq) * (inv * inv); k[i] = (k[i] * sck) * inv; }
  __syncthreads();
  const float g = gb[0], beta = gb[1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int r = warp; r < RB; r += nw) {
    const int d = slice * RB + r;
    float* Sr = S + (int64_t(hv) * dv + d) * dk;
    float kv = 0.f;
    for (int i = lane; i < dk; i += 32) { const float s = Sr[i] * g; Sr[i] = s; kv += s * k[i]; }
    kv = warp_sum(kv);
    const float delta = (v[r] - kv) * beta;
    float y = 0.f;
    for (int i = lane; i < dk; i += 32) { const float s = Sr[i] + k[i] * delta; Sr[i] = s; y += s * q[i]; }
    y = warp_sum(y);
    if (lane == 0) a.y[hv * dv + d] = y;
  }
}

// ----------------------------------------------------------- attention ----
// Gated GQA decode for one token: q/k RMSNorm, partial NeoX RoPE, KV append,
// causal softmax(q k^T / sqrt(hd)) v split over context chunks, combine by the
// last CTA of each kv head, times sigmoid(gate) (QwenCPUModel.swift:285-367).
__device__ __forceinline__ void rope_inplace(float* x, int hd, int rot, int pos, float theta) {
  const int half = rot / 2;
  for (int j = threadIdx.x; j < half; j += blockDim.x) {
    const float invf = powf(theta, -float(2 * j) / float(rot));
    const float ang = float(pos) * invf;
    const float c = cosf(ang), s = sinf(ang);
    const float xa = x[j], xb = x[half + j];
    x[j] = xa * c - xb * s;
    x[half + j] = xb * c + xa * s;
  }
}

__global__ void __launch_bounds__(256) k_attn(const AttnArgs a) {
  extern __shared__ __align__(16) float sm[];
  const int hd = a.hd, G = a.H / a.Hkv, kvh = blockIdx.x, chunk = blockIdx.y;
  float* q = sm;                 // [G][hd]
  float* kn = q + G * hd;        // [hd]
  float* vn = kn + hd;           // [hd]
  float* sc = vn + hd;           // [G][chunk_cap]
  float* red = sc + G * a.chunk_cap;  // [32]
  __shared__ bool last;
  pdl_wait();
  const StateDev* sd = a.sd;
  const int pos = *sd->pos;
  float* Kc = sd->kc[a.layer];
  float* Vc = sd->vc[a.layer];
  // stage q heads of this group, new k, new v
  for (int i = threadIdx.x; i < G * hd; i += blockDim.x) {
    const int h = kvh * G + i / hd, d = i % hd;
    q[i] = a.qout[h * 2 * hd + d];
  }
  for (int i = threadIdx.x; i < hd; i += blockDim.x) { kn[i] = a.knew[kvh * hd + i]; vn[i] = a.vnew[kvh * hd + i]; }
  __syncthreads();
  pdl_launch();
  // RMSNorm with weight (eps = rms_norm_eps), one head at a time
  for (int h = 0; h <= G; ++h) {
    float* x = h < G ? q + h * hd : kn;
    const float* w = h < G ? a.qn : a.kn;
    float ss = 0.f;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) ss += x[i] * x[i];
    ss = block_sum(ss, red);
    const float scale = 1.f / sqrtf(ss / float(hd) + a.eps);
    for (int i = threadIdx.x; i < hd; i += blockDim.x) x[i] *= scale * w[i];
    __syncthreads();
    rope_inplace(x, hd, a.rot, pos, a.rope_theta);
    __syncthreads();
  }
  if (chunk == 0)
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
      Kc[(int64_t(pos) * a.Hkv + kvh) * hd + i] = kn[i];
      Vc[(int64_t(pos) * a.Hkv + kvh) * hd + i] = vn[i];
    }
  const int ctx = pos + 1;
  const int per = (ctx + a.nchunks - 1) / a.nchunks;
  const int p0 = chunk * per, p1 = min(ctx, p0 + per);
  const int n = max(0, p1 - p0);
  const float scale = 1.f / sqrtf(float(hd));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  // scores
  for (int j = warp; j < n; j += nw) {
    const int p = p0 + j;
    const float* kr = p == pos ? kn : Kc + (int64_t(p) * a.Hkv + kvh) * hd;
    for (int h = 0; h < G; ++h) {
      float d = 0.f;
      for (int i = lane; i < hd; i += 32) d += q[h * hd + i] * kr[i];
      d = warp_sum(d);
      if (lane == 0) sc[h * a.chunk_cap + j] = d * scale;
    }
  }
  __syncthreads();
  // per-head chunk max and exp-sum (one warp per head)
  __shared__ float hm[64], hl[64];
  for (int h = warp; h < G; h += nw) {
    float m = -INFINITY;
    for (int j = lane; j < n; j += 32) m = fmaxf(m, sc[h * a.chunk_cap + j]);
    m = warp_max(m);
    float l = 0.f;
    for (int j = lane; j < n; j += 32) { const float e = expf(sc[h * a.chunk_cap + j] - m); sc[h * a.chunk_cap + j] = e; l += e; }
    l = warp_sum(l);
    if (lane == 0) { hm[h] = n > 0 ? m : -INFINITY; hl[h] = l; }
  }
  __syncthreads();
  float* part = a.part + (int64_t(kvh) * a.nchunks + chunk) * G * (hd + 2);
  for (int i = threadIdx.x; i < G * hd; i += blockDim.x) {
    const int h = i / hd, d = i % hd;
    float acc = 0.f;
    for (int j = 0; j < n; ++j) {
      const int p = p0 + j;
      const float vv = p == pos ? vn[d] : Vc[(int64_t(p) * a.Hkv + kvh) * hd + d];
      acc += sc[h * a.chunk_cap + j] * vv;
    }
    part[h * (hd + 2) + 2 + d] = acc;
  }
  for (int h = threadIdx.x; h < G; h += blockDim.x) { part[h * (hd + 2)] = hm[h]; part[h * (hd + 2) + 1] = hl[h]; }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(a.counters + kvh, 1u) == a.nchunks - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  const float* pk = a.part + int64_t(kvh) * a.nchunks * G * (hd + 2);
  for (int i = threadIdx.x; i < G * hd; i += blockDim.x) {
    const int h = i / hd, d = i % hd;
    float m = -INFINITY;
    for (int c = 0; c < a.nchunks; ++c) m = fmaxf(m, __ldcg(pk + (int64_t(c) * G + h) * (hd + 2)));
    float l = 0.f, o = 0.f;
    for (int c = 0; c < a.nchunks; ++c) {
      const float* pc = pk + (int64_t(c) * G + h) * (hd + 2);
      const float mc = __ldcg(pc);
      if (mc == -INFINITY) continue;
      const float f = expf(mc - m);
      l += __ldcg(pc + 1) * f;
      o += __ldcg(pc + 2 + d) * f;
    }
    const int head = kvh * G + h;
    const float gate = a.qout[head * 2 * hd + hd + d];
    a.out[head * hd + d] = (o / l) * sigmoid_ref(gate);
  }
  if (threadIdx.x == 0) a.counters[kvh] = 0u;
}

// --------------------------------------------------------------- embed ----
__global__ void k_embed(const EmbedArgs a, int D) {
  pdl_wait();
  const int tok = a.tokens[*a.cursor];
  pdl_launch();
  if (tok < 0 || tok >= a.vocab) {
    if (threadIdx.x == 0) *a.err = 1;
    for (int i = threadIdx.x; i < D; i += blockDim.x) a.h[i] = 0.f;
    return;
  }
  const QLin& L = a.table;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float v;
    if (L.bits) {
      const int per = 32 / L.bits;
      const uint32_t word = reinterpret_cast<const uint32_t*>(L.w + int64_t(tok) * L.row_bytes)[i / per];
      const uint32_t q = (word >> (L.bits * (i % per))) & ((1u << L.bits) - 1u);
      const int64_t g = int64_t(tok) * L.srow + i / L.gs;
      v = __fadd_rn(__fmul_rn(load_scalar(L.s, L.dt, g), float(q)), load_scalar(L.b, L.dt, g));
    } else {
      v = load_scalar(L.w, L.dt, int64_t(tok) * D + i);
    }
    a.h[i] = v;
  }
}

// Dequantised rows (bit-exact w = fl(fl(scale * q) + bias), two roundings).
__global__ void k_dequant(const QLin L, int64_t r0, int64_t r1, float* out) {
  const int64_t cols = L.in, n = (r1 - r0) * cols;
  for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < n; t += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = r0 + t / cols, i = t % cols;
    float v;
    if (L.bits) {
      const int per = 32 / L.bits;
      const uint32_t word = reinterpret_cast<const uint32_t*>(L.w + r * L.row_bytes)[i / per];
      const uint32_t q = (word >> (L.bits * (i % per))) & ((1u << L.bits) - 1u);
      const int64_t g = r * L.srow + i / L.gs;
      v = __fadd_rn(__fmul_rn(load_scalar(L.s, L.dt, g), float(q)), load_scalar(L.b, L.dt, g));
    } else {
      v = load_scalar(L.w, L.dt, r * cols + i);
    }
    out[t] = v;
  }
}

// ------------------------------------------------------------- launches --
int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

static int lanes_per_row(int64_t row_bytes) {
  const int64_t nch = row_bytes >> 4;
  int l = 32;
  while (l > 1 && l > nch) l >>= 1;
  return l;
}
static int wpc_of(int bits, int dt) { return bits == 4 ? 32 : bits == 8 ? 16 : (dt == DT_F32 ? 4 : 8); }

#define SWL_DISPATCH(BITS_, DT_, FN)                                              \
  do {                                                                            \
    const int b_ = (BITS_), d_ = (DT_);                                           \
    if (b_ == 4 && d_ == DT_BF16) { FN(4, DT_BF16); }                             \
    else if (b_ == 4 && d_ == DT_F32) { FN(4, DT_F32); }                          \
    else if (b_ == 4 && d_ == DT_F16) { FN(4, DT_F16); }                          \
    else if (b_ == 8 && d_ == DT_BF16) { FN(8, DT_BF16); }                        \
    else if (b_ == 8 && d_ == DT_F32) { FN(8, DT_F32); }                          \
    else if (b_ == 8 && d_ == DT_F16) { FN(8, DT_F16); }                          \
    else if (b_ == 0 && d_ == DT_F32) { FN(0, DT_F32); }                          \
    else if (b_ == 0 && d_ == DT_BF16) { FN(0, DT_BF16); }                        \
    else if (b_ == 0 && d_ == DT_F16) { FN(0, DT_F16); }                          \
    else throw Error(ERR_UNSUPPORTED, "unsupported weight format");               \
  } while (0)

void launch_gemv(const GemvArgs& a, cudaStream_t st, bool pdl) {
  const QLin& l0 = a.seg[0].lin;
  for (int s = 1; s < a.nseg; ++s)
    if (a.seg[s].lin.bits != l0.bits || a.seg[s].lin.dt != l0.dt || a.seg[s].lin.row_bytes != l0.row_bytes)
      throw Error(ERR_UNSUPPORTED, "fused GEMV segments differ in format");
  int total = 0;
  for (int s = 0; s < a.nseg; ++s) total += (a.seg[s].lin.out + GEMV_R - 1) / GEMV_R;
  const int LPR = lanes_per_row(l0.row_bytes);
  const int tasks_per_block_pass = (GEMV_THREADS / 32) * (32 / LPR);
  int grid = std::min((total + tasks_per_block_pass - 1) / tasks_per_block_pass, sm_count() * 4);
  grid = std::max(grid, 1);
  int tpb = (total + grid - 1) / grid;
  if (a.argmax_out) grid = std::min(grid, 1024);
  tpb = (total + grid - 1) / grid;
  grid = (total + tpb - 1) / tpb;
  const int wpc = wpc_of(l0.bits, l0.dt);
  const size_t smem = size_t(a.in + a.in / wpc + 4 + 32) * 4;
#define GEMV_FN(B, D) launch(k_gemv<B, D>, dim3(grid), dim3(GEMV_THREADS), smem, st, pdl, a, LPR, total, tpb)
  SWL_DISPATCH(l0.bits, l0.dt, GEMV_FN);
#undef GEMV_FN
}

void launch_router(const RouterArgs& r, int E, cudaStream_t st, bool pdl) {
  if (r.gate.bits != r.sgate.bits || r.gate.dt != r.sgate.dt || r.gate.row_bytes != r.sgate.row_bytes)
    throw Error(ERR_UNSUPPORTED, "router and shared-expert gate differ in format");
  const int total = (E + GEMV_R - 1) / GEMV_R + 1;
  const int LPR = lanes_per_row(r.gate.row_bytes);
  const int per = (GEMV_THREADS / 32) * (32 / LPR);
  const int grid = std::max(1, std::min((total + per - 1) / per, sm_count()));
  const int tpb = (total + grid - 1) / grid;
  const int g2 = (total + tpb - 1) / tpb;
  const int wpc = wpc_of(r.gate.bits, r.gate.dt);
  const size_t smem = size_t(std::max(r.gate.in + r.gate.in / wpc + 4 + 32, E + 32)) * 4;
#define ROUTER_FN(B, D) launch(k_router<B, D>, dim3(g2), dim3(GEMV_THREADS), smem, st, pdl, r, E, LPR, total, tpb)
  SWL_DISPATCH(r.gate.bits, r.gate.dt, ROUTER_FN);
#undef ROUTER_FN
}

void launch_moe_gateup(const MoeArgs& m, cudaStream_t st, bool pdl) {
  const QLin& g = m.g.lin;
  if (m.sg.bits != g.bits || m.sg.dt != g.dt || m.sg.row_bytes != g.row_bytes || m.u.lin.row_bytes != g.row_bytes)
    throw Error(ERR_UNSUPPORTED, "shared and routed experts differ in format");
  const int tr = (g.out + MOE_RG - 1) / MOE_RG, ts = (m.sg.out + MOE_RG - 1) / MOE_RG;
  const int total = tr * m.topk + ts;
  const int LPR = lanes_per_row(g.row_bytes);
  const int per = (GEMV_THREADS / 32) * (32 / LPR);
  int grid = std::max(1, std::min((total + per - 1) / per, sm_count() * 4));
  const int tpb = (total + grid - 1) / grid;
  grid = (total + tpb - 1) / tpb;
  const int wpc = wpc_of(g.bits, g.dt);
  const size_t smem = size_t(g.in + g.in / wpc + 4 + 32) * 4;
#define GU_FN(B, D) launch(k_moe_gateup<B, D>, dim3(grid), dim3(GEMV_THREADS), smem, st, pdl, m, LPR, tr, ts, tpb)
  SWL_DISPATCH(g.bits, g.dt, GU_FN);
#undef GU_FN
}

void launch_moe_down(const MoeArgs& m, cudaStream_t st, bool pdl) {
  const QLin& d = m.d.lin;
  if (m.sd.bits != d.bits || m.sd.dt != d.dt)
    throw Error(ERR_UNSUPPORTED, "shared and routed experts differ in format");
  if (m.topk > 64) throw Error(ERR_UNSUPPORTED, "top-k above 64");
  const int LPR = std::min(lanes_per_row(d.row_bytes), lanes_per_row(m.sd.row_bytes));
  const int per = (128 / 32) * (32 / LPR);
  const int D = d.out;
  int grid = std::max(1, (D + per - 1) / per);
  const int tpb = (D + grid - 1) / grid;
  grid = (D + tpb - 1) / tpb;
  const int wpc = wpc_of(d.bits, d.dt);
  const size_t smem = size_t(m.topk + 1) * size_t(m.hmid_stride + m.hmid_stride / wpc + 4) * 4;
#define DOWN_FN(B, D_) launch(k_moe_down<B, D_>, dim3(grid), dim3(128), smem, st, pdl, m, LPR, tpb)
  SWL_DISPATCH(d.bits, d.dt, DOWN_FN);
#undef DOWN_FN
}

void launch_delta(const DeltaArgs& a, cudaStream_t st, bool pdl) {
  const size_t smem = size_t(2 * a.dk + a.rows_per_block + 32) * 4;
  launch(k_delta, dim3(a.nv, a.dv / a.rows_per_block), dim3(128), smem, st, pdl, a);
}

void launch_attn(const AttnArgs& a, cudaStream_t st, bool pdl) {
  const int G = a.H / a.Hkv;
  const size_t smem = size_t(G * a.hd + 2 * a.hd + G * a.chunk_cap + 32) * 4;
  launch(k_attn, dim3(a.Hkv, a.nchunks), dim3(256), smem, st, pdl, a);
}

void launch_embed(const EmbedArgs& a, int hidden, cudaStream_t st, bool pdl) {
  launch(k_embed, dim3(1), dim3(256), 0, st, pdl, a, hidden);
}

void launch_dequant(const QLin& l, int64_t r0, int64_t r1, float* out, cudaStream_t st) {
  const int64_t n = (r1 - r0) * int64_t(l.in);
  const int grid = int(std::min<int64_t>((n + 255) / 256, 4096));
  launch(k_dequant, dim3(std::max(grid, 1)), dim3(256), 0, st, false, l, r0, r1, out);
}

}  // namespace swl
