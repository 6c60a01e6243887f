// Warp-specialised weight-streaming kernels of the decode step (B = 1):
// dense multi-segment GEMV (projections, lm_head with fused greedy argmax,
// router with its top-k epilogue), fused shared/routed expert gate/up, and
// expert down + combine + residual.
//
// At B = 1 every weight byte is used once per token, so a kernel's time is
// its dependency wait, the DRAM round trips it exposes after that wait, and
// its arithmetic. Here each CTA owns a contiguous slice of weight rows:
//   * warp SL_CW (the producer) copies the slice tile by tile into a ring of
//     shared-memory slots with bulk copies (cp.async.bulk, completion counted
//     on an mbarrier per slot), starting at kernel entry: weights never
//     depend on the previous kernel, so with programmatic dependent launch
//     they stream in while the previous kernel still runs (routed experts of
//     gate/up, known only once the router is done, are the exception);
//   * warps 0..SL_CW-1 (the consumers) wait for the previous grid, stage the
//     input vector (pre-scaled, chunk-interleaved, as the kernels of
//     gemv_impl.cuh) and keep their slice of it in registers, then walk the
//     tiles: read the row fragments from shared memory, free the slot, and
//     reduce. Rows longer than one register window (64 activations per lane)
//     are split over W warp groups whose partial sums meet in shared memory.
// Every wait on an mbarrier is bounded (mbar_wait); a wait that gives up sets
// bit 0 of SliceTab::status and the CTA finishes without its result.
#pragma once

#include "gemv_impl.cuh"
#include "slice.h"

namespace swl {

template <int BITS, int DT>
struct SliceFmt {
  static constexpr int WPC = ChunkInfo<BITS, DT>::WPC;
  static constexpr int CPL = 64 / WPC;  // chunks per lane: 64 activations in registers
  static constexpr int SB = DT == DT_F32 ? 4 : 2;
};

template <typename P>
__device__ __forceinline__ P seg_pick(const P (&v)[4], int k) {
  return k == 0 ? v[0] : k == 1 ? v[1] : k == 2 ? v[2] : v[3];
}

__device__ __forceinline__ void sl_fail(const SliceTab& T) {
  if (T.status) atomicOr(T.status, 1);
}

// Scale / bias entry i of a row held in shared memory.
template <int DT>
__device__ __forceinline__ float sm_scalar(const uint8_t* p, int i) {
  if constexpr (DT == DT_F32) {
    return reinterpret_cast<const float*>(p)[i];
  } else {
    const uint16_t u = reinterpret_cast<const uint16_t*>(p)[i];
    return DT == DT_BF16 ? bf16_to_f32(u) : f16_bits_to_f32(u);
  }
}

// One lane's fragment of a row held in shared memory (zeros when !valid).
template <int BITS, int DT, int CPL>
__device__ __forceinline__ void smem_row(RowFrag<BITS, DT, CPL>& f, const LaneChunks<BITS, DT, CPL>& lc,
                                         const uint8_t* w, const uint8_t* s, const uint8_t* b, bool valid) {
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const bool ok = valid && lc.ok[i];
    f.w[i] = ok ? *reinterpret_cast<const uint4*>(w + lc.off[i]) : make_uint4(0, 0, 0, 0);
    if constexpr (BITS != 0) {
      f.s[i] = ok ? sm_scalar<DT>(s, lc.grp[i]) : 0.f;
      f.b[i] = ok ? sm_scalar<DT>(b, lc.grp[i]) : 0.f;
    }
  }
}

// Bytes of n rows of one matrix in a slot (weights + scales + biases).
template <int BITS, int DT>
__device__ __forceinline__ unsigned sl_bytes(const SliceTab& T, int n) {
  const unsigned w = unsigned(n) * unsigned(T.rb);
  return BITS != 0 ? w + 2u * unsigned(n) * unsigned(T.srow * SliceFmt<BITS, DT>::SB) : w;
}
// Issues the bulk copies of rows [row, row + n) of one matrix into a slot
// laid out as [TR rows of weights][TR rows of scales][TR rows of biases].
template <int BITS, int DT>
__device__ __forceinline__ void sl_copy(const SliceTab& T, uint8_t* d, uint64_t* bar, const uint8_t* w,
                                        const uint8_t* s, const uint8_t* b, int row, int n, uint64_t pol) {
  constexpr int SB = SliceFmt<BITS, DT>::SB;
  bulk_g2s(d, w + int64_t(row) * T.rb, unsigned(n) * unsigned(T.rb), bar, pol);
  if constexpr (BITS != 0) {
    const int ss = T.srow * SB;
    bulk_g2s(d + T.TR * T.rb, s + int64_t(row) * ss, unsigned(n * ss), bar, pol);
    bulk_g2s(d + T.TR * T.rb + T.TR * ss, b + int64_t(row) * ss, unsigned(n * ss), bar, pol);
  }
}
// Before the producer exits: no copy of this CTA may still be in flight.
// Tiles older than the last S were consumed (their slots were reused).
__device__ __forceinline__ void sl_drain(uint64_t* full, int S, int issued) {
  for (int k = max(0, issued - S); k < issued; ++k) mbar_wait(full + (k % S), unsigned(k / S) & 1u);
}
__device__ __forceinline__ void sl_init_barriers(uint64_t* full, uint64_t* empty, int S) {
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, SL_CW);
    }
    mbar_init_fence();
  }
  __syncthreads();
}

// Sum over the NT consumer threads; `red` holds >= NT / 32 floats.
template <int NT = SL_NT>
__device__ __forceinline__ float sl_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  bar_sync_n(NT);
  if (l == 0) red[w] = v;
  bar_sync_n(NT);
  v = l < NT / 32 ? red[l] : 0.f;
  return warp_sum(v);
}

// Pre-scaled, chunk-interleaved copy (xs) and chunk sums (cs) of n plain
// values in shared memory (consumer threads; the caller synchronises before
// and after). Work item idx covers float4 jq of chunk c with c = idx % nch and
// jq rotated by c, so that consecutive threads read and write distinct bank
// groups; each chunk sum reads its chunk in the same rotated order.
template <int BITS, int DT, int NT = SL_NT>
__device__ __forceinline__ void sl_interleave(const float* plain, int n, float* xs, float* cs) {
  constexpr int WPC = ChunkInfo<BITS, DT>::WPC, Q = WPC / 4;
  const int tid = threadIdx.x, nch = n / WPC;
  const float4* p4 = reinterpret_cast<const float4*>(plain);
  float4* x4 = reinterpret_cast<float4*>(xs);
  for (int idx = tid; idx < nch * Q; idx += NT) {
    const int c = idx % nch, jq = (idx / nch + c) % Q;
    float4 v = p4[c * Q + jq];
    if constexpr (BITS != 0) {
      const int k = (c * Q + jq) * 4;
      v.x *= prescale<BITS>(k);
      v.y *= prescale<BITS>(k + 1);
      v.z *= prescale<BITS>(k + 2);
      v.w *= prescale<BITS>(k + 3);
    }
    x4[jq * nch + c] = v;
  }
  if constexpr (BITS != 0) {
    for (int c = tid; c < nch; c += NT) {
      float s = 0.f;
#pragma unroll
      for (int t = 0; t < Q; ++t) {
        const float4 v = p4[c * Q + (t + c) % Q];
        s += (v.x + v.y) + (v.z + v.w);
      }
      cs[c] = s;
    }
  }
}

__device__ __forceinline__ float4 f4_zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }
__device__ __forceinline__ float f4_sq(const float4 v) { return (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w); }

// Consumer-side staging of the input vector (in <= 4096, 16-byte aligned
// inputs): every float4 is loaded in one round trip (float4 i*SL_NT + tid goes
// to register i), transformed (Prologue) and written plain to `plain` (in
// floats of shared memory; sl_stage then interleaves it into xs / cs). red
// holds SL_RED floats.
template <int NT = SL_NT>
__device__ __forceinline__ void sl_stage_plain(const GemvArgs& a, float* red, float* plain) {
  constexpr int MAXQ = 4096 / (4 * NT);
  const int in = a.in, nq = in >> 2, tid = threadIdx.x, lane = tid & 31;
  const bool norm = a.prologue == PRO_RMSNORM, gated = a.prologue == PRO_GATEDNORM;
  const float4* x4 = reinterpret_cast<const float4*>(a.x);
  const float4* u4 = reinterpret_cast<const float4*>(a.aux);
  const float4* w4 = reinterpret_cast<const float4*>(a.aux2);
  const int hq = gated ? a.head_dim >> 2 : 1;
  float4 v[MAXQ], u[MAXQ], w[MAXQ];
#pragma unroll
  for (int i = 0; i < MAXQ; ++i) {
    const int q = i * NT + tid;
    const bool ok = q < nq;
    v[i] = ok ? __ldcg(x4 + q) : f4_zero();
    u[i] = ok && (norm || gated) ? __ldcg(u4 + q) : f4_zero();
    w[i] = ok && gated ? __ldcg(w4 + q % hq) : f4_zero();
  }
  if (norm) {
    // QwenCPUModel.rmsNorm (QwenCPUModel.swift:47-59)
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXQ; ++i) ss += f4_sq(v[i]);
    ss = sl_sum<NT>(ss, red);
    const float scale = 1.f / sqrtf(ss / float(in) + a.eps);
#pragma unroll
    for (int i = 0; i < MAXQ; ++i) {
      v[i].x = v[i].x * (scale * u[i].x);
      v[i].y = v[i].y * (scale * u[i].y);
      v[i].z = v[i].z * (scale * u[i].z);
      v[i].w = v[i].w * (scale * u[i].w);
    }
  } else if (gated) {
    // DeltaNet output gate (QwenCPUModel.swift:490-493): per head RMSNorm with
    // weight, times silu(z) (u holds silu(z)). Eight lanes hold 32 consecutive
    // values of one head (head_dim % 32 == 0): three shuffle rounds give the
    // segment's sum of squares; one thread per head then forms its scale.
    float* hs = red + 32;         // [in / 32] segment sums of squares
    float* hsc = red + 32 + 128;  // [in / head_dim] head scales
    float q2[MAXQ];
#pragma unroll
    for (int i = 0; i < MAXQ; ++i) q2[i] = f4_sq(v[i]);
#pragma unroll
    for (int o = 1; o < 8; o <<= 1)
#pragma unroll
      for (int i = 0; i < MAXQ; ++i) q2[i] += __shfl_xor_sync(0xffffffffu, q2[i], o);
#pragma unroll
    for (int i = 0; i < MAXQ; ++i) {
      const int q = i * NT + tid;
      if ((lane & 7) == 0 && q < nq) hs[q >> 3] = q2[i];
    }
    bar_sync_n(NT);
    const int hd = a.head_dim, per = hd >> 5, nh = in / hd;
    for (int h = tid; h < nh; h += NT) {
      float t = 0.f;
      for (int p = 0; p < per; ++p) t += hs[h * per + p];
      hsc[h] = 1.f / sqrtf(t / float(hd) + a.eps);
    }
    bar_sync_n(NT);
#pragma unroll
    for (int i = 0; i < MAXQ; ++i) {
      const int q = i * NT + tid;
      const float sc = q < nq ? hsc[q / hq] : 0.f;
      v[i].x = (v[i].x * (sc * w[i].x)) * u[i].x;
      v[i].y = (v[i].y * (sc * w[i].y)) * u[i].y;
      v[i].z = (v[i].z * (sc * w[i].z)) * u[i].z;
      v[i].w = (v[i].w * (sc * w[i].w)) * u[i].w;
    }
  }
  float4* p4 = reinterpret_cast<float4*>(plain);
  float4* o4 = (a.x_out && blockIdx.x == 0) ? reinterpret_cast<float4*>(a.x_out) : nullptr;
#pragma unroll
  for (int i = 0; i < MAXQ; ++i) {
    const int q = i * NT + tid;
    if (q < nq) {
      p4[q] = v[i];
      if (o4) o4[q] = v[i];
    }
  }
  bar_sync_n(NT);
}

template <int BITS, int DT>
__device__ __forceinline__ void sl_stage(const GemvArgs& a, float* xs, float* cs, float* red, float* plain) {
  sl_stage_plain(a, red, plain);
  sl_interleave<BITS, DT>(plain, a.in, xs, cs);
  bar_sync_n(SL_NT);
}

// Router epilogue (last CTA, consumer threads): softmax over E, top-k, combine
// weights (QwenCPUModel.swift:506-521, 546-550; routerPicks
// QwenMetalModel.swift:875-892). p holds E floats of shared memory.
template <int NT = SL_NT>
__device__ __forceinline__ void sl_router_tail(const RouterTail& rt, float* p, float* red) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, E = rt.E;
  float m = -INFINITY;
  for (int e = tid; e < E; e += NT) {
    p[e] = __ldcg(rt.logits + e);
    m = fmaxf(m, p[e]);
  }
  m = warp_max(m);
  bar_sync_n(NT);
  if (lane == 0) red[warp] = m;
  bar_sync_n(NT);
  m = -INFINITY;
  for (int w = 0; w < (NT / 32); ++w) m = fmaxf(m, red[w]);
  float sum = 0.f;
  for (int e = tid; e < E; e += NT) {
    p[e] = expf(p[e] - m);
    sum += p[e];
  }
  sum = sl_sum<NT>(sum, red + 8);
  for (int e = tid; e < E; e += NT) p[e] = p[e] / sum;
  bar_sync_n(NT);
  if (warp != 0) return;
  // top-k by repeated warp argmax; ties keep the lower expert id, the outcome
  // of the reference's insertion scan with a strict `>` (:516).
  __shared__ int ki[64];
  __shared__ float kp[64];
  for (int k = 0; k < rt.topk; ++k) {
    float bv = -1.f;
    int bi = 0x7fffffff;
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
    float score_sum = 0.f;
    for (int k = 0; k < rt.topk; ++k) score_sum += kp[k];
    for (int k = 0; k < rt.topk; ++k) {
      rt.pick_ids[k] = ki[k];
      rt.pick_w[k] = rt.norm_topk ? kp[k] / score_sum : kp[k];
    }
    *rt.shared_scale = sigmoid_ref(__ldcg(rt.logits + E));
    *rt.counter = 0u;
  }
}

// Greedy argmax over the rows this CTA wrote (consumer threads; (bv, bi) is
// the thread's best): per-CTA best, then the last CTA reduces them (first
// index wins on ties, TextGenerator.swift:90).
template <int NT = SL_NT>
__device__ __forceinline__ void sl_argmax_tail(const GemvArgs& a, float bv, int bi, float* red) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  int* ired = reinterpret_cast<int*>(red);
  bar_sync_n(NT);
  if (lane == 0) { red[warp] = bv; ired[8 + warp] = bi; }
  __threadfence();
  bar_sync_n(NT);
  if (tid == 0) {
    for (int w = 1; w < (NT / 32); ++w)
      if (red[w] > bv || (red[w] == bv && ired[8 + w] < bi)) { bv = red[w]; bi = ired[8 + w]; }
    a.argmax_val[blockIdx.x] = bv;
    a.argmax_idx[blockIdx.x] = bi;
    __threadfence();
    ired[16] = atomicAdd(a.counter, 1u) == gridDim.x - 1;
  }
  bar_sync_n(NT);
  if (ired[16] && warp == 0) {
    __threadfence();
    float gv = -INFINITY;
    int gi = 0x7fffffff;
    for (int b = lane; b < int(gridDim.x); b += 32) {
      const float v = __ldcg(a.argmax_val + b);
      const int i = __ldcg(a.argmax_idx + b);
      if (v > gv || (v == gv && i < gi)) { gv = v; gi = i; }
    }
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, gv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, gi, o);
      if (ov > gv || (ov == gv && oi < gi)) { gv = ov; gi = oi; }
    }
    if (lane == 0) {
      *a.argmax_out = gi;
      *a.counter = 0u;
    }
  }
}

// Router epilogue trigger: the last CTA to finish runs sl_router_tail.
template <int NT = SL_NT>
__device__ __forceinline__ void sl_router_done(const RouterTail& rt, float* p, float* red) {
  const int tid = threadIdx.x;
  int* ired = reinterpret_cast<int*>(red);
  __threadfence();
  bar_sync_n(NT);
  if (tid == 0) ired[16] = atomicAdd(rt.counter, 1u) == gridDim.x - 1;
  bar_sync_n(NT);
  if (ired[16]) {
    __threadfence();
    sl_router_tail<NT>(rt, p, red);
  }
}

// ------------------------------------------------------------ dense GEMV --
// y_seg[row] (=|+=) W_seg[row] . prologue(x) over the rows [b*rpc, (b+1)*rpc)
// of the concatenated segments; optional fused greedy argmax over segment 0
// (first index wins on ties, TextGenerator.swift:90) and router epilogue.
template <int BITS, int DT, int R>
__global__ void __launch_bounds__(SL_T, 2) k_sgemv(const GemvArgs a, const SliceTab T, const RouterTail rt) {
  using F = SliceFmt<BITS, DT>;
  constexpr int CPL = F::CPL, SB = F::SB;
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* ring = sm;
  float* xs = reinterpret_cast<float*>(sm + T.off_xs);
  float* cs = reinterpret_cast<float*>(sm + T.off_cs);
  float* red = reinterpret_cast<float*>(sm + T.off_red);
  float* part = reinterpret_cast<float*>(sm + T.off_part);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + T.off_bar);
  uint64_t* empty = full + T.S;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r0 = blockIdx.x * T.rpc, r1 = min(T.total, r0 + T.rpc);
  // The CTA's tiles: TR-row pieces of [r0, r1) inside one segment each.
  auto tiles = [&](auto&& f) {
    int idx = 0;
    for (int sg = 0; sg < T.nseg; ++sg) {
      const int a0 = max(r0, T.cum[sg]), a1 = min(r1, T.cum[sg + 1]);
      for (int r = a0; r < a1; r += T.TR) f(idx++, sg, r - T.cum[sg], min(T.TR, a1 - r), r - r0);
    }
  };
  sl_init_barriers(full, empty, T.S);
  if (warp == SL_CW) {  // producer
    if (lane == 0) {
      const uint64_t pol = l2_evict_first();
      int issued = 0;
      bool ok = true;
      tiles([&](int i, int sg, int row, int n, int) {
        if (!ok) return;
        const int s = i % T.S;
        if (i >= T.S && !mbar_wait(empty + s, unsigned(i / T.S - 1) & 1u)) { ok = false; return; }
        mbar_expect_tx(full + s, sl_bytes<BITS, DT>(T, n));
        sl_copy<BITS, DT>(T, ring + size_t(s) * T.slot, full + s, seg_pick(T.w, sg), seg_pick(T.s, sg),
                          seg_pick(T.b, sg), row, n, pol);
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
  sl_stage<BITS, DT>(a, xs, cs, red, reinterpret_cast<float*>(sm + T.off_raw));
  pdl_launch();
  const int LPR = T.LPR, spw = 32 / LPR, subw = lane / LPR, sl = lane % LPR;
  const int gw = SL_CW / T.W, g = warp / gw, j = (warp % gw) * spw + subw;
  const int nch = T.rb >> 4, c0 = g * LPR * CPL + sl, ss = T.srow * SB;
  XRegs<BITS, DT, CPL> xr;
  xr.load(XTile{reinterpret_cast<const float4*>(xs), cs, nch}, c0, LPR);
  trc.staged(a.trace);
  LaneChunks<BITS, DT, CPL> lc;
  lc.init(c0, LPR, nch, T.gs_shift);
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  auto epi = [&](int sg, int row, float v) {
    float* y = seg_pick(T.y, sg);
    if (a.epilogue == EPI_RESIDUAL) y[row] += v;
    else y[row] = v;
    if (sg == 0 && (v > bv || (v == bv && row < bi))) { bv = v; bi = row; }
  };
  bool dead = false;
  tiles([&](int i, int sg, int row, int n, int lo) {
    if (dead) return;
    const int s = i % T.S;
    if (!__all_sync(0xffffffffu, mbar_wait(full + s, unsigned(i / T.S) & 1u))) { dead = true; return; }
    const uint8_t* wt = ring + size_t(s) * T.slot;
    const uint8_t* st = wt + T.TR * T.rb;
    const uint8_t* bt = st + T.TR * ss;
    float p[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int rl = j * R + r;
      RowFrag<BITS, DT, CPL> f;
      smem_row(f, lc, wt + rl * T.rb, st + rl * ss, bt + rl * ss, rl < n);
      p[r] = dot_row<BITS, DT, CPL>(f, xr);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + s);
    int rr;
    const float v = reduce_rows<R>(p, LPR, sl, rr);
    const int rl = j * R + rr;
    if ((sl & (LPR / R - 1)) == 0 && rl < n) {
      if (T.W == 1) epi(sg, row + rl, v);
      else part[g * T.rpc + lo + rl] = v;
    }
  });
  trc.looped(a.trace);
  if (dead) sl_fail(T);
  if (T.W > 1) {
    bar_sync_n(SL_NT);
    for (int rl = tid; rl < r1 - r0; rl += SL_NT) {
      float v = 0.f;
      for (int q = 0; q < T.W; ++q) v += part[q * T.rpc + rl];
      const int row = r0 + rl;
      int sg = 0;
      while (sg + 1 < T.nseg && row >= T.cum[sg + 1]) ++sg;
      epi(sg, row - T.cum[sg], v);
    }
  }
  if (a.argmax_out) sl_argmax_tail(a, bv, bi, red);
  if (rt.logits) sl_router_done(rt, xs, red);
  trc.end(a.trace);
}

// ---------------------------------------------------------------- MoE ----
// Gate/up of the shared expert and the K routed experts with SiLU * up
// fused (encodePendingMoE QwenMetalModel.swift:806-841; QwenCPUModel.swift:
// 552-561). CTA b owns shared rows [b*sh_rpc, ...) and routed rows
// [b*rt_rpc, ...) of the K*inter routed rows; the shared tiles are copied
// before the dependency wait, the routed ones once the router is done. A
// slot holds TR gate rows, then TR up rows at slot/2.
constexpr int GR = 2;  // gate/up row pairs per sub-warp and tile

template <int BITS, int DT>
__global__ void __launch_bounds__(SL_T, 2) k_sgateup(const MoeArgs m, const SliceTab T) {
  using F = SliceFmt<BITS, DT>;
  constexpr int CPL = F::CPL, SB = F::SB;
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* ring = sm;
  float* xs = reinterpret_cast<float*>(sm + T.off_xs);
  float* cs = reinterpret_cast<float*>(sm + T.off_cs);
  float* red = reinterpret_cast<float*>(sm + T.off_red);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + T.off_bar);
  uint64_t* empty = full + T.S;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = m.topk, inter = m.g.lin.out, sh = m.sg.out, nq = K * inter;
  const int s0 = min(sh, int(blockIdx.x) * T.sh_rpc), s1 = min(sh, s0 + T.sh_rpc);
  const int q0 = min(nq, int(blockIdx.x) * T.rt_rpc), q1 = min(nq, q0 + T.rt_rpc);
  auto tiles = [&](auto&& f) {  // f(tile, slot (K = shared), row, n)
    int idx = 0;
    for (int r = s0; r < s1; r += T.TR) f(idx++, K, r, min(T.TR, s1 - r));
    for (int q = q0; q < q1;) {
      const int k = q / inter, row = q - k * inter;
      const int n = min(T.TR, min(q1 - q, inter - row));
      f(idx++, k, row, n);
      q += n;
    }
  };
  const int half = T.slot / 2;
  sl_init_barriers(full, empty, T.S);
  if (warp == SL_CW) {  // producer
    if (lane == 0) {
      const uint64_t pol = l2_evict_first();
      int issued = 0;
      bool ok = true, waited = false;
      tiles([&](int i, int k, int row, int n) {
        if (!ok) return;
        if (k < K && !waited) { pdl_wait(); waited = true; }  // routing comes from the previous grid
        const int s = i % T.S;
        if (i >= T.S && !mbar_wait(empty + s, unsigned(i / T.S - 1) & 1u)) { ok = false; return; }
        QLin G = m.sg, U = m.su;
        if (k < K) {
          const int id = __ldcg(m.pick_ids + k);
          G = expert_lin(m.g, id);
          U = expert_lin(m.u, id);
        }
        uint8_t* d = ring + size_t(s) * T.slot;
        mbar_expect_tx(full + s, 2u * sl_bytes<BITS, DT>(T, n));
        sl_copy<BITS, DT>(T, d, full + s, G.w, G.s, G.b, row, n, pol);
        sl_copy<BITS, DT>(T, d + half, full + s, U.w, U.s, U.b, row, n, pol);
        issued = i + 1;
      });
      // Dependents are released only after the router grid is complete: the
      // down kernel reads the routing before its own dependency wait.
      if (!waited) pdl_wait();
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
  GemvArgs a;
  a.in = m.g.lin.in; a.prologue = PRO_COPY; a.x = m.x;
  sl_stage<BITS, DT>(a, xs, cs, red, reinterpret_cast<float*>(sm + T.off_raw));
  pdl_launch();
  const int LPR = T.LPR, spw = 32 / LPR, subw = lane / LPR, sl = lane % LPR;
  const int j = warp * spw + subw;
  const int nch = T.rb >> 4, ss = T.srow * SB;
  XRegs<BITS, DT, CPL> xr;
  xr.load(XTile{reinterpret_cast<const float4*>(xs), cs, nch}, sl, LPR);
  trc.staged(m.trace);
  LaneChunks<BITS, DT, CPL> lc;
  lc.init(sl, LPR, nch, T.gs_shift);
  bool dead = false;
  tiles([&](int i, int k, int row, int n) {
    if (dead) return;
    const int s = i % T.S;
    if (!__all_sync(0xffffffffu, mbar_wait(full + s, unsigned(i / T.S) & 1u))) { dead = true; return; }
    const uint8_t* gt = ring + size_t(s) * T.slot;
    const uint8_t* ut = gt + half;
    const int so = T.TR * T.rb, bo = T.TR * T.rb + T.TR * ss;
    float p[2 * GR];  // GR gate rows, then the same GR up rows
#pragma unroll
    for (int r = 0; r < GR; ++r) {
      const int rl = j * GR + r;
      RowFrag<BITS, DT, CPL> fg, fu;
      smem_row(fg, lc, gt + rl * T.rb, gt + so + rl * ss, gt + bo + rl * ss, rl < n);
      smem_row(fu, lc, ut + rl * T.rb, ut + so + rl * ss, ut + bo + rl * ss, rl < n);
      p[r] = dot_row<BITS, DT, CPL>(fg, xr);
      p[GR + r] = dot_row<BITS, DT, CPL>(fu, xr);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + s);
    int rr;
    const float v = reduce_rows<2 * GR>(p, LPR, sl, rr);
    // the first exchange round (lane bit LPR/2) split gate rows from up rows
    const float uv = __shfl_xor_sync(0xffffffffu, v, LPR >> 1);
    const int rl = j * GR + rr;
    if (rr < GR && (sl & (LPR / (2 * GR) - 1)) == 0 && rl < n)
      m.hmid[k * m.hmid_stride + row + rl] = silu_ref(v) * uv;
  });
  trc.looped(m.trace);
  if (dead) sl_fail(T);
  trc.end(m.trace);
}

// Down projections of the K routed experts and the shared expert for the
// CTA's output rows [b*rpc, ...), router-weighted combine and residual add
// (weighted_accum Kernels.metal.txt:463-478; QwenCPUModel.swift:555-566).
// Tile e holds expert slot e's rows of the CTA (slot K: the shared expert);
// warp e % SL_CW reduces it in items of DR rows per sub-warp into part[e][row]
// and the consumers finally combine part over the experts. Every weight is
// known before the dependency wait: the routing was written by the router
// grid, which completed before this grid was launched (the gate/up grid
// releases its dependents only after its own wait on the router).
constexpr int DR = 4;  // rows per down work item

template <int BITS, int DT>
__global__ void __launch_bounds__(SL_T, 2) k_sdown(const MoeArgs m, const SliceTab T) {
  using F = SliceFmt<BITS, DT>;
  constexpr int CPL = F::CPL, SB = F::SB, WPC = F::WPC;
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* ring = sm;
  float* xs = reinterpret_cast<float*>(sm + T.off_xs);
  float* cs = reinterpret_cast<float*>(sm + T.off_cs);
  float* part = reinterpret_cast<float*>(sm + T.off_part);
  float* raw = reinterpret_cast<float*>(sm + T.off_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + T.off_bar);
  uint64_t* empty = full + T.S;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = m.topk, D = m.d.lin.out, inter = m.d.lin.in;
  const int o0 = int(blockIdx.x) * T.rpc, o1 = min(D, o0 + T.rpc), nrow = o1 - o0;
  sl_init_barriers(full, empty, T.S);
  if (warp == SL_CW) {  // producer
    if (lane == 0) {
      const uint64_t pol = l2_evict_first();
      int issued = 0;
      bool ok = true;
      for (int e = 0; e <= K && ok; ++e) {
        const int s = e % T.S;
        if (e >= T.S && !mbar_wait(empty + s, unsigned(e / T.S - 1) & 1u)) { ok = false; break; }
        const QLin L = e < K ? expert_lin(m.d, __ldcg(m.pick_ids + e)) : m.sd;
        mbar_expect_tx(full + s, sl_bytes<BITS, DT>(T, nrow));
        sl_copy<BITS, DT>(T, ring + size_t(s) * T.slot, full + s, L.w, L.s, L.b, o0, nrow, pol);
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
  // stage the K + 1 SwiGLU outputs: one asynchronous round trip, then the
  // chunk-interleaved layout per expert slot
  const int xstride = m.hmid_stride, cstride = m.hmid_stride / WPC + 4, nch = T.rb >> 4;
  const int nfl = (K + 1) * m.hmid_stride;
  for (int i = tid; i < (nfl >> 2); i += SL_NT) cp_async16(raw + 4 * i, m.hmid + 4 * i);
  cp_async_wait_all();
  bar_sync_n(SL_NT);
  for (int e = 0; e <= K; ++e) sl_interleave<BITS, DT>(raw + e * m.hmid_stride, inter, xs + e * xstride, cs + e * cstride);
  bar_sync_n(SL_NT);
  pdl_launch();
  trc.staged(m.trace);
  const int LPR = T.LPR, spw = 32 / LPR, subw = lane / LPR, sl = lane % LPR, ss = T.srow * SB;
  const int G = (nrow + DR - 1) / DR, rounds = (G + spw - 1) / spw;
  LaneChunks<BITS, DT, CPL> lc;
  lc.init(sl, LPR, nch, T.gs_shift);
  bool dead = false;
  for (int e = 0; e <= K && !dead; ++e) {
    const int s = e % T.S;
    if (!__all_sync(0xffffffffu, mbar_wait(full + s, unsigned(e / T.S) & 1u))) { dead = true; break; }
    if (e % SL_CW == warp) {
      const uint8_t* dt = ring + size_t(s) * T.slot;
      XRegs<BITS, DT, CPL> xr;
      xr.load(XTile{reinterpret_cast<const float4*>(xs + e * xstride), cs + e * cstride, nch}, sl, LPR);
      for (int q = 0; q < rounds; ++q) {
        const int g = q * spw + subw;
        float p[DR];
#pragma unroll
        for (int r = 0; r < DR; ++r) {
          const int rl = g * DR + r;
          RowFrag<BITS, DT, CPL> f;
          smem_row(f, lc, dt + rl * T.rb, dt + T.TR * T.rb + rl * ss, dt + T.TR * T.rb + T.TR * ss + rl * ss,
                   rl < nrow);
          p[r] = dot_row<BITS, DT, CPL>(f, xr);
        }
        int rr;
        const float v = reduce_rows<DR>(p, LPR, sl, rr);
        const int rl = g * DR + rr;
        if ((sl & (LPR / DR - 1)) == 0 && rl < nrow) part[e * T.rpc + rl] = v;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + s);
  }
  trc.looped(m.trace);
  if (dead) sl_fail(T);
  bar_sync_n(SL_NT);
  for (int rl = tid; rl < nrow; rl += SL_NT) {
    float acc = 0.f;
    for (int e = 0; e <= K; ++e)
      acc = fmaf(e < K ? __ldcg(m.pick_w + e) : __ldcg(m.shared_scale), part[e * T.rpc + rl], acc);
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
template <int B, int D>
void sgemv_fmt(const GemvArgs& a, const SliceTab& T, const RouterTail& rt, int R, int grid, size_t smem,
               cudaStream_t st, bool pdl) {
  if (R == 4) launch(k_sgemv<B, D, 4>, dim3(grid), dim3(SL_T), smem, st, pdl, a, T, rt);
  else launch(k_sgemv<B, D, 1>, dim3(grid), dim3(SL_T), smem, st, pdl, a, T, rt);
}
template <int B, int D>
void sgateup_fmt(const MoeArgs& m, const SliceTab& T, int grid, size_t smem, cudaStream_t st, bool pdl) {
  launch(k_sgateup<B, D>, dim3(grid), dim3(SL_T), smem, st, pdl, m, T);
}
template <int B, int D>
void sdown_fmt(const MoeArgs& m, const SliceTab& T, int grid, size_t smem, cudaStream_t st, bool pdl) {
  launch(k_sdown<B, D>, dim3(grid), dim3(SL_T), smem, st, pdl, m, T);
}

#define SWL_INSTANTIATE_SLICE(B, D)                                                                                    \
  template void sgemv_fmt<B, D>(const GemvArgs&, const SliceTab&, const RouterTail&, int, int, size_t, cudaStream_t,   \
                                bool);                                                                                 \
  template void sgateup_fmt<B, D>(const MoeArgs&, const SliceTab&, int, size_t, cudaStream_t, bool);                   \
  template void sdown_fmt<B, D>(const MoeArgs&, const SliceTab&, int, size_t, cudaStream_t, bool);

}  // namespace swl
