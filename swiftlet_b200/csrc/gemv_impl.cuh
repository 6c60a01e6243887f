// Weight-streaming kernels of the decode step (templates; instantiated per
// weight format in gemv_fmt_*.cu): multi-segment GEMV (dense projections,
// lm_head with fused greedy argmax), router + top-k, and the fused
// routed/shared expert SwiGLU (gate/up, then down + combine + residual).
//
// Structure shared by all four (B = 1 decode is latency bound):
//   * grids are one wave (all CTAs resident), so a CTA can signal
//     griddepcontrol.launch_dependents right after its prologue: the next
//     kernel's CTAs then start on the free half of each SM and load their
//     first weights while this kernel streams;
//   * weights never depend on the previous kernel, so each sub-warp loads
//     its first task's weights BEFORE griddepcontrol.wait;
//   * a sub-warp of LPR lanes owns a task of R rows; lane l always handles
//     chunks l, l + LPR, ... of a row, so its per-chunk offsets, group
//     indices and (for rows of <= 64 chunks... CPL <= 2) its slice of x are
//     computed or loaded once and every row streams past them.
#pragma once

#include <algorithm>

#include "kcommon.cuh"
#include "kernels.h"
#include "launch.h"

namespace swl {

constexpr int GT = 128;  // threads per block

// Lean, per-launch description of up to four same-format matrices.
struct SegTab {
  const uint8_t* w[4];
  const uint8_t* s[4];
  const uint8_t* b[4];
  float* y[4];
  int task0[5];  // cumulative task starts (R rows per task)
  int rows[4];
  int nseg;
};

// Per-lane constants of a row walk: chunk byte offsets, scale/bias group
// index, validity (nslab = 1: the lane's chunks are the same for every row).
template <int BITS, int DT, int CPL>
struct LaneChunks {
  int off[CPL];  // byte offset of the chunk in the row
  int grp[CPL];  // group index of the chunk in the row
  bool ok[CPL];
  __device__ __forceinline__ void init(int c0, int LPR, int nch, int gs_shift) {
    constexpr int WPC = ChunkInfo<BITS, DT>::WPC;
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      const int c = c0 + i * LPR;
      ok[i] = c < nch;
      off[i] = c << 4;
      grp[i] = (c * WPC) >> gs_shift;
    }
  }
};

// Loads R consecutive rows starting at wrow / srow_s / srow_b (row strides
// rb bytes and sr scale entries).
template <int BITS, int DT, int R, int CPL>
__device__ __forceinline__ void load_rows(RowFrag<BITS, DT, CPL> (&f)[R], const LaneChunks<BITS, DT, CPL>& lc,
                                          const uint8_t* wrow, const uint8_t* sbase, const uint8_t* bbase, int rb,
                                          int sr, int nr) {
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      const bool ok = r < nr && lc.ok[i];
      f[r].w[i] = ok ? ld_stream(wrow + r * rb + lc.off[i]) : make_uint4(0, 0, 0, 0);
      if constexpr (BITS != 0) {
        const int idx = r * sr + lc.grp[i];
        f[r].s[i] = ok ? load_scalar(sbase, DT, idx) : 0.f;
        f[r].b[i] = ok ? load_scalar(bbase, DT, idx) : 0.f;
      }
    }
}

// ------------------------------------------------------------ dense GEMV --
// Prologue of the dense GEMV: the inputs are copied to shared memory in one
// asynchronous round trip (raw), then x is transformed and staged (see
// Prologue). Shared layout: xs[in] | cs[in/WPC + 4] | red[32 + heads] |
// raw[in] | raw2[in] | raw3[head_dim].
template <int BITS, int DT>
__device__ __forceinline__ void stage_gemv_x(const GemvArgs& a, float* xs, float* cs, float* red, float* raw) {
  const int in = a.in;
  float* raw2 = raw + in;
  float* raw3 = raw2 + in;
  float* xo = (a.x_out && blockIdx.x == 0) ? a.x_out : nullptr;
  // GATEDNORM stages z and the norm weight only (y is read from global), so
  // the largest case (in = 4096) stays within 48 KB of shared memory.
  if (a.prologue == PRO_GATEDNORM) {
    raw2 = raw;
    raw3 = raw + in;
    copy_async(raw2, a.aux, in);
    copy_async(raw3, a.aux2, a.head_dim);
  } else {
    copy_async(raw, a.x, in);
    if (a.prologue == PRO_RMSNORM) copy_async(raw2, a.aux, in);
  }
  cp_async_wait_all();
  __syncthreads();
  if (a.prologue == PRO_RMSNORM) {
    float ss = 0.f;
    for (int k = threadIdx.x; k < in; k += blockDim.x) { const float v = raw[k]; ss += v * v; }
    ss = block_sum(ss, red);
    const float scale = 1.f / sqrtf(ss / float(in) + a.eps);  // QwenCPUModel.rmsNorm :47-59
    stage_vec<BITS, DT>(in, xs, cs, [&](int k) {
      const float v = raw[k] * (scale * raw2[k]);
      if (xo) xo[k] = v;
      return v;
    });
  } else if (a.prologue == PRO_GATEDNORM) {
    // DeltaNet output gate (QwenCPUModel.swift:490-493): per v-head RMSNorm
    // with weight, times silu(z) (aux holds silu(z), computed by the DeltaNet
    // kernel). Head scales first (one warp per head).
    float* hscale = red + 32;
    const int hd = a.head_dim, nh = in / hd, w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int h = w; h < nh; h += nw) {
      float ss = 0.f;
      for (int i = l; i < hd; i += 32) { const float v = a.x[h * hd + i]; ss += v * v; }
      ss = warp_sum(ss);
      if (l == 0) hscale[h] = 1.f / sqrtf(ss / float(hd) + a.eps);
    }
    __syncthreads();
    stage_vec<BITS, DT>(in, xs, cs, [&](int k) {
      const int h = k / hd;
      const float v = (a.x[k] * (hscale[h] * raw3[k - h * hd])) * raw2[k];
      if (xo) xo[k] = v;
      return v;
    });
  } else {
    stage_vec<BITS, DT>(in, xs, cs, [&](int k) {
      const float v = raw[k];
      if (xo) xo[k] = v;
      return v;
    });
  }
  __syncthreads();
}

struct TaskPtrs {
  const uint8_t* w;
  const uint8_t* s;
  const uint8_t* b;
  float* y;
  int row0, nr;
};

template <int R>
__device__ __forceinline__ TaskPtrs seg_task(const SegTab& T, int t, int rb, int sr, int sb) {
  int k = 0;
  if (T.nseg > 1 && t >= T.task0[1]) k = 1;
  if (T.nseg > 2 && t >= T.task0[2]) k = 2;
  if (T.nseg > 3 && t >= T.task0[3]) k = 3;
  TaskPtrs p;
  const int tb = t - (k == 0 ? 0 : k == 1 ? T.task0[1] : k == 2 ? T.task0[2] : T.task0[3]);
  const int rows = k == 0 ? T.rows[0] : k == 1 ? T.rows[1] : k == 2 ? T.rows[2] : T.rows[3];
  p.row0 = tb * R;
  p.nr = t < T.task0[T.nseg] ? min(R, rows - p.row0) : 0;
  const uint8_t* w = k == 0 ? T.w[0] : k == 1 ? T.w[1] : k == 2 ? T.w[2] : T.w[3];
  const uint8_t* s = k == 0 ? T.s[0] : k == 1 ? T.s[1] : k == 2 ? T.s[2] : T.s[3];
  const uint8_t* b = k == 0 ? T.b[0] : k == 1 ? T.b[1] : k == 2 ? T.b[2] : T.b[3];
  p.y = k == 0 ? T.y[0] : k == 1 ? T.y[1] : k == 2 ? T.y[2] : T.y[3];
  p.w = w + int64_t(p.row0) * rb;
  p.s = s + int64_t(p.row0) * sr * sb;
  p.b = b + int64_t(p.row0) * sr * sb;
  return p;
}

// Streams the tasks of a multi-segment GEMV. `prologue()` runs after the
// first task's weights are in flight and stages x (chunk-interleaved) in
// xs/cs; `epi(y, row, value)` consumes finished rows. Rows longer than
// CPL * LPR chunks are walked in nslab slabs.
template <int BITS, int DT, int R, int CPL, typename Pro, typename Epi>
__device__ __forceinline__ void gemv_stream(const SegTab& T, int rb, int sr, int gs_shift, int LPR, int nslab,
                                            const float* xs, const float* cs, Pro prologue, Epi epi) {
  using Frag = RowFrag<BITS, DT, CPL>;
  constexpr int SB = DT == DT_F32 ? 4 : 2;
  constexpr bool XR = CPL <= 2;  // lanes keep their x chunks in registers (nslab == 1)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int spw = 32 / LPR, subw = lane / LPR, sl = lane % LPR;
  const int nsub = gridDim.x * nw * spw;
  const int gsub = (blockIdx.x * nw + warp) * spw + subw;
  const int total = T.task0[T.nseg];
  const int iters = (total + nsub - 1) / nsub;
  const int nch = rb >> 4;
  const XTile xt{reinterpret_cast<const float4*>(xs), cs, nch};
  Frag f[R];
  LaneChunks<BITS, DT, CPL> lc;
  lc.init(sl, LPR, nch, gs_shift);
  auto load_task = [&](int t, int slab) {
    const TaskPtrs p = seg_task<R>(T, t, rb, sr, SB);
    LaneChunks<BITS, DT, CPL> ls = lc;
    if (slab) {
#pragma unroll
      for (int i = 0; i < CPL; ++i) {
        const int c = sl + (slab * CPL + i) * LPR;
        ls.ok[i] = c < nch;
        ls.off[i] = c << 4;
        ls.grp[i] = (c * ChunkInfo<BITS, DT>::WPC) >> gs_shift;
      }
    }
    load_rows<BITS, DT, R, CPL>(f, ls, p.w, p.s, p.b, rb, sr, p.nr);
  };
  if (iters > 0) load_task(gsub, 0);
  prologue();
  XRegs<BITS, DT, CPL> xr;
  if constexpr (XR) xr.load(xt, sl, LPR);
  for (int it = 0; it < iters; ++it) {
    const int t = gsub + it * nsub;
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.f;
    for (int slab = 0; slab < nslab; ++slab) {
      if (it > 0 || slab > 0) load_task(t, slab);
      const int c0 = sl + slab * CPL * LPR;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if constexpr (XR) acc[r] += dot_row<BITS, DT, CPL>(f[r], xr);
        else acc[r] += dot_row<BITS, DT, CPL>(f[r], xt, c0, LPR);
      }
    }
    const TaskPtrs p = seg_task<R>(T, t, rb, sr, SB);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float v = sub_sum(acc[r], LPR);
      if (sl == 0 && r < p.nr) epi(p.y, p.row0 + r, v);
    }
  }
}

template <int BITS, int DT, int R, int CPL>
__global__ void __launch_bounds__(GT) k_gemv(const GemvArgs a, const SegTab T, int gs_shift, int LPR, int nslab) {
  extern __shared__ __align__(16) float smem[];
  constexpr int WPC = ChunkInfo<BITS, DT>::WPC;
  float* xs = smem;
  float* cs = smem + a.in;
  float* red = cs + a.in / WPC + 4;
  float* raw = red + 32 + (a.prologue == PRO_GATEDNORM ? a.in / a.head_dim : 0);
  raw += (4 - (reinterpret_cast<uintptr_t>(raw) >> 2) % 4) % 4;  // 16-byte aligned
  const int rb = int(a.seg[0].lin.row_bytes), sr = int(a.seg[0].lin.srow);
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  TraceRec trc;
  trc.start(a.trace);
  gemv_stream<BITS, DT, R, CPL>(
      T, rb, sr, gs_shift, LPR, nslab, xs, cs,
      [&] {
        pdl_wait();
        trc.waited(a.trace);
        stage_gemv_x<BITS, DT>(a, xs, cs, red, raw);
        pdl_launch();
      },
      [&](float* y, int row, float v) {
        if (a.epilogue == EPI_RESIDUAL) y[row] += v;
        else y[row] = v;
        if (v > bv || (v == bv && row < bi)) { bv = v; bi = row; }
      });
  if (a.argmax_out) {
    // Fused greedy argmax over segment 0 (first index wins on ties, as the
    // reference's `logits[v] > logits[best]` scan, TextGenerator.swift:90).
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
      for (int w = 1; w < int(blockDim.x >> 5); ++w)
        if (wv[w] > bv || (wv[w] == bv && wi[w] < bi)) { bv = wv[w]; bi = wi[w]; }
      a.argmax_val[blockIdx.x] = bv;
      a.argmax_idx[blockIdx.x] = bi;
      __threadfence();
      last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (last && threadIdx.x < 32) {
      __threadfence();
      float gv = -INFINITY;
      int gi = 0x7fffffff;
      for (int b = threadIdx.x; b < int(gridDim.x); b += 32) {
        const float v = __ldcg(a.argmax_val + b);
        const int i = __ldcg(a.argmax_idx + b);
        if (v > gv || (v == gv && i < gi)) { gv = v; gi = i; }
      }
      for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, gv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, gi, o);
        if (ov > gv || (ov == gv && oi < gi)) { gv = ov; gi = oi; }
      }
      if (threadIdx.x == 0) {
        *a.argmax_out = gi;
        *a.counter = 0u;
      }
    }
  }
  trc.end(a.trace);
}

// ------------------------------------------------------------- router ----
// Post-attention RMSNorm + router GEMV + shared-expert gate logit; the last
// CTA computes softmax, top-k and the combine weights (QwenCPUModel.swift:
// 506-521, 546-550; routerPicks QwenMetalModel.swift:875-892).
template <int BITS, int DT, int R, int CPL>
__global__ void __launch_bounds__(GT) k_router(const RouterArgs ra, const SegTab T, int E, int gs_shift, int LPR,
                                               int nslab) {
  extern __shared__ __align__(16) float smem[];
  constexpr int WPC = ChunkInfo<BITS, DT>::WPC;
  const int D = ra.gate.in;
  float* xs = smem;
  float* cs = smem + D;
  float* red = cs + D / WPC + 4;
  float* raw = red + 32;
  raw += (4 - (reinterpret_cast<uintptr_t>(raw) >> 2) % 4) % 4;
  GemvArgs a;
  a.in = D; a.prologue = PRO_RMSNORM; a.x = ra.h; a.aux = ra.norm_w; a.eps = ra.eps; a.x_out = ra.x_out;
  TraceRec trc;
  trc.start(ra.trace);
  gemv_stream<BITS, DT, R, CPL>(
      T, int(ra.gate.row_bytes), int(ra.gate.srow), gs_shift, LPR, nslab, xs, cs,
      [&] {
        pdl_wait();
        trc.waited(ra.trace);
        stage_gemv_x<BITS, DT>(a, xs, cs, red, raw);
        pdl_launch();
      },
      [&](float* y, int row, float v) { y[row] = v; });
  __shared__ bool last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(ra.counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) {
    trc.end(ra.trace);
    return;
  }
  __threadfence();
  // softmax over E (max-subtracted, QwenCPUModel.softmaxRow :65-71)
  float* p = smem;
  __shared__ float red2[32];
  float m = -INFINITY;
  for (int e = threadIdx.x; e < E; e += blockDim.x) { p[e] = __ldcg(ra.logits + e); m = fmaxf(m, p[e]); }
  m = warp_max(m);
  __shared__ float wm[32];
  __syncthreads();
  if ((threadIdx.x & 31) == 0) wm[threadIdx.x >> 5] = m;
  __syncthreads();
  m = -INFINITY;
  for (int w = 0; w < int(blockDim.x >> 5); ++w) m = fmaxf(m, wm[w]);
  float sum = 0.f;
  for (int e = threadIdx.x; e < E; e += blockDim.x) { p[e] = expf(p[e] - m); sum += p[e]; }
  sum = block_sum(sum, red2);
  for (int e = threadIdx.x; e < E; e += blockDim.x) p[e] = p[e] / sum;
  __syncthreads();
  // top-k by repeated warp argmax; ties keep the lower expert id, which is
  // the outcome of the reference's insertion scan with a strict `>` (:516).
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    __shared__ int ki[64];
    __shared__ float kp[64];
    for (int k = 0; k < ra.topk; ++k) {
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
      for (int k = 0; k < ra.topk; ++k) score_sum += kp[k];
      for (int k = 0; k < ra.topk; ++k) {
        ra.pick_ids[k] = ki[k];
        ra.pick_w[k] = ra.norm_topk ? kp[k] / score_sum : kp[k];
      }
      *ra.shared_scale = sigmoid_ref(__ldcg(ra.logits + E));
      *ra.counter = 0u;
    }
  }
  trc.end(ra.trace);
}

// ---------------------------------------------------------------- MoE ----
__device__ __forceinline__ QLin expert_lin(const ExpertProj& p, int id) {
  QLin l = p.lin;
  l.w += int64_t(id) * p.wstride;
  l.s += int64_t(id) * p.sstride;
  l.b += int64_t(id) * p.bstride;
  return l;
}

// Gate/up of the shared expert and the K routed experts with SiLU * up
// fused (encodePendingMoE QwenMetalModel.swift:806-841; QwenCPUModel.swift:
// 552-561). Task order: shared expert rows first (their weights are known
// before the router finishes, so they are loaded before the wait).
template <int BITS, int DT, int R, int CPL>
__global__ void __launch_bounds__(GT) k_moe_gateup(const MoeArgs m, int gs_shift, int LPR, int tr, int ts, int nslab) {
  using Frag = RowFrag<BITS, DT, CPL>;
  extern __shared__ __align__(16) float smem[];
  constexpr bool XR = CPL <= 2;
  const int D = m.g.lin.in;
  float* xs = smem;
  float* cs = smem + D;
  const int total = ts + tr * m.topk;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int spw = 32 / LPR, subw = lane / LPR, sl = lane % LPR;
  const int nsub = gridDim.x * nw * spw;
  const int gsub = (blockIdx.x * nw + warp) * spw + subw;
  const int iters = (total + nsub - 1) / nsub;
  const int rb = int(m.g.lin.row_bytes), sr = int(m.g.lin.srow), nch = rb >> 4;
  const XTile xt{reinterpret_cast<const float4*>(xs), cs, nch};
  LaneChunks<BITS, DT, CPL> lc;
  lc.init(sl, LPR, nch, gs_shift);
  Frag fg[R], fu[R];
  struct Task { QLin G, U; int slot, row0, nr; };
  auto task = [&](int t) {
    Task k;
    if (t < ts) {
      k.G = m.sg; k.U = m.su; k.slot = m.topk; k.row0 = t * R;
    } else {
      const int tt = t - ts, slot = tt / tr;
      const int id = t < total ? m.pick_ids[slot] : 0;
      k.G = expert_lin(m.g, id); k.U = expert_lin(m.u, id); k.slot = slot; k.row0 = (tt - slot * tr) * R;
    }
    k.nr = t < total ? min(R, k.G.out - k.row0) : 0;
    return k;
  };
  constexpr int SB = DT == DT_F32 ? 4 : 2;
  auto load_task = [&](int t, int slab) {
    const Task k = task(t);
    LaneChunks<BITS, DT, CPL> ls = lc;
    if (slab) {
#pragma unroll
      for (int i = 0; i < CPL; ++i) {
        const int c = sl + (slab * CPL + i) * LPR;
        ls.ok[i] = c < nch;
        ls.off[i] = c << 4;
        ls.grp[i] = (c * ChunkInfo<BITS, DT>::WPC) >> gs_shift;
      }
    }
    const int64_t ro = int64_t(k.row0);
    load_rows<BITS, DT, R, CPL>(fg, ls, k.G.w + ro * rb, k.G.s + ro * sr * SB, k.G.b + ro * sr * SB, rb, sr, k.nr);
    load_rows<BITS, DT, R, CPL>(fu, ls, k.U.w + ro * rb, k.U.s + ro * sr * SB, k.U.b + ro * sr * SB, rb, sr, k.nr);
  };
  TraceRec trc;
  trc.start(m.trace);
  const bool early = iters > 0 && gsub < ts;  // shared-expert task: weights known now
  if (early) load_task(gsub, 0);
  pdl_wait();
  trc.waited(m.trace);
  if (!early && iters > 0) load_task(gsub, 0);
  float* raw = cs + D / ChunkInfo<BITS, DT>::WPC + 4;
  raw += (4 - (reinterpret_cast<uintptr_t>(raw) >> 2) % 4) % 4;
  copy_async(raw, m.x, D);
  cp_async_wait_all();
  __syncthreads();
  stage_vec<BITS, DT>(D, xs, cs, [&](int k) { return raw[k]; });
  __syncthreads();
  pdl_launch();
  XRegs<BITS, DT, CPL> xr;
  if constexpr (XR) xr.load(xt, sl, LPR);
  for (int it = 0; it < iters; ++it) {
    const int t = gsub + it * nsub;
    float ag[R], au[R];
#pragma unroll
    for (int r = 0; r < R; ++r) ag[r] = au[r] = 0.f;
    for (int slab = 0; slab < nslab; ++slab) {
      if (it > 0 || slab > 0) load_task(t, slab);
      const int c0 = sl + slab * CPL * LPR;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if constexpr (XR) {
          ag[r] += dot_row<BITS, DT, CPL>(fg[r], xr);
          au[r] += dot_row<BITS, DT, CPL>(fu[r], xr);
        } else {
          ag[r] += dot_row<BITS, DT, CPL>(fg[r], xt, c0, LPR);
          au[r] += dot_row<BITS, DT, CPL>(fu[r], xt, c0, LPR);
        }
      }
    }
    const Task k = task(t);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float gv = sub_sum(ag[r], LPR), uv = sub_sum(au[r], LPR);
      if (sl == 0 && r < k.nr) m.hmid[k.slot * m.hmid_stride + k.row0 + r] = silu_ref(gv) * uv;
    }
  }
  trc.end(m.trace);
}

// Down projections of the K routed experts + the shared expert for R output
// rows per sub-warp task, router-weighted combine and residual add
// (weighted_accum Kernels.metal.txt:463-478; QwenCPUModel.swift:555-566).
// All NE experts' chunks of the task's rows are in flight at once.
template <int BITS, int DT, int NE, int R>
__global__ void __launch_bounds__(GT) k_moe_down(const MoeArgs m, int gs_shift, int LPR, int nslab) {
  using Frag = RowFrag<BITS, DT, 1>;
  extern __shared__ __align__(16) float smem[];
  constexpr int WPC = ChunkInfo<BITS, DT>::WPC;
  constexpr int SB = DT == DT_F32 ? 4 : 2;
  const int K = m.topk, D = m.d.lin.out;
  const int xstride = m.hmid_stride, cstride = m.hmid_stride / WPC + 4;
  float* xs = smem;                    // [(K+1) * xstride]
  float* cs = xs + (K + 1) * xstride;  // [(K+1) * cstride]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int spw = 32 / LPR, subw = lane / LPR, sl = lane % LPR;
  const int nsub = gridDim.x * nw * spw;
  const int gsub = (blockIdx.x * nw + warp) * spw + subw;
  const int tasks = (D + R - 1) / R;
  const int iters = (tasks + nsub - 1) / nsub;
  const int rb = int(m.d.lin.row_bytes), sr = int(m.d.lin.srow), nch = rb >> 4;
  // routing was written two kernels back (router): complete before this grid started.
  // Routed experts differ only by the blob offset id * stride; -1 marks the shared expert.
  int64_t eoff[NE];
  float wts[NE];
#pragma unroll
  for (int e = 0; e < NE; ++e) {
    eoff[e] = e < K ? int64_t(m.pick_ids[e]) * m.d.wstride : -1;
    wts[e] = e < K ? m.pick_w[e] : (e == K ? *m.shared_scale : 0.f);
  }
  Frag f[NE][R];
  auto load_task = [&](int t, int slab) {
    const int row0 = t * R;
    const int nr = t < tasks ? min(R, D - row0) : 0;
    LaneChunks<BITS, DT, 1> lc;
    lc.init(sl + slab * LPR, LPR, nch, gs_shift);
    const int64_t ro = int64_t(row0);
#pragma unroll
    for (int e = 0; e < NE; ++e) {
      Frag(&fe)[R] = f[e];
      const bool routed = eoff[e] >= 0;
      const uint8_t* w = routed ? m.d.lin.w + eoff[e] : m.sd.w;
      const uint8_t* sp = routed ? m.d.lin.s + eoff[e] : m.sd.s;
      const uint8_t* bp = routed ? m.d.lin.b + eoff[e] : m.sd.b;
      load_rows<BITS, DT, R, 1>(fe, lc, w + ro * rb, sp + ro * sr * SB, bp + ro * sr * SB, rb, sr, e <= K ? nr : 0);
    }
  };
  TraceRec trc;
  trc.start(m.trace);
  if (iters > 0) load_task(gsub, 0);
  pdl_wait();
  trc.waited(m.trace);
  float* raw = cs + (K + 1) * cstride;
  raw += (4 - (reinterpret_cast<uintptr_t>(raw) >> 2) % 4) % 4;
  copy_async(raw, m.hmid, (K + 1) * m.hmid_stride);
  cp_async_wait_all();
  __syncthreads();
  for (int e = 0; e <= K; ++e) {
    const float* src = raw + e * m.hmid_stride;
    stage_vec<BITS, DT>(m.d.lin.in, xs + e * xstride, cs + e * cstride, [&](int k) { return src[k]; });
  }
  __syncthreads();
  pdl_launch();
  for (int it = 0; it < iters; ++it) {
    const int t = gsub + it * nsub;
    float part[R];
#pragma unroll
    for (int r = 0; r < R; ++r) part[r] = 0.f;
    for (int slab = 0; slab < nslab; ++slab) {
      if (it > 0 || slab > 0) load_task(t, slab);
      const int c0 = sl + slab * LPR;
#pragma unroll
      for (int e = 0; e < NE; ++e)
        if (e <= K) {
          const XTile xt{reinterpret_cast<const float4*>(xs + e * xstride), cs + e * cstride, nch};
#pragma unroll
          for (int r = 0; r < R; ++r) part[r] = fmaf(wts[e], dot_row<BITS, DT, 1>(f[e][r], xt, c0, LPR), part[r]);
        }
    }
    const int row0 = t * R;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float v = sub_sum(part[r], LPR);
      if (sl == 0 && t < tasks && row0 + r < D) m.h[row0 + r] += v;
    }
  }
  if (m.advance_sd && blockIdx.x == 0 && threadIdx.x == 0) {
    // Advance the sequence position and the token cursor once the last
    // layer of the step is done (no other CTA of this grid reads them;
    // dependents read them only after this grid completes).
    *m.advance_sd->pos += 1;
    *m.advance_cursor += 1;
  }
  trc.end(m.trace);
}

// ------------------------------------------------- per-format launchers --
// Formats on the hot path (4/8-bit with bf16 or f32 scales) get every
// rows-per-task x chunks-per-lane variant; the others run one generic
// variant (R = 1, CPL = 4: loads past the row end are predicated off).
template <int BITS, int DT>
struct FullFormat {
  static constexpr bool value = BITS != 0 && DT != DT_F16;
};

template <int B, int D>
void gemv_fmt(const GemvArgs& a, const SegTab& T, int R, int CPL, int gs_shift, int LPR, int nslab, int grid,
              size_t smem, cudaStream_t st, bool pdl) {
#define SWL_G(R_, C_) launch(k_gemv<B, D, R_, C_>, dim3(grid), dim3(GT), smem, st, pdl, a, T, gs_shift, LPR, nslab)
  if constexpr (FullFormat<B, D>::value) {
    if (R == 4) { if (CPL == 1) SWL_G(4, 1); else if (CPL == 2) SWL_G(4, 2); else SWL_G(4, 4); }
    else if (R == 2) { if (CPL == 1) SWL_G(2, 1); else if (CPL == 2) SWL_G(2, 2); else SWL_G(2, 4); }
    else { if (CPL == 1) SWL_G(1, 1); else if (CPL == 2) SWL_G(1, 2); else SWL_G(1, 4); }
  } else {
    SWL_G(1, 4);
  }
#undef SWL_G
}

template <int B, int D>
void router_fmt(const RouterArgs& r, const SegTab& T, int E, int CPL, int gs_shift, int LPR, int nslab, int grid,
                size_t smem, cudaStream_t st, bool pdl) {
#define SWL_R(C_) launch(k_router<B, D, 1, C_>, dim3(grid), dim3(GT), smem, st, pdl, r, T, E, gs_shift, LPR, nslab)
  if constexpr (FullFormat<B, D>::value) {
    if (CPL == 1) SWL_R(1); else if (CPL == 2) SWL_R(2); else SWL_R(4);
  } else {
    SWL_R(4);
  }
#undef SWL_R
}

template <int B, int D>
void gateup_fmt(const MoeArgs& m, int R, int CPL, int gs_shift, int LPR, int tr, int ts, int nslab, int grid,
                size_t smem, cudaStream_t st, bool pdl) {
#define SWL_U(R_, C_) launch(k_moe_gateup<B, D, R_, C_>, dim3(grid), dim3(GT), smem, st, pdl, m, gs_shift, LPR, tr, ts, nslab)
  if constexpr (FullFormat<B, D>::value) {
    if (R == 2) { if (CPL == 1) SWL_U(2, 1); else if (CPL == 2) SWL_U(2, 2); else SWL_U(2, 4); }
    else { if (CPL == 1) SWL_U(1, 1); else if (CPL == 2) SWL_U(1, 2); else SWL_U(1, 4); }
  } else {
    SWL_U(1, 4);
  }
#undef SWL_U
}

template <int B, int D>
void down_fmt(const MoeArgs& m, int ne, int R, int gs_shift, int LPR, int nslab, int grid, size_t smem,
              cudaStream_t st, bool pdl) {
#define SWL_D(N, R_) launch(k_moe_down<B, D, N, R_>, dim3(grid), dim3(GT), smem, st, pdl, m, gs_shift, LPR, nslab)
  if constexpr (FullFormat<B, D>::value) {
    if (ne == 4) { if (R == 2) SWL_D(4, 2); else SWL_D(4, 1); }
    else if (ne == 9) { if (R == 2) SWL_D(9, 2); else SWL_D(9, 1); }
    else if (ne == 12) { if (R == 2) SWL_D(12, 2); else SWL_D(12, 1); }
    else SWL_D(16, 1);
  } else {
    if (ne == 4) SWL_D(4, 1); else if (ne == 9) SWL_D(9, 1); else if (ne == 12) SWL_D(12, 1); else SWL_D(16, 1);
  }
#undef SWL_D
}

#define SWL_INSTANTIATE_FORMAT(B, D)                                                                                  \
  template void gemv_fmt<B, D>(const GemvArgs&, const SegTab&, int, int, int, int, int, int, size_t, cudaStream_t, bool); \
  template void router_fmt<B, D>(const RouterArgs&, const SegTab&, int, int, int, int, int, int, size_t, cudaStream_t, bool); \
  template void gateup_fmt<B, D>(const MoeArgs&, int, int, int, int, int, int, int, int, size_t, cudaStream_t, bool);   \
  template void down_fmt<B, D>(const MoeArgs&, int, int, int, int, int, int, size_t, cudaStream_t, bool);

}  // namespace swl
