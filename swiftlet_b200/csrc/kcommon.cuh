// Device primitives shared by the decode kernels (sm_100a).
//
// Dequantisation without integer->float conversions: for a 4-bit nibble at
// bit 4j of a word w, (w & (0xF << 4j)) | 0x4B000000 is the float
// 2^23 + q * 2^(4j) exactly (j <= 4; nibbles 5..7 use w >> 12). One packed
// f32x2 subtract removes 2^23 and one packed f32x2 FMA multiplies by
// x * 2^-(4j), which the kernel stored pre-scaled (exact: powers of two).
// Per group, y += scale * sum(q*x) + bias * sum(x): the MLX affine form
// w = scale*q + bias (Checkpoint.swift:168-209) folded out of the inner loop.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.h"
#include "kernels.h"

namespace swl {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Streaming 16-byte load of read-only weights (no L1 allocation).
__device__ __forceinline__ uint4 ld_stream(const uint8_t* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
// Hint the L2 to fetch [p, p + bytes) (bytes a multiple of 16, p 16-byte aligned).
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Asynchronous 16-byte global->shared copies (L2 only); a block copies a
// whole input vector in one round trip instead of one load per iteration.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Waits until at most N committed groups of this thread are still in flight.
template <int N>
__device__ __forceinline__ void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
// Block-wide copy of n floats (n % 4 == 0, both pointers 16-byte aligned).
__device__ __forceinline__ void copy_async(float* dst, const float* src, int n) {
  for (int i = threadIdx.x; i < (n >> 2); i += blockDim.x) cp_async16(dst + 4 * i, src + 4 * i);
}

__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarriers and bulk (TMA, non-tensor) copies into shared memory ----
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ void mbar_init(uint64_t* b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
// Makes initialised barriers visible to the async (bulk copy) proxy.
__device__ __forceinline__ void mbar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* b, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Waits for the phase of parity `parity` to complete, for at most about two
// seconds (then returns false: the caller records an error and gives up).
// After a short burst of polls the waiting thread sleeps between polls, so a
// long wait (a producer waiting for a free slot) leaves the issue slots to
// the warps doing the work.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;
__device__ __forceinline__ bool mbar_wait_for(uint64_t* b, unsigned parity, unsigned long long limit_ns) {
  if (mbar_try(b, parity)) return true;
  const unsigned long long t0 = gtimer();
  for (int i = 0; i < (1 << 26); ++i) {
    if (mbar_try(b, parity)) return true;
    if (i >= 16) __nanosleep(i < 64 ? 64 : 256);
    if (gtimer() - t0 > limit_ns) break;
  }
  return false;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* b, unsigned parity) { return mbar_wait_for(b, parity, kWaitLimitNs); }
// L2 policy for weights that are read once per token: evict them first, so
// activations, recurrent state and the KV cache stay resident.
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// Bulk copy of `bytes` (multiple of 16; both addresses 16-byte aligned) from
// global to this CTA's shared memory, completing on mbarrier `b`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* b, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(b)), "l"(policy)
      : "memory");
}
// The same bulk copy with the default L2 policy (data that is read again, such
// as the KV cache).
__device__ __forceinline__ void bulk_g2s_keep(void* dst, const void* src, unsigned bytes, uint64_t* b) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(b))
               : "memory");
}
// Orders this thread's earlier shared-memory accesses (generic proxy) before
// its later bulk copies into the same memory (async proxy).
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// Named barrier 1 over the first n threads (the consumer warps of a
// warp-specialised block; the producer warp never joins it).
__device__ __forceinline__ void bar_sync_n(int n) { asm volatile("bar.sync 1, %0;" ::"r"(n) : "memory"); }

// ---- thread-block clusters: rank, barrier, distributed shared memory ----
__device__ __forceinline__ unsigned cluster_rank() {
  unsigned r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Barrier over every thread of the cluster; shared-memory writes before it
// are visible to every CTA of the cluster after it. All threads of all CTAs
// must reach it (no thread of the cluster may have exited).
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The two halves of cluster_sync, for work between them: after arrive the
// thread may not touch what it released to the cluster.
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// Address of the variable at `p` (this CTA's shared memory) in the shared
// memory of cluster CTA `rank` (same offset).
__device__ __forceinline__ uint32_t dsmem_map(const void* p, unsigned rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ float dsmem_ld(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void dsmem_st(uint32_t addr, unsigned v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
// Per-block timeline record (thread 0): see Trace.
struct TraceRec {
  unsigned long long t0 = 0, t1 = 0, t2 = 0, t3 = 0;
  __device__ __forceinline__ void start(const Trace& tr) { if (tr.buf && threadIdx.x == 0) t0 = gtimer(); }
  __device__ __forceinline__ void waited(const Trace& tr) { if (tr.buf && threadIdx.x == 0) t1 = gtimer(); }
  __device__ __forceinline__ void staged(const Trace& tr) { if (tr.buf && threadIdx.x == 0) t2 = gtimer(); }
  __device__ __forceinline__ void looped(const Trace& tr) { if (tr.buf && threadIdx.x == 0) t3 = gtimer(); }
  __device__ __forceinline__ void end(const Trace& tr) {
    if (tr.buf && threadIdx.x == 0) {
      const unsigned i = atomicAdd(tr.count, 1u);
      if (i < tr.cap) {
        unsigned long long* r = tr.buf + static_cast<unsigned long long>(kTraceFields) * i;
        r[0] = tr.tag;
        r[1] = blockIdx.x + 65536ull * blockIdx.y;
        r[2] = t0;
        r[3] = t1;
        r[4] = t2;
        r[5] = t3;
        r[6] = gtimer();
      }
    }
  }
};

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
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  v = l < nw ? red[l] : 0.f;
  return warp_sum(v);
}

// Index maps of a DeltaNet token's in-projection outputs (split qwen3_5
// layout, or qwen3_next's per-key-head interleaved qkvz / ba).
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
  if (a.split) return a.conv_dim + hv * a.dv + i;
  const int rep = a.nv / a.nk, chunk = 2 * a.dk + 2 * rep * a.dv, hk = hv / rep, ri = hv - hk * rep;
  return hk * chunk + 2 * a.dk + rep * a.dv + ri * a.dv + i;
}
__device__ __forceinline__ void delta_ba(const DeltaArgs& a, int hv, int& bi, int& ai) {
  const int valueDim = a.nv * a.dv;
  if (a.split) { bi = a.conv_dim + valueDim + hv; ai = a.conv_dim + valueDim + a.nv + hv; return; }
  const int keyDim = a.nk * a.dk, rep = a.nv / a.nk, hk = hv / rep, ri = hv - hk * rep;
  const int base = 2 * keyDim + 2 * valueDim + hk * 2 * rep;
  bi = base + ri; ai = base + rep + ri;
}

__device__ __forceinline__ float sigmoid_ref(float v) { return 1.f / (1.f + expf(-v)); }            // QwenCPUModel.swift:61
__device__ __forceinline__ float silu_ref(float v) { return v * sigmoid_ref(v); }                  // :62
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

// Sum over one 16-byte chunk of q * x' (quantised) or w * x (plain);
// xg(i) returns float4 number i of the chunk's (pre-scaled) activations.
template <int BITS, int DT, typename XG>
__device__ __forceinline__ float chunk_dot(const uint4 w, XG xg) {
  const uint32_t word[4] = {w.x, w.y, w.z, w.w};
  if constexpr (BITS == 4) {
    const float2 M = f2(-8388608.f, -8388608.f);
    float2 acc = f2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t lo = word[i], hi = lo >> 12;
      const float4 xa = xg(2 * i), xb = xg(2 * i + 1);
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
      const float4 xa = xg(i);
      const float2 p01 = __fadd2_rn(f2(__uint_as_float((lo & 0xFFu) | 0x4B000000u), __uint_as_float((lo & 0xFF00u) | 0x4B000000u)), M);
      const float2 p23 = __fadd2_rn(f2(__uint_as_float((hi & 0xFFu) | 0x4B000000u), __uint_as_float((hi & 0xFF00u) | 0x4B000000u)), M);
      acc = __ffma2_rn(p01, f2(xa.x, xa.y), acc);
      acc = __ffma2_rn(p23, f2(xa.z, xa.w), acc);
    }
    return acc.x + acc.y;
  } else if constexpr (DT == DT_F32) {
    const float4 xa = xg(0);
    return __uint_as_float(w.x) * xa.x + __uint_as_float(w.y) * xa.y + __uint_as_float(w.z) * xa.z + __uint_as_float(w.w) * xa.w;
  } else {
    float2 acc = f2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 xa = xg(i >> 1);
      const float xl = (i & 1) ? xa.z : xa.x, xh = (i & 1) ? xa.w : xa.y;
      float lo, hi;
      if constexpr (DT == DT_BF16) {
        lo = __uint_as_float(word[i] << 16);
        hi = __uint_as_float(word[i] & 0xFFFF0000u);
      } else {
        __half2_raw r;
        r.x = (unsigned short)(word[i] & 0xFFFF);
        r.y = (unsigned short)(word[i] >> 16);
        const float2 v = __half22float2(__half2(r));
        lo = v.x;
        hi = v.y;
      }
      acc = __ffma2_rn(f2(lo, hi), f2(xl, xh), acc);
    }
    return acc.x + acc.y;
  }
}

// One lane's share of one weight row: CPL chunks of 16 bytes and the scale
// and bias of the group each chunk lies in.
template <int BITS, int DT, int CPL>
struct RowFrag {
  uint4 w[CPL];
  float s[CPL], b[CPL];
};

// Loads chunks c0, c0 + LPR, ... (CPL of them, those < nch) of row `row`.
template <int BITS, int DT, int CPL>
__device__ __forceinline__ void load_row(RowFrag<BITS, DT, CPL>& f, const QLin& L, int64_t row, bool valid, int c0, int LPR) {
  constexpr int WPC = ChunkInfo<BITS, DT>::WPC;
  const int nch = int(L.row_bytes >> 4);
  const uint8_t* wr = L.w + row * L.row_bytes;
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const int c = c0 + i * LPR;
    const bool ok = valid && c < nch;
    f.w[i] = ok ? ld_stream(wr + (int64_t(c) << 4)) : make_uint4(0, 0, 0, 0);
    if constexpr (BITS != 0) {
      const int64_t g = row * L.srow + (c * WPC) / L.gs;
      f.s[i] = ok ? load_scalar(L.s, DT, g) : 0.f;
      f.b[i] = ok ? load_scalar(L.b, DT, g) : 0.f;
    }
  }
}

// Staged activations in shared memory, "chunk-interleaved": float4 number q
// of chunk c lives at xs4[q * nch + c], so the 32 lanes of a warp, which
// read consecutive chunks, hit consecutive 16-byte words (no bank
// conflicts). cs[c] is the sum of chunk c's unscaled values.
struct XTile {
  const float4* xs4;
  const float* cs;
  int nch;
};

// Partial dot of a row fragment with staged x.
template <int BITS, int DT, int CPL>
__device__ __forceinline__ float dot_row(const RowFrag<BITS, DT, CPL>& f, const XTile& x, int c0, int LPR) {
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const int c = c0 + i * LPR;
    if (c < x.nch) {
      const float d = chunk_dot<BITS, DT>(f.w[i], [&](int q) { return x.xs4[q * x.nch + c]; });
      if constexpr (BITS != 0) acc = fmaf(f.s[i], d, fmaf(f.b[i], x.cs[c], acc));
      else acc += d;
    }
  }
  return acc;
}

// A lane's fixed chunks of x held in registers (rows are streamed past them).
template <int BITS, int DT, int CPL>
struct XRegs {
  static constexpr int Q = ChunkInfo<BITS, DT>::WPC / 4;
  float4 x[CPL][Q];
  float cs[CPL];
  __device__ __forceinline__ void load(const XTile& t, int c0, int LPR) {
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      const int c = c0 + i * LPR;
#pragma unroll
      for (int q = 0; q < Q; ++q) x[i][q] = c < t.nch ? t.xs4[q * t.nch + c] : make_float4(0.f, 0.f, 0.f, 0.f);
      cs[i] = c < t.nch ? t.cs[c] : 0.f;
    }
  }
};

template <int BITS, int DT, int CPL>
__device__ __forceinline__ float dot_row(const RowFrag<BITS, DT, CPL>& f, const XRegs<BITS, DT, CPL>& x) {
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const float d = chunk_dot<BITS, DT>(f.w[i], [&](int q) { return x.x[i][q]; });
    if constexpr (BITS != 0) acc = fmaf(f.s[i], d, fmaf(f.b[i], x.cs[i], acc));
    else acc += d;
  }
  return acc;
}

// Transposed reduction of R per-lane partials (one per row) over the LPR
// lanes of a sub-warp (R <= LPR, powers of two): each exchange round halves
// the rows a lane holds, so R rows cost R - 1 + log2(LPR / R) shuffles
// instead of R * log2(LPR). Returns the full sum of row `row` of this lane;
// the lanes with sl % (LPR / R) == 0 hold distinct rows.
template <int R>
__device__ __forceinline__ float reduce_rows(float (&p)[R], int LPR, int sl, int& row) {
  row = 0;
  int o = LPR >> 1;
#pragma unroll
  for (int h = R >> 1; h >= 1; h >>= 1) {
    const bool hi = (sl & o) != 0;
#pragma unroll
    for (int i = 0; i < h; ++i) {
      const float send = hi ? p[i] : p[i + h];
      const float keep = hi ? p[i + h] : p[i];
      p[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
    if (hi) row += h;
    o >>= 1;
  }
  float v = p[0];
  for (; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Reduction over the LPR lanes of a sub-warp (all 32 lanes must call it).
__device__ __forceinline__ float sub_sum(float v, int LPR) {
  for (int o = LPR >> 1; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Stages x[0..n) (values from `get(k)`) pre-scaled into the chunk-
// interleaved layout of `xs` plus chunk sums `cs`. A warp covers 32
// consecutive elements, i.e. whole chunks when WPC in {16, 32}, so chunk
// sums are shuffle reductions.
template <int BITS, int DT, typename Get>
__device__ __forceinline__ void stage_vec(int n, float* xs, float* cs, Get get) {
  constexpr int WPC = ChunkInfo<BITS, DT>::WPC;
  const int nch = n / WPC;
  const int lane = threadIdx.x & 31;
  for (int k0 = threadIdx.x - lane; k0 < n; k0 += blockDim.x) {
    const int k = k0 + lane;
    const float v = k < n ? get(k) : 0.f;
    if (k < n) {
      const int c = k / WPC, j = k - c * WPC;
      xs[((j >> 2) * nch + c) * 4 + (j & 3)] = BITS != 0 ? v * prescale<BITS>(k) : v;
    }
    if constexpr (BITS != 0) {
      float s = v;
#pragma unroll
      for (int o = WPC >> 1; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if ((lane & (WPC - 1)) == 0 && k < n) cs[k / WPC] = s;
    }
  }
}

}  // namespace swl
