// Batched decode kernels (sm_100a): T <= BT_MAX sequences, one token each,
// through the dense projections, the router, the routed + shared experts and
// lm_head as one weight stream.
//
// Arithmetic is the B = 1 integer tensor-core scheme: each activation row is
// split per quantisation group into three signed base-254 digits
// (k_digitize, f32-level accuracy), weight codes are multiplied with them on
// mma.sync m16n8k32 u8 x s8 -> s32 and every group's int32 sums are scaled
// by the group's weight scale and digit scale in f32; the bias enters as
// bias_g * sum(x_g) (MLX affine w = scale * q + bias, Checkpoint.swift:168-209).
//
// k_bgemm is persistent: CTA c takes items c, c + grid, ...; an item is 64
// weight rows (two halves of 32, possibly from two matrices: gate and up of
// one expert) times a tile of up to 16 tokens. Its (item, input chunk)
// sequence streams through a four-stage cp.async ring: per stage the 64 rows
// x kc codes (16-byte chunks, XOR swizzle by row so the eight rows a warp
// reads at once fall on distinct banks), the rows' scale and bias windows,
// and the tokens' digit tables and group metadata. Warp w computes row
// fragment w % 4 (16 rows) for the token columns (token, digit) of column
// blocks w / 4, w / 4 + 2, ... or, with a single column block, half of the
// chunk's groups; the digits of a token are summed in the epilogue.
#include <algorithm>

#include "imma_impl.cuh"
#include "kernels.h"
#include "launch.h"

namespace swl {

constexpr int BG_THREADS = 256;
constexpr int BG_STAGES = 4;
constexpr int BG_MAXCB = 3;            // column blocks per warp (16 tokens x 3 digits = 6 blocks, 2 halves)
constexpr int BG_OCOLS = 3 * BG_TOK;   // epilogue columns per row
constexpr int BG_OBYTES = 2 * BG_ROWS * BG_OCOLS * 4;

__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// --------------------------------------------------------------- digits --
// One CTA per row: the prologue (QwenCPUModel.rmsNorm, QwenCPUModel.swift:
// 47-59; the DeltaNet gated norm, :490-493) in shared memory, then per group
// the digit scale 127 / max|x|, the three digits of every value (B-table
// entry (kb, t) of the 4-bit fragment order: codes 8t + 2j of block kb in the
// first word set, 8t + 2j + 1 in the second) and the group's (1 / scale, sum).
constexpr int DG_THREADS = 256;

template <int KPG>
__device__ __forceinline__ void digit_groups(const float* x, int in, int gs, uint2* bt, float2* meta) {
  const int tid = threadIdx.x;
  const int ng = in / gs, items = ng * 4;
  for (int base = 0; base < items; base += DG_THREADS) {
    const int it = base + tid;
    const bool ok = it < items;
    const int g = ok ? it >> 2 : 0, t = it & 3;
    float v[KPG][8];
    float m = 0.f, sum = 0.f;
    bool fin = true;
#pragma unroll
    for (int kk = 0; kk < KPG; ++kk) {
      entry_values<4>(x, g * KPG + kk, t, v[kk]);
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
#pragma unroll
      for (int kk = 0; kk < KPG; ++kk) entry_store<4>(v[kk], inv, bt + (g * KPG + kk) * 12 + t);
      if (t == 0) meta[g] = make_float2(rs, sum);
    }
  }
}

__global__ void __launch_bounds__(DG_THREADS) k_digitize(const DigitArgs a) {
  extern __shared__ __align__(16) float xs[];
  __shared__ float red[64];
  pdl_wait();
  const int row = blockIdx.x, tid = threadIdx.x, in = a.in;
  const float* x = a.x + row * a.x_stride;
  for (int i = tid; i < in; i += DG_THREADS) xs[i] = x[i];
  __syncthreads();
  if (a.prologue == PRO_RMSNORM) {
    float ss = 0.f;
    for (int i = tid; i < in; i += DG_THREADS) ss += xs[i] * xs[i];
    ss = block_sum(ss, red);
    const float scale = 1.f / sqrtf(ss / float(in) + a.eps);
    for (int i = tid; i < in; i += DG_THREADS) xs[i] = xs[i] * (scale * a.aux[i]);
  } else if (a.prologue == PRO_GATEDNORM) {
    // per head of head_dim values: rmsnorm with weight aux2, times silu(z)
    const float* z = a.aux + row * a.x_stride;
    const int hd = a.head_dim, nh = in / hd, warp = tid >> 5, lane = tid & 31;
    for (int hh = warp; hh < nh; hh += DG_THREADS / 32) {
      float ss = 0.f;
      for (int i = lane; i < hd; i += 32) ss += xs[hh * hd + i] * xs[hh * hd + i];
      ss = warp_sum(ss);
      const float sc = 1.f / sqrtf(ss / float(hd) + a.eps);
      for (int i = lane; i < hd; i += 32) {
        const int k = hh * hd + i;
        xs[k] = (xs[k] * (sc * a.aux2[i])) * z[k];
      }
    }
  }
  __syncthreads();
  pdl_launch();
  if (a.x_out)
    for (int i = tid; i < in; i += DG_THREADS) a.x_out[row * a.x_stride + i] = xs[i];
  uint2* bt = a.bt + row * a.bt_row;
  float2* meta = a.meta + row * a.meta_row;
  switch (a.gs >> 5) {
    case 1: digit_groups<1>(xs, in, a.gs, bt, meta); break;
    case 2: digit_groups<2>(xs, in, a.gs, bt, meta); break;
    default: digit_groups<4>(xs, in, a.gs, bt, meta); break;
  }
}

void launch_digitize(const DigitArgs& a, cudaStream_t st, bool pdl) {
  if (a.rows <= 0) return;
  if (a.in % a.gs || (a.gs != 32 && a.gs != 64 && a.gs != 128) || a.in > 16384)
    throw Error(ERR_UNSUPPORTED, "digitize: unsupported input size or group");
  launch(k_digitize, dim3(a.rows), dim3(DG_THREADS), size_t(a.in) * 4, st, pdl, a);
}

// ----------------------------------------------------------- GEMM items --
// The two 32-row halves and the token tile of item `it` (fields per half
// selected with conditionals, so the struct stays in registers).
struct BItem {
  const uint8_t *w0, *w1, *s0p, *s1p, *b0p, *b1p;
  int r0, r1;   // first row of each half in its matrix
  int nv0, nv1; // valid rows of each half (0..32)
  int64_t wrow, srow;
  int c;        // tokens of the tile
  int s0;       // first slot (expert launches) or token (dense)
  int seg;      // dense: segment; expert: expert id
  int orow;     // dense: first output row of the item in its segment; expert: first row
  __device__ __forceinline__ const uint8_t* w(int hf) const { return hf ? w1 : w0; }
  __device__ __forceinline__ const uint8_t* s(int hf) const { return hf ? s1p : s0p; }
  __device__ __forceinline__ const uint8_t* b(int hf) const { return hf ? b1p : b0p; }
  __device__ __forceinline__ int row(int hf) const { return hf ? r1 : r0; }
  __device__ __forceinline__ int nv(int hf) const { return hf ? nv1 : nv0; }
};

__device__ __forceinline__ int clamp32(int v) { return v < 0 ? 0 : (v > 32 ? 32 : v); }

__device__ __forceinline__ void bmat_half(const BMat& m, int e, int row0, BItem& d, int hf) {
  const uint8_t* w = m.w + e * m.ew;
  const uint8_t* s = m.s + e * m.es;
  const uint8_t* b = m.b + e * m.eb;
  const int nv = clamp32(m.rows - row0);
  if (hf) { d.w1 = w; d.s1p = s; d.b1p = b; d.r1 = row0; d.nv1 = nv; }
  else { d.w0 = w; d.s0p = s; d.b0p = b; d.r0 = row0; d.nv0 = nv; }
}

__device__ __forceinline__ BItem bitem(const BGemmArgs& a, int it) {
  BItem d;
  if (!a.expert_mode) {
    const int ntt = (a.ntok + BG_TOK - 1) / BG_TOK;
    const int rb = it / ntt, tt = it - rb * ntt;
    int sg = 0;
    while (sg + 1 < a.nseg && rb >= a.seg_rb[sg + 1]) ++sg;
    const int r = (rb - a.seg_rb[sg]) * BG_ROWS;
    const BMat& m = a.seg[sg];
    bmat_half(m, 0, r, d, 0);
    bmat_half(m, 0, r + 32, d, 1);
    d.wrow = m.wrow;
    d.srow = m.srow;
    d.s0 = tt * BG_TOK;
    d.c = min(BG_TOK, a.ntok - d.s0);
    d.seg = sg;
    d.orow = r;
  } else {
    const int4 q = a.items[it];
    const int e = q.x;
    const bool sh = e >= a.experts;
    const BMat& m0 = sh ? a.sg : a.eg;
    const int ee = sh ? 0 : e;
    if (a.mode == BM_SWIGLU) {
      const BMat& m1 = sh ? a.su : a.eu;
      bmat_half(m0, ee, q.y, d, 0);
      bmat_half(m1, ee, q.y, d, 1);
    } else {
      bmat_half(m0, ee, q.y, d, 0);
      bmat_half(m0, ee, q.y + 32, d, 1);
    }
    d.wrow = m0.wrow;
    d.srow = m0.srow;
    d.s0 = q.z;
    d.c = q.w;
    d.seg = e;
    d.orow = q.y;
  }
  return d;
}

// Per-thread copy plan of one item: chunk-0 sources and shared-memory
// offsets, computed once per item (later chunks add fixed strides). Thread
// tid copies weight chunks tid + 256u, the scale (even tid) or bias (odd
// tid) window of row tid / 2, digit chunks tid + 256u of the tile's tokens
// and metadata entry tid.
template <int BITS>
struct BPlan {
  static constexpr int WMAX = BITS == 4 ? 2 : 4;  // 64 rows x kcb / 16 chunks (kc <= 256)
  static constexpr int XMAX = 3;                  // 16 tokens x 48 chunks (kc <= 256)
  const uint8_t* wp[WMAX];
  const uint8_t* xp[XMAX];
  const uint8_t* sp;
  const uint8_t* mp;
  int wd[WMAX], xd[XMAX], sd, md;
  unsigned wm, xm;
  bool sv, mv;
  bool s8;  // the row's windows are 8 bytes per chunk and 8-byte aligned: one copy
};

template <int BITS, int DT>
__device__ __forceinline__ void bg_plan(const BGemmArgs& a, const BGLayout& L, const BItem& d, BPlan<BITS>& p) {
  const int tid = threadIdx.x;
  const int cpr = L.kcb >> 4, mask = min(cpr, 8) - 1;
  p.wm = 0u;
#pragma unroll
  for (int u = 0; u < BPlan<BITS>::WMAX; ++u) {
    const int i = tid + u * BG_THREADS, r = i / cpr, ch = i - r * cpr, hf = r >> 5, rr = r & 31;
    const bool ok = r < BG_ROWS && rr < d.nv(hf);
    p.wp[u] = ok ? d.w(hf) + int64_t(d.row(hf) + rr) * d.wrow + ch * 16 : nullptr;
    p.wd[u] = L.w_off + r * L.kcb + ((ch ^ (r & mask)) << 4);
    p.wm |= ok ? 1u << u : 0u;
  }
  {
    const int r = tid >> 1, which = tid & 1, hf = r >> 5, rr = r & 31;
    p.sv = r < BG_ROWS && rr < d.nv(hf);
    p.sp = p.sv ? (which ? d.b(hf) : d.s(hf)) + int64_t(d.row(hf) + rr) * d.srow : nullptr;
    p.sd = (which ? L.b_off : L.s_off) + r * L.sw;
    p.s8 = p.sv && L.gpc * (DT == DT_F32 ? 4 : 2) == 8 && (reinterpret_cast<uintptr_t>(p.sp) & 7) == 0;
  }
  const int n16 = (L.kc >> 5) * 6;  // 16-byte digit chunks per token per chunk (96 bytes per 32 values)
  p.xm = 0u;
#pragma unroll
  for (int u = 0; u < BPlan<BITS>::XMAX; ++u) {
    const int i = tid + u * BG_THREADS, j = i / n16, c16 = i - j * n16;
    const bool ok = j < d.c;
    int row = 0;
    if (ok) row = a.in_map ? a.in_map[d.s0 + j] : d.s0 + j;
    p.xp[u] = ok ? reinterpret_cast<const uint8_t*>(a.xbt + row * a.bt_row) + c16 * 16 : nullptr;
    p.xd[u] = L.x_off + j * L.bstride * 8 + c16 * 16;
    p.xm |= ok ? 1u << u : 0u;
  }
  {
    const int j = tid / L.gpc, g = tid - j * L.gpc;
    p.mv = j < d.c;
    int row = 0;
    if (p.mv) row = a.in_map ? a.in_map[d.s0 + j] : d.s0 + j;
    p.mp = p.mv ? reinterpret_cast<const uint8_t*>(a.xmeta + row * a.meta_row + g) : nullptr;
    p.md = L.m_off + (j * L.gpc + g) * 8;
  }
}

// Issues the copies of chunk kc of the planned item into stage buffer st.
template <int BITS, int DT>
__device__ __forceinline__ void bg_issue(const BGLayout& L, const BPlan<BITS>& p, int kc, uint8_t* st) {
  constexpr int SB = DT == DT_F32 ? 4 : 2;
#pragma unroll
  for (int u = 0; u < BPlan<BITS>::WMAX; ++u)
    if (p.wm & (1u << u)) cp_async16(st + p.wd[u], p.wp[u] + int64_t(kc) * L.kcb);
  if (p.s8) {
    cp_async8(st + p.sd, p.sp + kc * 8);
  } else if (p.sv) {
    // the 4-byte aligned words covering the chunk's entries of the row
    const int sbytes = L.gpc * SB;
    const uint8_t* base = p.sp + int64_t(kc) * sbytes;
    const uintptr_t a0 = reinterpret_cast<uintptr_t>(base) & ~uintptr_t(3);
    const uintptr_t a1 = (reinterpret_cast<uintptr_t>(base) + sbytes + 3) & ~uintptr_t(3);
    for (uintptr_t q = a0; q < a1; q += 4) cp_async4(st + p.sd + (q - a0), reinterpret_cast<const void*>(q));
  }
  const int64_t xstep = int64_t(L.kc >> 5) * 96;
#pragma unroll
  for (int u = 0; u < BPlan<BITS>::XMAX; ++u)
    if (p.xm & (1u << u)) cp_async16(st + p.xd[u], p.xp[u] + kc * xstep);
  if (p.mv) cp_async8(st + p.md, p.mp + int64_t(kc) * L.gpc * 8);
}

template <int DT>
__device__ __forceinline__ float sm_entry(const uint8_t* p) {
  if constexpr (DT == DT_F32) return *reinterpret_cast<const float*>(p);
  else if constexpr (DT == DT_BF16) return __uint_as_float(uint32_t(*reinterpret_cast<const uint16_t*>(p)) << 16);
  else return f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(p));
}

// Groups [G0, G0 + NG) of a chunk against NCB column blocks (1: the single
// block of a tile of at most two tokens, the warp's half of the groups; 3:
// blocks hw, hw + 2, hw + 4 over all groups) for the common layout of
// 256-value chunks and 64-value groups, fully unrolled so that every
// shared-memory access is a lane base plus a constant. W0 is the lane's
// first weight row (+ its word offset), sx the lane's swizzle term, X the
// stage's digit tables, M its metadata, S0/S1/B0/B1 the rows' scale and
// bias entries of group 0.
template <int BITS, int DT, int G0, int NG, int NCB>
__device__ __forceinline__ void bg_fast(const uint8_t* W0, int sx, const uint2* X, const float2* M,
                                        const int (&boff)[BG_MAXCB], const int (&cbv)[BG_MAXCB],
                                        const int (&mo0)[BG_MAXCB], const int (&mo1)[BG_MAXCB],
                                        const float (&wn0)[BG_MAXCB], const float (&wn1)[BG_MAXCB],
                                        const float (&z0)[BG_MAXCB], const float (&z1)[BG_MAXCB], const uint8_t* S0,
                                        const uint8_t* S1, const uint8_t* B0, const uint8_t* B1,
                                        float (&acc)[BG_MAXCB][4]) {
  constexpr int SB = DT == DT_F32 ? 4 : 2;
  constexpr int KCB = 32 * BITS;  // weight bytes per row per chunk
#pragma unroll
  for (int gg = 0; gg < NG; ++gg) {
    const int g = G0 + gg;
    int dd[NCB][4];
#pragma unroll
    for (int j = 0; j < NCB; ++j) dd[j][0] = dd[j][1] = dd[j][2] = dd[j][3] = 0;
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      const int kb = 2 * g + kk;
      uint32_t af[4];
      if constexpr (BITS == 4) {
        const int off = (kb << 4) ^ sx;
        const uint32_t u0 = *reinterpret_cast<const uint32_t*>(W0 + off);
        const uint32_t u1 = *reinterpret_cast<const uint32_t*>(W0 + 8 * KCB + off);
        af[0] = u0 & 0x0F0F0F0Fu;
        af[2] = (u0 >> 4) & 0x0F0F0F0Fu;
        af[1] = u1 & 0x0F0F0F0Fu;
        af[3] = (u1 >> 4) & 0x0F0F0F0Fu;
      } else {
        const int off = (kb << 5) ^ sx;
        const uint2 x0 = *reinterpret_cast<const uint2*>(W0 + off);
        const uint2 x1 = *reinterpret_cast<const uint2*>(W0 + 8 * KCB + off);
        af[0] = prmt(x0.x, x0.y, 0x6420u);
        af[2] = prmt(x0.x, x0.y, 0x7531u);
        af[1] = prmt(x1.x, x1.y, 0x6420u);
        af[3] = prmt(x1.x, x1.y, 0x7531u);
      }
#pragma unroll
      for (int j = 0; j < NCB; ++j)
        if (NCB == 1 || cbv[j]) {
          const uint2 bv = boff[j] >= 0 ? X[kb * 12 + boff[j]] : make_uint2(0u, 0u);
          mma_u8s8(dd[j], af, bv);
        }
    }
    const float s0v = sm_entry<DT>(S0 + g * SB), s1v = sm_entry<DT>(S1 + g * SB);
    const float b0v = sm_entry<DT>(B0 + g * SB), b1v = sm_entry<DT>(B1 + g * SB);
#pragma unroll
    for (int j = 0; j < NCB; ++j)
      if (NCB == 1 || cbv[j]) {
        const float2 m0 = mo0[j] >= 0 ? M[mo0[j] + g] : make_float2(0.f, 0.f);
        const float2 m1 = mo1[j] >= 0 ? M[mo1[j] + g] : make_float2(0.f, 0.f);
        const float f0 = m0.x * wn0[j], f1 = m1.x * wn1[j];
        const float c0 = z0[j] * m0.y, c1 = z1[j] * m1.y;
        acc[j][0] = fmaf(s0v * f0, i2f_small(dd[j][0]), fmaf(b0v, c0, acc[j][0]));
        acc[j][1] = fmaf(s0v * f1, i2f_small(dd[j][1]), fmaf(b0v, c1, acc[j][1]));
        acc[j][2] = fmaf(s1v * f0, i2f_small(dd[j][2]), fmaf(b1v, c0, acc[j][2]));
        acc[j][3] = fmaf(s1v * f1, i2f_small(dd[j][3]), fmaf(b1v, c1, acc[j][3]));
      }
  }
}

template <int BITS, int DT, bool FAST>
__global__ void __launch_bounds__(BG_THREADS) k_bgemm(const BGemmArgs a) {
  constexpr int SB = DT == DT_F32 ? 4 : 2;
  extern __shared__ __align__(128) uint8_t sm[];
  const BGLayout L = a.L;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gi = lane >> 2, t = lane & 3;
  const int rf = warp & 3, hw = warp >> 2;
  pdl_wait();
  const int nitems = a.expert_mode ? min(*a.nitems, a.max_items)
                                   : a.seg_rb[a.nseg] * ((a.ntok + BG_TOK - 1) / BG_TOK);
  const int nkc = a.in / L.kc;
  const int mine = nitems > int(blockIdx.x) ? (nitems - 1 - int(blockIdx.x)) / int(gridDim.x) + 1 : 0;
  const int nq = mine * nkc;
  // loader: (item, chunk) of the next chunk it issues, counted without
  // divisions; re-planned at each item's first chunk
  BPlan<BITS> lp;
  int l_m = 0, l_kc = 0;
  auto load = [&](int q) {
    if (l_kc == 0) bg_plan<BITS, DT>(a, L, bitem(a, int(blockIdx.x) + l_m * int(gridDim.x)), lp);
    bg_issue<BITS, DT>(L, lp, l_kc, sm + (q & (BG_STAGES - 1)) * L.stage);
    if (++l_kc == nkc) { l_kc = 0; ++l_m; }
  };
  // prologue: the first BG_STAGES - 1 chunks
#pragma unroll
  for (int q = 0; q < BG_STAGES - 1; ++q) {
    if (q < nq) load(q);
    cp_async_commit();
  }
  const int mask = min(L.kcb >> 4, 8) - 1;
  const int r0l = rf * 16 + gi, r1l = r0l + 8;  // this lane's two rows of the 64
  BItem d;
  int ncb = 0;
  bool ksplit = false;
  int boff[BG_MAXCB], cbv[BG_MAXCB];
  int mo0[BG_MAXCB], mo1[BG_MAXCB];
  float wn0[BG_MAXCB], wn1[BG_MAXCB], z0[BG_MAXCB], z1[BG_MAXCB];
  float acc[BG_MAXCB][4];
  int mis_s0 = 0, mis_s1 = 0, mis_b0 = 0, mis_b1 = 0;  // byte offset of the rows' first entry in their windows
  int c_m = 0, kc = 0;  // consumer's item and chunk
  for (int q = 0; q < nq; ++q, (++kc == nkc ? (kc = 0, ++c_m) : 0)) {
    cp_async_wait_group<BG_STAGES - 2>();
    __syncthreads();
    if (q + BG_STAGES - 1 < nq) load(q + BG_STAGES - 1);
    cp_async_commit();
    if (kc == 0) {
      d = bitem(a, int(blockIdx.x) + c_m * int(gridDim.x));
      ncb = (3 * d.c + 7) >> 3;
      ksplit = ncb == 1;
#pragma unroll
      for (int j = 0; j < BG_MAXCB; ++j) {
        const int cb = ksplit ? (j == 0 ? 0 : 99) : hw + 2 * j;
        cbv[j] = cb < ncb;
        const int cB = 8 * cb + gi, tB = cB / 3, nB = cB - 3 * tB;
        boff[j] = (cb < ncb && tB < d.c) ? tB * L.bstride + nB * 4 + t : -1;
        const int c0 = 8 * cb + 2 * t, c1 = c0 + 1;
        const int t0 = c0 / 3, n0 = c0 - 3 * t0, t1 = c1 / 3, n1 = c1 - 3 * t1;
        mo0[j] = (cb < ncb && t0 < d.c) ? t0 * L.gpc : -1;
        mo1[j] = (cb < ncb && t1 < d.c) ? t1 * L.gpc : -1;
        wn0[j] = n0 == 0 ? 1.f : (n0 == 1 ? 1.f / 254.f : 1.f / (254.f * 254.f));
        wn1[j] = n1 == 0 ? 1.f : (n1 == 1 ? 1.f / 254.f : 1.f / (254.f * 254.f));
        z0[j] = n0 == 0 ? 1.f : 0.f;
        z1[j] = n1 == 0 ? 1.f : 0.f;
#pragma unroll
        for (int u = 0; u < 4; ++u) acc[j][u] = 0.f;
      }
      const int h0 = r0l >> 5, h1 = r1l >> 5;
      mis_s0 = int(reinterpret_cast<uintptr_t>(d.s(h0) + int64_t(d.row(h0) + (r0l & 31)) * d.srow) & 3);
      mis_s1 = int(reinterpret_cast<uintptr_t>(d.s(h1) + int64_t(d.row(h1) + (r1l & 31)) * d.srow) & 3);
      mis_b0 = int(reinterpret_cast<uintptr_t>(d.b(h0) + int64_t(d.row(h0) + (r0l & 31)) * d.srow) & 3);
      mis_b1 = int(reinterpret_cast<uintptr_t>(d.b(h1) + int64_t(d.row(h1) + (r1l & 31)) * d.srow) & 3);
    }
    const uint8_t* st = sm + (q & (BG_STAGES - 1)) * L.stage;
    const uint8_t* W = st + L.w_off;
    const uint2* X = reinterpret_cast<const uint2*>(st + L.x_off);
    const float2* M = reinterpret_cast<const float2*>(st + L.m_off);
    const int cadv = (kc * L.gpc * SB) & 3;
    const uint8_t* S0 = st + L.s_off + r0l * L.sw + ((mis_s0 + cadv) & 3);
    const uint8_t* S1 = st + L.s_off + r1l * L.sw + ((mis_s1 + cadv) & 3);
    const uint8_t* B0 = st + L.b_off + r0l * L.sw + ((mis_b0 + cadv) & 3);
    const uint8_t* B1 = st + L.b_off + r1l * L.sw + ((mis_b1 + cadv) & 3);
    if constexpr (FAST) {
      const int sx = BITS == 4 ? (gi << 4) : ((((t >> 1) ^ gi) & 7) << 4);
      const uint8_t* W0 = W + r0l * (32 * BITS) + (BITS == 4 ? 4 * t : 8 * (t & 1));
      if (!ksplit)
        bg_fast<BITS, DT, 0, 4, 3>(W0, sx, X, M, boff, cbv, mo0, mo1, wn0, wn1, z0, z1, S0, S1, B0, B1, acc);
      else if (hw == 0)
        bg_fast<BITS, DT, 0, 2, 1>(W0, sx, X, M, boff, cbv, mo0, mo1, wn0, wn1, z0, z1, S0, S1, B0, B1, acc);
      else
        bg_fast<BITS, DT, 2, 2, 1>(W0, sx, X, M, boff, cbv, mo0, mo1, wn0, wn1, z0, z1, S0, S1, B0, B1, acc);
    }
    int g0 = 0, g1 = L.gpc;
    if (ksplit) { g0 = (hw * L.gpc) >> 1; g1 = ((hw + 1) * L.gpc) >> 1; }
    if (!FAST && cbv[0]) {
      for (int g = g0; g < g1; ++g) {
        int dd[BG_MAXCB][4];
#pragma unroll
        for (int j = 0; j < BG_MAXCB; ++j) dd[j][0] = dd[j][1] = dd[j][2] = dd[j][3] = 0;
        for (int kk = 0; kk < L.kpg; ++kk) {
          const int kb = g * L.kpg + kk;
          uint32_t af[4];
          if constexpr (BITS == 4) {
            const uint32_t u0 = *reinterpret_cast<const uint32_t*>(W + r0l * L.kcb + ((kb ^ (r0l & mask)) << 4) + 4 * t);
            const uint32_t u1 = *reinterpret_cast<const uint32_t*>(W + r1l * L.kcb + ((kb ^ (r1l & mask)) << 4) + 4 * t);
            af[0] = u0 & 0x0F0F0F0Fu;
            af[2] = (u0 >> 4) & 0x0F0F0F0Fu;
            af[1] = u1 & 0x0F0F0F0Fu;
            af[3] = (u1 >> 4) & 0x0F0F0F0Fu;
          } else {
            // 8-bit codes 8t..8t+7 of the block (words 2t, 2t + 1) in the
            // 4-bit fragment order: even codes first, odd codes second
            const int ch = 2 * kb + (t >> 1);
            const uint2 x0 = *reinterpret_cast<const uint2*>(W + r0l * L.kcb + ((ch ^ (r0l & mask)) << 4) + 8 * (t & 1));
            const uint2 x1 = *reinterpret_cast<const uint2*>(W + r1l * L.kcb + ((ch ^ (r1l & mask)) << 4) + 8 * (t & 1));
            af[0] = prmt(x0.x, x0.y, 0x6420u);
            af[2] = prmt(x0.x, x0.y, 0x7531u);
            af[1] = prmt(x1.x, x1.y, 0x6420u);
            af[3] = prmt(x1.x, x1.y, 0x7531u);
          }
#pragma unroll
          for (int j = 0; j < BG_MAXCB; ++j)
            if (cbv[j]) {
              const uint2 bv = boff[j] >= 0 ? X[kb * 12 + boff[j]] : make_uint2(0u, 0u);
              mma_u8s8(dd[j], af, bv);
            }
        }
        const float s0v = sm_entry<DT>(S0 + g * SB), s1v = sm_entry<DT>(S1 + g * SB);
        const float b0v = sm_entry<DT>(B0 + g * SB), b1v = sm_entry<DT>(B1 + g * SB);
#pragma unroll
        for (int j = 0; j < BG_MAXCB; ++j)
          if (cbv[j]) {
            const float2 m0 = mo0[j] >= 0 ? M[mo0[j] + g] : make_float2(0.f, 0.f);
            const float2 m1 = mo1[j] >= 0 ? M[mo1[j] + g] : make_float2(0.f, 0.f);
            const float f0 = m0.x * wn0[j], f1 = m1.x * wn1[j];
            const float c0 = z0[j] * m0.y, c1 = z1[j] * m1.y;
            acc[j][0] = fmaf(s0v * f0, i2f_small(dd[j][0]), fmaf(b0v, c0, acc[j][0]));
            acc[j][1] = fmaf(s0v * f1, i2f_small(dd[j][1]), fmaf(b0v, c1, acc[j][1]));
            acc[j][2] = fmaf(s1v * f0, i2f_small(dd[j][2]), fmaf(b1v, c0, acc[j][2]));
            acc[j][3] = fmaf(s1v * f1, i2f_small(dd[j][3]), fmaf(b1v, c1, acc[j][3]));
          }
      }
    }
    if (kc == nkc - 1) {
      // epilogue: per (row, column) results into O, the digit columns of a
      // token (and the two group halves of a split) summed per row
      __syncthreads();  // the stage may hold O: every warp is done reading it
      float* O = reinterpret_cast<float*>(L.o_off < 0 ? const_cast<uint8_t*>(st) : sm + L.o_off);
      const int ncol = 3 * d.c;
      float* Ob = O + (ksplit ? hw : 0) * BG_ROWS * BG_OCOLS;
#pragma unroll
      for (int j = 0; j < BG_MAXCB; ++j)
        if (cbv[j]) {
          const int cb = ksplit ? 0 : hw + 2 * j;
          const int c0 = 8 * cb + 2 * t;
          if (c0 < ncol) { Ob[r0l * BG_OCOLS + c0] = acc[j][0]; Ob[r1l * BG_OCOLS + c0] = acc[j][2]; }
          if (c0 + 1 < ncol) { Ob[r0l * BG_OCOLS + c0 + 1] = acc[j][1]; Ob[r1l * BG_OCOLS + c0 + 1] = acc[j][3]; }
        }
      __syncthreads();
      auto val = [&](int r, int tok) {
        const float* o = O + r * BG_OCOLS + 3 * tok;
        float v = (o[0] + o[1]) + o[2];
        if (ksplit) {
          const float* o2 = o + BG_ROWS * BG_OCOLS;
          v += (o2[0] + o2[1]) + o2[2];
        }
        return v;
      };
      if (a.mode == BM_SWIGLU) {
        for (int i = tid; i < 32 * d.c; i += BG_THREADS) {
          const int tok = i >> 5, r = i & 31;
          if (r < d.nv0 && r < d.nv1) {
            const float gv = val(r, tok), uv = val(32 + r, tok);
            a.out[int64_t(d.s0 + tok) * a.out_stride + d.orow + r] = silu_ref(gv) * uv;
          }
        }
      } else if (a.expert_mode) {
        for (int i = tid; i < BG_ROWS * d.c; i += BG_THREADS) {
          const int tok = i >> 6, r = i & 63;
          if ((r & 31) < d.nv(r >> 5)) a.out[int64_t(d.s0 + tok) * a.out_stride + d.orow + r] = val(r, tok);
        }
      } else {
        float* y = a.y[d.seg];
        for (int i = tid; i < BG_ROWS * d.c; i += BG_THREADS) {
          const int tok = i >> 6, r = i & 63;
          if ((r & 31) < d.nv(r >> 5)) {
            float* p = y + int64_t(d.s0 + tok) * a.y_stride + d.orow + r;
            const float v = val(r, tok);
            if (a.mode == BM_RESIDUAL) *p += v;
            else *p = v;
          }
        }
      }
    }
  }
  cp_async_wait_group<0>();
  pdl_launch();
}

bool bgemm_layout(int in, int bits, int dt, int gs, BGLayout& L) {
  if ((bits != 4 && bits != 8) || (gs != 32 && gs != 64 && gs != 128) || in % gs || in % 32) return false;
  int kc = 0;
  for (int c : {256, 128, 64, 32})
    if (in % c == 0 && c % gs == 0) { kc = c; break; }
  if (!kc) return false;
  const int SB = dtype_bytes(dt);
  L.kc = kc;
  L.kcb = kc * bits / 8;
  L.gpc = kc / gs;
  L.kpg = gs / 32;
  L.sw = (L.gpc * SB + 4 + 15) & ~15;
  const int kbc = kc / 32;
  L.bstride = kbc * 12 + ((12 - (kbc * 12) % 16) + 16) % 16;
  auto up = [](int v) { return (v + 127) & ~127; };
  L.w_off = 0;
  L.s_off = up(L.w_off + BG_ROWS * L.kcb);
  L.b_off = up(L.s_off + BG_ROWS * L.sw);
  L.x_off = up(L.b_off + BG_ROWS * L.sw);
  L.m_off = up(L.x_off + BG_TOK * L.bstride * 8);
  L.stage = up(L.m_off + BG_TOK * L.gpc * 8);
  if (L.stage >= BG_OBYTES) {
    L.o_off = -1;
    L.total = BG_STAGES * L.stage;
  } else {
    L.o_off = BG_STAGES * L.stage;
    L.total = L.o_off + BG_OBYTES;
  }
  return L.total <= 200 * 1024;
}

// The unrolled consumer serves 256-value chunks of 64-value groups.
static bool bg_fast_layout(const BGLayout& L) { return L.kc == 256 && L.kpg == 2 && L.gpc == 4; }

template <int BITS, int DT, bool FAST>
static int bg_grid_for(int smem) {
  static int cached[64] = {0};
  static bool opened = false;
  const int key = std::min(63, smem >> 12);
  if (!opened) {
    // the ceiling once, at the largest layout any launch uses: launches of
    // one instantiation differ in size, and a lower ceiling would reject them
    SWL_CUDA(cudaFuncSetAttribute(k_bgemm<BITS, DT, FAST>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    opened = true;
  }
  if (!cached[key]) {
    int per = 0;
    SWL_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, k_bgemm<BITS, DT, FAST>, BG_THREADS, smem));
    cached[key] = std::max(1, per);
  }
  return cached[key] * sm_count();
}

template <int BITS, int DT>
static int bg_grid2(const BGLayout& L) {
  return bg_fast_layout(L) ? bg_grid_for<BITS, DT, true>(L.total) : bg_grid_for<BITS, DT, false>(L.total);
}

int bgemm_grid(int bits, int dt, const BGLayout& L) {
  if (bits == 4) {
    if (dt == DT_BF16) return bg_grid2<4, DT_BF16>(L);
    if (dt == DT_F16) return bg_grid2<4, DT_F16>(L);
    return bg_grid2<4, DT_F32>(L);
  }
  if (dt == DT_BF16) return bg_grid2<8, DT_BF16>(L);
  if (dt == DT_F16) return bg_grid2<8, DT_F16>(L);
  return bg_grid2<8, DT_F32>(L);
}

template <int BITS, int DT>
static void bg_launch(const BGemmArgs& a, dim3 g, cudaStream_t st, bool pdl) {
  const size_t smem = size_t(a.L.total);
  if (bg_fast_layout(a.L)) launch(k_bgemm<BITS, DT, true>, g, dim3(BG_THREADS), smem, st, pdl, a);
  else launch(k_bgemm<BITS, DT, false>, g, dim3(BG_THREADS), smem, st, pdl, a);
}

void launch_bgemm(const BGemmArgs& a, int bits, int dt, int grid, cudaStream_t st, bool pdl) {
  const dim3 g(std::max(grid, 1));
  if (bits == 4) {
    if (dt == DT_BF16) bg_launch<4, DT_BF16>(a, g, st, pdl);
    else if (dt == DT_F16) bg_launch<4, DT_F16>(a, g, st, pdl);
    else bg_launch<4, DT_F32>(a, g, st, pdl);
  } else {
    if (dt == DT_BF16) bg_launch<8, DT_BF16>(a, g, st, pdl);
    else if (dt == DT_F16) bg_launch<8, DT_F16>(a, g, st, pdl);
    else bg_launch<8, DT_F32>(a, g, st, pdl);
  }
}

// -------------------------------------------------------------- routing --
// One CTA: warp w routes tokens w, w + 32 (warp_route: softmax weights,
// top-k with ties to the lower expert id, renormalisation, shared gate);
// then the picks are grouped by expert. A token picks an expert at most once,
// so a 64-bit token mask per expert gives each pick its rank (tokens below
// it with the same expert) and each expert its count; slots are
// expert-major in expert id order. Items: per active expert, token tiles of
// up to 16 slots times row blocks (gate/up: 32 intermediate rows of gate and
// of up; down: 64 hidden rows), tiles of one row block adjacent so that CTAs
// running together share its weights in L2; the shared expert's items last.
constexpr int BR_THREADS = 1024;
constexpr int BR_MAXE = 1024;

__global__ void __launch_bounds__(BR_THREADS) k_broute(const BRouteArgs a) {
  __shared__ int ids[BT_MAX * 32];
  __shared__ float wts[BT_MAX * 32];
  __shared__ float shs[BT_MAX];
  __shared__ unsigned long long msk[BR_MAXE];
  __shared__ int off[BR_MAXE + 1], tb[BR_MAXE + 1], tb5[BR_MAXE + 1];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T = a.T, E = a.E, K = a.K;
  const int e_lo = a.e_lo, e_hi = min(a.e_hi, E), sh_lo = min(a.sh_lo, T), sh_hi = min(a.sh_hi, T);
  pdl_wait();
  for (int e = tid; e < E; e += BR_THREADS) msk[e] = 0ull;
  for (int tok = warp; tok < T; tok += BR_THREADS / 32)
    warp_route(a.logits + int64_t(tok) * (E + 1), E, K, a.norm_topk, ids + tok * K, wts + tok * K, shs + tok);
  __syncthreads();
  for (int p = tid; p < T * K; p += BR_THREADS)
    if (ids[p] >= e_lo && ids[p] < e_hi) atomicOr(&msk[ids[p]], 1ull << (p / K));
  __syncthreads();
  if (warp == 0) {
    // exclusive scans of the counts (off) and of the token tiles (tb)
    int run_c = 0, run_t = 0, run_5 = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const int c = e < E ? __popcll(msk[e]) : 0, tt = (c + BG_TOK - 1) / BG_TOK, t5 = (c + 4) / 5;
      int ic = c, it = tt, i5 = t5;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int vc = __shfl_up_sync(0xffffffffu, ic, o), vt = __shfl_up_sync(0xffffffffu, it, o);
        const int v5 = __shfl_up_sync(0xffffffffu, i5, o);
        if (lane >= o) { ic += vc; it += vt; i5 += v5; }
      }
      if (e < E) { off[e] = run_c + ic - c; tb[e] = run_t + it - tt; tb5[e] = run_5 + i5 - t5; }
      run_c += __shfl_sync(0xffffffffu, ic, 31);
      run_t += __shfl_sync(0xffffffffu, it, 31);
      run_5 += __shfl_sync(0xffffffffu, i5, 31);
    }
    if (lane == 0) { off[E] = run_c; tb[E] = run_t; tb5[E] = run_5; }
  }
  __syncthreads();
  pdl_launch();
  for (int p = tid; p < T * K; p += BR_THREADS) {
    const int tok = p / K, e = ids[p];
    a.ids[p] = e;
    a.w[p] = wts[p];
    if (e < e_lo || e >= e_hi) {  // another rank's expert
      a.slot_of[p] = -1;
      continue;
    }
    const int rank = __popcll(msk[e] & ((1ull << tok) - 1ull));
    const int slot = off[e] + rank;
    a.slot_of[p] = slot;
    a.slot_tok[slot] = tok;
  }
  for (int tok = tid; tok < T; tok += BR_THREADS) {
    a.slot_tok[T * K + tok] = tok;
    a.sh[tok] = shs[tok];
  }
  const int rbg = (a.inter + 31) / 32, rbd = (a.hidden + 63) / 64, rbs = (a.shared_inter + 31) / 32;
  const int nsh = max(0, sh_hi - sh_lo), ntt_s = (nsh + BG_TOK - 1) / BG_TOK;
  // item i of a list belongs to the expert e with tb[e] * rb_n <= i <
  // tb[e + 1] * rb_n (binary search over the tile prefix sums); every thread
  // writes items, not one thread per expert
  auto routed_item = [&](int i, int rb_n, int rows) {
    int lo = 0, hi = E;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (tb[mid] * rb_n <= i) lo = mid;
      else hi = mid;
    }
    const int e = lo, c = __popcll(msk[e]), ntt = (c + BG_TOK - 1) / BG_TOK;
    const int r = i - tb[e] * rb_n, rb = r / ntt, tt = r - rb * ntt;
    return make_int4(e, rb * rows, off[e] + tt * BG_TOK, min(BG_TOK, c - tt * BG_TOK));
  };
  for (int i = tid; i < min(tb[E] * rbg, a.max_gu); i += BR_THREADS) a.items_gu[i] = routed_item(i, rbg, 32);
  for (int i = tid; i < min(tb[E] * rbd, a.max_dn); i += BR_THREADS) a.items_dn[i] = routed_item(i, rbd, 64);
  const int base_gu = tb[E] * rbg, base_dn = tb[E] * rbd;
  for (int i = tid; i < ntt_s * rbs; i += BR_THREADS) {
    const int rb = i / ntt_s, tt = i - rb * ntt_s;
    if (base_gu + i < a.max_gu)
      a.items_gu[base_gu + i] = make_int4(E, rb * 32, T * K + sh_lo + tt * BG_TOK, min(BG_TOK, nsh - tt * BG_TOK));
  }
  for (int i = tid; i < ntt_s * rbd; i += BR_THREADS) {
    const int rb = i / ntt_s, tt = i - rb * ntt_s;
    if (base_dn + i < a.max_dn)
      a.items_dn[base_dn + i] = make_int4(E, rb * 64, T * K + sh_lo + tt * BG_TOK, min(BG_TOK, nsh - tt * BG_TOK));
  }
  if (tid == 0) {
    a.nitems[0] = min(base_gu + ntt_s * rbs, a.max_gu);
    a.nitems[1] = min(base_dn + ntt_s * rbd, a.max_dn);
  }
  if (a.items_tgu) {
    // the tensor-core GEMM's lists: 64 intermediate rows of gate and up, 128
    // hidden rows; tiles of at most 5 slots (its narrow N = 16 items)
    constexpr int TT = 5;
    auto routed5 = [&](int i, int rb_n, int rows) {
      int lo = 0, hi = E;
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (tb5[mid] * rb_n <= i) lo = mid;
        else hi = mid;
      }
      const int e = lo, c = __popcll(msk[e]), ntt = (c + TT - 1) / TT;
      const int r = i - tb5[e] * rb_n, rb = r / ntt, tt = r - rb * ntt;
      return make_int4(e, rb * rows, off[e] + tt * TT, min(TT, c - tt * TT));
    };
    const int tg = (a.inter + 63) / 64, td = (a.hidden + 127) / 128, ts = (a.shared_inter + 63) / 64;
    const int nt5 = (nsh + TT - 1) / TT;
    for (int i = tid; i < min(tb5[E] * tg, a.max_tgu); i += BR_THREADS) a.items_tgu[i] = routed5(i, tg, 64);
    for (int i = tid; i < min(tb5[E] * td, a.max_tdn); i += BR_THREADS) a.items_tdn[i] = routed5(i, td, 128);
    const int bg = tb5[E] * tg, bd = tb5[E] * td;
    for (int i = tid; i < nt5 * ts; i += BR_THREADS) {
      const int rb = i / nt5, tt = i - rb * nt5;
      if (bg + i < a.max_tgu)
        a.items_tgu[bg + i] = make_int4(E, rb * 64, T * K + sh_lo + tt * TT, min(TT, nsh - tt * TT));
    }
    for (int i = tid; i < nt5 * td; i += BR_THREADS) {
      const int rb = i / nt5, tt = i - rb * nt5;
      if (bd + i < a.max_tdn)
        a.items_tdn[bd + i] = make_int4(E, rb * 128, T * K + sh_lo + tt * TT, min(TT, nsh - tt * TT));
    }
    for (int sl = off[E] + tid; sl < T * K; sl += BR_THREADS) a.slot_tok[sl] = 0;
    if (tid == 0) {
      a.ntitems[0] = min(bg + nt5 * ts, a.max_tgu);
      a.ntitems[1] = min(bd + nt5 * td, a.max_tdn);
    }
  }
}

void launch_broute(const BRouteArgs& a, cudaStream_t st, bool pdl) {
  if (a.T < 1 || a.T > BT_MAX || a.K > 32 || a.E > 512 || a.E < a.K)
    throw Error(ERR_UNSUPPORTED, "batched routing: unsupported batch or expert geometry");
  launch(k_broute, dim3(1), dim3(BR_THREADS), 0, st, pdl, a);
}

// -------------------------------------------------------------- combine --
// h[t] += sum_k w[t][k] * y[slot(t, k)] + sh[t] * y[T * K + t]: the routed
// experts in pick order, then the gated shared expert
// (QwenCPUModel.swift:552-566), added to the residual stream.
__global__ void k_bcombine(const BCombineArgs a) {
  pdl_wait();
  const int tok = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.D) return;
  float acc = 0.f;
  for (int k = 0; k < a.K; ++k)
    acc += a.w[tok * a.K + k] * a.ydown[int64_t(a.slot_of[tok * a.K + k]) * a.ystride + i];
  acc += a.sh[tok] * a.ydown[int64_t(a.T * a.K + tok) * a.ystride + i];
  a.h[int64_t(tok) * a.D + i] += acc;
  pdl_launch();
}

void launch_bcombine(const BCombineArgs& a, cudaStream_t st, bool pdl) {
  launch(k_bcombine, dim3((a.D + 255) / 256, a.T), dim3(256), 0, st, pdl, a);
}

// Expert-parallel form of k_bcombine (BCombineEpArgs): the partial sum of
// this rank's experts for every token of the step, with the shared expert and
// the residual added on the token's own rank only.
__global__ void k_bcombine_ep(const BCombineEpArgs a) {
  pdl_wait();
  const int tok = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.D) return;
  float acc = 0.f;
  for (int k = 0; k < a.K; ++k) {
    const int s = a.slot_of[tok * a.K + k];
    if (s >= 0) acc += a.w[tok * a.K + k] * a.ydown[int64_t(s) * a.ystride + i];
  }
  if (tok >= a.own_lo && tok < a.own_hi) {
    acc += a.sh[tok] * a.ydown[int64_t(a.T * a.K + tok) * a.ystride + i];
    acc += a.h[int64_t(tok - a.own_lo) * a.D + i];
  }
  a.part[int64_t(tok) * a.D + i] = acc;
  pdl_launch();
}

void launch_bcombine_ep(const BCombineEpArgs& a, cudaStream_t st, bool pdl) {
  launch(k_bcombine_ep, dim3((a.D + 255) / 256, a.T), dim3(256), 0, st, pdl, a);
}

// Every sequence of the step has consumed its tokens.
__global__ void k_badvance(const StateDev* sds, int S, const int* seq_n) {
  pdl_wait();
  if (int(threadIdx.x) < S) *sds[threadIdx.x].pos += seq_n ? seq_n[threadIdx.x] : 1;
}

void launch_badvance(const StateDev* sds, int S, const int* seq_n, cudaStream_t st, bool pdl) {
  launch(k_badvance, dim3(1), dim3(BT_MAX), 0, st, pdl, sds, S, seq_n);
}

// Greedy token per row: the first index of the largest logit
// (TextGenerator.swift:90).
__global__ void __launch_bounds__(1024) k_bargmax(const float* logits, int V, int* out) {
  __shared__ float bv[32];
  __shared__ int bi[32];
  pdl_wait();
  const float* l = logits + int64_t(blockIdx.x) * V;
  float v = -INFINITY;
  int idx = 0x7fffffff;
  auto take = [&](float x, int i) {
    if (x > v || (idx == 0x7fffffff)) { v = x; idx = i; }
  };
  if ((V & 3) == 0 && (reinterpret_cast<uintptr_t>(l) & 15) == 0) {
    // four 16-byte loads in flight per thread; each thread still meets its
    // indices in increasing order, so the first maximum wins as below
    const float4* l4 = reinterpret_cast<const float4*>(l);
    const int n4 = V >> 2, step = int(blockDim.x);
    for (int b = threadIdx.x; b < n4; b += 4 * step) {
      float4 q[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) q[u] = b + u * step < n4 ? l4[b + u * step] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i4 = b + u * step;
        if (i4 < n4) {
          take(q[u].x, 4 * i4);
          take(q[u].y, 4 * i4 + 1);
          take(q[u].z, 4 * i4 + 2);
          take(q[u].w, 4 * i4 + 3);
        }
      }
    }
  } else {
    for (int i = threadIdx.x; i < V; i += blockDim.x) take(l[i], i);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > v || (ov == v && oi < idx)) { v = ov; idx = oi; }
  }
  if (lane == 0) { bv[warp] = v; bi[warp] = idx; }
  __syncthreads();
  if (warp == 0) {
    v = lane < int(blockDim.x >> 5) ? bv[lane] : -INFINITY;
    idx = lane < int(blockDim.x >> 5) ? bi[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ov > v || (ov == v && oi < idx)) { v = ov; idx = oi; }
    }
    if (lane == 0) out[blockIdx.x] = idx;
  }
}

void launch_bargmax(const float* logits, int T, int V, int* out, cudaStream_t st, bool pdl) {
  launch(k_bargmax, dim3(T), dim3(1024), 0, st, pdl, logits, V, out);
}

}  // namespace swl
