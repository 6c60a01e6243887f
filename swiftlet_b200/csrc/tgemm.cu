// Grouped MLX-affine GEMMs of the batched decode and prefill launches on the
// 5th-generation tensor cores (tcgen05, sm_100a).
//
// Arithmetic (the same integer scheme as k_bgemm, exact to f32 level): each
// activation row is split per quantisation group into three signed base-254
// digits (k_digitize, tensor-core layout), the weight codes are multiplied
// with them as u8 x s8 -> s32 by tcgen05.mma kind::i8, and every group's int32
// sums are scaled in f32 by the group's weight scale and digit scale; the
// bias enters as bias_g * sum(x_g) (MLX affine w = scale * q + bias,
// Checkpoint.swift:168-209).
//
// One item is a 128-row weight tile (dense: 128 rows of a matrix; expert
// gate/up: 64 intermediate rows of gate on TMEM lanes 0-63 and of up on
// 64-127; expert down: 128 hidden rows) times up to 16 tokens or expert slots
// (N = 48 digit columns). The input dimension is walked in chunks of 256
// codes; per chunk the MMA warp issues, for each quantisation group, its
// K = 32 steps into that group's own TMEM accumulator (48 columns), so the
// epilogue can apply the per-(row, group) scales. Two accumulator sets
// alternate, so the MMAs of chunk j + 1 run while the epilogue reads chunk j.
//
// Warp roles of a CTA (256 threads, one CTA per SM, persistent over items
// c, c + grid, ...):
//   warps 0-3  epilogue: warp w reads TMEM lanes 32w..32w+31 (one weight row
//              per thread), accumulates each token in registers and writes
//              the item's outputs (SwiGLU: up rows pass through shared memory
//              to the gate rows);
//   warp 4     producer: TMA loads of the weight tile (128-byte swizzled
//              rows; 4-bit tiles packed) and the digit tile into a ring of
//              stages, completion on one mbarrier per stage;
//   warp 5     TMEM allocation and MMA issue (one thread), tcgen05.commit to
//              free a stage and to publish an accumulator set;
//   warps 6-7  4-bit weights only: unpack the packed tile into the 8-bit,
//              128-byte swizzled K-major layout the MMA reads (two LOP3 and
//              two PRMT per 8 codes), then fence the writes to the async
//              proxy.
// Every mbarrier wait is bounded (about 2 s): one that gives up sets bit 0
// of the status word and makes every role leave its loop; the MMA thread
// then waits for its last MMAs and the producer for its copies in flight
// before the TMEM is released.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "imma_impl.cuh"
#include "kernels.h"
#include "launch.h"

namespace swl {

constexpr int TG_THREADS = 256;
constexpr int TG_ROWS = 128;             // MMA M
constexpr int TG_KC = 256;               // codes per chunk
constexpr int TG_A_BYTES = TG_ROWS * TG_KC;        // unpacked 8-bit tile: two 128-byte atoms of 128 rows
constexpr int TG_P_BYTES = TG_ROWS * TG_KC / 2;    // packed 4-bit tile: one atom
constexpr int TG_DENSE_TOK = 16;                   // tokens per dense item (N = 48)

// Item width: N digit columns (three per token or slot); expert items are
// narrow (a routed expert sees a few tokens per step), so their MMAs, digit
// tiles and accumulators are a third the size and four accumulator sets fit.
template <int TN>
struct TgShape {
  static constexpr int N = TN;
  static constexpr int TOK = TN / 3;                 // 16 -> 5, 48 -> 16
  static constexpr int NACC = TN == 16 ? 4 : 2;      // accumulator sets in TMEM
  static constexpr int B_BYTES = TN * TG_KC;         // digit tile: two atoms of N rows
  static constexpr int XCHG = 64 * (TOK + 1);        // SwiGLU: up-row sums handed to the gate rows (padded rows)
  // kind::i8, D s32, A u8 (weight codes), B s8 (digits), both K-major, M 128
  static constexpr uint32_t IDESC = (2u << 4) | (0u << 7) | (1u << 10) | (uint32_t(TN >> 3) << 17) | (uint32_t(TG_ROWS >> 4) << 24);
};

struct TGemmMaps {
  CUtensorMap a[4];  // dense: segments; experts: routed gate (or down), routed up, shared gate (or down), shared up
  CUtensorMap b;     // digit matrix [rows][in] s8 as {128 B, rows, in / 128}
};

template <int BITS, int TN>
struct TgLayout {
  using Sh = TgShape<TN>;
  static constexpr int S = BITS == 4 ? (TN == 16 ? 4 : 3) : (TN == 16 ? 5 : 4);  // stages
  static constexpr int P_OFF = 0;
  static constexpr int P_SIZE = BITS == 4 ? TG_P_BYTES : 0;
  static constexpr int A_OFF = S * P_SIZE;
  static constexpr int B_OFF = A_OFF + S * TG_A_BYTES;
  static constexpr int X_OFF = B_OFF + S * Sh::B_BYTES;
  static constexpr int M_OFF = X_OFF + Sh::XCHG * 4;          // group metadata of two items [2][TOK][32] float2
  static constexpr int BAR_OFF = M_OFF + 2 * Sh::TOK * 32 * 8;
  // full[S], unpacked[S], empty[S], tfull[NACC], tempty[NACC], drain, tmem address, abort flag, step count
  static constexpr int TOTAL = BAR_OFF + (3 * S + 2 * Sh::NACC + 1) * 8 + 16;
};

// ---- tcgen05 / TMA primitives --------------------------------------------
__device__ __forceinline__ uint64_t tg_desc(uint32_t saddr) {
  // K-major operand, 128-byte swizzle: 8-row groups of 128-byte rows 1024
  // bytes apart (SBO), descriptor version 1 (sm_100)
  return uint64_t((saddr >> 4) & 0x3FFFu) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) | (uint64_t(1) << 46) |
         (uint64_t(2) << 61);
}
__device__ __forceinline__ void tg_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(uint32_t(accumulate))
      : "memory");
}
__device__ __forceinline__ void tg_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tg_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tg_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tg_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tg_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tg_tma3(void* dst, const CUtensorMap* m, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_u32(dst)),
      "l"(m), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tg_tma4(void* dst, const CUtensorMap* m, int x, int y, int z, int w, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(
          smem_u32(dst)),
      "l"(m), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ uint32_t tg_prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}
// Pipeline wait: polls without sleeping for the first ~4k tries (hand-offs
// between the roles are short), then backs off; gives up after about 2 s.
__device__ __forceinline__ bool tg_wait(uint64_t* b, unsigned parity) {
  if (mbar_try(b, parity)) return true;
  const unsigned long long t0 = gtimer();
  for (int i = 0; i < (1 << 26); ++i) {
    if (mbar_try(b, parity)) return true;
    if (i >= 4096) __nanosleep(128);
    if ((i & 255) == 0 && gtimer() - t0 > kWaitLimitNs) break;
  }
  return false;
}
// Exact float of an int32 partial sum (|v| < 2^22): magic-number conversion.
__device__ __forceinline__ float tg_i2f(uint32_t v) {
  return __int_as_float(int(v) + 0x4B400000) - 12582912.f;
}

// Item `it` of the launch: weight rows, first token / slot and its count.
struct TgItem {
  int mat;     // tensor map index (dense: segment; experts: 0 routed, 2 shared)
  int expert;  // routed expert id, or -1 (3-d map)
  int row0;    // first weight row in the matrix (SwiGLU: first intermediate row)
  int rows;    // valid weight rows of the matrix from row0 (up to 128; SwiGLU: up to 64)
  int s0, nt;  // first token / slot and tokens in the tile
  const uint8_t* s;   // scales of row row0 (SwiGLU: of gate)
  const uint8_t* b;
  const uint8_t* s2;  // SwiGLU: up's scales / biases of row row0
  const uint8_t* b2;
  int64_t srow;       // scale (bias) bytes per row
};

__device__ __forceinline__ TgItem tg_item(const TGemmArgs& a, int it) {
  TgItem d;
  if (!a.expert_mode) {
    const int ntt = (a.ntok + TG_DENSE_TOK - 1) / TG_DENSE_TOK;
    const int rb = it / ntt, tt = it - rb * ntt;
    int sg = 0;
    while (sg + 1 < a.nseg && rb >= a.seg_rb[sg + 1]) ++sg;
    const BMat& m = a.seg[sg];
    d.mat = sg;
    d.expert = -1;
    d.row0 = (rb - a.seg_rb[sg]) * TG_ROWS;
    d.rows = min(TG_ROWS, m.rows - d.row0);
    d.s0 = tt * TG_DENSE_TOK;
    d.nt = min(TG_DENSE_TOK, a.ntok - d.s0);
    d.srow = m.srow;
    d.s = m.s + d.row0 * m.srow;
    d.b = m.b + d.row0 * m.srow;
    d.s2 = d.b2 = nullptr;
  } else {
    const int4 q = a.items[it];
    const bool sh = q.x >= a.experts;
    const BMat& g = sh ? a.sg : a.eg;
    const int e = sh ? 0 : q.x;
    d.mat = sh ? 2 : 0;
    d.expert = sh ? -1 : q.x;
    d.row0 = q.y;
    d.rows = min(a.mode == BM_SWIGLU ? 64 : TG_ROWS, g.rows - q.y);
    d.s0 = q.z;
    d.nt = q.w;
    d.srow = g.srow;
    d.s = g.s + e * g.es + q.y * g.srow;
    d.b = g.b + e * g.eb + q.y * g.srow;
    if (a.mode == BM_SWIGLU) {
      const BMat& u = sh ? a.su : a.eu;
      d.s2 = u.s + e * u.es + q.y * u.srow;
      d.b2 = u.b + e * u.eb + q.y * u.srow;
    } else {
      d.s2 = d.b2 = nullptr;
    }
  }
  return d;
}

__device__ __forceinline__ int tg_nitems(const TGemmArgs& a) {
  if (!a.expert_mode) return a.seg_rb[a.nseg] * ((a.ntok + TG_DENSE_TOK - 1) / TG_DENSE_TOK);
  return min(*a.nitems, a.max_items);
}

template <int BITS, int TN>
__global__ void __launch_bounds__(TG_THREADS, 1) k_tgemm(const TGemmArgs a, const __grid_constant__ TGemmMaps M) {
  using Lay = TgLayout<BITS, TN>;
  using Sh = TgShape<TN>;
  constexpr int S = Lay::S, NACC = Sh::NACC, TOK = Sh::TOK, TG_N = Sh::N;
  extern __shared__ __align__(1024) uint8_t tg_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tg_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + Lay::BAR_OFF);
  uint64_t* unpacked = full + S;
  uint64_t* empty = unpacked + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + NACC;
  uint64_t* drain = tempty + NACC;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* issued_ctr = const_cast<int*>(abort_flag) + 1;
  float* xchg = reinterpret_cast<float*>(sm + Lay::X_OFF);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int in = a.in, nkc = in / TG_KC, gpc = TG_KC / a.gs, kpg = a.gs / 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&unpacked[s], 64);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < NACC; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    *issued_ctr = 0;
    mbar_init_fence();
  }
  if (warp == 5) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tg_fence_before();
  __syncthreads();
  tg_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();
  const int nit = tg_nitems(a);
  auto fail = [&]() {
    if (a.status) atomicOr(a.status, 1);
    *abort_flag = 1;
  };

  if (warp == 4) {
    // ---------------------------------------------------- producer ------
    if (lane == 0) {
      int j = 0;
      for (int it = blockIdx.x; it < nit && !*abort_flag; it += gridDim.x) {
        const TgItem d = tg_item(a, it);
        for (int kc = 0; kc < nkc; ++kc, ++j) {
          const int s = j % S;
          const unsigned ph = (j / S) & 1;
          if (!tg_wait(&empty[s], ph ^ 1)) { fail(); break; }
          if (*abort_flag) break;
          uint8_t* A = sm + Lay::A_OFF + s * TG_A_BYTES;
          uint8_t* B = sm + Lay::B_OFF + s * Sh::B_BYTES;
          const bool two = a.expert_mode && a.mode == BM_SWIGLU;  // gate rows 0-63, up rows 64-127
          const unsigned abytes = BITS == 4 ? TG_P_BYTES : TG_A_BYTES;
          mbar_expect_tx(&full[s], abytes + Sh::B_BYTES);
          const int nseg_k = BITS == 4 ? 1 : 2;  // 128-byte K segments of weights per chunk
          for (int q = 0; q < nseg_k; ++q) {
            uint8_t* dst = BITS == 4 ? sm + Lay::P_OFF + s * TG_P_BYTES : A + q * (TG_ROWS * 128);
            const int seg = kc * nseg_k + q;
            const CUtensorMap* m0 = &M.a[d.mat];
            if (!two) {
              if (d.expert < 0) tg_tma3(dst, m0, 0, d.row0, seg, &full[s]);
              else tg_tma4(dst, m0, 0, d.row0, seg, d.expert, &full[s]);
            } else {
              const CUtensorMap* m1 = &M.a[d.mat + 1];
              if (d.expert < 0) {
                tg_tma3(dst, m0, 0, d.row0, seg, &full[s]);
                tg_tma3(dst + 64 * 128, m1, 0, d.row0, seg, &full[s]);
              } else {
                tg_tma4(dst, m0, 0, d.row0, seg, d.expert, &full[s]);
                tg_tma4(dst + 64 * 128, m1, 0, d.row0, seg, d.expert, &full[s]);
              }
            }
          }
          for (int q = 0; q < 2; ++q) tg_tma3(B + q * (TG_N * 128), &M.b, 0, 3 * d.s0, 2 * kc + q, &full[s]);
          *issued_ctr = j + 1;
        }
        if (*abort_flag) break;
      }
    }
  } else if (warp == 5) {
    // ---------------------------------------------------- MMA issue -----
    if (lane == 0) {
      int j = 0;
      for (int it = blockIdx.x; it < nit && !*abort_flag; it += gridDim.x) {
        for (int kc = 0; kc < nkc; ++kc, ++j) {
          const int s = j % S, acc = j % NACC;
          const unsigned ph = (j / S) & 1, aph = (j / NACC) & 1;
          if (!tg_wait(&full[s], ph) || (BITS == 4 && !tg_wait(&unpacked[s], ph))) { fail(); break; }
          if (!tg_wait(&tempty[acc], aph ^ 1)) { fail(); break; }
          if (*abort_flag) break;
          tg_fence_after();
          // descriptors of the stage's tiles; a K step adds its byte offset
          // (>> 4) to the start-address field
          const uint64_t ad = tg_desc(smem_u32(sm + Lay::A_OFF + s * TG_A_BYTES));
          const uint64_t bd = tg_desc(smem_u32(sm + Lay::B_OFF + s * Sh::B_BYTES));
          const uint32_t dacc = tmem + uint32_t(acc * gpc * TG_N);
#pragma unroll
          for (int i = 0; i < TG_KC / 32; ++i) {  // eight K = 32 steps: group i / kpg
            const int atom = i >> 2, off = (i & 3) * 32;
            const int g = i / kpg;
            tg_mma(dacc + uint32_t(g * TG_N), ad + uint64_t((atom * (TG_ROWS * 128) + off) >> 4),
                   bd + uint64_t((atom * (TG_N * 128) + off) >> 4), Sh::IDESC, (i % kpg) != 0);
          }
          tg_commit(&empty[s]);
          tg_commit(&tfull[acc]);
        }
        if (*abort_flag) break;
      }
      // every MMA issued above has completed once this commit arrives
      tg_commit(drain);
      if (!tg_wait(drain, 0)) fail();
    }
  } else if (warp >= 6) {
    // ---------------------------------------------------- 4-bit unpack --
    if constexpr (BITS == 4) {
      const int ut = threadIdx.x - 192;  // 0..63
      int j = 0;
      for (int it = blockIdx.x; it < nit && !*abort_flag; it += gridDim.x) {
        for (int kc = 0; kc < nkc; ++kc, ++j) {
          const int s = j % S;
          const unsigned ph = (j / S) & 1;
          if (!tg_wait(&full[s], ph)) { fail(); break; }
          const uint8_t* P = sm + Lay::P_OFF + s * TG_P_BYTES;
          uint8_t* A = sm + Lay::A_OFF + s * TG_A_BYTES;
          // thread ut owns rows ut and ut + 64: all eight packed 16-byte
          // chunks of a row are loaded before any is unpacked (eight loads in
          // flight; the lanes of a quarter-warp are eight consecutive rows,
          // which the swizzle puts on distinct banks), then chunk c's 32 codes
          // go to 32 bytes of atom c / 4. Measured alone on B200: 590 cycles
          // per 128 x 256-code stage, against 1,380 with units walked rows
          // fastest four at a time.
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int r = ut + 64 * h, sw = r & 7;
            uint4 w[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) w[c] = *reinterpret_cast<const uint4*>(P + r * 128 + ((c ^ sw) << 4));
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              uint32_t o[8];
              const uint32_t wv[4] = {w[c].x, w[c].y, w[c].z, w[c].w};
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                // codes 0, 2, 4, 6 of the word, then 1, 3, 5, 7: the digit
                // matrix of 4-bit launches holds its values in that order
                o[2 * q] = wv[q] & 0x0F0F0F0Fu;
                o[2 * q + 1] = (wv[q] >> 4) & 0x0F0F0F0Fu;
              }
              uint8_t* atom = A + (c >> 2) * (TG_ROWS * 128) + r * 128;
              const int ch = 2 * (c & 3);
              *reinterpret_cast<uint4*>(atom + ((ch ^ sw) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
              *reinterpret_cast<uint4*>(atom + (((ch + 1) ^ sw) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
            }
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          mbar_arrive(&unpacked[s]);
        }
        if (*abort_flag) break;
      }
    }
  } else {
    // ---------------------------------------------------- epilogue ------
    // Per item, each thread holds its weight row's scales and biases (bf16,
    // up to 32 groups) in registers and the item's group metadata sits in a
    // shared-memory slot; both are fetched for the next item while this one
    // runs, so the per-chunk loop reads only TMEM, registers and shared memory.
    const int r = threadIdx.x;  // TMEM lane = tile row
    const uint32_t lane_base = tmem + (uint32_t(32 * warp) << 16);
    const int ng = in / a.gs;   // groups per row (<= 32)
    float2* meta_s = reinterpret_cast<float2*>(sm + Lay::M_OFF);  // [2][TOK][32]
    uint4 sc_cur[4], bi_cur[4], sc_nxt[4], bi_nxt[4];
    auto fetch_rows = [&](const TgItem& d, uint4 (&sc)[4], uint4 (&bi)[4]) {
      const bool swg = a.expert_mode && a.mode == BM_SWIGLU;
      const bool upr = swg && r >= 64;
      const int mrow = swg ? (r & 63) : r;
      const bool ok = mrow < d.rows;
      const uint4* sp = reinterpret_cast<const uint4*>((upr ? d.s2 : d.s) + int64_t(mrow) * d.srow);
      const uint4* bp = reinterpret_cast<const uint4*>((upr ? d.b2 : d.b) + int64_t(mrow) * d.srow);
      const int nq = (ng * 2 + 15) / 16;  // 16-byte pieces of a row
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        sc[q] = (ok && q < nq) ? __ldg(sp + q) : make_uint4(0, 0, 0, 0);
        bi[q] = (ok && q < nq) ? __ldg(bp + q) : make_uint4(0, 0, 0, 0);
      }
    };
    auto fetch_meta = [&](const TgItem& d, int slot) {
      float2* dst = meta_s + slot * (TOK * 32);
      for (int i = r; i < d.nt * ng; i += 128) {
        const int t = i / ng, g = i - t * ng;
        dst[t * 32 + g] = __ldg(a.meta + int64_t(d.s0 + t) * a.meta_row + g);
      }
    };
    auto bf = [](const uint4 (&v)[4], int g) -> float {
      // selects, not an indexed load: the arrays stay in registers
      const int qi = g >> 3, wi = (g >> 1) & 3;
      const uint4 q = qi == 0 ? v[0] : qi == 1 ? v[1] : qi == 2 ? v[2] : v[3];
      const uint32_t w = wi == 0 ? q.x : wi == 1 ? q.y : wi == 2 ? q.z : q.w;
      return __uint_as_float((g & 1) ? (w & 0xFFFF0000u) : (w << 16));
    };
    int j = 0, nslot = 0;
    int it = blockIdx.x;
    TgItem d;
    if (it < nit) {
      d = tg_item(a, it);
      fetch_rows(d, sc_cur, bi_cur);
      fetch_meta(d, 0);
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    for (; it < nit && !*abort_flag; it += gridDim.x) {
      const bool swiglu = a.expert_mode && a.mode == BM_SWIGLU;
      const bool up = swiglu && r >= 64;
      const int mrow = swiglu ? (r & 63) : r;
      const bool valid = mrow < d.rows;
      // the next item's descriptor, scales and metadata, in flight meanwhile
      const int itn = it + gridDim.x;
      TgItem dn = d;
      if (itn < nit) {
        dn = tg_item(a, itn);
        fetch_rows(dn, sc_nxt, bi_nxt);
        fetch_meta(dn, nslot ^ 1);
      }
      const float2* mcur = meta_s + nslot * (TOK * 32);
      float acc_t[TOK];
#pragma unroll
      for (int t = 0; t < TOK; ++t) acc_t[t] = 0.f;
      bool bad = false;
      for (int kc = 0; kc < nkc; ++kc, ++j) {
        const int acc = j % NACC;
        const unsigned aph = (j / NACC) & 1;
        // warp-uniform outcome: the TMEM loads below are warp-collective
        if (!__all_sync(0xffffffffu, tg_wait(&tfull[acc], aph) ? 1 : 0)) { fail(); bad = true; break; }
        tg_fence_after();
        // narrow items: every group's 16 columns in flight before one wait
        uint32_t w4[4][16];
        if constexpr (TN == 16) {
#pragma unroll
          for (int g = 0; g < 4; ++g)
            if (g < gpc) tg_ld16(lane_base + uint32_t(acc * gpc * TG_N + g * TG_N), w4[g]);
          tg_ld_wait();
        }
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          if (g >= gpc) break;
          uint32_t v0[16], v1[16], v2[16];
          if constexpr (TN == 16) {
#pragma unroll
            for (int q = 0; q < 16; ++q) v0[q] = w4[g][q];
          } else {
            const uint32_t col = lane_base + uint32_t(acc * gpc * TG_N + g * TG_N);
            tg_ld16(col, v0);
            tg_ld16(col + 16, v1);
            tg_ld16(col + 32, v2);
            tg_ld_wait();
          }
          const int gi = kc * gpc + g;
          const float s_rg = bf(sc_cur, gi), b_rg = bf(bi_cur, gi);
          if constexpr (TN == 16) {
            // every token slot, branch-free (slots past the item's get zero
            // weight): independent chains across tokens
#pragma unroll
            for (int t = 0; t < TOK; ++t) {
              const float2 m = t < d.nt ? mcur[t * 32 + gi] : make_float2(0.f, 0.f);
              // v = P0 + P1 / 254 + P2 / 254^2 as (254 P0 + P1 + P2 / 254) / 254
              const int q = int(v0[3 * t]) * 254 + int(v0[3 * t + 1]);
              const float vv = fmaf(float(int(v0[3 * t + 2])), 1.f / 254.f, float(q));
              acc_t[t] = fmaf(s_rg * m.x * (1.f / 254.f), vv, fmaf(b_rg, m.y, acc_t[t]));
            }
          } else {
            // wide items: every token slot, branch-free (slots past the
            // item's read zero metadata), the digit columns merged in
            // integers as for narrow items
            const float sr = s_rg * (1.f / 254.f);
#pragma unroll
            for (int t = 0; t < TOK; ++t) {
              const int c0 = 3 * t;
              auto pick = [&](int c) -> uint32_t { return c < 16 ? v0[c] : (c < 32 ? v1[c - 16] : v2[c - 32]); };
              const float2 m = t < d.nt ? mcur[t * 32 + gi] : make_float2(0.f, 0.f);
              const int q = int(pick(c0)) * 254 + int(pick(c0 + 1));
              const float vv = fmaf(float(int(pick(c0 + 2))), 1.f / 254.f, float(q));
              acc_t[t] = fmaf(sr * m.x, vv, fmaf(b_rg, m.y, acc_t[t]));
            }
          }
        }
        tg_fence_before();
        mbar_arrive(&tempty[acc]);
      }
      // the four epilogue warps leave together (the SwiGLU hand-over below
      // uses a named barrier among them)
      int stop = (bad || *abort_flag) ? 1 : 0;
      asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.s32 p, %1, 0;\n\tbar.red.or.pred q, 1, 128, p;\n\tselp.s32 %0, 1, 0, q;\n\t}"
                   : "=r"(stop) : "r"(stop) : "memory");
      if (stop) break;
      // ---- outputs of the item ----
      if (!a.expert_mode) {
        float* y = a.y[d.mat];
        if (valid)
#pragma unroll
          for (int t = 0; t < TOK; ++t) {
            if (t >= d.nt) break;
            float* o = y + int64_t(d.s0 + t) * a.y_stride + d.row0 + r;
            if (a.mode == BM_RESIDUAL) *o += acc_t[t];
            else *o = acc_t[t];
          }
      } else if (!swiglu) {
        if (valid)
#pragma unroll
          for (int t = 0; t < TOK; ++t) {
            if (t >= d.nt) break;
            a.out[int64_t(d.s0 + t) * a.out_stride + d.row0 + r] = acc_t[t];
          }
      } else {
        // up rows hand their sums to the gate rows through shared memory
        if (up)
#pragma unroll
          for (int t = 0; t < TOK; ++t) xchg[(r - 64) * (TOK + 1) + t] = acc_t[t];
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (!up && valid)
#pragma unroll
          for (int t = 0; t < TOK; ++t) {
            if (t >= d.nt) break;
            const float g = acc_t[t], u = xchg[r * (TOK + 1) + t];
            a.out[int64_t(d.s0 + t) * a.out_stride + d.row0 + r] = (g / (1.f + expf(-g))) * u;
          }
      }
      // the next item's metadata slot is complete; this item's may be reused
      asm volatile("bar.sync 1, 128;" ::: "memory");
      d = dn;
      nslot ^= 1;
#pragma unroll
      for (int q = 0; q < 4; ++q) { sc_cur[q] = sc_nxt[q]; bi_cur[q] = bi_nxt[q]; }
    }
  }
  // ---- tear-down: nothing of this CTA may still be in flight ----
  __syncthreads();
  if (warp == 4 && lane == 0 && *abort_flag) {
    // copies issued for stages no role consumed: wait for them to land
    const int issued = *issued_ctr;
    for (int jj = max(0, issued - S); jj < issued; ++jj) mbar_wait(&full[jj % S], (jj / S) & 1);
  }
  tg_fence_before();
  __syncthreads();
  pdl_launch();
  if (warp == 5) {
    tg_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
  }
}

// ------------------------------------------------------------------ host --
static PFN_cuTensorMapEncodeTiled_v12000 tg_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// {128 bytes, rows, row_bytes / 128 segments[, experts]} with a box of
// {128, box_rows, 1[, 1]}, 128-byte swizzle.
static bool tg_map(CUtensorMap* m, const void* base, int64_t rows, int64_t rb, int box_rows, int experts,
                   int64_t estride) {
  auto enc = tg_encoder();
  if (!enc || rows < 1 || rb % 128 || (reinterpret_cast<uintptr_t>(base) & 15) || (experts > 0 && estride % 16))
    return false;
  const int rank = experts > 0 ? 4 : 3;
  cuuint64_t dims[4] = {128, cuuint64_t(rows), cuuint64_t(rb / 128), cuuint64_t(experts > 0 ? experts : 1)};
  cuuint64_t strides[3] = {cuuint64_t(rb), 128, cuuint64_t(estride)};
  cuuint32_t boxd[4] = {128, cuuint32_t(box_rows), 1, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, rank, const_cast<void*>(base), dims, strides, boxd, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool tg_disabled() {
  static const int off = std::getenv("SWL_NO_TCGEN05") ? 1 : 0;  // diagnostics: the mma.sync grouped GEMM
  return off != 0;
}

bool tgemm_supported(int in, int bits, int dt, int gs) {
  return !tg_disabled() && (bits == 4 || bits == 8) && dt == DT_BF16 && (gs == 64 || gs == 128) && in % TG_KC == 0 &&
         in / gs <= 32 && (in / gs) % 8 == 0;
}

// Weight rows whole 128-byte segments; scale and bias rows 16-byte pieces
// at 16-byte aligned addresses (the epilogue reads them as such).
static bool tg_mat_ok(const BMat& m, int in, int bits) {
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  return m.w && m.wrow == int64_t(in) * bits / 8 && m.wrow % 128 == 0 && al(m.s) && al(m.b) && m.srow % 16 == 0 &&
         m.es % 16 == 0 && m.eb % 16 == 0;
}

bool launch_tgemm(const TGemmArgs& a, int bits, int grid, cudaStream_t st, bool pdl) {
  if (!tgemm_supported(a.in, bits, a.scale_f32 ? DT_F32 : DT_BF16, a.gs) || !a.dg || !a.meta || a.dg_rows < 1)
    return false;
  TGemmMaps M;
  memset(&M, 0, sizeof M);
  const int64_t rb = int64_t(a.in) * bits / 8;
  if (!a.expert_mode) {
    if (a.nseg < 1 || a.nseg > 4 || a.ntok < 1) return false;
    for (int s = 0; s < a.nseg; ++s)
      if (!tg_mat_ok(a.seg[s], a.in, bits) || !tg_map(&M.a[s], a.seg[s].w, a.seg[s].rows, rb, TG_ROWS, 0, 0))
        return false;
  } else {
    const int box = a.mode == BM_SWIGLU ? 64 : TG_ROWS;
    if (!tg_mat_ok(a.eg, a.in, bits) || !tg_mat_ok(a.sg, a.in, bits)) return false;
    if (!tg_map(&M.a[0], a.eg.w, a.eg.rows, rb, box, a.experts, a.eg.ew) ||
        !tg_map(&M.a[2], a.sg.w, a.sg.rows, rb, box, 0, 0))
      return false;
    if (a.mode == BM_SWIGLU) {
      if (!tg_mat_ok(a.eu, a.in, bits) || !tg_mat_ok(a.su, a.in, bits)) return false;
      if (!tg_map(&M.a[1], a.eu.w, a.eu.rows, rb, box, a.experts, a.eu.ew) ||
          !tg_map(&M.a[3], a.su.w, a.su.rows, rb, box, 0, 0))
        return false;
    }
  }
  // expert items: at most TG_EXPERT_TOK slots (N = 16); dense items: 16 tokens (N = 48)
  const int tn = a.expert_mode ? 16 : 48;
  if (!tg_map(&M.b, a.dg, a.dg_rows, a.in, tn, 0, 0)) return false;
  if (a.expert_mode) {
    if (bits == 4) launch(k_tgemm<4, 16>, dim3(grid), dim3(TG_THREADS), size_t(TgLayout<4, 16>::TOTAL) + 1024, st, pdl, a, M);
    else launch(k_tgemm<8, 16>, dim3(grid), dim3(TG_THREADS), size_t(TgLayout<8, 16>::TOTAL) + 1024, st, pdl, a, M);
  } else {
    if (bits == 4) launch(k_tgemm<4, 48>, dim3(grid), dim3(TG_THREADS), size_t(TgLayout<4, 48>::TOTAL) + 1024, st, pdl, a, M);
    else launch(k_tgemm<8, 48>, dim3(grid), dim3(TG_THREADS), size_t(TgLayout<8, 48>::TOTAL) + 1024, st, pdl, a, M);
  }
  path_note("tgemm");
  return true;
}

// ------------------------------------------------ digits, tensor layout --
// One CTA per output row i (expert slot or token): the source row in_map[i]
// (or i), the prologue as k_digitize, then per quantisation group the digit
// scale 127 / max|x| and the three base-254 digits of every value in natural
// order: digit d of value k at dg[(3 i + d) * in + k]; meta[i][g] = (1 / scale,
// sum of the group).
__global__ void __launch_bounds__(256) k_tdigit(const DigitArgs a, const int* in_map, int8_t* dg, int perm4) {
  extern __shared__ __align__(16) float xs[];
  __shared__ float red[64];
  pdl_wait();
  const int row = blockIdx.x, tid = threadIdx.x, in = a.in;
  const int src = in_map ? in_map[row] : row;
  const float* x = a.x + int64_t(src) * a.x_stride;
  for (int i = tid; i < in; i += 256) xs[i] = x[i];
  __syncthreads();
  if (a.prologue == PRO_RMSNORM) {
    float ss = 0.f;
    for (int i = tid; i < in; i += 256) ss += xs[i] * xs[i];
    ss = block_sum(ss, red);
    const float scale = 1.f / sqrtf(ss / float(in) + a.eps);
    for (int i = tid; i < in; i += 256) xs[i] = xs[i] * (scale * a.aux[i]);
  } else if (a.prologue == PRO_GATEDNORM) {
    const float* z = a.aux + int64_t(src) * a.x_stride;
    const int hd = a.head_dim, nh = in / hd, warp = tid >> 5, lane = tid & 31;
    for (int hh = warp; hh < nh; hh += 8) {
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
    for (int i = tid; i < in; i += 256) a.x_out[int64_t(row) * a.x_stride + i] = xs[i];
  // quads of 4 values; a group of gs values is gs / 4 consecutive lanes (16 or 32)
  const int gl = a.gs >> 2;
  int8_t* d0 = dg + int64_t(3 * row) * in;
  for (int base = 0; base < in; base += 1024) {
    const int k = base + 4 * tid;
    const bool ok = k < in;
    const float4 v = ok ? *reinterpret_cast<const float4*>(xs + k) : make_float4(0.f, 0.f, 0.f, 0.f);
    float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    bool fin = isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w);
    float sum = (v.x + v.y) + (v.z + v.w);
    if (!fin) m = INFINITY;
    for (int o = 1; o < gl; o <<= 1) {
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      sum += __shfl_xor_sync(0xffffffffu, sum, o);
    }
    float inv, rs;
    digit_scale(m, inv, rs);
    uint32_t b[3] = {0u, 0u, 0u};
    put_digits(v.x * inv, 0, b);
    put_digits(v.y * inv, 1, b);
    put_digits(v.z * inv, 2, b);
    put_digits(v.w * inv, 3, b);
    if (perm4) {
      // 4-bit weights: within each block of 8 values the order is
      // 0, 2, 4, 6, 1, 3, 5, 7 (the tensor-core unpack's nibble order); the
      // thread of values 0-3 writes the first word, its neighbour the second
      const bool first = (tid & 1) == 0;
#pragma unroll
      for (int dd = 0; dd < 3; ++dd) {
        const uint32_t other = __shfl_xor_sync(0xffffffffu, b[dd], 1);
        const uint32_t lo = first ? b[dd] : other, hi = first ? other : b[dd];  // values 0-3 | 4-7
        b[dd] = first ? __byte_perm(lo, hi, 0x6420) : __byte_perm(lo, hi, 0x7531);
      }
    }
    if (ok) {
#pragma unroll
      for (int dd = 0; dd < 3; ++dd) *reinterpret_cast<uint32_t*>(d0 + int64_t(dd) * in + k) = b[dd];
      if ((tid & (gl - 1)) == 0) a.meta[int64_t(row) * a.meta_row + k / a.gs] = make_float2(rs, sum);
    }
  }
}

void launch_tdigit(const DigitArgs& a, const int* in_map, int8_t* dg, int bits, cudaStream_t st, bool pdl) {
  if (a.rows <= 0) return;
  if (a.in % 256 || (a.gs != 64 && a.gs != 128) || a.in > 16384)
    throw Error(ERR_UNSUPPORTED, "tensor-core digits: unsupported input size or group");
  launch(k_tdigit, dim3(a.rows), dim3(256), size_t(a.in) * 4, st, pdl, a, in_map, dg, bits == 4 ? 1 : 0);
}

}  // namespace swl
