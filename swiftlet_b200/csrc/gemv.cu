// Host-side dispatch of the weight-streaming kernels (kernels in
// gemv_impl.cuh, instantiated per weight format in gemv_fmt_*.cu).
//
// Grids are sized to one wave of at most kBlocksPerSm CTAs per SM so that
// every CTA is resident at once and the next kernel (programmatic dependent
// launch) can start on the rest of each SM.
#include <algorithm>
#include <cstdlib>
#include <mutex>

#include <cudaTypedefs.h>

#include "kernels.h"
#include "launch.h"
#include "slice.h"

namespace swl {

struct SegTab {
  const uint8_t* w[4];
  const uint8_t* s[4];
  const uint8_t* b[4];
  float* y[4];
  int task0[5];
  int rows[4];
  int nseg;
};

template <int B, int D>
void gemv_fmt(const GemvArgs&, const SegTab&, int, int, int, int, int, int, size_t, cudaStream_t, bool);
template <int B, int D>
void router_fmt(const RouterArgs&, const SegTab&, int, int, int, int, int, int, size_t, cudaStream_t, bool);
template <int B, int D>
void gateup_fmt(const MoeArgs&, int, int, int, int, int, int, int, int, size_t, cudaStream_t, bool);
template <int B, int D>
void down_fmt(const MoeArgs&, int, int, int, int, int, int, size_t, cudaStream_t, bool);
template <int B, int D>
void sgemv_fmt(const GemvArgs&, const SliceTab&, const RouterTail&, int, int, size_t, cudaStream_t, bool);
template <int B, int D>
void sgateup_fmt(const MoeArgs&, const SliceTab&, int, size_t, cudaStream_t, bool);
template <int B, int D>
void sdown_fmt(const MoeArgs&, const SliceTab&, int, size_t, cudaStream_t, bool);
template <int B, int D>
void igemv_fmt(const GemvArgs&, const SliceTab&, const TileMaps&, const RouterTail&, int, int, size_t, cudaStream_t,
               bool);
template <int B, int D>
void igateup_fmt(const MoeArgs&, const SliceTab&, const TileMaps&, int, int, size_t, cudaStream_t, bool);
template <int B, int D>
void idown_fmt(const MoeArgs&, const SliceTab&, const TileMaps&, int, int, size_t, cudaStream_t, bool);
constexpr int kImmaWarps = 8;  // consumer warps of the tensor-core kernels (IW)

constexpr int GT = 128;
static constexpr int kBlocksPerSm = 2;

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

static bool full_format(int bits, int dt) { return bits != 0 && dt != DT_F16; }
static int lanes_per_row(int64_t row_bytes) {
  const int64_t nch = row_bytes >> 4;
  int l = 32;
  while (l > 1 && l > nch) l >>= 1;
  return l;
}
static int wpc_of(int bits, int dt) { return bits == 4 ? 32 : bits == 8 ? 16 : (dt == DT_F32 ? 4 : 8); }
static int cpl_of(const QLin& l, int LPR) {
  if (!full_format(l.bits, l.dt)) return 4;
  const int64_t need = ((l.row_bytes >> 4) + LPR - 1) / LPR;
  return need <= 1 ? 1 : need <= 2 ? 2 : 4;
}
static int slabs_of(int64_t row_bytes, int LPR, int CPL) {
  const int64_t per = int64_t(LPR) * CPL;
  return int(((row_bytes >> 4) + per - 1) / per);
}
static int gs_shift_of(const QLin& l) {
  if (!l.bits) return 0;
  int s = 0;
  while ((1 << s) < l.gs) ++s;
  if ((1 << s) != l.gs) throw Error(ERR_UNSUPPORTED, "group size must be a power of two");
  return s;
}
static int slots(int spw) { return sm_count() * kBlocksPerSm * (GT / 32) * spw; }
// Rows per task: the largest R that still gives every sub-warp slot a task.
static int pick_r(const QLin& l, int rows, int spw, int rmax) {
  if (!full_format(l.bits, l.dt)) return 1;
  const int n = slots(spw);
  if (rmax >= 4 && (rows + 3) / 4 >= n) return 4;
  if (rmax >= 2 && (rows + 1) / 2 >= n) return 2;
  return 1;
}
static int grid_for(int tasks, int spw) {
  const int per_block = (GT / 32) * spw;
  return std::max(1, std::min((tasks + per_block - 1) / per_block, sm_count() * kBlocksPerSm));
}

#define SWL_DISPATCH_FMT(BITS_, DT_, CALL)                               \
  do {                                                                   \
    const int b_ = (BITS_), d_ = (DT_);                                  \
    if (b_ == 4 && d_ == DT_BF16) CALL(4, DT_BF16);                      \
    else if (b_ == 4 && d_ == DT_F32) CALL(4, DT_F32);                   \
    else if (b_ == 4 && d_ == DT_F16) CALL(4, DT_F16);                   \
    else if (b_ == 8 && d_ == DT_BF16) CALL(8, DT_BF16);                 \
    else if (b_ == 8 && d_ == DT_F32) CALL(8, DT_F32);                   \
    else if (b_ == 8 && d_ == DT_F16) CALL(8, DT_F16);                   \
    else if (b_ == 0 && d_ == DT_F32) CALL(0, DT_F32);                   \
    else if (b_ == 0 && d_ == DT_BF16) CALL(0, DT_BF16);                 \
    else if (b_ == 0 && d_ == DT_F16) CALL(0, DT_F16);                   \
    else throw Error(ERR_UNSUPPORTED, "unsupported weight format");      \
  } while (0)

#define SWL_DISPATCH_IMMA(BITS_, DT_, CALL)                              \
  do {                                                                   \
    const int b_ = (BITS_), d_ = (DT_);                                  \
    if (b_ == 4 && d_ == DT_BF16) CALL(4, DT_BF16);                      \
    else if (b_ == 4 && d_ == DT_F32) CALL(4, DT_F32);                   \
    else if (b_ == 4 && d_ == DT_F16) CALL(4, DT_F16);                   \
    else if (b_ == 8 && d_ == DT_BF16) CALL(8, DT_BF16);                 \
    else if (b_ == 8 && d_ == DT_F32) CALL(8, DT_F32);                   \
    else if (b_ == 8 && d_ == DT_F16) CALL(8, DT_F16);                   \
    else throw Error(ERR_UNSUPPORTED, "unsupported weight format");      \
  } while (0)

static SegTab make_tab(const QLin* lins, float* const* ys, int n, int R) {
  SegTab T = {};
  T.nseg = n;
  T.task0[0] = 0;
  for (int s = 0; s < 4; ++s) {
    const QLin& l = lins[s < n ? s : 0];
    T.w[s] = l.w; T.s[s] = l.s; T.b[s] = l.b; T.y[s] = ys[s < n ? s : 0]; T.rows[s] = s < n ? l.out : 0;
    T.task0[s + 1] = T.task0[s] + (s < n ? (l.out + R - 1) / R : 0);
  }
  return T;
}

// ------------------------------------------------------ slice planning --
// Shared memory per slice CTA: at most about half an SM, so that the CTA of
// the next kernel (programmatic dependent launch) fits beside it and copies
// its weights while this one runs.
static constexpr size_t kSliceSmem = 110 * 1024;
// Budget of the launch being planned (GemvArgs / MoeArgs::smem_kb, else the
// default above): a kernel whose neighbours in the launch sequence are small
// may take more, so that all of its tiles are copied before its wait.
static thread_local size_t g_budget = kSliceSmem;
struct BudgetScope {
  size_t old;
  explicit BudgetScope(int kb) : old(g_budget) { g_budget = kb > 0 ? size_t(kb) * 1024 : kSliceSmem; }
  ~BudgetScope() { g_budget = old; }
};

static bool slice_enabled() {
  static const int on = std::getenv("SWL_LEGACY_GEMV") ? 0 : 1;  // diagnostics: the register-streaming kernels
  return on != 0;
}
static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
static int scale_bytes(int dt) { return dt == DT_F32 ? 4 : 2; }

// Formats and layouts the slice kernels take: 16-byte aligned rows, scale rows
// and base pointers (bulk copies), inputs of at most 4096 values (staging
// registers), power-of-two groups.
static bool slice_fmt_ok(const QLin& l) {
  if (l.bits != 0 && l.bits != 4 && l.bits != 8) return false;
  if (l.row_bytes % 16 || !aligned16(l.w) || l.in > 4096 || l.in % 32) return false;
  if (l.bits) {
    if ((l.srow * scale_bytes(l.dt)) % 16 || !aligned16(l.s) || !aligned16(l.b)) return false;
    if (l.gs <= 0 || (l.gs & (l.gs - 1))) return false;
  }
  return true;
}
static int row_total(const QLin& l) {
  return int(l.row_bytes) + (l.bits ? 2 * int(l.srow) * scale_bytes(l.dt) : 0);
}
// Lanes per row, K windows and rows per tile for R rows per sub-warp.
static void slice_geom(const QLin& l, int R, SliceTab& T) {
  const int cpl = 64 / wpc_of(l.bits, l.dt), nch = int(l.row_bytes >> 4);
  int lpr = 1;
  while (lpr < 32 && lpr * cpl < nch) lpr <<= 1;
  T.LPR = lpr;
  T.W = std::max(1, (nch + 32 * cpl - 1) / (32 * cpl));
  T.TR = (SL_CW / T.W) * (32 / lpr) * R;
  T.rb = int(l.row_bytes);
  T.srow = l.bits ? int(l.srow) : 0;
  T.gs_shift = gs_shift_of(l);
}
// Lays out [ring | xs | cs | red | part | raw | barriers]; returns the bytes.
static size_t slice_layout(SliceTab& T, int xs_f, int cs_f, int part_f, int raw_f) {
  auto al = [](size_t v, size_t a) { return (v + a - 1) / a * a; };
  size_t off = size_t(T.S) * T.slot;
  off = al(off, 16); T.off_xs = int(off); off += size_t(xs_f) * 4;
  off = al(off, 16); T.off_cs = int(off); off += size_t(cs_f) * 4;
  off = al(off, 16); T.off_red = int(off); off += SL_RED * 4;
  off = al(off, 16); T.off_part = int(off); off += size_t(part_f) * 4;
  off = al(off, 16); T.off_raw = int(off); off += size_t(raw_f) * 4;
  off = al(off, 8); T.off_bar = int(off); off += size_t(2 * T.S) * 8;
  return off;
}
// Ring slots: as many tiles as the CTA has, within the shared-memory budget.
static bool slice_ring(SliceTab& T, int max_tiles, int xs_f, int cs_f, int part_f, int raw_f, size_t& smem) {
  T.S = 0;
  const size_t stage = slice_layout(T, xs_f, cs_f, part_f, raw_f);
  if (stage + size_t(T.slot) + 16 > g_budget) return false;
  const int fit = int((g_budget - stage - 16) / (size_t(T.slot) + 16));
  T.S = std::max(1, std::min({max_tiles, fit, 32}));
  smem = slice_layout(T, xs_f, cs_f, part_f, raw_f);
  return smem <= g_budget;
}

// Dense GEMV over up to four same-format segments; R = rows per sub-warp and tile.
static bool plan_dense(const QLin* lins, float* const* ys, int nseg, int in, int prologue, int head_dim,
                       const float* x, const float* aux, const float* aux2, const float* x_out, int* status,
                       SliceTab& T, int& R, int& grid, size_t& smem) {
  if (!slice_enabled()) return false;
  const QLin& l0 = lins[0];
  for (int s = 0; s < nseg; ++s) if (!slice_fmt_ok(lins[s]) || lins[s].in != in) return false;
  if (prologue == PRO_GATEDNORM && (head_dim <= 0 || head_dim % 32)) return false;
  if (!aligned16(x) || !aligned16(aux) || !aligned16(aux2) || !aligned16(x_out)) return false;
  T = SliceTab{};
  slice_geom(l0, 1, T);
  R = T.LPR >= 4 ? 4 : 1;
  slice_geom(l0, R, T);
  T.nseg = nseg;
  T.cum[0] = 0;
  for (int s = 0; s < 4; ++s) {
    const int k = s < nseg ? s : 0;
    T.w[s] = lins[k].w; T.s[s] = lins[k].s; T.b[s] = lins[k].b; T.y[s] = ys[k];
    T.cum[s + 1] = T.cum[s] + (s < nseg ? lins[s].out : 0);
  }
  T.total = T.cum[nseg];
  if (T.total <= 0) return false;
  T.rpc = std::max((T.total + sm_count() - 1) / sm_count(), T.TR);
  grid = (T.total + T.rpc - 1) / T.rpc;
  T.slot = T.TR * row_total(l0);
  const int max_tiles = (T.rpc + T.TR - 1) / T.TR + nseg - 1;
  const int wpc = wpc_of(l0.bits, l0.dt);
  T.status = status;
  return slice_ring(T, max_tiles, in, in / wpc + 4, T.W > 1 ? T.W * T.rpc : 0, in, smem);
}

// ------------------------------------------------------- tensor maps -----
// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against the driver library).
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    cudaGetLastError();
  });
  return fn;
}
// Map of a row-major matrix of `rows` rows of rb bytes (rb % 128 == 0) as
// {128 bytes, rows, rb / 128 segments[, experts at estride bytes]}: a box of
// `box` rows lands in shared memory as [segment][row][128 bytes], 128-byte
// swizzled (16-byte chunk c of row r at chunk c ^ (r & 7)).
static bool encode_rows(CUtensorMap* m, const void* base, int64_t rows, int64_t rb, int box, int experts,
                        int64_t estride) {
  auto enc = tensor_map_encoder();
  if (!enc || rows < 1 || rb % 128 || rb / 128 > 256 || !aligned16(base) || (experts > 0 && estride % 16)) return false;
  const int rank = experts > 0 ? 4 : 3;
  cuuint64_t dims[4] = {128, cuuint64_t(rows), cuuint64_t(rb / 128), cuuint64_t(experts > 0 ? experts : 1)};
  cuuint64_t strides[3] = {cuuint64_t(rb), 128, cuuint64_t(estride)};
  cuuint32_t boxd[4] = {128, cuuint32_t(box), cuuint32_t(rb / 128), 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, rank, const_cast<void*>(base), dims, strides, boxd, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
static int round1024(int v) { return (v + 1023) / 1024 * 1024; }

// ------------------------------------------- integer tensor-core planning --
// 4/8-bit weights with groups of >= 32 take the mma.sync (u8 x s8) kernels of
// imma_impl.cuh; slots hold rows at a 16-byte padded pitch.
static bool imma_enabled() {
  static const int on = std::getenv("SWL_NO_IMMA") ? 0 : 1;  // diagnostics: the f32 slice kernels
  return on != 0;
}
static bool imma_fmt_ok(const QLin& l) {
  return slice_fmt_ok(l) && (l.bits == 4 || l.bits == 8) && l.gs >= 32 && l.gs <= 128 && (l.in / l.gs) % 4 == 0;
}
// Warps per tile (K split) and ring slots for a CTA of `tiles` tiles
// (`max_tiles` at most) and `ngroups` quantisation groups per row: the fewest
// rounds of tile work, counting a split tile as 1 / KS of a tile plus a small
// cost for the combine. Tile i goes to warp group i % NG (NG = warps / KS);
// when slots are reused (more tiles than slots) the slot count must be a
// multiple of NG, so that every slot belongs to one group, which waits for its
// phases in order (a wait on the parity of a phase two ahead would alias).
// Lays out the shared memory for the chosen slot count.
static bool settle_ks(SliceTab& T, int tiles, int max_tiles, int ngroups, int xs_f, int cs_f, int part_f, int raw_f,
                      size_t& smem) {
  int best = 0, best_s = 0;
  double best_cost = 1e30;
  for (int ks : {1, 2, 4, 8}) {
    if (ngroups % (4 * ks)) continue;  // whole steps of four groups per warp, each starting on a 128-byte segment
    const int ng = kImmaWarps / ks;
    int S = T.S;
    if (max_tiles > S) S = S / ng * ng;
    if (S < 1) continue;
    // a combine (named barrier, partials through shared memory) costs about
    // 0.3 of a whole tile's reduction on B200: measured as the decode step's
    // time with this weight swept from 0.08 to 2 (best at 0.3; at 0.08 the
    // 6-tile in-projections split 4 ways over 3 rounds)
    const double cost = double((tiles + ng - 1) / ng) * (1.0 / ks + (ks > 1 ? 0.3 : 0.0));
    if (cost < best_cost - 1e-9) { best_cost = cost; best = ks; best_s = S; }
  }
  if (!best) return false;
  T.W = best;
  T.S = best_s;
  smem = slice_layout(T, xs_f, cs_f, part_f, raw_f);
  if (smem > g_budget) return false;
  smem += 1024;  // the kernel aligns its ring to 1024 bytes
  return true;
}
// One matrix block of a slot: box rows of weights, scale rows and bias rows,
// rounded to 1024 bytes (the next block's swizzled weights stay aligned).
static int imma_block_bytes(const QLin& l, int box) {
  return round1024(box * (int(l.row_bytes) + 2 * int(l.srow) * scale_bytes(l.dt)));
}

static bool plan_idense(const QLin* lins, float* const* ys, int nseg, int in, int prologue, int head_dim,
                        const float* x, const float* aux, const float* aux2, const float* x_out, int* status,
                        SliceTab& T, TileMaps& M, int& grid, size_t& smem) {
  if (!slice_enabled() || !imma_enabled()) return false;
  const QLin& l0 = lins[0];
  for (int s = 0; s < nseg; ++s) if (!imma_fmt_ok(lins[s]) || lins[s].in != in) return false;
  if (prologue == PRO_GATEDNORM && (head_dim <= 0 || head_dim % 32)) return false;
  if (!aligned16(x) || !aligned16(aux) || !aligned16(aux2) || !aligned16(x_out)) return false;
  T = SliceTab{};
  T.rb = int(l0.row_bytes);
  T.srow = int(l0.srow);
  T.gs_shift = gs_shift_of(l0);
  T.TR = 16;
  T.nseg = nseg;
  T.cum[0] = 0;
  for (int s = 0; s < 4; ++s) {
    const int k = s < nseg ? s : 0;
    T.w[s] = lins[k].w; T.s[s] = lins[k].s; T.b[s] = lins[k].b; T.y[s] = ys[k];
    T.cum[s + 1] = T.cum[s] + (s < nseg ? lins[s].out : 0);
  }
  T.total = T.cum[nseg];
  if (T.total <= 0) return false;
  // Large launches (in_proj of the DeltaNet layers, lm_head) take two CTAs
  // per SM, each within 112 KB of shared memory so both stay resident: twice
  // the warps hide the tile loop's dependent latencies (B = 1 decode 501.5 ->
  // 510.2 tok/s on B200, same inputs).
  const bool two = T.total >= 4 * 16 * sm_count();
  const int ctas = two ? 2 * sm_count() : sm_count();
  T.rpc = std::max((T.total + ctas - 1) / ctas, 16);
  grid = (T.total + T.rpc - 1) / T.rpc;
  if (two && g_budget > 112 * 1024) g_budget = 112 * 1024;  // restored by the caller's BudgetScope
  for (int sg = 0; sg < nseg; ++sg)
    if (!encode_rows(&M.m[sg], lins[sg].w, lins[sg].out, lins[sg].row_bytes, 16, 0, 0)) return false;
  T.slot = imma_block_bytes(l0, 16);
  const int max_tiles = (T.rpc + 15) / 16 + nseg - 1;
  T.status = status;
  // xs: B table (3 bytes per input), cs: group sums then group digit scales,
  // part: K-split partials, raw: the staged input
  const int xs_f = 3 * in / 4, cs_f = 2 * (((in >> T.gs_shift) + 3) & ~3) + 4, part_f = 2 * kImmaWarps * 16;
  return slice_ring(T, max_tiles, xs_f, cs_f, part_f, in, smem) &&
         settle_ks(T, (T.rpc + 15) / 16, max_tiles, in >> T.gs_shift, xs_f, cs_f, part_f, in, smem);
}

static bool expert_strides_ok(const ExpertProj& p) {
  return p.wstride % 16 == 0 && p.sstride % 16 == 0 && p.bstride % 16 == 0;
}

// Gate/up: CTA b takes a share of the shared expert's rows and of the routed rows.
static bool plan_gateup(const MoeArgs& m, SliceTab& T, int& grid, size_t& smem) {
  if (!slice_enabled()) return false;
  const QLin& g = m.g.lin;
  if (!slice_fmt_ok(g) || !slice_fmt_ok(m.u.lin) || !slice_fmt_ok(m.sg) || !slice_fmt_ok(m.su)) return false;
  if (!expert_strides_ok(m.g) || !expert_strides_ok(m.u) || m.su.out != m.sg.out || m.sg.in != g.in) return false;
  if (!aligned16(m.x)) return false;
  T = SliceTab{};
  slice_geom(g, 2, T);  // two gate/up row pairs per sub-warp and tile
  if (T.W != 1 || T.LPR < 4) return false;
  const int sh = m.sg.out, nq = m.topk * g.out, n = sm_count();
  T.sh_rpc = std::max(1, (sh + n - 1) / n);
  T.rt_rpc = nq > 0 ? std::max(1, (nq + n - 1) / n) : 0;
  grid = std::max(1, std::max((sh + T.sh_rpc - 1) / T.sh_rpc, nq > 0 ? (nq + T.rt_rpc - 1) / T.rt_rpc : 0));
  T.slot = 2 * T.TR * row_total(g);
  const int max_tiles = (T.sh_rpc + T.TR - 1) / T.TR +
                        (nq > 0 ? (T.rt_rpc + T.TR - 1) / T.TR + (T.rt_rpc + g.out - 1) / g.out + 1 : 0);
  T.status = m.status;
  const int wpc = wpc_of(g.bits, g.dt);
  return slice_ring(T, max_tiles, g.in, g.in / wpc + 4, 0, g.in, smem);
}

// Gate/up: one item of BR rows of one gate/up pair per CTA (the shared
// expert's items first, then K routed slots of ipe items each). BR is the
// smallest multiple of 8 (>= 16) whose items fit one CTA per SM, else two
// CTAs per SM (shared memory permitting), within the shared-memory budget;
// the item's BR / 8 MMA tiles are split over warp groups (KS warps each).
static bool plan_igateup(const MoeArgs& m, SliceTab& T, TileMaps& M, int& grid, size_t& smem) {
  if (!slice_enabled() || !imma_enabled()) return false;
  const QLin& g = m.g.lin;
  if (!imma_fmt_ok(g) || !imma_fmt_ok(m.u.lin) || !imma_fmt_ok(m.sg) || !imma_fmt_ok(m.su)) return false;
  if (!expert_strides_ok(m.g) || !expert_strides_ok(m.u) || m.su.out != m.sg.out || m.sg.in != g.in) return false;
  if (!aligned16(m.x) || g.in > 4096 || m.topk > 16 || m.sg.out < 8 || (m.topk > 0 && g.out < 8)) return false;
  T = SliceTab{};
  T.rb = int(g.row_bytes);
  T.srow = int(g.srow);
  T.gs_shift = gs_shift_of(g);
  T.status = m.status;
  const int sh = m.sg.out, inter = g.out, K = m.topk, sms = sm_count(), ngroups = g.in >> T.gs_shift;
  const int xs_f = 3 * g.in / 4, cs_f = 2 * ((ngroups + 3) & ~3) + 4, part_f = 2 * kImmaWarps * 16;
  const int max_br = std::min(256, (std::min(sh, K > 0 ? inter : sh) / 8) * 8);
  int br = 0;
  size_t br_smem = 0;
  for (int pass = 0; pass < 2 && !br; ++pass) {
    for (int c = 16; c <= max_br && !br; c += 8) {
      const int items = (sh + c - 1) / c + K * ((inter + c - 1) / c);
      T.TR = c;
      T.S = 1;
      T.slot = 2 * imma_block_bytes(g, c);
      const size_t need = slice_layout(T, xs_f, cs_f, part_f, g.in) + 1024;  // + the ring's 1024-byte alignment
      if (need > g_budget) break;  // larger items only need more
      if (pass == 0 ? items <= sms : (items <= 2 * sms && need <= 113 * 1024)) {
        br = c;
        br_smem = need;
      }
    }
  }
  if (!br) return false;
  T.TR = br;
  T.S = 1;
  T.slot = 2 * imma_block_bytes(g, br);
  smem = br_smem;
  slice_layout(T, xs_f, cs_f, part_f, g.in);
  grid = (sh + br - 1) / br + K * ((inter + br - 1) / br);
  if (!encode_rows(&M.m[0], m.sg.w, m.sg.out, m.sg.row_bytes, br, 0, 0) ||
      !encode_rows(&M.m[1], m.su.w, m.su.out, m.su.row_bytes, br, 0, 0))
    return false;
  if (K > 0 && (m.g.count < 1 || m.u.count < 1 ||
                !encode_rows(&M.m[2], g.w, g.out, g.row_bytes, br, m.g.count, m.g.wstride) ||
                !encode_rows(&M.m[3], m.u.lin.w, m.u.lin.out, m.u.lin.row_bytes, br, m.u.count, m.u.wstride)))
    return false;
  // warp groups per item: the fewest rounds of tile work, a combine costing
  // 0.3 of a tile (as settle_ks)
  const int tiles = br / 8;
  double best_cost = 1e30;
  T.W = 0;
  for (int ks : {1, 2, 4, 8}) {
    if (ngroups % (4 * ks)) continue;
    const int ng = kImmaWarps / ks;
    const double cost = double((tiles + ng - 1) / ng) * (1.0 / ks + (ks > 1 ? 0.3 : 0.0));
    if (cost < best_cost - 1e-9) { best_cost = cost; T.W = ks; }
  }
  return T.W > 0;
}

static bool plan_idown(const MoeArgs& m, SliceTab& T, TileMaps& M, int& grid, size_t& smem) {
  if (!slice_enabled() || !imma_enabled()) return false;
  const QLin& d = m.d.lin;
  if (!imma_fmt_ok(d) || !imma_fmt_ok(m.sd) || !expert_strides_ok(m.d)) return false;
  if (m.topk + 1 > 16 || !aligned16(m.hmid) || m.hmid_stride % 4 || m.sd.in != d.in) return false;
  T = SliceTab{};
  T.rb = int(d.row_bytes);
  T.srow = int(d.srow);
  T.gs_shift = gs_shift_of(d);
  const int D = d.out, K1 = m.topk + 1;
  T.total = D;
  T.rpc = std::min(16, (D + sm_count() - 1) / sm_count());
  T.TR = T.rpc;
  grid = (D + T.rpc - 1) / T.rpc;
  if (!encode_rows(&M.m[0], m.sd.w, m.sd.out, m.sd.row_bytes, 16, 0, 0)) return false;
  if (m.topk > 0 && (m.d.count < 1 || !encode_rows(&M.m[2], d.w, d.out, d.row_bytes, 16, m.d.count, m.d.wstride)))
    return false;
  T.slot = imma_block_bytes(d, 16);
  T.status = m.status;
  const int nkb = d.in >> 5;
  // one slot per expert slot (warp e % 8 waits on slot e only once)
  if (!slice_ring(T, K1, K1 * nkb * 24, 2 * ((K1 * (d.in >> T.gs_shift) + 3) & ~3) + 4, K1 * T.rpc,
                  K1 * m.hmid_stride, smem) || T.S != K1)
    return false;
  smem += 1024;  // the kernel aligns its ring to 1024 bytes
  return true;
}

bool moe_routes_from_logits(const MoeArgs& m, int experts) {
  SliceTab T;
  TileMaps M;
  int grid = 0;
  size_t smem = 0;
  return experts <= 512 && m.topk <= 16 && plan_igateup(m, T, M, grid, smem) && plan_idown(m, T, M, grid, smem);
}

// Down: CTA b takes output rows [b*rpc, (b+1)*rpc) of every picked expert.
static bool plan_down(const MoeArgs& m, SliceTab& T, int& grid, size_t& smem) {
  if (!slice_enabled()) return false;
  const QLin& d = m.d.lin;
  if (!slice_fmt_ok(d) || !slice_fmt_ok(m.sd) || !expert_strides_ok(m.d)) return false;
  if (m.topk + 1 > 16 || !aligned16(m.hmid) || m.hmid_stride % 4 || m.sd.in != d.in) return false;
  T = SliceTab{};
  slice_geom(d, 1, T);
  if (T.W != 1 || T.LPR < 4) return false;
  const int D = d.out, K1 = m.topk + 1, wpc = wpc_of(d.bits, d.dt);
  T.total = D;
  T.rpc = (D + sm_count() - 1) / sm_count();
  if (T.rpc > 64) return false;
  grid = (D + T.rpc - 1) / T.rpc;
  T.TR = T.rpc;  // one tile per expert: the CTA's rows
  T.slot = T.TR * row_total(d);
  const int max_tiles = K1;
  T.status = m.status;
  return slice_ring(T, max_tiles, K1 * m.hmid_stride, K1 * (m.hmid_stride / wpc + 4), K1 * T.rpc, K1 * m.hmid_stride,
                    smem);
}

void launch_gemv(const GemvArgs& a, cudaStream_t st, bool pdl) {
  const BudgetScope budget(a.smem_kb);
  const QLin& l0 = a.seg[0].lin;
  for (int s = 1; s < a.nseg; ++s)
    if (a.seg[s].lin.bits != l0.bits || a.seg[s].lin.dt != l0.dt || a.seg[s].lin.row_bytes != l0.row_bytes ||
        a.seg[s].lin.srow != l0.srow)
      throw Error(ERR_UNSUPPORTED, "fused GEMV segments differ in format");
  int rows = 0;
  for (int s = 0; s < a.nseg; ++s) rows += a.seg[s].lin.out;
  const int LPR = lanes_per_row(l0.row_bytes), spw = 32 / LPR;
  const int CPL = cpl_of(l0, LPR), nslab = slabs_of(l0.row_bytes, LPR, CPL);
  const int R = pick_r(l0, rows, spw, CPL >= 4 ? 2 : 4);
  QLin lins[4];
  float* ys[4];
  for (int s = 0; s < a.nseg; ++s) { lins[s] = a.seg[s].lin; ys[s] = a.seg[s].y; }
  {
    SliceTab ST;
    int sgrid = 0, sR = 1;
    size_t ssmem = 0;
    TileMaps TM;
    if (plan_idense(lins, ys, a.nseg, a.in, a.prologue, a.head_dim, a.x, a.aux, a.aux2, a.x_out, a.status, ST, TM,
                    sgrid, ssmem)) {
      const RouterTail none;
#define CALL(B, D) igemv_fmt<B, D>(a, ST, TM, none, ST.kpg(), sgrid, ssmem, st, pdl)
      SWL_DISPATCH_IMMA(l0.bits, l0.dt, CALL);
#undef CALL
      path_note("igemv");
      return;
    }
    if (plan_dense(lins, ys, a.nseg, a.in, a.prologue, a.head_dim, a.x, a.aux, a.aux2, a.x_out, a.status, ST, sR,
                   sgrid, ssmem)) {
      const RouterTail none;
#define CALL(B, D) sgemv_fmt<B, D>(a, ST, none, sR, sgrid, ssmem, st, pdl)
      SWL_DISPATCH_FMT(l0.bits, l0.dt, CALL);
#undef CALL
      path_note("sgemv");
      return;
    }
  }
  const SegTab T = make_tab(lins, ys, a.nseg, R);
  int grid = grid_for(T.task0[a.nseg], spw);
  if (a.argmax_out) grid = std::min(grid, 1024);
  const int wpc = wpc_of(l0.bits, l0.dt);
  const int nh = a.prologue == PRO_GATEDNORM ? a.in / std::max(a.head_dim, 1) : 0;
  const size_t smem = size_t(a.in + a.in / wpc + 4 + 32 + nh + 4 + (a.prologue == PRO_RMSNORM ? 2 : 1) * a.in +
                             (a.prologue == PRO_GATEDNORM ? a.head_dim : 0)) * 4;
  const int gss = gs_shift_of(l0);
#define CALL(B, D) gemv_fmt<B, D>(a, T, R, CPL, gss, LPR, nslab, grid, smem, st, pdl)
  SWL_DISPATCH_FMT(l0.bits, l0.dt, CALL);
#undef CALL
  path_note("gemv");
}

void launch_router(const RouterArgs& r, int E, cudaStream_t st, bool pdl) {
  if (r.gate.bits != r.sgate.bits || r.gate.dt != r.sgate.dt || r.gate.row_bytes != r.sgate.row_bytes ||
      r.gate.srow != r.sgate.srow)
    throw Error(ERR_UNSUPPORTED, "router and shared-expert gate differ in format");
  if (r.topk > 64) throw Error(ERR_UNSUPPORTED, "top-k above 64");
  const QLin lins[2] = {r.gate, r.sgate};
  float* const ys[2] = {r.logits, r.logits + E};
  {
    SliceTab ST;
    int sgrid = 0, sR = 1;
    size_t ssmem = 0;
    TileMaps TM;
    const bool imma = E <= r.gate.in && plan_idense(lins, ys, 2, r.gate.in, PRO_RMSNORM, 0, r.h, r.norm_w, nullptr,
                                                    r.x_out, r.status, ST, TM, sgrid, ssmem);
    if (imma || (E <= r.gate.in && plan_dense(lins, ys, 2, r.gate.in, PRO_RMSNORM, 0, r.h, r.norm_w, nullptr, r.x_out,
                                              r.status, ST, sR, sgrid, ssmem))) {
      GemvArgs a;
      a.seg[0].lin = r.gate; a.seg[0].y = r.logits; a.seg[1].lin = r.sgate; a.seg[1].y = r.logits + E;
      a.nseg = 2; a.in = r.gate.in; a.prologue = PRO_RMSNORM; a.epilogue = EPI_STORE;
      a.x = r.h; a.aux = r.norm_w; a.eps = r.eps; a.x_out = r.x_out; a.status = r.status; a.trace = r.trace;
      RouterTail rt;
      if (!r.skip_topk) rt.logits = r.logits;
      rt.E = E; rt.topk = r.topk; rt.norm_topk = r.norm_topk;
      rt.pick_ids = r.pick_ids; rt.pick_w = r.pick_w; rt.shared_scale = r.shared_scale; rt.counter = r.counter;
      if (imma) {
#define CALL(B, D) igemv_fmt<B, D>(a, ST, TM, rt, ST.kpg(), sgrid, ssmem, st, pdl)
        SWL_DISPATCH_IMMA(r.gate.bits, r.gate.dt, CALL);
#undef CALL
        path_note("igemv");
      } else {
#define CALL(B, D) sgemv_fmt<B, D>(a, ST, rt, sR, sgrid, ssmem, st, pdl)
        SWL_DISPATCH_FMT(r.gate.bits, r.gate.dt, CALL);
#undef CALL
        path_note("sgemv");
      }
      return;
    }
  }
  const int LPR = lanes_per_row(r.gate.row_bytes), spw = 32 / LPR;
  const int CPL = cpl_of(r.gate, LPR), nslab = slabs_of(r.gate.row_bytes, LPR, CPL);
  const SegTab T = make_tab(lins, ys, 2, 1);
  const int grid = grid_for(T.task0[2], spw);
  const int wpc = wpc_of(r.gate.bits, r.gate.dt);
  const size_t smem = size_t(std::max(r.gate.in + r.gate.in / wpc + 4 + 32 + 4 + 2 * r.gate.in, E + 32)) * 4;
  const int gss = gs_shift_of(r.gate);
#define CALL(B, D) router_fmt<B, D>(r, T, E, CPL, gss, LPR, nslab, grid, smem, st, pdl)
  SWL_DISPATCH_FMT(r.gate.bits, r.gate.dt, CALL);
#undef CALL
  path_note("router");
}

void launch_moe_gateup(const MoeArgs& m, cudaStream_t st, bool pdl) {
  const BudgetScope budget(m.smem_kb);
  const QLin& g = m.g.lin;
  if (m.sg.bits != g.bits || m.sg.dt != g.dt || m.sg.row_bytes != g.row_bytes || m.u.lin.row_bytes != g.row_bytes ||
      m.su.row_bytes != g.row_bytes || m.sg.srow != g.srow)
    throw Error(ERR_UNSUPPORTED, "shared and routed experts differ in format");
  {
    SliceTab ST;
    int sgrid = 0;
    size_t ssmem = 0;
    TileMaps TM;
    if (plan_igateup(m, ST, TM, sgrid, ssmem)) {
#define CALL(B, D) igateup_fmt<B, D>(m, ST, TM, ST.kpg(), sgrid, ssmem, st, pdl)
      SWL_DISPATCH_IMMA(g.bits, g.dt, CALL);
#undef CALL
      path_note("igateup");
      return;
    }
    if (plan_gateup(m, ST, sgrid, ssmem)) {
#define CALL(B, D) sgateup_fmt<B, D>(m, ST, sgrid, ssmem, st, pdl)
      SWL_DISPATCH_FMT(g.bits, g.dt, CALL);
#undef CALL
      path_note("sgateup");
      return;
    }
  }
  const int LPR = lanes_per_row(g.row_bytes), spw = 32 / LPR;
  const int CPL = cpl_of(g, LPR), nslab = slabs_of(g.row_bytes, LPR, CPL);
  const int R = pick_r(g, (m.topk + 1) * g.out, spw, CPL >= 4 ? 1 : 2);
  const int tr = (g.out + R - 1) / R, ts = (m.sg.out + R - 1) / R;
  const int grid = grid_for(tr * m.topk + ts, spw);
  const int wpc = wpc_of(g.bits, g.dt);
  const size_t smem = size_t(g.in + g.in / wpc + 4 + 4 + g.in) * 4;
  const int gss = gs_shift_of(g);
#define CALL(B, D) gateup_fmt<B, D>(m, R, CPL, gss, LPR, tr, ts, nslab, grid, smem, st, pdl)
  SWL_DISPATCH_FMT(g.bits, g.dt, CALL);
#undef CALL
  path_note("gateup");
}

void launch_moe_down(const MoeArgs& m, cudaStream_t st, bool pdl) {
  const QLin& d = m.d.lin;
  if (m.sd.bits != d.bits || m.sd.dt != d.dt || m.sd.row_bytes != d.row_bytes || m.sd.srow != d.srow)
    throw Error(ERR_UNSUPPORTED, "shared and routed experts differ in format");
  if (m.topk + 1 > 16) throw Error(ERR_UNSUPPORTED, "more than 15 routed experts per token");
  {
    SliceTab ST;
    int sgrid = 0;
    size_t ssmem = 0;
    TileMaps TM;
    if (plan_idown(m, ST, TM, sgrid, ssmem)) {
#define CALL(B, D_) idown_fmt<B, D_>(m, ST, TM, ST.kpg(), sgrid, ssmem, st, pdl)
      SWL_DISPATCH_IMMA(d.bits, d.dt, CALL);
#undef CALL
      path_note("idown");
      return;
    }
    if (plan_down(m, ST, sgrid, ssmem)) {
#define CALL(B, D_) sdown_fmt<B, D_>(m, ST, sgrid, ssmem, st, pdl)
      SWL_DISPATCH_FMT(d.bits, d.dt, CALL);
#undef CALL
      path_note("sdown");
      return;
    }
  }
  const int LPR = lanes_per_row(d.row_bytes), spw = 32 / LPR;
  const int nslab = int(((d.row_bytes >> 4) + LPR - 1) / LPR);
  const int D = d.out;
  const int R = full_format(d.bits, d.dt) && m.topk + 1 <= 12 && (D + 1) / 2 >= slots(spw) ? 2 : 1;
  if (m.d.wstride != m.d.sstride || m.d.wstride != m.d.bstride)
    throw Error(ERR_UNSUPPORTED, "expert sections must share one blob stride");
  const int grid = grid_for((D + R - 1) / R, spw);
  const int wpc = wpc_of(d.bits, d.dt);
  const size_t smem = (size_t(m.topk + 1) * size_t(2 * m.hmid_stride + m.hmid_stride / wpc + 4) + 4) * 4;
  const int ne = m.topk + 1 <= 4 ? 4 : m.topk + 1 <= 9 ? 9 : m.topk + 1 <= 12 ? 12 : 16;
  const int gss = gs_shift_of(d);
#define CALL(B, D_) down_fmt<B, D_>(m, ne, R, gss, LPR, nslab, grid, smem, st, pdl)
  SWL_DISPATCH_FMT(d.bits, d.dt, CALL);
#undef CALL
  path_note("down");
}

}  // namespace swl
