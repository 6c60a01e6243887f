// Host-side dispatch of the weight-streaming kernels (kernels in
// gemv_impl.cuh, instantiated per weight format in gemv_fmt_*.cu).
//
// Grids are sized to one wave of at most kBlocksPerSm CTAs per SM so that
// every CTA is resident at once and the next kernel (programmatic dependent
// launch) can start on the rest of each SM.
#include <algorithm>

#include "kernels.h"

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

void launch_gemv(const GemvArgs& a, cudaStream_t st, bool pdl) {
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
}

void launch_router(const RouterArgs& r, int E, cudaStream_t st, bool pdl) {
  if (r.gate.bits != r.sgate.bits || r.gate.dt != r.sgate.dt || r.gate.row_bytes != r.sgate.row_bytes ||
      r.gate.srow != r.sgate.srow)
    throw Error(ERR_UNSUPPORTED, "router and shared-expert gate differ in format");
  if (r.topk > 64) throw Error(ERR_UNSUPPORTED, "top-k above 64");
  const int LPR = lanes_per_row(r.gate.row_bytes), spw = 32 / LPR;
  const int CPL = cpl_of(r.gate, LPR), nslab = slabs_of(r.gate.row_bytes, LPR, CPL);
  const QLin lins[2] = {r.gate, r.sgate};
  float* const ys[2] = {r.logits, r.logits + E};
  const SegTab T = make_tab(lins, ys, 2, 1);
  const int grid = grid_for(T.task0[2], spw);
  const int wpc = wpc_of(r.gate.bits, r.gate.dt);
  const size_t smem = size_t(std::max(r.gate.in + r.gate.in / wpc + 4 + 32 + 4 + 2 * r.gate.in, E + 32)) * 4;
  const int gss = gs_shift_of(r.gate);
#define CALL(B, D) router_fmt<B, D>(r, T, E, CPL, gss, LPR, nslab, grid, smem, st, pdl)
  SWL_DISPATCH_FMT(r.gate.bits, r.gate.dt, CALL);
#undef CALL
}

void launch_moe_gateup(const MoeArgs& m, cudaStream_t st, bool pdl) {
  const QLin& g = m.g.lin;
  if (m.sg.bits != g.bits || m.sg.dt != g.dt || m.sg.row_bytes != g.row_bytes || m.u.lin.row_bytes != g.row_bytes ||
      m.su.row_bytes != g.row_bytes || m.sg.srow != g.srow)
    throw Error(ERR_UNSUPPORTED, "shared and routed experts differ in format");
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
}

void launch_moe_down(const MoeArgs& m, cudaStream_t st, bool pdl) {
  const QLin& d = m.d.lin;
  if (m.sd.bits != d.bits || m.sd.dt != d.dt || m.sd.row_bytes != d.row_bytes || m.sd.srow != d.srow)
    throw Error(ERR_UNSUPPORTED, "shared and routed experts differ in format");
  if (m.topk + 1 > 16) throw Error(ERR_UNSUPPORTED, "more than 15 routed experts per token");
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
}

}  // namespace swl
