// Launch descriptor of the warp-specialised "slice" weight-streaming kernels
// (slice_impl.cuh): each CTA owns a contiguous slice of weight rows, which a
// producer warp bulk-copies into a ring of shared-memory tiles, before the
// kernel's dependency wait where the weights allow it. Shared by host
// dispatch (gemv.cu) and device code.
#pragma once

#include <cstdint>

#include <cuda.h>

namespace swl {

constexpr int SL_CW = 4;                // consumer warps per CTA
constexpr int SL_NT = SL_CW * 32;       // consumer threads
constexpr int SL_T = SL_NT + 32;        // + one producer warp
constexpr int SL_RED = 288;             // floats of reduction scratch (32 + 2 * 128)

struct SliceTab {
  // up to four same-format matrices, rows concatenated (dense GEMV / router)
  const uint8_t* w[4];
  const uint8_t* s[4];
  const uint8_t* b[4];
  float* y[4];
  int cum[5];        // cumulative row starts of the segments
  int nseg;
  int total;         // rows over all segments (dense), output rows (down)
  int rpc;           // rows per CTA (dense / down); CTA b owns [b*rpc, (b+1)*rpc)
  int sh_rpc;        // gate/up: shared-expert rows per CTA
  int rt_rpc;        // gate/up: routed rows per CTA (over topk * inter)
  int rb;            // weight row bytes
  int srow;          // scale (and bias) entries per row
  int TR;            // rows per tile
  int S;             // ring slots
  int slot;          // bytes per slot
  int LPR;           // lanes per row (power of two)
  int W;             // K windows (warp groups splitting a row's chunks)
  int gs_shift;      // log2(group size)
  int off_xs, off_cs, off_red, off_part, off_raw, off_bar;  // dynamic smem offsets (ring at 0)
  int* status;       // bit 0 set when a bounded wait gave up (may be null)
  int kpg() const { return (1 << gs_shift) >> 5; }  // 32-weight blocks per group
};

// Tensor maps of the weight matrices an integer tensor-core launch streams,
// each {128 bytes, rows, row / 128 segments[, experts]} with the 128-byte
// swizzle (dense: one per segment; gate/up: shared gate, shared up, routed
// gate, routed up; down: shared down, -, routed down). Passed by value as a
// __grid_constant__ kernel parameter.
struct TileMaps {
  CUtensorMap m[4];
};

// Router epilogue run by the last CTA: softmax over E logits, top-k and the
// combine weights, sigmoid of the shared-expert gate logit.
struct RouterTail {
  const float* logits = nullptr;  // [E + 1] (null: no router epilogue)
  int E = 0;
  int topk = 0;
  int norm_topk = 0;
  int* pick_ids = nullptr;
  float* pick_w = nullptr;
  float* shared_scale = nullptr;
  unsigned* counter = nullptr;
};

}  // namespace swl
