// Launch interface of the decode-path kernels (sm_100a).
#pragma once

#include "common.h"

namespace swl {

// Per-sequence device state, reached through one indirection so that a
// captured CUDA graph serves every sequence: the host copies the sequence's
// descriptor into the model's "current" slot before replaying.
struct StateDev {
  int* pos;         // tokens already processed (RoPE offset, ring slot)
  float** conv;     // [layers] conv ring [conv_k][conv_dim] (slot = pos % conv_k), DeltaNet layers
  float** dstate;   // [layers] delta state [nv][dv][dk]
  float** kc;       // [layers] K cache [kv_heads][max_ctx][head_dim], attention layers
  float** vc;       // [layers] V cache
  int max_ctx;
};

// Optional per-block timeline (SWL_TRACE): each CTA appends one record of
// {kernel tag, block, start ns, after-dependency-wait ns, inputs-staged ns,
// main-loop-done ns, end ns} (the two middle marks are 0 where a kernel does
// not set them).
constexpr int kTraceFields = 7;
struct Trace {
  unsigned long long* buf = nullptr;  // [cap][kTraceFields]
  unsigned* count = nullptr;
  unsigned cap = 0;
  unsigned tag = 0;
};

// Input transform applied by a GEMV prologue while staging x in shared memory.
enum Prologue : int {
  PRO_COPY = 0,      // x as given
  PRO_RMSNORM = 1,   // rmsnorm(x) * w (eps)
  PRO_GATEDNORM = 2, // per head: rmsnorm(y) * w * g, g = silu(z) given (DeltaNet output gate)
};
enum Epilogue : int {
  EPI_STORE = 0,     // y[row] = acc
  EPI_RESIDUAL = 1,  // y[row] += acc
};

struct GemvSeg {
  QLin lin;
  float* y;
};

struct GemvArgs {
  GemvSeg seg[4];
  int nseg = 0;
  int in = 0;
  int prologue = PRO_COPY;
  int epilogue = EPI_STORE;
  const float* x = nullptr;     // input vector [in] (PRO_GATEDNORM: y)
  const float* aux = nullptr;   // norm weight (RMSNORM) / silu(z) vector (GATEDNORM)
  const float* aux2 = nullptr;  // GATEDNORM: per-dim norm weight [head_dim]
  int head_dim = 0;             // GATEDNORM head size
  float eps = 1e-6f;
  float* x_out = nullptr;       // block 0 stores the prepared x here (optional)
  int* argmax_out = nullptr;    // optional fused greedy argmax over segment 0 rows
  float* argmax_val = nullptr;  // scratch [gridDim] values for argmax
  int* argmax_idx = nullptr;    // scratch [gridDim] indices
  unsigned* counter = nullptr;  // last-block counter for argmax
  int* status = nullptr;        // bit 0: a bounded wait inside the kernel gave up
  int smem_kb = 0;              // shared-memory budget of the streaming kernel (0: default)
  Trace trace;
};

struct RouterArgs {
  QLin gate;        // [E, D]
  QLin sgate;       // shared_expert_gate [1, D]
  const float* h;   // residual stream
  const float* norm_w;
  float eps;
  float* x_out;     // normalised input for the experts [D]
  float* logits;    // scratch [E + 1]
  int* pick_ids;    // [K]
  float* pick_w;    // [K] combine weights (renormalised when norm_topk)
  float* shared_scale;  // sigmoid(shared gate logit)
  unsigned* counter;
  int topk;
  int norm_topk;
  const uint8_t* pool;        // expert blobs of this layer (L2 prefetch of the picks), may be null
  int64_t pool_stride;
  uint32_t prefetch_bytes;    // bytes per expert to prefetch (multiple of 16)
  int* status = nullptr;      // bit 0: a bounded wait inside the kernel gave up
  int skip_topk = 0;          // the expert kernels route from the logits themselves
  Trace trace;
};

struct MoeArgs {
  ExpertProj g, u, d;          // routed experts of this layer (pool addressing)
  QLin sg, su, sd;             // shared expert
  const float* x;              // [D] normalised
  int* pick_ids;
  float* pick_w;
  float* shared_scale;
  float* hmid;                 // [(K+1) * max_inter]
  int hmid_stride;
  int topk;
  float* h;                    // residual stream (down + combine adds here)
  const StateDev* advance_sd;  // when set: ++*advance_sd->pos and ++*advance_cursor after the layer
  int* advance_cursor;
  int* status = nullptr;       // bit 0: a bounded wait inside the kernel gave up
  // When set (integer tensor-core kernels only): the expert kernels compute
  // the routing themselves from the router's E + 1 logits (the router then
  // skips its top-k); gate/up CTA 0 also stores pick_ids / pick_w /
  // shared_scale for observers.
  const float* logits = nullptr;
  int experts = 0;
  int norm_topk = 0;
  int smem_kb = 0;             // shared-memory budget of the gate/up kernel (0: default)
  Trace trace;
};

struct DeltaArgs {
  const float* proj;       // in-projection outputs of this token
  int split;               // 1: [qkv | z | b | a]; 0: qwen3_next interleaved qkvz then ba
  int nk, nv, dk, dv, conv_k, conv_dim;
  const float* conv_w;     // [conv_dim][conv_k]
  const float* a_log;      // [nv]
  const float* dt_bias;    // [nv]
  const StateDev* sd;
  int layer;
  int rows_per_block;      // dv rows per block
  float* y;                // [nv*dv] raw recurrence output
  float* z;                // [nv*dv] silu of the gate input, de-interleaved
  Trace trace;
};

struct AttnArgs {
  const float* qout;       // [H * 2 * hd] (per head: q | gate)
  const float* knew;       // [Hkv * hd]
  const float* vnew;       // [Hkv * hd]
  const float* qn;         // q_norm weight [hd]
  const float* kn;         // k_norm weight [hd]
  float eps;
  float rope_theta;
  int rot;
  int H, Hkv, hd;
  int nchunks;             // grid.y: context chunks per kv head
  int chunk_cap;           // max positions per chunk (smem sizing)
  const StateDev* sd;
  int layer;
  float* part;             // [Hkv][nchunks / 8][G][hd + 2] per-cluster partials
  unsigned* counters;      // [Hkv][8] per kv head and combine slice
  float* out;              // [H * hd] gated attention output
  int* status = nullptr;   // bit 0: a bounded wait inside the kernel gave up
  Trace trace;
};

struct EmbedArgs {
  QLin table;
  const int* tokens;
  const int* cursor;
  float* h;
  int vocab;
  int* err;
  Trace trace;
};

// All launches go to `stream`; `pdl` enables programmatic dependent launch.
void launch_gemv(const GemvArgs& a, cudaStream_t stream, bool pdl);
void launch_router(const RouterArgs& a, int experts, cudaStream_t stream, bool pdl);
void launch_moe_gateup(const MoeArgs& a, cudaStream_t stream, bool pdl);
void launch_moe_down(const MoeArgs& a, cudaStream_t stream, bool pdl);
// True when both expert launches for `a` take the integer tensor-core kernels,
// which can compute the routing from the router logits (MoeArgs::logits).
bool moe_routes_from_logits(const MoeArgs& a, int experts);
void launch_delta(const DeltaArgs& a, cudaStream_t stream, bool pdl);
void launch_attn(const AttnArgs& a, cudaStream_t stream, bool pdl);
void launch_embed(const EmbedArgs& a, int hidden, cudaStream_t stream, bool pdl);
// Debug/test helper: dequantise rows [r0, r1) of a module to f32.
void launch_dequant(const QLin& l, int64_t r0, int64_t r1, float* out, cudaStream_t stream);

int sm_count();

}  // namespace swl
