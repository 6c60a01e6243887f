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
  // Batched decode (grid.z = sequences): sequence b reads sd[b], proj +
  // b * proj_stride and writes y / z + b * nv * dv. 0 for one sequence.
  int64_t proj_stride = 0;
  // Chunked steps (k_delta_seq, k_conv_ring): sequence s owns token rows
  // [seq_first[s], seq_first[s] + seq_n[s]) of proj / y / z, in order.
  const int* seq_first = nullptr;
  const int* seq_n = nullptr;
  Trace trace;
};

// Chunked-parallel delta rule (delta_wy.cu) of a prompt launch: per token the
// normalised q / k rows, v rows and (log g, beta) pairs that k_delta_prep
// writes, per sequence (blockIdx.z) its token range; the state is each
// sequence's own (sd) or, for the kernel-level entry point, one direct state.
struct WyArgs {
  const float* q = nullptr;   // [tokens][q_stride], key head h at h * dk
  const float* k = nullptr;
  const float* v = nullptr;   // [tokens][v_stride], value head h at h * dv
  const float* lg = nullptr;  // [tokens][gb_stride]: (log g, beta) of value head h at 2h, 2h + 1
  float *qw = nullptr, *kw = nullptr, *vw = nullptr, *lgw = nullptr;  // the same buffers, written by the prep
  int64_t q_stride = 0, k_stride = 0, v_stride = 0, gb_stride = 0;
  int nk = 0, nv = 0, dk = 0, dv = 0;
  const StateDev* sd = nullptr;
  int layer = 0;
  float* state = nullptr;     // direct state [nv][dv][dk] (kernel-level entry; sd unused)
  const int* seq_first = nullptr;  // token range of sequence blockIdx.z (null: tokens [0, ntok))
  const int* seq_n = nullptr;
  const int* tok_seq = nullptr;    // prep: sequence and offset of each token
  const int* tok_off = nullptr;
  int ntok = 0;
  float* y = nullptr;         // [tokens][y_stride] recurrence output
  int64_t y_stride = 0;
};
bool delta_wy_supported(int dk, int dv, int nk, int nv, int conv_dim);
void launch_delta_prep(const DeltaArgs& a, const WyArgs& w, int T, cudaStream_t stream, bool pdl);
void launch_delta_wy(const WyArgs& a, int S, cudaStream_t stream, bool pdl);
// Decode step of T sequences (one token each): the per-token inputs
// (k_delta_prep_dec, which also advances the conv ring), then the state.
void launch_delta_prep_dec(const DeltaArgs& a, const WyArgs& w, int T, cudaStream_t stream, bool pdl);
void launch_delta_step(const WyArgs& a, int T, cudaStream_t stream, bool pdl);

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
  // Batched decode (grid.z = sequences): sequence b reads sd[b] and its
  // projections at qout / knew / vnew + b * proj_stride, uses its own
  // partials and counters, and writes out + b * H * hd.
  int64_t proj_stride = 0;
  // Chunked steps (grid.z = tokens): token z belongs to sequence tok_seq[z]
  // at position *pos + tok_off[z]; every key and value of the chunk is
  // already in the cache (k_kv_append), so none is appended or injected.
  const int* tok_seq = nullptr;
  const int* tok_off = nullptr;
  Trace trace;
};

struct EmbedArgs {
  QLin table;
  const int* tokens;
  const int* cursor;       // token index; null: row blockIdx.y takes tokens[blockIdx.y] (batched)
  float* h;
  int vocab;
  int* err;
  Trace trace;
};

// ---------------------------------------------------- batched decode ----
// Several sequences, one token each, go through every layer together: the
// dense projections, the router and lm_head run as one weight stream for all
// of them, and the routed experts as a grouped GEMM over the tokens that
// picked each expert (QwenCPUModel.swift:500-569 computes the same per token).
constexpr int BT_MAX = 64;   // sequences per batched step
constexpr int BG_TOK = 16;   // tokens per GEMM token tile
constexpr int BG_ROWS = 64;  // weight rows per GEMM item (two halves of 32)

// One MLX-affine matrix in HBM, or a stack of same-shaped experts (expert e
// at w + e * ew, s + e * es, b + e * eb).
struct BMat {
  const uint8_t* w = nullptr;
  const uint8_t* s = nullptr;
  const uint8_t* b = nullptr;
  int64_t wrow = 0;  // bytes per weight row
  int64_t srow = 0;  // bytes per scale (and bias) row
  int64_t ew = 0, es = 0, eb = 0;
  int rows = 0;
};

// Activation rows -> integer digit tables for k_bgemm: per row, the
// prologue's output split into three signed base-254 digits per value
// (B-fragment order of the 4-bit weights) and per quantisation group the
// reconstruction scale and the sum of the values.
struct DigitArgs {
  const float* x = nullptr;
  int64_t x_stride = 0;        // floats between input rows
  int rows = 0, in = 0, gs = 0;
  int prologue = PRO_COPY;     // PRO_COPY, PRO_RMSNORM, PRO_GATEDNORM
  const float* aux = nullptr;  // RMSNORM: weight [in]; GATEDNORM: silu(z) rows (x_stride apart)
  const float* aux2 = nullptr; // GATEDNORM: norm weight [head_dim]
  int head_dim = 0;
  float eps = 1e-6f;
  float* x_out = nullptr;      // optional copy of the prepared rows (x_stride apart)
  uint2* bt = nullptr;         // [rows][bt_row]
  float2* meta = nullptr;      // [rows][meta_row] (scale, sum) per group
  int64_t bt_row = 0, meta_row = 0;
};

enum BMode : int { BM_STORE = 0, BM_RESIDUAL = 1, BM_SWIGLU = 2 };

// Shared-memory layout of k_bgemm (bytes), chosen by the launcher.
struct BGLayout {
  int kc = 0;           // input values per pipeline chunk
  int kcb = 0;          // weight bytes per row per chunk
  int gpc = 0, kpg = 0; // quantisation groups per chunk, 32-value blocks per group
  int sw = 0;           // bytes per row of a staged scale (or bias) window
  int bstride = 0;      // uint2 per token in a staged digit table
  int w_off = 0, s_off = 0, b_off = 0, x_off = 0, m_off = 0, stage = 0;
  int o_off = 0;        // epilogue buffer; < 0: reuse the stage just consumed
  int total = 0;
};

struct BGemmArgs {
  int mode = BM_STORE;
  int in = 0;
  BGLayout L;
  // dense launches: up to four segments over one input; item = 64-row block
  // x token tile, rows of segment s at y[s] + token * y_stride
  BMat seg[4];
  float* y[4] = {nullptr, nullptr, nullptr, nullptr};
  int nseg = 0;
  int seg_rb[5] = {0, 0, 0, 0, 0};  // cumulative 64-row blocks
  int64_t y_stride = 0;
  int ntok = 0;
  // expert launches: items {expert, first row, first slot, tokens} from
  // k_broute; expert == experts selects the shared expert
  int expert_mode = 0;
  BMat eg, eu;  // routed: gate and up (SWIGLU) or down (STORE)
  BMat sg, su;  // shared expert: the same roles
  int experts = 0;
  const int4* items = nullptr;
  const int* nitems = nullptr;
  int max_items = 0;
  const int* in_map = nullptr;  // input row of slot s (null: s)
  float* out = nullptr;         // expert outputs, slot-major
  int64_t out_stride = 0;
  // digitised inputs (k_digitize)
  const uint2* xbt = nullptr;
  const float2* xmeta = nullptr;
  int64_t bt_row = 0, meta_row = 0;
};

// Grouped GEMM on the tcgen05 tensor cores (tgemm.cu): the operations of
// BGemmArgs with 128-row items (dense: 128 rows of a segment; expert gate/up:
// 64 intermediate rows of gate and of up; expert down: 128 hidden rows) and
// tiles of up to 16 tokens, reading the activations as a digit matrix from
// launch_tdigit (three rows of base-254 digits per token or slot).
struct TGemmArgs {
  int mode = BM_STORE;
  int in = 0, gs = 64;
  int scale_f32 = 0;            // scales/biases f32 (else bf16)
  // dense launches: up to four segments over one input
  BMat seg[4];
  float* y[4] = {nullptr, nullptr, nullptr, nullptr};
  int nseg = 0;
  int seg_rb[5] = {0, 0, 0, 0, 0};  // cumulative 128-row blocks
  int64_t y_stride = 0;
  int ntok = 0;
  // expert launches: items {expert, first row, first slot, slots} from
  // k_broute's tensor-core lists (expert == experts: the shared expert)
  int expert_mode = 0;
  BMat eg, eu, sg, su;
  int experts = 0;
  const int4* items = nullptr;
  const int* nitems = nullptr;
  int max_items = 0;
  float* out = nullptr;         // expert outputs, slot-major
  int64_t out_stride = 0;
  // digitised inputs (launch_tdigit)
  const int8_t* dg = nullptr;   // [dg_rows][in]
  int64_t dg_rows = 0;
  const float2* meta = nullptr; // [rows][meta_row] (1 / digit scale, sum) per group
  int64_t meta_row = 0;
  int* status = nullptr;        // bit 0: a bounded wait inside the kernel gave up
};
// Whether the tensor-core GEMM takes matrices of this format; false also
// when SWL_NO_TCGEN05 is set.
bool tgemm_supported(int in, int bits, int dt, int gs);
// Launches it (grid = persistent CTAs); false, with nothing launched, when
// the shapes or tensor maps do not fit it.
bool launch_tgemm(const TGemmArgs& a, int bits, int grid, cudaStream_t stream, bool pdl);
// Digits of `rows` rows in the tensor-core layout: row i reads source row
// in_map[i] (or i) of a.x, applies a.prologue, and writes dg[(3i + d) * in + k]
// and a.meta[i * a.meta_row + g]; a.bt is unused. For 4-bit weights (bits 4)
// the values of each block of 8 are stored in the order 0, 2, 4, 6, 1, 3, 5, 7,
// the order the GEMM's unpack leaves the weight codes in.
void launch_tdigit(const DigitArgs& a, const int* in_map, int8_t* dg, int bits, cudaStream_t stream, bool pdl);

// Routing and grouping of a batch: per token the softmax top-k of the router
// logits (QwenCPUModel.swift:506-521), then picks sorted by expert into
// slots (expert-major, tokens ascending within an expert; the shared expert
// takes slots T*K + t) and the gate/up and down work items.
struct BRouteArgs {
  const float* logits = nullptr;  // [T][E + 1] (router logits, shared-gate logit)
  int T = 0, E = 0, K = 0, norm_topk = 0;
  int* ids = nullptr;             // [T][K]
  float* w = nullptr;             // [T][K] combine weights
  float* sh = nullptr;            // [T] sigmoid of the shared-gate logit
  int* slot_of = nullptr;         // [T][K]
  int* slot_tok = nullptr;        // [T * (K + 1)]
  int4* items_gu = nullptr;       // gate/up items (32 intermediate rows each)
  int4* items_dn = nullptr;       // down items (64 hidden rows each)
  int* nitems = nullptr;          // [2] gate/up, down
  int inter = 0, shared_inter = 0, hidden = 0;
  int max_gu = 0, max_dn = 0;
  // Expert parallelism: only experts [e_lo, e_hi) get slots and items (the
  // other picks get slot -1), and only tokens [sh_lo, sh_hi) get shared-expert
  // items. The defaults cover every expert and token.
  int e_lo = 0, e_hi = 1 << 30, sh_lo = 0, sh_hi = 1 << 30;
  // Optional item lists of the tensor-core GEMM: gate/up items of 64
  // intermediate rows, down items of 128 hidden rows; counts in ntitems[2].
  // Slots past the routed ones get slot_tok 0 so digit rows can be made for
  // every slot index.
  int4* items_tgu = nullptr;
  int4* items_tdn = nullptr;
  int* ntitems = nullptr;
  int max_tgu = 0, max_tdn = 0;
};

// Expert-parallel combine: part[t] = sum of the weighted outputs of this
// rank's picks of token t, plus, for the rank's own tokens [own_lo, own_hi),
// the gated shared expert and the residual h[t - own_lo]. A reduce-scatter of
// part over the ranks then yields each rank's new residual stream.
struct BCombineEpArgs {
  const float* h = nullptr;       // [own_hi - own_lo][D]
  float* part = nullptr;          // [T][D]
  const float* ydown = nullptr;   // [slots][ystride]
  int64_t ystride = 0;
  const int* slot_of = nullptr;   // [T][K], -1 for another rank's expert
  const float* w = nullptr;
  const float* sh = nullptr;
  int T = 0, K = 0, D = 0, own_lo = 0, own_hi = 0;
};

struct BCombineArgs {
  float* h = nullptr;             // [T][D] residual stream
  const float* ydown = nullptr;   // [slots][ystride]
  int64_t ystride = 0;
  const int* slot_of = nullptr;
  const float* w = nullptr;
  const float* sh = nullptr;
  int T = 0, K = 0, D = 0;
};

// On-device sampling (SwiftletSession.sample, SwiftletSession.swift:226-273),
// one row of logits per sequence.
constexpr int SMP_KMAX = 1024;  // largest top_k (when below the vocabulary)
struct SampleArgs {
  const float* logits = nullptr;  // [nseq][row_stride]
  int64_t row_stride = 0;
  int nseq = 0, vocab = 0;
  float temperature = 0.f, top_p = 1.f, presence = 0.f, frequency = 0.f;
  int top_k = 1;
  const int* suppress = nullptr;  // ids set to -inf in every row
  int n_suppress = 0;
  const int* eos = nullptr;       // ids set to -inf in rows that ban EOS
  int n_eos = 0;
  const int* ban_eos = nullptr;   // [nseq] nonzero: ban EOS; null: every row
  int* counts = nullptr;          // [nseq][vocab] times each token was generated (may be null)
  int update_counts = 0;          // add the sampled token to counts
  const float* uniform = nullptr; // [nseq] uniform [0, 1) draws
  int* out = nullptr;             // [nseq] sampled ids
};
void launch_sample(const SampleArgs& a, cudaStream_t stream);

void launch_digitize(const DigitArgs& a, cudaStream_t stream, bool pdl);
// Fills a.L for the matrices of the launch (all with these bits / scale
// dtype / group size) and returns whether the shapes are supported.
bool bgemm_layout(int in, int bits, int dt, int gs, BGLayout& L);
void launch_bgemm(const BGemmArgs& a, int bits, int dt, int grid, cudaStream_t stream, bool pdl);
int bgemm_grid(int bits, int dt, const BGLayout& L);
void launch_broute(const BRouteArgs& a, cudaStream_t stream, bool pdl);
void launch_bcombine(const BCombineArgs& a, cudaStream_t stream, bool pdl);
void launch_bcombine_ep(const BCombineEpArgs& a, cudaStream_t stream, bool pdl);
// Sequence s of the step has consumed seq_n[s] tokens (1 when seq_n is null).
void launch_badvance(const StateDev* sds, int S, const int* seq_n, cudaStream_t stream, bool pdl);
// Chunked steps: the DeltaNet recurrence over each sequence's tokens in order
// (grid: v-heads x sequences), then the conv rings' last conv_k positions.
void launch_delta_seq(const DeltaArgs& a, int S, cudaStream_t stream, bool pdl);
void launch_conv_ring(const DeltaArgs& a, int S, cudaStream_t stream, bool pdl);
// Chunked steps: every token's key (RMSNorm, RoPE) and value into the cache.
void launch_kv_append(const AttnArgs& a, int T, cudaStream_t stream, bool pdl);
void launch_bargmax(const float* logits, int T, int V, int* out, cudaStream_t stream, bool pdl);
void launch_bembed(const EmbedArgs& a, int hidden, int T, cudaStream_t stream, bool pdl);

// All launches go to `stream`; `pdl` enables programmatic dependent launch.
void launch_gemv(const GemvArgs& a, cudaStream_t stream, bool pdl);
void launch_router(const RouterArgs& a, int experts, cudaStream_t stream, bool pdl);
void launch_moe_gateup(const MoeArgs& a, cudaStream_t stream, bool pdl);
void launch_moe_down(const MoeArgs& a, cudaStream_t stream, bool pdl);
// True when both expert launches for `a` take the integer tensor-core kernels,
// which can compute the routing from the router logits (MoeArgs::logits).
bool moe_routes_from_logits(const MoeArgs& a, int experts);
void launch_delta(const DeltaArgs& a, cudaStream_t stream, bool pdl);
// The same for T sequences of a batched step (grid.z = T).
void launch_delta_batch(const DeltaArgs& a, int T, cudaStream_t stream, bool pdl);
// T > 1: T sequences of a batched step (grid.z = T).
void launch_attn(const AttnArgs& a, cudaStream_t stream, bool pdl, int T = 1);
void launch_embed(const EmbedArgs& a, int hidden, cudaStream_t stream, bool pdl);
// Test helper: a bounded mbarrier wait that nothing completes gives up after
// limit_ns and sets bit 0 of *status (the decode kernels' timeout report).
void launch_wait_probe(int* status, unsigned long long limit_ns, cudaStream_t stream);
// Debug/test helper: dequantise rows [r0, r1) of a module to f32.
void launch_dequant(const QLin& l, int64_t r0, int64_t r1, float* out, cudaStream_t stream);

int sm_count();

}  // namespace swl
