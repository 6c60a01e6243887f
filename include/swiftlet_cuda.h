/*
 * swiftlet_cuda.h — C ABI of the B200 (sm_100a) decode backend for
 * Qwen3-Next / Qwen3.5-MoE hybrid models.
 *
 * This is the drop-in boundary for Swiftlet's GPU backend. Each entry point
 * names the Swiftlet interface it replaces (paths inside the Swiftlet tree).
 * Every function returns 0 (SWL_OK) or a negative SWL_ERR_* status; the
 * message of the last failure on the calling thread is swl_last_error().
 *
 * Threading: calls on one model are serialised by the caller, as with
 * QwenMetalModel (SwiftletSession.swift:139-169 serialises under genLock).
 * Device state is keyed per swl_state, so several sequences can be
 * interleaved on one model.
 */
#ifndef SWIFTLET_CUDA_H
#define SWIFTLET_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct swl_model swl_model;
typedef struct swl_state swl_state;

enum {
  SWL_OK = 0,
  SWL_ERR_INVALID = -1,     /* bad argument (null handle, token out of range, ...) */
  SWL_ERR_IO = -2,          /* missing or unreadable file */
  SWL_ERR_FORMAT = -3,      /* malformed config / safetensors / .qpack */
  SWL_ERR_CUDA = -4,        /* CUDA runtime failure */
  SWL_ERR_OOM = -5,         /* device allocation failed */
  SWL_ERR_UNSUPPORTED = -6, /* valid but unsupported format (e.g. 2-bit) */
  SWL_ERR_CAPACITY = -7     /* context or pool capacity exceeded */
};

/* Model configuration: the fields of QwenConfig (QwenConfig.swift:10-50). */
typedef struct swl_config {
  int32_t hidden_size, num_hidden_layers, num_attention_heads, num_key_value_heads, head_dim;
  int32_t vocab_size, full_attention_interval;
  int32_t linear_num_value_heads, linear_num_key_heads, linear_key_head_dim, linear_value_head_dim;
  int32_t linear_conv_kernel_dim;
  int32_t num_experts, num_experts_per_tok, moe_intermediate_size, shared_expert_intermediate_size;
  int32_t norm_topk_prob, tie_word_embeddings;
  int32_t split_delta_layout; /* 1: qwen3_5 in_proj_qkv/z/b/a; 0: qwen3_next in_proj_qkvz/ba */
  int32_t rotary_dims;
  double rope_theta, partial_rotary_factor, rms_norm_eps;
} swl_config;

/* Expert pool statistics (ExpertCache.swift:11,21-22,40-41). The pool is
 * HBM-resident: every expert of every layer is uploaded once at open
 * (counted as misses); each routed expert use during decode is a hit. */
typedef struct swl_pool_info {
  int64_t expert_stride;   /* bytes per expert blob (ExpertCache.stride) */
  int64_t slot_count;      /* ExpertCache.slotCount */
  int64_t allocated_slots; /* ExpertCache.allocatedSlots */
  int64_t hits, misses;    /* ExpertCache.hits / .misses */
  int64_t resident_bytes;  /* HBM held by the pool */
} swl_pool_info;

/* Message of the last failed call on this thread ("" if none). */
const char* swl_last_error(void);

/* Replaces QwenMetalModel.init(modelDir:cacheBudgetGB:) (QwenMetalModel.swift:104).
 * `dir` is an mlx-lm checkpoint directory, a .qpack container
 * (Qpack.swift:3-16) or a synthetic checkpoint (config.json with a
 * "synthetic" block). pool_gb caps the HBM expert pool; <= 0 means no cap.
 * A pool that does not fit the cap fails with SWL_ERR_CAPACITY. */
int swl_model_open(const char* dir, double pool_gb, int device, swl_model** out);

/* Releases every device buffer of the model. States must be freed first. */
int swl_model_close(swl_model* model);

/* InferenceModel.config (TextGenerator.swift:5). */
int swl_model_config(const swl_model* model, swl_config* out);

/* Replaces QwenCPUModel.DecodeState() (QwenCPUModel.swift:183-193): a fresh
 * sequence at position 0 with room for max_ctx tokens of KV cache. */
int swl_state_new(swl_model* model, int32_t max_ctx, swl_state** out);
int swl_state_free(swl_state* state);
/* DecodeState.position (QwenCPUModel.swift:185). */
int32_t swl_state_position(const swl_state* state);

/* Conversation-state reuse (SwiftletSession.swift:114-132 keeps one
 * DecodeState across turns; :193-213 decides when a follow-up extends it).
 * swl_state_reset replaces SwiftletSession.resetConversation (a fresh
 * DecodeState): position 0, zeroed recurrent state. swl_state_copy forks a
 * sequence: dst (same model, max_ctx >= src position) gets src's position,
 * conv rings, delta states and KV rows. swl_state_save writes a host snapshot
 * of the whole decode state (NULL out: *written = bytes needed;
 * SWL_ERR_CAPACITY if out_bytes is short); swl_state_load restores one into
 * any state of a model with the same shape (SWL_ERR_FORMAT otherwise;
 * SWL_ERR_CAPACITY when the state's max_ctx is below the snapshot's
 * position). Decoding from a restored or copied state gives the same logits
 * as continuing the original. */
int swl_state_reset(swl_state* state);
int swl_state_copy(swl_state* dst, const swl_state* src);
int swl_state_save(const swl_state* state, void* out, int64_t out_bytes, int64_t* written);
int swl_state_load(swl_state* state, const void* in, int64_t in_bytes);

/* Replaces InferenceModel.step(_:state:) (TextGenerator.swift:7;
 * QwenMetalModel.swift:359-366): consumes n >= 1 tokens, advances the
 * state's position by n and writes the LAST position's logits (vocab_size
 * floats, host memory) to logits_out. */
int swl_step(swl_model* model, swl_state* state, const int32_t* tokens, int32_t n, float* logits_out);

/* Batched form: sequence i consumes counts[i] tokens (concatenated in
 * `tokens`); logits_out receives nseq rows of vocab_size floats (each
 * sequence's last position). Replaces the per-session loop a caller runs
 * over InferenceModel.step (TextGenerator.swift:84-94) for several sessions.
 * With two or more sequences and a model whose formats the batched kernels
 * take (swl_batch_supported), the sequences advance together: round r runs
 * the r-th token of every sequence that has one, up to 64 sequences per
 * launch. A state may appear only once per call. */
int swl_step_batch(swl_model* model, swl_state** states, const int32_t* tokens, const int32_t* counts, int32_t nseq,
                   float* logits_out);

/* One decode token for each of nseq sequences with device-resident inputs
 * and outputs: d_tokens [nseq]; d_logits (may be NULL) [nseq][vocab_size];
 * d_greedy (may be NULL, may equal d_tokens) [nseq] the first argmax of each
 * row (TextGenerator.swift:90). Work is queued on the model's stream. */
int swl_step_batch_device(swl_model* model, swl_state** states, int32_t nseq, const int32_t* d_tokens, float* d_logits,
                          int32_t* d_greedy);

/* 1 when swl_step_batch runs this model's sequences through the batched
 * kernels (every linear module MLX-affine 4/8-bit with group 32/64/128,
 * routed and shared experts of one format), 0 when it steps them one by one;
 * `why` (may be NULL) receives the reason for 0. Negative on error. */
int swl_batch_supported(swl_model* model, char* why, int32_t why_len);

/* Expert parallelism for batched decode. The reference runs on one Metal
 * device and has no counterpart; the sharding follows the MoE block it
 * computes (QwenMetalModel.swift:798-873, QwenCPUModel.swift:506-566): the
 * routed experts of every layer are split by id over `world` ranks, one
 * process and GPU per rank, each with its own model opened from the same
 * checkpoint. NCCL (libnccl.so.2) is loaded on first use.
 *
 * swl_ep_unique_id writes a communicator id (SWL_EP_ID_BYTES bytes) that one
 * rank makes and hands to the others out of band. swl_ep_init joins the group
 * (blocks until every rank has joined): from then on, a decode launch of
 * swl_step_batch / swl_step_batch_device with one token for each of exactly
 * tokens_per_rank sequences routes all ranks' tokens together. Per MoE layer
 * the ranks all-gather the tokens' quantised inputs and router logits, rank r
 * computes experts [r * E / world, (r + 1) * E / world) for every token and
 * the shared expert for its own tokens, and a reduce-scatter returns each
 * token's sum to its rank. 2 <= tokens_per_rank, tokens_per_rank * world <= 64.
 * Every rank must make the same decode calls in the same order; a decode call
 * with another number of sequences returns SWL_ERR_INVALID before any launch.
 * Prompt calls (a sequence with two or more tokens) and swl_step stay on the
 * rank, which keeps every expert resident. */
#define SWL_EP_ID_BYTES 128
int swl_ep_unique_id(void* out, int32_t out_len);
int swl_ep_init(swl_model* model, int32_t rank, int32_t world, const void* id, int32_t id_len,
                int32_t tokens_per_rank);
/* Failure path of expert parallelism. Every rank's decode step waits in
 * NCCL for the others, so a rank that leaves would leave its peers waiting:
 * the host tells the library instead. Before each expert-parallel decode
 * step the library calls fn(ctx, step) (step = expert-parallel steps this
 * model has made); the callback confirms, out of band (a store, a heartbeat),
 * that every peer is alive and at this step, and returns 0, or nonzero when a
 * peer is gone. A nonzero answer, or an error NCCL reports for the
 * communicator, ends expert parallelism on the model before anything is
 * launched: that call and every later decode call return SWL_ERR_CUDA. NULL
 * removes the callback. */
typedef int (*swl_ep_liveness_fn)(void* ctx, int32_t step);
int swl_ep_set_liveness(swl_model* model, swl_ep_liveness_fn fn, void* ctx);
/* Collective timing of expert parallelism, for finding where a step's time
 * goes (no counterpart in the reference, whose decode runs on one device).
 * Active only when the model's expert parallelism was initialised with the
 * environment variables SWL_EP_TIMING=1 and SWL_EP_NO_GRAPH=1 (steps launched
 * directly, CUDA events around every exchange). Writes out[0] = timed steps,
 * out[1] = their total ms, out[2] = collectives (grouped all-gathers and
 * reduce-scatters), out[3] = their total ms (each including its wait for the
 * slowest peer); synchronises the model's stream; reset != 0 starts the
 * counts again. Returns 1 when timing is active, 0 when not (out all 0). */
int swl_ep_timing(swl_model* model, int32_t reset, double* out);
/* 1 when expert parallelism is on (rank, world and the owned expert range are
 * written; each pointer may be NULL), 0 when off (0, 1, 0, E). */
int swl_ep_info(const swl_model* model, int32_t* rank, int32_t* world, int32_t* expert_lo, int32_t* expert_hi);

/* Same as swl_step with device-resident tokens and logits (either logits
 * pointer may be NULL); `greedy_out` (device, may be NULL) receives the
 * argmax of the last logits (first index on ties, as TextGenerator.swift:90). */
int swl_step_device(swl_model* model, swl_state* state, const int32_t* d_tokens, int32_t n, float* d_logits,
                    int32_t* d_greedy_out);

/* ExpertCache counters (ExpertCache.swift:21-22,40-41). */
int swl_pool_stats(const swl_model* model, swl_pool_info* out);

/* Replaces QwenMetalModel.shrinkCache(toGB:) (QwenMetalModel.swift:324). The
 * HBM pool holds the full expert set; a budget below it returns
 * SWL_ERR_CAPACITY and leaves the pool untouched. */
int swl_pool_resize(swl_model* model, double gb);

/* Container verification (scripts/verify_container.py; manifest fields
 * Qpack.swift:38-46). Every file named in `hashes_json` (NULL:
 * <dir>/hashes.json, {"files": {relative path: sha256 hex}}) is hashed (host
 * threads in parallel) and compared; a file whose size differs from the
 * size manifest.json lists for it counts as corrupt. Returns SWL_OK when all
 * match, SWL_ERR_FORMAT when any file is corrupt or missing (SWL_ERR_IO when
 * the hash list cannot be read). With delete_corrupt != 0 the corrupt files
 * and manifest.json are deleted, as the script does, so the installer reads
 * the container as incomplete and fetches just those files again. `out` (may
 * be NULL) receives the counts either way. No GPU is used. */
typedef struct swl_verify_report {
  int64_t checked, ok, corrupt, missing;
  char first_bad[256]; /* relative path of the first bad file ("" if none) */
} swl_verify_report;
int swl_qpack_verify(const char* dir, const char* hashes_json, int32_t delete_corrupt, swl_verify_report* out);
/* SHA-256 of a file as 64 lowercase hex digits plus a terminator (hex_out
 * holds 65 bytes). */
int swl_sha256_file(const char* path, char* hex_out);

/* Runs all work of `model` on this CUDA stream (cudaStream_t); NULL selects
 * the model's own stream. Graphs are re-captured on the new stream. */
int swl_set_stream(swl_model* model, void* cuda_stream);

/* ---- inspection entry points used by the parity tests ------------------ */

/* Dequantised rows [r0, r1) of a linear module (Checkpoint.moduleWeightSlice,
 * Checkpoint.swift:148-155), as host f32. */
int swl_debug_dequant(swl_model* model, const char* module, int64_t r0, int64_t r1, float* out);
/* Raw device bytes of elements [e0, e1) of a stored tensor (packed words,
 * scales, biases or expert sections; plain tensors are held as f32). */
int swl_debug_tensor_bytes(swl_model* model, const char* name, int64_t e0, int64_t e1, void* out, int64_t out_bytes);
/* One decoder layer for one token at the state's position (the state
 * advances only through swl_step): h_in/h_out are host [hidden_size];
 * pick_ids/pick_w (host, may be NULL) receive the layer's top-k routing. */
int swl_debug_layer(swl_model* model, swl_state* state, int32_t layer, const float* h_in, float* h_out,
                    int32_t* pick_ids, float* pick_w);
/* Delta-rule state of a DeltaNet layer ([nv][dv][dk] f32, host). */
int swl_debug_delta_state(swl_model* model, swl_state* state, int32_t layer, float* out);
/* Kernel family of every launch of one single-token decode step (embedding,
 * layers, lm_head with greedy argmax), comma-separated into out (out_len
 * bytes including the terminator; SWL_ERR_CAPACITY if too small). Families:
 * embed, igemv / sgemv / gemv (dense projections, router, lm_head), router,
 * delta, attn, igateup / sgateup / gateup, idown / sdown / down (the integer
 * tensor-core, slice and register-streaming kernels). Nothing runs. */
int swl_debug_kernel_path(swl_model* model, char* out, int32_t out_len);
/* Runs one bounded mbarrier wait that nothing completes, with a limit of
 * limit_us microseconds (1 .. 1e6), through the same status word the decode
 * kernels report their timeouts in: returns SWL_ERR_CUDA once the wait has
 * given up, the way a decode step reports a weight copy that never arrived,
 * and leaves the model usable. */
int swl_debug_wait_timeout(swl_model* model, int32_t limit_us);

/* Expert-GEMV sweep for the roofline measurement: `iters` passes over all
 * layers of the fused routed+shared expert kernels (gate/up + SiLU, then
 * down + combine), using the routing left by the last step, timed with CUDA
 * events on the model's stream. Outputs the elapsed milliseconds, the
 * algorithmic bytes one layer's pair of launches must read (K routed + 1
 * shared expert: packed words, scales, biases) and the kernel launch count.
 * Needs one prior swl_step; modifies only model scratch. */
int swl_bench_expert_sweep(swl_model* model, int32_t iters, float* ms_out, double* bytes_per_layer,
                           int32_t* launches_out);

/* Batched expert sweep for the expert-GEMM roofline at B = T (2..64): the
 * MoE block of the batched path (router, routing, grouped gate/up and down
 * GEMMs, combine) over every layer for the T tokens the last batched decode
 * step left in the model's scratch, `iters` times, timed with CUDA events.
 * Outputs the elapsed ms, the algorithmic bytes of one sweep (the distinct
 * routed experts each layer's routing picked, counted on the host from one
 * untimed pass, plus the shared expert and router of every layer), that
 * distinct-expert count and the launches. Modifies only model scratch. */
int swl_bench_moe_sweep(swl_model* model, int32_t T, int32_t iters, float* ms_out, double* bytes_out,
                        int32_t* unique_experts_out, int32_t* launches_out);
/* DeltaNet step sweep: the decode recurrence of every DeltaNet layer for one
 * token (T = 1, the state of the last swl_step) or for the T sequences of the
 * last batched decode step, `iters` times, timed with CUDA events; bytes =
 * state read + written, conv taps, projections in, y and z out, per sequence
 * and layer. Benchmark only: it advances those states' recurrences. */
int swl_bench_delta_sweep(swl_model* model, int32_t T, int32_t iters, float* ms_out, double* bytes_out,
                          int32_t* launches_out);

/* Kernel timeline: with SWL_TRACE=<records> set when the model was opened,
 * every CTA of every decode kernel appends {tag, block, start, after the
 * dependency wait, end} (ns, %globaltimer); tag = kind + 16 * (layer + 1)
 * with kind 1 embed, 2 in-projection, 3 DeltaNet/attention, 4 out-projection,
 * 5 router, 6 expert gate/up, 7 expert down, 8 lm_head. Writes the records
 * as CSV to `path` and clears the buffer. */
int swl_trace_dump(swl_model* model, const char* path);

/* On-device sampling: SwiftletSession.sample (SwiftletSession.swift:226-273)
 * for nseq rows of logits (device buffers, row i at d_logits + i * row_stride;
 * not modified). Per row, as the reference: ids in d_suppress, and the ids in
 * d_eos when the row bans EOS (d_ban_eos[i] != 0; d_ban_eos NULL bans them in
 * every row), become -inf; with d_counts ([nseq][vocab], times each token was
 * generated; may be NULL) every token seen n > 0 times loses
 * presence_penalty + frequency_penalty * n; temperature <= 0 takes the first
 * maximum; otherwise the top_k largest (top_k <= 1024 unless >= vocab; ties
 * at the k-th value and in the ordering go to the lower id) are weighted by
 * exp((l - l_max) / temperature), cut at the first cumulative share >= top_p,
 * and d_uniform[i] (a [0, 1) draw per row; the caller's RNG replaces
 * Float.random) picks the token. d_out[i] gets the id; update_counts != 0 adds
 * it to d_counts. Queued on cuda_stream (NULL: the default stream). */
typedef struct swl_sample_options {
  float temperature, top_p, presence_penalty, frequency_penalty;
  int32_t top_k;
} swl_sample_options;
int swl_sample_device(const float* d_logits, int32_t nseq, int32_t vocab, int64_t row_stride,
                      const swl_sample_options* opt, const int32_t* d_suppress, int32_t n_suppress,
                      const int32_t* d_eos, int32_t n_eos, const int32_t* d_ban_eos, int32_t* d_counts,
                      int32_t update_counts, const float* d_uniform, int32_t* d_out, void* cuda_stream);

/* Model-free kernels on host buffers, for kernel-level parity tests:
 * y = W x for one MLX-affine matrix (sdtype 0 f32, 1 bf16, 2 f16) ... */
int swl_kernel_gemv_affine(const uint32_t* packed, const void* scales, const void* biases, int sdtype, int out_dim,
                           int in_dim, int group, int bits, const float* x, float* y);
/* ... and one expert's SwiGLU, y = down(silu(gate x) * (up x))
 * (QwenCPUModel.swift:552-555), through the fused expert kernels; gate/up are
 * [inter, hidden], down [hidden, inter], all with the same bits/group/sdtype. */
int swl_kernel_expert_swiglu(const uint32_t* gate_w, const void* gate_s, const void* gate_b, const uint32_t* up_w,
                             const void* up_s, const void* up_b, const uint32_t* down_w, const void* down_s,
                             const void* down_b, int sdtype, int bits, int group, int hidden, int inter, const float* x,
                             float* y);

/* ... and the gated delta rule over T tokens (the recurrence of
 * QwenCPUModel.swift:459-488 on given inputs, as MetalKernelTests.swift:
 * 194-220 constructs it) through the chunked-parallel prompt kernel:
 * q, k [T][Hk][Dk], v [T][Hv][Dv], g, beta [T][Hv], state [Hv][Dv][Dk]
 * (updated in place), y [T][Hv][Dv]. Needs Dk = 128 and Dv a multiple of 32. */
int swl_kernel_gated_delta(const float* q, const float* k, const float* v, const float* g, const float* beta,
                           float* state, float* y, int32_t T, int32_t Hk, int32_t Hv, int32_t Dk, int32_t Dv);

/* Timing of that chunked prompt kernel on device-resident inputs of T tokens
 * (a fixed input pattern shaped like the prompt path's), `iters` launches
 * timed with CUDA events; flops_out = the chunked algorithm's multiply-add
 * work x 2 over all launches. */
int swl_bench_gated_delta(int32_t T, int32_t Hk, int32_t Hv, int32_t Dk, int32_t Dv, int32_t iters, float* ms_out,
                          double* flops_out);

/* ---- allocation-free entry point (no counterpart in the reference) ----- */

/* A device-resident MLX-affine matrix: uint32 words packed low bits first,
 * [rows][cols * bits / 32] (16-byte aligned rows and pointer), and one scale
 * and one bias per `group` inputs, [rows][cols / group]. */
typedef struct swl_affine_matrix {
  const void* weight;
  const void* scales;
  const void* biases;
  int32_t rows, cols, bits, group;
  int32_t scale_dtype; /* 0 f32, 1 bf16, 2 f16 */
} swl_affine_matrix;

/* One expert's SwiGLU, y = down(silu(gate x) * (up x)), with device-resident
 * x [hidden] (16-byte aligned) and y [hidden], that allocates no device
 * memory: for callers that cannot call cudaMalloc (a host runtime that owns
 * all device memory in its own arena, a plugin that must not grow the
 * process's device footprint). No counterpart in the reference.
 * The intermediate vector lives in one library-wide __device__ array that
 * holds at most 16384 values (moe_intermediate_size); a larger expert fails
 * with SWL_ERR_CAPACITY. Every GPU that loads the library keeps that array
 * (64 KiB) until exit, and every call shares it: calls that overlap on the
 * GPU (different streams without ordering) race on it. Work is queued on
 * `stream` (a cudaStream_t; NULL = legacy default stream) and not waited
 * for. The first call on a device looks up the array's device address
 * (host-side set-up); make that first call before any stream capture.
 * d_status (device int32, may be NULL): the kernels OR bit 0 into it when a
 * bounded wait for their weight copies gave up (about 2 s), in which case y
 * is incomplete; the call never clears it, so the caller zeroes it once and
 * reads it after synchronising. With NULL such a timeout goes unreported. */
int swl_expert_swiglu_noalloc(const swl_affine_matrix* gate, const swl_affine_matrix* up,
                              const swl_affine_matrix* down, const float* x, float* y, int32_t* d_status,
                              void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SWIFTLET_CUDA_H */
