/*
 * qwen_b200.h — C ABI of the B200 ragged hybrid-Qwen decode step.
 *
 * This header replaces the reference's native/mlx_bridge.h for the decode path:
 * the Rust executor (src/serving/native_device.rs:1087-1207,
 * src/serving/native_mtp_device.rs:332-393) binds these symbols unchanged.
 * Every declaration cites the reference declaration it replaces.
 *
 * Conventions (all inherited from the reference, native/mlx_bridge.cpp:19-31):
 *  - functions returning int return 0 on success and -1 on error; on error a
 *    NUL-terminated message is written into error[capacity];
 *  - constructors return NULL on error with the same message convention;
 *  - no C++ exception ever crosses this boundary;
 *  - every handle is worker-confined: one host thread uses a handle at a time
 *    (native/mlx_bridge.h:7); the library keeps no internal locks;
 *  - callers own every host buffer; inputs are copied before the call returns.
 *
 * The library has no CPU path: a session can only be created on a CUDA device
 * of compute capability 10.0 (B200). A missing or different device is an error.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* Model geometry and execution knobs; field order and size are the
 * reference's rs_qwen_config (native/mlx_bridge.h:50-53, 132 bytes), mirrored
 * in Rust by #[repr(C)] Architecture (src/serving/native_qwen.rs:62-98).
 * Knobs that steer MLX graph construction (layer_group, fused_recurrent,
 * compiled_decode, fused_attention, expert_kernel) are validated for range and
 * otherwise ignored: this backend always runs its fused CUDA kernels. */
typedef struct {
  int32_t hidden, layers, vocab, q_heads, kv_heads, head_dim, key_heads, value_heads,
      key_dim, value_dim, conv, interval, experts, top, intermediate, shared, group, bits,
      context, chunk, rope_dims, activation_precision, layer_group, fused_recurrent,
      execution_timing, compiled_decode, operator_profile, fused_attention, validation_mode,
      validation_interval, expert_kernel;
  float epsilon, theta;
} rs_qwen_config;

/* Layer program entry (native/mlx_bridge.h:54): mixer 1 = gated attention,
 * 0 = Gated-DeltaNet; mixer == ((index+1) % interval == 0). */
typedef struct { uint32_t index, mixer; } rs_qwen_layer;

/* Generation-checked state version handle (native/mlx_bridge.h:72-75,
 * native/state_table.h:11-13). 40 bytes. */
#ifndef RS_QWEN_STATE_ID_DEFINED
#define RS_QWEN_STATE_ID_DEFINED
typedef struct StateId { uint64_t owner, slot, generation, position, bytes; } StateId;
#endif

/* ---- weight store (native/mlx_bridge.h:30-32, mlx_bridge.cpp:98-119) ---- */

/* Replaces rs_mlx_weights_create (native/mlx_bridge.h:30). Creates an empty
 * device weight store on the calling thread's current CUDA device. */
void* rs_mlx_weights_create(char* error, size_t capacity);
/* Replaces rs_mlx_weights_destroy (native/mlx_bridge.h:31). */
void rs_mlx_weights_destroy(void* store);
/* Replaces rs_mlx_weights_load (native/mlx_bridge.h:32). Reading safetensors
 * shards is not implemented by this backend yet: returns -1 with a message. */
int rs_mlx_weights_load(void* store, const char* file, char* error, size_t capacity);
/* Replaces rs_qwen_quant (native/mlx_bridge.h:55, native/qwen_model.inc:273-276):
 * per-module quantization override. This backend's kernels implement 4-bit
 * affine, group 64; any other (group, bits) is rejected with a message. */
int rs_qwen_quant(void* store, const char* module, int group, int bits, char* error,
                  size_t capacity);
/* Replaces rs_mlx_weight_bytes (native/mlx_bridge.h:64, mlx_bridge.cpp:177-187):
 * copies bytes of a named tensor in the reference's canonical layout
 * (packed uint32 [rows, cols*bits/32] for ".weight", float32 for ".scales",
 * ".biases" and unquantized vectors) starting at byte `offset`.
 * dtype: 0 float32, 2 uint32 (the reference's rs_mlx_input codes). */
int rs_mlx_weight_bytes(void* store, const char* name, const int32_t* shape, size_t rank,
                        int dtype, size_t offset, uint8_t* output, size_t count, char* error,
                        size_t capacity);

/* Replaces rs_qwen_forward (native/mlx_bridge.h:56-57, native/qwen_model.inc:278-377;
 * declared at src/serving/native_qwen.rs:566): one-shot forward of `count`
 * (1..chunk <= 8) tokens at `offset`. old_state (rs_qwen_state_count floats,
 * NULL / 0 iff offset == 0) is the state before the tokens in the reference
 * layout; new_state (same layout and count) receives the state after them and
 * logits (vocab floats) the last token's logits. gpu must be 1 (this backend
 * has no CPU path). projection_checks, projection_outputs and trace are MLX
 * diagnostics this backend does not provide: they must be 0 / NULL. Uses a
 * private device session kept in the store (rebuilt when `config` changes),
 * so calls on one store must come from one thread at a time. K/V rows of
 * old_state are held in the session's bf16 cache. */
int rs_qwen_forward(void* store, int gpu, const rs_qwen_config* config, const rs_qwen_layer* layers,
                    size_t layer_count, const uint32_t* tokens, size_t count, size_t offset,
                    const float* old_state, size_t old_count, float* new_state, size_t new_count,
                    float* logits, size_t logits_count, int projection_checks,
                    const uint32_t* projection_outputs, size_t projection_output_count, float* trace,
                    size_t trace_count, char* error, size_t capacity);

/* ---- MLX graph builder (native/mlx_bridge.h:8-43; declared at
 * src/serving/native_mlx.rs:574-636). The reference's in-process MLX graph
 * executor has no counterpart on this backend: rs_mlx_create returns NULL and
 * the other builders return -1, each with a message; rs_mlx_destroy and
 * rs_mlx_cleanup do nothing. They exist so the Rust crate links unchanged. */
/* Replaces rs_mlx_create (native/mlx_bridge.h:8). */
void* rs_mlx_create(int gpu, char* error, size_t capacity);
/* Replaces rs_mlx_destroy (native/mlx_bridge.h:9). */
void rs_mlx_destroy(void* graph);
/* Replaces rs_mlx_input (native/mlx_bridge.h:10-11). */
int rs_mlx_input(void* graph, int dtype, const void* data, const int32_t* shape, size_t rank, char* error,
                 size_t capacity);
/* Replaces rs_mlx_op (native/mlx_bridge.h:12-13). */
int rs_mlx_op(void* graph, int op, const uint32_t* inputs, size_t count, int group, float epsilon,
              char* error, size_t capacity);
/* Replaces rs_mlx_finish (native/mlx_bridge.h:14-15). */
int rs_mlx_finish(void* graph, uint32_t output, void* data, size_t elements, char* error, size_t capacity);
/* Replaces rs_mlx_kernel (native/mlx_bridge.h:41-43). */
int rs_mlx_kernel(void* graph, int op, const uint32_t* inputs, size_t count, const int32_t* ints, size_t ni,
                  const float* floats, size_t nf, char* error, size_t capacity);
/* Replaces rs_mlx_parameter (native/mlx_bridge.h:33-34). */
int rs_mlx_parameter(void* graph, void* store, const char* name, const int32_t* shape, size_t rank,
                     int dtype, char* error, size_t capacity);
/* Replaces rs_mlx_cleanup (native/mlx_bridge.h:23; native/mlx_bridge.cpp:96
 * clears MLX streams at executor-thread exit). Sessions own their CUDA streams,
 * so there is nothing per-thread to release. */
void rs_mlx_cleanup(void);

/* NEW (no reference counterpart; the reference loads a private checkpoint,
 * src/serving/qwen_tests.rs:17-243 builds a synthetic one): fill `store` with
 * seeded random-init weights of the given architecture, generated on the
 * device: every matrix is N(0, 0.02) quantized to 4-bit affine g64 with bf16
 * scale and bias; RMSNorm gains are 1; conv, A_log and dt_bias are N(0, 0.02).
 * with_mtp != 0 also creates the MTP head ("language_model.mtp.*").
 * The same generator is restated in the test oracle (bit-identical bytes). */
int rs_qwen_weights_synthetic(void* store, const rs_qwen_config* config, uint64_t seed,
                              int with_mtp, char* error, size_t capacity);

/* ---- device session (native/qwen_device.inc) ---- */

/* Replaces rs_qwen_device_create (native/mlx_bridge.h:76, qwen_device.inc:13-32).
 * gpu must be 1 (the reference's "GPU" code); 0 (CPU) is rejected because this
 * backend has no CPU path. slots = maximum live state versions (target +
 * draft); bytes = resident state budget (KV pages + DeltaNet state) charged
 * in StateId.bytes. Unlike the reference, any architecture the kernels
 * support is accepted (hidden, expert and head widths multiples of 64). */
void* rs_qwen_device_create(void* weights, int gpu, const rs_qwen_config* config,
                            const rs_qwen_layer* layers, size_t count, size_t slots,
                            uint64_t bytes, char* error, size_t capacity);
/* Replaces rs_qwen_device_destroy (native/mlx_bridge.h:86). */
void rs_qwen_device_destroy(void* session);

/* Replaces rs_qwen_device_decode_batch (native/mlx_bridge.h:77,
 * qwen_batch.inc:77-125). One token per row; unlike the reference (B <= 3,
 * equal positions) any batch size and any mix of positions is accepted.
 * logits_count = batch * vocab, row-major. */
int rs_qwen_device_decode_batch(void* session, const StateId* parents, const uint32_t* tokens,
                                size_t batch, StateId* outputs, float* logits,
                                size_t logits_count, char* error, size_t capacity);
/* Replaces rs_qwen_device_step (native/mlx_bridge.h:78, qwen_device.inc:33-50):
 * previous is NULL iff position == 0; count <= config.chunk; logits of the
 * last input token (vocab floats). trace must be NULL/0 (diagnostic traces are
 * an MLX-baseline feature not offered by this backend). */
int rs_qwen_device_step(void* session, const StateId* previous, size_t position,
                        const uint32_t* tokens, size_t count, StateId* output, float* logits,
                        size_t logits_count, float* trace, size_t trace_count, char* error,
                        size_t capacity);
/* Replaces rs_qwen_device_step_sampled (native/mlx_bridge.h:79): greedy
 * total-order argmax on the device, only the token returns. */
int rs_qwen_device_step_sampled(void* session, const StateId* previous, size_t position,
                                const uint32_t* tokens, size_t count, StateId* output,
                                uint32_t* token, char* error, size_t capacity);
/* Replaces rs_qwen_device_block (native/mlx_bridge.h:80-81): position-major
 * logits for every input token (count * vocab floats). */
int rs_qwen_device_block(void* session, const StateId* previous, size_t position,
                         const uint32_t* tokens, size_t count, StateId* output, float* logits,
                         size_t logits_count, char* error, size_t capacity);
/* Replace rs_qwen_device_hidden_step / _hidden_block (native/mlx_bridge.h:94-95):
 * as step / block, and the new version also keeps the post-final-norm hidden
 * rows of its input tokens (read with rs_qwen_device_hidden_snapshot, and the
 * MTP head's input). */
int rs_qwen_device_hidden_step(void* session, const StateId* previous, size_t position,
                               const uint32_t* tokens, size_t count, StateId* output,
                               float* logits, size_t logits_count, char* error,
                               size_t capacity);
int rs_qwen_device_hidden_block(void* session, const StateId* previous, size_t position,
                                const uint32_t* tokens, size_t count, StateId* output,
                                float* logits, size_t logits_count, char* error,
                                size_t capacity);
/* Replaces rs_qwen_device_hidden_snapshot (native/mlx_bridge.h:96). */
int rs_qwen_device_hidden_snapshot(void* session, const StateId* id, float* output,
                                   size_t count, char* error, size_t capacity);
/* Replaces rs_qwen_device_release (native/mlx_bridge.h:82, qwen_device.inc:55). */
int rs_qwen_device_release(void* session, const StateId* id, char* error, size_t capacity);
/* Replaces rs_qwen_device_snapshot (native/mlx_bridge.h:83, qwen_device.inc:56-61):
 * exports a version's state as float32 in the reference layout
 * (native/qwen_model.inc:268-271): per layer in order, DeltaNet conv
 * [conv-1, 2*kd+vd] then S [hv, dv, dk]; attention K [kv, context, d] then V,
 * positions >= version position zero. count = rs_qwen_state_count(). */
int rs_qwen_device_snapshot(void* session, const StateId* id, float* output, size_t count,
                            char* error, size_t capacity);
/* Replaces rs_qwen_device_stats (native/mlx_bridge.h:84, qwen_device.inc:62):
 * count must be 17 + 19*3 = 74; same slot meaning (residents, bytes, exports,
 * uploads, steps, device bytes in use, peak, timing calls/completed/graph_ns/
 * wait_ns/export_ns/wall_ns/groups, graphs/graph misses/graph launches, then
 * per-stage calls/host_ns/wait_ns for the 19 operator stages). */
int rs_qwen_device_stats(void* session, uint64_t* output, size_t count, char* error,
                         size_t capacity);
/* Replaces rs_qwen_device_drain (native/mlx_bridge.h:85, qwen_device.inc:65). */
int rs_qwen_device_drain(void* session, uint64_t* invalidated, char* error, size_t capacity);

/* ---- MTP draft head (native/qwen_mtp.inc) ---- */

/* Replaces rs_qwen_device_mtp_attach (native/mlx_bridge.h:103, qwen_mtp.inc:127-131).
 * The MTP weights live in the same store as the target ("language_model.mtp.*");
 * `weights` must be that store or a store with the MTP head. Must precede
 * any admission. */
int rs_qwen_device_mtp_attach(void* session, void* weights, char* error, size_t capacity);
/* Replaces rs_qwen_device_mtp_step (native/mlx_bridge.h:104, qwen_mtp.inc:133-181). */
int rs_qwen_device_mtp_step(void* session, const StateId* previous, const StateId* source,
                            int draft_source, size_t row, const uint32_t* tokens, size_t count,
                            StateId* output, float* logits, size_t logits_count,
                            int diagnostics, char* error, size_t capacity);
/* Replaces rs_qwen_device_mtp_release (native/mlx_bridge.h:105). */
int rs_qwen_device_mtp_release(void* session, const StateId* id, char* error, size_t capacity);
/* Replaces rs_qwen_device_mtp_snapshot (native/mlx_bridge.h:112): draft KV
 * [kv, context, d] K then V, then the hidden rows. count = id.bytes/4 is not
 * used here; count = 2*kv*context*d + rows*hidden. */
int rs_qwen_device_mtp_snapshot(void* session, const StateId* id, float* output, size_t count,
                                char* error, size_t capacity);

/* ---- NEW ragged entry points (additive; no reference counterpart) ---- */

/* Flags for rs_qwen_device_step_ragged. */
#define RS_QWEN_RAGGED_SAMPLED 1u      /* write greedy tokens (one per output row) */
#define RS_QWEN_RAGGED_LOGITS 2u       /* write fp32 logits (vocab per output row) */
#define RS_QWEN_RAGGED_ALL_ROWS 4u     /* output rows = every input token, else last per sequence */
#define RS_QWEN_RAGGED_HIDDEN 8u       /* keep post-norm hidden rows in each new version */
#define RS_QWEN_RAGGED_CONSUME 16u     /* parents are released by the call (in-place DeltaNet
                                          state update, no second state slot) */

/* One step over a ragged batch: sequence s feeds counts[s] tokens starting at
 * positions[s] (parents[s] is a zeroed StateId iff positions[s] == 0; its
 * position must equal positions[s]). Tokens are packed sequence-major in
 * tokens_flat. Prefill chunks and decode tokens mix freely. Packing (prefix
 * sums, per-token sequence/position, paged-KV block tables and DeltaNet slot
 * indices) is built on the device. Outputs: outs[s] for every sequence; per
 * output row (see flags) a sampled token and/or vocab logits.
 * Generalises rs_qwen_device_decode_batch (qwen_batch.inc:77-125) and
 * rs_qwen_device_step (qwen_device.inc:33-54). */
int rs_qwen_device_step_ragged(void* session, size_t n_seq, const StateId* parents,
                               const uint32_t* positions, const uint32_t* counts,
                               const uint32_t* tokens_flat, uint32_t flags, StateId* outs,
                               uint32_t* sampled, size_t sampled_count, float* logits,
                               size_t logits_count, char* error, size_t capacity);

/* rs_qwen_device_step_ragged with constrained greedy selection: the device
 * version of the reference's host-side select(logits, allowed)
 * (src/serving/choices.rs:65-98), which the Rust batch transaction applies to
 * rows that carry an allowed-token set (batch_transaction.rs:193-235). Output
 * row r (rows as in step_ragged) picks among allowed_ids[allowed_offsets[r],
 * allowed_offsets[r+1]) the id with the largest logit on the IEEE total order,
 * the lowest id on ties; a row whose range is empty picks over the whole
 * vocabulary. allowed_offsets has rows + 1 entries, starts at 0 and ends at
 * allowed_count. Every logit of every row must be finite (else -1,
 * "nonfinite device state"); an id >= vocab is rejected ("invalid legal
 * token"). An empty range means "no constraint", so the reference's
 * "empty legal token set" error (a constrained row with no legal id) is
 * raised by the caller before the call. Requires RS_QWEN_RAGGED_SAMPLED;
 * logits may be returned as well. */
int rs_qwen_device_step_ragged_choices(void* session, size_t n_seq, const StateId* parents,
                                       const uint32_t* positions, const uint32_t* counts,
                                       const uint32_t* tokens_flat, uint32_t flags,
                                       const uint32_t* allowed_offsets, const uint32_t* allowed_ids,
                                       size_t allowed_count, StateId* outputs, uint32_t* sampled,
                                       size_t sampled_count, float* logits, size_t logits_count,
                                       char* error, size_t capacity);

/* Speculative verify + accept over a ragged batch, on the device.
 * Sequence s: parents[s] is a published version at position p; seeds[s] is
 * the greedy token after it (already emitted, not yet fed) and
 * drafts[s*width .. +ndraft[s]] (ndraft[s] <= width <= 8) are MTP proposals.
 * The call feeds [seed, drafts...] to the target in one ragged step (greedy
 * row r_j after fed token j), then applies the reference's plan() rule
 * (src/serving/native_speculative.rs:74-128): emit r_0, r_1, ... while
 * draft j == r_j and r_j is not an EOS; the first mismatch or EOS is emitted
 * and ends the plan; after all drafts match, the bonus r_k is emitted if the
 * context has room. accepted[s] = matched drafts (a matched EOS counts),
 * emitted[s*(width+1) ..] / n_emitted[s] = the emitted tokens, and outs[s] =
 * the version after [seed, d_0 .. d_{accepted-1}] (position p + 1 + accepted):
 * its DeltaNet state was written per token during the step and its KV pages
 * are the step's, truncated (compaction on the device; no replay). With
 * RS_QWEN_RAGGED_HIDDEN the version keeps the post-norm hidden rows of the
 * accepted tokens. Parents stay published. */
int rs_qwen_device_mtp_verify_accept(void* session, size_t n_seq, const StateId* parents,
                                     const uint32_t* seeds, const uint32_t* drafts,
                                     const uint32_t* ndraft, size_t width, const uint32_t* eos,
                                     size_t n_eos, uint32_t flags, StateId* outs,
                                     uint32_t* accepted, uint32_t* emitted,
                                     uint32_t* n_emitted, char* error, size_t capacity);

/* NEW: expert parallelism (the survey's multi-GPU mode b; no reference
 * counterpart). Rank 0 calls rs_qwen_ep_unique_id (128 bytes, NCCL unique id)
 * and shares it; every rank then calls rs_qwen_device_ep_init on its own
 * session (one GPU per process) with the same world size, its rank and the
 * same cap_tokens. From then on the target model's MoE layers compute only the
 * rank's block of routed experts [rank*E/world, (rank+1)*E/world) for the
 * rows of every rank, exchanged with NCCL send/recv over NVLink in
 * fixed-size stages of cap_tokens*top rows per peer; the shared expert and
 * everything else stay local, and logits equal the single-GPU ones bit for
 * bit. All ranks must step in lockstep (the same sequence of target steps,
 * each with at most cap_tokens tokens, and T >= 1); the MTP head stays local.
 * E must be a multiple of world. */
int rs_qwen_ep_unique_id(uint8_t* out, size_t out_bytes, char* error, size_t capacity);
int rs_qwen_device_ep_init(void* session, int world, int rank, const uint8_t* id, size_t id_bytes,
                           size_t cap_tokens, char* error, size_t capacity);
/* The same mode over direct NVLink stores instead of NCCL (one process per
 * GPU, all GPUs visible to every process): rs_qwen_device_ep_window allocates
 * this rank's window (the stages other ranks write to it and their epoch
 * flags) and returns its 64-byte CUDA IPC handle; once every rank has one,
 * rs_qwen_device_ep_connect(handles of ranks 0..world-1) maps the peers'
 * windows. The pack and return kernels then store only the valid rows into
 * the owner's window and raise a flag (bounded waits on the reader side);
 * same lockstep rules. Every rank must have finished its steps before any
 * session is destroyed. */
int rs_qwen_device_ep_window(void* session, int world, int rank, size_t cap_tokens, uint8_t* handle,
                             size_t handle_bytes, char* error, size_t capacity);
int rs_qwen_device_ep_connect(void* session, const uint8_t* handles, size_t handles_bytes, char* error,
                              size_t capacity);

/* NEW (no reference counterpart; stands in for a long prefill when measuring
 * decode at long contexts): create a published version at `position` whose
 * KV pages for [0, position) hold seeded bf16 N(0, 1) values, whose DeltaNet
 * state is fp32 N(0, 0.02) and conv history N(0, 1). The contents depend only
 * on (seed, position), not on the slot. */
int rs_qwen_device_synthetic_state(void* session, size_t position, uint64_t seed, StateId* out,
                                   char* error, size_t capacity);

/* NEW diagnostic (no reference counterpart; mirrors the role of the
 * reference's routing probe, native/operator_probe.inc:19-23): when enabled,
 * each step keeps its top-k expert ids; rs_qwen_device_debug_routing copies
 * the last step's ids as int32 [moe layers][tokens][top]. */
int rs_qwen_device_set_capture(void* session, int routing, char* error, size_t capacity);
int rs_qwen_device_debug_routing(void* session, int32_t* out, size_t count, char* error,
                                 size_t capacity);
/* NEW diagnostic: the last step's device intermediates, as raw bytes.
 * what: 0 router logits fp32 [moe layers][T][experts+1] (last column = shared
 * gate), 1 expert offsets int32 [moe layers][experts+2], 2 sorted->flat
 * permutation int32 [moe layers][T*(top+1)], 3 packing int32 blob
 * {n, T, R, n_new, SeqDesc[n] (12 ints), new pages[n_new], cu_seqlens[n+1],
 * token_seq[T], token_pos[T], slot_mapping[T] (low 32 bits), out_token[R]},
 * 4 block-table rows int32 [n][pages] of the step's children (rows padded to
 * the longest). Capture must be enabled before the step (routing != 0).
 * count is the byte capacity of out; returns the byte count written in
 * *written. */
int rs_qwen_device_debug_capture(void* session, int what, void* out, size_t count, size_t* written,
                                 char* error, size_t capacity);

/* NEW diagnostic: device-side timing from CUDA events on the session stream.
 * profile != 0 additionally brackets every operator stage with events
 * (the 19 stages of native/operator_timing.h:5-9). rs_qwen_device_timing
 * writes count = 3 + 19 doubles: last step device ms, cumulative device ms,
 * timed steps, then cumulative device ms per stage (zeros unless profiling). */
int rs_qwen_device_set_profile(void* session, int profile, char* error, size_t capacity);
int rs_qwen_device_timing(void* session, double* out, size_t count, char* error, size_t capacity);

/* NEW diagnostic: run one dense 4-bit GEMM of the model on caller inputs.
 * which: 0 = layer `layer` mixer input projection, 1 = its output projection,
 * 2 = its MoE router (+ shared gate), 3 = lm_head. x: T rows of IEEE half
 * bits, the projection input type (row width = the matrix's input width). y: T x rows fp32 (split-K partials
 * summed). engine: 0 = tcgen05 kernel, 1 = CUDA-core reference kernel.
 * ms: device time of the GEMM launch(es). Returns 0/-1. */
int rs_qwen_debug_gemm(void* session, int which, int layer, const uint16_t* x, size_t T, float* y,
                       size_t y_count, int engine, double* ms, char* error, size_t capacity);

/* Allocation-free dense projection. No counterpart in the reference: it exists
 * for callers that must not allocate device memory while they run, e.g. a
 * server that has handed the device to the session's KV page pool and
 * DeltaNet state slots (the pool takes what the byte budget leaves, so a
 * later cudaMalloc can fail), or a latency-critical loop where cudaMalloc /
 * cudaFree would synchronise the device. It allocates nothing, on the device
 * or the host, when it succeeds.
 *
 * y_device (fp32, T x rows, device) = x_device (IEEE half, T x k, device,
 * 16-byte aligned) times the selected matrix; `which` and `layer` select it
 * as in rs_qwen_debug_gemm (tcgen05 engine). The split-K partials live in a
 * fixed 16 MiB static device array per device, so T x rows may not exceed
 * 4,194,240 floats; larger calls return -1 with an error naming the limit.
 * Work is enqueued on `stream` (NULL: the session's stream); the call then
 * synchronises that stream and returns once the result is in y_device. It
 * runs on the session's device and leaves the calling thread's current device
 * as it found it. The first call on each device resolves the scratch address
 * (a one-time set-up); make that call before any stream capture begins.
 * Every call on a device shares the one array: calls that overlap in time
 * (several host threads, or several sessions on one device) race and corrupt
 * each other's results, so serialise them. Returns 0/-1. */
int rs_qwen_project_noalloc(void* session, int which, int layer, const void* x_device, size_t T,
                            float* y_device, size_t y_count, void* stream, char* error, size_t capacity);

/* Number of floats of a version's reference-layout snapshot
 * (native/qwen_model.inc:268-271 qwen_state_count). */
size_t rs_qwen_state_count(const rs_qwen_config* config);

/* Version string of this backend (replaces rs_mlx_version, native/mlx_bridge.h:16). */
const char* rs_mlx_version(void);

#ifdef __cplusplus
}
#endif
