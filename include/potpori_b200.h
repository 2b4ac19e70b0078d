/*
 * potpori_b200 — C ABI of the B200 (sm_100a) per-shard Qwen3 verify pass.
 *
 * One handle is one shard: a contiguous layer range [layer_begin, layer_end) of a Qwen3
 * model with its own F32 KV cache, on one CUDA device. It replaces the reference's
 * `Shard<R: QwenRuntime>` (src/qwen/shard.rs:17-133) and the CUDA `QwenRuntime` adapter
 * behind it (src/qwen/runtime/mod.rs:24-43, src/qwen/runtime/cuda.rs:54-190), and offers
 * the `ShardEngine` surface (src/node.rs:55-86) as plain functions over plain pointers.
 *
 * Threading: a handle is used from one host thread at a time (the reference's runtime is
 * not Sync either). Handles on different devices may run concurrently.
 * Memory: all device memory is owned by the handle; host buffers are owned by the caller.
 * Errors: every call returns a pp_status; pp_last_error() gives the message of the last
 * failure on a handle (or of pp_shard_create when the handle is NULL).
 */
#ifndef POTPORI_B200_H
#define POTPORI_B200_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

typedef enum pp_status {
  PP_OK = 0,
  PP_E_INVALID = 1,     /* rejected before launch: src/qwen/model.rs:373-395 rules */
  PP_E_NONFINITE = 2,   /* non-finite logits at the tail (src/node.rs:266-272) */
  PP_E_CUDA = 3,        /* a CUDA runtime/driver call failed */
  PP_E_TIMEOUT = 4,     /* a bounded device wait expired */
  PP_E_OOM = 5,         /* device allocation failed */
  PP_E_UNSUPPORTED = 6, /* a geometry this build does not run */
  PP_E_MISSING = 7      /* a parameter of the shard was never loaded */
} pp_status;

typedef enum pp_dtype { PP_F32 = 0, PP_BF16 = 1 } pp_dtype;

/* Model geometry: src/qwen/model.rs:11-21 (QwenConfig), field for field. */
typedef struct pp_config {
  uint32_t layers, hidden, intermediate, head_dim, n_heads, n_kv_heads, vocab_size;
  float rms_norm_eps, rope_theta;
} pp_config;

/* Shard description: the arguments of QwenGraph::build (src/qwen/model.rs:198-205) and
 * Shard::load_chunked (src/qwen/shard.rs:28-38). first/last are implied by the range. */
typedef struct pp_shard_desc {
  pp_config cfg;
  uint32_t layer_begin, layer_end;
  uint32_t capacity; /* KV positions (max_seq) */
  uint32_t chunk;    /* verify chunk (gamma + 1), at most 16; 0 = any size up to 16. Chunks
                        of 9..16 rows need n_heads / n_kv_heads <= 4. */
  int32_t cuda_device;
} pp_shard_desc;

/* What the tail returns for one chunk (src/node.rs:265-278, src/engine.rs:14-29,
 * src/specdecode.rs:92-98). Arrays have one entry per chunk row. */
typedef struct pp_verify_out {
  int32_t* argmax;  /* [m], or NULL; -1 for a row with a non-finite logit */
  float* top1;      /* [m], or NULL: largest logit */
  float* top2;      /* [m], or NULL: second largest logit (a tie counts twice) */
  float* logits;    /* [m][vocab] row form, or NULL (not computed when NULL) */
  int32_t n_accepted; /* longest prefix with drafts[i] == argmax[i] */
  int32_t correction; /* argmax[n_accepted] */
  int32_t nonfinite_rows; /* bit r set when row r had a non-finite logit */
} pp_verify_out;

typedef struct pp_shard pp_shard;

/* QwenGraph::build + QwenRuntime::compile (src/qwen/model.rs:198-337,
 * src/qwen/runtime/cuda.rs:64-147): validates the range (model.rs:206-217), allocates the
 * device arena (weights, KV cache, RoPE table, activations) and zeroes the KV cache. */
pp_status pp_shard_create(const pp_shard_desc* desc, pp_shard** out);
void pp_shard_destroy(pp_shard* shard);

/* One parameter by checkpoint name and shape (src/qwen/hf.rs:227-272 load_inputs): matrices
 * as BF16 bits or F32 (rounded to BF16), names containing "norm" as F32 or BF16 (widened).
 * Names of other shards' parameters are accepted and ignored. */
pp_status pp_shard_set_tensor(pp_shard* shard, const char* name, pp_dtype dtype,
                              const void* host_data, uint64_t elements);
/* Every parameter of the shard from a prepared safetensors file
 * (model_combined_bf16_v1.safetensors layout, src/qwen/hf.rs:20,85-91,227-272). */
pp_status pp_shard_load_safetensors(pp_shard* shard, const char* path);
/* Every parameter from the seeded generator: matrices N(0, std) rounded to BF16 (Irwin-Hall
 * of twelve 16-bit uniforms, counter-based by tensor name), norms 1. */
pp_status pp_shard_init_random(pp_shard* shard, uint64_t seed, float std);
/* Number of parameters not yet loaded; names ';'-separated into buf when given. */
int32_t pp_shard_missing(const pp_shard* shard, char* buf, size_t len);

/* ShardEngine::forward_tokens (src/node.rs:70, src/qwen/shard.rs:124-126): first shard.
 * m tokens at absolute positions pos..pos+m-1. out_hidden: [m][hidden] for a non-last shard
 * (may be NULL). verify: results on the last shard (may be NULL); drafts for the accept
 * compare are tokens[1..m-1]. */
pp_status pp_shard_forward_tokens(pp_shard* shard, uint32_t pos, const int32_t* tokens,
                                  uint32_t m, float* out_hidden, pp_verify_out* verify);
/* Greedy decode of n single tokens on a whole-model shard (first and last), the draft's
 * gamma loop of src/qwen/draft.rs:14-93: step i feeds token t_i at position pos + i, with
 * t_0 = token and t_{i+1} = the greedy pick of step i; out[i] = pick i (n <= 64). The picks
 * are fed to the next step on the device, so the host waits once for the n steps instead of
 * once per token. PP_E_NONFINITE when a step produced non-finite logits (the picks after it
 * are then undefined). */
pp_status pp_shard_decode_greedy(pp_shard* shard, uint32_t pos, int32_t token, uint32_t n,
                                 int32_t* out);
/* ShardEngine::forward_hidden (src/node.rs:73, src/qwen/shard.rs:127-129): non-first shard.
 * hidden: [m][hidden] F32 (finite, src/qwen/model.rs:390-392). drafts: [n_drafts] tokens
 * for the tail's accept compare (may be NULL). */
pp_status pp_shard_forward_hidden(pp_shard* shard, uint32_t pos, uint32_t m, const float* hidden,
                                  const int32_t* drafts, uint32_t n_drafts, float* out_hidden,
                                  pp_verify_out* verify);

/* Device-resident step for in-box pipeline stages (replaces the QUIC hop of
 * src/node.rs:466-496 with device buffers). The step reads its input from the shard's own
 * input buffer (pp_shard_buffers) and its step header from the device header buffer, both
 * of which a peer copy may fill (pp_shard_handoff, pp_shard_recv); no host synchronisation. stream: a
 * cudaStream_t (NULL = the shard's stream). max_rows selects the compiled chunk width
 * (1, 2, 4, 8 or 16 rows). */
pp_status pp_shard_step_device(pp_shard* shard, uint32_t max_rows, void* stream);
/* Host-side enqueue of the step header (pos, m, tokens, drafts) for pp_shard_step_device.
 * flags: bit 0 = also write the full logits (last shard); the other bits travel with the
 * header unchanged (pipeline stages use them to mark a timed window). */
pp_status pp_shard_set_step(pp_shard* shard, uint32_t pos, uint32_t m, const int32_t* tokens,
                            const int32_t* drafts, uint32_t n_drafts, int32_t flags,
                            void* stream);
/* Device pointers of the shard's resident buffers: hidden [max_rows][hidden] F32 (input of
 * a non-first shard, output of a non-last one), the step header (pp_step_header layout, 144
 * bytes) and the step result (pp_step_result layout). */
pp_status pp_shard_buffers(pp_shard* shard, void** hidden, void** header, void** result);
/* Read the device step result after a device step (synchronises the stream). */
pp_status pp_shard_read_result(pp_shard* shard, uint32_t m, pp_verify_out* verify, void* stream);

/* In-box stage handoff (replaces the hidden-state frame of src/node.rs:476-489 and
 * src/transport.rs:425-489): enqueue on `to`'s stream a copy of `from`'s output rows
 * [m][hidden] into `to`'s input buffer, ordered after the work already enqueued on `from`
 * (a peer copy over NVLink when the devices differ). No host synchronisation. */
pp_status pp_shard_handoff(pp_shard* from, pp_shard* to, uint32_t m);
/* Enqueue the device-to-host copy of the step result into result slot `slot` (0..63). */
pp_status pp_shard_result_enqueue(pp_shard* shard, uint32_t slot);
/* Wait for result slot `slot` and fill `verify` (m rows); the status of that step. */
pp_status pp_shard_result_wait(pp_shard* shard, uint32_t slot, uint32_t m, pp_verify_out* verify);

/* Cross-process stage link inside one box: the hop between the nodes of a chain
 * (ChainLink::send_chunk and serve_middle/serve_tail, src/node.rs:242-342,466-535; the frames
 * of src/transport.rs:425-489) when consecutive stages run in different processes, one per
 * GPU. The receiving stage exports an inbox of `slots` chunk slots (step header + hidden rows)
 * in its device memory as a 64-byte CUDA IPC handle; the sending stage opens it and, after
 * its step, copies the chunk's header and hidden rows into slot seq % slots on the copy
 * engines (NVLink), then writes the slot's two mailbox words (mail[1] = info, then
 * mail[0] = seq + 1) with stream-ordered writes into host memory that both processes share
 * (registered with pp_host_register). No SM takes part in a transfer. The receiving process
 * waits for mail[0] on the host, then pp_shard_recv copies the slot into the shard's input
 * and header buffers, ordered before its next step. m = 0 sends only the mailbox words (the
 * end of a session). */
pp_status pp_shard_inbox_export(pp_shard* shard, uint32_t slots, void* handle);
pp_status pp_shard_outbox_open(pp_shard* shard, const void* handle, uint32_t slots);
pp_status pp_shard_send(pp_shard* shard, uint32_t seq, uint32_t m, uint32_t* mail, uint32_t info);
pp_status pp_shard_recv(pp_shard* shard, uint32_t seq, uint32_t m);
/* Last stage: copy the step result into host memory (registered, shared with the head's
 * process: the direct return of the result to the head) and then write `value` into *mail. */
pp_status pp_shard_send_result(pp_shard* shard, void* host_result, uint32_t* mail, uint32_t value);
/* Page-lock and map host memory for the device (a shared-memory segment of the chain). */
pp_status pp_host_register(void* ptr, size_t bytes);
pp_status pp_host_unregister(void* ptr);

/* ShardEngine::reset (src/qwen/runtime/cuda.rs:181-189): KV cache back to zeros. */
pp_status pp_shard_reset(pp_shard* shard);
/* Seeded N(0,1) KV rows [0, rows) in every layer (benchmark warm context; the oracle's
 * or_shard_fill_kv writes the same values). */
pp_status pp_shard_fill_kv(pp_shard* shard, uint64_t seed, uint32_t rows);

/* ShardEngine getters (src/node.rs:57-67, src/qwen/shard.rs:106-123). */
uint32_t pp_shard_capacity(const pp_shard* shard);
uint32_t pp_shard_chunk_size(const pp_shard* shard);
void pp_shard_range(const pp_shard* shard, uint32_t* begin, uint32_t* end);
uint32_t pp_shard_hidden_dim(const pp_shard* shard);
uint32_t pp_shard_vocab_size(const pp_shard* shard);
uint32_t pp_shard_model_layers(const pp_shard* shard);
/* Bytes of device memory the handle holds. */
uint64_t pp_shard_device_bytes(const pp_shard* shard);

/* Kernel kinds reported by pp_shard_profile_kernels. */
typedef enum pp_kernel_kind {
  PP_K_BEGIN = 0,        /* step header check */
  PP_K_EMBED = 1,        /* embedding gather (first shard) */
  PP_K_QKV = 2,          /* input norm + QKV + QK-norm + RoPE + KV write */
  PP_K_ATTN = 3,         /* split-KV attention */
  PP_K_ATTN_COMBINE = 4, /* merge of the splits */
  PP_K_O = 5,            /* O projection + residual */
  PP_K_GATE_UP = 6,      /* post-attention norm + gate/up + SwiGLU */
  PP_K_DOWN = 7,         /* down projection + residual */
  PP_K_HEAD = 8,         /* final norm + vocab projection + argmax/top-2/accept */
  PP_K_DECODE = 9        /* every layer of a 1-row step in one persistent kernel */
} pp_kernel_kind;

/* Time every kernel of one step: the step is captured into a graph with an event after each
 * kernel (which also serialises them) and replayed `iters` times; ms[k] is the mean duration
 * of the k-th kernel and kinds[k] its pp_kernel_kind. *count = kernels per step. */
pp_status pp_shard_profile_kernels(pp_shard* shard, uint32_t max_rows, uint32_t iters, float* ms,
                                   int32_t* kinds, uint32_t cap, uint32_t* count);
/* The shard's own CUDA stream (a cudaStream_t). */
void* pp_shard_stream(const pp_shard* shard);

/* Kernel launches of the last forward (for the benchmark's launch count). */
uint32_t pp_shard_last_launches(const pp_shard* shard);
/* Enable (1) / disable (0) CUDA-graph replay of the step (default on) and programmatic
 * dependent launch between kernels (default on). */
pp_status pp_shard_set_graphs(pp_shard* shard, int32_t enabled);
pp_status pp_shard_set_pdl(pp_shard* shard, int32_t enabled);
/* Most CTAs (one per SM) any kernel of this shard launches; 0 = every SM, the default. The
 * split-K GEMVs and the split attention assume all their CTAs are resident at once, so SMs
 * held by other work on the device (another model's long-running kernels, or transfer
 * kernels of a communication library) must be left out of the budget, or the CTAs that do
 * not fit run as a second wave.
 * No counterpart in the reference. Must be at least n_kv_heads. Results stay within the
 * parity tolerances: the split partition (the summation order) depends on the budget. */
pp_status pp_shard_set_sm_limit(pp_shard* shard, uint32_t ctas);
uint32_t pp_shard_sm_limit(const pp_shard* shard);

/* Prompt prefill of a first shard: positions pos .. pos + t - 1 (t <= 2048) of the prompt
 * `tokens` go through all its layers at once and their K/V rows are written into the cache,
 * as the reference's prefill does in chunk-sized verify steps (src/qwen/target.rs:62-84,
 * src/node.rs:538-566). The projections run on the tensor cores (pp_rows_gemm), the causal
 * attention flash-style over the whole chunk. It produces no logits: the caller runs the last
 * prompt token as a 1-row step for its greedy pick. A shard that is not the last leaves the t
 * output rows of its last layer in its prefill buffer for the next stage. Allocates its row
 * buffers (about 0.2 GB for Qwen3-0.6B, 0.5 GB for 4B) on first use. PP_E_UNSUPPORTED for a
 * head size other than 128 or other than 1, 2, 4 or 8 query heads per KV head. Synchronous. */
pp_status pp_shard_prefill(pp_shard* shard, uint32_t pos, const int32_t* tokens, uint32_t t);
/* The same pass on a later stage over the t rows in its prefill buffer, which
 * pp_shard_prefill_handoff (same process) or pp_shard_prefill_send (another process) filled,
 * or `hidden` ([t][hidden] F32 host rows, finite) when not NULL. Synchronous. */
pp_status pp_shard_prefill_hidden(pp_shard* shard, uint32_t pos, uint32_t t, const float* hidden);
/* The t output rows a prefill pass left in a shard that is not the last ([t][hidden] F32). */
pp_status pp_shard_prefill_read(pp_shard* shard, uint32_t t, float* out);
/* Copy `from`'s t prefill output rows into the prefill buffer of the next stage `to` (a peer
 * copy when the devices differ). */
pp_status pp_shard_prefill_handoff(pp_shard* from, pp_shard* to, uint32_t t);
/* Across processes: the receiving stage exports its prefill buffer (64-byte CUDA IPC handle),
 * the sending stage opens it and, after its pass, copies its t output rows into it on the
 * copy engines, then writes the mailbox words (mail[1] = info, mail[0] = seq + 1) as
 * pp_shard_send does. */
pp_status pp_shard_prefill_export(pp_shard* shard, void* handle);
pp_status pp_shard_prefill_open(pp_shard* shard, const void* handle);
pp_status pp_shard_prefill_send(pp_shard* shard, uint32_t seq, uint32_t t, uint32_t* mail,
                                uint32_t info);

/* Run every 1-row step of a shard that holds all layers (a draft model's greedy decode, the
 * single-token verify steps) as one persistent cooperative kernel over the shard's SM budget
 * followed by the vocabulary head, instead of six kernels per layer (enabled = 1; 0 returns
 * to the per-layer kernels). The kernel streams a row-major copy of the layer weights (K
 * padded to a multiple of 512, of 1024 above 4096 and of 2048 above 8192), made on first use
 * after every weight upload and held until the shard is destroyed (0.9 GB for Qwen3-0.6B).
 * Same step semantics as the per-layer path (src/qwen/model.rs:366-412 for one token); the
 * F32 summation order differs, within the parity tolerances. PP_E_UNSUPPORTED for a shard
 * without every layer or outside the kernel's sizes (hidden <= 8192, q_dim and intermediate
 * <= 16384, all multiples of 8; head size 128 with 1, 2 or 4 query heads per KV head and at
 * most 8 KV heads). No counterpart in the reference. */
pp_status pp_shard_set_decode_kernel(pp_shard* shard, int32_t enabled);
int32_t pp_shard_decode_kernel(const pp_shard* shard);

/* Prompt-sized projection on the 5th-generation tensor cores (tcgen05 MMA, TMEM accumulator):
 * with device pointers,
 *   y[i][j] = sum_c W[j][c] * x[i][c]    for i < t rows, j < n, c < k,
 * the linear of src/qwen/model.rs:166-183 at prefill sizes (a 2048-token prompt chunk is a
 * dense contraction, not a skinny GEMV). W is BF16 in the tiled layout described at
 * pp_norm_gemv_static (the shards' layout), x is [t][k] and y [t][n] F32. x is split into
 * BF16 hi + lo parts in `work` (caller-owned device memory, 1024-byte aligned, at least
 * pp_rows_gemm_work_bytes(t, k) bytes) and every K step accumulates W.hi + W.lo in F32, the
 * reference's F32 arithmetic to about 2^-17 relative per product. *err (device memory, zero
 * before the call) gets a nonzero bit when a bounded wait on the device expired. Asynchronous
 * on `stream` (a cudaStream_t, NULL = default). */
uint64_t pp_rows_gemm_work_bytes(uint32_t t, uint32_t k);
pp_status pp_rows_gemm(const uint16_t* w_tiled, uint32_t n, uint32_t k, const float* x, uint32_t t,
                       float* y, void* work, uint64_t work_bytes, uint32_t* err, void* stream);

/* Allocation-free RMSNorm + skinny GEMV (no counterpart in the reference; an addition for
 * callers that cannot allocate device memory: code running inside a host framework or memory
 * pool that owns every allocation, or a context where cudaMalloc/cudaFree and their implicit
 * synchronisation are not allowed). With every pointer a device pointer:
 *   y[i][j] = sum_c W[j][c] * (x[i][c] / sqrt(mean_c x[i][c]^2 + eps) * norm_w[c])
 * for i < m <= 8 rows, j < n, c < k (k a multiple of 8). x is [m][k] F32, y is [m][n] F32,
 * norm_w is [k] F32, and W is BF16 in the tiled layout the shards use: element (j, c) at
 *   ((((j/128)*kc + c/64)*128 + j%128) * 64) + ((((c%64)/8) ^ (j%8)) * 8) + c%8
 * with kc = ceil(k/64), the buffer holding ceil(n/128)*kc blocks of 128x64, padding zero.
 * The call allocates nothing: its split-K scratch is a static device array of about 1.2 MB
 * (partial sums for 148 CTAs and counters for n <= 8192*128 rows) that every GPU loading the
 * library holds until exit; it rejects larger sizes with PP_E_INVALID. The first call on a
 * device looks the array up with that device current and should come before any stream
 * capture. Every call shares the array and clears the counters it needs: calls that overlap
 * on the GPU (two streams at once) race on it. *err (device memory, zero before the call, or
 * NULL) gets status bits: 2 when x holds a non-finite value, 4 when a bounded wait on the
 * device expired, in which case y is undefined (the call itself still returned PP_OK, since it
 * only enqueues). stream: a cudaStream_t (NULL = default). */
pp_status pp_norm_gemv_static(const uint16_t* w_tiled, const float* x, const float* norm_w,
                              float eps, uint32_t n, uint32_t k, uint32_t m, float* y,
                              uint32_t* err, void* stream);

/* Test hook of the decode kernel's bounded waits (no counterpart in the reference; the
 * reference bounds its own waits, src/node.rs:47-50): limit_us sets the time limit of its grid
 * and head barriers (0: the default 200 ms); unreachable = 1 makes every grid barrier wait for
 * one CTA more than the grid has, so the step's first barrier can only end by running out of
 * time: the kernel then records the timeout, drains its copies and returns, and the step
 * reports PP_E_TIMEOUT. The shard stays usable; unreachable = 0 restores normal steps. */
pp_status pp_shard_set_wait_test(pp_shard* shard, uint32_t limit_us, int32_t unreachable);

/* Tapped-layer outputs: TappedShards (src/node.rs:108-223) and LayerTap
 * (src/transport.rs:148-179). After every step the output rows [m][hidden] of each layer in
 * `layers` (model layer numbers inside the shard's range and below the model's last layer,
 * which feeds the logits: src/node.rs:118-124) are kept on the device; duplicates are dropped,
 * the order is ascending, n = 0 ends tapping. One shard taps any of its layers, where the
 * reference cuts a node into one shard per tap. 1-row steps of a shard with the decode kernel
 * run on the per-layer kernels while layers are tapped. */
pp_status pp_shard_set_taps(pp_shard* shard, const uint32_t* layers, uint32_t n);
/* The tapped layers (ascending) into layers[0..cap); returns their number. */
uint32_t pp_shard_tap_layers(const pp_shard* shard, uint32_t* layers, uint32_t cap);
/* The last step's tapped outputs for its m rows, [n_taps][m][hidden]: F32 into f32 and/or
 * BF16 bits rounded to nearest even into bf16 (LayerTap::from_f32, the wire form); either may
 * be NULL. Synchronises the shard's stream. */
pp_status pp_shard_read_taps(pp_shard* shard, uint32_t m, float* f32, uint16_t* bf16);

/* Message of the last error on the handle (or of the last failed create when NULL). */
size_t pp_last_error(const pp_shard* shard, char* buf, size_t len);
/* Library version string. */
const char* pp_version(void);

#ifdef __cplusplus
}
#endif
#endif
