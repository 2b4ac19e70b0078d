/*
 * Oracle: a CPU restatement of potpori's per-shard Qwen3 forward.
 *
 * TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and the cpu_baseline /
 * reference legs of bench.py may load this library, and only as the checker or the timed
 * CPU baseline; the product path never calls it.
 *
 * What it restates (reference paths are relative to the potpori repository):
 *   - src/qwen/tiny.rs:9-132     the scalar Qwen3 forward: RMSNorm, projections as
 *                                row . input sums, per-head QK-RMSNorm, rotate-half RoPE,
 *                                causal GQA softmax attention, SwiGLU, tied output head.
 *   - src/qwen/model.rs:198-337  the shard cut: layers [a,b), embedding on the first shard,
 *                                final norm + tied vocab projection on the last shard,
 *                                F32 KV cache [capacity, kv_dim] per layer written at
 *                                absolute positions (rollback = overwrite).
 *   - src/qwen/model.rs:373-412  step validation (chunk in {1, chunk}, end <= capacity,
 *                                token range, finite hidden input) and gather = 0..end.
 *   - src/engine.rs:14-29        greedy argmax: first index of the strict maximum, no
 *                                result for an empty row or any non-finite value.
 *   - src/qwen/hf.rs:85-91,227-272  parameter dtypes: matrices BF16, names containing
 *                                "norm" F32; an F32 matrix is rounded to BF16 on load.
 *
 * Parity is pinned by tests against the reference's golden vectors
 * (tests/fixtures/dspark_tiny: transformers logits and per-layer features of a 6-layer
 * tiny Qwen3) and against transformers' Qwen3ForCausalLM run in F32 on the same weights.
 */
#ifndef POTPORI_ORACLE_H
#define POTPORI_ORACLE_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

typedef struct or_config {
  int32_t layers, hidden, intermediate, head_dim, n_heads, n_kv_heads, vocab_size;
  float rms_norm_eps, rope_theta;
} or_config;

typedef struct or_shard or_shard;

enum { OR_OK = 0, OR_E_INVALID = 1, OR_E_NONFINITE = 2, OR_E_MISSING = 3 };
enum { OR_F32 = 0, OR_BF16 = 1 };
/* RoPE angle evaluation. 0: angle = pos * theta^(-2i/d) in double, cos/sin in double,
 * rounded to f32 (the table the CUDA path uses). 1: tiny.rs:29-30 verbatim in f32:
 * angle = (float)pos / powf(theta, 2i/d), sinf/cosf. */
enum { OR_ROPE_F64 = 0, OR_ROPE_F32 = 1 };

or_shard *or_shard_create(const or_config *cfg, int32_t layer_begin, int32_t layer_end,
                          int32_t capacity, int32_t chunk);
void or_shard_destroy(or_shard *s);
/* Set one parameter by its checkpoint name. dtype OR_F32 or OR_BF16 (raw bits). */
int or_shard_set_tensor(or_shard *s, const char *name, int32_t dtype, const void *data,
                        int64_t elements);
/* Fill every parameter from the seeded generator (matrices N(0,std) -> BF16, norms 1). */
int or_shard_init_random(or_shard *s, uint64_t seed, float std);
/* Fill KV rows [0, rows) of every layer with seeded N(0,1) values (bench warm context). */
int or_shard_fill_kv(or_shard *s, uint64_t seed, int32_t rows);
int or_shard_missing(const or_shard *s, char *buf, int64_t len);
void or_shard_set_rope_mode(or_shard *s, int32_t mode);
/* One forward of m rows at absolute position pos. The first shard takes tokens, others
 * take hidden [m, hidden]. out: hidden [m, hidden], or logits [m, vocab] (row form) on the
 * last shard. taps (optional): [layers_in_shard][m][hidden], the output of every layer. */
int or_shard_forward(or_shard *s, int32_t pos, int32_t m, const int32_t *tokens,
                     const float *hidden, float *out, float *taps);
void or_shard_reset(or_shard *s);
/* engine.rs:14-29. Returns 1 and sets *index, or 0 for an empty or non-finite row. */
int or_argmax(const float *row, int64_t n, int32_t *index);
/* Largest and second-largest value of a finite row (ties count twice). */
void or_top2(const float *row, int64_t n, float *top1, float *top2);
void or_set_threads(int32_t n);
int32_t or_get_threads(void);
/* Seeded generator, exposed so tests can compare the device generator bit for bit. */
void or_gen_bf16(uint64_t seed, const char *name, int64_t start, int64_t count, float std,
                 uint16_t *out);
uint64_t or_name_hash(const char *name);

#ifdef __cplusplus
}
#endif
#endif
