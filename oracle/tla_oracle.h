/*
 * CPU oracle for the three-llm attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY: this library is the checker for the CUDA path
 * (parity tests, smoke check, and the timed CPU baseline in bench.py). The
 * product library never links or calls it.
 *
 * It restates, in C, the reference's TypeScript CPU attention with the
 * reference's numerics: every arithmetic step runs in IEEE double (JS
 * `number`) and values are rounded to float32 exactly where the TypeScript
 * stores into a Float32Array.
 *
 *   orc_rope_parameters  <- packages/three-llm/src/runtime/rope.ts:4-52
 *   orc_apply_rope       <- packages/three-llm/src/runtime/math.ts:118-152
 *   orc_softmax          <- packages/three-llm/src/runtime/math.ts:60-76
 *   orc_rms_norm         <- packages/three-llm/src/runtime/math.ts:78-97
 *   orc_rms_norm_packed_heads <- packages/three-llm/src/runtime/math.ts:154-167
 *   orc_causal_attention <- packages/three-llm/src/runtime/math.ts:179-276
 *
 * Batch, ragged and prefill wrappers loop the single-sequence function the
 * way the reference's runners do (one runner per sequence; prefill replays
 * the one-token step per prompt position, decoder/DecoderTSLRunner.ts:504-530).
 */
#ifndef TLA_ORACLE_H
#define TLA_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  ORC_ROPE_NONE = 0,   /* no scaling object */
  ORC_ROPE_LINEAR = 1,
  ORC_ROPE_YARN = 2,
  ORC_ROPE_LLAMA3 = 3,
};

enum {
  ORC_OK = 0,
  ORC_ERR_ROPE_DIM = -1,      /* 'RoPE dimension must be a non-negative even integer.' */
  ORC_ERR_ROPE_THETA = -2,    /* 'RoPE theta must be finite and greater than one.' */
  ORC_ERR_ROPE_FACTOR = -3,   /* 'RoPE scaling factor must be finite and at least one.' */
  ORC_ERR_YARN_RANGE = -4,    /* 'Invalid YaRN context or beta range.' */
  ORC_ERR_YARN_FACTOR = -5,   /* 'Invalid YaRN attention factor.' */
  ORC_ERR_LLAMA3_RANGE = -6,  /* 'Invalid Llama 3 RoPE frequency range.' */
  ORC_ERR_ARG = -7,           /* bad sizes or pointers passed to a wrapper */
};

typedef struct orc_rope_scaling {
  int32_t type;                   /* ORC_ROPE_* */
  double factor;
  double original_context_length; /* yarn, llama3 */
  double beta_fast, beta_slow;    /* yarn */
  int32_t has_attention_factor;   /* yarn: 0 => 1 + 0.1*ln(factor) */
  double attention_factor;
  double low_freq_factor, high_freq_factor; /* llama3 */
} orc_rope_scaling;

typedef struct orc_attn_options {
  int32_t head_count;
  int32_t kv_head_count;
  int32_t head_dim;
  int32_t rotary_dim;       /* rotaryDim (default head_dim) */
  int32_t rope_freq_dim;    /* ropeFreqDim (0 => rotary_dim) */
  int32_t rope_pair_count;  /* ropePairCount (<0 => rotary_dim/2) */
  double rope_theta;        /* 0 disables RoPE */
  orc_rope_scaling scaling; /* type ORC_ROPE_NONE => no scaling */
  int32_t sliding_window;   /* 0 => unlimited */
  int32_t has_attn_scale;   /* 0 => 1/sqrt(head_dim) */
  double attn_scale;
  const float* q_norm_weight; /* NULL => no Q norm */
  const float* k_norm_weight; /* NULL => no K norm */
  double rms_epsilon;
  int32_t offset_rms_norm;
  int32_t query_only;
  int32_t write_cache;
  int32_t v_norm;
} orc_attn_options;

const char* orc_error_string(int code);

int orc_rope_parameters(int32_t dim, double theta, const orc_rope_scaling* scaling,
                        float* inv_freq, double* attention_factor);
int orc_apply_rope(float* vector, int32_t head_offset, int32_t rotary_dim, int32_t position,
                   double theta, int32_t rope_freq_dim, int32_t rope_pair_count,
                   const orc_rope_scaling* scaling);
void orc_softmax(const float* values, int32_t n, float* target);
void orc_rms_norm(const float* input, int32_t n, const float* weight, double epsilon,
                  int32_t offset_weight, float* target);
void orc_rms_norm_packed_heads(float* vector, int32_t head_count, int32_t head_dim,
                               const float* weight, double epsilon, int32_t offset_weight);

/* One token of causal attention for one sequence.
 * qkv: packed [Q (Hq*D) | K (Hk*D) | V (Hk*D)] for the token at `position`.
 * key_cache/value_cache: token-major [max_tokens][Hk*D] float32.
 * gate: NULL or [Hq*D] (output *= sigmoid(gate), math.ts:271-273).
 * output: [Hq*D]. */
int orc_causal_attention(const float* qkv, int32_t position, float* key_cache, float* value_cache,
                         const orc_attn_options* o, const float* gate, float* output);

/* Batched / ragged decode: sequence b uses caches + b*max_tokens*kv_size.
 * qkv [B][Hq+2Hk][D], positions [B], gate NULL or [B][Hq*D], out [B][Hq*D].
 * threads > 1 runs (sequence, head) work items on OpenMP threads; the
 * numerics do not depend on the thread count. */
int orc_decode_batch(const float* qkv, const int32_t* positions, int32_t batch, int32_t max_tokens,
                     float* key_cache, float* value_cache, const orc_attn_options* o,
                     const float* gate, float* out, int32_t threads);

/* Prefill as the reference runs it: S one-token steps at start_pos[b]+t
 * (decoder/DecoderTSLRunner.ts:472-480, 504-530), each with the decode
 * graph's output gate when gate != NULL.
 * qkv [B][S][Hq+2Hk][D], gate NULL or [B][S][Hq*D], out [B][S][Hq*D].
 * The per-token norm / RoPE / append steps run in token order within a
 * sequence; the attention of the (token, head) pairs runs on `threads`
 * OpenMP threads. The values equal the token-by-token replay. */
int orc_prefill(const float* qkv, const int32_t* start_pos, const float* gate, int32_t batch, int32_t seq_len,
                int32_t max_tokens, float* key_cache, float* value_cache, const orc_attn_options* o,
                float* out, int32_t threads);

/* linear (packages/three-llm/src/runtime/math.ts:6-25) for `rows` independent
 * inputs: target[r][o] = bias[o] + sum_i input[r][i] * weight[i][o], the sum in
 * double (JS numbers), the result stored as float32. weight is the reference's
 * [inputSize][outputSize] layout; bias may be NULL. Rows run on `threads`. */
int orc_linear(const float* input, int32_t rows, const float* weight, const float* bias, int32_t in_size,
               int32_t out_size, float* target, int32_t threads);

/* Attention of the listed query heads only, over an already-filled cache
 * (no append): used to time a bounded sample of a large decode workload.
 * q_rot: post-RoPE queries [B][Hq*D]. */
int orc_attend_heads(const float* q_rot, const int32_t* positions, int32_t batch, int32_t max_tokens,
                     const float* key_cache, const float* value_cache, const orc_attn_options* o,
                     int32_t head_begin, int32_t head_end, float* out, int32_t threads);

#ifdef __cplusplus
}
#endif
#endif
