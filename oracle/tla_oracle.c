/*
 * CPU oracle for the three-llm attention hot path (TEST INFRASTRUCTURE ONLY).
 *
 * Numerics follow the reference's JavaScript: `double` for every operation,
 * `(float)` casts exactly where the TypeScript writes into a Float32Array.
 * Build with -ffp-contract=off so that no fused multiply-add changes a
 * double result (JS engines do not contract).
 */
#include "tla_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

const char* orc_error_string(int code) {
  switch (code) {
    case ORC_OK: return "ok";
    case ORC_ERR_ROPE_DIM: return "RoPE dimension must be a non-negative even integer.";
    case ORC_ERR_ROPE_THETA: return "RoPE theta must be finite and greater than one.";
    case ORC_ERR_ROPE_FACTOR: return "RoPE scaling factor must be finite and at least one.";
    case ORC_ERR_YARN_RANGE: return "Invalid YaRN context or beta range.";
    case ORC_ERR_YARN_FACTOR: return "Invalid YaRN attention factor.";
    case ORC_ERR_LLAMA3_RANGE: return "Invalid Llama 3 RoPE frequency range.";
    case ORC_ERR_ARG: return "invalid argument";
    default: return "unknown error";
  }
}

/* rope.ts:4-52 */
int orc_rope_parameters(int32_t dim, double theta, const orc_rope_scaling* scaling, float* inv_freq,
                        double* attention_factor_out) {
  if (dim < 0 || dim % 2 != 0) return ORC_ERR_ROPE_DIM;                 /* :5-6 */
  if (!isfinite(theta) || theta <= 1) return ORC_ERR_ROPE_THETA;        /* :7 */
  const orc_rope_scaling* s = (scaling && scaling->type != ORC_ROPE_NONE) ? scaling : NULL;
  const int is_yarn = s && s->type == ORC_ROPE_YARN;                    /* :10-11 */
  double attention_factor = 1;
  double low = 0, high = 0;
  if (s && (!isfinite(s->factor) || s->factor < 1)) return ORC_ERR_ROPE_FACTOR; /* :14-15 */
  if (is_yarn) {                                                        /* :16-28 */
    if (!isfinite(s->original_context_length) || !isfinite(s->beta_fast) || !isfinite(s->beta_slow))
      return ORC_ERR_YARN_RANGE;
    if (!(s->original_context_length > 0 && s->beta_fast > 0 && s->beta_slow > 0 &&
          s->beta_fast >= s->beta_slow))
      return ORC_ERR_YARN_RANGE;
    attention_factor = s->has_attention_factor ? s->attention_factor : 1 + 0.1 * log(s->factor);
    if (!isfinite(attention_factor) || attention_factor <= 0) return ORC_ERR_YARN_FACTOR;
    const double cf = (dim * log(s->original_context_length / (s->beta_fast * 2 * M_PI))) / (2 * log(theta));
    const double cs = (dim * log(s->original_context_length / (s->beta_slow * 2 * M_PI))) / (2 * log(theta));
    low = fmax(0, floor(cf));
    high = fmin(dim - 1, ceil(cs));
    if (low == high) high += 0.001;
  }
  for (int32_t i = 0; i < dim / 2; i++) {                               /* :29-50 */
    double frequency = 1 / pow(theta, (2.0 * i) / dim);
    if (s && s->type == ORC_ROPE_LINEAR) frequency /= s->factor;
    if (is_yarn) {
      const double ramp = fmin(1, fmax(0, (i - low) / (high - low)));
      frequency *= 1 - ramp + ramp / s->factor;
    }
    if (s && s->type == ORC_ROPE_LLAMA3) {
      const double ocl = s->original_context_length, lf = s->low_freq_factor, hf = s->high_freq_factor;
      if (!isfinite(ocl) || !isfinite(lf) || !isfinite(hf)) return ORC_ERR_LLAMA3_RANGE;
      if (!(ocl > 0 && lf > 0 && hf > lf)) return ORC_ERR_LLAMA3_RANGE;
      const double wavelength = (2 * M_PI) / frequency;
      if (wavelength > ocl / lf) {
        frequency /= s->factor;
      } else if (wavelength >= ocl / hf) {
        const double smooth = (ocl / wavelength - lf) / (hf - lf);
        frequency *= (1 - smooth) / s->factor + smooth;
      }
    }
    if (inv_freq) inv_freq[i] = (float)frequency;                       /* Float32Array store */
  }
  if (attention_factor_out) *attention_factor_out = attention_factor;
  return ORC_OK;
}

/* math.ts:118-152 (rotate-half / NeoX layout) */
int orc_apply_rope(float* vector, int32_t head_offset, int32_t rotary_dim, int32_t position, double theta,
                   int32_t rope_freq_dim, int32_t rope_pair_count, const orc_rope_scaling* scaling) {
  if (rotary_dim <= 0) return ORC_OK;                                   /* :126 */
  if (rotary_dim % 2 != 0) return ORC_ERR_ROPE_DIM;
  const int32_t half = rotary_dim / 2;
  const int32_t freq_dim = rope_freq_dim ? rope_freq_dim : rotary_dim;  /* :129 */
  const int32_t pair_count = rope_pair_count >= 0 ? rope_pair_count : half;
  if (freq_dim < 0 || freq_dim % 2 != 0) return ORC_ERR_ROPE_DIM;
  float* inv_freq = (float*)malloc(sizeof(float) * (size_t)(freq_dim / 2 + 1));
  float* rotated = (float*)malloc(sizeof(float) * (size_t)rotary_dim);
  double attention_factor = 1;
  int rc = orc_rope_parameters(freq_dim, theta, scaling, inv_freq, &attention_factor);
  if (rc != ORC_OK) {
    free(inv_freq);
    free(rotated);
    return rc;
  }
  for (int32_t i = 0; i < rotary_dim; i++) {
    const double x = vector[head_offset + i];
    const int32_t freq_index = i < half ? i : i - half;
    if (freq_index >= pair_count) {
      rotated[i] = (float)x;
      continue;
    }
    const double partner = i < half ? -(double)vector[head_offset + i + half] : (double)vector[head_offset + i - half];
    /* invFreq[k] beyond its length is `undefined` in JS, which makes the angle NaN. */
    const double angle = freq_index < freq_dim / 2 ? (double)position * (double)inv_freq[freq_index] : NAN;
    rotated[i] = (float)((x * cos(angle) + partner * sin(angle)) * attention_factor);
  }
  for (int32_t i = 0; i < rotary_dim; i++) vector[head_offset + i] = rotated[i];
  free(inv_freq);
  free(rotated);
  return ORC_OK;
}

/* math.ts:60-76; the running sum stays a double, the stores are float32 */
void orc_softmax(const float* values, int32_t n, float* target) {
  double max_value = -INFINITY;
  for (int32_t i = 0; i < n; i++) {
    const double v = values[i];
    max_value = (isnan(v) || isnan(max_value)) ? NAN : fmax(max_value, v);
  }
  double sum = 0;
  for (int32_t i = 0; i < n; i++) {
    const double value = exp((double)values[i] - max_value);
    target[i] = (float)value;
    sum += value;
  }
  for (int32_t i = 0; i < n; i++) target[i] = (float)((double)target[i] / sum);
}

/* math.ts:78-97 */
void orc_rms_norm(const float* input, int32_t n, const float* weight, double epsilon, int32_t offset_weight,
                  float* target) {
  double sum_squares = 0;
  for (int32_t i = 0; i < n; i++) sum_squares += (double)input[i] * (double)input[i];
  const double inv_rms = 1 / sqrt(sum_squares / n + epsilon);
  for (int32_t i = 0; i < n; i++) {
    const double scale = weight == NULL ? 1 : offset_weight ? 1 + (double)weight[i] : (double)weight[i];
    target[i] = (float)((double)input[i] * inv_rms * scale);
  }
}

/* math.ts:154-167 */
void orc_rms_norm_packed_heads(float* vector, int32_t head_count, int32_t head_dim, const float* weight,
                               double epsilon, int32_t offset_weight) {
  float* tmp = (float*)malloc(sizeof(float) * (size_t)head_dim);
  for (int32_t head = 0; head < head_count; head++) {
    float* slice = vector + (size_t)head * head_dim;
    orc_rms_norm(slice, head_dim, weight, epsilon, offset_weight, tmp);
    memcpy(slice, tmp, sizeof(float) * (size_t)head_dim);
  }
  free(tmp);
}

static double opt_attn_scale(const orc_attn_options* o) {
  return o->has_attn_scale ? o->attn_scale : 1 / sqrt((double)o->head_dim);   /* math.ts:190 */
}

static int32_t first_token(const orc_attn_options* o, int32_t position) {    /* math.ts:208 */
  if (o->sliding_window > 0) {
    const int32_t f = position - o->sliding_window + 1;
    return f > 0 ? f : 0;
  }
  return 0;
}

/* math.ts:204-238: QK-norm, RoPE, cache append. Writes the rotated query into q_out. */
static int prepare_token(const float* qkv, int32_t position, float* key_cache, float* value_cache,
                         const orc_attn_options* o, float* q_out) {
  const int32_t D = o->head_dim, Hq = o->head_count, Hk = o->kv_head_count;
  const int32_t q_size = Hq * D, kv_size = Hk * D;
  const int32_t rotary = o->rotary_dim;
  float* key = (float*)malloc(sizeof(float) * (size_t)kv_size);
  float* value = (float*)malloc(sizeof(float) * (size_t)kv_size);
  memcpy(q_out, qkv, sizeof(float) * (size_t)q_size);
  memcpy(key, qkv + q_size, sizeof(float) * (size_t)kv_size);
  int rc = ORC_OK;
  if (o->q_norm_weight) orc_rms_norm_packed_heads(q_out, Hq, D, o->q_norm_weight, o->rms_epsilon, o->offset_rms_norm);
  if (!o->query_only && o->k_norm_weight)
    orc_rms_norm_packed_heads(key, Hk, D, o->k_norm_weight, o->rms_epsilon, o->offset_rms_norm);
  if (o->rope_theta > 0) {
    const int32_t freq_dim = o->rope_freq_dim ? o->rope_freq_dim : rotary;
    for (int32_t h = 0; h < Hq && rc == ORC_OK; h++)
      rc = orc_apply_rope(q_out, h * D, rotary, position, o->rope_theta, freq_dim, o->rope_pair_count, &o->scaling);
    if (!o->query_only)
      for (int32_t h = 0; h < Hk && rc == ORC_OK; h++)
        rc = orc_apply_rope(key, h * D, rotary, position, o->rope_theta, freq_dim, o->rope_pair_count, &o->scaling);
  }
  if (rc == ORC_OK && !o->query_only && o->write_cache) {
    memcpy(value, qkv + q_size + kv_size, sizeof(float) * (size_t)kv_size);
    if (o->v_norm) orc_rms_norm_packed_heads(value, Hk, D, NULL, o->rms_epsilon, 0);
    memcpy(key_cache + (size_t)position * kv_size, key, sizeof(float) * (size_t)kv_size);
    memcpy(value_cache + (size_t)position * kv_size, value, sizeof(float) * (size_t)kv_size);
  }
  free(key);
  free(value);
  return rc;
}

/* math.ts:242-269 for one query head, plus the gate of :271-273 */
static void attend_head(const float* q_rot, int32_t position, const float* key_cache, const float* value_cache,
                        const orc_attn_options* o, int32_t head, const float* gate, float* output) {
  const int32_t D = o->head_dim, Hq = o->head_count, Hk = o->kv_head_count;
  const int32_t kv_size = Hk * D;
  const int32_t q_off = head * D;
  const int32_t kv_head = (int32_t)(((int64_t)head * Hk) / Hq);              /* :244 */
  const int32_t kv_off = kv_head * D;
  const int32_t first = first_token(o, position);
  const int32_t n = position - first + 1;
  const double scale = opt_attn_scale(o);
  float* scores = (float*)malloc(sizeof(float) * (size_t)n);
  float* weights = (float*)malloc(sizeof(float) * (size_t)n);
  for (int32_t t = first; t <= position; t++) {
    double dot = 0;
    const float* k = key_cache + (size_t)t * kv_size + kv_off;
    for (int32_t i = 0; i < D; i++) dot += (double)q_rot[q_off + i] * (double)k[i];
    scores[t - first] = (float)(dot * scale);
  }
  orc_softmax(scores, n, weights);
  for (int32_t i = 0; i < D; i++) {
    double sum = 0;
    for (int32_t t = first; t <= position; t++)
      sum += (double)weights[t - first] * (double)value_cache[(size_t)t * kv_size + kv_off + i];
    float out = (float)sum;
    if (gate) out = (float)((double)out * (1 / (1 + exp(-(double)gate[q_off + i]))));   /* :278-280 */
    output[q_off + i] = out;
  }
  free(scores);
  free(weights);
}

int orc_causal_attention(const float* qkv, int32_t position, float* key_cache, float* value_cache,
                         const orc_attn_options* o, const float* gate, float* output) {
  if (!o || o->head_count <= 0 || o->kv_head_count <= 0 || o->head_dim <= 0 || position < 0) return ORC_ERR_ARG;
  float* q = (float*)malloc(sizeof(float) * (size_t)o->head_count * o->head_dim);
  int rc = prepare_token(qkv, position, key_cache, value_cache, o, q);
  if (rc == ORC_OK)
    for (int32_t h = 0; h < o->head_count; h++) attend_head(q, position, key_cache, value_cache, o, h, gate, output);
  free(q);
  return rc;
}

static void set_threads(int32_t threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
}

int orc_decode_batch(const float* qkv, const int32_t* positions, int32_t batch, int32_t max_tokens,
                     float* key_cache, float* value_cache, const orc_attn_options* o, const float* gate,
                     float* out, int32_t threads) {
  if (!o || batch < 0 || max_tokens <= 0) return ORC_ERR_ARG;
  const int32_t D = o->head_dim, Hq = o->head_count, Hk = o->kv_head_count;
  const size_t row = (size_t)(Hq + 2 * Hk) * D, q_size = (size_t)Hq * D;
  const size_t cache_seq = (size_t)max_tokens * Hk * D;
  for (int32_t b = 0; b < batch; b++)
    if (positions[b] < 0 || positions[b] >= max_tokens) return ORC_ERR_ARG;
  float* q = (float*)malloc(sizeof(float) * q_size * (size_t)(batch > 0 ? batch : 1));
  int rc = ORC_OK;
  set_threads(threads);
#pragma omp parallel for schedule(static) if (threads > 1)
  for (int32_t b = 0; b < batch; b++) {
    int r = prepare_token(qkv + b * row, positions[b], key_cache + b * cache_seq, value_cache + b * cache_seq, o,
                          q + b * q_size);
    if (r != ORC_OK) {
#pragma omp critical
      rc = r;
    }
  }
  if (rc == ORC_OK) {
    const int64_t items = (int64_t)batch * Hq;
#pragma omp parallel for schedule(dynamic, 1) if (threads > 1)
    for (int64_t it = 0; it < items; it++) {
      const int32_t b = (int32_t)(it / Hq), h = (int32_t)(it % Hq);
      attend_head(q + b * q_size, positions[b], key_cache + b * cache_seq, value_cache + b * cache_seq, o, h,
                  gate ? gate + b * q_size : NULL, out + b * q_size);
    }
  }
  free(q);
  return rc;
}

int orc_prefill(const float* qkv, const int32_t* start_pos, const float* gate, int32_t batch, int32_t seq_len,
                int32_t max_tokens, float* key_cache, float* value_cache, const orc_attn_options* o, float* out,
                int32_t threads) {
  if (!o || batch < 0 || seq_len < 0 || max_tokens <= 0) return ORC_ERR_ARG;
  const int32_t D = o->head_dim, Hq = o->head_count, Hk = o->kv_head_count;
  const size_t row = (size_t)(Hq + 2 * Hk) * D, q_size = (size_t)Hq * D;
  const size_t cache_seq = (size_t)max_tokens * Hk * D;
  for (int32_t b = 0; b < batch; b++)
    if (start_pos[b] < 0 || (int64_t)start_pos[b] + seq_len > max_tokens) return ORC_ERR_ARG;
  const size_t tokens = (size_t)batch * seq_len;
  float* q = (float*)malloc(sizeof(float) * q_size * (tokens > 0 ? tokens : 1));
  int rc = ORC_OK;
  set_threads(threads);
  /* The reference replays causalAttention (math.ts:179-276) token by token.
   * Token t's attention reads cache slots [window start, start + t] only, all
   * written by then, so running every token's QK-norm / RoPE / append first
   * (in token order within a sequence) and the attention of all
   * (token, head) pairs afterwards gives the same values as the replay. */
#pragma omp parallel for schedule(dynamic, 1) if (threads > 1)
  for (int32_t b = 0; b < batch; b++) {
    for (int32_t t = 0; t < seq_len; t++) {
      const size_t i = (size_t)b * seq_len + t;
      int r = prepare_token(qkv + i * row, start_pos[b] + t, key_cache + b * cache_seq, value_cache + b * cache_seq,
                            o, q + i * q_size);
      if (r != ORC_OK) {
#pragma omp critical
        rc = r;
        break;
      }
    }
  }
  if (rc == ORC_OK) {
    const int64_t items = (int64_t)tokens * Hq;
#pragma omp parallel for schedule(dynamic, 64) if (threads > 1)
    for (int64_t it = 0; it < items; it++) {
      const size_t i = (size_t)(it / Hq);
      const int32_t h = (int32_t)(it % Hq), b = (int32_t)(i / (size_t)seq_len), t = (int32_t)(i % (size_t)seq_len);
      attend_head(q + i * q_size, start_pos[b] + t, key_cache + b * cache_seq, value_cache + b * cache_seq, o, h,
                  gate ? gate + i * q_size : NULL, out + i * q_size);
    }
  }
  free(q);
  return rc;
}

int orc_linear(const float* input, int32_t rows, const float* weight, const float* bias, int32_t in_size,
               int32_t out_size, float* target, int32_t threads) {
  if (!input || !weight || !target || rows < 0 || in_size <= 0 || out_size <= 0) return ORC_ERR_ARG;
  set_threads(threads);
#pragma omp parallel for schedule(static) if (threads > 1)
  for (int32_t r = 0; r < rows; r++) {
    const float* x = input + (size_t)r * in_size;
    float* y = target + (size_t)r * out_size;
    double* sum = (double*)malloc(sizeof(double) * (size_t)out_size);
    for (int32_t o = 0; o < out_size; o++) sum[o] = bias ? (double)bias[o] : 0;   /* math.ts:15 */
    for (int32_t i = 0; i < in_size; i++) {                                        /* math.ts:17-19 */
      const double xi = (double)x[i];
      const float* w = weight + (size_t)i * out_size;
      for (int32_t o = 0; o < out_size; o++) sum[o] += xi * (double)w[o];
    }
    for (int32_t o = 0; o < out_size; o++) y[o] = (float)sum[o];                  /* :21, Float32Array store */
    free(sum);
  }
  return ORC_OK;
}

int orc_attend_heads(const float* q_rot, const int32_t* positions, int32_t batch, int32_t max_tokens,
                     const float* key_cache, const float* value_cache, const orc_attn_options* o,
                     int32_t head_begin, int32_t head_end, float* out, int32_t threads) {
  if (!o || batch < 0 || head_begin < 0 || head_end > o->head_count || head_begin > head_end) return ORC_ERR_ARG;
  const int32_t D = o->head_dim, Hq = o->head_count, Hk = o->kv_head_count;
  const size_t q_size = (size_t)Hq * D, cache_seq = (size_t)max_tokens * Hk * D;
  const int32_t nh = head_end - head_begin;
  const int64_t items = (int64_t)batch * nh;
  set_threads(threads);
#pragma omp parallel for schedule(dynamic, 1) if (threads > 1)
  for (int64_t it = 0; it < items; it++) {
    const int32_t b = (int32_t)(it / nh), h = head_begin + (int32_t)(it % nh);
    attend_head(q_rot + b * q_size, positions[b], key_cache + b * cache_seq, value_cache + b * cache_seq, o, h,
                NULL, out + b * q_size);
  }
  return ORC_OK;
}
