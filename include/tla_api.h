/*
 * tla_api.h - C ABI of the B200 attention path for three-llm.
 *
 * This is the boundary a three-llm host binds (N-API addon, FFI or ctypes) in
 * place of the WebGPU operator `TSLAttention`
 * (packages/three-llm/src/tsl/TSLAttention.ts:19-448). Plain C types only:
 * device buffers are `void*` / typed pointers that the caller owns, streams
 * are `cudaStream_t` passed as `void*` (NULL = legacy default stream).
 * Every call returns a tla_status (0 = ok, < 0 = error); nothing throws.
 *
 * Threading: a tla_ctx (and every layer made from it) is used from one host
 * thread and one CUDA stream at a time. Calls are stream-ordered and do not
 * block, except tla_cache_read/tla_cache_write/tla_get_error, which
 * synchronise the device.
 */
#ifndef TLA_API_H
#define TLA_API_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. The RoPE codes carry the reference's error messages
 * (packages/three-llm/src/runtime/rope.ts:5-41); tla_status_string returns them. */
typedef enum tla_status {
  TLA_OK = 0,
  TLA_ERR_INVALID_ARG = -1,
  TLA_ERR_ROPE_DIM = -2,      /* RoPE dimension must be a non-negative even integer. (rope.ts:5-6) */
  TLA_ERR_ROPE_THETA = -3,    /* RoPE theta must be finite and greater than one. (rope.ts:7) */
  TLA_ERR_ROPE_FACTOR = -4,   /* RoPE scaling factor must be finite and at least one. (rope.ts:14-15) */
  TLA_ERR_YARN_RANGE = -5,    /* Invalid YaRN context or beta range. (rope.ts:17-20) */
  TLA_ERR_YARN_FACTOR = -6,   /* Invalid YaRN attention factor. (rope.ts:22) */
  TLA_ERR_LLAMA3_RANGE = -7,  /* Invalid Llama 3 RoPE frequency range. (rope.ts:38-41) */
  TLA_ERR_ROTARY_DIM = -8,    /* Invalid rotary dimension (load/DecoderRecipe.ts:409-415) */
  TLA_ERR_UNSUPPORTED = -9,   /* shape outside what the kernels implement */
  TLA_ERR_CUDA = -10,         /* a CUDA runtime call failed */
  TLA_ERR_OUT_OF_MEMORY = -11,
  TLA_ERR_POSITION = -12,     /* device-reported: a position outside [0, max_tokens) */
  TLA_ERR_TIMEOUT = -13,      /* device-reported: a bounded in-kernel wait expired */
  TLA_ERR_NO_DEVICE = -14,
  TLA_ERR_SHARED = -15,       /* operation not allowed on a layer that borrows another's cache */
  TLA_ERR_SCRATCH_LIMIT = -16, /* request exceeds the fixed scratch of tla_decode_noalloc */
  TLA_ERR_BOUNDS = -17         /* device-reported, bounds-check builds only: an index outside its buffer
                                  (the access was skipped) */
} tla_status;

/* RoPE scaling: RopeScalingConfig | YarnRoPEConfig (packages/three-llm/src/types.ts:245-256). */
typedef enum tla_rope_type {
  TLA_ROPE_NONE = 0,
  TLA_ROPE_LINEAR = 1,
  TLA_ROPE_YARN = 2,
  TLA_ROPE_LLAMA3 = 3
} tla_rope_type;

typedef struct tla_rope_scaling {
  int32_t type;                   /* tla_rope_type */
  double factor;
  double original_context_length; /* yarn, llama3 */
  double beta_fast, beta_slow;    /* yarn */
  int32_t has_attention_factor;   /* yarn: 0 => 1 + 0.1*ln(factor) */
  double attention_factor;
  double low_freq_factor, high_freq_factor; /* llama3 */
} tla_rope_scaling;

/* Flag bits of tla_attn_config.flags */
enum {
  TLA_FLAG_OFFSET_RMS_NORM = 1u << 0, /* offsetRMSNorm: QK-norm scale is (1 + w) */
  TLA_FLAG_V_NORM = 1u << 1,          /* vNorm: weightless RMS norm of V before caching */
  TLA_FLAG_IO_FP32 = 1u << 2,         /* qkv, gate and out are float32 (default: fp16) */
  TLA_FLAG_CACHE_FP32 = 1u << 3       /* K/V cache in float32 (default: fp16) */
};

/* AttentionKernelOptions (packages/three-llm/src/types.ts:288-312) plus the
 * TSLAttention constructor's sizes (TSLAttention.ts:64-70). */
typedef struct tla_attn_config {
  int32_t head_count;      /* headCount */
  int32_t kv_head_count;   /* kvHeadCount; 0 => head_count */
  int32_t head_dim;        /* headDim */
  int32_t max_tokens;      /* maxTokens: cache slots per sequence */
  int32_t max_batch;       /* sequences the cache holds (the reference has one) */
  int32_t rotary_dim;      /* rotaryDim; -1 => head_dim */
  int32_t rope_freq_dim;   /* ropeFreqDim; 0 => rotary_dim */
  int32_t rope_pair_count; /* ropePairCount; -1 => rotary_dim / 2 */
  double rope_theta;       /* ropeTheta; 0 disables RoPE */
  tla_rope_scaling rope_scaling; /* ropeScaling ?? yarn; type NONE => none */
  int32_t sliding_window;  /* slidingWindow; 0 => none */
  int32_t has_attn_scale;  /* 0 => attnScale = 1/sqrt(head_dim) */
  double attn_scale;
  double rms_epsilon;      /* rmsEpsilon; 0 => 1e-6 */
  uint32_t flags;          /* TLA_FLAG_* */
} tla_attn_config;

typedef struct tla_ctx tla_ctx;
typedef struct tla_layer tla_layer;

/* Physical cache view (for zero-copy host bindings and tests). Element
 * (seq, kv_head, token, d) lives at base + seq*seq_stride + kv_head*head_stride
 * + token*token_stride + d, strides in elements. */
typedef struct tla_cache_view {
  void* key;
  void* value;
  int64_t seq_stride, head_stride, token_stride;
  int32_t elem_bytes;      /* 2 (fp16) or 4 (fp32) */
} tla_cache_view;

const char* tla_status_string(int status);

/* Context: one per device. Owns the error word and the split-KV scratch. */
int tla_create(int device, tla_ctx** out);
int tla_destroy(tla_ctx* ctx);

/* Device-reported errors since the last reset (synchronises the device).
 * Replaces the reference's absence of a GPU error channel. With reset != 0
 * the error word is cleared and, when an error was recorded, so are the
 * context's split-KV completion counters, so the next launch on the context
 * starts from a clean state. */
int tla_get_error(tla_ctx* ctx, int reset);

/* ropeParameters (packages/three-llm/src/runtime/rope.ts:4-52):
 * inv_freq[dim/2] float32 and the YaRN attention factor. */
int tla_rope_parameters(int32_t dim, double theta, const tla_rope_scaling* scaling, float* inv_freq,
                        double* attention_factor);

/* new TSLAttention(qkv, hiddenSize, headCount, maxTokens, options)
 * (TSLAttention.ts:64-166). q_norm_weight / k_norm_weight: host float32
 * [head_dim] or NULL (qNormWeight / kNormWeight). Allocates and zeroes the
 * K/V cache [max_batch][kv_head_count][max_tokens][head_dim]. */
int tla_layer_create(tla_ctx* ctx, const tla_attn_config* config, const float* q_norm_weight,
                     const float* k_norm_weight, tla_layer** out);
/* sharedAttention (TSLAttention.ts:122-139): dst reads src's cache and
 * stops appending to it (no copy step, TSLAttention.ts:154-156). Shapes must match. */
int tla_layer_share_cache(tla_layer* dst, const tla_layer* src);
int tla_layer_destroy(tla_layer* layer);
int tla_layer_cache_view(const tla_layer* layer, tla_cache_view* view);

/* One decode step for `batch` sequences (TSLAttention.compute, TSLAttention.ts:443-447,
 * with its four kernels fused: copy-KV :252-286, query :288-304, scores :306-356,
 * softmax+PV :358-428).
 *   qkv       device [batch][head_count + 2*kv_head_count][head_dim]  ([Q | K | V])
 *   positions device int32 [batch]: the new token's position (positionNode)
 *   gate      device [batch][head_count][head_dim] or NULL (gateNode: out *= sigmoid(gate))
 *   out       device [batch][head_count][head_dim]
 * The new K (after QK-norm and RoPE) and V are written to slot positions[b]. */
int tla_decode(tla_layer* layer, const void* qkv, const int32_t* positions, const void* gate, void* out,
               int32_t batch, void* stream);

/* queryAttribute (TSLAttention.ts:53, written by the query kernel :288-304):
 * the rotated queries of a decode step, QK-norm then RoPE at positions[b]
 * exactly as tla_decode forms them, as float32 [batch][head_count][head_dim].
 * Reads qkv only (nothing is appended). */
int tla_query(tla_layer* layer, const void* qkv, const int32_t* positions, float* query_out, int32_t batch,
              void* stream);

/* scoreAttribute (TSLAttention.ts:52, written by the score kernel :306-356):
 * scores_out[b][h][t] = attnScale * <query[b][h], K[b][kv(h)][t]> for every
 * cache slot t in [window start, positions[b]], over the cache as it holds
 * now (so after tla_decode it includes the appended token); slots outside
 * that range are left untouched, as in the reference's buffer.
 *   query      device float32 [batch][head_count][head_dim] (tla_query's output)
 *   scores_out device float32 [batch][head_count][max_tokens]
 * An inspection and test path: tla_decode never materialises its scores. */
int tla_scores(tla_layer* layer, const float* query, const int32_t* positions, float* scores_out, int32_t batch,
               void* stream);

/* Causal prefill of seq_len tokens per sequence starting at start_pos[b]:
 * equal to seq_len decode steps at start_pos[b] + t
 * (DecoderTSLRunner.prefillTokens, packages/three-llm/src/decoder/DecoderTSLRunner.ts:504-530,
 * which replays the one-token graph, output gate included, per prompt position).
 *   qkv       device [batch][seq_len][head_count + 2*kv_head_count][head_dim]
 *   start_pos device int32 [batch]
 *   gate      device [batch][seq_len][head_count][head_dim] or NULL
 *             (gateNode, TSLAttention.ts:418-423: out *= sigmoid(gate))
 *   out       device [batch][seq_len][head_count][head_dim] */
int tla_prefill(tla_layer* layer, const void* qkv, const int32_t* start_pos, const void* gate, int32_t seq_len,
                void* out, int32_t batch, void* stream);

/* The QKV projection feeding this layer (TSLLinear, packages/three-llm/src/tsl/TSLLinear.ts:56-75,
 * wired at decoder/DecoderTSLRunner.ts:293-297; CPU linear, runtime/math.ts:6-25), fused with the
 * attention's front end: [Q | K | V] = x W + bias runs on the tensor cores and its epilogue applies the
 * QK-norm and RoPE at each row's position, appends K and V (vNorm) to the cache and hands the rotated
 * queries to the attention kernel, so the raw [Q | K | V] rows never go through HBM. The result equals
 * tla_decode / tla_prefill on qkv = x W + bias.
 *   x      device fp16 [batch][hidden] (decode) or [batch][seq_len][hidden] (prefill)
 *   weight device fp16 [hidden][(head_count + 2*kv_head_count) * head_dim]: the reference's
 *          [inputSize][outputSize] layout
 *   bias   device float32 [(head_count + 2*kv_head_count) * head_dim] or NULL
 * hidden must be a multiple of 8; fp16 I/O and cache, head_dim 64 or 128 (else TLA_ERR_UNSUPPORTED). */
int tla_qkv_decode(tla_layer* layer, const void* x, const void* weight, const float* bias, int32_t hidden,
                   const int32_t* positions, const void* gate, void* out, int32_t batch, void* stream);
int tla_qkv_prefill(tla_layer* layer, const void* x, const void* weight, const float* bias, int32_t hidden,
                    const int32_t* start_pos, const void* gate, int32_t seq_len, void* out, int32_t batch,
                    void* stream);

/* The attention output projection and the residual add after it (DecoderTSLRunner.ts:299-309, 353-356:
 * attnProj TSLLinear, then TSLAdd): y = residual + attn W + bias on the tensor cores.
 *   attn     device fp16 [rows][in_features] (attention output rows)
 *   weight   device fp16 [in_features][hidden] (the reference's [inputSize][outputSize] layout)
 *   bias     device float32 [hidden] or NULL; residual device [rows][hidden] or NULL
 *   y        device [rows][hidden]
 * With TLA_FLAG_IO_FP32 in io_flags, residual and y are float32 (else fp16). in_features and hidden
 * must be multiples of 64. With head-sharded attention, the rank's attention columns and the matching
 * rows of W give this rank's partial product (bias and residual NULL, float32 y), which the ranks sum. */
int tla_out_proj(tla_ctx* ctx, const void* attn, const void* weight, const float* bias, const void* residual,
                 void* y, int32_t rows, int32_t in_features, int32_t hidden, uint32_t io_flags, void* stream);

/* Sequence-sharded decode building block: attend over cache slots
 * [0, local_tokens) that hold global positions [slot_offset, slot_offset +
 * local_tokens), and emit per query head the partial triple
 * partial[b][h] = {m (log2 domain), l, o[head_dim] (unnormalised)} as float32
 * [batch][head_count][head_dim + 2]. If append != 0 the new token (global
 * position positions[b]) is written to slot positions[b] - slot_offset and
 * included. Slots outside [window start, positions[b]] are excluded. */
int tla_decode_partial(tla_layer* layer, const void* qkv, const int32_t* positions, int32_t slot_offset,
                       int32_t local_tokens, int32_t append, float* partial, int32_t batch, void* stream);

/* Log-sum-exp merge of `ranks` partial triples laid out
 * [ranks][batch][head_count][head_dim + 2] into out [batch][head_count][head_dim]
 * (fp16, or float32 with TLA_FLAG_IO_FP32 in io_flags), times sigmoid(gate) if gate != NULL. */
int tla_combine_lse(const float* partials, int32_t ranks, int32_t batch, int32_t head_count, int32_t head_dim,
                    const void* gate, void* out, uint32_t io_flags, void* stream);

/* Peer-memory exchange for sequence-sharded decode across the GPUs of one
 * node (no counterpart in the reference, which runs on one device). Each
 * rank creates its exchange buffer (returning a 64-byte IPC handle), the
 * ranks swap handles out of band, connect, and then per layer
 * tla_exchange_combine pushes this rank's partial triples
 * ([batch][head_count][head_dim + 2], as from tla_decode_partial) into every
 * peer's buffer over NVLink, waits (bounded; TLA_ERR_TIMEOUT via
 * tla_get_error) for all peers' triples of the same step and writes the
 * log-sum-exp merge to out ([batch][head_count][head_dim], fp16 or with
 * TLA_FLAG_IO_FP32 float32). Every rank must call it the same number of
 * times; the step counter lives on the device, so the call can be captured
 * in a CUDA graph. batch * head_count <= 1024. */
typedef struct tla_exchange tla_exchange;
int tla_exchange_create(tla_ctx* ctx, int32_t rank, int32_t ranks, size_t slot_bytes, tla_exchange** out,
                        void* ipc_handle_out);
int tla_exchange_connect(tla_exchange* exchange, const void* ipc_handles /* [ranks][64] */);
int tla_exchange_combine(tla_exchange* exchange, const float* partial, int32_t batch, int32_t head_count,
                         int32_t head_dim, const void* gate, void* out, uint32_t io_flags, void* stream);
/* Same-process alternative to the IPC handles: tla_exchange_buffer returns
 * this rank's buffer, tla_exchange_connect_buffers takes every rank's buffer
 * as a device pointer this device can address (ranks on one device, or
 * buffers the caller mapped itself). */
int tla_exchange_buffer(tla_exchange* exchange, void** buffer_out);
int tla_exchange_connect_buffers(tla_exchange* exchange, void* const* buffers /* [ranks] */);
int tla_exchange_destroy(tla_exchange* exchange);

/* tla_out_proj across the GPUs of a head-sharded layer (no counterpart in the reference, which runs on
 * one device). attn [rows][in_features] holds this rank's query heads' attention output and weight
 * ([in_features][hidden] fp16) the matching rows of W. The product runs on the tensor cores and its
 * epilogue stores each partial tile over NVLink straight into the exchange buffer of the rank that owns
 * those hidden columns (hidden / ranks each: a reduce-scatter fused into the GEMM); then one kernel sums
 * the owned block over every rank, adds bias and residual and sends the block to every rank, so each rank
 * ends with y = residual + sum over ranks of attn_r W_r + bias, [rows][hidden] (fp16, or float32 with
 * TLA_FLAG_IO_FP32). The exchange's slot_bytes must hold 2 * rows * hidden / ranks floats and hidden must
 * be a multiple of 64 * ranks. Every rank calls it with the same shapes, the same number of times; the
 * waits are bounded (TLA_ERR_TIMEOUT through tla_get_error). */
int tla_out_proj_allreduce(tla_exchange* exchange, const void* attn, const void* weight, const float* bias,
                           const void* residual, void* y, int32_t rows, int32_t in_features, int32_t hidden,
                           uint32_t io_flags, void* stream);

/* tla_decode_partial fused with the exchange: this rank's split-KV decode
 * over its token block, then one kernel that merges each query row's segments,
 * exchanges the row's triple with every rank of `exchange` and writes the
 * merged output ([batch][head_count][head_dim], the layer's I/O type, times
 * sigmoid(gate) when gate is given). partial: caller scratch of
 * batch * head_count * (head_dim + 2) floats. Every rank calls it once per
 * step. No counterpart in the reference. */
int tla_decode_exchange(tla_layer* layer, tla_exchange* exchange, const void* qkv, const int32_t* positions,
                        int32_t slot_offset, int32_t local_tokens, int32_t append, float* partial, const void* gate,
                        void* out, int32_t batch, void* stream);

/* reset() (TSLAttention.ts:434-441): zero the cache. A borrowing layer is a no-op. */
int tla_cache_reset(tla_layer* layer, void* stream);

/* Test / binding view of the cache as the reference lays it out
 * (token-major float32 [count][kv_head_count*head_dim], TSLAttention.ts:120):
 * keyCacheAttribute / valueCacheAttribute. Synchronises. NULL outputs skip. */
int tla_cache_read(const tla_layer* layer, int32_t seq, int32_t token_begin, int32_t count, float* key_out,
                   float* value_out);
/* Inverse of tla_cache_read: host float32 token-major rows into the cache. */
int tla_cache_write(tla_layer* layer, int32_t seq, int32_t token_begin, int32_t count, const float* key,
                    const float* value);

/* Allocation-free decode. No counterpart in the reference: this entry point
 * serves hosts that cannot call cudaMalloc - hosts whose device memory is all
 * owned by their own pool or a fixed budget, and serving loops that must not
 * take cudaMalloc's implicit device-wide synchronisation - so it needs no
 * tla_ctx or tla_layer and allocates nothing.
 *
 * It runs the same decode step as tla_decode on the calling thread's current
 * device, with the caller's buffers: config as for tla_layer_create (fp16
 * cache, head_dim 64 or 128, head_count a multiple of kv_head_count with a
 * ratio of at most 16, max_batch <= 1024); key_cache / value_cache laid out
 * [max_batch][kv_head_count][max_tokens][head_dim] (the new token is appended
 * there); q_norm_weight / k_norm_weight device float32 [head_dim] or NULL;
 * qkv, positions, gate, out as for tla_decode; status a device int32 that
 * receives device-detected errors (TLA_ERR_POSITION, TLA_ERR_TIMEOUT) or NULL.
 *
 * Its scratch (split-KV partial results, completion counters, the RoPE table)
 * is one static 8 MiB device array in the library, which every GPU that loads
 * the library holds until the process exits. batch * kv_head_count may not
 * exceed 16384 (TLA_ERR_SCRATCH_LIMIT otherwise). The first call on a device
 * looks up that array's device address, so make that first call before any
 * stream capture. Every call shares the array and keeps the last call's
 * contents; calls whose execution overlaps on the GPU (for example on two
 * streams) race on it and must be serialised by the caller. */
int tla_decode_noalloc(const tla_attn_config* config, void* key_cache, void* value_cache,
                       const float* q_norm_weight, const float* k_norm_weight, const void* qkv,
                       const int32_t* positions, const void* gate, void* out, int32_t* status, int32_t batch,
                       void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TLA_API_H */
