// Host-side state and kernel entry points shared by the translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "tla_api.h"

struct tla_ctx {
  int device = 0;
  int sm_count = 0;
  int* d_error = nullptr;  // sticky device error word (first error wins)
  // split-KV scratch: partial triples of the persistent decode kernel and the
  // per-(sequence, kv head) completion counters (zero between launches)
  float* d_partials = nullptr;
  size_t partial_floats = 0;
  int32_t* d_counters = nullptr;
  size_t counter_count = 0;
  // prefill / generic-path query scratch (rotated queries)
  void* d_qscratch = nullptr;
  size_t qscratch_bytes = 0;
  // split-K projection workspace: fp32 partial sums and per-tile tickets,
  // zero between launches
  float* d_proj_ws = nullptr;
  size_t proj_ws_floats = 0;
  int* d_proj_cnt = nullptr;
  size_t proj_cnt_count = 0;
  PFN_cuTensorMapEncodeTiled_v12000 encode_tiled = nullptr;
};

struct tla_layer {
  tla_ctx* ctx = nullptr;
  tla_attn_config cfg{};
  int Hq = 0, Hk = 0, D = 0, G = 0;
  int max_tokens = 0, max_batch = 0;
  int rotary = 0, freq_half = 0, pair_count = 0, sliding = 0;
  float attn_scale = 0.f, attn_factor = 1.f, rms_eps = 1e-6f;
  bool io_fp32 = false, cache_fp32 = false, v_norm = false, offset_rms = false;
  bool has_qnorm = false, has_knorm = false;
  bool borrowed = false;        // sharedAttention: cache belongs to another layer
  void* k_cache = nullptr;
  void* v_cache = nullptr;
  float* d_inv_freq = nullptr;  // [max(freq_half, 1)]
  float* d_qnorm = nullptr;     // [D] or null
  float* d_knorm = nullptr;     // [D] or null
  // fast decode path (fp16 cache, D in {64, 128}, G <= 16)
  bool fast_decode = false;
  int decode_grid = 0;          // persistent CTAs per launch
  size_t decode_smem = 0;
  CUtensorMap tmap_k{}, tmap_v{};
  // tensor-core prefill path (cache maps with 128-token boxes)
  bool fast_prefill = false;
  size_t prefill_smem = 0;
  CUtensorMap tmap_k128{}, tmap_v128{};  // 128-token boxes
};

namespace tla {

// Launch with programmatic dependent launch allowed: the kernel may start
// while the previous kernel in the stream finishes; it waits (griddep_wait)
// before touching anything that kernel produces.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), unsigned grid, unsigned block, size_t smem, cudaStream_t stream,
                       Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}


// Parameters shared by all decode / prefill kernels of one layer.
struct LayerArgs {
  void* k_cache;
  void* v_cache;
  const float* inv_freq;
  const float* q_norm;  // null => none
  const float* k_norm;  // null => none
  int* error;
  int Hq, Hk, D, G;
  int max_tokens, max_batch;
  int rotary, freq_half, pair_count, sliding;
  float attn_scale, attn_factor, rms_eps;
  int v_norm, offset_rms;
};

LayerArgs layer_args(const tla_layer* L);

// cudaFuncAttributeMaxDynamicSharedMemorySize is a property of a kernel
// instance on the current device, shared by every layer that launches it:
// raise it to `bytes` if it is lower, never lower it.
cudaError_t raise_smem_limit(const void* kernel, int bytes);
// Resident blocks per SM of a kernel instance at (threads, dynamic smem) on
// the current device, cached per (device, kernel, threads, smem).
cudaError_t cached_occupancy(const void* kernel, int threads, int smem, int* blocks);

// Generic path (any head_dim <= 256, any GQA ratio, fp16 or fp32 cache).
// rope_append: per (b, t) token at pos = start[b] + t: QK-norm + RoPE of Q into
// qscr (float32 [B][S][Hq][D]); if append, K (norm + RoPE) and V (vNorm) into
// cache slot pos - slot_offset.
cudaError_t launch_rope_append(const tla_layer* L, const void* qkv, const int32_t* start, int batch, int seq_len,
                               int slot_offset, int append, float* qscr, cudaStream_t stream);
// attend: output or partial triples for each (b, t, h) query over cache slots
// [max(window start, slot_offset), min(pos, slot_offset + local_tokens - 1)] - slot_offset.
cudaError_t launch_attend_generic(const tla_layer* L, const float* qscr, const int32_t* start, int batch,
                                  int seq_len, int slot_offset, int local_tokens, const void* gate, void* out,
                                  float* partial, cudaStream_t stream);
// scaled scores of one decode step: scores[b][h][t] for t in [window start, pos[b]].
cudaError_t launch_scores(const tla_layer* L, const float* query, const int32_t* positions, int batch, float* scores,
                          cudaStream_t stream);
// rope_append with the rotated queries written as fp16 [B][Hq][S][D] (fp16 cache only).
cudaError_t launch_rope_append_half_q(const tla_layer* L, const void* qkv, const int32_t* start, int batch,
                                      int seq_len, __half* qscr, cudaStream_t stream);
// Fast persistent split-KV decode (TMA + tensor-core tiles); partial != null
// switches to partial-triple output (sequence sharding).
cudaError_t launch_decode_fast(const tla_layer* L, const void* qkv, const int32_t* positions, const void* gate,
                               void* out, float* partial, int batch, int slot_offset, int local_tokens, int append,
                               cudaStream_t stream);
// Peer exchange (exchange.cu / exchange.cuh): device view of a connected exchange.
struct ExchangeDev;
bool exchange_device_view(const tla_exchange* ex, ExchangeDev* out);
size_t exchange_slot_bytes(const tla_exchange* ex);
// Sequence-shard decode fused with the exchange: the split-KV kernel writes
// this rank's segments (partial: [B][Hq][D+2] for pairs held by one CTA), then
// one kernel merges each query row's segments, exchanges the row's triple with
// every rank and writes the merged output.
cudaError_t launch_decode_exchange(const tla_layer* L, const ExchangeDev& x, const void* qkv,
                                   const int32_t* positions, const void* gate, void* out, float* partial, int batch,
                                   int slot_offset, int local_tokens, int append, cudaStream_t stream);
cudaError_t decode_fast_configure(tla_layer* L);
cudaError_t launch_combine_lse(const float* partials, int ranks, int batch, int Hq, int D, const void* gate,
                               void* out, bool io_fp32, cudaStream_t stream);
// Tensor-core prefill (tcgen05/TMEM/TMA), fp16 cache, D in {64, 128}.
cudaError_t prefill_fast_configure(tla_layer* L);
// gate: null or [batch][seq_len][Hq][D] in the layer's I/O type.
cudaError_t launch_prefill_fast(const tla_layer* L, const void* qkv, const int32_t* start, const void* gate, int batch,
                                int seq_len, void* out, cudaStream_t stream);

// The causal attention kernel alone, over rotated queries already in the
// context's query scratch ([B][Hq][S][D] fp16) and K/V already appended.
// Query scratch bytes the tensor-core prefill of a chunk needs: the rotated
// queries [B][Hq][S][D] fp16 (rounded up to 256 bytes), then, when the chunk
// is split into KV-range pieces, their partial rows.
size_t prefill_scratch_bytes(const tla_layer* L, int batch, int seq_len);
cudaError_t launch_prefill_attention(const tla_layer* L, const int32_t* start, const void* gate, int batch,
                                     int seq_len, void* out, cudaStream_t stream);
// Decode over rotated queries [B][Hq][D] fp16 whose new K/V rows are already
// in the cache (the fused QKV projection's output).
cudaError_t launch_decode_fast_qrot(const tla_layer* L, const __half* qrot, const int32_t* positions,
                                    const void* gate, void* out, int batch, cudaStream_t stream);
// Grows the context's split-K workspace (zeroed) to at least the given size.
cudaError_t ensure_proj_workspace(tla_ctx* ctx, size_t floats, size_t tiles);
// Tensor-core projections (proj_tc.cu). QKV: x [rows][hidden] fp16 times
// weight [hidden][(Hq+2Hk)D] fp16 (+ bias), epilogue QK-norm / RoPE / append,
// rotated queries to qout. Output projection: y = residual + attn W + bias
// (or the bare product with y float32 and no residual / bias).
cudaError_t launch_qkv_proj(const tla_layer* L, const void* x, const void* weight, const float* bias, int hidden,
                            const int32_t* pos, int rows, int seq_len, bool prefill, __half* qout,
                            cudaStream_t stream);
// Head-sharded output projection: this rank's partial product tiles are stored
// over NVLink into the exchange buffer of the rank owning their columns, then
// one kernel sums the owned block, adds bias + residual and all-gathers.
cudaError_t launch_out_proj_allreduce(tla_ctx* ctx, const ExchangeDev& x, const void* attn,
                                      const void* weight, const float* bias, const void* residual, bool f32, void* y,
                                      int rows, int in_features, int hidden, cudaStream_t stream);
cudaError_t launch_out_proj(tla_ctx* ctx, const void* attn, const void* weight, const float* bias,
                            const void* residual, bool residual_f32, void* y, bool y_f32, int rows, int in_features,
                            int hidden, cudaStream_t stream);

}  // namespace tla
