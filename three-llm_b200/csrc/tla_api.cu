// C ABI of the attention path: contexts, layers (the TSLAttention operator
// surface, packages/three-llm/src/tsl/TSLAttention.ts:19-448), argument
// validation and kernel dispatch.
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "tla_device.cuh"
#include "exchange.cuh"
#include "tla_internal.h"

namespace tla {
size_t decode_fast_scratch_floats(const tla_layer* L);

LayerArgs layer_args(const tla_layer* L) {
  LayerArgs a;
  a.k_cache = L->k_cache;
  a.v_cache = L->v_cache;
  a.inv_freq = L->d_inv_freq;
  a.q_norm = L->d_qnorm;
  a.k_norm = L->d_knorm;
  a.error = L->ctx->d_error;
  a.Hq = L->Hq;
  a.Hk = L->Hk;
  a.D = L->D;
  a.G = L->G;
  a.max_tokens = L->max_tokens;
  a.max_batch = L->max_batch;
  a.rotary = L->rotary;
  a.freq_half = L->freq_half;
  a.pair_count = L->pair_count;
  a.sliding = L->sliding;
  a.attn_scale = L->attn_scale;
  a.attn_factor = L->attn_factor;
  a.rms_eps = L->rms_eps;
  a.v_norm = L->v_norm ? 1 : 0;
  a.offset_rms = L->offset_rms ? 1 : 0;
  return a;
}

namespace {
struct SmemLimit {
  int device;
  const void* kernel;
  int bytes;
};
struct Occupancy {
  int device;
  const void* kernel;
  int threads, smem, blocks;
};
std::mutex g_attr_mu;
std::vector<SmemLimit> g_smem_limits;
std::vector<Occupancy> g_occupancy;
}  // namespace

cudaError_t raise_smem_limit(const void* kernel, int bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(g_attr_mu);
  for (SmemLimit& s : g_smem_limits) {
    if (s.device != dev || s.kernel != kernel) continue;
    if (bytes <= s.bytes) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) s.bytes = bytes;
    return e;
  }
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) g_smem_limits.push_back({dev, kernel, bytes});
  return e;
}

cudaError_t ensure_proj_workspace(tla_ctx* ctx, size_t floats, size_t tiles) {
  if (floats <= ctx->proj_ws_floats && tiles <= ctx->proj_cnt_count) return cudaSuccess;
  cudaError_t e = cudaSuccess;
  if (floats > ctx->proj_ws_floats) {
    cudaFree(ctx->d_proj_ws);
    ctx->d_proj_ws = nullptr;
    ctx->proj_ws_floats = 0;
    e = cudaMalloc(&ctx->d_proj_ws, floats * sizeof(float));
    if (e == cudaSuccess) e = cudaMemset(ctx->d_proj_ws, 0, floats * sizeof(float));
    if (e != cudaSuccess) return e;
    ctx->proj_ws_floats = floats;
  }
  if (tiles > ctx->proj_cnt_count) {
    cudaFree(ctx->d_proj_cnt);
    ctx->d_proj_cnt = nullptr;
    ctx->proj_cnt_count = 0;
    e = cudaMalloc(&ctx->d_proj_cnt, tiles * sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(ctx->d_proj_cnt, 0, tiles * sizeof(int));
    if (e != cudaSuccess) return e;
    ctx->proj_cnt_count = tiles;
  }
  return cudaSuccess;
}

cudaError_t cached_occupancy(const void* kernel, int threads, int smem, int* blocks) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(g_attr_mu);
  for (const Occupancy& o : g_occupancy)
    if (o.device == dev && o.kernel == kernel && o.threads == threads && o.smem == smem) {
      *blocks = o.blocks;
      return cudaSuccess;
    }
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, kernel, threads, smem);
  if (e == cudaSuccess) g_occupancy.push_back({dev, kernel, threads, smem, *blocks});
  return e;
}
}  // namespace tla

namespace {

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

int from_cuda(cudaError_t e) {
  if (e == cudaSuccess) return TLA_OK;
  if (getenv("TLA_DEBUG")) fprintf(stderr, "tla: CUDA error %d: %s\n", static_cast<int>(e), cudaGetErrorString(e));
  if (e == cudaErrorMemoryAllocation) return TLA_ERR_OUT_OF_MEMORY;
  return TLA_ERR_CUDA;
}

// ropeParameters, packages/three-llm/src/runtime/rope.ts:4-52: double
// arithmetic, float32 table.
int rope_parameters(int32_t dim, double theta, const tla_rope_scaling* scaling, float* inv_freq, double* af_out) {
  if (dim < 0 || dim % 2 != 0) return TLA_ERR_ROPE_DIM;
  if (!isfinite(theta) || theta <= 1) return TLA_ERR_ROPE_THETA;
  const tla_rope_scaling* s = (scaling && scaling->type != TLA_ROPE_NONE) ? scaling : nullptr;
  const bool yarn = s && s->type == TLA_ROPE_YARN;
  double af = 1, low = 0, high = 0;
  if (s && (!isfinite(s->factor) || s->factor < 1)) return TLA_ERR_ROPE_FACTOR;
  if (yarn) {
    if (!isfinite(s->original_context_length) || !isfinite(s->beta_fast) || !isfinite(s->beta_slow))
      return TLA_ERR_YARN_RANGE;
    if (!(s->original_context_length > 0 && s->beta_fast > 0 && s->beta_slow > 0 && s->beta_fast >= s->beta_slow))
      return TLA_ERR_YARN_RANGE;
    af = s->has_attention_factor ? s->attention_factor : 1 + 0.1 * log(s->factor);
    if (!isfinite(af) || af <= 0) return TLA_ERR_YARN_FACTOR;
    auto correction = [&](double rotations) {
      return (dim * log(s->original_context_length / (rotations * 2 * M_PI))) / (2 * log(theta));
    };
    low = fmax(0, floor(correction(s->beta_fast)));
    high = fmin(dim - 1, ceil(correction(s->beta_slow)));
    if (low == high) high += 0.001;
  }
  for (int32_t i = 0; i < dim / 2; ++i) {
    double f = 1 / pow(theta, (2.0 * i) / dim);
    if (s && s->type == TLA_ROPE_LINEAR) f /= s->factor;
    if (yarn) {
      const double ramp = fmin(1, fmax(0, (i - low) / (high - low)));
      f *= 1 - ramp + ramp / s->factor;
    }
    if (s && s->type == TLA_ROPE_LLAMA3) {
      const double ocl = s->original_context_length, lf = s->low_freq_factor, hf = s->high_freq_factor;
      if (!isfinite(ocl) || !isfinite(lf) || !isfinite(hf) || !(ocl > 0 && lf > 0 && hf > lf))
        return TLA_ERR_LLAMA3_RANGE;
      const double wavelength = (2 * M_PI) / f;
      if (wavelength > ocl / lf) {
        f /= s->factor;
      } else if (wavelength >= ocl / hf) {
        const double smooth = (ocl / wavelength - lf) / (hf - lf);
        f *= (1 - smooth) / s->factor + smooth;
      }
    }
    if (inv_freq) inv_freq[i] = static_cast<float>(f);
  }
  if (af_out) *af_out = af;
  return TLA_OK;
}

template <typename T>
int dev_alloc(T** p, size_t count) {
  *p = nullptr;
  if (count == 0) return TLA_OK;
  return from_cuda(cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T)));
}

int ensure_qscratch(tla_ctx* ctx, size_t bytes) {
  if (bytes <= ctx->qscratch_bytes) return TLA_OK;
  if (ctx->d_qscratch) cudaFree(ctx->d_qscratch);
  ctx->d_qscratch = nullptr;
  ctx->qscratch_bytes = 0;
  cudaError_t e = cudaMalloc(&ctx->d_qscratch, bytes);
  if (e != cudaSuccess) return from_cuda(e);
  ctx->qscratch_bytes = bytes;
  return TLA_OK;
}

bool valid_layer(const tla_layer* L) { return L && L->ctx && L->k_cache && L->v_cache; }

}  // namespace

extern "C" {

const char* tla_status_string(int status) {
  switch (status) {
    case TLA_OK: return "ok";
    case TLA_ERR_INVALID_ARG: return "invalid argument";
    case TLA_ERR_ROPE_DIM: return "RoPE dimension must be a non-negative even integer.";
    case TLA_ERR_ROPE_THETA: return "RoPE theta must be finite and greater than one.";
    case TLA_ERR_ROPE_FACTOR: return "RoPE scaling factor must be finite and at least one.";
    case TLA_ERR_YARN_RANGE: return "Invalid YaRN context or beta range.";
    case TLA_ERR_YARN_FACTOR: return "Invalid YaRN attention factor.";
    case TLA_ERR_LLAMA3_RANGE: return "Invalid Llama 3 RoPE frequency range.";
    case TLA_ERR_ROTARY_DIM: return "Invalid rotary dimension: expected an even integer within the head dimension.";
    case TLA_ERR_UNSUPPORTED: return "unsupported attention shape";
    case TLA_ERR_CUDA: return "CUDA runtime error";
    case TLA_ERR_OUT_OF_MEMORY: return "out of device memory";
    case TLA_ERR_POSITION: return "position outside the KV cache";
    case TLA_ERR_TIMEOUT: return "in-kernel wait timed out";
    case TLA_ERR_NO_DEVICE: return "no CUDA device";
    case TLA_ERR_SHARED: return "layer borrows another layer's cache";
    case TLA_ERR_SCRATCH_LIMIT: return "request exceeds the fixed scratch of the allocation-free decode";
    case TLA_ERR_BOUNDS: return "index outside its buffer (bounds-check build)";
    default: return "unknown status";
  }
}

int tla_rope_parameters(int32_t dim, double theta, const tla_rope_scaling* scaling, float* inv_freq,
                        double* attention_factor) {
  return rope_parameters(dim, theta, scaling, inv_freq, attention_factor);
}

int tla_create(int device, tla_ctx** out) {
  if (!out) return TLA_ERR_INVALID_ARG;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return TLA_ERR_NO_DEVICE;
  if (device < 0 || device >= n) return TLA_ERR_INVALID_ARG;
  DeviceGuard g(device);
  tla_ctx* ctx = new tla_ctx();
  ctx->device = device;
  cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device);
  int rc = dev_alloc(&ctx->d_error, 1);
  if (rc == TLA_OK) rc = from_cuda(cudaMemset(ctx->d_error, 0, sizeof(int)));
  if (rc != TLA_OK) {
    tla_destroy(ctx);
    return rc;
  }
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    ctx->encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  *out = ctx;
  return TLA_OK;
}

int tla_destroy(tla_ctx* ctx) {
  if (!ctx) return TLA_OK;
  DeviceGuard g(ctx->device);
  cudaFree(ctx->d_error);
  cudaFree(ctx->d_partials);
  cudaFree(ctx->d_counters);
  cudaFree(ctx->d_qscratch);
  cudaFree(ctx->d_proj_ws);
  cudaFree(ctx->d_proj_cnt);
  delete ctx;
  return TLA_OK;
}

int tla_get_error(tla_ctx* ctx, int reset) {
  if (!ctx) return TLA_ERR_INVALID_ARG;
  DeviceGuard g(ctx->device);
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return from_cuda(e);
  int v = 0;
  e = cudaMemcpy(&v, ctx->d_error, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return from_cuda(e);
  if (reset) {
    e = cudaMemset(ctx->d_error, 0, sizeof(int));
    // A launch that reported an error may have ended before the CTA that
    // completes a split (sequence, kv head) pair zeroed that pair's counter;
    // the next launch's tickets need every counter at zero.
    if (e == cudaSuccess && v != 0 && ctx->d_counters)
      e = cudaMemset(ctx->d_counters, 0, ctx->counter_count * sizeof(int32_t));
    if (e == cudaSuccess && v != 0 && ctx->d_proj_ws)
      e = cudaMemset(ctx->d_proj_ws, 0, ctx->proj_ws_floats * sizeof(float));
    if (e == cudaSuccess && v != 0 && ctx->d_proj_cnt)
      e = cudaMemset(ctx->d_proj_cnt, 0, ctx->proj_cnt_count * sizeof(int));
    if (e != cudaSuccess) return from_cuda(e);
  }
  return v;
}

int tla_layer_create(tla_ctx* ctx, const tla_attn_config* cfg, const float* q_norm_weight, const float* k_norm_weight,
                     tla_layer** out) {
  if (!ctx || !cfg || !out) return TLA_ERR_INVALID_ARG;
  *out = nullptr;
  const int Hq = cfg->head_count, D = cfg->head_dim;
  const int Hk = cfg->kv_head_count > 0 ? cfg->kv_head_count : Hq;
  if (Hq <= 0 || D <= 0 || Hk > Hq || cfg->max_tokens <= 0 || cfg->max_batch <= 0 || cfg->sliding_window < 0)
    return TLA_ERR_INVALID_ARG;
  if (D > 256) return TLA_ERR_UNSUPPORTED;
  const int rotary = cfg->rotary_dim < 0 ? D : cfg->rotary_dim;
  if (rotary % 2 != 0 || rotary > D) return TLA_ERR_ROTARY_DIM;  // load/DecoderRecipe.ts:409-415
  const bool rope_on = cfg->rope_theta > 0 && rotary > 0;       // math.ts:217, TSLAttention.ts:84-87
  const int freq_dim = cfg->rope_freq_dim > 0 ? cfg->rope_freq_dim : rotary;
  const int pair_count = cfg->rope_pair_count >= 0 ? cfg->rope_pair_count : rotary / 2;
  std::vector<float> inv(static_cast<size_t>(freq_dim / 2) + 1, 0.f);
  double af = 1;
  if (rope_on) {
    int rc = rope_parameters(freq_dim, cfg->rope_theta, &cfg->rope_scaling, inv.data(), &af);
    if (rc != TLA_OK) return rc;
    // invFreq[k] past the table would be undefined (NaN) in the reference.
    if (pair_count > freq_dim / 2) return TLA_ERR_INVALID_ARG;
  }
  DeviceGuard g(ctx->device);
  tla_layer* L = new tla_layer();
  L->ctx = ctx;
  L->cfg = *cfg;
  L->Hq = Hq;
  L->Hk = Hk;
  L->D = D;
  L->G = (Hq % Hk == 0) ? Hq / Hk : 0;
  L->max_tokens = cfg->max_tokens;
  L->max_batch = cfg->max_batch;
  L->rotary = rope_on ? rotary : 0;
  L->freq_half = rope_on ? freq_dim / 2 : 0;
  L->pair_count = rope_on ? (pair_count < rotary / 2 ? pair_count : rotary / 2) : 0;
  L->sliding = cfg->sliding_window;
  L->attn_scale = static_cast<float>(cfg->has_attn_scale ? cfg->attn_scale : 1 / sqrt(static_cast<double>(D)));
  L->attn_factor = static_cast<float>(af);
  L->rms_eps = static_cast<float>(cfg->rms_epsilon > 0 ? cfg->rms_epsilon : 1e-6);
  L->io_fp32 = (cfg->flags & TLA_FLAG_IO_FP32) != 0;
  L->cache_fp32 = (cfg->flags & TLA_FLAG_CACHE_FP32) != 0;
  L->v_norm = (cfg->flags & TLA_FLAG_V_NORM) != 0;
  L->offset_rms = (cfg->flags & TLA_FLAG_OFFSET_RMS_NORM) != 0;
  const size_t elems = static_cast<size_t>(L->max_batch) * Hk * L->max_tokens * D;
  const size_t ebytes = L->cache_fp32 ? 4 : 2;
  int rc = from_cuda(cudaMalloc(&L->k_cache, elems * ebytes));
  if (rc == TLA_OK) rc = from_cuda(cudaMalloc(&L->v_cache, elems * ebytes));
  if (rc == TLA_OK) rc = from_cuda(cudaMemset(L->k_cache, 0, elems * ebytes));
  if (rc == TLA_OK) rc = from_cuda(cudaMemset(L->v_cache, 0, elems * ebytes));
  if (rc == TLA_OK) rc = dev_alloc(&L->d_inv_freq, inv.size());
  if (rc == TLA_OK)
    rc = from_cuda(cudaMemcpy(L->d_inv_freq, inv.data(), inv.size() * sizeof(float), cudaMemcpyHostToDevice));
  if (rc == TLA_OK && q_norm_weight) {
    rc = dev_alloc(&L->d_qnorm, D);
    if (rc == TLA_OK) rc = from_cuda(cudaMemcpy(L->d_qnorm, q_norm_weight, D * sizeof(float), cudaMemcpyHostToDevice));
  }
  if (rc == TLA_OK && k_norm_weight) {
    rc = dev_alloc(&L->d_knorm, D);
    if (rc == TLA_OK) rc = from_cuda(cudaMemcpy(L->d_knorm, k_norm_weight, D * sizeof(float), cudaMemcpyHostToDevice));
  }
  L->has_qnorm = q_norm_weight != nullptr;
  L->has_knorm = k_norm_weight != nullptr;
  if (rc == TLA_OK && L->G > 0) rc = from_cuda(tla::decode_fast_configure(L));
  if (rc == TLA_OK && L->fast_decode) {
    const size_t need = tla::decode_fast_scratch_floats(L);
    if (need > ctx->partial_floats) {
      cudaFree(ctx->d_partials);
      ctx->partial_floats = 0;
      rc = dev_alloc(&ctx->d_partials, need);
      if (rc == TLA_OK) ctx->partial_floats = need;
    }
    const size_t counters = static_cast<size_t>(L->max_batch) * Hk;
    if (rc == TLA_OK && counters > ctx->counter_count) {
      cudaFree(ctx->d_counters);
      ctx->counter_count = 0;
      rc = dev_alloc(&ctx->d_counters, counters);
      if (rc == TLA_OK) rc = from_cuda(cudaMemset(ctx->d_counters, 0, counters * sizeof(int32_t)));
      if (rc == TLA_OK) ctx->counter_count = counters;
    }
  }
  if (rc == TLA_OK) rc = from_cuda(tla::prefill_fast_configure(L));
  if (rc != TLA_OK) {
    tla_layer_destroy(L);
    return rc;
  }
  *out = L;
  return TLA_OK;
}

int tla_layer_share_cache(tla_layer* dst, const tla_layer* src) {
  if (!valid_layer(dst) || !valid_layer(src) || dst == src) return TLA_ERR_INVALID_ARG;
  if (dst->Hk != src->Hk || dst->D != src->D || dst->max_tokens != src->max_tokens ||
      dst->max_batch != src->max_batch || dst->cache_fp32 != src->cache_fp32 || dst->ctx != src->ctx)
    return TLA_ERR_INVALID_ARG;
  DeviceGuard g(dst->ctx->device);
  if (!dst->borrowed) {
    cudaFree(dst->k_cache);
    cudaFree(dst->v_cache);
  }
  dst->k_cache = src->k_cache;
  dst->v_cache = src->v_cache;
  dst->borrowed = true;
  dst->tmap_k = src->tmap_k;
  dst->tmap_v = src->tmap_v;
  return TLA_OK;
}

int tla_layer_destroy(tla_layer* L) {
  if (!L) return TLA_OK;
  DeviceGuard g(L->ctx->device);
  if (!L->borrowed) {
    cudaFree(L->k_cache);
    cudaFree(L->v_cache);
  }
  cudaFree(L->d_inv_freq);
  cudaFree(L->d_qnorm);
  cudaFree(L->d_knorm);
  delete L;
  return TLA_OK;
}

int tla_layer_cache_view(const tla_layer* L, tla_cache_view* view) {
  if (!valid_layer(L) || !view) return TLA_ERR_INVALID_ARG;
  view->key = L->k_cache;
  view->value = L->v_cache;
  view->token_stride = L->D;
  view->head_stride = static_cast<int64_t>(L->max_tokens) * L->D;
  view->seq_stride = view->head_stride * L->Hk;
  view->elem_bytes = L->cache_fp32 ? 4 : 2;
  return TLA_OK;
}

int tla_decode(tla_layer* L, const void* qkv, const int32_t* positions, const void* gate, void* out, int32_t batch,
               void* stream) {
  if (!valid_layer(L) || !qkv || !positions || !out || batch < 0 || batch > L->max_batch) return TLA_ERR_INVALID_ARG;
  if (batch == 0) return TLA_OK;
  DeviceGuard g(L->ctx->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int append = L->borrowed ? 0 : 1;
  if (L->fast_decode)
    return from_cuda(tla::launch_decode_fast(L, qkv, positions, gate, out, nullptr, batch, 0, L->max_tokens, append, st));
  int rc = ensure_qscratch(L->ctx, static_cast<size_t>(batch) * L->Hq * L->D * sizeof(float));
  if (rc != TLA_OK) return rc;
  float* qs = static_cast<float*>(L->ctx->d_qscratch);
  rc = from_cuda(tla::launch_rope_append(L, qkv, positions, batch, 1, 0, append, qs, st));
  if (rc != TLA_OK) return rc;
  return from_cuda(tla::launch_attend_generic(L, qs, positions, batch, 1, 0, L->max_tokens, gate, out, nullptr, st));
}

int tla_query(tla_layer* L, const void* qkv, const int32_t* positions, float* query_out, int32_t batch,
              void* stream) {
  if (!valid_layer(L) || !qkv || !positions || !query_out || batch < 0 || batch > L->max_batch)
    return TLA_ERR_INVALID_ARG;
  if (batch == 0) return TLA_OK;
  DeviceGuard g(L->ctx->device);
  return from_cuda(tla::launch_rope_append(L, qkv, positions, batch, 1, 0, 0, query_out,
                                           static_cast<cudaStream_t>(stream)));
}

int tla_scores(tla_layer* L, const float* query, const int32_t* positions, float* scores_out, int32_t batch,
               void* stream) {
  if (!valid_layer(L) || !query || !positions || !scores_out || batch < 0 || batch > L->max_batch)
    return TLA_ERR_INVALID_ARG;
  if (batch == 0) return TLA_OK;
  DeviceGuard g(L->ctx->device);
  return from_cuda(tla::launch_scores(L, query, positions, batch, scores_out, static_cast<cudaStream_t>(stream)));
}

int tla_prefill(tla_layer* L, const void* qkv, const int32_t* start_pos, const void* gate, int32_t seq_len, void* out,
                int32_t batch, void* stream) {
  if (!valid_layer(L) || !qkv || !start_pos || !out || batch < 0 || batch > L->max_batch || seq_len < 0 ||
      seq_len > L->max_tokens)
    return TLA_ERR_INVALID_ARG;
  if (batch == 0 || seq_len == 0) return TLA_OK;
  DeviceGuard g(L->ctx->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (L->fast_prefill && !L->borrowed) {
    int rc = ensure_qscratch(L->ctx, tla::prefill_scratch_bytes(L, batch, seq_len));
    if (rc != TLA_OK) return rc;
    return from_cuda(tla::launch_prefill_fast(L, qkv, start_pos, gate, batch, seq_len, out, st));
  }
  int rc = ensure_qscratch(L->ctx, static_cast<size_t>(batch) * seq_len * L->Hq * L->D * sizeof(float));
  if (rc != TLA_OK) return rc;
  float* qs = static_cast<float*>(L->ctx->d_qscratch);
  rc = from_cuda(tla::launch_rope_append(L, qkv, start_pos, batch, seq_len, 0, L->borrowed ? 0 : 1, qs, st));
  if (rc != TLA_OK) return rc;
  return from_cuda(
      tla::launch_attend_generic(L, qs, start_pos, batch, seq_len, 0, L->max_tokens, gate, out, nullptr, st));
}

int tla_qkv_decode(tla_layer* L, const void* x, const void* weight, const float* bias, int32_t hidden,
                   const int32_t* positions, const void* gate, void* out, int32_t batch, void* stream) {
  if (!valid_layer(L) || !x || !weight || !positions || !out || batch < 0 || batch > L->max_batch || hidden <= 0 ||
      hidden % 8 != 0)
    return TLA_ERR_INVALID_ARG;
  if (!L->fast_decode || L->io_fp32 || L->cache_fp32) return TLA_ERR_UNSUPPORTED;
  if (L->borrowed) return TLA_ERR_SHARED;
  if (batch == 0) return TLA_OK;
  DeviceGuard g(L->ctx->device);
  int rc = ensure_qscratch(L->ctx, static_cast<size_t>(batch) * L->Hq * L->D * sizeof(__half));
  if (rc != TLA_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  __half* q = static_cast<__half*>(L->ctx->d_qscratch);
  rc = from_cuda(tla::launch_qkv_proj(L, x, weight, bias, hidden, positions, batch, 1, false, q, st));
  if (rc != TLA_OK) return rc;
  return from_cuda(tla::launch_decode_fast_qrot(L, q, positions, gate, out, batch, st));
}

int tla_qkv_prefill(tla_layer* L, const void* x, const void* weight, const float* bias, int32_t hidden,
                    const int32_t* start_pos, const void* gate, int32_t seq_len, void* out, int32_t batch,
                    void* stream) {
  if (!valid_layer(L) || !x || !weight || !start_pos || !out || batch < 0 || batch > L->max_batch || seq_len < 0 ||
      seq_len > L->max_tokens || hidden <= 0 || hidden % 8 != 0)
    return TLA_ERR_INVALID_ARG;
  if (!L->fast_prefill || L->io_fp32 || L->cache_fp32) return TLA_ERR_UNSUPPORTED;
  if (L->borrowed) return TLA_ERR_SHARED;
  if (batch == 0 || seq_len == 0) return TLA_OK;
  DeviceGuard g(L->ctx->device);
  int rc = ensure_qscratch(L->ctx, tla::prefill_scratch_bytes(L, batch, seq_len));
  if (rc != TLA_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  __half* q = static_cast<__half*>(L->ctx->d_qscratch);
  rc = from_cuda(tla::launch_qkv_proj(L, x, weight, bias, hidden, start_pos, batch * seq_len, seq_len, true, q, st));
  if (rc != TLA_OK) return rc;
  return from_cuda(tla::launch_prefill_attention(L, start_pos, gate, batch, seq_len, out, st));
}

int tla_out_proj(tla_ctx* ctx, const void* attn, const void* weight, const float* bias, const void* residual, void* y,
                 int32_t rows, int32_t in_features, int32_t hidden, uint32_t io_flags, void* stream) {
  if (!ctx || !attn || !weight || !y || rows < 0 || in_features <= 0 || hidden <= 0 || in_features % 64 != 0 ||
      hidden % 64 != 0)
    return TLA_ERR_INVALID_ARG;
  if (ctx->encode_tiled == nullptr) return TLA_ERR_UNSUPPORTED;
  if (rows == 0) return TLA_OK;
  DeviceGuard g(ctx->device);
  const bool f32 = (io_flags & TLA_FLAG_IO_FP32) != 0;
  return from_cuda(tla::launch_out_proj(ctx, attn, weight, bias, residual, f32, y, f32, rows, in_features, hidden,
                                        static_cast<cudaStream_t>(stream)));
}

int tla_decode_partial(tla_layer* L, const void* qkv, const int32_t* positions, int32_t slot_offset,
                       int32_t local_tokens, int32_t append, float* partial, int32_t batch, void* stream) {
  if (!valid_layer(L) || !qkv || !positions || !partial || batch < 0 || batch > L->max_batch || slot_offset < 0 ||
      local_tokens < 0 || local_tokens > L->max_tokens)
    return TLA_ERR_INVALID_ARG;
  if (append && L->borrowed) return TLA_ERR_SHARED;
  if (batch == 0) return TLA_OK;
  DeviceGuard g(L->ctx->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (L->fast_decode)
    return from_cuda(tla::launch_decode_fast(L, qkv, positions, nullptr, nullptr, partial, batch, slot_offset,
                                             local_tokens, append ? 1 : 0, st));
  int rc = ensure_qscratch(L->ctx, static_cast<size_t>(batch) * L->Hq * L->D * sizeof(float));
  if (rc != TLA_OK) return rc;
  float* qs = static_cast<float*>(L->ctx->d_qscratch);
  rc = from_cuda(tla::launch_rope_append(L, qkv, positions, batch, 1, slot_offset, append ? 1 : 0, qs, st));
  if (rc != TLA_OK) return rc;
  return from_cuda(tla::launch_attend_generic(L, qs, positions, batch, 1, slot_offset, local_tokens, nullptr, nullptr,
                                              partial, st));
}

int tla_decode_exchange(tla_layer* L, tla_exchange* ex, const void* qkv, const int32_t* positions, int32_t slot_offset,
                        int32_t local_tokens, int32_t append, float* partial, const void* gate, void* out, int32_t batch,
                        void* stream) {
  if (!valid_layer(L) || !ex || !qkv || !positions || !partial || !out || batch < 0 || batch > L->max_batch ||
      slot_offset < 0 || local_tokens < 0 || local_tokens > L->max_tokens)
    return TLA_ERR_INVALID_ARG;
  if (append && L->borrowed) return TLA_ERR_SHARED;
  if (batch == 0) return TLA_OK;
  const size_t need = static_cast<size_t>(batch) * L->Hq * (L->D + 2) * sizeof(float);
  if (need > tla::exchange_slot_bytes(ex)) return TLA_ERR_INVALID_ARG;
  if (!L->fast_decode) {  // generic shapes: the partial kernel, then the exchange kernel
    int rc = tla_decode_partial(L, qkv, positions, slot_offset, local_tokens, append, partial, batch, stream);
    if (rc != TLA_OK) return rc;
    return tla_exchange_combine(ex, partial, batch, L->Hq, L->D, gate, out, L->io_fp32 ? TLA_FLAG_IO_FP32 : 0u,
                                stream);
  }
  tla::ExchangeDev x;
  if (!tla::exchange_device_view(ex, &x)) return TLA_ERR_INVALID_ARG;
  DeviceGuard g(L->ctx->device);
  return from_cuda(tla::launch_decode_exchange(L, x, qkv, positions, gate, out, partial, batch, slot_offset,
                                               local_tokens, append ? 1 : 0, static_cast<cudaStream_t>(stream)));
}

int tla_combine_lse(const float* partials, int32_t ranks, int32_t batch, int32_t head_count, int32_t head_dim,
                    const void* gate, void* out, uint32_t io_flags, void* stream) {
  if (!partials || !out || ranks <= 0 || batch < 0 || head_count <= 0 || head_dim <= 0) return TLA_ERR_INVALID_ARG;
  return from_cuda(tla::launch_combine_lse(partials, ranks, batch, head_count, head_dim, gate, out,
                                           (io_flags & TLA_FLAG_IO_FP32) != 0, static_cast<cudaStream_t>(stream)));
}

int tla_cache_reset(tla_layer* L, void* stream) {
  if (!valid_layer(L)) return TLA_ERR_INVALID_ARG;
  if (L->borrowed) return TLA_OK;  // TSLAttention.ts:435
  DeviceGuard g(L->ctx->device);
  const size_t bytes =
      static_cast<size_t>(L->max_batch) * L->Hk * L->max_tokens * L->D * (L->cache_fp32 ? 4 : 2);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = from_cuda(cudaMemsetAsync(L->k_cache, 0, bytes, st));
  if (rc == TLA_OK) rc = from_cuda(cudaMemsetAsync(L->v_cache, 0, bytes, st));
  return rc;
}

static int cache_copy(const tla_layer* L, int32_t seq, int32_t begin, int32_t count, float* k_host, float* v_host,
                      const float* k_in, const float* v_in) {
  if (!valid_layer(L) || seq < 0 || seq >= L->max_batch || begin < 0 || count < 0 ||
      static_cast<int64_t>(begin) + count > L->max_tokens)
    return TLA_ERR_INVALID_ARG;
  DeviceGuard g(L->ctx->device);
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return from_cuda(e);
  const int D = L->D, Hk = L->Hk;
  const size_t eb = L->cache_fp32 ? 4 : 2;
  std::vector<uint8_t> buf(static_cast<size_t>(count) * D * eb);
  for (int which = 0; which < 2; ++which) {
    float* host_out = which == 0 ? k_host : v_host;
    const float* host_in = which == 0 ? k_in : v_in;
    if (!host_out && !host_in) continue;
    uint8_t* base = static_cast<uint8_t*>(which == 0 ? L->k_cache : L->v_cache);
    for (int kh = 0; kh < Hk; ++kh) {
      uint8_t* dev = base + ((static_cast<size_t>(seq) * Hk + kh) * L->max_tokens + begin) * D * eb;
      if (host_out) {
        e = cudaMemcpy(buf.data(), dev, buf.size(), cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) return from_cuda(e);
        for (int t = 0; t < count; ++t)
          for (int d = 0; d < D; ++d) {
            const size_t i = static_cast<size_t>(t) * D + d;
            const float v = eb == 4 ? reinterpret_cast<float*>(buf.data())[i]
                                    : __half2float(reinterpret_cast<__half*>(buf.data())[i]);
            host_out[(static_cast<size_t>(t) * Hk + kh) * D + d] = v;
          }
      } else {
        for (int t = 0; t < count; ++t)
          for (int d = 0; d < D; ++d) {
            const size_t i = static_cast<size_t>(t) * D + d;
            const float v = host_in[(static_cast<size_t>(t) * Hk + kh) * D + d];
            if (eb == 4)
              reinterpret_cast<float*>(buf.data())[i] = v;
            else
              reinterpret_cast<__half*>(buf.data())[i] = __float2half_rn(v);
          }
        e = cudaMemcpy(dev, buf.data(), buf.size(), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return from_cuda(e);
      }
    }
  }
  return TLA_OK;
}

int tla_cache_read(const tla_layer* L, int32_t seq, int32_t token_begin, int32_t count, float* key_out,
                   float* value_out) {
  return cache_copy(L, seq, token_begin, count, key_out, value_out, nullptr, nullptr);
}

int tla_cache_write(tla_layer* L, int32_t seq, int32_t token_begin, int32_t count, const float* key,
                    const float* value) {
  if (L && L->borrowed) return TLA_ERR_SHARED;
  return cache_copy(L, seq, token_begin, count, nullptr, nullptr, key, value);
}

}  // extern "C"
