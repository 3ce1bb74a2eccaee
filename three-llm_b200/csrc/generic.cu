// Generic attention path: any head_dim <= 256, any GQA ratio, fp16 or fp32
// cache. Used for shapes the tensor-core kernels do not cover (the reference's
// own test shapes use head_dim 2, 4 and 8) and for float32 caches.
//
// rope_append_kernel  <- TSLAttention copy-KV and query kernels
//                        (packages/three-llm/src/tsl/TSLAttention.ts:252-304)
//                        and causalAttention's QK-norm / RoPE / append steps
//                        (packages/three-llm/src/runtime/math.ts:211-238)
// attend_generic_kernel <- scores + softmax/PV kernels (TSLAttention.ts:306-428),
//                        math.ts:242-273, as a single online-softmax pass.
#include <math.h>

#include "tla_device.cuh"
#include "tla_internal.h"

namespace tla {

namespace {

constexpr int kThreads = 128;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float block_reduce_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  v = red[0];
#pragma unroll
  for (int i = 1; i < kThreads / 32; ++i) v = fmaxf(v, red[i]);
  return v;
}

__device__ __forceinline__ float block_reduce_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  v = 0.f;
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) v += red[i];
  return v;
}

// One block per (t, b) token row of qkv.
// QH: rotated queries as fp16 head-major [B][Hq][S][D] (the tensor-core
// prefill's TMA source) instead of float32 [B][S][Hq][D].
template <typename IO, typename CT, bool QH>
__global__ void __launch_bounds__(kThreads) rope_append_kernel(LayerArgs a, const IO* __restrict__ qkv,
                                                               const int32_t* __restrict__ start, int seq_len,
                                                               int slot_offset, int append, void* __restrict__ qscr) {
  extern __shared__ float smem[];
  const int t = blockIdx.x, b = blockIdx.y;
  const int D = a.D, Hq = a.Hq, Hk = a.Hk;
  const int heads = Hq + 2 * Hk;
  const int pos = start[b] + t;
  const int slot = pos - slot_offset;
  if (pos < 0 || (append && (slot < 0 || slot >= a.max_tokens))) {
    if (threadIdx.x == 0) report_error(a.error, TLA_ERR_POSITION);
    return;
  }
  float* x = smem;                       // [heads * D]
  float* cs = smem + heads * D;          // [rotary/2] cos
  float* sn = cs + (a.rotary / 2 + 1);   // [rotary/2] sin
  float* red = sn + (a.rotary / 2 + 1);  // [4]
  (void)red;
  const IO* row = qkv + (static_cast<size_t>(b) * seq_len + t) * heads * D;
  const int nload = (append ? heads : Hq) * D;
  for (int i = threadIdx.x; i < nload; i += kThreads) x[i] = to_f32(row[i]);
  const int half = a.rotary / 2;
  for (int j = threadIdx.x; j < half; j += kThreads) {
    float c = 1.f, s = 0.f;
    if (j < a.pair_count) rope_cos_sin(pos, a.inv_freq[j], &c, &s);
    cs[j] = c;
    sn[j] = s;
  }
  __syncthreads();
  // Per-head RMS norms (math.ts:78-97 / :154-167): one warp per head.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int norm_heads = append ? heads : Hq;
  for (int h = warp; h < norm_heads; h += kThreads / 32) {
    const float* w = nullptr;
    bool on = false;
    if (h < Hq) {
      w = a.q_norm;
      on = w != nullptr;
    } else if (h < Hq + Hk) {
      w = a.k_norm;
      on = w != nullptr;
    } else {
      on = a.v_norm != 0;  // weightless
    }
    if (!on) continue;
    float* v = x + h * D;
    float ss = 0.f;
    for (int d = lane; d < D; d += 32) ss += v[d] * v[d];
    ss = warp_sum(ss);
    const float inv_rms = 1.f / sqrtf(ss / static_cast<float>(D) + a.rms_eps);
    __syncwarp();
    for (int d = lane; d < D; d += 32) {
      const float scale = w == nullptr ? 1.f : (a.offset_rms ? 1.f + w[d] : w[d]);
      v[d] = v[d] * inv_rms * scale;
    }
  }
  __syncthreads();
  // RoPE, rotate-half layout (math.ts:134-147) and the stores.
  const int rope_heads = append ? Hq + Hk : Hq;
  for (int i = threadIdx.x; i < rope_heads * D; i += kThreads) {
    const int h = i / D, d = i - h * D;
    const float* v = x + h * D;
    float val = v[d];
    if (half > 0 && d < a.rotary) {
      const int j = d < half ? d : d - half;
      if (j < a.pair_count) {
        const float partner = d < half ? -v[d + half] : v[d - half];
        val = (val * cs[j] + partner * sn[j]) * a.attn_factor;
      }
    }
    if (h < Hq) {
      if (QH)
        static_cast<__half*>(qscr)[((static_cast<size_t>(b) * Hq + h) * seq_len + t) * D + d] = __float2half_rn(val);
      else
        static_cast<float*>(qscr)[((static_cast<size_t>(b) * seq_len + t) * Hq + h) * D + d] = val;
    } else {
      const int kh = h - Hq;
      CT* kc = static_cast<CT*>(a.k_cache);
      const size_t ci = ((static_cast<size_t>(b) * Hk + kh) * a.max_tokens + slot) * D + d;
      if (TLA_IN_BOUNDS(ci, static_cast<long long>(a.max_batch) * Hk * a.max_tokens * D, a.error))
        kc[ci] = from_f32<CT>(val);
    }
  }
  if (append) {
    CT* vc = static_cast<CT*>(a.v_cache);
    for (int i = threadIdx.x; i < Hk * D; i += kThreads) {
      const int kh = i / D, d = i - kh * D;
      const size_t ci = ((static_cast<size_t>(b) * Hk + kh) * a.max_tokens + slot) * D + d;
      if (TLA_IN_BOUNDS(ci, static_cast<long long>(a.max_batch) * Hk * a.max_tokens * D, a.error))
        vc[ci] = from_f32<CT>(x[(Hq + Hk + kh) * D + d]);
    }
  }
}

// One block per (h, t, b) query; online softmax over 128-token chunks.
template <typename CT, typename IO>
__global__ void __launch_bounds__(kThreads)
    attend_generic_kernel(LayerArgs a, const float* __restrict__ qscr, const int32_t* __restrict__ start, int seq_len,
                          int slot_offset, int local_tokens, const IO* __restrict__ gate, IO* __restrict__ out,
                          float* __restrict__ partial) {
  extern __shared__ float smem[];
  const int h = blockIdx.x, t = blockIdx.y, b = blockIdx.z;
  const int D = a.D, Hq = a.Hq, Hk = a.Hk;
  const int pos = start[b] + t;
  if (pos < 0) return;  // reported by rope_append_kernel
  float* q = smem;            // [D]
  float* o = q + D;           // [D]
  float* p = o + D;           // [kThreads]
  float* red = p + kThreads;  // [4]
  const int kvh = static_cast<int>((static_cast<long long>(h) * Hk) / Hq);  // TSLAttention.ts:340
  const size_t qrow = (static_cast<size_t>(b) * seq_len + t) * Hq + h;
  for (int d = threadIdx.x; d < D; d += kThreads) {
    q[d] = qscr[qrow * D + d];
    o[d] = 0.f;
  }
  const int first = a.sliding > 0 ? max(0, pos - a.sliding + 1) : 0;  // math.ts:208
  const int lo = max(first, slot_offset) - slot_offset;
  const int hi = min(pos, slot_offset + local_tokens - 1) - slot_offset;
  const CT* kc = static_cast<const CT*>(a.k_cache) + (static_cast<size_t>(b) * Hk + kvh) * a.max_tokens * D;
  const CT* vc = static_cast<const CT*>(a.v_cache) + (static_cast<size_t>(b) * Hk + kvh) * a.max_tokens * D;
  const float scale = a.attn_scale * kLog2e;
  float m = -INFINITY, l = 0.f;
  __syncthreads();
  for (int c = lo; c <= hi; c += kThreads) {
    const int tok = c + threadIdx.x;
    float s = -INFINITY;
    if (tok <= hi && TLA_IN_BOUNDS(tok, a.max_tokens, a.error)) {
      const CT* kr = kc + static_cast<size_t>(tok) * D;
      float dot = 0.f;
      for (int d = 0; d < D; ++d) dot += q[d] * to_f32(kr[d]);
      s = dot * scale;
    }
    const float m_new = fmaxf(m, block_reduce_max(s, red));
    const float alpha = ex2(m - m_new);
    const float pv = tok <= hi ? ex2(s - m_new) : 0.f;
    p[threadIdx.x] = pv;
    l = l * alpha + block_reduce_sum(pv, red);
    const int n = min(kThreads, hi - c + 1);
    for (int d = threadIdx.x; d < D; d += kThreads) {
      float acc = o[d] * alpha;
      const CT* vr = vc + static_cast<size_t>(c) * D + d;
      for (int j = 0; j < n; ++j) acc += p[j] * to_f32(vr[static_cast<size_t>(j) * D]);
      o[d] = acc;
    }
    m = m_new;
    __syncthreads();
  }
  if (partial) {
    float* pr = partial + qrow * (D + 2);
    if (threadIdx.x == 0) {
      pr[0] = m;
      pr[1] = l;
    }
    for (int d = threadIdx.x; d < D; d += kThreads) pr[2 + d] = o[d];
    return;
  }
  const float inv_l = l > 0.f ? 1.f / l : 0.f;
  for (int d = threadIdx.x; d < D; d += kThreads) {
    float v = o[d] * inv_l;
    if (gate) v = v * (1.f / (1.f + expf(-to_f32(gate[qrow * D + d]))));  // math.ts:271-273
    out[qrow * D + d] = from_f32<IO>(v);
  }
}

template <typename IO, typename CT, bool QH = false>
cudaError_t rope_append_t(const tla_layer* L, const void* qkv, const int32_t* start, int batch, int seq_len,
                          int slot_offset, int append, void* qscr, cudaStream_t stream) {
  const LayerArgs a = layer_args(L);
  const size_t smem = sizeof(float) * (static_cast<size_t>(L->Hq + 2 * L->Hk) * L->D + 2 * (L->rotary / 2 + 1) + 4);
  auto k = rope_append_kernel<IO, CT, QH>;
  if (smem > 48 * 1024) {
    cudaError_t e = raise_smem_limit(reinterpret_cast<const void*>(k), static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  k<<<dim3(seq_len, batch), kThreads, smem, stream>>>(a, static_cast<const IO*>(qkv), start, seq_len, slot_offset,
                                                      append, qscr);
  return cudaGetLastError();
}

template <typename CT, typename IO>
cudaError_t attend_t(const tla_layer* L, const float* qscr, const int32_t* start, int batch, int seq_len,
                     int slot_offset, int local_tokens, const void* gate, void* out, float* partial,
                     cudaStream_t stream) {
  const LayerArgs a = layer_args(L);
  const size_t smem = sizeof(float) * (2 * static_cast<size_t>(L->D) + kThreads + 4);
  attend_generic_kernel<CT, IO><<<dim3(L->Hq, seq_len, batch), kThreads, smem, stream>>>(
      a, qscr, start, seq_len, slot_offset, local_tokens, static_cast<const IO*>(gate), static_cast<IO*>(out),
      partial);
  return cudaGetLastError();
}

}  // namespace

// EPL consecutive elements as floats, with a single vector load.
template <typename IO, int EPL>
__device__ __forceinline__ void load_vec(const IO* p, float (&x)[EPL]) {
  if constexpr (sizeof(IO) == 2 && EPL == 2) {
    const __half2 h = *reinterpret_cast<const __half2*>(p);
    x[0] = __low2float(h);
    x[1] = __high2float(h);
  } else if constexpr (sizeof(IO) == 2 && EPL == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const __half2 a = *reinterpret_cast<const __half2*>(&u.x), b = *reinterpret_cast<const __half2*>(&u.y);
    x[0] = __low2float(a);
    x[1] = __high2float(a);
    x[2] = __low2float(b);
    x[3] = __high2float(b);
  } else if constexpr (EPL == 2) {
    const float2 f = *reinterpret_cast<const float2*>(p);
    x[0] = f.x;
    x[1] = f.y;
  } else {
    const float4 f = *reinterpret_cast<const float4*>(p);
    x[0] = f.x;
    x[1] = f.y;
    x[2] = f.z;
    x[3] = f.w;
  }
}

// Warp-per-token variant for head_dim 64 / 128 and an fp16 cache: lane l holds
// elements [l*EPL, (l+1)*EPL) of every head of the token, head norms are warp
// reductions and the rotate-half partner comes from lane +/- half/EPL.
template <typename IO, int D>
__global__ void __launch_bounds__(128) rope_append_warp_kernel(LayerArgs a, const IO* __restrict__ qkv,
                                                               const int32_t* __restrict__ start, int seq_len,
                                                               int tokens, __half* __restrict__ qscr) {
  constexpr int EPL = D / 32;
  const int lane = threadIdx.x & 31;
  const int ti = blockIdx.x * 4 + (threadIdx.x >> 5);
  if (ti >= tokens) return;
  const int b = ti / seq_len, t = ti - b * seq_len;
  const int Hq = a.Hq, Hk = a.Hk;
  const int pos = start[b] + t;
  if (pos < 0 || pos >= a.max_tokens) {
    if (lane == 0) report_error(a.error, TLA_ERR_POSITION);
    return;
  }
  const int half = a.rotary / 2;
  const int d0 = lane * EPL;
  const bool lo_side = d0 < half;
  const bool rot = half > 0 && d0 < a.rotary;
  const int src = !rot ? lane : (lo_side ? lane + half / EPL : lane - half / EPL);
  float c_[EPL], sn[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    c_[e] = 1.f;
    sn[e] = 0.f;
    const int j = lo_side ? d0 + e : d0 + e - half;
    if (rot && j < a.pair_count) rope_cos_sin(pos, a.inv_freq[j], &c_[e], &sn[e]);
  }
  const int heads = Hq + 2 * Hk;
  const IO* row = qkv + static_cast<size_t>(ti) * heads * D;
  __half* kc = static_cast<__half*>(a.k_cache);
  __half* vc = static_cast<__half*>(a.v_cache);
  constexpr int kChunk = 8;  // heads whose loads are in flight together
  for (int h0 = 0; h0 < heads; h0 += kChunk) {
    float xs[kChunk][EPL];
#pragma unroll
    for (int c = 0; c < kChunk; ++c) {
      if (h0 + c < heads)
        load_vec<IO, EPL>(row + (h0 + c) * D + d0, xs[c]);  // one 4-16 byte load per lane and head
      else
#pragma unroll
        for (int e = 0; e < EPL; ++e) xs[c][e] = 0.f;
    }
#pragma unroll
    for (int c = 0; c < kChunk; ++c) {
      const int hh = h0 + c;
      if (hh >= heads) break;
      float* x = xs[c];
      const float* w = hh < Hq ? a.q_norm : (hh < Hq + Hk ? a.k_norm : nullptr);
      const bool norm = hh < Hq + Hk ? w != nullptr : a.v_norm != 0;
      if (norm) {  // math.ts:78-97
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < EPL; ++e) ss += x[e] * x[e];
        ss = warp_sum(ss);
        const float inv_rms = 1.f / sqrtf(ss / static_cast<float>(D) + a.rms_eps);
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          const float sc = w == nullptr ? 1.f : (a.offset_rms ? 1.f + w[d0 + e] : w[d0 + e]);
          x[e] = x[e] * inv_rms * sc;
        }
      }
      if (hh < Hq + Hk) {  // RoPE, math.ts:134-147
        float y[EPL];
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          const float partner = __shfl_sync(0xffffffffu, x[e], src);
          y[e] = x[e];
          const int j = lo_side ? d0 + e : d0 + e - half;
          if (rot && j < a.pair_count) y[e] = (x[e] * c_[e] + (lo_side ? -partner : partner) * sn[e]) * a.attn_factor;
        }
#pragma unroll
        for (int e = 0; e < EPL; ++e) x[e] = y[e];
      }
      __half hv[EPL];
#pragma unroll
      for (int e = 0; e < EPL; ++e) hv[e] = __float2half_rn(x[e]);
      __half* dst;
      if (hh < Hq)
        dst = qscr + ((static_cast<size_t>(b) * Hq + hh) * seq_len + t) * D + d0;
      else if (hh < Hq + Hk)
        dst = kc + ((static_cast<size_t>(b) * Hk + (hh - Hq)) * a.max_tokens + pos) * D + d0;
      else
        dst = vc + ((static_cast<size_t>(b) * Hk + (hh - Hq - Hk)) * a.max_tokens + pos) * D + d0;
      if constexpr (EPL == 2)
        *reinterpret_cast<__half2*>(dst) = __halves2half2(hv[0], hv[1]);
      else
        *reinterpret_cast<uint2*>(dst) = make_uint2(*reinterpret_cast<uint32_t*>(&hv[0]),
                                                    *reinterpret_cast<uint32_t*>(&hv[2]));
    }
  }
}

// Register budget of rope_rows_kernel: at head_dim 64 at least 6 resident
// 128-thread blocks per SM (80 registers; 5 warp-wide loads per round = 20
// heads, e.g. 14 + 2 + 2), at 128 at least 5 (96 registers; 8 loads = 16
// heads), both without spills. The kernel is issue-bound, so resident warps
// matter more than loads in flight per warp.
template <int D>
constexpr int rope_min_blocks() {
  return D == 64 ? 6 : 5;
}

// fp16 rows, head_dim 64 or 128: a warp per token, each lane owns 16 bytes
// (8 dims) of a head, so one warp-wide load covers 32 / (D / 8) heads and the
// whole qkv row is in flight in a few loads; the rotate-half partner is
// (rotary / 16) lanes away (a power of two: xor shuffle within the head's
// lane group), RMS norms reduce over the group, and cos/sin are computed once
// per token (lane k: pairs k and k + 32) and gathered by shuffles.
template <int D>
__global__ void __launch_bounds__(128, rope_min_blocks<D>()) rope_rows_kernel(LayerArgs a, const __half* __restrict__ qkv,
                                                        const int32_t* __restrict__ start, int seq_len, int tokens,
                                                        __half* __restrict__ qscr) {
  constexpr int L = D / 8;     // lanes per head
  constexpr int HPW = 32 / L;  // heads per warp-wide load
  constexpr int kLoads = D == 64 ? 5 : 8;  // warp-wide loads in flight per round
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const int ti = blockIdx.x * 4 + (threadIdx.x >> 5);
  griddep_wait();  // qkv, start and the cache may come from the previous kernel
  if (ti >= tokens) return;
  const int b = ti / seq_len, t = ti - b * seq_len;
  const int Hq = a.Hq, Hk = a.Hk, heads = Hq + 2 * Hk;
  const int g = lane / L, d0 = 8 * (lane % L);
  const __half* row = qkv + static_cast<size_t>(ti) * heads * D;
  // the first round of loads goes out before the position is known
  uint4 raw[kLoads];
#pragma unroll
  for (int c = 0; c < kLoads; ++c) {
    const int hh = c * HPW + g;
    raw[c] = hh < heads ? *reinterpret_cast<const uint4*>(row + hh * D + d0) : make_uint4(0, 0, 0, 0);
  }
  const int pos = start[b] + t;
  if (pos < 0 || pos >= a.max_tokens) {
    if (lane == 0) report_error(a.error, TLA_ERR_POSITION);
    return;
  }
  const int half = a.rotary / 2, hl = half / 8;
  const bool rot = d0 < a.rotary, lo_side = d0 < half;
  float c0 = 1.f, s0 = 0.f, c1 = 1.f, s1 = 0.f;
  if (lane < a.pair_count && lane < half) rope_cos_sin(pos, a.inv_freq[lane], &c0, &s0);
  if (lane + 32 < a.pair_count && lane + 32 < half) rope_cos_sin(pos, a.inv_freq[lane + 32], &c1, &s1);
  // cos/sin of this lane's 8 dims, with the attention factor folded in
  float cs[8], sn[8];
  bool turn[8];
  const int jb = lo_side ? d0 : d0 - half;
  const bool wide = half > 32;  // pairs 32.. exist (the same for every thread)
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int j = jb + e, src = j & 31;
    float cc = __shfl_sync(full, c0, src), ss = __shfl_sync(full, s0, src);
    if (wide) {
      const float cc1 = __shfl_sync(full, c1, src), ss1 = __shfl_sync(full, s1, src);
      if (j >= 32) {
        cc = cc1;
        ss = ss1;
      }
    }
    turn[e] = rot && j < a.pair_count;
    cs[e] = cc * a.attn_factor;
    sn[e] = ss * a.attn_factor;
  }
  __half* kc = static_cast<__half*>(a.k_cache);
  __half* vc = static_cast<__half*>(a.v_cache);
  const bool any_norm = a.q_norm != nullptr || a.k_norm != nullptr || a.v_norm != 0;
  for (int h0 = 0; h0 < heads; h0 += kLoads * HPW) {
    if (h0 > 0) {
#pragma unroll
      for (int c = 0; c < kLoads; ++c) {
        const int hh = h0 + c * HPW + g;
        raw[c] = hh < heads ? *reinterpret_cast<const uint4*>(row + hh * D + d0) : make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int c = 0; c < kLoads; ++c) {
      if (h0 + c * HPW >= heads) break;  // warp-uniform
      const int hh = h0 + c * HPW + g;
      float x[8];
      const __half2* hp = reinterpret_cast<const __half2*>(&raw[c]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        x[2 * e] = __low2float(hp[e]);
        x[2 * e + 1] = __high2float(hp[e]);
      }
      const float* w = hh < Hq ? a.q_norm : (hh < Hq + Hk ? a.k_norm : nullptr);
      const bool norm = hh < Hq + Hk ? w != nullptr : a.v_norm != 0;
      float ss = 0.f;
      if (any_norm) {  // the same for every thread: the shuffles stay warp-wide
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += x[e] * x[e];
#pragma unroll
        for (int o = L / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(full, ss, o);
      }
      if (norm) {  // math.ts:78-97
        const float inv_rms = 1.f / sqrtf(ss / static_cast<float>(D) + a.rms_eps);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float sc = w == nullptr ? 1.f : (a.offset_rms ? 1.f + w[d0 + e] : w[d0 + e]);
          x[e] = x[e] * inv_rms * sc;
        }
      }
      float pt[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) pt[e] = __shfl_xor_sync(full, x[e], hl);
      if (hh < Hq + Hk) {  // RoPE, math.ts:134-147
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (turn[e]) x[e] = x[e] * cs[e] + (lo_side ? -pt[e] : pt[e]) * sn[e];
      }
      if (hh >= heads) continue;
      uint4 outv;
      uint32_t* ov = reinterpret_cast<uint32_t*>(&outv);
#pragma unroll
      for (int e = 0; e < 4; ++e) ov[e] = pack_half2(x[2 * e], x[2 * e + 1]);
      __half* dst;
      if (hh < Hq)
        dst = qscr + ((static_cast<size_t>(b) * Hq + hh) * seq_len + t) * D + d0;
      else if (hh < Hq + Hk)
        dst = kc + ((static_cast<size_t>(b) * Hk + (hh - Hq)) * a.max_tokens + pos) * D + d0;
      else
        dst = vc + ((static_cast<size_t>(b) * Hk + (hh - Hq - Hk)) * a.max_tokens + pos) * D + d0;
      if (TLA_IN_BOUNDS(hh < Hq ? ((static_cast<long long>(b) * Hq + hh) * seq_len + t) * D + d0 + 7
                                : ((static_cast<long long>(b) * Hk + (hh - Hq) % Hk) * a.max_tokens + pos) * D + d0 + 7,
                        hh < Hq ? static_cast<long long>(tokens) * Hq * D
                                : static_cast<long long>(a.max_batch) * Hk * a.max_tokens * D,
                        a.error))
        *reinterpret_cast<uint4*>(dst) = outv;
    }
  }
  griddep_launch_dependents();  // the attention kernel may start its prologue
}

template <int D>
cudaError_t rope_rows_t(const tla_layer* L, const void* qkv, const int32_t* start, int batch, int seq_len,
                        __half* qscr, cudaStream_t stream) {
  const int tokens = batch * seq_len;
  return launch_pdl(rope_rows_kernel<D>, (tokens + 3) / 4, 128, 0, stream, layer_args(L),
                    static_cast<const __half*>(qkv), start, seq_len, tokens, qscr);
}

template <typename IO, int D>
cudaError_t rope_warp_t(const tla_layer* L, const void* qkv, const int32_t* start, int batch, int seq_len,
                        __half* qscr, cudaStream_t stream) {
  const int tokens = batch * seq_len;
  rope_append_warp_kernel<IO, D><<<(tokens + 3) / 4, 128, 0, stream>>>(layer_args(L), static_cast<const IO*>(qkv),
                                                                         start, seq_len, tokens, qscr);
  return cudaGetLastError();
}

cudaError_t launch_rope_append_half_q(const tla_layer* L, const void* qkv, const int32_t* start, int batch,
                                      int seq_len, __half* qscr, cudaStream_t stream) {
  const int epl = L->D / 32;
  const bool warp_ok = !L->cache_fp32 && (L->D == 64 || L->D == 128) && ((L->rotary / 2) % epl == 0);
  const int hl = L->rotary / 16;
  const bool rows_ok = warp_ok && !L->io_fp32 && (L->rotary / 2) % 8 == 0 && (hl & (hl - 1)) == 0;
  if (rows_ok) return L->D == 64 ? rope_rows_t<64>(L, qkv, start, batch, seq_len, qscr, stream)
                                 : rope_rows_t<128>(L, qkv, start, batch, seq_len, qscr, stream);
  if (warp_ok) {
    if (L->D == 64)
      return L->io_fp32 ? rope_warp_t<float, 64>(L, qkv, start, batch, seq_len, qscr, stream)
                        : rope_warp_t<__half, 64>(L, qkv, start, batch, seq_len, qscr, stream);
    return L->io_fp32 ? rope_warp_t<float, 128>(L, qkv, start, batch, seq_len, qscr, stream)
                      : rope_warp_t<__half, 128>(L, qkv, start, batch, seq_len, qscr, stream);
  }
  if (L->io_fp32) return rope_append_t<float, __half, true>(L, qkv, start, batch, seq_len, 0, 1, qscr, stream);
  return rope_append_t<__half, __half, true>(L, qkv, start, batch, seq_len, 0, 1, qscr, stream);
}

cudaError_t launch_rope_append(const tla_layer* L, const void* qkv, const int32_t* start, int batch, int seq_len,
                               int slot_offset, int append, float* qscr, cudaStream_t stream) {
  if (L->io_fp32)
    return L->cache_fp32 ? rope_append_t<float, float>(L, qkv, start, batch, seq_len, slot_offset, append, qscr, stream)
                         : rope_append_t<float, __half>(L, qkv, start, batch, seq_len, slot_offset, append, qscr, stream);
  return L->cache_fp32 ? rope_append_t<__half, float>(L, qkv, start, batch, seq_len, slot_offset, append, qscr, stream)
                       : rope_append_t<__half, __half>(L, qkv, start, batch, seq_len, slot_offset, append, qscr, stream);
}

cudaError_t launch_attend_generic(const tla_layer* L, const float* qscr, const int32_t* start, int batch,
                                  int seq_len, int slot_offset, int local_tokens, const void* gate, void* out,
                                  float* partial, cudaStream_t stream) {
  if (L->io_fp32)
    return L->cache_fp32
               ? attend_t<float, float>(L, qscr, start, batch, seq_len, slot_offset, local_tokens, gate, out, partial,
                                        stream)
               : attend_t<__half, float>(L, qscr, start, batch, seq_len, slot_offset, local_tokens, gate, out, partial,
                                         stream);
  return L->cache_fp32
             ? attend_t<float, __half>(L, qscr, start, batch, seq_len, slot_offset, local_tokens, gate, out, partial,
                                       stream)
             : attend_t<__half, __half>(L, qscr, start, batch, seq_len, slot_offset, local_tokens, gate, out, partial,
                                        stream);
}

// ---------------------------------------------------------------- scores (scoreAttribute)
namespace {
// One block per (h, b): the block's threads walk the window's slots; the
// query row is staged in shared memory (TSLAttention.ts:306-356).
template <typename CT>
__global__ void __launch_bounds__(kThreads) scores_kernel(LayerArgs a, const float* __restrict__ query,
                                                          const int32_t* __restrict__ positions,
                                                          float* __restrict__ scores) {
  extern __shared__ float q[];  // [D]
  const int h = blockIdx.x, b = blockIdx.y;
  const int D = a.D, Hq = a.Hq, Hk = a.Hk;
  const int pos = positions[b];
  if (pos < 0 || pos >= a.max_tokens) {
    if (threadIdx.x == 0) report_error(a.error, TLA_ERR_POSITION);
    return;
  }
  const size_t qrow = static_cast<size_t>(b) * Hq + h;
  for (int d = threadIdx.x; d < D; d += kThreads) q[d] = query[qrow * D + d];
  __syncthreads();
  const int kvh = static_cast<int>((static_cast<long long>(h) * Hk) / Hq);  // TSLAttention.ts:340
  const int first = a.sliding > 0 ? max(0, pos - a.sliding + 1) : 0;       // :330-334
  const CT* kc = static_cast<const CT*>(a.k_cache) + (static_cast<size_t>(b) * Hk + kvh) * a.max_tokens * D;
  for (int t = first + threadIdx.x; t <= pos; t += kThreads) {
    const CT* kr = kc + static_cast<size_t>(t) * D;
    float dot = 0.f;
    for (int d = 0; d < D; ++d) dot += q[d] * to_f32(kr[d]);
    scores[qrow * a.max_tokens + t] = dot * a.attn_scale;
  }
}
}  // namespace

cudaError_t launch_scores(const tla_layer* L, const float* query, const int32_t* positions, int batch, float* scores,
                          cudaStream_t stream) {
  const LayerArgs a = layer_args(L);
  const size_t smem = sizeof(float) * L->D;
  if (L->cache_fp32)
    scores_kernel<float><<<dim3(L->Hq, batch), kThreads, smem, stream>>>(a, query, positions, scores);
  else
    scores_kernel<__half><<<dim3(L->Hq, batch), kThreads, smem, stream>>>(a, query, positions, scores);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- LSE combine
namespace {
template <typename IO>
__global__ void combine_lse_kernel(const float* __restrict__ partials, int ranks, int rows, int D,
                                   const IO* __restrict__ gate, IO* __restrict__ out) {
  const int row = blockIdx.x;  // (b, h)
  const size_t stride = static_cast<size_t>(rows) * (D + 2);
  float M = -INFINITY;
  for (int r = 0; r < ranks; ++r) M = fmaxf(M, partials[r * stride + static_cast<size_t>(row) * (D + 2)]);
  float Lsum = 0.f;
  for (int r = 0; r < ranks; ++r) {
    const float* p = partials + r * stride + static_cast<size_t>(row) * (D + 2);
    Lsum += p[1] * ex2(p[0] - M);
  }
  const float inv = Lsum > 0.f ? 1.f / Lsum : 0.f;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int r = 0; r < ranks; ++r) {
      const float* p = partials + r * stride + static_cast<size_t>(row) * (D + 2);
      acc += p[2 + d] * ex2(p[0] - M);
    }
    float v = acc * inv;
    if (gate) v = v * (1.f / (1.f + expf(-to_f32(gate[static_cast<size_t>(row) * D + d]))));
    out[static_cast<size_t>(row) * D + d] = from_f32<IO>(v);
  }
}
}  // namespace

cudaError_t launch_combine_lse(const float* partials, int ranks, int batch, int Hq, int D, const void* gate,
                               void* out, bool io_fp32, cudaStream_t stream) {
  const int rows = batch * Hq;
  if (rows == 0) return cudaSuccess;
  const int threads = D >= 128 ? 128 : (D >= 64 ? 64 : 32);
  if (io_fp32)
    combine_lse_kernel<float><<<rows, threads, 0, stream>>>(partials, ranks, rows, D, static_cast<const float*>(gate),
                                                            static_cast<float*>(out));
  else
    combine_lse_kernel<__half><<<rows, threads, 0, stream>>>(partials, ranks, rows, D,
                                                             static_cast<const __half*>(gate), static_cast<__half*>(out));
  return cudaGetLastError();
}

}  // namespace tla
