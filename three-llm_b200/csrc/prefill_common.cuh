// Pieces shared by the two tensor-core prefill kernels (prefill_tc.cu: one
// query tile per CTA pipeline, any head_dim; prefill_pp.cu: two query tiles
// per CTA sharing the K/V steps, head_dim 64): parameters, the softmax
// arithmetic helpers, TMEM row loads and the TMA maps of the queries and the cache.
#pragma once

#include <math.h>

#include "tcgen05.cuh"
#include "tla_device.cuh"
#include "tla_internal.h"

namespace tla {
namespace prefill {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.f;  // a row's reference maximum moves only when exceeded by 2^8

struct PrefillParams {
  CUtensorMap tm_q;  // rotated queries [B*Hq][S][D] fp16, 128-row boxes
  CUtensorMap tm_k;  // cache [max_batch*Hk][max_tokens][D] fp16, 128-token boxes
  CUtensorMap tm_v;
  void* out;
  const void* gate;  // null, or [B][S][Hq][D] like out: out *= sigmoid(gate)
  const int32_t* start;
  int* error;
  int S, Hq, Hk, G, sliding, batch, num_m;
  float scale_log2;
  // two-tile kernel: with piece_len > 0, each pair's KV steps are cut into
  // pieces of about piece_len steps, every piece leaves fp32 partial rows in
  // `part`, and a merge kernel writes the output (0: whole pairs)
  int piece_len;
  float* part;
};

// 2^x on the FMA pipe, for part of the softmax exponentials (the MUFU unit is the
// bottleneck at head_dim 64). Cody-Waite split x = j + f with j = rint(x) (the
// 1.5 * 2^23 rounding trick, j ends up in the low mantissa bits), f in [-0.5, 0.5];
// 2^f from a cubic least-squares fit on Chebyshev nodes of [-0.5, 0.5]
// (max relative error 7.7e-5, below fp16 resolution); 2^j is added to the
// exponent field. Inputs below -126 (masked scores) give a subnormal that
// rounds to 0 in fp16.
__device__ __forceinline__ float ex2_poly(float x) {
  x = fmaxf(x, -126.f);
  const float t = x + 12582912.f;
  const float f = x - (t - 12582912.f);
  const float p = fmaf(fmaf(fmaf(0.05508868f, f, 0.24260405f), f, 0.69327623f), f, 0.99992895f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}


#ifndef TLA_PREFILL_POLY_EVERY
#define TLA_PREFILL_POLY_EVERY 0  // head_dim 128 kernel: every n-th pair of exponentials on the FMA pipe (0: none)
#endif
#ifndef TLA_PP_POLY_EVERY
// two-tile head_dim 64 kernel: every 8th pair of exponentials on the FMA pipe
// (config 3: 0.0779 against 0.0780-0.0785 ms without; every 16th: 0.0788)
#define TLA_PP_POLY_EVERY 8
#endif

// Whether pair `i` of a row's exponentials is evaluated with ex2_poly, for
// every EVERY-th pair (none when EVERY is 0).
template <int EVERY>
__device__ __forceinline__ constexpr bool poly_pair_every(int i) {
  if constexpr (EVERY > 0) {
    return i % EVERY == EVERY - 1;
  } else {
    return i < 0;
  }
}
__device__ __forceinline__ constexpr bool poly_pair(int i) { return poly_pair_every<TLA_PREFILL_POLY_EVERY>(i); }

// Packed fp32 pairs (sm_100 f32x2 arithmetic: one instruction for two
// columns' FMA or add, each element rounded as its scalar counterpart).
__device__ __forceinline__ uint64_t pack_f32x2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
// (a0, a1) * b2 + c2
__device__ __forceinline__ void fma_f32x2(float a0, float a1, uint64_t b2, uint64_t c2, float& r0, float& r1) {
  asm("{\n\t.reg .b64 a, d;\n\tmov.b64 a, {%2, %3};\n\tfma.rn.f32x2 d, a, %4, %5;\n\tmov.b64 {%0, %1}, d;\n\t}"
      : "=f"(r0), "=f"(r1)
      : "f"(a0), "f"(a1), "l"(b2), "l"(c2));
}
// acc += (e0, e1)
__device__ __forceinline__ void add_f32x2(uint64_t& acc, float e0, float e1) {
  asm("{\n\t.reg .b64 e;\n\tmov.b64 e, {%1, %2};\n\tadd.rn.f32x2 %0, %0, e;\n\t}" : "+l"(acc) : "f"(e0), "f"(e1));
}
__device__ __forceinline__ float sum_f32x2(uint64_t v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return lo + hi;
}

// 64 consecutive fp32 columns of this thread's TMEM lane (two loads, one wait).
__device__ __forceinline__ void tmem_ld64x(uint32_t taddr, uint32_t (&r)[64]) {
#pragma unroll
  for (int k = 0; k < 2; ++k)
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[k * 32 + 0]), "=r"(r[k * 32 + 1]), "=r"(r[k * 32 + 2]), "=r"(r[k * 32 + 3]), "=r"(r[k * 32 + 4]),
          "=r"(r[k * 32 + 5]), "=r"(r[k * 32 + 6]), "=r"(r[k * 32 + 7]), "=r"(r[k * 32 + 8]), "=r"(r[k * 32 + 9]),
          "=r"(r[k * 32 + 10]), "=r"(r[k * 32 + 11]), "=r"(r[k * 32 + 12]), "=r"(r[k * 32 + 13]),
          "=r"(r[k * 32 + 14]), "=r"(r[k * 32 + 15]), "=r"(r[k * 32 + 16]), "=r"(r[k * 32 + 17]),
          "=r"(r[k * 32 + 18]), "=r"(r[k * 32 + 19]), "=r"(r[k * 32 + 20]), "=r"(r[k * 32 + 21]),
          "=r"(r[k * 32 + 22]), "=r"(r[k * 32 + 23]), "=r"(r[k * 32 + 24]), "=r"(r[k * 32 + 25]),
          "=r"(r[k * 32 + 26]), "=r"(r[k * 32 + 27]), "=r"(r[k * 32 + 28]), "=r"(r[k * 32 + 29]),
          "=r"(r[k * 32 + 30]), "=r"(r[k * 32 + 31])
        : "r"(taddr + k * 32));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 consecutive values of a gate row, as floats (16-byte loads).
template <typename T>
__device__ __forceinline__ void load_row32(const T* src, float (&v)[32]) {
  if constexpr (sizeof(T) == 2) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 u = *reinterpret_cast<const uint4*>(src + 8 * i);
      const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        v[8 * i + 2 * k] = __low2float(h[k]);
        v[8 * i + 2 * k + 1] = __high2float(h[k]);
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 f = *reinterpret_cast<const float4*>(src + 4 * i);
      v[4 * i] = f.x;
      v[4 * i + 1] = f.y;
      v[4 * i + 2] = f.z;
      v[4 * i + 3] = f.w;
    }
  }
}

// Item index of this CTA's k-th item (snake order over the grid), or -1.
__device__ __forceinline__ int prefill_item_of(int k, int num_items) {
  const int G = static_cast<int>(gridDim.x), c = static_cast<int>(blockIdx.x);
  const int it = k * G + ((k & 1) ? G - 1 - c : c);
  return it < num_items ? it : -1;
}

inline CUresult make_map(const tla_layer* L, void* base, uint64_t rows, uint64_t planes, CUtensorMap* map,
                        uint32_t box_rows = 128) {
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(L->D), rows, planes};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(L->D) * 2, static_cast<cuuint64_t>(L->D) * 2 * rows};
  const cuuint32_t box[3] = {64, box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return L->ctx->encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, base, dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

// The two-tile kernel (prefill_pp.cu, head_dim 64, fp16 cache).
cudaError_t pp_configure(const tla_layer* L);
size_t pp_smem();
cudaError_t launch_pp(const tla_layer* L, const PrefillParams& p, cudaStream_t stream);
// Scratch bytes the two-tile kernel needs past the rotated queries for a
// chunk of batch x seq_len (0: the chunk has enough work items unsplit).
size_t pp_partial_bytes(const tla_layer* L, int batch, int seq_len);

}  // namespace prefill
}  // namespace tla
