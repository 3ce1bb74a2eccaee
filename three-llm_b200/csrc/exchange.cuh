// Device side of the peer-memory exchange (tla_exchange_*): the {value, epoch}
// word protocol shared by exchange_combine_kernel (exchange.cu) and the fused
// decode + exchange kernel (decode_fast.cu).
//
// Buffer of one rank: [2 parities][ranks][slot words] 8-byte {value, epoch}
// words, then the epoch counter, the CTA ticket and the abort word on their
// own 128-byte lines. A row of W floats (W even) of rank s lives at words
// [parity][s][row * W ..]. Call number e (the device-side counter + 1) uses
// parity e & 1: a rank cannot finish call e+1 before every peer has stored
// its call e+1 words, which each does only after its call e kernel (all reads
// of parity e & 1) has completed, so a region is never overwritten while a
// peer reads it. An aligned 8-byte store is never torn, so a reader that sees
// the epoch in a word also sees its value: no fence and no separate flag.
// The last CTA of each call (ticket) advances the epoch counter, so a
// captured CUDA graph can replay the step.
#pragma once

#include <math.h>
#include <stdint.h>

#include "tla_device.cuh"

namespace tla {

constexpr int kXchMaxRanks = 16;
constexpr int kXchCtrlBytes = 3 * 128;  // epoch, ticket, abort

struct ExchangeDev {
  uint8_t* const* peers;  // device array: every rank's buffer (peers[rank] is local)
  int rank, ranks;
  size_t region_bytes;    // one parity region
  size_t slot_words;      // words of one rank's slot
};

__device__ __forceinline__ uint4 xch_ld_v4(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ void xch_st_v4(void* p, uint4 v) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ int* xch_epoch_ptr(const ExchangeDev& x) {
  return reinterpret_cast<int*>(x.peers[x.rank] + 2 * x.region_bytes);
}

// The call's epoch number, read by thread 0 and broadcast through shared memory.
__device__ __forceinline__ unsigned xch_epoch(const ExchangeDev& x, int* smem_slot) {
  if (threadIdx.x == 0) *smem_slot = *reinterpret_cast<volatile int*>(xch_epoch_ptr(x)) + 1;
  __syncthreads();
  return static_cast<unsigned>(*smem_slot);
}

// Store this rank's row (W floats at src, W even, 8-byte aligned) into slot
// [rank] of every rank's buffer; threads of the block share the pairs.
__device__ __forceinline__ void xch_push_row(const ExchangeDev& x, unsigned epoch, int row, const float* src, int W) {
  const size_t base = static_cast<size_t>(epoch & 1u) * x.region_bytes;
  const size_t word0 = static_cast<size_t>(x.rank) * x.slot_words + static_cast<size_t>(row) * W;
  const float2* s2 = reinterpret_cast<const float2*>(src);
  for (int i = threadIdx.x; i < W / 2; i += blockDim.x) {
    const float2 f = s2[i];
    const uint4 w = make_uint4(__float_as_uint(f.x), epoch, __float_as_uint(f.y), epoch);
    for (int r = 0; r < x.ranks; ++r) xch_st_v4(x.peers[r] + base + (word0 + 2 * i) * 8, w);
  }
}

// Gather every rank's row from the local buffer into vals[ranks][W] (shared
// memory): all loads are issued, then the words whose epoch is not yet there
// are polled again, bounded by kWaitLimitNs (then TLA_ERR_TIMEOUT, and the
// abort word tells the other threads of this call to stop waiting).
__device__ __forceinline__ void xch_gather_row(const ExchangeDev& x, unsigned epoch, int row, int W, float* vals,
                                               int* error) {
  const uint8_t* mine = x.peers[x.rank] + static_cast<size_t>(epoch & 1u) * x.region_bytes;
  volatile int* abort_p = reinterpret_cast<volatile int*>(x.peers[x.rank] + 2 * x.region_bytes + 256);
  for (int i = threadIdx.x; i < W / 2; i += blockDim.x) {
    uint4 w[kXchMaxRanks];
#pragma unroll
    for (int r = 0; r < kXchMaxRanks; ++r)
      if (r < x.ranks)
        w[r] = xch_ld_v4(mine + ((static_cast<size_t>(r) * x.slot_words + static_cast<size_t>(row) * W) + 2 * i) * 8);
    unsigned long long t0 = 0;
    for (;;) {
      bool done = true;
#pragma unroll
      for (int r = 0; r < kXchMaxRanks; ++r)
        if (r < x.ranks && (w[r].y != epoch || w[r].w != epoch)) {
          done = false;
          w[r] = xch_ld_v4(mine +
                           ((static_cast<size_t>(r) * x.slot_words + static_cast<size_t>(row) * W) + 2 * i) * 8);
        }
      if (done) break;
      if (*abort_p == static_cast<int>(epoch)) break;  // another thread already gave up on this call
      const unsigned long long now = globaltimer();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > kWaitLimitNs) {
        report_error(error, TLA_ERR_TIMEOUT);
        *abort_p = static_cast<int>(epoch);
        break;
      }
    }
#pragma unroll
    for (int r = 0; r < kXchMaxRanks; ++r)
      if (r < x.ranks) {
        vals[r * W + 2 * i] = __uint_as_float(w[r].x);
        vals[r * W + 2 * i + 1] = __uint_as_float(w[r].z);
      }
  }
}

// Log-sum-exp merge of the gathered rows vals[ranks][W] (W = D + 2: m, l,
// o[D]) into out[0 .. D) (times sigmoid(gate) when gate is given). Whole
// block; wts holds kXchMaxRanks floats, ls one.
template <typename IO>
__device__ __forceinline__ void xch_merge_row(const float* vals, int ranks, int D, const IO* gate, IO* out,
                                              float* wts, float* ls) {
  const int W = D + 2;
  __syncthreads();
  if (threadIdx.x < 32) {
    float M = -INFINITY;
    for (int r = 0; r < ranks; ++r) M = fmaxf(M, vals[r * W]);
    float L = 0.f;
    for (int r = threadIdx.x; r < ranks; r += 32) {
      const float w = M == -INFINITY ? 0.f : ex2(vals[r * W] - M);
      wts[r] = w;
      L += vals[r * W + 1] * w;
    }
    L = warp_sum(L);
    if (threadIdx.x == 0) *ls = L;
  }
  __syncthreads();
  const float L = *ls;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int r = 0; r < ranks; ++r) acc += vals[r * W + 2 + d] * wts[r];
    float v = L > 0.f ? acc / L : 0.f;
    if (gate) v = v * (1.f / (1.f + expf(-to_f32(gate[d]))));
    out[d] = from_f32<IO>(v);
  }
  __syncthreads();  // vals / wts reuse by the next row
}

// The last CTA of the call advances the epoch (every CTA read it at its start).
__device__ __forceinline__ void xch_finish(const ExchangeDev& x, unsigned epoch) {
  if (threadIdx.x == 0) {
    int* epoch_p = xch_epoch_ptr(x);
    int* ticket_p = reinterpret_cast<int*>(x.peers[x.rank] + 2 * x.region_bytes + 128);
    __threadfence();
    if (atomicAdd(ticket_p, 1) == static_cast<int>(gridDim.x) - 1) {
      *ticket_p = 0;
      *reinterpret_cast<volatile int*>(epoch_p) = static_cast<int>(epoch);
      __threadfence();
    }
  }
}

}  // namespace tla
