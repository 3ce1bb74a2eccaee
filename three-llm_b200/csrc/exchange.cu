// Peer-memory exchange of sequence-shard partial triples over NVLink.
//
// Long-context decode shards one sequence's cache by token blocks; every rank
// produces (m, l, o) per query head (tla_decode_partial) and needs everyone's
// triples to merge. Instead of a collective library call followed by a merge
// kernel, one kernel per layer, one CTA per query row: the CTA stores its
// row's triple into slot [rank] of every rank's buffer with plain 16-byte
// stores over NVLink, each 4-byte value paired with the call's epoch number
// (an 8-byte {value, epoch} word is never torn, so a reader that sees the
// epoch also sees the value: no fence or separate flag round trip). It then
// polls its row's words of every rank in its own buffer until all carry the
// epoch (bounded, ~2 s) and does the log-sum-exp merge.
//
// Buffer of one rank: [2 parities][ranks][slot words] {value, epoch} words,
// then the epoch counter, the CTA ticket and the abort word on their own
// 128-byte lines. Call number e (the device-side counter + 1) uses parity
// e & 1: a rank cannot finish call e+1 before every peer has stored its call
// e+1 words, which each does only after its call e kernel (all reads of
// parity e & 1) has completed, so a region is never overwritten while a peer
// reads it. The counter is advanced by the last CTA of each call (ticket), so
// a captured CUDA graph can replay the step. No multicast and no TMA touch
// peer memory: only ordinary ld/st.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <vector>

#include "tla_device.cuh"
#include "tla_internal.h"

struct tla_exchange {
  tla_ctx* ctx = nullptr;
  int rank = 0, ranks = 1;
  size_t slot_bytes = 0;    // bytes of one rank's float triples (multiple of 16)
  size_t region_bytes = 0;  // one parity region: ranks * slot_bytes * 2 ({value, epoch} words)
  uint8_t* local = nullptr; // [2][region] + epoch / ticket / abort lines
  size_t local_bytes = 0;
  std::vector<uint8_t*> peers;  // every rank's buffer (peers[rank] == local)
  std::vector<char> opened;     // peers[r] came from cudaIpcOpenMemHandle
  uint8_t** d_peers = nullptr;  // device copy of peers
  int connected = 0;
};

namespace tla {
namespace {

constexpr int kMaxRanks = 16;
constexpr int kCtrlBytes = 3 * 128;  // epoch, ticket, abort

__device__ __forceinline__ uint4 ld_volatile_v4(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ void st_volatile_v4(void* p, uint4 v) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// block = 128; CTA c owns rows c, c + grid, ... (grid <= rows, at most one
// CTA per SM, so every CTA that a peer's CTA waits for is resident). Every
// CTA first pushes all its rows, then gathers and merges them.
// W = D + 2 values per row (m, l, o[D]).
template <typename IO>
__global__ void __launch_bounds__(128) exchange_combine_kernel(uint8_t* const* peers, int rank, int ranks,
                                                               size_t region_bytes, size_t slot_words,
                                                               const float* __restrict__ partial, int rows, int D,
                                                               const IO* __restrict__ gate, IO* __restrict__ out,
                                                               int* error) {
  extern __shared__ float vals[];  // [ranks][W]
  __shared__ int epoch_s;
  __shared__ float wts[kMaxRanks];
  __shared__ float Ls;
  const int W = D + 2, tid = threadIdx.x;
  uint8_t* local = peers[rank];
  int* epoch_p = reinterpret_cast<int*>(local + 2 * region_bytes);
  int* ticket_p = reinterpret_cast<int*>(local + 2 * region_bytes + 128);
  volatile int* abort_p = reinterpret_cast<volatile int*>(local + 2 * region_bytes + 256);
  if (tid == 0) epoch_s = *reinterpret_cast<volatile int*>(epoch_p) + 1;
  __syncthreads();
  const unsigned epoch = static_cast<unsigned>(epoch_s);
  const size_t base = static_cast<size_t>(epoch & 1u) * region_bytes;
  // ---- push this rank's rows to every rank: {value, epoch, value, epoch}
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const size_t row_word = static_cast<size_t>(row) * W;  // W is even: 16-byte aligned pairs
    const float2* src = reinterpret_cast<const float2*>(partial + row_word);
    for (int i = tid; i < W / 2; i += blockDim.x) {
      const float2 f = src[i];
      const uint4 w = make_uint4(__float_as_uint(f.x), epoch, __float_as_uint(f.y), epoch);
      for (int r = 0; r < ranks; ++r)
        st_volatile_v4(peers[r] + base + ((static_cast<size_t>(rank) * slot_words + row_word) + 2 * i) * 8, w);
    }
  }
  const uint8_t* mine = local + base;
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const size_t row_word = static_cast<size_t>(row) * W;
    // ---- gather every rank's row from the local buffer: issue all loads, then re-poll stragglers
    for (int i = tid; i < W / 2; i += blockDim.x) {
      uint4 w[kMaxRanks];
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r)
        if (r < ranks) w[r] = ld_volatile_v4(mine + ((static_cast<size_t>(r) * slot_words + row_word) + 2 * i) * 8);
      unsigned long long t0 = 0;
      for (;;) {
        bool done = true;
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r)
          if (r < ranks && (w[r].y != epoch || w[r].w != epoch)) {
            done = false;
            w[r] = ld_volatile_v4(mine + ((static_cast<size_t>(r) * slot_words + row_word) + 2 * i) * 8);
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
      for (int r = 0; r < kMaxRanks; ++r)
        if (r < ranks) {
          vals[r * W + 2 * i] = __uint_as_float(w[r].x);
          vals[r * W + 2 * i + 1] = __uint_as_float(w[r].z);
        }
    }
    __syncthreads();
    // ---- log-sum-exp merge of the row
    if (tid < 32) {
      float M = -INFINITY;
      for (int r = 0; r < ranks; ++r) M = fmaxf(M, vals[r * W]);
      float L = 0.f;
      for (int r = tid; r < ranks; r += 32) {
        const float w = M == -INFINITY ? 0.f : ex2(vals[r * W] - M);
        wts[r] = w;
        L += vals[r * W + 1] * w;
      }
      L = warp_sum(L);
      if (tid == 0) Ls = L;
    }
    __syncthreads();
    const float L = Ls;
    for (int d = tid; d < D; d += blockDim.x) {
      float acc = 0.f;
      for (int r = 0; r < ranks; ++r) acc += vals[r * W + 2 + d] * wts[r];
      float v = L > 0.f ? acc / L : 0.f;
      const size_t oi = static_cast<size_t>(row) * D + d;
      if (gate) v = v * (1.f / (1.f + expf(-to_f32(gate[oi]))));
      out[oi] = from_f32<IO>(v);
    }
    __syncthreads();  // vals / wts reuse by the next row
  }
  // ---- the last CTA of the call advances the epoch (every CTA read it above)
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(ticket_p, 1) == static_cast<int>(gridDim.x) - 1) {
      *ticket_p = 0;
      *reinterpret_cast<volatile int*>(epoch_p) = static_cast<int>(epoch);
      __threadfence();
    }
  }
}

}  // namespace
}  // namespace tla

extern "C" {

int tla_exchange_create(tla_ctx* ctx, int32_t rank, int32_t ranks, size_t slot_bytes, tla_exchange** out,
                        void* handle_out) {
  if (!ctx || !out || !handle_out || ranks <= 0 || ranks > tla::kMaxRanks || rank < 0 || rank >= ranks || slot_bytes == 0)
    return TLA_ERR_INVALID_ARG;
  *out = nullptr;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(ctx->device);
  tla_exchange* ex = new tla_exchange();
  ex->ctx = ctx;
  ex->rank = rank;
  ex->ranks = ranks;
  ex->slot_bytes = (slot_bytes + 15) & ~size_t(15);
  ex->region_bytes = 2 * ex->slot_bytes * ranks;
  ex->local_bytes = 2 * ex->region_bytes + tla::kCtrlBytes;
  cudaError_t e = cudaMalloc(&ex->local, ex->local_bytes);
  if (e == cudaSuccess) e = cudaMemset(ex->local, 0, ex->local_bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle_out), ex->local);
  if (e == cudaSuccess) e = cudaMalloc(&ex->d_peers, sizeof(uint8_t*) * ranks);
  if (prev >= 0) cudaSetDevice(prev);
  if (e != cudaSuccess) {
    tla_exchange_destroy(ex);
    return e == cudaErrorMemoryAllocation ? TLA_ERR_OUT_OF_MEMORY : TLA_ERR_CUDA;
  }
  ex->peers.assign(ranks, nullptr);
  ex->opened.assign(ranks, 0);
  ex->peers[rank] = ex->local;
  *out = ex;
  return TLA_OK;
}

int tla_exchange_connect(tla_exchange* ex, const void* handles) {
  if (!ex || !handles || ex->connected) return TLA_ERR_INVALID_ARG;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(ex->ctx->device);
  cudaError_t e = cudaSuccess;
  for (int r = 0; r < ex->ranks && e == cudaSuccess; ++r) {
    if (r == ex->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const uint8_t*>(handles) + static_cast<size_t>(r) * sizeof(cudaIpcMemHandle_t), sizeof(h));
    void* p = nullptr;
    e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    ex->peers[r] = static_cast<uint8_t*>(p);
    ex->opened[r] = e == cudaSuccess;
  }
  if (e == cudaSuccess)
    e = cudaMemcpy(ex->d_peers, ex->peers.data(), sizeof(uint8_t*) * ex->ranks, cudaMemcpyHostToDevice);
  if (prev >= 0) cudaSetDevice(prev);
  if (e != cudaSuccess) return TLA_ERR_CUDA;
  ex->connected = 1;
  return TLA_OK;
}

int tla_exchange_buffer(tla_exchange* ex, void** buffer_out) {
  if (!ex || !buffer_out) return TLA_ERR_INVALID_ARG;
  *buffer_out = ex->local;
  return TLA_OK;
}

int tla_exchange_connect_buffers(tla_exchange* ex, void* const* buffers) {
  if (!ex || !buffers || ex->connected) return TLA_ERR_INVALID_ARG;
  for (int r = 0; r < ex->ranks; ++r)
    if (!buffers[r] || (r == ex->rank && buffers[r] != ex->local)) return TLA_ERR_INVALID_ARG;
  for (int r = 0; r < ex->ranks; ++r) ex->peers[r] = static_cast<uint8_t*>(buffers[r]);
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(ex->ctx->device);
  const cudaError_t e =
      cudaMemcpy(ex->d_peers, ex->peers.data(), sizeof(uint8_t*) * ex->ranks, cudaMemcpyHostToDevice);
  if (prev >= 0) cudaSetDevice(prev);
  if (e != cudaSuccess) return TLA_ERR_CUDA;
  ex->connected = 1;
  return TLA_OK;
}

int tla_exchange_combine(tla_exchange* ex, const float* partial, int32_t batch, int32_t head_count, int32_t head_dim,
                         const void* gate, void* out, uint32_t io_flags, void* stream) {
  if (!ex || !ex->connected || !partial || !out || batch <= 0 || head_count <= 0 || head_dim <= 0 || head_dim % 2)
    return TLA_ERR_INVALID_ARG;
  const size_t need = static_cast<size_t>(batch) * head_count * (head_dim + 2) * sizeof(float);
  if (need > ex->slot_bytes) return TLA_ERR_INVALID_ARG;
  const long long rows = static_cast<long long>(batch) * head_count;
  if (rows > 0x7fffffffLL) return TLA_ERR_UNSUPPORTED;
  const size_t smem = static_cast<size_t>(ex->ranks) * (head_dim + 2) * sizeof(float);
  if (smem > 48 * 1024) return TLA_ERR_UNSUPPORTED;
  const size_t slot_words = ex->slot_bytes / sizeof(float);
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(ex->ctx->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>(rows < ex->ctx->sm_count ? rows : ex->ctx->sm_count);
  if (io_flags & TLA_FLAG_IO_FP32)
    tla::exchange_combine_kernel<float><<<grid, 128, smem, st>>>(ex->d_peers, ex->rank, ex->ranks, ex->region_bytes,
                                                                 slot_words, partial, static_cast<int>(rows), head_dim,
                                                                 static_cast<const float*>(gate),
                                                                 static_cast<float*>(out), ex->ctx->d_error);
  else
    tla::exchange_combine_kernel<__half><<<grid, 128, smem, st>>>(ex->d_peers, ex->rank, ex->ranks,
                                                                  ex->region_bytes, slot_words, partial, static_cast<int>(rows),
                                                                  head_dim, static_cast<const __half*>(gate),
                                                                  static_cast<__half*>(out), ex->ctx->d_error);
  const cudaError_t e = cudaGetLastError();
  if (prev >= 0) cudaSetDevice(prev);
  return e == cudaSuccess ? TLA_OK : TLA_ERR_CUDA;
}

int tla_exchange_destroy(tla_exchange* ex) {
  if (!ex) return TLA_OK;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(ex->ctx->device);
  for (int r = 0; r < static_cast<int>(ex->peers.size()); ++r)
    if (ex->opened[r]) cudaIpcCloseMemHandle(ex->peers[r]);
  cudaFree(ex->local);
  cudaFree(ex->d_peers);
  if (prev >= 0) cudaSetDevice(prev);
  delete ex;
  return TLA_OK;
}

}  // extern "C"
