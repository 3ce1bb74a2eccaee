// Peer-memory exchange of sequence-shard partial triples over NVLink.
//
// Long-context decode shards one sequence's cache by token blocks; every rank
// produces (m, l, o) per query head (tla_decode_partial) and needs everyone's
// triples to merge. Instead of a collective library call followed by a merge
// kernel, one kernel per layer: pushes this rank's triples into slot [rank]
// of every peer's gather buffer with plain stores over NVLink, publishes a
// per-rank epoch flag with system-scope release, waits (bounded, ~2 s) until
// every peer's flag for this epoch has arrived in its own buffer, then does
// the log-sum-exp merge. The epoch counter lives in device memory and is
// advanced by the kernel, so a captured CUDA graph can replay the step.
// No multicast and no TMA touch peer memory: only ordinary ld/st.
#include <cuda_runtime.h>
#include <stdint.h>
#include <math.h>
#include <string.h>

#include <vector>

#include "tla_device.cuh"
#include "tla_internal.h"

struct tla_exchange {
  tla_ctx* ctx = nullptr;
  int rank = 0, ranks = 1;
  size_t slot_bytes = 0;    // bytes of one rank's triples (multiple of 16)
  uint8_t* local = nullptr; // [2][ranks][slot_bytes] gather + [ranks] flags (128 B apart) + epoch
  size_t local_bytes = 0;
  std::vector<uint8_t*> peers;  // every rank's buffer (peers[rank] == local)
  std::vector<char> opened;     // peers[r] came from cudaIpcOpenMemHandle
  uint8_t** d_peers = nullptr;  // device copy of peers
  int connected = 0;
};

namespace tla {
namespace {

constexpr int kFlagStride = 128;  // bytes between flags (own cache line each)

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

constexpr int kMaxWeights = 8192;  // rows * ranks held in shared memory

// Buffer of one rank: [2 parities][ranks][stride] triples, then [ranks] epoch
// flags (kFlagStride apart), then this rank's epoch counter. Epoch e uses
// parity e & 1: a rank can be at most one epoch ahead of the slowest peer
// (it cannot finish epoch e+1 before every peer has published e+1, which each
// does only after merging e), so the slot it overwrites is never being read.
template <typename IO>
__global__ void __launch_bounds__(256) exchange_combine_kernel(uint8_t* const* peers, int rank, int ranks,
                                                               size_t stride, size_t bytes,
                                                               const float* __restrict__ partial, int rows, int D,
                                                               const IO* __restrict__ gate, IO* __restrict__ out,
                                                               int* error) {
  __shared__ int epoch_s;
  __shared__ float wsh[kMaxWeights];  // [rows][ranks] merge weights
  __shared__ float lsh[1024];         // [rows] merged sums (rows <= 1024)
  uint8_t* local = peers[rank];
  const size_t flags_off = 2 * static_cast<size_t>(ranks) * stride;
  int* epoch_p = reinterpret_cast<int*>(local + flags_off + static_cast<size_t>(ranks) * kFlagStride);
  const int tid = threadIdx.x;
  if (tid == 0) epoch_s = *epoch_p + 1;
  __syncthreads();
  const int epoch = epoch_s;
  const size_t base = static_cast<size_t>(epoch & 1) * ranks * stride;
  // push this rank's triples into slot [rank] of every buffer (its own included)
  const int n16 = static_cast<int>(bytes / 16);
  const uint4* src = reinterpret_cast<const uint4*>(partial);
  for (int r = 0; r < ranks; ++r) {
    uint4* dst = reinterpret_cast<uint4*>(peers[r] + base + static_cast<size_t>(rank) * stride);
    for (int i = tid; i < n16; i += blockDim.x) dst[i] = src[i];
  }
  __threadfence_system();  // this thread's stores before the flags below
  __syncthreads();
  if (tid < ranks)  // publish to rank tid: data, then flag, at system scope
    st_release_sys(reinterpret_cast<int*>(peers[tid] + flags_off + static_cast<size_t>(rank) * kFlagStride), epoch);
  if (tid < ranks) {  // wait for rank tid's flag of this epoch in the local buffer (bounded)
    const int* f = reinterpret_cast<const int*>(local + flags_off + static_cast<size_t>(tid) * kFlagStride);
    const unsigned long long t0 = globaltimer();
    while (ld_acquire_sys(f) < epoch) {
      if (globaltimer() - t0 > kWaitLimitNs) {
        report_error(error, TLA_ERR_TIMEOUT);
        break;
      }
    }
  }
  __syncthreads();
  __threadfence();
  if (tid == 0) *epoch_p = epoch;
  // log-sum-exp merge of the gathered triples (read past L1: written by peers)
  const float* g = reinterpret_cast<const float*>(local + base);
  const size_t slot_f = stride / 4;
  for (int row = tid; row < rows; row += blockDim.x) {
    float M = -INFINITY;
    for (int r = 0; r < ranks; ++r) M = fmaxf(M, __ldcg(g + r * slot_f + static_cast<size_t>(row) * (D + 2)));
    float L = 0.f;
    for (int r = 0; r < ranks; ++r) {
      const float* pr = g + r * slot_f + static_cast<size_t>(row) * (D + 2);
      const float w = M == -INFINITY ? 0.f : ex2(__ldcg(pr) - M);
      wsh[row * ranks + r] = w;
      L += __ldcg(pr + 1) * w;
    }
    lsh[row] = L;
  }
  __syncthreads();
  for (int i = tid; i < rows * D; i += blockDim.x) {
    const int row = i / D, d = i - row * D;
    float acc = 0.f;
    for (int r = 0; r < ranks; ++r)
      acc += __ldcg(g + r * slot_f + static_cast<size_t>(row) * (D + 2) + 2 + d) * wsh[row * ranks + r];
    const float L = lsh[row];
    float v = L > 0.f ? acc / L : 0.f;
    if (gate) v = v * (1.f / (1.f + expf(-to_f32(gate[i]))));
    out[i] = from_f32<IO>(v);
  }
}

}  // namespace
}  // namespace tla

extern "C" {

int tla_exchange_create(tla_ctx* ctx, int32_t rank, int32_t ranks, size_t slot_bytes, tla_exchange** out,
                        void* handle_out) {
  if (!ctx || !out || !handle_out || ranks <= 0 || ranks > 256 || rank < 0 || rank >= ranks || slot_bytes == 0)
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
  ex->local_bytes = 2 * ex->slot_bytes * ranks + static_cast<size_t>(ranks) * tla::kFlagStride + tla::kFlagStride;
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
  if (!ex || !ex->connected || !partial || !out || batch <= 0 || head_count <= 0 || head_dim <= 0)
    return TLA_ERR_INVALID_ARG;
  const size_t need = static_cast<size_t>(batch) * head_count * (head_dim + 2) * sizeof(float);
  const long long rows_ll = static_cast<long long>(batch) * head_count;
  if (need > ex->slot_bytes || need % 16 != 0) return TLA_ERR_INVALID_ARG;
  if (rows_ll > 1024 || rows_ll * ex->ranks > tla::kMaxWeights) return TLA_ERR_UNSUPPORTED;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(ex->ctx->device);
  const int rows = batch * head_count;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (io_flags & TLA_FLAG_IO_FP32)
    tla::exchange_combine_kernel<float><<<1, 256, 0, st>>>(ex->d_peers, ex->rank, ex->ranks, ex->slot_bytes, need,
                                                          partial, rows,
                                                          head_dim, static_cast<const float*>(gate),
                                                          static_cast<float*>(out), ex->ctx->d_error);
  else
    tla::exchange_combine_kernel<__half><<<1, 256, 0, st>>>(ex->d_peers, ex->rank, ex->ranks, ex->slot_bytes, need,
                                                           partial, rows,
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
