// Peer-memory exchange of sequence-shard partial triples over NVLink.
//
// Long-context decode shards one sequence's cache by token blocks; every rank
// produces (m, l, o) per query head (tla_decode_partial) and needs everyone's
// triples to merge. Instead of a collective library call followed by a merge
// kernel, one kernel per layer, CTAs over query rows: each stores its rows'
// triples into slot [rank] of every rank's buffer with plain 16-byte stores
// over NVLink, then polls its rows' words of every rank in its own buffer and
// does the log-sum-exp merge (protocol: exchange.cuh). The fused
// decode + exchange kernel (decode_fast.cu) uses the same buffers.
// No multicast and no TMA touch peer memory: only ordinary ld/st.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <vector>

#include "exchange.cuh"
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

bool exchange_device_view(const tla_exchange* ex, ExchangeDev* out) {
  if (!ex || !ex->connected) return false;
  out->peers = ex->d_peers;
  out->rank = ex->rank;
  out->ranks = ex->ranks;
  out->region_bytes = ex->region_bytes;
  out->slot_words = ex->slot_bytes / sizeof(float);
  return true;
}

size_t exchange_slot_bytes(const tla_exchange* ex) { return ex ? ex->slot_bytes : 0; }

namespace {

// block = 128; CTA c owns rows c, c + grid, ... (grid <= rows, at most one
// CTA per SM, so every CTA that a peer's CTA waits for is resident). Every
// CTA first pushes all its rows, then gathers and merges them.
// W = D + 2 values per row (m, l, o[D]).
template <typename IO>
__global__ void __launch_bounds__(128) exchange_combine_kernel(ExchangeDev x, const float* __restrict__ partial,
                                                               int rows, int D, const IO* __restrict__ gate,
                                                               IO* __restrict__ out, int* error) {
  extern __shared__ float vals[];  // [ranks][W]
  __shared__ int epoch_s;
  __shared__ float wts[kXchMaxRanks];
  __shared__ float ls;
  const int W = D + 2;
  const unsigned epoch = xch_epoch(x, &epoch_s);
  for (int row = blockIdx.x; row < rows; row += gridDim.x)
    xch_push_row(x, epoch, row, partial + static_cast<size_t>(row) * W, W);
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    xch_gather_row(x, epoch, row, W, vals, error);
    xch_merge_row<IO>(vals, x.ranks, D, gate ? gate + static_cast<size_t>(row) * D : nullptr,
                      out + static_cast<size_t>(row) * D, wts, &ls);
  }
  xch_finish(x, epoch);
}

}  // namespace
}  // namespace tla

extern "C" {

int tla_exchange_create(tla_ctx* ctx, int32_t rank, int32_t ranks, size_t slot_bytes, tla_exchange** out,
                        void* handle_out) {
  if (!ctx || !out || !handle_out || ranks <= 0 || ranks > tla::kXchMaxRanks || rank < 0 || rank >= ranks || slot_bytes == 0)
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
  ex->local_bytes = 2 * ex->region_bytes + tla::kXchCtrlBytes;
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
  tla::ExchangeDev x;
  tla::exchange_device_view(ex, &x);
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(ex->ctx->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>(rows < ex->ctx->sm_count ? rows : ex->ctx->sm_count);
  if (io_flags & TLA_FLAG_IO_FP32)
    tla::exchange_combine_kernel<float><<<grid, 128, smem, st>>>(x, partial, static_cast<int>(rows), head_dim,
                                                                 static_cast<const float*>(gate),
                                                                 static_cast<float*>(out), ex->ctx->d_error);
  else
    tla::exchange_combine_kernel<__half><<<grid, 128, smem, st>>>(x, partial, static_cast<int>(rows), head_dim,
                                                                  static_cast<const __half*>(gate),
                                                                  static_cast<__half*>(out), ex->ctx->d_error);
  const cudaError_t e = cudaGetLastError();
  if (prev >= 0) cudaSetDevice(prev);
  return e == cudaSuccess ? TLA_OK : TLA_ERR_CUDA;
}

int tla_out_proj_allreduce(tla_exchange* ex, const void* attn, const void* weight, const float* bias,
                           const void* residual, void* y, int32_t rows, int32_t in_features, int32_t hidden,
                           uint32_t io_flags, void* stream) {
  if (!ex || !ex->connected || !attn || !weight || !y || rows < 0 || in_features <= 0 || in_features % 64 != 0 ||
      hidden <= 0 || hidden % (64 * ex->ranks) != 0)
    return TLA_ERR_INVALID_ARG;
  if (2 * static_cast<size_t>(rows) * (hidden / ex->ranks) * sizeof(float) > ex->slot_bytes)
    return TLA_ERR_INVALID_ARG;
  if (ex->ctx->encode_tiled == nullptr) return TLA_ERR_UNSUPPORTED;
  if (rows == 0) return TLA_OK;
  tla::ExchangeDev x;
  tla::exchange_device_view(ex, &x);
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(ex->ctx->device);
  const cudaError_t e =
      tla::launch_out_proj_allreduce(ex->ctx, x, attn, weight, bias, residual, (io_flags & TLA_FLAG_IO_FP32) != 0, y,
                                     rows, in_features, hidden, static_cast<cudaStream_t>(stream));
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
