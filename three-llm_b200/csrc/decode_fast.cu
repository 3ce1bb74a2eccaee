// Persistent split-KV decode attention for B200 (sm_100a), fp16 K/V cache,
// head_dim 64 or 128, GQA group <= 16.
//
// Replaces the four WebGPU kernels of one TSLAttention decode step
// (packages/three-llm/src/tsl/TSLAttention.ts:252-428): copy-KV (RoPE and
// QK-norm of the new K, append), query (RoPE and QK-norm of Q), scores and the
// two-pass softmax + PV. Semantics follow causalAttention
// (packages/three-llm/src/runtime/math.ts:179-276).
//
// Work split: the (sequence, kv head) pairs' token ranges are cut into
// 64-token tiles; the grid is persistent (a fixed number of CTAs per SM) and
// CTA c takes the contiguous global tile range [c*T/C, (c+1)*T/C), so every
// CTA streams the same number of bytes whatever the per-sequence lengths.
// A CTA's range may start or end inside a pair: such partial segments leave
// (m, l, o) triples in scratch, and the CTA that completes a pair's tile count
// (an atomic ticket, no spinning) merges them with a log-sum-exp combine.
//
// CTA: 4 consumer warps + 1 producer warp. The producer's lane 0 streams K and
// V tiles with TMA (cp.async.bulk.tensor, 128-byte swizzle) into a ring of
// shared-memory stages guarded by mbarriers. Each consumer warp owns 16 tokens
// of a tile: S = Q K^T and O += P V run as m16n8k16 tensor-core tiles (the
// GQA group's query heads are the 16 rows), the online softmax keeps fp32
// running max / sum per row, reduced across the 4 lanes that share a row with
// warp shuffles. All smem reads are ldmatrix on the swizzled layout.
#include <math.h>

#include <mutex>

#include "exchange.cuh"
#include "tla_device.cuh"
#include "tla_internal.h"

namespace tla {

namespace {

constexpr int kTile = 64;            // tokens per pipeline stage
constexpr int kConsumerWarps = 4;    // 16 tokens each
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kMaxBatch = 1024;      // prefix table in shared memory

// Pipeline depth per head_dim: at 2 resident CTAs per SM a 4-stage (D=64) or
// 2-stage (D=128) ring keeps 64-128 KB of K/V in flight per SM.
// A pair split over more than this many CTAs (segments) is merged by
// decode_merge_kernel instead of by the last CTA in the decode kernel.
#ifndef TLA_DEFER_MERGE_SEGMENTS
#define TLA_DEFER_MERGE_SEGMENTS 4
#endif

#ifndef TLA_DECODE_STAGES_D64
#define TLA_DECODE_STAGES_D64 4
#endif
#ifndef TLA_DECODE_STAGES_D128
#define TLA_DECODE_STAGES_D128 2
#endif

#ifdef TLA_DECODE_TRACE
// Optional per-CTA timeline (builds with -DTLA_DECODE_TRACE only): globaltimer
// at [cta][0] entry, [1] partition done, [2] first tile landed (consumer warp
// 0), [3] last tile consumed, [4] exit, [5] first TMA issued, [6] first
// segment's query set-up done, [7] set-up loads stored, [8] norms done,
// [10] query rows stored, [11] RoPE factors stored, [12] RoPE applied,
// [13] producer has the first position, [14] partition re-checked after the
// wait, [15] consumer has the first position; read with
// tla_debug_decode_trace. The timer read is a compiler memory barrier, so an
// event follows the memory operations before it in program order.
__device__ unsigned long long g_decode_trace[2048][16];
#define DTRACE(ev) \
  do { \
    unsigned long long t_; \
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_)::"memory"); \
    if (blockIdx.x < 2048) g_decode_trace[blockIdx.x][(ev)] = t_; \
  } while (0)
#define DTRACE_AFTER(ev, v) \
  do { \
    asm volatile("" ::"r"(v)); \
    DTRACE(ev); \
  } while (0)
#else
#define DTRACE(ev) \
  do { \
  } while (0)
#define DTRACE_AFTER(ev, v) \
  do { \
  } while (0)
#endif

template <int D>
struct Cfg {
  static constexpr int kStages = D == 64 ? TLA_DECODE_STAGES_D64 : TLA_DECODE_STAGES_D128;
  // A cache row of D fp16 is viewed as kHalves consecutive 128-byte rows, so a
  // 64-token tile is one contiguous [kHalves * 64][64] box (16 KB for D=128).
  static constexpr int kHalves = D / 64;
  static constexpr int kTileBytes = kTile * kHalves * 128;   // K (or V) of one tile
  static constexpr int kStageBytes = 2 * kTileBytes;         // K + V
  static constexpr int kQPitch = D * 2 + 16;                 // padded row pitch of the Q tile
  static constexpr int kMinBlocks = 2;
};

struct DecodeParams {
  CUtensorMap tmap_k;
  CUtensorMap tmap_v;
  LayerArgs a;
  const void* qkv;
  const int32_t* positions;
  const void* gate;
  void* out;
  float* partial_out;  // sequence-shard mode: [B][Hq][D + 2]; null => out
  const __half* qrot;  // null, or the rotated queries [B][Hq][D] fp16 from the fused QKV projection
                       // (which also appended the new K/V): no QK-norm / RoPE / append here
  float* scratch;      // [grid][2][G][D + 2]
  int32_t* counters;   // [B * Hk], zero between launches
  long long scratch_floats, counter_count;  // extents (bounds-check builds)
  int batch, slot_offset, local_tokens, append;
  int defer_merge;  // 1: split pairs are merged by decode_merge_kernel instead of the last CTA
  int small_grid;   // CTAs for a small launch (one per SM; 0: always the whole grid), see effective_grid
};

struct SmemLayout {
  // byte offsets from the 1024-aligned base
  int stages, q, qf, kvf, cs, newkv, red, prefix, spos, bars, flags, total;
};

template <int D>
__host__ __device__ inline SmemLayout smem_layout(int G, int batch) {
  using C = Cfg<D>;
  SmemLayout s;
  int off = 0;
  s.stages = off;
  off += C::kStages * C::kStageBytes;
  s.q = off;
  off += 16 * C::kQPitch;
  s.qf = off;
  off += 16 * D * 4;
  s.kvf = off;
  off += 2 * D * 4;
  s.cs = off;
  off += D * 4;  // cos[D/2], sin[D/2]
  s.newkv = off;
  off += 2 * D * 2;
  s.red = off;
  off += kConsumerWarps * G * (D + 2) * 4;
  s.prefix = off;
  off += (batch + 1) * 4;
  s.spos = off;  // the positions, as read after the wait
  off += batch * 4;
  off = (off + 7) & ~7;
  s.bars = off;
  off += 2 * C::kStages * 8;
  s.flags = off;
  off += 16;
  s.total = off + 1024;  // alignment slack
  return s;
}

// Local slot range [lo, hi] a sequence attends over (math.ts:208 window,
// sequence-shard clipping), or lo > hi if empty.
__device__ __forceinline__ void seq_range(const LayerArgs& a, int pos, int slot_offset, int local_tokens, int* lo,
                                          int* hi) {
  const int first = a.sliding > 0 ? max(0, pos - a.sliding + 1) : 0;
  *lo = max(first, slot_offset) - slot_offset;
  *hi = min(pos, slot_offset + local_tokens - 1) - slot_offset;
}

// First unit of CTA c. The set-up runs it a few times on its critical path:
// a 32-bit division when c * total fits (c <= grid <= 16 D <= 4096), else
// 64-bit.
__device__ __forceinline__ long long cta_begin(int c, long long total, int grid) {
  if (total < (1LL << 31) / 4096)
    return static_cast<long long>(static_cast<unsigned>(c * static_cast<int>(total)) / static_cast<unsigned>(grid));
  return (static_cast<long long>(c) * total) / grid;
}

// CTAs that take part in a launch of `total` units: a small launch (fewer
// than 8 units per SM) runs on one CTA per SM, so each CTA streams more tiles
// and a pair is cut into fewer segments (measured: config 2 at batch 1); the
// decode, merge and exchange kernels all derive it from the same total.
__device__ __forceinline__ int effective_grid(long long total, int grid, int small) {
  return (small > 0 && small < grid && total < 8LL * small) ? small : grid;
}

// Largest c with cta_begin(c) <= g.
__device__ __forceinline__ int cta_of(long long g, long long total, int grid) {
  int c = total < (1LL << 31) / 4096
              ? static_cast<int>(static_cast<unsigned>(static_cast<int>(g) * grid) / static_cast<unsigned>(total))
              : static_cast<int>((g * grid) / total);
  while (c + 1 < grid && cta_begin(c + 1, total, grid) <= g) ++c;
  while (c > 0 && cta_begin(c, total, grid) > g) --c;
  return c;
}

// The stream-K split is over partition units: every (sequence, kv head) pair
// with tiles takes kSetup units before its tiles, so a CTA that starts
// several pairs (each with a query set-up and an epilogue) gets fewer tiles.
// The weights are measured optima (B200, configs 2 and 4 and their head
// shards): a pair's set-up and epilogue cost about as much as streaming
// twelve 64-token tiles at head_dim 64, four at head_dim 128.
template <int D>
struct Units {
  static constexpr int kSetup = D == 64 ? 12 : 4;
};

// The pair holding unit g of sequence b (prefix[b] <= g < prefix[b + 1]) and
// this CTA's share of it, for a CTA whose range ends at te.
struct Seg {
  int kvh, tiles, lt, n;  // n: this CTA's tiles of the pair, from tile lt (may be 0)
  long long start;        // the pair's first unit (its set-up units included)
  long long first_tile;   // the unit of its tile 0
  long long next;         // where this CTA's next pair starts
};
template <typename PT>
__device__ __forceinline__ Seg seg_at(const PT* prefix, int b, int Hk, int setup, long long g, long long te) {
  Seg sg;
  // (a sequence's units fit in 32 bits: Hk * (max_tokens / 64 + setup))
  const int per = static_cast<int>(prefix[b + 1] - prefix[b]) / Hk;  // units per pair: tiles + setup
  sg.tiles = per - setup;
  sg.kvh = static_cast<int>(g - prefix[b]) / per;
  sg.start = prefix[b] + static_cast<long long>(sg.kvh) * per;
  sg.first_tile = sg.start + setup;
  const long long end = min(te, sg.first_tile + sg.tiles);
  sg.lt = static_cast<int>(max(0LL, g - sg.first_tile));
  sg.n = static_cast<int>(max(0LL, end - (sg.first_tile + sg.lt)));
  sg.next = end;
  return sg;
}

// Tiles of a sequence at position pos in this launch (0 when the position is
// invalid; *ok says whether it was valid). With append, the new token must be the last
// local slot (always true for plain decode, where the local range is the whole
// cache).
__device__ __forceinline__ int pair_tiles(const DecodeParams& p, int pos, bool* ok_out) {
  const LayerArgs& a = p.a;
  int lo, hi;
  seq_range(a, pos, p.slot_offset, p.local_tokens, &lo, &hi);
  const bool ok = pos >= 0 && (p.partial_out != nullptr || pos < a.max_tokens) &&
                  (!p.append || (pos - p.slot_offset >= 0 && pos - p.slot_offset < a.max_tokens &&
                                 pos - p.slot_offset == hi));
  if (ok_out) *ok_out = ok;
  return ok && hi >= lo ? (hi - lo + kTile) / kTile : 0;
}

// Partition units of a sequence with `tiles` tiles per kv head (none if empty).
template <int D>
__device__ __forceinline__ int pair_units(int tiles, int Hk) {
  return tiles > 0 ? (tiles + Units<D>::kSetup) * Hk : 0;
}

// Inclusive scan of prefix[1..batch] by warp 0 (prefix[0] = 0).
__device__ __forceinline__ void scan_prefix(int* prefix, int batch, int warp, int lane) {
  if (warp != 0) return;
  int carry = 0;
  for (int base = 1; base <= batch; base += 32) {
    const int i = base + lane;
    int v = i <= batch ? prefix[i] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += n;
    }
    if (i <= batch) prefix[i] = v + carry;
    carry += __shfl_sync(0xffffffffu, v, 31);
  }
}

// L2 prefetch of the K and V boxes of this CTA's first kPrefetchTiles tiles
// under the given partition (a hint only: the tensor maps bound every box).
constexpr int kPrefetchTiles = 4;
__device__ __forceinline__ void tma_prefetch_l2_3d(const CUtensorMap* map, int x, int y, int z) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(z)
               : "memory");
}
template <int D>
__device__ __forceinline__ void prefetch_first_tiles(const DecodeParams& p, const int* prefix, int cta, int grid) {
  const long long total = prefix[p.batch];
  if (total == 0) return;
  const long long tb = cta_begin(cta, total, grid), te = cta_begin(cta + 1, total, grid);
  const int Hk = p.a.Hk;
  int b = 0, done = 0;
  for (long long g = tb; g < te && done < kPrefetchTiles;) {
    while (prefix[b + 1] <= g) ++b;
    const Seg sg = seg_at(prefix, b, Hk, Units<D>::kSetup, g, te);
    const int kvh = sg.kvh, lt = sg.lt, n = sg.n;
    int lo, hi;
    seq_range(p.a, p.positions[b], p.slot_offset, p.local_tokens, &lo, &hi);
    for (int j = lt; j < lt + n && done < kPrefetchTiles; ++j, ++done) {
      const int y = (lo + j * kTile) * Cfg<D>::kHalves, z = b * Hk + kvh;
      tma_prefetch_l2_3d(&p.tmap_k, 0, y, z);
      tma_prefetch_l2_3d(&p.tmap_v, 0, y, z);
    }
    g = sg.next;
  }
}

// L2 prefetch of the set-up inputs of this CTA's first segment (the group's
// query rows, the new K/V rows, the RoPE frequencies) by the consumer
// threads, from the speculative partition, before the wait. A hint only: L2
// receives the previous kernel's writes, so no stale line survives there.
// (An L1 prefetch after the wait was measured slower.)
template <int D, typename IO>
__device__ __forceinline__ void prefetch_first_rows(const DecodeParams& p, const int* prefix, int cta, int grid,
                                                    int tid) {
  const long long total = prefix[p.batch];
  if (total == 0) return;
  const long long tb = cta_begin(cta, total, grid), te = cta_begin(cta + 1, total, grid);
  if (tb >= te) return;
  const LayerArgs& a = p.a;
  int b = 0;
  while (prefix[b + 1] <= tb) ++b;
  const int kvh = seg_at(prefix, b, a.Hk, Units<D>::kSetup, tb, te).kvh;
  if (p.qrot != nullptr) {  // the group's rotated query rows only
    const char* q = reinterpret_cast<const char*>(p.qrot + (static_cast<size_t>(b) * a.Hq + kvh * a.G) * D);
    if (tid < a.G * D * 2 / 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(q + tid * 128));
    return;
  }
  const char* row = static_cast<const char*>(p.qkv) + static_cast<size_t>(b) * (a.Hq + 2 * a.Hk) * D * sizeof(IO);
  constexpr int kRowLines = D * sizeof(IO) / 128;  // 128-byte lines per head row (D * sizeof(IO) >= 128)
  const int q_lines = a.G * kRowLines;
  const char* addr = nullptr;
  if (tid < q_lines) {
    addr = row + (static_cast<size_t>(kvh) * a.G * D) * sizeof(IO) + tid * 128;
  } else if (tid < q_lines + 2 * kRowLines) {
    const int i = tid - q_lines, which = i / kRowLines;
    addr = row + (static_cast<size_t>(a.Hq + which * a.Hk + kvh) * D) * sizeof(IO) + (i - which * kRowLines) * 128;
  } else if (tid < q_lines + 2 * kRowLines + 2 && a.inv_freq != nullptr) {
    addr = reinterpret_cast<const char*>(a.inv_freq) + (tid - q_lines - 2 * kRowLines) * 128;
  }
  if (addr) asm volatile("prefetch.global.L2 [%0];" ::"l"(addr));
}

template <int D, typename IO, bool TWO_ROWS>
__global__ void __launch_bounds__(kThreads, Cfg<D>::kMinBlocks)
    decode_fast_kernel(const __grid_constant__ DecodeParams p) {
  using C = Cfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const LayerArgs& a = p.a;
  const int G = a.G, Hk = a.Hk, Hq = a.Hq;
  const SmemLayout L = smem_layout<D>(G, p.batch);
  int* prefix = reinterpret_cast<int*>(smem + L.prefix);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + C::kStages;
  volatile int* flags = reinterpret_cast<volatile int*>(smem + L.flags);  // [0] abort, [1] last-CTA ticket
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int launch_grid = gridDim.x, cta = blockIdx.x;
  if (tid == 0) DTRACE(0);
  if (tid == 0) {
    flags[0] = 0;
    flags[1] = 0;
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  // ---- partition: tiles per sequence, prefix over (sequence, kv head) pairs.
  // It is first built from the positions as they read while the previous
  // kernel may still be running, and only used to prefetch this CTA's first
  // tiles into L2 (a prefetch cannot return stale data: L2 is where writes
  // land); after the wait the positions are read again and the partition is
  // rebuilt only if one of them changed.
  for (int b = tid; b < p.batch; b += kThreads) prefix[b + 1] = pair_units<D>(pair_tiles(p, p.positions[b], nullptr), Hk);
  if (tid == 0) prefix[0] = 0;
  __syncthreads();
  scan_prefix(prefix, p.batch, warp, lane);
  __syncthreads();
  int grid = effective_grid(prefix[p.batch], launch_grid, p.small_grid);
  if (warp == kConsumerWarps) {
    if (lane == 0 && cta < grid) prefetch_first_tiles<D>(p, prefix, cta, grid);
  } else {
    if (cta < grid) prefetch_first_rows<D, IO>(p, prefix, cta, grid, tid);
    // rows G..15 of the query tile stay zero (the m16 MMA's padding rows)
    __half* q_pad = reinterpret_cast<__half*>(smem + L.q);
    for (int i = tid; i < (16 - G) * D; i += kConsumerWarps * 32) {
      const int r = G + i / D, d = i - (i / D) * D;
      q_pad[r * (C::kQPitch / 2) + d] = __float2half_rn(0.f);
    }
  }
  // inputs (positions, qkv, the cache, the scratch) may come from the previous
  // kernel; once they are visible, the next kernel may start its prologue
  griddep_wait();
  griddep_launch_dependents();
  int* spos = reinterpret_cast<int*>(smem + L.spos);
  bool changed = false;
  for (int b = tid; b < p.batch; b += kThreads) {
    bool ok;
    const int pos = p.positions[b];
    spos[b] = pos;
    const int tiles = pair_tiles(p, pos, &ok);
    if (!ok && cta == 0) report_error(a.error, TLA_ERR_POSITION);
    changed |= pair_units<D>(tiles, Hk) != prefix[b + 1] - prefix[b];
  }
  if (__syncthreads_or(changed)) {
    for (int b = tid; b < p.batch; b += kThreads) prefix[b + 1] = pair_units<D>(pair_tiles(p, spos[b], nullptr), Hk);
    __syncthreads();
    scan_prefix(prefix, p.batch, warp, lane);
    __syncthreads();
  }
  if (tid == 0) DTRACE(14);
  const long long total = prefix[p.batch];
  grid = effective_grid(total, launch_grid, p.small_grid);

  // Sequence-shard mode: pairs with no local tokens still emit an empty triple.
  if (p.partial_out != nullptr) {
    for (int b = cta; b < p.batch; b += grid) {
      if (prefix[b + 1] != prefix[b]) continue;
      for (int i = tid; i < Hq * (D + 2); i += kThreads) {
        const int h = i / (D + 2), e = i - h * (D + 2);
        p.partial_out[(static_cast<size_t>(b) * Hq + h) * (D + 2) + e] = e == 0 ? -INFINITY : 0.f;
      }
    }
  }
  if (tid == 0) DTRACE(1);
  if (total == 0 || cta >= grid) return;  // (CTAs past a small launch's grid have no units)
  const long long tb = cta_begin(cta, total, grid);
  const long long te = cta_begin(cta + 1, total, grid);
  if (tb >= te) return;

  uint8_t* stages = smem + L.stages;

  if (warp == kConsumerWarps) {
    // ================================================================ producer
    if (lane == 0) {
      tma_prefetch(&p.tmap_k);
      tma_prefetch(&p.tmap_v);
      uint32_t it = 0;
      int b = 0;
      for (long long g = tb; g < te;) {
        while (prefix[b + 1] <= g) ++b;
        const Seg sg = seg_at(prefix, b, Hk, Units<D>::kSetup, g, te);
        const int kvh = sg.kvh, lt = sg.lt, n = sg.n;
        int lo, hi;
        seq_range(a, spos[b], p.slot_offset, p.local_tokens, &lo, &hi);
        if (it == 0) DTRACE(13);
        for (int j = lt; j < lt + n; ++j, ++it) {
          const int s = it % C::kStages;
          const uint32_t ph = (it / C::kStages) & 1u;
          if (flags[0] || !mbar_wait(&empty[s], ph ^ 1u, a.error)) {
            flags[0] = 1;
            continue;
          }
          mbar_arrive_expect_tx(&full[s], C::kStageBytes);
          uint8_t* kst = stages + s * C::kStageBytes;
          const int y = lo + j * kTile, z = b * Hk + kvh;
          tma_load_3d(kst, &p.tmap_k, &full[s], 0, y * C::kHalves, z);
          tma_load_3d(kst + C::kTileBytes, &p.tmap_v, &full[s], 0, y * C::kHalves, z);
          if (it == 0) DTRACE(5);
        }
        g = sg.next;
      }
      // Do not leave the CTA with copies in flight: the last stages' loads
      // have landed once their full barriers completed.
      const uint32_t first = it > static_cast<uint32_t>(C::kStages) ? it - C::kStages : 0u;
      for (uint32_t i = first; i < it; ++i)
        if (!flags[0]) mbar_wait(&full[i % C::kStages], (i / C::kStages) & 1u, a.error);
    }
    return;
  }

  // ================================================================== consumers
  const IO* qkv = static_cast<const IO*>(p.qkv);
  __half* q_s = reinterpret_cast<__half*>(smem + L.q);
  float* qf = reinterpret_cast<float*>(smem + L.qf);
  float* kvf = reinterpret_cast<float*>(smem + L.kvf);
  float* cs = reinterpret_cast<float*>(smem + L.cs);
  __half* newkv = reinterpret_cast<__half*>(smem + L.newkv);
  float* red = reinterpret_cast<float*>(smem + L.red);
  const int half = a.rotary / 2;
  const float scale = a.attn_scale * kLog2e;
  const int g_row = lane >> 2, t4 = lane & 3;
  const int row_stride = (Hq + 2 * Hk) * D;
  uint32_t it = 0;
  int b = 0;

  for (long long g = tb; g < te;) {
    while (prefix[b + 1] <= g) ++b;
    const Seg sg = seg_at(prefix, b, Hk, Units<D>::kSetup, g, te);
    const int tiles = sg.tiles, kvh = sg.kvh, lt = sg.lt, n = sg.n;
    if (n == 0) {  // this CTA ends inside the pair's set-up units
      g = sg.next;
      continue;
    }
    const int pos = spos[b];
    int lo, hi;
    seq_range(a, pos, p.slot_offset, p.local_tokens, &lo, &hi);
    const int slot_new = pos - p.slot_offset;
    if (tid == 0 && it == 0) DTRACE_AFTER(15, pos);
    const bool has_new = p.append && (lt + n == tiles);
    const bool qready = p.qrot != nullptr;
    const IO* row = qready ? nullptr : qkv + static_cast<size_t>(b) * row_stride;

    // ---- segment setup: QK-norm + RoPE of the group's queries (and the new K/V)
    // All global loads of the set-up go out together (read-only path) before
    // any shared-memory store, so the set-up costs one memory round trip
    // instead of one per loop trip.
    {
      constexpr int kQPer = 16 * D / 128;  // elements per thread for up to 16 query rows
      float qv[kQPer];
      if (qready) {
        const __half* qr = p.qrot + (static_cast<size_t>(b) * Hq + kvh * G) * D;
#pragma unroll
        for (int u = 0; u < kQPer; ++u) {
          const int i = tid + 128 * u;
          qv[u] = i < G * D ? __half2float(qr[i]) : 0.f;
        }
      } else {
        const IO* qsrc = row + kvh * G * D;
#pragma unroll
        for (int u = 0; u < kQPer; ++u) {
          const int i = tid + 128 * u;
          qv[u] = i < G * D ? to_f32(__ldg(qsrc + i)) : 0.f;
        }
      }
      float kv0 = 0.f, kv1 = 0.f, kv2 = 0.f, kv3 = 0.f;  // the new K/V: D <= 256 values each
      if (has_new && (D >= 128 || tid < D)) {  // (at D = 64 a wider read would run past the last V row)
        kv0 = to_f32(__ldg(row + (Hq + kvh) * D + tid));
        kv1 = to_f32(__ldg(row + (Hq + Hk + kvh) * D + tid));
        if (D > 128 && 128 + tid < D) {
          kv2 = to_f32(__ldg(row + (Hq + kvh) * D + 128 + tid));
          kv3 = to_f32(__ldg(row + (Hq + Hk + kvh) * D + 128 + tid));
        }
      }
      const float f = (tid < half && tid < a.pair_count) ? __ldg(a.inv_freq + tid) : 0.f;
#pragma unroll
      for (int u = 0; u < kQPer; ++u) {
        const int i = tid + 128 * u;
        if (i < G * D) qf[i] = qv[u];
      }
      if (tid == 0 && it == 0) DTRACE(10);
      if (has_new) {
        if (tid < D) {
          kvf[tid] = kv0;
          kvf[D + tid] = kv1;
        }
        if (D > 128) {
          kvf[128 + tid] = kv2;
          kvf[D + 128 + tid] = kv3;
        }
      }
      if (tid < half) {  // half <= D / 2 <= 128
        float c = 1.f, sn = 0.f;
        if (tid < a.pair_count) rope_cos_sin(pos, f, &c, &sn);
        cs[tid] = c;
        cs[D / 2 + tid] = sn;
      }
      if (tid == 0 && it == 0) DTRACE(11);
    }
    named_barrier_sync(1, 128);
    if (tid == 0 && it == 0) DTRACE(7);
    for (int h = warp; h < G + 2; h += kConsumerWarps) {  // per-head RMS norms, math.ts:154-167
      const float* w;
      float* v;
      if (h < G) {
        if (a.q_norm == nullptr || qready) continue;
        w = a.q_norm;
        v = qf + h * D;
      } else if (h == G) {
        if (!has_new || a.k_norm == nullptr) continue;
        w = a.k_norm;
        v = kvf;
      } else {
        if (!has_new || !a.v_norm) continue;
        w = nullptr;
        v = kvf + D;
      }
      float ss = 0.f;
      for (int d = lane; d < D; d += 32) ss += v[d] * v[d];
      ss = warp_sum(ss);
      const float inv_rms = 1.f / sqrtf(ss / static_cast<float>(D) + a.rms_eps);
      __syncwarp();
      for (int d = lane; d < D; d += 32) {
        const float sc = w == nullptr ? 1.f : (a.offset_rms ? 1.f + w[d] : w[d]);
        v[d] = v[d] * inv_rms * sc;
      }
    }
    named_barrier_sync(1, 128);
    if (tid == 0 && it == 0) DTRACE(8);
    auto rope = [&](const float* v, int d) -> float {
      float val = v[d];
      if (d < a.rotary) {
        const int j = d < half ? d : d - half;
        if (j < a.pair_count) {
          const float partner = d < half ? -v[d + half] : v[d - half];
          val = (val * cs[j] + partner * cs[D / 2 + j]) * a.attn_factor;
        }
      }
      return val;
    };
    for (int i = tid; i < G * D; i += 128) {  // rows G..15 were zeroed at the start
      const int r = i / D, d = i - r * D;
      q_s[r * (C::kQPitch / 2) + d] = __float2half_rn(qready ? qf[r * D + d] : rope(qf + r * D, d));
    }
    if (has_new)
      for (int d = tid; d < D; d += 128) {
        newkv[d] = __float2half_rn(rope(kvf, d));
        newkv[D + d] = __float2half_rn(kvf[D + d]);
      }
    named_barrier_sync(1, 128);
    if (has_new && tid < D / 8) {  // append to the cache (copy-KV, TSLAttention.ts:280-281)
      const size_t base = ((static_cast<size_t>(b) * Hk + kvh) * a.max_tokens + slot_new) * D + tid * 8;
      if (TLA_IN_BOUNDS(base + 7, static_cast<long long>(a.max_batch) * Hk * a.max_tokens * D, a.error)) {
        reinterpret_cast<uint4*>(static_cast<__half*>(a.k_cache) + base)[0] =
            reinterpret_cast<const uint4*>(newkv)[tid];
        reinterpret_cast<uint4*>(static_cast<__half*>(a.v_cache) + base)[0] =
            reinterpret_cast<const uint4*>(newkv + D)[tid];
      }
    }
    if (tid == 0 && it == 0) DTRACE(12);
    uint32_t qa[D / 16][4];
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const int r = (lane & 7) + ((lane >> 3) & 1) * 8;
      const int ch = 2 * kk + (lane >> 4);
      ldsm_x4(smem_u32(q_s) + r * C::kQPitch + ch * 16, qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
    }

    float o[D / 8][4];
#pragma unroll
    for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    if (tid == 0 && it == 0) DTRACE(6);

    // ---- stream the segment's tiles
    for (int j = lt; j < lt + n; ++j, ++it) {
      const int s = it % C::kStages;
      const uint32_t ph = (it / C::kStages) & 1u;
      if (!flags[0] && !mbar_wait(&full[s], ph, a.error)) flags[0] = 1;
      __syncwarp();
      if (tid == 0 && it == 0) DTRACE(2);
      uint8_t* kst = stages + s * C::kStageBytes;
      uint8_t* vst = kst + C::kTileBytes;
      const int y0 = lo + j * kTile;
      const int tok0 = warp * 16;
      bool wrote = false;
      if (has_new && j == tiles - 1) {  // the new token's row holds the fresh K/V
        const int r = slot_new - y0;
        if (r >= tok0 && r < tok0 + 16 && lane < D / 8) {
          const int box = lane >> 3, ch = lane & 7;
          *reinterpret_cast<uint4*>(kst + sw128(r * C::kHalves + box, ch)) =
              reinterpret_cast<const uint4*>(newkv)[lane];
          *reinterpret_cast<uint4*>(vst + sw128(r * C::kHalves + box, ch)) =
              reinterpret_cast<const uint4*>(newkv + D)[lane];
          wrote = true;
        }
        __syncwarp();
      }
      // S = Q K^T over this warp's 16 tokens
      float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      const uint32_t kbase = smem_u32(kst);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const int tok = tok0 + (lane & 7) + ((lane >> 4) << 3);
        const int chunk = 2 * kk + ((lane >> 3) & 1);
        uint32_t r0, r1, r2, r3;
        ldsm_x4(kbase + sw128(tok * C::kHalves + (chunk >> 3), chunk & 7), r0, r1, r2, r3);
        mma_16816(acc[0], qa[kk], r0, r1);
        mma_16816(acc[1], qa[kk], r2, r3);
      }
      // mask + online softmax (log2 domain)
      float x[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int tok = y0 + tok0 + nt * 8 + 2 * t4 + (e & 1);
          x[nt][e] = tok <= hi ? acc[nt][e] * scale : -INFINITY;
        }
      float mt0 = fmaxf(fmaxf(x[0][0], x[0][1]), fmaxf(x[1][0], x[1][1]));
      mt0 = fmaxf(mt0, __shfl_xor_sync(0xffffffffu, mt0, 1));
      mt0 = fmaxf(mt0, __shfl_xor_sync(0xffffffffu, mt0, 2));
      const float mn0 = fmaxf(m0, mt0);
      const float mu0 = mn0 == -INFINITY ? 0.f : mn0;
      const float al0 = ex2(m0 - mu0);
      m0 = mn0;
      float pr[2][4];
      pr[0][0] = ex2(x[0][0] - mu0);
      pr[0][1] = ex2(x[0][1] - mu0);
      pr[1][0] = ex2(x[1][0] - mu0);
      pr[1][1] = ex2(x[1][1] - mu0);
      l0 = l0 * al0 + (pr[0][0] + pr[0][1]) + (pr[1][0] + pr[1][1]);
      float al1 = 1.f;
      if (TWO_ROWS) {
        float mt1 = fmaxf(fmaxf(x[0][2], x[0][3]), fmaxf(x[1][2], x[1][3]));
        mt1 = fmaxf(mt1, __shfl_xor_sync(0xffffffffu, mt1, 1));
        mt1 = fmaxf(mt1, __shfl_xor_sync(0xffffffffu, mt1, 2));
        const float mn1 = fmaxf(m1, mt1);
        const float mu1 = mn1 == -INFINITY ? 0.f : mn1;
        al1 = ex2(m1 - mu1);
        m1 = mn1;
        pr[0][2] = ex2(x[0][2] - mu1);
        pr[0][3] = ex2(x[0][3] - mu1);
        pr[1][2] = ex2(x[1][2] - mu1);
        pr[1][3] = ex2(x[1][3] - mu1);
        l1 = l1 * al1 + (pr[0][2] + pr[0][3]) + (pr[1][2] + pr[1][3]);
      }
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        o[i][0] *= al0;
        o[i][1] *= al0;
        if (TWO_ROWS) {
          o[i][2] *= al1;
          o[i][3] *= al1;
        }
      }
      uint32_t pa[4];
      pa[0] = pack_half2(pr[0][0], pr[0][1]);
      pa[1] = TWO_ROWS ? pack_half2(pr[0][2], pr[0][3]) : 0u;
      pa[2] = pack_half2(pr[1][0], pr[1][1]);
      pa[3] = TWO_ROWS ? pack_half2(pr[1][2], pr[1][3]) : 0u;
      // O += P V
      const uint32_t vbase = smem_u32(vst);
#pragma unroll
      for (int dd = 0; dd < D / 16; ++dd) {
        const int tok = tok0 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int chunk = 2 * dd + (lane >> 4);
        uint32_t r0, r1, r2, r3;
        ldsm_x4_t(vbase + sw128(tok * C::kHalves + (chunk >> 3), chunk & 7), r0, r1, r2, r3);
        mma_16816(o[2 * dd], pa, r0, r1);
        mma_16816(o[2 * dd + 1], pa, r2, r3);
      }
      if (wrote) fence_proxy_async_smem();  // generic writes before the next TMA into this stage
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }

    if (tid == 0) DTRACE(3);
    // ---- merge the 4 warps' (m, l, O)
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    if (TWO_ROWS) {
      l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
      l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    }
    float* rw = red + warp * G * (D + 2);
    if (g_row < G) {
      float* rr = rw + g_row * (D + 2);
      if (t4 == 0) {
        rr[0] = m0;
        rr[1] = l0;
      }
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        rr[2 + i * 8 + 2 * t4] = o[i][0];
        rr[2 + i * 8 + 2 * t4 + 1] = o[i][1];
      }
    }
    if (TWO_ROWS && g_row + 8 < G) {
      float* rr = rw + (g_row + 8) * (D + 2);
      if (t4 == 0) {
        rr[0] = m1;
        rr[1] = l1;
      }
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        rr[2 + i * 8 + 2 * t4] = o[i][2];
        rr[2 + i * 8 + 2 * t4 + 1] = o[i][3];
      }
    }
    named_barrier_sync(1, 128);
    const bool whole = (lt == 0 && n == tiles);
    const int slot = (g == tb) ? 0 : 1;
    float* mine = p.scratch + (static_cast<size_t>(cta) * 2 + slot) * G * (D + 2);
    for (int i = tid; i < G * (D + 2); i += 128) {
      const int r = i / (D + 2), e = i - r * (D + 2);
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, red[(w * G + r) * (D + 2)]);
      float v = 0.f;
      if (e == 0) {
        v = M;
      } else if (M != -INFINITY) {
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) {
          const float* rr = red + (w * G + r) * (D + 2);
          v += rr[e] * ex2(rr[0] - M);
        }
      }
      if (!whole) {
        if (TLA_IN_BOUNDS((static_cast<long long>(cta) * 2 + slot) * G * (D + 2) + i, p.scratch_floats, a.error))
          mine[i] = v;
      } else if (!TLA_IN_BOUNDS(static_cast<long long>(b) * Hq + kvh * G + r, static_cast<long long>(p.batch) * Hq,
                                a.error)) {
      } else if (p.partial_out) {
        p.partial_out[(static_cast<size_t>(b) * Hq + kvh * G + r) * (D + 2) + e] = v;
      } else if (e >= 2) {
        // out = O / l (x sigmoid(gate)); l is red-combined in the e == 1 slot
        float Lsum = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) {
          const float* rr = red + (w * G + r) * (D + 2);
          Lsum += rr[1] * ex2(rr[0] - M);
        }
        float val = v / Lsum;
        const size_t oi = (static_cast<size_t>(b) * Hq + kvh * G + r) * D + (e - 2);
        if (p.gate) val = val * (1.f / (1.f + expf(-to_f32(static_cast<const IO*>(p.gate)[oi]))));
        static_cast<IO*>(p.out)[oi] = from_f32<IO>(val);
      }
    }
    if (!whole && !p.defer_merge) {
      // ---- ticket: the CTA that completes the pair merges all its segments
      __threadfence();
      named_barrier_sync(1, 128);
      const int pair = b * Hk + kvh;
      if (tid == 0) {
        const int old = TLA_IN_BOUNDS(pair, p.counter_count, a.error) ? atomicAdd(&p.counters[pair], n) : -1;
        flags[1] = (old + n == tiles) ? 1 : 0;
      }
      named_barrier_sync(1, 128);
      if (flags[1]) {
        // Merge every segment of this pair. The loads of different segments
        // are independent, so the maxima and sums are block reductions and
        // the output rows loop over segments without serial dependences.
        __threadfence();
        const long long start = prefix[b] + static_cast<long long>(kvh) * (tiles + Units<D>::kSetup);
        const long long first_tile = start + Units<D>::kSetup;
        const int c0 = cta_of(first_tile, total, grid), c1 = cta_of(first_tile + tiles - 1, total, grid);
        // Slot of each contributing CTA (-1: empty range), computed once; qf is
        // free here and holds 16*D ints (the host keeps grid <= 16*D). A CTA
        // whose range starts at or after the pair's first unit holds the pair
        // as its first segment (slot 0), otherwise as its last (slot 1).
        int* slot_of = reinterpret_cast<int*>(qf);
        for (int c = c0 + tid; c <= c1; c += 128) {
          const long long cb = cta_begin(c, total, grid);
          slot_of[c - c0] = cta_begin(c + 1, total, grid) == cb ? -1 : c * 2 + (cb >= start ? 0 : 1);
        }
        named_barrier_sync(1, 128);
        auto seg = [&](int c) -> const float* {  // this pair's triple block in CTA c's scratch, or null
          const int sl = slot_of[c - c0];
          if (sl < 0 || !TLA_IN_BOUNDS((static_cast<long long>(sl) + 1) * G * (D + 2) - 1, p.scratch_floats, a.error))
            return nullptr;
          return p.scratch + static_cast<size_t>(sl) * G * (D + 2);
        };
        float lm[16], ll[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
          lm[r] = -INFINITY;
          ll[r] = 0.f;
        }
        for (int c = c0 + tid; c <= c1; c += 128) {
          const float* sp = seg(c);
          if (sp == nullptr) continue;
#pragma unroll
          for (int r = 0; r < 16; ++r)
            if (r < G) lm[r] = fmaxf(lm[r], __ldcg(sp + r * (D + 2)));
        }
        float* sred = red;                     // [4][G] maxima
        float* sM = red + 8 * G;               // [G] merged maxima
#pragma unroll
        for (int r = 0; r < 16; ++r) {
          if (r < G) {
            float v = lm[r];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
            if (lane == 0) sred[warp * G + r] = v;
          }
        }
        named_barrier_sync(1, 128);
        if (tid < G)
          sM[tid] = fmaxf(fmaxf(sred[tid], sred[G + tid]), fmaxf(sred[2 * G + tid], sred[3 * G + tid]));
        named_barrier_sync(1, 128);
        for (int c = c0 + tid; c <= c1; c += 128) {
          const float* sp = seg(c);
          if (sp == nullptr) continue;
#pragma unroll
          for (int r = 0; r < 16; ++r)
            if (r < G) ll[r] += __ldcg(sp + r * (D + 2) + 1) * ex2(__ldcg(sp + r * (D + 2)) - sM[r]);
        }
        float* ssum = red + 4 * G;             // [4][G] sums
        float* sL = red + 9 * G;               // [G] merged sums
#pragma unroll
        for (int r = 0; r < 16; ++r) {
          if (r < G) {
            const float v = warp_sum(ll[r]);
            if (lane == 0) ssum[warp * G + r] = v;
          }
        }
        named_barrier_sync(1, 128);
        if (tid < G) sL[tid] = (ssum[tid] + ssum[G + tid]) + (ssum[2 * G + tid] + ssum[3 * G + tid]);
        named_barrier_sync(1, 128);
        for (int i = tid; i < G * D; i += 128) {
          const int r = i / D, d = i - r * D;
          const float M = sM[r];
          float acc = 0.f;
#pragma unroll 8
          for (int c = c0; c <= c1; ++c) {
            const float* sp = seg(c);
            if (sp == nullptr) continue;
            const float* row = sp + r * (D + 2);
            acc += __ldcg(row + 2 + d) * ex2(__ldcg(row) - M);
          }
          const size_t hrow = static_cast<size_t>(b) * Hq + kvh * G + r;
          if (p.partial_out) {
            p.partial_out[hrow * (D + 2) + 2 + d] = acc;
            if (d == 0) {
              p.partial_out[hrow * (D + 2)] = M;
              p.partial_out[hrow * (D + 2) + 1] = sL[r];
            }
          } else {
            float val = acc / sL[r];
            const size_t oi = hrow * D + d;
            if (p.gate) val = val * (1.f / (1.f + expf(-to_f32(static_cast<const IO*>(p.gate)[oi]))));
            static_cast<IO*>(p.out)[oi] = from_f32<IO>(val);
          }
        }
        if (tid == 0 && TLA_IN_BOUNDS(pair, p.counter_count, a.error)) p.counters[pair] = 0;
      }
    }
    named_barrier_sync(1, 128);  // red / q_s / flags reuse by the next segment
    g = min(te, prefix[b] + static_cast<long long>(kvh) * (tiles + Units<D>::kSetup) + Units<D>::kSetup + tiles);
  }
  if (tid == 0) DTRACE(4);
}

// Deferred merge for pairs split across many CTAs (few, long sequences): one
// block of 4 warps per (pair, query row); when a pair spans 64 or more CTAs
// (one long sequence per kv head: up to the whole grid), one block of 16 warps
// per (pair, query row, 32-column slice), so D / 32 times more SMs read the
// segments. The segment table (the scratch slot of every contributing CTA)
// is built in shared memory before the decode kernel has finished; then, in
// one pass, warp w folds segments w, w + NT / 32, ... into a running triple
// (maximum, sum, this lane's output columns) with 8 or 12 segments' loads in
// flight at a time, and the warps' triples are combined through shared memory.
// Pairs covered by a single CTA were written by the decode kernel and are
// skipped.
constexpr int kMaxGrid = 16 * 128;  // the host keeps decode_grid <= 16 * D
constexpr int kMergeThreads = 128;

template <int D, typename IO, int NT>
__global__ void __launch_bounds__(NT) decode_merge_kernel(const __grid_constant__ DecodeParams p,
                                                                     int grid) {
  constexpr int kWarps = NT / 32;
  // 16-warp blocks take one 32-column slice of the row each (D / 32 blocks per
  // row), so a pair split over the whole grid is read by D / 32 times more SMs
  constexpr bool kSliced = NT >= 512;
  constexpr int kSlices = kSliced ? D / 32 : 1;
  constexpr int kCols = D / kSlices;  // output columns of this block
  constexpr int kPer = kCols / 32;    // output columns per lane (float2 loads when 2)
  __shared__ long long prefix[kMaxBatch + 1];
  __shared__ int seg_slot[kMaxGrid];   // scratch slot of segment k, -1 if none
  __shared__ float red[2][kWarps];
  __shared__ float rows_s[kWarps][kCols];
  // The next kernel may launch as soon as every block of this one is
  // resident: it can only start its own prologue (its griddepcontrol.wait
  // waits for this grid to complete), and these blocks need no more resources
  // to finish, so its CTAs can take the SMs that the decode kernel frees and
  // start their L2 prefetches early.
  griddep_launch_dependents();
  const LayerArgs& a = p.a;
  const int G = a.G, Hk = a.Hk;
  const int slice = static_cast<int>(blockIdx.x) % kSlices, row_id = static_cast<int>(blockIdx.x) / kSlices;
  const int pair = row_id / G, r = row_id - pair * G;
  const int b = pair / Hk, kvh = pair - b * Hk;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // the decode kernel's partition, recomputed: tile counts in parallel, then a serial scan
  for (int bb = tid; bb < p.batch; bb += NT) {
    const int pos = p.positions[bb];
    int lo, hi;
    seq_range(a, pos, p.slot_offset, p.local_tokens, &lo, &hi);
    const bool ok = pos >= 0 && (p.partial_out != nullptr || pos < a.max_tokens) &&
                    (!p.append || (pos - p.slot_offset >= 0 && pos - p.slot_offset < a.max_tokens &&
                                   pos - p.slot_offset == hi));
    prefix[bb + 1] = pair_units<D>((ok && hi >= lo) ? (hi - lo + kTile) / kTile : 0, Hk);
  }
  __syncthreads();
  if (tid == 0) {
    long long acc = 0;
    prefix[0] = 0;
    for (int bb = 1; bb <= p.batch; ++bb) {
      acc += prefix[bb];
      prefix[bb] = acc;
    }
  }
  __syncthreads();
  const long long total = prefix[p.batch];
  grid = effective_grid(total, grid, p.small_grid);  // as the decode kernel took it
  if (prefix[b + 1] == prefix[b]) return;  // no tiles
  const Seg sg = seg_at(prefix, b, Hk, Units<D>::kSetup, prefix[b] + (prefix[b + 1] - prefix[b]) / Hk * kvh, total);
  const int tiles = sg.tiles;
  const int c0 = cta_of(sg.first_tile, total, grid), c1 = cta_of(sg.first_tile + tiles - 1, total, grid);
  if (c0 == c1) return;  // one CTA held the whole pair
  const int S = c1 - c0 + 1;
  // the segment table (computed before the decode kernel has finished)
  for (int k = tid; k < S; k += NT) {
    const int c = c0 + k;
    const long long cb = cta_begin(c, total, grid);
    seg_slot[k] = cta_begin(c + 1, total, grid) == cb ? -1 : c * 2 + (cb >= sg.start ? 0 : 1);
  }
  __syncthreads();
  griddep_wait();  // the decode kernel's segments are complete and visible
  // One pass: warp w folds segments w, w + NT / 32, ... with a running
  // maximum (the online softmax across segments), loading the triples of kB
  // segments at once; then the warps' partial triples are combined.
  constexpr int kB = kSliced ? 12 : 8;
  const float* rowp = p.scratch + static_cast<size_t>(r) * (D + 2);
  const size_t slot_stride = static_cast<size_t>(G) * (D + 2);
  float mw = -INFINITY, lw = 0.f;
  float acc[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) acc[j] = 0.f;
  for (int k = warp; k < S; k += kB * kWarps) {
    float mk[kB], lk[kB], v[kB][kPer];
#pragma unroll
    for (int u = 0; u < kB; ++u) {
      const int ku = k + u * kWarps;
      int sl = ku < S ? seg_slot[ku] : -1;
      if (sl >= 0 && !TLA_IN_BOUNDS((static_cast<long long>(sl) + 1) * G * (D + 2) - 1, p.scratch_floats, a.error))
        sl = -1;
      mk[u] = -INFINITY;
      lk[u] = 0.f;
#pragma unroll
      for (int j = 0; j < kPer; ++j) v[u][j] = 0.f;
      if (sl >= 0) {
        const float* sp = rowp + static_cast<size_t>(sl) * slot_stride;
        mk[u] = __ldcg(sp);
        lk[u] = __ldcg(sp + 1);
        if constexpr (kPer >= 2) {
#pragma unroll
          for (int j = 0; j < kPer / 2; ++j) {
            const float2 t = __ldcg(reinterpret_cast<const float2*>(sp + 2) + lane + 32 * j);
            v[u][2 * j] = t.x;
            v[u][2 * j + 1] = t.y;
          }
        } else {
          v[u][0] = __ldcg(sp + 2 + slice * kCols + lane);
        }
      }
    }
    float mb = mw;
#pragma unroll
    for (int u = 0; u < kB; ++u) mb = fmaxf(mb, mk[u]);
    if (mb == -INFINITY) continue;
    const float sc = mw == -INFINITY ? 0.f : ex2(mw - mb);
    lw *= sc;
#pragma unroll
    for (int j = 0; j < kPer; ++j) acc[j] *= sc;
#pragma unroll
    for (int u = 0; u < kB; ++u) {
      const float w = mk[u] == -INFINITY ? 0.f : ex2(mk[u] - mb);
      lw += lk[u] * w;
#pragma unroll
      for (int j = 0; j < kPer; ++j) acc[j] += v[u][j] * w;
    }
    mw = mb;
  }
  if (lane == 0) {
    red[0][warp] = mw;
    red[1][warp] = lw;
  }
  if constexpr (kPer >= 2) {
#pragma unroll
    for (int j = 0; j < kPer / 2; ++j) {
      rows_s[warp][2 * (lane + 32 * j)] = acc[2 * j];
      rows_s[warp][2 * (lane + 32 * j) + 1] = acc[2 * j + 1];
    }
  } else {
    rows_s[warp][lane] = acc[0];
  }
  __syncthreads();
  float M = red[0][0];
#pragma unroll
  for (int w = 1; w < kWarps; ++w) M = fmaxf(M, red[0][w]);
  float wt[kWarps];
  float L = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    wt[w] = red[0][w] == -INFINITY ? 0.f : ex2(red[0][w] - M);
    L += red[1][w] * wt[w];
  }
  const size_t hrow = static_cast<size_t>(b) * a.Hq + kvh * G + r;
  if (!TLA_IN_BOUNDS(hrow, static_cast<long long>(p.batch) * a.Hq, a.error)) return;
  for (int c = tid; c < kCols; c += NT) {
    float o = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) o += rows_s[w][c] * wt[w];
    const int d = slice * kCols + c;
    if (p.partial_out) {
      p.partial_out[hrow * (D + 2) + 2 + d] = o;
      if (d == 0) {
        p.partial_out[hrow * (D + 2)] = M;
        p.partial_out[hrow * (D + 2) + 1] = L;
      }
    } else {
      float val = o / L;
      const size_t oi = hrow * D + d;
      if (p.gate) val = val * (1.f / (1.f + expf(-to_f32(static_cast<const IO*>(p.gate)[oi]))));
      static_cast<IO*>(p.out)[oi] = from_f32<IO>(val);
    }
  }
}

// Sequence-shard decode fused with the peer exchange: one 4-warp block per
// SM walks query rows (b, h). For each row it merges this rank's split-KV
// segments exactly like decode_merge_kernel (or takes the triple the decode
// kernel wrote when one CTA held the whole pair), stores the row's triple
// into every rank's exchange buffer, and after all its rows are out, gathers
// every rank's triple of each row and writes the log-sum-exp merge.
template <int D, typename IO>
__global__ void __launch_bounds__(kMergeThreads) decode_exchange_kernel(const __grid_constant__ DecodeParams p,
                                                                        int grid, ExchangeDev x) {
  constexpr int kWarps = kMergeThreads / 32;
  constexpr int kPer = D / 32;
  constexpr int W = D + 2;
  __shared__ long long prefix[kMaxBatch + 1];
  __shared__ int seg_slot[kMaxGrid];
  __shared__ float seg_w[kMaxGrid];
  __shared__ float seg_l[kMaxGrid];
  __shared__ float red[2][kWarps];
  __shared__ float rows_s[kWarps][D];
  __shared__ __align__(16) float trip[W];
  __shared__ __align__(16) float vals[kXchMaxRanks * W];
  __shared__ int epoch_s;
  __shared__ float wts[kXchMaxRanks];
  __shared__ float ls;
  const LayerArgs& a = p.a;
  const int G = a.G, Hk = a.Hk, Hq = a.Hq;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int bb = tid; bb < p.batch; bb += kMergeThreads) {
    const int pos = p.positions[bb];
    int lo, hi;
    seq_range(a, pos, p.slot_offset, p.local_tokens, &lo, &hi);
    const bool ok = pos >= 0 && (!p.append || (pos - p.slot_offset >= 0 && pos - p.slot_offset < a.max_tokens &&
                                                pos - p.slot_offset == hi));
    prefix[bb + 1] = pair_units<D>((ok && hi >= lo) ? (hi - lo + kTile) / kTile : 0, Hk);
  }
  __syncthreads();
  if (tid == 0) {
    long long acc = 0;
    prefix[0] = 0;
    for (int bb = 1; bb <= p.batch; ++bb) {
      acc += prefix[bb];
      prefix[bb] = acc;
    }
  }
  griddep_wait();  // the decode kernel's segments are complete and visible
  griddep_launch_dependents();
  const unsigned epoch = xch_epoch(x, &epoch_s);  // syncs the block
  const long long total = prefix[p.batch];
  grid = effective_grid(total, grid, p.small_grid);  // as the decode kernel took it
  const int rows = p.batch * Hq;
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const int b = row / Hq, h = row - b * Hq, kvh = h / G, r = h - kvh * G;
    const bool empty = prefix[b + 1] == prefix[b];
    Seg sg{};
    if (!empty)
      sg = seg_at(prefix, b, Hk, Units<D>::kSetup, prefix[b] + (prefix[b + 1] - prefix[b]) / Hk * kvh, total);
    const int tiles = empty ? 0 : sg.tiles;
    const int c0 = tiles ? cta_of(sg.first_tile, total, grid) : 0;
    const int c1 = tiles ? cta_of(sg.first_tile + tiles - 1, total, grid) : 0;
    if (tiles == 0 || c0 == c1) {  // written by the decode kernel (empty pair: m = -inf)
      for (int e = tid; e < W; e += kMergeThreads) trip[e] = __ldcg(p.partial_out + static_cast<size_t>(row) * W + e);
    } else {
      const int S = c1 - c0 + 1;
      float m = -INFINITY;
      for (int k = tid; k < S; k += kMergeThreads) {
        const int c = c0 + k;
        const long long cb = cta_begin(c, total, grid);
        const int sl = cta_begin(c + 1, total, grid) == cb ? -1 : c * 2 + (cb >= sg.start ? 0 : 1);
        seg_slot[k] = sl;
        float mk = -INFINITY, lk = 0.f;
        if (sl >= 0) {
          const float* sp = p.scratch + (static_cast<size_t>(sl) * G + r) * W;
          mk = __ldcg(sp);
          lk = __ldcg(sp + 1);
        }
        seg_w[k] = mk;
        seg_l[k] = lk;
        m = fmaxf(m, mk);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane == 0) red[0][warp] = m;
      __syncthreads();
      float M = red[0][0];
#pragma unroll
      for (int w = 1; w < kWarps; ++w) M = fmaxf(M, red[0][w]);
      float l = 0.f;
      for (int k = tid; k < S; k += kMergeThreads) {
        const float w = (seg_slot[k] < 0 || M == -INFINITY) ? 0.f : ex2(seg_w[k] - M);
        seg_w[k] = w;
        l += seg_l[k] * w;
      }
      l = warp_sum(l);
      if (lane == 0) red[1][warp] = l;
      __syncthreads();
      const float2* col = reinterpret_cast<const float2*>(p.scratch + static_cast<size_t>(r) * W + 2) + lane;
      const size_t slot_stride2 = static_cast<size_t>(G) * W / 2;
      float2 acc[kPer / 2];
#pragma unroll
      for (int j = 0; j < kPer / 2; ++j) acc[j] = make_float2(0.f, 0.f);
      int k = warp;
      for (; k + 7 * kWarps < S; k += 8 * kWarps) {  // eight segments' loads in flight
        float2 v[8][kPer / 2];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int sl = seg_slot[k + u * kWarps];
#pragma unroll
          for (int j = 0; j < kPer / 2; ++j)
            v[u][j] = sl >= 0 ? __ldcg(col + static_cast<size_t>(sl) * slot_stride2 + j * 32) : make_float2(0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float w = seg_w[k + u * kWarps];
#pragma unroll
          for (int j = 0; j < kPer / 2; ++j) {
            acc[j].x += v[u][j].x * w;
            acc[j].y += v[u][j].y * w;
          }
        }
      }
      for (; k < S; k += kWarps) {
        const int sl = seg_slot[k];
        if (sl < 0) continue;
        const float w = seg_w[k];
#pragma unroll
        for (int j = 0; j < kPer / 2; ++j) {
          const float2 v = __ldcg(col + static_cast<size_t>(sl) * slot_stride2 + j * 32);
          acc[j].x += v.x * w;
          acc[j].y += v.y * w;
        }
      }
#pragma unroll
      for (int j = 0; j < kPer / 2; ++j) {
        rows_s[warp][2 * (lane + 32 * j)] = acc[j].x;
        rows_s[warp][2 * (lane + 32 * j) + 1] = acc[j].y;
      }
      __syncthreads();
      for (int d = tid; d < D; d += kMergeThreads) {
        float o = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) o += rows_s[w][d];
        trip[2 + d] = o;
      }
      if (tid == 0) {
        trip[0] = M;
        trip[1] = red[1][0] + red[1][1] + red[1][2] + red[1][3];
      }
    }
    __syncthreads();
    xch_push_row(x, epoch, row, trip, W);
    __syncthreads();  // trip and the segment tables are reused by the next row
  }
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    xch_gather_row(x, epoch, row, W, vals, a.error);
    xch_merge_row<IO>(vals, x.ranks, D, p.gate ? static_cast<const IO*>(p.gate) + static_cast<size_t>(row) * D : nullptr,
                      static_cast<IO*>(p.out) + static_cast<size_t>(row) * D, wts, &ls);
  }
  xch_finish(x, epoch);
}

template <int D, typename IO, bool TWO>
cudaError_t launch_t(const tla_layer* L, const DecodeParams& p, const ExchangeDev* x, cudaStream_t stream) {
  const SmemLayout s = smem_layout<D>(L->G, p.batch);
  cudaError_t e = launch_pdl(decode_fast_kernel<D, IO, TWO>, L->decode_grid, kThreads, s.total, stream, p);
  if (e != cudaSuccess) return e;
  if (x != nullptr) {
    const int rows = p.batch * L->Hq;
    const int grid = rows < L->ctx->sm_count ? rows : L->ctx->sm_count;
    return launch_pdl(decode_exchange_kernel<D, IO>, grid, kMergeThreads, 0, stream, p, L->decode_grid, *x);
  }
  if (!p.defer_merge) return e;
  const int pairs = p.batch * L->Hk;
  if (L->decode_grid >= 64 * pairs)  // 16 warps per block, one 32-column slice per block
    return launch_pdl(decode_merge_kernel<D, IO, 512>, pairs * L->G * (D / 32), 512, 0, stream, p, L->decode_grid);
  return launch_pdl(decode_merge_kernel<D, IO, kMergeThreads>, pairs * L->G, kMergeThreads, 0, stream, p,
                    L->decode_grid);
}

template <int D, typename IO, bool TWO>
cudaError_t configure_t(tla_layer* L, int* blocks) {
  // A launch of `batch` sequences uses smem_layout(G, batch) <= this layer's
  // worst case; the limit is shared with every other layer on this instance.
  const SmemLayout s = smem_layout<D>(L->G, L->max_batch);
  const void* k = reinterpret_cast<const void*>(decode_fast_kernel<D, IO, TWO>);
  cudaError_t e = raise_smem_limit(k, s.total);
  if (e != cudaSuccess) return e;
  L->decode_smem = s.total;
  return cached_occupancy(k, kThreads, s.total, blocks);
}

template <int D>
cudaError_t dispatch_configure(tla_layer* L, int* blocks) {
  const bool two = L->G > 8;
  if (L->io_fp32) return two ? configure_t<D, float, true>(L, blocks) : configure_t<D, float, false>(L, blocks);
  return two ? configure_t<D, __half, true>(L, blocks) : configure_t<D, __half, false>(L, blocks);
}

template <int D>
cudaError_t dispatch_launch(const tla_layer* L, const DecodeParams& p, const ExchangeDev* x, cudaStream_t stream) {
  const bool two = L->G > 8;
  if (L->io_fp32)
    return two ? launch_t<D, float, true>(L, p, x, stream) : launch_t<D, float, false>(L, p, x, stream);
  return two ? launch_t<D, __half, true>(L, p, x, stream) : launch_t<D, __half, false>(L, p, x, stream);
}

CUresult make_cache_map(const tla_layer* L, void* base, CUtensorMap* map) {
  // 3-D view of the cache with 128-byte rows: x = 64 fp16 of a row half,
  // y = (token slot, half), z = (sequence, kv head)
  const cuuint64_t halves = static_cast<cuuint64_t>(L->D / 64);
  const cuuint64_t dims[3] = {64, halves * L->max_tokens, static_cast<cuuint64_t>(L->max_batch) * L->Hk};
  const cuuint64_t strides[2] = {128, 128 * halves * L->max_tokens};
  const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(kTile * halves), 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return L->ctx->encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, base, dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

}  // namespace

cudaError_t decode_fast_configure(tla_layer* L) {
  L->fast_decode = false;
  if (L->cache_fp32 || (L->D != 64 && L->D != 128) || L->Hq % L->Hk != 0 || L->G > 16 ||
      L->max_batch > kMaxBatch || L->ctx->encode_tiled == nullptr)
    return cudaSuccess;
  if (make_cache_map(L, L->k_cache, &L->tmap_k) != CUDA_SUCCESS ||
      make_cache_map(L, L->v_cache, &L->tmap_v) != CUDA_SUCCESS)
    return cudaSuccess;  // fall back to the generic path
  int blocks = 0;
  cudaError_t e = L->D == 64 ? dispatch_configure<64>(L, &blocks) : dispatch_configure<128>(L, &blocks);
  if (e != cudaSuccess) return e;
  if (blocks <= 0) return cudaSuccess;
#ifdef TLA_DECODE_CTAS_PER_SM
  if (blocks > TLA_DECODE_CTAS_PER_SM) blocks = TLA_DECODE_CTAS_PER_SM;
#endif
  L->decode_grid = blocks * L->ctx->sm_count;
  if (L->decode_grid > 16 * L->D) L->decode_grid = 16 * L->D;  // merge slot table lives in the 16*D-float Q staging
  L->fast_decode = true;
  return cudaSuccess;
}

size_t decode_fast_scratch_floats(const tla_layer* L) {
  return static_cast<size_t>(L->decode_grid) * 2 * L->G * (L->D + 2);
}

namespace {
DecodeParams decode_params(const tla_layer* L, const void* qkv, const int32_t* positions, const void* gate, void* out,
                           float* partial, int batch, int slot_offset, int local_tokens, int append) {
  DecodeParams p;
  p.tmap_k = L->tmap_k;
  p.tmap_v = L->tmap_v;
  p.a = layer_args(L);
  p.qkv = qkv;
  p.qrot = nullptr;
  p.positions = positions;
  p.gate = gate;
  p.out = out;
  p.partial_out = partial;
  p.scratch = L->ctx->d_partials;
  p.counters = L->ctx->d_counters;
  p.scratch_floats = static_cast<long long>(L->ctx->partial_floats);
  p.counter_count = static_cast<long long>(L->ctx->counter_count);
  p.batch = batch;
  p.slot_offset = slot_offset;
  p.local_tokens = local_tokens;
  p.append = append;
  // Few, long sequences split each (sequence, kv head) over many CTAs: merge
  // those in a separate, fully parallel kernel instead of in the last CTA.
  p.defer_merge = L->decode_grid > TLA_DEFER_MERGE_SEGMENTS * batch * L->Hk ? 1 : 0;
  p.small_grid = L->decode_grid > L->ctx->sm_count ? L->ctx->sm_count : 0;
  return p;
}
}  // namespace

cudaError_t launch_decode_fast(const tla_layer* L, const void* qkv, const int32_t* positions, const void* gate,
                               void* out, float* partial, int batch, int slot_offset, int local_tokens, int append,
                               cudaStream_t stream) {
  const DecodeParams p = decode_params(L, qkv, positions, gate, out, partial, batch, slot_offset, local_tokens, append);
  return L->D == 64 ? dispatch_launch<64>(L, p, nullptr, stream) : dispatch_launch<128>(L, p, nullptr, stream);
}

cudaError_t launch_decode_fast_qrot(const tla_layer* L, const __half* qrot, const int32_t* positions, const void* gate,
                                    void* out, int batch, cudaStream_t stream) {
  DecodeParams p = decode_params(L, nullptr, positions, gate, out, nullptr, batch, 0, L->max_tokens, 0);
  p.qrot = qrot;
  return L->D == 64 ? dispatch_launch<64>(L, p, nullptr, stream) : dispatch_launch<128>(L, p, nullptr, stream);
}

cudaError_t launch_decode_exchange(const tla_layer* L, const ExchangeDev& x, const void* qkv,
                                   const int32_t* positions, const void* gate, void* out, float* partial, int batch,
                                   int slot_offset, int local_tokens, int append, cudaStream_t stream) {
  DecodeParams p = decode_params(L, qkv, positions, gate, out, partial, batch, slot_offset, local_tokens, append);
  p.defer_merge = 1;  // the segments are merged by decode_exchange_kernel
  return L->D == 64 ? dispatch_launch<64>(L, p, &x, stream) : dispatch_launch<128>(L, p, &x, stream);
}

}  // namespace tla

// ============================================================================
// Allocation-free decode: the same persistent split-KV kernel, with its
// scratch in a fixed static device array instead of memory owned by a tla_ctx.
// ============================================================================
namespace tla {
namespace {

// Per-device static scratch (every GPU that loads the library holds it until exit):
//   [0, 64 KiB)            completion counters, int32[kStaticMaxPairs]
//   [64 KiB, +256)         status word used when the caller passes none
//   [+256, +512)           RoPE inverse frequencies, float[64]
//   [+512, 8 MiB)          split-KV partial triples
constexpr size_t kStaticScratchBytes = size_t(8) << 20;
constexpr int kStaticMaxPairs = 16384;  // batch * kv_head_count
constexpr size_t kStaticStatusOff = size_t(kStaticMaxPairs) * 4;
constexpr size_t kStaticInvFreqOff = kStaticStatusOff + 256;
constexpr size_t kStaticPartialOff = kStaticInvFreqOff + 256;
constexpr int kStaticMaxDevices = 64;

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

struct StaticScratchSlot {
  std::once_flag once;
  cudaError_t status = cudaSuccess;
  unsigned char* ptr = nullptr;
};
StaticScratchSlot g_static_slots[kStaticMaxDevices];
std::once_flag g_static_encode_once;
PFN_cuTensorMapEncodeTiled_v12000 g_static_encode = nullptr;

// The RoPE table travels by value in the kernel parameters, so no host
// buffer has to outlive the call.
struct InvFreqTable {
  float v[64];
};
__global__ void store_inv_freq_kernel(float* dst, InvFreqTable t) { dst[threadIdx.x] = t.v[threadIdx.x]; }

}  // namespace
}  // namespace tla

extern "C" int tla_decode_noalloc(const tla_attn_config* cfg, void* key_cache, void* value_cache,
                                  const float* q_norm_weight, const float* k_norm_weight, const void* qkv,
                                  const int32_t* positions, const void* gate, void* out, int32_t* status,
                                  int32_t batch, void* stream) {
  using namespace tla;
  if (!cfg || !key_cache || !value_cache || !qkv || !positions || !out || batch < 0) return TLA_ERR_INVALID_ARG;
  const int Hq = cfg->head_count, D = cfg->head_dim;
  const int Hk = cfg->kv_head_count > 0 ? cfg->kv_head_count : Hq;
  if (Hq <= 0 || D <= 0 || Hk > Hq || cfg->max_tokens <= 0 || cfg->max_batch <= 0 || batch > cfg->max_batch ||
      cfg->sliding_window < 0)
    return TLA_ERR_INVALID_ARG;
  // Only the shapes of the fast kernel: fp16 cache, head_dim 64/128, GQA group <= 16.
  if ((cfg->flags & TLA_FLAG_CACHE_FP32) || (D != 64 && D != 128) || Hq % Hk != 0 || Hq / Hk > 16 ||
      cfg->max_batch > kMaxBatch)
    return TLA_ERR_UNSUPPORTED;
  if (static_cast<long long>(batch) * Hk > kStaticMaxPairs) return TLA_ERR_SCRATCH_LIMIT;
  const int rotary = cfg->rotary_dim < 0 ? D : cfg->rotary_dim;
  if (rotary % 2 != 0 || rotary > D) return TLA_ERR_ROTARY_DIM;
  const bool rope_on = cfg->rope_theta > 0 && rotary > 0;
  const int freq_dim = cfg->rope_freq_dim > 0 ? cfg->rope_freq_dim : rotary;
  const int pair_count = cfg->rope_pair_count >= 0 ? cfg->rope_pair_count : rotary / 2;
  InvFreqTable inv = {};
  double af = 1;
  if (rope_on) {
    if (freq_dim / 2 > 64) return TLA_ERR_UNSUPPORTED;
    const int rc = tla_rope_parameters(freq_dim, cfg->rope_theta, &cfg->rope_scaling, inv.v, &af);
    if (rc != TLA_OK) return rc;
    if (pair_count > freq_dim / 2) return TLA_ERR_INVALID_ARG;
  }
  if (batch == 0) return TLA_OK;

  // One-time set-up per device, with that device current: the device address
  // of the static array (its name is only a stand-in in host code).
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kStaticMaxDevices) return TLA_ERR_NO_DEVICE;
  StaticScratchSlot& slot = g_static_slots[dev];
  std::call_once(slot.once, [&slot] {
    slot.status = cudaGetSymbolAddress(reinterpret_cast<void**>(&slot.ptr), g_static_scratch);
  });
  if (slot.status != cudaSuccess || slot.ptr == nullptr) return TLA_ERR_CUDA;
  std::call_once(g_static_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_static_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (g_static_encode == nullptr) return TLA_ERR_CUDA;

  // Host-side descriptions only: nothing below allocates device memory.
  tla_ctx ctx;
  ctx.device = dev;
  if (cudaDeviceGetAttribute(&ctx.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return TLA_ERR_CUDA;
  ctx.d_error = status ? status : reinterpret_cast<int*>(slot.ptr + kStaticStatusOff);
  ctx.d_counters = reinterpret_cast<int32_t*>(slot.ptr);
  ctx.counter_count = kStaticMaxPairs;
  ctx.d_partials = reinterpret_cast<float*>(slot.ptr + kStaticPartialOff);
  ctx.partial_floats = (kStaticScratchBytes - kStaticPartialOff) / sizeof(float);
  ctx.encode_tiled = g_static_encode;
  tla_layer L;
  L.ctx = &ctx;
  L.cfg = *cfg;
  L.Hq = Hq;
  L.Hk = Hk;
  L.D = D;
  L.G = Hq / Hk;
  L.max_tokens = cfg->max_tokens;
  L.max_batch = cfg->max_batch;
  L.rotary = rope_on ? rotary : 0;
  L.freq_half = rope_on ? freq_dim / 2 : 0;
  L.pair_count = rope_on ? (pair_count < rotary / 2 ? pair_count : rotary / 2) : 0;
  L.sliding = cfg->sliding_window;
  L.attn_scale = static_cast<float>(cfg->has_attn_scale ? cfg->attn_scale : 1 / sqrt(static_cast<double>(D)));
  L.attn_factor = static_cast<float>(af);
  L.rms_eps = static_cast<float>(cfg->rms_epsilon > 0 ? cfg->rms_epsilon : 1e-6);
  L.io_fp32 = (cfg->flags & TLA_FLAG_IO_FP32) != 0;
  L.v_norm = (cfg->flags & TLA_FLAG_V_NORM) != 0;
  L.offset_rms = (cfg->flags & TLA_FLAG_OFFSET_RMS_NORM) != 0;
  L.k_cache = key_cache;
  L.v_cache = value_cache;
  L.d_inv_freq = reinterpret_cast<float*>(slot.ptr + kStaticInvFreqOff);
  L.d_qnorm = const_cast<float*>(q_norm_weight);
  L.d_knorm = const_cast<float*>(k_norm_weight);
  if (decode_fast_configure(&L) != cudaSuccess || !L.fast_decode) return TLA_ERR_UNSUPPORTED;
  const int per_cta = 2 * L.G * (D + 2);
  const int max_grid = static_cast<int>(ctx.partial_floats / per_cta);
  if (max_grid < 1) return TLA_ERR_SCRATCH_LIMIT;
  if (L.decode_grid > max_grid) L.decode_grid = max_grid;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The array keeps the previous call's contents: reload the RoPE table and
  // zero the completion counters this launch uses.
  store_inv_freq_kernel<<<1, 64, 0, st>>>(L.d_inv_freq, inv);
  if (cudaGetLastError() != cudaSuccess) return TLA_ERR_CUDA;
  if (cudaMemsetAsync(ctx.d_counters, 0, sizeof(int32_t) * batch * Hk, st) != cudaSuccess) return TLA_ERR_CUDA;
  const cudaError_t e =
      launch_decode_fast(&L, qkv, positions, gate, out, nullptr, batch, 0, cfg->max_tokens, 1, st);
  return e == cudaSuccess ? TLA_OK : TLA_ERR_CUDA;
}

#ifdef TLA_DECODE_TRACE
extern "C" int tla_debug_decode_trace(unsigned long long* host, int count) {
  return cudaMemcpyFromSymbol(host, tla::g_decode_trace, sizeof(unsigned long long) * count) == cudaSuccess ? 0 : -1;
}
#endif
