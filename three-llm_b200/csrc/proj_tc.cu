// Dense projections on the 5th-generation tensor cores (tcgen05): fp16
// operands fed by TMA, fp32 accumulation in TMEM, with the attention's front
// and back ends fused into the epilogue.
//
//  - QKV projection (TSLLinear, packages/three-llm/src/tsl/TSLLinear.ts:56-75;
//    CPU linear, runtime/math.ts:6-25; wired at decoder/DecoderTSLRunner.ts:
//    293-297): [Q | K | V] = x W + bias, then per head the QK-norm and RoPE
//    at the row's position (TSLAttention.ts:168-304), K and V (vNorm)
//    appended to the cache (copy-KV, :252-286) and the rotated queries handed
//    to the attention kernel, so the raw [Q | K | V] rows never reach HBM.
//  - Output projection and residual (DecoderTSLRunner.ts:299-309, 353-356:
//    the attnProj TSLLinear, then TSLAdd): y = residual + attn W_o + bias, or
//    one rank's fp32 partial product when the heads are sharded.
//
// Tile: 128 rows (the TMEM lanes) x NT columns (64..256; whole heads for the
// QKV epilogue), the reduction dimension in 64-element stages. Warp 0 lane 0
// issues the TMA loads of x (K-major, 128-byte swizzle) and W (stored
// [in][out], i.e. MN-major for the MMA's B operand, in 64-column boxes) into a
// ring of shared-memory stages; warp 1 owns TMEM and its lane 0 issues
// tcgen05.mma (M = 128, N = NT, K = 16) per stage and commits the stage back
// to the producer; then all four warps run the epilogue, thread = row = TMEM
// lane. Every mbarrier wait is bounded (TLA_ERR_TIMEOUT).
#include <math.h>

#include "exchange.cuh"
#include "tcgen05.cuh"
#include "tla_device.cuh"
#include "tla_internal.h"

namespace tla {

namespace {

constexpr int kThreads = 256;  // warps 0-3: TMA / MMA, then epilogue; all 8 warps run the epilogue
constexpr int kXStage = 128 * 128;  // x: 128 rows x 64 fp16 (one 128-byte row each)
constexpr int kWBox = 64 * 128;     // W: 64 rows of the reduction dim x 64 fp16 columns
enum : int { kQkvDecode = 0, kQkvPrefill = 1, kOutProj = 2, kOutPush = 3 };


struct ProjParams {
  CUtensorMap tm_x;  // [rows][K] fp16, box {64, 128}
  CUtensorMap tm_w;  // [K][N] fp16, box {64, 64}
  int rows, K, N, NT, stages, m_tiles;
  uint32_t tmem_cols;
  int mode;
  const float* bias;  // [N] or null
  int* error;
  // QKV modes
  LayerArgs a;
  const int32_t* pos;  // decode: positions [B]; prefill: start positions [B]
  int S;               // prefill: tokens per sequence
  __half* qout;        // decode: [B][Hq][D]; prefill: [B][Hq][S][D] (the prefill kernel's TMA source)
  // output projection
  const void* residual;  // [rows][N] or null
  void* y;               // [rows][N]
  int y_f32, res_f32;    // float32 (else fp16) output / residual
  // head-sharded output projection: the partial tile goes over NVLink to the
  // rank that owns its columns (cols = hidden / ranks each), as {value, epoch}
  // words in that rank's exchange buffer, slot [this rank], first half
  ExchangeDev x;
  int cols;
  // split-K (few rows, decode): ksplit CTAs share a tile; each adds its fp32
  // partial into ws [rows][N] and the last one (tile_cnt ticket) runs the
  // epilogue from ws and zeroes it again
  int ksplit;
  float* ws;
  int* tile_cnt;  // [m_tiles * (N / NT)], zero between launches
};

#ifdef TLA_PROJ_TRACE
// Optional per-CTA timeline (builds with -DTLA_PROJ_TRACE only): globaltimer at
// [cta][0] entry, [1] after the dependency wait, [2] accumulator complete,
// [3] split-K partial added and ticket taken, [4] epilogue tables ready,
// [5] exit of a CTA that ran the epilogue, [6] QKV: a head's values loaded,
// [7] its rotated rows stored; read with tla_debug_proj_trace.
__device__ unsigned long long g_proj_trace[1024][8];
#define PRTRACE(ev)                                                                       \
  do {                                                                                    \
    if (threadIdx.x == 0 && blockIdx.x < 1024) g_proj_trace[blockIdx.x][(ev)] = globaltimer(); \
  } while (0)
// out_allreduce_kernel per CTA: [0] entry, [1] after the wait, [2] own block
// summed and sent, [3] exit; read with tla_debug_allreduce_trace
__device__ unsigned long long g_ar_trace[256][4];
#define ARTRACE(ev)                                                                     \
  do {                                                                                  \
    if (threadIdx.x == 0 && blockIdx.x < 256) g_ar_trace[blockIdx.x][(ev)] = globaltimer(); \
  } while (0)
#else
#define PRTRACE(ev) \
  do {              \
  } while (0)
#define ARTRACE(ev) \
  do {              \
  } while (0)
#endif

__host__ __device__ inline int stage_bytes(int NT) { return kXStage + (NT / 64) * kWBox; }

template <int D>
__host__ __device__ inline int epilogue_bytes(int mode) {
  return mode >= kOutProj ? 0 : 3 * 128 * (D + 1) * 4;  // each row's cos / sin, and its head values per warp set
}

// Bytes below the barriers: the stage ring, and the epilogue's tables and
// rows, which reuse it.
template <int D>
__host__ __device__ inline int region_bytes(int ring, int mode) {
  const int epi = epilogue_bytes<D>(mode);
  return ring > epi ? ring : epi;
}

template <int D>
__global__ void __launch_bounds__(kThreads, 2) proj_tc_kernel(const __grid_constant__ ProjParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int sb = stage_bytes(p.NT);
  const int ring = p.stages * sb;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + region_bytes<D>(ring, p.mode));
  uint64_t* empty = full + p.stages;
  uint64_t* accb = empty + p.stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accb + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_tiles = p.N / p.NT;
  const int tile = static_cast<int>(blockIdx.x) % (p.m_tiles * n_tiles);
  const int ks = static_cast<int>(blockIdx.x) / (p.m_tiles * n_tiles);
  const int m0 = (tile % p.m_tiles) * 128;
  const int n0 = (tile / p.m_tiles) * p.NT;
  const int kc_all = (p.K + 63) / 64;
  const int kc0 = (ks * kc_all) / p.ksplit, kc1 = ((ks + 1) * kc_all) / p.ksplit;
  const int kchunks = kc1 - kc0;  // this CTA's 64-element chunks of the reduction dim
  PRTRACE(0);
  if (tid == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accb, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(p.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();  // x, positions and the residual may come from the previous kernel
  PRTRACE(1);
  __shared__ int epoch_s;
  const unsigned epoch = p.mode == kOutPush ? xch_epoch(p.x, &epoch_s) : 0u;  // (block-uniform branch)
  auto wait = [&](uint64_t* bar, uint32_t parity) {
    if (*abort_flag) return;
    if (!mbar_wait(bar, parity, p.error)) *abort_flag = 1;
  };
  // QKV modes: this thread's tile row position (threads 0-127, one row each;
  // -1: no row, or a position outside the cache), loaded now so that its
  // latency overlaps the mainloop.
  __shared__ int row_pos[128];
  int my_pos = -1;
  if ((p.mode == kQkvDecode || p.mode == kQkvPrefill) && tid < 128 && m0 + tid < p.rows) {
    const int grow = m0 + tid;
    if (p.mode == kQkvDecode) {
      my_pos = p.pos[grow];
    } else {
      const int bb = grow / p.S;
      my_pos = p.pos[bb] + (grow - bb * p.S);
    }
    if (my_pos < 0 || my_pos >= p.a.max_tokens) my_pos = -1;
  }
  // The rows' positions into row_pos and, for a tile of Q or K heads, their
  // RoPE factors at tbl + r (D + 1): cos [half], sin [half]. Each factor is
  // one dependent chain, so all threads share them.
  auto fill_rope = [&](float* tbl) {
    const LayerArgs& a = p.a;
    if (tid < 128) row_pos[tid] = my_pos;
    __syncthreads();
    const int half = a.rotary / 2;
    if (half == 0 || n0 / D >= a.Hq + a.Hk) return;  // V heads: no RoPE
    for (int e = tid; e < 128 * half; e += kThreads) {  // entry (row rr, pair i) at index rr half + i
      const int rr = e / half, i = e - rr * half;
      if (m0 + rr >= p.rows) break;  // rows only grow with e
      const int ps = row_pos[rr];
      if (ps < 0) continue;
      float c = 1.f, sn = 0.f;
      if (i < a.pair_count) rope_cos_sin(ps, __ldg(a.inv_freq + i), &c, &sn);
      float* cr = tbl + rr * (D + 1);
      cr[i] = c;
      cr[half + i] = sn;
    }
  };

  if (warp == 0 && lane == 0) {
    // ---------------------------------------------------------------- TMA producer
    tma_prefetch(&p.tm_x);
    tma_prefetch(&p.tm_w);
    for (int c = 0; c < kchunks; ++c) {
      const int s = c % p.stages;
      wait(&empty[s], ((c / p.stages) & 1) ^ 1);
      if (*abort_flag) continue;
      uint8_t* st = smem + s * sb;
      mbar_arrive_expect_tx(&full[s], sb);
      const int kx = (kc0 + c) * 64;
      tma_load_2d(st, &p.tm_x, &full[s], kx, m0);
      for (int i = 0; i < p.NT / 64; ++i) tma_load_2d(st + kXStage + i * kWBox, &p.tm_w, &full[s], n0 + 64 * i, kx);
    }
    for (int c = kchunks > p.stages ? kchunks - p.stages : 0; c < kchunks; ++c)  // no copies in flight at exit
      wait(&full[c % p.stages], (c / p.stages) & 1);
  } else if (warp == 1 && lane == 0) {
    // ---------------------------------------------------------------- MMA issuer
    const uint32_t idesc = idesc_f16(128, p.NT, true);
    // Descriptors are linear in the start address (no carry below 256 KB):
    // stage and k-step offsets are plain adds. x: K-major, 32 bytes per k-step;
    // W: MN-major, 64-column boxes kWBox apart, 16 rows (2048 bytes) per k-step.
    const uint64_t dx = sdesc(smem_u32(smem), 16, 1024);
    const uint64_t dw = sdesc(smem_u32(smem + kXStage), kWBox, 1024);
    for (int c = 0; c < kchunks; ++c) {
      const int s = c % p.stages;
      wait(&full[s], (c / p.stages) & 1);
      tc_fence_after();
      if (!*abort_flag) {
        const uint64_t so = static_cast<uint64_t>((s * sb) >> 4);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) mma_f16(tmem, dx + so + kk * 2, dw + so + kk * 128, idesc, (c | kk) ? 1u : 0u);
      }
      mma_commit(&empty[s]);
    }
    mma_commit(accb);
  }
  __syncwarp();
  wait(accb, 0);
  __syncwarp();
  tc_fence_after();
  PRTRACE(2);

  // Epilogue: thread = row (TMEM lane) in each of two warp sets (warps 0-3 and
  // 4-7 read the same lanes), which take alternate 32-column chunks or heads.
  const int set = warp >> 2, r = tid & 127, row = m0 + r;
  const bool valid = row < p.rows;
  const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
  if (p.ksplit > 1) {
    // The output projection's epilogue inputs that do not depend on the
    // other splits (this row's residual and bias columns) are brought into L1
    // now, so that the last CTA's epilogue waits only on the workspace.
    if (p.mode == kOutProj && valid) {
      for (int c = set; c < p.NT / 32; c += 2) {
        const size_t o = static_cast<size_t>(row) * p.N + n0 + 32 * c;
        if (p.residual) {
          const char* rp = static_cast<const char*>(p.residual) + o * (p.res_f32 ? 4 : 2);
          asm volatile("prefetch.global.L1 [%0];" ::"l"(rp));
          if (p.res_f32) asm volatile("prefetch.global.L1 [%0];" ::"l"(rp + 64));
        }
        if (p.bias && r == 0) asm volatile("prefetch.global.L1 [%0];" ::"l"(p.bias + n0 + 32 * c));
      }
    }
    // add this CTA's partial tile into the workspace; the last CTA of the tile
    // goes on to the epilogue, reading the complete sums from the workspace
    for (int c = set; c < p.NT / 32; c += 2) {
      float v[32];
      tmem_ld32(lane_base + 32 * c, v);
      if (!valid || !TLA_IN_BOUNDS(static_cast<long long>(row) * p.N + n0 + 32 * c + 31,
                                   static_cast<long long>(p.rows) * p.N, p.error))
        continue;
      float* dst = p.ws + static_cast<size_t>(row) * p.N + n0 + 32 * c;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst + 4 * i), "f"(v[4 * i]),
                     "f"(v[4 * i + 1]), "f"(v[4 * i + 2]), "f"(v[4 * i + 3])
                     : "memory");
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) epoch_s = atomicAdd(p.tile_cnt + tile, 1) == p.ksplit - 1 ? 1 : 0;
    __syncthreads();
    const bool last = epoch_s != 0;
    PRTRACE(3);
    __syncthreads();  // epoch_s is reused by the push epilogue
    if (!last) {
      tc_fence_before();
      __syncthreads();
      if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(p.tmem_cols) : "memory");
      }
      return;
    }
    __threadfence();
    if (tid == 0) p.tile_cnt[tile] = 0;
  }
  // The tile's accumulator columns [c0, c0 + 32) of this thread's row: from
  // TMEM (warp-collective), or, split-K, from the workspace.
  auto load_acc = [&](int c0, float (&v)[32]) {
    if (p.ksplit == 1) {
      tmem_ld32(lane_base + c0, v);
    } else if (valid) {
      const float4* src = reinterpret_cast<const float4*>(p.ws + static_cast<size_t>(row) * p.N + n0 + c0);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 q = __ldcg(src + i);
        v[4 * i] = q.x;
        v[4 * i + 1] = q.y;
        v[4 * i + 2] = q.z;
        v[4 * i + 3] = q.w;
      }
    }
  };
  // Split-K: zero the workspace columns [c0, c0 + 32) of this thread's row
  // for the next launch once they have been read (kept apart from the loads,
  // so that no store waits behind a load of the same address).
  auto clear_acc = [&](int c0) {
    if (p.ksplit == 1 || !valid) return;
    float4* dst = reinterpret_cast<float4*>(p.ws + static_cast<size_t>(row) * p.N + n0 + c0);
#pragma unroll
    for (int i = 0; i < 8; ++i) __stcg(dst + i, make_float4(0.f, 0.f, 0.f, 0.f));
  };
  // bias columns [c0, c0 + 32) of the tile (zeros without a bias)
  const bool bias_v4 = (reinterpret_cast<uintptr_t>(p.bias) & 15) == 0;
  auto load_bias = [&](int c0, float (&bv)[32]) {
    if (p.bias == nullptr) {
#pragma unroll
      for (int i = 0; i < 32; ++i) bv[i] = 0.f;
    } else if (bias_v4) {
      const float4* src = reinterpret_cast<const float4*>(p.bias + n0 + c0);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 q = __ldg(src + i);
        bv[4 * i] = q.x;
        bv[4 * i + 1] = q.y;
        bv[4 * i + 2] = q.z;
        bv[4 * i + 3] = q.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) bv[i] = __ldg(p.bias + n0 + c0 + i);
    }
  };
  if (p.mode == kQkvDecode || p.mode == kQkvPrefill) {
    // ---------------------------------------------------------------- QKV epilogue
    const LayerArgs& a = p.a;
    constexpr int kRow = D + 1;  // padded row of the tables (floats)
    float* const tbl = reinterpret_cast<float*>(smem);  // over the stage ring
    fill_rope(tbl);
    __syncthreads();
    PRTRACE(4);
    int b = 0, t = 0;
    const int pos = row_pos[r];
    if (valid) {
      if (p.mode == kQkvDecode) {
        b = row;
      } else {
        b = row / p.S;
        t = row - b * p.S;
      }
    }
    const bool ok = valid && pos >= 0;
    if (valid && !ok && n0 == 0 && set == 0) report_error(a.error, TLA_ERR_POSITION);  // the row is skipped
    float* cs = tbl + r * kRow;  // cos [half], sin [half]
    float* hrow = reinterpret_cast<float*>(smem) + (1 + set) * 128 * kRow + r * kRow;  // padded rows
    const int half = a.rotary / 2;
    const int head0 = n0 / D, heads = p.NT / D;
    const bool full_rope = a.rotary == D && a.pair_count == D / 2;
    for (int j = set; j < heads; j += 2) {
      const int hh = head0 + j;
      float ss = 0.f;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float v[32], bv[32];
        load_acc(j * D + 32 * c, v);  // TMEM: warp-collective, every lane loads
        load_bias(j * D + 32 * c, bv);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float x = v[i] + bv[i];
          hrow[32 * c + i] = x;
          ss += x * x;
        }
      }
#pragma unroll
      for (int c = 0; c < D / 32; ++c) clear_acc(j * D + 32 * c);
      PRTRACE(6);
      if (!ok) continue;
      const bool isq = hh < a.Hq, isk = !isq && hh < a.Hq + a.Hk;
      const float* w = isq ? a.q_norm : (isk ? a.k_norm : nullptr);
      const bool norm = (isq || isk) ? w != nullptr : a.v_norm != 0;  // rmsNormPackedHeads, math.ts:154-167
      const float inv = norm ? 1.f / sqrtf(ss / static_cast<float>(D) + a.rms_eps) : 1.f;
      auto val = [&](int d) -> float {
        float x = hrow[d] * inv;
        if (w) x *= a.offset_rms ? 1.f + __ldg(w + d) : __ldg(w + d);
        return x;
      };
      __half* dst;
      long long di, dn;  // element offset of dst and the buffer's extent (bounds-check builds)
      if (isq) {
        di = p.mode == kQkvDecode ? (static_cast<long long>(b) * a.Hq + hh) * D
                                  : ((static_cast<long long>(b) * a.Hq + hh) * p.S + t) * D;
        dn = static_cast<long long>(p.rows) * a.Hq * D;
        dst = p.qout + di;
      } else {
        di = ((static_cast<long long>(b) * a.Hk + (hh - a.Hq) % a.Hk) * a.max_tokens + pos) * D;
        dn = static_cast<long long>(a.max_batch) * a.Hk * a.max_tokens * D;
        dst = static_cast<__half*>(isk ? a.k_cache : a.v_cache) + di;
      }
      if (!TLA_IN_BOUNDS(di + D - 1, dn, a.error)) continue;
      const bool rope = (isq || isk) && half > 0;
      if (rope && full_rope) {
        // rotate-half RoPE over the whole head (math.ts:134-147), dims i and
        // i + D/2 together, branch-free
#pragma unroll
        for (int i0 = 0; i0 < D / 2; i0 += 8) {
          uint32_t lo[4], hi[4];
#pragma unroll
          for (int e = 0; e < 8; e += 2) {
            float l2[2], h2[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int i = i0 + e + u;
              const float x = val(i), y = val(i + D / 2), c = cs[i], sn = cs[D / 2 + i];
              l2[u] = (x * c - y * sn) * a.attn_factor;
              h2[u] = (y * c + x * sn) * a.attn_factor;
            }
            lo[e / 2] = pack_half2(l2[0], l2[1]);
            hi[e / 2] = pack_half2(h2[0], h2[1]);
          }
          *reinterpret_cast<uint4*>(dst + i0) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
          *reinterpret_cast<uint4*>(dst + D / 2 + i0) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        }
        PRTRACE(7);
        continue;
      }
      for (int d0 = 0; d0 < D; d0 += 8) {
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          float y[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int d = d0 + e + u;
            float x = val(d);
            if (rope && d < a.rotary) {  // rotate-half RoPE, math.ts:134-147 (partial rotary / pair count)
              const int jj = d < half ? d : d - half;
              if (jj < a.pair_count) {
                const float partner = d < half ? -val(d + half) : val(d - half);
                x = (x * cs[jj] + partner * cs[half + jj]) * a.attn_factor;
              }
            }
            y[u] = x;
          }
          pk[e / 2] = pack_half2(y[0], y[1]);
        }
        *reinterpret_cast<uint4*>(dst + d0) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
    }
  } else if (p.mode == kOutPush) {
    // ---------------------------------------------------------------- partial tile -> its owner over NVLink
    const int owner = n0 / p.cols;  // NT divides cols: the tile lies in one owner's block
    uint8_t* dst = p.x.peers[owner] + static_cast<size_t>(epoch & 1u) * p.x.region_bytes;
    const size_t word0 = static_cast<size_t>(p.x.rank) * p.x.slot_words + static_cast<size_t>(row) * p.cols +
                         (n0 - owner * p.cols);
    for (int c = set; c < p.NT / 32; c += 2) {
      float v[32];
      load_acc(32 * c, v);
      if (!valid) continue;
#pragma unroll
      for (int i = 0; i < 16; ++i)
        xch_st_v4(dst + (word0 + 32 * c + 2 * i) * 8,
                  make_uint4(__float_as_uint(v[2 * i]), epoch, __float_as_uint(v[2 * i + 1]), epoch));
      clear_acc(32 * c);
    }
  } else {
    // ---------------------------------------------------------------- output projection epilogue
    for (int c = set; c < p.NT / 32; c += 2) {
      float v[32], bv[32];
      load_acc(32 * c, v);
      load_bias(32 * c, bv);
      if (!valid) continue;
      const int col = n0 + 32 * c;
      const size_t o = static_cast<size_t>(row) * p.N + col;
      if (!TLA_IN_BOUNDS(o + 31, static_cast<long long>(p.rows) * p.N, p.error)) continue;
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] += bv[i];
      if (p.residual) {
        if (p.res_f32) {
          const float4* res = reinterpret_cast<const float4*>(static_cast<const float*>(p.residual) + o);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 q = res[i];
            v[4 * i] += q.x;
            v[4 * i + 1] += q.y;
            v[4 * i + 2] += q.z;
            v[4 * i + 3] += q.w;
          }
        } else {
          const uint4* res = reinterpret_cast<const uint4*>(static_cast<const __half*>(p.residual) + o);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint4 q = res[i];
            const __half2* h = reinterpret_cast<const __half2*>(&q);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              v[8 * i + 2 * k] += __low2float(h[k]);
              v[8 * i + 2 * k + 1] += __high2float(h[k]);
            }
          }
        }
      }
      if (p.y_f32) {
        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.y) + o);
#pragma unroll
        for (int i = 0; i < 8; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
      } else {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(p.y) + o);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          dst[i] = make_uint4(pack_half2(v[8 * i], v[8 * i + 1]), pack_half2(v[8 * i + 2], v[8 * i + 3]),
                              pack_half2(v[8 * i + 4], v[8 * i + 5]), pack_half2(v[8 * i + 6], v[8 * i + 7]));
      }
      clear_acc(32 * c);
    }
  }
  PRTRACE(5);
  griddep_launch_dependents();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(p.tmem_cols) : "memory");
  }
}

CUresult make_map_2d(const tla_ctx* ctx, const void* base, uint64_t inner, uint64_t outer, uint32_t box_outer,
                     CUtensorMap* map) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {inner * 2};
  const cuuint32_t box[2] = {64, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return ctx->encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

// Widest tile (<= 256 columns, a multiple of `unit` dividing N) that still gives
// every SM a tile; the narrowest if none does (few rows: decode, where split-K
// then supplies the CTAs; a wider tile there was measured slower, its split-K
// sums being larger than the weights it saves reading as wider row pieces).
int choose_nt(int N, int unit, int m_tiles, int sms) {
  int best = 0;
  for (int nt = unit; nt <= 256; nt += unit) {
    if (N % nt) continue;
    if (best == 0 || static_cast<long long>(m_tiles) * (N / nt) >= sms) best = nt;
  }
  return best;
}

template <int D>
cudaError_t launch_proj_t(tla_ctx* ctx, ProjParams& p, cudaStream_t stream) {
  const int sb = stage_bytes(p.NT);
  const int n_tiles = p.N / p.NT, tiles = p.m_tiles * n_tiles, kc_all = (p.K + 63) / 64;
  // Few tiles (decode rows): split the reduction dimension so that about two
  // CTAs per SM stream the weights (4 stages each, so two fit on an SM).
  p.ksplit = 1;
  if (tiles < ctx->sm_count && kc_all >= 4) {
    int ks = (2 * ctx->sm_count) / tiles;  // one resident wave at two CTAs per SM
    if (ks > kc_all / 2) ks = kc_all / 2;  // at least two 64-element chunks per CTA
    if (ks > 1) {
      const size_t ws = static_cast<size_t>(p.rows) * p.N;
      if (ensure_proj_workspace(ctx, ws, tiles) == cudaSuccess) {
        p.ksplit = ks;
        p.ws = ctx->d_proj_ws;
        p.tile_cnt = ctx->d_proj_cnt;
      }
    }
  }
  int stages = p.ksplit > 1 ? 4 : (200 * 1024) / sb;
  if (stages > 8) stages = 8;
  if (stages < 2) stages = 2;
  p.stages = stages;
  p.tmem_cols = p.NT <= 64 ? 64 : (p.NT <= 128 ? 128 : 256);
  const int ring = stages * sb;
  const int smem = region_bytes<D>(ring, p.mode) + (2 * stages + 1) * 8 + 16 + 1024;
  const void* k = reinterpret_cast<const void*>(proj_tc_kernel<D>);
  cudaError_t e = raise_smem_limit(k, smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(proj_tc_kernel<D>, static_cast<unsigned>(tiles * p.ksplit), kThreads, smem, stream, p);
}

// Second half of the head-sharded output projection, one CTA per SM at most
// (every CTA a peer waits for is resident), with blocks wide enough (up to
// 512 threads) that each thread has about one pair: each thread takes pairs
// of this rank's column block, loads the pair's bias and residual, waits
// (bounded) for every rank's partial words of the pair, sums them in rank
// order, adds bias and residual, keeps the result and stores it into slot
// [this rank], second half, of every rank's buffer; then it collects the
// other ranks' finished blocks. Every CTA finishes its own block's pairs
// before it waits on another rank's.
template <typename OUT>
__global__ void __launch_bounds__(512) out_allreduce_kernel(ExchangeDev x, int rows, int hidden, int cols,
                                                            const float* __restrict__ bias, const void* residual,
                                                            int res_f32, OUT* __restrict__ y, int* error) {
  __shared__ int epoch_s;
  ARTRACE(0);
  griddep_wait();  // the partial tiles of this rank's GEMM are out
  ARTRACE(1);
  const unsigned epoch = xch_epoch(x, &epoch_s);
  const uint8_t* mine = x.peers[x.rank] + static_cast<size_t>(epoch & 1u) * x.region_bytes;
  volatile int* abort_p = reinterpret_cast<volatile int*>(x.peers[x.rank] + 2 * x.region_bytes + 256);
  const size_t half_words = static_cast<size_t>(rows) * cols;  // second half of a slot
  const int pairs = static_cast<int>(half_words / 2);
  const int stride = static_cast<int>(gridDim.x * blockDim.x);
  auto wait_words = [&](uint4 (&w)[kXchMaxRanks], size_t word) {  // every rank's word of a pair
    auto load = [&](int r) { return xch_ld_v4(mine + (static_cast<size_t>(r) * x.slot_words + word) * 8); };
#pragma unroll
    for (int r = 0; r < kXchMaxRanks; ++r)
      if (r < x.ranks) w[r] = load(r);
    unsigned long long t0 = 0;
    for (;;) {
      bool done = true;
#pragma unroll
      for (int r = 0; r < kXchMaxRanks; ++r)
        if (r < x.ranks && (w[r].y != epoch || w[r].w != epoch)) {
          done = false;
          w[r] = load(r);
        }
      if (done || *abort_p == static_cast<int>(epoch)) return;
      const unsigned long long now = globaltimer();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > kWaitLimitNs) {
        report_error(error, TLA_ERR_TIMEOUT);
        *abort_p = static_cast<int>(epoch);
        return;
      }
    }
  };
  auto store = [&](int row, int col, float v0, float v1) {
    const size_t o = static_cast<size_t>(row) * hidden + col;
    if constexpr (sizeof(OUT) == 4)
      *reinterpret_cast<float2*>(y + o) = make_float2(v0, v1);
    else
      *reinterpret_cast<uint32_t*>(y + o) = pack_half2(v0, v1);
  };
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < pairs; i += stride) {
    const int row = (2 * i) / cols, lc = 2 * i - row * cols, col = x.rank * cols + lc;
    // bias and residual first: their loads overlap the wait for the partial words
    float b0 = 0.f, b1 = 0.f;
    if (bias) {
      b0 = __ldg(bias + col);
      b1 = __ldg(bias + col + 1);
    }
    if (residual) {
      const size_t o = static_cast<size_t>(row) * hidden + col;
      if (res_f32) {
        const float2 q = *reinterpret_cast<const float2*>(static_cast<const float*>(residual) + o);
        b0 += q.x;
        b1 += q.y;
      } else {
        const __half2 q = *reinterpret_cast<const __half2*>(static_cast<const __half*>(residual) + o);
        b0 += __low2float(q);
        b1 += __high2float(q);
      }
    }
    uint4 w[kXchMaxRanks];
    wait_words(w, static_cast<size_t>(2 * i));
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int r = 0; r < kXchMaxRanks; ++r)
      if (r < x.ranks) {
        s0 += __uint_as_float(w[r].x);
        s1 += __uint_as_float(w[r].z);
      }
    s0 += b0;
    s1 += b1;
    store(row, col, s0, s1);
    const uint4 out = make_uint4(__float_as_uint(s0), epoch, __float_as_uint(s1), epoch);
    const size_t word = static_cast<size_t>(x.rank) * x.slot_words + half_words + 2 * i;
    for (int q = 0; q < x.ranks; ++q)
      if (q != x.rank) xch_st_v4(x.peers[q] + static_cast<size_t>(epoch & 1u) * x.region_bytes + word * 8, out);
  }
  ARTRACE(2);
  for (int q = 0; q < x.ranks; ++q) {
    if (q == x.rank) continue;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < pairs; i += stride) {
      const int row = (2 * i) / cols, lc = 2 * i - row * cols;
      const uint8_t* src = mine + (static_cast<size_t>(q) * x.slot_words + half_words + 2 * i) * 8;
      uint4 w = xch_ld_v4(src);
      unsigned long long t0 = 0;
      while ((w.y != epoch || w.w != epoch) && *abort_p != static_cast<int>(epoch)) {
        const unsigned long long now = globaltimer();
        if (t0 == 0) {
          t0 = now;
        } else if (now - t0 > kWaitLimitNs) {
          report_error(error, TLA_ERR_TIMEOUT);
          *abort_p = static_cast<int>(epoch);
          break;
        }
        w = xch_ld_v4(src);
      }
      store(row, q * cols + lc, __uint_as_float(w.x), __uint_as_float(w.z));
    }
  }
  xch_finish(x, epoch);
  ARTRACE(3);
}

}  // namespace

cudaError_t launch_out_proj_allreduce(tla_ctx* ctx, const ExchangeDev& x, const void* attn,
                                      const void* weight, const float* bias, const void* residual, bool f32, void* y,
                                      int rows, int in_features, int hidden, cudaStream_t stream) {
  ProjParams p{};
  if (make_map_2d(ctx, attn, in_features, rows, 128, &p.tm_x) != CUDA_SUCCESS ||
      make_map_2d(ctx, weight, hidden, in_features, 64, &p.tm_w) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  p.rows = rows;
  p.K = in_features;
  p.N = hidden;
  p.cols = hidden / x.ranks;
  p.m_tiles = (rows + 127) / 128;
  p.NT = choose_nt(p.cols, 64, p.m_tiles * x.ranks, ctx->sm_count);  // NT divides an owner's block
  if (p.NT == 0) return cudaErrorInvalidValue;
  p.mode = kOutPush;
  p.error = ctx->d_error;
  p.x = x;
  cudaError_t e = launch_proj_t<64>(ctx, p, stream);
  if (e != cudaSuccess) return e;
  const int pairs = rows * p.cols / 2;
  int block = 128;  // widened until one pass of the grid covers every pair (at most 512)
  while (block < 512 && static_cast<long long>(block) * ctx->sm_count < pairs) block *= 2;
  int grid = (pairs + block - 1) / block;
  if (grid > ctx->sm_count) grid = ctx->sm_count;
  if (f32)
    return launch_pdl(out_allreduce_kernel<float>, static_cast<unsigned>(grid), static_cast<unsigned>(block), 0,
                      stream, x, rows, hidden, p.cols, bias, residual, 1, static_cast<float*>(y), ctx->d_error);
  return launch_pdl(out_allreduce_kernel<__half>, static_cast<unsigned>(grid), static_cast<unsigned>(block), 0,
                    stream, x, rows, hidden, p.cols, bias, residual, 0, static_cast<__half*>(y), ctx->d_error);
}

cudaError_t launch_qkv_proj(const tla_layer* L, const void* x, const void* weight, const float* bias, int hidden,
                            const int32_t* pos, int rows, int seq_len, bool prefill, __half* qout,
                            cudaStream_t stream) {
  ProjParams p{};
  const int N = (L->Hq + 2 * L->Hk) * L->D;
  if (make_map_2d(L->ctx, x, hidden, rows, 128, &p.tm_x) != CUDA_SUCCESS ||
      make_map_2d(L->ctx, weight, N, hidden, 64, &p.tm_w) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  p.rows = rows;
  p.K = hidden;
  p.N = N;
  p.m_tiles = (rows + 127) / 128;
  p.NT = choose_nt(N, L->D, p.m_tiles, L->ctx->sm_count);
#ifdef TLA_QKV_SPLIT_NT
  if (p.m_tiles * (N / p.NT) < L->ctx->sm_count && N % TLA_QKV_SPLIT_NT == 0 && TLA_QKV_SPLIT_NT % L->D == 0)
    p.NT = TLA_QKV_SPLIT_NT;
#endif
  if (p.NT == 0) return cudaErrorInvalidValue;
  p.mode = prefill ? kQkvPrefill : kQkvDecode;
  p.bias = bias;
  p.error = L->ctx->d_error;
  p.a = layer_args(L);
  p.pos = pos;
  p.S = seq_len;
  p.qout = qout;
  return L->D == 64 ? launch_proj_t<64>(L->ctx, p, stream) : launch_proj_t<128>(L->ctx, p, stream);
}

cudaError_t launch_out_proj(tla_ctx* ctx, const void* attn, const void* weight, const float* bias,
                            const void* residual, bool residual_f32, void* y, bool y_f32, int rows, int in_features,
                            int hidden, cudaStream_t stream) {
  ProjParams p{};
  if (make_map_2d(ctx, attn, in_features, rows, 128, &p.tm_x) != CUDA_SUCCESS ||
      make_map_2d(ctx, weight, hidden, in_features, 64, &p.tm_w) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  p.rows = rows;
  p.K = in_features;
  p.N = hidden;
  p.m_tiles = (rows + 127) / 128;
  p.NT = choose_nt(hidden, 64, p.m_tiles, ctx->sm_count);
  if (p.NT == 0) return cudaErrorInvalidValue;
  p.mode = kOutProj;
  p.bias = bias;
  p.error = ctx->d_error;
  p.residual = residual;
  p.res_f32 = residual_f32 ? 1 : 0;
  p.y = y;
  p.y_f32 = y_f32 ? 1 : 0;
  return launch_proj_t<64>(ctx, p, stream);
}

}  // namespace tla

#ifdef TLA_PROJ_TRACE
extern "C" int tla_debug_proj_trace(unsigned long long* host, int count) {
  return cudaMemcpyFromSymbol(host, tla::g_proj_trace, sizeof(unsigned long long) * count) == cudaSuccess ? 0 : -1;
}
extern "C" int tla_debug_allreduce_trace(unsigned long long* host, int count) {
  return cudaMemcpyFromSymbol(host, tla::g_ar_trace, sizeof(unsigned long long) * count) == cudaSuccess ? 0 : -1;
}
#endif

