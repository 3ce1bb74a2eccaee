// Causal prefill attention at head_dim 64 with two query tiles per CTA that
// share every K/V step ("ping-pong" over the exponential unit).
//
// At head_dim 64 a 128 x 128 step costs the tensor pipe about 614 cycles
// (S = Q K^T: four M=128 N=128 K=16 MMAs at 64 cycles; P V: eight N=64 MMAs
// with P in TMEM at about 45) and the exponential unit 1024 cycles (16384
// exponentials at 4 per cycle per sub-partition). One softmax warp per
// sub-partition cannot keep that unit busy, so each CTA here runs two
// softmax warpgroups on two 128-row query tiles of the same (sequence, kv
// head), with the K/V tiles loaded once for both. The rows of a step leave
// TMEM for registers at its start and P goes to its own TMEM columns, so the
// next S of a tile is computed while that tile's exponentials run.
//
// Warp roles (512 threads):
//   warp 0           TMA: lane 0 the Q tiles and K steps, lane 1 the V steps
//   warp 1           S issuer (both tiles), warp 3 P V issuer (both tiles)
//   warp 2           TMEM owner
//   warps 4-7 / 8-11 softmax of tile 0 / 1 (thread = query row = TMEM lane)
//   warps 12-15      epilogue: O / l, the output gate, rows out via shared memory
// A sub-partition runs warps w, w + 4, w + 8 and w + 12; a busy softmax pair
// beside an MMA issuer slows its issue (an M=128 N=64 MMA: 45 cycles alone,
// 55-85 with such neighbours), so the issuers' latency shows in each step.
// Registers: the launch gives 128 per thread; setmaxnreg moves them to the
// softmax warpgroups (184) from the epilogue (88) and control (56) warpgroups:
// 2 x 184 + 88 + 56 = 512 = 4 x 128.
// TMEM columns: S of tile t at 128 t, P (fp16 pairs) at 256 + 64 t, O at
// 384 + 64 t.
//
// Work items: the (query head, 128-row tile) units of one (sequence, kv head)
// are listed longest first (tile index descending, heads in order) and taken
// in pairs, so both tiles of an item read the same K/V steps; an item's step
// range is the union of its tiles' ranges and a tile takes part only in its
// own steps (a pair can straddle two tile rows when the group size is odd).
// Items of all (sequence, kv head) pairs are interleaved, longest first, and
// dealt to the persistent CTAs in snake order.
//
// Every mbarrier wait is bounded; on timeout the CTA records TLA_ERR_TIMEOUT,
// stops waiting and issuing, waits for the copies it issued, and frees TMEM.
#include <limits.h>

#include <algorithm>
#include <vector>

#include "prefill_common.cuh"

namespace tla {

namespace {

using namespace prefill;

#ifdef TLA_PREFILL_TRACE
// Optional pipeline trace (builds with -DTLA_PREFILL_TRACE only): SM clock of
// block 0's events, [step][event]; read with tla_debug_pp_trace. Softmax of
// tile t (its first warp, per tile step): [5 t] S seen complete, [5 t + 1] S
// loaded, [5 t + 2] maximum applied, [5 t + 3] exponentials done, [5 t + 4] P
// stored. Per union step: [10]/[11] S issue start/end, [12]/[13] P V issue
// start/end. An observer lane records [14] S of tile 0 complete and [15] P V
// of tile 1 complete (first 16 steps). Such a trace showed S complete well
// before the softmax reached its wait: the step's time outside the
// exponentials is the softmax warps' own.
__device__ unsigned long long g_pp_trace[64][16];
// per CTA: globaltimer at entry, after set-up, when the softmax of tile 0
// finished, at exit; and the union steps the CTA ran
__device__ unsigned long long g_pp_cta[256][5];
#define PPTRACE(n, ev)                                                                            \
  do {                                                                                            \
    if (blockIdx.x == 0 && (n) < 64) g_pp_trace[(n)][(ev)] = static_cast<unsigned long long>(clock64()); \
  } while (0)
#else
#define PPTRACE(n, ev) \
  do {                 \
  } while (0)
#endif

struct PP {
  static constexpr int D = 64;
  static constexpr int kThreads = 512;
  static constexpr int kTile = 128 * 128;  // bytes of a 128-row x 64 fp16 tile (Q, K or V)
  static constexpr int kST = 3;            // K and V stages
  static constexpr int kQ = 0;             // Q tiles [tile][item % 2]
  static constexpr int kK = kQ + 4 * kTile;
  static constexpr int kV = kK + kST * kTile;
  static constexpr int kOut = kV + kST * kTile;  // epilogue staging: 4 warps x 32 rows x D x up to 4 bytes
  static constexpr int kOutBytes = 4 * 32 * D * 4;
  static constexpr int kL = kOut + kOutBytes;  // row sums, then row maxima: [tile][item % 2][128] fp32 each
  static constexpr int kBar = kL + 2 * 4 * 128 * 4;
  // q_full[4], q_empty[4], k_full, v_full, k_empty, v_empty [kST], s_full[2],
  // s_free[2], p_full[2], o_done[2], o_free[2], l_full[4]
  static constexpr int kNumBars = 8 + 4 * kST + 10 + 4;
  static constexpr int kSmem = kBar + kNumBars * 8 + 16 + 1024;
  static constexpr uint32_t kS = 0, kP = 256, kO = 384, kCols = 512;
  // warpgroups by role: the MMA issuers and the TMA warp as warps 0-3 took
  // config 3 from 0.0799 to 0.0787 ms against warps 12-15
  static constexpr int kCtrlWg = 0, kSoftWg0 = 1, kEpiWg = 3;
  static constexpr int kTmaWarp = 4 * kCtrlWg, kSWarp = kTmaWarp + 1, kAllocWarp = kTmaWarp + 2,
                       kPvWarp = kTmaWarp + 3;
};
static_assert(PP::kSmem <= 232448, "shared memory");

// A pair of (head, query tile) units of one (sequence, kv head); n[t] == 0
// when the pair has only its first unit.
struct PairItem {
  int b, kvh, start, J0, NJ;
  int h[2], row0[2], rows[2], j0[2], n[2];
};

// One tile of a pair, picked with selects (no local-memory array indexing
// when t is not a compile-time constant).
struct PairTile {
  int h, row0, rows, j0, n;
};
__device__ __forceinline__ PairTile tile_of(const PairItem& w, int t) {
  const bool z = t == 0;
  return {z ? w.h[0] : w.h[1], z ? w.row0[0] : w.row0[1], z ? w.rows[0] : w.rows[1], z ? w.j0[0] : w.j0[1],
          z ? w.n[0] : w.n[1]};
}

__host__ __device__ __forceinline__ int pair_count(int G, int num_m, int batch, int Hk) {
  return ((G * num_m + 1) / 2) * batch * Hk;
}
__device__ __forceinline__ int pair_count(const PrefillParams& p) {
  return pair_count(p.G, p.num_m, p.batch, p.Hk);
}

// Pair q (unsplit): units 2q and 2q + 1 of its (sequence, kv head) list.
__device__ __forceinline__ PairItem pair_base(const PrefillParams& p, int q) {
  PairItem w;
  const int nbk = p.batch * p.Hk;
  const int qq = q / nbk, bk = q - qq * nbk;
  w.b = bk / p.Hk;
  w.kvh = bk - w.b * p.Hk;
  w.start = p.start[w.b];
  const int units = p.G * p.num_m;
  int lo = INT_MAX, hi = 0;
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int u = 2 * qq + t;
    w.h[t] = w.row0[t] = w.rows[t] = w.j0[t] = w.n[t] = 0;
    if (u >= units) continue;
    const int mi = u / p.G;
    w.h[t] = w.kvh * p.G + (u - mi * p.G);
    w.row0[t] = (p.num_m - 1 - mi) * 128;
    w.rows[t] = min(128, p.S - w.row0[t]);
    const int first_min = p.sliding > 0 ? max(0, w.start + w.row0[t] - p.sliding + 1) : 0;
    w.j0[t] = first_min / 128;
    w.n[t] = (w.start + w.row0[t] + w.rows[t] - 1) / 128 - w.j0[t] + 1;
    lo = min(lo, w.j0[t]);
    hi = max(hi, w.j0[t] + w.n[t]);
  }
  w.J0 = lo;
  w.NJ = hi - lo;
  return w;
}

// Pieces (piece_len > 0): pfx[q] = the first item of pair q, pfx[pairs] = the
// number of items; each pair is cut into ceil(NJ / piece_len) pieces (at most
// kMaxPieces). By the
// block's threads (pairs <= kMaxPiecePairs), with a warp scan at the end.
constexpr int kMaxPiecePairs = 320, kMaxPieces = 8, kMergeCols = 8;
__device__ __forceinline__ void piece_prefix(const PrefillParams& p, int* pfx, int pairs) {
  for (int q = threadIdx.x; q < pairs; q += blockDim.x) {
    const int nj = pair_base(p, q).NJ;
    pfx[q + 1] = min(kMaxPieces, max(1, (nj + p.piece_len - 1) / p.piece_len));
  }
  __syncthreads();
  if (threadIdx.x < 32) {  // lane l takes a run of consecutive pairs, then a shuffle scan over the runs
    constexpr int kRun = kMaxPiecePairs / 32;
    const int lane = threadIdx.x, per = (pairs + 31) / 32;
    const int q0 = min(pairs, lane * per), q1 = min(pairs, q0 + per);
    int cts[kRun], run = 0;
#pragma unroll
    for (int i = 0; i < kRun; ++i) {
      cts[i] = q0 + i < q1 ? pfx[q0 + i + 1] : 0;
      run += cts[i];
    }
    __syncwarp();  // every count is read before any prefix overwrites it
    int incl = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int acc = incl - run;  // this lane's exclusive prefix
#pragma unroll
    for (int i = 0; i < kRun; ++i) {
      if (q0 + i < q1) pfx[q0 + i] = acc;
      acc += cts[i];
    }
    if (lane == 31) pfx[pairs] = incl;  // the total (lanes past the last run add nothing)
  }
  __syncthreads();
}

// Work item `it`: pair it (piece_len == 0), or piece k of the pair q that
// covers item it: steps [J0 + k NJ / c, J0 + (k + 1) NJ / c) of the pair's
// union range (c pieces), each tile clipped to it (n[t] == 0: no step of the
// tile in the piece).
template <bool PIECES>
__device__ __forceinline__ PairItem pair_item(const PrefillParams& p, int it, const int* pfx, int pairs) {
  if constexpr (!PIECES) return pair_base(p, it);
  int lo_q = 0, hi_q = pairs - 1;  // the last q with pfx[q] <= it
  while (lo_q < hi_q) {
    const int mid = (lo_q + hi_q + 1) >> 1;
    if (pfx[mid] <= it)
      lo_q = mid;
    else
      hi_q = mid - 1;
  }
  PairItem w = pair_base(p, lo_q);
  const int k = it - pfx[lo_q], c = pfx[lo_q + 1] - pfx[lo_q];
  const int p0 = w.J0 + (k * w.NJ) / c, p1 = w.J0 + ((k + 1) * w.NJ) / c;
  int lo = INT_MAX, hi = 0;
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int a = max(w.j0[t], p0), e = min(w.j0[t] + w.n[t], p1);
    if (w.n[t] == 0 || e <= a) {
      w.n[t] = 0;
      continue;
    }
    w.j0[t] = a;
    w.n[t] = e - a;
    lo = min(lo, a);
    hi = max(hi, e);
  }
  w.J0 = hi == 0 ? 0 : lo;  // (an empty piece: NJ = 0)
  w.NJ = hi - w.J0;
  return w;
}

template <typename OUT, bool PIECES>
__global__ void __launch_bounds__(PP::kThreads, 1) prefill_pp_kernel(const __grid_constant__ PrefillParams p) {
  constexpr int kT = 128, D = PP::D;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + PP::kBar);
  uint64_t* q_full = bars;  // [2 t + item % 2]
  uint64_t* q_empty = bars + 4;
  uint64_t* k_full = bars + 8;
  uint64_t* v_full = k_full + PP::kST;
  uint64_t* k_empty = v_full + PP::kST;
  uint64_t* v_empty = k_empty + PP::kST;
  uint64_t* s_full = v_empty + PP::kST;  // [t]
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_free + 2;
  uint64_t* o_done = p_full + 2;
  uint64_t* o_free = o_done + 2;
  uint64_t* l_full = o_free + 2;  // [2 t + item % 2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + PP::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* l_buf = reinterpret_cast<float*>(smem + PP::kL);  // [2 t + item % 2][128]
  const int pairs = pair_count(p);
  __shared__ int pfx[kMaxPiecePairs + 1];  // pieces: the first item of each pair
#ifdef TLA_PREFILL_TRACE
  if (tid == 0 && blockIdx.x < 256) g_pp_cta[blockIdx.x][0] = globaltimer();
#endif

  if (tid == 0) {
    for (int i = 0; i < 8 + 4 * PP::kST; ++i) mbar_init(&bars[i], 1);  // q, k, v rings
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&s_free[t], 128);
      mbar_init(&p_full[t], 128);
      mbar_init(&o_done[t], 1);
      mbar_init(&o_free[t], 128);
      mbar_init(&l_full[2 * t], 128);
      mbar_init(&l_full[2 * t + 1], 128);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == PP::kAllocWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(PP::kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();  // the RoPE/append kernel's queries and cache rows are complete
#ifdef TLA_PREFILL_TRACE
  if (tid == 0 && blockIdx.x < 256) g_pp_cta[blockIdx.x][1] = globaltimer();
#endif
  if constexpr (PIECES) {
    piece_prefix(p, pfx, pairs);  // (the start positions may come from the kernel before)
    // the merge kernel may launch now: it builds its piece table, then waits
    // for this grid to complete (its CTAs take the SMs this grid leaves)
    griddep_launch_dependents();
  }
  const int num_items = PIECES ? pfx[pairs] : pairs;
  auto wait = [&](uint64_t* bar, uint32_t parity) {
    if (*abort_flag) return;
    if (!mbar_wait(bar, parity, p.error)) *abort_flag = 1;
  };
  auto spin = [&](uint64_t* bar, uint32_t parity) {
    if (!*abort_flag && !mbar_spin(bar, parity, p.error)) *abort_flag = 1;
  };

  const int wg = warp >> 2;
  const int role = wg == PP::kCtrlWg ? 3 : wg == PP::kEpiWg ? 2 : wg - PP::kSoftWg0;  // 0 / 1 softmax of tile 0 / 1

  if (role == 3) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 56;" ::: "memory");
    if (warp == PP::kTmaWarp && lane < 2) {
      // ============================================================ TMA producer
      const CUtensorMap* map = lane == 0 ? &p.tm_k : &p.tm_v;
      uint64_t* full = lane == 0 ? k_full : v_full;
      uint64_t* empty = lane == 0 ? k_empty : v_empty;
      uint8_t* ring = smem + (lane == 0 ? PP::kK : PP::kV);
      tma_prefetch(map);
      if (lane == 0) tma_prefetch(&p.tm_q);
      int g = 0, kq[2] = {0, 0};  // K/V loads issued; Q loads issued per tile
      for (int k = 0;; ++k) {
        const int it = prefill_item_of(k, num_items);
        if (it < 0) break;
        const PairItem w = pair_item<PIECES>(p, it, pfx, pairs);
        if (lane == 0) {
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            if (w.n[t] == 0) continue;
            const int slot = 2 * t + (kq[t] & 1);
            wait(&q_empty[slot], ((kq[t] >> 1) & 1) ^ 1);
            if (*abort_flag) break;
            mbar_arrive_expect_tx(&q_full[slot], PP::kTile);
            tma_load_3d(smem + PP::kQ + slot * PP::kTile, &p.tm_q, &q_full[slot], 0, w.row0[t], w.b * p.Hq + w.h[t]);
            ++kq[t];
          }
        }
        const int z = w.b * p.Hk + w.kvh;
        for (int n = 0; n < w.NJ && !*abort_flag; ++n) {
          const int st = g % PP::kST;
          wait(&empty[st], ((g / PP::kST) & 1) ^ 1);
          if (*abort_flag) break;
          mbar_arrive_expect_tx(&full[st], PP::kTile);
          tma_load_3d(ring + st * PP::kTile, map, &full[st], 0, (w.J0 + n) * kT, z);
          ++g;
        }
        if (*abort_flag) break;
      }
      // no copies in flight at exit: only the last kST loads of a ring (and
      // the last Q load of each slot) can still be running
      for (int q = max(0, g - PP::kST); q < g; ++q) mbar_wait(&full[q % PP::kST], (q / PP::kST) & 1, p.error);
      if (lane == 0) {
        for (int t = 0; t < 2; ++t)
          for (int c = max(0, kq[t] - 2); c < kq[t]; ++c) mbar_wait(&q_full[2 * t + (c & 1)], (c >> 1) & 1, p.error);
      }
#ifdef TLA_PREFILL_TRACE
    } else if (warp == PP::kAllocWarp && lane == 0 && blockIdx.x == 0) {
      // observer (trace builds): when S of tile 0's first 16 steps completes
      // ([14]) and when P V of tile 1 completes ([15], from a second lane)
      for (int c = 0; c < 16 && !*abort_flag; ++c) {
        for (int i = 0; i < (1 << 24) && !mbar_test_wait(&s_full[0], c & 1); ++i) {
        }
        PPTRACE(c, 14);
      }
    } else if (warp == PP::kAllocWarp && lane == 1 && blockIdx.x == 0) {
      for (int c = 0; c < 16 && !*abort_flag; ++c) {
        for (int i = 0; i < (1 << 24) && !mbar_test_wait(&o_done[1], c & 1); ++i) {
        }
        PPTRACE(c, 15);
      }
#endif
    } else if ((warp == PP::kSWarp || warp == PP::kPvWarp) && lane == 0) {
      // ============================================================ MMA issuers
      // Warp 1 issues every S (both tiles), warp 3 every P V, so one
      // thread's waits overlap the other's MMAs. Both poll their barriers
      // without suspending (about 1% faster at config 3 than try_wait). S of a tile is issued once
      // that tile's softmax has read the previous S into registers (s_free);
      // P V once the softmax has stored P (p_full) and, for a tile's first
      // step of an item, once the epilogue has read that tile's O (o_free).
      if (warp == PP::kSWarp) {
        constexpr uint32_t kIdS = idesc_f16(128, kT, false);
        const uint64_t dq = sdesc(smem_u32(smem + PP::kQ), 16, 1024);
        const uint64_t dk = sdesc(smem_u32(smem + PP::kK), 16, 1024);
        int g = 0, kq[2] = {0, 0}, sc[2] = {0, 0};  // steps, items per tile, S per tile
        for (int k = 0;; ++k) {
          const int it = prefill_item_of(k, num_items);
          if (it < 0) break;
          const PairItem w = pair_item<PIECES>(p, it, pfx, pairs);
          for (int n = 0; n < w.NJ; ++n, ++g) {
            const int st = g % PP::kST, J = w.J0 + n;
            spin(&k_full[st], (g / PP::kST) & 1);
            PPTRACE(g, 10);
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              const int jl = J - w.j0[t];
              if (jl < 0 || jl >= w.n[t]) continue;
              const int slot = 2 * t + (kq[t] & 1);
              if (jl == 0) spin(&q_full[slot], (kq[t] >> 1) & 1);
              if (sc[t] > 0) spin(&s_free[t], (sc[t] - 1) & 1);
              tc_fence_after();
              const uint64_t qb = dq + static_cast<uint64_t>(slot * (PP::kTile >> 4));
              const uint64_t kb = dk + static_cast<uint64_t>(st * (PP::kTile >> 4));
              if (!*abort_flag) {
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                  mma_f16(tmem + PP::kS + 128 * t, qb + 2 * kk, kb + 2 * kk, kIdS, kk > 0 ? 1u : 0u);
              }
              mma_commit(&s_full[t]);
              ++sc[t];
              if (jl == w.n[t] - 1) {  // the tile's last S of this item: its Q slot is free
                mma_commit(&q_empty[slot]);
                ++kq[t];
              }
            }
            mma_commit(&k_empty[st]);
            PPTRACE(g, 11);
          }
        }
      } else {
        constexpr uint32_t kIdO = idesc_f16(128, D, true);
        const uint64_t dv = sdesc(smem_u32(smem + PP::kV), PP::kTile, 1024);
        int g = 0, kq[2] = {0, 0}, pc[2] = {0, 0};  // steps, items per tile, P V per tile
        for (int k = 0;; ++k) {
          const int it = prefill_item_of(k, num_items);
          if (it < 0) break;
          const PairItem w = pair_item<PIECES>(p, it, pfx, pairs);
          for (int n = 0; n < w.NJ; ++n, ++g) {
            const int st = g % PP::kST, J = w.J0 + n;
            spin(&v_full[st], (g / PP::kST) & 1);
            PPTRACE(g, 12);
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              const int jl = J - w.j0[t];
              if (jl < 0 || jl >= w.n[t]) continue;
              if (jl == 0 && kq[t] > 0) spin(&o_free[t], (kq[t] - 1) & 1);
              spin(&p_full[t], pc[t] & 1);
              tc_fence_after();
              const uint64_t vb = dv + static_cast<uint64_t>(st * (PP::kTile >> 4));
              if (!*abort_flag) {
#pragma unroll
                for (int kk = 0; kk < kT / 16; ++kk)
                  mma_f16_ts(tmem + PP::kO + 64 * t, tmem + PP::kP + 64 * t + 8 * kk, vb + 128 * kk, kIdO,
                             (jl > 0 || kk > 0) ? 1u : 0u);
              }
              mma_commit(&o_done[t]);
              ++pc[t];
              if (jl == w.n[t] - 1) ++kq[t];
            }
            mma_commit(&v_empty[st]);
            PPTRACE(g, 13);
          }
        }
      }
    }
  } else if (role == 2) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 88;" ::: "memory");
    // ================================================================ epilogue
    // For each tile of each item: wait for its row sums and its last P V,
    // normalise O, apply the output gate, and store whole rows through this
    // warp's shared-memory stage; then free the tile's O columns.
    const int r = tid & 127;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    constexpr int kRowBytes = D * static_cast<int>(sizeof(OUT));
    constexpr int kChunks = kRowBytes / 16;
    constexpr int kRowsPer = 32 / kChunks;
    uint8_t* stage = smem + PP::kOut + (warp & 3) * 32 * kRowBytes;
    const size_t row_stride = static_cast<size_t>(p.Hq) * D;  // elements between consecutive tokens
    [[maybe_unused]] const long long out_elems = static_cast<long long>(p.batch) * p.S * p.Hq * D;
    int kq[2] = {0, 0}, c[2] = {0, 0};  // items and P V steps per tile
    for (int k = 0;; ++k) {
      const int it = prefill_item_of(k, num_items);
      if (it < 0) break;
      const PairItem w = pair_item<PIECES>(p, it, pfx, pairs);
#pragma unroll 1
      for (int t = 0; t < 2; ++t) {
        const PairTile u = tile_of(w, t);
        if (u.n == 0) continue;
        int& ct = t == 0 ? c[0] : c[1];
        int& kt = t == 0 ? kq[0] : kq[1];
        ct += u.n;
        const int slot = 2 * t + (kt & 1);
        wait(&l_full[slot], (kt >> 1) & 1);
        wait(&o_done[t], (ct - 1) & 1);
        __syncwarp();
        tc_fence_after();
        const float le = l_buf[slot * 128 + r];
        const float inv = le > 0.f ? 1.f / le : 0.f;
        const long long base = ((static_cast<long long>(w.b) * p.S + u.row0) * p.Hq + u.h) * D;
        const int rows = u.rows;
        const uint32_t oe = tmem + lane_base + PP::kO + 64 * t;
        if constexpr (PIECES) {
          // a piece: the row's unnormalised O, its maximum and its sum, fp32,
          // column-major per (item, tile) block [D + 2][128] so that a warp's
          // rows are 32 consecutive words (the merge kernel writes the output)
          float* dst = p.part + (static_cast<size_t>(it) * 2 + t) * (D + 2) * 128 + r;
#pragma unroll 1
          for (int cc = 0; cc < D / 16; ++cc) {
            uint32_t ou[16];
            tmem_ld16(oe + 16 * cc, ou);
            if (r < rows) {
#pragma unroll
              for (int i = 0; i < 16; ++i) dst[(16 * cc + i) * 128] = __uint_as_float(ou[i]);
            }
          }
          if (r < rows) {
            dst[D * 128] = l_buf[512 + slot * 128 + r];
            dst[(D + 1) * 128] = le;
          }
          tc_fence_before();
          mbar_arrive(&o_free[t]);
          ++kt;
        } else {
#pragma unroll 1
          for (int cc = 0; cc < D / 16; ++cc) {  // 16 columns at a time
            uint32_t ou[16];
            tmem_ld16(oe + 16 * cc, ou);
            float o[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = __uint_as_float(ou[i]) * inv;
            // output gate (TSLAttention.ts:418-423, math.ts:271-273): times
            // sigmoid(gate) in fp32 before the conversion to OUT
            if (p.gate != nullptr && r < rows &&
                TLA_IN_BOUNDS(base + r * row_stride + 16 * cc + 15, out_elems, p.error)) {
              const OUT* gsrc = static_cast<const OUT*>(p.gate) + base + r * row_stride + 16 * cc;
#pragma unroll
              for (int i0 = 0; i0 < 16; i0 += 8) {
                float gv[8];
                if constexpr (sizeof(OUT) == 2) {
                  const uint4 u = *reinterpret_cast<const uint4*>(gsrc + i0);
                  const __half2* h2 = reinterpret_cast<const __half2*>(&u);
#pragma unroll
                  for (int j = 0; j < 4; ++j) {
                    gv[2 * j] = __low2float(h2[j]);
                    gv[2 * j + 1] = __high2float(h2[j]);
                  }
                } else {
                  const float4 a = *reinterpret_cast<const float4*>(gsrc + i0);
                  const float4 b = *reinterpret_cast<const float4*>(gsrc + i0 + 4);
                  gv[0] = a.x, gv[1] = a.y, gv[2] = a.z, gv[3] = a.w;
                  gv[4] = b.x, gv[5] = b.y, gv[6] = b.z, gv[7] = b.w;
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) o[i0 + j] *= 1.f / (1.f + expf(-gv[j]));
              }
            }
            // into the stage: 16-byte chunks XOR-swizzled by row
            constexpr int kPer16 = static_cast<int>(sizeof(OUT));  // 16-byte chunks per 16 values
#pragma unroll
            for (int i = 0; i < kPer16; ++i) {
              uint4 v;
              if constexpr (sizeof(OUT) == 2) {
                const float* f = o + 8 * i;
                v = make_uint4(pack_half2(f[0], f[1]), pack_half2(f[2], f[3]), pack_half2(f[4], f[5]),
                               pack_half2(f[6], f[7]));
              } else {
                const float* f = o + 4 * i;
                v = make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                               __float_as_uint(f[3]));
              }
              const int q = cc * kPer16 + i;
              *reinterpret_cast<uint4*>(stage + lane * kRowBytes + ((q ^ (lane & 7)) << 4)) = v;
            }
          }
          // O has been read: the tile's next item may start accumulating
          tc_fence_before();
          mbar_arrive(&o_free[t]);
          ++kt;
          __syncwarp();
          // whole rows out: a warp-wide store covers kRowsPer rows
          const int q = lane % kChunks;
          const uint8_t* src = stage + (lane / kChunks) * kRowBytes;
          int row = (warp & 3) * 32 + lane / kChunks;
          uint8_t* dst = reinterpret_cast<uint8_t*>(static_cast<OUT*>(p.out) + base + row * row_stride) + (q << 4);
          const size_t dst_step = kRowsPer * row_stride * sizeof(OUT);
#pragma unroll 1
          for (int i = 0; i < kChunks; ++i, row += kRowsPer, src += kRowsPer * kRowBytes, dst += dst_step) {
            const uint4 v = *reinterpret_cast<const uint4*>(src + ((q ^ (row & 7)) << 4));
            if (row < rows && TLA_IN_BOUNDS(base + row * row_stride + ((q + 1) * 16) / sizeof(OUT) - 1, out_elems,
                                            p.error))
              *reinterpret_cast<uint4*>(dst) = v;
          }
          __syncwarp();  // the stage is reused by the next tile
        }
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 184;" ::: "memory");
    // ================================================================ softmax
    const int t = role;        // this warpgroup's tile
    const int r = tid & 127;   // query row = TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t s_addr = tmem + lane_base + PP::kS + 128 * t;
    const uint32_t p_addr = tmem + lane_base + PP::kP + 64 * t;
    const uint32_t o_addr = tmem + lane_base + PP::kO + 64 * t;
    const float sl2 = p.scale_log2;
    const uint32_t ninf = __float_as_uint(-INFINITY);
    int c = 0, kq = 0;  // this tile's steps and items so far
    for (int k = 0;; ++k) {
      const int it = prefill_item_of(k, num_items);
      if (it < 0) break;
      const PairItem w = pair_item<PIECES>(p, it, pfx, pairs);
      const PairTile u = tile_of(w, t);
      if (u.n == 0) continue;
      const int pr = w.start + u.row0 + r;
      const int first_r = p.sliding > 0 ? max(0, pr - p.sliding + 1) : 0;
      float m_run = -INFINITY, l_run = 0.f;
      uint32_t sv[128];  // this step's S row (fp32 bits)
      // P = 2^(S scale_log2 - mu) as fp16 pairs into this tile's P columns, in
      // quarters of 32 columns stored as soon as they are done (one basic
      // block, so the quarters' instructions interleave); returns the row sum
      // of the step.
      auto run_exps = [&](float mu) -> float {
        const uint64_t sl2x2 = pack_f32x2(sl2, sl2), nmu2 = pack_f32x2(-mu, -mu);
        uint64_t sum2[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const int kc = 32 * h + i;
            const bool poly = poly_pair_every<TLA_PP_POLY_EVERY>(kc / 2);
            float x0, x1;
            fma_f32x2(__uint_as_float(sv[kc]), __uint_as_float(sv[kc + 1]), sl2x2, nmu2, x0, x1);
            const float e0 = poly ? ex2_poly(x0) : ex2(x0);
            const float e1 = poly ? ex2_poly(x1) : ex2(x1);
            add_f32x2(sum2[(i >> 1) & 3], e0, e1);
            pk[i / 2] = pack_half2(e0, e1);
          }
          if (h == 0 && c > 0) {  // P V of the previous step has read this tile's P columns
            wait(&o_done[t], (c - 1) & 1);
            __syncwarp();
            tc_fence_after();
          }
          tmem_st16(p_addr + 16 * h, pk);
        }
        return (sum_f32x2(sum2[0]) + sum_f32x2(sum2[1])) + (sum_f32x2(sum2[2]) + sum_f32x2(sum2[3]));
      };
#pragma unroll 1
      for (int jl = 0; jl < u.n; ++jl, ++c) {
        const bool tr = (warp & 3) == 0 && lane == 0;
        wait(&s_full[t], c & 1);
        if (tr) PPTRACE(c, 5 * t);
        __syncwarp();
        tc_fence_after();
        tmem_ld64x(s_addr, *reinterpret_cast<uint32_t(*)[64]>(&sv[0]));
        tmem_ld64x(s_addr + 64, *reinterpret_cast<uint32_t(*)[64]>(&sv[64]));
        tc_fence_before();
        mbar_arrive(&s_free[t]);  // the S issuer may overwrite this tile's S
        if (tr) PPTRACE(c, 5 * t + 1);
        const int tok0 = (u.j0 + jl) * kT;
        if (tok0 + kT - 1 > pr || tok0 < first_r) {
          // valid columns [lo, lo + span] (first_r <= pr); one unsigned
          // compare and a select per column, no branch
          const int lo = first_r - tok0;
          const uint32_t span = static_cast<uint32_t>(pr - first_r);
#pragma unroll
          for (int i = 0; i < 128; ++i) sv[i] = static_cast<uint32_t>(i - lo) <= span ? sv[i] : ninf;
        }
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int i = 0; i < 128; i += 8) {  // four independent chains of three-input maxima
          mx[0] = fmax3(mx[0], __uint_as_float(sv[i]), __uint_as_float(sv[i + 1]));
          mx[1] = fmax3(mx[1], __uint_as_float(sv[i + 2]), __uint_as_float(sv[i + 3]));
          mx[2] = fmax3(mx[2], __uint_as_float(sv[i + 4]), __uint_as_float(sv[i + 5]));
          mx[3] = fmax3(mx[3], __uint_as_float(sv[i + 6]), __uint_as_float(sv[i + 7]));
        }
        const float m_tile = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * sl2;
        // The row's reference maximum moves (and O is rescaled in TMEM, after
        // P V of the previous step) only when exceeded by more than 2^8.
        const bool grow = m_tile > m_run + kRescaleLog2;
        if (__any_sync(0xffffffffu, grow)) {
          const float m_new = grow ? m_tile : m_run;
          // 0 while the row has seen no unmasked token (O and l are still zero), 1 when unchanged
          const float alpha = m_run == -INFINITY ? 0.f : ex2(m_run - m_new);
          if (jl > 0) {
            wait(&o_done[t], (c - 1) & 1);
            __syncwarp();
            tc_fence_after();
#pragma unroll 1
            for (int cc = 0; cc < D / 16; ++cc) {  // 16 columns at a time: the row's S is still live
              uint32_t o[16];
              tmem_ld16(o_addr + 16 * cc, o);
#pragma unroll
              for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
              tmem_st16(o_addr + 16 * cc, o);
            }
          }
          l_run *= alpha;
          m_run = m_new;
        }
        if (tr) PPTRACE(c, 5 * t + 2);
        l_run += run_exps(m_run == -INFINITY ? 0.f : m_run);
        if (tr) PPTRACE(c, 5 * t + 3);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[t]);
        if (tr) PPTRACE(c, 5 * t + 4);
      }
      // the row sum for the epilogue
      const int slot = 2 * t + (kq & 1);
      l_buf[slot * 128 + r] = l_run;
      l_buf[512 + slot * 128 + r] = m_run;  // (read only for partial rows)
      mbar_arrive(&l_full[slot]);
      ++kq;
    }
#ifdef TLA_PREFILL_TRACE
    if (r == 0 && t == 0 && blockIdx.x < 256) {
      g_pp_cta[blockIdx.x][2] = globaltimer();
      g_pp_cta[blockIdx.x][4] = static_cast<unsigned long long>(c);
    }
#endif
  }
  tc_fence_before();
  __syncthreads();
  if (warp == PP::kAllocWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(PP::kCols) : "memory");
  }
#ifdef TLA_PREFILL_TRACE
  if (tid == 0 && blockIdx.x < 256) g_pp_cta[blockIdx.x][3] = globaltimer();
#endif
}

// Merge of the KV-range pieces (piece_len > 0): one CTA per (pair, tile,
// group of kMergeCols columns), a thread per output row, whose pieces' loads
// all go out in one round (the partial blocks are column-major, so a warp's
// loads are 32 consecutive words). The pieces' unnormalised (O, m, l) combine
// by the log-sum-exp rule (m in the log2 domain), then O / l times the output
// gate (TSLAttention.ts:418-423) goes out.
template <typename OUT>
__global__ void __launch_bounds__(128) prefill_pp_merge_kernel(const __grid_constant__ PrefillParams p) {
  constexpr int D = PP::D, kCols = kMergeCols;
  __shared__ int pfx[kMaxPiecePairs + 1];
  __shared__ int in_piece[kMaxPieces];  // the tile has steps in piece k
  __shared__ int tile_b, tile_row0, tile_h, tile_rows;
  const int r = threadIdx.x;
  const int col0 = (static_cast<int>(blockIdx.x) % (D / kCols)) * kCols;
  const int pt = static_cast<int>(blockIdx.x) / (D / kCols);
  const int pq = pt >> 1, t = pt & 1;
  const int pairs = pair_count(p);
  // The piece table before the wait: the start positions were final before
  // the attention kernel started (it waited for them itself).
  piece_prefix(p, pfx, pairs);
  const int first = pfx[pq], pieces = pfx[pq + 1] - first;
  if (r == 0) {
    const PairItem w = pair_base(p, pq);
    const PairTile u = tile_of(w, t);
    tile_b = w.b;
    tile_row0 = u.row0;
    tile_h = u.h;
    tile_rows = u.rows;
    for (int k = 0; k < kMaxPieces; ++k) {  // as pair_item cuts the pieces
      const int p0 = w.J0 + (k * w.NJ) / max(pieces, 1), p1 = w.J0 + ((k + 1) * w.NJ) / max(pieces, 1);
      in_piece[k] = k < pieces && min(u.j0 + u.n, p1) > max(u.j0, p0);
    }
  }
  __syncthreads();
  griddep_wait();  // the pieces are complete and visible
  if (r >= tile_rows) return;
  constexpr size_t kBlock = static_cast<size_t>(D + 2) * 128;  // floats of one (item, tile) block
  const float* rowp = p.part + static_cast<size_t>(first * 2 + t) * kBlock + r;
  float mk[kMaxPieces], lk[kMaxPieces], ok[kMaxPieces][kCols];
  float mx = -INFINITY;
#pragma unroll
  for (int k = 0; k < kMaxPieces; ++k) {
    const float* src = rowp + k * 2 * kBlock;
    const bool in = in_piece[k] != 0;
    mk[k] = in ? __ldcg(src + D * 128) : -INFINITY;
    lk[k] = in ? __ldcg(src + (D + 1) * 128) : 0.f;
#pragma unroll
    for (int i = 0; i < kCols; ++i) ok[k][i] = in ? __ldcg(src + (col0 + i) * 128) : 0.f;
    mx = fmaxf(mx, mk[k]);
  }
  float acc[kCols];
#pragma unroll
  for (int i = 0; i < kCols; ++i) acc[i] = 0.f;
  float l = 0.f;
#pragma unroll
  for (int k = 0; k < kMaxPieces; ++k) {
    // (not in the piece, or no unmasked column of the row there: weight 0)
    const float f = mk[k] == -INFINITY ? 0.f : ex2(mk[k] - mx);
    l += f * lk[k];
#pragma unroll
    for (int i = 0; i < kCols; ++i) acc[i] += f * ok[k][i];
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  const long long base = ((static_cast<long long>(tile_b) * p.S + tile_row0 + r) * p.Hq + tile_h) * D + col0;
  if (!TLA_IN_BOUNDS(base + kCols - 1, static_cast<long long>(p.batch) * p.S * p.Hq * D, p.error)) return;
  const OUT* gs = p.gate != nullptr ? static_cast<const OUT*>(p.gate) + base : nullptr;
  OUT* dst = static_cast<OUT*>(p.out) + base;
#pragma unroll
  for (int i = 0; i < kCols; i += 8) {
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      o[j] = acc[i + j] * inv;
      if (gs != nullptr) o[j] *= 1.f / (1.f + expf(-to_f32(gs[i + j])));  // in fp32 before the conversion
    }
    if constexpr (sizeof(OUT) == 2) {
      *reinterpret_cast<uint4*>(dst + i) = make_uint4(pack_half2(o[0], o[1]), pack_half2(o[2], o[3]),
                                                      pack_half2(o[4], o[5]), pack_half2(o[6], o[7]));
    } else {
      *reinterpret_cast<float4*>(dst + i) = make_float4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<float4*>(dst + i + 4) = make_float4(o[4], o[5], o[6], o[7]);
    }
  }
}

}  // namespace

namespace prefill {

#ifdef TLA_PREFILL_TRACE
extern "C" int tla_debug_pp_trace(unsigned long long* host, int count) {
  return cudaMemcpyFromSymbol(host, g_pp_trace, sizeof(unsigned long long) * count) == cudaSuccess ? 0 : -1;
}
extern "C" int tla_debug_pp_cta(unsigned long long* host, int count) {
  return cudaMemcpyFromSymbol(host, g_pp_cta, sizeof(unsigned long long) * count) == cudaSuccess ? 0 : -1;
}
#endif

cudaError_t pp_configure(const tla_layer* L) {
  cudaError_t e = L->io_fp32
                      ? raise_smem_limit(reinterpret_cast<const void*>(prefill_pp_kernel<float, false>), PP::kSmem)
                      : raise_smem_limit(reinterpret_cast<const void*>(prefill_pp_kernel<__half, false>), PP::kSmem);
  if (e != cudaSuccess) return e;
  return L->io_fp32 ? raise_smem_limit(reinterpret_cast<const void*>(prefill_pp_kernel<float, true>), PP::kSmem)
                    : raise_smem_limit(reinterpret_cast<const void*>(prefill_pp_kernel<__half, true>), PP::kSmem);
}

size_t pp_smem() { return PP::kSmem; }

// Piece length (KV steps) for a chunk, 0 for whole pairs. Each piece costs a
// query-tile load, a first step from cold, a partial-row epilogue and a share
// of the merge kernel, so the chunk is cut only when it has at most one pair
// per two SMs (measured: one pair per SM gained nothing), and then into the
// longest pieces that still fit in one wave of items: the smallest length L
// with sum over pairs of min(kMaxPieces, ceil(NJ / L)) <= SMs, the pairs'
// step counts NJ taken at start position 0.
int pp_piece_len(const tla_layer* L, int batch, int seq_len) {
  const int num_m = (seq_len + 127) / 128, G = L->G;
  const long long pairs = pair_count(G, num_m, batch, L->Hk);
  const int sms = L->ctx->sm_count;
  if (pairs <= 0 || sms <= 0 || 2 * pairs > sms || pairs > kMaxPiecePairs) return 0;
  // step counts of one (sequence, kv head)'s pairs (the same for all of them at start 0)
  const int units = G * num_m, per = (units + 1) / 2;
  std::vector<int> nj(per);
  int max_nj = 0;
  for (int q = 0; q < per; ++q) {
    int lo = 1 << 30, hi = 0;
    for (int u = 2 * q; u < 2 * q + 2 && u < units; ++u) {
      const int row0 = (num_m - 1 - u / G) * 128, rows = std::min(128, seq_len - row0);
      const int j0 = (L->sliding > 0 ? std::max(0, row0 - L->sliding + 1) : 0) / 128;
      lo = std::min(lo, j0);
      hi = std::max(hi, (row0 + rows - 1) / 128 + 1);
    }
    nj[q] = hi - lo;
    max_nj = std::max(max_nj, nj[q]);
  }
  const long long copies = pairs / per;  // (sequence, kv head) lists
  for (int len = 2; len < max_nj; ++len) {
    long long items = 0;
    for (int q = 0; q < per; ++q) items += std::min(kMaxPieces, (nj[q] + len - 1) / len);
    if (items * copies <= sms) return len;
  }
  return 0;
}

size_t pp_partial_bytes(const tla_layer* L, int batch, int seq_len) {
  if (pp_piece_len(L, batch, seq_len) == 0) return 0;
  const int pairs = pair_count(L->G, (seq_len + 127) / 128, batch, L->Hk);
  return static_cast<size_t>(pairs) * kMaxPieces * 2 * (PP::D + 2) * 128 * sizeof(float);
}

cudaError_t launch_pp(const tla_layer* L, const PrefillParams& p0, cudaStream_t stream) {
  PrefillParams p = p0;
  const int pairs = pair_count(p.G, p.num_m, p.batch, p.Hk);
  p.piece_len = pp_piece_len(L, p.batch, p.S);
  // the pieces' partial blocks follow the rotated queries [B][Hq][S][D] fp16 in the query scratch
  const size_t q_bytes = (static_cast<size_t>(p.batch) * p.Hq * p.S * PP::D * sizeof(__half) + 255) & ~size_t(255);
  p.part = p.piece_len > 0 ? reinterpret_cast<float*>(static_cast<uint8_t*>(L->ctx->d_qscratch) + q_bytes) : nullptr;
  const int sms = L->ctx->sm_count;
  const unsigned grid = static_cast<unsigned>(p.piece_len > 0 ? sms : (pairs < sms ? pairs : sms));
  // (pieces get their own instance, so that whole-pair chunks run the kernel without the piece code)
  cudaError_t e;
  if (p.piece_len > 0)
    e = L->io_fp32 ? launch_pdl(prefill_pp_kernel<float, true>, grid, PP::kThreads, PP::kSmem, stream, p)
                   : launch_pdl(prefill_pp_kernel<__half, true>, grid, PP::kThreads, PP::kSmem, stream, p);
  else
    e = L->io_fp32 ? launch_pdl(prefill_pp_kernel<float, false>, grid, PP::kThreads, PP::kSmem, stream, p)
                   : launch_pdl(prefill_pp_kernel<__half, false>, grid, PP::kThreads, PP::kSmem, stream, p);
  if (e != cudaSuccess || p.piece_len == 0) return e;
  const unsigned mgrid = static_cast<unsigned>(pairs) * 2 * (PP::D / kMergeCols);  // a CTA per (pair, tile, columns)
  return L->io_fp32 ? launch_pdl(prefill_pp_merge_kernel<float>, mgrid, 128, 0, stream, p)
                    : launch_pdl(prefill_pp_merge_kernel<__half>, mgrid, 128, 0, stream, p);
}

}  // namespace prefill
}  // namespace tla
