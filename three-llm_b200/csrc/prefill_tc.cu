// Causal prefill attention on the 5th-generation tensor cores (tcgen05),
// fp16 K/V cache, head_dim 64 or 128.
//
// The reference has no prefill kernel: it replays the one-token decode graph
// for every prompt position (packages/three-llm/src/decoder/DecoderTSLRunner.ts:
// 472-480, 504-530), so position p attends to cache slots [window start, p]
// with every earlier prompt token already appended. This kernel computes the
// same outputs for a whole prompt chunk at once: a RoPE/append kernel
// (generic.cu) first writes the rotated queries (fp16, [B][Hq][S][D]) and
// appends the chunk's K/V to the cache, then prefill_tc_kernel runs one
// persistent CTA per SM over the work items (128-row query tile, head,
// sequence), longest first.
// Every mbarrier wait is bounded; on timeout the CTA records TLA_ERR_TIMEOUT,
// stops waiting, runs its remaining control flow and frees its TMEM.
#include <math.h>

#include "prefill_common.cuh"

namespace tla {

namespace {

using namespace prefill;

#ifdef TLA_PREFILL_TRACE
// Optional pipeline trace (builds with -DTLA_PREFILL_TRACE only): SM clock of
// each event of block 0's first 64 global steps, [step][event]; read with
// tla_debug_prefill_trace. Softmax (warp 0 unless noted): [0] S(g) complete,
// [1] after the fence that follows it, [2] S(g) loaded, [3 + w] warp w's P(g)
// stored. S issuer: [8]/[9] S(g) issue start/end. P V issuer: [12]/[13]
// before/after the V(g) wait, [10]/[11] P V(g) issue start/end.
__device__ unsigned long long g_prefill_trace[64][16];
#define PTRACE(ev, n) \
  do { \
    if (blockIdx.x == 0 && pipe == 0 && (n) < 64) g_prefill_trace[(n)][(ev)] = clock64(); \
  } while (0)
#else
#define PTRACE(ev, n) \
  do { \
  } while (0)
#endif

#ifndef TLA_PREFILL_PP
#define TLA_PREFILL_PP 1  // head_dim 64: the two-tile kernel of prefill_pp.cu (0: prefill_tc_kernel)
#endif

#ifndef TLA_PREFILL_DUAL
#define TLA_PREFILL_DUAL 0  // head_dim 64: two pipelines per CTA (measured slower; 0: one)
#endif

// ---------------------------------------------------------------- the kernel
// Persistent: one CTA per SM walks a fixed list of work items, an item being
// one 128-row query tile of one (head, sequence), K/V in 128-token steps.
// Items are ordered longest first and dealt to the CTAs in snake order
// (c, 2G-1-c, 2G+c, ...), so every CTA gets a similar amount of work; the
// step counter g runs across a CTA's items, so the TMA rings, the S buffers
// and the barriers flow from one item into the next without a drain, and the
// next item's Q load and first S MMAs overlap the current item's epilogue.
//
// The tcgen05 pipe runs one MMA at a time and an issuing thread waits for
// each to be accepted. Two issuing threads share it: one issues every S(g),
// the other every P V(g), so one's waits, commits and bookkeeping overlap the
// other's MMAs. NS TMEM S buffers let S run NS steps ahead of P V: S(g) is
// issued once P V(g - NS) has completed (it read P(g - NS) from the buffer
// S(g) overwrites), which gives the order S(0) .. S(NS-1) PV(0) S(NS) PV(1)
// ..., so S(g) is usually finished when the softmax warpgroup reaches step g.
// N = 128 for the S MMAs (full rate) and N = head_dim for P V.
// Softmax thread = one query row (TMEM lane), all 128 columns of the step in
// registers (one pass). P(g) is written as fp16 pairs over the first 64
// columns of its own S buffer and read from there as the A operand of P V;
// S(g+NS) reuses the buffer only after P V(g) has completed. The scale and
// subtract and the row sums run as packed fp32 pairs. (Splitting the columns
// over two warps per sub-partition, with a per-step exchange of the row
// maxima, gained about 2% for eight more warps and was not kept.) O
// accumulates in TMEM, double-buffered by
// item where TMEM has room (head_dim 64), so the next item's P V can start
// before this item's epilogue has read its O (o_free); likewise the Q tile in
// shared memory (head_dim 64; at 128 the K/V stages take the room). A row's reference maximum only moves when a step's maximum
// exceeds it by more than 2^8 (O is then rescaled in TMEM after the previous
// P V finished), so P stays <= 256 in fp16.
// P V(g) completion is signalled on o_done[g & 1]. A softmax thread can be up
// to two P V steps behind the issuer, which one barrier's phase parity cannot
// tell apart; with two barriers each barrier is at most one phase from any
// phase a thread waits for: S(g) is issued only after P V(g - NS) (NS <= 3)
// has completed, so once S(g) is complete P V(g-3) is too, and the rescale at
// step g (waiting for P V(g-1), whose barrier last completed for P V(g-3)) and
// the item epilogue (P V(g-2), then P V(g-1)) wait on a barrier at most one
// phase behind. The softmax therefore waits for O only when it reads it.
// The S issuer's own wait for P V(g - NS) is not overtaken by P V(g-1) on the
// same barrier: P V(g-1) needs P(g-1), which the softmax releases only after
// it has loaded S(g), also across items.
// TMEM columns: S/P buffer j at 128 j (j < NS), O buffer i at 128 NS + D i (i < NO).
// Warp roles. One pipeline: warps 0-3 softmax, 4 TMA, 5 P V issuer (and TMEM
// owner), 6 S issuer (224 threads). Two pipelines (DUAL, head_dim 64): each
// CTA runs two independent copies of that pipeline over alternate work items,
// each with one TMEM S buffer, so one pipeline's exponentials overlap the
// other's MMAs and loads: warps 0-3 / 4-7 softmax of pipeline 0 / 1, 8-9 TMA,
// 10-11 P V issuers (warp 10 owns TMEM), 12-13 S issuers, 14-15 idle (they
// complete the fourth warpgroup for setmaxnreg), 512 threads.
enum : int { kRoleSoftmax = 0, kRoleTma = 1, kRolePv = 2, kRoleS = 3, kRoleIdle = 4 };

template <int D, bool DUAL = false>
struct PCfg {
  static constexpr int kPipes = DUAL ? 2 : 1;
  static constexpr int kThreads = DUAL ? 512 : 224;
  static constexpr int kAllocWarp = DUAL ? 10 : 5;
  static constexpr int kBoxes = D / 64;
  static constexpr int kBox = 128 * 128;         // [128 rows][64 fp16]
  static constexpr int kTile = kBoxes * kBox;    // Q tile, or K (V) of one step
  static constexpr int kNS = DUAL ? 1 : 3;       // TMEM S buffers (per pipeline)
  static constexpr int kNO = D == 64 ? 2 : 1;    // TMEM O buffers (by item)
  static constexpr int kNQ = (D == 64 && !DUAL) ? 2 : 1;  // Q tiles in shared memory (by item)
  static constexpr int kST = DUAL ? 2 : (D == 64 ? 4 : 3);  // K/V stages (K and V rings filled independently)
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + kNQ * kTile;
  static constexpr int kV = kK + kST * kTile;
  // per-warp staging of the item epilogue's output rows (32 rows x D x up to 4
  // bytes), so the global stores cover whole rows; head_dim 64 only (at 128
  // the K/V stages take the room)
  static constexpr int kOut = kV + kST * kTile;
  static constexpr int kOutBytes = D == 64 ? 4 * 32 * D * 4 : 0;
  static constexpr int kPipeBytes = kOut + kOutBytes;  // one pipeline's shared memory (1024-aligned)
  static constexpr int kBar = kPipes * kPipeBytes;
  // per pipeline: q_full, q_empty [2]; k_full, v_full, k_empty, v_empty [kST];
  // s_full, p_full [kNS]; o_done, o_free [2]
  static constexpr int kNumBars = 4 + 4 * kST + 2 * kNS + 4;
  static constexpr int kSmem = kBar + kPipes * kNumBars * 8 + 16 + 1024;
  static constexpr uint32_t kO = 128 * kNS, kCols = 512, kPipeCols = kCols / kPipes;
  static_assert(kO + kNO * D <= kPipeCols, "TMEM columns");
  static_assert(kPipeBytes % 1024 == 0, "pipeline base alignment");
};

// A work item and its step range: item it (longest first) -> query tile m of
// (sequence b, head h); the tile's steps are the 128-token KV tiles j0 .. j0+N-1.
struct PrefillItem {
  int b, h, row0, rows, j0, N, start;
};

__device__ __forceinline__ PrefillItem prefill_item(const PrefillParams& p, int it) {
  PrefillItem w;
  const int bh_count = p.batch * p.Hq;
  const int m = p.num_m - 1 - it / bh_count;
  const int bh = it % bh_count;
  w.b = bh / p.Hq;
  w.h = bh - w.b * p.Hq;
  w.start = p.start[w.b];
  w.row0 = m * 128;
  w.rows = min(128, p.S - w.row0);
  const int first_min = p.sliding > 0 ? max(0, w.start + w.row0 - p.sliding + 1) : 0;
  w.j0 = first_min / 128;
  w.N = (w.start + w.row0 + w.rows - 1) / 128 - w.j0 + 1;
  return w;
}


template <int D, typename OUT, bool DUAL>
__global__ void __launch_bounds__(PCfg<D, DUAL>::kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ PrefillParams p) {
  using C = PCfg<D, DUAL>;
  constexpr int kT = 128, NS = C::kNS;
  static_assert(NS <= 3, "the o_done parity argument needs S(g) to be issued after P V(g-3) or later");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int role, pipe = 0;
  if constexpr (DUAL) {
    role = warp < 8 ? kRoleSoftmax : (warp < 10 ? kRoleTma : (warp < 12 ? kRolePv : (warp < 14 ? kRoleS : kRoleIdle)));
    pipe = warp < 8 ? warp >> 2 : (warp - 8) & 1;
  } else {
    role = warp < 4 ? kRoleSoftmax : (warp == 4 ? kRoleTma : (warp == 5 ? kRolePv : kRoleS));
  }
  uint8_t* const ps = smem + pipe * C::kPipeBytes;  // this pipeline's shared memory
  uint64_t* const bars0 = reinterpret_cast<uint64_t*>(smem + C::kBar);
  uint64_t* bars = bars0 + pipe * C::kNumBars;
  uint64_t* q_full = bars;  // [item % NQ]
  uint64_t* q_empty = bars + 2;
  uint64_t* k_full = bars + 4;
  uint64_t* v_full = k_full + C::kST;
  uint64_t* k_empty = v_full + C::kST;
  uint64_t* v_empty = k_empty + C::kST;
  uint64_t* s_full = v_empty + C::kST;  // [g % NS]
  uint64_t* p_full = s_full + NS;       // [g % NS]
  uint64_t* o_done = p_full + NS;       // [g & 1]
  uint64_t* o_free = o_done + 2;        // [item % NO]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars0 + C::kPipes * C::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int num_items = p.num_m * p.batch * p.Hq;

  if (tid == 0) {
    for (int pp = 0; pp < C::kPipes; ++pp) {
      uint64_t* b = bars0 + pp * C::kNumBars;
      for (int i = 0; i < 4 + 4 * C::kST; ++i) mbar_init(&b[i], 1);  // q, k, v rings
      for (int i = 0; i < NS; ++i) {
        mbar_init(&b[4 + 4 * C::kST + i], 1);       // s_full
        mbar_init(&b[4 + 4 * C::kST + NS + i], 128);  // p_full
      }
      mbar_init(&b[4 + 4 * C::kST + 2 * NS], 1);        // o_done [2]
      mbar_init(&b[4 + 4 * C::kST + 2 * NS + 1], 1);
      mbar_init(&b[4 + 4 * C::kST + 2 * NS + 2], 128);  // o_free [2]
      mbar_init(&b[4 + 4 * C::kST + 2 * NS + 3], 128);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == C::kAllocWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot + static_cast<uint32_t>(pipe) * C::kPipeCols;  // this pipeline's columns
  griddep_wait();  // the RoPE/append kernel's queries and cache rows are complete
  auto wait = [&](uint64_t* bar, uint32_t parity) {
    if (*abort_flag) return;
    if (!mbar_wait(bar, parity, p.error)) *abort_flag = 1;
  };

  if (role != kRoleSoftmax) {
  // Two pipelines: 512 threads x 128 registers at launch; the two control
  // warpgroups (warps 8-15) give theirs down to 56 and the two softmax
  // warpgroups take 200 (2 x 128 x 56 + 2 x 128 x 200 = 65536, the launch's
  // total). setmaxnreg is issued once per warpgroup branch, by all four of its
  // warps.
  if constexpr (DUAL) asm volatile("setmaxnreg.dec.sync.aligned.u32 56;" ::: "memory");
  if (role == kRoleTma) {
    // ================================================================ TMA producer
    // lane 0: Q of each item, then its K tiles; lane 1: the V tiles. S runs
    // up to NS steps ahead of P V, so K must not queue behind V.
    if (lane < 2) {
      const CUtensorMap* map = lane == 0 ? &p.tm_k : &p.tm_v;
      uint64_t* full = lane == 0 ? k_full : v_full;
      uint64_t* empty = lane == 0 ? k_empty : v_empty;
      uint8_t* ring = ps + (lane == 0 ? C::kK : C::kV);
      tma_prefetch(map);
      if (lane == 0) tma_prefetch(&p.tm_q);
      int g = 0;
      for (int k = 0;; ++k) {
        const int it = prefill_item_of(k * C::kPipes + pipe, num_items);
        if (it < 0) break;
        const PrefillItem w = prefill_item(p, it);
        const int z = w.b * p.Hk + w.h / p.G;
        if (lane == 0) {
          const int qi = k % C::kNQ;
          wait(&q_empty[qi], ((k / C::kNQ) & 1) ^ 1);
          if (!*abort_flag) {
            mbar_arrive_expect_tx(&q_full[qi], C::kTile);
#pragma unroll
            for (int x = 0; x < C::kBoxes; ++x)
              tma_load_3d(ps + C::kQ + qi * C::kTile + x * C::kBox, &p.tm_q, &q_full[qi], x * 64, w.row0,
                          w.b * p.Hq + w.h);
          }
        }
        for (int n = 0; n < w.N; ++n, ++g) {
          const int st = g % C::kST;
          wait(&empty[st], ((g / C::kST) & 1) ^ 1);
          if (!*abort_flag) {
            mbar_arrive_expect_tx(&full[st], C::kTile);
#pragma unroll
            for (int x = 0; x < C::kBoxes; ++x)
              tma_load_3d(ring + st * C::kTile + x * C::kBox, map, &full[st], x * 64, (w.j0 + n) * kT, z);
          }
        }
      }
      for (int q = max(0, g - C::kST); q < g; ++q)  // no copies in flight at exit
        wait(&full[q % C::kST], (q / C::kST) & 1);
    }
  } else if (role == kRolePv || role == kRoleS) {
    // ================================================================ MMA issuers
    // Two issuing threads, so that one's waits, commits and bookkeeping
    // overlap the other's MMAs: warp kSWarp issues every S(g) (S(g) for
    // g >= NS once P V(g - NS) has completed, i.e. has read P(g - NS) from
    // the buffer S(g) overwrites), warp kMmaWarp every P V(g) once the
    // softmax has stored P(g). A tcgen05.commit tracks the issuing thread's
    // own MMAs, and each barrier has a single committing thread.
    if (lane == 0) {
      constexpr uint32_t kIdS = idesc_f16(128, kT, false);
      constexpr uint32_t kIdO = idesc_f16(128, D, true);
      auto spin = [&](uint64_t* bar, uint32_t parity) {
        if (!*abort_flag && !mbar_spin(bar, parity, p.error)) *abort_flag = 1;
      };
      // Descriptors are linear in the start address (bits 0-13 = addr >> 4, no
      // carry below 256 KB), so buffer, stage, box and k-step offsets are plain adds.
      const uint64_t dq = sdesc(smem_u32(ps + C::kQ), 16, 1024);
      const uint64_t dk = sdesc(smem_u32(ps + C::kK), 16, 1024);
      const uint64_t dv = sdesc(smem_u32(ps + C::kV), C::kBox, 1024);
      if (role == kRoleS) {
        // S cursor: item ks, local step ns, global step gs
        int ks = 0, ns = 0, gs = 0, its = prefill_item_of(pipe, num_items);
        int Ns = its >= 0 ? prefill_item(p, its).N : 0;
        while (its >= 0) {  // S(gs) = Q K(gs)^T into buffer gs % NS
          // P V(gs - NS) has read P from this buffer (its barrier last
          // completed for P V(gs - NS - 2), which the previous wait covers)
          if (gs >= NS) wait(&o_done[(gs - NS) & 1], ((gs - NS) >> 1) & 1);
          if (ns == 0) spin(&q_full[ks % C::kNQ], (ks / C::kNQ) & 1);
          const int st = gs % C::kST;
          spin(&k_full[st], (gs / C::kST) & 1);
          PTRACE(8, gs);
          const uint64_t qb = dq + static_cast<uint64_t>((ks % C::kNQ) * (C::kTile >> 4));
          const uint64_t kb = dk + static_cast<uint64_t>(st * (C::kTile >> 4));
          const uint32_t d = tmem + 128 * (gs % NS);
          if (!*abort_flag) {
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t off = ((kk >> 2) * C::kBox + (kk & 3) * 32) >> 4;
              mma_f16(d, qb + off, kb + off, kIdS, kk > 0 ? 1u : 0u);
            }
          }
          mma_commit(&s_full[gs % NS]);
          mma_commit(&k_empty[st]);
          PTRACE(9, gs);
          ++gs;
          if (++ns == Ns) {  // this item's last S: its Q tile is free
            mma_commit(&q_empty[ks % C::kNQ]);
            ns = 0;
            its = prefill_item_of(++ks * C::kPipes + pipe, num_items);
            Ns = its >= 0 ? prefill_item(p, its).N : 0;
          }
        }
      } else {
        // P V cursor: item kp, local step np, global step gp
        int kp = 0, np = 0, gp = 0, itp = prefill_item_of(pipe, num_items);
        int Np = itp >= 0 ? prefill_item(p, itp).N : 0;
        while (itp >= 0) {  // O(item) += P(gp) V(gp) once the softmax step is done
          const int st = gp % C::kST;
          if (np == 0 && kp >= C::kNO)  // the epilogue of item kp - NO has read this O buffer
            spin(&o_free[kp % C::kNO], ((kp / C::kNO) - 1) & 1);
          PTRACE(12, gp);
          spin(&v_full[st], (gp / C::kST) & 1);
          PTRACE(13, gp);
          // the softmax step is usually still running: sleep on the barrier
          // instead of spinning, which would take issue slots from the softmax
          // warp on this sub-partition
          wait(&p_full[gp % NS], (gp / NS) & 1);
          tc_fence_after();
          PTRACE(10, gp);
          const uint64_t vb = dv + static_cast<uint64_t>(st * (C::kTile >> 4));
          const uint32_t a = tmem + 128 * (gp % NS);
          const uint32_t o = tmem + C::kO + D * (kp % C::kNO);
          if (!*abort_flag) {
#pragma unroll
            for (int kk = 0; kk < kT / 16; ++kk)
              mma_f16_ts(o, a + kk * 8, vb + 128 * kk, kIdO, (np > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&o_done[gp & 1]);
          mma_commit(&v_empty[st]);
          PTRACE(11, gp);
          ++gp;
          if (++np == Np) {
            np = 0;
            itp = prefill_item_of(++kp * C::kPipes + pipe, num_items);
            Np = itp >= 0 ? prefill_item(p, itp).N : 0;
          }
        }
      }
    }
  }
  } else {
    if constexpr (DUAL) asm volatile("setmaxnreg.inc.sync.aligned.u32 200;" ::: "memory");
    // ================================================================ softmax
    const int r = tid & 127;  // query row = TMEM lane
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const float sl2 = p.scale_log2;
    int g = 0;
    // The completion wait of a step's P stores and its p_full arrival are
    // deferred until the next step's S is loaded, so the TMEM store and load
    // latencies overlap (different S buffers; the MMA issuer only needs P(g)
    // before P V(g)).
    int pend_j = -1;
    auto release_p = [&]() {
      if (pend_j >= 0) {
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[pend_j]);
        pend_j = -1;
      }
    };
    // Item epilogue: normalise and store this row's outputs of item ke (its
    // last step is global step last), then free its O buffer. It runs inside
    // the first step of the next item, after that step's P is stored, so the
    // softmax goes on to the next item's S without waiting for P V(last)
    // (O is double-buffered by item at head_dim 64; at 128 the next item's
    // first P V waits for o_free). There, S(last + 1) complete implies
    // P V(last - 2), and P(last + 1) is not yet released, so the barrier of
    // P V(last - 1) is one phase from it, and so is that of P V(last) once
    // P V(last - 1) has completed. After the last item the same waits hold
    // with S(last) seen (P V(last - 3) complete).
    auto epilogue = [&](int ke, long long base, int rows, float le, int last) {
      // (one pipeline per CTA: P V(last - 1) first, so that no wait here is on an
      // ambiguous phase; two pipelines: P V(last) implies P V(last - 1), the
      // same thread's earlier MMAs, and P V(last + 1) may have completed)
      if (!DUAL && last >= 1) wait(&o_done[(last - 1) & 1], ((last - 1) >> 1) & 1);
      wait(&o_done[last & 1], (last >> 1) & 1);
      __syncwarp();
      tc_fence_after();
      const uint32_t oe = lane_addr + C::kO + D * (ke % C::kNO);
      const float inv = le > 0.f ? 1.f / le : 0.f;
      const size_t row_stride = static_cast<size_t>(p.Hq) * D;  // elements between consecutive tokens
      OUT* const dst0 = static_cast<OUT*>(p.out) + base;        // row 0 of the item's tile
      // Output gate (TSLAttention.ts:418-423, math.ts:271-273): this row's 32
      // columns times sigmoid(gate), in fp32 before the conversion to OUT.
      auto gate_cols = [&](float (&o)[32], int c) {
        if (p.gate == nullptr || r >= rows) return;
        if (!TLA_IN_BOUNDS(base + r * row_stride + 32 * c + 31, static_cast<long long>(p.batch) * p.S * p.Hq * D,
                           p.error))
          return;
        float gv[32];
        load_row32(static_cast<const OUT*>(p.gate) + base + r * row_stride + 32 * c, gv);
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = o[i] * (1.f / (1.f + expf(-gv[i])));
      };
      if constexpr (C::kOutBytes > 0) {
        // Rows go through this warp's shared-memory stage (16-byte chunks
        // XOR-swizzled by row, so neither side has bank conflicts) and leave
        // as whole 128- or 256-byte rows: a warp-wide store covers 4 (2) rows
        // instead of 16 bytes of 32 rows.
        constexpr int kRowBytes = D * static_cast<int>(sizeof(OUT));
        constexpr int kChunks = kRowBytes / 16;
        constexpr int kPer32 = 32 * static_cast<int>(sizeof(OUT)) / 16;  // chunks per 32 values
        uint8_t* stage = ps + C::kOut + (warp & 3) * 32 * kRowBytes;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          float o[32];
          tmem_ld32(oe + 32 * c, o);
          gate_cols(o, c);
#pragma unroll
          for (int i = 0; i < kPer32; ++i) {
            uint4 v;
            if constexpr (sizeof(OUT) == 2) {
              const float* f = o + 8 * i;
              v = make_uint4(pack_half2(f[0] * inv, f[1] * inv), pack_half2(f[2] * inv, f[3] * inv),
                             pack_half2(f[4] * inv, f[5] * inv), pack_half2(f[6] * inv, f[7] * inv));
            } else {
              const float* f = o + 4 * i;
              v = make_uint4(__float_as_uint(f[0] * inv), __float_as_uint(f[1] * inv), __float_as_uint(f[2] * inv),
                             __float_as_uint(f[3] * inv));
            }
            const int q = c * kPer32 + i;
            *reinterpret_cast<uint4*>(stage + lane * kRowBytes + ((q ^ (lane & 7)) << 4)) = v;
          }
        }
        __syncwarp();
        constexpr int kRowsPer = 32 / kChunks;
        const int q = lane % kChunks;
        const uint8_t* src = stage + (lane / kChunks) * kRowBytes;
        int row = (warp & 3) * 32 + lane / kChunks;
        uint8_t* dst = reinterpret_cast<uint8_t*>(dst0 + row * row_stride) + (q << 4);
        const size_t dst_step = kRowsPer * row_stride * sizeof(OUT);
#pragma unroll 1
        for (int it = 0; it < kChunks; ++it, row += kRowsPer, src += kRowsPer * kRowBytes, dst += dst_step) {
          const uint4 v = *reinterpret_cast<const uint4*>(src + ((q ^ (row & 7)) << 4));
          if (row < rows &&
              TLA_IN_BOUNDS(base + row * row_stride + ((q + 1) * 16) / sizeof(OUT) - 1,
                            static_cast<long long>(p.batch) * p.S * p.Hq * D, p.error))
            *reinterpret_cast<uint4*>(dst) = v;
        }
        __syncwarp();  // the stage is reused by the next epilogue
      } else {
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          float o[32];
          tmem_ld32(oe + 32 * c, o);
          gate_cols(o, c);
          if (r < rows && TLA_IN_BOUNDS(base + r * row_stride + 32 * c + 31,
                                        static_cast<long long>(p.batch) * p.S * p.Hq * D, p.error)) {
            OUT* dst = dst0 + r * row_stride + 32 * c;
            if constexpr (sizeof(OUT) == 2) {
#pragma unroll
              for (int i = 0; i < 32; i += 8)
                *reinterpret_cast<uint4*>(dst + i) =
                    make_uint4(pack_half2(o[i] * inv, o[i + 1] * inv), pack_half2(o[i + 2] * inv, o[i + 3] * inv),
                               pack_half2(o[i + 4] * inv, o[i + 5] * inv), pack_half2(o[i + 6] * inv, o[i + 7] * inv));
            } else {
#pragma unroll
              for (int i = 0; i < 32; i += 4)
                *reinterpret_cast<float4*>(dst + i) =
                    make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv, o[i + 3] * inv);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&o_free[ke % C::kNO]);
    };
    int e_k = -1, e_last = 0, e_rows = 0;  // the item whose epilogue is pending, its last step, its rows,
    long long e_base = 0;                  // the output offset of its first row,
    float e_l = 0.f;                       // and this row's softmax sum
    const uint32_t ninf = __float_as_uint(-INFINITY);
    int sj = 0;        // g % NS, kept incrementally (no division on the loop head)
    uint32_t sph = 0;  // (g / NS) & 1
    for (int k = 0;; ++k) {
      const int it = prefill_item_of(k * C::kPipes + pipe, num_items);
      if (it < 0) break;
      const PrefillItem w = prefill_item(p, it);
      const uint32_t o_addr = lane_addr + C::kO + D * (k % C::kNO);
      const int pr = w.start + w.row0 + r;
      const int first_r = p.sliding > 0 ? max(0, pr - p.sliding + 1) : 0;
      float m_run = -INFINITY, l_run = 0.f;
      for (int n = 0; n < w.N; ++n, ++g) {
        const int j = sj;
        const uint32_t buf = lane_addr + 128 * j;
        wait(&s_full[j], sph);
        if (++sj == NS) {
          sj = 0;
          sph ^= 1u;
        }
        if (tid == 0) PTRACE(0, g);
        __syncwarp();
        tc_fence_after();
        if (tid == 0) PTRACE(1, g);
        // Row maximum of the step -> moves the row's reference maximum (and
        // rescales O in TMEM) when exceeded by more than 2^8; returns the
        // maximum the exponentials subtract.
        auto apply_max = [&](float m_tile) -> float {
          const bool grow = m_tile > m_run + kRescaleLog2;
          if (__any_sync(0xffffffffu, grow)) {
            const float m_new = grow ? m_tile : m_run;
            // 0 while the row has seen no unmasked token (O and l are still zero), 1 when unchanged
            const float alpha = m_run == -INFINITY ? 0.f : ex2(m_run - m_new);
            if (n > 0) {  // rescale O in TMEM once P V(g-1) finished
              wait(&o_done[(g - 1) & 1], ((g - 1) >> 1) & 1);
              __syncwarp();
              tc_fence_after();
#pragma unroll
              for (int c = 0; c < D / 32; ++c) {
                float o[32];
                uint32_t u[32];
                tmem_ld32(o_addr + 32 * c, o);
#pragma unroll
                for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(o[i] * alpha);
                tmem_st32(o_addr + 32 * c, u);
              }
            }
            l_run *= alpha;
            m_run = m_new;
          }
          return m_run == -INFINITY ? 0.f : m_run;
        };
        if constexpr (!DUAL) {
          uint32_t sv[128];
          tmem_ld64x(buf, *reinterpret_cast<uint32_t(*)[64]>(&sv[0]));
          tmem_ld64x(buf + 64, *reinterpret_cast<uint32_t(*)[64]>(&sv[64]));
          if (tid == 0) PTRACE(2, g);
          release_p();  // the previous step's P (its P V may now be issued)
          const int tok0 = (w.j0 + n) * kT;
          const bool masked = tok0 + kT - 1 > pr || tok0 < first_r;
          float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
          if (masked) {
            // valid columns [lo, hi] (lo <= hi: first_r <= pr); one unsigned
            // compare and a select per column, no branch
            const int lo = first_r - tok0;
            const uint32_t span = static_cast<uint32_t>(pr - first_r);
#pragma unroll
            for (int i = 0; i < 128; ++i) sv[i] = static_cast<uint32_t>(i - lo) <= span ? sv[i] : ninf;
          }
#pragma unroll
          for (int i = 0; i < 128; i += 8) {  // four independent chains of three-input maxima
            mx[0] = fmax3(mx[0], __uint_as_float(sv[i]), __uint_as_float(sv[i + 1]));
            mx[1] = fmax3(mx[1], __uint_as_float(sv[i + 2]), __uint_as_float(sv[i + 3]));
            mx[2] = fmax3(mx[2], __uint_as_float(sv[i + 4]), __uint_as_float(sv[i + 5]));
            mx[3] = fmax3(mx[3], __uint_as_float(sv[i + 6]), __uint_as_float(sv[i + 7]));
          }
          const float mu = apply_max(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * sl2);
          // x = S * scale_log2 - mu and the row sum, two columns per instruction
          const uint64_t sl2x2 = pack_f32x2(sl2, sl2), nmu2 = pack_f32x2(-mu, -mu);
          uint64_t sum2[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t pk[32];
#pragma unroll
            for (int i = 0; i < 64; i += 2) {
              const int kc = 64 * c + i;
              const bool poly = poly_pair(kc / 2);
              float x0, x1;
              fma_f32x2(__uint_as_float(sv[kc]), __uint_as_float(sv[kc + 1]), sl2x2, nmu2, x0, x1);
              const float e0 = poly ? ex2_poly(x0) : ex2(x0);
              const float e1 = poly ? ex2_poly(x1) : ex2(x1);
              add_f32x2(sum2[(i >> 1) & 3], e0, e1);
              pk[i / 2] = pack_half2(e0, e1);
            }
            tmem_st32(buf + 32 * c, pk);
          }
          l_run += (sum_f32x2(sum2[0]) + sum_f32x2(sum2[1])) + (sum_f32x2(sum2[2]) + sum_f32x2(sum2[3]));
        } else {
          // Half width (two pipelines share the SM's registers): columns 0..63
          // stay in registers, the maximum of 64..127 is taken in 32-column
          // pieces; after the exponentials of the first half (P over S columns
          // 0..31, already read) the second half is reloaded (P over S columns
          // 32..63, also already read).
          const int tok0 = (w.j0 + n) * kT;
          const bool masked = tok0 + kT - 1 > pr || tok0 < first_r;
          const int lo = first_r - tok0;
          const uint32_t span = static_cast<uint32_t>(pr - first_r);
          uint32_t sa[64];
          tmem_ld64x(buf, sa);
          if (tid == 0) PTRACE(2, g);
          if (masked) {
#pragma unroll
            for (int i = 0; i < 64; ++i) sa[i] = static_cast<uint32_t>(i - lo) <= span ? sa[i] : ninf;
          }
          float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
          for (int i = 0; i < 64; i += 8) {
            mx[0] = fmax3(mx[0], __uint_as_float(sa[i]), __uint_as_float(sa[i + 1]));
            mx[1] = fmax3(mx[1], __uint_as_float(sa[i + 2]), __uint_as_float(sa[i + 3]));
            mx[2] = fmax3(mx[2], __uint_as_float(sa[i + 4]), __uint_as_float(sa[i + 5]));
            mx[3] = fmax3(mx[3], __uint_as_float(sa[i + 6]), __uint_as_float(sa[i + 7]));
          }
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            float t[32];
            tmem_ld32(buf + 64 + 32 * c, t);
            if (masked) {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                t[i] = static_cast<uint32_t>(64 + 32 * c + i - lo) <= span ? t[i] : -INFINITY;
            }
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              mx[0] = fmax3(mx[0], t[i], t[i + 1]);
              mx[1] = fmax3(mx[1], t[i + 2], t[i + 3]);
              mx[2] = fmax3(mx[2], t[i + 4], t[i + 5]);
              mx[3] = fmax3(mx[3], t[i + 6], t[i + 7]);
            }
          }
          const float mu = apply_max(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * sl2);
          const uint64_t sl2x2 = pack_f32x2(sl2, sl2), nmu2 = pack_f32x2(-mu, -mu);
          uint64_t sum2[4] = {0ull, 0ull, 0ull, 0ull};
          auto exps = [&](const uint32_t (&v)[64], int c0, uint32_t dst) {
            uint32_t pk[32];
#pragma unroll
            for (int i = 0; i < 64; i += 2) {
              const bool poly = poly_pair((c0 + i) / 2);
              float x0, x1;
              fma_f32x2(__uint_as_float(v[i]), __uint_as_float(v[i + 1]), sl2x2, nmu2, x0, x1);
              const float e0 = poly ? ex2_poly(x0) : ex2(x0);
              const float e1 = poly ? ex2_poly(x1) : ex2(x1);
              add_f32x2(sum2[(i >> 1) & 3], e0, e1);
              pk[i / 2] = pack_half2(e0, e1);
            }
            tmem_st32(dst, pk);
          };
          exps(sa, 0, buf);
          tmem_ld64x(buf + 64, sa);
          if (masked) {
#pragma unroll
            for (int i = 0; i < 64; ++i) sa[i] = static_cast<uint32_t>(64 + i - lo) <= span ? sa[i] : ninf;
          }
          exps(sa, 64, buf + 32);
          l_run += (sum_f32x2(sum2[0]) + sum_f32x2(sum2[1])) + (sum_f32x2(sum2[2]) + sum_f32x2(sum2[3]));
        }
        if (lane == 0) PTRACE(3 + warp, g);
        pend_j = j;
        // two pipelines: the next S of this pipeline waits for this step's P V
        // (one S buffer), so P is released at once
        if constexpr (DUAL) release_p();
        if (n == 0 && e_k >= 0) {  // the previous item's epilogue (its last P V is done by now)
          epilogue(e_k, e_base, e_rows, e_l, e_last);
          e_k = -1;
        }
      }
      e_k = k;
      e_base = ((static_cast<long long>(w.b) * p.S + w.row0) * p.Hq + w.h) * D;
      e_rows = w.rows;
      e_l = l_run;
      e_last = g - 1;
    }
    release_p();
    if (e_k >= 0) epilogue(e_k, e_base, e_rows, e_l, e_last);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == C::kAllocWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(*tmem_slot), "r"(C::kCols) : "memory");
  }
}

template <int D, typename OUT, bool DUAL>
cudaError_t set_smem() {
  return raise_smem_limit(reinterpret_cast<const void*>(prefill_tc_kernel<D, OUT, DUAL>), PCfg<D, DUAL>::kSmem);
}

}  // namespace

#ifdef TLA_PREFILL_TRACE
extern "C" int tla_debug_prefill_trace(unsigned long long* host, int count) {
  return cudaMemcpyFromSymbol(host, g_prefill_trace, sizeof(unsigned long long) * count) == cudaSuccess ? 0 : -1;
}
#endif

cudaError_t prefill_fast_configure(tla_layer* L) {
  L->fast_prefill = false;
  if (L->cache_fp32 || (L->D != 64 && L->D != 128) || L->G <= 0 || L->ctx->encode_tiled == nullptr) return cudaSuccess;
  const uint64_t planes = static_cast<uint64_t>(L->max_batch) * L->Hk;
  if (make_map(L, L->k_cache, L->max_tokens, planes, &L->tmap_k128) != CUDA_SUCCESS ||
      make_map(L, L->v_cache, L->max_tokens, planes, &L->tmap_v128) != CUDA_SUCCESS)
    return cudaSuccess;
  cudaError_t e;
  if (L->D == 64 && TLA_PREFILL_PP) {  // two query tiles per CTA
    e = pp_configure(L);
    L->prefill_smem = pp_smem();
  } else if (L->D == 64) {
    constexpr bool kDual = TLA_PREFILL_DUAL != 0;
    e = L->io_fp32 ? set_smem<64, float, kDual>() : set_smem<64, __half, kDual>();
    L->prefill_smem = PCfg<64, kDual>::kSmem;
  } else {
    e = L->io_fp32 ? set_smem<128, float, false>() : set_smem<128, __half, false>();
    L->prefill_smem = PCfg<128>::kSmem;
  }
  if (e != cudaSuccess) return e;
  L->fast_prefill = true;
  return cudaSuccess;
}

size_t prefill_scratch_bytes(const tla_layer* L, int batch, int seq_len) {
  const size_t q = (static_cast<size_t>(batch) * L->Hq * seq_len * L->D * sizeof(__half) + 255) & ~size_t(255);
  return q + ((L->D == 64 && TLA_PREFILL_PP && L->fast_prefill) ? pp_partial_bytes(L, batch, seq_len) : 0);
}

cudaError_t launch_prefill_fast(const tla_layer* L, const void* qkv, const int32_t* start, const void* gate, int batch,
                                int seq_len, void* out, cudaStream_t stream) {
  __half* qh = static_cast<__half*>(L->ctx->d_qscratch);
  cudaError_t e = launch_rope_append_half_q(L, qkv, start, batch, seq_len, qh, stream);
  if (e != cudaSuccess) return e;
  return launch_prefill_attention(L, start, gate, batch, seq_len, out, stream);
}

cudaError_t launch_prefill_attention(const tla_layer* L, const int32_t* start, const void* gate, int batch,
                                     int seq_len, void* out, cudaStream_t stream) {
  __half* qh = static_cast<__half*>(L->ctx->d_qscratch);
  PrefillParams p;
  if (make_map(L, qh, seq_len, static_cast<uint64_t>(batch) * L->Hq, &p.tm_q) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  p.tm_k = L->tmap_k128;
  p.tm_v = L->tmap_v128;
  p.out = out;
  p.gate = gate;
  p.start = start;
  p.error = L->ctx->d_error;
  p.piece_len = 0;
  p.part = nullptr;
  p.S = seq_len;
  p.Hq = L->Hq;
  p.Hk = L->Hk;
  p.G = L->G;
  p.sliding = L->sliding;
  p.batch = batch;
  p.scale_log2 = L->attn_scale * kLog2e;
  p.num_m = (seq_len + 127) / 128;
  if (L->D == 64 && TLA_PREFILL_PP) return launch_pp(L, p, stream);
  const int items = p.num_m * batch * L->Hq;
  const dim3 grid(static_cast<unsigned>(items < L->ctx->sm_count ? items : L->ctx->sm_count));
  if (L->D == 64) {
    constexpr bool kDual = TLA_PREFILL_DUAL != 0;
    using C = PCfg<64, kDual>;
    if (L->io_fp32)
      return launch_pdl(prefill_tc_kernel<64, float, kDual>, grid.x, C::kThreads, C::kSmem, stream, p);
    else
      return launch_pdl(prefill_tc_kernel<64, __half, kDual>, grid.x, C::kThreads, C::kSmem, stream, p);
  } else {
    using C = PCfg<128>;
    if (L->io_fp32)
      return launch_pdl(prefill_tc_kernel<128, float, false>, grid.x, C::kThreads, C::kSmem, stream, p);
    else
      return launch_pdl(prefill_tc_kernel<128, __half, false>, grid.x, C::kThreads, C::kSmem, stream, p);
  }
  return cudaGetLastError();
}

}  // namespace tla
