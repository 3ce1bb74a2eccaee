// Causal prefill attention on the 5th-generation tensor cores (tcgen05),
// fp16 K/V cache, head_dim 64 or 128.
//
// The reference has no prefill kernel: it replays the one-token decode graph
// for every prompt position (packages/three-llm/src/decoder/DecoderTSLRunner.ts:
// 472-480, 504-530), so position p attends to cache slots [window start, p]
// with every earlier prompt token already appended. This kernel computes the
// same outputs for a whole prompt chunk at once.
//
// One CTA per (128-row query tile, head, sequence), longest tiles first.
// Warp roles (kSoftmaxGroups * 128 + 64 threads):
//   warps 0..4*NW-1  softmax: NW warpgroups; thread (g, r) owns query row r
//                    (TMEM lane r) and columns [g*128/NW, (g+1)*128/NW) of
//                    each S tile and [g*D/NW, (g+1)*D/NW) of the output row.
//                    The NW partial row maxima meet in shared memory once per
//                    tile; the row sums stay split until the epilogue.
//   warp 4*NW        TMA producer (Q tile once, then K/V tiles through a 2-stage ring)
//   warp 4*NW+1      MMA issuer: S = Q K^T (M=128, N=128, K=head_dim) into one of
//                    two TMEM S buffers, O_tile = P V (M=128, N=head_dim, K=128)
//                    into one of two TMEM O buffers; tcgen05.commit signals mbarriers.
// P goes through shared memory in the canonical 128-byte-swizzled K-major
// layout. The softmax warps keep the running max / sum and their output
// columns in fp32 registers and fold each O_tile in one tile late, so the
// tensor core computes S(n+1) and PV(n) while the softmax works on tile n.
// Every mbarrier wait is bounded; on timeout the CTA records TLA_ERR_TIMEOUT,
// stops waiting, runs its remaining control flow and frees its TMEM.
#include <math.h>

#include "tla_device.cuh"
#include "tla_internal.h"

namespace tla {

namespace {

constexpr int kRows = 128;       // query rows per CTA (TMEM lanes)
constexpr int kCols = 128;       // kv tokens per tile
constexpr int kNW = 4;                          // softmax warpgroups
constexpr int kThreads = kNW * 128 + 64;
constexpr int kSoftmaxThreads = kNW * 128;
constexpr float kLog2e = 1.4426950408889634f;

template <int D>
struct PCfg {
  static constexpr int kBoxes = D / 64;
  static constexpr int kBoxBytes = 128 * 128;          // [128 rows][64 fp16]
  static constexpr int kTileBytes = kBoxes * kBoxBytes;
  static constexpr int kPB = D == 64 ? 2 : 1;           // P buffers
  static constexpr int kPBytes = 2 * kBoxBytes;        // [128 rows][128 fp16]
  static constexpr int kQ = 0;
  static constexpr int kST = D == 64 ? 3 : 2;          // K/V ring stages
  static constexpr int kK = kQ + kTileBytes;
  static constexpr int kV = kK + kST * kTileBytes;
  static constexpr int kP = kV + kST * kTileBytes;
  static constexpr int kBar = kP + kPB * kPBytes;
  // q_full, k_full/v_full/k_empty/v_empty [kST], s_full/s_free [2], p_full/p_free [kPB], o_full/o_free [2]
  static constexpr int kNumBars = 1 + 4 * kST + 4 + 2 * kPB + 4;
  static constexpr int kRed = kBar + kNumBars * 8 + 16;      // [2][kNW][128] row-max partials
  static constexpr int kSmem = kRed + 2 * kNW * 128 * 4 + 1024;
  static constexpr uint32_t kTmemCols = 512;           // S 2x128 + O 2xD
  static constexpr int kTmemO = 256;
};

struct PrefillParams {
  CUtensorMap tm_q;  // rotated queries [B*Hq][S][D] fp16
  CUtensorMap tm_k;  // cache [max_batch*Hk][max_tokens][D] fp16, 128-token boxes
  CUtensorMap tm_v;
  void* out;
  const int32_t* start;
  int* error;
  int S, Hq, Hk, G, sliding, batch, num_m;
  float scale_log2;
};

// ---------------------------------------------------------------- tcgen05 helpers
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  // sm_100 shared-memory matrix descriptor, 128-byte swizzle, version 1
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// kind::f16 instruction descriptor: fp16 A and B, fp32 accumulator, A K-major.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool b_mn_major) {
  return (1u << 4) | (b_mn_major ? (1u << 16) : 0u) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float (&v)[N]) {
  static_assert(N % 16 == 0, "TMEM loads come in 16-column pieces");
  if constexpr (N % 32 == 0) {
#pragma unroll
    for (int c = 0; c < N / 32; ++c) tmem_ld32(taddr + c * 32, *reinterpret_cast<float(*)[32]>(&v[c * 32]));
  } else {
#pragma unroll
    for (int c = 0; c < N / 16; ++c) tmem_ld16(taddr + c * 16, *reinterpret_cast<float(*)[16]>(&v[c * 16]));
  }
}

template <int D, typename OUT>
__global__ void __launch_bounds__(kThreads, 1) prefill_tc_kernel(const __grid_constant__ PrefillParams p) {
  using C = PCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + C::kST;
  uint64_t* k_empty = v_full + C::kST;
  uint64_t* v_empty = k_empty + C::kST;
  uint64_t* s_full = v_empty + C::kST;
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_free + 2;
  uint64_t* p_free = p_full + C::kPB;
  uint64_t* o_full = p_free + C::kPB;
  uint64_t* o_free = o_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // ---- work unit
  const int bh_count = p.batch * p.Hq;
  const int m = p.num_m - 1 - static_cast<int>(blockIdx.x) / bh_count;
  const int bh = static_cast<int>(blockIdx.x) % bh_count;
  const int b = bh / p.Hq, h = bh - b * p.Hq, kvh = h / p.G;
  const int start = p.start[b];
  const int row0 = m * kRows;
  const int rows = min(kRows, p.S - row0);
  const int pmin = start + row0, pmax = start + row0 + rows - 1;
  const int first_min = p.sliding > 0 ? max(0, pmin - p.sliding + 1) : 0;
  const int j0 = first_min / kCols, j1 = pmax / kCols;
  const int ntiles = j1 - j0 + 1;

  if (tid == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < C::kST; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], kSoftmaxThreads);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], kSoftmaxThreads);
    }
    for (int i = 0; i < C::kPB; ++i) {
      mbar_init(&p_full[i], kSoftmaxThreads);
      mbar_init(&p_free[i], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  constexpr int kProducerWarp = kNW * 4, kMmaWarp = kNW * 4 + 1;
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto wait = [&](uint64_t* bar, uint32_t parity) {
    if (*abort_flag) return;
    if (!mbar_wait(bar, parity, p.error)) *abort_flag = 1;
  };

  if (warp == kProducerWarp) {
    // ================================================================ TMA producer
    if (lane == 0) {
      tma_prefetch(&p.tm_q);
      tma_prefetch(&p.tm_k);
      tma_prefetch(&p.tm_v);
      mbar_arrive_expect_tx(q_full, C::kTileBytes);
#pragma unroll
      for (int x = 0; x < C::kBoxes; ++x)
        tma_load_3d(smem + C::kQ + x * C::kBoxBytes, &p.tm_q, q_full, x * 64, row0, b * p.Hq + h);
      for (int n = 0; n < ntiles; ++n) {
        const int st = n % C::kST;
        const uint32_t ph = ((n / C::kST) & 1) ^ 1;
        const int y = (j0 + n) * kCols, z = b * p.Hk + kvh;
        wait(&k_empty[st], ph);  // freed once S of the tile that used it completed
        if (!*abort_flag) {
          mbar_arrive_expect_tx(&k_full[st], C::kTileBytes);
#pragma unroll
          for (int x = 0; x < C::kBoxes; ++x)
            tma_load_3d(smem + C::kK + st * C::kTileBytes + x * C::kBoxBytes, &p.tm_k, &k_full[st], x * 64, y, z);
        }
        wait(&v_empty[st], ph);  // freed once its P V completed
        if (!*abort_flag) {
          mbar_arrive_expect_tx(&v_full[st], C::kTileBytes);
#pragma unroll
          for (int x = 0; x < C::kBoxes; ++x)
            tma_load_3d(smem + C::kV + st * C::kTileBytes + x * C::kBoxBytes, &p.tm_v, &v_full[st], x * 64, y, z);
        }
      }
      // no copies may be in flight when the CTA exits
      for (int n = max(0, ntiles - C::kST); n < ntiles; ++n) {
        wait(&k_full[n % C::kST], (n / C::kST) & 1);
        wait(&v_full[n % C::kST], (n / C::kST) & 1);
      }
    }
  } else if (warp == kMmaWarp) {
    // ================================================================ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdS = idesc_f16(kRows, kCols, false);
      constexpr uint32_t kIdO = idesc_f16(kRows, D, true);
      const uint32_t q_base = smem_u32(smem + C::kQ);
      wait(q_full, 0);
      for (int n = 0; n <= ntiles; ++n) {
        if (n < ntiles) {
          const int st = n % C::kST, sb = n & 1;
          wait(&k_full[st], (n / C::kST) & 1);
          wait(&s_free[sb], ((n >> 1) & 1) ^ 1);
          tc_fence_after();
          const uint32_t k_base = smem_u32(smem + C::kK + st * C::kTileBytes);
          if (!*abort_flag) {
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t off = (kk >> 2) * C::kBoxBytes + (kk & 3) * 32;
              mma_f16(tmem + sb * kCols, sdesc(q_base + off, 16, 1024), sdesc(k_base + off, 16, 1024), kIdS,
                      kk > 0 ? 1u : 0u);
            }
          }
          mma_commit(&s_full[sb]);
          mma_commit(&k_empty[st]);
        }
        if (n >= 1) {
          const int q = n - 1, st = q % C::kST, ob = q & 1, pb = q % C::kPB;
          wait(&p_full[pb], (q / C::kPB) & 1);
          wait(&v_full[st], (q / C::kST) & 1);
          wait(&o_free[ob], ((q >> 1) & 1) ^ 1);
          tc_fence_after();
          const uint32_t p_base = smem_u32(smem + C::kP + pb * C::kPBytes);
          const uint32_t v_base = smem_u32(smem + C::kV + st * C::kTileBytes);
          if (!*abort_flag) {
#pragma unroll
            for (int kk = 0; kk < kCols / 16; ++kk)
              mma_f16(tmem + C::kTmemO + ob * D, sdesc(p_base + (kk >> 2) * C::kBoxBytes + (kk & 3) * 32, 16, 1024),
                      sdesc(v_base + kk * 2048, C::kBoxBytes, 1024), kIdO, kk > 0 ? 1u : 0u);
          }
          mma_commit(&o_full[ob]);
          mma_commit(&v_empty[st]);
          mma_commit(&p_free[pb]);
        }
      }
    }
  } else {
    // ================================================================ softmax
    constexpr int CW = kCols / kNW;  // S columns per thread
    constexpr int DW = D / kNW;      // output columns per thread
    const int g = warp >> 2;         // warpgroup
    const int r = tid & 127;         // query row = TMEM lane
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const int pr = start + row0 + r;
    const int first_r = p.sliding > 0 ? max(0, pr - p.sliding + 1) : 0;
    const float sl2 = p.scale_log2;
    float* red = reinterpret_cast<float*>(smem + C::kRed);  // [2][kNW][128]
    float o[DW];
#pragma unroll
    for (int i = 0; i < DW; ++i) o[i] = 0.f;
    float m_run = -INFINITY, l_part = 0.f, alpha_prev = 0.f;
    auto absorb = [&](int q) {
      const int ob = q & 1;
      wait(&o_full[ob], (q >> 1) & 1);
      __syncwarp();
      tc_fence_after();
      float v[DW];
      tmem_ld<DW>(lane_addr + C::kTmemO + ob * D + g * DW, v);
#pragma unroll
      for (int i = 0; i < DW; ++i) o[i] = fmaf(o[i], alpha_prev, v[i]);
      tc_fence_before();
      mbar_arrive(&o_free[ob]);
    };
    for (int n = 0; n < ntiles; ++n) {
      const int sb = n & 1, pb = n % C::kPB;
      const int tok0 = (j0 + n) * kCols + g * CW;  // first token of this thread's columns
      const bool masked = tok0 + CW - 1 > pr || tok0 < first_r;
      wait(&s_full[sb], (n >> 1) & 1);
      __syncwarp();
      tc_fence_after();
      float sv[CW];
      tmem_ld<CW>(lane_addr + sb * kCols + g * CW, sv);
      if (masked) {
#pragma unroll
        for (int i = 0; i < CW; ++i) {
          const int tok = tok0 + i;
          sv[i] = (tok >= first_r && tok <= pr) ? sv[i] : -INFINITY;
        }
      }
      float mx[4] = {sv[0], sv[1], sv[2], sv[3]};
#pragma unroll
      for (int i = 4; i < CW; i += 4) {
        mx[0] = fmaxf(mx[0], sv[i]);
        mx[1] = fmaxf(mx[1], sv[i + 1]);
        mx[2] = fmaxf(mx[2], sv[i + 2]);
        mx[3] = fmaxf(mx[3], sv[i + 3]);
      }
      float* rb = red + (n & 1) * kNW * 128;
      rb[g * 128 + r] = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      named_barrier_sync(1, kSoftmaxThreads);
      float mt = rb[r];
#pragma unroll
      for (int k = 1; k < kNW; ++k) mt = fmaxf(mt, rb[k * 128 + r]);
      const float m_new = fmaxf(m_run, mt * sl2);
      const float mu = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = ex2(m_run - mu);
      wait(&p_free[pb], ((n / C::kPB) & 1) ^ 1);
      __syncwarp();
      float sum[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pk[CW / 2];
#pragma unroll
      for (int i = 0; i < CW; i += 2) {
        const float e0 = ex2(fmaf(sv[i], sl2, -mu));  // exp2(-inf) = 0 for masked tokens
        const float e1 = ex2(fmaf(sv[i + 1], sl2, -mu));
        sum[(i >> 1) & 3] += e0 + e1;
        pk[i / 2] = pack_half2(e0, e1);
      }
      uint8_t* prow = smem + C::kP + pb * C::kPBytes + r * 128;
#pragma unroll
      for (int q4 = 0; q4 < CW / 8; ++q4) {
        const int cc = g * (CW / 8) + q4;  // 16-byte chunk 0..15 of the 256-byte P row
        const int box = cc >> 3, ch = cc & 7;
        *reinterpret_cast<uint4*>(prow + box * C::kBoxBytes + ((ch ^ (r & 7)) << 4)) =
            make_uint4(pk[q4 * 4], pk[q4 * 4 + 1], pk[q4 * 4 + 2], pk[q4 * 4 + 3]);
      }
      l_part = fmaf(l_part, alpha, (sum[0] + sum[1]) + (sum[2] + sum[3]));
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[pb]);
      mbar_arrive(&s_free[sb]);
      if (n >= 1) absorb(n - 1);
      alpha_prev = alpha;
      m_run = m_new;
    }
    absorb(ntiles - 1);
    // ---- epilogue: total row sum, normalise and store this thread's columns
    float* rl = red + (ntiles & 1) * kNW * 128;  // the buffer the last tile did not use
    rl[g * 128 + r] = l_part;
    named_barrier_sync(1, kSoftmaxThreads);
    float l_run = 0.f;
#pragma unroll
    for (int k = 0; k < kNW; ++k) l_run += rl[k * 128 + r];
    if (r < rows) {
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      OUT* dst = static_cast<OUT*>(p.out) + ((static_cast<size_t>(b) * p.S + row0 + r) * p.Hq + h) * D + g * DW;
      if constexpr (sizeof(OUT) == 2) {
#pragma unroll
        for (int i = 0; i < DW; i += 8) {
          uint4 u = make_uint4(pack_half2(o[i] * inv, o[i + 1] * inv), pack_half2(o[i + 2] * inv, o[i + 3] * inv),
                               pack_half2(o[i + 4] * inv, o[i + 5] * inv), pack_half2(o[i + 6] * inv, o[i + 7] * inv));
          *reinterpret_cast<uint4*>(dst + i) = u;
        }
      } else {
#pragma unroll
        for (int i = 0; i < DW; i += 4)
          *reinterpret_cast<float4*>(dst + i) = make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv, o[i + 3] * inv);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kTmemCols) : "memory");
  }
}

// ---------------------------------------------------------------- head_dim 64: two Q tiles per CTA
// Two 128-row query tiles (Q0, Q1) of one (head, sequence) share every K/V
// tile. Each tile has its own softmax warpgroup in which a thread owns one
// whole row (no cross-warpgroup exchange), and the MMA warp alternates
// between them: while warpgroup 0 turns S0(n) into P0(n), the tensor core
// computes S1(n) and P1(n-1) V, and the other way round. P is written to
// TMEM with tcgen05.st and read from there as the A operand of P V; O
// accumulates in TMEM across tiles. A row's reference maximum only moves when
// the tile maximum exceeds it by more than 2^8 (then O is rescaled in TMEM,
// warp-uniformly, after the previous P V finished), so P stays <= 256 in fp16
// and most tiles need no correction.
constexpr int kThreads2 = 576;  // warps 0-15: four softmax warpgroups, 16: TMA, 17: MMA
constexpr float kRescaleLog2 = 8.f;

struct P2Cfg {
  static constexpr int kTile = 128 * 128;  // one [128][64] fp16 box
  static constexpr int kST = 3;            // K/V stages
  static constexpr int kQ0 = 0, kQ1 = kTile;
  static constexpr int kK = 2 * kTile;
  static constexpr int kV = kK + kST * kTile;
  static constexpr int kBar = kV + kST * kTile;
  // q_full, k_full/v_full/k_empty/v_empty [kST], s_full [2], p_full [2], o_done [2]
  static constexpr int kNumBars = 1 + 4 * kST + 6;
  static constexpr int kXch = kBar + kNumBars * 8 + 16;  // [2][2 tiles][2 halves][128] row maxima / sums
  static constexpr int kSmem = kXch + 2 * 2 * 2 * 128 * 4 + 1024;
  // TMEM columns
  static constexpr uint32_t kS = 0, kP = 256, kO = 384, kCols = 512;
};

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}



// Two 32-column loads in flight before one wait.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
  uint32_t r[64];
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
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// D (TMEM) += A (TMEM) * B (shared memory descriptor)
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}

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

#ifdef TLA_PREFILL_TRACE
// Optional pipeline trace (builds with -DTLA_PREFILL_TRACE only): SM clock of
// each event of block 0, [tile][event]; read with tla_debug_prefill_trace.
__device__ unsigned long long g_prefill_trace[64][16];
#define PTRACE(ev, n) \
  do { \
    if (blockIdx.x == 0 && (n) < 64) g_prefill_trace[(n)][(ev)] = clock64(); \
  } while (0)
#else
#define PTRACE(ev, n) \
  do { \
  } while (0)
#endif

#ifndef TLA_PREFILL_POLY_EVERY
#define TLA_PREFILL_POLY_EVERY 0  // every n-th pair of exponentials goes to the FMA pipe (0: none)
#endif

template <typename OUT>
__global__ void __launch_bounds__(kThreads2, 1) prefill_tc2_kernel(const __grid_constant__ PrefillParams p) {
  using C = P2Cfg;
  constexpr int D = 64;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + C::kST;
  uint64_t* k_empty = v_full + C::kST;
  uint64_t* v_empty = k_empty + C::kST;
  uint64_t* s_full = v_empty + C::kST;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_done = p_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const int bh_count = p.batch * p.Hq;
  const int m = p.num_m - 1 - static_cast<int>(blockIdx.x) / bh_count;  // 256-row block, longest first
  const int bh = static_cast<int>(blockIdx.x) % bh_count;
  const int b = bh / p.Hq, h = bh - b * p.Hq, kvh = h / p.G;
  const int start = p.start[b];
  const int row0 = m * 256;
  const int rows = min(256, p.S - row0);
  const int pmin = start + row0, pmax = start + row0 + rows - 1;
  const int first_min = p.sliding > 0 ? max(0, pmin - p.sliding + 1) : 0;
  const int j0 = first_min / kCols, j1 = pmax / kCols;
  const int N = j1 - j0 + 1;

  if (tid == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < C::kST; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 256);
      mbar_init(&o_done[i], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 17) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto wait = [&](uint64_t* bar, uint32_t parity) {
    if (*abort_flag) return;
    if (!mbar_wait(bar, parity, p.error)) *abort_flag = 1;
  };

  if (warp == 16) {
    // ================================================================ TMA producer
    if (lane == 0) {
      tma_prefetch(&p.tm_q);
      tma_prefetch(&p.tm_k);
      tma_prefetch(&p.tm_v);
      mbar_arrive_expect_tx(q_full, 2 * C::kTile);
      tma_load_3d(smem + C::kQ0, &p.tm_q, q_full, 0, row0, b * p.Hq + h);
      tma_load_3d(smem + C::kQ1, &p.tm_q, q_full, 0, row0 + 128, b * p.Hq + h);
      for (int n = 0; n < N; ++n) {
        const int st = n % C::kST;
        const uint32_t ph = ((n / C::kST) & 1) ^ 1;
        const int y = (j0 + n) * kCols, z = b * p.Hk + kvh;
        wait(&k_empty[st], ph);
        if (!*abort_flag) {
          mbar_arrive_expect_tx(&k_full[st], C::kTile);
          tma_load_3d(smem + C::kK + st * C::kTile, &p.tm_k, &k_full[st], 0, y, z);
        }
        wait(&v_empty[st], ph);
        if (!*abort_flag) {
          mbar_arrive_expect_tx(&v_full[st], C::kTile);
          tma_load_3d(smem + C::kV + st * C::kTile, &p.tm_v, &v_full[st], 0, y, z);
        }
      }
      for (int n = max(0, N - C::kST); n < N; ++n) {  // no copies in flight at exit
        wait(&k_full[n % C::kST], (n / C::kST) & 1);
        wait(&v_full[n % C::kST], (n / C::kST) & 1);
      }
    }
  } else if (warp == 17) {
    // ================================================================ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdS = idesc_f16(128, kCols, false);
      constexpr uint32_t kIdO = idesc_f16(128, D, true);
      const uint32_t q0 = smem_u32(smem + C::kQ0), q1 = smem_u32(smem + C::kQ1);
      auto issue_s = [&](int t, int n) {  // S_t = Q_t K(n)^T
        const uint32_t kb = smem_u32(smem + C::kK + (n % C::kST) * C::kTile);
        const uint32_t qb = t == 0 ? q0 : q1;
        if (!*abort_flag) {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            mma_f16(tmem + C::kS + t * 128, sdesc(qb + kk * 32, 16, 1024), sdesc(kb + kk * 32, 16, 1024), kIdS,
                    kk > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[t]);
      };
      auto issue_pv = [&](int t, int n) {  // O_t += P_t V(n)
        const uint32_t vb = smem_u32(smem + C::kV + (n % C::kST) * C::kTile);
        if (!*abort_flag) {
#pragma unroll
          for (int kk = 0; kk < kCols / 16; ++kk)
            mma_f16_ts(tmem + C::kO + t * D, tmem + C::kP + t * 64 + kk * 8, sdesc(vb + kk * 2048, 16384, 1024),
                       kIdO, (n > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&o_done[t]);
      };
      wait(q_full, 0);
      wait(&k_full[0], 0);
      tc_fence_after();
      issue_s(0, 0);
      issue_s(1, 0);
      mma_commit(&k_empty[0]);
      for (int n = 0; n < N; ++n) {
        const bool more = n + 1 < N;
        const int st1 = (n + 1) % C::kST;
        wait(&p_full[0], n & 1);  // S0(n) consumed, P0(n) in TMEM
        PTRACE(8, n);
        if (more) wait(&k_full[st1], ((n + 1) / C::kST) & 1);
        wait(&v_full[n % C::kST], (n / C::kST) & 1);
        tc_fence_after();
        PTRACE(9, n);
        if (more) issue_s(0, n + 1);
        issue_pv(0, n);
        wait(&p_full[1], n & 1);
        tc_fence_after();
        PTRACE(10, n);
        if (more) {
          issue_s(1, n + 1);
          mma_commit(&k_empty[st1]);
        }
        issue_pv(1, n);
        mma_commit(&v_empty[n % C::kST]);
        PTRACE(11, n);
      }
    }
  } else {
    // ================================================================ softmax
    // warpgroup g: Q tile t = g >> 1, column half hc = g & 1. The two warpgroups
    // of a tile hold the same rows (TMEM lanes); they meet once per tile in
    // shared memory for the row maximum and keep separate row sums.
    const int g = warp >> 2, t = g >> 1, hc = g & 1;
    const int r = tid & 127;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const uint32_t s_addr = lane_addr + C::kS + t * 128 + hc * 64;  // this half's 64 S columns
    const uint32_t p_addr = lane_addr + C::kP + t * 64 + hc * 32;   // its 32 columns of fp16 pairs
    const uint32_t o_addr = lane_addr + C::kO + t * D + hc * 32;    // its 32 output columns
    float* xch = reinterpret_cast<float*>(smem + C::kXch);
    auto xslot = [&](int buf, int half) -> float& { return xch[((buf * 2 + t) * 2 + half) * 128 + r]; };
    const bool tracer = hc == 0 && (warp & 3) == 0 && lane == 0;
    const int pr = start + row0 + t * 128 + r;
    const int first_r = p.sliding > 0 ? max(0, pr - p.sliding + 1) : 0;
    const float sl2 = p.scale_log2;
    float m_run = -INFINITY, l_part = 0.f;
    for (int n = 0; n < N; ++n) {
      const int tok0 = (j0 + n) * kCols + hc * 64;  // first token of this half
      const bool masked = tok0 + 63 > pr || tok0 < first_r;
      const int lo = first_r - tok0, hi = pr - tok0;  // valid columns [lo, hi] of this half
      wait(&s_full[t], n & 1);
      __syncwarp();
      tc_fence_after();
      if (tracer) PTRACE(4 * t + 0, n);
      // pass 1: this half's maximum, then the row maximum with the other half
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll 1
      for (int ch = 0; ch < 2; ++ch) {
        float v[32];
        tmem_ld32(s_addr + ch * 32, v);
        if (!masked) {
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            mx[0] = fmaxf(mx[0], v[i]);
            mx[1] = fmaxf(mx[1], v[i + 1]);
            mx[2] = fmaxf(mx[2], v[i + 2]);
            mx[3] = fmaxf(mx[3], v[i + 3]);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int k = ch * 32 + i;
            mx[i & 3] = fmaxf(mx[i & 3], (k >= lo && k <= hi) ? v[i] : -INFINITY);
          }
        }
      }
      const float pm = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      xslot(n & 1, hc) = pm;
      named_barrier_sync(1 + t, 256);
      const float m_tile = fmaxf(pm, xslot(n & 1, hc ^ 1)) * sl2;
      if (tracer) PTRACE(4 * t + 2, n);
      // move the reference maximum only when this tile exceeds it by more than 2^8
      const bool grow = m_tile > m_run + kRescaleLog2;
      if (n > 0) {  // P_t is free and O_t stable once the previous P V finished
        wait(&o_done[t], (n - 1) & 1);
        __syncwarp();
        tc_fence_after();
      }
      if (tracer) PTRACE(4 * t + 1, n);
      if (__any_sync(0xffffffffu, grow)) {
        const float m_new = grow ? m_tile : m_run;
        // 0 while the row has seen no unmasked token (O and l are still zero), 1 when unchanged
        const float alpha = m_run == -INFINITY ? 0.f : ex2(m_run - m_new);
        if (n > 0) {  // rescale this half of O in TMEM
          float o[32];
          uint32_t u[32];
          tmem_ld32(o_addr, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(o[i] * alpha);
          tmem_st32(o_addr, u);
        }
        l_part *= alpha;
        m_run = m_new;
      }
      const float mu = m_run == -INFINITY ? 0.f : m_run;
      // pass 2: P = 2^(s*scale - mu) to TMEM as fp16 pairs
      float sum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
      for (int ch = 0; ch < 2; ++ch) {
        float v[32];
        tmem_ld32(s_addr + ch * 32, v);
        uint32_t pk[16];
        if (!masked) {
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const bool poly = TLA_PREFILL_POLY_EVERY > 0 && (i / 2) % TLA_PREFILL_POLY_EVERY == TLA_PREFILL_POLY_EVERY - 1;
            const float x0 = fmaf(v[i], sl2, -mu), x1 = fmaf(v[i + 1], sl2, -mu);
            const float e0 = poly ? ex2_poly(x0) : ex2(x0);
            const float e1 = poly ? ex2_poly(x1) : ex2(x1);
            sum[(i >> 1) & 3] += e0 + e1;
            pk[i / 2] = pack_half2(e0, e1);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const int k = ch * 32 + i;
            const float e0 = (k >= lo && k <= hi) ? ex2(fmaf(v[i], sl2, -mu)) : 0.f;
            const float e1 = (k + 1 >= lo && k + 1 <= hi) ? ex2(fmaf(v[i + 1], sl2, -mu)) : 0.f;
            sum[(i >> 1) & 3] += e0 + e1;
            pk[i / 2] = pack_half2(e0, e1);
          }
        }
        tmem_st16(p_addr + ch * 16, pk);
      }
      tmem_wait_st();
      l_part += (sum[0] + sum[1]) + (sum[2] + sum[3]);
      tc_fence_before();
      mbar_arrive(&p_full[t]);
      if (tracer) PTRACE(4 * t + 3, n);
    }
    // ---- epilogue: row sum of both halves, normalise and store this half's 32 columns
    xslot(N & 1, hc) = l_part;
    named_barrier_sync(1 + t, 256);
    const float l_run = l_part + xslot(N & 1, hc ^ 1);
    wait(&o_done[t], (N - 1) & 1);
    __syncwarp();
    tc_fence_after();
    const int row = row0 + t * 128 + r;
    const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
    float o[32];
    tmem_ld32(o_addr, o);
    if (row < p.S) {
      OUT* dst = static_cast<OUT*>(p.out) + ((static_cast<size_t>(b) * p.S + row) * p.Hq + h) * D + hc * 32;
      if constexpr (sizeof(OUT) == 2) {
#pragma unroll
        for (int i = 0; i < 32; i += 8)
          *reinterpret_cast<uint4*>(dst + i) =
              make_uint4(pack_half2(o[i] * inv, o[i + 1] * inv), pack_half2(o[i + 2] * inv, o[i + 3] * inv),
                         pack_half2(o[i + 4] * inv, o[i + 5] * inv), pack_half2(o[i + 6] * inv, o[i + 7] * inv));
      } else {
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          *reinterpret_cast<float4*>(dst + i) = make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv, o[i + 3] * inv);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 17) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kCols) : "memory");
  }
}

CUresult make_map(const tla_layer* L, void* base, uint64_t rows, uint64_t planes, CUtensorMap* map) {
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(L->D), rows, planes};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(L->D) * 2, static_cast<cuuint64_t>(L->D) * 2 * rows};
  const cuuint32_t box[3] = {64, 128, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return L->ctx->encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, base, dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

template <int D, typename OUT>
cudaError_t set_smem() {
  return cudaFuncSetAttribute(prefill_tc_kernel<D, OUT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              PCfg<D>::kSmem);
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
  if (L->D == 64) {
    e = L->io_fp32 ? cudaFuncSetAttribute(prefill_tc2_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          P2Cfg::kSmem)
                   : cudaFuncSetAttribute(prefill_tc2_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          P2Cfg::kSmem);
    L->prefill_smem = P2Cfg::kSmem;
  } else {
    e = L->io_fp32 ? set_smem<128, float>() : set_smem<128, __half>();
    L->prefill_smem = PCfg<128>::kSmem;
  }
  if (e != cudaSuccess) return e;
  L->fast_prefill = true;
  return cudaSuccess;
}

cudaError_t launch_prefill_fast(const tla_layer* L, const void* qkv, const int32_t* start, int batch, int seq_len,
                                void* out, cudaStream_t stream) {
  __half* qh = static_cast<__half*>(L->ctx->d_qscratch);
  cudaError_t e = launch_rope_append_half_q(L, qkv, start, batch, seq_len, qh, stream);
  if (e != cudaSuccess) return e;
  PrefillParams p;
  if (make_map(L, qh, seq_len, static_cast<uint64_t>(batch) * L->Hq, &p.tm_q) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  p.tm_k = L->tmap_k128;
  p.tm_v = L->tmap_v128;
  p.out = out;
  p.start = start;
  p.error = L->ctx->d_error;
  p.S = seq_len;
  p.Hq = L->Hq;
  p.Hk = L->Hk;
  p.G = L->G;
  p.sliding = L->sliding;
  p.batch = batch;
  p.scale_log2 = L->attn_scale * kLog2e;
  if (L->D == 64) {
    p.num_m = (seq_len + 255) / 256;
    const dim3 grid(static_cast<unsigned>(p.num_m * batch * L->Hq));
    if (L->io_fp32)
      prefill_tc2_kernel<float><<<grid, kThreads2, P2Cfg::kSmem, stream>>>(p);
    else
      prefill_tc2_kernel<__half><<<grid, kThreads2, P2Cfg::kSmem, stream>>>(p);
  } else {
    p.num_m = (seq_len + kRows - 1) / kRows;
    const dim3 grid(static_cast<unsigned>(p.num_m * batch * L->Hq));
    if (L->io_fp32)
      prefill_tc_kernel<128, float><<<grid, kThreads, PCfg<128>::kSmem, stream>>>(p);
    else
      prefill_tc_kernel<128, __half><<<grid, kThreads, PCfg<128>::kSmem, stream>>>(p);
  }
  return cudaGetLastError();
}

}  // namespace tla
