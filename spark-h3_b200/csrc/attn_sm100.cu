// Sparse attention forward on the 5th-generation tensor cores (sm_100a), bf16, D = 128.
//
// One CTA per (128-row query tile, head, batch).  Roles (384 threads):
//   warps 0-3  softmax group 0: row r = TMEM lane r, key columns 0-63 of every tile
//   warps 4-7  softmax group 1: row r = TMEM lane r, key columns 64-127 of every tile
//   warp 8     TMA producer of Q and the K (or AK summary) tiles, 2 stages
//   warp 9     TMA producer of the V (or AV summary) tiles, 3 stages (2 on long sequences)
//   warp 10    tcgen05 issuer of S = Q K^T (one 128 x 64 product per group); owns TMEM
//   warp 11    tcgen05 issuer of O += P V (one per group)
// Issuing one tcgen05.mma occupies its thread for about as long as a third of the MMA's
// execution, so two issuers keep the tensor pipe fed where one would stall it on every
// wait and commit.
// TMEM (512 columns): S double buffer at [0,128) and [128,256); O_A at [256,384) and
// O_B at [384,512).  Each softmax group keeps its own running max, sum and output
// accumulator (O_A += P_A V[0:64), O_B += P_B V[64:128)) and has its own S product,
// P.V product and barriers, so the groups never synchronise inside the key loop and
// drift out of step: the two warps that share a scheduler (one per group) then take
// turns on the exponential unit instead of contending for it.  The epilogue merges the
// two partial softmaxes.
// P is written back over the group's own S columns as packed bf16 pairs and feeds the
// P.V product straight from TMEM.
//
// A query tile is two 64-row halves; each half has its own exact key-block set (with
// 64-row blocks the halves are different query blocks).  Exact work is enumerated in
// 64-key granules over the union of both halves' sets, two granules per 128-key tile;
// softmax group g handles granule slot g, so its visibility is one flag per row half.
// Summary tiles cover 128 summary entries (one per key block); an entry is visible to
// a half when its block is not exact for that half.
#include "common.cuh"
#include "attn_common.cuh"
#include "sm100_ptx.cuh"

// Optional per-event clock trace of one CTA (compile with -DSB_TRACE; off in the product).
#ifdef SB_TRACE
namespace sb {
__device__ long long g_trace[24][4096];
__device__ int g_trace_cta;
}
#define SB_TRACE_POINT(on, ev, j) \
  do { if ((on) && (j) < 4096) ::sb::g_trace[ev][j] = clock64(); } while (0)
#define SB_TRACE_CTA() ((int)blockIdx.x == ::sb::g_trace_cta && blockIdx.y == 0 && blockIdx.z == 0)
// Start and end (%globaltimer, ns) and SM of every CTA of the first 64k.
namespace sb {
__device__ unsigned long long g_cta_time[65536][3];
}
__device__ __forceinline__ unsigned long long sb_globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned sb_smid() {
  unsigned r;
  asm volatile("mov.u32 %0, %smid;" : "=r"(r));
  return r;
}
#define SB_CTA_TIME(slot)                                                                          \
  do {                                                                                             \
    const unsigned cta_ = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);          \
    if (cta_ < 65536u) {                                                                           \
      ::sb::g_cta_time[cta_][slot] = sb_globaltimer();                                             \
      if ((slot) == 0) ::sb::g_cta_time[cta_][2] = sb_smid();                                      \
    }                                                                                              \
  } while (0)
#else
#define SB_TRACE_POINT(on, ev, j) do { } while (0)
#define SB_TRACE_CTA() false
#define SB_CTA_TIME(slot) do { } while (0)
#endif

namespace sb {
namespace {

using namespace sm100;

constexpr int kThreads = 384;
constexpr int kProducerWarp = 8;   // Q and K
constexpr int kProducerVWarp = 9;  // V
constexpr int kMmaWarp = 10;       // S issuer
constexpr int kPvWarp = 11;        // P.V issuer
// Ring depths when they fit; 2 + 2 on long sequences (below).  Measured at config 1 (A/B in
// one session, attention kernel): K 2 + V 3 27.75-27.98 ms, K 3 + V 2 28.15-28.24 ms.
#ifndef SB_K_STAGES
#define SB_K_STAGES 2
#endif
#ifndef SB_V_STAGES
#define SB_V_STAGES 3
#endif
constexpr int kKStages = SB_K_STAGES;
constexpr int kVStages = SB_V_STAGES;
constexpr int kMaxStages = kKStages > kVStages ? kKStages : kVStages;
constexpr uint32_t kSmemLimit = 227 * 1024;
static_assert(kKStages >= 2 && kVStages >= 2, "both rings need two stages for the long-sequence layout");
constexpr int kTileBytes = 128 * 128 * 2;  // one 128 x 128 bf16 operand tile
constexpr int kHalfBytes = 128 * 64 * 2;   // one 64-column half of it
constexpr int kBoxBytes = 64 * 64 * 2;     // one TMA box (64 columns x 64 rows)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColOA = 256;
constexpr uint32_t kColOB = 384;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: lazy O rescale
// Every kPolyEvery-th pair of exponentials on the fast path runs on the FMA pipe (0: none).
// Measured at config 1 (attention kernel): 0 -- all on the MUFU unit -- 30.6-30.9 ms,
// 1 in 16 31.0, 1 in 8 31.8, 1 in 4 33.9, 1 in 2 38.2 ms: the softmax is short of issue
// slots, not of MUFU throughput.
#ifndef SB_POLY_EVERY
#define SB_POLY_EVERY 0
#endif
constexpr int kPolyEvery = SB_POLY_EVERY;

// Bits [a, b) of a 32-bit word, clamped to [0, 32).
__device__ __forceinline__ uint32_t range_bits(int a, int b) {
  a = max(a, 0);
  b = min(b, 32);
  if (a >= b) return 0u;
  const uint32_t upto_b = b == 32 ? 0xffffffffu : ((1u << b) - 1u);
  return upto_b & ~((1u << a) - 1u);
}

struct __align__(8) Control {
  uint64_t bar_q_full;
  uint64_t bar_k_full[kKStages], bar_k_empty[kKStages];
  uint64_t bar_v_full[kVStages], bar_v_empty[kVStages];
  uint64_t bar_s_full[2][2];   // [group][buffer]: the group's S columns have landed
  uint64_t bar_p_full[2][2];   // [group][buffer]: the group's P is in TMEM (one arrival per warp)
  uint64_t bar_pv_done[2][2];  // [group][buffer]: the group's P.V has completed
  uint64_t bar_xsum;       // both groups have published their final max and sum (256)
  uint64_t bar_o_final;    // P.V issuer: every P.V (hence every S) has completed
  uint64_t bar_s_final;    // S issuer: its last MMA has completed (drain before exit)
  uint32_t tmem_base;
  int abort_flag;
  int exact_granules;
  int has_summary;
  float xmax[2][128];  // [group][row] final running max
  float xsum[2][128];  // [group][row] final partial sums
};

struct SmemLayout {
  uint32_t q, k, v;  // byte offsets from the 1024-aligned base (stages are consecutive)
  uint32_t ctrl, ebits, ubits, lm, glist;
  uint32_t total;
  int k_stages, v_stages;
};

// The per-sequence tables (route words, summary log-masses, granule list) grow with T; when
// three V stages no longer fit beside them the ring drops to two.  With 64-key blocks that
// moves the longest accepted sequence from about 330k to about 660k tokens (128-key blocks:
// about 500k to 990k).
__host__ __device__ inline SmemLayout smem_layout_stages(int words_blk, int words_gran, int nb_pad, int k_stages,
                                                         int v_stages) {
  SmemLayout L;
  L.k_stages = k_stages;
  L.v_stages = v_stages;
  L.q = 0;
  L.k = kTileBytes;
  L.v = L.k + k_stages * kTileBytes;
  L.ctrl = L.v + v_stages * kTileBytes;
  L.ebits = L.ctrl + (uint32_t)((sizeof(Control) + 15) / 16 * 16);  // Control is small
  L.ubits = L.ebits + (uint32_t)((2 * words_blk * 4 + 15) / 16 * 16);  // every region 16-byte aligned
  L.lm = L.ubits + (uint32_t)((words_gran * 4 + 15) / 16 * 16);
  L.glist = L.lm + (uint32_t)(nb_pad * 4);  // LM * log2(e) of every key block
  L.total = L.glist + (uint32_t)((words_gran * 32 * 2 + 15) / 16 * 16);  // exact granules in order (uint16)
  return L;
}

__host__ __device__ inline SmemLayout smem_layout(int words_blk, int words_gran, int nb_pad) {
  const SmemLayout L = smem_layout_stages(words_blk, words_gran, nb_pad, kKStages, kVStages);
  return L.total <= kSmemLimit ? L : smem_layout_stages(words_blk, words_gran, nb_pad, 2, 2);
}

// 2^x on the FMA/ALU pipes (offloads the MUFU unit): round-to-nearest range reduction
// x = j + f with f in [-0.5, 0.5], a degree-3 polynomial for 2^f (least-squares fit on
// Chebyshev nodes, max relative error 2.2e-4, below bf16 rounding), and j added to the
// exponent field.  Inputs below -126 give a value below 2^-125 (effectively zero).
[[maybe_unused]] __device__ __forceinline__ float exp2_poly(float x) {
  x = fmaxf(x, -126.f);
  const float shifter = 12582912.f;  // 1.5 * 2^23: rounds x to an integer in the mantissa
  const float t = x + shifter;
  const float j = t - shifter;
  const float f = x - j;
  float p = fmaf(0.05294328f, f, 0.24218228f);
  p = fmaf(p, f, 0.6935803f);
  p = fmaf(p, f, 0.99996096f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

// exp2_poly on a pair, with the float arithmetic in packed fp32x2 instructions.
__device__ __forceinline__ void exp2_poly2(float x0, float x1, float& y0, float& y1) {
  x0 = fmaxf(x0, -126.f);
  x1 = fmaxf(x1, -126.f);
  const uint64_t shifter = f2_pack(12582912.f, 12582912.f);
  const uint64_t neg_shifter = f2_pack(-12582912.f, -12582912.f);
  const uint64_t x = f2_pack(x0, x1);
  const uint64_t t = f2_add(x, shifter);
  const uint64_t j = f2_add(t, neg_shifter);
  const uint64_t f = f2_fma(j, f2_pack(-1.f, -1.f), x);
  uint64_t p = f2_fma(f2_pack(0.05294328f, 0.05294328f), f, f2_pack(0.24218228f, 0.24218228f));
  p = f2_fma(p, f, f2_pack(0.6935803f, 0.6935803f));
  p = f2_fma(p, f, f2_pack(0.99996096f, 0.99996096f));
  float p0, p1, t0, t1;
  f2_unpack(p, p0, p1);
  f2_unpack(t, t0, t1);
  y0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
  y1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
}


__global__ void __launch_bounds__(kThreads, 1)
sparse_attention_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                              const __grid_constant__ CUtensorMap tm_k,
                              const __grid_constant__ CUtensorMap tm_v,
                              const __grid_constant__ CUtensorMap tm_ak,
                              const __grid_constant__ CUtensorMap tm_av, AttnParams p) {
  // The dynamic window starts 1024-byte aligned (the kernel has no static shared
  // memory); the 128-byte swizzle atoms of the operand tiles rely on it.
  extern __shared__ __align__(1024) uint8_t smem[];
  if ((sm100::smem_u32(smem) & 1023u) != 0u) {
    if (threadIdx.x == 0 && p.status) atomicExch(p.status, 900);
    return;
  }
  const int words_blk = p.words;
  const int n64 = ceil_div(p.T, 64);
  const int words_gran = ceil_div(n64, 32);
  const int nb_pad = 128 * ceil_div(p.NB, 128);  // whole summary tiles
  const SmemLayout L = smem_layout(words_blk, words_gran, nb_pad);
  Control& C = *reinterpret_cast<Control*>(smem + L.ctrl);
  float* lm_s = reinterpret_cast<float*>(smem + L.lm);  // [nb_pad]
  uint32_t* ebits = reinterpret_cast<uint32_t*>(smem + L.ebits);  // [2][words_blk]
  uint32_t* ubits = reinterpret_cast<uint32_t*>(smem + L.ubits);  // [words_gran]
  uint16_t* glist = reinterpret_cast<uint16_t*>(smem + L.glist);  // [exact granules]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tid = threadIdx.x;
  // First rows of the tile's two 64-row halves (-1: an empty half).  The dense suffix tiles
  // launch first.
  int hb[2];
  if (p.pairs != nullptr) {
    const int suffix_tiles = ceil_div(p.row_hi - p.query_tokens, 128);
    if ((int)blockIdx.x < suffix_tiles) {
      hb[0] = p.query_tokens + 128 * (suffix_tiles - 1 - (int)blockIdx.x);
      hb[1] = hb[0] + 64;
    } else {
      const int32_t* pr = p.pairs + (((int64_t)blockIdx.z * p.H + blockIdx.y) * p.pair_tiles +
                                     ((int)blockIdx.x - suffix_tiles)) * 2;
      hb[0] = pr[0] >= 0 ? pr[0] * p.block : -1;
      hb[1] = pr[1] >= 0 ? pr[1] * p.block : -1;
    }
  } else {
    hb[0] = 128 * (ceil_div(p.row_hi, 128) - 1 - (int)blockIdx.x);
    hb[1] = hb[0] + 64;
  }
  const int h = blockIdx.y, b = blockIdx.z;
  const int gshift = p.block == 128 ? 1 : 0;
  [[maybe_unused]] const bool trace = SB_TRACE_CTA();
  if (threadIdx.x == 0) SB_CTA_TIME(0);

  // ---------------------------------------------------------------- setup
  if (tid == 0) {
    mbar_init(smem_u32(&C.bar_q_full), 1);
    for (int s = 0; s < L.k_stages; ++s) {
      mbar_init(smem_u32(&C.bar_k_full[s]), 1);
      mbar_init(smem_u32(&C.bar_k_empty[s]), 1);
    }
    for (int s = 0; s < L.v_stages; ++s) {
      mbar_init(smem_u32(&C.bar_v_full[s]), 1);
      mbar_init(smem_u32(&C.bar_v_empty[s]), 1);
    }
    for (int g = 0; g < 2; ++g)
      for (int s = 0; s < 2; ++s) {
        mbar_init(smem_u32(&C.bar_s_full[g][s]), 1);
        mbar_init(smem_u32(&C.bar_p_full[g][s]), 4);
        mbar_init(smem_u32(&C.bar_pv_done[g][s]), 1);
      }
    mbar_init(smem_u32(&C.bar_o_final), 1);
    mbar_init(smem_u32(&C.bar_s_final), 1);
    mbar_init(smem_u32(&C.bar_xsum), 256);
    C.abort_flag = 0;
    C.exact_granules = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(&C.tmem_base), kTmemCols);
    tmem_relinquish();
  }
  if (warp == kProducerWarp && lane == 0) {
    prefetch_tensormap(&tm_q);
    prefetch_tensormap(&tm_k);
    prefetch_tensormap(&tm_v);
    prefetch_tensormap(&tm_ak);
    prefetch_tensormap(&tm_av);
  }
  // LM * log2(e) of every key block: the copies are issued first, so their latency overlaps
  // the route words below.
  {
    const bool any_routed = ((hb[0] >= 0 && hb[0] < p.query_tokens) || (hb[1] >= 0 && hb[1] < p.query_tokens)) &&
                            p.lm != nullptr;  // summaries present
    const int lm_end = any_routed ? p.NB : 0;
    for (int e = tid; e < nb_pad; e += kThreads) {
      if (e < lm_end)
        cp_async4(lm_s + e, p.lm + ((int64_t)b * p.H + h) * p.NB + e);
      else
        lm_s[e] = 0.f;
    }
    cp_async_commit();
  }
  // Exact block sets of the two 64-row halves (block units): the route word, the sink range
  // and the local band as whole-word masks.
  for (int idx = tid; idx < 2 * words_blk; idx += kThreads) {
    const int half = idx / words_blk, w = idx % words_blk;
    const int hrow = hb[half];
    uint32_t bits = 0u;
    if (hrow >= 0 && hrow < p.T) {
      const int lo = 32 * w;
      if (hrow < p.query_tokens) {
        const int qb = hrow / p.block;
        bits = (uint32_t)p.packed[(((int64_t)b * p.QB + qb) * p.H + h) * p.words + w];
        bits |= range_bits(p.sink_first - lo, p.sink_last - lo);
        if (p.local_radius >= 0) bits |= range_bits(qb - p.local_radius - lo, qb + p.local_radius + 1 - lo);
      } else {
        bits = 0xffffffffu;  // dense suffix rows: every key block exact
      }
      bits &= range_bits(0, p.NB - lo);
    }
    ebits[idx] = bits;
  }
  __syncthreads();
  // Exact 64-key granules of either half.  (A whole-word form of this loop, with 128-key
  // blocks spreading each block bit over two granule bits, costs the softmax loop registers:
  // the kernel sits at its 168-register cap.)
  for (int w = tid; w < words_gran; w += kThreads) {
    uint32_t bits = 0u;
    for (int i = 0; i < 32; ++i) {
      const int g = 32 * w + i;
      if (g >= n64) break;
      const int kb = g >> gshift;  // granule -> key block (block is 64 or 128)
      const uint32_t either = ebits[kb >> 5] | ebits[words_blk + (kb >> 5)];
      if ((either >> (kb & 31)) & 1u) bits |= 1u << i;
    }
    ubits[w] = bits;
  }
  cp_async_wait<0>();
  for (int e = tid; e < nb_pad; e += kThreads) lm_s[e] *= kLog2e;  // this thread's own copies
  __syncthreads();
  if (warp == 0) {
    // The exact granules in ascending order (granule ids are below 65536: T <= 2^22).
    int cnt = 0;
    for (int w0 = 0; w0 < words_gran; w0 += 32) {
      const int w = w0 + lane;
      uint32_t bits = w < words_gran ? ubits[w] : 0u;
      const int own = __popc(bits);
      int incl = own;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      int pos = cnt + incl - own;
      while (bits) {
        glist[pos++] = (uint16_t)(32 * w + __ffs(bits) - 1);
        bits &= bits - 1u;
      }
      cnt += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      C.exact_granules = cnt;
      const bool routed0 = hb[0] >= 0 && hb[0] < p.query_tokens && hb[0] < p.T;
      const bool routed1 = hb[1] >= 0 && hb[1] < p.query_tokens && hb[1] < p.T;
      C.has_summary = (routed0 || routed1) && p.lm != nullptr ? 1 : 0;  // no summaries: exact keys only
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const uint32_t tmem = C.tmem_base;
  const int exact_tiles = (C.exact_granules + 1) / 2;
  const int summary_tiles = C.has_summary ? ceil_div(p.NB, 128) : 0;
  const int total_tiles = exact_tiles + summary_tiles;
  volatile int* abort_flag = &C.abort_flag;
  const uint32_t base = smem_u32(smem);
  const uint32_t sQ = base + L.q;
  const uint32_t sK0 = base + L.k;
  const uint32_t sV0 = base + L.v;

  if (warp == kProducerWarp || warp == kProducerVWarp) {
    // ----------------------------------------------------------- producers
    // Warp 8 streams Q and the K side, warp 9 the V side; both walk the same tile list,
    // so a slow P.V never delays the next K tile.  Q streams through L2 once (evict first);
    // K, V and the summaries are read again by every query tile of the head (evict last).
    if (lane == 0) {
      const bool is_k = warp == kProducerWarp;
      const int stages = is_k ? L.k_stages : L.v_stages;
      const CUtensorMap* exact_map = is_k ? &tm_k : &tm_v;
      const CUtensorMap* summ_map = is_k ? &tm_ak : &tm_av;
      const uint32_t s_base = is_k ? sK0 : sV0;
      uint64_t* full = is_k ? C.bar_k_full : C.bar_v_full;
      uint64_t* empty = is_k ? C.bar_k_empty : C.bar_v_empty;
      const uint32_t bq = smem_u32(&C.bar_q_full);
      const uint64_t keep = l2_policy_evict_last();
      if (is_k) {
        const uint64_t once = l2_policy_evict_first();
        mbar_arrive_expect_tx(bq, kTileBytes);
        for (int dh = 0; dh < 2; ++dh)
          for (int rh = 0; rh < 2; ++rh)
            tma_load_3d_hint(sQ + dh * kHalfBytes + rh * kBoxBytes, &tm_q, bq, h * 128 + 64 * dh,
                             hb[rh] >= 0 ? hb[rh] : p.T, b,
                             once);
      }
      const int n_gran = C.exact_granules;
      int armed[kMaxStages] = {};
      int s = 0, use = 0;  // stage and how many times it has been filled before
      for (int j = 0; j < total_tiles; ++j) {
        int g0 = 0, g1 = 0;
        const bool exact = j < exact_tiles;
        if (exact) {
          g0 = glist[2 * j];
          g1 = 2 * j + 1 < n_gran ? (int)glist[2 * j + 1] : g0;  // an odd last granule fills both slots
        }
        const int cc = j - exact_tiles;
        const uint32_t bar = smem_u32(&full[s]);
        if (!mbar_wait(smem_u32(&empty[s]), (uint32_t)((use & 1) ^ 1), abort_flag, p.status, is_k ? 101 : 102)) break;
        mbar_arrive_expect_tx(bar, kTileBytes);
        SB_TRACE_POINT(trace, is_k ? 0 : 1, j);
        ++armed[s];
        const uint32_t st = s_base + s * kTileBytes;
        for (int slot = 0; slot < 2; ++slot) {
          for (int dh = 0; dh < 2; ++dh) {
            const uint32_t dst = st + dh * kHalfBytes + slot * kBoxBytes;
            if (exact)
              tma_load_3d_hint(dst, exact_map, bar, h * 128 + 64 * dh, (slot ? g1 : g0) * 64, b, keep);
            else
              tma_load_3d_hint(dst, summ_map, bar, 64 * dh, cc * 128 + 64 * slot, b * p.H + h, keep);
          }
        }
        if (++s == stages) {
          s = 0;
          ++use;
        }
      }
      // Every armed load must land before the CTA may exit.
      for (int st = 0; st < stages; ++st)
        if (armed[st] > 0) mbar_drain(smem_u32(&full[st]), (uint32_t)((armed[st] - 1) & 1));
      if (is_k) mbar_drain(bq, 0);
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------- S issuer
    // Two S products per tile, one per softmax group (N = 64: the group's granule slot),
    // each with its own barriers, so the groups run out of step: while one group works
    // through its exponentials the other can wait, load and reduce.
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_bf16_f32(128, 64, false);
      bool ok = mbar_wait(smem_u32(&C.bar_q_full), 0, abort_flag, p.status, 201);
      // Descriptors differ only in the start-address field (bits 0-13, in 16-byte units).
      const uint64_t qdesc0 = smem_desc_sw128(sQ, 16, 1024);
      const uint64_t kdesc0 = smem_desc_sw128(sK0, 16, 1024);
      int ks = 0, kuse = 0;
      for (int j = 0; ok && j < total_tiles; ++j) {
        const int s = j & 1;
        if (!mbar_wait(smem_u32(&C.bar_k_full[ks]), (uint32_t)(kuse & 1), abort_flag, p.status, 204)) break;
        SB_TRACE_POINT(trace, 2, j);
        const uint64_t kdesc = kdesc0 + (uint64_t)((ks * kTileBytes) >> 4);
        for (int g = 0; ok && g < 2; ++g) {
          // The group's S columns of buffer s still hold its P of tile j-2 until that P.V
          // completes.  The barrier cannot run two phases ahead: P.V of tile j needs S_j.
          if (j >= 2 && !mbar_wait(smem_u32(&C.bar_pv_done[g][s]), (uint32_t)(((j - 2) >> 1) & 1), abort_flag,
                                   p.status, 205)) {
            ok = false;
            break;
          }
          SB_TRACE_POINT(trace, g ? 18 : 12, j);
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t off = (uint64_t)(((kk >> 2) * kHalfBytes + (kk & 3) * 32) >> 4);
            mma_ss(tmem + s * 128 + 64 * g, qdesc0 + off, kdesc + off + (uint64_t)((g * kBoxBytes) >> 4), idesc_qk,
                   kk > 0 ? 1u : 0u);
          }
          tc_commit(smem_u32(&C.bar_s_full[g][s]));
        }
        if (!ok) break;
        SB_TRACE_POINT(trace, 3, j);
        tc_commit(smem_u32(&C.bar_k_empty[ks]));
        if (++ks == L.k_stages) {
          ks = 0;
          ++kuse;
        }
      }
      tc_commit(smem_u32(&C.bar_s_final));
    }
  } else if (warp == kPvWarp) {
    // ----------------------------------------------------------- P.V issuer
    // O_A += P_A V[0:64), O_B += P_B V[64:128), each as soon as its group's P is in TMEM.
    // Per group, a commit tells the S issuer and the group that the P.V has finished; one
    // commit after both releases the V stage.
    if (lane == 0) {
      constexpr uint32_t idesc_pv = idesc_bf16_f32(128, 128, true);
      const uint64_t vdesc0 = smem_desc_sw128(sV0, kHalfBytes, 1024);
      bool ok = true;
      int vs = 0, vuse = 0;  // V stage and how many times it has been filled before
      for (int i = 0; ok && i < total_tiles; ++i) {
        const int s = i & 1;  // S/P buffer (two in TMEM)
        const uint32_t par = (i >> 1) & 1;
        const uint64_t vdesc = vdesc0 + (uint64_t)((vs * kTileBytes) >> 4);
        if (!mbar_wait(smem_u32(&C.bar_v_full[vs]), (uint32_t)(vuse & 1), abort_flag, p.status, 203)) break;
        SB_TRACE_POINT(trace, 16, i);
        for (int g = 0; g < 2; ++g) {
          if (!mbar_wait(smem_u32(&C.bar_p_full[g][s]), par, abort_flag, p.status, 202)) {
            ok = false;
            break;
          }
          SB_TRACE_POINT(trace, g ? 17 : 4, i);
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_ts(tmem + (g ? kColOB : kColOA), tmem + s * 128 + 64 * g + kk * 8,
                   vdesc + (uint64_t)(((4 * g + kk) * 2048) >> 4), idesc_pv, (i > 0 || kk > 0) ? 1u : 0u);
          tc_commit(smem_u32(&C.bar_pv_done[g][s]));
        }
        if (!ok) break;
        tc_commit(smem_u32(&C.bar_v_empty[vs]));
        SB_TRACE_POINT(trace, 5, i);
        if (++vs == L.v_stages) {
          vs = 0;
          ++vuse;
        }
      }
      tc_commit(smem_u32(&C.bar_o_final));
    }
  } else {
    // --------------------------------------------------------------- softmax
    const int grp = warp >> 2;        // 0: key columns 0-63, 1: key columns 64-127
    const int row = tid & 127;        // TMEM lane = query row of the tile
    const int half = row >> 6;
    const int half_row0 = hb[half];  // -1: this half holds no rows
    const int grow = half_row0 >= 0 ? half_row0 + (row & 63) : -1;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t s_col = 64 * grp;  // this group's S columns inside a buffer
    const uint32_t* ehalf = ebits + half * words_blk;
    const float scale_log2 = 0.08838834764831845f * kLog2e;
    float m_run = -INFINITY, l_run = 0.f;
    // Tile j's exact 64-key granule for this group is glist[2j + grp] (none past the end).
    // Both shared-memory reads behind its visibility (the list entry and the exact-block
    // word of the row half) are issued a tile ahead, so their latency -- long while the
    // tensor pipe streams operands out of shared memory -- hides behind the exponentials.
    const int n_gran = C.exact_granules;
    auto granule = [&](int t) -> int {
      const int i = 2 * t + grp;
      return (t < exact_tiles && i < n_gran) ? (int)glist[i] : -1;
    };
    int g_cur = granule(0);
    uint32_t w_cur = g_cur >= 0 ? ehalf[(g_cur >> gshift) >> 5] : 0u;
    bool ok = true;
    for (int j = 0; j < total_tiles; ++j) {
      SB_TRACE_POINT(trace && row == 0, grp ? 19 : 13, j);
      const int s = j & 1;
      const uint32_t par = (j >> 1) & 1;
      const bool exact = j < exact_tiles;
      // Visibility of this group's 64 keys for this row half.
      bool vis = true, masked = false;
      int key0 = 0;
      if (exact) {
        vis = g_cur >= 0 && ((w_cur >> ((g_cur >> gshift) & 31)) & 1u);
        key0 = g_cur * 64;
        masked = vis && key0 + 64 > p.T;
      }
      const int g_nxt = granule(j + 1);
      SB_TRACE_POINT(trace && tid == 0, 14, j);
      const bool got_s = mbar_wait(smem_u32(&C.bar_s_full[grp][s]), par, abort_flag, p.status, 301);
      if (!__all_sync(0xffffffffu, got_s)) {
        ok = false;
        break;
      }
      SB_TRACE_POINT(trace && row == 0, grp ? 10 : 7, j);
      tc_fence_after();
      uint32_t r[64];
      const bool any_vis = __any_sync(0xffffffffu, vis || !exact);
      if (any_vis) {
        tmem_ld32(tmem + lane_base + s * 128 + s_col, r);
        tmem_ld32(tmem + lane_base + s * 128 + s_col + 32, r + 32);
        tmem_wait_ld();
      }
      SB_TRACE_POINT(trace && tid == 0, 6, j);
      // fast: unmasked exact keys, r holds raw scores; otherwise r is rewritten in place
      // with scaled (and, for summary tiles, LM-biased) logits, -inf where invisible.
      const bool fast = exact && vis && !masked;
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (fast) {
#pragma unroll
        for (int i = 0; i < 64; i += 2)
          mx[(i >> 1) & 3] = max3(mx[(i >> 1) & 3], __uint_as_float(r[i]), __uint_as_float(r[i + 1]));
#pragma unroll
        for (int i = 0; i < 4; ++i) mx[i] *= scale_log2;
      } else if (!exact) {
        // Summary entries e0 .. e0+63 of this group: logit + LM * log2(e), or -inf when the
        // block is exact for this half (or past the last block).
        const int e0 = (j - exact_tiles) * 128 + (int)s_col;
#pragma unroll
        for (int wq = 0; wq < 2; ++wq) {
          const int eb = e0 + 32 * wq;
          const uint32_t ex = eb < p.NB ? ehalf[eb >> 5] : 0xffffffffu;
          const int valid = p.NB - eb;
          const uint32_t live = valid >= 32 ? ~ex : (valid <= 0 ? 0u : (~ex & ((1u << valid) - 1u)));
          const float4* lm4 = reinterpret_cast<const float4*>(lm_s + eb);
#pragma unroll
          for (int i4 = 0; i4 < 8; ++i4) {
            const float4 l4 = lm4[i4];
            const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int i = 4 * i4 + u;
              const float v = ((live >> i) & 1u) ? fmaf(__uint_as_float(r[32 * wq + i]), scale_log2, lv[u]) : -INFINITY;
              r[32 * wq + i] = __float_as_uint(v);
              mx[i & 3] = fmaxf(mx[i & 3], v);
            }
          }
        }
      } else if (vis) {
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const float v = key0 + i < p.T ? __uint_as_float(r[i]) * scale_log2 : -INFINITY;
          r[i] = __float_as_uint(v);
          mx[i & 3] = fmaxf(mx[i & 3], v);
        }
      }
      const float tile_max = fmaxf(max3(mx[0], mx[1], mx[2]), mx[3]);
      SB_TRACE_POINT(trace && row == 0 && grp == 0, 8, j);
      const uint32_t w_nxt = g_nxt >= 0 ? ehalf[(g_nxt >> gshift) >> 5] : 0u;
      // Lazy rescale of this group's O: only when the running max grows by more than the
      // threshold (or becomes finite for the first time).
      const float m_new = fmaxf(m_run, tile_max);
      const bool need = (m_new > m_run + kRescaleThreshold) || (m_run == -INFINITY && m_new != -INFINITY);
      float alpha = 1.f;
      if (need) {
        alpha = m_run == -INFINITY ? 0.f : ex2_approx(m_run - m_new);
        m_run = m_new;
      }
      // The group's P.V of tile j-1 has finished; that barrier cannot be two phases
      // ahead, since the group's P.V of tile j+1 needs its P of tile j+1.
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        const bool got_o = mbar_wait(smem_u32(&C.bar_pv_done[grp][(j - 1) & 1]), (uint32_t)(((j - 1) >> 1) & 1),
                                     abort_flag, p.status, 302);
        if (!__all_sync(0xffffffffu, got_o)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t o[32];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t ta = tmem + lane_base + (grp ? kColOB : kColOA) + 32 * c;
          tmem_ld32(ta, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(ta, o);
        }
        tmem_wait_st();
      }
      l_run *= alpha;
      const float base_m = m_run == -INFINITY ? 0.f : m_run;
      uint32_t pk[32];
      float ps[4] = {0.f, 0.f, 0.f, 0.f};  // partial sums: even pairs in 0-1, odd pairs in 2-3
      if (!exact || vis) {
        // p = 2^(s * scale - m) (fast path) or 2^(logit - m).  Scalar FFMA and FADD, not the
        // packed fp32x2 forms: measured at config 1, 27.6 ms against 28.0 ms with both
        // packed and 29.3-29.9 ms with only one of them packed (same results bit for bit).
        // kPolyEvery > 0 moves a share of the fast path's exponentials to the polynomial
        // on the FMA pipe.
        const float mul = fast ? scale_log2 : 1.f;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float a0 = fmaf(__uint_as_float(r[2 * c]), mul, -base_m);
          const float a1 = fmaf(__uint_as_float(r[2 * c + 1]), mul, -base_m);
          float p0, p1;
          if (kPolyEvery > 0 && fast && (c % (kPolyEvery > 0 ? kPolyEvery : 1)) == kPolyEvery - 1) {
            exp2_poly2(a0, a1, p0, p1);
          } else {
            p0 = ex2_approx(a0);
            p1 = ex2_approx(a1);
          }
          ps[2 * (c & 1)] += p0;
          ps[2 * (c & 1) + 1] += p1;
          pk[c] = cvt_bf16x2(p0, p1);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 32; ++c) pk[c] = 0u;
      }
      l_run += (ps[0] + ps[1]) + (ps[2] + ps[3]);
      SB_TRACE_POINT(trace && row == 0, grp ? 20 : 15, j);
      tmem_st32(tmem + lane_base + s * 128 + s_col, pk);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&C.bar_p_full[grp][s]));
      SB_TRACE_POINT(trace && row == 0, grp ? 11 : 9, j);
      g_cur = g_nxt;
      w_cur = w_nxt;
    }
    // Epilogue: merge the two groups' partial softmaxes (bounded mbarrier exchange);
    // group g writes head-dim columns 64g .. 64g+63 of the output row.
    const bool got_final = ok && mbar_wait(smem_u32(&C.bar_o_final), 0, abort_flag, p.status, 303);
    C.xmax[grp][row] = m_run;
    C.xsum[grp][row] = l_run;
    mbar_arrive(smem_u32(&C.bar_xsum));
    const bool got_sum = got_final && mbar_wait(smem_u32(&C.bar_xsum), 0, abort_flag, p.status, 306);
    if (__all_sync(0xffffffffu, got_sum)) {
      tc_fence_after();
      const float ma = C.xmax[0][row], mb = C.xmax[1][row];
      const float la = C.xsum[0][row], lb = C.xsum[1][row];
      const float m = fmaxf(ma, mb);
      const float fa = ma == -INFINITY ? 0.f : ex2_approx(ma - m);
      const float fb = mb == -INFINITY ? 0.f : ex2_approx(mb - m);
      const float l = la * fa + lb * fb;
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const bool row_ok = grow >= p.row_lo && grow < p.row_hi;
      __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out) + (((int64_t)b * p.T + grow) * p.H + h) * 128 + 64 * grp;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t oa[32], ob[32];
        tmem_ld32(tmem + lane_base + kColOA + 64 * grp + 32 * c, oa);
        tmem_ld32(tmem + lane_base + kColOB + 64 * grp + 32 * c, ob);
        tmem_wait_ld();
        if (row_ok) {
#pragma unroll
          for (int v8 = 0; v8 < 4; ++v8) {
            float f[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
              f[i] = (__uint_as_float(oa[8 * v8 + i]) * fa + __uint_as_float(ob[8 * v8 + i]) * fb) * inv;
            store8(out + 32 * c + 8 * v8, f);
          }
        }
      }
      if (grp == 0 && row_ok && p.lse != nullptr)
        p.lse[((int64_t)b * p.T + grow) * p.H + h] = l > 0.f ? (m + __log2f(l)) * kLn2 : -INFINITY;
    }
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    // The two final commits cover every MMA this CTA issued.
    mbar_drain(smem_u32(&C.bar_o_final), 0);
    mbar_drain(smem_u32(&C.bar_s_final), 0);
    tmem_dealloc(tmem, kTmemCols);
    if (lane == 0) SB_CTA_TIME(1);
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// 3-D bf16 map {inner, rows, outer} with a 64 x 64 box and 128-byte swizzle.
int make_map(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t outer,
             uint64_t row_stride_bytes, uint64_t outer_stride_bytes) {
  EncodeTiledFn encode = get_encode_fn();
  if (encode == nullptr) {
    set_error("sb_sparse_attention: cuTensorMapEncodeTiled is unavailable");
    return SB_ERR_CUDA;
  }
  const cuuint64_t dims[3] = {inner, rows, outer};
  const cuuint64_t strides[2] = {row_stride_bytes, outer_stride_bytes};
  const cuuint32_t box[3] = {64, 64, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("sb_sparse_attention: cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
    return SB_ERR_CUDA;
  }
  return SB_OK;
}

}  // namespace

int launch_sparse_attention_sm100(const AttnParams& p, cudaStream_t s) {
  const uint64_t HD = (uint64_t)p.H * 128;
  CUtensorMap mq, mk, mv, mak, mav;
  int rc;
  if ((rc = make_map(&mq, p.q, HD, p.T, p.B, HD * 2, HD * 2 * p.T)) != SB_OK) return rc;
  if ((rc = make_map(&mk, p.k, HD, p.T, p.B, HD * 2, HD * 2 * p.T)) != SB_OK) return rc;
  if ((rc = make_map(&mv, p.v, HD, p.T, p.B, HD * 2, HD * 2 * p.T)) != SB_OK) return rc;
  if (p.ak != nullptr) {
    if ((rc = make_map(&mak, p.ak, 128, p.NB, (uint64_t)p.B * p.H, 256, 256ull * p.NB)) != SB_OK) return rc;
    if ((rc = make_map(&mav, p.av, 128, p.NB, (uint64_t)p.B * p.H, 256, 256ull * p.NB)) != SB_OK) return rc;
  } else {
    mak = mk;
    mav = mv;
  }
  const int n64 = ceil_div(p.T, 64);
  const SmemLayout L = smem_layout(p.words, ceil_div(n64, 32), 128 * ceil_div(p.NB, 128));
  const size_t smem = L.total;
  if (smem > kSmemLimit) {
    set_error("sb_sparse_attention: sequence too long for the tensor-core kernel (%zu bytes of shared memory)", smem);
    return SB_ERR_UNSUPPORTED;
  }
  cudaError_t err = cudaFuncSetAttribute(sparse_attention_sm100_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
  if (err != cudaSuccess) return cuda_error(err, "sb_sparse_attention: set smem");
  const int tiles = p.pairs != nullptr ? p.pair_tiles + ceil_div(p.row_hi - p.query_tokens, 128)
                                       : ceil_div(p.row_hi, 128) - p.row_lo / 128;
  dim3 grid(tiles, p.H, p.B);
  sparse_attention_sm100_kernel<<<grid, kThreads, smem, s>>>(mq, mk, mv, mak, mav, p);
  SB_CHECK_LAUNCH("sb_sparse_attention: sm100 launch");
  return SB_OK;
}

}  // namespace sb

#ifdef SB_TRACE
extern "C" int sb_trace_setup(int cta) { return (int)cudaMemcpyToSymbol(sb::g_trace_cta, &cta, sizeof(int)); }
extern "C" int sb_trace_dump(long long* host) {
  return (int)cudaMemcpyFromSymbol(host, sb::g_trace, sizeof(long long) * 24 * 4096);
}
extern "C" int sb_cta_time_dump(unsigned long long* host) {
  return (int)cudaMemcpyFromSymbol(host, sb::g_cta_time, sizeof(unsigned long long) * 65536 * 3);
}
#endif
