// Block scores (pooled Q . pooled K) and exact per-row Top-K with the lowest-index
// tie rule, emitting the packed int32 route and ascending block indices.
//
// score = fp32(sequential fused multiply-add over d of qc[d] * kc[d]) * scale_log2.
// The CPU oracle computes the identical chain, so selections agree bit for bit.
#include <algorithm>
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "sm100_ptx.cuh"

namespace sb {

constexpr int kScoreTile = 128;  // query blocks x key blocks per CTA
constexpr int kScoreThreads = 256;
constexpr int kKeyStride = kScoreTile + 4;  // floats per d-row of the key tile (16-byte rows)

// grid (splits, ceil(QB/128), B*H).  A CTA keeps one 128-query-block tile's means in shared
// memory and walks the candidate tiles blockIdx.x, blockIdx.x + splits, ...; the next
// tile's key means are fetched into registers while the current tile is scored.  Thread
// (ty, tx) of a 16 x 16 grid computes 8 x 8 scores: query rows ty + 16 i (i < 8) and key
// columns 2 tx + 32 p + {0, 1} (p < 4), each one fma chain over d in order.  Two chains
// advance per instruction (fma.rn.f32x2 on a pair of key columns: each lane is the same
// single-rounded fma as the scalar form, so the scores are unchanged bit for bit); the query
// means sit in shared memory as (a, a) pairs so both operands load as 64-bit words.
template <typename TK> struct KeyChunk;  // 16 bytes of one key-mean row
template <> struct KeyChunk<__nv_bfloat16> {
  static constexpr int kElems = 8;
  __device__ static void to_f(const uint4& raw, float* out) {
    const __nv_bfloat162* x = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(x[i]);
      out[2 * i] = f.x;
      out[2 * i + 1] = f.y;
    }
  }
};
template <> struct KeyChunk<float> {
  static constexpr int kElems = 4;
  __device__ static void to_f(const uint4& raw, float* out) {
    out[0] = __uint_as_float(raw.x);
    out[1] = __uint_as_float(raw.y);
    out[2] = __uint_as_float(raw.z);
    out[3] = __uint_as_float(raw.w);
  }
};

template <typename TK, int D>
__global__ void __launch_bounds__(kScoreThreads)
block_scores_kernel(const float* __restrict__ qc, const TK* __restrict__ kc, int QB, int NB, int H,
                    int C, float scale_log2, float* __restrict__ scores) {
  constexpr int EL = KeyChunk<TK>::kElems;
  constexpr int CHUNKS = D / EL;                           // 16-byte chunks per key row
  constexpr int PER = kScoreTile * CHUNKS / kScoreThreads;  // chunks a thread fetches per tile
  extern __shared__ __align__(16) float score_smem[];
  float2* sq = reinterpret_cast<float2*>(score_smem);  // [128 rows][D] of (a, a)
  float* sk = score_smem + 2 * kScoreTile * D;         // [D][kKeyStride]
  const int bh = blockIdx.z, b = bh / H, h = bh % H;
  const int q0 = blockIdx.y * kScoreTile;
  const int tid = threadIdx.x;
  for (int idx = tid; idx < kScoreTile * D / 4; idx += kScoreThreads) {
    const int r = idx / (D / 4), d4 = idx % (D / 4);
    const int qi = q0 + r;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    if (qi < QB) a = __ldg(reinterpret_cast<const float4*>(qc + (((int64_t)b * NB + qi) * H + h) * D) + d4);
    float4* dst = reinterpret_cast<float4*>(sq + r * D + 4 * d4);
    dst[0] = make_float4(a.x, a.x, a.y, a.y);
    dst[1] = make_float4(a.z, a.z, a.w, a.w);
  }
  // Key-mean tile c: thread t fetches chunks t, t + 256, ... with the row fastest
  // (row = chunk % 128), so a warp's stores into the [d][row] tile hit 32 different banks.
  uint4 next[PER];
  auto fetch = [&](int c0) {
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int chunk = tid + kScoreThreads * k;
      const int r = chunk % kScoreTile, part = chunk / kScoreTile;
      const int ci = c0 + r;
      next[k] = ci < C ? __ldg(reinterpret_cast<const uint4*>(kc + (((int64_t)b * NB + ci) * H + h) * D) + part)
                       : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  const int tiles = ceil_div(C, kScoreTile);
  const int tx = tid % 16, ty = tid / 16;
  int ct = blockIdx.x;
  if (ct < tiles) fetch(ct * kScoreTile);
  for (; ct < tiles; ct += gridDim.x) {
    const int c0 = ct * kScoreTile;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int chunk = tid + kScoreThreads * k;
      const int r = chunk % kScoreTile, part = chunk / kScoreTile;
      float f[EL];
      KeyChunk<TK>::to_f(next[k], f);
#pragma unroll
      for (int e = 0; e < EL; ++e) sk[(part * EL + e) * kKeyStride + r] = f[e];
    }
    __syncthreads();
    if (ct + (int)gridDim.x < tiles) fetch((ct + gridDim.x) * kScoreTile);
    uint64_t acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0ull;
#pragma unroll 2
    for (int d = 0; d < D; ++d) {
      uint64_t a[8], w[4];
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = *reinterpret_cast<const uint64_t*>(sq + (ty + 16 * i) * D + d);
#pragma unroll
      for (int j = 0; j < 4; ++j) w[j] = *reinterpret_cast<const uint64_t*>(sk + d * kKeyStride + 2 * tx + 32 * j);
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = sm100::f2_fma(a[i], w[j], acc[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int qi = q0 + ty + 16 * i;
      if (qi >= QB) continue;
      float* row = scores + (((int64_t)b * QB + qi) * H + h) * C;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int ci = c0 + 2 * tx + 32 * j;
        float lo, hi;
        sm100::f2_unpack(acc[i][j], lo, hi);
        if (ci + 1 < C && (C & 1) == 0) {
          *reinterpret_cast<float2*>(row + ci) = make_float2(__fmul_rn(lo, scale_log2), __fmul_rn(hi, scale_log2));
        } else {
          if (ci < C) row[ci] = __fmul_rn(lo, scale_log2);
          if (ci + 1 < C) row[ci + 1] = __fmul_rn(hi, scale_log2);
        }
      }
    }
    __syncthreads();  // every thread is done with this key tile before the next overwrites it
  }
}

// Order-preserving map from fp32 to uint32 (larger float -> larger key).
__device__ __forceinline__ uint32_t float_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// One warp per (b, query block, head) row, several rows per CTA, no CTA barriers: the row's
// keys sit in the warp's slice of shared memory; a radix select (8-bit digits) with per-warp
// histograms finds the key of the k-th largest score; then 32 candidates at a time, the
// keys above it and the lowest-index keys equal to it are taken (each ballot is one packed
// route word).  Ties at the cut go to the lowest candidate index.
// The row's scores reach shared memory by cp.async copies issued all at once (a row is read
// with many loads in flight, not one dependent load per lane and step), and the key bits
// that every candidate of the row shares (sign, exponent and leading mantissa bits of
// clustered scores) are known without a pass, so the digits start below them.  Four warps
// per CTA let several CTAs share an SM, so one row's copies overlap another's passes.
//
// k is `topk` for every row, or, with per-head budgets (head_budget.py:7-19), head_topk[h]
// for the row's head h = row % H, clamped to [0, C].  Index rows are `index_width` wide;
// positions past the row's k are written as -1.
constexpr int kTopkWarpMaxRows = 4;
constexpr int kHistCopies = 1;

__global__ void __launch_bounds__(32 * kTopkWarpMaxRows)
topk_rows_warp_kernel(const float* __restrict__ scores, int64_t rows, int C, int topk, int words,
                      const int32_t* __restrict__ head_topk, int H, int index_width,
                      int32_t* __restrict__ packed, int32_t* __restrict__ indices) {
  extern __shared__ uint32_t warp_smem[];  // per warp: hist[kHistCopies][256] then keys[C]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
  if (row >= rows) return;
  int k = topk;
  if (head_topk != nullptr) k = min(max(__ldg(head_topk + row % H), 0), C);
  int32_t* prow = packed + row * words;
  if (k == 0) {  // nothing routed: every candidate is summarised
    for (int w = lane; w < words; w += 32) prow[w] = 0;
    if (indices != nullptr)
      for (int i = lane; i < index_width; i += 32) indices[row * index_width + i] = -1;
    return;
  }
  uint32_t* hist = warp_smem + (size_t)warp * (kHistCopies * 256 + C);
  uint32_t* keys = hist + kHistCopies * 256;
  uint32_t* my_hist = hist + 256 * (lane % kHistCopies);
  const float* src = scores + row * C;
  for (int i = lane; i < C; i += 32)
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((uint32_t)__cvta_generic_to_shared(keys + i)),
                 "l"(src + i)
                 : "memory");
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncwarp();
  uint32_t all_and = 0xffffffffu, all_or = 0u;
  for (int i = lane; i < C; i += 32) {
    const uint32_t kk = float_key(__uint_as_float(keys[i]));
    keys[i] = kk;
    all_and &= kk;
    all_or |= kk;
  }
  all_and = __reduce_and_sync(0xffffffffu, all_and);
  all_or = __reduce_or_sync(0xffffffffu, all_or);
  // Bits above `remaining` are common to every key: they are part of the threshold already.
  int remaining = 32 - __clz(all_and ^ all_or);  // 0 when every key is equal
  uint32_t prefix = remaining == 32 ? 0u : (all_and & (0xffffffffu << remaining));
  uint32_t need = (uint32_t)k;
#pragma unroll 1
  while (remaining > 0) {
    const int width = remaining < 8 ? remaining : 8;
    const int shift = remaining - width;
    const uint32_t mask_hi = remaining == 32 ? 0u : (0xffffffffu << remaining);
    const uint32_t dmask = (1u << width) - 1u;
#pragma unroll
    for (int i = 0; i < kHistCopies * 8; ++i) hist[lane + 32 * i] = 0u;
    __syncwarp();
    for (int i = lane; i < C; i += 32) {
      const uint32_t kk = keys[i];
      if ((kk & mask_hi) == prefix) atomicAdd(&my_hist[(kk >> shift) & dmask], 1u);
    }
    __syncwarp();
    // Lane l owns digits 255 - 8l .. 248 - 8l (descending); an exclusive prefix over lanes of
    // the counts above gives each lane the number of keys in higher digits.
    uint32_t c[8], own = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int dg = 255 - 8 * lane - i;
      c[i] = 0u;
#pragma unroll
      for (int cp = 0; cp < kHistCopies; ++cp) c[i] += hist[256 * cp + dg];
      own += c[i];
    }
    uint32_t incl = own;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    uint32_t above = incl - own;
    int digit = -1;
    uint32_t above_digit = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (digit < 0 && above + c[i] >= need) {
        digit = 255 - 8 * lane - i;
        above_digit = above;
      }
      above += c[i];
    }
    // The selected digit is the first (highest) one where the running count reaches need;
    // digit 0 takes whatever remains.
    const unsigned has = __ballot_sync(0xffffffffu, digit >= 0);
    const int src_lane = has ? __ffs(has) - 1 : 31;
    int sel_digit = __shfl_sync(0xffffffffu, digit, src_lane);
    uint32_t sel_above = __shfl_sync(0xffffffffu, above_digit, src_lane);
    if (!has) {
      sel_digit = 0;
      sel_above = __shfl_sync(0xffffffffu, incl, 31) - __shfl_sync(0xffffffffu, c[7], 31);
    }
    prefix |= (uint32_t)sel_digit << shift;
    need -= sel_above;
    remaining = shift;
    __syncwarp();
  }
  const uint32_t thresh = prefix, take_equal = need;
  uint32_t eq_seen = 0;
  int out_pos = 0;
  for (int w = 0; w < words; ++w) {
    const int i = 32 * w + lane;
    const uint32_t kk = i < C ? keys[i] : 0u;
    const bool eq = i < C && kk == thresh;
    const unsigned eq_mask = __ballot_sync(0xffffffffu, eq);
    const uint32_t eq_before = eq_seen + __popc(eq_mask & ((1u << lane) - 1u));
    const bool sel = i < C && (kk > thresh || (eq && eq_before < take_equal));
    const unsigned sel_mask = __ballot_sync(0xffffffffu, sel);
    if (sel && indices != nullptr) {
      const int pos = out_pos + __popc(sel_mask & ((1u << lane) - 1u));
      if (pos < index_width) indices[row * index_width + pos] = i;
    }
    if (lane == 0) prow[w] = (int32_t)sel_mask;
    eq_seen += __popc(eq_mask);
    out_pos += __popc(sel_mask);
  }
  if (indices != nullptr)
    for (int i = k + lane; i < index_width; i += 32) indices[row * index_width + i] = -1;
}

// ---------------------------------------------------------------- query-block pairing
// With 64-token blocks the attention kernel's 128-row tiles hold two query blocks and do the
// exact key work of the union of their sets.  Pairing each block with the unpaired block of
// the largest route overlap among the next kPairWindow (ties: the nearer one), in block
// order, shrinks that union: on the config-2 route from 1.32 k to 1.24 k at top-k 0.1.
// Blocks left without a partner are paired with each other in order, so every (b, h) has
// exactly ceil(blocks / 2) tiles.  The pairing is a scheduling choice of this library (the
// reference runs one 64-row block per tile); attention outputs are unchanged up to the
// order of the online-softmax accumulation.
constexpr int kPairWindow = 64;

// ov[(b h) a][j] = popcount(route[a] & route[a + 1 + j]), 0 past the last block.  A CTA
// takes kPairRows consecutive blocks of one (b, h): their routes and the window's
// (kPairRows + kPairWindow rows) are staged in shared memory once, then thread (a, jg)
// counts the overlaps of block a with eight candidates.
constexpr int kPairRows = 32;
constexpr int kPairThreads = kPairRows * (kPairWindow / 8);  // 256

__global__ void __launch_bounds__(kPairThreads)
block_pair_overlap_kernel(const int32_t* __restrict__ packed, int QB, int H, int words, int blocks,
                          uint16_t* __restrict__ ov) {
  extern __shared__ uint32_t rows_s[];  // [kPairRows + kPairWindow][words]
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int a0 = blockIdx.x * kPairRows;
  const int nrows = min(kPairRows + kPairWindow, blocks - a0);
  const uint32_t* route = reinterpret_cast<const uint32_t*>(packed);
  for (int i = threadIdx.x; i < nrows * words; i += kPairThreads) {
    const int r = i / words, w = i % words;
    rows_s[i] = __ldg(route + (((int64_t)b * QB + a0 + r) * H + h) * words + w);
  }
  __syncthreads();
  const int al = threadIdx.x / (kPairWindow / 8), jg = threadIdx.x % (kPairWindow / 8);
  const int a = a0 + al;
  if (a >= blocks) return;
  int cnt[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  const uint32_t* ra = rows_s + al * words;
  for (int w = 0; w < words; ++w) {
    const uint32_t x = ra[w];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int r = al + 1 + 8 * jg + k;  // candidate a + 1 + j, j = 8 jg + k, as a staged row
      if (r < nrows) cnt[k] += __popc(x & rows_s[r * words + w]);
    }
  }
  uint16_t* out = ov + ((int64_t)bh * blocks + a) * kPairWindow + 8 * jg;
#pragma unroll
  for (int k = 0; k < 8; ++k) out[k] = (uint16_t)cnt[k];
}

// The greedy pass of one (b, h): one warp walks the blocks in order; an unpaired block takes
// the unpaired candidate of the largest overlap (one warp max over (overlap, nearness)).  The
// paired flags of blocks a .. a + 127 live in two 64-bit registers that every lane holds
// alike (a partner is never more than kPairWindow ahead, so a block beyond that is still
// free).  The overlap rows come through a two-chunk shared-memory ring that cp.async fills a
// chunk ahead.
constexpr int kPairChunk = 32;
constexpr int kPairChunkBytes = kPairChunk * kPairWindow * 2;

__global__ void __launch_bounds__(32)
block_pair_greedy_kernel(const uint16_t* __restrict__ ov, int blocks, int tiles, int32_t* __restrict__ pairs) {
  extern __shared__ __align__(16) uint8_t pair_smem[];
  uint16_t* ring = reinterpret_cast<uint16_t*>(pair_smem);            // [2][kPairChunk][kPairWindow]
  int* singles = reinterpret_cast<int*>(pair_smem + 2 * kPairChunkBytes);  // [blocks]
  const int lane = threadIdx.x;
  const int bh = blockIdx.x;
  const uint16_t* ovb = ov + (int64_t)bh * blocks * kPairWindow;
  const int chunks = ceil_div(blocks, kPairChunk);
  auto load_chunk = [&](int c) {  // one commit group per call, empty past the end
    if (c < chunks) {
      const int rows = min(kPairChunk, blocks - c * kPairChunk);
      const uint16_t* src = ovb + (int64_t)c * kPairChunk * kPairWindow;
      uint16_t* dst = ring + (c & 1) * kPairChunk * kPairWindow;
      for (int o = lane; o < rows * (kPairWindow / 8); o += 32) cp_async16(dst + 8 * o, src + 8 * o);
    }
    cp_async_commit();
  };
  load_chunk(0);
  load_chunk(1);
  int32_t* out = pairs + (int64_t)bh * tiles * 2;
  int n_pairs = 0, n_single = 0;
  uint64_t lo = 0ull, hi = 0ull;  // paired flags of blocks a .. a + 63 and a + 64 .. a + 127
  for (int a = 0; a < blocks; ++a) {
    if ((a & (kPairChunk - 1)) == 0) {
      const int c = a / kPairChunk;
      if (c > 0) {
        __syncwarp();  // chunk c - 1 is read by every lane: its buffer takes chunk c + 1
        load_chunk(c + 1);
      }
      cp_async_wait<1>();  // chunk c has landed (only chunk c + 1 may be in flight)
      __syncwarp();
    }
    if (!(lo & 1ull)) {
      const uint16_t* row = ring + ((a / kPairChunk) & 1) * kPairChunk * kPairWindow +
                            (a & (kPairChunk - 1)) * kPairWindow;
      // lane l looks at candidates a + 1 + l and a + 33 + l (flag bits 1 + l and 33 + l)
      uint32_t best = 0u;  // (overlap + 1) << 8 | (255 - j): larger overlap, then smaller j
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int j = lane + 32 * half, c = a + 1 + j;
        const bool busy = j == 63 ? (hi & 1ull) : ((lo >> (j + 1)) & 1ull);
        if (c < blocks && !busy) {
          const uint32_t key = ((uint32_t)row[j] + 1u) << 8 | (uint32_t)(255 - j);
          best = key > best ? key : best;
        }
      }
      best = __reduce_max_sync(0xffffffffu, best);
      if (best == 0u) {
        if (lane == 0) singles[n_single] = a;
        ++n_single;
      } else {
        const int j = 255 - (int)(best & 255u);
        if (lane == 0) {
          out[2 * n_pairs] = a;
          out[2 * n_pairs + 1] = a + 1 + j;
        }
        ++n_pairs;
        if (j == 63) hi |= 1ull; else lo |= 1ull << (j + 1);
      }
    }
    lo = (lo >> 1) | (hi << 63);  // advance the window by one block
    hi >>= 1;
  }
  cp_async_wait<0>();
  __syncwarp();
  // blocks without a partner in reach: paired with each other in block order
  for (int i = lane; 2 * i < n_single; i += 32) {
    out[2 * (n_pairs + i)] = singles[2 * i];
    out[2 * (n_pairs + i) + 1] = 2 * i + 1 < n_single ? singles[2 * i + 1] : -1;
  }
}

}  // namespace sb

using namespace sb;

// cuda_error with the failing entry point's name in front of the step.
static int cuda_error_at(cudaError_t err, const char* who, const char* what) {
  char buf[160];
  snprintf(buf, sizeof(buf), "%s: %s", who, what);
  return cuda_error(err, buf);
}

template <typename TK, int D>
static size_t score_smem_bytes() {
  return (size_t)(2 * kScoreTile * D + D * kKeyStride) * sizeof(float);
}

// Raises the dynamic shared-memory limit of the score kernel for (TK, D); `who` names the
// entry point in the error text.
template <typename TK, int D>
static int prepare_scores(const char* who) {
  cudaError_t err = cudaFuncSetAttribute(block_scores_kernel<TK, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)score_smem_bytes<TK, D>());
  if (err != cudaSuccess) return cuda_error_at(err, who, "set score smem");
  return SB_OK;
}

template <typename TK, int D>
static int launch_scores(const char* who, dim3 grid, const float* qc, const void* kc, int QB, int NB, int H, int C,
                         float scale_log2, float* scores, cudaStream_t s) {
  block_scores_kernel<TK, D><<<grid, kScoreThreads, score_smem_bytes<TK, D>(), s>>>(qc, (const TK*)kc, QB, NB, H, C,
                                                                                 scale_log2, scores);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return cuda_error_at(err, who, "score launch");
  return SB_OK;
}

// Score grid: one CTA row per (query tile, head), and as many CTAs sharing its candidate
// tiles as bring the launch to about two waves of the device's SMs (one CTA fits an SM).
static dim3 score_grid(int candidates, int query_blocks, int heads) {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      sms = 148;
  }
  const int q_tiles = ceil_div(query_blocks, kScoreTile), c_tiles = ceil_div(candidates, kScoreTile);
  const int64_t rows = (int64_t)q_tiles * heads;
  const int splits = (int)std::max<int64_t>(1, std::min<int64_t>(c_tiles, (2 * sms + rows - 1) / rows));
  return dim3(splits, q_tiles, heads);
}

// Score-kernel dispatch on the key-centroid dtype and the head dim (prepare_scores first).
static int scores_for(const char* who, int kc_dtype, int D, dim3 grid, const float* qc, const void* kc, int QB, int NB,
                      int H, int C, float scale_log2, float* scores, cudaStream_t s) {
  if (kc_dtype == SB_BF16)
    return D == 128 ? launch_scores<__nv_bfloat16, 128>(who, grid, qc, kc, QB, NB, H, C, scale_log2, scores, s)
                    : launch_scores<__nv_bfloat16, 64>(who, grid, qc, kc, QB, NB, H, C, scale_log2, scores, s);
  return D == 128 ? launch_scores<float, 128>(who, grid, qc, kc, QB, NB, H, C, scale_log2, scores, s)
                  : launch_scores<float, 64>(who, grid, qc, kc, QB, NB, H, C, scale_log2, scores, s);
}

static int prepare_scores_for(const char* who, int kc_dtype, int D) {
  if (kc_dtype == SB_BF16) return D == 128 ? prepare_scores<__nv_bfloat16, 128>(who) : prepare_scores<__nv_bfloat16, 64>(who);
  return D == 128 ? prepare_scores<float, 128>(who) : prepare_scores<float, 64>(who);
}

// Top-K of `rows` score rows of C candidates: warps of one row each, as many per CTA as their
// keys (C x 4 B + a 1 KB histogram each) fit in 200 KB of shared memory.
struct TopkLaunch {
  int warps;
  size_t smem;
};

static TopkLaunch topk_shape(int C) {
  const size_t per_warp = (size_t)(kHistCopies * 256 + C) * sizeof(uint32_t);
  const int warps = (int)std::min<size_t>(kTopkWarpMaxRows, std::max<size_t>(1, (200 * 1024) / per_warp));
  return TopkLaunch{warps, per_warp * warps};
}

static int prepare_topk(const char* who, int C) {
  const TopkLaunch t = topk_shape(C);
  if (t.smem > 200 * 1024) {
    set_error("%s: too many candidate blocks (%d)", who, C);
    return SB_ERR_INVALID;
  }
  cudaError_t err = cudaFuncSetAttribute(topk_rows_warp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)t.smem);
  if (err != cudaSuccess) return cuda_error_at(err, who, "set top-k smem");
  return SB_OK;
}

static int launch_topk(const char* who, const float* scores, int64_t rows, int C, int topk, int words,
                       const int32_t* head_topk, int H, int index_width, int32_t* packed, int32_t* indices,
                       cudaStream_t s) {
  const TopkLaunch t = topk_shape(C);
  topk_rows_warp_kernel<<<(unsigned)((rows + t.warps - 1) / t.warps), 32 * t.warps, t.smem, s>>>(
      scores, rows, C, topk, words, head_topk, H, index_width, packed, indices);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return cuda_error_at(err, who, "top-k launch");
  return SB_OK;
}

extern "C" int64_t sb_route_workspace_bytes(int B, int QB, int H, int candidates) {
  if (B <= 0 || QB <= 0 || H <= 0 || candidates <= 0) return 0;
  return (int64_t)B * QB * H * candidates * (int64_t)sizeof(float);
}

// Shared argument checks of the route entry points (`who` names the caller in the message).
static int check_route_args(const char* who, const float* qc, const void* kc, int kc_dtype, int B, int QB, int NB,
                            int H, int D, int candidates) {
  SB_CHECK_ARG(qc && kc, "%s: null pointer", who);
  SB_CHECK_ARG(kc_dtype == SB_F32 || kc_dtype == SB_BF16, "%s: bad key-centroid dtype", who);
  SB_CHECK_ARG(B > 0 && QB > 0 && NB > 0 && H > 0, "%s: sizes must be positive", who);
  SB_CHECK_ARG(QB <= NB, "%s: QB (%d) exceeds NB (%d)", who, QB, NB);
  SB_CHECK_ARG(D == 64 || D == 128, "%s: head dim must be 64 or 128", who);
  SB_CHECK_ARG(candidates >= 1 && candidates <= NB, "%s: candidates must lie in [1, NB], got %d", who, candidates);
  SB_CHECK_ARG(ceil_div(NB, 32) <= 256, "%s: at most 8192 key blocks are supported", who);
  SB_CHECK_ARG((size_t)candidates * sizeof(uint32_t) <= 200 * 1024, "%s: too many candidate blocks (%d)", who,
               candidates);
  SB_CHECK_ARG((int64_t)B * QB * H < (1ll << 31), "%s: too many rows", who);
  return SB_OK;
}

// Scores into `workspace`, then the Top-K of every row (a fixed k, or per-head budgets).
static int route_with_workspace(const char* who, const float* qc, const void* kc, int kc_dtype, int B, int QB, int NB,
                                int H, int D, int candidates, int topk, const int32_t* head_topk, int index_width,
                                float scale_log2, void* workspace, int32_t* packed_route, int32_t* indices,
                                cudaStream_t s) {
  int rc = prepare_scores_for(who, kc_dtype, D);
  if (rc == SB_OK) rc = prepare_topk(who, candidates);
  if (rc != SB_OK) return rc;
  float* scores = (float*)workspace;
  dim3 grid = score_grid(candidates, QB, B * H);
  rc = scores_for(who, kc_dtype, D, grid, qc, kc, QB, NB, H, candidates, scale_log2, scores, s);
  if (rc != SB_OK) return rc;
  return launch_topk(who, scores, (int64_t)B * QB * H, candidates, topk, ceil_div(NB, 32), head_topk, H, index_width,
                     packed_route, indices, s);
}

extern "C" int sb_route_topk(const float* qc, const void* kc, int kc_dtype, int B, int QB, int NB,
                             int H, int D, int candidates, int topk, float scale_log2,
                             void* workspace, int32_t* packed_route, int32_t* indices,
                             void* stream) {
  const char* who = "sb_route_topk";
  int rc = check_route_args(who, qc, kc, kc_dtype, B, QB, NB, H, D, candidates);
  if (rc != SB_OK) return rc;
  SB_CHECK_ARG(workspace && packed_route, "%s: null pointer", who);
  SB_CHECK_ARG(topk >= 1 && topk <= candidates, "%s: topk must lie in [1, candidates], got %d", who, topk);
  return route_with_workspace(who, qc, kc, kc_dtype, B, QB, NB, H, D, candidates, topk, nullptr, topk, scale_log2,
                              workspace, packed_route, indices, (cudaStream_t)stream);
}

extern "C" int sb_route_topk_head_budgets(const float* qc, const void* kc, int kc_dtype, int B, int QB, int NB,
                                          int H, int D, int candidates, const int32_t* head_topk, int index_width,
                                          float scale_log2, void* workspace, int32_t* packed_route,
                                          int32_t* indices, void* stream) {
  const char* who = "sb_route_topk_head_budgets";
  int rc = check_route_args(who, qc, kc, kc_dtype, B, QB, NB, H, D, candidates);
  if (rc != SB_OK) return rc;
  SB_CHECK_ARG(head_topk && workspace && packed_route, "%s: null pointer", who);
  SB_CHECK_ARG(indices == nullptr || (index_width >= 1 && index_width <= candidates),
               "%s: index_width must lie in [1, candidates], got %d", who, index_width);
  return route_with_workspace(who, qc, kc, kc_dtype, B, QB, NB, H, D, candidates, 0, head_topk,
                              indices ? index_width : 0, scale_log2, workspace, packed_route, indices,
                              (cudaStream_t)stream);
}

// ------------------------------------------------------------------------------------------
// Allocation-free variant of sb_route_topk.
//
// Some callers cannot hand this library a device workspace: a host that binds only this C ABI
// through a thin FFI and owns no device allocator, or a serving loop that will not accept the
// implicit device synchronisation cudaMalloc performs.  sb_route_topk_noalloc keeps the block
// scores in the file-scope array below instead, and works through the query blocks in chunks
// whose scores fit it, so any size whose per-query-block scores (H * candidates floats) fit
// the array is accepted.
constexpr int64_t kNoAllocScoreFloats = SB_ROUTE_NOALLOC_SCRATCH_FLOATS;
static __device__ __align__(256) float g_route_noalloc_scratch[kNoAllocScoreFloats];

// Device address of the scratch array on the current device, looked up once per device
// (the symbol name is only a host-side stand-in; a kernel must be given this address).
static float* route_noalloc_scratch(int* status) {
  static std::mutex mu;
  static float* cached[64] = {nullptr};
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) {
    *status = cuda_error(err, "sb_route_topk_noalloc: cudaGetDevice");
    return nullptr;
  }
  if (dev < 0 || dev >= 64) {
    set_error("sb_route_topk_noalloc: device ordinal %d out of range", dev);
    *status = SB_ERR_UNSUPPORTED;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev] == nullptr) {
    void* ptr = nullptr;
    err = cudaGetSymbolAddress(&ptr, g_route_noalloc_scratch);
    if (err != cudaSuccess) {
      *status = cuda_error(err, "sb_route_topk_noalloc: cudaGetSymbolAddress of the scratch array");
      return nullptr;
    }
    cached[dev] = static_cast<float*>(ptr);
  }
  return cached[dev];
}

extern "C" int sb_route_topk_noalloc(const float* qc, const void* kc, int kc_dtype, int B, int QB, int NB, int H,
                                     int D, int candidates, int topk, float scale_log2, int32_t* packed_route,
                                     int32_t* indices, void* stream) {
  const char* who = "sb_route_topk_noalloc";
  int rc = check_route_args(who, qc, kc, kc_dtype, B, QB, NB, H, D, candidates);
  if (rc != SB_OK) return rc;
  SB_CHECK_ARG(packed_route, "%s: null pointer", who);
  SB_CHECK_ARG(topk >= 1 && topk <= candidates, "%s: topk must lie in [1, candidates], got %d", who, topk);
  const int64_t per_block = (int64_t)H * candidates;
  SB_CHECK_ARG(per_block <= kNoAllocScoreFloats,
               "%s: H * candidates = %lld exceeds the %lld-float scratch array "
               "(SB_ROUTE_NOALLOC_SCRATCH_FLOATS); use sb_route_topk with a caller workspace",
               who, (long long)per_block, (long long)kNoAllocScoreFloats);
  int status = SB_OK;
  float* scratch = route_noalloc_scratch(&status);
  if (scratch == nullptr) return status;
  // Kernel attributes are set once, before the chunk loop.
  rc = prepare_scores_for(who, kc_dtype, D);
  if (rc == SB_OK) rc = prepare_topk(who, candidates);
  if (rc != SB_OK) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  const int chunk = (int)std::min<int64_t>(QB, kNoAllocScoreFloats / per_block);
  const int words = ceil_div(NB, 32);
  const size_t kc_elem = kc_dtype == SB_BF16 ? 2 : 4;
  for (int b = 0; b < B; ++b) {
    const char* kc_b = static_cast<const char*>(kc) + (size_t)b * NB * H * D * kc_elem;
    for (int q0 = 0; q0 < QB; q0 += chunk) {
      const int n = std::min(chunk, QB - q0);
      const float* qc_c = qc + ((int64_t)b * NB + q0) * H * D;
      dim3 grid = score_grid(candidates, n, H);
      rc = scores_for(who, kc_dtype, D, grid, qc_c, kc_b, n, NB, H, candidates, scale_log2, scratch, s);
      if (rc != SB_OK) return rc;
      const int64_t row0 = ((int64_t)b * QB + q0) * H;
      rc = launch_topk(who, scratch, (int64_t)n * H, candidates, topk, words, nullptr, H, topk,
                       packed_route + row0 * words, indices ? indices + row0 * topk : nullptr, s);
      if (rc != SB_OK) return rc;
    }
  }
  return SB_OK;
}

extern "C" int64_t sb_route_pair_workspace_bytes(int B, int H, int blocks) {
  if (B <= 0 || H <= 0 || blocks <= 0) return 0;
  return (int64_t)B * H * blocks * kPairWindow * (int64_t)sizeof(uint16_t);
}

extern "C" int sb_route_pair_blocks(const int32_t* packed_route, int B, int QB, int H, int words, int blocks,
                                    void* workspace, int32_t* pairs, void* stream) {
  SB_CHECK_ARG(packed_route && workspace && pairs, "sb_route_pair_blocks: null pointer");
  SB_CHECK_ARG(B > 0 && H > 0 && QB > 0 && blocks >= 1 && blocks <= QB,
               "sb_route_pair_blocks: need B, H > 0 and 1 <= blocks (%d) <= QB (%d)", blocks, QB);
  SB_CHECK_ARG(words >= 1 && words <= 256, "sb_route_pair_blocks: route words must lie in [1, 256], got %d", words);
  SB_CHECK_ARG((int64_t)B * H < 65536 * 32768LL, "sb_route_pair_blocks: too many (batch, head) rows");
  cudaStream_t s = (cudaStream_t)stream;
  uint16_t* ov = static_cast<uint16_t*>(workspace);
  SB_CHECK_ARG(B * H <= 65535, "sb_route_pair_blocks: B * H must be at most 65535");
  const size_t rows_smem = (size_t)(kPairRows + kPairWindow) * words * sizeof(uint32_t);
  cudaError_t err = cudaFuncSetAttribute(block_pair_overlap_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)rows_smem);
  if (err != cudaSuccess) return cuda_error(err, "sb_route_pair_blocks: set smem");
  block_pair_overlap_kernel<<<dim3(ceil_div(blocks, kPairRows), B * H), kPairThreads, rows_smem, s>>>(
      packed_route, QB, H, words, blocks, ov);
  SB_CHECK_LAUNCH("sb_route_pair_blocks: overlap launch");
  const int tiles = ceil_div(blocks, 2);
  const size_t smem = 2 * (size_t)kPairChunkBytes + (size_t)blocks * 4;
  SB_CHECK_ARG(smem <= 200 * 1024, "sb_route_pair_blocks: %d blocks need too much shared memory", blocks);
  err = cudaFuncSetAttribute(block_pair_greedy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return cuda_error(err, "sb_route_pair_blocks: set smem");
  block_pair_greedy_kernel<<<B * H, 32, smem, s>>>(ov, blocks, tiles, pairs);
  SB_CHECK_LAUNCH("sb_route_pair_blocks: greedy launch");
  return SB_OK;
}
