// Sparse attention forward on the 5th-generation tensor cores (sm_100a), bf16, D = 128.
//
// One CTA per (128-row query tile, head, batch).  Roles:
//   warps 0-3  softmax: thread r owns query row r of the tile (TMEM lane r)
//   warp 4     TMA producer: Q once, then K/V tiles of the exact key blocks, then
//              AK/AV summary tiles
//   warp 5     tcgen05 issuer; also owns the TMEM allocation
// TMEM (512 columns): S/P double buffer at columns [0,128) and [128,256), O at [256,384).
// P overwrites the first 64 columns of its S buffer as packed bf16 pairs and feeds the
// P.V product directly from TMEM.
//
// A query tile is two 64-row halves; each half has its own exact key-block set (with
// 64-row blocks the halves are different query blocks).  Exact work is enumerated in
// 64-key granules over the union of both halves' sets, two granules per 128-key tile,
// with per-half visibility masks.  Summary tiles cover 128 summary entries (one per key
// block) each; an entry is visible to a half when its block is not exact for that half.
#include "common.cuh"
#include "attn_common.cuh"
#include "sm100_ptx.cuh"

namespace sb {
namespace {

using namespace sm100;

constexpr int kThreads = 192;
constexpr int kTileBytes = 128 * 128 * 2;  // one 128 x 128 bf16 operand tile
constexpr int kHalfBytes = 128 * 64 * 2;   // one 64-column half of it
constexpr int kBoxBytes = 64 * 64 * 2;     // one TMA box (64 columns x 64 rows)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 256;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: lazy O rescale

struct __align__(8) Control {
  uint64_t bar_q_full;
  uint64_t bar_k_full[2], bar_k_empty[2];
  uint64_t bar_v_full[2], bar_v_empty[2];
  uint64_t bar_s_full[2], bar_p_full[2];
  uint64_t bar_o_done, bar_o_final;
  uint32_t tmem_base;
  int abort_flag;
  int exact_granules;
  int has_summary;
};

// Walks the set bits of the granule bitset in ascending order.
struct GranuleWalker {
  const uint32_t* words;
  int nwords, w;
  uint32_t bits;
  __device__ void init(const uint32_t* u, int n) {
    words = u;
    nwords = n;
    w = 0;
    bits = n > 0 ? u[0] : 0u;
  }
  __device__ int next() {
    while (bits == 0u) {
      if (++w >= nwords) return -1;
      bits = words[w];
    }
    const int g = 32 * w + __ffs(bits) - 1;
    bits &= bits - 1u;
    return g;
  }
};

struct SmemLayout {
  uint32_t q, k0, k1, v0, v1;  // byte offsets from the 1024-aligned base
  uint32_t ctrl, ebits, ubits;
  uint32_t total;
};

__host__ __device__ inline SmemLayout smem_layout(int words_blk, int words_gran) {
  SmemLayout L;
  L.q = 0;
  L.k0 = kTileBytes;
  L.k1 = 2 * kTileBytes;
  L.v0 = 3 * kTileBytes;
  L.v1 = 4 * kTileBytes;
  L.ctrl = 5 * kTileBytes;
  L.ebits = L.ctrl + (uint32_t)((sizeof(Control) + 15) / 16 * 16);
  L.ubits = L.ebits + (uint32_t)(2 * words_blk * 4);
  L.total = L.ubits + (uint32_t)(words_gran * 4);
  return L;
}

__global__ void __launch_bounds__(kThreads, 1)
sparse_attention_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                              const __grid_constant__ CUtensorMap tm_k,
                              const __grid_constant__ CUtensorMap tm_v,
                              const __grid_constant__ CUtensorMap tm_ak,
                              const __grid_constant__ CUtensorMap tm_av, AttnParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // Align the operand region to 1024 bytes (128-byte swizzle atoms).
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int words_blk = p.words;
  const int n64 = ceil_div(p.T, 64);
  const int words_gran = ceil_div(n64, 32);
  const SmemLayout L = smem_layout(words_blk, words_gran);
  Control& C = *reinterpret_cast<Control*>(smem + L.ctrl);
  uint32_t* ebits = reinterpret_cast<uint32_t*>(smem + L.ebits);  // [2][words_blk]
  uint32_t* ubits = reinterpret_cast<uint32_t*>(smem + L.ubits);  // [words_gran]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tid = threadIdx.x;
  const int n_tiles = ceil_div(p.T, 128);
  const int tile = n_tiles - 1 - (int)blockIdx.x;  // the dense suffix tile launches first
  const int h = blockIdx.y, b = blockIdx.z;
  const int row0 = tile * 128;

  // ---------------------------------------------------------------- setup
  if (tid == 0) {
    mbar_init(smem_u32(&C.bar_q_full), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&C.bar_k_full[s]), 1);
      mbar_init(smem_u32(&C.bar_k_empty[s]), 1);
      mbar_init(smem_u32(&C.bar_v_full[s]), 1);
      mbar_init(smem_u32(&C.bar_v_empty[s]), 1);
      mbar_init(smem_u32(&C.bar_s_full[s]), 1);
      mbar_init(smem_u32(&C.bar_p_full[s]), 128);
    }
    mbar_init(smem_u32(&C.bar_o_done), 1);
    mbar_init(smem_u32(&C.bar_o_final), 1);
    C.abort_flag = 0;
    C.exact_granules = 0;
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(&C.tmem_base), kTmemCols);
    tmem_relinquish();
  }
  if (warp == 4 && lane == 0) {
    prefetch_tensormap(&tm_q);
    prefetch_tensormap(&tm_k);
    prefetch_tensormap(&tm_v);
    prefetch_tensormap(&tm_ak);
    prefetch_tensormap(&tm_av);
  }
  // Exact block sets of the two 64-row halves (block units).
  for (int idx = tid; idx < 2 * words_blk; idx += kThreads) {
    const int half = idx / words_blk, w = idx % words_blk;
    const int hrow = row0 + 64 * half;
    uint32_t bits = 0u;
    if (hrow < p.T) {
      const int lo = 32 * w;
      if (hrow < p.query_tokens) {
        const int qb = hrow / p.block;
        bits = (uint32_t)p.packed[(((int64_t)b * p.QB + qb) * p.H + h) * p.words + w];
        for (int i = 0; i < 32; ++i) {
          const int kb = lo + i;
          if (kb >= p.NB) break;
          const bool sink = kb >= p.sink_first && kb < p.sink_last;
          const int dist = qb > kb ? qb - kb : kb - qb;
          const bool local = p.local_radius >= 0 && dist <= p.local_radius;
          if (sink || local) bits |= 1u << i;
        }
      } else {
        bits = 0xffffffffu;  // dense suffix rows: every key block exact
      }
      const int valid = p.NB - lo;
      if (valid < 32) bits &= valid <= 0 ? 0u : ((1u << valid) - 1u);
    }
    ebits[idx] = bits;
  }
  __syncthreads();
  for (int w = tid; w < words_gran; w += kThreads) {
    uint32_t bits = 0u;
    for (int i = 0; i < 32; ++i) {
      const int g = 32 * w + i;
      if (g >= n64) break;
      const int kb = g * 64 / p.block;
      const uint32_t either = ebits[kb >> 5] | ebits[words_blk + (kb >> 5)];
      if ((either >> (kb & 31)) & 1u) bits |= 1u << i;
    }
    ubits[w] = bits;
  }
  __syncthreads();
  if (warp == 0) {
    int cnt = 0;
    for (int w = lane; w < words_gran; w += 32) cnt += __popc(ubits[w]);
    for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    if (lane == 0) {
      C.exact_granules = cnt;
      const bool routed0 = row0 < p.query_tokens && row0 < p.T;
      const bool routed1 = row0 + 64 < p.query_tokens && row0 + 64 < p.T;
      C.has_summary = (routed0 || routed1) ? 1 : 0;
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
  const uint32_t sK[2] = {base + L.k0, base + L.k1};
  const uint32_t sV[2] = {base + L.v0, base + L.v1};

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint32_t bq = smem_u32(&C.bar_q_full);
      mbar_arrive_expect_tx(bq, kTileBytes);
      for (int dh = 0; dh < 2; ++dh)
        for (int rh = 0; rh < 2; ++rh)
          tma_load_3d(sQ + dh * kHalfBytes + rh * kBoxBytes, &tm_q, bq, h * 128 + 64 * dh, row0 + 64 * rh, b);
      GranuleWalker walk;
      walk.init(ubits, words_gran);
      int armed_k[2] = {0, 0}, armed_v[2] = {0, 0};
      for (int j = 0; j < total_tiles; ++j) {
        const int s = j & 1;
        const uint32_t par = ((j >> 1) & 1) ^ 1;
        int g0 = 0, g1 = 0;
        const bool exact = j < exact_tiles;
        if (exact) {
          g0 = walk.next();
          g1 = walk.next();
          if (g1 < 0) g1 = g0;
        }
        const int cc = j - exact_tiles;
        const uint32_t bk = smem_u32(&C.bar_k_full[s]);
        if (!mbar_wait(smem_u32(&C.bar_k_empty[s]), par, abort_flag, p.status, 101)) break;
        mbar_arrive_expect_tx(bk, kTileBytes);
        ++armed_k[s];
        for (int slot = 0; slot < 2; ++slot) {
          for (int dh = 0; dh < 2; ++dh) {
            const uint32_t dst = sK[s] + dh * kHalfBytes + slot * kBoxBytes;
            if (exact)
              tma_load_3d(dst, &tm_k, bk, h * 128 + 64 * dh, (slot ? g1 : g0) * 64, b);
            else
              tma_load_3d(dst, &tm_ak, bk, 64 * dh, cc * 128 + 64 * slot, b * p.H + h);
          }
        }
        const uint32_t bv = smem_u32(&C.bar_v_full[s]);
        if (!mbar_wait(smem_u32(&C.bar_v_empty[s]), par, abort_flag, p.status, 102)) break;
        mbar_arrive_expect_tx(bv, kTileBytes);
        ++armed_v[s];
        for (int slot = 0; slot < 2; ++slot) {
          for (int dh = 0; dh < 2; ++dh) {
            const uint32_t dst = sV[s] + dh * kHalfBytes + slot * kBoxBytes;
            if (exact)
              tma_load_3d(dst, &tm_v, bv, h * 128 + 64 * dh, (slot ? g1 : g0) * 64, b);
            else
              tma_load_3d(dst, &tm_av, bv, 64 * dh, cc * 128 + 64 * slot, b * p.H + h);
          }
        }
      }
      // Every armed load must land before the CTA may exit.
      for (int st = 0; st < 2; ++st) {
        if (armed_k[st] > 0) mbar_drain(smem_u32(&C.bar_k_full[st]), (uint32_t)((armed_k[st] - 1) & 1));
        if (armed_v[st] > 0) mbar_drain(smem_u32(&C.bar_v_full[st]), (uint32_t)((armed_v[st] - 1) & 1));
      }
      mbar_drain(bq, 0);
    }
  } else if (warp == 5) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_bf16_f32(128, 128, false);
      constexpr uint32_t idesc_pv = idesc_bf16_f32(128, 128, true);
      bool ok = mbar_wait(smem_u32(&C.bar_q_full), 0, abort_flag, p.status, 201);
      auto issue_pv = [&](int i) -> bool {
        const int s = i & 1;
        const uint32_t par = (i >> 1) & 1;
        if (!mbar_wait(smem_u32(&C.bar_p_full[s]), par, abort_flag, p.status, 202)) return false;
        if (!mbar_wait(smem_u32(&C.bar_v_full[s]), par, abort_flag, p.status, 203)) return false;
        tc_fence_after();
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t bdesc = smem_desc_sw128(sV[s] + kk * 2048, kHalfBytes, 1024);
          mma_ts(tmem + kColO, tmem + s * 128 + kk * 8, bdesc, idesc_pv, (i > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(smem_u32(&C.bar_v_empty[s]));
        tc_commit(smem_u32(&C.bar_o_done));
        return true;
      };
      for (int j = 0; ok && j < total_tiles; ++j) {
        const int s = j & 1;
        const uint32_t par = (j >> 1) & 1;
        if (!mbar_wait(smem_u32(&C.bar_k_full[s]), par, abort_flag, p.status, 204)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
          const uint64_t adesc = smem_desc_sw128(sQ + off, 16, 1024);
          const uint64_t bdesc = smem_desc_sw128(sK[s] + off, 16, 1024);
          mma_ss(tmem + s * 128, adesc, bdesc, idesc_qk, kk > 0 ? 1u : 0u);
        }
        tc_commit(smem_u32(&C.bar_s_full[s]));
        tc_commit(smem_u32(&C.bar_k_empty[s]));
        if (j >= 1 && !issue_pv(j - 1)) ok = false;
      }
      if (ok && total_tiles > 0) issue_pv(total_tiles - 1);
      tc_commit(smem_u32(&C.bar_o_final));
    }
  } else {
    // --------------------------------------------------------------- softmax
    const int row = tid;  // 0..127, TMEM lane
    const int half = row >> 6;
    const int grow = row0 + row;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const uint32_t* ehalf = ebits + half * words_blk;
    const float scale_log2 = 0.08838834764831845f * kLog2e;
    const float* lm_row = p.lm ? p.lm + ((int64_t)b * p.H + h) * p.NB : nullptr;
    float m_run = -INFINITY, l_run = 0.f;
    GranuleWalker walk;
    walk.init(ubits, words_gran);
    bool ok = true;
    for (int j = 0; j < total_tiles; ++j) {
      const int s = j & 1;
      const uint32_t par = (j >> 1) & 1;
      const bool exact = j < exact_tiles;
      int g0 = 0, g1 = -1;
      if (exact) {
        g0 = walk.next();
        g1 = walk.next();
      }
      const bool got_s = mbar_wait(smem_u32(&C.bar_s_full[s]), par, abort_flag, p.status, 301);
      if (!__all_sync(0xffffffffu, got_s)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float x[128];
      {
        uint32_t r[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tmem + lane_base + s * 128 + 32 * c, r + 32 * c);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 128; ++i) x[i] = __uint_as_float(r[i]);
      }
      float tile_max = -INFINITY;
      if (exact) {
        bool vis[2];
        int key0[2];
        const int gs[2] = {g0, g1};
#pragma unroll
        for (int slot = 0; slot < 2; ++slot) {
          const int g = gs[slot];
          bool v = g >= 0;
          if (v) {
            const int kb = g * 64 / p.block;
            v = (ehalf[kb >> 5] >> (kb & 31)) & 1u;
          }
          vis[slot] = v;
          key0[slot] = g * 64;
        }
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          const int slot = c >> 6;
          const bool visible = vis[slot] && (key0[slot] + (c & 63) < p.T);
          const float val = visible ? x[c] * scale_log2 : -INFINITY;
          x[c] = val;
          tile_max = fmaxf(tile_max, val);
        }
      } else {
        const int e0 = (j - exact_tiles) * 128;
#pragma unroll
        for (int wq = 0; wq < 4; ++wq) {
          const int e_base = e0 + 32 * wq;
          const uint32_t ex = e_base < p.NB ? ehalf[e_base >> 5] : 0xffffffffu;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int c = 32 * wq + i;
            const int ee = e_base + i;
            const bool visible = ee < p.NB && !((ex >> i) & 1u);
            const float bias = visible ? __ldg(lm_row + ee) * kLog2e : 0.f;
            const float val = visible ? fmaf(x[c], scale_log2, bias) : -INFINITY;
            x[c] = val;
            tile_max = fmaxf(tile_max, val);
          }
        }
      }
      // Lazy rescale: only when the running max grows by more than the threshold.
      const float m_new = fmaxf(m_run, tile_max);
      const bool need = (m_new > m_run + kRescaleThreshold) || (m_run == -INFINITY && m_new != -INFINITY);
      float alpha = 1.f;
      if (need) {
        alpha = m_run == -INFINITY ? 0.f : ex2_approx(m_run - m_new);
        m_run = m_new;
      }
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        const bool got_o = mbar_wait(smem_u32(&C.bar_o_done), (uint32_t)((j - 1) & 1), abort_flag, p.status, 302);
        if (!__all_sync(0xffffffffu, got_o)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t r[32];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t ta = tmem + lane_base + kColO + 32 * c;
          tmem_ld32(ta, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          tmem_st32(ta, r);
        }
        tmem_wait_st();
      }
      l_run *= alpha;
      const float base_m = m_run == -INFINITY ? 0.f : m_run;
      float sum = 0.f;
      uint32_t pk[64];
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const float p0 = ex2_approx(x[2 * c] - base_m);
        const float p1 = ex2_approx(x[2 * c + 1] - base_m);
        sum += p0 + p1;
        __nv_bfloat162 pair = __floats2bfloat162_rn(p0, p1);
        pk[c] = *reinterpret_cast<uint32_t*>(&pair);
      }
      l_run += sum;
      tmem_st32(tmem + lane_base + s * 128, pk);
      tmem_st32(tmem + lane_base + s * 128 + 32, pk + 32);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(smem_u32(&C.bar_p_full[s]));
    }
    // Epilogue: O / l -> bf16, and the natural-log LSE.
    const bool got_final = ok && mbar_wait(smem_u32(&C.bar_o_final), 0, abort_flag, p.status, 303);
    if (__all_sync(0xffffffffu, got_final)) {
      tc_fence_after();
      const bool row_ok = grow < p.T;
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out) + (((int64_t)b * p.T + grow) * p.H + h) * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + kColO + 32 * c, r);
        tmem_wait_ld();
        if (row_ok) {
#pragma unroll
          for (int v8 = 0; v8 < 4; ++v8) {
            float f[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) f[i] = __uint_as_float(r[8 * v8 + i]) * inv;
            store8(out + 32 * c + 8 * v8, f);
          }
        }
      }
      if (row_ok && p.lse != nullptr)
        p.lse[((int64_t)b * p.T + grow) * p.H + h] = l_run > 0.f ? (m_run + __log2f(l_run)) * kLn2 : -INFINITY;
    }
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    // The final commit covers every MMA this CTA issued.
    mbar_drain(smem_u32(&C.bar_o_final), 0);
    tmem_dealloc(tmem, kTmemCols);
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
  const SmemLayout L = smem_layout(p.words, ceil_div(n64, 32));
  const size_t smem = L.total + 1024;  // slack for the 1024-byte alignment of the base
  if (smem > 227 * 1024) {
    set_error("sb_sparse_attention: sequence too long for the tensor-core kernel (%zu bytes of shared memory)", smem);
    return SB_ERR_UNSUPPORTED;
  }
  cudaError_t err = cudaFuncSetAttribute(sparse_attention_sm100_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
  if (err != cudaSuccess) return cuda_error(err, "sb_sparse_attention: set smem");
  dim3 grid(ceil_div(p.T, 128), p.H, p.B);
  sparse_attention_sm100_kernel<<<grid, kThreads, smem, s>>>(mq, mk, mv, mak, mav, p);
  SB_CHECK_LAUNCH("sb_sparse_attention: sm100 launch");
  return SB_OK;
}

}  // namespace sb
