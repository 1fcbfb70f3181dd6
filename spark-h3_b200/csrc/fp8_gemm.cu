// e4m3 linears on sm_100a: row / tensor quantisers and a persistent tcgen05 GEMM
//   Y[m, n] = (sum_k A[m, k] * B[n, k]) * a_scale[m] * b_scale[n]  (+ bias[n]) -> bf16
// with fp32 accumulation in TMEM (kind::f8f6f4, K = 32 per MMA).
//
// The GEMM runs on CTA pairs (clusters of two) with tcgen05.mma.cta_group::2: 256 x 256
// output tiles, 256-byte K stages through a 3-stage ring (64 KB per CTA per stage), two
// TMEM accumulators per CTA so the epilogue of one tile overlaps the main loop of the next.
// Roles per CTA (192 threads): warps 0-3 epilogue (thread r owns accumulator row r), warp 4
// TMA producer, warp 5 MMA issuer (rank 0 only) and TMEM owner.
#include <algorithm>

#include "common.cuh"
#include "sm100_ptx.cuh"

namespace sb {
namespace {

using namespace sm100;

constexpr int kBK = 128;          // TMA box inner extent: one 128-byte swizzle span of K
constexpr int kGemmThreads = 192;  // warps 0-3 epilogue, 4 TMA producer, 5 MMA issuer
constexpr int kGroupM = 16;        // tiles are visited in groups of 16 row-tiles, rows fastest

// Instruction descriptor for kind::f8f6f4 with e4m3 A and B, fp32 accumulation, K-major.
__host__ __device__ constexpr uint32_t idesc_e4m3_f32(int M, int N) {
  return (1u << 4)                     // D format: f32
         | (0u << 7) | (0u << 10)      // A, B format: e4m3
         | ((uint32_t)(N >> 3) << 17)  // K-major A and B
         | ((uint32_t)(M >> 4) << 24);
}

struct GemmParams {
  const float* a_scale;
  const float* b_scale;
  int a_scale_stride, b_scale_stride;  // 1: one scale per row / column, 0: one per tensor
  const __nv_bfloat16* bias;
  const __nv_bfloat16* residual;  // optional: out = residual + gate[n] * (scaled product + bias)
  const float* gate;              // [N], required with residual
  __nv_bfloat16* out;
  int tma_out;  // 1: the plain / residual output is written by TMA stores (tm_out); 0: row stores
  int* status;
  int64_t M;
  int N, K;
  int m_tiles, n_tiles, k_steps;
  // Attention-input producer (the fused QKV projection), active when qkv_out[0] is set:
  // columns [0, H*128) are the q heads, then the k heads, then the v heads.  q and k get a
  // per-head RMSNorm (weights norm_w[0] / norm_w[1], eps) of the bf16-rounded projection and
  // the rotary embedding (pair j rotates by rope[j * rope_stride + coords[m, rope_axis[j]]],
  // stored as (cos, sin)); v is stored as projected.  Head h of row m goes to
  // qkv_out[section] + ((h / hp * M + m) * hp + h % hp) * 128, hp = heads / shards: the send
  // layout of the sequence-to-head all-to-all.
  __nv_bfloat16* qkv_out[3];
  // With qkv_peers ([3][shards] device pointers, one receive buffer per section and rank),
  // head h of row m goes to qkv_peers[section][h / hp] + ((peer_rank * M + m) * hp + h % hp)
  // * 128 instead: the all-to-all itself, done by the epilogue's stores over NVLink.
  __nv_bfloat16* const* qkv_peers;
  int peer_rank;
  const float* norm_w[2];
  const float2* rope;
  const int32_t* coords;
  const int8_t* rope_axis;
  int rope_stride, heads, shards;
  float eps;
};

// Projection of 32 accumulator columns to bf16-representable fp32 values (scales, bias).
__device__ __forceinline__ void project_chunk(const uint32_t (&r)[32], float sa, float sb_l, float bias_l, float (&f)[32]) {
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float y = __uint_as_float(r[i]) * sa * __shfl_sync(0xffffffffu, sb_l, i);
    f[i] = __bfloat162float(__float2bfloat16_rn(y + __shfl_sync(0xffffffffu, bias_l, i)));
  }
}

// ------------------------------------------------------------------ CTA-pair GEMM
// A cluster of two CTAs computes a 256 x 256 tile with tcgen05.mma.cta_group::2: CTA rank r
// holds A rows [128r, 128r + 128) and B rows [128r, 128r + 128) of the tile in its own shared
// memory, the pair's MMA (issued by rank 0) reads both halves, and each CTA's TMEM receives
// its 128 rows x 256 columns of the accumulator.  Per SM this halves the operand bytes that
// shared memory serves per MMA, which bounds the single-CTA 128 x 256 tile.
//   full[s]      rank 0 only: armed by rank 0 for both CTAs' bytes; both CTAs' TMA loads
//                complete on it (cta_group::2 loads with rank 0's barrier address)
//   empty[s]     both CTAs: the MMA's commit to each CTA releases the stage
//   acc_full[b]  both CTAs: the MMA's commit after the last K step of a tile
//   acc_empty[b] rank 0 only: one arrival per epilogue warp of both CTAs (8)
//   mma_done     both CTAs: final commit, waited before TMEM is freed
constexpr int kPairStages = 3;
constexpr int kPairBK = 256;                          // K bytes per stage: two 128-byte swizzle spans
constexpr int kPairSpanBytes = 128 * 128;             // 16 KB: 128 rows x 128 K bytes
constexpr int kPairOpBytes = 2 * kPairSpanBytes;      // one operand's rows of a stage (32 KB)
constexpr int kPairStageBytes = 2 * kPairOpBytes;     // A half + B half per CTA (64 KB)
constexpr uint32_t kPairAccCols = 256;
constexpr int kPairOutBox = 32 * 64 * 2;         // one epilogue warp's 32 rows x 64 columns (4 KB)
constexpr int kPairOutBytes = 4 * 2 * kPairOutBox;  // four epilogue warps, two staging buffers each

struct __align__(8) PairControl {
  uint64_t full[kPairStages], empty[kPairStages];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar_cluster, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}
__device__ __forceinline__ void mma_f8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u)
      : "memory");
}
__device__ __forceinline__ void tc_commit_pair(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
               : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t holder_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(holder_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Grouped raster: groups of kGroupM row-tiles; inside a group rows move fastest, so the
// pairs running at one time share a few B panels and a few A panels (both stay in L2).
__device__ __forceinline__ void tile_coords(int64_t t, int m_tiles, int n_tiles, int& mt, int& nt) {
  const int64_t per_group = (int64_t)kGroupM * n_tiles;
  const int group = (int)(t / per_group);
  const int first_m = group * kGroupM;
  const int gm = min(kGroupM, m_tiles - first_m);
  const int within = (int)(t - (int64_t)group * per_group);
  mt = first_m + within % gm;
  nt = within / gm;
}

__global__ void __launch_bounds__(kGemmThreads, 1)
fp8_gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                     const __grid_constant__ CUtensorMap tm_out, GemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  // Same layout in both CTAs, so both take the same branch here.
  const bool aligned = (smem_u32(smem) & 1023u) == 0u;
  uint8_t* sOut = smem + kPairStages * kPairStageBytes;  // output staging of the TMA-store epilogue
  PairControl& C = *reinterpret_cast<PairControl*>(sOut + kPairOutBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  if (aligned && threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(smem_u32(&C.full[s]), 1);
      mbar_init(smem_u32(&C.empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&C.acc_full[b]), 1);
      mbar_init(smem_u32(&C.acc_empty[b]), 8);
    }
    mbar_init(smem_u32(&C.mma_done), 1);
    C.abort_flag = 0;
    fence_barrier_init();
  }
  cluster_sync_all();  // every barrier of the pair exists before either CTA signals one
  if (!aligned) {
    if (threadIdx.x == 0 && p.status) atomicExch(p.status, 911);
    return;
  }
  if (warp == 5) {
    tmem_alloc_pair(smem_u32(&C.tmem_base), 2 * kPairAccCols);
    tmem_relinquish_pair();
  }
  if (warp == 4 && lane == 0) {
    prefetch_tensormap(&tm_a);
    prefetch_tensormap(&tm_b);
    if (p.tma_out) prefetch_tensormap(&tm_out);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = C.tmem_base;
  volatile int* abort_flag = &C.abort_flag;
  const uint32_t base = smem_u32(smem);
  const int64_t pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
  const int64_t total_tiles = (int64_t)p.m_tiles * p.n_tiles;  // 256 x 256 tiles

  if (warp == 4) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      int s = 0, use = 0;
      int armed[kPairStages] = {};
      bool ok = true;
      for (int64_t t = pair; ok && t < total_tiles; t += pairs) {
        int mt, nt;
        tile_coords(t, p.m_tiles, p.n_tiles, mt, nt);
        for (int ks = 0; ks < p.k_steps; ++ks) {
          if (!mbar_wait(smem_u32(&C.empty[s]), (uint32_t)((use & 1) ^ 1), abort_flag, p.status, 421)) {
            ok = false;
            break;
          }
          const uint32_t full_leader = mapa_shared(smem_u32(&C.full[s]), 0);
          if (leader) mbar_arrive_expect_tx(smem_u32(&C.full[s]), 2 * kPairStageBytes);
          ++armed[s];
          const uint32_t st = base + s * kPairStageBytes;
#pragma unroll
          for (int kh = 0; kh < 2; ++kh) {
            tma_load_2d_pair(st + kh * kPairSpanBytes, &tm_a, full_leader, ks * kPairBK + kh * 128,
                             mt * 256 + (int)rank * 128);
            tma_load_2d_pair(st + kPairOpBytes + kh * kPairSpanBytes, &tm_b, full_leader, ks * kPairBK + kh * 128,
                             nt * 256 + (int)rank * 128);
          }
          if (++s == kPairStages) {
            s = 0;
            ++use;
          }
        }
      }
      // rank 0's full barriers complete only once both CTAs' bytes have landed
      if (leader)
        for (int st = 0; st < kPairStages; ++st)
          if (armed[st] > 0) mbar_drain(smem_u32(&C.full[st]), (uint32_t)((armed[st] - 1) & 1));
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer (rank 0)
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = idesc_e4m3_f32(256, 256);
      const uint64_t adesc0 = smem_desc_sw128(base, 16, 1024);
      int s = 0, use = 0, local = 0;
      bool ok = true;
      for (int64_t t = pair; ok && t < total_tiles; t += pairs, ++local) {
        const int buf = local & 1;
        if (local >= 2 && !mbar_wait(smem_u32(&C.acc_empty[buf]), (uint32_t)(((local - 2) >> 1) & 1), abort_flag,
                                     p.status, 422)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + buf * kPairAccCols;
        for (int ks = 0; ks < p.k_steps; ++ks) {
          if (!mbar_wait(smem_u32(&C.full[s]), (uint32_t)(use & 1), abort_flag, p.status, 423)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t sa = adesc0 + (uint64_t)((s * kPairStageBytes) >> 4);
          const uint64_t sb = sa + (uint64_t)(kPairOpBytes >> 4);
#pragma unroll
          for (int kk = 0; kk < kPairBK / 32; ++kk) {
            const uint64_t off = (uint64_t)(((kk >> 2) * kPairSpanBytes + (kk & 3) * 32) >> 4);
            mma_f8_pair(acc, sa + off, sb + off, idesc, (ks > 0 || kk > 0) ? 1u : 0u);
          }
          const uint32_t e = smem_u32(&C.empty[s]);
          tc_commit_pair(mapa_shared(e, 0));
          tc_commit_pair(mapa_shared(e, 1));
          if (++s == kPairStages) {
            s = 0;
            ++use;
          }
        }
        if (!ok) break;
        const uint32_t f = smem_u32(&C.acc_full[buf]);
        tc_commit_pair(mapa_shared(f, 0));
        tc_commit_pair(mapa_shared(f, 1));
      }
      const uint32_t d = smem_u32(&C.mma_done);  // covers every MMA of the pair
      tc_commit_pair(mapa_shared(d, 0));
      tc_commit_pair(mapa_shared(d, 1));
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int row = threadIdx.x;  // TMEM lane of this CTA: tile row 128 * rank + row
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    // TMA-store epilogue: warp w stages its 32 rows of each 64-column group in a 128-byte-
    // swizzled box (16-byte chunk c of row r at c ^ (r & 7)) and stores it with one TMA store;
    // two buffers alternate, a buffer being reused once its store has read it.
    const uint32_t out_stage = smem_u32(sOut) + (uint32_t)(warp * 2 * kPairOutBox);
    uint32_t groups_stored = 0;
    int local = 0;
    for (int64_t t = pair; t < total_tiles; t += pairs, ++local) {
      const int buf = local & 1;
      const bool got = mbar_wait(smem_u32(&C.acc_full[buf]), (uint32_t)((local >> 1) & 1), abort_flag, p.status, 424);
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      int mt, nt;
        tile_coords(t, p.m_tiles, p.n_tiles, mt, nt);
      const int64_t m = (int64_t)mt * 256 + rank * 128 + row;
      const int n0 = nt * 256;
      const bool row_ok = m < p.M;
      const float sa = row_ok ? __ldg(p.a_scale + m * p.a_scale_stride) : 0.f;
      __nv_bfloat16* out_row = p.out + m * p.N;
      if (p.heads > 0) {
        // ------------------------------------------------ attention-input producer
        const int HD = p.heads * 128;
        const int section = n0 / HD;  // a 256-column tile never straddles q / k / v
        const int hp = p.heads / p.shards;
#pragma unroll 1
        for (int hh = 0; hh < 2; ++hh) {
          const int h = (n0 - section * HD) / 128 + hh;
          __nv_bfloat16* dst =
              p.qkv_peers != nullptr
                  ? p.qkv_peers[section * p.shards + h / hp] + (((int64_t)p.peer_rank * p.M + m) * hp + h % hp) * 128
                  : p.qkv_out[section] + (((int64_t)(h / hp) * p.M + m) * hp + h % hp) * 128;
          const uint32_t col0 = buf * kPairAccCols + 128 * hh;
          float rstd = 1.f;
          if (section < 2) {
            float ss = 0.f;
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
              uint32_t r[32];
              tmem_ld32(tmem + lane_base + col0 + 32 * c, r);
              const int nl = n0 + 128 * hh + 32 * c + lane;
              const float sb_l = __ldg(p.b_scale + (int64_t)nl * p.b_scale_stride);
              const float bias_l = p.bias != nullptr ? __bfloat162float(p.bias[nl]) : 0.f;
              tmem_wait_ld();
              float f[32];
              project_chunk(r, sa, sb_l, bias_l, f);
#pragma unroll
              for (int i = 0; i < 32; ++i) ss = fmaf(f[i], f[i], ss);
            }
            rstd = rsqrtf(ss / 128.f + p.eps);
          }
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t r[32];
            tmem_ld32(tmem + lane_base + col0 + 32 * c, r);
            const int nl = n0 + 128 * hh + 32 * c + lane;
            const float sb_l = __ldg(p.b_scale + (int64_t)nl * p.b_scale_stride);
            const float bias_l = p.bias != nullptr ? __bfloat162float(p.bias[nl]) : 0.f;
            const float w_l = section < 2 ? __ldg(p.norm_w[section] + 32 * c + lane) : 1.f;
            tmem_wait_ld();
            float f[32];
            project_chunk(r, sa, sb_l, bias_l, f);
            if (section < 2) {
#pragma unroll
              for (int i = 0; i < 32; ++i) f[i] = f[i] * rstd * __shfl_sync(0xffffffffu, w_l, i);
              if (row_ok) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  const int j = 16 * c + i;  // rotation pair (32c + 2i, 32c + 2i + 1)
                  const float2 cs = __ldg(p.rope + (int64_t)j * p.rope_stride + p.coords[m * 3 + p.rope_axis[j]]);
                  const float x0 = f[2 * i], x1 = f[2 * i + 1];
                  f[2 * i] = x0 * cs.x - x1 * cs.y;
                  f[2 * i + 1] = x0 * cs.y + x1 * cs.x;
                }
              }
            }
            if (row_ok) {
#pragma unroll
              for (int v = 0; v < 4; ++v) store8(dst + 32 * c + 8 * v, f + 8 * v);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&C.acc_empty[buf]), 0));
        continue;
      }
#pragma unroll 1
      for (int c = 0; c < 256 / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + buf * kPairAccCols + 32 * c, r);
        // this chunk's 32 column scales and biases: one load per lane, broadcast by shuffle
        const int nc = n0 + 32 * c;
        const int nl = nc + lane;
        const float sb_l = nl < p.N ? __ldg(p.b_scale + (int64_t)nl * p.b_scale_stride) : 0.f;
        const float bias_l = (p.bias != nullptr && nl < p.N) ? __bfloat162float(p.bias[nl]) : 0.f;
        const float gate_l = (p.residual != nullptr && nl < p.N) ? __ldg(p.gate + nl) : 0.f;
        tmem_wait_ld();
        float f[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float y = __uint_as_float(r[i]) * sa * __shfl_sync(0xffffffffu, sb_l, i);
          f[i] = y + __shfl_sync(0xffffffffu, bias_l, i);
        }
        if (p.residual != nullptr) {
          float res[32];
          const __nv_bfloat16* res_row = p.residual + m * p.N;
          if (row_ok && nc + 32 <= p.N && (p.N % 8) == 0) {
#pragma unroll
            for (int v = 0; v < 4; ++v) load8(res_row + nc + 8 * v, res + 8 * v);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) res[i] = (row_ok && nc + i < p.N) ? __bfloat162float(res_row[nc + i]) : 0.f;
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) f[i] = fmaf(__shfl_sync(0xffffffffu, gate_l, i), f[i], res[i]);
        }
        if (p.tma_out) {
          const uint32_t stage = out_stage + (groups_stored & 1u) * kPairOutBox;
          if ((c & 1) == 0) {
            if (lane == 0) bulk_wait_group_read<1>();  // the store that last read this buffer
            __syncwarp();
          }
          const uint32_t rowp = stage + (uint32_t)(lane * 128);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int chunk = (c & 1) * 4 + q;
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) w[e] = cvt_bf16x2(f[8 * q + 2 * e], f[8 * q + 2 * e + 1]);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(rowp + (uint32_t)((chunk ^ (lane & 7)) * 16)),
                         "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3])
                         : "memory");
          }
          if (c & 1) {
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {  // rows past M and columns past N are clipped by the store
              tma_store_2d(&tm_out, stage, n0 + 64 * (c >> 1), (int)(mt * 256 + rank * 128 + warp * 32));
              bulk_commit_group();
            }
            ++groups_stored;
          }
          continue;
        }
        if (row_ok && nc < p.N) {
          if (nc + 32 <= p.N && (p.N % 8) == 0) {
            // The output is written once: evict-first keeps the A and B panels in L2.
            const uint64_t once = l2_evict_first_policy();
#pragma unroll
            for (int v = 0; v < 4; ++v) store8_hint(out_row + nc + 8 * v, f + 8 * v, once);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (nc + i < p.N) out_row[nc + i] = __float2bfloat16_rn(f[i]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&C.acc_empty[buf]), 0));
    }
    if (p.qkv_peers != nullptr) __threadfence_system();  // the stores to peer buffers, before exit
    if (p.tma_out) {
      if (lane == 0) bulk_wait_group<0>();  // every output store has landed before the CTA exits
      __syncwarp();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    mbar_drain(smem_u32(&C.mma_done), 0);  // rank 0's MMAs write both CTAs' TMEM
  }
  cluster_sync_all();  // no signal to the peer's shared memory is still in flight
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 2 * kPairAccCols);
  }
}

// Row loaders for the quantisers: 8 consecutive fp32 values of row `row` from column c.
template <typename T>
struct PlainRows {
  const T* x;
  int K;
  __device__ void load(int64_t row, int c, float* v) const {
    const T* xr = x + row * K;
    if (c + 8 <= K && (K % 8) == 0) {  // rows are 16-byte aligned only when K % 8 == 0
      load8(xr + c, v);
    } else {
      for (int i = 0; i < 8; ++i) v[i] = c + i < K ? Elem<T>::to_f(xr[c + i]) : 0.f;
    }
  }
};

// a * silu(gate) of a [M, 2K] projection (value half first, gate half second), evaluated
// in fp32 as a * g * sigmoid(g).
template <typename T>
struct SwigluRows {
  const T* h;
  int K;
  __device__ void load(int64_t row, int c, float* v) const {
    const T* hr = h + row * 2 * K;
    float a[8], g[8];
    if (c + 8 <= K && (K % 8) == 0) {
      load8(hr + c, a);
      load8(hr + K + c, g);
    } else {
      for (int i = 0; i < 8; ++i) {
        a[i] = c + i < K ? Elem<T>::to_f(hr[c + i]) : 0.f;
        g[i] = c + i < K ? Elem<T>::to_f(hr[K + c + i]) : 0.f;
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = a[i] * g[i] * (1.f / (1.f + __expf(-g[i])));
  }
};

// The eager spelling divides a tensor by the Python scalar 448, which torch evaluates as a
// multiplication by the fp32 reciprocal; the scale is taken the same way.
constexpr float kInv448 = 1.0f / 448.0f;

// GELU(x) = x * Phi(x) (erf form) of one [M, K] row.
template <typename T>
struct GeluRows {
  const T* x;
  int K;
  __device__ void load(int64_t row, int c, float* v) const {
    const T* xr = x + row * K;
    if (c + 8 <= K && (K % 8) == 0) {
      load8(xr + c, v);
    } else {
      for (int i = 0; i < 8; ++i) v[i] = c + i < K ? Elem<T>::to_f(xr[c + i]) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.5f * v[i] * (1.f + erff(v[i] * 0.70710678118654752f));
  }
};

// Row m of a matrix stored as `segments` consecutive [M, seg] blocks (seg columns each,
// seg_stride elements apart): the layout an all-to-all returns when every peer sends one
// column block of every row.
template <typename T>
struct SegmentRows {
  const T* x;
  int seg;
  int64_t seg_stride;
  __device__ void load(int64_t row, int c, float* v) const {
    const int s = c / seg, off = c - s * seg;  // seg is a multiple of 8: one segment per vector
    load8(x + s * seg_stride + row * seg + off, v);
  }
};

__device__ __forceinline__ void store_e4m3x8(uint8_t* yr, int c, int K, const float* v, float scale) {
  uint16_t packed[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float lo = fminf(fmaxf(__fdiv_rn(v[2 * i], scale), -448.f), 448.f);
    const float hi = fminf(fmaxf(__fdiv_rn(v[2 * i + 1], scale), -448.f), 448.f);
    uint16_t pr;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(pr) : "f"(hi), "f"(lo));
    packed[i] = pr;
  }
  if (c + 8 <= K && (K % 8) == 0) {
    *reinterpret_cast<uint2*>(yr + c) = *reinterpret_cast<uint2*>(packed);
  } else {
    const uint8_t* bytes = reinterpret_cast<const uint8_t*>(packed);
    for (int i = 0; i < 8 && c + i < K; ++i) yr[c + i] = bytes[i];
  }
}

// One warp per row: absmax, scale = max(absmax * fp32(1/448), 1e-12), y = sat_e4m3(x / scale).  The
// second sweep over the row is served from L1/L2.
template <typename Rows>
__global__ void quantize_rows_kernel(Rows rows, int64_t M, int K, uint8_t* __restrict__ y,
                                     float* __restrict__ scales) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  float amax = 0.f;
  for (int c = lane * 8; c < K; c += 256) {
    float v[8];
    rows.load(row, c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
  }
  amax = warp_max(amax);
  const float scale = fmaxf(amax * kInv448, 1e-12f);
  if (lane == 0) scales[row] = scale;
  uint8_t* yr = y + row * K;
  for (int c = lane * 8; c < K; c += 256) {
    float v[8];
    rows.load(row, c, v);
    store_e4m3x8(yr, c, K, v, scale);
  }
}

// Whole-tensor absmax in one read: per-CTA partial maximum, one atomic per CTA.  Absolute
// values are non-negative, so their bit patterns order like unsigned integers.
template <typename T>
__global__ void absmax_kernel(const T* __restrict__ x, int64_t n, unsigned int* __restrict__ amax_bits) {
  float m = 0.f;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x * 8;
  for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8; i < n; i += stride) {
    float v[8];
    if (i + 8 <= n) {
      load8(x + i, v);
    } else {
      for (int j = 0; j < 8; ++j) v[j] = i + j < n ? Elem<T>::to_f(x[i + j]) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(v[j]));
  }
  m = warp_max(m);
  __shared__ float part[32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float w = threadIdx.x < blockDim.x / 32 ? part[threadIdx.x] : 0.f;
    w = warp_max(w);
    if (threadIdx.x == 0) atomicMax(amax_bits, __float_as_uint(w));
  }
}

// y = sat_e4m3(x / scale) with scale = max(amax / 448, 1e-12) taken from the absmax pass.
template <typename T>
__global__ void cast_scaled_kernel(const T* __restrict__ x, int64_t n, const unsigned int* __restrict__ amax_bits,
                                   uint8_t* __restrict__ y, float* __restrict__ scale_out) {
  const float scale = fmaxf(__uint_as_float(*amax_bits) * kInv448, 1e-12f);
  if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = scale;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x * 8;
  for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8; i < n; i += stride) {
    float v[8];
    if (i + 8 <= n) {
      load8(x + i, v);
    } else {
      for (int j = 0; j < 8; ++j) v[j] = i + j < n ? Elem<T>::to_f(x[i + j]) : 0.f;
    }
    const int64_t rest = n - i;
    store_e4m3x8(y + i, 0, rest < 8 ? (int)rest : 8, v, scale);
  }
}

// a * silu(gate) rounded to bf16 (the per-tensor SwiGLU path quantises this tensor).
template <typename T>
__global__ void swiglu_kernel(const T* __restrict__ h, int64_t M, int K, __nv_bfloat16* __restrict__ act) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  SwigluRows<T> rows{h, K};
  __nv_bfloat16* ar = act + row * K;
  for (int c = lane * 8; c < K; c += 256) {
    float v[8];
    rows.load(row, c, v);
    if (c + 8 <= K && (K % 8) == 0) {
      store8(ar + c, v);
    } else {
      for (int i = 0; i < 8 && c + i < K; ++i) ar[c + i] = __float2bfloat16_rn(v[i]);
    }
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
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

// bf16 output [rows, cols] as a store target: 64-column x 32-row boxes, 128-byte swizzle.
int make_out_map(CUtensorMap* map, void* base, uint64_t cols, uint64_t rows) {
  EncodeTiledFn encode = encode_fn();
  if (encode == nullptr) {
    set_error("sb_fp8_gemm: cuTensorMapEncodeTiled is unavailable");
    return SB_ERR_CUDA;
  }
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {64, 32};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("sb_fp8_gemm: cuTensorMapEncodeTiled (output) failed (CUresult %d)", (int)r);
    return SB_ERR_CUDA;
  }
  return SB_OK;
}

int make_map_u8(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint32_t box_rows) {
  EncodeTiledFn encode = encode_fn();
  if (encode == nullptr) {
    set_error("sb_fp8_gemm: cuTensorMapEncodeTiled is unavailable");
    return SB_ERR_CUDA;
  }
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols};
  const cuuint32_t box[2] = {(cuuint32_t)kBK, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("sb_fp8_gemm: cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
    return SB_ERR_CUDA;
  }
  return SB_OK;
}

}  // namespace
}  // namespace sb

using namespace sb;

namespace {
constexpr int kRowsPerCta = 8;

template <typename Rows>
int launch_rows(Rows rows, int64_t M, int K, uint8_t* out, float* scales, cudaStream_t s, const char* what) {
  const int64_t grid = (M + kRowsPerCta - 1) / kRowsPerCta;
  SB_CHECK_ARG(grid < (1ll << 31), "%s: too many rows", what);
  quantize_rows_kernel<Rows><<<(unsigned)grid, 32 * kRowsPerCta, 0, s>>>(rows, M, K, out, scales);
  SB_CHECK_LAUNCH(what);
  return SB_OK;
}

int elementwise_grid(int64_t n) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (n + 256 * 8 - 1) / (256 * 8);
  return (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)sms * 8));
}
}  // namespace

extern "C" int sb_fp8_quantize_rows(const void* x, int dtype, int64_t M, int K, uint8_t* out, float* scales,
                                    void* stream) {
  SB_CHECK_ARG(x && out && scales, "sb_fp8_quantize_rows: null pointer");
  SB_CHECK_ARG(dtype == SB_F32 || dtype == SB_BF16, "sb_fp8_quantize_rows: bad dtype");
  SB_CHECK_ARG(M > 0 && K > 0, "sb_fp8_quantize_rows: M and K must be positive");
  SB_CHECK_ARG(((uintptr_t)x % 16) == 0 && ((uintptr_t)out % 8) == 0,
               "sb_fp8_quantize_rows: x must be 16-byte and out 8-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == SB_BF16)
    return launch_rows(PlainRows<__nv_bfloat16>{(const __nv_bfloat16*)x, K}, M, K, out, scales, s,
                       "sb_fp8_quantize_rows launch");
  return launch_rows(PlainRows<float>{(const float*)x, K}, M, K, out, scales, s, "sb_fp8_quantize_rows launch");
}

extern "C" int sb_fp8_swiglu_quantize_rows(const void* h, int dtype, int64_t M, int K, uint8_t* out, float* scales,
                                           void* stream) {
  SB_CHECK_ARG(h && out && scales, "sb_fp8_swiglu_quantize_rows: null pointer");
  SB_CHECK_ARG(dtype == SB_F32 || dtype == SB_BF16, "sb_fp8_swiglu_quantize_rows: bad dtype");
  SB_CHECK_ARG(M > 0 && K > 0, "sb_fp8_swiglu_quantize_rows: M and K must be positive");
  SB_CHECK_ARG(((uintptr_t)h % 16) == 0 && ((uintptr_t)out % 8) == 0,
               "sb_fp8_swiglu_quantize_rows: h must be 16-byte and out 8-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == SB_BF16)
    return launch_rows(SwigluRows<__nv_bfloat16>{(const __nv_bfloat16*)h, K}, M, K, out, scales, s,
                       "sb_fp8_swiglu_quantize_rows launch");
  return launch_rows(SwigluRows<float>{(const float*)h, K}, M, K, out, scales, s,
                     "sb_fp8_swiglu_quantize_rows launch");
}

extern "C" int sb_fp8_gelu_quantize_rows(const void* x, int dtype, int64_t M, int K, uint8_t* out, float* scales,
                                         void* stream) {
  SB_CHECK_ARG(x && out && scales, "sb_fp8_gelu_quantize_rows: null pointer");
  SB_CHECK_ARG(dtype == SB_F32 || dtype == SB_BF16, "sb_fp8_gelu_quantize_rows: bad dtype");
  SB_CHECK_ARG(M > 0 && K > 0, "sb_fp8_gelu_quantize_rows: M and K must be positive");
  SB_CHECK_ARG(((uintptr_t)x % 16) == 0 && ((uintptr_t)out % 8) == 0,
               "sb_fp8_gelu_quantize_rows: x must be 16-byte and out 8-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == SB_BF16)
    return launch_rows(GeluRows<__nv_bfloat16>{(const __nv_bfloat16*)x, K}, M, K, out, scales, s,
                       "sb_fp8_gelu_quantize_rows launch");
  return launch_rows(GeluRows<float>{(const float*)x, K}, M, K, out, scales, s, "sb_fp8_gelu_quantize_rows launch");
}

extern "C" int sb_fp8_quantize_segments(const void* x, int64_t M, int K, int seg, int64_t seg_stride, uint8_t* out,
                                        float* scales, void* stream) {
  SB_CHECK_ARG(x && out && scales, "sb_fp8_quantize_segments: null pointer");
  SB_CHECK_ARG(M > 0 && K > 0 && seg > 0 && seg % 8 == 0 && K % seg == 0,
               "sb_fp8_quantize_segments: K must be a whole number of segments of a multiple of 8 columns");
  SB_CHECK_ARG(seg_stride >= M * (int64_t)seg, "sb_fp8_quantize_segments: segments overlap");
  SB_CHECK_ARG(((uintptr_t)x % 16) == 0 && ((uintptr_t)out % 8) == 0,
               "sb_fp8_quantize_segments: x must be 16-byte and out 8-byte aligned");
  return launch_rows(SegmentRows<__nv_bfloat16>{(const __nv_bfloat16*)x, seg, seg_stride}, M, K, out, scales,
                     (cudaStream_t)stream, "sb_fp8_quantize_segments launch");
}

extern "C" int sb_fp8_quantize_tensor(const void* x, int dtype, int64_t n, uint8_t* out, float* scale,
                                      float* workspace, void* stream) {
  SB_CHECK_ARG(x && out && scale && workspace, "sb_fp8_quantize_tensor: null pointer");
  SB_CHECK_ARG(dtype == SB_F32 || dtype == SB_BF16, "sb_fp8_quantize_tensor: bad dtype");
  SB_CHECK_ARG(n > 0, "sb_fp8_quantize_tensor: n must be positive");
  SB_CHECK_ARG(((uintptr_t)x % 16) == 0 && ((uintptr_t)out % 8) == 0,
               "sb_fp8_quantize_tensor: x must be 16-byte and out 8-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  unsigned int* amax = reinterpret_cast<unsigned int*>(workspace);
  cudaError_t err = cudaMemsetAsync(amax, 0, sizeof(unsigned int), s);
  if (err != cudaSuccess) return cuda_error(err, "sb_fp8_quantize_tensor: clear absmax");
  const int grid = elementwise_grid(n);
  if (dtype == SB_BF16) {
    absmax_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>((const __nv_bfloat16*)x, n, amax);
    cast_scaled_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>((const __nv_bfloat16*)x, n, amax, out, scale);
  } else {
    absmax_kernel<float><<<grid, 256, 0, s>>>((const float*)x, n, amax);
    cast_scaled_kernel<float><<<grid, 256, 0, s>>>((const float*)x, n, amax, out, scale);
  }
  SB_CHECK_LAUNCH("sb_fp8_quantize_tensor launch");
  return SB_OK;
}

extern "C" int sb_fp8_swiglu(const void* h, int dtype, int64_t M, int K, void* act, void* stream) {
  SB_CHECK_ARG(h && act, "sb_fp8_swiglu: null pointer");
  SB_CHECK_ARG(dtype == SB_F32 || dtype == SB_BF16, "sb_fp8_swiglu: bad dtype");
  SB_CHECK_ARG(M > 0 && K > 0 && K % 8 == 0, "sb_fp8_swiglu: M > 0 and K a positive multiple of 8");
  SB_CHECK_ARG(((uintptr_t)h % 16) == 0 && ((uintptr_t)act % 16) == 0, "sb_fp8_swiglu: 16-byte aligned rows");
  const int64_t grid = (M + kRowsPerCta - 1) / kRowsPerCta;
  SB_CHECK_ARG(grid < (1ll << 31), "sb_fp8_swiglu: too many rows");
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == SB_BF16)
    swiglu_kernel<__nv_bfloat16><<<(unsigned)grid, 32 * kRowsPerCta, 0, s>>>((const __nv_bfloat16*)h, M, K,
                                                                          (__nv_bfloat16*)act);
  else
    swiglu_kernel<float><<<(unsigned)grid, 32 * kRowsPerCta, 0, s>>>((const float*)h, M, K, (__nv_bfloat16*)act);
  SB_CHECK_LAUNCH("sb_fp8_swiglu launch");
  return SB_OK;
}

namespace {
struct ProducerArgs {
  void* qkv_out[3];
  void* const* peers;  // optional [3][shards] device table of receive buffers
  int rank;
  const float* norm_w[2];
  const float* rope;
  const int32_t* coords;
  const int8_t* axis;
  int rope_stride, heads, shards;
  float eps;
};

int launch_fp8_gemm(const uint8_t* a, const float* a_scale, int a_scale_stride, const uint8_t* b,
                    const float* b_scale, int b_scale_stride, int64_t M, int N, int K, const void* bias,
                    const void* residual, const float* gate, void* out, int num_ctas, void* stream,
                    const ProducerArgs* prod = nullptr) {
  SB_CHECK_ARG(a && a_scale && b && b_scale && out, "sb_fp8_gemm: null pointer");
  SB_CHECK_ARG(residual == nullptr || (gate != nullptr && ((uintptr_t)residual % 16) == 0),
               "sb_fp8_gemm: a residual needs a gate vector and 16-byte alignment");
  SB_CHECK_ARG(M > 0 && N > 0 && K > 0, "sb_fp8_gemm: M, N, K must be positive");
  SB_CHECK_ARG(K % 16 == 0, "sb_fp8_gemm: K must be a multiple of 16 (TMA row pitch), got %d", K);
  SB_CHECK_ARG(((uintptr_t)a % 16) == 0 && ((uintptr_t)b % 16) == 0 && ((uintptr_t)out % 16) == 0,
               "sb_fp8_gemm: A, B and the output must be 16-byte aligned");
  SB_CHECK_ARG(M < (1ll << 31), "sb_fp8_gemm: M must be below 2^31");
  SB_CHECK_ARG((a_scale_stride == 0 || a_scale_stride == 1) && (b_scale_stride == 0 || b_scale_stride == 1),
               "sb_fp8_gemm: scale strides must be 0 (per tensor) or 1 (per row / column)");
  int* status = device_status_ptr();
  if (status == nullptr) return cuda_error(cudaGetLastError(), "sb_fp8_gemm: status word");
  CUtensorMap ma, mb;
  int rc;
  if ((rc = make_map_u8(&ma, a, (uint64_t)K, (uint64_t)M, 128)) != SB_OK) return rc;
  if ((rc = make_map_u8(&mb, b, (uint64_t)K, (uint64_t)N, 128)) != SB_OK) return rc;
  GemmParams p{};
  p.a_scale = a_scale;
  p.b_scale = b_scale;
  p.a_scale_stride = a_scale_stride;
  p.b_scale_stride = b_scale_stride;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.residual = static_cast<const __nv_bfloat16*>(residual);
  p.gate = gate;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.status = status;
  p.M = M;
  p.N = N;
  p.K = K;
  p.m_tiles = (int)((M + 255) / 256);
  p.n_tiles = (N + 255) / 256;
  p.k_steps = (K + kPairBK - 1) / kPairBK;
  if (prod != nullptr) {
    for (int i = 0; i < 3; ++i) p.qkv_out[i] = static_cast<__nv_bfloat16*>(prod->qkv_out[i]);
    p.qkv_peers = reinterpret_cast<__nv_bfloat16* const*>(prod->peers);
    p.peer_rank = prod->rank;
    p.norm_w[0] = prod->norm_w[0];
    p.norm_w[1] = prod->norm_w[1];
    p.rope = reinterpret_cast<const float2*>(prod->rope);
    p.coords = prod->coords;
    p.rope_axis = prod->axis;
    p.rope_stride = prod->rope_stride;
    p.heads = prod->heads;
    p.shards = prod->shards;
    p.eps = prod->eps;
  }
  // Plain and residual outputs with 16-byte rows go out through TMA stores.
  CUtensorMap mo = ma;
  if (prod == nullptr && N % 8 == 0 && ((uintptr_t)out % 16) == 0) {
    if ((rc = make_out_map(&mo, out, (uint64_t)N, (uint64_t)M)) != SB_OK) return rc;
    p.tma_out = 1;
  }
  const size_t smem = (size_t)kPairStages * kPairStageBytes + kPairOutBytes + sizeof(PairControl);
  cudaError_t err = cudaFuncSetAttribute(fp8_gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return cuda_error(err, "sb_fp8_gemm: set smem");
  int ctas = num_ctas;
  if (ctas <= 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&ctas, cudaDevAttrMultiProcessorCount, dev);
  }
  const int64_t tiles = (int64_t)p.m_tiles * p.n_tiles;
  const int pairs = (int)std::max<int64_t>(1, std::min<int64_t>(tiles, ctas / 2));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  err = cudaLaunchKernelEx(&cfg, fp8_gemm_pair_kernel, ma, mb, mo, p);
  if (err != cudaSuccess) return cuda_error(err, "sb_fp8_gemm: cluster launch");
  SB_CHECK_LAUNCH("sb_fp8_gemm launch");
  return SB_OK;
}
}  // namespace

extern "C" int sb_fp8_gemm(const uint8_t* a, const float* a_scale, int a_scale_stride, const uint8_t* b,
                           const float* b_scale, int b_scale_stride, int64_t M, int N, int K, const void* bias,
                           void* out, int num_ctas, void* stream) {
  return launch_fp8_gemm(a, a_scale, a_scale_stride, b, b_scale, b_scale_stride, M, N, K, bias, nullptr, nullptr, out,
                         num_ctas, stream);
}

extern "C" int sb_fp8_gemm_residual(const uint8_t* a, const float* a_scale, int a_scale_stride, const uint8_t* b,
                                    const float* b_scale, int b_scale_stride, int64_t M, int N, int K, const void* bias,
                                    const void* residual, const float* gate, void* out, int num_ctas, void* stream) {
  SB_CHECK_ARG(residual != nullptr, "sb_fp8_gemm_residual: null residual");
  return launch_fp8_gemm(a, a_scale, a_scale_stride, b, b_scale, b_scale_stride, M, N, K, bias, residual, gate, out,
                         num_ctas, stream);
}

extern "C" int sb_fp8_gemm_qkv_rope(const uint8_t* a, const float* a_scale, const uint8_t* b, const float* b_scale,
                                    int64_t M, int heads, int K, const void* bias, const float* norm_q,
                                    const float* norm_k, const float* rope, int rope_stride, const int32_t* coords,
                                    const int8_t* axis, int shards, float eps, void* q, void* k, void* v, int num_ctas,
                                    void* stream) {
  SB_CHECK_ARG(q && k && v && norm_q && norm_k && rope && coords && axis, "sb_fp8_gemm_qkv_rope: null pointer");
  SB_CHECK_ARG(heads > 0 && heads % 2 == 0, "sb_fp8_gemm_qkv_rope: heads must be even (a tile holds two heads)");
  SB_CHECK_ARG(shards > 0 && heads % shards == 0, "sb_fp8_gemm_qkv_rope: heads must split evenly across shards");
  SB_CHECK_ARG(rope_stride > 0, "sb_fp8_gemm_qkv_rope: bad rope table stride");
  SB_CHECK_ARG((((uintptr_t)q | (uintptr_t)k | (uintptr_t)v) % 16) == 0,
               "sb_fp8_gemm_qkv_rope: q, k, v must be 16-byte aligned");
  ProducerArgs prod{};
  prod.qkv_out[0] = q;
  prod.qkv_out[1] = k;
  prod.qkv_out[2] = v;
  prod.norm_w[0] = norm_q;
  prod.norm_w[1] = norm_k;
  prod.rope = rope;
  prod.coords = coords;
  prod.axis = axis;
  prod.rope_stride = rope_stride;
  prod.heads = heads;
  prod.shards = shards;
  prod.eps = eps;
  return launch_fp8_gemm(a, a_scale, 1, b, b_scale, 1, M, 3 * heads * 128, K, bias, nullptr, nullptr, q, num_ctas,
                         stream, &prod);
}

extern "C" int sb_fp8_gemm_qkv_rope_peers(const uint8_t* a, const float* a_scale, const uint8_t* b,
                                          const float* b_scale, int64_t M, int heads, int K, const void* bias,
                                          const float* norm_q, const float* norm_k, const float* rope,
                                          int rope_stride, const int32_t* coords, const int8_t* axis, int shards,
                                          int rank, float eps, void* const* peers, int num_ctas, void* stream) {
  SB_CHECK_ARG(peers && norm_q && norm_k && rope && coords && axis, "sb_fp8_gemm_qkv_rope_peers: null pointer");
  SB_CHECK_ARG(heads > 0 && heads % 2 == 0, "sb_fp8_gemm_qkv_rope_peers: heads must be even");
  SB_CHECK_ARG(shards > 0 && heads % shards == 0 && rank >= 0 && rank < shards,
               "sb_fp8_gemm_qkv_rope_peers: bad shard count or rank");
  SB_CHECK_ARG(rope_stride > 0, "sb_fp8_gemm_qkv_rope_peers: bad rope table stride");
  ProducerArgs prod{};
  prod.peers = peers;
  prod.rank = rank;
  prod.norm_w[0] = norm_q;
  prod.norm_w[1] = norm_k;
  prod.rope = rope;
  prod.coords = coords;
  prod.axis = axis;
  prod.rope_stride = rope_stride;
  prod.heads = heads;
  prod.shards = shards;
  prod.eps = eps;
  // `out` is not written in producer mode; any 16-byte-aligned pointer passes the checks.
  return launch_fp8_gemm(a, a_scale, 1, b, b_scale, 1, M, 3 * heads * 128, K, bias, nullptr, nullptr,
                         const_cast<uint8_t*>(a), num_ctas, stream, &prod);
}
