// Landmark-tree-v2 reblocking on sm_100a: the per-(batch, head, side) token permutation
// that groups similar tokens into 64-token blocks before Spark routing.
//
//   metric     ridged second moments of N/64 Hilbert-midpoint samples of Q and of K and their
//              Cholesky factors (one CTA per matrix, factorisation in shared memory)
//   transform  features = [K . L_Q ; Q . L_K] in bf16: a persistent tcgen05 GEMM (TMA tiles
//              of 128 tokens x 128 dims, the factor resident in shared memory, two TMEM
//              accumulators so the store of one tile overlaps the MMA of the next)
//   tree       per splitting round: 32 midpoint landmarks and a binary proxy tree per node
//              (one warp per node), cosine split scores per token (bandwidth-bound gather of
//              the token's feature row), exact-capacity routing by (score, token id) with a
//              radix select per internal proxy node, and a stable partition into the children
//              (one CTA per node)
//
// The tree is bit-exact with the CPU restatement: every fp32 reduction follows one canonical
// order.  A 128-vector lives on a warp with lane l holding elements 4l .. 4l+3; a dot product
// is the lane's fma chain over its four elements followed by xor-butterfly sums over offsets
// 16, 8, 4, 2, 1; unit(x) = x / max(sqrt(dot(x, x)), 1e-12) with IEEE division and square
// root; weighted landmark means are fma chains over the 32 landmarks in index order.
#include <algorithm>
#include <cstdio>
#include <vector>

#include "common.cuh"
#include "sm100_ptx.cuh"

namespace sb {
namespace {

using namespace sm100;

constexpr int kDim = 128;
constexpr int kLandmarks = 32;
constexpr int kMaxChildren = 64;
constexpr int kNodeInts = 4 + kMaxChildren;  // start, tokens, children, unused, capacities
constexpr int kPlanHeader = 8;
constexpr int kLevelInts = 8;  // nodes, node table offset, tile table offset, P, score stride
constexpr unsigned kFull = 0xffffffffu;

// ------------------------------------------------------------ canonical arithmetic
__device__ __forceinline__ float butterfly(float p) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) p = __fadd_rn(p, __shfl_xor_sync(kFull, p, o));
  return p;
}

__device__ __forceinline__ float lane_dot4(const float* a, const float* b) {
  float p = __fmul_rn(a[0], b[0]);
  p = __fmaf_rn(a[1], b[1], p);
  p = __fmaf_rn(a[2], b[2], p);
  return __fmaf_rn(a[3], b[3], p);
}

__device__ __forceinline__ void unit4(const float* x, float* u) {
  const float den = fmaxf(__fsqrt_rn(butterfly(lane_dot4(x, x))), 1e-12f);
#pragma unroll
  for (int i = 0; i < 4; ++i) u[i] = __fdiv_rn(x[i], den);
}

__device__ __forceinline__ void load_row4(const __nv_bfloat16* row, int lane, float* x) {
  const uint2 raw = __ldg(reinterpret_cast<const uint2*>(row + 4 * lane));
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
  const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
  x[0] = a.x, x[1] = a.y, x[2] = b.x, x[3] = b.y;
}

// Monotone unsigned key of an fp32 value; -0 and +0 map to the same key.
__device__ __forceinline__ uint32_t order_key(float f) {
  if (f == 0.0f) f = 0.0f;
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Reduce-scatter of P per-lane partials with the butterfly's summation tree: on return
// lane l holds, in v[0 .. P/32) (or v[0] when P <= 32), the full sums of value indices
//   P >= 32: (P/32) * l + i;   P < 32: l / (32 / P).
template <int P>
__device__ __forceinline__ void reduce_scatter(float (&v)[P], int lane) {
  int m = P;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    if (m > 1) {
      const int half = m / 2;
      const bool upper = (lane & o) != 0;
#pragma unroll
      for (int i = 0; i < P / 2; ++i) {
        if (i < half) {
          const float send = upper ? v[i] : v[half + i];
          const float keep = upper ? v[half + i] : v[i];
          v[i] = __fadd_rn(keep, __shfl_xor_sync(kFull, send, o));
        }
      }
      m = half;
    } else {
      v[0] = __fadd_rn(v[0], __shfl_xor_sync(kFull, v[0], o));
    }
  }
}

// ===================================================================== metric
// M[r] = X^T X / S over the S sampled tokens of one (side, batch, head); 16 rows per CTA.
template <typename T>
__global__ void __launch_bounds__(256) metric_moment_kernel(const T* __restrict__ q, const T* __restrict__ k, int T_,
                                                            int H, int BH, const int32_t* __restrict__ samples, int S,
                                                            float* __restrict__ moments) {
  __shared__ float xs[32][kDim + 1];
  const int r = blockIdx.y;
  const int side = r / BH, bh = r % BH, b = bh / H, h = bh % H;
  const T* src = side == 0 ? q : k;  // rows [0, BH): moments of Q; [BH, 2BH): moments of K
  const int j = threadIdx.x & 127;
  const int i0 = blockIdx.x * 16 + (threadIdx.x >> 7) * 8;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int s0 = 0; s0 < S; s0 += 32) {
    __syncthreads();
    for (int e = threadIdx.x; e < 32 * kDim; e += 256) {
      const int s = s0 + e / kDim, d = e % kDim;
      xs[e / kDim][d] = s < S ? Elem<T>::to_f(src[(((int64_t)b * T_ + samples[s]) * H + h) * kDim + d]) : 0.f;
    }
    __syncthreads();
    const int count = min(32, S - s0);
    for (int s = 0; s < count; ++s) {
      const float xj = xs[s][j];
#pragma unroll
      for (int a = 0; a < 8; ++a) acc[a] = __fmaf_rn(xs[s][i0 + a], xj, acc[a]);
    }
  }
  float* m = moments + (int64_t)r * kDim * kDim;
#pragma unroll
  for (int a = 0; a < 8; ++a) m[(i0 + a) * kDim + j] = __fdiv_rn(acc[a], (float)S);
}

// Symmetrise, add ridge * trace / D to the diagonal and factor L L^T in place (lower).
__global__ void __launch_bounds__(256) cholesky_kernel(float* __restrict__ factors, float ridge) {
  extern __shared__ float A[];  // [128][129]
  constexpr int ld = kDim + 1;
  float* m = factors + (int64_t)blockIdx.x * kDim * kDim;
  for (int e = threadIdx.x; e < kDim * kDim; e += blockDim.x) A[(e / kDim) * ld + e % kDim] = m[e];
  __syncthreads();
  for (int e = threadIdx.x; e < kDim * kDim; e += blockDim.x) {
    const int i = e / kDim, j = e % kDim;
    if (i > j) {
      const float s = __fmul_rn(0.5f, __fadd_rn(A[i * ld + j], A[j * ld + i]));
      A[i * ld + j] = s;
      A[j * ld + i] = s;
    }
  }
  __syncthreads();
  __shared__ float ridge_add;
  if (threadIdx.x == 0) {
    float tr = 0.f;
    for (int i = 0; i < kDim; ++i) tr = __fadd_rn(tr, A[i * ld + i]);
    ridge_add = __fmul_rn(ridge, __fdiv_rn(tr, (float)kDim));
  }
  __syncthreads();
  if (threadIdx.x < kDim) A[threadIdx.x * ld + threadIdx.x] = __fadd_rn(A[threadIdx.x * ld + threadIdx.x], ridge_add);
  __syncthreads();
  __shared__ float pivot;
  for (int c = 0; c < kDim; ++c) {
    if (threadIdx.x == 0) {
      pivot = __fsqrt_rn(A[c * ld + c]);
      A[c * ld + c] = pivot;
    }
    __syncthreads();
    for (int i = c + 1 + threadIdx.x; i < kDim; i += blockDim.x) A[i * ld + c] = __fdiv_rn(A[i * ld + c], pivot);
    __syncthreads();
    const int rest = kDim - c - 1;
    for (int e = threadIdx.x; e < rest * rest; e += blockDim.x) {
      const int i = c + 1 + e / rest, j = c + 1 + e % rest;
      if (j <= i) A[i * ld + j] = __fsub_rn(A[i * ld + j], __fmul_rn(A[i * ld + c], A[j * ld + c]));
    }
    __syncthreads();
  }
  for (int e = threadIdx.x; e < kDim * kDim; e += blockDim.x) {
    const int i = e / kDim, j = e % kDim;
    m[e] = j <= i ? A[i * ld + j] : 0.f;
  }
}

// ================================================================== transform
constexpr int kTfThreads = 192;  // warps 0-3 epilogue, 4 TMA producer, 5 MMA issuer
constexpr int kTfStages = 3;
constexpr int kTfTileBytes = 128 * kDim * 2;  // 32 KB: two 64-column halves of 128 rows
constexpr int kTfHalfBytes = kTfTileBytes / 2;
constexpr int kTfWarpOutBytes = 32 * kDim * 2;  // one epilogue warp's 32 output rows (8 KB)
constexpr int kTfOutBytes = 2 * 4 * kTfWarpOutBytes;  // double-buffered, four epilogue warps

struct __align__(8) TfControl {
  uint64_t full[kTfStages], empty[kTfStages];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
};

struct TfParams {
  const float* factors;
  __nv_bfloat16* features;
  int* status;
  int T, H, BH, video, tiles, splits;
};

__global__ void __launch_bounds__(kTfThreads) reblock_transform_kernel(const __grid_constant__ CUtensorMap tm_k,
                                                                       const __grid_constant__ CUtensorMap tm_q,
                                                                       const __grid_constant__ CUtensorMap tm_out,
                                                                       TfParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  if ((smem_u32(smem) & 1023u) != 0u) {
    if (threadIdx.x == 0 && p.status) atomicExch(p.status, 920);
    return;
  }
  uint8_t* sB = smem;                                   // L^T, K-major, two 64-column halves
  uint8_t* sA = smem + kTfTileBytes;                    // token tiles
  uint8_t* sOut = smem + (1 + kTfStages) * kTfTileBytes;  // [2][4 warps][2 halves][32 rows][128 B]
  TfControl& C = *reinterpret_cast<TfControl*>(sOut + kTfOutBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.y;
  const int side = r / p.BH, bh = r % p.BH, b = bh / p.H, h = bh % p.H;
  const CUtensorMap* map = side == 0 ? &tm_k : &tm_q;  // rows [0, BH): K . L_Q; [BH, 2BH): Q . L_K
  if (threadIdx.x == 0) {
    for (int s = 0; s < kTfStages; ++s) {
      mbar_init(smem_u32(&C.full[s]), 1);
      mbar_init(smem_u32(&C.empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&C.acc_full[a]), 1);
      mbar_init(smem_u32(&C.acc_empty[a]), 128);
    }
    mbar_init(smem_u32(&C.mma_done), 1);
    C.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp < 4) {
    // B[n][k] = bf16(L[k][n]) in the 128-byte-swizzled K-major layout.
    const int n = threadIdx.x;
    const float* L = p.factors + (int64_t)r * kDim * kDim;
#pragma unroll 1
    for (int kh = 0; kh < 2; ++kh)
#pragma unroll 1
      for (int c = 0; c < 8; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int k0 = kh * 64 + c * 8 + 2 * e;
          w[e] = cvt_bf16x2(L[k0 * kDim + n], L[(k0 + 1) * kDim + n]);
        }
        *reinterpret_cast<uint4*>(sB + kh * kTfHalfBytes + n * 128 + ((c ^ (n & 7)) * 16)) =
            make_uint4(w[0], w[1], w[2], w[3]);
      }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(&C.tmem_base), 256);
    tmem_relinquish();
  }
  if (warp == 4 && lane == 0) {
    prefetch_tensormap(map);
    prefetch_tensormap(&tm_out);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = C.tmem_base;
  volatile int* abort_flag = &C.abort_flag;
  const uint32_t a_base = smem_u32(sA), b_base = smem_u32(sB);

  if (warp == 4) {
    if (lane == 0) {
      int armed[kTfStages] = {};
      int local = 0;
      for (int tile = blockIdx.x; tile < p.tiles; tile += p.splits, ++local) {
        const int s = local % kTfStages;
        if (!mbar_wait(smem_u32(&C.empty[s]), (uint32_t)(((local / kTfStages) & 1) ^ 1), abort_flag, p.status, 501))
          break;
        const uint32_t bar = smem_u32(&C.full[s]);
        mbar_arrive_expect_tx(bar, kTfTileBytes);
        ++armed[s];
        const uint32_t dst = a_base + s * kTfTileBytes;
        for (int dh = 0; dh < 2; ++dh)
          for (int rh = 0; rh < 2; ++rh)
            tma_load_3d(dst + dh * kTfHalfBytes + rh * (kTfHalfBytes / 2), map, bar, h * kDim + 64 * dh,
                        tile * 128 + 64 * rh, b);
      }
      for (int s = 0; s < kTfStages; ++s)
        if (armed[s] > 0) mbar_drain(smem_u32(&C.full[s]), (uint32_t)((armed[s] - 1) & 1));
    }
  } else if (warp == 5) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(128, 128, false);
      int local = 0;
      for (int tile = blockIdx.x; tile < p.tiles; tile += p.splits, ++local) {
        const int s = local % kTfStages, buf = local & 1;
        if (local >= 2 && !mbar_wait(smem_u32(&C.acc_empty[buf]), (uint32_t)(((local - 2) >> 1) & 1), abort_flag,
                                     p.status, 502))
          break;
        if (!mbar_wait(smem_u32(&C.full[s]), (uint32_t)((local / kTfStages) & 1), abort_flag, p.status, 503)) break;
        tc_fence_after();
        const uint32_t acc = tmem + buf * 128;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t ad = smem_desc_sw128(a_base + s * kTfTileBytes + (kk >> 2) * kTfHalfBytes, 16, 1024) +
                              (uint64_t)((kk & 3) * 2);
          const uint64_t bd = smem_desc_sw128(b_base + (kk >> 2) * kTfHalfBytes, 16, 1024) + (uint64_t)((kk & 3) * 2);
          mma_ss(acc, ad, bd, idesc, kk > 0 ? 1u : 0u);
        }
        tc_commit(smem_u32(&C.empty[s]));
        tc_commit(smem_u32(&C.acc_full[buf]));
      }
      tc_commit(smem_u32(&C.mma_done));
    }
  } else {
    // Epilogue: warp w owns rows 32w .. 32w + 31 of each tile.  It converts its rows to bf16
    // into a 128-byte-swizzled staging buffer (16-byte chunk c of row r at c ^ (r & 7), the
    // layout of a SWIZZLE_128B box) and writes them with two TMA stores (one per 64-column
    // half); two buffers alternate, and a buffer is reused once its store has read it.
    const int row = threadIdx.x;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const uint32_t out_base = smem_u32(sOut) + (uint32_t)(warp * 2 * kTfWarpOutBytes);
    int local = 0;
    for (int tile = blockIdx.x; tile < p.tiles; tile += p.splits, ++local) {
      const int buf = local & 1;
      const bool got = mbar_wait(smem_u32(&C.acc_full[buf]), (uint32_t)((local >> 1) & 1), abort_flag, p.status, 504);
      if (!__all_sync(kFull, got)) break;
      tc_fence_after();
      if (lane == 0) bulk_wait_group_read<1>();  // the store that last read this buffer is done
      __syncwarp();
      const uint32_t stage = out_base + (uint32_t)(buf * kTfWarpOutBytes);
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_base + buf * 128 + 32 * c, v);
        tmem_wait_ld();
        const uint32_t half = stage + (uint32_t)((c >> 1) * (kTfWarpOutBytes / 2)) + (uint32_t)(lane * 128);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int chunk = (c & 1) * 4 + q;  // 16-byte chunk of the 128-byte half row
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            w[e] = cvt_bf16x2(__uint_as_float(v[8 * q + 2 * e]), __uint_as_float(v[8 * q + 2 * e + 1]));
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(half + (uint32_t)((chunk ^ (lane & 7)) * 16)),
                       "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3])
                       : "memory");
        }
      }
      tc_fence_before();
      mbar_arrive(smem_u32(&C.acc_empty[buf]));  // TMEM columns are free once loaded
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const int y = tile * 128 + warp * 32;  // rows past the video end are clipped by the store
        tma_store_3d(&tm_out, stage, 0, y, r);
        tma_store_3d(&tm_out, stage + kTfWarpOutBytes / 2, 64, y, r);
        bulk_commit_group();
      }
    }
    if (lane == 0) bulk_wait_group<0>();  // every store has landed before the CTA exits
    __syncwarp();
    (void)row;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    mbar_drain(smem_u32(&C.mma_done), 0);
    tmem_dealloc(tmem, 256);
  }
}

// ======================================================================= tree
// Root order without the protected remainder: the N mod 64 tokens of largest squared
// feature norm (equal norms: lower id) go to the tail of the permutation in root order.
// With `frozen` ([rows][N mod 64] token ids, the caller's excluded_indices) those tokens form
// the tail instead; an id out of range is skipped, and a tail of the wrong size (out-of-range
// or repeated ids) sets status 612.  Every write stays inside the row either way.
__global__ void __launch_bounds__(1024) reblock_root_kernel(const __nv_bfloat16* __restrict__ F, int N, int active,
                                                            const int32_t* __restrict__ root_order,
                                                            const int32_t* __restrict__ frozen,
                                                            float* __restrict__ norms, int32_t* __restrict__ idx0,
                                                            int32_t* __restrict__ perm, int direct,
                                                            int* __restrict__ status) {
  const int r = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rem = N - active;
  float* nr = norms + (int64_t)r * N;
  __shared__ float best_v[32];
  __shared__ int best_i[32];
  __shared__ int counts[32][2];
  __shared__ int base[2];
  if (rem > 0 && frozen != nullptr) {
    for (int t = threadIdx.x; t < N; t += 1024) nr[t] = 0.f;
    __syncthreads();
    if (threadIdx.x < rem) {
      const int id = frozen[(int64_t)r * rem + threadIdx.x];
      if (id >= 0 && id < N) nr[id] = -1.0f;
    }
    __syncthreads();
  } else if (rem > 0) {
    for (int t = warp; t < N; t += 32) {
      float x[4];
      load_row4(F + ((int64_t)r * N + t) * kDim, lane, x);
      const float n2 = butterfly(lane_dot4(x, x));
      if (lane == 0) nr[t] = n2;
    }
    __syncthreads();
    for (int k = 0; k < rem; ++k) {
      float v = -2.f;
      int vi = 0x7fffffff;
      for (int t = threadIdx.x; t < N; t += 1024) {
        const float x = nr[t];
        if (x > v) v = x, vi = t;  // t increases: the first maximum stays
      }
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {
        const float ov = __shfl_xor_sync(kFull, v, o);
        const int oi = __shfl_xor_sync(kFull, vi, o);
        if (ov > v || (ov == v && oi < vi)) v = ov, vi = oi;
      }
      if (lane == 0) best_v[warp] = v, best_i[warp] = vi;
      __syncthreads();
      if (warp == 0) {
        v = best_v[lane];
        vi = best_i[lane];
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
          const float ov = __shfl_xor_sync(kFull, v, o);
          const int oi = __shfl_xor_sync(kFull, vi, o);
          if (ov > v || (ov == v && oi < vi)) v = ov, vi = oi;
        }
        if (lane == 0) nr[vi] = -1.0f;  // excluded (norms are never negative)
      }
      __syncthreads();
    }
  }
  if (threadIdx.x == 0) base[0] = 0, base[1] = 0;
  __syncthreads();
  int32_t* act_out = direct ? perm + (int64_t)r * N : idx0 + (int64_t)r * N;
  for (int c0 = 0; c0 < N; c0 += 1024) {
    const int pos = c0 + threadIdx.x;
    const bool valid = pos < N;
    const int id = valid ? (root_order ? root_order[pos] : pos) : 0;
    const bool ex = valid && rem > 0 && nr[id] == -1.0f;
    const unsigned m_ex = __ballot_sync(kFull, valid && ex), m_in = __ballot_sync(kFull, valid && !ex);
    if (lane == 0) counts[warp][0] = __popc(m_in), counts[warp][1] = __popc(m_ex);
    __syncthreads();
    int before_in = 0, before_ex = 0, tot_in = 0, tot_ex = 0;
    for (int w = 0; w < 32; ++w) {
      if (w < warp) before_in += counts[w][0], before_ex += counts[w][1];
      tot_in += counts[w][0], tot_ex += counts[w][1];
    }
    const unsigned lt = (1u << lane) - 1u;
    if (valid) {
      if (ex)
        perm[(int64_t)r * N + active + base[1] + before_ex + __popc(m_ex & lt)] = id;
      else
        act_out[base[0] + before_in + __popc(m_in & lt)] = id;
    }
    __syncthreads();
    if (threadIdx.x == 0) base[0] += tot_in, base[1] += tot_ex;
    __syncthreads();
  }
  if (threadIdx.x == 0 && base[1] != rem && status) atomicExch(status, 612);
}

struct TreeLevel {
  const int32_t* nodes;  // [nodes][kNodeInts]
  const int32_t* tiles;  // [active / 64] node of each 64-position tile, -1 when not split
  int count, P, S;
};

// The binary proxy tree over a node's C children (h3_sparse_attention
// landmark_v2_terminal.py:11-33, split_topology): the internal node of children [s0, s1)
// splits them at mid = s0 + (s1 - s0 + 1) / 2, internal nodes are numbered breadth first,
// and a child range of one child is finished.  Tags below kFinished name an internal node;
// kFinished + c names finished child c.  For a power-of-two C this is the heap: node h has
// children 2h + 1 and 2h + 2 and every child finishes at the last depth.
constexpr int kFinished = 64;
constexpr int kMaxDepths = 7;  // ceil(log2 64) depths of internal nodes, plus one

struct Topology {
  int lc[kMaxChildren], rc[kMaxChildren];  // token capacities of the left and right children
  uint8_t s0[kMaxChildren], mid[kMaxChildren], s1[kMaxChildren];
  uint8_t ltag[kMaxChildren], rtag[kMaxChildren];
  uint8_t first[kMaxDepths + 1];  // first internal node of each depth; first[depths] = C - 1
  int depths;
};

// Breadth-first construction by one thread (C <= 64: at most 63 internal nodes); caps holds
// the C child capacities in tokens.
__device__ void build_topology(int C, const int32_t* caps, Topology& t) {
  int count = 1, depth = 0;
  t.s0[0] = 0;
  t.s1[0] = (uint8_t)C;
  t.first[0] = 0;
  int depth_end = 1;  // one past the last node of the current depth
  for (int k = 0; k < count; ++k) {
    if (k == depth_end) {
      t.first[++depth] = (uint8_t)k;
      depth_end = count;
    }
    const int a = t.s0[k], b = t.s1[k], m = a + (b - a + 1) / 2;
    t.mid[k] = (uint8_t)m;
    if (m - a == 1) {
      t.ltag[k] = (uint8_t)(kFinished + a);
    } else {
      t.s0[count] = (uint8_t)a, t.s1[count] = (uint8_t)m, t.ltag[k] = (uint8_t)count++;
    }
    if (b - m == 1) {
      t.rtag[k] = (uint8_t)(kFinished + m);
    } else {
      t.s0[count] = (uint8_t)m, t.s1[count] = (uint8_t)b, t.rtag[k] = (uint8_t)count++;
    }
  }
  t.depths = depth + 1;
  t.first[t.depths] = (uint8_t)count;
  for (int k = 0; k < count; ++k) {
    int l = 0, r = 0;
    for (int c = t.s0[k]; c < t.mid[k]; ++c) l += caps[c];
    for (int c = t.mid[k]; c < t.s1[k]; ++c) r += caps[c];
    t.lc[k] = l;
    t.rc[k] = r;
  }
}

// One CTA of four warps per (node, row): midpoint landmarks, their unit vectors and pairwise
// cosine distances (four threads per vector), then the binary proxy tree with the internal
// nodes of one depth spread over the warps; directions are written by topology node.
constexpr int kProxyThreads = 128;

// act (the landmark weights each internal node of a depth passes down, two depths) comes last
// and is sized per level: [2][max(1, fanout / 2)][kLandmarks] ints (a depth of a C-child tree
// holds at most C / 2 internal nodes).
struct ProxySmem {
  __nv_bfloat16 x[kLandmarks][kDim];
  float n[kLandmarks][kDim];
  float dist[kLandmarks][kLandmarks + 1];
  int id[kLandmarks], w[kLandmarks];
  Topology topo;
  int act[1];
};

__host__ __device__ constexpr int proxy_act_rows(int fanout) { return fanout / 2 > 1 ? fanout / 2 : 1; }

inline size_t proxy_smem_bytes(int fanout) {
  return offsetof(ProxySmem, act) + sizeof(int) * 2 * proxy_act_rows(fanout) * kLandmarks;
}

// Canonical dot products with four threads per 128-vector: thread t4 of the group holds the
// lane groups l = t4 + 4j (j = 0..7), so the butterfly's offsets 16, 8 and 4 pair lane groups
// inside the thread (j ^ 4, j ^ 2, j ^ 1) and only offsets 2 and 1 cross threads.  The
// summation tree is the one of the 32-lane form, term for term.
__device__ __forceinline__ float tree8(const float* p) {
  float a[4], b[2];
#pragma unroll
  for (int j = 0; j < 4; ++j) a[j] = __fadd_rn(p[j], p[j + 4]);
#pragma unroll
  for (int j = 0; j < 2; ++j) b[j] = __fadd_rn(a[j], a[j + 2]);
  return __fadd_rn(b[0], b[1]);
}

__device__ __forceinline__ uint64_t tree8x2(const uint64_t* p) {
  uint64_t a[4], b[2];
#pragma unroll
  for (int j = 0; j < 4; ++j) a[j] = f2_add(p[j], p[j + 4]);
#pragma unroll
  for (int j = 0; j < 2; ++j) b[j] = f2_add(a[j], a[j + 2]);
  return f2_add(b[0], b[1]);
}

// Full canonical dot of two quarter-held vectors (all four threads get the result).
__device__ __forceinline__ float quad_dot(const float (&a)[8][4], const float (&b)[8][4]) {
  float p[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) p[j] = lane_dot4(a[j], b[j]);
  float v = tree8(p);
  v = __fadd_rn(v, __shfl_xor_sync(kFull, v, 2));
  return __fadd_rn(v, __shfl_xor_sync(kFull, v, 1));
}

// unit(x) of a quarter-held vector, in place.
__device__ __forceinline__ void quad_unit(float (&x)[8][4]) {
  const float den = fmaxf(__fsqrt_rn(quad_dot(x, x)), 1e-12f);
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) x[j][e] = __fdiv_rn(x[j][e], den);
}

// kIters: mean-update passes of the proxy tree, 0, 1, 2 (production) or 4; kEndpoint: seeds are
// the lowest and highest valid landmark instead of the farthest pair (landmark_v2_terminal.py:43-50).
template <int kIters, bool kEndpoint>
__global__ void __launch_bounds__(kProxyThreads, 7) reblock_proxy_kernel(const __nv_bfloat16* __restrict__ F, int N,
                                                                       int active, TreeLevel lv,
                                                                       const int32_t* __restrict__ idx_in,
                                                                       float* __restrict__ dirs) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  ProxySmem& S = *reinterpret_cast<ProxySmem*>(smem_raw);
  const int act_rows = proxy_act_rows(lv.P);
  auto act = [&](int buf, int j) -> int* { return S.act + (buf * act_rows + j) * kLandmarks; };
  const int node = blockIdx.x, r = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int32_t* tbl = lv.nodes + (int64_t)node * kNodeInts;
  const int start = tbl[0], n = tbl[1], C = tbl[2];
  const int32_t* caps = tbl + 4;
  const int32_t* ids = idx_in + (int64_t)r * N + start;
  const __nv_bfloat16* Fr = F + (int64_t)r * N * kDim;
  if (tid < kLandmarks) {  // midpoint of each of 32 equal intervals, weighted by its length
    const int64_t lo = (int64_t)tid * n / kLandmarks, hi = (int64_t)(tid + 1) * n / kLandmarks;
    S.id[tid] = ids[lo + (hi - lo) / 2];
    S.w[tid] = (int)(hi - lo);
  }
  if (tid == kLandmarks) build_topology(C, caps, S.topo);
  __syncthreads();
  for (int i = warp; i < kLandmarks; i += 4)
    *reinterpret_cast<uint2*>(&S.x[i][4 * lane]) =
        __ldg(reinterpret_cast<const uint2*>(Fr + (int64_t)S.id[i] * kDim + 4 * lane));
  __syncthreads();
  const int g = tid >> 2, t4 = tid & 3;  // four threads per landmark vector
  {
    float u[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) u[j][e] = __bfloat162float(S.x[g][4 * (t4 + 4 * j) + e]);
    quad_unit(u);
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) S.n[g][4 * (t4 + 4 * j) + e] = u[j][e];
  }
  __syncthreads();
  {
    // rows a and 31 - a (31 pairs together); the two halves of the groups take alternate pairs
    const int a = g & 15, b = 31 - a, half = g >> 4;
    for (int t = half; t < 31; t += 2) {
      const int i = t < 31 - a ? a : b;
      const int k = t < 31 - a ? a + 1 + t : b + 1 + (t - (31 - a));
      float ni[8][4], nk[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          ni[j][e] = S.n[i][4 * (t4 + 4 * j) + e];
          nk[j][e] = S.n[k][4 * (t4 + 4 * j) + e];
        }
      const float d = __fsub_rn(1.0f, quad_dot(ni, nk));
      if (t4 == 0) S.dist[i][k] = d;
    }
  }
  if (tid < kLandmarks) act(0, 0)[tid] = S.w[tid];
  __syncthreads();
  float* out = dirs + ((int64_t)r * lv.count + node) * lv.S * kDim;
  const Topology& topo = S.topo;
  int cur = 0;
  for (int depth = 0; depth < topo.depths; ++depth) {
    const int k0 = topo.first[depth], next0 = topo.first[depth + 1];
    for (int j = warp; j < next0 - k0; j += 4) {
      const int hnode = k0 + j;
      const int lc = topo.lc[hnode], rc = topo.rc[hnode];
      const int aw = act(cur, j)[lane];
      const unsigned vmask = __ballot_sync(kFull, aw > 0);
      int first = vmask ? __ffs(vmask) - 1 : 0, second = first;
      if (kEndpoint && __popc(vmask) >= 2) {
        second = 31 - __clz(vmask);  // the lowest and the highest valid landmark
      } else if (__popc(vmask) >= 2) {
        // farthest valid pair, first in row-major (i, k) order
        float bv = 0.f;
        int bk = -1;
        if (aw > 0)
          for (int k = lane + 1; k < kLandmarks; ++k)
            if ((vmask >> k) & 1u) {
              const float d = S.dist[lane][k];
              if (bk < 0 || d > bv) bv = d, bk = k;
            }
        int bi = lane;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
          const float ov = __shfl_xor_sync(kFull, bv, o);
          const int ok = __shfl_xor_sync(kFull, bk, o), oi = __shfl_xor_sync(kFull, bi, o);
          const bool take = ok >= 0 && (bk < 0 || ov > bv || (ov == bv && oi < bi));
          if (take) bv = ov, bk = ok, bi = oi;
        }
        first = bi;
        second = bk;
      }
      float left[4], right[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        left[e] = __bfloat162float(S.x[first][4 * lane + e]);
        right[e] = __bfloat162float(S.x[second][4 * lane + e]);
      }
      int lw = 0, rw = 0;
      // max(1, passes) assignments; with zero updates the one assignment only hands the
      // children their landmark weights, and the seeds give the direction
      for (int it = 0; it < (kIters > 0 ? kIters : 1); ++it) {
        float ul[4], ur[4], dir[4];
        unit4(left, ul);
        unit4(right, ur);
#pragma unroll
        for (int e = 0; e < 4; ++e) dir[e] = __fsub_rn(ur[e], ul[e]);
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float nn[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) nn[e] = S.n[i][4 * lane + e];
          v[i] = lane_dot4(nn, dir);
        }
        reduce_scatter<32>(v, lane);
        const float my_s = v[0];  // score of landmark `lane`
        int rank = 0;
        for (int jj = 0; jj < 32; ++jj) {
          const float sj = __shfl_sync(kFull, my_s, jj);
          rank += (sj < my_s || (sj == my_s && jj < lane)) ? 1 : 0;
        }
        int before = 0;
        for (int jj = 0; jj < 32; ++jj) {
          const int rj = __shfl_sync(kFull, rank, jj), aj = __shfl_sync(kFull, aw, jj);
          if (rj < rank) before += aj;
        }
        lw = min(max(lc - before, 0), aw);
        rw = aw - lw;
        if (it >= kIters) break;
        float accl[4] = {0.f, 0.f, 0.f, 0.f}, accr[4] = {0.f, 0.f, 0.f, 0.f};
        for (int jj = 0; jj < 32; ++jj) {
          const float wl = (float)__shfl_sync(kFull, lw, jj), wr = (float)__shfl_sync(kFull, rw, jj);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float xj = __bfloat162float(S.x[jj][4 * lane + e]);
            accl[e] = __fmaf_rn(wl, xj, accl[e]);
            accr[e] = __fmaf_rn(wr, xj, accr[e]);
          }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          left[e] = __fdiv_rn(accl[e], (float)lc);
          right[e] = __fdiv_rn(accr[e], (float)rc);
        }
      }
      float ul[4], ur[4], dir[4];
      unit4(left, ul);
      unit4(right, ur);
#pragma unroll
      for (int e = 0; e < 4; ++e) dir[e] = __fsub_rn(ur[e], ul[e]);
      *reinterpret_cast<float4*>(out + (int64_t)hnode * kDim + 4 * lane) = make_float4(dir[0], dir[1], dir[2], dir[3]);
      // internal children take their weights at their place in the next depth
      if (topo.ltag[hnode] < kFinished) act(cur ^ 1, topo.ltag[hnode] - next0)[lane] = lw;
      if (topo.rtag[hnode] < kFinished) act(cur ^ 1, topo.rtag[hnode] - next0)[lane] = rw;
    }
    __syncthreads();
    cur ^= 1;
  }
}

// Split scores of every token of the splitting nodes: s[h] = dot(unit(x), dir_h); four
// threads per token, directions paired for packed f32x2 multiply-adds.  A CTA walks
// kScoreTiles consecutive 64-token tiles (reloading the directions only when the node
// changes) and fetches the next tile's feature rows while it scores the current one.
constexpr int kScoreTiles = 8;

// Reduce-scatter of the P scores of one token over the four threads of its quad (offsets 2
// and 1 of the butterfly), then the store of this thread's share.
template <int P>
__device__ __forceinline__ void score_reduce_store(float (&v)[P], int t4, int C, float* out) {
  int m = P;
#pragma unroll
  for (int o = 2; o >= 1; o >>= 1) {
    if (m > 1) {
      const int half = m / 2;
      const bool upper = (t4 & o) != 0;
#pragma unroll
      for (int i = 0; i < P / 2; ++i) {
        if (i < half) {
          const float send = upper ? v[i] : v[half + i];
          const float keep = upper ? v[half + i] : v[i];
          v[i] = __fadd_rn(keep, __shfl_xor_sync(kFull, send, o));
        }
      }
      m = half;
    } else {
      v[0] = __fadd_rn(v[0], __shfl_xor_sync(kFull, v[0], o));
    }
  }
  if (P >= 4) {
#pragma unroll
    for (int i = 0; i < (P >= 4 ? P / 4 : 1); ++i) {
      const int hh = t4 * (P / 4) + i;
      if (hh < C - 1) out[hh] = v[i];
    }
  } else if ((t4 & 1) == 0 && (t4 >> 1) < C - 1) {
    out[t4 >> 1] = v[0];
  }
}

// TT tokens per quad share every direction element read from shared memory.
template <int P, int TT>
__device__ __forceinline__ void score_tokens(const uint2 (&raw)[TT][8], const float2 (*sd)[kDim], int t4, int C,
                                             float* const (&out)[TT]) {
  float u[TT][8][4];
#pragma unroll
  for (int t = 0; t < TT; ++t) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[t][j]);
      const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
      u[t][j][0] = a.x, u[t][j][1] = a.y, u[t][j][2] = b.x, u[t][j][3] = b.y;
    }
    quad_unit(u[t]);
  }
  float v[TT][P];
#pragma unroll
  for (int q = 0; q < P / 2; ++q) {
    uint64_t c[TT][8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4* dp = reinterpret_cast<const float4*>(&sd[q][4 * (t4 + 4 * j)]);
      const float4 d01 = dp[0], d23 = dp[1];  // (h0, h1) pairs of elements 0..3
#pragma unroll
      for (int t = 0; t < TT; ++t) {
        uint64_t acc = f2_mul(f2_pack(u[t][j][0], u[t][j][0]), f2_pack(d01.x, d01.y));
        acc = f2_fma(f2_pack(u[t][j][1], u[t][j][1]), f2_pack(d01.z, d01.w), acc);
        acc = f2_fma(f2_pack(u[t][j][2], u[t][j][2]), f2_pack(d23.x, d23.y), acc);
        c[t][j] = f2_fma(f2_pack(u[t][j][3], u[t][j][3]), f2_pack(d23.z, d23.w), acc);
      }
    }
#pragma unroll
    for (int t = 0; t < TT; ++t) f2_unpack(tree8x2(c[t]), v[t][2 * q], v[t][2 * q + 1]);
  }
#pragma unroll
  for (int t = 0; t < TT; ++t) score_reduce_store<P>(v[t], t4, C, out[t]);
}

template <int P>
__device__ __forceinline__ void score_token(const uint2 (&raw)[8], const float2 (*sd)[kDim], int t4, int C,
                                            float* out) {
  float u[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[j]);
    const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
    u[j][0] = a.x, u[j][1] = a.y, u[j][2] = b.x, u[j][3] = b.y;
  }
  quad_unit(u);
  float v[P];
#pragma unroll
  for (int q = 0; q < P / 2; ++q) {
    uint64_t c[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4* dp = reinterpret_cast<const float4*>(&sd[q][4 * (t4 + 4 * j)]);
      const float4 d01 = dp[0], d23 = dp[1];  // (h0, h1) pairs of elements 0..3
      uint64_t acc = f2_mul(f2_pack(u[j][0], u[j][0]), f2_pack(d01.x, d01.y));
      acc = f2_fma(f2_pack(u[j][1], u[j][1]), f2_pack(d01.z, d01.w), acc);
      acc = f2_fma(f2_pack(u[j][2], u[j][2]), f2_pack(d23.x, d23.y), acc);
      c[j] = f2_fma(f2_pack(u[j][3], u[j][3]), f2_pack(d23.z, d23.w), acc);
    }
    f2_unpack(tree8x2(c), v[2 * q], v[2 * q + 1]);
  }
  // offsets 2 and 1: reduce-scatter of the P values over the four threads
  int m = P;
#pragma unroll
  for (int o = 2; o >= 1; o >>= 1) {
    if (m > 1) {
      const int half = m / 2;
      const bool upper = (t4 & o) != 0;
#pragma unroll
      for (int i = 0; i < P / 2; ++i) {
        if (i < half) {
          const float send = upper ? v[i] : v[half + i];
          const float keep = upper ? v[half + i] : v[i];
          v[i] = __fadd_rn(keep, __shfl_xor_sync(kFull, send, o));
        }
      }
      m = half;
    } else {
      v[0] = __fadd_rn(v[0], __shfl_xor_sync(kFull, v[0], o));
    }
  }
  if (P >= 4) {
#pragma unroll
    for (int i = 0; i < (P >= 4 ? P / 4 : 1); ++i) {
      const int hh = t4 * (P / 4) + i;
      if (hh < C - 1) out[hh] = v[i];
    }
  } else if ((t4 & 1) == 0 && (t4 >> 1) < C - 1) {
    out[t4 >> 1] = v[0];
  }
}

template <int P>
__global__ void __launch_bounds__(256) reblock_score_kernel(const __nv_bfloat16* __restrict__ F, int N, int active,
                                                            TreeLevel lv, const int32_t* __restrict__ idx_in,
                                                            const float* __restrict__ dirs,
                                                            float* __restrict__ scores) {
  static_assert(P >= 2 && (P & (P - 1)) == 0, "P is a power of two");
  __shared__ __align__(16) float2 sd[P / 2][kDim];
  __shared__ int s_node[kScoreTiles];
  const int r = blockIdx.y;
  const int tiles = active / 64;
  const int tile0 = blockIdx.x * kScoreTiles;
  const int ntiles = min(kScoreTiles, tiles - tile0);
  if (threadIdx.x < kScoreTiles) s_node[threadIdx.x] = threadIdx.x < ntiles ? lv.tiles[tile0 + threadIdx.x] : -1;
  __syncthreads();
  const int tk = threadIdx.x >> 2, t4 = threadIdx.x & 3;
  const __nv_bfloat16* Fr = F + (int64_t)r * N * kDim;
  const int32_t* ir = idx_in + (int64_t)r * N;
  auto fetch = [&](int tile, uint2 (&raw)[8]) {
    const int id = ir[tile * 64 + tk];
    const __nv_bfloat16* row = Fr + (int64_t)id * kDim;
#pragma unroll
    for (int j = 0; j < 8; ++j) raw[j] = __ldg(reinterpret_cast<const uint2*>(row + 4 * (t4 + 4 * j)));
  };
  int i = 0;
  while (i < ntiles && s_node[i] < 0) ++i;
  if (i == ntiles) return;
  uint2 cur[8], nxt[8];
  fetch(tile0 + i, cur);
  int loaded = -1, C = 2;
  while (i < ntiles) {
    const int node = s_node[i];
    int next = i + 1;
    while (next < ntiles && s_node[next] < 0) ++next;
    if (next < ntiles) fetch(tile0 + next, nxt);
    if (node != loaded) {
      __syncthreads();
      C = lv.nodes[(int64_t)node * kNodeInts + 2];
      const float* nd = dirs + ((int64_t)r * lv.count + node) * lv.S * kDim;
      for (int e = threadIdx.x; e < (P / 2) * kDim; e += blockDim.x) {
        const int q = e / kDim, d = e % kDim;
        sd[q][d] = make_float2(2 * q < C - 1 ? nd[(2 * q) * kDim + d] : 0.f,
                               2 * q + 1 < C - 1 ? nd[(2 * q + 1) * kDim + d] : 0.f);
      }
      __syncthreads();
      loaded = node;
    }
    const int pos = (tile0 + i) * 64 + tk;
    score_token<P>(cur, sd, t4, C, scores + ((int64_t)r * active + pos) * lv.S);
#pragma unroll
    for (int j = 0; j < 8; ++j) cur[j] = nxt[j];
    i = next;
  }
}

// The same scores with the gathered feature rows staged in shared memory.  A CTA first
// copies the ids of its tiles, then streams the rows of up to two tiles ahead into a
// three-stage ring with cp.async (16-byte chunks, XOR-swizzled by row so that the eight quads
// of a warp read distinct banks) while it scores the current tile out of shared memory: the
// loads in flight no longer cost registers.  Two tokens per quad (tokens tk and tk + 32 of a
// 64-token tile) share each direction element read from shared memory; the arithmetic is
// score_tokens<P, 2>.
constexpr int kScoreStages = 3;
constexpr int kScoreRowBytes = kDim * 2;  // one bf16 feature row
constexpr int kScoreStageBytes = 64 * kScoreRowBytes;
constexpr int kScoreRingBytes = kScoreStages * kScoreStageBytes;

template <int P>
__global__ void __launch_bounds__(128) reblock_score3_kernel(const __nv_bfloat16* __restrict__ F, int N, int active,
                                                             TreeLevel lv, const int32_t* __restrict__ idx_in,
                                                             const float* __restrict__ dirs,
                                                             float* __restrict__ scores) {
  static_assert(P >= 2 && (P & (P - 1)) == 0 && P <= 16, "P is a power of two up to 16");
  extern __shared__ __align__(16) uint8_t ring[];  // [kScoreStages][64 rows][256 bytes]
  __shared__ __align__(16) float2 sd[P / 2][kDim];
  __shared__ int s_ids[kScoreTiles][64];
  __shared__ int s_tile[kScoreTiles], s_node[kScoreTiles], s_count;
  const int r = blockIdx.y;
  const int tiles = active / 64;
  const int tile0 = blockIdx.x * kScoreTiles;
  const int ntiles = min(kScoreTiles, tiles - tile0);
  const int tid = threadIdx.x;
  const __nv_bfloat16* Fr = F + (int64_t)r * N * kDim;
  const int32_t* ir = idx_in + (int64_t)r * N + (int64_t)tile0 * 64;
  for (int c = tid; c < ntiles * 64; c += blockDim.x) cp_async4(&s_ids[c >> 6][c & 63], ir + c);
  cp_async_commit();
  if (tid == 0) {
    int m = 0;
    for (int i = 0; i < ntiles; ++i) {
      const int node = lv.tiles[tile0 + i];
      if (node >= 0) {
        s_tile[m] = i;
        s_node[m] = node;
        ++m;
      }
    }
    s_count = m;
  }
  cp_async_wait<0>();
  __syncthreads();
  const int M = s_count;
  if (M == 0) return;
  // Rows of the k-th listed tile into stage k mod kScoreStages: 16 threads per row, eight
  // rows per thread.  One commit group per call (empty past the end), so that the group
  // count is the same for every thread and every call.
  auto issue = [&](int k) {
    if (k < M) {
      const int* ids = s_ids[s_tile[k]];
      uint8_t* st = ring + (k % kScoreStages) * kScoreStageBytes;
      const int chunk = tid & 15;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int row = (tid >> 4) + 8 * q;
        cp_async16(st + row * kScoreRowBytes + ((chunk ^ (row & 15)) << 4), Fr + (int64_t)ids[row] * kDim + chunk * 8);
      }
    }
    cp_async_commit();
  };
  issue(0);
  issue(1);
  const int tk = tid >> 2, t4 = tid & 3;  // tokens tk and tk + 32 of a tile
  int loaded = -1, C = 2;
  for (int k = 0; k < M; ++k) {
    cp_async_wait<1>();  // tile k's group has landed: only the newest group, tile k + 1's, may be in flight
    __syncthreads();     // every thread's rows are visible, and stage (k + 2) mod 3 (tile k - 1) is free
    const int node = s_node[k];
    if (node != loaded) {
      C = lv.nodes[(int64_t)node * kNodeInts + 2];
      const float* nd = dirs + ((int64_t)r * lv.count + node) * lv.S * kDim;
      for (int e = tid; e < (P / 2) * kDim; e += blockDim.x) {
        const int q = e / kDim, d = e % kDim;
        sd[q][d] = make_float2(2 * q < C - 1 ? nd[(2 * q) * kDim + d] : 0.f,
                               2 * q + 1 < C - 1 ? nd[(2 * q + 1) * kDim + d] : 0.f);
      }
      __syncthreads();
      loaded = node;
    }
    issue(k + 2);
    const uint8_t* st = ring + (k % kScoreStages) * kScoreStageBytes;
    uint2 raw[2][8];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const int row = tk + 32 * t;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int byte = 8 * (t4 + 4 * j);  // elements 4 (t4 + 4 j) .. +3 of the row
        raw[t][j] = *reinterpret_cast<const uint2*>(st + row * kScoreRowBytes + (((byte >> 4) ^ (row & 15)) << 4) +
                                                    (byte & 15));
      }
    }
    const int pos = (tile0 + s_tile[k]) * 64 + tk;
    float* const outs[2] = {scores + ((int64_t)r * active + pos) * lv.S,
                            scores + ((int64_t)r * active + pos + 32) * lv.S};
    score_tokens<P, 2>(raw, sd, t4, C, outs);
  }
}

// Exact-capacity routing of one node (per internal proxy node: the left capacity goes to the
// smallest (score, id) keys) and the stable partition into the children.  Nodes of up to
// 1024 tokens sort (proxy node, score key, id) in shared memory each depth; larger nodes find
// the cut with a radix select over the score key (ids break equal keys).
constexpr int kRouteThreads = 512;
constexpr int kRouteWarps = kRouteThreads / 32;
constexpr int kSortMax = 1024;
constexpr int kUnroll = 8;

template <int THREADS, bool RADIX>
__global__ void __launch_bounds__(THREADS) reblock_route_kernel(int N, int active, TreeLevel lv,
                                                                      const int32_t* __restrict__ idx_in,
                                                                      const float* __restrict__ scores,
                                                                      uint32_t* __restrict__ keys,
                                                                      uint8_t* __restrict__ state,
                                                                      int32_t* __restrict__ idx_out,
                                                                      int32_t* __restrict__ perm,
                                                                      int* __restrict__ status) {
  // radix histograms (32 nodes x 256 digits), or the sort keys
  __shared__ __align__(16) uint8_t scratch[RADIX ? 32 * 256 * 4 : kSortMax * 8];
  __shared__ int target[32], ties[32], need_ids[32], seg[32];
  __shared__ uint32_t prefix[32], id_prefix[32];
  __shared__ unsigned long long cut[32];  // small nodes: the key of the target-th smallest token
  __shared__ int any_ids;
  __shared__ int warp_cnt[(THREADS / 32)][kMaxChildren];
  __shared__ int warp_off[(THREADS / 32)][kMaxChildren];
  __shared__ int running[kMaxChildren], child_off[kMaxChildren];
  __shared__ Topology topo;
  int(*hist)[256] = reinterpret_cast<int(*)[256]>(scratch);
  unsigned long long* sk = reinterpret_cast<unsigned long long*>(scratch);
  const int node = blockIdx.x, r = blockIdx.y;
  const int32_t* tbl = lv.nodes + (int64_t)node * kNodeInts;
  const int start = tbl[0], n = tbl[1], C = tbl[2];
  const int32_t* caps = tbl + 4;
  const int32_t* ids = idx_in + (int64_t)r * N + start;
  const float* sc = scores + ((int64_t)r * active + start) * lv.S;
  uint32_t* key = keys + (int64_t)r * active + start;
  uint8_t* st = state + (int64_t)r * active + start;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool small = n <= kSortMax;
  if (!RADIX && !small) {  // the launcher sends larger nodes to the radix form; refuse uniformly
    if (threadIdx.x == 0 && status) atomicExch(status, 611);
    return;
  }
  int n2 = 1;
  while (n2 < n) n2 <<= 1;
  for (int t = tid; t < n; t += THREADS) st[t] = 0;
  if (tid == 0) build_topology(C, caps, topo);
  __syncthreads();
  // st[t]: the token's internal proxy node, or kFinished + child once its child is decided
  for (int depth = 0; depth < topo.depths; ++depth) {
    const int first_node = topo.first[depth];
    const int nd = topo.first[depth + 1] - first_node;
    if (tid < nd) {
      // the node's left capacity; the tokens of the depth's earlier nodes (their whole
      // capacities) come before its own in the sorted keys
      const int k = first_node + tid;
      int before = 0;
      for (int jn = first_node; jn < k; ++jn) before += topo.lc[jn] + topo.rc[jn];
      target[tid] = topo.lc[k];
      seg[tid] = before;
      prefix[tid] = 0;
      id_prefix[tid] = 0;
    }
    if (small) {
      // (proxy node, score key, token id) as one unique 64-bit key per token; the sort only
      // has to find, per proxy node, the key of its target-th smallest token (the cut), and
      // every token then compares its own key with its node's cut.
      unsigned long long mine[kSortMax / THREADS];
#pragma unroll
      for (int q = 0; q < kSortMax / THREADS; ++q) {
        const int e = tid + q * THREADS;
        unsigned long long k64 = ~0ull;  // padding and finished tokens sort last
        if (e < n && st[e] < kFinished) {
          const int h = st[e];
          const uint32_t kk = order_key(sc[(int64_t)e * lv.S + h]);
          k64 = ((unsigned long long)(h - first_node) << 57) | ((unsigned long long)kk << 25) |
                (unsigned long long)(uint32_t)ids[e];
        }
        mine[q] = k64;
        if (e < n2) sk[e] = k64;
      }
      __syncthreads();
      // Bitonic sort, one compare-exchange per thread and step: only the first n2 / 2 threads
      // (at least one warp) take part, synchronised by a named barrier of their own.
      const int pairs = n2 >> 1;
      const int sorters = pairs < 32 ? 32 : (pairs < THREADS ? pairs : THREADS);
      if (tid < sorters) {
        for (int k = 2; k <= n2; k <<= 1)
          for (int j = k >> 1; j > 0; j >>= 1) {
            for (int p = tid; p < pairs; p += THREADS) {
              const int i = ((p & ~(j - 1)) << 1) | (p & (j - 1));  // bit j of i is clear
              const unsigned long long a = sk[i], b = sk[i | j];
              if ((a > b) == ((i & k) == 0)) {
                sk[i] = b;
                sk[i | j] = a;
              }
            }
            if (sorters == 32)
              __syncwarp();
            else
              asm volatile("bar.sync 1, %0;" ::"r"(sorters) : "memory");
          }
      }
      __syncthreads();
      if (tid < nd) cut[tid] = target[tid] > 0 ? sk[seg[tid] + target[tid] - 1] : 0ull;
      __syncthreads();
#pragma unroll
      for (int q = 0; q < kSortMax / THREADS; ++q) {
        const int e = tid + q * THREADS;
        if (e < n && mine[q] != ~0ull) {
          const int j = (int)(mine[q] >> 57);
          const int hnode = first_node + j;
          st[e] = target[j] > 0 && mine[q] <= cut[j] ? topo.ltag[hnode] : topo.rtag[hnode];
        }
      }
      __syncthreads();
    } else if constexpr (RADIX) {
      for (int t0 = tid; t0 < n; t0 += kUnroll * THREADS) {
        int hs[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int t = t0 + u * THREADS;
          hs[u] = t < n ? st[t] : kFinished;
        }
        float vs[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int t = t0 + u * THREADS;
          vs[u] = hs[u] < kFinished ? sc[(int64_t)t * lv.S + hs[u]] : 0.f;
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int t = t0 + u * THREADS;
          if (hs[u] < kFinished) key[t] = order_key(vs[u]);
        }
      }
      __syncthreads();
      // radix select on the score key, most significant byte first
      for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        for (int e = tid; e < nd * 256; e += THREADS) hist[e >> 8][e & 255] = 0;
        __syncthreads();
        for (int t0 = tid; t0 < n; t0 += kUnroll * THREADS) {
          uint32_t ks[kUnroll];
          int js[kUnroll];
#pragma unroll
          for (int u = 0; u < kUnroll; ++u) {
            const int t = t0 + u * THREADS;
            const int h = t < n ? st[t] : kFinished;
            js[u] = h < kFinished ? h - first_node : -1;
            ks[u] = h < kFinished ? key[t] : 0u;
          }
#pragma unroll
          for (int u = 0; u < kUnroll; ++u) {
            const int j = js[u];
            if (j >= 0 && (pass == 0 || (ks[u] >> (shift + 8)) == (prefix[j] >> (shift + 8))))
              atomicAdd(&hist[j][(ks[u] >> shift) & 255], 1);
          }
        }
        __syncthreads();
        if (tid < nd) {
          int cum = 0, want = target[tid];
          for (int bin = 0; bin < 256; ++bin) {
            const int c = hist[tid][bin];
            if (cum + c >= want) {
              prefix[tid] |= (uint32_t)bin << shift;
              target[tid] = want - cum;
              ties[tid] = c;
              break;
            }
            cum += c;
          }
        }
        __syncthreads();
      }
      if (tid == 0) {
        int any = 0;
        for (int j = 0; j < nd; ++j) {
          need_ids[j] = target[j] < ties[j] ? 1 : 0;
          any |= need_ids[j];
        }
        any_ids = any;
      }
      __syncthreads();
      if (any_ids) {
        // equal scores at the cut: the lowest token ids among them go left
        for (int pass = 0; pass < 4; ++pass) {
          const int shift = 24 - 8 * pass;
          for (int e = tid; e < nd * 256; e += THREADS) hist[e >> 8][e & 255] = 0;
          __syncthreads();
          for (int t = tid; t < n; t += THREADS) {
            const int h = st[t];
            if (h >= kFinished) continue;
            const int j = h - first_node;
            if (!need_ids[j] || key[t] != prefix[j]) continue;
            const uint32_t id = (uint32_t)ids[t];
            if (pass == 0 || (id >> (shift + 8)) == (id_prefix[j] >> (shift + 8)))
              atomicAdd(&hist[j][(id >> shift) & 255], 1);
          }
          __syncthreads();
          if (tid < nd && need_ids[tid]) {
            int cum = 0, want = target[tid];
            for (int bin = 0; bin < 256; ++bin) {
              const int c = hist[tid][bin];
              if (cum + c >= want) {
                id_prefix[tid] |= (uint32_t)bin << shift;
                target[tid] = want - cum;
                break;
              }
              cum += c;
            }
          }
          __syncthreads();
        }
      }
      for (int t0 = tid; t0 < n; t0 += kUnroll * THREADS) {
        int hs[kUnroll];
        uint32_t ks[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int t = t0 + u * THREADS;
          hs[u] = t < n ? st[t] : kFinished;
          ks[u] = hs[u] < kFinished ? key[t] : 0u;
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int t = t0 + u * THREADS;
          if (hs[u] >= kFinished) continue;
          const int j = hs[u] - first_node;
          const bool left = ks[u] < prefix[j] ||
                            (ks[u] == prefix[j] && (!need_ids[j] || (uint32_t)ids[t] <= id_prefix[j]));
          st[t] = left ? topo.ltag[hs[u]] : topo.rtag[hs[u]];
        }
      }
      __syncthreads();
    }
  }
  // stable partition by child label
  if (tid < C) {
    int off = 0;
    for (int c = 0; c < tid; ++c) off += caps[c];
    child_off[tid] = off;
    running[tid] = 0;
  }
  __syncthreads();
  const int label_base = kFinished;
  int32_t* out_next = idx_out + (int64_t)r * N + start;
  int32_t* out_leaf = perm + (int64_t)r * N + start;
  const unsigned lt = (1u << lane) - 1u;
  for (int c0 = 0; c0 < n; c0 += THREADS) {
    for (int c = lane; c < C; c += 32) warp_cnt[warp][c] = 0;
    __syncwarp();
    const int t = c0 + tid;
    const bool valid = t < n;
    const int label = valid ? st[t] - label_base : -1;
    const int id = valid ? ids[t] : 0;
    const unsigned peers = __match_any_sync(kFull, label);
    const int rank = __popc(peers & lt);
    if (valid && rank == 0) warp_cnt[warp][label] = __popc(peers);
    __syncthreads();
    if (tid < C) {
      int base = running[tid];
      for (int w = 0; w < (THREADS / 32); ++w) {
        warp_off[w][tid] = base;
        base += warp_cnt[w][tid];
      }
      running[tid] = base;
    }
    __syncthreads();
    if (valid) {
      const int dst = child_off[label] + warp_off[warp][label] + rank;
      (caps[label] == 64 ? out_leaf : out_next)[dst] = id;
    }
  }
  __syncthreads();
  if (tid < C && running[tid] != caps[tid] && status) atomicExch(status, 610);
}

// The root round's one node per row spread over a cluster of kRootCluster CTAs (the one-CTA
// kernel leaves most SMs idle there: one CTA per row).  Every CTA takes a contiguous slice of
// the node's tokens; the per-pass histograms of the slices are summed through distributed
// shared memory, and every CTA derives the same cut from the sum.  The stable partition
// offsets each CTA by the child counts of the lower-ranked slices, so keys, cuts and output
// order are those of reblock_route_kernel's radix path exactly.
constexpr int kRootCluster = 8;
constexpr int kClusterMaxNodes = 16;  // internal proxy nodes per depth: fanout up to 32

__global__ void __cluster_dims__(kRootCluster, 1, 1) __launch_bounds__(kRouteThreads)
    reblock_route_cluster_kernel(int N, int active, TreeLevel lv, const int32_t* __restrict__ idx_in,
                                 const float* __restrict__ scores, uint32_t* __restrict__ keys,
                                 uint8_t* __restrict__ state, int32_t* __restrict__ idx_out,
                                 int32_t* __restrict__ perm, int* __restrict__ status) {
  __shared__ __align__(16) int hist[kClusterMaxNodes][256];   // this CTA's slice
  __shared__ __align__(16) int total[kClusterMaxNodes][256];  // summed over the cluster
  __shared__ int target[kClusterMaxNodes], ties[kClusterMaxNodes], need_ids[kClusterMaxNodes];
  __shared__ uint32_t prefix[kClusterMaxNodes], id_prefix[kClusterMaxNodes];
  __shared__ int any_ids;
  __shared__ int warp_cnt[kRouteWarps][kMaxChildren];
  __shared__ int warp_off[kRouteWarps][kMaxChildren];
  __shared__ int running[kMaxChildren], child_off[kMaxChildren], slice_cnt[kMaxChildren];
  const uint32_t crank = cluster_ctarank();
  const int node = blockIdx.x / kRootCluster, r = blockIdx.y;
  const int32_t* tbl = lv.nodes + (int64_t)node * kNodeInts;
  const int start = tbl[0], n_node = tbl[1], C = tbl[2];
  const int32_t* caps = tbl + 4;
  const int chunk = (n_node + kRootCluster - 1) / kRootCluster;
  const int lo = min(n_node, (int)crank * chunk);
  const int n = min(n_node, lo + chunk) - lo;  // this CTA's slice: tokens [lo, lo + n) of the node
  const int32_t* ids = idx_in + (int64_t)r * N + start + lo;
  const float* sc = scores + ((int64_t)r * active + start + lo) * lv.S;
  uint32_t* key = keys + (int64_t)r * active + start + lo;
  uint8_t* st = state + (int64_t)r * active + start + lo;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // total = the sum of every slice's hist over the first `bins` bins.  The first barrier
  // publishes the slices' counts; the second keeps any CTA from clearing its counts for the
  // next pass while another still reads them.
  auto cluster_sum = [&](int bins) {
    cluster_sync_all();
    for (int e = tid; e < bins; e += kRouteThreads) {
      const uint32_t a = smem_u32(&hist[0][0] + e);
      int sum = 0;
#pragma unroll
      for (int k = 0; k < kRootCluster; ++k) sum += (int)ld_shared_cluster_u32(mapa_shared(a, (uint32_t)k));
      (&total[0][0])[e] = sum;
    }
    cluster_sync_all();
  };
  // The cut of every node of this depth from the summed histogram (one thread per node).
  auto pick = [&](int nd, int shift, uint32_t* pre, bool key_pass) {
    if (tid < nd && (key_pass || need_ids[tid])) {
      int cum = 0;
      const int want = target[tid];
      for (int bin = 0; bin < 256; ++bin) {
        const int c = total[tid][bin];
        if (cum + c >= want) {
          pre[tid] |= (uint32_t)bin << shift;
          target[tid] = want - cum;
          if (key_pass) ties[tid] = c;
          break;
        }
        cum += c;
      }
    }
    __syncthreads();
  };
  for (int t = tid; t < n; t += kRouteThreads) st[t] = 0;
  __syncthreads();
  int depth_nodes = 1, first_heap = 0, span = C;
  while (span > 1) {
    const int nd = depth_nodes;
    if (tid < nd) {
      const int s0 = tid * span, mid = s0 + span / 2;
      int lc = 0;
      for (int c = s0; c < mid; ++c) lc += caps[c];
      target[tid] = lc;
      prefix[tid] = 0;
      id_prefix[tid] = 0;
    }
    for (int t0 = tid; t0 < n; t0 += kUnroll * kRouteThreads) {
      int hs[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int t = t0 + u * kRouteThreads;
        hs[u] = t < n ? st[t] : 0;
      }
      float vs[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int t = t0 + u * kRouteThreads;
        vs[u] = t < n ? sc[(int64_t)t * lv.S + hs[u]] : 0.f;
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int t = t0 + u * kRouteThreads;
        if (t < n) key[t] = order_key(vs[u]);
      }
    }
    __syncthreads();
    // radix select on the score key, most significant byte first
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      for (int e = tid; e < nd * 256; e += kRouteThreads) hist[e >> 8][e & 255] = 0;
      __syncthreads();
      for (int t0 = tid; t0 < n; t0 += kUnroll * kRouteThreads) {
        uint32_t ks[kUnroll];
        int js[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int t = t0 + u * kRouteThreads;
          js[u] = t < n ? st[t] - first_heap : -1;
          ks[u] = t < n ? key[t] : 0u;
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int j = js[u];
          if (j >= 0 && (pass == 0 || (ks[u] >> (shift + 8)) == (prefix[j] >> (shift + 8))))
            atomicAdd(&hist[j][(ks[u] >> shift) & 255], 1);
        }
      }
      cluster_sum(nd * 256);
      pick(nd, shift, prefix, true);
    }
    if (tid == 0) {
      int any = 0;
      for (int j = 0; j < nd; ++j) {
        need_ids[j] = target[j] < ties[j] ? 1 : 0;
        any |= need_ids[j];
      }
      any_ids = any;
    }
    __syncthreads();
    if (any_ids) {  // the same in every CTA: it derives from the summed histograms
      // equal scores at the cut: the lowest token ids among them go left
      for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        for (int e = tid; e < nd * 256; e += kRouteThreads) hist[e >> 8][e & 255] = 0;
        __syncthreads();
        for (int t = tid; t < n; t += kRouteThreads) {
          const int j = st[t] - first_heap;
          if (!need_ids[j] || key[t] != prefix[j]) continue;
          const uint32_t id = (uint32_t)ids[t];
          if (pass == 0 || (id >> (shift + 8)) == (id_prefix[j] >> (shift + 8)))
            atomicAdd(&hist[j][(id >> shift) & 255], 1);
        }
        cluster_sum(nd * 256);
        pick(nd, shift, id_prefix, false);
      }
    }
    for (int t0 = tid; t0 < n; t0 += kUnroll * kRouteThreads) {
      int hs[kUnroll];
      uint32_t ks[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int t = t0 + u * kRouteThreads;
        hs[u] = t < n ? st[t] : 0;
        ks[u] = t < n ? key[t] : 0u;
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int t = t0 + u * kRouteThreads;
        if (t >= n) continue;
        const int j = hs[u] - first_heap;
        const bool left = ks[u] < prefix[j] ||
                          (ks[u] == prefix[j] && (!need_ids[j] || (uint32_t)ids[t] <= id_prefix[j]));
        st[t] = (uint8_t)(left ? 2 * hs[u] + 1 : 2 * hs[u] + 2);
      }
    }
    __syncthreads();
    first_heap += depth_nodes;
    depth_nodes *= 2;
    span /= 2;
  }
  // stable partition by child label; this slice starts after the lower-ranked slices' tokens
  // of each label
  const int label_base = C - 1;
  for (int c = tid; c < C; c += kRouteThreads) slice_cnt[c] = 0;
  __syncthreads();
  for (int w0 = tid - lane; w0 < n; w0 += kRouteThreads) {  // warp-uniform trip count
    const int t = w0 + lane;
    const int label = t < n ? st[t] - label_base : -1;
    const unsigned peers = __match_any_sync(kFull, label);
    if (label >= 0 && lane == __ffs(peers) - 1) atomicAdd(&slice_cnt[label], __popc(peers));
  }
  cluster_sync_all();
  if (tid < C) {
    int off = 0;
    for (int c = 0; c < tid; ++c) off += caps[c];
    child_off[tid] = off;
    const uint32_t a = smem_u32(&slice_cnt[tid]);
    int before = 0;
    for (uint32_t k = 0; k < crank; ++k) before += (int)ld_shared_cluster_u32(mapa_shared(a, k));
    running[tid] = before;
  }
  cluster_sync_all();  // no CTA reads slice_cnt any more; running and child_off are set
  int32_t* out_next = idx_out + (int64_t)r * N + start;
  int32_t* out_leaf = perm + (int64_t)r * N + start;
  const unsigned lt = (1u << lane) - 1u;
  for (int c0 = 0; c0 < n; c0 += kRouteThreads) {
    for (int c = lane; c < C; c += 32) warp_cnt[warp][c] = 0;
    __syncwarp();
    const int t = c0 + tid;
    const bool valid = t < n;
    const int label = valid ? st[t] - label_base : -1;
    const int id = valid ? ids[t] : 0;
    const unsigned peers = __match_any_sync(kFull, label);
    const int rnk = __popc(peers & lt);
    if (valid && rnk == 0) warp_cnt[warp][label] = __popc(peers);
    __syncthreads();
    if (tid < C) {
      int base = running[tid];
      for (int w = 0; w < kRouteWarps; ++w) {
        warp_off[w][tid] = base;
        base += warp_cnt[w][tid];
      }
      running[tid] = base;
    }
    __syncthreads();
    if (valid) {
      const int dst = child_off[label] + warp_off[warp][label] + rnk;
      (caps[label] == 64 ? out_leaf : out_next)[dst] = id;
    }
  }
  __syncthreads();
  // the last slice ends every child: its running counts are the whole node's
  if (crank == kRootCluster - 1 && tid < C && running[tid] != caps[tid] && status) atomicExch(status, 610);
}

__global__ void reblock_inverse_kernel(const int32_t* __restrict__ perm, int N, int64_t total,
                                       int32_t* __restrict__ inverse) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int64_t r = i / N;
  const int32_t p = perm[i];
  // a malformed caller tail (status 612) can leave positions of perm unwritten
  if (p >= 0 && p < N) inverse[r * N + p] = (int32_t)(i - r * N);
}

// ----------------------------------------------------------------- host helpers
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

// {H*D, T, B} bf16 map, 64 x 64 box, 128-byte swizzle.
int make_bthd_map(CUtensorMap* map, const void* base, int B, int T, int H) {
  EncodeTiledFn encode = encode_fn();
  if (encode == nullptr) {
    set_error("sb_reblock_transform: cuTensorMapEncodeTiled is unavailable");
    return SB_ERR_CUDA;
  }
  const uint64_t HD = (uint64_t)H * kDim;
  const cuuint64_t dims[3] = {HD, (cuuint64_t)T, (cuuint64_t)B};
  const cuuint64_t strides[2] = {HD * 2, HD * 2 * (uint64_t)T};
  const cuuint32_t box[3] = {64, 64, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult res = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS) {
    set_error("sb_reblock_transform: cuTensorMapEncodeTiled failed (CUresult %d)", (int)res);
    return SB_ERR_CUDA;
  }
  return SB_OK;
}

// Features [rows, video, 128] bf16 as a store target: boxes of 64 columns x 32 rows, 128-byte
// swizzle (one epilogue warp's rows of one 64-column half).
int make_features_map(CUtensorMap* map, void* base, int rows, int video) {
  EncodeTiledFn encode = encode_fn();
  if (encode == nullptr) {
    set_error("sb_reblock_transform: cuTensorMapEncodeTiled is unavailable");
    return SB_ERR_CUDA;
  }
  const cuuint64_t dims[3] = {(cuuint64_t)kDim, (cuuint64_t)video, (cuuint64_t)rows};
  const cuuint64_t strides[2] = {(cuuint64_t)kDim * 2, (cuuint64_t)kDim * 2 * (uint64_t)video};
  const cuuint32_t box[3] = {64, 32, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult res = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS) {
    set_error("sb_reblock_transform: cuTensorMapEncodeTiled (features) failed (CUresult %d)", (int)res);
    return SB_ERR_CUDA;
  }
  return SB_OK;
}

int sm_count() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

struct WorkspaceLayout {
  size_t idx, scores, dirs, keys, state, total;
};

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

WorkspaceLayout workspace_layout(const int32_t* plan, int rows) {
  const int64_t N = plan[1], A = plan[2], max_nodes = plan[3], max_s = std::max(1, plan[4] - 1);
  WorkspaceLayout w{};
  size_t off = 0;
  w.idx = off;
  off = align256(off + 2 * sizeof(int32_t) * (size_t)rows * N);
  w.scores = off;
  off = align256(off + sizeof(float) * (size_t)rows * A * max_s);
  w.dirs = off;
  off = align256(off + sizeof(float) * (size_t)rows * std::max<int64_t>(max_nodes, 1) * max_s * kDim);
  w.keys = off;
  off = align256(off + sizeof(uint32_t) * (size_t)rows * std::max(N, A));
  w.state = off;
  off = align256(off + (size_t)rows * A);
  w.total = off;
  return w;
}

}  // namespace
}  // namespace sb

using namespace sb;

extern "C" int sb_reblock_metric(const void* q, const void* k, int dtype, int B, int T, int H, int D,
                                 const int32_t* samples, int num_samples, float ridge, float* factors, void* stream) {
  SB_CHECK_ARG(q && k && samples && factors, "sb_reblock_metric: null pointer");
  SB_CHECK_ARG(dtype == SB_F32 || dtype == SB_BF16, "sb_reblock_metric: bad dtype");
  SB_CHECK_ARG(D == kDim, "sb_reblock_metric: head dimension must be 128, got %d", D);
  SB_CHECK_ARG(B > 0 && T > 0 && H > 0 && num_samples > 0, "sb_reblock_metric: empty input");
  SB_CHECK_ARG(ridge >= 0.f, "sb_reblock_metric: ridge must be non-negative");
  cudaStream_t s = (cudaStream_t)stream;
  const int BH = B * H;
  dim3 grid(kDim / 16, 2 * BH);
  if (dtype == SB_BF16)
    metric_moment_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>((const __nv_bfloat16*)q, (const __nv_bfloat16*)k, T, H,
                                                             BH, samples, num_samples, factors);
  else
    metric_moment_kernel<float><<<grid, 256, 0, s>>>((const float*)q, (const float*)k, T, H, BH, samples, num_samples,
                                                     factors);
  SB_CHECK_LAUNCH("sb_reblock_metric: moments");
  const int smem = kDim * (kDim + 1) * (int)sizeof(float);
  cudaError_t err = cudaFuncSetAttribute(cholesky_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (err != cudaSuccess) return cuda_error(err, "sb_reblock_metric: set smem");
  cholesky_kernel<<<2 * BH, 256, smem, s>>>(factors, ridge);
  SB_CHECK_LAUNCH("sb_reblock_metric: cholesky");
  return SB_OK;
}

// Splits of each row's token tiles across CTAs, chosen so the rows x splits CTAs fill whole
// waves of the resident slots (two CTAs per SM): with 64 rows on 296 slots, 5 splits (320
// CTAs) leave 24 CTAs running alone in a second wave, while 37 splits make exactly 8 waves.
// Among splits that give every CTA at least 8 tiles, the one with the least idle slot time
// wins (ties: fewer splits).
static int transform_splits(int tiles, int rows, int slots) {
  int best = 1;
  double best_eff = 0.0;
  const int max_splits = std::max(1, tiles / 8);
  for (int sp = 1; sp <= max_splits; ++sp) {
    const int64_t ctas = (int64_t)rows * sp;
    const int64_t waves = (ctas + slots - 1) / slots;
    const double eff = (double)ctas / (double)(waves * slots);
    if (eff > best_eff + 1e-9) {
      best_eff = eff;
      best = sp;
    }
    if (eff >= 0.999) break;
  }
  return best;
}

extern "C" int sb_reblock_transform(const void* q, const void* k, int B, int T, int H, int D, int video_tokens,
                                    const float* factors, void* features, void* stream) {
  SB_CHECK_ARG(q && k && factors && features, "sb_reblock_transform: null pointer");
  SB_CHECK_ARG(D == kDim, "sb_reblock_transform: head dimension must be 128, got %d", D);
  SB_CHECK_ARG(B > 0 && H > 0 && video_tokens > 0 && video_tokens <= T, "sb_reblock_transform: bad shape");
  SB_CHECK_ARG(((uintptr_t)q % 16) == 0 && ((uintptr_t)k % 16) == 0 && ((uintptr_t)features % 16) == 0,
               "sb_reblock_transform: tensors must be 16-byte aligned");
  int* status = device_status_ptr();
  if (status == nullptr) return cuda_error(cudaGetLastError(), "sb_reblock_transform: status word");
  CUtensorMap mk, mq, mo;
  int rc;
  if ((rc = make_bthd_map(&mk, k, B, T, H)) != SB_OK) return rc;
  if ((rc = make_bthd_map(&mq, q, B, T, H)) != SB_OK) return rc;
  if ((rc = make_features_map(&mo, features, 2 * B * H, video_tokens)) != SB_OK) return rc;
  TfParams p{};
  p.factors = factors;
  p.features = static_cast<__nv_bfloat16*>(features);
  p.status = status;
  p.T = T;
  p.H = H;
  p.BH = B * H;
  p.video = video_tokens;
  p.tiles = ceil_div(video_tokens, 128);
  const int rows = 2 * p.BH;
  p.splits = transform_splits(p.tiles, rows, sm_count());  // one CTA per SM
  const size_t smem = (size_t)(1 + kTfStages) * kTfTileBytes + kTfOutBytes + sizeof(TfControl);
  cudaError_t err = cudaFuncSetAttribute(reblock_transform_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
  if (err != cudaSuccess) return cuda_error(err, "sb_reblock_transform: set smem");
  reblock_transform_kernel<<<dim3(p.splits, rows), kTfThreads, smem, (cudaStream_t)stream>>>(mk, mq, mo, p);
  SB_CHECK_LAUNCH("sb_reblock_transform launch");
  return SB_OK;
}

extern "C" int64_t sb_reblock_plan(const int32_t* schedule, int schedule_len, int tokens, int32_t* plan,
                                   int64_t capacity) {
  SB_CHECK_ARG(schedule && schedule_len > 0, "sb_reblock_plan: empty schedule");
  SB_CHECK_ARG(tokens >= 64, "sb_reblock_plan: at least 64 tokens are required, got %d", tokens);
  const int active = tokens - tokens % 64;
  const int tiles = active / 64;
  struct Seg {
    int start, leaves;
  };
  std::vector<Seg> segs{{0, tiles}};
  std::vector<std::vector<int32_t>> level_nodes;
  std::vector<int> level_P;
  const int levels = schedule[0];
  int pos = 1;
  for (int level = 0; level < levels; ++level) {
    SB_CHECK_ARG(pos < schedule_len, "sb_reblock_plan: schedule truncated");
    const int entries = schedule[pos];
    const int level_pos = pos + 1;
    int p = level_pos;
    for (int e = 0; e < entries; ++e) {
      SB_CHECK_ARG(p + 1 < schedule_len, "sb_reblock_plan: schedule truncated");
      p += 2 + schedule[p + 1];
    }
    SB_CHECK_ARG(p <= schedule_len, "sb_reblock_plan: schedule truncated");
    pos = p;
    std::vector<Seg> next;
    std::vector<int32_t> nodes;
    int maxC = 2;
    for (const Seg& sg : segs) {
      if (sg.leaves <= 1) continue;
      int q = level_pos, found = -1;
      for (int e = 0; e < entries; ++e) {
        if (schedule[q] == sg.leaves) {
          found = q;
          break;
        }
        q += 2 + schedule[q + 1];
      }
      SB_CHECK_ARG(found >= 0, "sb_reblock_plan: no budget for a node of %d leaves at round %d", sg.leaves, level);
      const int C = schedule[found + 1];
      SB_CHECK_ARG(C >= 2 && C <= kMaxChildren, "sb_reblock_plan: the CUDA tree takes 2 to 64 children, got %d", C);
      std::vector<int32_t> rec(kNodeInts, 0);
      rec[0] = sg.start * 64;
      rec[1] = sg.leaves * 64;
      rec[2] = C;
      int off = sg.start, sum = 0;
      for (int c = 0; c < C; ++c) {
        const int budget = schedule[found + 2 + c];
        SB_CHECK_ARG(budget >= 1, "sb_reblock_plan: empty child");
        rec[4 + c] = 64 * budget;
        next.push_back({off, budget});
        off += budget;
        sum += budget;
      }
      SB_CHECK_ARG(sum == sg.leaves, "sb_reblock_plan: child budgets do not cover the node");
      nodes.insert(nodes.end(), rec.begin(), rec.end());
      maxC = std::max(maxC, C);
    }
    for (const Seg& sg : segs)
      if (sg.leaves <= 1) next.push_back(sg);
    std::sort(next.begin(), next.end(), [](const Seg& a, const Seg& b) { return a.start < b.start; });
    segs.swap(next);
    if (!nodes.empty()) {
      // kernels are instantiated per power-of-two fanout; a level runs with the smallest one
      // that holds its largest node (the score kernels store only a node's C - 1 scores)
      int P = 2;
      while (P < maxC) P *= 2;
      level_nodes.push_back(std::move(nodes));
      level_P.push_back(P);
    }
  }
  for (const Seg& sg : segs)
    SB_CHECK_ARG(sg.leaves == 1, "sb_reblock_plan: the schedule ends before every node is a leaf");
  const int L = (int)level_nodes.size();
  int64_t length = kPlanHeader + (int64_t)kLevelInts * L;
  int max_nodes = 0, maxP = 2;
  for (int l = 0; l < L; ++l) {
    length += (int64_t)level_nodes[l].size() + tiles;
    max_nodes = std::max(max_nodes, (int)(level_nodes[l].size() / kNodeInts));
    maxP = std::max(maxP, level_P[l]);
  }
  if (plan == nullptr) return length;
  SB_CHECK_ARG(capacity >= length, "sb_reblock_plan: plan buffer holds %lld ints, %lld needed", (long long)capacity,
               (long long)length);
  std::fill(plan, plan + length, 0);
  plan[0] = L;
  plan[1] = tokens;
  plan[2] = active;
  plan[3] = max_nodes;
  plan[4] = maxP;
  plan[5] = (int32_t)length;
  plan[6] = 2;  // proxy controls (sb_reblock_plan_proxy): two mean updates from the farthest pair
  plan[7] = 0;
  int64_t off = kPlanHeader + (int64_t)kLevelInts * L;
  for (int l = 0; l < L; ++l) {
    int32_t* lv = plan + kPlanHeader + kLevelInts * l;
    const int count = (int)(level_nodes[l].size() / kNodeInts);
    lv[0] = count;
    lv[1] = (int32_t)off;
    std::copy(level_nodes[l].begin(), level_nodes[l].end(), plan + off);
    off += (int64_t)level_nodes[l].size();
    lv[2] = (int32_t)off;
    int32_t* tile_tbl = plan + off;
    std::fill(tile_tbl, tile_tbl + tiles, -1);
    for (int j = 0; j < count; ++j) {
      const int32_t* rec = plan + lv[1] + (int64_t)j * kNodeInts;
      for (int t = rec[0] / 64; t < (rec[0] + rec[1]) / 64; ++t) tile_tbl[t] = j;
    }
    off += tiles;
    lv[3] = level_P[l];
    lv[4] = level_P[l] - 1;
  }
  return length;
}

extern "C" int sb_reblock_plan_proxy(int32_t* plan, int proxy_iterations, int endpoint_seeds) {
  SB_CHECK_ARG(plan != nullptr, "sb_reblock_plan_proxy: null plan");
  SB_CHECK_ARG(proxy_iterations == 0 || proxy_iterations == 1 || proxy_iterations == 2 || proxy_iterations == 4,
               "sb_reblock_plan_proxy: proxy_iterations must be 0, 1, 2, or 4, got %d", proxy_iterations);
  SB_CHECK_ARG(endpoint_seeds == 0 || endpoint_seeds == 1,
               "sb_reblock_plan_proxy: endpoint_seeds must be 0 (farthest_pair) or 1 (endpoint_order)");
  plan[6] = proxy_iterations;
  plan[7] = endpoint_seeds;
  return SB_OK;
}

using ProxyKernel = void (*)(const __nv_bfloat16*, int, int, TreeLevel, const int32_t*, float*);

// The proxy kernel for the plan's controls (validated by the caller).
static ProxyKernel proxy_kernel_for(int iterations, int endpoint_seeds) {
  switch (iterations * 2 + endpoint_seeds) {
    case 0: return reblock_proxy_kernel<0, false>;
    case 1: return reblock_proxy_kernel<0, true>;
    case 2: return reblock_proxy_kernel<1, false>;
    case 3: return reblock_proxy_kernel<1, true>;
    case 5: return reblock_proxy_kernel<2, true>;
    case 8: return reblock_proxy_kernel<4, false>;
    case 9: return reblock_proxy_kernel<4, true>;
    default: return reblock_proxy_kernel<2, false>;
  }
}

// The largest node of a plan level (lh: the level's header in the plan).
static int level_max_tokens(const int32_t* plan, const int32_t* lh) {
  int most = 0;
  for (int j = 0; j < lh[0]; ++j) most = std::max(most, plan[lh[1] + (int64_t)j * kNodeInts + 1]);
  return most;
}

extern "C" int64_t sb_reblock_workspace_bytes(const int32_t* plan, int rows) {
  SB_CHECK_ARG(plan && rows > 0, "sb_reblock_workspace_bytes: bad arguments");
  return (int64_t)workspace_layout(plan, rows).total;
}

// The tree's CUDA errors name the entry point the caller used.
static int tree_cuda_error(cudaError_t err, const char* who, const char* what) {
  char buf[160];
  snprintf(buf, sizeof(buf), "%s: %s", who, what);
  return cuda_error(err, buf);
}
#define TREE_CHECK_LAUNCH(who, what)                                     \
  do {                                                                   \
    cudaError_t err__ = cudaGetLastError();                              \
    if (err__ != cudaSuccess) return tree_cuda_error(err__, who, what);  \
  } while (0)

static int reblock_tree(const char* who, const void* features, int rows, int tokens, int D, const int32_t* root_order,
                        const int32_t* frozen, const int32_t* plan_host, const int32_t* plan_device, void* workspace,
                        int64_t workspace_bytes, int32_t* perm, int32_t* inverse, void* stream) {
  SB_CHECK_ARG(features && plan_host && plan_device && workspace && perm && inverse, "%s: null pointer", who);
  SB_CHECK_ARG(D == kDim, "%s: feature dimension must be 128, got %d", who, D);
  SB_CHECK_ARG(rows > 0 && rows < 65536, "%s: rows must lie in [1, 65535]", who);
  SB_CHECK_ARG(plan_host[1] == tokens, "%s: the plan was built for %d tokens, not %d", who, plan_host[1],
               tokens);
  SB_CHECK_ARG(tokens < (1 << 25), "%s: at most 2^25 - 1 tokens per row", who);
  SB_CHECK_ARG(((uintptr_t)features % 16) == 0 && ((uintptr_t)workspace % 256) == 0,
               "%s: features must be 16-byte and the workspace 256-byte aligned", who);
  SB_CHECK_ARG((plan_host[6] == 0 || plan_host[6] == 1 || plan_host[6] == 2 || plan_host[6] == 4) &&
                   (plan_host[7] == 0 || plan_host[7] == 1),
               "%s: the plan's proxy controls are invalid", who);
  const WorkspaceLayout W = workspace_layout(plan_host, rows);
  SB_CHECK_ARG((size_t)workspace_bytes >= W.total, "%s: workspace holds %lld bytes, %zu needed", who,
               (long long)workspace_bytes, W.total);
  int* status = device_status_ptr();
  if (status == nullptr) return tree_cuda_error(cudaGetLastError(), who, "status word");
  cudaStream_t s = (cudaStream_t)stream;
  const __nv_bfloat16* F = static_cast<const __nv_bfloat16*>(features);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int32_t* idx[2] = {reinterpret_cast<int32_t*>(ws + W.idx),
                     reinterpret_cast<int32_t*>(ws + W.idx) + (size_t)rows * tokens};
  float* scores = reinterpret_cast<float*>(ws + W.scores);
  float* dirs = reinterpret_cast<float*>(ws + W.dirs);
  uint32_t* keys = reinterpret_cast<uint32_t*>(ws + W.keys);
  uint8_t* state = ws + W.state;
  const int L = plan_host[0], active = plan_host[2];
  reblock_root_kernel<<<rows, 1024, 0, s>>>(F, tokens, active, root_order, frozen, reinterpret_cast<float*>(keys),
                                            idx[0], perm, L == 0 ? 1 : 0, status);
  TREE_CHECK_LAUNCH(who, "root");
  const ProxyKernel proxy_kernel = proxy_kernel_for(plan_host[6], plan_host[7]);
  cudaError_t err = cudaFuncSetAttribute(proxy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)proxy_smem_bytes(kMaxChildren));
  if (err != cudaSuccess) return tree_cuda_error(err, who, "set smem");
  for (const void* fn : {(const void*)reblock_score3_kernel<2>, (const void*)reblock_score3_kernel<4>,
                         (const void*)reblock_score3_kernel<8>, (const void*)reblock_score3_kernel<16>}) {
    err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kScoreRingBytes);
    if (err != cudaSuccess) return tree_cuda_error(err, who, "set smem");
  }
  int cur = 0;
  for (int l = 0; l < L; ++l) {
    const int32_t* lh = plan_host + kPlanHeader + kLevelInts * l;
    TreeLevel lv{plan_device + lh[1], plan_device + lh[2], lh[0], lh[3], lh[4]};
    proxy_kernel<<<dim3(lv.count, rows), kProxyThreads, proxy_smem_bytes(lv.P), s>>>(F, tokens, active, lv, idx[cur],
                                                                                      dirs);
    TREE_CHECK_LAUNCH(who, "proxy");
    const dim3 sgrid(ceil_div(active / 64, kScoreTiles), rows);
    switch (lv.P) {
      case 2: reblock_score3_kernel<2><<<sgrid, 128, kScoreRingBytes, s>>>(F, tokens, active, lv, idx[cur], dirs,
                                                                            scores); break;
      case 4: reblock_score3_kernel<4><<<sgrid, 128, kScoreRingBytes, s>>>(F, tokens, active, lv, idx[cur], dirs,
                                                                            scores); break;
      case 8: reblock_score3_kernel<8><<<sgrid, 128, kScoreRingBytes, s>>>(F, tokens, active, lv, idx[cur], dirs,
                                                                            scores); break;
      case 16: reblock_score3_kernel<16><<<sgrid, 128, kScoreRingBytes, s>>>(F, tokens, active, lv, idx[cur], dirs,
                                                                              scores); break;
      case 32: reblock_score_kernel<32><<<sgrid, 256, 0, s>>>(F, tokens, active, lv, idx[cur], dirs, scores); break;
      case 64: reblock_score_kernel<64><<<sgrid, 256, 0, s>>>(F, tokens, active, lv, idx[cur], dirs, scores); break;
      default: set_error("%s: bad plan fanout %d", who, lv.P); return SB_ERR_INVALID;
    }
    TREE_CHECK_LAUNCH(who, "scores");
    const int32_t* first = plan_host + lh[1];  // the level's first node record (start, tokens, children)
    // the cluster form walks the heap of a power-of-two fanout; other roots take the radix form
    if (lv.count == 1 && first[1] > kSortMax && first[2] <= 2 * kClusterMaxNodes && (first[2] & (first[2] - 1)) == 0)
      reblock_route_cluster_kernel<<<dim3(kRootCluster, rows), kRouteThreads, 0, s>>>(
          tokens, active, lv, idx[cur], scores, keys, state, idx[cur ^ 1], perm, status);
    else if (level_max_tokens(plan_host, lh) <= kSortMax)  // every node sorts: 128-thread CTAs
      reblock_route_kernel<128, false><<<dim3(lv.count, rows), 128, 0, s>>>(tokens, active, lv, idx[cur], scores,
                                                                            keys, state, idx[cur ^ 1], perm, status);
    else
      reblock_route_kernel<kRouteThreads, true><<<dim3(lv.count, rows), kRouteThreads, 0, s>>>(
          tokens, active, lv, idx[cur], scores, keys, state, idx[cur ^ 1], perm, status);
    TREE_CHECK_LAUNCH(who, "route");
    cur ^= 1;
  }
  const int64_t total = (int64_t)rows * tokens;
  reblock_inverse_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(perm, tokens, total, inverse);
  TREE_CHECK_LAUNCH(who, "inverse");
  return SB_OK;
}

extern "C" int sb_reblock_tree(const void* features, int rows, int tokens, int D, const int32_t* root_order,
                               const int32_t* plan_host, const int32_t* plan_device, void* workspace,
                               int64_t workspace_bytes, int32_t* perm, int32_t* inverse, void* stream) {
  return reblock_tree("sb_reblock_tree", features, rows, tokens, D, root_order, nullptr, plan_host, plan_device,
                      workspace, workspace_bytes, perm, inverse, stream);
}

extern "C" int sb_reblock_tree_frozen(const void* features, int rows, int tokens, int D, const int32_t* root_order,
                                      const int32_t* excluded, const int32_t* plan_host, const int32_t* plan_device,
                                      void* workspace, int64_t workspace_bytes, int32_t* perm, int32_t* inverse,
                                      void* stream) {
  SB_CHECK_ARG(excluded != nullptr || tokens % 64 == 0,
               "sb_reblock_tree_frozen: excluded ids are required for the %d remainder tokens", tokens % 64);
  return reblock_tree("sb_reblock_tree_frozen", features, rows, tokens, D, root_order, excluded, plan_host,
                      plan_device, workspace, workspace_bytes, perm, inverse, stream);
}

extern "C" int sb_reblock_remainder(const void* features, int rows, int tokens, int D, void* workspace,
                                    int64_t workspace_bytes, int32_t* excluded, void* stream) {
  const char* who = "sb_reblock_remainder";
  SB_CHECK_ARG(features && workspace, "%s: null pointer", who);
  SB_CHECK_ARG(D == kDim, "%s: feature dimension must be 128, got %d", who, D);
  SB_CHECK_ARG(rows > 0 && rows < 65536, "%s: rows must lie in [1, 65535]", who);
  SB_CHECK_ARG(tokens >= 64 && tokens < (1 << 25), "%s: tokens must lie in [64, 2^25)", who);
  SB_CHECK_ARG(((uintptr_t)features % 16) == 0 && ((uintptr_t)workspace % 256) == 0,
               "%s: features must be 16-byte and the workspace 256-byte aligned", who);
  SB_CHECK_ARG(workspace_bytes >= 8 * (int64_t)rows * tokens, "%s: workspace holds %lld bytes, %lld needed", who,
               (long long)workspace_bytes, 8ll * rows * tokens);
  const int rem = tokens % 64, active = tokens - rem;
  if (rem == 0) return SB_OK;
  SB_CHECK_ARG(excluded != nullptr, "%s: null excluded buffer for %d remainder tokens", who, rem);
  int* status = device_status_ptr();
  if (status == nullptr) return tree_cuda_error(cudaGetLastError(), who, "status word");
  cudaStream_t s = (cudaStream_t)stream;
  float* norms = static_cast<float*>(workspace);
  int32_t* order = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(workspace) + 4 * (size_t)rows * tokens);
  // The root kernel in its direct form over the flat order: the tail of each row of `order`
  // holds the remainder in ascending id order.
  reblock_root_kernel<<<rows, 1024, 0, s>>>(static_cast<const __nv_bfloat16*>(features), tokens, active, nullptr,
                                            nullptr, norms, order, order, 1, status);
  TREE_CHECK_LAUNCH(who, "root");
  const cudaError_t err = cudaMemcpy2DAsync(excluded, sizeof(int32_t) * rem, order + active,
                                            sizeof(int32_t) * tokens, sizeof(int32_t) * rem, rows,
                                            cudaMemcpyDeviceToDevice, s);
  if (err != cudaSuccess) return tree_cuda_error(err, who, "copy");
  return SB_OK;
}
