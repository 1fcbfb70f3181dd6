// Block scores (pooled Q . pooled K) and exact per-row Top-K with the lowest-index
// tie rule, emitting the packed int32 route and ascending block indices.
//
// score = fp32(sequential fused multiply-add over d of qc[d] * kc[d]) * scale_log2.
// The CPU oracle computes the identical chain, so selections agree bit for bit.
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace sb {

constexpr int kScoreTile = 64;  // query blocks x key blocks per CTA
constexpr int kScoreThreads = 256;

// grid (ceil(C/64), ceil(QB/64), B*H).  Thread (ty, tx) computes 4x4 scores:
// query rows ty + 16*i and key columns tx + 16*j.
template <typename TK, int D>
__global__ void __launch_bounds__(kScoreThreads)
block_scores_kernel(const float* __restrict__ qc, const TK* __restrict__ kc, int QB, int NB, int H,
                    int C, float scale_log2, float* __restrict__ scores) {
  extern __shared__ float score_smem[];
  float (*sq)[D + 1] = reinterpret_cast<float (*)[D + 1]>(score_smem);
  float (*sk)[kScoreTile + 1] = reinterpret_cast<float (*)[kScoreTile + 1]>(score_smem + kScoreTile * (D + 1));
  const int bh = blockIdx.z, b = bh / H, h = bh % H;
  const int q0 = blockIdx.y * kScoreTile, c0 = blockIdx.x * kScoreTile;
  const int tid = threadIdx.x;
  for (int idx = tid; idx < kScoreTile * D; idx += kScoreThreads) {
    const int r = idx / D, d = idx % D;
    const int qi = q0 + r, ci = c0 + r;
    sq[r][d] = qi < QB ? qc[(((int64_t)b * NB + qi) * H + h) * D + d] : 0.f;
    sk[d][r] = ci < C ? Elem<TK>::to_f(kc[(((int64_t)b * NB + ci) * H + h) * D + d]) : 0.f;
  }
  __syncthreads();
  const int tx = tid % 16, ty = tid / 16;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
#pragma unroll 4
  for (int d = 0; d < D; ++d) {
    float a[4], w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) a[i] = sq[ty + 16 * i][d];
#pragma unroll
    for (int j = 0; j < 4; ++j) w[j] = sk[d][tx + 16 * j];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = __fmaf_rn(a[i], w[j], acc[i][j]);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int qi = q0 + ty + 16 * i;
    if (qi >= QB) continue;
    float* row = scores + (((int64_t)b * QB + qi) * H + h) * C;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int ci = c0 + tx + 16 * j;
      if (ci < C) row[ci] = __fmul_rn(acc[i][j], scale_log2);
    }
  }
}

// Order-preserving map from fp32 to uint32 (larger float -> larger key).
__device__ __forceinline__ uint32_t float_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr int kTopkThreads = 256;

// One CTA per (b, query block, head) row.  Radix select (4 x 8 bits) finds the key of
// the topk-th largest score; every score above it is kept, and of the scores equal to
// it the lowest-index ones fill the remaining slots.
__global__ void __launch_bounds__(kTopkThreads)
topk_rows_kernel(const float* __restrict__ scores, int C, int topk, int words,
                 int32_t* __restrict__ packed, int32_t* __restrict__ indices) {
  extern __shared__ uint32_t keys[];  // [C]
  __shared__ uint32_t hist[256];
  __shared__ uint32_t sel_prefix, sel_need;
  __shared__ uint32_t route_words[256];
  __shared__ int warp_counts[kTopkThreads / 32];
  __shared__ int eq_base;
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* src = scores + row * C;
  for (int i = tid; i < C; i += kTopkThreads) keys[i] = float_key(src[i]);
  if (tid == 0) {
    sel_prefix = 0;
    sel_need = (uint32_t)topk;
  }
  __syncthreads();

  // Radix select from the most significant byte.
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    const uint32_t mask_hi = pass == 0 ? 0u : (0xffffffffu << (32 - 8 * pass));
    for (int i = tid; i < 256; i += kTopkThreads) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = sel_prefix;
    for (int i = tid; i < C; i += kTopkThreads) {
      const uint32_t kk = keys[i];
      if ((kk & mask_hi) == prefix) atomicAdd(&hist[(kk >> shift) & 0xff], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      uint32_t need = sel_need, above = 0;
      int digit = 255;
      for (; digit > 0; --digit) {
        if (above + hist[digit] >= need) break;
        above += hist[digit];
      }
      sel_prefix = prefix | ((uint32_t)digit << shift);
      sel_need = need - above;
    }
    __syncthreads();
  }
  const uint32_t thresh = sel_prefix;
  const uint32_t take_equal = sel_need;  // how many entries equal to thresh to keep

  // Exclusive scan of "equal to thresh" flags in index order gives the lowest-index rule;
  // a second scan of the final selection writes ascending indices.
  for (int i = tid; i < words; i += kTopkThreads) route_words[i] = 0;
  if (tid == 0) eq_base = 0;
  __syncthreads();
  int out_base = 0;
  for (int start = 0; start < C; start += kTopkThreads) {
    const int i = start + tid;
    const uint32_t kk = i < C ? keys[i] : 0u;
    const bool eq = i < C && kk == thresh;
    const unsigned eq_mask = __ballot_sync(0xffffffffu, eq);
    if (lane == 0) warp_counts[warp] = __popc(eq_mask);
    __syncthreads();
    int eq_before = eq_base;
    for (int w = 0; w < warp; ++w) eq_before += warp_counts[w];
    eq_before += __popc(eq_mask & ((1u << lane) - 1u));
    const bool sel = i < C && (kk > thresh || (eq && (uint32_t)eq_before < take_equal));
    __syncthreads();
    if (tid == 0) {
      int tot = 0;
      for (int w = 0; w < kTopkThreads / 32; ++w) tot += warp_counts[w];
      eq_base += tot;
    }
    const unsigned sel_mask = __ballot_sync(0xffffffffu, sel);
    __syncthreads();
    if (lane == 0) warp_counts[warp] = __popc(sel_mask);
    __syncthreads();
    int pos = out_base;
    for (int w = 0; w < warp; ++w) pos += warp_counts[w];
    pos += __popc(sel_mask & ((1u << lane) - 1u));
    if (sel) {
      atomicOr(&route_words[i >> 5], 1u << (i & 31));
      if (indices != nullptr && pos < topk) indices[row * topk + pos] = i;
    }
    for (int w = 0; w < kTopkThreads / 32; ++w) out_base += warp_counts[w];
    __syncthreads();
  }
  for (int i = tid; i < words; i += kTopkThreads) packed[row * words + i] = (int32_t)route_words[i];
}

}  // namespace sb

using namespace sb;

template <typename TK, int D>
static int launch_scores(dim3 grid, const float* qc, const void* kc, int QB, int NB, int H, int C,
                         float scale_log2, float* scores, cudaStream_t s) {
  const size_t smem = (size_t)(kScoreTile * (D + 1) + D * (kScoreTile + 1)) * sizeof(float);
  auto kern = block_scores_kernel<TK, D>;
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return cuda_error(err, "sb_route_topk: set score smem");
  kern<<<grid, kScoreThreads, smem, s>>>(qc, (const TK*)kc, QB, NB, H, C, scale_log2, scores);
  SB_CHECK_LAUNCH("sb_route_topk: score launch");
  return SB_OK;
}

extern "C" int64_t sb_route_workspace_bytes(int B, int QB, int H, int candidates) {
  if (B <= 0 || QB <= 0 || H <= 0 || candidates <= 0) return 0;
  return (int64_t)B * QB * H * candidates * (int64_t)sizeof(float);
}

extern "C" int sb_route_topk(const float* qc, const void* kc, int kc_dtype, int B, int QB, int NB,
                             int H, int D, int candidates, int topk, float scale_log2,
                             void* workspace, int32_t* packed_route, int32_t* indices,
                             void* stream) {
  SB_CHECK_ARG(qc && kc && workspace && packed_route, "sb_route_topk: null pointer");
  SB_CHECK_ARG(kc_dtype == SB_F32 || kc_dtype == SB_BF16, "sb_route_topk: bad key-centroid dtype");
  SB_CHECK_ARG(B > 0 && QB > 0 && NB > 0 && H > 0, "sb_route_topk: sizes must be positive");
  SB_CHECK_ARG(QB <= NB, "sb_route_topk: QB (%d) exceeds NB (%d)", QB, NB);
  SB_CHECK_ARG(D == 64 || D == 128, "sb_route_topk: head dim must be 64 or 128");
  SB_CHECK_ARG(candidates >= 1 && candidates <= NB,
               "sb_route_topk: candidates must lie in [1, NB], got %d", candidates);
  SB_CHECK_ARG(topk >= 1 && topk <= candidates, "sb_route_topk: topk must lie in [1, candidates], got %d", topk);
  const int words = ceil_div(NB, 32);
  SB_CHECK_ARG(words <= 256, "sb_route_topk: at most 8192 key blocks are supported");
  const size_t key_smem = (size_t)candidates * sizeof(uint32_t);
  SB_CHECK_ARG(key_smem <= 200 * 1024, "sb_route_topk: too many candidate blocks (%d)", candidates);
  cudaStream_t s = (cudaStream_t)stream;
  float* scores = (float*)workspace;
  dim3 grid(ceil_div(candidates, kScoreTile), ceil_div(QB, kScoreTile), B * H);
  int rc = SB_OK;
  if (kc_dtype == SB_BF16)
    rc = D == 128 ? launch_scores<__nv_bfloat16, 128>(grid, qc, kc, QB, NB, H, candidates, scale_log2, scores, s)
                  : launch_scores<__nv_bfloat16, 64>(grid, qc, kc, QB, NB, H, candidates, scale_log2, scores, s);
  else
    rc = D == 128 ? launch_scores<float, 128>(grid, qc, kc, QB, NB, H, candidates, scale_log2, scores, s)
                  : launch_scores<float, 64>(grid, qc, kc, QB, NB, H, candidates, scale_log2, scores, s);
  if (rc != SB_OK) return rc;
  cudaError_t err = cudaFuncSetAttribute(topk_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)key_smem);
  if (err != cudaSuccess) return cuda_error(err, "sb_route_topk: set smem");
  const int64_t rows = (int64_t)B * QB * H;
  SB_CHECK_ARG(rows < (1ll << 31), "sb_route_topk: too many rows");
  topk_rows_kernel<<<(unsigned)rows, kTopkThreads, key_smem, s>>>(scores, candidates, topk, words, packed_route, indices);
  SB_CHECK_LAUNCH("sb_route_topk: top-k launch");
  return SB_OK;
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
  SB_CHECK_ARG(qc && kc && packed_route, "sb_route_topk_noalloc: null pointer");
  SB_CHECK_ARG(kc_dtype == SB_F32 || kc_dtype == SB_BF16, "sb_route_topk_noalloc: bad key-centroid dtype");
  SB_CHECK_ARG(B > 0 && QB > 0 && NB > 0 && H > 0, "sb_route_topk_noalloc: sizes must be positive");
  SB_CHECK_ARG(QB <= NB, "sb_route_topk_noalloc: QB (%d) exceeds NB (%d)", QB, NB);
  SB_CHECK_ARG(D == 64 || D == 128, "sb_route_topk_noalloc: head dim must be 64 or 128");
  SB_CHECK_ARG(candidates >= 1 && candidates <= NB,
               "sb_route_topk_noalloc: candidates must lie in [1, NB], got %d", candidates);
  SB_CHECK_ARG(topk >= 1 && topk <= candidates,
               "sb_route_topk_noalloc: topk must lie in [1, candidates], got %d", topk);
  const int words = ceil_div(NB, 32);
  SB_CHECK_ARG(words <= 256, "sb_route_topk_noalloc: at most 8192 key blocks are supported");
  const size_t key_smem = (size_t)candidates * sizeof(uint32_t);
  SB_CHECK_ARG(key_smem <= 200 * 1024, "sb_route_topk_noalloc: too many candidate blocks (%d)", candidates);
  const int64_t per_block = (int64_t)H * candidates;
  SB_CHECK_ARG(per_block <= kNoAllocScoreFloats,
               "sb_route_topk_noalloc: H * candidates = %lld exceeds the %lld-float scratch array "
               "(SB_ROUTE_NOALLOC_SCRATCH_FLOATS); use sb_route_topk with a caller workspace",
               (long long)per_block, (long long)kNoAllocScoreFloats);
  int status = SB_OK;
  float* scratch = route_noalloc_scratch(&status);
  if (scratch == nullptr) return status;
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t err = cudaFuncSetAttribute(topk_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)key_smem);
  if (err != cudaSuccess) return cuda_error(err, "sb_route_topk_noalloc: set smem");
  const int chunk = (int)std::min<int64_t>(QB, kNoAllocScoreFloats / per_block);
  const size_t kc_elem = kc_dtype == SB_BF16 ? 2 : 4;
  for (int b = 0; b < B; ++b) {
    const char* kc_b = static_cast<const char*>(kc) + (size_t)b * NB * H * D * kc_elem;
    for (int q0 = 0; q0 < QB; q0 += chunk) {
      const int n = std::min(chunk, QB - q0);
      const float* qc_c = qc + ((int64_t)b * NB + q0) * H * D;
      dim3 grid(ceil_div(candidates, kScoreTile), ceil_div(n, kScoreTile), H);
      int rc;
      if (kc_dtype == SB_BF16)
        rc = D == 128 ? launch_scores<__nv_bfloat16, 128>(grid, qc_c, kc_b, n, NB, H, candidates, scale_log2, scratch, s)
                      : launch_scores<__nv_bfloat16, 64>(grid, qc_c, kc_b, n, NB, H, candidates, scale_log2, scratch, s);
      else
        rc = D == 128 ? launch_scores<float, 128>(grid, qc_c, kc_b, n, NB, H, candidates, scale_log2, scratch, s)
                      : launch_scores<float, 64>(grid, qc_c, kc_b, n, NB, H, candidates, scale_log2, scratch, s);
      if (rc != SB_OK) return rc;
      const int64_t row0 = ((int64_t)b * QB + q0) * H;
      topk_rows_kernel<<<(unsigned)((int64_t)n * H), kTopkThreads, key_smem, s>>>(
          scratch, candidates, topk, words, packed_route + row0 * words, indices ? indices + row0 * topk : nullptr);
      SB_CHECK_LAUNCH("sb_route_topk_noalloc: top-k launch");
    }
  }
  return SB_OK;
}
