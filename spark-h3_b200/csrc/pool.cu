// Block pooling of Q and K, the global query anchor, and the anchor-weighted key/value
// summaries.  All three are HBM-bound single passes with 16-byte vector accesses.
//
// Canonical arithmetic (the CPU oracle in oracle/spark_oracle.c repeats it exactly):
//   a block's sum is formed per 64-row sub-block, each a sequential fp32 sum over rows
//   in token order starting from 0, and the sub-block sums are then added in order;
//   the mean is that sum divided (IEEE fp32) by the rows present in the block.
#include "common.cuh"

namespace sb {

// grid (NB, B), block (H*D/8).  Each thread owns 8 adjacent columns of the H*D row.
template <typename T>
__global__ void pool_queries_kernel(const T* __restrict__ q, int T_, int HD, int block,
                                    float* __restrict__ qc) {
  const int j = blockIdx.x, b = blockIdx.y;
  const int col = threadIdx.x * 8;
  if (col >= HD) return;
  const int row0 = j * block;
  const int rows = min(block, T_ - row0);
  const T* base = q + ((int64_t)b * T_ + row0) * HD + col;
  float total[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) total[i] = 0.f;
  for (int s = 0; s < rows; s += 64) {
    const int sub = min(64, rows - s);
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    int r = 0;
    for (; r + 4 <= sub; r += 4) {
      float x0[8], x1[8], x2[8], x3[8];
      load8(base + (int64_t)(s + r) * HD, x0);
      load8(base + (int64_t)(s + r + 1) * HD, x1);
      load8(base + (int64_t)(s + r + 2) * HD, x2);
      load8(base + (int64_t)(s + r + 3) * HD, x3);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        acc[i] = __fadd_rn(acc[i], x0[i]);
        acc[i] = __fadd_rn(acc[i], x1[i]);
        acc[i] = __fadd_rn(acc[i], x2[i]);
        acc[i] = __fadd_rn(acc[i], x3[i]);
      }
    }
    for (; r < sub; ++r) {
      float x0[8];
      load8(base + (int64_t)(s + r) * HD, x0);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], x0[i]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) total[i] = __fadd_rn(total[i], acc[i]);
  }
  const float cnt = (float)rows;
  float out[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) out[i] = __fdiv_rn(total[i], cnt);
  store8(qc + ((int64_t)b * gridDim.x + j) * HD + col, out);
}

// grid (ceil(H*D/128), B), block 128: one thread per (b, h, d) column.
template <typename TA>
__global__ void query_anchor_kernel(const float* __restrict__ qc, int NB, int HD, int block,
                                    int prefix_blocks, TA* __restrict__ anchor) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x, b = blockIdx.y;
  if (col >= HD) return;
  const float* p = qc + (int64_t)b * NB * HD + col;
  const float scale = (float)block;
  float acc = 0.f;
  for (int j = 0; j < prefix_blocks; ++j) acc = __fadd_rn(acc, __fmul_rn(__ldg(p + (int64_t)j * HD), scale));
  const float mean = __fdiv_rn(acc, (float)prefix_blocks * (float)block);
  anchor[(int64_t)b * HD + col] = Elem<TA>::from_f(mean);
}

// One CTA per (key block, head, batch), 128 threads.  K and V rows of the block are
// staged in shared memory as fp32 (block <= 128 rows, D <= 128).
template <typename T, typename TA, int D>
__global__ void __launch_bounds__(128)
pool_keys_summaries_kernel(const T* __restrict__ k, const T* __restrict__ v,
                           const TA* __restrict__ anchor, int T_, int H, int block,
                           int weighted_kv, int mass_bias, T* __restrict__ kc,
                           T* __restrict__ ak, T* __restrict__ av, float* __restrict__ lm) {
  extern __shared__ float smem[];
  const int kb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int NB = gridDim.x;
  const int HD = H * D;
  const int row0 = kb * block;
  const int rows = min(block, T_ - row0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool want_sum = (ak != nullptr || av != nullptr || lm != nullptr);
  float* sk = smem;                   // [block][D]
  float* sv = sk + block * D;         // [block][D]
  float* sa = sv + block * D;         // [D]
  float* sp = sa + D;                 // [block] probabilities
  float* red = sp + block;            // [8] reductions

  // Stage K (and V, when summaries are wanted).  8 columns per thread-step.
  constexpr int C8 = D / 8;
  for (int idx = tid; idx < rows * C8; idx += blockDim.x) {
    const int r = idx / C8, c = (idx % C8) * 8;
    const int64_t g = ((int64_t)b * T_ + row0 + r) * HD + (int64_t)h * D + c;
    load8(k + g, sk + r * D + c);
    if (want_sum) load8(v + g, sv + r * D + c);
  }
  if (want_sum && anchor != nullptr) {
    for (int d = tid; d < D; d += blockDim.x) sa[d] = Elem<TA>::to_f(anchor[((int64_t)b * H + h) * D + d]);
  }
  __syncthreads();

  // Key block mean (routing centroid) in the canonical order.
  if (kc != nullptr) {
    for (int d = tid; d < D; d += blockDim.x) {
      float total = 0.f;
      for (int s = 0; s < rows; s += 64) {
        const int sub = min(64, rows - s);
        float acc = 0.f;
        for (int r = 0; r < sub; ++r) acc = __fadd_rn(acc, sk[(s + r) * D + d]);
        total = __fadd_rn(total, acc);
      }
      kc[(((int64_t)b * NB + kb) * H + h) * D + d] = Elem<T>::from_f(__fdiv_rn(total, (float)rows));
    }
  }
  if (!want_sum) return;

  const float scale = rsqrtf((float)D);
  const float scale_log2 = scale * kLog2e;
  const float cnt = (float)rows;
  float maximum = 0.f, den = 1.f;
  if (weighted_kv || mass_bias) {
    // logits[r] = (a . k_r) * scale * log2(e): warps split rows, lanes split d.
    for (int r = warp; r < rows; r += 4) {
      float part = 0.f;
      for (int d = lane; d < D; d += 32) part = fmaf(sa[d], sk[r * D + d], part);
      part = warp_sum(part);
      if (lane == 0) sp[r] = part * scale_log2;
    }
    __syncthreads();
    float m = -INFINITY;
    for (int r = tid; r < rows; r += blockDim.x) m = fmaxf(m, sp[r]);
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    maximum = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    __syncthreads();
    float s = 0.f;
    for (int r = tid; r < rows; r += blockDim.x) {
      const float p = exp2f(sp[r] - maximum);
      sp[r] = p;
      s += p;
    }
    s = warp_sum(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    den = (red[0] + red[1]) + (red[2] + red[3]);
    __syncthreads();
  }

  // Weighted (or plain) means.  The weights are rounded to the K/V element type
  // before the products, as the tensor-core dot of the reference does.
  T* ak_row = ak ? ak + (((int64_t)b * H + h) * NB + kb) * D : nullptr;
  T* av_row = av ? av + (((int64_t)b * H + h) * NB + kb) * D : nullptr;
  float shift_part = 0.f;
  for (int d = tid; d < D; d += blockDim.x) {
    float key_sum = 0.f, val_sum = 0.f;
    if (weighted_kv) {
      for (int r = 0; r < rows; ++r) {
        const float w = Elem<T>::to_f(Elem<T>::from_f(sp[r]));
        key_sum = fmaf(w, sk[r * D + d], key_sum);
        val_sum = fmaf(w, sv[r * D + d], val_sum);
      }
      key_sum /= den;
      val_sum /= den;
    } else {
      for (int r = 0; r < rows; ++r) {
        key_sum += sk[r * D + d];
        val_sum += sv[r * D + d];
      }
      key_sum /= cnt;
      val_sum /= cnt;
    }
    const T key_stored = Elem<T>::from_f(key_sum);
    if (ak_row) ak_row[d] = key_stored;
    if (av_row) av_row[d] = Elem<T>::from_f(val_sum);
    if (mass_bias) shift_part = fmaf(sa[d], Elem<T>::to_f(key_stored), shift_part);
  }
  if (lm == nullptr) return;
  if (mass_bias) {
    shift_part = warp_sum(shift_part);
    if (lane == 0) red[4 + warp] = shift_part;
    __syncthreads();
    if (tid == 0) {
      const float shift = ((red[4] + red[5]) + (red[6] + red[7])) * scale;
      lm[((int64_t)b * H + h) * NB + kb] = (maximum + log2f(den)) * kLn2 - shift;
    }
  } else if (tid == 0) {
    lm[((int64_t)b * H + h) * NB + kb] = logf(cnt);
  }
}

}  // namespace sb

using namespace sb;

extern "C" int sb_pool_queries(const void* q, int dtype, int B, int T, int H, int D, int block,
                               float* qc, void* stream) {
  SB_CHECK_ARG(q && qc, "sb_pool_queries: null pointer");
  SB_CHECK_ARG(dtype == SB_F32 || dtype == SB_BF16, "sb_pool_queries: dtype must be SB_F32 or SB_BF16");
  SB_CHECK_ARG(B > 0 && T > 0 && H > 0, "sb_pool_queries: B, T, H must be positive");
  SB_CHECK_ARG(D == 64 || D == 128, "sb_pool_queries: head dim must be 64 or 128, got %d", D);
  SB_CHECK_ARG(block == 64 || block == 128, "sb_pool_queries: block must be 64 or 128, got %d", block);
  SB_CHECK_ARG(((uintptr_t)q % 16) == 0 && ((uintptr_t)qc % 16) == 0, "sb_pool_queries: pointers must be 16-byte aligned");
  const int HD = H * D;
  SB_CHECK_ARG(HD / 8 <= 1024, "sb_pool_queries: H * D must be at most 8192");
  const int NB = ceil_div(T, block);
  dim3 grid(NB, B), threads(HD / 8);
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == SB_BF16)
    pool_queries_kernel<__nv_bfloat16><<<grid, threads, 0, s>>>((const __nv_bfloat16*)q, T, HD, block, qc);
  else
    pool_queries_kernel<float><<<grid, threads, 0, s>>>((const float*)q, T, HD, block, qc);
  SB_CHECK_LAUNCH("sb_pool_queries launch");
  return SB_OK;
}

extern "C" int sb_query_anchor(const float* qc, int B, int NB, int H, int D, int block,
                               int prefix_blocks, void* anchor, int anchor_dtype, void* stream) {
  SB_CHECK_ARG(qc && anchor, "sb_query_anchor: null pointer");
  SB_CHECK_ARG(anchor_dtype == SB_F32 || anchor_dtype == SB_BF16, "sb_query_anchor: bad anchor dtype");
  SB_CHECK_ARG(B > 0 && H > 0 && D > 0 && NB > 0, "sb_query_anchor: sizes must be positive");
  SB_CHECK_ARG(prefix_blocks >= 1 && prefix_blocks <= NB,
               "sb_query_anchor: prefix_blocks must lie in [1, NB], got %d", prefix_blocks);
  const int HD = H * D;
  dim3 grid(ceil_div(HD, 128), B);
  cudaStream_t s = (cudaStream_t)stream;
  if (anchor_dtype == SB_BF16)
    query_anchor_kernel<__nv_bfloat16><<<grid, 128, 0, s>>>(qc, NB, HD, block, prefix_blocks, (__nv_bfloat16*)anchor);
  else
    query_anchor_kernel<float><<<grid, 128, 0, s>>>(qc, NB, HD, block, prefix_blocks, (float*)anchor);
  SB_CHECK_LAUNCH("sb_query_anchor launch");
  return SB_OK;
}

template <typename T, typename TA, int D>
static int launch_pool_keys(const void* k, const void* v, const void* anchor, int B, int tokens, int H,
                            int block, int weighted_kv, int mass_bias, void* kc, void* ak, void* av,
                            float* lm, cudaStream_t s) {
  const int NB = ceil_div(tokens, block);
  const size_t smem = (size_t)(2 * block * D + D + block + 8) * sizeof(float);
  auto kern = pool_keys_summaries_kernel<T, TA, D>;
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return cuda_error(err, "sb_pool_keys_summaries: set smem");
  dim3 grid(NB, H, B);
  kern<<<grid, 128, smem, s>>>((const T*)k, (const T*)v, (const TA*)anchor, tokens, H, block, weighted_kv,
                              mass_bias, (T*)kc, (T*)ak, (T*)av, lm);
  SB_CHECK_LAUNCH("sb_pool_keys_summaries launch");
  return SB_OK;
}

extern "C" int sb_pool_keys_summaries(const void* k, const void* v, const void* anchor, int dtype,
                                      int anchor_dtype, int B, int T, int H, int D, int block,
                                      int weighted_kv, int mass_bias, void* kc, void* ak, void* av,
                                      float* lm, void* stream) {
  const bool want_sum = ak || av || lm;
  SB_CHECK_ARG(k, "sb_pool_keys_summaries: null K");
  SB_CHECK_ARG(!want_sum || v, "sb_pool_keys_summaries: summaries need V");
  SB_CHECK_ARG(!want_sum || !(weighted_kv || mass_bias) || anchor,
               "sb_pool_keys_summaries: weighted summaries need the anchor");
  SB_CHECK_ARG(dtype == SB_F32 || dtype == SB_BF16, "sb_pool_keys_summaries: bad dtype");
  SB_CHECK_ARG(anchor_dtype == SB_F32 || anchor_dtype == SB_BF16, "sb_pool_keys_summaries: bad anchor dtype");
  SB_CHECK_ARG(B > 0 && T > 0 && H > 0, "sb_pool_keys_summaries: B, T, H must be positive");
  SB_CHECK_ARG(D == 64 || D == 128, "sb_pool_keys_summaries: head dim must be 64 or 128");
  SB_CHECK_ARG(block == 64 || block == 128, "sb_pool_keys_summaries: block must be 64 or 128");
  SB_CHECK_ARG(((uintptr_t)k % 16) == 0 && (!v || ((uintptr_t)v % 16) == 0),
               "sb_pool_keys_summaries: K/V must be 16-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  const bool abf = anchor_dtype == SB_BF16;
  if (dtype == SB_BF16) {
    if (D == 128)
      return abf ? launch_pool_keys<__nv_bfloat16, __nv_bfloat16, 128>(k, v, anchor, B, T, H, block, weighted_kv, mass_bias, kc, ak, av, lm, s)
                 : launch_pool_keys<__nv_bfloat16, float, 128>(k, v, anchor, B, T, H, block, weighted_kv, mass_bias, kc, ak, av, lm, s);
    return abf ? launch_pool_keys<__nv_bfloat16, __nv_bfloat16, 64>(k, v, anchor, B, T, H, block, weighted_kv, mass_bias, kc, ak, av, lm, s)
               : launch_pool_keys<__nv_bfloat16, float, 64>(k, v, anchor, B, T, H, block, weighted_kv, mass_bias, kc, ak, av, lm, s);
  }
  SB_CHECK_ARG(!abf, "sb_pool_keys_summaries: float32 K/V need a float32 anchor");
  if (D == 128)
    return launch_pool_keys<float, float, 128>(k, v, anchor, B, T, H, block, weighted_kv, mass_bias, kc, ak, av, lm, s);
  return launch_pool_keys<float, float, 64>(k, v, anchor, B, T, H, block, weighted_kv, mass_bias, kc, ak, av, lm, s);
}
