// SIMT sparse attention for the inputs the tensor-core kernel does not take (float32
// elements, or head dim 64).  One warp per query row; lanes split the head dim.
// Semantics are those of sb_sparse_attention in include/spark_h3_b200.h.
#include "common.cuh"
#include "attn_common.cuh"

namespace sb {

template <typename T, int D>
__global__ void __launch_bounds__(128)
sparse_attention_simt_kernel(AttnParams p) {
  constexpr int PER = D / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = p.row_lo + blockIdx.x * 4 + warp;
  const int h = blockIdx.y, b = blockIdx.z;
  if (t >= p.row_hi) return;
  const T* q = static_cast<const T*>(p.q);
  const T* k = static_cast<const T*>(p.k);
  const T* v = static_cast<const T*>(p.v);
  const T* ak = static_cast<const T*>(p.ak);
  const T* av = static_cast<const T*>(p.av);
  const int64_t HD = (int64_t)p.H * D;
  const float scale_log2 = rsqrtf((float)D) * kLog2e;

  float qv[PER], acc[PER];
  const int64_t qoff = ((int64_t)b * p.T + t) * HD + (int64_t)h * D;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    qv[i] = Elem<T>::to_f(q[qoff + lane + 32 * i]);
    acc[i] = 0.f;
  }
  float m = -INFINITY, l = 0.f;

  const bool routed = t < p.query_tokens;
  const int qb = t / p.block;
  const int32_t* words = routed ? p.packed + (((int64_t)b * p.QB + qb) * p.H + h) * p.words : nullptr;

  for (int kb = 0; kb < p.NB; ++kb) {
    const bool exact = !routed || block_is_exact(words, kb, qb, p.sink_first, p.sink_last, p.local_radius);
    if (exact) {
      const int r0 = kb * p.block, r1 = min(p.T, r0 + p.block);
      for (int r = r0; r < r1; ++r) {
        const int64_t koff = ((int64_t)b * p.T + r) * HD + (int64_t)h * D;
        float part = 0.f;
#pragma unroll
        for (int i = 0; i < PER; ++i) part = fmaf(qv[i], Elem<T>::to_f(k[koff + lane + 32 * i]), part);
        const float x = warp_sum(part) * scale_log2;
        const float m_new = fmaxf(m, x);
        const float alpha = exp2f(m - m_new), pr = exp2f(x - m_new);
        l = l * alpha + pr;
#pragma unroll
        for (int i = 0; i < PER; ++i) acc[i] = acc[i] * alpha + pr * Elem<T>::to_f(v[koff + lane + 32 * i]);
        m = m_new;
      }
    } else if (p.lm != nullptr) {  // without summaries, routed rows see their exact keys only
      const int64_t soff = (((int64_t)b * p.H + h) * p.NB + kb) * D;
      float part = 0.f;
#pragma unroll
      for (int i = 0; i < PER; ++i) part = fmaf(qv[i], Elem<T>::to_f(ak[soff + lane + 32 * i]), part);
      const float x = warp_sum(part) * scale_log2 + p.lm[((int64_t)b * p.H + h) * p.NB + kb] * kLog2e;
      const float m_new = fmaxf(m, x);
      const float alpha = exp2f(m - m_new), pr = exp2f(x - m_new);
      l = l * alpha + pr;
#pragma unroll
      for (int i = 0; i < PER; ++i) acc[i] = acc[i] * alpha + pr * Elem<T>::to_f(av[soff + lane + 32 * i]);
      m = m_new;
    }
  }
  T* out = static_cast<T*>(p.out);
  const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) out[qoff + lane + 32 * i] = Elem<T>::from_f(acc[i] * inv);
  if (p.lse != nullptr && lane == 0)
    p.lse[((int64_t)b * p.T + t) * p.H + h] = l > 0.f ? (m + log2f(l)) * kLn2 : -INFINITY;
}

int launch_sparse_attention_simt(const AttnParams& p, int dtype, int D, cudaStream_t s) {
  dim3 grid(ceil_div(p.row_hi - p.row_lo, 4), p.H, p.B);
  if (dtype == SB_BF16) {
    if (D == 128) sparse_attention_simt_kernel<__nv_bfloat16, 128><<<grid, 128, 0, s>>>(p);
    else sparse_attention_simt_kernel<__nv_bfloat16, 64><<<grid, 128, 0, s>>>(p);
  } else {
    if (D == 128) sparse_attention_simt_kernel<float, 128><<<grid, 128, 0, s>>>(p);
    else sparse_attention_simt_kernel<float, 64><<<grid, 128, 0, s>>>(p);
  }
  SB_CHECK_LAUNCH("sb_sparse_attention: SIMT launch");
  return SB_OK;
}

}  // namespace sb
