// Pooled tails of the Spark layer: the reference's tail granularities "block" and "block8x8"
// (sol_numerator_virtual_q.py:193-242, 415-499, 528-596).  The exact part comes from the
// attention kernels run without summary columns (exact output and its LSE); here the
// skipped key blocks are attended once per query group through the group's mean query, and
// the two partial softmaxes are merged row by row:
//   tail_summaries8_kernel  anchor-weighted summaries of every 8 keys (block8x8 only)
//   tail_merge_kernel       per query group (a whole block, or 8 rows): mean query rounded to
//                           the Q dtype, online softmax over the summary entries whose key
//                           block is not exact, then out = (we * exact + wa * tail) / (we + wa)
//                           with we, wa the exponentials of the two LSEs relative to their max.
#include "common.cuh"
#include "attn_common.cuh"

namespace sb {
namespace {

constexpr int kDim = 128;
constexpr int kTailThreads = 128;  // 4 warps; a lane holds 4 of the 128 dimensions

// One warp per 8-key group (sol_numerator_virtual_q.py:193-242): p = 2^(a.k/sqrt(D) log2 e
// - max) in fp32, AK = sum p k / sum p, AV likewise (or plain means), stored in the K/V dtype;
// LM = (max + log2 sum p) ln 2 - a.AK/sqrt(D) with the stored key (or the fp32 mean), or
// log(keys in the group) without the mass bias.
template <typename T, typename TA>
__global__ void __launch_bounds__(kTailThreads) tail_summaries8_kernel(
    const T* __restrict__ k, const T* __restrict__ v, const TA* __restrict__ anchor, int Tn, int H, int n8,
    int weighted_kv, int mass_bias, int pre_round, T* __restrict__ ak8, T* __restrict__ av8, float* __restrict__ lm8) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x * (kTailThreads / 32) + warp;
  const int h = blockIdx.y, b = blockIdx.z;
  if (g >= n8) return;
  const int d0 = 4 * lane;
  const int64_t HD = (int64_t)H * kDim;
  float a[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) a[i] = Elem<TA>::to_f(anchor[((int64_t)b * H + h) * kDim + d0 + i]);
  const int row0 = 8 * g;
  const int count = min(8, Tn - row0);
  const float scale = rsqrtf((float)kDim);
  float kr[8][4], vr[8][4], logit[8];
  float mx = -INFINITY;
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    float part = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) kr[r][i] = vr[r][i] = 0.f;
    if (r < count) {
      const int64_t off = ((int64_t)b * Tn + row0 + r) * HD + (int64_t)h * kDim + d0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        kr[r][i] = Elem<T>::to_f(k[off + i]);
        vr[r][i] = Elem<T>::to_f(v[off + i]);
        part = fmaf(kr[r][i], a[i], part);
      }
    }
    logit[r] = r < count ? warp_sum(part) * scale * kLog2e : -INFINITY;  // count is warp-uniform
    mx = fmaxf(mx, logit[r]);
  }
  float den = 0.f, p[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    p[r] = r < count ? exp2f(logit[r] - mx) : 0.f;
    den += p[r];
  }
  den = fmaxf(den, 1e-30f);
  float key[4], val[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float sk = 0.f, sv = 0.f;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const float w = weighted_kv ? p[r] : (r < count ? 1.f : 0.f);
      sk = fmaf(w, kr[r][i], sk);
      sv = fmaf(w, vr[r][i], sv);
    }
    const float norm = weighted_kv ? den : (float)count;
    key[i] = sk / norm;
    val[i] = sv / norm;
  }
  const int64_t so = (((int64_t)b * H + h) * n8 + g) * kDim + d0;
  float shift = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const T ks = Elem<T>::from_f(key[i]);
    ak8[so + i] = ks;
    av8[so + i] = Elem<T>::from_f(val[i]);
    shift = fmaf(a[i], pre_round ? key[i] : Elem<T>::to_f(ks), shift);
  }
  shift = warp_sum(shift) * scale;
  if (lane == 0)
    lm8[((int64_t)b * H + h) * n8 + g] = mass_bias ? (mx + log2f(den)) * kLn2 - shift : logf((float)count);
}

// One CTA per (query block, head, batch), serving the block's NG query groups of G rows
// (NG = block / G: one group for "block", eight or sixteen of 8 rows for "block8x8"), which
// share the block's exact set.  Summary entry e covers keys [e*E, e*E + E) of key block
// (e*E) / block; it is skipped when that block is exact for the query block (route bit, sink
// range or local radius).  A warp takes 32 entries at a time, one per lane: the lane scores
// its entry against every group mean (full 128-term dot products, the means read from shared
// memory as broadcasts), one warp max per group rescales the chunk, and the probabilities
// reach the lanes that own the value dimensions by shuffles.  That is about 2.5 times fewer
// instructions per entry than a warp-wide dot product per group and entry.
template <typename T, int NG>
__global__ void __launch_bounds__(kTailThreads) tail_merge_kernel(
    const T* __restrict__ q, const T* __restrict__ tk, const T* __restrict__ tv, const float* __restrict__ lmass,
    const int32_t* __restrict__ packed, int QB, int words, int Tn, int H, int n_entries, int entry_tokens,
    int block, int sink_first, int sink_last, int local_radius, T* __restrict__ out, float* __restrict__ lse) {
  constexpr int kWarps = kTailThreads / 32;
  __shared__ __align__(16) float qmean[NG][kDim];
  __shared__ float wm[kWarps][NG], wden[kWarps][NG];
  __shared__ float wacc[kWarps][NG][kDim];
  __shared__ float row_w[2][kTailThreads];  // per row of the block (at most 128): exact and tail weights
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int G = block / NG;  // rows per query group
  const int row0 = qb * block;
  const int64_t HD = (int64_t)H * kDim;
  // Mean query of every group, in fp32 and rounded to the Q dtype (the reference's qmean).
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    const int r0 = row0 + g * G, rows = min(G, Tn - r0);
    float s = 0.f;
    for (int r = 0; r < rows; ++r) s += Elem<T>::to_f(q[((int64_t)b * Tn + r0 + r) * HD + (int64_t)h * kDim + tid]);
    qmean[g][tid] = Elem<T>::to_f(Elem<T>::from_f(s / (float)max(rows, 1)));
  }
  __syncthreads();
  const int32_t* wrow = packed + (((int64_t)b * QB + qb) * H + h) * words;
  const int d0 = 4 * lane;
  const float scale_log2 = rsqrtf((float)kDim) * kLog2e;
  float m[NG], den[NG], acc[NG][4];
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    m[g] = -INFINITY;
    den[g] = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[g][i] = 0.f;
  }
  const int64_t ebase = ((int64_t)b * H + h) * n_entries;
  float dl[NG];  // this lane's share of each group's denominator
#pragma unroll
  for (int g = 0; g < NG; ++g) dl[g] = 0.f;
  // TT entries per lane: each group mean read from shared memory serves TT key rows.
  constexpr int TT = NG >= 16 ? 1 : (NG >= 8 ? 2 : 4);
  for (int c0 = warp * 32 * TT; c0 < n_entries; c0 += kWarps * 32 * TT) {
    bool live[TT];
    float sc[TT][NG];
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      const int e = c0 + 32 * t + lane;
      live[t] = e < n_entries;
      if (live[t])
        live[t] = !block_is_exact(wrow, (e * entry_tokens) / block, qb, sink_first, sink_last, local_radius);
#pragma unroll
      for (int g = 0; g < NG; ++g) sc[t][g] = 0.f;
    }
#pragma unroll 2
    for (int d = 0; d < kDim; d += 8) {
      float kf[TT][8];
#pragma unroll
      for (int t = 0; t < TT; ++t) {
        if (live[t]) {
          load8(tk + (ebase + c0 + 32 * t + lane) * kDim + d, kf[t]);
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) kf[t][i] = 0.f;
        }
      }
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        const float4 qa = *reinterpret_cast<const float4*>(&qmean[g][d]);
        const float4 qc = *reinterpret_cast<const float4*>(&qmean[g][d + 4]);
#pragma unroll
        for (int t = 0; t < TT; ++t) {
          float x = fmaf(kf[t][0], qa.x, sc[t][g]);
          x = fmaf(kf[t][1], qa.y, x);
          x = fmaf(kf[t][2], qa.z, x);
          x = fmaf(kf[t][3], qa.w, x);
          x = fmaf(kf[t][4], qc.x, x);
          x = fmaf(kf[t][5], qc.y, x);
          x = fmaf(kf[t][6], qc.z, x);
          sc[t][g] = fmaf(kf[t][7], qc.w, x);
        }
      }
    }
    float lm2[TT];
#pragma unroll
    for (int t = 0; t < TT; ++t) lm2[t] = live[t] ? lmass[ebase + c0 + 32 * t + lane] * kLog2e : 0.f;
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      float score[TT], cm = -INFINITY;
#pragma unroll
      for (int t = 0; t < TT; ++t) {
        score[t] = live[t] ? sc[t][g] * scale_log2 + lm2[t] : -INFINITY;
        cm = fmaxf(cm, score[t]);
      }
      const float m_new = fmaxf(m[g], warp_max(cm));
      const float factor = m[g] == -INFINITY ? 0.f : exp2f(m[g] - m_new);
      float pr_sum = 0.f;
#pragma unroll
      for (int t = 0; t < TT; ++t) {
        const float pr = live[t] ? exp2f(score[t] - m_new) : 0.f;
        pr_sum += pr;
        sc[t][g] = pr;
      }
      dl[g] = fmaf(dl[g], factor, pr_sum);
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[g][i] *= factor;
      m[g] = m_new;
    }
    // P.V over the chunk's live entries: lane j's probabilities against entry j's values.
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      for (unsigned bits = __ballot_sync(0xffffffffu, live[t]); bits; bits &= bits - 1u) {
        const int j = __ffs(bits) - 1;
        const T* vp = tv + (ebase + c0 + 32 * t + j) * kDim + d0;
        float vv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) vv[i] = Elem<T>::to_f(vp[i]);
#pragma unroll
        for (int g = 0; g < NG; ++g) {
          const float pj = __shfl_sync(0xffffffffu, sc[t][g], j);
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[g][i] = fmaf(pj, vv[i], acc[g][i]);
        }
      }
    }
  }
#pragma unroll
  for (int g = 0; g < NG; ++g) den[g] = warp_sum(dl[g]);
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    if (lane == 0) {
      wm[warp][g] = m[g];
      wden[warp][g] = den[g];
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) wacc[warp][g][d0 + i] = acc[g][i];
  }
  __syncthreads();
  // Per group: merge the warps' partial softmaxes into the pooled tail and its LSE; then one
  // thread per row computes the blend weights, and every thread blends its dimension.
  float tail[NG], al[NG];
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, wm[w][g]);
    float D = 0.f, A = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float f = wm[w][g] == -INFINITY ? 0.f : exp2f(wm[w][g] - M);
      D = fmaf(wden[w][g], f, D);
      A = fmaf(wacc[w][g][tid], f, A);
    }
    tail[g] = D > 0.f ? A / D : 0.f;
    al[g] = D > 0.f ? (M + log2f(D)) * kLn2 : -INFINITY;
  }
  const int rows = min(block, Tn - row0);
  if (tid < rows) {
    float a_row = al[0];
#pragma unroll
    for (int g = 1; g < NG; ++g)
      if (tid / G == g) a_row = al[g];
    const int64_t rl = ((int64_t)b * Tn + row0 + tid) * H + h;
    const float el = lse[rl];
    const float mx = fmaxf(el, a_row);
    const float we = mx == -INFINITY ? 0.f : expf(el - mx);
    const float wa = mx == -INFINITY ? 0.f : expf(a_row - mx);
    row_w[0][tid] = we;
    row_w[1][tid] = wa;
    lse[rl] = we + wa > 0.f ? mx + logf(we + wa) : -INFINITY;
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    const int r0 = g * G, r1 = min(r0 + G, rows);
    for (int r = r0; r < r1; ++r) {
      const float we = row_w[0][r], wa = row_w[1][r];
      const int64_t o = ((int64_t)b * Tn + row0 + r) * HD + (int64_t)h * kDim + tid;
      const float exact = Elem<T>::to_f(out[o]);
      const float merged =
          ((we > 0.f ? we * exact : 0.f) + (wa > 0.f ? wa * tail[g] : 0.f)) / fmaxf(we + wa, 1e-30f);
      out[o] = Elem<T>::from_f(merged);
    }
  }
}

}  // namespace
}  // namespace sb

using namespace sb;

extern "C" int sb_tail_summaries8(const void* k, const void* v, const void* anchor, int dtype, int anchor_dtype, int B,
                                  int T, int H, int D, int weighted_kv, int mass_bias, int numerics, void* ak8,
                                  void* av8, float* lm8, void* stream) {
  SB_CHECK_ARG(k && v && anchor && ak8 && av8 && lm8, "sb_tail_summaries8: null pointer");
  SB_CHECK_ARG(dtype == SB_BF16, "sb_tail_summaries8: K/V must be bf16");
  SB_CHECK_ARG(anchor_dtype == SB_BF16 || anchor_dtype == SB_F32, "sb_tail_summaries8: bad anchor dtype");
  SB_CHECK_ARG(B > 0 && T > 0 && H > 0 && D == kDim, "sb_tail_summaries8: needs B, T, H > 0 and D = 128");
  SB_CHECK_ARG((numerics & ~SB_SUMMARY_PRE_ROUND_LOGMASS) == 0,
               "sb_tail_summaries8: eight-key summaries take only SB_SUMMARY_PRE_ROUND_LOGMASS");
  const int n8 = ceil_div(T, 8);
  dim3 grid(ceil_div(n8, kTailThreads / 32), H, B);
  cudaStream_t s = (cudaStream_t)stream;
  const int pre = (numerics & SB_SUMMARY_PRE_ROUND_LOGMASS) ? 1 : 0;
  if (anchor_dtype == SB_BF16)
    tail_summaries8_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, kTailThreads, 0, s>>>(
        (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, (const __nv_bfloat16*)anchor, T, H, n8, weighted_kv,
        mass_bias, pre, (__nv_bfloat16*)ak8, (__nv_bfloat16*)av8, lm8);
  else
    tail_summaries8_kernel<__nv_bfloat16, float><<<grid, kTailThreads, 0, s>>>(
        (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, (const float*)anchor, T, H, n8, weighted_kv, mass_bias,
        pre, (__nv_bfloat16*)ak8, (__nv_bfloat16*)av8, lm8);
  SB_CHECK_LAUNCH("sb_tail_summaries8 launch");
  return SB_OK;
}

extern "C" int sb_tail_merge(const void* q, const void* ak, const void* av, const float* lm, int dtype, int B, int T,
                             int H, int D, int entry_tokens, int group_tokens, int block,
                             const int32_t* packed_route, int QB, int query_tokens, int sink_first, int sink_last,
                             int local_radius, void* out, float* lse, void* stream) {
  SB_CHECK_ARG(q && ak && av && lm && packed_route && out && lse, "sb_tail_merge: null pointer");
  SB_CHECK_ARG(dtype == SB_BF16, "sb_tail_merge: Q and the output must be bf16");
  SB_CHECK_ARG(B > 0 && T > 0 && H > 0 && D == kDim, "sb_tail_merge: needs B, T, H > 0 and D = 128");
  SB_CHECK_ARG(block == 64 || block == 128, "sb_tail_merge: block must be 64 or 128");
  SB_CHECK_ARG((entry_tokens == block && group_tokens == block) || (entry_tokens == 8 && group_tokens == 8),
               "sb_tail_merge: entries and query groups are both whole blocks or both 8 tokens");
  SB_CHECK_ARG(query_tokens >= 0 && query_tokens <= T && query_tokens % block == 0,
               "sb_tail_merge: query_tokens must be a block multiple in [0, T]");
  const int NB = ceil_div(T, block);
  SB_CHECK_ARG(QB >= query_tokens / block && QB <= NB, "sb_tail_merge: QB out of range");
  SB_CHECK_ARG(sink_first >= 0 && sink_first <= sink_last && sink_last <= NB, "sb_tail_merge: bad sink range");
  if (query_tokens == 0) return SB_OK;
  const int n_entries = ceil_div(T, entry_tokens);
  dim3 grid(query_tokens / block, H, B);
  cudaStream_t s = (cudaStream_t)stream;
  const auto* qq = (const __nv_bfloat16*)q;
  const auto* kk = (const __nv_bfloat16*)ak;
  const auto* vv = (const __nv_bfloat16*)av;
  auto* oo = (__nv_bfloat16*)out;
  const int words = ceil_div(NB, 32);
  if (group_tokens == block)
    tail_merge_kernel<__nv_bfloat16, 1><<<grid, kTailThreads, 0, s>>>(
        qq, kk, vv, lm, packed_route, QB, words, T, H, n_entries, entry_tokens, block, sink_first, sink_last,
        local_radius, oo, lse);
  else if (block == 64)
    tail_merge_kernel<__nv_bfloat16, 8><<<grid, kTailThreads, 0, s>>>(
        qq, kk, vv, lm, packed_route, QB, words, T, H, n_entries, entry_tokens, block, sink_first, sink_last,
        local_radius, oo, lse);
  else
    tail_merge_kernel<__nv_bfloat16, 16><<<grid, kTailThreads, 0, s>>>(
        qq, kk, vv, lm, packed_route, QB, words, T, H, n_entries, entry_tokens, block, sink_first, sink_last,
        local_radius, oo, lse);
  SB_CHECK_LAUNCH("sb_tail_merge launch");
  return SB_OK;
}
