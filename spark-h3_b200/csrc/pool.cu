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

// One CTA per (key block, batch) covering every head: thread t owns 16 adjacent columns
// of the H*D token row (D/16 threads per head), so each row is read with 32- or 64-byte
// vector loads by the whole CTA.  Pass 1 streams K once: key block means (canonical
// order) and the anchor logits.  Pass 2 re-reads K (an L2 hit) and streams V for the
// weighted means; the weights are rounded to the K/V element type before the products,
// as the tensor-core dot of the reference does.
constexpr int kCPT = 16;  // columns per thread

template <typename T> __device__ __forceinline__ void load16(const T* p, float* out);
template <> __device__ __forceinline__ void load16<__nv_bfloat16>(const __nv_bfloat16* p, float* out) {
  load8(p, out);
  load8(p + 8, out + 8);
}
template <> __device__ __forceinline__ void load16<float>(const float* p, float* out) {
  load8(p, out);
  load8(p + 8, out + 8);
}

template <int GROUP>
__device__ __forceinline__ float group_sum(float x) {
#pragma unroll
  for (int o = GROUP / 2; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}
template <int GROUP>
__device__ __forceinline__ float group_max(float x) {
#pragma unroll
  for (int o = GROUP / 2; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

template <typename T, typename TA, int D>
__global__ void __launch_bounds__(256)
pool_keys_summaries_kernel(const T* __restrict__ k, const T* __restrict__ v,
                           const TA* __restrict__ anchor, int T_, int H, int block,
                           int weighted_kv, int mass_bias, int numerics, T* __restrict__ kc,
                           T* __restrict__ ak, T* __restrict__ av, float* __restrict__ lm) {
  constexpr int G = D / kCPT;  // threads per head
  extern __shared__ float plog[];  // [H][block] logits, then probabilities
  __shared__ float head_max[64], head_den[64];
  const int kb = blockIdx.x, b = blockIdx.y;
  const int NB = gridDim.x;
  const int HD = H * D;
  const int tid = threadIdx.x;
  const int col = tid * kCPT;
  const bool active = col < HD;
  const int h = col / D, dcol = col % D;
  const int glane = tid % G;
  const int row0 = kb * block;
  const int rows = min(block, T_ - row0);
  const bool want_sum = (ak != nullptr || av != nullptr || lm != nullptr);
  const bool need_logits = want_sum && (weighted_kv || mass_bias);
  const float scale = rsqrtf((float)D);
  const float scale_log2 = scale * kLog2e;

  float a[kCPT];
#pragma unroll
  for (int i = 0; i < kCPT; ++i) a[i] = 0.f;
  if (active && need_logits) {
#pragma unroll
    for (int i = 0; i < kCPT; ++i) a[i] = Elem<TA>::to_f(anchor[((int64_t)b * H + h) * D + dcol + i]);
  }
  const T* kbase = k + ((int64_t)b * T_ + row0) * HD + col;
  const T* vbase = v ? v + ((int64_t)b * T_ + row0) * HD + col : nullptr;

  // Pass 1: K block means and anchor logits.
  float total[kCPT];
#pragma unroll
  for (int i = 0; i < kCPT; ++i) total[i] = 0.f;
  for (int s = 0; s < rows; s += 64) {
    const int sub = min(64, rows - s);
    float acc[kCPT];
#pragma unroll
    for (int i = 0; i < kCPT; ++i) acc[i] = 0.f;
    int r = 0;
    for (; r + 2 <= sub; r += 2) {
      float x0[kCPT], x1[kCPT];
      if (active) {
        load16<T>(kbase + (int64_t)(s + r) * HD, x0);
        load16<T>(kbase + (int64_t)(s + r + 1) * HD, x1);
      }
      float d0 = 0.f, d1 = 0.f;
#pragma unroll
      for (int i = 0; i < kCPT; ++i) {
        acc[i] = __fadd_rn(acc[i], x0[i]);
        acc[i] = __fadd_rn(acc[i], x1[i]);
        d0 = fmaf(a[i], x0[i], d0);
        d1 = fmaf(a[i], x1[i], d1);
      }
      if (need_logits) {
        d0 = group_sum<G>(d0);
        d1 = group_sum<G>(d1);
        if (active && glane == 0) {
          plog[h * block + s + r] = d0 * scale_log2;
          plog[h * block + s + r + 1] = d1 * scale_log2;
        }
      }
    }
    for (; r < sub; ++r) {
      float x0[kCPT];
      if (active) load16<T>(kbase + (int64_t)(s + r) * HD, x0);
      float d0 = 0.f;
#pragma unroll
      for (int i = 0; i < kCPT; ++i) {
        acc[i] = __fadd_rn(acc[i], x0[i]);
        d0 = fmaf(a[i], x0[i], d0);
      }
      if (need_logits) {
        d0 = group_sum<G>(d0);
        if (active && glane == 0) plog[h * block + s + r] = d0 * scale_log2;
      }
    }
#pragma unroll
    for (int i = 0; i < kCPT; ++i) total[i] = __fadd_rn(total[i], acc[i]);
  }
  if (kc != nullptr && active) {
    float out[kCPT];
#pragma unroll
    for (int i = 0; i < kCPT; ++i) out[i] = __fdiv_rn(total[i], (float)rows);
    T* dst = kc + (((int64_t)b * NB + kb) * H + h) * D + dcol;
    store8(dst, out);
    store8(dst + 8, out + 8);
  }
  if (!want_sum) return;

  // Softmax over the block's rows, per head (the G threads of a head cooperate).
  if (need_logits) {
    __syncthreads();
    float m = -INFINITY;
    if (active)
      for (int r = glane; r < rows; r += G) m = fmaxf(m, plog[h * block + r]);
    m = group_max<G>(m);
    float sum = 0.f;
    if (active)
      for (int r = glane; r < rows; r += G) {
        const float p = exp2f(plog[h * block + r] - m);
        plog[h * block + r] = p;
        sum += p;
      }
    sum = group_sum<G>(sum);
    if (active && glane == 0) {
      head_max[h] = m;
      head_den[h] = sum;
    }
    __syncthreads();
  }
  // Inactive lanes (H*D not a multiple of 512) stay for the group shuffles below.
  const float maximum = need_logits && active ? head_max[h] : 0.f;
  const float den = need_logits && active ? head_den[h] : 1.f;

  // Pass 2: weighted (or plain) means of K and V.
  float sk[kCPT], sv[kCPT];
#pragma unroll
  for (int i = 0; i < kCPT; ++i) sk[i] = sv[i] = 0.f;
  for (int r = 0; active && r < rows; ++r) {
    float x[kCPT], y[kCPT];
    load16<T>(kbase + (int64_t)r * HD, x);
    load16<T>(vbase + (int64_t)r * HD, y);
    // The probability enters the weighted sums rounded to the K/V dtype (the reference's
    // tensor-core summaries), or in fp32 with SB_SUMMARY_FP32_WEIGHTS (its comfy_fp32 mode).
    const float pr = plog[h * block + r];
    const float w = weighted_kv ? ((numerics & SB_SUMMARY_FP32_WEIGHTS) ? pr : Elem<T>::to_f(Elem<T>::from_f(pr))) : 1.f;
#pragma unroll
    for (int i = 0; i < kCPT; ++i) {
      sk[i] = fmaf(w, x[i], sk[i]);
      sv[i] = fmaf(w, y[i], sv[i]);
    }
  }
  const float norm = weighted_kv ? den : (float)rows;
  float key_out[kCPT], val_out[kCPT];
  float shift = 0.f;
#pragma unroll
  for (int i = 0; i < kCPT; ++i) {
    const float key = sk[i] / norm;
    key_out[i] = Elem<T>::to_f(Elem<T>::from_f(key));
    val_out[i] = sv[i] / norm;
    // The log-mass shift uses the stored (rounded) key, or the fp32 mean with
    // SB_SUMMARY_PRE_ROUND_LOGMASS.
    shift = fmaf(a[i], (numerics & SB_SUMMARY_PRE_ROUND_LOGMASS) ? key : key_out[i], shift);
  }
  const int64_t srow = (((int64_t)b * H + h) * NB + kb) * D + dcol;
  if (ak && active) {
    store8(ak + srow, key_out);
    store8(ak + srow + 8, key_out + 8);
  }
  if (av && active) {
    store8(av + srow, val_out);
    store8(av + srow + 8, val_out + 8);
  }
  shift = group_sum<G>(shift);
  if (lm != nullptr && active && glane == 0) {
    const float value = mass_bias ? (maximum + log2f(den)) * kLn2 - shift * scale : logf((float)rows);
    lm[((int64_t)b * H + h) * NB + kb] = value;
  }
}


// bf16 K/V: one CTA per (key block, head, batch entry).  The block's K and V rows of the
// head are staged in shared memory by 16-byte cp.async copies, so each is read from HBM
// exactly once (the all-heads kernel above re-reads K for its weighted sums); the key
// means (canonical order), the anchor logits, the block softmax and the weighted means
// then run out of shared memory.  Three CTAs fit an SM, so one CTA's copies overlap
// another's arithmetic.  Heads are the fastest grid index (x = key block * H + head), so
// the CTAs in flight read whole token rows of consecutive blocks.
constexpr int kHeadThreads = 256;

template <int D, int BLOCK>
struct HeadSmem {
  static constexpr size_t kTile = (size_t)BLOCK * D * sizeof(__nv_bfloat16);
  // K tile, V tile, logits [BLOCK], mean partials [2][D], anchor [D], statistics
  static constexpr size_t kBytes = 2 * kTile + BLOCK * sizeof(float) + 3 * D * sizeof(float) + 64;
  // The weighted-sum partials ([kHeadThreads / (D / 8)][D] for K and for V) reuse the tiles.
  static_assert(2 * (kHeadThreads / (D / 8)) * D * sizeof(float) <= 2 * kTile, "partials must fit the tiles");
};

template <typename TA, int D, int BLOCK>
__global__ void __launch_bounds__(kHeadThreads)
kv_summaries_head_kernel(const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
                         const TA* __restrict__ anchor, int T_, int H, int weighted_kv, int mass_bias, int numerics,
                         __nv_bfloat16* __restrict__ kc, __nv_bfloat16* __restrict__ ak,
                         __nv_bfloat16* __restrict__ av, float* __restrict__ lm) {
  using S = HeadSmem<D, BLOCK>;
  constexpr int CH = D * 2 / 16;  // 16-byte chunks per row
  extern __shared__ __align__(16) uint8_t head_smem[];
  __nv_bfloat16* ks = reinterpret_cast<__nv_bfloat16*>(head_smem);
  __nv_bfloat16* vs = reinterpret_cast<__nv_bfloat16*>(head_smem + S::kTile);
  float* plog = reinterpret_cast<float*>(head_smem + 2 * S::kTile);  // [BLOCK]
  float* part_k = plog + BLOCK;                                     // [2][D] key-mean partials
  float* a_s = part_k + 2 * D;                                      // [D] anchor
  float* stat = a_s + D;                                            // max, den, 8 warp partials

  const int kb = blockIdx.x / H, h = blockIdx.x % H, b = blockIdx.y;
  const int NB = ceil_div(T_, BLOCK);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row0 = kb * BLOCK;
  const int rows = min(BLOCK, T_ - row0);
  const bool want_sum = (ak != nullptr || av != nullptr || lm != nullptr);
  const bool need_logits = want_sum && (weighted_kv || mass_bias);
  const float scale = rsqrtf((float)D);
  const float scale_log2 = scale * kLog2e;
  const int64_t HD = (int64_t)H * D;
  const __nv_bfloat16* kbase = k + ((int64_t)b * T_ + row0) * HD + (int64_t)h * D;

  // The anchor row is fetched into a register before the tiles are waited on, so its L2
  // latency overlaps the K and V copies instead of following the key means.
  float anchor_col = 0.f;
  if (need_logits && tid < D) anchor_col = Elem<TA>::to_f(anchor[((int64_t)b * H + h) * D + tid]);
  for (int i = tid; i < rows * CH; i += kHeadThreads) {
    const int r = i / CH, c = i % CH;
    cp_async16(ks + r * D + c * 8, kbase + r * HD + c * 8);
  }
  cp_async_commit();
  if (want_sum) {
    const __nv_bfloat16* vbase = v + ((int64_t)b * T_ + row0) * HD + (int64_t)h * D;
    for (int i = tid; i < rows * CH; i += kHeadThreads) {
      const int r = i / CH, c = i % CH;
      cp_async16(vs + r * D + c * 8, vbase + r * HD + c * 8);
    }
  }
  cp_async_commit();
  if (need_logits && tid < D) a_s[tid] = anchor_col;
  cp_async_wait<1>();  // K has landed; V may still be in flight
  __syncthreads();

  constexpr int OCT = D / 8;                  // 8-column octets of a row (one 16-byte chunk)
  constexpr int GROUPS = kHeadThreads / OCT;  // row groups of the weighted sums
  const int oct = tid % OCT, grp = tid / OCT;
  // Key means: thread (column pair c, sub-block s) sums columns 2c, 2c + 1 over the rows of
  // 64-row sub-block s in token order (two chains, one 32-bit read per row); the sub-block
  // sums are then added in order and divided by the rows present (the canonical order).
  const int nsub = (rows + 63) / 64;
  {
    const int pair = tid % (D / 2), sb = tid / (D / 2);
    if (sb < nsub) {
      float acc0 = 0.f, acc1 = 0.f;
      const int r1 = min(rows, 64 * sb + 64);
      const __nv_bfloat162* src = reinterpret_cast<const __nv_bfloat162*>(ks) + pair;
      if (r1 - 64 * sb == 64) {
        // A full sub-block: 16 rows' reads are issued ahead of their (in-order) adds.
#pragma unroll 16
        for (int r = 64 * sb; r < 64 * sb + 64; ++r) {
          const float2 f = __bfloat1622float2(src[r * (D / 2)]);
          acc0 = __fadd_rn(acc0, f.x);
          acc1 = __fadd_rn(acc1, f.y);
        }
      } else {
        for (int r = 64 * sb; r < r1; ++r) {
          const float2 f = __bfloat1622float2(src[r * (D / 2)]);
          acc0 = __fadd_rn(acc0, f.x);
          acc1 = __fadd_rn(acc1, f.y);
        }
      }
      part_k[sb * D + 2 * pair] = acc0;
      part_k[sb * D + 2 * pair + 1] = acc1;
    }
  }
  // Anchor logits: PER = 256 / BLOCK threads per row, each a dot over D / PER columns in
  // 16-byte chunks.  Chunk order is rotated by (thread & 7), so the eight threads of a
  // shared-memory phase read eight different bank groups; the anchor sits in shared memory.
  constexpr int PER = kHeadThreads / BLOCK;  // 2 (128-row blocks) or 4 (64-row blocks)
  constexpr int CPT = D / 8 / PER;          // 16-byte chunks per thread
  if (need_logits) {
    const int r = tid / PER, part = tid % PER;
    float d0 = 0.f, d1 = 0.f;
    if (r < rows) {
#pragma unroll
      for (int j = 0; j < CPT; ++j) {
        const int chunk = part * CPT + ((j + tid) & (CPT - 1));
        const uint4 raw = *reinterpret_cast<const uint4*>(ks + r * D + chunk * 8);
        const float4 a0 = *reinterpret_cast<const float4*>(a_s + chunk * 8);
        const float4 a1 = *reinterpret_cast<const float4*>(a_s + chunk * 8 + 4);
        const __nv_bfloat162* x = reinterpret_cast<const __nv_bfloat162*>(&raw);
        const float2 x0 = __bfloat1622float2(x[0]), x1 = __bfloat1622float2(x[1]);
        const float2 x2 = __bfloat1622float2(x[2]), x3 = __bfloat1622float2(x[3]);
        d0 = fmaf(a0.x, x0.x, d0);
        d1 = fmaf(a0.y, x0.y, d1);
        d0 = fmaf(a0.z, x1.x, d0);
        d1 = fmaf(a0.w, x1.y, d1);
        d0 = fmaf(a1.x, x2.x, d0);
        d1 = fmaf(a1.y, x2.y, d1);
        d0 = fmaf(a1.z, x3.x, d0);
        d1 = fmaf(a1.w, x3.y, d1);
      }
    }
    float d = d0 + d1;
#pragma unroll
    for (int o = PER / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
    if (r < rows && part == 0) plog[r] = d * scale_log2;
  }
  __syncthreads();
  if (kc != nullptr && tid < D) {
    float total = 0.f;
    for (int sb = 0; sb < nsub; ++sb) total = __fadd_rn(total, part_k[sb * D + tid]);
    kc[(((int64_t)b * NB + kb) * H + h) * D + tid] = __float2bfloat16_rn(__fdiv_rn(total, (float)rows));
  }
  if (!want_sum) return;

  // Softmax over the block's rows (warp 0).
  if (need_logits && warp == 0) {
    float m = -INFINITY;
    for (int r = lane; r < rows; r += 32) m = fmaxf(m, plog[r]);
    m = warp_max(m);
    float sum = 0.f;
    for (int r = lane; r < rows; r += 32) {
      const float pr = exp2f(plog[r] - m);
      plog[r] = pr;
      sum += pr;
    }
    sum = warp_sum(sum);
    if (lane == 0) {
      stat[0] = m;
      stat[1] = sum;
    }
  }
  cp_async_wait<0>();
  __syncthreads();
  const float maximum = need_logits ? stat[0] : 0.f;
  const float den = need_logits ? stat[1] : 1.f;

  // Weighted (or plain) sums: thread (octet o, group g) accumulates the 8 columns of octet o
  // over rows g, g + GROUPS, ... from 16-byte shared-memory reads.  The probability enters
  // rounded to bf16 (the reference's tensor-core summaries), or in fp32 with
  // SB_SUMMARY_FP32_WEIGHTS (its comfy_fp32 mode).  The group partials are then summed per
  // column, in group order, through shared memory (the K tile's space, no longer read).
  float sk[8], sv[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) sk[e] = sv[e] = 0.f;
  for (int r = grp; r < rows; r += GROUPS) {
    const float pr = plog[r];
    const float w = weighted_kv ? ((numerics & SB_SUMMARY_FP32_WEIGHTS) ? pr : __bfloat162float(__float2bfloat16_rn(pr)))
                                : 1.f;
    const uint4 kraw = *reinterpret_cast<const uint4*>(ks + r * D + oct * 8);
    const uint4 vraw = *reinterpret_cast<const uint4*>(vs + r * D + oct * 8);
    const __nv_bfloat162* kx = reinterpret_cast<const __nv_bfloat162*>(&kraw);
    const __nv_bfloat162* vx = reinterpret_cast<const __nv_bfloat162*>(&vraw);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 kf = __bfloat1622float2(kx[e]), vf = __bfloat1622float2(vx[e]);
      sk[2 * e] = fmaf(w, kf.x, sk[2 * e]);
      sk[2 * e + 1] = fmaf(w, kf.y, sk[2 * e + 1]);
      sv[2 * e] = fmaf(w, vf.x, sv[2 * e]);
      sv[2 * e + 1] = fmaf(w, vf.y, sv[2 * e + 1]);
    }
  }
  __syncthreads();  // every K and V read is done: the tiles' space takes the partials
  float* red_k = reinterpret_cast<float*>(head_smem);  // [GROUPS][D]
  float* red_v = red_k + GROUPS * D;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    red_k[grp * D + oct * 8 + e] = sk[e];
    red_v[grp * D + oct * 8 + e] = sv[e];
  }
  __syncthreads();
  if (tid < D) {
    const int col = tid;
    float sum_k = 0.f, sum_v = 0.f;
    for (int g = 0; g < GROUPS; ++g) {
      sum_k += red_k[g * D + col];
      sum_v += red_v[g * D + col];
    }
    const float norm = weighted_kv ? den : (float)rows;
    const float key = sum_k / norm;
    const __nv_bfloat16 key_b = __float2bfloat16_rn(key);
    const int64_t srow = (((int64_t)b * H + h) * NB + kb) * D + col;
    if (ak) ak[srow] = key_b;
    if (av) av[srow] = __float2bfloat16_rn(sum_v / norm);
    // Log-mass shift: a . key over the head's columns, from the stored (rounded) key or, with
    // SB_SUMMARY_PRE_ROUND_LOGMASS, the fp32 mean.
    float shift = 0.f;
    if (lm != nullptr && mass_bias) {
      const float a_c = a_s[col];  // written at the start: mass_bias implies need_logits
      shift = a_c * ((numerics & SB_SUMMARY_PRE_ROUND_LOGMASS) ? key : __bfloat162float(key_b));
    }
    shift = warp_sum(shift);
    if (lane == 0) stat[2 + warp] = shift;
  }
  __syncthreads();
  if (tid == 0 && lm != nullptr) {
    float shift = 0.f;
    for (int w = 0; w < D / 32; ++w) shift += stat[2 + w];
    lm[((int64_t)b * H + h) * NB + kb] =
        mass_bias ? (maximum + log2f(den)) * kLn2 - shift * scale : logf((float)rows);
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
                            int block, int weighted_kv, int mass_bias, int numerics, void* kc, void* ak,
                            void* av, float* lm, cudaStream_t s) {
  const int NB = ceil_div(tokens, block);
  const int threads = ceil_div(H * D / kCPT, 32) * 32;
  if (threads > 256 || H > 64) {
    set_error("sb_pool_keys_summaries: H * D must be at most 4096 and H at most 64");
    return SB_ERR_INVALID;
  }
  const size_t smem = (size_t)H * block * sizeof(float);
  auto kern = pool_keys_summaries_kernel<T, TA, D>;
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return cuda_error(err, "sb_pool_keys_summaries: set smem");
  dim3 grid(NB, B);
  kern<<<grid, threads, smem, s>>>((const T*)k, (const T*)v, (const TA*)anchor, tokens, H, block, weighted_kv,
                              mass_bias, numerics, (T*)kc, (T*)ak, (T*)av, lm);
  SB_CHECK_LAUNCH("sb_pool_keys_summaries launch");
  return SB_OK;
}

template <typename TA, int D, int BLOCK>
static int launch_kv_head(const void* k, const void* v, const void* anchor, int B, int tokens, int H,
                          int weighted_kv, int mass_bias, int numerics, void* kc, void* ak, void* av, float* lm,
                          cudaStream_t s) {
  const size_t smem = HeadSmem<D, BLOCK>::kBytes;
  auto kern = kv_summaries_head_kernel<TA, D, BLOCK>;
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return cuda_error(err, "sb_pool_keys_summaries: set smem");
  if ((int64_t)ceil_div(tokens, BLOCK) * H >= (1ll << 31) || B > 65535) {
    set_error("sb_pool_keys_summaries: too many key blocks x heads");
    return SB_ERR_INVALID;
  }
  dim3 grid(ceil_div(tokens, BLOCK) * H, B);
  kern<<<grid, kHeadThreads, smem, s>>>((const __nv_bfloat16*)k, (const __nv_bfloat16*)v, (const TA*)anchor, tokens,
                                        H, weighted_kv, mass_bias, numerics, (__nv_bfloat16*)kc,
                                        (__nv_bfloat16*)ak, (__nv_bfloat16*)av, lm);
  SB_CHECK_LAUNCH("sb_pool_keys_summaries launch");
  return SB_OK;
}

template <typename TA>
static int launch_kv_head_for(int D, int block, const void* k, const void* v, const void* anchor, int B, int tokens,
                              int H, int weighted_kv, int mass_bias, int numerics, void* kc, void* ak, void* av,
                              float* lm, cudaStream_t s) {
  if (D == 128)
    return block == 128 ? launch_kv_head<TA, 128, 128>(k, v, anchor, B, tokens, H, weighted_kv, mass_bias, numerics, kc, ak, av, lm, s)
                        : launch_kv_head<TA, 128, 64>(k, v, anchor, B, tokens, H, weighted_kv, mass_bias, numerics, kc, ak, av, lm, s);
  return block == 128 ? launch_kv_head<TA, 64, 128>(k, v, anchor, B, tokens, H, weighted_kv, mass_bias, numerics, kc, ak, av, lm, s)
                      : launch_kv_head<TA, 64, 64>(k, v, anchor, B, tokens, H, weighted_kv, mass_bias, numerics, kc, ak, av, lm, s);
}

extern "C" int sb_pool_keys_summaries(const void* k, const void* v, const void* anchor, int dtype,
                                      int anchor_dtype, int B, int T, int H, int D, int block,
                                      int weighted_kv, int mass_bias, int numerics, void* kc, void* ak,
                                      void* av, float* lm, void* stream) {
  const bool want_sum = ak || av || lm;
  SB_CHECK_ARG(k, "sb_pool_keys_summaries: null K");
  SB_CHECK_ARG(!want_sum || v, "sb_pool_keys_summaries: summaries need V");
  SB_CHECK_ARG(!want_sum || !(weighted_kv || mass_bias) || anchor,
               "sb_pool_keys_summaries: weighted summaries need the anchor");
  SB_CHECK_ARG(dtype == SB_F32 || dtype == SB_BF16, "sb_pool_keys_summaries: bad dtype");
  SB_CHECK_ARG((numerics & ~(SB_SUMMARY_PRE_ROUND_LOGMASS | SB_SUMMARY_FP32_WEIGHTS)) == 0,
               "sb_pool_keys_summaries: unknown numerics flags %d", numerics);
  SB_CHECK_ARG(anchor_dtype == SB_F32 || anchor_dtype == SB_BF16, "sb_pool_keys_summaries: bad anchor dtype");
  SB_CHECK_ARG(B > 0 && T > 0 && H > 0, "sb_pool_keys_summaries: B, T, H must be positive");
  SB_CHECK_ARG(D == 64 || D == 128, "sb_pool_keys_summaries: head dim must be 64 or 128");
  SB_CHECK_ARG(block == 64 || block == 128, "sb_pool_keys_summaries: block must be 64 or 128");
  SB_CHECK_ARG(((uintptr_t)k % 16) == 0 && (!v || ((uintptr_t)v % 16) == 0),
               "sb_pool_keys_summaries: K/V must be 16-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  const bool abf = anchor_dtype == SB_BF16;
  if (dtype == SB_BF16)  // one CTA per (key block, head): K and V read once
    return abf ? launch_kv_head_for<__nv_bfloat16>(D, block, k, v, anchor, B, T, H, weighted_kv, mass_bias, numerics,
                                                   kc, ak, av, lm, s)
               : launch_kv_head_for<float>(D, block, k, v, anchor, B, T, H, weighted_kv, mass_bias, numerics, kc, ak,
                                           av, lm, s);
  SB_CHECK_ARG(!abf, "sb_pool_keys_summaries: float32 K/V need a float32 anchor");
  if (D == 128)
    return launch_pool_keys<float, float, 128>(k, v, anchor, B, T, H, block, weighted_kv, mass_bias, numerics, kc, ak, av, lm, s);
  return launch_pool_keys<float, float, 64>(k, v, anchor, B, T, H, block, weighted_kv, mass_bias, numerics, kc, ak, av, lm, s);
}
