// Pointwise kernels of the synthetic DiT block stack, fused around the
// fp8 GEMMs and the head-sharded attention:
//   norm_modulate_quantize  RMSNorm of a hidden row, adaLN modulation x * (1 + scale) + shift,
//                           and the per-token e4m3 quantisation the next GEMM consumes
//   qkv_norm_rope           per-head RMSNorm of q and k (learned weight), 3-D rotary embedding
//                           over (t, h, w) coordinates, written straight into the layout of the
//                           sequence-to-head all-to-all: [shard][token][head in shard][dim]
#include "common.cuh"

namespace sb {
namespace {

constexpr int kNormThreads = 128;
constexpr int kMaxVec = 8;  // up to 8 x 8 x 128 = 8192 columns per row

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < kNormThreads / 32 ? red[lane] : 0.f;
  return warp_sum(t);
}

__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < kNormThreads / 32 ? red[lane] : 0.f;
  return warp_max(t);
}

// One CTA per row: y = x / rms(x) * (1 + scale) + shift, then e4m3 with one scale per row
// (scale = max(absmax * fp32(1/448), 1e-12), codes = sat_e4m3(y / scale)).
__global__ void __launch_bounds__(kNormThreads) norm_modulate_quantize_kernel(
    const __nv_bfloat16* __restrict__ x, const float* __restrict__ shift, const float* __restrict__ scale, int C,
    float eps, uint8_t* __restrict__ out, float* __restrict__ scales) {
  __shared__ float red[kNormThreads / 32];
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * C;
  float v[kMaxVec][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int c = (j * kNormThreads + threadIdx.x) * 8;
    if (c < C) {
      load8(xr + c, v[j]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(v[j][e], v[j][e], ss);
    }
  }
  const float rstd = rsqrtf(block_sum(ss, red) / (float)C + eps);
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int c = (j * kNormThreads + threadIdx.x) * 8;
    if (c < C) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        v[j][e] = fmaf(v[j][e] * rstd, 1.f + __ldg(scale + c + e), __ldg(shift + c + e));
        amax = fmaxf(amax, fabsf(v[j][e]));
      }
    }
  }
  amax = block_max(amax, red);
  const float q = fmaxf(amax * (1.0f / 448.0f), 1e-12f);
  if (threadIdx.x == 0) scales[row] = q;
  uint8_t* orow = out + row * C;
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int c = (j * kNormThreads + threadIdx.x) * 8;
    if (c < C) {
      uint16_t packed[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float lo = fminf(fmaxf(__fdiv_rn(v[j][2 * i], q), -448.f), 448.f);
        const float hi = fminf(fmaxf(__fdiv_rn(v[j][2 * i + 1], q), -448.f), 448.f);
        uint16_t pr;
        asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(pr) : "f"(hi), "f"(lo));
        packed[i] = pr;
      }
      *reinterpret_cast<uint2*>(orow + c) = *reinterpret_cast<uint2*>(packed);
    }
  }
}

constexpr int kRopeThreads = 256;  // 8 warps: heads h, h + 8, ... of one token
constexpr int kHeadDim = 128;

// One CTA per token.  The token's 64 rotation angles (pair j of the head dimension rotates by
// coord[axis(j)] * inv_freq[j]) are computed once and shared by every head.
__global__ void __launch_bounds__(kRopeThreads) qkv_norm_rope_kernel(
    const __nv_bfloat16* __restrict__ qkv, const float* __restrict__ wq, const float* __restrict__ wk,
    const int32_t* __restrict__ coords, const float* __restrict__ inv_freq, const int8_t* __restrict__ axis,
    int64_t M, int H, int shards, float eps, __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ k,
    __nv_bfloat16* __restrict__ v) {
  __shared__ float cs[kHeadDim / 2], sn[kHeadDim / 2];
  const int64_t m = blockIdx.x;
  if (threadIdx.x < kHeadDim / 2) {
    const int j = threadIdx.x;
    const float angle = (float)coords[m * 3 + axis[j]] * inv_freq[j];
    float s, c;
    sincosf(angle, &s, &c);
    cs[j] = c;
    sn[j] = s;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hp = H / shards;
  const __nv_bfloat16* row = qkv + m * 3 * H * kHeadDim;
  for (int h = warp; h < H; h += kRopeThreads / 32) {
    const int shard = h / hp, hl = h - shard * hp;
    const int64_t o = ((int64_t)(shard * M + m) * hp + hl) * kHeadDim + 4 * lane;
    for (int which = 0; which < 3; ++which) {
      const __nv_bfloat16* src = row + ((int64_t)which * H + h) * kHeadDim + 4 * lane;
      const uint2 raw = *reinterpret_cast<const uint2*>(src);
      if (which == 2) {
        *reinterpret_cast<uint2*>(v + o) = raw;
        continue;
      }
      const __nv_bfloat162* hv = reinterpret_cast<const __nv_bfloat162*>(&raw);
      const float2 a = __bfloat1622float2(hv[0]), b = __bfloat1622float2(hv[1]);
      float x[4] = {a.x, a.y, b.x, b.y};
      const float ss = warp_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]);
      const float rstd = rsqrtf(ss / (float)kHeadDim + eps);
      const float* w = which == 0 ? wq : wk;
#pragma unroll
      for (int e = 0; e < 4; ++e) x[e] = x[e] * rstd * __ldg(w + 4 * lane + e);
      float y[4];
#pragma unroll
      for (int pr = 0; pr < 2; ++pr) {
        const int j = 2 * lane + pr;  // pair (4 lane + 2 pr, 4 lane + 2 pr + 1)
        const float c = cs[j], s = sn[j];
        y[2 * pr] = x[2 * pr] * c - x[2 * pr + 1] * s;
        y[2 * pr + 1] = x[2 * pr] * s + x[2 * pr + 1] * c;
      }
      __nv_bfloat162 out2[2] = {__floats2bfloat162_rn(y[0], y[1]), __floats2bfloat162_rn(y[2], y[3])};
      *reinterpret_cast<uint2*>((which == 0 ? q : k) + o) = *reinterpret_cast<uint2*>(out2);
    }
  }
}

}  // namespace
}  // namespace sb

using namespace sb;

extern "C" int sb_dit_norm_modulate_quantize(const void* x, const float* shift, const float* scale, int64_t M, int C,
                                             float eps, uint8_t* out, float* scales, void* stream) {
  SB_CHECK_ARG(x && shift && scale && out && scales, "sb_dit_norm_modulate_quantize: null pointer");
  SB_CHECK_ARG(M > 0 && M < (1ll << 31), "sb_dit_norm_modulate_quantize: bad row count");
  SB_CHECK_ARG(C > 0 && C % 8 == 0 && C <= kMaxVec * kNormThreads * 8,
               "sb_dit_norm_modulate_quantize: C must be a multiple of 8 up to %d", kMaxVec * kNormThreads * 8);
  SB_CHECK_ARG(((uintptr_t)x % 16) == 0 && ((uintptr_t)out % 8) == 0,
               "sb_dit_norm_modulate_quantize: x must be 16-byte and out 8-byte aligned");
  norm_modulate_quantize_kernel<<<(unsigned)M, kNormThreads, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)x, shift, scale, C, eps, out, scales);
  SB_CHECK_LAUNCH("sb_dit_norm_modulate_quantize launch");
  return SB_OK;
}

extern "C" int sb_dit_qkv_norm_rope(const void* qkv, const float* wq, const float* wk, const int32_t* coords,
                                    const float* inv_freq, const int8_t* axis, int64_t M, int H, int D, int shards,
                                    float eps, void* q, void* k, void* v, void* stream) {
  SB_CHECK_ARG(qkv && wq && wk && coords && inv_freq && axis && q && k && v, "sb_dit_qkv_norm_rope: null pointer");
  SB_CHECK_ARG(D == kHeadDim, "sb_dit_qkv_norm_rope: head dimension must be 128, got %d", D);
  SB_CHECK_ARG(M > 0 && M < (1ll << 31) && H > 0 && shards > 0 && H % shards == 0,
               "sb_dit_qkv_norm_rope: heads must split evenly across shards");
  qkv_norm_rope_kernel<<<(unsigned)M, kRopeThreads, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)qkv, wq, wk, coords, inv_freq, axis, M, H, shards, eps, (__nv_bfloat16*)q,
      (__nv_bfloat16*)k, (__nv_bfloat16*)v);
  SB_CHECK_LAUNCH("sb_dit_qkv_norm_rope launch");
  return SB_OK;
}
