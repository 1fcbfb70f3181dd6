// Head-wise gather of the video prefix: dst[b, t, h, :] = src[b, perm[b, h, t], h, :].
// Each CTA writes whole [H*D] token rows, so stores are contiguous 16-byte vectors;
// each gathered (token, head) segment is a contiguous D-element read.
#include "common.cuh"

namespace sb {

constexpr int kPermuteRows = 8;

template <typename I>
__global__ void headwise_permute_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                        const I* __restrict__ perm, int T_, int H, int vec_per_head,
                                        int video_tokens) {
  const int b = blockIdx.y;
  const int row_vecs = H * vec_per_head;
  const int c = threadIdx.x;
  if (c >= row_vecs) return;
  const int h = c / vec_per_head;
  for (int rr = 0; rr < kPermuteRows; ++rr) {
    const int t = blockIdx.x * kPermuteRows + rr;
    if (t >= T_) return;
    int64_t s = t;
    if (t < video_tokens) s = (int64_t)__ldg(perm + ((int64_t)b * H + h) * video_tokens + t);
    dst[((int64_t)b * T_ + t) * row_vecs + c] = __ldg(src + ((int64_t)b * T_ + s) * row_vecs + c);
  }
}

}  // namespace sb

using namespace sb;

extern "C" int sb_headwise_permute(const void* src, void* dst, const void* perm, int index_bytes,
                                   int B, int T, int H, int D, int elem_bytes, int video_tokens,
                                   void* stream) {
  SB_CHECK_ARG(src && dst && perm, "sb_headwise_permute: null pointer");
  SB_CHECK_ARG(index_bytes == 4 || index_bytes == 8, "sb_headwise_permute: index_bytes must be 4 or 8");
  SB_CHECK_ARG(elem_bytes == 2 || elem_bytes == 4, "sb_headwise_permute: elem_bytes must be 2 or 4");
  SB_CHECK_ARG(B > 0 && T > 0 && H > 0 && D > 0, "sb_headwise_permute: sizes must be positive");
  SB_CHECK_ARG(video_tokens >= 0 && video_tokens <= T, "sb_headwise_permute: video_tokens is outside [0, T]");
  SB_CHECK_ARG((D * elem_bytes) % 16 == 0, "sb_headwise_permute: D * elem_bytes must be a multiple of 16");
  SB_CHECK_ARG(((uintptr_t)src % 16) == 0 && ((uintptr_t)dst % 16) == 0, "sb_headwise_permute: pointers must be 16-byte aligned");
  const int64_t bytes = (int64_t)B * T * H * D * elem_bytes;
  const char* s0 = (const char*)src;
  const char* d0 = (const char*)dst;
  SB_CHECK_ARG(d0 + bytes <= s0 || s0 + bytes <= d0, "sb_headwise_permute: src and dst overlap");
  const int vec_per_head = D * elem_bytes / 16;
  const int row_vecs = H * vec_per_head;
  SB_CHECK_ARG(row_vecs <= 1024, "sb_headwise_permute: H * D * elem_bytes must be at most 16 KiB");
  dim3 grid(ceil_div(T, kPermuteRows), B);
  cudaStream_t s = (cudaStream_t)stream;
  if (index_bytes == 4)
    headwise_permute_kernel<int32_t><<<grid, row_vecs, 0, s>>>((const uint4*)src, (uint4*)dst, (const int32_t*)perm, T, H, vec_per_head, video_tokens);
  else
    headwise_permute_kernel<int64_t><<<grid, row_vecs, 0, s>>>((const uint4*)src, (uint4*)dst, (const int64_t*)perm, T, H, vec_per_head, video_tokens);
  SB_CHECK_LAUNCH("sb_headwise_permute launch");
  return SB_OK;
}
