// Parameters and exact-block rule shared by the sparse attention kernels.
#pragma once

#include "common.cuh"

namespace sb {

struct AttnParams {
  const void* q;
  const void* k;
  const void* v;
  const int32_t* packed;  // [B, QB, H, words]
  const void* ak;         // [B, H, NB, D]
  const void* av;         // [B, H, NB, D]
  const float* lm;        // [B, H, NB]
  void* out;              // [B, T, H, D]
  float* lse;             // [B, T, H] or null
  int* status;            // device status word (bounded waits)
  int B, T, H, block, NB, QB, words;
  int query_tokens, sink_first, sink_last, local_radius;
  int row_lo, row_hi;     // query rows computed and stored: [row_lo, row_hi)
  // Optional query-block pairs (64-token blocks, sm100 kernel): tile t of (b, h) holds blocks
  // pairs[((b * H + h) * pair_tiles + t) * 2 + {0, 1}] (-1: no block); rows past the routed
  // prefix form 128-row tiles from query_tokens on.  Null: tile t holds rows 128 t .. 128 t + 127.
  const int32_t* pairs;
  int pair_tiles;
};

// Key block kb is evaluated exactly for routed query block qb when the route marks it,
// when it lies in the sink range, or when it is within the explicit local radius.
// Mirrors sol_attn/sm90/mainloop.py:590-667 for packed external routes.
__host__ __device__ __forceinline__ bool block_is_exact(const int32_t* words, int kb, int qb,
                                                        int sink_first, int sink_last,
                                                        int local_radius) {
  if ((words[kb >> 5] >> (kb & 31)) & 1) return true;
  if (kb >= sink_first && kb < sink_last) return true;
  if (local_radius >= 0) {
    const int dist = qb > kb ? qb - kb : kb - qb;
    if (dist <= local_radius) return true;
  }
  return false;
}

int launch_sparse_attention_simt(const AttnParams& p, int dtype, int D, cudaStream_t s);
int launch_sparse_attention_sm100(const AttnParams& p, cudaStream_t s);

}  // namespace sb
