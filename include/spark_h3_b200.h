/*
 * spark_h3_b200.h -- C ABI of the B200 (sm_100a) Spark-H3 sparse-attention hot path.
 *
 * Every entry point takes plain device pointers, explicit sizes and a cudaStream_t
 * passed as void*.  Nothing here allocates device memory: outputs and workspaces are
 * owned by the caller.  No entry point synchronises the host with the device.
 * Return value: 0 on success, a negative SB_ERR_* code on failure; sb_last_error()
 * returns the message of the last failure on the calling host thread.
 *
 * Tensor layouts (row-major, innermost last):
 *   Q, K, V, O        [B, T, H, D]        token-major "BTHD", as the reference's
 *                                          spark_attention_bthd consumes them
 *   query block means [B, NB, H, D] fp32  NB = ceil(T / block)
 *   key block means   [B, NB, H, D] dtype
 *   anchor            [B, H, D]     dtype (one global video anchor per head)
 *   AK, AV            [B, H, NB, D] dtype (anchor-weighted key/value summaries)
 *   LM                [B, H, NB]    fp32  (log-mass correction, natural log)
 *   packed route      [B, QB, H, W] int32 W = ceil(NB / 32); bit (kb % 32) of word
 *                                          (kb / 32) marks key block kb as exact
 *   top-k indices     [B, QB, H, k] int32 ascending block indices
 *   LSE               [B, T, H]     fp32  natural-log softmax normaliser
 *
 * dtype codes: SB_F32 (float32) or SB_BF16 (bfloat16).  The tensor-core attention
 * path handles bf16 with D = 128; float32 inputs or D = 64 use the SIMT path of the
 * same library (still on the GPU).  Block sizes 64 and 128 are supported.
 */
#ifndef SPARK_H3_B200_H
#define SPARK_H3_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SB_F32 0
#define SB_BF16 1

#define SB_OK 0
#define SB_ERR_INVALID -1     /* bad argument: shape, dtype, alignment, null pointer */
#define SB_ERR_CUDA -2        /* a CUDA runtime/driver call failed */
#define SB_ERR_UNSUPPORTED -3 /* valid arguments this build does not implement */

/* Library version (major * 10000 + minor * 100 + patch). */
int sb_version(void);

/* Message of the last failing call on this host thread ("" if none). */
const char* sb_last_error(void);

/* Device-side status word written by kernels whose waits are bounded.  Returns the
 * value the last completed kernel left in it (0 = no timeout) and clears it.  This
 * is the only entry point that synchronises the stream. */
int sb_read_device_status(void* stream);

/*
 * Self-check of the bounded waits every kernel uses (no counterpart in the reference): one
 * CTA whose warp 0 waits on an mbarrier that nothing arrives on, for limit_cycles, then raises
 * the CTA abort flag and records SB_SELFTEST_WAIT_SITE in the device status word; warp 1,
 * waiting on another such barrier with the normal two-second limit, must leave when the flag
 * rises.  result (device, 4 ints): per warp, whether its wait succeeded (expected 0) and
 * whether it left within a bounded time (expected 1).  Nothing faults; the context stays
 * usable.  limit_cycles in (0, 1e8].
 */
#define SB_SELFTEST_WAIT_SITE 990
int sb_selftest_wait_timeout(long long limit_cycles, int* result, void* stream);

/*
 * Peer memory between the processes of one node (one per GPU; no counterpart in the
 * reference): sb_ipc_alloc allocates a device buffer whose CUDA IPC handle (64 bytes,
 * sb_ipc_handle) another process maps with sb_ipc_open (peer access enabled lazily) and
 * unmaps with sb_ipc_close; sb_ipc_free releases the allocation.
 */
int sb_ipc_alloc(int64_t bytes, void** ptr);
int sb_ipc_free(void* ptr);
int sb_ipc_handle(const void* ptr, uint8_t* handle);
int sb_ipc_open(const uint8_t* handle, void** ptr);
int sb_ipc_close(void* ptr);

/*
 * Query block pooling.  Replaces the query-centroid half of
 * h3_sparse_attention/spark_integration.py:111-127 (_sol_topk_policy_scores) and the
 * per-64-row partial sums of sol_numerator_virtual_q.py:268-285 (_anchor_parts).
 * qc[b, j, h, :] = (sum of the rows of block j, fp32, rows in order) / rows_in_block.
 */
int sb_pool_queries(const void* q, int dtype, int B, int T, int H, int D, int block,
                    float* qc, void* stream);

/*
 * Global video anchor of each head, from the query block means.  Replaces
 * sol_numerator_virtual_q.py:287-302 (_anchors_from_parts / build_virtual_anchors for
 * the single global parent of landmark_virtual_q.py:54-65 with levels_up = 99).
 * anchor[b, h, :] = (sum_j qc[b, j, h, :] * block) / (prefix_blocks * block), j in
 * order, then rounded to anchor_dtype.
 */
int sb_query_anchor(const float* qc, int B, int NB, int H, int D, int block,
                    int prefix_blocks, void* anchor, int anchor_dtype, void* stream);

/*
 * One pass over K and V: key block means (routing) and anchor-weighted summaries.
 * Replaces sol_attn/preprocess.py:16-52 (_reduce_kc_kernel) and
 * sol_numerator_virtual_q.py:93-135 (_summaries) for the global parent.
 * weighted_kv != 0: AK/AV are softmax(anchor . k / sqrt(D))-weighted means, else plain
 * means.  mass_bias != 0: LM = logsumexp(a.k/sqrt(D)) - a.AK_stored/sqrt(D), else
 * LM = log(rows in block).  Any of kc / ak / av / lm may be NULL to skip that output
 * (anchor may be NULL when ak, av and lm are all NULL).  numerics selects the reference's
 * summary ablations (sol_numerator_virtual_q.py:93-193, processor.py:61-68): 0 is its
 * default (probabilities rounded to the K/V dtype in the weighted sums, LM shift from the
 * stored key); SB_SUMMARY_PRE_ROUND_LOGMASS takes the shift from the fp32 key mean
 * (sol_reweight_logmass_key = "pre_round"); SB_SUMMARY_FP32_WEIGHTS keeps the
 * probabilities in fp32 (sol_reweight_summary_math = "comfy_fp32").
 */
#define SB_SUMMARY_PRE_ROUND_LOGMASS 1
#define SB_SUMMARY_FP32_WEIGHTS 2
int sb_pool_keys_summaries(const void* k, const void* v, const void* anchor,
                           int dtype, int anchor_dtype, int B, int T, int H, int D,
                           int block, int weighted_kv, int mass_bias, int numerics,
                           void* kc, void* ak, void* av, float* lm, void* stream);

/*
 * Block scores and per-row Top-K.  Replaces spark_integration.py:94-175
 * (_sol_topk_policy_scores + _sol_topk_route_from_scores) and
 * sol_topk_cutoff.py:416-480 (gemm_topk_packed_route, including the packing kernel
 * at :19-44).  score[b, i, h, j] = fp32(dot(qc[b,i,h,:], kc[b,j,h,:])) * scale_log2
 * for j < candidates (dot = sequential fused multiply-add over d); each row keeps the
 * topk largest scores, ties going to the lower block index.  packed_route must hold
 * B*QB*H*ceil(NB/32) words; bits >= candidates are never set.
 * workspace: at least sb_route_workspace_bytes(B, QB, H, candidates) bytes.
 * indices may be NULL.
 */
int64_t sb_route_workspace_bytes(int B, int QB, int H, int candidates);
int sb_route_topk(const float* qc, const void* kc, int kc_dtype, int B, int QB, int NB,
                  int H, int D, int candidates, int topk, float scale_log2,
                  void* workspace, int32_t* packed_route, int32_t* indices,
                  void* stream);

/*
 * Top-K with one budget per head.  Replaces head_budget.py:7-19 (route_with_head_budgets,
 * reached from spark_integration.py:1344-1351 when the controller carries
 * head_topk_budget): row (b, i, h) keeps the head_topk[h] largest of its candidate scores
 * in stable descending order (ties to the lower block index), the budget clamped to
 * [0, candidates].  head_topk: device int32 [H].  Scores, packed_route and the workspace are
 * as for sb_route_topk.  indices (may be NULL) is [B, QB, H, index_width] with
 * 1 <= index_width <= candidates: a row's ascending selections, -1 past its budget; a budget
 * above index_width fills the row and the remaining selections appear only in packed_route.
 * The caller makes the blocks past the candidates exact (the reference routes every block
 * >= candidates when there are sink tokens or a partial video block).
 */
int sb_route_topk_head_budgets(const float* qc, const void* kc, int kc_dtype, int B, int QB, int NB,
                               int H, int D, int candidates, const int32_t* head_topk,
                               int index_width, float scale_log2, void* workspace,
                               int32_t* packed_route, int32_t* indices, void* stream);

/*
 * Allocation-free variant of sb_route_topk; no counterpart in the reference.
 * For callers that cannot pass a device workspace, for instance a host that binds only this
 * library through a thin FFI and owns no device allocator, or a serving loop that cannot
 * accept the device synchronisation cudaMalloc implies.  The block scores live in a
 * file-scope device array of SB_ROUTE_NOALLOC_SCRATCH_FLOATS floats (16 MiB), which every GPU
 * that loads the library holds until the process exits.  Query blocks are processed in
 * chunks that fit it, so the outputs equal sb_route_topk's; sizes with
 * H * candidates > SB_ROUTE_NOALLOC_SCRATCH_FLOATS are rejected with SB_ERR_INVALID.
 * No cudaMalloc, cudaFree or allocating library routine is called.  The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress) and caches it; make
 * that first call before any stream capture.  All calls share the one array: calls that
 * overlap on the GPU (other streams, other host threads) race and must be serialised by
 * the caller.  Every score a call reads was written earlier in the same call.
 */
#define SB_ROUTE_NOALLOC_SCRATCH_FLOATS (4 * 1024 * 1024)
int sb_route_topk_noalloc(const float* qc, const void* kc, int kc_dtype, int B, int QB, int NB,
                          int H, int D, int candidates, int topk, float scale_log2,
                          int32_t* packed_route, int32_t* indices, void* stream);

/*
 * Sparse attention forward.  Replaces sol_numerator_virtual_q.py:717-977
 * (_fused_virtual -> SparkReweightForwardSm*) with the semantics of the streamed
 * oracle at sol_numerator_virtual_q.py:596-652 and
 * tests/test_spark_installer.py:559-570:
 *   for a query row in routed query block i (i < query_tokens / block):
 *     exact key blocks E = route bits of (b, i, h)  U  [sink_first, sink_last)
 *                          U  {|i - kb| <= local_radius}  (local_radius < 0: none)
 *     logits = q.k / sqrt(D) over the tokens of E, and q.AK[kb] / sqrt(D) + LM[kb]
 *     over every key block kb not in E; O = softmax(logits) @ [V ; AV].
 *   rows >= query_tokens attend every key exactly (the dense suffix).
 * packed_route: [B, QB, H, ceil(NB/32)] with QB >= query_tokens / block.
 * ak/av/lm: summaries of the single global parent ([B, H, NB, D] / [B, H, NB]); all three
 * NULL leaves the summary columns out, so routed rows attend their exact blocks only (the
 * exact_attention stage of the reference's block tails, sol_numerator_virtual_q.py:655-660).
 * lse may be NULL.
 */
int sb_sparse_attention(const void* q, const void* k, const void* v, int dtype,
                        int B, int T, int H, int D, int block,
                        const int32_t* packed_route, int QB,
                        const void* ak, const void* av, const float* lm,
                        int query_tokens, int sink_first, int sink_last,
                        int local_radius, void* out, float* lse, void* stream);

/*
 * Pairing of 64-token query blocks for the tensor-core kernel (no reference counterpart: a
 * scheduling choice of this library; the reference runs one 64-row block per tile,
 * spark_reweight_sm100.py:1495-1700).  Its 128-row tiles hold two query blocks and do the
 * exact key work of the union of their route sets; this pairs, per (b, h) and in block
 * order, each unpaired block among the first `blocks` of packed_route with the unpaired block
 * of the largest route overlap among the next 64 (ties: the nearer), then the blocks left
 * without a partner with each other in order.
 * packed_route: [B, QB, H, words] (words <= 256); pairs: [B, H, ceil(blocks/2), 2] int32,
 * -1 for the empty half of an odd count.  workspace: sb_route_pair_workspace_bytes(B, H,
 * blocks) bytes of device memory.
 */
int64_t sb_route_pair_workspace_bytes(int B, int H, int blocks);
int sb_route_pair_blocks(const int32_t* packed_route, int B, int QB, int H, int words, int blocks,
                         void* workspace, int32_t* pairs, void* stream);

/*
 * sb_sparse_attention with the routed query blocks tiled by block_pairs (as produced by
 * sb_route_pair_blocks over the query_tokens / 64 routed blocks; block must be 64); the rows
 * from query_tokens on form tiles of 128 in order.  Every row's result is sb_sparse_attention's
 * up to the order of its online-softmax accumulation.  block_pairs NULL: sb_sparse_attention.
 * The fp32 / D = 64 kernel works row by row and ignores the pairs.
 */
int sb_sparse_attention_pairs(const void* q, const void* k, const void* v, int dtype,
                              int B, int T, int H, int D, int block,
                              const int32_t* packed_route, int QB,
                              const void* ak, const void* av, const float* lm,
                              int query_tokens, int sink_first, int sink_last,
                              int local_radius, const int32_t* block_pairs, void* out, float* lse,
                              void* stream);

/*
 * Dense attention of query rows [row_lo, row_hi) over all T keys (softmax scale D^-1/2); the
 * other rows of out / lse are not written.  Replaces the dense-suffix SDPA overwrite of
 * h3_sparse_attention/spark_integration.py:1238-1260 for the rows a padded sparse prefix
 * covered (sol_video_tail_mode = "pad": the context rows that filled the final video query
 * block, spark_integration.py:1173-1187).  Shapes, dtype and alignment as sb_sparse_attention.
 */
int sb_dense_rows_attention(const void* q, const void* k, const void* v, int dtype, int B, int T, int H, int D,
                            int row_lo, int row_hi, void* out, float* lse, void* stream);

/*
 * Eight-key anchor summaries for the block8x8 tail.  Replaces sol_numerator_virtual_q.py:
 * 193-242 (_summaries_block8) for the global parent: per group of 8 keys g (the last may be
 * short), p = 2^(a.k / sqrt(D) log2 e - max) in fp32, AK8 = sum p k / sum p and AV8 likewise
 * (plain means without weighted_kv), stored bf16; LM8 = (max + log2 sum p) ln 2 -
 * a.AK8 / sqrt(D) with the stored key (SB_SUMMARY_PRE_ROUND_LOGMASS: the fp32 mean), or
 * log(keys in the group) without mass_bias.  K, V [B, T, H, 128] bf16; anchor [B, H, 128]
 * (anchor_dtype); ak8, av8 [B, H, ceil(T/8), 128] bf16; lm8 [B, H, ceil(T/8)] fp32.
 */
int sb_tail_summaries8(const void* k, const void* v, const void* anchor, int dtype, int anchor_dtype, int B, int T,
                       int H, int D, int weighted_kv, int mass_bias, int numerics, void* ak8, void* av8, float* lm8,
                       void* stream);

/*
 * Pooled tail merge for the tail granularities "block" (group_tokens = entry_tokens = block)
 * and "block8x8" (8 and 8).  Replaces sol_numerator_virtual_q.py:415-499
 * (_skip_merge_chunk_block, _skip_merge_chunk_block8) for the global parent.  out / lse hold
 * the exact-keys-only output and its LSE (sb_sparse_attention without summaries) and are
 * updated in place for the routed rows (< query_tokens): per query group of group_tokens
 * rows, the mean query (fp32, rounded to bf16) takes an online softmax over the summary
 * entries (ak, av [B, H, ceil(T / entry_tokens), 128] bf16, lm fp32) whose key block
 * (entry * entry_tokens / block) is not exact for the group's query block, and each row
 * becomes (we * out + wa * tail) / (we + wa), with we, wa = exp(lse_exact - m),
 * exp(lse_tail - m), m their max; lse becomes m + log(we + wa).
 */
int sb_tail_merge(const void* q, const void* ak, const void* av, const float* lm, int dtype, int B, int T, int H,
                  int D, int entry_tokens, int group_tokens, int block, const int32_t* packed_route, int QB,
                  int query_tokens, int sink_first, int sink_last, int local_radius, void* out, float* lse,
                  void* stream);

/*
 * Head-wise token permutation of the video prefix.  Replaces
 * spark_integration.py:308-362 (_headwise_permute_video_tokens) and
 * landmark_tree_v2_triton.py:19-90 (headwise_permute_bthd).
 * dst[b, t, h, :] = src[b, perm[b, h, t], h, :] for t < video_tokens, and
 * dst[b, t, h, :] = src[b, t, h, :] for t >= video_tokens.  perm is int32 or int64
 * (index_bytes 4 or 8).  src and dst must not overlap.
 */
int sb_headwise_permute(const void* src, void* dst, const void* perm, int index_bytes,
                        int B, int T, int H, int D, int elem_bytes, int video_tokens,
                        void* stream);

/*
 * e4m3 row quantiser.  Replaces h3_sparse_attention/fp8_linear.py:75-145 (_quantize_rows_kernel
 * / quantize_rows_reference): per row, scale = max(absmax * fp32(1/448), 1e-12) (fp32, as torch evaluates x / 448) and
 * out = e4m3(clamp(x / scale, -448, 448)) with round-to-nearest-even.  Used for per-token
 * activation scales and per-output-channel weight scales.  x: [M, K] (dtype), out: [M, K]
 * bytes, scales: [M] fp32.  x must be 16-byte aligned (rows use 16-byte loads when K % 8 == 0).
 */
int sb_fp8_quantize_rows(const void* x, int dtype, int64_t M, int K, uint8_t* out,
                         float* scales, void* stream);

/*
 * Fused SwiGLU + e4m3 row quantiser.  Replaces fp8_linear.py:92-108/128-138
 * (_swiglu_quantize_kernel / swiglu_quantize): h is the [M, 2K] projection output (value
 * half first, gate half second); the row quantiser above is applied to a * g * sigmoid(g)
 * evaluated in fp32, without writing the activation.  out: [M, K] bytes, scales: [M] fp32.
 */
int sb_fp8_swiglu_quantize_rows(const void* h, int dtype, int64_t M, int K, uint8_t* out,
                                float* scales, void* stream);

/*
 * Per-tensor e4m3 quantiser.  Replaces fp8_linear.py:160-180/201-214 (_absmax_kernel,
 * _cast_scaled_kernel, quantize_tensor): one absmax over all n values, then
 * scale = max(absmax * fp32(1/448), 1e-12) and out = e4m3(clamp(x / scale)).  scale: 1 fp32 (device),
 * workspace: 1 fp32 of scratch (device).  Nothing is synchronised.
 */
int sb_fp8_quantize_tensor(const void* x, int dtype, int64_t n, uint8_t* out, float* scale,
                           float* workspace, void* stream);

/*
 * act = bf16(a * g * sigmoid(g)) of a [M, 2K] projection output, the bf16 intermediate that
 * the per-tensor SwiGLU path quantises (fp8_linear.py:182-198/223-239).  act: [M, K] bf16.
 */
int sb_fp8_swiglu(const void* h, int dtype, int64_t M, int K, void* act, void* stream);

/*
 * e4m3 GEMM with per-row scales on both operands, bf16 output.  Replaces the
 * torch._scaled_mm call of fp8_linear.py:280-287 (Fp8Linear.forward_quantized):
 *   out[m, n] = bf16(sum_k a[m, k] * b[n, k] * a_scale[m * sa] * b_scale[n * sb] + bias[n])
 * with sa = a_scale_stride and sb = b_scale_stride, each 1 (per-token / per-output-channel
 * scales) or 0 (one scale for the tensor).  a: [M, K] e4m3, b: [N, K] e4m3 (the weight,
 * K-major), bias: [N] bf16 or NULL, out: [M, N] bf16.  K must be a multiple of 16.
 * num_ctas <= 0 launches one persistent CTA per SM.
 */
int sb_fp8_gemm(const uint8_t* a, const float* a_scale, int a_scale_stride, const uint8_t* b,
                const float* b_scale, int b_scale_stride, int64_t M, int N, int K, const void* bias,
                void* out, int num_ctas, void* stream);

/*
 * fp8 GEMM with a gated residual epilogue for the DiT block stack (which
 * the build writes itself; no counterpart in the reference's attention path):
 *   out[m, n] = residual[m, n] + gate[n] * (sum_k a[m, k] b[n, k] a_scale[m] b_scale[n] + bias[n])
 * residual / out: [M, N] bf16 (they may be the same buffer); gate: [N] fp32.  Otherwise as
 * sb_fp8_gemm.
 */
int sb_fp8_gemm_residual(const uint8_t* a, const float* a_scale, int a_scale_stride, const uint8_t* b,
                         const float* b_scale, int b_scale_stride, int64_t M, int N, int K,
                         const void* bias, const void* residual, const float* gate, void* out,
                         int num_ctas, void* stream);

/*
 * Attention-input producer for the DiT stack (config 4; the fused projection / RoPE producer
 * the reference's ComfyUI path builds in native/spark_split/producer.cu): the fused QKV fp8
 * GEMM (A [M, K] e4m3 with per-token scales, B [3 * heads * 128, K] e4m3 with per-channel
 * scales, optional bf16 bias) whose epilogue, per head, rounds the projection to bf16, applies
 * RMSNorm (q with norm_q, k with norm_k, both [128] fp32, eps) and the rotary embedding to q
 * and k, and writes q, k and v head rows as [shards][M][heads / shards][128] bf16: the send
 * layout of the sequence-to-head all-to-all.  Pair j of the head dimension rotates by
 * rope[(j * rope_stride + coords[m, axis[j]]) * 2 + {0: cos, 1: sin}], coords [M, 3] int32,
 * axis [64] int8.  heads must be even.  Replaces sb_fp8_gemm followed by sb_dit_qkv_norm_rope
 * (no qkv intermediate).
 */
int sb_fp8_gemm_qkv_rope(const uint8_t* a, const float* a_scale, const uint8_t* b, const float* b_scale,
                         int64_t M, int heads, int K, const void* bias, const float* norm_q, const float* norm_k,
                         const float* rope, int rope_stride, const int32_t* coords, const int8_t* axis, int shards,
                         float eps, void* q, void* k, void* v, int num_ctas, void* stream);

/*
 * sb_fp8_gemm_qkv_rope whose epilogue performs the sequence-to-head all-to-all itself:
 * peers is a device table [3][shards] of receive buffers (q, k, v; entry [s][r] is rank r's
 * buffer, [shards][M][heads / shards][128] bf16 each, mapped into this process with
 * sb_ipc_open), and head h of row m is stored over NVLink to
 * peers[section][h / hp] + ((rank * M + m) * hp + h % hp) * 128.  The caller orders the
 * ranks' kernels before any rank reads its buffers (a stream-ordered collective serves).
 */
int sb_fp8_gemm_qkv_rope_peers(const uint8_t* a, const float* a_scale, const uint8_t* b, const float* b_scale,
                               int64_t M, int heads, int K, const void* bias, const float* norm_q,
                               const float* norm_k, const float* rope, int rope_stride, const int32_t* coords,
                               const int8_t* axis, int shards, int rank, float eps, void* const* peers, int num_ctas,
                               void* stream);

/*
 * GELU (erf form) fused with the e4m3 row quantiser: quantize_rows(gelu(x)) of an FFN up
 * projection without writing the activation (config 4; the reference's SwiGLU counterpart is
 * fp8_linear.py:128-138).  x: [M, K] (dtype), out: [M, K] bytes, scales: [M] fp32.
 */
int sb_fp8_gelu_quantize_rows(const void* x, int dtype, int64_t M, int K, uint8_t* out,
                              float* scales, void* stream);

/*
 * e4m3 row quantiser over a matrix stored as K / seg consecutive [M, seg] bf16 blocks,
 * `seg_stride` elements apart: the attention output as the head-to-sequence all-to-all
 * returns it (one block of heads per peer), quantised for the output projection without a
 * reordering copy.  out: [M, K] bytes (row-major), scales: [M] fp32.
 */
int sb_fp8_quantize_segments(const void* x, int64_t M, int K, int seg, int64_t seg_stride,
                             uint8_t* out, float* scales, void* stream);

/*
 * DiT block pointwise stage (config 4): per row, y = x / rms(x) * (1 + scale) + shift (RMSNorm
 * with eps, adaLN modulation), quantised to e4m3 with one scale per row for the next GEMM.
 * x: [M, C] bf16, shift / scale: [C] fp32, out: [M, C] bytes, scales: [M] fp32.
 */
int sb_dit_norm_modulate_quantize(const void* x, const float* shift, const float* scale, int64_t M,
                                  int C, float eps, uint8_t* out, float* scales, void* stream);

/*
 * DiT attention input stage (config 4): from the fused projection qkv [M, 3, H, 128] bf16,
 * per-head RMSNorm of q and k (weights wq, wk [128]) and the 3-D rotary embedding (pair j of
 * the head dimension rotates by coords[m, axis[j]] * inv_freq[j]; coords [M, 3] int32 holds
 * each token's (t, h, w)), written as q, k, v [shards][M][H / shards][128] bf16: the send
 * layout of the sequence-to-head all-to-all.
 */
int sb_dit_qkv_norm_rope(const void* qkv, const float* wq, const float* wk, const int32_t* coords,
                         const float* inv_freq, const int8_t* axis, int64_t M, int H, int D,
                         int shards, float eps, void* q, void* k, void* v, void* stream);

/*
 * Strided copy (rows of `width` bytes, `height` rows) between host and device memory in either
 * direction, asynchronous on `stream`: moves one head chunk of a BTHD tensor between a pinned
 * host tensor and a contiguous device buffer.  No counterpart in the reference (its layer
 * takes device tensors); the streamed layer of the Python API uses it to overlap transfers
 * with compute.
 */
int sb_memcpy2d(void* dst, int64_t dpitch, const void* src, int64_t spitch, int64_t width,
                int64_t height, void* stream);

/*
 * Reblock metric factors.  Replaces h3_sparse_attention/landmark_direction.py:60-104 with
 * mahalanobis_kmeans.py:309-388 (landmark_direction_factors / batched_cross_metric_factors,
 * raw moments, m2_side "both"): for every (batch, head) the non-centred second moment of the
 * sampled Q rows and of the sampled K rows, M = X^T X / S, symmetrised, with
 * ridge * trace(M) / D added to the diagonal, factored as L L^T (Cholesky, fp32).
 * q, k: BTHD (dtype), D = 128.  samples: [S] token ids (device), the Hilbert-midpoint
 * samples of mahalanobis_kmeans.py:87-96.  factors: [2*B*H, D, D] fp32 lower-triangular,
 * rows [0, BH) = chol(M(Q)) (applied to K), rows [BH, 2BH) = chol(M(K)) (applied to Q).
 */
int sb_reblock_metric(const void* q, const void* k, int dtype, int B, int T, int H, int D,
                      const int32_t* samples, int num_samples, float ridge, float* factors,
                      void* stream);

/*
 * Reblock features.  Replaces the two bf16 bmm calls of spark_integration.py:561-585:
 * features[r] = bf16(X_r . bf16(L_r)) over the first video_tokens tokens, X_r = K[b, :, h]
 * for r = b*H + h < BH and Q[b, :, h] for r - BH.  q, k: BTHD bf16, D = 128;
 * factors: as written by sb_reblock_metric; features: [2*B*H, video_tokens, D] bf16.
 */
int sb_reblock_transform(const void* q, const void* k, int B, int T, int H, int D,
                         int video_tokens, const float* factors, void* features, void* stream);

/*
 * Reblock plan.  The splitting rounds of reblock_hierarchy.py:108-234
 * (ReblockHierarchy.split_budgets) turned into per-round node tables for sb_reblock_tree.
 * schedule: [rounds, then per round: entries, then per entry: leaves, children,
 * budget_0 .. budget_{children-1}] (host).  plan: host buffer of `capacity` ints, or NULL
 * to query the length.  Returns the plan length in ints, or a negative error.  The caller
 * keeps the host plan and a device copy of the same ints.
 */
int64_t sb_reblock_plan(const int32_t* schedule, int schedule_len, int tokens, int32_t* plan,
                        int64_t capacity);

/*
 * Proxy controls of a plan (host), before its device copy is made.  Replaces the
 * proxy_iterations / seed_rule arguments of landmark_tree_v2.py:790-832 and
 * landmark_v2_terminal.py:43-50 (_normalize_proxy_controls): proxy_iterations mean-update
 * passes of every proxy node, 0, 1, 2 or 4 (with 0, one assignment pass hands the children
 * their landmark weights and the seed pair gives the split direction); endpoint_seeds 0 seeds
 * each proxy node with its farthest valid landmark pair (seed_rule "farthest_pair"), 1 with
 * its lowest and highest valid landmark ("endpoint_order").  sb_reblock_plan sets the
 * production controls, 2 and 0.  Returns 0, or SB_ERR_INVALID for other values.
 */
int sb_reblock_plan_proxy(int32_t* plan, int proxy_iterations, int endpoint_seeds);

/* Scratch bytes sb_reblock_tree needs for `rows` feature rows under `plan` (host plan). */
int64_t sb_reblock_workspace_bytes(const int32_t* plan, int rows);

/*
 * Landmark-tree-v2 permutation.  Replaces landmark_tree_v2.py:297-787
 * (_recursive_landmark_tree_v2 with the defaults of PreparedLandmarkTreeV2Permutation:
 * cosine distance, group size 1, 32 midpoint landmarks, linear aggregation, parent order,
 * two mean-update proxy iterations from the farthest pair; any fanout mode, i.e. nodes of 2
 * to 64 children over the split topology of landmark_v2_terminal.py:11-33) and
 * landmark_tree_clustering.py:56-146, 290-565 (remainder, exact routing, stable partition).
 * features: [rows, tokens, D] bf16, D = 128.  root_order: [tokens] device ids of the initial
 * order, or NULL for the flat order.  perm / inverse: [rows, tokens] int32; perm holds the
 * 64-token leaves in order, then the tokens mod 64 protected remainder tokens (largest
 * squared feature norm, lower id first among equals) in root order.
 */
int sb_reblock_tree(const void* features, int rows, int tokens, int D, const int32_t* root_order,
                    const int32_t* plan_host, const int32_t* plan_device, void* workspace,
                    int64_t workspace_bytes, int32_t* perm, int32_t* inverse, void* stream);

/*
 * The protected remainder of each feature row, alone: the tokens mod 64 tokens of largest
 * squared feature norm (equal norms: lower id), ascending ids.  Replaces
 * landmark_tree_clustering.py:56-82 (_largest_norm_remainder) where spark_integration.py:
 * 597-693 freezes the tail of the baseline (both-side Hilbert M2) features for the M2
 * ablations, before the tree runs on other features (sb_reblock_tree_frozen).
 * features: [rows, tokens, 128] bf16; workspace: 8 * rows * tokens bytes, 256-byte aligned;
 * excluded: [rows, tokens mod 64] int32 (untouched when tokens is a multiple of 64).
 */
int sb_reblock_remainder(const void* features, int rows, int tokens, int D, void* workspace,
                         int64_t workspace_bytes, int32_t* excluded, void* stream);

/*
 * sb_reblock_tree with the protected remainder chosen by the caller: the excluded_indices
 * argument of landmark_tree_v2.py:790-832 and landmark_tree_clustering.py:85-119
 * (_initial_hilbert_partition's frozen tail).  excluded: [rows, tokens mod 64] device int32
 * token ids, unique and in [0, tokens) per row (NULL allowed when tokens is a multiple of 64);
 * those tokens form the tail of each permutation in root order, whatever their norms.  The
 * caller validates the ids: an out-of-range id is skipped and a tail of the wrong size sets
 * device status 612 (sb_read_device_status), with every write still inside the row.
 */
int sb_reblock_tree_frozen(const void* features, int rows, int tokens, int D, const int32_t* root_order,
                           const int32_t* excluded, const int32_t* plan_host, const int32_t* plan_device,
                           void* workspace, int64_t workspace_bytes, int32_t* perm, int32_t* inverse,
                           void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPARK_H3_B200_H */
