/*
 * One Spark layer through the C ABI alone: include/spark_h3_b200.h, libsparkh3b200 and the
 * CUDA runtime, no Python or torch.  The sequence is the one a C host of the reference's
 * attention seam runs (spark_attention_bthd, spark_integration.py:883-1283, with the video
 * prefix first and no context):
 *   pool Q -> global anchor -> key means + summaries -> scores + Top-K -> sparse attention.
 *
 * usage: spark_layer T H D block topk scale_log2 q.bin k.bin v.bin outdir
 *   q/k/v.bin: bf16 [1, T, H, D] raw.  scale_log2 is a C99 hex float.
 * writes outdir/packed.bin (int32 [1, QB, H, words]), indices.bin (int32 [1, QB, H, topk]),
 * out.bin (bf16 [1, T, H, D]) and lse.bin (fp32 [1, T, H]).  Exit status 0 on success.
 */
#include <cuda_runtime_api.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "spark_h3_b200.h"

#define SB(call)                                                                  \
  do {                                                                            \
    int rc_ = (call);                                                             \
    if (rc_ != SB_OK) {                                                           \
      fprintf(stderr, "%s failed (%d): %s\n", #call, rc_, sb_last_error());       \
      exit(2);                                                                    \
    }                                                                             \
  } while (0)
#define CU(call)                                                                  \
  do {                                                                            \
    cudaError_t e_ = (call);                                                      \
    if (e_ != cudaSuccess) {                                                      \
      fprintf(stderr, "%s failed: %s\n", #call, cudaGetErrorString(e_));          \
      exit(3);                                                                    \
    }                                                                             \
  } while (0)

static void* device_from_file(const char* path, size_t bytes) {
  void* host = malloc(bytes);
  FILE* f = fopen(path, "rb");
  if (!host || !f || fread(host, 1, bytes, f) != bytes) {
    fprintf(stderr, "cannot read %zu bytes from %s\n", bytes, path);
    exit(4);
  }
  fclose(f);
  void* dev = NULL;
  CU(cudaMalloc(&dev, bytes));
  CU(cudaMemcpy(dev, host, bytes, cudaMemcpyHostToDevice));
  free(host);
  return dev;
}

static void device_to_file(const void* dev, size_t bytes, const char* dir, const char* name) {
  char path[4096];
  snprintf(path, sizeof(path), "%s/%s", dir, name);
  void* host = malloc(bytes);
  CU(cudaMemcpy(host, dev, bytes, cudaMemcpyDeviceToHost));
  FILE* f = fopen(path, "wb");
  if (!host || !f || fwrite(host, 1, bytes, f) != bytes) {
    fprintf(stderr, "cannot write %s\n", path);
    exit(4);
  }
  fclose(f);
  free(host);
}

static void* device_alloc(size_t bytes) {
  void* p = NULL;
  CU(cudaMalloc(&p, bytes));
  return p;
}

int main(int argc, char** argv) {
  if (argc != 11) {
    fprintf(stderr, "usage: %s T H D block topk scale_log2 q.bin k.bin v.bin outdir\n", argv[0]);
    return 1;
  }
  const int B = 1, T = atoi(argv[1]), H = atoi(argv[2]), D = atoi(argv[3]), block = atoi(argv[4]);
  const int topk = atoi(argv[5]);
  const float scale_log2 = strtof(argv[6], NULL);
  const char* outdir = argv[10];
  const int NB = (T + block - 1) / block;
  const int candidates = T / block;                 /* complete video blocks */
  const int query_tokens = candidates * block;      /* sparse query prefix */
  const int QB = candidates;
  const int words = (NB + 31) / 32;
  const int sink_first = candidates, sink_last = candidates;  /* no context suffix */
  const size_t tokens = (size_t)B * T * H * D;

  if (sb_version() <= 0) {
    fprintf(stderr, "bad library version\n");
    return 5;
  }
  void* q = device_from_file(argv[7], tokens * 2);
  void* k = device_from_file(argv[8], tokens * 2);
  void* v = device_from_file(argv[9], tokens * 2);
  float* qc = (float*)device_alloc((size_t)B * NB * H * D * 4);
  void* anchor = device_alloc((size_t)B * H * D * 2);
  void* kc = device_alloc((size_t)B * NB * H * D * 2);
  void* ak = device_alloc((size_t)B * H * NB * D * 2);
  void* av = device_alloc((size_t)B * H * NB * D * 2);
  float* lm = (float*)device_alloc((size_t)B * H * NB * 4);
  const int64_t ws_bytes = sb_route_workspace_bytes(B, QB, H, candidates);
  if (ws_bytes < 0) {
    fprintf(stderr, "sb_route_workspace_bytes: %s\n", sb_last_error());
    return 2;
  }
  void* ws = device_alloc((size_t)ws_bytes);
  int32_t* packed = (int32_t*)device_alloc((size_t)B * QB * H * words * 4);
  int32_t* indices = (int32_t*)device_alloc((size_t)B * QB * H * topk * 4);
  void* out = device_alloc(tokens * 2);
  float* lse = (float*)device_alloc((size_t)B * T * H * 4);

  cudaStream_t stream;
  CU(cudaStreamCreate(&stream));
  SB(sb_pool_queries(q, SB_BF16, B, T, H, D, block, qc, stream));
  SB(sb_query_anchor(qc, B, NB, H, D, block, candidates, anchor, SB_BF16, stream));
  SB(sb_pool_keys_summaries(k, v, anchor, SB_BF16, SB_BF16, B, T, H, D, block, 1, 1, 0, kc, ak, av, lm,
                            stream));
  SB(sb_route_topk(qc, kc, SB_BF16, B, QB, NB, H, D, candidates, topk, scale_log2, ws, packed, indices,
                   stream));
  SB(sb_sparse_attention(q, k, v, SB_BF16, B, T, H, D, block, packed, QB, ak, av, lm, query_tokens, sink_first,
                         sink_last, -1, out, lse, stream));
  CU(cudaStreamSynchronize(stream));
  const int status = sb_read_device_status(stream);
  if (status != 0) {
    fprintf(stderr, "device status %d\n", status);
    return 6;
  }

  device_to_file(packed, (size_t)B * QB * H * words * 4, outdir, "packed.bin");
  device_to_file(indices, (size_t)B * QB * H * topk * 4, outdir, "indices.bin");
  device_to_file(out, tokens * 2, outdir, "out.bin");
  device_to_file(lse, (size_t)B * T * H * 4, outdir, "lse.bin");

  void* bufs[] = {q, k, v, qc, anchor, kc, ak, av, lm, ws, packed, indices, out, lse};
  for (size_t i = 0; i < sizeof(bufs) / sizeof(bufs[0]); ++i) CU(cudaFree(bufs[i]));
  CU(cudaStreamDestroy(stream));
  printf("spark_layer ok: T=%d H=%d block=%d topk=%d\n", T, H, block, topk);
  return 0;
}
