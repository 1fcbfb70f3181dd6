// C-ABI plumbing: error reporting, the device status word, and the sparse attention
// dispatcher (tensor-core kernel for bf16 / D = 128, SIMT kernel otherwise).
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "attn_common.cuh"
#include "sm100_ptx.cuh"

namespace sb {

static thread_local char g_error[1024] = "";

void set_error(const char* fmt, ...) {
  va_list args;
  va_start(args, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, args);
  va_end(args);
}

int cuda_error(cudaError_t err, const char* what) {
  set_error("%s: %s (%s)", what, cudaGetErrorString(err), cudaGetErrorName(err));
  return SB_ERR_CUDA;
}

// Written by kernels whose waits gave up (value = a site code), read by
// sb_read_device_status.  One copy per device that loads the library.
__device__ int g_device_status;

int* device_status_ptr() {
  static std::mutex mu;
  static int* cached[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_device_status) != cudaSuccess) return nullptr;
    cached[dev] = static_cast<int*>(ptr);
  }
  return cached[dev];
}

}  // namespace sb

using namespace sb;

extern "C" int sb_version(void) { return 100; }

extern "C" int sb_memcpy2d(void* dst, int64_t dpitch, const void* src, int64_t spitch, int64_t width, int64_t height,
                           void* stream) {
  SB_CHECK_ARG(dst && src, "sb_memcpy2d: null pointer");
  SB_CHECK_ARG(width >= 0 && height >= 0 && dpitch >= width && spitch >= width, "sb_memcpy2d: bad extents");
  if (width == 0 || height == 0) return SB_OK;
  cudaError_t err = cudaMemcpy2DAsync(dst, (size_t)dpitch, src, (size_t)spitch, (size_t)width, (size_t)height,
                                      cudaMemcpyDefault, (cudaStream_t)stream);
  if (err != cudaSuccess) return cuda_error(err, "sb_memcpy2d");
  return SB_OK;
}

extern "C" const char* sb_last_error(void) { return g_error; }

extern "C" int sb_read_device_status(void* stream) {
  int* ptr = device_status_ptr();
  if (ptr == nullptr) return cuda_error(cudaGetLastError(), "sb_read_device_status: symbol address");
  cudaStream_t s = (cudaStream_t)stream;
  int value = 0;
  cudaError_t err = cudaMemcpyAsync(&value, ptr, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (err == cudaSuccess) err = cudaStreamSynchronize(s);
  if (err != cudaSuccess) return cuda_error(err, "sb_read_device_status: read");
  const int zero = 0;
  err = cudaMemcpyAsync(ptr, &zero, sizeof(int), cudaMemcpyHostToDevice, s);
  if (err == cudaSuccess) err = cudaStreamSynchronize(s);
  if (err != cudaSuccess) return cuda_error(err, "sb_read_device_status: clear");
  return value;
}

extern "C" int sb_sparse_attention_pairs(const void* q, const void* k, const void* v, int dtype, int B,
                                         int T, int H, int D, int block, const int32_t* packed_route,
                                         int QB, const void* ak, const void* av, const float* lm,
                                         int query_tokens, int sink_first, int sink_last,
                                         int local_radius, const int32_t* block_pairs, void* out, float* lse,
                                         void* stream) {
  SB_CHECK_ARG(q && k && v && out, "sb_sparse_attention: null Q/K/V/out");
  SB_CHECK_ARG(dtype == SB_F32 || dtype == SB_BF16, "sb_sparse_attention: bad dtype");
  SB_CHECK_ARG(B > 0 && T > 0 && H > 0, "sb_sparse_attention: B, T, H must be positive");
  SB_CHECK_ARG(D == 64 || D == 128, "sb_sparse_attention: head dim must be 64 or 128, got %d", D);
  SB_CHECK_ARG(block == 64 || block == 128, "sb_sparse_attention: block must be 64 or 128, got %d", block);
  SB_CHECK_ARG(T <= (1 << 22), "sb_sparse_attention: at most 4194304 tokens are supported");
  SB_CHECK_ARG(query_tokens >= 0 && query_tokens <= T && query_tokens % block == 0,
               "sb_sparse_attention: query_tokens must be a block multiple in [0, T], got %d", query_tokens);
  const int NB = ceil_div(T, block);
  const int routed_blocks = query_tokens / block;
  if (routed_blocks > 0) {
    SB_CHECK_ARG(packed_route, "sb_sparse_attention: routed queries need the route");
    SB_CHECK_ARG((ak && av && lm) || (!ak && !av && !lm),
                 "sb_sparse_attention: pass all of AK, AV and LM, or none (exact keys only)");
    SB_CHECK_ARG(QB >= routed_blocks && QB <= NB, "sb_sparse_attention: QB (%d) must lie in [%d, %d]", QB, routed_blocks, NB);
  }
  SB_CHECK_ARG(sink_first >= 0 && sink_first <= sink_last && sink_last <= NB,
               "sb_sparse_attention: sink range [%d, %d) is outside [0, %d]", sink_first, sink_last, NB);
  SB_CHECK_ARG(local_radius >= -1, "sb_sparse_attention: local_radius must be >= -1");
  const uintptr_t mis = (uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out |
                        (uintptr_t)ak | (uintptr_t)av;
  SB_CHECK_ARG(mis % 16 == 0, "sb_sparse_attention: tensors must be 16-byte aligned");
  AttnParams p{};
  p.q = q; p.k = k; p.v = v; p.packed = packed_route; p.ak = ak; p.av = av; p.lm = lm;
  p.out = out; p.lse = lse;
  p.status = device_status_ptr();
  if (p.status == nullptr) return cuda_error(cudaGetLastError(), "sb_sparse_attention: status word");
  p.B = B; p.T = T; p.H = H; p.block = block; p.NB = NB; p.QB = QB; p.words = ceil_div(NB, 32);
  p.query_tokens = query_tokens; p.sink_first = sink_first; p.sink_last = sink_last;
  p.local_radius = local_radius;
  p.row_lo = 0;
  p.row_hi = T;
  if (block_pairs != nullptr) {
    SB_CHECK_ARG(block == 64, "sb_sparse_attention_pairs: query-block pairs need 64-token blocks");
    SB_CHECK_ARG(routed_blocks >= 1, "sb_sparse_attention_pairs: pairs need routed query blocks");
    p.pairs = block_pairs;
    p.pair_tiles = ceil_div(routed_blocks, 2);
  }
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == SB_BF16 && D == 128) return launch_sparse_attention_sm100(p, s);
  return launch_sparse_attention_simt(p, dtype, D, s);  // row by row: pairs do not apply
}

extern "C" int sb_sparse_attention(const void* q, const void* k, const void* v, int dtype, int B,
                                   int T, int H, int D, int block, const int32_t* packed_route,
                                   int QB, const void* ak, const void* av, const float* lm,
                                   int query_tokens, int sink_first, int sink_last,
                                   int local_radius, void* out, float* lse, void* stream) {
  return sb_sparse_attention_pairs(q, k, v, dtype, B, T, H, D, block, packed_route, QB, ak, av, lm, query_tokens,
                                   sink_first, sink_last, local_radius, nullptr, out, lse, stream);
}

extern "C" int sb_dense_rows_attention(const void* q, const void* k, const void* v, int dtype, int B, int T, int H,
                                       int D, int row_lo, int row_hi, void* out, float* lse, void* stream) {
  SB_CHECK_ARG(q && k && v && out, "sb_dense_rows_attention: null Q/K/V/out");
  SB_CHECK_ARG(dtype == SB_F32 || dtype == SB_BF16, "sb_dense_rows_attention: bad dtype");
  SB_CHECK_ARG(B > 0 && T > 0 && H > 0, "sb_dense_rows_attention: B, T, H must be positive");
  SB_CHECK_ARG(D == 64 || D == 128, "sb_dense_rows_attention: head dim must be 64 or 128, got %d", D);
  SB_CHECK_ARG(T <= (1 << 22), "sb_dense_rows_attention: at most 4194304 tokens are supported");
  SB_CHECK_ARG(row_lo >= 0 && row_lo <= row_hi && row_hi <= T,
               "sb_dense_rows_attention: rows [%d, %d) are outside [0, %d]", row_lo, row_hi, T);
  SB_CHECK_ARG((((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) % 16) == 0,
               "sb_dense_rows_attention: tensors must be 16-byte aligned");
  if (row_lo == row_hi) return SB_OK;
  AttnParams p{};
  p.q = q; p.k = k; p.v = v; p.out = out; p.lse = lse;
  p.status = device_status_ptr();
  if (p.status == nullptr) return cuda_error(cudaGetLastError(), "sb_dense_rows_attention: status word");
  // Every row is a dense-suffix row: no route, no summaries, every key block exact.
  p.B = B; p.T = T; p.H = H; p.block = 128; p.NB = ceil_div(T, 128); p.QB = 0; p.words = ceil_div(p.NB, 32);
  p.query_tokens = 0; p.sink_first = 0; p.sink_last = 0; p.local_radius = -1;
  p.row_lo = row_lo;
  p.row_hi = row_hi;
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == SB_BF16 && D == 128) return launch_sparse_attention_sm100(p, s);
  return launch_sparse_attention_simt(p, dtype, D, s);
}

// ------------------------------------------------------------------ bounded-wait self-check
namespace sb {
namespace {

constexpr int kSelfTestSite = SB_SELFTEST_WAIT_SITE;

// Warp 0 waits on an mbarrier that nothing arrives on, with a short limit: it gives up,
// raises the CTA abort flag and records its site code.  Warp 1 waits on a second such
// barrier with the kernels' normal two-second limit and must leave as soon as the flag is
// up.  No fault, no unbounded wait: the kernel ends after about `limit` cycles.
__global__ void wait_timeout_kernel(long long limit, int* status, int* result) {
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    sm100::mbar_init(sm100::smem_u32(&bars[0]), 1);
    sm100::mbar_init(sm100::smem_u32(&bars[1]), 1);
    sm100::fence_barrier_init();
    abort_flag = 0;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5;
  const long long t0 = clock64();
  const bool got = warp == 0 ? sm100::mbar_wait_limit(sm100::smem_u32(&bars[0]), 0, &abort_flag, status,
                                                      kSelfTestSite, limit)
                             : sm100::mbar_wait(sm100::smem_u32(&bars[1]), 0, &abort_flag, status, kSelfTestSite + 1);
  const long long dt = clock64() - t0;
  if ((threadIdx.x & 31) == 0) {
    result[2 * warp] = got ? 1 : 0;
    result[2 * warp + 1] = dt < 4 * limit + 1000000 ? 1 : 0;  // left within a bounded time
  }
}

}  // namespace
}  // namespace sb

extern "C" int sb_selftest_wait_timeout(long long limit_cycles, int* result, void* stream) {
  SB_CHECK_ARG(result, "sb_selftest_wait_timeout: null result");
  SB_CHECK_ARG(limit_cycles > 0 && limit_cycles <= 100000000ll,
               "sb_selftest_wait_timeout: limit must lie in (0, 1e8] cycles");
  int* status = device_status_ptr();
  if (status == nullptr) return cuda_error(cudaGetLastError(), "sb_selftest_wait_timeout: status word");
  wait_timeout_kernel<<<1, 64, 0, (cudaStream_t)stream>>>(limit_cycles, status, result);
  SB_CHECK_LAUNCH("sb_selftest_wait_timeout launch");
  return SB_OK;
}

// ------------------------------------------------------------------ peer memory (CUDA IPC)
// Receive buffers that other processes of the node write into directly (one process per
// GPU): allocated here so that the IPC handle covers exactly the buffer.
extern "C" int sb_ipc_alloc(int64_t bytes, void** ptr) {
  SB_CHECK_ARG(ptr && bytes > 0, "sb_ipc_alloc: bad arguments");
  *ptr = nullptr;
  cudaError_t err = cudaMalloc(ptr, (size_t)bytes);
  if (err != cudaSuccess) return cuda_error(err, "sb_ipc_alloc");
  return SB_OK;
}

extern "C" int sb_ipc_free(void* ptr) {
  if (ptr == nullptr) return SB_OK;
  cudaError_t err = cudaFree(ptr);
  if (err != cudaSuccess) return cuda_error(err, "sb_ipc_free");
  return SB_OK;
}

extern "C" int sb_ipc_handle(const void* ptr, uint8_t* handle) {
  SB_CHECK_ARG(ptr && handle, "sb_ipc_handle: null pointer");
  cudaIpcMemHandle_t h;
  cudaError_t err = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (err != cudaSuccess) return cuda_error(err, "sb_ipc_handle");
  memcpy(handle, &h, sizeof(h));
  return SB_OK;
}

extern "C" int sb_ipc_open(const uint8_t* handle, void** ptr) {
  SB_CHECK_ARG(handle && ptr, "sb_ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  cudaError_t err = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (err != cudaSuccess) return cuda_error(err, "sb_ipc_open");
  return SB_OK;
}

extern "C" int sb_ipc_close(void* ptr) {
  if (ptr == nullptr) return SB_OK;
  cudaError_t err = cudaIpcCloseMemHandle(ptr);
  if (err != cudaSuccess) return cuda_error(err, "sb_ipc_close");
  return SB_OK;
}
