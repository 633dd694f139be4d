// Row-parallel projection + norm epilogue for callers that cannot allocate device memory.
//
// morj_gemm_bf16_peer followed by morj_peer_reduce needs scratch beyond the caller's inputs and outputs: the BF16
// projection rows C = A . B^T and the per-block arrival counters, which the Python engine allocates through torch.
// Some callers of this library have no device allocator they may use: a host process that binds the C-ABI from
// another language, owns only the buffers it was handed and may not call cudaMalloc itself (its memory is managed
// elsewhere, or its budget is fixed at start-up). morj_gemm_norm_epilogue_noalloc runs the same two kernels for one
// rank with that scratch in a fixed array compiled into the library (kScratchBytes, every GPU that loads the library
// holds it until exit), so it calls no cudaMalloc, cudaFree or other allocating routine.
//
// The array is shared by every call on a device and keeps the last call's contents: each call clears the counters
// it uses (cudaMemsetAsync on its stream) before the GEMM, and the projection rows are fully rewritten. Two calls
// that overlap on the GPU (different streams, or different host threads without ordering) race on the array.
#include <mutex>

#include "common.cuh"

namespace morj {
namespace noalloc {

constexpr size_t kPartBytes = size_t(8) << 20;  // BF16 projection rows: M * N * 2 bytes at most
constexpr int kMaxBlocks = 1024;                // row blocks of 128 (M <= 131072), one counter pair each
constexpr size_t kScratchBytes = kPartBytes + 2 * kMaxBlocks * sizeof(unsigned long long);

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

// The device address of g_scratch on the current device. In host code `g_scratch` names a host-side stand-in, not
// device memory, so the address is looked up once per device (with that device current) and cached for the life of
// the process. The cache is keyed by device number: after cudaDeviceReset (or from a second context on the same
// device) the cached address is stale, so a process that resets a device must not call this entry point again.
static int scratch_address(unsigned char** out) {
  constexpr int kMaxDevices = 64;
  static unsigned char* addr[kMaxDevices] = {};
  static std::mutex lock;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(MORJ_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return set_error(MORJ_ERR_UNSUPPORTED, "device %d beyond %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> g(lock);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess) return set_error(MORJ_ERR_CUDA, "cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    addr[dev] = static_cast<unsigned char*>(p);
  }
  *out = addr[dev];
  return MORJ_OK;
}

}  // namespace noalloc
}  // namespace morj

extern "C" int morj_gemm_norm_epilogue_noalloc(const void* A, long long lda, const void* B, long long ldb, int M,
                                               int N, int K, int mode, void* x, void* h, const void* w_a,
                                               const void* scalar, const void* w_b, float eps, int has_next,
                                               void* stream) {
  using namespace morj;
  if (M == 0) return MORJ_OK;
  if (M < 0 || N <= 0 || K <= 0 || !x || (mode != 0 && mode != 1) || ((mode == 0 || has_next) && !h))
    return set_error(MORJ_ERR_ARG, "morj_gemm_norm_epilogue_noalloc: bad arguments (M=%d N=%d K=%d mode=%d)", M, N,
                     K, mode);
  const long long blocks = (M + 127) / 128;
  if ((unsigned long long)M * (unsigned long long)N * 2 > noalloc::kPartBytes)
    return set_error(MORJ_ERR_ARG,
                     "morj_gemm_norm_epilogue_noalloc: M x N = %d x %d needs %lld bytes of projection scratch, above "
                     "the library's fixed %zu",
                     M, N, (long long)M * N * 2, noalloc::kPartBytes);
  if (blocks > noalloc::kMaxBlocks)
    return set_error(MORJ_ERR_ARG,
                     "morj_gemm_norm_epilogue_noalloc: M = %d rows need %lld row blocks of 128, above the library's "
                     "fixed %d counter pairs (M <= %d)",
                     M, blocks, noalloc::kMaxBlocks, noalloc::kMaxBlocks * 128);
  unsigned char* scratch = nullptr;
  int st = noalloc::scratch_address(&scratch);
  if (st) return st;
  unsigned long long* counters = reinterpret_cast<unsigned long long*>(scratch + noalloc::kPartBytes);
  morj_peer_t d{};
  d.world = 1;
  d.rank = 0;
  d.max_blocks = (int)blocks;
  d.hidden = N;
  d.part[0] = scratch;
  d.x[0] = x;
  d.h[0] = h ? h : x;  // (an MLP epilogue without a next layer writes no h)
  d.partials[0] = counters;
  d.rows[0] = counters + blocks;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // the counters of the previous call are still there: this call's must start at zero
  const cudaError_t e = cudaMemsetAsync(counters, 0, 2 * blocks * sizeof(unsigned long long), s);
  if (e != cudaSuccess) return set_error(MORJ_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
  st = morj_gemm_bf16_peer(A, lda, B, ldb, M, N, K, &d, stream);
  if (st) return st;
  // one site, one rank: every block's counter reaches 4 epilogue warps x N columns
  return morj_peer_reduce(&d, mode, M, w_a, scalar, w_b, eps, has_next, 0, 4ull * (unsigned long long)N, stream);
}
