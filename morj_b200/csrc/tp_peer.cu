// Tensor parallelism over peer memory: the owner-side reduction of the row-parallel O / down projections and the
// hand-back of the reduced rows, replacing an NCCL all-reduce followed by replicated epilogues.
//
// Row block b (128 rows) belongs to rank b % world. Every rank's row-parallel GEMM (morj_gemm_bf16_peer) has stored
// its BF16 partial rows in its own part buffer and counted the columns of block b on the owner's counter. Here the
// owner
//   1. waits (one thread per CTA, acquire at system scope, bounded) until block b's counter holds every rank's
//      columns for this site,
//   2. reads block b's partial rows from every rank (NVLink loads from the peers' part buffers), sums them in rank
//      order in FP32 and rounds to BF16,
//   3. applies the post-attention or post-MLP epilogue (the math of morj_attn_epilogue / morj_mlp_epilogue) to its
//      rows, and
//   4. stores the new h rows (and x rows, when asked) into every rank's buffers over NVLink, then counts one row on
//      each rank's row counter for block b (after a CTA barrier, release at system scope).
// morj_peer_wait then holds each rank's stream until all of h has arrived. Counters only grow; the host passes
// cumulative targets, and the last CTA of every reduce pads the blocks beyond this call's rows so that every block
// advances by the same amount per site. Plain stores and atomics to peer memory only: no multicast, no NVLS.
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace morj {
namespace peer {

MORJ_DEV unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
MORJ_DEV void red_release_sys_add(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Spin (bounded) until *p >= target. Returns false after reporting `code` when the limit passes.
MORJ_DEV bool wait_at_least(const unsigned long long* p, unsigned long long target, int code) {
  if (ld_acquire_sys(p) >= target) return true;
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (ld_acquire_sys(p) >= target) return true;
    if ((i & 15) == 0) {
      if (global_ns() - t0 > kWaitLimitNs) {
        report(code);
        return false;
      }
      __nanosleep(64);
    }
  }
}

// One CTA per row of this rank's row blocks below n, plus one last CTA that pads the blocks past n. The row's x
// (this rank's own memory, written only by its own earlier kernels) is loaded before the counter wait and the ranks'
// partials right after it, as packed BF16, two ranks at a time with the loop over ranks unrolled to W (the group
// size rounded up to 2, 4 or 8): a runtime loop over ranks left one load round trip per rank and vector in the
// chain, and holding all W partials at once cut the CTAs per SM to one at W = 8. The partials go through L2 only
// (`ld.cg`): the peers' GEMMs write them while this kernel may run. The row's stores are published by one barrier
// and the release atomics that count the row (release is cumulative over the barrier, as in a stream-K fix-up's
// arrival); a system fence in every thread stalled the kernel most of its time.
template <int VPT, int MODE, int W>
__global__ void __launch_bounds__(ROW_THREADS, W == 2 ? 4 : 3)
    reduce_kernel(const morj_peer_t p, int n, const __nv_bfloat16* __restrict__ w_a,
                  const __nv_bfloat16* __restrict__ scalar, const __nv_bfloat16* __restrict__ w_b, float eps,
                  int has_next, int push_x, unsigned long long partial_target) {
  pdl_wait();  // the previous kernel on the stream has completed
  pdl_trigger();
  __shared__ float red[2][32];  // one array per reduction
  __shared__ int ok_s;
  const int H = p.hidden, world = p.world, rank = p.rank;
  const int n_blocks = (n + 127) / 128;
  if (blockIdx.x == gridDim.x - 1) {
    // padding: every rank's share of the partial columns for blocks >= n_blocks, and this rank's rows of its own
    // blocks >= n_blocks, so every block's counters advance by the same amount at every site
    for (int b = n_blocks + (int)threadIdx.x; b < p.max_blocks; b += ROW_THREADS) {
      red_release_sys_add(p.partials[b % world] + b, 4ull * (unsigned long long)H);
      if (b % world == rank)
        for (int r = 0; r < world; ++r) red_release_sys_add(p.rows[r] + b, 128ull);
    }
    return;
  }
  const int blk = rank + (int)(blockIdx.x / 128) * world;
  const int row = blk * 128 + (int)(blockIdx.x % 128);
  const bool live = row < n;  // rows past n in the last block only count
  __nv_bfloat16* x = reinterpret_cast<__nv_bfloat16*>(p.x[rank]) + (size_t)row * H;
  uint4 x_raw[VPT];
  if (live) {
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int c = (threadIdx.x + k * ROW_THREADS) * 8;
      if (c < H) x_raw[k] = *reinterpret_cast<const uint4*>(x + c);
    }
  }
  if (threadIdx.x == 0) ok_s = wait_at_least(p.partials[rank] + blk, partial_target, kErrTimeoutPeerPartials);
  __syncthreads();
  if (!ok_s) return;  // the peers' waits for this block's rows run out and report too
  if (live) {
    float ov[VPT][8];
#pragma unroll
    for (int s0 = 0; s0 < W; s0 += 2) {
      uint4 raw[2][VPT];
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int c = (threadIdx.x + k * ROW_THREADS) * 8;
        if (c < H) {
#pragma unroll
          for (int j = 0; j < 2; ++j)
            if (s0 + j < world)
              raw[j][k] = __ldcg(reinterpret_cast<const uint4*>(
                  reinterpret_cast<const __nv_bfloat16*>(p.part[s0 + j]) + (size_t)row * H + c));
        }
      }
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int c = (threadIdx.x + k * ROW_THREADS) * 8;
        if (c < H) {
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            if (s0 + j < world) {
              float pv[8];
              unpack8(raw[j][k], pv);
#pragma unroll
              for (int e = 0; e < 8; ++e) ov[k][e] = (s0 + j == 0) ? pv[e] : ov[k][e] + pv[e];  // FP32, rank order
            }
          }
        }
      }
    }
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int c = (threadIdx.x + k * ROW_THREADS) * 8;
      if (c < H) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          ov[k][e] = bf16_round(ov[k][e]);  // the reduced BF16 projection
          ss += ov[k][e] * ov[k][e];
        }
      }
    }
    const float sc = MODE == 1 ? __bfloat162float(scalar[0]) : 1.f;
    const float inv1 = 1.0f / sqrtf(block_sum_fresh(ss, red[0]) / H + eps);
    float ss2 = 0.f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int c = (threadIdx.x + k * ROW_THREADS) * 8;
      if (c < H) {
        float xv[8], wv[8];
        unpack8(x_raw[k], xv);
        load8(w_a + c, wv);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float on = bf16_round(ov[k][e] * inv1 * wv[e]);
          const float xa = bf16_round(xv[e] + on);
          ov[k][e] = MODE == 1 ? bf16_round(xa * sc) : xa;  // the new residual
          ss2 += ov[k][e] * ov[k][e];
        }
#pragma unroll
        for (int r = 0; r < W; ++r)
          if (r < world && (r == rank || push_x))
            store8(reinterpret_cast<__nv_bfloat16*>(p.x[r]) + (size_t)row * H + c, ov[k]);
      }
    }
    if (MODE == 0 || has_next) {
      const float inv2 = 1.0f / sqrtf(block_sum_fresh(ss2, red[1]) / H + eps);
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int c = (threadIdx.x + k * ROW_THREADS) * 8;
        if (c < H) {
          float wv[8], hv[8];
          load8(w_b + c, wv);
#pragma unroll
          for (int e = 0; e < 8; ++e) hv[e] = ov[k][e] * inv2 * wv[e];
#pragma unroll
          for (int r = 0; r < W; ++r)
            if (r < world) store8(reinterpret_cast<__nv_bfloat16*>(p.h[r]) + (size_t)row * H + c, hv);
        }
      }
    }
  }
  __syncthreads();  // every thread's stores of this row precede the release below
  if ((int)threadIdx.x < world) red_release_sys_add(p.rows[threadIdx.x] + blk, 1ull);
}

__global__ void __launch_bounds__(ROW_THREADS) wait_kernel(const unsigned long long* rows, int n_blocks,
                                                          unsigned long long target) {
  pdl_wait();  // the previous kernel on the stream has completed
  pdl_trigger();
  for (int b = threadIdx.x; b < n_blocks; b += ROW_THREADS)
    if (!wait_at_least(rows + b, target, kErrTimeoutPeerRows)) return;
}

static int check_peer(const morj_peer_t* p, const char* who) {
  if (!p || p->world < 1 || p->world > MORJ_MAX_RANKS || p->rank < 0 || p->rank >= p->world || p->max_blocks <= 0 ||
      p->hidden <= 0 || p->hidden % 8)
    return set_error(MORJ_ERR_ARG, "%s: bad exchange description", who);
  for (int r = 0; r < p->world; ++r)
    if (!p->part[r] || !p->x[r] || !p->h[r] || !p->partials[r] || !p->rows[r] ||
        ((reinterpret_cast<uintptr_t>(p->part[r]) | reinterpret_cast<uintptr_t>(p->x[r]) |
          reinterpret_cast<uintptr_t>(p->h[r])) & 15) ||
        ((reinterpret_cast<uintptr_t>(p->partials[r]) | reinterpret_cast<uintptr_t>(p->rows[r])) & 7))
      return set_error(MORJ_ERR_ARG, "%s: rank %d's buffers are missing or unaligned", who, r);
  return MORJ_OK;
}

typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

static AddressRangeFn address_range_fn() {
  static AddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(f);
  });
  return fn;
}

}  // namespace peer
}  // namespace morj

using namespace morj;

extern "C" int morj_ipc_export(const void* ptr, void* handle) {
  if (!ptr || !handle) return set_error(MORJ_ERR_ARG, "morj_ipc_export: null argument");
  peer::AddressRangeFn range = peer::address_range_fn();
  if (!range) return set_error(MORJ_ERR_CUDA, "morj_ipc_export: cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return set_error(MORJ_ERR_ARG, "morj_ipc_export: not a device allocation");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return set_error(MORJ_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  static_assert(sizeof(cudaIpcMemHandle_t) + 8 == MORJ_IPC_HANDLE_BYTES, "handle layout");
  const unsigned long long offset = reinterpret_cast<CUdeviceptr>(ptr) - base;
  std::memcpy(handle, &h, sizeof(h));
  std::memcpy(static_cast<char*>(handle) + sizeof(h), &offset, 8);
  return MORJ_OK;
}

extern "C" int morj_ipc_import(const void* handle, void** ptr) {
  if (!handle || !ptr) return set_error(MORJ_ERR_ARG, "morj_ipc_import: null argument");
  cudaIpcMemHandle_t h;
  unsigned long long offset = 0;
  std::memcpy(&h, handle, sizeof(h));
  std::memcpy(&offset, static_cast<const char*>(handle) + sizeof(h), 8);
  void* base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_error(MORJ_ERR_CUDA, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  *ptr = static_cast<char*>(base) + offset;
  return MORJ_OK;
}

extern "C" int morj_ipc_close(void* ptr, const void* handle) {
  if (!ptr || !handle) return set_error(MORJ_ERR_ARG, "morj_ipc_close: null argument");
  unsigned long long offset = 0;
  std::memcpy(&offset, static_cast<const char*>(handle) + sizeof(cudaIpcMemHandle_t), 8);
  const cudaError_t e = cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset);
  if (e != cudaSuccess) return set_error(MORJ_ERR_CUDA, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
  return MORJ_OK;
}

extern "C" int morj_peer_reduce(const morj_peer_t* p, int mode, int n, const void* w_a, const void* scalar,
                                const void* w_b, float eps, int has_next, int push_x,
                                unsigned long long partial_target, void* stream) {
  int st = peer::check_peer(p, "morj_peer_reduce");
  if (st) return st;
  if (n < 0 || n > p->max_blocks * 128 || (mode != 0 && mode != 1) || !w_a || (mode == 1 && !scalar) ||
      ((mode == 0 || has_next) && !w_b))
    return set_error(MORJ_ERR_ARG, "morj_peer_reduce: bad arguments (mode=%d n=%d)", mode, n);
  const int H = p->hidden;
  const int n_blocks = (n + 127) / 128;
  const int owned = n_blocks > p->rank ? (n_blocks - p->rank + p->world - 1) / p->world : 0;
  const unsigned grid = (unsigned)owned * 128 + 1;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const __nv_bfloat16* wa = static_cast<const __nv_bfloat16*>(w_a);
  const __nv_bfloat16* sc = static_cast<const __nv_bfloat16*>(scalar);
  const __nv_bfloat16* wb = static_cast<const __nv_bfloat16*>(w_b);
  const int hn = mode == 0 ? 1 : has_next;
  int st2 = MORJ_OK;
#define MORJ_REDUCE(MODE, W)                                                                                     \
  MORJ_VPT_SWITCH(H, (st2 = launch_pdl("peer::reduce_kernel", peer::reduce_kernel<V, MODE, W>, dim3(grid),       \
                                       dim3(ROW_THREADS), 0, s, *p, n, wa, sc, wb, eps, hn, push_x, partial_target)))
  if (p->world <= 2) {
    if (mode == 0) { MORJ_REDUCE(0, 2); } else { MORJ_REDUCE(1, 2); }
  } else if (p->world <= 4) {
    if (mode == 0) { MORJ_REDUCE(0, 4); } else { MORJ_REDUCE(1, 4); }
  } else {
    if (mode == 0) { MORJ_REDUCE(0, 8); } else { MORJ_REDUCE(1, 8); }
  }
#undef MORJ_REDUCE
  return st2;
}

extern "C" int morj_peer_wait(const morj_peer_t* p, int n, unsigned long long row_target, void* stream) {
  int st = peer::check_peer(p, "morj_peer_wait");
  if (st) return st;
  if (n < 0 || n > p->max_blocks * 128) return set_error(MORJ_ERR_ARG, "morj_peer_wait: n=%d out of range", n);
  if (n == 0) return MORJ_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return launch_pdl("peer::wait_kernel", peer::wait_kernel, dim3(1), dim3(ROW_THREADS), 0, s,
                    (const unsigned long long*)p->rows[p->rank], (n + 127) / 128, row_target);
}
