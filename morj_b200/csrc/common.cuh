// Shared device helpers for the sm_100a kernels: mbarriers with bounded waits, TMA tile loads, tcgen05 (TMEM
// allocation, UMMA issue/commit, TMEM loads), shared-memory matrix descriptors, BF16 packing, and the library's
// error reporting. Every wait in this library is bounded: when a wait runs out, the kernel records the site in
// the device error word, raises its CTA's abort flag, and returns through its normal exit path (TMEM freed).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "morj_b200.h"

#define MORJ_DEV __device__ __forceinline__

namespace morj {

// ---------------------------------------------------------------------------------------------------------------
// Error word shared by all kernels of the library (one per device): 0 = clean; otherwise the first failure's code.
// Defined in rowops.cu; the library is built with relocatable device code so every kernel sees the same word.
// ---------------------------------------------------------------------------------------------------------------
extern __device__ int g_device_error;

enum DeviceError : int {
  kErrNone = 0,
  kErrTimeoutGemmProducer = 0x101,
  kErrTimeoutGemmMma = 0x102,
  kErrTimeoutGemmEpilogue = 0x103,
  kErrTimeoutPeerPartials = 0x104,
  kErrTimeoutPeerRows = 0x105,
  kErrTimeoutGemmSplit = 0x106,
  kErrTimeoutAttention = 0x201,
  kErrBadIndex = 0x301,
  kErrBadAlignment = 0x302,
};

// a wait that has not completed after this long is treated as a hang
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

MORJ_DEV unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

MORJ_DEV void report(int code) { atomicCAS(&g_device_error, 0, code); }

MORJ_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// ---------------------------------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------------------------------
MORJ_DEV void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
MORJ_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
MORJ_DEV void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
MORJ_DEV void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
MORJ_DEV bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: a waiting thread is suspended (it takes no issue slots from the warps that are
// working) until the phase completes or about `ns` nanoseconds pass.
MORJ_DEV bool mbar_test_suspend(uint32_t bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// Wait for the phase with `parity` to complete. Returns false (after reporting `code` and raising `*abort`) when
// the wait runs past the limit, or as soon as another thread of the CTA raised `*abort` (checked every 64 tries;
// each try suspends for at most 20 us).
MORJ_DEV bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort, int code) {
  if (mbar_test(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_test_suspend(bar, parity, 20000)) return true;
    if ((i & 63) == 0) {
      if (*abort) return false;
      if (global_ns() - t0 > kWaitLimitNs) {
        *abort = 1;
        report(code);
        return false;
      }
    }
  }
}

// Wait for a phase on the exit path (copies or MMAs this CTA issued must finish before it frees its resources):
// bounded, and independent of the abort flag.
MORJ_DEV bool mbar_wait_landed(uint32_t bar, uint32_t parity) {
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 0;; ++i) {
    if (mbar_test(bar, parity)) return true;
    if ((i & 63) == 63 && global_ns() - t0 > kWaitLimitNs) return false;
  }
}

// ---------------------------------------------------------------------------------------------------------------
// TMA (tiled, no multicast anywhere in this library)
// ---------------------------------------------------------------------------------------------------------------
MORJ_DEV void tma_prefetch(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
MORJ_DEV void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
MORJ_DEV void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}
MORJ_DEV uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
MORJ_DEV uint64_t policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}
MORJ_DEV uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
MORJ_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---------------------------------------------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, commit, loads
// ---------------------------------------------------------------------------------------------------------------
MORJ_DEV void tmem_alloc(uint32_t slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem), "r"(ncols)
               : "memory");
}
MORJ_DEV void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
MORJ_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
MORJ_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
MORJ_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, BF16 inputs, FP32 accumulator; `accumulate` = 0 overwrites D.
MORJ_DEV void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D (TMEM) (+)= A . B with A read from TMEM (128 lanes = rows, 16-bit elements packed in pairs along K per column)
MORJ_DEV void umma_bf16_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// the mbarrier receives one arrival once every MMA issued so far by this thread has completed
MORJ_DEV void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives lane (base + i), columns [col, col + 32)
MORJ_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
MORJ_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 16 consecutive 32-bit columns (as tmem_ld32, half the columns)
MORJ_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// 32 lanes x 32 consecutive 32-bit columns from registers into TMEM (the inverse of tmem_ld32)
MORJ_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
MORJ_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 2^x with the SFU's approximate exponential (PTX ex2.approx.ftz.f32)
MORJ_DEV float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Shared-memory matrix descriptor for a 128-byte-swizzled tile whose 8-row groups are 1024 bytes apart
// (K-major operand, or MN-major operand with `lbo` = distance between 64-element column groups).
MORJ_DEV uint64_t sw128_desc(uint32_t saddr, uint32_t lbo_bytes = 16) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  d |= (uint64_t)2 << 61;  // 128-byte swizzle
  return d;
}

// Instruction descriptor: BF16 x BF16 -> FP32, M x N tile; `b_mn_major` when B is stored N-contiguous.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool b_mn_major = false) {
  return (1u << 4)                      // D format: FP32
         | (1u << 7)                    // A format: BF16
         | (1u << 10)                   // B format: BF16
         | ((b_mn_major ? 1u : 0u) << 16)
         | ((uint32_t)(N >> 3) << 17)   // N / 8
         | ((uint32_t)(M >> 4) << 24);  // M / 16
}

// byte offset of 16-byte chunk `c` (0..7) of row `r` inside a 128-byte-swizzled [rows x 128 B] block
MORJ_DEV uint32_t sw128_offset(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

// ---------------------------------------------------------------------------------------------------------------
// 2-CTA clusters: the pair of SMs that share one tcgen05.mma.cta_group::2 (no multicast loads anywhere)
// ---------------------------------------------------------------------------------------------------------------
MORJ_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// the address of the same shared-memory location in CTA `rank` of the cluster
MORJ_DEV uint32_t map_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
MORJ_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrival on a barrier that may live in the peer CTA of the pair. Relaxed: it signals that this warp's reads of the
// accumulator (completed by tcgen05.wait::ld before it) are done, and orders none of the warp's global stores, which
// a release at cluster scope would make it wait for.
MORJ_DEV void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// TMA tile load whose completion is counted on an mbarrier that may live in the peer CTA of the pair
MORJ_DEV void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar_cluster, int x, int y,
                               uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
MORJ_DEV void tmem_alloc_pair(uint32_t slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem), "r"(ncols)
               : "memory");
}
MORJ_DEV void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
MORJ_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D (both CTAs' TMEM, 128 rows each) (+)= A (128 rows in each CTA) * B^T (N/2 rows in each CTA)
MORJ_DEV void umma_bf16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// one arrival on the barrier at the same offset in both CTAs once the pair's MMAs issued so far have completed
MORJ_DEV void umma_commit_pair(uint32_t bar) {
  const uint16_t both = 0x3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"(both)
      : "memory");
}

// ---------------------------------------------------------------------------------------------------------------
// numerics helpers
// ---------------------------------------------------------------------------------------------------------------
MORJ_DEV float bf16_round(float x) { return __bfloat162float(__float2bfloat16(x)); }
MORJ_DEV uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
MORJ_DEV float2 unpack_bf16x2(uint32_t v) {
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&v);
  return __bfloat1622float2(b);
}
MORJ_DEV void unpack8_bf16(uint4 u, float (&v)[8]) {
  const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), c = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
  v[0] = a.x, v[1] = a.y, v[2] = b.x, v[3] = b.y, v[4] = c.x, v[5] = c.y, v[6] = d.x, v[7] = d.y;
}

// ---------------------------------------------------------------------------------------------------------------
// row helpers (one CTA per token row, 8-wide BF16 vectors, FP32 reductions)
// ---------------------------------------------------------------------------------------------------------------
constexpr int ROW_THREADS = 256;

MORJ_DEV float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  __syncthreads();  // red may still be read by a previous reduction
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  const int nw = blockDim.x / 32;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

// block_sum into a `red` array that no earlier reduction of this CTA has used: one barrier instead of two (a CTA
// that reduces twice per row gives each reduction its own array)
MORJ_DEV float block_sum_fresh(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = v;
  __syncthreads();
  float t = 0.f;
  const int nw = blockDim.x / 32;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

MORJ_DEV void load8(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), c = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
}
MORJ_DEV void unpack8(const uint4& u, float (&v)[8]) {
  float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), c = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
}
MORJ_DEV uint4 pack8(const float (&v)[8]) {
  uint4 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  u.z = pack_bf16x2(v[4], v[5]);
  u.w = pack_bf16x2(v[6], v[7]);
  return u;
}
MORJ_DEV void store8(__nv_bfloat16* p, const float (&v)[8]) {
  uint4 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  u.z = pack_bf16x2(v[4], v[5]);
  u.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

// hidden sizes up to 16384: VPT = 8-element vectors per thread of a ROW_THREADS-thread row CTA
inline int vpt_for(int H) { return (H / 8 + ROW_THREADS - 1) / ROW_THREADS; }
#define MORJ_VPT_SWITCH(H, CALL)                                                      \
  switch (vpt_for(H)) {                                                               \
    case 1: { constexpr int V = 1; CALL; break; }                                     \
    case 2: { constexpr int V = 2; CALL; break; }                                     \
    case 3: { constexpr int V = 3; CALL; break; }                                     \
    case 4: { constexpr int V = 4; CALL; break; }                                     \
    case 5: { constexpr int V = 5; CALL; break; }                                     \
    case 6: { constexpr int V = 6; CALL; break; }                                     \
    case 7: { constexpr int V = 7; CALL; break; }                                     \
    case 8: { constexpr int V = 8; CALL; break; }                                     \
    default: return set_error(MORJ_ERR_UNSUPPORTED, "hidden size %d above 16384", H); \
  }

// GELU, tanh form, computed as the reference's GeGLU kernel computes it (FlashInfer `gelu_tanh_and_mul`,
// `lean_core.py:685`): x * (0.5 * (1 + tanh(sqrt(2 / pi) * (x + 0.044715 x^3)))) with the hardware tanh approximation
// (PTX `tanh.approx.f32`, one instruction).
MORJ_DEV float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
MORJ_DEV float gelu_tanh(float x) {
  const float cdf = 0.5f * (1.0f + tanh_approx(0.7978845608028654f * (x + 0.044715f * x * x * x)));
  return x * cdf;
}

// host side: status and the calling thread's last error message (rowops.cu)
int set_error(int code, const char* fmt, ...);
int check_launch(const char* what);

// ---------------------------------------------------------------------------------------------------------------
// Programmatic dependent launch. Every kernel of this library is launched with launch_pdl, so the GPU may schedule
// it (and it may run its prologue: barrier set-up, TMEM allocation, tensor-map prefetch) while the previous kernel on
// the stream is still finishing. pdl_wait() returns once that kernel has completed and its memory operations are
// visible: each kernel calls it before its first access to global memory. pdl_trigger() lets the next kernel's CTAs
// be scheduled; it orders nothing, the next kernel's own pdl_wait() does.
// ---------------------------------------------------------------------------------------------------------------
MORJ_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
MORJ_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline int launch_pdl(const char* what, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                      cudaStream_t stream, Args... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) return set_error(MORJ_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
  return MORJ_OK;
}

// host side: tiled tensor maps (driver entry point resolved at run time; gemm_sm100.cu)
int encode_tiled(CUtensorMap* map, CUtensorMapDataType type, int rank, const void* ptr, const unsigned long long* dims,
                 const unsigned long long* strides_bytes, const unsigned* box, CUtensorMapSwizzle swizzle);
int num_sms();

}  // namespace morj
