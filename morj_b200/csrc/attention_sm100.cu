// Tree-masked paged prefill attention for sm_100a.
//
// One CTA (4 warps) handles one work tile: a segment's block of 128/G consecutive queries for one KV head, with the
// G = hq/hk query heads that share that KV head packed into the 128 MMA rows (row = query * G + head). For every
// chunk of 64 keys of the segment's key list it
//   1. gathers the K and V rows of the chunk from the paged pool (slot = page * page_size + offset) into 128-byte-
//      swizzled shared memory with cp.async (double-buffered: the next chunk loads while this one computes),
//   2. issues S = Q K^T on the tensor cores (tcgen05.mma, M=128, N=64, accumulator in TMEM),
//   3. reads S back (thread = row), applies the tree mask (bottom-right causal, sliding window, bidirectional image
//      blocks) and the online softmax in FP32, and writes P as BF16 to shared memory,
//   4. issues O_chunk = P V (tcgen05.mma with V as an N-major operand, so K and V share one shared-memory layout),
//   5. accumulates O_chunk into registers with the softmax rescale.
// The key range of a tile is cut to what its queries can see (the window and causal bounds), so a sliding layer's
// long prefix costs O(window) per tile.
#include "common.cuh"

namespace morj {
namespace attn {

constexpr int ROWS = 128;
constexpr int BN = 64;
constexpr int THREADS = 128;
constexpr int TMEM_COLS = 256;  // S at columns [0, 64), O chunk at [128, 128 + D)
constexpr float LOG2E = 1.4426950408889634f;

template <int D>
struct Smem {
  static constexpr int Q_BYTES = ROWS * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int P_BYTES = ROWS * BN * 2;
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + Q_BYTES;       // 2 buffers
  static constexpr int V_OFF = K_OFF + 2 * KV_BYTES;  // 2 buffers
  static constexpr int P_OFF = V_OFF + 2 * KV_BYTES;
  static constexpr int BAR_OFF = P_OFF + P_BYTES;
  // barriers; the dynamic shared window starts 1024-byte aligned (checked in the kernel), so two CTAs fit an SM
  static constexpr int TOTAL = BAR_OFF + 64;
};

MORJ_DEV void cp_async16(uint32_t dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
MORJ_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
MORJ_DEV void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

struct Segment {
  int q_start, q_len, kv_base, kv_len;
};

// pool slot of key position t of a segment
MORJ_DEV int key_slot(const int* __restrict__ kv_indices, int kv_base, int t, int page_size) {
  if (page_size == 1) return __ldg(kv_indices + kv_base + t);
  const int page = __ldg(kv_indices + kv_base + t / page_size);
  return page * page_size + t % page_size;
}

// gather K and V rows of keys [t0, t0 + BN) (zeros past t_end) into one buffer pair
template <int D>
MORJ_DEV void load_kv_chunk(uint32_t k_dst, uint32_t v_dst, const __nv_bfloat16* __restrict__ k_pool,
                            const __nv_bfloat16* __restrict__ v_pool, const int* __restrict__ kv_indices,
                            const Segment& sg, int t0, int t_end, int hk, int h, int page_size) {
  constexpr int CH = D / 8;  // 16-byte chunks per row
  for (int id = threadIdx.x; id < BN * CH; id += THREADS) {
    const int k = id / CH, c16 = id % CH;
    const int t = t0 + k;
    const bool ok = t < t_end;
    const size_t row = ok ? ((size_t)key_slot(kv_indices, sg.kv_base, t, page_size) * hk + h) * D : 0;
    const uint32_t off = (uint32_t)((c16 >> 3) * (BN * 128)) + sw128_offset(k, c16 & 7);
    cp_async16(k_dst + off, k_pool + row + c16 * 8, ok ? 16u : 0u);
    cp_async16(v_dst + off, v_pool + row + c16 * 8, ok ? 16u : 0u);
  }
}

template <int D>
__global__ void __launch_bounds__(THREADS, 2)
    tree_attention_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k_pool,
                          const __nv_bfloat16* __restrict__ v_pool, __nv_bfloat16* __restrict__ out,
                          const int* __restrict__ qo_indptr, const int* __restrict__ kv_indptr,
                          const int* __restrict__ kv_indices, const int* __restrict__ kv_last_page_len, int n_bidir,
                          int hq, int hk, int page_size, int window, float scale_log2, const int* __restrict__ work) {
  using L = Smem<D>;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  if (sbase & 1023) {  // the swizzled operand tiles need 1024-byte alignment
    if (threadIdx.x == 0) report(kErrBadAlignment);
    return;
  }
  const uint32_t bar_s = sbase + L::BAR_OFF, bar_o = bar_s + 8, bar_d = bar_s + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::BAR_OFF + 24);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::BAR_OFF + 28);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int seg = work[2 * blockIdx.x], q0 = work[2 * blockIdx.x + 1];
  const int h = blockIdx.y;
  const int G = hq / hk;
  const int QT = ROWS / G;

  Segment sg;
  sg.q_start = qo_indptr[seg];
  sg.q_len = qo_indptr[seg + 1] - sg.q_start;
  sg.kv_base = kv_indptr[seg];
  const int pages = kv_indptr[seg + 1] - sg.kv_base;
  sg.kv_len = page_size == 1 ? pages
                             : (pages - 1) * page_size + (kv_last_page_len ? kv_last_page_len[seg] : page_size);
  const bool bidir = seg < n_bidir;
  const int q_last = min(q0 + QT, sg.q_len) - 1;  // last valid query of the tile
  const int diag = sg.kv_len - sg.q_len;          // key aligned with query 0

  // key range the tile can see
  int t_begin, t_end;
  if (bidir) {
    t_end = sg.kv_len;
    t_begin = window > 0 ? max(0, diag + min(0, q0 - (window - 1))) : 0;
  } else {
    t_end = diag + q_last + 1;
    t_begin = window > 0 ? max(0, diag + q0 - (window - 1)) : 0;
  }
  const int n_chunks = (t_end - t_begin + BN - 1) / BN;

  if (threadIdx.x == 0) {
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    mbar_init(bar_d, 1);
    *abort = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }

  // Q tile: row r = query (r / G) of the tile, head h * G + r % G; zeros past the segment
  {
    constexpr int CH = D / 8;
    for (int id = threadIdx.x; id < ROWS * CH; id += THREADS) {
      const int r = id / CH, c16 = id % CH;
      const int qi = q0 + r / G;
      const bool ok = qi < sg.q_len;
      const size_t src = ok ? ((size_t)(sg.q_start + qi) * hq + h * G + r % G) * D : 0;
      const uint32_t off = (uint32_t)((c16 >> 3) * (ROWS * 128)) + sw128_offset(r, c16 & 7);
      cp_async16(sbase + L::Q_OFF + off, q + src + c16 * 8, ok ? 16u : 0u);
    }
  }
  load_kv_chunk<D>(sbase + L::K_OFF, sbase + L::V_OFF, k_pool, v_pool, kv_indices, sg, t_begin, t_end, hk, h,
                   page_size);
  cp_async_commit();

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_lane = tmem + ((uint32_t)(warp * 32) << 16);
  const uint32_t tm_s = t_lane, tm_o = t_lane + 128;  // this warp's lanes of S and O

  // this thread's row
  const int r = threadIdx.x;
  const int qi = q0 + r / G;
  const bool row_ok = qi < sg.q_len;
  int lo, hi;  // visible key positions [lo, hi]
  if (bidir) {
    hi = sg.kv_len - 1;
    lo = window > 0 ? diag + min(0, qi - (window - 1)) : 0;
  } else {
    hi = diag + qi;
    lo = window > 0 ? hi - (window - 1) : 0;
  }
  if (!row_ok) {
    lo = 1;
    hi = 0;
  }

  float o_acc[D];
#pragma unroll
  for (int i = 0; i < D; ++i) o_acc[i] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;

  constexpr uint32_t IDESC_S = idesc_bf16(ROWS, BN);
  constexpr uint32_t IDESC_O = idesc_bf16(ROWS, D, /*b_mn_major=*/true);
  bool failed = false;

  for (int ci = 0; ci < n_chunks; ++ci) {
    const int buf = ci & 1;
    const int t0 = t_begin + ci * BN;
    if (ci + 1 < n_chunks) {
      const int nb = buf ^ 1;
      load_kv_chunk<D>(sbase + L::K_OFF + nb * L::KV_BYTES, sbase + L::V_OFF + nb * L::KV_BYTES, k_pool, v_pool,
                       kv_indices, sg, t0 + BN, t_end, hk, h, page_size);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    const uint32_t k_s = sbase + L::K_OFF + buf * L::KV_BYTES;
    const uint32_t v_s = sbase + L::V_OFF + buf * L::KV_BYTES;
    if (threadIdx.x == 0) {
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t qa = sbase + L::Q_OFF + (kk >> 2) * (ROWS * 128) + (kk & 3) * 32;
        const uint32_t kb = k_s + (kk >> 2) * (BN * 128) + (kk & 3) * 32;
        umma_bf16(tmem, sw128_desc(qa), sw128_desc(kb), IDESC_S, kk > 0);
      }
      umma_commit(bar_s);
    }
    // every warp's lane 0 waits; the CTA acts on one verdict so no thread is left at a barrier alone
    int ok = lane == 0 ? (int)mbar_wait(bar_s, ci & 1, abort, kErrTimeoutAttention) : 1;
    ok = __syncthreads_and(ok);
    if (!ok) {
      failed = true;
      break;
    }
    tc_fence_after();

    // scores of this row for keys t0 .. t0 + 63
    uint32_t sr[2][32];
    tmem_ld32(tm_s, sr[0]);
    tmem_ld32(tm_s + 32, sr[1]);
    tmem_wait_ld();
    float s[BN];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < BN; ++j) {
      const int t = t0 + j;
      const bool vis = t >= lo && t <= hi;
      s[j] = vis ? __uint_as_float(sr[j >> 5][j & 31]) * scale_log2 : -INFINITY;
      mx = fmaxf(mx, s[j]);
    }
    const float m_new = fmaxf(m_run, mx);
    const float alpha = (m_run == -INFINITY) ? 0.f : exp2f(m_run - m_new);
    float psum = 0.f;
    uint32_t pk[BN / 2];
#pragma unroll
    for (int j = 0; j < BN; j += 2) {
      const float p0 = (s[j] == -INFINITY) ? 0.f : exp2f(s[j] - m_new);
      const float p1 = (s[j + 1] == -INFINITY) ? 0.f : exp2f(s[j + 1] - m_new);
      psum += p0 + p1;
      pk[j / 2] = pack_bf16x2(p0, p1);
    }
    l_run = l_run * alpha + psum;
    m_run = m_new;
    // P row r -> shared memory (K-major, one 128-byte swizzle atom wide)
    {
      uint8_t* prow = smem + L::P_OFF;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 v = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        *reinterpret_cast<uint4*>(prow + sw128_offset(r, c)) = v;
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x == 0) {
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk) {
        const uint32_t pa = sbase + L::P_OFF + kk * 32;
        const uint32_t vb = v_s + kk * 2048;
        umma_bf16(tmem + 128, sw128_desc(pa), sw128_desc(vb, BN * 128), IDESC_O, kk > 0);
      }
      umma_commit(bar_o);
    }
    ok = lane == 0 ? (int)mbar_wait(bar_o, ci & 1, abort, kErrTimeoutAttention) : 1;
    ok = __syncthreads_and(ok);
    if (!ok) {
      failed = true;
      break;
    }
    tc_fence_after();
#pragma unroll
    for (int c = 0; c < D; c += 32) {
      uint32_t orr[32];
      tmem_ld32(tm_o + c, orr);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) o_acc[c + i] = o_acc[c + i] * alpha + __uint_as_float(orr[i]);
    }
  }

  if (!failed && row_ok) {
    const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
    __nv_bfloat16* dst = out + ((size_t)(sg.q_start + qi) * hq + h * G + r % G) * D;
#pragma unroll
    for (int c = 0; c < D; c += 8) {
      uint4 v;
      v.x = pack_bf16x2(o_acc[c + 0] * inv, o_acc[c + 1] * inv);
      v.y = pack_bf16x2(o_acc[c + 2] * inv, o_acc[c + 3] * inv);
      v.z = pack_bf16x2(o_acc[c + 4] * inv, o_acc[c + 5] * inv);
      v.w = pack_bf16x2(o_acc[c + 6] * inv, o_acc[c + 7] * inv);
      *reinterpret_cast<uint4*>(dst + c) = v;
    }
  }
  // exit: no copy or MMA of this CTA may be in flight when its shared memory and TMEM go away
  cp_async_wait<0>();
  if (failed && threadIdx.x == 0) {
    umma_commit(bar_d);
    mbar_wait_landed(bar_d, 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

template <int D>
static int launch(const void* q, const void* k_pool, const void* v_pool, void* out, const int* qo_indptr,
                  const int* kv_indptr, const int* kv_indices, const int* kv_last_page_len, int n_bidir, int hq,
                  int hk, int page_size, int window, float sm_scale, const int* work, int n_work,
                  cudaStream_t stream) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(tree_attention_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Smem<D>::TOTAL);
    if (e != cudaSuccess) return set_error(MORJ_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    configured = true;
  }
  dim3 grid(n_work, hk);
  tree_attention_kernel<D><<<grid, THREADS, Smem<D>::TOTAL, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(q), reinterpret_cast<const __nv_bfloat16*>(k_pool),
      reinterpret_cast<const __nv_bfloat16*>(v_pool), reinterpret_cast<__nv_bfloat16*>(out), qo_indptr, kv_indptr,
      kv_indices, kv_last_page_len, n_bidir, hq, hk, page_size, window, sm_scale * LOG2E, work);
  return check_launch("tree_attention_kernel");
}

}  // namespace attn
}  // namespace morj

extern "C" int morj_tree_attention_work(const int* qo_indptr_host, int n_segments, int hq, int hk, int* work_host,
                                        int cap) {
  using namespace morj;
  if (!qo_indptr_host || n_segments < 0 || hk <= 0 || hq <= 0 || hq % hk) {
    set_error(MORJ_ERR_ARG, "morj_tree_attention_work: bad arguments");
    return -1;
  }
  const int G = hq / hk;
  if (attn::ROWS % G) {
    set_error(MORJ_ERR_ARG, "morj_tree_attention_work: group %d does not divide 128", G);
    return -1;
  }
  const int QT = attn::ROWS / G;
  int n = 0;
  // within a segment, later tiles first: they see the most keys under the causal mask
  for (int s = 0; s < n_segments; ++s) {
    const int len = qo_indptr_host[s + 1] - qo_indptr_host[s];
    for (int q0 = ((len - 1) / QT) * QT; q0 >= 0 && len > 0; q0 -= QT) {
      if (n < cap && work_host) {
        work_host[2 * n] = s;
        work_host[2 * n + 1] = q0;
      }
      ++n;
    }
  }
  if (n > cap) {
    set_error(MORJ_ERR_ARG, "morj_tree_attention_work: %d tiles exceed capacity %d", n, cap);
    return -1;
  }
  return n;
}

extern "C" int morj_tree_attention(const void* q, const void* k_pool, const void* v_pool, void* out,
                                   const int* qo_indptr, const int* kv_indptr, const int* kv_indices,
                                   const int* kv_last_page_len, int n_segments, int n_bidir, int hq, int hk, int d,
                                   int page_size, int window, float sm_scale, const int* work, int n_work,
                                   void* stream) {
  using namespace morj;
  if (n_work == 0 || n_segments == 0) return MORJ_OK;
  if (!q || !k_pool || !v_pool || !out || !qo_indptr || !kv_indptr || !kv_indices || !work || n_work < 0)
    return set_error(MORJ_ERR_ARG, "morj_tree_attention: null pointer or negative size");
  if (hq <= 0 || hk <= 0 || hq % hk || attn::ROWS % (hq / hk))
    return set_error(MORJ_ERR_ARG, "morj_tree_attention: hq=%d hk=%d unsupported", hq, hk);
  if (page_size <= 0 || n_bidir < 0 || n_bidir > n_segments)
    return set_error(MORJ_ERR_ARG, "morj_tree_attention: bad page_size %d or n_bidir %d", page_size, n_bidir);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (d == 128)
    return attn::launch<128>(q, k_pool, v_pool, out, qo_indptr, kv_indptr, kv_indices, kv_last_page_len, n_bidir, hq,
                             hk, page_size, window, sm_scale, work, n_work, s);
  if (d == 64)
    return attn::launch<64>(q, k_pool, v_pool, out, qo_indptr, kv_indptr, kv_indices, kv_last_page_len, n_bidir, hq,
                            hk, page_size, window, sm_scale, work, n_work, s);
  return set_error(MORJ_ERR_UNSUPPORTED, "morj_tree_attention: head_dim %d unsupported (64, 128)", d);
}
