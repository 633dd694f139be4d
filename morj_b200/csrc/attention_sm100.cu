// Tree-masked paged prefill attention for sm_100a.
//
// One CTA handles one work tile: a segment's block of 128/G consecutive queries for one KV head, the G = hq/hk query
// heads that share that KV head packed into the 128 MMA rows (row = query * G + head). The CTA is warp-specialised:
//   warp 0      loader: gathers the K and V rows of each 64-key chunk from the paged pool (slot = page * page_size +
//               offset) into 128-byte-swizzled shared memory with cp.async, two chunks in flight
//   warp 1      MMA issuer (one thread): S_c = Q K_c^T into one of two TMEM score buffers, then O += P_{c-1} V_{c-1}
//               into the TMEM output, so the tensor cores compute chunk c+1's scores while the softmax works on c
//   warps 2-5   softmax (thread = row): tree mask (bottom-right causal bound, sliding window, image-block rule), online
//               softmax in FP32 with a lazily rescaled running maximum (O in TMEM is rescaled only when a row's
//               maximum grows by more than 2^8), P as BF16 to shared memory, and the final O / l store
// V is read as an N-major operand, so one shared-memory layout serves K (for QK^T) and V (for PV). The key range of a
// tile is cut to what its queries can see, so a sliding layer's long prefix costs O(window) per tile.
#include "common.cuh"

namespace morj {
namespace attn {

constexpr int ROWS = 128;
constexpr int BN = 64;
constexpr int THREADS = 192;
constexpr int TMEM_COLS = 256;  // S buffers at columns [0, 64) and [64, 128), O at [128, 128 + D)
constexpr float LOG2E = 1.4426950408889634f;
constexpr float RESCALE_LOG2 = 8.0f;  // rescale O only when a row maximum grows by more than 2^8

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
  // barriers: kv_full[2], kv_empty[2], s_full[2], s_free[2], p_full, o_done, done; then the TMEM slot and abort flag.
  // The dynamic shared window starts 1024-byte aligned (checked in the kernel), so two CTAs fit an SM.
  static constexpr int TOTAL = BAR_OFF + 128;
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

// warp-level wait: lane 0 polls the barrier, the warp follows its verdict
MORJ_DEV bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
  int ok = (threadIdx.x & 31) == 0 ? (int)mbar_wait(bar, parity, abort, kErrTimeoutAttention) : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// one warp gathers the K and V rows of keys [t0, t0 + BN) (zeros past t_end) into one buffer pair
template <int D>
MORJ_DEV void load_kv_chunk(uint32_t k_dst, uint32_t v_dst, const __nv_bfloat16* __restrict__ k_pool,
                            const __nv_bfloat16* __restrict__ v_pool, const int* __restrict__ kv_indices,
                            const Segment& sg, int t0, int t_end, int hk, int h, int page_size, int lane) {
  constexpr int CH = D / 8;  // 16-byte chunks per row
  for (int k = lane; k < BN; k += 32) {
    const int t = t0 + k;
    const bool ok = t < t_end;
    const size_t row = ok ? ((size_t)key_slot(kv_indices, sg.kv_base, t, page_size) * hk + h) * D : 0;
    const __nv_bfloat16* ks = k_pool + row;
    const __nv_bfloat16* vs = v_pool + row;
#pragma unroll
    for (int c16 = 0; c16 < CH; ++c16) {
      const uint32_t off = (uint32_t)((c16 >> 3) * (BN * 128)) + sw128_offset(k, c16 & 7);
      cp_async16(k_dst + off, ks + c16 * 8, ok ? 16u : 0u);
      cp_async16(v_dst + off, vs + c16 * 8, ok ? 16u : 0u);
    }
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
  const uint32_t bar0 = sbase + L::BAR_OFF;
  const uint32_t kv_full = bar0, kv_empty = bar0 + 16, s_full = bar0 + 32, s_free = bar0 + 48;
  const uint32_t p_full = bar0 + 64, o_done = bar0 + 72, done = bar0 + 80;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::BAR_OFF + 96);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::BAR_OFF + 100);

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
    for (int b = 0; b < 2; ++b) {
      mbar_init(kv_full + 8 * b, 1);
      mbar_init(kv_empty + 8 * b, 1);
      mbar_init(s_full + 8 * b, 1);
      mbar_init(s_free + 8 * b, 4);
    }
    mbar_init(p_full, 4);
    mbar_init(o_done, 1);
    mbar_init(done, 1);
    *abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- loader ----------------
    // chunk c goes to buffer c & 1; chunk 0's copy group also carries the Q tile
    constexpr int CH = D / 8;
    for (int id = lane; id < ROWS * CH; id += 32) {
      const int r = id / CH, c16 = id % CH;
      const int qi = q0 + r / G;
      const bool ok = qi < sg.q_len;
      const size_t src = ok ? ((size_t)(sg.q_start + qi) * hq + h * G + r % G) * D : 0;
      const uint32_t off = (uint32_t)((c16 >> 3) * (ROWS * 128)) + sw128_offset(r, c16 & 7);
      cp_async16(sbase + L::Q_OFF + off, q + src + c16 * 8, ok ? 16u : 0u);
    }
    // Chunk c is published (kv_full) as soon as it has landed, before the loader waits for a buffer to reuse: the
    // issuer needs chunk c's keys to run S_c and then PV_{c-1}, and that PV is what frees the buffer of chunk c + 1.
    load_kv_chunk<D>(sbase + L::K_OFF, sbase + L::V_OFF, k_pool, v_pool, kv_indices, sg, t_begin, t_end, hk, h,
                     page_size, lane);
    cp_async_commit();
    bool ok = true;
    for (int c = 1; c < n_chunks; ++c) {
      cp_async_wait<0>();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(kv_full + 8 * ((c - 1) & 1));
      const int b = c & 1;
      if (c >= 2 && !warp_wait(kv_empty + 8 * b, ((c >> 1) - 1) & 1, abort)) {
        ok = false;
        break;
      }
      load_kv_chunk<D>(sbase + L::K_OFF + b * L::KV_BYTES, sbase + L::V_OFF + b * L::KV_BYTES, k_pool, v_pool,
                       kv_indices, sg, t_begin + c * BN, t_end, hk, h, page_size, lane);
      cp_async_commit();
    }
    cp_async_wait<0>();
    if (ok) {
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(kv_full + 8 * ((n_chunks - 1) & 1));
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t IDESC_S = idesc_bf16(ROWS, BN);
      constexpr uint32_t IDESC_O = idesc_bf16(ROWS, D, /*b_mn_major=*/true);
      bool ok = true;
      auto issue_pv = [&](int j) -> bool {
        if (!mbar_wait(p_full, j & 1, abort, kErrTimeoutAttention)) return false;
        tc_fence_after();
        const uint32_t v_s = sbase + L::V_OFF + (j & 1) * L::KV_BYTES;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint32_t pa = sbase + L::P_OFF + kk * 32;
          const uint32_t vb = v_s + kk * 2048;
          umma_bf16(tmem + 128, sw128_desc(pa), sw128_desc(vb, BN * 128), IDESC_O, (j | kk) != 0);
        }
        umma_commit(o_done);
        umma_commit(kv_empty + 8 * (j & 1));
        return true;
      };
      for (int c = 0; c < n_chunks && ok; ++c) {
        const int b = c & 1;
        if (!mbar_wait(kv_full + 8 * b, (c >> 1) & 1, abort, kErrTimeoutAttention)) {
          ok = false;
          break;
        }
        if (c >= 2 && !mbar_wait(s_free + 8 * b, ((c >> 1) - 1) & 1, abort, kErrTimeoutAttention)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k_s = sbase + L::K_OFF + b * L::KV_BYTES;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t qa = sbase + L::Q_OFF + (kk >> 2) * (ROWS * 128) + (kk & 3) * 32;
          const uint32_t kb = k_s + (kk >> 2) * (BN * 128) + (kk & 3) * 32;
          umma_bf16(tmem + b * BN, sw128_desc(qa), sw128_desc(kb), IDESC_S, kk > 0);
        }
        umma_commit(s_full + 8 * b);
        if (c >= 1) ok = issue_pv(c - 1);
      }
      if (ok) issue_pv(n_chunks - 1);
      // TMEM is freed only after every MMA issued here has completed
      umma_commit(done);
      mbar_wait_landed(done, 0);
    }
  } else {
    // ---------------- softmax warpgroup ----------------
    const int quarter = warp & 3;  // TMEM lanes 32 * quarter .. + 31
    const int r = quarter * 32 + lane;
    const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
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
    float m_used = -INFINITY, l_run = 0.f;
    bool ok = true;
    uint8_t* prow = smem + L::P_OFF;
    for (int c = 0; c < n_chunks; ++c) {
      const int b = c & 1;
      if (!warp_wait(s_full + 8 * b, (c >> 1) & 1, abort)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[2][32];
      tmem_ld32(t_lane + b * BN, sr[0]);
      tmem_ld32(t_lane + b * BN + 32, sr[1]);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free + 8 * b);
      const int t0 = t_begin + c * BN;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < BN; ++j) {
        const int t = t0 + j;
        const float v = (t >= lo && t <= hi) ? __uint_as_float(sr[j >> 5][j & 31]) * scale_log2 : -INFINITY;
        sr[j >> 5][j & 31] = __float_as_uint(v);
        mx = fmaxf(mx, v);
      }
      float alpha = 1.f;
      if (mx > m_used + RESCALE_LOG2 || m_used == -INFINITY) {
        if (m_used != -INFINITY) alpha = fast_exp2(m_used - mx);
        if (mx != -INFINITY) m_used = mx;
      }
      l_run *= alpha;
      float psum = 0.f;
      uint32_t pk[BN / 2];
#pragma unroll
      for (int j = 0; j < BN; j += 2) {
        const float s0 = __uint_as_float(sr[j >> 5][j & 31]);
        const float s1 = __uint_as_float(sr[(j + 1) >> 5][(j + 1) & 31]);
        const float p0 = s0 == -INFINITY ? 0.f : fast_exp2(s0 - m_used);
        const float p1 = s1 == -INFINITY ? 0.f : fast_exp2(s1 - m_used);
        psum += p0 + p1;
        pk[j / 2] = pack_bf16x2(p0, p1);
      }
      l_run += psum;
      // P and O are free once the previous chunk's PV has completed
      if (c >= 1) {
        if (!warp_wait(o_done, (c - 1) & 1, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
          for (int col = 0; col < D; col += 32) {
            uint32_t o[32];
            tmem_ld32(t_lane + 128 + col, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(t_lane + 128 + col, o);
          }
          tmem_wait_st();
        }
      }
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        uint4 v = make_uint4(pk[4 * cc], pk[4 * cc + 1], pk[4 * cc + 2], pk[4 * cc + 3]);
        *reinterpret_cast<uint4*>(prow + sw128_offset(r, cc)) = v;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (ok && warp_wait(o_done, (n_chunks - 1) & 1, abort)) {
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      __nv_bfloat16* dst = out + ((size_t)(sg.q_start + qi) * hq + h * G + r % G) * D;
#pragma unroll 1
      for (int col = 0; col < D; col += 32) {
        uint32_t o[32];
        tmem_ld32(t_lane + 128 + col, o);
        tmem_wait_ld();
        if (row_ok) {
#pragma unroll
          for (int v8 = 0; v8 < 4; ++v8) {
            uint4 v;
            v.x = pack_bf16x2(__uint_as_float(o[v8 * 8 + 0]) * inv, __uint_as_float(o[v8 * 8 + 1]) * inv);
            v.y = pack_bf16x2(__uint_as_float(o[v8 * 8 + 2]) * inv, __uint_as_float(o[v8 * 8 + 3]) * inv);
            v.z = pack_bf16x2(__uint_as_float(o[v8 * 8 + 4]) * inv, __uint_as_float(o[v8 * 8 + 5]) * inv);
            v.w = pack_bf16x2(__uint_as_float(o[v8 * 8 + 6]) * inv, __uint_as_float(o[v8 * 8 + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + col + v8 * 8) = v;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
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
