// Tree-masked paged prefill attention for sm_100a.
//
// One CTA handles one work tile: a segment's block of 128/G consecutive queries for one KV head, the G = hq/hk query
// heads that share that KV head packed into the 128 MMA rows (row = query * G + head). The CTA is warp-specialised:
//   warp 0      K loader: the Q tile (TMA), then each 64-key chunk's K rows into a two-deep ring: one TMA tile load
//               per head-dim half when the chunk's pool slots are contiguous (tree nodes own contiguous slot runs;
//               pages hold 64 slots), a cp.async row gather otherwise
//   warp 1      MMA issuer (one thread): S_c = Q K_c^T into TMEM buffer c % 2, and O += P_c V_c with P read from
//               TMEM, so the tensor cores compute chunk c+1's scores while the softmax works on c
//   warp 2      V loader: the same for V, on its own ring (K of chunk c+2 is fetched as soon as S_c is done)
//   warps 4-7   softmax (thread = row): tree mask (bottom-right causal bound, sliding window, image-block rule), online
//               softmax in FP32 with a lazily rescaled running maximum (O in TMEM is rescaled only when a row's
//               maximum grows by more than 2^8), P as BF16 written over its own scores in TMEM, and the final O / l
//               store
// P never leaves TMEM: chunk c's P is packed over the first half of S_c's columns and consumed there by the PV MMA, so
// two score buffers double-buffer P too. S_{c+2} is issued into buffer c % 2 right after P_c V_c: the MMAs of one
// thread run in issue order, so the PV reads P_c before the next QK^T overwrites it. The same ordering frees the K
// and V buffers: a loader reuses a K buffer once S_{c-2} is complete and a V buffer once P_{c-2} V_{c-2} is, and the
// MMA issuer posts two commits per chunk (S_c complete, P_c V_c complete).
// V is read as an N-major operand, so one shared-memory layout serves K (for QK^T) and V (for PV). The key range of a
// tile is cut to what its queries can see, so a sliding layer's long prefix costs O(window) per tile.
#include <algorithm>
#include <array>
#include <vector>

#include "common.cuh"

namespace morj {
namespace attn {

constexpr int ROWS = 128;
constexpr int BN = 64;
constexpr int THREADS = 256;
constexpr int TMEM_COLS = 256;  // S/P buffers at columns [0, 64) and [64, 128), O at [128, 128 + D)
constexpr float LOG2E = 1.4426950408889634f;
constexpr float RESCALE_LOG2 = 8.0f;  // rescale O only when a row maximum grows by more than 2^8

template <int D>
struct Smem {
  static constexpr int Q_BYTES = ROWS * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + Q_BYTES;       // 2 buffers
  static constexpr int V_OFF = K_OFF + 2 * KV_BYTES;  // 2 buffers
  static constexpr int BAR_OFF = V_OFF + 2 * KV_BYTES;
  // barriers (8 B each): q_full, k_full[2], v_full[2], (2 x 2 unused), s_full[2], p_full[2], pv_done[2], done; then
  // the TMEM slot and the abort flag. The dynamic shared window starts 1024-byte aligned (checked in the
  // kernel), so two CTAs fit an SM.
  static constexpr int TOTAL = BAR_OFF + 160;
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

// Packed pairs of FP32 values (one 64-bit register): fma / add on both lanes in one instruction, and a three-input
// maximum.
MORJ_DEV uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
MORJ_DEV uint64_t f2_bits(uint32_t lo, uint32_t hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}
MORJ_DEV void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
MORJ_DEV uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
MORJ_DEV uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
MORJ_DEV float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// warp-level wait: lane 0 polls the barrier, the warp follows its verdict
MORJ_DEV bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
  int ok = (threadIdx.x & 31) == 0 ? (int)mbar_wait(bar, parity, abort, kErrTimeoutAttention) : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// One loader warp fills buffer `dst` with the rows of keys [t0, t0 + BN) of one pool (K or V) for KV head h and
// completes `full`: one TMA tile load per 64-column half when the 64 slots are consecutive and all keys are inside
// the list, otherwise a cp.async row gather with zeros past t_end (so a masked key never brings a NaN into P V).
template <int D>
MORJ_DEV void load_chunk(uint32_t dst, uint32_t full, const CUtensorMap* map, const __nv_bfloat16* __restrict__ pool,
                         const int* __restrict__ kv_indices, const Segment& sg, int t0, int t_end, int hk, int h,
                         int page_size, int lane) {
  const int ta = t0 + 2 * lane, tb = ta + 1;
  const int sa = ta < t_end ? key_slot(kv_indices, sg.kv_base, ta, page_size) : -1;
  const int sb = tb < t_end ? key_slot(kv_indices, sg.kv_base, tb, page_size) : -1;
  const int s0 = __shfl_sync(0xffffffffu, sa, 0);
  const bool contiguous = __all_sync(0xffffffffu, sa == s0 + 2 * lane && sb == s0 + 2 * lane + 1);
  if (contiguous) {
    if (lane == 0) {
      mbar_arrive_expect_tx(full, BN * D * 2);
#pragma unroll
      for (int half = 0; half < D / 64; ++half) tma_load_3d(dst + half * (BN * 128), map, full, half * 64, h, s0);
    }
    return;
  }
  constexpr int CH = D / 8;  // 16-byte chunks per row
#pragma unroll
  for (int k2 = 0; k2 < 2; ++k2) {
    const int k = 2 * lane + k2;
    const int slot = k2 ? sb : sa;
    const bool ok = slot >= 0;
    const __nv_bfloat16* src = pool + (ok ? ((size_t)slot * hk + h) * D : 0);
#pragma unroll
    for (int c16 = 0; c16 < CH; ++c16) {
      const uint32_t off = (uint32_t)((c16 >> 3) * (BN * 128)) + sw128_offset(k, c16 & 7);
      cp_async16(dst + off, src + c16 * 8, ok ? 16u : 0u);
    }
  }
  cp_async_commit();
  cp_async_wait<0>();
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) mbar_arrive(full);
}

template <int D>
__global__ void __launch_bounds__(THREADS, 2)
    tree_attention_kernel(const __grid_constant__ CUtensorMap q_map, const __grid_constant__ CUtensorMap k_map,
                          const __grid_constant__ CUtensorMap v_map, const __nv_bfloat16* __restrict__ k_pool,
                          const __nv_bfloat16* __restrict__ v_pool, __nv_bfloat16* __restrict__ out,
                          const int* __restrict__ qo_indptr, const int* __restrict__ kv_indptr,
                          const int* __restrict__ kv_indices, const int* __restrict__ kv_last_page_len, int n_bidir,
                          int hq, int hk, int page_size, int window, float scale_log2, const int* __restrict__ work) {
  pdl_wait();  // the previous kernel on the stream has completed
  pdl_trigger();
  using L = Smem<D>;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  if (sbase & 1023) {  // the swizzled operand tiles need 1024-byte alignment
    if (threadIdx.x == 0) report(kErrBadAlignment);
    return;
  }
  const uint32_t bar0 = sbase + L::BAR_OFF;
  const uint32_t q_full = bar0, k_full = bar0 + 8, v_full = bar0 + 24;
  const uint32_t s_full = bar0 + 72, p_full = bar0 + 88, pv_done = bar0 + 104, done = bar0 + 120;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::BAR_OFF + 128);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::BAR_OFF + 132);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // CTAs run in grid order, so the KV head is the fast index: every head of the longest tile starts first
  const int item = blockIdx.x / hk, h = blockIdx.x % hk;
  const int seg = work[2 * item], q0 = work[2 * item + 1];
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

  // key range the tile can see; the start is rounded down to a chunk boundary so chunks line up with 64-slot pages
  int t_begin, t_end;
  if (bidir) {
    t_end = sg.kv_len;
    t_begin = window > 0 ? max(0, diag + min(0, q0 - (window - 1))) : 0;
  } else {
    t_end = diag + q_last + 1;
    t_begin = window > 0 ? max(0, diag + q0 - (window - 1)) : 0;
  }
  t_begin -= t_begin % BN;
  const int n_chunks = (t_end - t_begin + BN - 1) / BN;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(k_full + 8 * b, 1);
      mbar_init(v_full + 8 * b, 1);
      mbar_init(s_full + 8 * b, 1);
      mbar_init(p_full + 8 * b, 4);  // one arrival per softmax warp
      mbar_init(pv_done + 8 * b, 1);
    }
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

  if (warp == 0 || warp == 2) {
    // ---------------- K loader (warp 0) / V loader (warp 2) ----------------
    const bool is_k = warp == 0;
    if (is_k && lane == 0) {
      tma_prefetch(&q_map);
      tma_prefetch(&k_map);
      // Q tile: rows (query, head) of queries [q0, q0 + QT) and heads [h * G, h * G + G); rows past the tensor read 0
      mbar_arrive_expect_tx(q_full, ROWS * D * 2);
#pragma unroll
      for (int half = 0; half < D / 64; ++half)
        tma_load_3d(sbase + L::Q_OFF + half * (ROWS * 128), &q_map, q_full, half * 64, h * G, sg.q_start + q0);
    }
    if (!is_k && lane == 0) tma_prefetch(&v_map);
    const uint32_t base = sbase + (is_k ? L::K_OFF : L::V_OFF);
    // a K buffer is free once the scores of the chunk two back are complete, a V buffer once its PV is
    const uint32_t full = is_k ? k_full : v_full, empty = is_k ? s_full : pv_done;
    for (int c = 0; c < n_chunks; ++c) {
      const int b = c & 1;
      if (c >= 2 && !warp_wait(empty + 8 * b, ((c >> 1) - 1) & 1, abort)) break;
      load_chunk<D>(base + b * L::KV_BYTES, full + 8 * b, is_k ? &k_map : &v_map, is_k ? k_pool : v_pool,
                    kv_indices, sg, t_begin + c * BN, t_end, hk, h, page_size, lane);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t IDESC_S = idesc_bf16(ROWS, BN);
      constexpr uint32_t IDESC_O = idesc_bf16(ROWS, D, /*b_mn_major=*/true);
      bool ok = mbar_wait(q_full, 0, abort, kErrTimeoutAttention);
      // operand descriptors: one per buffer, advanced per 16-deep K step by the byte offset (>> 4)
      const uint64_t q_desc = sw128_desc(sbase + L::Q_OFF);
      const uint64_t k_desc0 = sw128_desc(sbase + L::K_OFF), v_desc0 = sw128_desc(sbase + L::V_OFF, BN * 128);
      constexpr uint64_t KV_STEP = L::KV_BYTES >> 4;
      auto issue_qk = [&](int c) -> bool {
        const int b = c & 1;
        if (!mbar_wait(k_full + 8 * b, (c >> 1) & 1, abort, kErrTimeoutAttention)) return false;
        tc_fence_after();
        const uint64_t k_desc = k_desc0 + b * KV_STEP;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t qa = ((kk >> 2) * (ROWS * 128) + (kk & 3) * 32) >> 4;
          const uint32_t kb = ((kk >> 2) * (BN * 128) + (kk & 3) * 32) >> 4;
          umma_bf16(tmem + b * BN, q_desc + qa, k_desc + kb, IDESC_S, kk > 0);
        }
        umma_commit(s_full + 8 * b);
        return true;
      };
      if (ok) ok = issue_qk(0);
      if (ok && n_chunks > 1) ok = issue_qk(1);
      for (int c = 0; c < n_chunks && ok; ++c) {
        const int b = c & 1;
        // O += P_c V_c, P_c from TMEM buffer b (packed BF16 pairs, 8 columns per 16 keys)
        if (!mbar_wait(p_full + 8 * b, (c >> 1) & 1, abort, kErrTimeoutAttention) ||
            !mbar_wait(v_full + 8 * b, (c >> 1) & 1, abort, kErrTimeoutAttention)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t v_desc = v_desc0 + b * KV_STEP;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          umma_bf16_tmem_a(tmem + 128, tmem + b * BN + kk * 8, v_desc + kk * (2048 >> 4), IDESC_O, (c | kk) != 0);
        umma_commit(pv_done + 8 * b);
        if (c + 2 < n_chunks) ok = issue_qk(c + 2);  // in issue order after this PV, which reads P_c first
      }
      // TMEM is freed only after every MMA issued here has completed
      umma_commit(done);
      mbar_wait_landed(done, 0);
    }
  } else if (warp >= 4) {
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
      const int t0 = t_begin + c * BN;
      // Scores are kept raw; the softmax works in the log2 domain with the scale folded into one FMA per element.
      // Chunks every key of which this row sees (the bulk of a long prefix) skip the per-key mask.
      // (the row maximum and sum run over 8 independent partials: short dependency chains)
      const bool full = t0 >= lo && t0 + BN - 1 <= hi;
      float m8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) m8[i] = -INFINITY;
      if (__all_sync(0xffffffffu, full)) {
#pragma unroll
        for (int j = 0; j < BN; j += 2)
          m8[(j >> 1) & 7] = max3f(m8[(j >> 1) & 7], __uint_as_float(sr[j >> 5][j & 31]),
                                   __uint_as_float(sr[(j + 1) >> 5][(j + 1) & 31]));
      } else {
#pragma unroll
        for (int j = 0; j < BN; ++j) {
          const int t = t0 + j;
          const float v = (t >= lo && t <= hi) ? __uint_as_float(sr[j >> 5][j & 31]) : -INFINITY;
          sr[j >> 5][j & 31] = __float_as_uint(v);
          m8[j & 7] = fmaxf(m8[j & 7], v);
        }
      }
      float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                       fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
      mx *= scale_log2;  // scale > 0: the maximum of the scaled scores
      float alpha = 1.f;
      if (mx > m_used + RESCALE_LOG2 || m_used == -INFINITY) {
        if (m_used != -INFINITY) alpha = fast_exp2(m_used - mx);
        if (mx != -INFINITY) m_used = mx;
      }
      l_run *= alpha;
      // exp2(-inf) = 0 for masked keys; a row with no visible key yet keeps m_used = -inf and p = 0
      const float neg_m = m_used == -INFINITY ? 0.f : -m_used;
      // scores in pairs: one packed FMA scales and shifts two of them, one packed add sums two probabilities
      const uint64_t scale2 = f2_pack(scale_log2, scale_log2), neg_m2 = f2_pack(neg_m, neg_m);
      uint64_t s4[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) s4[i] = f2_pack(0.f, 0.f);
      uint32_t pk[BN / 2];
#pragma unroll
      for (int j = 0; j < BN; j += 2) {
        float x0, x1;
        f2_unpack(f2_fma(f2_bits(sr[j >> 5][j & 31], sr[(j + 1) >> 5][(j + 1) & 31]), scale2, neg_m2), x0, x1);
        const float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
        s4[(j >> 1) & 3] = f2_add(s4[(j >> 1) & 3], f2_pack(p0, p1));
        pk[j / 2] = pack_bf16x2(p0, p1);
      }
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float lo, hi;
        f2_unpack(s4[i], lo, hi);
        sum += lo + hi;
      }
      l_run += sum;
      // a rescale of O waits until the previous chunk's PV has completed (the next one needs this chunk's P)
      if (c >= 1 && __any_sync(0xffffffffu, alpha != 1.f)) {
        if (!warp_wait(pv_done + 8 * (b ^ 1), ((c - 1) >> 1) & 1, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int col = 0; col < D; col += 32) {
          uint32_t o[32];
          tmem_ld32(t_lane + 128 + col, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(t_lane + 128 + col, o);
        }
      }
      tmem_st32(t_lane + b * BN, pk);  // P_c over the first 32 columns of S_c
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full + 8 * b);
    }
    if (ok && warp_wait(pv_done + 8 * ((n_chunks - 1) & 1), ((n_chunks - 1) >> 1) & 1, abort)) {
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
  // (warp 3 has no role)

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

template <int D>
static int launch(const void* q, int n_q, const void* k_pool, const void* v_pool, int pool_slots, void* out,
                  const int* qo_indptr, const int* kv_indptr, const int* kv_indices, const int* kv_last_page_len,
                  int n_bidir, int hq, int hk, int page_size, int window, float sm_scale, const int* work, int n_work,
                  cudaStream_t stream) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(tree_attention_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Smem<D>::TOTAL);
    if (e != cudaSuccess) return set_error(MORJ_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    configured = true;
  }
  const int G = hq / hk;
  CUtensorMap qm, km, vm;
  {  // q [n_q, hq, D]: box = 64 columns x G heads x 128/G queries
    const unsigned long long dims[3] = {(unsigned long long)D, (unsigned long long)hq, (unsigned long long)n_q};
    const unsigned long long strides[2] = {(unsigned long long)D * 2, (unsigned long long)hq * D * 2};
    const unsigned box[3] = {64u, (unsigned)G, (unsigned)(ROWS / G)};
    int st = encode_tiled(&qm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
  }
  {  // pools [slots, hk, D]: box = 64 columns x 1 head x 64 slots
    const unsigned long long dims[3] = {(unsigned long long)D, (unsigned long long)hk, (unsigned long long)pool_slots};
    const unsigned long long strides[2] = {(unsigned long long)D * 2, (unsigned long long)hk * D * 2};
    const unsigned box[3] = {64u, 1u, (unsigned)BN};
    int st = encode_tiled(&km, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, k_pool, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    st = encode_tiled(&vm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, v_pool, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
  }
  dim3 grid(n_work * hk);  // (tile, KV head) pairs, longest tile first
  return launch_pdl("tree_attention_kernel", tree_attention_kernel<D>, grid, dim3(THREADS), Smem<D>::TOTAL, stream,
                    qm, km, vm, reinterpret_cast<const __nv_bfloat16*>(k_pool),
                    reinterpret_cast<const __nv_bfloat16*>(v_pool), reinterpret_cast<__nv_bfloat16*>(out), qo_indptr,
                    kv_indptr, kv_indices, kv_last_page_len, n_bidir, hq, hk, page_size, window, sm_scale * LOG2E,
                    work);
}

}  // namespace attn
}  // namespace morj

extern "C" int morj_tree_attention_work(const int* qo_indptr_host, const int* kv_indptr_host,
                                        const int* kv_last_page_len_host, int n_segments, int n_bidir, int hq, int hk,
                                        int page_size, int window, int* work_host, int cap) {
  using namespace morj;
  if (!qo_indptr_host || !kv_indptr_host || n_segments < 0 || hk <= 0 || hq <= 0 || hq % hk || page_size <= 0) {
    set_error(MORJ_ERR_ARG, "morj_tree_attention_work: bad arguments");
    return -1;
  }
  const int G = hq / hk;
  if (attn::ROWS % G) {
    set_error(MORJ_ERR_ARG, "morj_tree_attention_work: group %d does not divide 128", G);
    return -1;
  }
  const int QT = attn::ROWS / G;
  // every tile with the number of key chunks it will walk (the same range the kernel computes)
  std::vector<std::array<int, 3>> tiles;  // (chunks, segment, first query)
  for (int s = 0; s < n_segments; ++s) {
    const int q_len = qo_indptr_host[s + 1] - qo_indptr_host[s];
    const int pages = kv_indptr_host[s + 1] - kv_indptr_host[s];
    const int kv_len = page_size == 1 ? pages
                                      : (pages - 1) * page_size +
                                            (kv_last_page_len_host ? kv_last_page_len_host[s] : page_size);
    const int diag = kv_len - q_len;
    for (int q0 = 0; q0 < q_len; q0 += QT) {
      const int q_last = std::min(q0 + QT, q_len) - 1;
      int t_begin, t_end;
      if (s < n_bidir) {
        t_end = kv_len;
        t_begin = window > 0 ? std::max(0, diag + std::min(0, q0 - (window - 1))) : 0;
      } else {
        t_end = diag + q_last + 1;
        t_begin = window > 0 ? std::max(0, diag + q0 - (window - 1)) : 0;
      }
      t_begin -= t_begin % attn::BN;
      tiles.push_back({(t_end - t_begin + attn::BN - 1) / attn::BN, s, q0});
    }
  }
  const int n = (int)tiles.size();
  if (n > cap) {
    set_error(MORJ_ERR_ARG, "morj_tree_attention_work: %d tiles exceed capacity %d", n, cap);
    return -1;
  }
  // longest first: the grid's last wave then holds the short tiles
  std::stable_sort(tiles.begin(), tiles.end(), [](const std::array<int, 3>& a, const std::array<int, 3>& b) {
    return a[0] > b[0];
  });
  if (work_host) {
    for (int i = 0; i < n; ++i) {
      work_host[2 * i] = tiles[i][1];
      work_host[2 * i + 1] = tiles[i][2];
    }
  }
  return n;
}

extern "C" int morj_tree_attention(const void* q, int n_q, const void* k_pool, const void* v_pool, int pool_slots,
                                   void* out, const int* qo_indptr, const int* kv_indptr, const int* kv_indices,
                                   const int* kv_last_page_len, int n_segments, int n_bidir, int hq, int hk, int d,
                                   int page_size, int window, float sm_scale, const int* work, int n_work,
                                   void* stream) {
  using namespace morj;
  if (n_work == 0 || n_segments == 0) return MORJ_OK;
  if (!q || !k_pool || !v_pool || !out || !qo_indptr || !kv_indptr || !kv_indices || !work || n_work < 0 ||
      n_q <= 0 || pool_slots <= 0)
    return set_error(MORJ_ERR_ARG, "morj_tree_attention: null pointer or bad size");
  if (hq <= 0 || hk <= 0 || hq % hk || attn::ROWS % (hq / hk))
    return set_error(MORJ_ERR_ARG, "morj_tree_attention: hq=%d hk=%d unsupported", hq, hk);
  if (page_size <= 0 || n_bidir < 0 || n_bidir > n_segments)
    return set_error(MORJ_ERR_ARG, "morj_tree_attention: bad page_size %d or n_bidir %d", page_size, n_bidir);
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_pool) | reinterpret_cast<uintptr_t>(v_pool)) &
      15)
    return set_error(MORJ_ERR_ARG, "morj_tree_attention: q and pools must be 16-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (d == 128)
    return attn::launch<128>(q, n_q, k_pool, v_pool, pool_slots, out, qo_indptr, kv_indptr, kv_indices,
                             kv_last_page_len, n_bidir, hq, hk, page_size, window, sm_scale, work, n_work, s);
  if (d == 64)
    return attn::launch<64>(q, n_q, k_pool, v_pool, pool_slots, out, qo_indptr, kv_indptr, kv_indices,
                            kv_last_page_len, n_bidir, hq, hk, page_size, window, sm_scale, work, n_work, s);
  return set_error(MORJ_ERR_UNSUPPORTED, "morj_tree_attention: head_dim %d unsupported (64, 128)", d);
}
