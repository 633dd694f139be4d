// BF16 projection GEMM for sm_100a: C = A . B^T with FP32 accumulation in TMEM.
//
// Persistent, warp-specialised kernel, one CTA per SM:
//   warp 0      TMA producer: A [128 x 64] and B [BN x 64] tiles (128-byte swizzle) into a 4-6 stage ring
//   warp 1      MMA issuer: one thread issues tcgen05.mma (M=128, N=BN, K=16) into a TMEM accumulator, commits each
//               stage back to the producer and each finished tile to the epilogue
//   warps 2-5   epilogue: tcgen05.ld of the accumulator (thread = row), BF16 rounding and the fused epilogue
// Two accumulators (all 512 TMEM columns) let the epilogue of tile i overlap the main loop of i+1. The tile width
// BN (128..256) is chosen per shape so the tile count fills whole waves of the 148 SMs; with a caller-registered
// workspace the SM-pair kernel instead shares the k-blocks of its last waves evenly between the pairs (split tiles).
// Tiles are walked in groups of 16 row-blocks so the activation slice and the weight tiles of the CTAs in flight
// stay in L2. No TMA multicast is used, so the kernel is valid whichever GPU's memory the pointers refer to.
#include <mutex>

#include "common.cuh"

namespace morj {
namespace gemm {

constexpr int BM = 128, BK = 64;
constexpr int A_BYTES = BM * BK * 2;
constexpr int TMEM_COLS = 512;  // two accumulators, at columns 0 and 256
constexpr int THREADS = 192;
constexpr int GROUP_M = 16;

// Tile width BN (a multiple of 16, at most 256): the host picks it per shape so the tile count fills whole waves of
// the SMs; the stage ring is as deep as shared memory allows.
template <int BN>
struct Cfg {
  static_assert(BN % 16 == 0 && BN >= 64 && BN <= 256, "tile width");
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (220 * 1024) / STAGE_BYTES > 6 ? 6 : (220 * 1024) / STAGE_BYTES;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  static constexpr uint32_t IDESC = idesc_bf16(BM, BN);
};

struct TileCoord {
  int m, n;
};

// Operands of the fused QKV epilogue: per-head RMSNorm (q, k weighted; v unweighted) of the BF16-rounded projection,
// BF16 rounding, rotate-half RoPE on q and k, and the scatter of q to its packed rows and of k / v to pool slots.
struct QkvEpi {
  int hq, hk, has_v;
  const __nv_bfloat16* q_norm;
  const __nv_bfloat16* k_norm;
  const int* positions;
  const float4* rope;  // RoPE table by position: D / 2 (cos, sin) pairs per position
  int rope_rows;
  const int* slots;
  float eps;
  __nv_bfloat16* q_out;
  __nv_bfloat16* k_pool;
  __nv_bfloat16* v_pool;
};

// Operands of the partial epilogue (tensor parallelism over peer memory): the output rows go to this rank's part
// buffer and the columns written for row block b are counted on the counter b of its owner, rank b % world. (Storing
// the rows straight into the owner's memory instead, so that NVLink would carry them while later tiles compute,
// measured slower: at 4 ranks the row-parallel GEMMs took 68 instead of 30 ms per latency tree, the epilogue warps'
// remote stores and system fences holding the accumulators, for a 13 ms saving in the reduction.)
constexpr int EPI_PEER = 4;
struct PeerEpi {
  __nv_bfloat16* part;
  unsigned long long* partials[MORJ_MAX_RANKS];
  int world;
};

// Split tiles of the pair kernel. When the tiles do not fill whole waves of SM pairs, the tiles of the last one to
// two waves are cut along K so that every pair gets the same number of k-blocks. Tiles [0, dp_tiles) go whole to
// pair t % pairs. The k-blocks of tiles [dp_tiles, tiles), `units` of them in tile-major order, are cut into `pairs`
// contiguous ranges of equal length (to one k-block), range p going to pair p. The host splits between `pairs` and
// 2 * pairs - 1 tiles this way, so a range is at least one tile long and a tile is cut at most once: its k-head
// [0, b) ends range p and its k-tail [b, kb) starts range p + 1. A pair walks its range from the end: the head
// piece first (kHead: its FP32 partial goes to the pair's workspace slot), then its whole tiles, the tail piece last
// (kTail: adds the slot of pair p - 1, written at that pair's start, then runs the epilogue). A pair thus only waits
// on a lower pair, for a partial written early in that pair's share of the split tiles.
struct Split {
  float4* ws;       // partial tiles: [pair][rank][epilogue warp][kSlotChunks float4 columns][32 rows]
  unsigned* flags;  // [pair][rank][epilogue warp]: 1 while the slot holds a partial not yet added
  int dp_tiles;
  long long units;
};
constexpr int kSlotChunks = 256 / 4;                                  // float4 columns of a 256-wide partial row
constexpr size_t kSlotBytesPerPair = 2ull * 4 * kSlotChunks * 32 * 16;  // both CTAs, 4 warps of 32 rows each
constexpr size_t kFlagBytesPerPair = 2 * 4 * sizeof(unsigned);

enum : int { kWhole = 0, kHead = 1, kTail = 2 };
struct Item {
  int tile, k0, k1, kind;  // k-blocks [k0, k1) of `tile`
};
struct Walk {
  int pairs, kb, dp_tiles, t;
  long long lo, hi;  // what is left of this pair's range of split k-blocks, taken from the end
  __host__ __device__ Walk(int pair, int pairs_, int kb_, int dp, long long units)
      : pairs(pairs_), kb(kb_), dp_tiles(dp), t(pair), lo(units * pair / pairs_), hi(units * (pair + 1) / pairs_) {}
  __host__ __device__ bool next(Item& it) {
    if (t < dp_tiles) {
      it = Item{t, 0, kb, kWhole};
      t += pairs;
      return true;
    }
    if (hi <= lo) return false;
    const long long first = (hi - 1) / kb * kb;  // first k-block of the tile that holds k-block hi - 1
    const long long s = first > lo ? first : lo;
    it.tile = dp_tiles + (int)((hi - 1) / kb);
    it.k0 = (int)(s - first);
    it.k1 = (int)(hi - first);
    it.kind = it.k0 > 0 ? kTail : (it.k1 < kb ? kHead : kWhole);
    hi = s;
    return true;
  }
};

// The split of `tiles` tiles of `kb` k-blocks over `pairs` SM pairs (no split: dp_tiles = tiles, units = 0).
__host__ __device__ inline void split_schedule(int tiles, int pairs, int kb, int* dp_tiles, long long* units) {
  *dp_tiles = tiles;
  *units = 0;
  if (pairs < 2 || tiles <= pairs || tiles % pairs == 0) return;
  *dp_tiles = (tiles / pairs - 1) * pairs;
  *units = (long long)(tiles - *dp_tiles) * kb;
}

MORJ_DEV unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
MORJ_DEV void st_release_gpu(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
MORJ_DEV void st_relaxed_gpu(unsigned* p, unsigned v) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// kHead: this warp's 32 accumulator rows (FP32) to its slot, column-chunk-major so each store is one 512-byte line
// per warp; then the flag, released after every lane's stores.
template <int BN>
MORJ_DEV void save_partial(uint32_t tacc, float4* slot, unsigned* flag, int lane) {
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    uint32_t r[32];
    tmem_ld32(tacc + c, r);
    tmem_wait_ld();
#pragma unroll
    for (int v = 0; v < 8; ++v)
      __stcg(slot + (c / 4 + v) * 32 + lane, make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                                         __uint_as_float(r[4 * v + 2]),
                                                         __uint_as_float(r[4 * v + 3])));
  }
  __threadfence();
  __syncwarp();
  if (lane == 0) st_release_gpu(flag, 1u);
}

// kTail: wait (bounded) for the head's partial, add it into this warp's accumulator rows in TMEM and clear the flag
// for the next launch. Returns false when the wait gave up (device error recorded, CTA abort raised).
template <int BN>
MORJ_DEV bool add_partial(uint32_t tacc, const float4* slot, unsigned* flag, int lane, volatile int* abort) {
  int ok = 1;
  if (lane == 0) {
    const unsigned long long t0 = global_ns();
    for (uint32_t i = 0; ld_acquire_gpu(flag) == 0; ++i) {
      if ((i & 63) == 63) {
        if (*abort) {
          ok = 0;
          break;
        }
        if (global_ns() - t0 > kWaitLimitNs) {
          *abort = 1;
          report(kErrTimeoutGemmSplit);
          ok = 0;
          break;
        }
      }
      __nanosleep(128);
    }
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (!ok) return false;
  (void)ld_acquire_gpu(flag);  // (every lane acquires the head's stores)
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    uint32_t r[32];
    tmem_ld32(tacc + c, r);
    tmem_wait_ld();
#pragma unroll
    for (int v = 0; v < 8; ++v) {
      const float4 p = __ldcg(slot + (c / 4 + v) * 32 + lane);
      r[4 * v] = __float_as_uint(__uint_as_float(r[4 * v]) + p.x);
      r[4 * v + 1] = __float_as_uint(__uint_as_float(r[4 * v + 1]) + p.y);
      r[4 * v + 2] = __float_as_uint(__uint_as_float(r[4 * v + 2]) + p.z);
      r[4 * v + 3] = __float_as_uint(__uint_as_float(r[4 * v + 3]) + p.w);
    }
    tmem_st32(tacc + c, r);
  }
  tmem_wait_st();
  __syncwarp();
  if (lane == 0) st_relaxed_gpu(flag, 0u);
  return true;
}

// (after a system fence by every lane and a warp barrier, which order the warp's stores before it)
MORJ_DEV void red_relaxed_sys_add(unsigned long long* p, unsigned long long v) {
  asm volatile("red.relaxed.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

MORJ_DEV void store32_bf16(__nv_bfloat16* dst, const float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 pk;
    pk.x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
    pk.y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
    pk.z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
    pk.w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
    reinterpret_cast<uint4*>(dst)[q] = pk;
  }
}

// One 128-row tile of the QKV projection, D-wide heads: thread = token row (reference `_qkv_post` numerics).
template <int BN, int D>
MORJ_DEV void epilogue_qkv(uint32_t tacc, int row, int n_blk, bool row_ok, const QkvEpi& e, int N) {
  // the norm weights and the (cos, sin) pairs are read 8 weights / 2 pairs per load
  constexpr int HALF = D / 2;
  const int n_heads = N / D;
  int pos = row_ok ? e.positions[row] : 0;
  if ((unsigned)pos >= (unsigned)e.rope_rows) {
    if (row_ok) report(kErrBadIndex);
    row_ok = false;
    pos = 0;
  }
  const float4* rope = e.rope + (size_t)pos * (HALF / 2);
  const size_t slot = (row_ok && e.hk) ? (size_t)e.slots[row] : 0;
#pragma unroll 1
  for (int hh = 0; hh < BN / D; ++hh) {
    const int head = (n_blk * BN) / D + hh;
    if (head >= n_heads) break;
    const uint32_t tb = tacc + hh * D;
    const bool is_q = head < e.hq;
    const bool is_k = !is_q && head < e.hq + e.hk;
    float ss = 0.f;
#pragma unroll 1
    for (int c = 0; c < D; c += 32) {
      uint32_t r[32];
      tmem_ld32(tb + c, r);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float v = bf16_round(__uint_as_float(r[i]));
        ss += v * v;
      }
    }
    const float inv = 1.0f / sqrtf(ss / D + e.eps);
    const __nv_bfloat16* w = is_q ? e.q_norm : e.k_norm;
    __nv_bfloat16* dst;
    __nv_bfloat16* dst_v = nullptr;  // full-attention layers: V is the unweighted norm of the K projection
    if (is_q) {
      dst = e.q_out + ((size_t)row * e.hq + head) * D;
    } else if (is_k) {
      dst = e.k_pool + (slot * e.hk + (head - e.hq)) * D;
      if (!e.has_v) dst_v = e.v_pool + (slot * e.hk + (head - e.hq)) * D;
    } else {
      dst = e.v_pool + (slot * e.hk + (head - e.hq - e.hk)) * D;
    }
#pragma unroll 1
    for (int c = 0; c < HALF; c += 32) {
      uint32_t r1[32], r2[32];
      tmem_ld32(tb + c, r1);
      tmem_ld32(tb + HALF + c, r2);
      tmem_wait_ld();
      float o1[32], o2[32];
      if (is_q || is_k) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          float w1[8], w2[8];
          unpack8_bf16(*reinterpret_cast<const uint4*>(w + c + j), w1);
          unpack8_bf16(*reinterpret_cast<const uint4*>(w + HALF + c + j), w2);
#pragma unroll
          for (int u = 0; u < 8; u += 2) {
            const float4 cs = rope[(c + j + u) / 2];  // (cos, sin) of pairs c+j+u and c+j+u+1
#pragma unroll
            for (int v = 0; v < 2; ++v) {
              const int i = j + u + v;
              const float co = v ? cs.z : cs.x, sn = v ? cs.w : cs.y;
              const float a = bf16_round(__uint_as_float(r1[i])) * inv;
              const float b = bf16_round(__uint_as_float(r2[i])) * inv;
              const float y1 = bf16_round(a * w1[u + v]);  // rounded before RoPE, as the reference
              const float y2 = bf16_round(b * w2[u + v]);
              o1[i] = y1 * co - y2 * sn;
              o2[i] = y2 * co + y1 * sn;
            }
          }
        }
        if (row_ok) {
          store32_bf16(dst + c, o1);
          store32_bf16(dst + HALF + c, o2);
        }
        if (dst_v != nullptr) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            o1[i] = bf16_round(__uint_as_float(r1[i])) * inv;
            o2[i] = bf16_round(__uint_as_float(r2[i])) * inv;
          }
          if (row_ok) {
            store32_bf16(dst_v + c, o1);
            store32_bf16(dst_v + HALF + c, o2);
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          o1[i] = bf16_round(__uint_as_float(r1[i])) * inv;
          o2[i] = bf16_round(__uint_as_float(r2[i])) * inv;
        }
        if (row_ok) {
          store32_bf16(dst + c, o1);
          store32_bf16(dst + HALF + c, o2);
        }
      }
    }
  }
}

MORJ_DEV TileCoord tile_coord(int t, int num_m, int num_n) {
  const int per_group = GROUP_M * num_n;
  const int group = t / per_group;
  const int first_m = group * GROUP_M;
  const int gm = min(GROUP_M, num_m - first_m);
  const int local = t - group * per_group;
  return {first_m + local % gm, local / gm};
}

// BF16 store of one accumulator row (this thread's) of tile column block n_blk into crow[n_blk * BN ...].
template <int BN>
MORJ_DEV void store_row(uint32_t tacc, __nv_bfloat16* crow, int n_blk, bool row_ok, int N) {
  const int lim = min(N, (n_blk + 1) * BN);  // this tile's columns (the last 32-column load may run past BN)
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    uint32_t r[32];
    tmem_ld32(tacc + c, r);
    tmem_wait_ld();
    const int col = n_blk * BN + c;
    if (row_ok && col < lim) {
      uint4* dst = reinterpret_cast<uint4*>(crow + col);
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        if (col + v * 8 < lim) {
          uint4 pk;
          pk.x = pack_bf16x2(__uint_as_float(r[v * 8 + 0]), __uint_as_float(r[v * 8 + 1]));
          pk.y = pack_bf16x2(__uint_as_float(r[v * 8 + 2]), __uint_as_float(r[v * 8 + 3]));
          pk.z = pack_bf16x2(__uint_as_float(r[v * 8 + 4]), __uint_as_float(r[v * 8 + 5]));
          pk.w = pack_bf16x2(__uint_as_float(r[v * 8 + 6]), __uint_as_float(r[v * 8 + 7]));
          dst[v] = pk;
        }
      }
    }
  }
}

// Partial epilogue: this thread's row of the tile goes to this rank's part buffer (the STORE epilogue's stores);
// the tile's column count for the row block's owner is returned, to be posted by `peer_arrive`. Row blocks wholly
// past M (the pair kernel's padding) neither store nor count.
template <int BN>
MORJ_DEV void epilogue_peer(uint32_t tacc, int row, int n_blk, int M, int N, const PeerEpi& pe,
                            unsigned long long*& count, unsigned long long& cols) {
  const int blk = row / 128;
  if (blk * 128 >= M) return;
  store_row<BN>(tacc, pe.part + (size_t)row * N, n_blk, row < M, N);
  count = pe.partials[blk % pe.world] + blk;
  cols = (unsigned long long)(min(N, (n_blk + 1) * BN) - n_blk * BN);
}

// The arrival of a written tile (deferred to the warp's next accumulator wait, where the system fence's round trip
// is hidden under the main loop): every lane's stores are ordered system-wide before lane 0's add.
MORJ_DEV void peer_arrive(unsigned long long*& count, unsigned long long cols, int lane) {
  if (count == nullptr) return;
  __threadfence_system();
  __syncwarp();
  if (lane == 0) red_relaxed_sys_add(count, cols);
  count = nullptr;
}

// ---- epilogue stores through a per-warp shared-memory transpose (SM-pair kernel) ----
// The accumulator gives each epilogue lane one row, so a direct 16-byte store per lane makes every store instruction
// touch 32 rows: 32 L1 wavefronts and 32 partial-sector L2 writes, and on the last tile of a pair (the one whose
// epilogue nothing overlaps) those stores cost up to 5-7 us per launch (measured by leaving them out). Here a
// 64-column BF16 chunk (8 x 16 bytes per row) goes through the warp's 4 KB buffer: each lane writes its row
// (128 bytes, 16-byte units XOR-swizzled by row & 7, so eight consecutive rows cover all 32 banks), then each of 8
// read instructions takes 4 rows x 8 units and stores 4 whole 128-byte row segments. Measured: O projection 0.0695
// -> 0.0666 ms, QKV with the head epilogue 0.1424 -> 0.1392 ms, down 0.3369 -> 0.3347 ms.
constexpr int kStageBytesPerWarp = 32 * 128;

MORJ_DEV void stage_st16(uint32_t addr, const uint4& v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
MORJ_DEV uint4 stage_ld16(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
               : "memory");
  return v;
}

// Stores this warp's 32 rows x 64 BF16 columns (lane = row; v = the lane's 8 units of 8 columns). dst(r, u) gives
// the address of unit u of warp row r, or nullptr to skip it.
template <class Dst>
MORJ_DEV void staged_store64(uint32_t buf, const uint4 (&v)[8], int lane, const Dst& dst) {
  __syncwarp();  // the previous chunk's reads of the buffer are done
#pragma unroll
  for (int u = 0; u < 8; ++u) stage_st16(buf + lane * 128 + ((u ^ (lane & 7)) << 4), v[u]);
  __syncwarp();
  const int unit = lane & 7;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = i * 4 + (lane >> 3);
    const uint4 val = stage_ld16(buf + r * 128 + ((unit ^ (r & 7)) << 4));
    __nv_bfloat16* p = dst(r, unit);
    if (p != nullptr) *reinterpret_cast<uint4*>(p) = val;
  }
}

// BF16 store of this warp's 32 accumulator rows of tile column block n_blk (row_base = the warp's first row) into
// C[row][n_blk * BN ...], rows below M and columns below N only.
template <int BN>
MORJ_DEV void store_rows_staged(uint32_t tacc, uint32_t buf, __nv_bfloat16* C, long long ldc, int row_base, int M,
                                int n_blk, int N, int lane) {
  const int lim = min(N, (n_blk + 1) * BN);
#pragma unroll 1
  for (int c = 0; c < BN; c += 64) {
    uint32_t r0[32], r1[32];
    tmem_ld32(tacc + c, r0);
    tmem_ld32(tacc + c + 32, r1);  // (past BN only when BN % 64 != 0: accumulator columns left unstored)
    tmem_wait_ld();
    uint4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const uint32_t* r = u < 4 ? r0 : r1;
      const int o = (u & 3) * 8;
      v[u].x = pack_bf16x2(__uint_as_float(r[o + 0]), __uint_as_float(r[o + 1]));
      v[u].y = pack_bf16x2(__uint_as_float(r[o + 2]), __uint_as_float(r[o + 3]));
      v[u].z = pack_bf16x2(__uint_as_float(r[o + 4]), __uint_as_float(r[o + 5]));
      v[u].w = pack_bf16x2(__uint_as_float(r[o + 6]), __uint_as_float(r[o + 7]));
    }
    const int col0 = n_blk * BN + c;
    staged_store64(buf, v, lane, [&](int r, int u) -> __nv_bfloat16* {
      const int row = row_base + r, col = col0 + u * 8;
      return (row < M && col < lim) ? C + (size_t)row * ldc + col : nullptr;
    });
  }
}

// The head epilogue of the SM-pair kernel: the numerics of epilogue_qkv, with each head's D output columns of the
// warp's 32 rows assembled in the warp's store buffer (D / 64 chunks of 32 rows x 128 bytes, units swizzled as in
// staged_store64) and written 4 rows x 128 bytes per store instruction; each row's destination offset (its q row or
// K / V pool slot) is shuffled to the lanes that store it.
MORJ_DEV void stage_put32(uint32_t buf, int lane, int col, const float (&o)[32]) {
  const uint32_t chunk = buf + (uint32_t)(col >> 6) * kStageBytesPerWarp + lane * 128;
  const int unit0 = (col & 63) >> 3;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 v;
    v.x = pack_bf16x2(o[i * 8 + 0], o[i * 8 + 1]);
    v.y = pack_bf16x2(o[i * 8 + 2], o[i * 8 + 3]);
    v.z = pack_bf16x2(o[i * 8 + 4], o[i * 8 + 5]);
    v.w = pack_bf16x2(o[i * 8 + 6], o[i * 8 + 7]);
    stage_st16(chunk + (((unit0 + i) ^ (lane & 7)) << 4), v);
  }
}

// Writes the staged head (D columns of 32 rows) to base + off(row) for every row whose offset is >= 0.
template <int D>
MORJ_DEV void stage_flush_head(uint32_t buf, int lane, __nv_bfloat16* base, long long off) {
  __syncwarp();
  const int unit = lane & 7;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = i * 4 + (lane >> 3);
    const long long o = __shfl_sync(0xffffffffu, off, r);
#pragma unroll
    for (int k = 0; k < D / 64; ++k) {
      const uint4 val = stage_ld16(buf + k * kStageBytesPerWarp + r * 128 + ((unit ^ (r & 7)) << 4));
      if (o >= 0) *reinterpret_cast<uint4*>(base + o + k * 64 + unit * 8) = val;
    }
  }
}

template <int BN, int D>
MORJ_DEV void epilogue_qkv_staged(uint32_t tacc, uint32_t buf, int row, int n_blk, bool row_ok, const QkvEpi& e,
                                  int N, int lane) {
  static_assert(D % 64 == 0, "head width");
  constexpr int HALF = D / 2;
  const int n_heads = N / D;
  int pos = row_ok ? e.positions[row] : 0;
  if ((unsigned)pos >= (unsigned)e.rope_rows) {
    if (row_ok) report(kErrBadIndex);
    row_ok = false;
    pos = 0;
  }
  const float4* rope = e.rope + (size_t)pos * (HALF / 2);
  const long long slot = (row_ok && e.hk) ? (long long)e.slots[row] : 0;
#pragma unroll 1
  for (int hh = 0; hh < BN / D; ++hh) {
    const int head = (n_blk * BN) / D + hh;
    if (head >= n_heads) break;  // (warp-uniform)
    const uint32_t tb = tacc + hh * D;
    const bool is_q = head < e.hq;
    const bool is_k = !is_q && head < e.hq + e.hk;
    float ss = 0.f;
#pragma unroll 1
    for (int c = 0; c < D; c += 32) {
      uint32_t r[32];
      tmem_ld32(tb + c, r);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float v = bf16_round(__uint_as_float(r[i]));
        ss += v * v;
      }
    }
    const float inv = 1.0f / sqrtf(ss / D + e.eps);
    const __nv_bfloat16* w = is_q ? e.q_norm : e.k_norm;
    __nv_bfloat16* base;
    __nv_bfloat16* base_v = nullptr;  // full-attention layers: V is the unweighted norm of the K projection
    long long off;
    if (is_q) {
      base = e.q_out;
      off = ((long long)row * e.hq + head) * D;
    } else if (is_k) {
      base = e.k_pool;
      off = (slot * e.hk + (head - e.hq)) * D;
      if (!e.has_v) base_v = e.v_pool;
    } else {
      base = e.v_pool;
      off = (slot * e.hk + (head - e.hq - e.hk)) * D;
    }
    if (!row_ok) off = -1;
    __syncwarp();  // the previous head's flush has read the buffer
#pragma unroll 1
    for (int c = 0; c < HALF; c += 32) {
      uint32_t r1[32], r2[32];
      tmem_ld32(tb + c, r1);
      tmem_ld32(tb + HALF + c, r2);
      tmem_wait_ld();
      float o1[32], o2[32];
      if (is_q || is_k) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          float w1[8], w2[8];
          unpack8_bf16(*reinterpret_cast<const uint4*>(w + c + j), w1);
          unpack8_bf16(*reinterpret_cast<const uint4*>(w + HALF + c + j), w2);
#pragma unroll
          for (int u = 0; u < 8; u += 2) {
            const float4 cs = rope[(c + j + u) / 2];  // (cos, sin) of pairs c+j+u and c+j+u+1
#pragma unroll
            for (int v = 0; v < 2; ++v) {
              const int i = j + u + v;
              const float co = v ? cs.z : cs.x, sn = v ? cs.w : cs.y;
              const float a = bf16_round(__uint_as_float(r1[i])) * inv;
              const float b = bf16_round(__uint_as_float(r2[i])) * inv;
              const float y1 = bf16_round(a * w1[u + v]);  // rounded before RoPE, as the reference
              const float y2 = bf16_round(b * w2[u + v]);
              o1[i] = y1 * co - y2 * sn;
              o2[i] = y2 * co + y1 * sn;
            }
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          o1[i] = bf16_round(__uint_as_float(r1[i])) * inv;
          o2[i] = bf16_round(__uint_as_float(r2[i])) * inv;
        }
      }
      stage_put32(buf, lane, c, o1);
      stage_put32(buf, lane, HALF + c, o2);
    }
    stage_flush_head<D>(buf, lane, base, off);
    if (base_v != nullptr) {
      __syncwarp();
#pragma unroll 1
      for (int c = 0; c < HALF; c += 32) {
        uint32_t r1[32], r2[32];
        tmem_ld32(tb + c, r1);
        tmem_ld32(tb + HALF + c, r2);
        tmem_wait_ld();
        float o1[32], o2[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          o1[i] = bf16_round(__uint_as_float(r1[i])) * inv;
          o2[i] = bf16_round(__uint_as_float(r2[i])) * inv;
        }
        stage_put32(buf, lane, c, o1);
        stage_put32(buf, lane, HALF + c, o2);
      }
      stage_flush_head<D>(buf, lane, base_v, off);
    }
  }
}

template <int EPI, int BN>
MORJ_DEV void epilogue_tile(uint32_t tacc, int row, int n_blk, bool row_ok, __nv_bfloat16* C, long long ldc, int N) {
  if constexpr (EPI == MORJ_EPI_STORE) {
    store_row<BN>(tacc, C + (size_t)row * ldc, n_blk, row_ok, N);
  } else {
    // gate columns [0, 128), up columns [128, 256) of this tile -> 128 outputs
    const int F = N / 2;
    __nv_bfloat16* crow = C + (size_t)row * ldc;
#pragma unroll 1
    for (int c = 0; c < BN / 2; c += 32) {
      uint32_t g[32], u[32];
      tmem_ld32(tacc + c, g);
      tmem_ld32(tacc + BN / 2 + c, u);
      tmem_wait_ld();
      const int col = n_blk * (BN / 2) + c;
      if (row_ok && col < F) {
        uint4* dst = reinterpret_cast<uint4*>(crow + col);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          float o[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float gv = bf16_round(__uint_as_float(g[v * 8 + e]));
            const float uv = bf16_round(__uint_as_float(u[v * 8 + e]));
            o[e] = gelu_tanh(gv) * uv;
          }
          uint4 pk;
          pk.x = pack_bf16x2(o[0], o[1]);
          pk.y = pack_bf16x2(o[2], o[3]);
          pk.z = pack_bf16x2(o[4], o[5]);
          pk.w = pack_bf16x2(o[6], o[7]);
          dst[v] = pk;
        }
      }
    }
  }
}

template <int EPI, int BN>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                __nv_bfloat16* __restrict__ C, long long ldc, int M, int N, int K, const QkvEpi qe,
                const PeerEpi pe) {
  using C_ = Cfg<BN>;
  constexpr int STAGES = C_::STAGES, STAGE_BYTES = C_::STAGE_BYTES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  // bars: full[STAGES], empty[STAGES], acc_full[2], acc_empty[2], done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES);
  const uint32_t accf0 = smem_u32(bars + 2 * STAGES), acce0 = smem_u32(bars + 2 * STAGES + 2);
  const uint32_t done0 = smem_u32(bars + 2 * STAGES + 4);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf0 + 8 * b, 1);
      mbar_init(acce0 + 8 * b, 128);
    }
    mbar_init(done0, 1);
    *abort = 0;
    fence_mbar_init();
    tma_prefetch(&map_a);
    tma_prefetch(&map_b);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // (set-up above touches no global memory) the previous kernel on the stream has completed
  pdl_trigger();

  const int num_m = (M + BM - 1) / BM, num_n = (N + BN - 1) / BN;
  const int tiles = num_m * num_n;
  const int kblocks = (K + BK - 1) / BK;
  const uint32_t smem_base = smem_u32(smem);

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_a = policy_evict_last();
      const uint64_t pol_b = policy_evict_normal();
      int stage = 0, issued = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < tiles && !*abort; t += gridDim.x) {
        const TileCoord tc = tile_coord(t, num_m, num_n);
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, abort, kErrTimeoutGemmProducer)) {
            ok = false;
            break;
          }
          const uint32_t sa = smem_base + stage * STAGE_BYTES;
          mbar_arrive_expect_tx(full0 + 8 * stage, STAGE_BYTES);
          tma_load_2d(sa, &map_a, full0 + 8 * stage, kb * BK, tc.m * BM, pol_a);
          tma_load_2d(sa + A_BYTES, &map_b, full0 + 8 * stage, kb * BK, tc.n * BN, pol_b);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
      }
      // no copy may still be in flight when the CTA exits: wait for the last fills to land
      const int pending = issued < STAGES ? issued : STAGES;
      for (int j = 1; j <= pending; ++j) {
        const int s = (stage - j + STAGES) % STAGES;
        const uint32_t ph = (stage - j >= 0) ? phase : (phase ^ 1);
        mbar_wait_landed(full0 + 8 * s, ph);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
        if (!mbar_wait(acce0 + 8 * acc, acc_phase ^ 1, abort, kErrTimeoutGemmMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * 256;
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(full0 + 8 * stage, phase, abort, kErrTimeoutGemmMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_base + stage * STAGE_BYTES;
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            umma_bf16(d_tmem, sw128_desc(sa + 32 * k), sw128_desc(sb + 32 * k), C_::IDESC, (kb | k) != 0);
          }
          umma_commit(empty0 + 8 * stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(accf0 + 8 * acc);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      // TMEM is freed below only after every MMA issued here has completed
      umma_commit(done0);
      mbar_wait_landed(done0, 0);
    }
  } else {
    // epilogue warps 2..5: warp w reads TMEM lanes 32 * (w % 4) .. + 31
    const int quarter = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    unsigned long long* pend = nullptr;  // partial-delivery epilogue: the arrival still to post
    unsigned long long pend_cols = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      const TileCoord tc = tile_coord(t, num_m, num_n);
      // lane 0 waits for the accumulator; the warp follows its verdict (tcgen05.ld below is warp-collective)
      int ok = lane == 0 ? (int)mbar_wait(accf0 + 8 * acc, acc_phase, abort, kErrTimeoutGemmEpilogue) : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if constexpr (EPI == EPI_PEER) peer_arrive(pend, pend_cols, lane);
      if (!ok) break;
      tc_fence_after();
      const int row = tc.m * BM + quarter * 32 + lane;
      const uint32_t tacc = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * 256;
      if constexpr (EPI == MORJ_EPI_QKV_D128) {
        epilogue_qkv<BN, 128>(tacc, row, tc.n, row < M, qe, N);
      } else if constexpr (EPI == MORJ_EPI_QKV_D64) {
        epilogue_qkv<BN, 64>(tacc, row, tc.n, row < M, qe, N);
      } else if constexpr (EPI == EPI_PEER) {
        epilogue_peer<BN>(tacc, row, tc.n, M, N, pe, pend, pend_cols);
      } else {
        epilogue_tile<EPI, BN>(tacc, row, tc.n, row < M, C, ldc, N);
      }
      tc_fence_before();
      mbar_arrive(acce0 + 8 * acc);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if constexpr (EPI == EPI_PEER) peer_arrive(pend, pend_cols, lane);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Pair kernel: a cluster of two CTAs on two SMs computes a 256 x BN tile with tcgen05.mma.cta_group::2. CTA r loads
// A rows [128 r, 128 r + 128) of the tile and B rows [r BN / 2, (r + 1) BN / 2); the MMA issued by CTA 0 reads both
// CTAs' shared memory and leaves rows [128 r, 128 r + 128) of the accumulator in CTA r's TMEM. Each SM fills only
// half of the B tile per k-block, so the L2-to-shared-memory traffic per FLOP drops by a third against the one-CTA
// kernel. The epilogues are the one-CTA kernel's (each CTA drains its own 128 rows).
// ---------------------------------------------------------------------------------------------------------------
template <int BN>
struct Cfg2 {
  static_assert(BN % 32 == 0 || BN % 16 == 0, "tile width");
  static constexpr int B_HALF_BYTES = (BN / 2) * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_HALF_BYTES;
  static constexpr int STAGES = (200 * 1024) / STAGE_BYTES > 8 ? 8 : (200 * 1024) / STAGE_BYTES;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  static constexpr uint32_t IDESC = idesc_bf16(2 * BM, BN);
};

// Store buffers of the pair kernel's four epilogue warps (after the stage ring): one 64-column chunk per warp for the
// plain epilogue and the D = 64 head epilogue, a whole 128-column head for the D = 128 head epilogue, none for the
// GeGLU and partial epilogues (direct stores).
template <int EPI>
constexpr int pair_stage_out_bytes() {
  return EPI == MORJ_EPI_QKV_D128                                  ? 4 * 2 * kStageBytesPerWarp
         : (EPI == MORJ_EPI_STORE || EPI == MORJ_EPI_QKV_D64) ? 4 * kStageBytesPerWarp
                                                              : 0;
}
template <int EPI, int BN>
constexpr int pair_smem_bytes() {
  return Cfg2<BN>::SMEM_BYTES + pair_stage_out_bytes<EPI>();
}

template <int EPI, int BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    gemm2_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                 __nv_bfloat16* __restrict__ C, long long ldc, int M, int N, int K, const QkvEpi qe,
                 const PeerEpi pe, const Split sp) {
  using C_ = Cfg2<BN>;
  constexpr int STAGES = C_::STAGES, STAGE_BYTES = C_::STAGE_BYTES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  static_assert(pair_smem_bytes<EPI, BN>() <= 232448, "shared memory per CTA");
  constexpr int STAGE_OUT = pair_stage_out_bytes<EPI>() / 4;  // per epilogue warp
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES + 4 * STAGE_OUT);
  // bars: full[STAGES] (used in CTA 0), empty[STAGES], acc_full[2], acc_empty[2] (used in CTA 0), done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_rank();
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES);
  const uint32_t accf0 = smem_u32(bars + 2 * STAGES), acce0 = smem_u32(bars + 2 * STAGES + 2);
  const uint32_t done0 = smem_u32(bars + 2 * STAGES + 4);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf0 + 8 * b, 1);
      mbar_init(acce0 + 8 * b, 8);  // one arrival per epilogue warp of each CTA of the pair
    }
    mbar_init(done0, 1);
    *abort = 0;
    fence_mbar_init();
    tma_prefetch(&map_a);
    tma_prefetch(&map_b);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs are initialised before either CTA signals the other's
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // (set-up above touches no global memory) the previous kernel on the stream has completed
  pdl_trigger();

  const int num_m = (M + 2 * BM - 1) / (2 * BM), num_n = (N + BN - 1) / BN;
  const int kblocks = (K + BK - 1) / BK;
  const uint32_t smem_base = smem_u32(smem);
  const int cluster = blockIdx.x / 2, n_clusters = gridDim.x / 2;

  if (warp == 0) {
    if (lane == 0) {
      // this CTA's loads complete on CTA 0's full barriers; CTA 0 posts the byte count of both CTAs
      const uint32_t full0_leader = map_shared(full0, 0);
      const uint64_t pol_a = policy_evict_last();
      const uint64_t pol_b = policy_evict_normal();
      int stage = 0, issued = 0;
      uint32_t phase = 0;
      Walk walk(cluster, n_clusters, kblocks, sp.dp_tiles, sp.units);
      Item it;
      while (!*abort && walk.next(it)) {
        const TileCoord tc = tile_coord(it.tile, num_m, num_n);
        bool ok = true;
        for (int kb = it.k0; kb < it.k1; ++kb) {
          if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, abort, kErrTimeoutGemmProducer)) {
            ok = false;
            break;
          }
          const uint32_t sa = smem_base + stage * STAGE_BYTES;
          if (rank == 0) mbar_arrive_expect_tx(full0 + 8 * stage, 2 * STAGE_BYTES);
          tma_load_2d_pair(sa, &map_a, full0_leader + 8 * stage, kb * BK, tc.m * 2 * BM + rank * BM, pol_a);
          tma_load_2d_pair(sa + A_BYTES, &map_b, full0_leader + 8 * stage, kb * BK,
                           tc.n * BN + rank * (BN / 2), pol_b);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
      }
      // no copy of this CTA may still be in flight when it leaves: its last fills are consumed (empty) first
      const int pending = issued < STAGES ? issued : STAGES;
      for (int j = 0; j < pending; ++j) {
        if (!mbar_wait_landed(empty0 + 8 * stage, phase ^ 1)) break;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      Walk walk(cluster, n_clusters, kblocks, sp.dp_tiles, sp.units);
      Item it;
      while (walk.next(it)) {
        if (!mbar_wait(acce0 + 8 * acc, acc_phase ^ 1, abort, kErrTimeoutGemmMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * 256;
        bool ok = true;
        for (int kb = it.k0; kb < it.k1; ++kb) {
          if (!mbar_wait(full0 + 8 * stage, phase, abort, kErrTimeoutGemmMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_base + stage * STAGE_BYTES;
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            umma_bf16_pair(d_tmem, sw128_desc(sa + 32 * k), sw128_desc(sb + 32 * k), C_::IDESC,
                           ((kb - it.k0) | k) != 0);
          }
          umma_commit_pair(empty0 + 8 * stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair(accf0 + 8 * acc);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      umma_commit_pair(done0);
      mbar_wait_landed(done0, 0);
    }
  } else {
    // epilogue warps 2..5 of each CTA drain that CTA's 128 accumulator rows
    const int quarter = warp & 3;
    const uint32_t acce_leader = map_shared(acce0, 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    unsigned long long* pend = nullptr;  // partial-delivery epilogue: the arrival still to post
    unsigned long long pend_cols = 0;
    Walk walk(cluster, n_clusters, kblocks, sp.dp_tiles, sp.units);
    Item it;
    while (walk.next(it)) {
      const TileCoord tc = tile_coord(it.tile, num_m, num_n);
      int ok = lane == 0 ? (int)mbar_wait(accf0 + 8 * acc, acc_phase, abort, kErrTimeoutGemmEpilogue) : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if constexpr (EPI == EPI_PEER) peer_arrive(pend, pend_cols, lane);
      if (!ok) break;
      tc_fence_after();
      const int row = tc.m * 2 * BM + rank * BM + quarter * 32 + lane;
      const uint32_t tacc = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * 256;
      const int slot = (cluster * 2 + (int)rank) * 4 + quarter;  // this warp's slot (and flag) in pair `cluster`
      if (it.kind == kHead) {
        save_partial<BN>(tacc, sp.ws + (size_t)slot * kSlotChunks * 32, sp.flags + slot, lane);
      } else if (it.kind == kTail && !add_partial<BN>(tacc, sp.ws + (size_t)(slot - 8) * kSlotChunks * 32,
                                                       sp.flags + slot - 8, lane, abort)) {
        break;
      } else if constexpr (EPI == MORJ_EPI_QKV_D128) {
        epilogue_qkv_staged<BN, 128>(tacc, smem_u32(smem) + STAGES * STAGE_BYTES + quarter * STAGE_OUT, row, tc.n,
                                     row < M, qe, N, lane);
      } else if constexpr (EPI == MORJ_EPI_QKV_D64) {
        epilogue_qkv_staged<BN, 64>(tacc, smem_u32(smem) + STAGES * STAGE_BYTES + quarter * STAGE_OUT, row, tc.n,
                                    row < M, qe, N, lane);
      } else if constexpr (EPI == EPI_PEER) {
        epilogue_peer<BN>(tacc, row, tc.n, M, N, pe, pend, pend_cols);
      } else if constexpr (EPI == MORJ_EPI_STORE) {
        store_rows_staged<BN>(tacc, smem_u32(smem) + STAGES * STAGE_BYTES + quarter * STAGE_OUT, C, ldc, row - lane,
                              M, tc.n, N, lane);
      } else {
        // GeGLU writes half as many columns per tile; staged, it measured the same (0.6271 against 0.6266 ms),
        // so its stores stay direct
        epilogue_tile<EPI, BN>(tacc, row, tc.n, row < M, C, ldc, N);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acce_leader + 8 * acc);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if constexpr (EPI == EPI_PEER) peer_arrive(pend, pend_cols, lane);
  }

  tc_fence_before();
  cluster_sync();  // neither CTA leaves while the pair's MMAs or the peer's signals may still touch it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Skinny kernel, M <= 16 activation rows (the last layer's readout rows): C = X . W^T is computed as W . X^T, so the
// weights are the MMA's A operand (128 weight rows per tile, M = 128) and stream through the SMs once, and the
// activation rows are its B operand (N = 16; rows past M are zero-filled by TMA). The (tile, k-block) units,
// tile-major, are cut into one contiguous range per CTA, one CTA per SM, so every SM streams the same number of
// weight bytes whatever the tile count (the 42 tiles of a 5376-wide projection would leave 106 of 148 SMs idle). A
// range's piece of a tile accumulates in TMEM and goes to the workspace as an FP32 [128 x 16] partial; the piece that
// completes a tile (an atomic count per tile, or per gate/up tile pair with the GeGLU epilogue) adds the tile's
// pieces in k order (so the sum does not depend on arrival order), rounds, and stores the output columns of the M
// rows.
// ---------------------------------------------------------------------------------------------------------------
constexpr int SK_N = 16;
constexpr int SK_B_BYTES = SK_N * BK * 2;
constexpr int SK_STAGE = A_BYTES + SK_B_BYTES;  // 18 KB, a multiple of the 1 KB swizzle atom
constexpr int SK_STAGES = 11;
constexpr int SK_SMEM = SK_STAGES * SK_STAGE + 1024 /*align*/ + 256 /*barriers*/;
constexpr int SK_SLOT_FLOATS = BM * SK_N;  // one piece: [128 weight rows][16 activation rows] FP32
constexpr int SK_TMEM_COLS = 32;           // two 16-column accumulators
constexpr uint32_t SK_IDESC = idesc_bf16(BM, SK_N);

struct Skinny {
  float* slots;      // [tiles][pmax][SK_SLOT_FLOATS]
  unsigned* counts;  // per tile (store) or tile pair (GeGLU): pieces arrived this launch; 0 at rest
  int pmax;
};

// The CTA whose range holds unit u when `units` units are cut into `ctas` ranges [units * g / ctas, ...).
__host__ __device__ inline int sk_owner(long long u, int ctas, long long units) {
  return (int)(((u + 1) * ctas + units - 1) / units) - 1;
}
__host__ __device__ inline int sk_pieces(int t, int kb, int ctas, long long units) {
  return sk_owner((long long)t * kb + kb - 1, ctas, units) - sk_owner((long long)t * kb, ctas, units) + 1;
}
// CTA `cta`'s range of units [lo, hi) (non-empty: ctas <= units), its tiles [t_first, t_last] and each tile's
// k-blocks [k0(t), k1(t)); the piece it computes of tile t is cta - sk_owner(t * kb).
struct SkRange {
  long long lo, hi;
  int kb, t_first, t_last;
  __host__ __device__ SkRange(int cta, int ctas, int tiles, int kb_)
      : lo((long long)tiles * kb_ * cta / ctas), hi((long long)tiles * kb_ * (cta + 1) / ctas), kb(kb_),
        t_first((int)(lo / kb_)), t_last((int)((hi - 1) / kb_)) {}
  __host__ __device__ int k0(int t) const { return (int)(lo > (long long)t * kb ? lo - (long long)t * kb : 0); }
  __host__ __device__ int k1(int t) const { return (int)(hi < (long long)(t + 1) * kb ? hi - (long long)t * kb : kb); }
};

MORJ_DEV void sk_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }  // the four epilogue warps

// Sum of tile t's pieces for weight row r (k order).
MORJ_DEV void sk_sum(const Skinny& sk, int t, int r, int pieces, float (&acc)[SK_N]) {
#pragma unroll
  for (int m = 0; m < SK_N; ++m) acc[m] = 0.f;
  for (int q = 0; q < pieces; ++q) {
    const float4* src =
        reinterpret_cast<const float4*>(sk.slots + ((size_t)t * sk.pmax + q) * SK_SLOT_FLOATS + r * SK_N);
#pragma unroll
    for (int v = 0; v < SK_N / 4; ++v) {
      const float4 x = __ldcg(src + v);
      acc[4 * v] += x.x;
      acc[4 * v + 1] += x.y;
      acc[4 * v + 2] += x.z;
      acc[4 * v + 3] += x.w;
    }
  }
}

template <int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    skinny_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                  __nv_bfloat16* __restrict__ C, long long ldc, int M, int N, int K, const Skinny sk) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SK_STAGES * SK_STAGE);
  // bars: full[SK_STAGES], empty[SK_STAGES], acc_full[2], acc_empty[2], done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * SK_STAGES + 5);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + SK_STAGES);
  const uint32_t accf0 = smem_u32(bars + 2 * SK_STAGES), acce0 = smem_u32(bars + 2 * SK_STAGES + 2);
  const uint32_t done0 = smem_u32(bars + 2 * SK_STAGES + 4);
  if (threadIdx.x == 0) {
    for (int s = 0; s < SK_STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf0 + 8 * b, 1);
      mbar_init(acce0 + 8 * b, 128);
    }
    mbar_init(done0, 1);
    *abort = 0;
    fence_mbar_init();
    tma_prefetch(&map_w);
    tma_prefetch(&map_x);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), SK_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // (set-up above touches no global memory) the previous kernel on the stream has completed
  pdl_trigger();

  const int tiles = (N + BM - 1) / BM, kb = (K + BK - 1) / BK;
  const long long units = (long long)tiles * kb;
  const int ctas = (int)gridDim.x;
  const SkRange range((int)blockIdx.x, ctas, tiles, kb);
  const int t_first = range.t_first, t_last = range.t_last;
  const uint32_t smem_base = smem_u32(smem);

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();  // every weight byte is read once
      const uint64_t pol_x = policy_evict_last();   // the activation rows are read by every CTA
      int stage = 0, issued = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = t_first; t <= t_last && ok && !*abort; ++t) {
        const int k0 = range.k0(t), k1 = range.k1(t);
        for (int k = k0; k < k1; ++k) {
          if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, abort, kErrTimeoutGemmProducer)) {
            ok = false;
            break;
          }
          const uint32_t sa = smem_base + stage * SK_STAGE;
          mbar_arrive_expect_tx(full0 + 8 * stage, SK_STAGE);
          tma_load_2d(sa, &map_w, full0 + 8 * stage, k * BK, t * BM, pol_w);
          tma_load_2d(sa + A_BYTES, &map_x, full0 + 8 * stage, k * BK, 0, pol_x);
          ++issued;
          if (++stage == SK_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // no copy may still be in flight when the CTA exits: wait for the last fills to land
      const int pending = issued < SK_STAGES ? issued : SK_STAGES;
      for (int j = 1; j <= pending; ++j) {
        const int s = (stage - j + SK_STAGES) % SK_STAGES;
        const uint32_t ph = (stage - j >= 0) ? phase : (phase ^ 1);
        mbar_wait_landed(full0 + 8 * s, ph);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int t = t_first; t <= t_last && ok; ++t) {
        const int k0 = range.k0(t), k1 = range.k1(t);
        if (!mbar_wait(acce0 + 8 * acc, acc_phase ^ 1, abort, kErrTimeoutGemmMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * SK_N;
        for (int k = k0; k < k1; ++k) {
          if (!mbar_wait(full0 + 8 * stage, phase, abort, kErrTimeoutGemmMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_base + stage * SK_STAGE;
#pragma unroll
          for (int j = 0; j < BK / 16; ++j)
            umma_bf16(d_tmem, sw128_desc(sa + 32 * j), sw128_desc(sa + A_BYTES + 32 * j), SK_IDESC,
                      (k != k0) || j != 0);
          umma_commit(empty0 + 8 * stage);
          if (++stage == SK_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(accf0 + 8 * acc);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      // TMEM is freed below only after every MMA issued here has completed
      umma_commit(done0);
      mbar_wait_landed(done0, 0);
    }
  } else {
    // epilogue warps 2..5: warp w reads TMEM lanes 32 (w % 4) .. + 31, i.e. weight row r of the tile
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = t_first; t <= t_last; ++t) {
      int ok = lane == 0 ? (int)mbar_wait(accf0 + 8 * acc, acc_phase, abort, kErrTimeoutGemmEpilogue) : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;  // (a phase that completed completes for every warp: all four leave at the same tile)
      tc_fence_after();
      uint32_t v[SK_N];
      tmem_ld16(tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * SK_N, v);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(acce0 + 8 * acc);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
      const int first = sk_owner((long long)t * kb, ctas, units);
      float4* slot = reinterpret_cast<float4*>(
          sk.slots + ((size_t)t * sk.pmax + (blockIdx.x - first)) * SK_SLOT_FLOATS + r * SK_N);
#pragma unroll
      for (int q = 0; q < SK_N / 4; ++q)
        slot[q] = make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]), __uint_as_float(v[4 * q + 2]),
                              __uint_as_float(v[4 * q + 3]));
      __threadfence();
      sk_bar();
      const int c = EPI == MORJ_EPI_GEGLU ? t / 2 : t;
      if (warp == 2 && lane == 0) {
        int expected = sk_pieces(t, kb, ctas, units);
        if constexpr (EPI == MORJ_EPI_GEGLU) expected += sk_pieces(t ^ 1, kb, ctas, units);
        *last = atomicAdd(sk.counts + c, 1u) + 1 == (unsigned)expected;
      }
      sk_bar();
      if (*last) {
        __threadfence();
        if constexpr (EPI == MORJ_EPI_GEGLU) {
          // gate rows: tile 2c, up rows: tile 2c + 1 -> output columns [128 c, 128 c + 128)
          float g[SK_N], u[SK_N];
          const int tg = 2 * c;
          sk_sum(sk, tg, r, sk_pieces(tg, kb, ctas, units), g);
          sk_sum(sk, tg + 1, r, sk_pieces(tg + 1, kb, ctas, units), u);
          const int col = c * BM + r;
          if (col < N / 2) {
#pragma unroll
            for (int m = 0; m < SK_N; ++m)
              if (m < M) C[(size_t)m * ldc + col] = __float2bfloat16(gelu_tanh(bf16_round(g[m])) * bf16_round(u[m]));
          }
        } else {
          float a[SK_N];
          sk_sum(sk, t, r, sk_pieces(t, kb, ctas, units), a);
          const int col = t * BM + r;
          if (col < N) {
#pragma unroll
            for (int m = 0; m < SK_N; ++m)
              if (m < M) C[(size_t)m * ldc + col] = __float2bfloat16(a[m]);
          }
        }
        if (warp == 2 && lane == 0) sk.counts[c] = 0;  // every piece of this count has arrived: back to rest
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, SK_TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

}  // namespace gemm

int encode_tiled(CUtensorMap* map, CUtensorMapDataType type, int rank, const void* ptr, const unsigned long long* dims,
                 const unsigned long long* strides_bytes, const unsigned* box, CUtensorMapSwizzle swizzle) {
  gemm::EncodeTiledFn fn = gemm::encode_fn();
  if (!fn) return set_error(MORJ_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) st[i] = strides_bytes[i];
  }
  CUresult r = fn(map, type, rank, const_cast<void*>(ptr), d, st, b, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(MORJ_ERR_ARG, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return MORJ_OK;
}

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

namespace gemm {

// 2D BF16 tensor map over a row-major [rows, cols] matrix with leading dimension ld, box [box_rows, 64 cols].
static int make_map(CUtensorMap* map, const void* ptr, long long rows, long long cols, long long ld, int box_rows) {
  const unsigned long long dims[2] = {(unsigned long long)cols, (unsigned long long)rows};
  const unsigned long long strides[1] = {(unsigned long long)(ld * 2)};
  const unsigned box[2] = {(unsigned)BK, (unsigned)box_rows};
  return encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ptr, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int EPI, int BN>
static int launch(const void* A, long long lda, const void* B, long long ldb, void* C, long long ldc, int M, int N,
                  int K, cudaStream_t stream, const QkvEpi& qe = QkvEpi{}, const PeerEpi& pe = PeerEpi{}) {
  using C_ = Cfg<BN>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(gemm_kernel<EPI, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C_::SMEM_BYTES);
    if (e != cudaSuccess) return set_error(MORJ_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    configured = true;
  }
  CUtensorMap ma, mb;
  int st = make_map(&ma, A, M, K, lda, BM);
  if (st) return st;
  st = make_map(&mb, B, N, K, ldb, BN);
  if (st) return st;
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int grid = tiles < num_sms() ? tiles : num_sms();
  return launch_pdl("gemm_kernel", gemm_kernel<EPI, BN>, dim3(grid), dim3(THREADS), C_::SMEM_BYTES, stream, ma, mb,
                    reinterpret_cast<__nv_bfloat16*>(C), ldc, M, N, K, qe, pe);
}

// Split-tile workspaces, one per (device, stream), registered by the caller (morj_gemm_workspace_set): the pair
// kernel's FP32 partial tiles and their flags live in memory the caller owns, so no launch allocates and launches on
// different streams never share one.
struct Workspace {
  int dev;
  cudaStream_t stream;
  void* ptr;
};
constexpr int kMaxWorkspaces = 64;
static Workspace g_ws[kMaxWorkspaces];
static int g_ws_count = 0;
static std::mutex g_ws_lock;

static unsigned long long workspace_bytes() {
  return (unsigned long long)(num_sms() / 2) * (kSlotBytesPerPair + kFlagBytesPerPair);
}

// The workspace registered for `stream` on the current device, or nullptr.
static void* workspace_for(cudaStream_t stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> g(g_ws_lock);
  for (int i = 0; i < g_ws_count; ++i)
    if (g_ws[i].dev == dev && g_ws[i].stream == stream) return g_ws[i].ptr;
  return nullptr;
}

template <int EPI, int BN>
static int launch2(const void* A, long long lda, const void* B, long long ldb, void* C, long long ldc, int M, int N,
                   int K, cudaStream_t stream, const QkvEpi& qe = QkvEpi{}, const PeerEpi& pe = PeerEpi{}) {
  using C_ = Cfg2<BN>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(gemm2_kernel<EPI, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (pair_smem_bytes<EPI, BN>()));
    if (e != cudaSuccess) return set_error(MORJ_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    configured = true;
  }
  CUtensorMap ma, mb;
  int st = make_map(&ma, A, M, K, lda, BM);
  if (st) return st;
  st = make_map(&mb, B, N, K, ldb, BN / 2);
  if (st) return st;
  const int tiles = ((M + 2 * BM - 1) / (2 * BM)) * ((N + BN - 1) / BN);
  const int pairs = num_sms() / 2;
  const int clusters = tiles < pairs ? tiles : pairs;
  Split sp{nullptr, nullptr, tiles, 0};
  if (void* ws = workspace_for(stream)) {
    split_schedule(tiles, pairs, (K + BK - 1) / BK, &sp.dp_tiles, &sp.units);
    if (sp.units) {  // (only when tiles > pairs: every pair of the grid takes part)
      sp.ws = static_cast<float4*>(ws);
      sp.flags = reinterpret_cast<unsigned*>(static_cast<char*>(ws) + (size_t)pairs * kSlotBytesPerPair);
    }
  }
  return launch_pdl("gemm2_kernel", gemm2_kernel<EPI, BN>, dim3(2 * clusters), dim3(THREADS), (pair_smem_bytes<EPI, BN>()), stream,
                    ma, mb, reinterpret_cast<__nv_bfloat16*>(C), ldc, M, N, K, qe, pe, sp);
}

// Kernel and tile width: the smallest (waves x per-tile time) over the candidates. A wave is one tile per SM (one
// 256-row tile per SM pair for the pair kernel); a tile's time per 64-deep k-block is the larger of its MMA time
// (2 x BN cycles) and the time to fill its stage from L2 (about 1.46 cycles per 128-byte row, measured on the 31B
// shapes: 128 + BN rows for one CTA, 128 + BN / 2 per SM for the pair). With split tiles (`split`: a workspace is
// registered for the stream) the pair kernel's last waves are shared out evenly, so its wave count is fractional
// once there are more tiles than pairs. Ties go to the pair kernel, then to the wider tile.
// The skinny kernel for M <= 16 rows when a workspace is registered for the stream and the partials fit it;
// returns kSkinnyNo when it does not apply (the tiled kernels run instead).
constexpr int kSkinnyNo = -1;
template <int EPI>
static int launch_skinny(const void* A, long long lda, const void* B, long long ldb, void* C, long long ldc, int M,
                         int N, int K, cudaStream_t stream) {
  void* ws = workspace_for(stream);
  if (M > SK_N || !ws) return kSkinnyNo;
  const int tiles = (N + BM - 1) / BM, kb = (K + BK - 1) / BK;
  const long long units = (long long)tiles * kb;
  const int ctas = units < num_sms() ? (int)units : num_sms();
  int pmax = 1;
  for (int t = 0; t < tiles; ++t) {
    const int p = sk_pieces(t, kb, ctas, units);
    pmax = p > pmax ? p : pmax;
  }
  const size_t pairs = num_sms() / 2;
  if ((size_t)tiles * pmax * SK_SLOT_FLOATS * sizeof(float) > pairs * kSlotBytesPerPair ||
      (size_t)tiles * sizeof(unsigned) > pairs * kFlagBytesPerPair)
    return kSkinnyNo;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(skinny_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, SK_SMEM);
    if (e != cudaSuccess) return set_error(MORJ_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    configured = true;
  }
  CUtensorMap mw, mx;
  int st = make_map(&mw, B, N, K, ldb, BM);
  if (st) return st;
  st = make_map(&mx, A, M, K, lda, SK_N);
  if (st) return st;
  // the split-tile workspace's slot area holds the partials, its flag area the counts (both idle between launches)
  const Skinny sk{static_cast<float*>(ws),
                  reinterpret_cast<unsigned*>(static_cast<char*>(ws) + pairs * kSlotBytesPerPair), pmax};
  return launch_pdl("skinny_kernel", skinny_kernel<EPI>, dim3(ctas), dim3(THREADS), SK_SMEM, stream, mw, mx,
                    reinterpret_cast<__nv_bfloat16*>(C), ldc, M, N, K, sk);
}

struct Choice {
  int bn;
  bool pair;
};
static Choice pick(int M, int N, const int* cand, int n_cand, int force, bool split = false) {
  const int sms = num_sms();
  Choice best{cand[0], false};
  double best_cost = -1;
  for (int p = 1; p >= 0; --p) {
    if ((force == 1 && p == 0) || (force == 2 && p == 1)) continue;
    for (int i = 0; i < n_cand; ++i) {
      const int bn = cand[i];
      const long long rows = p ? (M + 2 * BM - 1) / (2 * BM) : (M + BM - 1) / BM;
      const long long tiles = rows * ((N + bn - 1) / bn);
      const int slots = p ? sms / 2 : sms;
      const double fill = 1.46 * (BM + (p ? bn / 2 : bn));
      const double per_tile = 2.0 * bn > fill ? 2.0 * bn : fill;
      const double waves = (p && split && tiles > slots) ? (double)tiles / slots : (double)((tiles + slots - 1) / slots);
      const double cost = waves * per_tile;
      if (best_cost < 0 || cost < best_cost - 1e-9) {
        best_cost = cost;
        best = Choice{bn, p == 1};
      }
    }
  }
  return best;
}

}  // namespace gemm
}  // namespace morj

extern "C" int morj_gemm_bf16(const void* A, long long lda, const void* B, long long ldb, void* C, long long ldc,
                              int M, int N, int K, int epilogue, void* stream) {
  using namespace morj;
  if (M == 0 || N == 0) return MORJ_OK;
  if (!A || !B || !C || M < 0 || N < 0 || K <= 0)
    return set_error(MORJ_ERR_ARG, "morj_gemm_bf16: bad pointers or sizes (M=%d N=%d K=%d)", M, N, K);
  if (K % 8 || lda % 8 || ldb % 8 || ldc % 8 || lda < K || ldb < K)
    return set_error(MORJ_ERR_ARG, "morj_gemm_bf16: K and leading dimensions must be multiples of 8 (K=%d)", K);
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B) | reinterpret_cast<uintptr_t>(C)) & 15)
    return set_error(MORJ_ERR_ARG, "morj_gemm_bf16: pointers must be 16-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int force = (epilogue & MORJ_GEMM_FORCE_PAIR) ? 1 : (epilogue & MORJ_GEMM_FORCE_SINGLE) ? 2 : 0;
  epilogue &= 0xff;
  if (epilogue == MORJ_EPI_STORE) {
    if (N % 16 || ldc < N) return set_error(MORJ_ERR_ARG, "morj_gemm_bf16: N must be a multiple of 16 (N=%d)", N);
    if (!force) {
      const int st = gemm::launch_skinny<MORJ_EPI_STORE>(A, lda, B, ldb, C, ldc, M, N, K, s);
      if (st != gemm::kSkinnyNo) return st;
    }
    static const int cand[] = {256, 240, 224, 208, 192, 176, 160, 128};
    const gemm::Choice c = gemm::pick(M, N, cand, 8, force, gemm::workspace_for(s) != nullptr);
#define MORJ_STORE_CASE(W)                                                                   \
  case W:                                                                                    \
    return c.pair ? gemm::launch2<MORJ_EPI_STORE, W>(A, lda, B, ldb, C, ldc, M, N, K, s)     \
                  : gemm::launch<MORJ_EPI_STORE, W>(A, lda, B, ldb, C, ldc, M, N, K, s);
    switch (c.bn) {
      MORJ_STORE_CASE(240)
      MORJ_STORE_CASE(224)
      MORJ_STORE_CASE(208)
      MORJ_STORE_CASE(192)
      MORJ_STORE_CASE(176)
      MORJ_STORE_CASE(160)
      MORJ_STORE_CASE(128)
      default:
        return c.pair ? gemm::launch2<MORJ_EPI_STORE, 256>(A, lda, B, ldb, C, ldc, M, N, K, s)
                      : gemm::launch<MORJ_EPI_STORE, 256>(A, lda, B, ldb, C, ldc, M, N, K, s);
    }
#undef MORJ_STORE_CASE
  }
  if (epilogue == MORJ_EPI_GEGLU) {
    if (N % 256 || ldc < N / 2)
      return set_error(MORJ_ERR_ARG, "morj_gemm_bf16: GEGLU needs N a multiple of 256 (N=%d)", N);
    if (!force) {
      const int st = gemm::launch_skinny<MORJ_EPI_GEGLU>(A, lda, B, ldb, C, ldc, M, N, K, s);
      if (st != gemm::kSkinnyNo) return st;
    }
    static const int cand[] = {256};
    if (gemm::pick(M, N, cand, 1, force, gemm::workspace_for(s) != nullptr).pair)
      return gemm::launch2<MORJ_EPI_GEGLU, 256>(A, lda, B, ldb, C, ldc, M, N, K, s);
    return gemm::launch<MORJ_EPI_GEGLU, 256>(A, lda, B, ldb, C, ldc, M, N, K, s);
  }
  return set_error(MORJ_ERR_ARG, "morj_gemm_bf16: unknown epilogue %d", epilogue);
}

extern "C" int morj_gemm_bf16_peer(const void* A, long long lda, const void* B, long long ldb, int M, int N, int K,
                                   const morj_peer_t* peer, void* stream) {
  using namespace morj;
  if (M == 0) return MORJ_OK;
  if (!A || !B || !peer || M < 0 || N <= 0 || K <= 0)
    return set_error(MORJ_ERR_ARG, "morj_gemm_bf16_peer: bad pointers or sizes (M=%d N=%d K=%d)", M, N, K);
  if (peer->world < 1 || peer->world > MORJ_MAX_RANKS || peer->rank < 0 || peer->rank >= peer->world ||
      N != peer->hidden || M > peer->max_blocks * 128)
    return set_error(MORJ_ERR_ARG, "morj_gemm_bf16_peer: exchange buffers do not fit (M=%d N=%d)", M, N);
  if (N % 16 || K % 8 || lda % 8 || ldb % 8 || lda < K || ldb < K)
    return set_error(MORJ_ERR_ARG, "morj_gemm_bf16_peer: N % 16, K and leading dimensions % 8 required");
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) & 15)
    return set_error(MORJ_ERR_ARG, "morj_gemm_bf16_peer: pointers must be 16-byte aligned");
  gemm::PeerEpi pe{};
  for (int r = 0; r < peer->world; ++r) {
    if (!peer->partials[r] || (reinterpret_cast<uintptr_t>(peer->partials[r]) & 7))
      return set_error(MORJ_ERR_ARG, "morj_gemm_bf16_peer: rank %d's counters are missing or unaligned", r);
    pe.partials[r] = peer->partials[r];
  }
  if (!peer->part[peer->rank] || (reinterpret_cast<uintptr_t>(peer->part[peer->rank]) & 15))
    return set_error(MORJ_ERR_ARG, "morj_gemm_bf16_peer: part buffer missing or unaligned");
  pe.part = reinterpret_cast<__nv_bfloat16*>(peer->part[peer->rank]);
  pe.world = peer->world;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  static const int cand[] = {256, 208, 192, 128};
  // (the widths the STORE path picks for these shapes)
  const gemm::Choice c = gemm::pick(M, N, cand, 4, 0, gemm::workspace_for(s) != nullptr);
  const gemm::QkvEpi qe{};
#define MORJ_PEER_CASE(W)                                                                                        \
  case W:                                                                                                        \
    return c.pair ? gemm::launch2<gemm::EPI_PEER, W>(A, lda, B, ldb, nullptr, 0, M, N, K, s, qe, pe)             \
                  : gemm::launch<gemm::EPI_PEER, W>(A, lda, B, ldb, nullptr, 0, M, N, K, s, qe, pe);
  switch (c.bn) {
    MORJ_PEER_CASE(208)
    MORJ_PEER_CASE(192)
    MORJ_PEER_CASE(128)
    default:
      return c.pair ? gemm::launch2<gemm::EPI_PEER, 256>(A, lda, B, ldb, nullptr, 0, M, N, K, s, qe, pe)
                    : gemm::launch<gemm::EPI_PEER, 256>(A, lda, B, ldb, nullptr, 0, M, N, K, s, qe, pe);
  }
#undef MORJ_PEER_CASE
}

extern "C" int morj_gemm_qkv_rope(const void* A, long long lda, const void* W, long long ldw, int M, int K, int hq,
                                  int hk, int has_v, int d, const void* q_norm, const void* k_norm,
                                  const int* positions, const void* rope, int rope_rows, const int* slots, float eps,
                                  void* q_out, void* k_pool, void* v_pool, void* stream) {
  using namespace morj;
  if (M == 0 || hq + hk == 0) return MORJ_OK;
  if (!A || !W || !positions || !rope || rope_rows <= 0 || M < 0 || K <= 0 || hq < 0 || hk < 0 ||
      (hq && (!q_out || !q_norm)) || (hk && (!k_pool || !v_pool || !slots || !k_norm)))
    return set_error(MORJ_ERR_ARG, "morj_gemm_qkv_rope: bad pointers or sizes");
  if ((reinterpret_cast<uintptr_t>(rope) | reinterpret_cast<uintptr_t>(q_norm) |
       reinterpret_cast<uintptr_t>(k_norm)) & 15)
    return set_error(MORJ_ERR_ARG, "morj_gemm_qkv_rope: rope table and norm weights must be 16-byte aligned");
  if (K % 8 || lda % 8 || ldw % 8 || lda < K || ldw < K)
    return set_error(MORJ_ERR_ARG, "morj_gemm_qkv_rope: K and leading dimensions must be multiples of 8");
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(W)) & 15)
    return set_error(MORJ_ERR_ARG, "morj_gemm_qkv_rope: pointers must be 16-byte aligned");
  const int force = (has_v & MORJ_GEMM_FORCE_PAIR) ? 1 : (has_v & MORJ_GEMM_FORCE_SINGLE) ? 2 : 0;
  has_v &= 0xff;
  const int N = (hq + (has_v ? 2 : 1) * hk) * d;
  gemm::QkvEpi e{hq, hk, has_v ? 1 : 0, (const __nv_bfloat16*)q_norm, (const __nv_bfloat16*)k_norm, positions,
                 (const float4*)rope, rope_rows, slots, eps, (__nv_bfloat16*)q_out, (__nv_bfloat16*)k_pool,
                 (__nv_bfloat16*)v_pool};
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // The head epilogue costs about as much per 128 columns as 35 k-blocks of main loop, which the cost model does not
  // see: 128-wide tiles pay it twice as often. So without split tiles (or with at most one 256-row block) the
  // one-CTA kernel unless forced (2040 x 8192 x 5376: 0.20 ms pair at BN 128, 0.158 ms one-CTA); with them, BN 256
  // and the kernel per shape (2040 x 8192 x 5376: the pair kernel, 0.146 ms).
  static const int cand[] = {256, 128};
  const bool split = gemm::workspace_for(s) != nullptr && M > 2 * gemm::BM;
  const gemm::Choice c = gemm::pick(M, N, cand, split ? 1 : 2, force ? force : (split ? 0 : 2), split);
  if (d == 128) {
    if (c.bn == 128)
      return c.pair ? gemm::launch2<MORJ_EPI_QKV_D128, 128>(A, lda, W, ldw, nullptr, 0, M, N, K, s, e)
                    : gemm::launch<MORJ_EPI_QKV_D128, 128>(A, lda, W, ldw, nullptr, 0, M, N, K, s, e);
    return c.pair ? gemm::launch2<MORJ_EPI_QKV_D128, 256>(A, lda, W, ldw, nullptr, 0, M, N, K, s, e)
                  : gemm::launch<MORJ_EPI_QKV_D128, 256>(A, lda, W, ldw, nullptr, 0, M, N, K, s, e);
  }
  if (d == 64) {
    if (c.bn == 128)
      return c.pair ? gemm::launch2<MORJ_EPI_QKV_D64, 128>(A, lda, W, ldw, nullptr, 0, M, N, K, s, e)
                    : gemm::launch<MORJ_EPI_QKV_D64, 128>(A, lda, W, ldw, nullptr, 0, M, N, K, s, e);
    return c.pair ? gemm::launch2<MORJ_EPI_QKV_D64, 256>(A, lda, W, ldw, nullptr, 0, M, N, K, s, e)
                  : gemm::launch<MORJ_EPI_QKV_D64, 256>(A, lda, W, ldw, nullptr, 0, M, N, K, s, e);
  }
  return set_error(MORJ_ERR_UNSUPPORTED, "morj_gemm_qkv_rope: head_dim %d unsupported (64, 128)", d);
}

extern "C" int morj_gemm_workspace_bytes(unsigned long long* bytes) {
  if (!bytes) return morj::set_error(MORJ_ERR_ARG, "morj_gemm_workspace_bytes: null output");
  *bytes = morj::gemm::workspace_bytes();
  return MORJ_OK;
}

extern "C" int morj_gemm_workspace_set(void* stream, void* ptr, unsigned long long bytes) {
  using namespace morj;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(MORJ_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (ptr) {
    const unsigned long long need = gemm::workspace_bytes();
    if (reinterpret_cast<uintptr_t>(ptr) & 255)
      return set_error(MORJ_ERR_ARG, "morj_gemm_workspace_set: the workspace must be 256-byte aligned");
    if (bytes < need)
      return set_error(MORJ_ERR_ARG, "morj_gemm_workspace_set: %llu bytes given, %llu needed", bytes, need);
    const size_t pairs = num_sms() / 2;
    e = cudaMemsetAsync(static_cast<char*>(ptr) + pairs * gemm::kSlotBytesPerPair, 0,
                        pairs * gemm::kFlagBytesPerPair, s);
    if (e != cudaSuccess) return set_error(MORJ_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
  }
  std::lock_guard<std::mutex> g(gemm::g_ws_lock);
  for (int i = 0; i < gemm::g_ws_count; ++i) {
    if (gemm::g_ws[i].dev == dev && gemm::g_ws[i].stream == s) {
      if (ptr)
        gemm::g_ws[i].ptr = ptr;
      else
        gemm::g_ws[i] = gemm::g_ws[--gemm::g_ws_count];
      return MORJ_OK;
    }
  }
  if (!ptr) return MORJ_OK;
  if (gemm::g_ws_count == gemm::kMaxWorkspaces)
    return set_error(MORJ_ERR_UNSUPPORTED, "morj_gemm_workspace_set: more than %d streams", gemm::kMaxWorkspaces);
  gemm::g_ws[gemm::g_ws_count++] = gemm::Workspace{dev, s, ptr};
  return MORJ_OK;
}

extern "C" int morj_gemm_workspace_remove(const void* ptr) {
  using namespace morj;
  std::lock_guard<std::mutex> g(gemm::g_ws_lock);
  for (int i = 0; i < gemm::g_ws_count;) {
    if (gemm::g_ws[i].ptr == ptr)
      gemm::g_ws[i] = gemm::g_ws[--gemm::g_ws_count];
    else
      ++i;
  }
  return MORJ_OK;
}

extern "C" int morj_gemm_skinny_walk(int tiles, int kblocks, int ctas, int cta, int* items, int cap) {
  using namespace morj::gemm;
  if (tiles < 1 || kblocks < 1 || ctas < 1 || (long long)ctas > (long long)tiles * kblocks || cta < 0 ||
      cta >= ctas || cap < 0 || (cap && !items))
    return -1;
  const long long units = (long long)tiles * kblocks;
  const SkRange range(cta, ctas, tiles, kblocks);
  int n = 0;
  for (int t = range.t_first; t <= range.t_last; ++t) {
    if (n == cap) return -1;
    items[5 * n] = t;
    items[5 * n + 1] = range.k0(t);
    items[5 * n + 2] = range.k1(t);
    items[5 * n + 3] = cta - sk_owner((long long)t * kblocks, ctas, units);
    items[5 * n + 4] = sk_pieces(t, kblocks, ctas, units);
    ++n;
  }
  return n;
}

extern "C" int morj_gemm_split_walk(int tiles, int pairs, int kblocks, int pair, int* items, int cap) {
  using namespace morj::gemm;
  if (tiles < 0 || pairs < 1 || kblocks < 1 || pair < 0 || pair >= pairs || cap < 0 || (cap && !items)) return -1;
  int dp = 0;
  long long units = 0;
  split_schedule(tiles, pairs, kblocks, &dp, &units);
  Walk walk(pair, pairs, kblocks, dp, units);
  Item it;
  int n = 0;
  while (walk.next(it)) {
    if (n == cap) return -1;
    items[4 * n] = it.tile;
    items[4 * n + 1] = it.k0;
    items[4 * n + 2] = it.k1;
    items[4 * n + 3] = it.kind;
    ++n;
  }
  return n;
}
