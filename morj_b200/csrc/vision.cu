// Row kernels of the image path (the vision tower that turns image patches into soft tokens, and the projection into
// the text model's embedding space). The tower's projections, GeGLU MLP and residual epilogues run on the library's
// GEMM and row kernels and its attention on the tree attention kernel (one bidirectional segment per image); what is
// particular to images is here:
//   * patch prologue: pixel values in [0, 1] rescaled to [-1, 1] in BF16 arithmetic (2 * (p - 0.5));
//   * position add: each patch adds the sum of its x and y rows of the two learned position tables (zero for padding
//     patches);
//   * head epilogue: per head RMSNorm (q, k weighted; v unweighted) and 2-D rotary embedding, the first half of the
//     head dims rotated by the patch's x position and the second half by its y position, each half rotating pairs
//     (i, i + d/4); BF16 rounding after every elementwise step, as a BF16 module computes it;
//   * pooling: the average of each k x k cell of patches (FP32 sum, padding patches excluded) times sqrt(hidden);
//   * row norm: RMSNorm with or without a weight.
// The numerics follow the reference's image path (`aleria_judge/lean_core.py:745-781`, transformers' Gemma 4 vision
// model in BF16). Every kernel reads and writes only the rows it is given; no waits, no scratch memory.
#include "common.cuh"

namespace morj {
namespace vision {

constexpr int THREADS = 256;

MORJ_DEV float bf(float v) { return bf16_round(v); }

// x[i] = bf16(2 * bf16(x[i] - 0.5)), in place, n elements (n % 8 == 0)
__global__ void __launch_bounds__(THREADS) patch_prologue_kernel(__nv_bfloat16* __restrict__ x, long long n8) {
  pdl_wait();
  pdl_trigger();
  for (long long i = blockIdx.x * (long long)THREADS + threadIdx.x; i < n8; i += (long long)gridDim.x * THREADS) {
    float v[8];
    load8(x + i * 8, v);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = bf(2.f * bf(v[e] - 0.5f));
    store8(x + i * 8, v);
  }
}

// x[r] = bf16(x[r] + bf16(table[0][px] + table[1][py])) for patches with a position; padding patches (-1, -1) keep x
__global__ void __launch_bounds__(THREADS) position_add_kernel(__nv_bfloat16* __restrict__ x,
                                                               const int* __restrict__ pos,
                                                               const __nv_bfloat16* __restrict__ table, int H,
                                                               int table_rows) {
  pdl_wait();
  pdl_trigger();
  const size_t r = blockIdx.x;
  const int px = pos[2 * r], py = pos[2 * r + 1];
  if (px < 0 && py < 0) return;
  if (px < 0 || py < 0 || px >= table_rows || py >= table_rows) {
    if (threadIdx.x == 0) report(kErrBadIndex);
    return;
  }
  const __nv_bfloat16* tx = table + (size_t)px * H;
  const __nv_bfloat16* ty = table + ((size_t)table_rows + py) * H;
  for (int c = threadIdx.x * 8; c < H; c += THREADS * 8) {
    float xv[8], a[8], b[8];
    load8(x + r * H + c, xv);
    load8(tx + c, a);
    load8(ty + c, b);
#pragma unroll
    for (int e = 0; e < 8; ++e) xv[e] = bf(xv[e] + bf(a[e] + b[e]));
    store8(x + r * H + c, xv);
  }
}

// One warp per (token, head) of the fused [q | k | v] projection rows (ld elements apart); lane l holds elements
// [l * E, l * E + E) of each quarter of the head (E = D / 128, D in {64, 128}).
template <int D>
__global__ void __launch_bounds__(THREADS) head_epilogue_kernel(const __nv_bfloat16* __restrict__ qkv, long long ld,
                                                                int heads, const __nv_bfloat16* __restrict__ q_norm,
                                                                const __nv_bfloat16* __restrict__ k_norm,
                                                                const int* __restrict__ pos,
                                                                const float* __restrict__ inv_freq, float eps,
                                                                __nv_bfloat16* __restrict__ q_out,
                                                                __nv_bfloat16* __restrict__ k_out,
                                                                __nv_bfloat16* __restrict__ v_out, int n) {
  pdl_wait();
  pdl_trigger();
  constexpr int Q4 = D / 4;   // rotated pairs per spatial dimension
  constexpr int E = Q4 / 32;  // elements per lane in each quarter (D = 128: 1; D = 64: handled with a lane mask)
  constexpr int EL = E > 0 ? E : 1;
  const int warp = blockIdx.x * (THREADS / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int tok = warp / (3 * heads), hh = warp % (3 * heads);
  if (tok >= n) return;
  const int kind = hh / heads, head = hh % heads;  // 0 q, 1 k, 2 v
  const __nv_bfloat16* src = qkv + (size_t)tok * ld + (size_t)hh * D;
  const bool active = E > 0 || lane < Q4;  // D = 64: 16 pairs per quarter, lanes 16..31 idle
  // element j of quarter g: index g * Q4 + i, i = lane * EL + j
  float v[4][EL];
  float ss = 0.f;
#pragma unroll
  for (int g = 0; g < 4; ++g)
#pragma unroll
    for (int j = 0; j < EL; ++j) {
      const int i = lane * EL + j;
      v[g][j] = active ? __bfloat162float(src[g * Q4 + i]) : 0.f;
      ss += v[g][j] * v[g][j];
    }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (!active) return;
  const float inv = 1.0f / sqrtf(ss / D + eps);
  const __nv_bfloat16* w = kind == 0 ? q_norm : k_norm;
  float y[4][EL];
#pragma unroll
  for (int g = 0; g < 4; ++g)
#pragma unroll
    for (int j = 0; j < EL; ++j) {
      const int i = lane * EL + j;
      const float wv = kind < 2 ? __bfloat162float(w[g * Q4 + i]) : 1.f;
      y[g][j] = bf(v[g][j] * inv * wv);  // the norm's BF16 output
    }
  __nv_bfloat16* dst = (kind == 0 ? q_out : kind == 1 ? k_out : v_out) + ((size_t)tok * heads + head) * D;
  if (kind == 2) {
#pragma unroll
    for (int g = 0; g < 4; ++g)
#pragma unroll
      for (int j = 0; j < EL; ++j) dst[g * Q4 + lane * EL + j] = __float2bfloat16(y[g][j]);
    return;
  }
  // quarters 0, 1: the x half (pairs (i, i + Q4)); quarters 2, 3: the y half
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const float p = (float)pos[2 * tok + half];
#pragma unroll
    for (int j = 0; j < EL; ++j) {
      const int i = lane * EL + j;
      float sn, cs;
      sincosf(p * inv_freq[i], &sn, &cs);
      const float c = bf(cs), s = bf(sn);  // the rotary tables are BF16 in a BF16 module
      const float a = y[2 * half][j], b = y[2 * half + 1][j];
      dst[(2 * half) * Q4 + i] = __float2bfloat16(bf(a * c) + bf(-b * s));
      dst[(2 * half + 1) * Q4 + i] = __float2bfloat16(bf(b * c) + bf(a * s));
    }
  }
}

// out[c] = bf16(bf16(sum over rows of cell c of x[row] / k2) * scale)
__global__ void __launch_bounds__(THREADS) pool_kernel(const __nv_bfloat16* __restrict__ x, int H,
                                                       const int* __restrict__ cell_indptr,
                                                       const int* __restrict__ cell_rows, float inv_k2, float scale,
                                                       __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int cell = blockIdx.x;
  const int r0 = cell_indptr[cell], r1 = cell_indptr[cell + 1];
  for (int c = threadIdx.x * 8; c < H; c += THREADS * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = r0; r < r1; ++r) {
      float v[8];
      load8(x + (size_t)cell_rows[r] * H + c, v);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += v[e] * inv_k2;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = bf(bf(acc[e]) * scale);
    store8(out + (size_t)cell * H + c, acc);
  }
}

// out[r] = bf16(x[r] * rsqrt(mean(x[r]^2) + eps) * w), w = 1 when null
template <int VPT>
__global__ void __launch_bounds__(THREADS) norm_kernel(const __nv_bfloat16* __restrict__ x,
                                                       const __nv_bfloat16* __restrict__ w, int H, float eps,
                                                       __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  const size_t base = (size_t)blockIdx.x * H;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = (threadIdx.x + k * THREADS) * 8;
    if (c < H) {
      load8(x + base + c, v[k]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[k][e] * v[k][e];
    }
  }
  const float inv = 1.0f / sqrtf(block_sum(ss, red) / H + eps);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = (threadIdx.x + k * THREADS) * 8;
    if (c < H) {
      float wv[8], o[8];
      if (w) load8(w + c, wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = v[k][e] * inv * (w ? wv[e] : 1.f);
      store8(out + base + c, o);
    }
  }
}

}  // namespace vision
}  // namespace morj

using namespace morj;

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

extern "C" int morj_vision_patch_prologue(void* pixels, long long n, void* stream) {
  if (n == 0) return MORJ_OK;
  if (!pixels || n < 0 || n % 8 || !aligned16(pixels))
    return set_error(MORJ_ERR_ARG, "morj_vision_patch_prologue: bad arguments (n=%lld)", n);
  const long long n8 = n / 8;
  const unsigned grid = (unsigned)std::min<long long>((n8 + vision::THREADS - 1) / vision::THREADS, 4096);
  return launch_pdl("patch_prologue_kernel", vision::patch_prologue_kernel, dim3(grid), dim3(vision::THREADS), 0,
                    reinterpret_cast<cudaStream_t>(stream), (__nv_bfloat16*)pixels, n8);
}

extern "C" int morj_vision_position_add(void* x, const int* positions, const void* table, int table_rows, int n,
                                        int H, void* stream) {
  if (n == 0) return MORJ_OK;
  if (!x || !positions || !table || n < 0 || H <= 0 || H % 8 || table_rows <= 0 || !aligned16(x) ||
      !aligned16(table))
    return set_error(MORJ_ERR_ARG, "morj_vision_position_add: bad arguments (n=%d H=%d)", n, H);
  return launch_pdl("position_add_kernel", vision::position_add_kernel, dim3(n), dim3(vision::THREADS), 0,
                    reinterpret_cast<cudaStream_t>(stream), (__nv_bfloat16*)x, positions,
                    (const __nv_bfloat16*)table, H, table_rows);
}

extern "C" int morj_vision_head_epilogue(const void* qkv, long long ld, int n, int heads, int d, const void* q_norm,
                                         const void* k_norm, const int* positions, const float* inv_freq, float eps,
                                         void* q_out, void* k_out, void* v_out, void* stream) {
  if (n == 0) return MORJ_OK;
  if (!qkv || !q_norm || !k_norm || !positions || !inv_freq || !q_out || !k_out || !v_out || n < 0 || heads <= 0 ||
      ld < 3LL * heads * d)
    return set_error(MORJ_ERR_ARG, "morj_vision_head_epilogue: bad arguments (n=%d heads=%d d=%d)", n, heads, d);
  const long long warps = (long long)n * 3 * heads;
  const unsigned grid = (unsigned)((warps + vision::THREADS / 32 - 1) / (vision::THREADS / 32));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const auto* a = (const __nv_bfloat16*)qkv;
  const auto* qn = (const __nv_bfloat16*)q_norm;
  const auto* kn = (const __nv_bfloat16*)k_norm;
  if (d == 128)
    return launch_pdl("head_epilogue_kernel", vision::head_epilogue_kernel<128>, dim3(grid), dim3(vision::THREADS),
                      0, s, a, ld, heads, qn, kn, positions, inv_freq, eps, (__nv_bfloat16*)q_out,
                      (__nv_bfloat16*)k_out, (__nv_bfloat16*)v_out, n);
  if (d == 64)
    return launch_pdl("head_epilogue_kernel", vision::head_epilogue_kernel<64>, dim3(grid), dim3(vision::THREADS), 0,
                      s, a, ld, heads, qn, kn, positions, inv_freq, eps, (__nv_bfloat16*)q_out,
                      (__nv_bfloat16*)k_out, (__nv_bfloat16*)v_out, n);
  return set_error(MORJ_ERR_UNSUPPORTED, "morj_vision_head_epilogue: head_dim %d unsupported (64, 128)", d);
}

extern "C" int morj_vision_pool(const void* x, int H, const int* cell_indptr, const int* cell_rows, int n_cells,
                                float inv_k2, float scale, void* out, void* stream) {
  if (n_cells == 0) return MORJ_OK;
  if (!x || !cell_indptr || !cell_rows || !out || n_cells < 0 || H <= 0 || H % 8 || !aligned16(x) ||
      !aligned16(out))
    return set_error(MORJ_ERR_ARG, "morj_vision_pool: bad arguments (cells=%d H=%d)", n_cells, H);
  return launch_pdl("pool_kernel", vision::pool_kernel, dim3(n_cells), dim3(vision::THREADS), 0,
                    reinterpret_cast<cudaStream_t>(stream), (const __nv_bfloat16*)x, H, cell_indptr, cell_rows,
                    inv_k2, scale, (__nv_bfloat16*)out);
}

extern "C" int morj_rmsnorm_rows(const void* x, const void* w, int n, int H, float eps, void* out, void* stream) {
  if (n == 0) return MORJ_OK;
  if (!x || !out || n < 0 || H <= 0 || H % 8 || H > 8 * vision::THREADS * 8 || !aligned16(x) || !aligned16(out))
    return set_error(MORJ_ERR_ARG, "morj_rmsnorm_rows: bad arguments (n=%d H=%d)", n, H);
  int st = MORJ_OK;
  MORJ_VPT_SWITCH(H, (st = launch_pdl("norm_kernel", vision::norm_kernel<V>, dim3(n), dim3(vision::THREADS), 0,
                                      reinterpret_cast<cudaStream_t>(stream), (const __nv_bfloat16*)x,
                                      (const __nv_bfloat16*)w, H, eps, (__nv_bfloat16*)out)));
  return st;
}
