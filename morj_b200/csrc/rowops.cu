// Memory-bound row kernels of the tree-prefill forward (HBM roofline): embedding gather + input norm, the per-head
// q/k/v norm + RoPE + pool scatter, the post-attention and post-MLP residual epilogues (each fused with the next
// RMSNorm), the reference-layout GeGLU, row gathers/scatters and the label-restricted LM head.
// All norms accumulate in FP32 and round to BF16 exactly where the reference path rounds.
#include <cstdarg>
#include <cstdio>
#include <string>

#include "common.cuh"

namespace morj {

__device__ int g_device_error = 0;

namespace rows {

constexpr int THREADS = 256;

MORJ_DEV float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = -INFINITY;
  const int nw = blockDim.x / 32;
  for (int i = 0; i < nw; ++i) t = fmaxf(t, red[i]);
  return t;
}

// ---- embedding + image rows + input RMSNorm -------------------------------------------------------------------
template <int VPT>
__global__ void __launch_bounds__(THREADS) embed_rmsnorm_kernel(const int* __restrict__ tokens,
                                                                const int* __restrict__ feature_row,
                                                                const __nv_bfloat16* __restrict__ features,
                                                                const __nv_bfloat16* __restrict__ embed, int H,
                                                                float scale, const __nv_bfloat16* __restrict__ w,
                                                                float eps, __nv_bfloat16* __restrict__ x_out,
                                                                __nv_bfloat16* __restrict__ h_out) {
  pdl_wait();  // the previous kernel on the stream has completed
  pdl_trigger();
  __shared__ float red[32];
  const size_t row = blockIdx.x;
  const int fr = feature_row ? feature_row[row] : -1;
  const __nv_bfloat16* src = fr >= 0 ? features + (size_t)fr * H : embed + (size_t)tokens[row] * H;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = (threadIdx.x + k * THREADS) * 8;
    if (c < H) {
      load8(src + c, v[k]);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (fr < 0) v[k][e] = bf16_round(v[k][e] * scale);
        ss += v[k][e] * v[k][e];
      }
      store8(x_out + row * H + c, v[k]);
    }
  }
  const float inv = 1.0f / sqrtf(block_sum_fresh(ss, red) / H + eps);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = (threadIdx.x + k * THREADS) * 8;
    if (c < H) {
      float wv[8], o[8];
      load8(w + c, wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = v[k][e] * inv * wv[e];
      store8(h_out + row * H + c, o);
    }
  }
}

// ---- post-attention epilogue: x += rms(o) * w_post; h = rms(x) * w_pre -----------------------------------------
// Both rows a CTA reads from HBM (o and x) are loaded up front and kept as packed BF16, so a row waits on HBM once;
// the norm weights (shared by every row, L2-resident) are read where they are used.
template <int VPT>
__global__ void __launch_bounds__(THREADS) attn_epilogue_kernel(const __nv_bfloat16* __restrict__ o,
                                                                __nv_bfloat16* __restrict__ x,
                                                                __nv_bfloat16* __restrict__ h_out,
                                                                const __nv_bfloat16* __restrict__ w_post,
                                                                const __nv_bfloat16* __restrict__ w_pre, int H,
                                                                float eps) {
  pdl_wait();  // the previous kernel on the stream has completed
  pdl_trigger();
  __shared__ float red[2][32];  // one array per reduction
  const size_t base = (size_t)blockIdx.x * H;
  uint4 o_raw[VPT], x_raw[VPT], w_raw[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = (threadIdx.x + k * THREADS) * 8;
    if (c < H) {
      o_raw[k] = *reinterpret_cast<const uint4*>(o + base + c);
      x_raw[k] = *reinterpret_cast<const uint4*>(x + base + c);
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = (threadIdx.x + k * THREADS) * 8;
    if (c < H) {
      float ov[8];
      unpack8(o_raw[k], ov);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += ov[e] * ov[e];
    }
  }
  const float inv1 = 1.0f / sqrtf(block_sum_fresh(ss, red[0]) / H + eps);
  float ss2 = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = (threadIdx.x + k * THREADS) * 8;
    if (c < H) {
      float ov[8], xv[8], wv[8];
      unpack8(o_raw[k], ov);
      unpack8(x_raw[k], xv);
      load8(w_post + c, wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float on = bf16_round(ov[e] * inv1 * wv[e]);
        xv[e] = bf16_round(xv[e] + on);  // the new residual
        ss2 += xv[e] * xv[e];
      }
      x_raw[k] = pack8(xv);
      *reinterpret_cast<uint4*>(x + base + c) = x_raw[k];
      w_raw[k] = *reinterpret_cast<const uint4*>(w_pre + c);
    }
  }
  const float inv2 = 1.0f / sqrtf(block_sum_fresh(ss2, red[1]) / H + eps);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = (threadIdx.x + k * THREADS) * 8;
    if (c < H) {
      float xv[8], wv[8], hv[8];
      unpack8(x_raw[k], xv);
      unpack8(w_raw[k], wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) hv[e] = xv[e] * inv2 * wv[e];
      store8(h_out + base + c, hv);
    }
  }
}

// ---- post-MLP epilogue: x = (x + rms(d) * w_post) * scalar; h = rms(x) * w_next ---------------------------------
// d and x are loaded up front as in the post-attention epilogue.
template <int VPT>
__global__ void __launch_bounds__(THREADS) mlp_epilogue_kernel(const __nv_bfloat16* __restrict__ d,
                                                               __nv_bfloat16* x, __nv_bfloat16* h_out,
                                                               const __nv_bfloat16* __restrict__ w_post,
                                                               const __nv_bfloat16* __restrict__ scalar,
                                                               const __nv_bfloat16* __restrict__ w_next, int H,
                                                               float eps, int has_next) {
  pdl_wait();  // the previous kernel on the stream has completed
  pdl_trigger();
  __shared__ float red[2][32];  // one array per reduction
  const size_t base = (size_t)blockIdx.x * H;
  const float sc = __bfloat162float(scalar[0]);
  uint4 d_raw[VPT], x_raw[VPT], w_raw[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = (threadIdx.x + k * THREADS) * 8;
    if (c < H) {
      d_raw[k] = *reinterpret_cast<const uint4*>(d + base + c);
      x_raw[k] = *reinterpret_cast<const uint4*>(x + base + c);
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = (threadIdx.x + k * THREADS) * 8;
    if (c < H) {
      float dv[8];
      unpack8(d_raw[k], dv);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += dv[e] * dv[e];
    }
  }
  const float inv1 = 1.0f / sqrtf(block_sum_fresh(ss, red[0]) / H + eps);
  float ss2 = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = (threadIdx.x + k * THREADS) * 8;
    if (c < H) {
      float dv[8], xv[8], wv[8];
      unpack8(d_raw[k], dv);
      unpack8(x_raw[k], xv);
      load8(w_post + c, wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float dn = bf16_round(dv[e] * inv1 * wv[e]);
        const float xa = bf16_round(xv[e] + dn);
        xv[e] = bf16_round(xa * sc);
        ss2 += xv[e] * xv[e];
      }
      x_raw[k] = pack8(xv);
      *reinterpret_cast<uint4*>(x + base + c) = x_raw[k];
      if (has_next) w_raw[k] = *reinterpret_cast<const uint4*>(w_next + c);
    }
  }
  if (!has_next) return;
  const float inv2 = 1.0f / sqrtf(block_sum_fresh(ss2, red[1]) / H + eps);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = (threadIdx.x + k * THREADS) * 8;
    if (c < H) {
      float xv[8], wv[8], hv[8];
      unpack8(x_raw[k], xv);
      unpack8(w_raw[k], wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) hv[e] = xv[e] * inv2 * wv[e];
      store8(h_out + base + c, hv);
    }
  }
}

// ---- q/k/v head norm + RoPE + scatter to the packed q and the K/V pools ------------------------------------------
// one warp per head; lane l holds elements [l*E, l*E + E) of each half (E = D / 64)
template <int D>
__global__ void __launch_bounds__(THREADS) qkv_post_kernel(const __nv_bfloat16* __restrict__ qkv, long long ld,
                                                           int hq, int hk, int has_v,
                                                           const __nv_bfloat16* __restrict__ q_norm,
                                                           const __nv_bfloat16* __restrict__ k_norm,
                                                           const int* __restrict__ positions,
                                                           const float* __restrict__ inv_freq,
                                                           const int* __restrict__ slots, float eps,
                                                           __nv_bfloat16* __restrict__ q_out,
                                                           __nv_bfloat16* __restrict__ k_pool,
                                                           __nv_bfloat16* __restrict__ v_pool) {
  pdl_wait();  // the previous kernel on the stream has completed
  pdl_trigger();
  constexpr int HALF = D / 2;
  constexpr int E = HALF / 32;
  const int tok = blockIdx.x;
  const int head = blockIdx.y * (THREADS / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (head >= hq + 2 * hk) return;
  const bool is_q = head < hq;
  const bool is_k = !is_q && head < hq + hk;
  const int hkk = head - hq, hvv = head - hq - hk;
  const int col = is_q ? head * D : (is_k ? (hq + hkk) * D : (hq + has_v * hk + hvv) * D);
  const __nv_bfloat16* src = qkv + (size_t)tok * ld + col;
  float x1[E], x2[E];
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    x1[e] = __bfloat162float(src[lane * E + e]);
    x2[e] = __bfloat162float(src[HALF + lane * E + e]);
    ss += x1[e] * x1[e] + x2[e] * x2[e];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = 1.0f / sqrtf(ss / D + eps);
  const __nv_bfloat16* w = is_q ? q_norm : k_norm;
  const float pos = (float)positions[tok];
  float o1[E], o2[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = lane * E + e;
    const float w1 = (is_q || is_k) ? __bfloat162float(w[i]) : 1.f;
    const float w2 = (is_q || is_k) ? __bfloat162float(w[HALF + i]) : 1.f;
    const float y1 = bf16_round(x1[e] * inv * w1);  // the normed vector is rounded to BF16 before RoPE
    const float y2 = bf16_round(x2[e] * inv * w2);
    if (is_q || is_k) {
      float sn, cs;
      sincosf(pos * inv_freq[i], &sn, &cs);
      o1[e] = y1 * cs - y2 * sn;
      o2[e] = y2 * cs + y1 * sn;
    } else {
      o1[e] = y1;
      o2[e] = y2;
    }
  }
  __nv_bfloat16* dst;
  if (is_q) {
    dst = q_out + ((size_t)tok * hq + head) * D;
  } else {
    const size_t slot = (size_t)slots[tok];
    dst = (is_k ? k_pool + (slot * hk + hkk) * D : v_pool + (slot * hk + hvv) * D);
  }
#pragma unroll
  for (int e = 0; e < E; ++e) {
    dst[lane * E + e] = __float2bfloat16(o1[e]);
    dst[HALF + lane * E + e] = __float2bfloat16(o2[e]);
  }
}

// ---- reference-layout GeGLU --------------------------------------------------------------------------------------
__global__ void geglu_kernel(const __nv_bfloat16* __restrict__ gu, int F, __nv_bfloat16* __restrict__ out) {
  pdl_wait();  // the previous kernel on the stream has completed
  pdl_trigger();
  const size_t row = blockIdx.y;
  for (int c = (blockIdx.x * blockDim.x + threadIdx.x) * 8; c < F; c += gridDim.x * blockDim.x * 8) {
    float g[8], u[8], o[8];
    load8(gu + row * 2 * F + c, g);
    load8(gu + row * 2 * F + F + c, u);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = gelu_tanh(g[e]) * u[e];
    store8(out + row * F + c, o);
  }
}

// ---- row gather / scatter ----------------------------------------------------------------------------------------
__global__ void copy_rows_kernel(const __nv_bfloat16* __restrict__ src, long long ld_src,
                                 const int* __restrict__ rows, int width, __nv_bfloat16* __restrict__ dst,
                                 long long ld_dst, int scatter) {
  pdl_wait();  // the previous kernel on the stream has completed
  pdl_trigger();
  const int i = blockIdx.x;
  const size_t s = scatter ? (size_t)i : (size_t)rows[i];
  const size_t d = scatter ? (size_t)rows[i] : (size_t)i;
  for (int c = threadIdx.x * 8; c < width; c += blockDim.x * 8)
    *reinterpret_cast<uint4*>(dst + d * ld_dst + c) = *reinterpret_cast<const uint4*>(src + s * ld_src + c);
}

// ---- label head: final norm, label-row logits, softcap, softmax ---------------------------------------------------
__global__ void __launch_bounds__(THREADS) label_head_kernel(const __nv_bfloat16* __restrict__ x, long long ld_x,
                                                             const int* __restrict__ seq_row,
                                                             const int* __restrict__ label_indptr,
                                                             const int* __restrict__ label_ids,
                                                             const __nv_bfloat16* __restrict__ norm_w,
                                                             const __nv_bfloat16* __restrict__ embed, int H,
                                                             float eps, float softcap, float* __restrict__ probs) {
  pdl_wait();  // the previous kernel on the stream has completed
  pdl_trigger();
  extern __shared__ float sh[];
  float* normed = sh;      // H
  float* logits = sh + H;  // labels of this sequence
  __shared__ float red[32];
  const int j = blockIdx.x;
  const __nv_bfloat16* xr = x + (size_t)seq_row[j] * ld_x;
  float ss = 0.f;
  for (int c = threadIdx.x; c < H; c += THREADS) {
    const float v = __bfloat162float(xr[c]);
    normed[c] = v;
    ss += v * v;
  }
  const float inv = 1.0f / sqrtf(block_sum(ss, red) / H + eps);
  for (int c = threadIdx.x; c < H; c += THREADS)
    normed[c] = bf16_round(normed[c] * inv * __bfloat162float(norm_w[c]));
  __syncthreads();
  const int l0 = label_indptr[j], nl = label_indptr[j + 1] - l0;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (int l = warp; l < nl; l += THREADS / 32) {
    const __nv_bfloat16* er = embed + (size_t)label_ids[l0 + l] * H;
    float acc = 0.f;
    for (int c = lane * 8; c < H; c += 256) {
      float ev[8];
      load8(er + c, ev);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc += normed[c + e] * ev[e];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) logits[l] = softcap * tanhf(acc / softcap);
  }
  __syncthreads();
  float mx = -INFINITY;
  for (int l = threadIdx.x; l < nl; l += THREADS) mx = fmaxf(mx, logits[l]);
  mx = block_max(mx, red);
  float se = 0.f;
  for (int l = threadIdx.x; l < nl; l += THREADS) se += expf(logits[l] - mx);
  se = block_sum(se, red);
  for (int l = threadIdx.x; l < nl; l += THREADS) probs[l0 + l] = expf(logits[l] - mx) / se;
}

// RoPE table by position: table[p][i] = (cos, sin)(p * inv_freq[i]) in FP32, the values the reference computes per
// step (`f = positions * inv_freq`, `f.cos()`, `f.sin()`).
__global__ void __launch_bounds__(256) rope_table_kernel(const float* __restrict__ inv_freq, int half, int rows,
                                                        float2* __restrict__ table) {
  pdl_wait();  // the previous kernel on the stream has completed
  pdl_trigger();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)rows * half) return;
  const int p = (int)(i / half), f = (int)(i % half);
  float sn, cs;
  sincosf((float)p * inv_freq[f], &sn, &cs);
  table[i] = make_float2(cs, sn);
}

}  // namespace rows

// ---------------------------------------------------------------------------------------------------------------
// host: errors
// ---------------------------------------------------------------------------------------------------------------
static thread_local std::string t_last_error;

int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(MORJ_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
  return MORJ_OK;
}

}  // namespace morj

using namespace morj;


extern "C" int morj_version(void) { return 100; }

extern "C" const char* morj_last_error(void) { return t_last_error.c_str(); }

extern "C" int morj_device_error(int* code, int clear, void* stream) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_device_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return set_error(MORJ_ERR_CUDA, "morj_device_error: %s", cudaGetErrorString(e));
  if (code) *code = v;
  if (clear && v) {
    static const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_device_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return set_error(MORJ_ERR_CUDA, "morj_device_error: %s", cudaGetErrorString(e));
  }
  return MORJ_OK;
}

extern "C" int morj_embed_rmsnorm(const int* tokens, const int* feature_row, const void* features, const void* embed,
                                  int n, int H, float scale, const void* norm_w, float eps, void* x_out, void* h_out,
                                  void* stream) {
  if (n == 0) return MORJ_OK;
  if (!tokens || !embed || !norm_w || !x_out || !h_out || n < 0 || H <= 0 || H % 8 || (feature_row && !features))
    return set_error(MORJ_ERR_ARG, "morj_embed_rmsnorm: bad arguments (n=%d H=%d)", n, H);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int st = MORJ_OK;
  MORJ_VPT_SWITCH(H, (st = launch_pdl("embed_rmsnorm_kernel", rows::embed_rmsnorm_kernel<V>, dim3(n),
                                      dim3(rows::THREADS), 0, s, tokens, feature_row,
                                      (const __nv_bfloat16*)features, (const __nv_bfloat16*)embed, H, scale,
                                      (const __nv_bfloat16*)norm_w, eps, (__nv_bfloat16*)x_out,
                                      (__nv_bfloat16*)h_out)));
  return st;
}

extern "C" int morj_attn_epilogue(const void* o, void* x, void* h_out, const void* w_post, const void* w_pre, int n,
                                  int H, float eps, void* stream) {
  if (n == 0) return MORJ_OK;
  if (!o || !x || !h_out || !w_post || !w_pre || n < 0 || H <= 0 || H % 8)
    return set_error(MORJ_ERR_ARG, "morj_attn_epilogue: bad arguments (n=%d H=%d)", n, H);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int st = MORJ_OK;
  MORJ_VPT_SWITCH(H, (st = launch_pdl("attn_epilogue_kernel", rows::attn_epilogue_kernel<V>, dim3(n),
                                      dim3(rows::THREADS), 0, s, (const __nv_bfloat16*)o, (__nv_bfloat16*)x,
                                      (__nv_bfloat16*)h_out, (const __nv_bfloat16*)w_post,
                                      (const __nv_bfloat16*)w_pre, H, eps)));
  return st;
}

extern "C" int morj_mlp_epilogue(const void* d, void* x, void* h_out, const void* w_post, const void* scalar,
                                 const void* w_next, int n, int H, float eps, int has_next, void* stream) {
  if (n == 0) return MORJ_OK;
  if (!d || !x || !w_post || !scalar || n < 0 || H <= 0 || H % 8 || (has_next && (!h_out || !w_next)))
    return set_error(MORJ_ERR_ARG, "morj_mlp_epilogue: bad arguments (n=%d H=%d)", n, H);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int st = MORJ_OK;
  MORJ_VPT_SWITCH(H, (st = launch_pdl("mlp_epilogue_kernel", rows::mlp_epilogue_kernel<V>, dim3(n),
                                      dim3(rows::THREADS), 0, s, (const __nv_bfloat16*)d, (__nv_bfloat16*)x,
                                      (__nv_bfloat16*)h_out, (const __nv_bfloat16*)w_post,
                                      (const __nv_bfloat16*)scalar, (const __nv_bfloat16*)w_next, H, eps,
                                      has_next)));
  return st;
}

extern "C" int morj_rope_table(const float* inv_freq, int half, int rows, void* table, void* stream) {
  if (rows == 0) return MORJ_OK;
  if (!inv_freq || !table || half <= 0 || half % 2 || rows < 0)
    return set_error(MORJ_ERR_ARG, "morj_rope_table: bad arguments (half=%d rows=%d)", half, rows);
  if (reinterpret_cast<uintptr_t>(table) & 15)
    return set_error(MORJ_ERR_ARG, "morj_rope_table: table must be 16-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const long long n = (long long)rows * half;
  return launch_pdl("rope_table_kernel", rows::rope_table_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s,
                    inv_freq, half, rows, reinterpret_cast<float2*>(table));
}

extern "C" int morj_qkv_post(const void* qkv, long long ld, int n, int hq, int hk, int has_v, int d,
                             const void* q_norm, const void* k_norm, const int* positions, const float* inv_freq,
                             const int* slots, float eps, void* q_out, void* k_pool, void* v_pool, void* stream) {
  if (n == 0 || hq + hk == 0) return MORJ_OK;
  if (!qkv || !positions || !inv_freq || n < 0 || hq < 0 || hk < 0 || (hq && (!q_out || !q_norm)) ||
      (hk && (!k_pool || !v_pool || !slots || !k_norm)))
    return set_error(MORJ_ERR_ARG, "morj_qkv_post: bad arguments");
  const int heads = hq + 2 * hk;
  const long long need = (long long)(hq + (has_v ? 2 : 1) * hk) * d;
  if (ld < need) return set_error(MORJ_ERR_ARG, "morj_qkv_post: leading dimension %lld < %lld", ld, need);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  dim3 grid(n, (heads + 7) / 8);
#define MORJ_QKV(DD)                                                                                             \
  launch_pdl("qkv_post_kernel", rows::qkv_post_kernel<DD>, grid, dim3(rows::THREADS), 0, s,                      \
             (const __nv_bfloat16*)qkv, ld, hq, hk, has_v, (const __nv_bfloat16*)q_norm,                          \
             (const __nv_bfloat16*)k_norm, positions, inv_freq, slots, eps, (__nv_bfloat16*)q_out,                \
             (__nv_bfloat16*)k_pool, (__nv_bfloat16*)v_pool)
  if (d == 64) return MORJ_QKV(64);
  if (d == 128) return MORJ_QKV(128);
  if (d == 256) return MORJ_QKV(256);
#undef MORJ_QKV
  return set_error(MORJ_ERR_UNSUPPORTED, "morj_qkv_post: head_dim %d unsupported", d);
}

extern "C" int morj_geglu(const void* gu, int n, int F, void* out, void* stream) {
  if (n == 0) return MORJ_OK;
  if (!gu || !out || n < 0 || F <= 0 || F % 8) return set_error(MORJ_ERR_ARG, "morj_geglu: bad arguments");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  dim3 grid((F / 8 + 255) / 256, n);
  return launch_pdl("geglu_kernel", rows::geglu_kernel, grid, dim3(256), 0, s, (const __nv_bfloat16*)gu, F,
                    (__nv_bfloat16*)out);
}

static int copy_rows(const void* src, long long ld_src, const int* rows_, int n, int width, void* dst,
                     long long ld_dst, void* stream, int scatter) {
  if (n == 0) return MORJ_OK;
  if (!src || !dst || !rows_ || n < 0 || width <= 0 || width % 8 || ld_src % 8 || ld_dst % 8 || ld_src < width ||
      ld_dst < width)
    return set_error(MORJ_ERR_ARG, "morj row copy: bad arguments (n=%d width=%d)", n, width);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int threads = width / 8 < 256 ? ((width / 8 + 31) / 32) * 32 : 256;
  return launch_pdl("copy_rows_kernel", rows::copy_rows_kernel, dim3(n), dim3(threads), 0, s,
                    (const __nv_bfloat16*)src, ld_src, rows_, width, (__nv_bfloat16*)dst, ld_dst, scatter);
}

extern "C" int morj_gather_rows(const void* src, long long ld_src, const int* rows_, int n, int width, void* dst,
                                long long ld_dst, void* stream) {
  return copy_rows(src, ld_src, rows_, n, width, dst, ld_dst, stream, 0);
}

extern "C" int morj_scatter_rows(const void* src, long long ld_src, const int* rows_, int n, int width, void* dst,
                                 long long ld_dst, void* stream) {
  return copy_rows(src, ld_src, rows_, n, width, dst, ld_dst, stream, 1);
}

extern "C" int morj_label_head(const void* x, long long ld_x, const int* seq_row, const int* label_indptr,
                               const int* label_ids, int n_seq, const void* norm_w, const void* embed, int H,
                               float eps, float softcap, float* probs, void* stream) {
  if (n_seq == 0) return MORJ_OK;
  if (!x || !seq_row || !label_indptr || !label_ids || !norm_w || !embed || !probs || n_seq < 0 || H <= 0 || H % 8)
    return set_error(MORJ_ERR_ARG, "morj_label_head: bad arguments");
  constexpr int kMaxLabels = 8192;
  const size_t smem = (size_t)(H + kMaxLabels) * sizeof(float);
  if (smem > 200 * 1024) return set_error(MORJ_ERR_UNSUPPORTED, "morj_label_head: hidden size %d too large", H);
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(rows::label_head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         200 * 1024);
    if (e != cudaSuccess) return set_error(MORJ_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    configured = true;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return launch_pdl("label_head_kernel", rows::label_head_kernel, dim3(n_seq), dim3(rows::THREADS), smem, s,
                    (const __nv_bfloat16*)x, ld_x, seq_row, label_indptr, label_ids, (const __nv_bfloat16*)norm_w,
                    (const __nv_bfloat16*)embed, H, eps, softcap, probs);
}
