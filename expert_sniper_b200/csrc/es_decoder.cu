// Caller-side helpers for the decoder around the MoE block (the per-layer
// loop of src/mlx_expert_sniper/generate.py:114-122): fused residual add +
// RMS norm, the per-head q/k RMS norm + rotary embedding + KV-cache write of
// Qwen3 attention, and a weight-streaming GEMV for the projections at batch
// 1-4. Plain kernels in fp32 arithmetic on bf16 tensors; no counterpart in
// the reference beyond the MLX ops they replace. All are launched as
// programmatic dependents (each waits for the kernel before it, then lets
// the next one launch), so a chain of them overlaps launch and ramp-up.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "es_common.cuh"
#include "es_kernels.cuh"
#include "es_moe.h"

namespace {

using es::launch_pdl;
using es::pdl_trigger;
using es::pdl_wait;

__device__ __forceinline__ float bf(uint16_t v) { return __uint_as_float((uint32_t)v << 16); }
__device__ __forceinline__ uint16_t to_bf(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

__device__ __forceinline__ float block_sum(float v, float* s_warp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) s_warp[warp] = v;
  __syncthreads();
  float t = 0.f;
  const int nw = (blockDim.x + 31) >> 5;
  for (int i = 0; i < nw; ++i) t += s_warp[i];
  __syncthreads();
  return t;
}

// one block per row: h += delta (if any); out = h * rsqrt(mean(h^2) + eps) * w.
// Each thread takes 8-column chunks (16-byte loads) and keeps the rounded
// residual of up to kNormChunks chunks in registers, so nothing is read back
// from memory between the update and the norm.
constexpr int kNormChunks = 4;
__global__ void add_rmsnorm_kernel(uint16_t* h, const uint16_t* delta, const uint16_t* w,
                                   uint16_t* out, int cols, float eps) {
  __shared__ float s_warp[32];
  pdl_trigger();
  pdl_wait();
  const size_t base = (size_t)blockIdx.x * cols;
  const int n8 = cols / 8;
  float r[kNormChunks][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kNormChunks; ++j) {
    const int c8 = threadIdx.x + j * blockDim.x;
    if (c8 < n8) {
      const uint4 hv = *reinterpret_cast<const uint4*>(h + base + (size_t)c8 * 8);
      const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
      uint32_t dw[4] = {0u, 0u, 0u, 0u};
      if (delta) {
        const uint4 dv = *reinterpret_cast<const uint4*>(delta + base + (size_t)c8 * 8);
        dw[0] = dv.x; dw[1] = dv.y; dw[2] = dv.z; dw[3] = dv.w;
      }
      uint32_t ow[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float lo = bf((uint16_t)(hw[q] & 0xffffu)), hi = bf((uint16_t)(hw[q] >> 16));
        if (delta) {
          // the residual stream stays bf16, as the model's
          lo = bf(to_bf(lo + bf((uint16_t)(dw[q] & 0xffffu))));
          hi = bf(to_bf(hi + bf((uint16_t)(dw[q] >> 16))));
        }
        r[j][2 * q] = lo;
        r[j][2 * q + 1] = hi;
        ss += lo * lo + hi * hi;
        ow[q] = (uint32_t)to_bf(lo) | ((uint32_t)to_bf(hi) << 16);
      }
      if (delta)
        *reinterpret_cast<uint4*>(h + base + (size_t)c8 * 8) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    }
  }
  const float rs = rsqrtf(block_sum(ss, s_warp) / cols + eps);
#pragma unroll
  for (int j = 0; j < kNormChunks; ++j) {
    const int c8 = threadIdx.x + j * blockDim.x;
    if (c8 < n8) {
      const uint4 wv = *reinterpret_cast<const uint4*>(w + (size_t)c8 * 8);
      const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t ow[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float o0 = r[j][2 * q] * rs * bf((uint16_t)(ww[q] & 0xffffu));
        const float o1 = r[j][2 * q + 1] * rs * bf((uint16_t)(ww[q] >> 16));
        ow[q] = (uint32_t)to_bf(o0) | ((uint32_t)to_bf(o1) << 16);
      }
      *reinterpret_cast<uint4*>(out + base + (size_t)c8 * 8) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    }
  }
}

// the same for rows that the vector form does not take (cols % 8, unaligned
// or longer than kNormChunks chunks per thread): scalar, two passes
__global__ void add_rmsnorm_scalar_kernel(uint16_t* h, const uint16_t* delta, const uint16_t* w,
                                          uint16_t* out, int cols, float eps) {
  __shared__ float s_warp[32];
  pdl_trigger();
  pdl_wait();
  const size_t base = (size_t)blockIdx.x * cols;
  float ss = 0.f;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    float v = bf(h[base + c]);
    if (delta) {
      v = bf(to_bf(v + bf(delta[base + c])));
      h[base + c] = to_bf(v);
    }
    ss += v * v;
  }
  const float r = rsqrtf(block_sum(ss, s_warp) / cols + eps);
  __syncthreads();
  for (int c = threadIdx.x; c < cols; c += blockDim.x)
    out[base + c] = to_bf(bf(h[base + c]) * r * bf(w[c]));
}

// one warp per (token, head) of the fused projection output
// qkv [B, (H + 2 KV) * hd]: RMS norm over hd (q and k heads), rotary on the
// two halves, q -> q_out [B, H, hd]; k, v -> caches [B, KV, max_ctx, hd] at
// position *pos
__global__ void qk_norm_rope_kv_kernel(const uint16_t* qkv, const uint16_t* qn, const uint16_t* kn,
                                       const float* cos_t, const float* sin_t, const int64_t* pos,
                                       uint16_t* q_out, uint16_t* kc, uint16_t* vc, int B, int H,
                                       int KV, int hd, int max_ctx, float eps) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int heads = H + 2 * KV;
  if (item >= B * heads) return;
  const int b = item / heads, hh = item - b * heads;
  const long long pl = *pos;
  if (pl < 0 || pl >= max_ctx) return;  // outside the cache: nothing written
  const int p = (int)pl;
  const uint16_t* src = qkv + (size_t)b * heads * hd + (size_t)hh * hd;
  const int half = hd >> 1;
  if (hh >= H + KV) {  // v head: copy into the cache
    const int kvh = hh - H - KV;
    uint16_t* dst = vc + (((size_t)b * KV + kvh) * max_ctx + p) * hd;
    for (int i = lane; i < hd; i += 32) dst[i] = src[i];
    return;
  }
  float ss = 0.f;
  for (int i = lane; i < hd; i += 32) {
    const float v = bf(src[i]);
    ss += v * v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(ss / hd + eps);
  const uint16_t* nw = hh < H ? qn : kn;
  uint16_t* dst = hh < H ? q_out + ((size_t)b * H + hh) * hd
                         : kc + (((size_t)b * KV + (hh - H)) * max_ctx + p) * hd;
  const float* cs = cos_t + (size_t)p * half;
  const float* sn = sin_t + (size_t)p * half;
  for (int i = lane; i < half; i += 32) {
    // round to bf16 after the norm, as the unfused path does
    const float x1 = bf(to_bf(bf(src[i]) * r * bf(nw[i])));
    const float x2 = bf(to_bf(bf(src[i + half]) * r * bf(nw[i + half])));
    dst[i] = to_bf(x1 * cs[i] - x2 * sn[i]);
    dst[i + half] = to_bf(x2 * cs[i] + x1 * sn[i]);
  }
}

// y[b][n] = sum_k W[n][k] x[b][k] for a few vectors (B <= kGemvMaxB): the
// weight-streaming shape of a decode step at batch 1-4. One warp per
// kGemvRows output rows; each lane reads 16-byte runs of the weight rows
// (coalesced: a warp covers 256 consecutive columns of a row per load),
// kGemvUnroll loads per row in flight, the next batch loading while the
// current one is used; the x vectors sit in shared memory; fp32
// accumulation, one warp reduction per (row, vector). Launched as a
// programmatic dependent: the first weight loads are issued before waiting
// for the kernel that writes x, so they stream while it finishes.
constexpr int kGemvMaxB = 4;
constexpr int kGemvRows = 2;
constexpr int kGemvWarps = 8;
constexpr int kGemvUnroll = 4;

template <int B>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_kernel(const uint16_t* __restrict__ w,
                                                               const uint16_t* __restrict__ x,
                                                               uint16_t* __restrict__ y, int N,
                                                               int K) {
  extern __shared__ uint4 s_x4[];  // [B][K / 8]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int k8 = K / 8;
  const int n0 = (blockIdx.x * kGemvWarps + warp) * kGemvRows;
  uint4 wv[2][kGemvUnroll][kGemvRows];
  auto load = [&](int c0, uint4 (&dst)[kGemvUnroll][kGemvRows]) {
#pragma unroll
    for (int u = 0; u < kGemvUnroll; ++u)
#pragma unroll
      for (int r = 0; r < kGemvRows; ++r) {
        const int c = c0 + 32 * u;
        dst[u][r] = (c < k8 && n0 + r < N)
                        ? __ldcs(reinterpret_cast<const uint4*>(w + (size_t)(n0 + r) * K) + c)
                        : make_uint4(0, 0, 0, 0);
      }
  };
  // weights do not depend on the previous kernel: start them first
  load(lane, wv[0]);
  if (32 * kGemvUnroll < k8) load(lane + 32 * kGemvUnroll, wv[1]);
  pdl_trigger();
  pdl_wait();
  for (int i = threadIdx.x; i < B * k8; i += blockDim.x)
    s_x4[i] = reinterpret_cast<const uint4*>(x)[i];
  __syncthreads();
  if (n0 >= N) return;
  float acc[kGemvRows][B];
#pragma unroll
  for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
    for (int b = 0; b < B; ++b) acc[r][b] = 0.f;
  int cur = 0;
  for (int c0 = lane; c0 < k8; c0 += 32 * kGemvUnroll, cur ^= 1) {
    // the batch after next goes into the buffer this iteration frees
    uint4 wc[kGemvUnroll][kGemvRows];
#pragma unroll
    for (int u = 0; u < kGemvUnroll; ++u)
#pragma unroll
      for (int r = 0; r < kGemvRows; ++r) wc[u][r] = cur ? wv[1][u][r] : wv[0][u][r];
    if (c0 + 64 * kGemvUnroll < k8) {
      if (cur) load(c0 + 64 * kGemvUnroll, wv[1]);
      else load(c0 + 64 * kGemvUnroll, wv[0]);
    }
#pragma unroll
    for (int u = 0; u < kGemvUnroll; ++u) {
      const int c = c0 + 32 * u;
      if (c >= k8) break;
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const uint4 xv = s_x4[b * k8 + c];
        const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int r = 0; r < kGemvRows; ++r) {
          const uint32_t ws[4] = {wc[u][r].x, wc[u][r].y, wc[u][r].z, wc[u][r].w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            acc[r][b] = fmaf(__uint_as_float(ws[q] << 16), __uint_as_float(xs[q] << 16), acc[r][b]);
            acc[r][b] = fmaf(__uint_as_float(ws[q] & 0xffff0000u),
                             __uint_as_float(xs[q] & 0xffff0000u), acc[r][b]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
    for (int b = 0; b < B; ++b) {
      float v = acc[r][b];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0 && n0 + r < N) y[(size_t)b * N + n0 + r] = to_bf(v);
    }
}

template <int B>
cudaError_t launch_gemv(const uint16_t* w, const uint16_t* x, uint16_t* y, int N, int K,
                        cudaStream_t st) {
  const size_t smem = (size_t)B * K * 2;
  if (smem > 48 * 1024) {
    const cudaError_t e =
        cudaFuncSetAttribute(gemv_kernel<B>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  const int rows_per_block = kGemvWarps * kGemvRows;
  return launch_pdl(gemv_kernel<B>, dim3((N + rows_per_block - 1) / rows_per_block),
                    dim3(kGemvWarps * 32), smem, st, w, x, y, N, K);
}

}  // namespace

extern "C" {

es_status es_dec_gemv(const void* weight, const void* x, void* y, int32_t batch, int32_t n,
                      int32_t k, es_stream_t stream) {
  if (!weight || !x || !y || batch < 0 || batch > kGemvMaxB || n <= 0 || k <= 0 || k % 8 ||
      (size_t)batch * k * 2 > 200 * 1024)
    return ES_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(weight) % 16 || reinterpret_cast<uintptr_t>(x) % 16)
    return ES_ERR_INVALID_ARG;
  if (batch == 0) return ES_OK;
  const auto* w = static_cast<const uint16_t*>(weight);
  const auto* xv = static_cast<const uint16_t*>(x);
  auto* yv = static_cast<uint16_t*>(y);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
  switch (batch) {
    case 1: e = launch_gemv<1>(w, xv, yv, n, k, st); break;
    case 2: e = launch_gemv<2>(w, xv, yv, n, k, st); break;
    case 3: e = launch_gemv<3>(w, xv, yv, n, k, st); break;
    default: e = launch_gemv<4>(w, xv, yv, n, k, st); break;
  }
  return e == cudaSuccess ? ES_OK : ES_ERR_CUDA;
}

es_status es_dec_add_rmsnorm(void* h, const void* delta, const void* weight, void* out,
                             int32_t rows, int32_t cols, float eps, es_stream_t stream) {
  if (!h || !weight || !out || rows < 0 || cols <= 0) return ES_ERR_INVALID_ARG;
  if (rows == 0) return ES_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uintptr_t al = reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(delta) |
                       reinterpret_cast<uintptr_t>(weight) | reinterpret_cast<uintptr_t>(out);
  const int n8 = cols / 8;
  // 8-column chunks: a thread per chunk up to 256 threads, up to
  // kNormChunks chunks per thread
  const int threads = std::min(256, ((n8 + 31) / 32) * 32);
  if (cols % 8 == 0 && al % 16 == 0 && n8 <= threads * kNormChunks) {
    if (launch_pdl(add_rmsnorm_kernel, dim3(rows), dim3(threads), 0, st,
                   static_cast<uint16_t*>(h), static_cast<const uint16_t*>(delta),
                   static_cast<const uint16_t*>(weight), static_cast<uint16_t*>(out), cols,
                   eps) != cudaSuccess)
      return ES_ERR_CUDA;
  } else {
    if (launch_pdl(add_rmsnorm_scalar_kernel, dim3(rows), dim3(cols >= 1024 ? 256 : 128), 0, st,
                   static_cast<uint16_t*>(h), static_cast<const uint16_t*>(delta),
                   static_cast<const uint16_t*>(weight), static_cast<uint16_t*>(out), cols,
                   eps) != cudaSuccess)
      return ES_ERR_CUDA;
  }
  return cudaGetLastError() == cudaSuccess ? ES_OK : ES_ERR_CUDA;
}

es_status es_dec_qk_norm_rope_kv(const void* qkv, const void* q_norm, const void* k_norm,
                                 const float* cos_table, const float* sin_table,
                                 const int64_t* pos, void* q_out, void* k_cache, void* v_cache,
                                 int32_t batch, int32_t heads, int32_t kv_heads,
                                 int32_t head_dim, int32_t max_ctx, float eps,
                                 es_stream_t stream) {
  if (!qkv || !q_norm || !k_norm || !cos_table || !sin_table || !pos || !q_out || !k_cache ||
      !v_cache || batch < 0 || heads <= 0 || kv_heads <= 0 || head_dim <= 0 || head_dim % 2 ||
      max_ctx <= 0)
    return ES_ERR_INVALID_ARG;
  if (batch == 0) return ES_OK;
  const int items = batch * (heads + 2 * kv_heads);
  const int warps = 8;
  return launch_pdl(qk_norm_rope_kv_kernel, dim3((items + warps - 1) / warps), dim3(warps * 32), 0,
                    static_cast<cudaStream_t>(stream), static_cast<const uint16_t*>(qkv),
                    static_cast<const uint16_t*>(q_norm), static_cast<const uint16_t*>(k_norm),
                    cos_table, sin_table, pos, static_cast<uint16_t*>(q_out),
                    static_cast<uint16_t*>(k_cache), static_cast<uint16_t*>(v_cache), batch,
                    heads, kv_heads, head_dim, max_ctx, eps) == cudaSuccess
             ? ES_OK
             : ES_ERR_CUDA;
}

}  // extern "C"
