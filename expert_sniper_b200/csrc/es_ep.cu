// Expert-parallel helpers: per-destination routing masks and the fixed-order
// sum of per-owner partials.
//
// The reference's Expert Network broadcasts each layer's request to every
// node; a node masks the top-k weights to its own partition and returns a
// partial (src/expert_network/node.py:142-172), and the driver sums the
// partials in fixed node order in fp32 (src/expert_network/reader.py:
// 278-286). Here the home GPU computes each destination's mask once
// (es_ep_mask), the owners run es_moe_expert_ffn on the rows they receive,
// and es_ep_combine adds the returned partials in rank order.
#include "es_common.cuh"
#include "es_kernels.cuh"
#include "es_moe.h"

namespace es {
namespace {

// one thread per (destination, token, slot)
__global__ void ep_mask_kernel(const int32_t* idx, const float* w, const int32_t* owner,
                               const int32_t* local_id, int E, int k, int T, int world,
                               int32_t* send_idx, float* send_w, uint32_t* err) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long total = (long long)world * T * k;
  pdl_wait();
  pdl_trigger();
  if (i >= total) return;
  const int d = (int)(i / ((long long)T * k));
  const long long tj = i - (long long)d * T * k;
  const int e = idx[tj];
  int l = -1;
  if (e >= 0 && e < E) {
    if (owner[e] == d) l = local_id[e];
  } else if (e != -1) {
    set_error(err, 0x1u);
  }
  send_idx[i] = l;
  send_w[i] = w[tj];
}

// out[t][c] = sum over ranks r in order of partials[r][t][c] (+ extra[t][c])
__global__ void ep_combine_kernel(const float* partials, const float* extra, int world, int T,
                                  int D, void* out, int out_f32) {
  const long long i4 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  const long long n = (long long)T * D;
  pdl_wait();
  pdl_trigger();
  if (i4 >= n) return;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int r = 0; r < world; ++r) {
    const float4 p = *reinterpret_cast<const float4*>(partials + (size_t)r * n + i4);
    acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
  }
  if (extra) {
    const float4 p = *reinterpret_cast<const float4*>(extra + i4);
    acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
  }
  if (out_f32) {
    *reinterpret_cast<float4*>(static_cast<float*>(out) + i4) = acc;
  } else {
    const uint32_t lo = (uint32_t)float_to_bf16_bits(acc.x) | ((uint32_t)float_to_bf16_bits(acc.y) << 16);
    const uint32_t hi = (uint32_t)float_to_bf16_bits(acc.z) | ((uint32_t)float_to_bf16_bits(acc.w) << 16);
    *reinterpret_cast<uint2*>(static_cast<uint16_t*>(out) + i4) = make_uint2(lo, hi);
  }
}

}  // namespace
}  // namespace es

extern "C" {

es_status es_ep_mask(const int32_t* topk_idx, const float* topk_w, const int32_t* owner,
                     const int32_t* local_id, int32_t num_experts, int32_t top_k, int32_t T,
                     int32_t world, int32_t* send_idx, float* send_w, void* workspace,
                     es_stream_t stream) {
  if (T < 0 || world < 1 || top_k < 1 || top_k > 16 || num_experts < 1) return ES_ERR_INVALID_ARG;
  if (T == 0) return ES_OK;
  if (!topk_idx || !topk_w || !owner || !local_id || !send_idx || !send_w) return ES_ERR_INVALID_ARG;
  const long long total = (long long)world * T * top_k;
  const int threads = 256;
  const long long blocks = (total + threads - 1) / threads;
  if (blocks > 0x7fffffffLL) return ES_ERR_UNSUPPORTED;
  uint32_t* err = static_cast<uint32_t*>(workspace);  // error word at offset 0, or NULL
  return es::launch_pdl(es::ep_mask_kernel, dim3((unsigned)blocks), dim3(threads), 0,
                        static_cast<cudaStream_t>(stream), topk_idx, topk_w, owner, local_id,
                        (int)num_experts, (int)top_k, (int)T, (int)world, send_idx, send_w, err) ==
                 cudaSuccess
             ? ES_OK
             : ES_ERR_CUDA;
}

es_status es_ep_combine(const float* partials, const float* extra, int32_t world, int32_t T,
                        int32_t D, void* out, int32_t out_dtype, es_stream_t stream) {
  if (world < 1 || T < 0 || D <= 0 || D % 4) return ES_ERR_INVALID_ARG;
  if (out_dtype != ES_DTYPE_BF16 && out_dtype != ES_DTYPE_F32) return ES_ERR_UNSUPPORTED;
  if (T == 0) return ES_OK;
  if (!partials || !out) return ES_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(partials) | reinterpret_cast<uintptr_t>(out) |
       reinterpret_cast<uintptr_t>(extra)) % 16)
    return ES_ERR_INVALID_ARG;
  const long long n4 = (long long)T * D / 4;
  const int threads = 256;
  const long long blocks = (n4 + threads - 1) / threads;
  return es::launch_pdl(es::ep_combine_kernel, dim3((unsigned)blocks), dim3(threads), 0,
                        static_cast<cudaStream_t>(stream), partials, extra, (int)world, (int)T,
                        (int)D, out, out_dtype == ES_DTYPE_F32 ? 1 : 0) == cudaSuccess
             ? ES_OK
             : ES_ERR_CUDA;
}

}  // extern "C"
