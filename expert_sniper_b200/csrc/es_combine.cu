// Combine: out[t] = sum_j w[t,j] * y[t,j] in ascending expert id order, in
// fp32, then + sgate[t] * y_shared[t]; cast to the output dtype. The
// per-pair rows y are fp32 (decode kernels) or fp16 (tensor-core path).
//
// Restates engine.py:40-41 ((out * top_k_weights[..., None]).sum(axis=-2))
// and the shared-expert add of generate.py:173-178. It is a gather: each
// thread owns four output columns of one token and reads that token's k
// expert rows in the expert-id order the dispatch recorded, so no
// floating-point atomics are involved and the sum order is fixed.
#include "es_common.cuh"
#include "es_kernels.cuh"

namespace es {
namespace {

constexpr int kThreads = 256;

ES_DEV float4 load_row4(const void* y, bool y_f16, size_t off) {
  if (y_f16) {
    const uint2 v = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(y) + off);
    return make_float4(lo_half_f(v.x), hi_half_f(v.x), lo_half_f(v.y), hi_half_f(v.y));
  }
  return *reinterpret_cast<const float4*>(static_cast<const float*>(y) + off);
}

template <bool kYF16>
__global__ void __launch_bounds__(kThreads) combine_kernel(CombineArgs a) {
  const int t = blockIdx.y;
  const int d = (blockIdx.x * kThreads + threadIdx.x) * 4;
  pdl_wait();
  pdl_trigger();
  if (d >= a.D) return;
  const int k = a.k;
  // all slot loads first, then all row loads, then the fixed-order sum: the
  // row loads are independent, so they overlap instead of forming a chain
  int ps[kMaxTopK];
  float ws[kMaxTopK];
#pragma unroll
  for (int r = 0; r < kMaxTopK; ++r) {
    ps[r] = r < k ? a.cs_pos[(size_t)t * k + r] : -1;
    ws[r] = r < k ? a.cs_w[(size_t)t * k + r] : 0.f;
  }
  float4 ys[kMaxTopK];
#pragma unroll
  for (int r = 0; r < kMaxTopK; ++r)
    ys[r] = ps[r] >= 0 ? load_row4(a.y_pair, kYF16, (size_t)ps[r] * a.D + d)
                       : make_float4(0.f, 0.f, 0.f, 0.f);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int r = 0; r < kMaxTopK; ++r) {
    if (ps[r] < 0) continue;  // masked slots (sorted last) add nothing
    acc.x = fmaf(ws[r], ys[r].x, acc.x);
    acc.y = fmaf(ws[r], ys[r].y, acc.y);
    acc.z = fmaf(ws[r], ys[r].z, acc.z);
    acc.w = fmaf(ws[r], ys[r].w, acc.w);
  }
  if (a.has_shared) {
    const int p = a.pos_shared[t];
    const float sg = a.sgate[t];
    const float4 y = load_row4(a.y_pair, kYF16, (size_t)p * a.D + d);
    acc.x = fmaf(sg, y.x, acc.x);
    acc.y = fmaf(sg, y.y, acc.y);
    acc.z = fmaf(sg, y.z, acc.z);
    acc.w = fmaf(sg, y.w, acc.w);
  }
  if (a.out_f32) {
    *reinterpret_cast<float4*>(static_cast<float*>(a.out) + (size_t)t * a.D + d) = acc;
  } else {
    const uint32_t lo = (uint32_t)float_to_bf16_bits(acc.x) | ((uint32_t)float_to_bf16_bits(acc.y) << 16);
    const uint32_t hi = (uint32_t)float_to_bf16_bits(acc.z) | ((uint32_t)float_to_bf16_bits(acc.w) << 16);
    *reinterpret_cast<uint2*>(static_cast<uint16_t*>(a.out) + (size_t)t * a.D + d) = make_uint2(lo, hi);
  }
}

}  // namespace

cudaError_t launch_combine(const CombineArgs& a, cudaStream_t st) {
  if (a.T <= 0) return cudaSuccess;
  dim3 grid((a.D / 4 + kThreads - 1) / kThreads, a.T);
  if (a.y_f16) return launch_pdl(combine_kernel<true>, grid, dim3(kThreads), 0, st, a);
  return launch_pdl(combine_kernel<false>, grid, dim3(kThreads), 0, st, a);
}

}  // namespace es
