// Combine: out[t] = sum_j w[t,j] * y[t,j] in ascending expert id order, in
// fp32, then + sgate[t] * y_shared[t]; cast to the output dtype.
//
// Restates engine.py:40-41 ((out * top_k_weights[..., None]).sum(axis=-2))
// and the shared-expert add of generate.py:173-178. It is a gather: each
// thread owns four output columns of one token and reads that token's k
// expert rows, so no floating-point atomics are involved and the sum order
// is fixed.
#include "es_common.cuh"
#include "es_kernels.cuh"

namespace es {
namespace {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads) combine_kernel(CombineArgs a) {
  const int t = blockIdx.y;
  const int d = (blockIdx.x * kThreads + threadIdx.x) * 4;
  if (d >= a.D) return;
  const int k = a.k, kk = k + (a.has_shared ? 1 : 0);
  int ids[kMaxTopK];
  int ps[kMaxTopK];
  float ws[kMaxTopK];
  int m = 0;
  for (int j = 0; j < k; ++j) {
    const int e = a.idx[(size_t)t * k + j];
    const int p = a.pos[(size_t)t * kk + j];
    if (e < 0 || p < 0) continue;
    const float w = a.w[(size_t)t * k + j];
    // insertion by expert id; equal ids keep slot order
    int i = m++;
    while (i > 0 && ids[i - 1] > e) {
      ids[i] = ids[i - 1]; ps[i] = ps[i - 1]; ws[i] = ws[i - 1];
      --i;
    }
    ids[i] = e; ps[i] = p; ws[i] = w;
  }
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int i = 0; i < m; ++i) {
    const float4 y = *reinterpret_cast<const float4*>(a.y_pair + (size_t)ps[i] * a.D + d);
    acc.x = fmaf(ws[i], y.x, acc.x);
    acc.y = fmaf(ws[i], y.y, acc.y);
    acc.z = fmaf(ws[i], y.z, acc.z);
    acc.w = fmaf(ws[i], y.w, acc.w);
  }
  if (a.has_shared) {
    const int p = a.pos[(size_t)t * kk + k];
    const float sg = a.sgate[t];
    const float4 y = *reinterpret_cast<const float4*>(a.y_pair + (size_t)p * a.D + d);
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
  combine_kernel<<<grid, kThreads, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace es
