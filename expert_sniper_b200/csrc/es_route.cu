// Router + per-token operand preparation, one warp per token.
//
// Restates src/mlx_expert_sniper/generate.py:122-136: logits (+ additive
// cache bias, fp32) -> softmax in fp32 -> top-k -> optional renormalisation.
// The selection ranks the biased fp32 logits, which orders experts exactly as
// the fp32 softmax does; equal keys go to the lower expert id. The same warp
// also marks each selected expert's token bitmap (the histogram the
// dispatch scans), computes the shared-expert gate, and rewrites the
// token's activation row into fragment order with per-group sums.
#include <math.h>

#include "es_common.cuh"
#include "es_kernels.cuh"

namespace es {
namespace {

constexpr int kRouteWarps = 4;

template <int VPL>
__global__ void __launch_bounds__(kRouteWarps * 32) route_kernel(RouteArgs a) {
  extern __shared__ __align__(16) uint16_t x_stage[];  // [kRouteWarps][D]
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int t = blockIdx.x * kRouteWarps + warp;
  if (t >= a.T) return;  // warp-uniform; only warp-level sync below
  const int E = a.E, k = a.k;

  int my_e = -1;  // lane j < k: expert of slot j
  if (a.logits) {
    float z[VPL];
    uint32_t key[VPL];
    float m = -INFINITY;
    bool nan_seen = false;
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      const int e = v * 32 + lane;
      float l = -INFINITY;
      if (e < E) {
        l = a.logits_f32 ? static_cast<const float*>(a.logits)[(size_t)t * E + e]
                         : bf16_bits_to_float(static_cast<const uint16_t*>(a.logits)[(size_t)t * E + e]);
        if (a.bias) l += a.bias[e];
        if (l != l) nan_seen = true; else m = fmaxf(m, l);
      }
      z[v] = l;
      key[v] = (e < E) ? ((l != l) ? 1u : float_key(l)) : 0u;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(full, m, o));
    float s = 0.f;
#pragma unroll
    for (int v = 0; v < VPL; ++v)
      if (v * 32 + lane < E && z[v] == z[v]) s += expf(z[v] - m);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(full, s, o);
    if (__any_sync(full, nan_seen) && lane == 0) set_error(a.err, 0x2u);

    float sel_w[kMaxTopK];
    int sel_e[kMaxTopK];
#pragma unroll
    for (int j = 0; j < kMaxTopK; ++j) {
      sel_e[j] = -1;
      sel_w[j] = 0.f;
      if (j < k) {
        uint32_t bk = 0u;
        int be = 0x7fffffff;
#pragma unroll
        for (int v = 0; v < VPL; ++v)
          if (key[v] > bk) { bk = key[v]; be = v * 32 + lane; }
        const uint32_t mk = __reduce_max_sync(full, bk);
        const unsigned cand = (bk == mk && bk != 0u) ? static_cast<unsigned>(be) : 0xffffffffu;
        const unsigned we = __reduce_min_sync(full, cand);
        float zv = 0.f;
#pragma unroll
        for (int v = 0; v < VPL; ++v)
          if (v * 32 + lane == static_cast<int>(we)) { zv = z[v]; key[v] = 0u; }
        zv = __shfl_sync(full, zv, we & 31);
        sel_e[j] = static_cast<int>(we);
        sel_w[j] = expf(zv - m) / s;
      }
    }
    if (a.renorm) {
      float tot = 0.f;
#pragma unroll
      for (int j = 0; j < kMaxTopK; ++j) if (j < k) tot += sel_w[j];
#pragma unroll
      for (int j = 0; j < kMaxTopK; ++j) sel_w[j] = sel_w[j] / tot;
    }
#pragma unroll
    for (int j = 0; j < kMaxTopK; ++j) {
      if (j < k && lane == j) {
        my_e = sel_e[j];
        if (a.out_idx) a.out_idx[(size_t)t * k + j] = sel_e[j];
        if (a.out_w) a.out_w[(size_t)t * k + j] = sel_w[j];
      }
    }
  } else if (a.in_idx) {
    if (lane < k) {
      my_e = a.in_idx[(size_t)t * k + lane];
      if (my_e < -1 || my_e >= E) {
        set_error(a.err, 0x1u);
        my_e = -1;
      }
    }
  }

  // histogram: token bitmap per expert (order-free, deterministic)
  if (a.bitmap) {
    const uint32_t bit = 1u << (t & 31);
    if (lane < k && my_e >= 0) atomicOr(&a.bitmap[(size_t)my_e * a.W + (t >> 5)], bit);
    if (a.has_shared && lane == 0) atomicOr(&a.bitmap[(size_t)E * a.W + (t >> 5)], bit);
  }

  if (!a.x) return;
  const int D = a.D;
  const uint16_t* xrow = a.x + (size_t)t * D;

  // shared-expert gate: sigmoid(x . w) (generate.py:173-178)
  if (a.has_shared && a.sgate) {
    float dot = 0.f;
    if (a.sg_w) {
      const uint32_t* x2 = reinterpret_cast<const uint32_t*>(xrow);
      const uint32_t* w2 = reinterpret_cast<const uint32_t*>(a.sg_w);
      for (int i = lane; i < D / 2; i += 32) {
        const uint32_t xv = x2[i], wv = w2[i];
        dot = fmaf(bf16_bits_to_float(xv & 0xffffu), bf16_bits_to_float(wv & 0xffffu), dot);
        dot = fmaf(bf16_bits_to_float(xv >> 16), bf16_bits_to_float(wv >> 16), dot);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(full, dot, o);
    }
    if (lane == 0) a.sgate[t] = a.sg_w ? 1.f / (1.f + expf(-dot)) : 1.f;
  }

  // activation row -> fragment order + per-group sums
  if (a.x_perm) {
    uint16_t* xs = x_stage + (size_t)warp * D;
    const uint4* src = reinterpret_cast<const uint4*>(xrow);
    for (int i = lane; i < D / 8; i += 32) reinterpret_cast<uint4*>(xs)[i] = src[i];
    __syncwarp();
    uint16_t* dst_row = a.x_perm + (size_t)t * D;
    for (int q = lane; q < D / 16; q += 32) {
      uint32_t wv[8];
#pragma unroll
      for (int w2 = 0; w2 < 8; ++w2) {
        const int s = w2 >> 1, slot = 2 * (w2 & 1);
        const uint32_t lo = xs[16 * q + s + 4 * slot];
        const uint32_t hi = xs[16 * q + s + 4 * (slot + 1)];
        wv[w2] = lo | (hi << 16);
      }
      uint4* d4 = reinterpret_cast<uint4*>(dst_row + 16 * q);
      d4[0] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
      d4[1] = make_uint4(wv[4], wv[5], wv[6], wv[7]);
    }
    const int GD = D / kGroup;
    for (int G = lane; G < GD; G += 32) {
      float sum = 0.f;
      for (int i = 0; i < kGroup; ++i) sum += bf16_bits_to_float(xs[G * kGroup + i]);
      a.xsum[(size_t)t * GD + G] = sum;
    }
  }
}

template <int VPL>
cudaError_t launch_vpl(const RouteArgs& a, cudaStream_t st) {
  const int blocks = (a.T + kRouteWarps - 1) / kRouteWarps;
  const size_t smem = a.x_perm ? (size_t)kRouteWarps * a.D * sizeof(uint16_t) : 0;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(route_kernel<VPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  route_kernel<VPL><<<blocks, kRouteWarps * 32, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_route(const RouteArgs& a, cudaStream_t st) {
  if (a.T <= 0) return cudaSuccess;
  const int vpl = (a.E + 31) / 32;
  if (vpl <= 1) return launch_vpl<1>(a, st);
  if (vpl <= 2) return launch_vpl<2>(a, st);
  if (vpl <= 4) return launch_vpl<4>(a, st);
  if (vpl <= 8) return launch_vpl<8>(a, st);
  if (vpl <= 16) return launch_vpl<16>(a, st);
  return launch_vpl<32>(a, st);
}

}  // namespace es
