// Per-token router, one warp per token (shared by the multi-block router and
// the single-CTA decode front end).
//
// Restates src/mlx_expert_sniper/generate.py:122-136: logits (+ additive
// cache bias, fp32) -> softmax in fp32 -> top-k -> optional renormalisation.
// Selection ranks the biased fp32 logits, which orders experts exactly as the
// fp32 softmax does; equal keys go to the lower expert id. Slot j (descending
// probability) ends up in lane j: (my_e, my_w). The loops over the k rounds
// are kept rolled so the kernel code stays small (these kernels run once per
// step and pay for every instruction-cache miss).
#pragma once

#include <math.h>

#include "es_common.cuh"

namespace es {

template <int VPL>
ES_DEV void route_token_warp(const void* logits, int logits_f32, const float* bias, int t, int E,
                             int k, int renorm, uint32_t* err, int& my_e, float& my_w) {
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  float z[VPL];
  uint32_t key[VPL];
  float m = -INFINITY;
  bool nan_seen = false;
#pragma unroll
  for (int v = 0; v < VPL; ++v) {
    const int e = v * 32 + lane;
    float l = -INFINITY;
    if (e < E) {
      l = logits_f32 ? static_cast<const float*>(logits)[(size_t)t * E + e]
                     : bf16_bits_to_float(static_cast<const uint16_t*>(logits)[(size_t)t * E + e]);
      if (bias) l += bias[e];
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
  if (__any_sync(full, nan_seen) && lane == 0) set_error(err, 0x2u);

  float my_z = -INFINITY;
  my_e = -1;
#pragma unroll 1
  for (int j = 0; j < k; ++j) {
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
    if (lane == j) { my_e = static_cast<int>(we); my_z = zv; }
  }
  my_w = lane < k ? expf(my_z - m) / s : 0.f;
  if (renorm) {
    float tot = my_w;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(full, tot, o);
    my_w = my_w / tot;
  }
}

// One 8-element chunk of an activation row -> fragment order (see
// es_layout.h): e[s] and e[s + 4] form word 2s + half of the 16-element
// chunk. Returns the chunk's sum.
ES_DEV float permute_chunk8(const uint16_t* x_row, uint16_t* perm_row, int q8, bool live) {
  uint4 v = make_uint4(0, 0, 0, 0);
  if (live) v = *reinterpret_cast<const uint4*>(x_row + q8 * 8);
  const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    sum += bf16_bits_to_float(w4[i] & 0xffffu) + bf16_bits_to_float(w4[i] >> 16);
  if (live) {
    const int half = q8 & 1, q = q8 >> 1;
    uint32_t* dst = reinterpret_cast<uint32_t*>(perm_row + 16 * q);
#pragma unroll
    for (int s2 = 0; s2 < 4; ++s2) {
      const uint32_t lo = (w4[s2 >> 1] >> (16 * (s2 & 1))) & 0xffffu;
      const uint32_t hi = (w4[(s2 + 4) >> 1] >> (16 * (s2 & 1))) & 0xffffu;
      dst[2 * s2 + half] = lo | (hi << 16);
    }
  }
  return sum;
}

// sigmoid(x . w) of one token, one warp (generate.py:173-178).
ES_DEV float shared_gate_warp(const uint16_t* xrow, const uint16_t* w, int D, bool x_f16 = false) {
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  if (!w) return 1.f;
  const uint32_t* x2 = reinterpret_cast<const uint32_t*>(xrow);
  const uint32_t* w2 = reinterpret_cast<const uint32_t*>(w);
  float dot = 0.f;
  for (int i = lane; i < D / 2; i += 32) {
    const uint32_t xv = x2[i], wv = w2[i];
    const float x0 = x_f16 ? half_bits_to_float(xv & 0xffffu) : bf16_bits_to_float(xv & 0xffffu);
    const float x1 = x_f16 ? half_bits_to_float(xv >> 16) : bf16_bits_to_float(xv >> 16);
    dot = fmaf(x0, bf16_bits_to_float(wv & 0xffffu), dot);
    dot = fmaf(x1, bf16_bits_to_float(wv >> 16), dot);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(full, dot, o);
  return 1.f / (1.f + expf(-dot));
}

// Slot order of one token for the combine: lane j < k holds expert e (or -1)
// and weight w; writes the token's slots sorted by expert id (masked last),
// the id in cs_pos (turned into a pair index by the dispatch) and the weight
// in cs_w. Returns the lane's slot (-1 for lanes >= k).
ES_DEV int sort_slots_warp(int32_t* cs_pos, float* cs_w, int k, int t, int e, float w) {
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const bool valid = lane < k && e >= 0;
  int rank = 0, nvalid = 0, ninv_before = 0;
  for (int j2 = 0; j2 < k; ++j2) {
    const int e2 = __shfl_sync(full, e, j2);
    const bool v2 = e2 >= 0;
    nvalid += v2;
    if (valid && v2 && (e2 < e || (e2 == e && j2 < lane))) ++rank;
    if (!v2 && j2 < lane) ++ninv_before;
  }
  if (lane >= k) return -1;
  const int r = valid ? rank : nvalid + ninv_before;
  cs_pos[(size_t)t * k + r] = valid ? e : -1;
  cs_w[(size_t)t * k + r] = w;
  return r;
}

}  // namespace es
