// The whole MoE block for tiny batches (T <= 16 tokens) in one cooperative
// kernel: router, gate/up + SwiGLU, down and combine, with three grid-wide
// barriers between the phases instead of four dependent launches.
//
// Restates generate.py:122-136 (router, once per CTA: every CTA routes the
// few tokens itself, so routing needs no grid-wide hand-off), engine.py:32-41
// (gather_qmm gate/up, SwiGLU, gather_qmm down, weighted sum) and
// generate.py:173-178 (shared expert, as one more expert whose per-token
// weight is the sigmoid gate).
//
// Phases (grid = one CTA per SM, all co-resident: cooperative launch):
//   0  every CTA: route the T tokens (warp t % 8 routes token t) while the
//      other warps stage x in fragment order with 64-group sums in shared
//      memory, then
//      list the distinct experts in ascending id with their (token, weight)
//      pairs, cut into entries of at most 8 pairs (the n = 8 columns of an
//      m16n8 MMA tile; an expert with more pairs takes several entries and
//      streams its weights once per entry)
//   1  gate/up: items (expert, 32-row pair of I, K share) dealt round the
//      CTAs; codes stream from HBM straight into registers (two groups in
//      flight), one m16n8k16 MMA step per 16 K on the exact 128 + q codes,
//      scale and bias applied per (row, group) in fp32: w = s q + b with no
//      weight rounding; each item writes its fp32 partial sums
//   -- barrier --
//   2  reduce: items (expert, row pair): the K shares summed in fixed order,
//      SwiGLU, h rounded once to fp16 (fragment order)
//   -- barrier --
//   3  down: items (expert, 64-row quad of D, I share) on fp16 1024 + q codes
//      and h, partial sums out
//   -- barrier --
//   4  combine: each output element sums its token's slots in ascending
//      expert id (the K shares of each in fixed order), then the shared
//      expert; bf16 or fp32 out, 16-column tiles per CTA
// All arithmetic is fixed-order, so results are bitwise repeatable. Every
// barrier wait is bounded (about a second) and reports ES_DEVERR_TIMEOUT;
// routing whose entries outgrow the split-K partials (experts repeated in
// given routing) reports ES_DEVERR_CAPACITY and writes zeros.
#include <atomic>

#include "es_common.cuh"
#include "es_kernels.cuh"
#include "es_route.cuh"

namespace es {
namespace {

constexpr int kSmWarps = 16;
constexpr int kSmThreads = kSmWarps * 32;
constexpr int kSmMaxT = kSmallMaxTokens;
constexpr int kRouteWarps = 8;  // warps that route (token t: warp t % 8); the rest stage x
static_assert(kRouteWarps < kSmWarps, "routing warps and staging warps are disjoint");
constexpr int kSmMaxPairs = kSmMaxT * kMaxTopK + kSmMaxT;  // routed + shared
constexpr uint32_t kErrCapacity = 0x4u;
constexpr uint32_t kErrTimeout = 0x8u;
constexpr uint32_t kErrRange = 0x10u;

// Grid barrier b (1, 2, 3) on a counter that is zero when the kernel starts:
// every CTA adds one with a release reduction (ordering the CTA's writes,
// collected by the block barrier, before it) and waits with acquire loads
// for b * gridDim.x arrivals (bounded).
ES_DEV void grid_barrier(unsigned* bar, unsigned b, uint32_t* err) {
  __syncthreads();
  if (threadIdx.x == 0) {
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;\n" ::"l"(bar) : "memory");
    const unsigned target = b * gridDim.x;
    const long long t0 = clock64();
    while (true) {
      unsigned v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(bar) : "memory");
      if (v >= target) break;
      if (clock64() - t0 > (1LL << 31)) {
        atomicOr(err, kErrTimeout);
        break;
      }
    }
  }
  __syncthreads();
}

// Shared-memory state of one CTA (identical in every CTA after phase 0).
struct SmallState {
  int n_pairs, n_act;
  int act_e[kSmMaxPairs];      // expert entries: runs of at most 8 of an
                               // expert's pairs, by ascending expert id
                               // (E = the shared expert)
  int act_off[kSmMaxPairs];    // their first pair
  int act_n[kSmMaxPairs];      // their pairs (1..8)
  int pair_tok[kSmMaxPairs];   // token of each pair
  float pair_w[kSmMaxPairs];   // its weight (shared expert: the sigmoid gate)
  int pair_u[kSmMaxPairs];     // its entry in act_*
  int slot_e[kSmMaxT * kMaxTopK];
  float slot_w[kSmMaxT * kMaxTopK];
  int ent[kSmMaxT * kMaxTopK];               // at an expert's first slot: its entries
  int n_ent;                                 // entries of the routed experts
  int tok_n[kSmMaxT];                        // pairs of each token
  int tok_pair[kSmMaxT * (kMaxTopK + 1)];    // their indices, ascending
  float sgate[kSmMaxT];
};

// x rows -> shared memory in fragment order, with 64-group sums, by the
// threads from tid0 up (whole warps); no barrier of its own
ES_DEV void small_stage_x(const SmallArgs& a, uint16_t* xs, float* xsum, int tid0) {
  const unsigned full = 0xffffffffu;
  const int chunks = a.D / 8, GD = a.D / kGroup;
  const int total = a.T * chunks, nthr = kSmThreads - tid0;
  for (int c0 = 0; c0 < total; c0 += nthr) {
    const int c = c0 + (int)threadIdx.x - tid0;
    const bool lv = c < total;
    const int tt = lv ? c / chunks : 0, q8 = lv ? c % chunks : 0;
    float sum = permute_chunk8(a.x + (size_t)tt * a.D, xs + (size_t)tt * a.D, q8, lv);
    sum += __shfl_xor_sync(full, sum, 1);
    sum += __shfl_xor_sync(full, sum, 2);
    sum += __shfl_xor_sync(full, sum, 4);
    if (lv && (q8 & 7) == 0) xsum[tt * GD + (q8 >> 3)] = sum;
  }
}

// Route: the T tokens (warp t routes token t) or read the given
// routing while the warps from kRouteWarps up stage x, and list the pairs in
// (expert id, token, slot) order.
template <int VPL>
ES_DEV void small_route(const SmallArgs& a, SmallState& st, uint16_t* xs, float* xsum) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int k = a.k, T = a.T;
  if (threadIdx.x == 0) st.n_ent = 0;
  if (warp < kRouteWarps) {
   for (int t = warp; t < T; t += kRouteWarps) {
    int my_e = -1;
    float my_w = 0.f;
    if (a.logits) {
      route_token_warp<VPL>(a.logits, a.logits_f32, a.bias, t, a.E, k, a.renorm,
                            blockIdx.x == 0 ? a.err : nullptr, my_e, my_w);
    } else if (lane < k) {
      my_e = a.in_idx[(size_t)t * k + lane];
      my_w = a.in_w[(size_t)t * k + lane];
      if (my_e < -1 || my_e >= a.E) {
        if (blockIdx.x == 0) set_error(a.err, 0x1u);
        my_e = -1;
      }
    }
    if (lane < k) {
      st.slot_e[t * k + lane] = my_e;
      st.slot_w[t * k + lane] = my_w;
      if (blockIdx.x == 0 && a.out_idx) {
        a.out_idx[(size_t)t * k + lane] = my_e;
        a.out_w[(size_t)t * k + lane] = my_w;
      }
    }
    if (a.has_shared) {
      const float gs = shared_gate_warp(a.x + (size_t)t * a.D, a.sg_w, a.D);
      if (lane == 0) st.sgate[t] = gs;
    }
   }
  } else {
    small_stage_x(a, xs, xsum, kRouteWarps * 32);
  }
  __syncthreads();
  // One thread per slot: its pair index (rank among the valid slots by
  // (expert, slot index)), its expert's slot count and its place among them.
  // An expert's pairs form entries of at most kSmallEntryPairs pairs (the
  // 8 columns of an m16n8 tile); an expert's first slot records how many.
  constexpr int S = kMaxTopK + 1;
  constexpr int EP = kSmallEntryPairs;
  const int ns = T * k;
  const int s = threadIdx.x;
  const bool valid = s < ns && st.slot_e[s] >= 0;
  int rank = 0, cnt_same = 0, wpos = 0;
  if (valid) {
    const int e = st.slot_e[s];
#pragma unroll 8
    for (int s2 = 0; s2 < ns; ++s2) {
      const int e2 = st.slot_e[s2];
      rank += (e2 >= 0 && (e2 < e || (e2 == e && s2 < s))) ? 1 : 0;
      cnt_same += e2 == e;
      wpos += (e2 == e && s2 < s) ? 1 : 0;
    }
  }
  const int n_entries_here = (valid && wpos == 0) ? (cnt_same + EP - 1) / EP : 0;
  if (s < ns) st.ent[s] = n_entries_here;
  if (n_entries_here) atomicAdd(&st.n_ent, n_entries_here);
  const int n_routed = __syncthreads_count(valid);
  // entry of each pair: the entries of the lower experts, then wpos / EP;
  // and the pair's place in its token's own list (ascending expert id)
  if (valid) {
    const int e = st.slot_e[s], t = s / k;
    int ubase = 0;
#pragma unroll 8
    for (int s2 = 0; s2 < ns; ++s2) {
      const int e2 = st.slot_e[s2];
      ubase += (e2 >= 0 && e2 < e) ? st.ent[s2] : 0;
    }
    int tpos = 0;
    for (int j = 0; j < k; ++j) {
      const int s2 = t * k + j, e2 = st.slot_e[s2];
      tpos += (e2 >= 0 && (e2 < e || (e2 == e && s2 < s))) ? 1 : 0;
    }
    const int u = ubase + wpos / EP;
    st.pair_tok[rank] = t;
    st.pair_w[rank] = st.slot_w[s];
    st.pair_u[rank] = u;
    st.tok_pair[t * S + tpos] = rank;
    if (wpos % EP == 0) {
      st.act_e[u] = e;
      st.act_off[u] = rank;
      st.act_n[u] = min(EP, cnt_same - wpos);
    }
  }
  // one thread per token: its pair count, and its shared-expert pair (the
  // last of its list, after every routed expert); the shared expert's pairs
  // form entries of EP tokens each
  const int n_ent = st.n_ent;
  if (s < T) {
    int nv = 0;
    for (int j = 0; j < k; ++j) nv += st.slot_e[s * k + j] >= 0 ? 1 : 0;
    if (a.has_shared) {
      const int p = n_routed + s, u = n_ent + s / EP;
      st.pair_tok[p] = s;
      st.pair_w[p] = st.sgate[s];
      st.pair_u[p] = u;
      st.tok_pair[s * S + nv] = p;
      ++nv;
      if (s % EP == 0) {
        st.act_e[u] = a.E;
        st.act_off[u] = p;
        st.act_n[u] = min(EP, T - s);
      }
    }
    st.tok_n[s] = nv;
  }
  if (s == 0) {
    st.n_act = n_ent + (a.has_shared ? (T + EP - 1) / EP : 0);
    st.n_pairs = n_routed + (a.has_shared ? T : 0);
  }
  __syncthreads();
}

// Gate/up item: expert entry u, row pair rp (32 rows of I: two 16-row
// blocks, gate and up), K share ks of GPI groups. Partial sums per lane:
// [block j][gate v0..3 | up v0..3] -> part[((u * RP + rp) * KS + ks) * 512].
ES_DEV void small_gateup_item(const SmallArgs& a, const SmallState& st, const uint16_t* xs,
                              const float* xsum, int u, int rp, int ks) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int GD = a.D / kGroup, RP = a.I / 32, KS = a.ks_gu, GPI = GD / KS;
  const int e = st.act_e[u], p0 = st.act_off[u], n = st.act_n[u];
  const uint8_t* base = a.packed + (size_t)e * a.expert_bytes;
  // weights are read once per call: first out of L2, so that the kernel's
  // code, x, the partials and h stay there
  const uint64_t pol = l2_evict_first_policy();
  const int tb = g < n ? st.pair_tok[p0 + g] : -1;
  const int tc0 = 2 * c < n ? st.pair_tok[p0 + 2 * c] : -1;
  const int tc1 = 2 * c + 1 < n ? st.pair_tok[p0 + 2 * c + 1] : -1;
  float acc[2][8];
#pragma unroll
  for (int j = 0; j < 2; ++j)
#pragma unroll
    for (int v = 0; v < 8; ++v) acc[j][v] = 0.f;
  uint4 cw[2][4];
  uint2 sb[2][4];
  auto load = [&](int G, uint4 (&w)[4], uint2 (&b)[4]) {
    const uint8_t* run = base + gateup_tile_off(GD, 2 * rp, G, 0);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      w[t] = ld_stream16_pol(run + t * kTileBytes + lane * 16, pol);
      b[t] = ld_nc8_pol(run + t * kTileBytes + kTileCodeBytes + g * 8, pol);
    }
  };
  const int G0 = ks * GPI;
  load(G0, cw[0], sb[0]);
  for (int i = 0; i < GPI; ++i) {
    const int G = G0 + i, cur = i & 1;
    if (i + 1 < GPI) {
      if (cur == 0) load(G + 1, cw[1], sb[1]);
      else load(G + 1, cw[0], sb[0]);
    }
    // B fragments of the pairs' tokens and their group sums, from shared memory
    uint32_t bw[8];
    {
      uint4 xa = make_uint4(0, 0, 0, 0), xb = xa;
      if (tb >= 0) {
        const uint4* xp = reinterpret_cast<const uint4*>(xs + (size_t)tb * a.D + G * kGroup + c * 16);
        xa = xp[0];
        xb = xp[1];
      }
      bw[0] = xa.x; bw[1] = xa.y; bw[2] = xa.z; bw[3] = xa.w;
      bw[4] = xb.x; bw[5] = xb.y; bw[6] = xb.z; bw[7] = xb.w;
    }
    const float xs0 = tc0 >= 0 ? xsum[tc0 * GD + G] : 0.f;
    const float xs1 = tc1 >= 0 ? xsum[tc1 * GD + G] : 0.f;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int j = t >> 1, proj = t & 1;  // tile order in a run: block, then (gate, up)
      const uint4 q = cur == 0 ? cw[0][t] : cw[1][t];
      const uint2 sbv = cur == 0 ? sb[0][t] : sb[1][t];
      const float s0 = lo_half_f(sbv.x), s8 = lo_half_f(sbv.y);
      const float b0 = fmaf(-128.f, s0, hi_half_f(sbv.x));
      const float b8 = fmaf(-128.f, s8, hi_half_f(sbv.y));
      float tmp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int s = 0; s < 4; ++s)
        mma_bf16(tmp, code_pair(q.x, s), code_pair(q.z, s), code_pair(q.y, s),
                 code_pair(q.w, s), bw[2 * s], bw[2 * s + 1], tmp);
      float* av = acc[j] + 4 * proj;
      av[0] = fmaf(s0, tmp[0], fmaf(b0, xs0, av[0]));
      av[1] = fmaf(s0, tmp[1], fmaf(b0, xs1, av[1]));
      av[2] = fmaf(s8, tmp[2], fmaf(b8, xs0, av[2]));
      av[3] = fmaf(s8, tmp[3], fmaf(b8, xs1, av[3]));
    }
  }
  float4* out = reinterpret_cast<float4*>(a.part + ((size_t)(u * RP + rp) * KS + ks) * 512) + lane * 4;
#pragma unroll
  for (int q = 0; q < 4; ++q)
    out[q] = make_float4(acc[q >> 1][(q & 1) * 4 + 0], acc[q >> 1][(q & 1) * 4 + 1],
                         acc[q >> 1][(q & 1) * 4 + 2], acc[q >> 1][(q & 1) * 4 + 3]);
}

// Reduce item (u, rp): the K shares summed in order, SwiGLU, h in fp16
// (fragment order) for the expert's pairs.
ES_DEV void small_reduce_item(const SmallArgs& a, const SmallState& st, int u, int rp) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int RP = a.I / 32, KS = a.ks_gu;
  const int p0 = st.act_off[u], n = st.act_n[u];
  float v[16];
#pragma unroll
  for (int q = 0; q < 16; ++q) v[q] = 0.f;
  const float4* src = reinterpret_cast<const float4*>(a.part + (size_t)(u * RP + rp) * KS * 512);
  // the shares in two batches of four, every load of a batch in flight
  // together; summed in share order
#pragma unroll
  for (int k0 = 0; k0 < kMaxSplitK; k0 += 4) {
    float4 t[4][4];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
#pragma unroll
      for (int q = 0; q < 4; ++q)
        t[kk][q] = k0 + kk < KS ? __ldcg(src + (size_t)(k0 + kk) * 128 + lane * 4 + q)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        v[4 * q] += t[kk][q].x; v[4 * q + 1] += t[kk][q].y;
        v[4 * q + 2] += t[kk][q].z; v[4 * q + 3] += t[kk][q].w;
      }
  }
  uint32_t range = 0;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int rb = 2 * rp + j;
#pragma unroll
    for (int vv = 0; vv < 4; ++vv) {
      const int row = vv < 2 ? g : g + 8;
      const int col = 2 * c + (vv & 1);
      if (col < n) {
        const float gv = v[j * 8 + vv], uv = v[j * 8 + 4 + vv];
        float h = gv / (1.f + expf(-gv)) * uv;
        if (!(fabsf(h) <= 65504.f)) { range = 1; h = h != h ? 0.f : copysignf(65504.f, h); }
        a.h16[(size_t)(p0 + col) * a.I + frag_pos(rb * 16 + row)] = __half_as_ushort(__float2half_rn(h));
      }
    }
  }
  if (range) set_error(a.err, kErrRange);
}

// Down item: expert entry u, row quad rq (64 rows of D), I share ks
// of GPI groups. fp16 codes 1024 + q against fp16 h (exact products), scale
// and bias per (row, group) on the fp32 sums. The weights and h of the next
// group are loaded while this one is multiplied. Partial sums per lane:
// [block j][v] -> part[((u * RQ + rq) * KS + ks) * 512].
ES_DEV void small_down_item(const SmallArgs& a, const SmallState& st, int u, int rq, int ks) {
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int GI = a.I / kGroup, RQ = a.D / 64, KS = a.ks_dn, GPI = GI / KS;
  const int e = st.act_e[u], p0 = st.act_off[u], n = st.act_n[u];
  const uint8_t* base = a.packed + (size_t)e * a.expert_bytes;
  // weights are read once per call: first out of L2, so that the kernel's
  // code, x, the partials and h stay there
  const uint64_t pol = l2_evict_first_policy();
  const uint4* hrow = g < n ? reinterpret_cast<const uint4*>(a.h16 + (size_t)(p0 + g) * a.I + c * 16)
                            : nullptr;
  float acc[4][4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int v = 0; v < 4; ++v) acc[j][v] = 0.f;
  uint4 cw[2][4];
  uint2 sb[2][4];
  uint4 hv[2][2];
  auto load_w = [&](int G, uint4 (&w)[4], uint2 (&b)[4]) {
    const uint8_t* run = base + down_tile_off(a.D, a.I, 4 * rq, G);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      w[t] = ld_stream16_pol(run + t * kTileBytes + lane * 16, pol);
      b[t] = ld_nc8_pol(run + t * kTileBytes + kTileCodeBytes + g * 8, pol);
    }
  };
  auto load_h = [&](int G, uint4 (&h)[2]) {
    if (hrow) {
      h[0] = __ldcg(hrow + G * (kGroup / 8));
      h[1] = __ldcg(hrow + G * (kGroup / 8) + 1);
    } else {
      h[0] = make_uint4(0, 0, 0, 0);
      h[1] = h[0];
    }
  };
  const int G0 = ks * GPI;
  load_w(G0, cw[0], sb[0]);
  load_h(G0, hv[0]);
  for (int i = 0; i < GPI; ++i) {
    const int G = G0 + i, cur = i & 1;
    if (i + 1 < GPI) {
      if (cur == 0) { load_w(G + 1, cw[1], sb[1]); load_h(G + 1, hv[1]); }
      else { load_w(G + 1, cw[0], sb[0]); load_h(G + 1, hv[0]); }
    }
    uint32_t hw[8];
    {
      const uint4 h0 = cur == 0 ? hv[0][0] : hv[1][0];
      const uint4 h1 = cur == 0 ? hv[0][1] : hv[1][1];
      hw[0] = h0.x; hw[1] = h0.y; hw[2] = h0.z; hw[3] = h0.w;
      hw[4] = h1.x; hw[5] = h1.y; hw[6] = h1.z; hw[7] = h1.w;
    }
    float hs = 0.f;
#pragma unroll
    for (int v = 0; v < 8; ++v) hs += lo_half_f(hw[v]) + hi_half_f(hw[v]);
    hs += __shfl_xor_sync(full, hs, 1);
    hs += __shfl_xor_sync(full, hs, 2);
    const float hs0 = __shfl_sync(full, hs, (2 * c) << 2);
    const float hs1 = __shfl_sync(full, hs, (2 * c + 1) << 2);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 q = cur == 0 ? cw[0][j] : cw[1][j];
      const uint2 sbv = cur == 0 ? sb[0][j] : sb[1][j];
      const float s0 = lo_half_f(sbv.x), s8 = lo_half_f(sbv.y);
      const float b0 = fmaf(-1024.f, s0, hi_half_f(sbv.x));
      const float b8 = fmaf(-1024.f, s8, hi_half_f(sbv.y));
      float tmp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int s = 0; s < 4; ++s)
        mma_f16(tmp, code_pair_f16(q.x, s), code_pair_f16(q.z, s), code_pair_f16(q.y, s),
                code_pair_f16(q.w, s), hw[2 * s], hw[2 * s + 1], tmp);
      acc[j][0] = fmaf(s0, tmp[0], fmaf(b0, hs0, acc[j][0]));
      acc[j][1] = fmaf(s0, tmp[1], fmaf(b0, hs1, acc[j][1]));
      acc[j][2] = fmaf(s8, tmp[2], fmaf(b8, hs0, acc[j][2]));
      acc[j][3] = fmaf(s8, tmp[3], fmaf(b8, hs1, acc[j][3]));
    }
  }
  float4* out = reinterpret_cast<float4*>(a.part + ((size_t)(u * RQ + rq) * KS + ks) * 512) + lane * 4;
#pragma unroll
  for (int j = 0; j < 4; ++j) out[j] = make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
}

// Combine: out[t][d] = sum over the token's pairs (ascending expert id, the
// shared expert last) of weight x (its down partials summed in share
// order). A CTA takes 16 columns at a time: one thread per (token, pair,
// column) loads and sums that pair's shares into shared memory, then one
// thread per (token, column) folds the pairs in order.
constexpr int kCombCols = 16;
ES_DEV void small_combine(const SmallArgs& a, const SmallState& st, float* ys) {
  const int RQ = a.D / 64, KS = a.ks_dn, T = a.T;
  constexpr int S = kMaxTopK + 1;
  const int n_tiles = a.D / kCombCols;
  for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
    const int d0 = tile * kCombCols;
    for (int w = threadIdx.x; w < T * S * kCombCols; w += kSmThreads) {
      const int dc = w % kCombCols, ts = w / kCombCols, t = ts / S, s = ts - t * S;
      if (s >= st.tok_n[t]) continue;
      const int p = st.tok_pair[t * S + s];
      const int d = d0 + dc, rq = d >> 6, j = (d >> 4) & 3, r = d & 15;
      const int u = st.pair_u[p], col = p - st.act_off[u];
      const float* src = a.part + (size_t)(u * RQ + rq) * KS * 512 +
                         ((r & 7) * 4 + (col >> 1)) * 16 + j * 4 + (r >= 8 ? 2 : 0) + (col & 1);
      float part[kMaxSplitK];
#pragma unroll
      for (int ks = 0; ks < kMaxSplitK; ++ks) part[ks] = ks < KS ? __ldcg(src + (size_t)ks * 512) : 0.f;
      float y = 0.f;
#pragma unroll
      for (int ks = 0; ks < kMaxSplitK; ++ks) y += part[ks];
      ys[w] = y;
    }
    __syncthreads();
    for (int w = threadIdx.x; w < T * kCombCols; w += kSmThreads) {
      const int t = w / kCombCols, dc = w % kCombCols;
      float acc = 0.f;
      for (int s = 0; s < st.tok_n[t]; ++s)
        acc = fmaf(st.pair_w[st.tok_pair[t * S + s]], ys[(t * S + s) * kCombCols + dc], acc);
      const size_t i = (size_t)t * a.D + d0 + dc;
      if (a.out_f32) static_cast<float*>(a.out)[i] = acc;
      else static_cast<uint16_t*>(a.out)[i] = float_to_bf16_bits(acc);
    }
    __syncthreads();
  }
}

template <int VPL>
__global__ void __launch_bounds__(kSmThreads, 1) small_block_kernel(SmallArgs a) {
  extern __shared__ __align__(16) uint8_t sm_dyn[];
  __shared__ SmallState st;
  __shared__ float ys[kSmMaxT * (kMaxTopK + 1) * kCombCols];
  uint16_t* xs = reinterpret_cast<uint16_t*>(sm_dyn);
  float* xsum = reinterpret_cast<float*>(sm_dyn + (size_t)a.T * a.D * 2);
  unsigned* bar = reinterpret_cast<unsigned*>(a.ctr);
  const int warp = threadIdx.x >> 5;
  // items go round the CTAs first, so a phase with fewer items than warps
  // still spreads its loads over every SM
  const int gw = warp * gridDim.x + blockIdx.x, nw = gridDim.x * kSmWarps;
  small_route<VPL>(a, st, xs, xsum);
  const int RP = a.I / 32, RQ = a.D / 64;
  // The partials are sized for the entries routing can make. Given routing
  // that repeats an expert inside a token's slots can cut more entries than
  // that: then the call reports ES_DEVERR_CAPACITY and writes zeros (every
  // CTA sees the same lists, so all take this path together).
  {
    const long long need_gu = (long long)st.n_act * RP * a.ks_gu;
    const long long need_dn = (long long)st.n_act * RQ * a.ks_dn;
    if (need_gu > a.part_slots || need_dn > a.part_slots) {
      if (blockIdx.x == 0 && threadIdx.x == 0) set_error(a.err, kErrCapacity);
      const size_t n_out = (size_t)a.T * a.D;
      for (size_t i = (size_t)blockIdx.x * kSmThreads + threadIdx.x; i < n_out;
           i += (size_t)gridDim.x * kSmThreads) {
        if (a.out_f32) static_cast<float*>(a.out)[i] = 0.f;
        else static_cast<uint16_t*>(a.out)[i] = 0;
      }
      return;
    }
  }
  // phase 1: gate/up partials
  {
    const int items = st.n_act * RP * a.ks_gu;
    for (int it = gw; it < items; it += nw) {
      const int ks = it % a.ks_gu, rest = it / a.ks_gu;
      small_gateup_item(a, st, xs, xsum, rest / RP, rest % RP, ks);
    }
  }
  grid_barrier(bar, 1, a.err);
  // phase 2: reduce + SwiGLU -> h
  for (int it = gw; it < st.n_act * RP; it += nw) small_reduce_item(a, st, it / RP, it % RP);
  grid_barrier(bar, 2, a.err);
  // phase 3: down partials
  {
    const int items = st.n_act * RQ * a.ks_dn;
    for (int it = gw; it < items; it += nw) {
      const int ks = it % a.ks_dn, rest = it / a.ks_dn;
      small_down_item(a, st, rest / RQ, rest % RQ, ks);
    }
  }
  grid_barrier(bar, 3, a.err);
  small_combine(a, st, ys);
  // the last CTA out returns both counters to zero for the next call
  __syncthreads();
  if (threadIdx.x == 0) {
    if (atomicAdd(bar + 1, 1u) == gridDim.x - 1) {
      bar[0] = 0u;
      bar[1] = 0u;
    }
  }
}

// largest divisor of n that is <= cap
int share_count(int n, int cap) {
  for (int s = cap; s > 1; --s)
    if (n % s == 0) return s;
  return 1;
}

template <int VPL>
cudaError_t launch_small_vpl(SmallArgs a, cudaStream_t st) {
  const size_t smem = (size_t)a.T * a.D * 2 + (size_t)a.T * (a.D / kGroup) * 4;
  // The shared-memory opt-in and the one-CTA-per-SM check are made once per
  // device for the largest size seen so far (a smaller call fits the same
  // opt-in and the same residency), not on every launch. A launch refused
  // after all (a new context on the device has no opt-in) makes them again
  // and retries once.
  constexpr int kMaxDev = 64;
  static std::atomic<size_t> checked[kMaxDev];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const bool cached = dev >= 0 && dev < kMaxDev &&
                      smem <= checked[dev].load(std::memory_order_acquire);
  if (!cached) {
    e = cudaFuncSetAttribute(small_block_kernel<VPL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, small_block_kernel<VPL>, kSmThreads,
                                                      smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    if (dev >= 0 && dev < kMaxDev) {
      size_t cur = checked[dev].load(std::memory_order_relaxed);
      while (smem > cur && !checked[dev].compare_exchange_weak(cur, smem)) {
      }
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sm_count());
  cfg.blockDim = dim3(kSmThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: grid barriers are safe
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, small_block_kernel<VPL>, a);
  if (e != cudaSuccess && cached) {
    (void)cudaGetLastError();
    checked[dev].store(0, std::memory_order_release);
    return launch_small_vpl<VPL>(a, st);
  }
  return e;
}

}  // namespace

bool small_path_fits(int T, int D, int I, int E, int k, int has_shared) {
  (void)E;
  (void)has_shared;
  return T >= 1 && T <= kSmallMaxTokens && D % 64 == 0 && D <= 4096 && I % 64 == 0 &&
         (I / 32) >= 1 && T * k <= kSmThreads;
}

cudaError_t launch_small(SmallArgs a, cudaStream_t st) {
  // above kSplitKMaxTokens tokens: up to twice the entries, half the shares,
  // so the partials fit the same workspace
  const int cap = a.T > kSplitKMaxTokens ? kSmallSplitKLarge : kMaxSplitK;
  a.ks_gu = share_count(a.D / kGroup, cap);
  a.ks_dn = share_count(a.I / kGroup, cap);
  const int vpl = (a.E + 31) / 32;
  if (vpl <= 1) return launch_small_vpl<1>(a, st);
  if (vpl <= 2) return launch_small_vpl<2>(a, st);
  if (vpl <= 4) return launch_small_vpl<4>(a, st);
  if (vpl <= 8) return launch_small_vpl<8>(a, st);
  if (vpl <= 16) return launch_small_vpl<16>(a, st);
  return launch_small_vpl<32>(a, st);
}

}  // namespace es
