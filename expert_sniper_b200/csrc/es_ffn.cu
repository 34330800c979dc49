// Decode expert FFN: 4-bit dequant-GEMV with warp-independent work items.
//
// Restates the three gather_qmm calls of run_expert_ffn
// (src/mlx_expert_sniper/engine.py:32-39) and the SwiGLU between them
// (engine.py:37) for every active expert, grouped by expert so each packed
// weight byte is read from HBM once per call however many tokens chose the
// expert.
//
// Arithmetic. A code q becomes the exact bf16 value 128 + q (gate/up, whose
// B operand is the bf16 activation) or the exact fp16 value 1024 + q (down,
// whose B operand is h rounded once to fp16), so the tensor core computes
// acc = sum_d (c0 + q_d) v_d exactly in fp32, and per (row, 64-group)
//     sum_d w_d v_d = scale * acc + (bias - c0 * scale) * sum_d v_d ,
// which is the MLX dequantisation w = scale * q + bias with no rounding of
// the weights. |h| beyond the fp16 range is saturated and flagged.
//
// Work. An item is (active expert, a run of rows, share of K): 32 rows
// (two 16-row blocks, gate and up) for gate/up, 64 rows (four blocks) for
// down. One warp owns an item from start to finish: lane 0 streams the
// item's packed tiles in chunks (the tiles sharing one activation fragment
// are contiguous in the packed layout) through the warp's own ring of
// shared-memory slots (bulk async copies, one mbarrier per slot, L2
// evict-first), and the warp converts codes in registers (one LOP3 per pair)
// and runs m16n8k16 MMAs against up to 16 tokens at a time, looping over
// further tokens if an expert has more. Each activation fragment (and, for
// down, its group sum) is loaded once per chunk and feeds 4 tiles. Warps
// never wait for each other: only as many warps take part as make the items
// whole rounds; after a first item given by its position, a warp claims
// items from a global counter (so experts with more tokens do not leave a
// tail), and the copy issuer runs up to a ring's depth ahead, across item
// boundaries. For very small batches K is split over KS warps;
// each writes its partial sums and the last to arrive (atomic counter, reset
// after use) adds the KS partials in fixed order, so results are
// deterministic.
#include "es_common.cuh"
#include "es_kernels.cuh"

namespace es {
namespace {

constexpr int kWarps = 16;       // warps per CTA, one CTA per SM
constexpr int kTiles = 2;        // n8 token tiles per pass: 16 tokens
constexpr int kQueue = 8;        // per-warp queue of claimed items
constexpr int kGUGroups = 2;     // 64-column groups per gate/up chunk
constexpr int kGUSlots = 3;      // gate/up ring depth
constexpr int kDNSlots = 4;      // down ring depth
constexpr uint32_t kGUChunk = kGUGroups * 4 * kTileBytes;  // 2 groups x 2 blocks x (gate, up)
constexpr uint32_t kDNChunk = 4 * kTileBytes;              // 1 group x 4 blocks
constexpr uint32_t kDevErrTimeout = 0x8u;
constexpr uint32_t kDevErrRange = 0x10u;

// Per-warp ring of `ns` chunk buffers, one mbarrier each.
struct WarpRing {
  uint8_t* buf;
  uint64_t* bars;
  uint32_t bytes;
  int ns;
  uint64_t pol;

  ES_DEV void init() {
    if ((threadIdx.x & 31) == 0) {
      for (int s = 0; s < ns; ++s) mbar_init(&bars[s], 1);
      fence_mbar_init();
    }
    __syncwarp();
  }
  ES_DEV void issue(int q, const void* src) {  // one lane
    const int s = q % ns;
    mbar_arrive_expect_tx(&bars[s], bytes);
    bulk_copy_g2s(buf + (size_t)s * bytes, src, bytes, &bars[s], pol);
  }
  ES_DEV const uint8_t* slot(int q) const { return buf + (size_t)(q % ns) * bytes; }
  // whole warp; false (after draining this warp's copies in flight) on timeout
  ES_DEV bool wait(int q, int issued, uint32_t* err) {
    const bool ok = mbar_wait_bounded(&bars[q % ns], (q / ns) & 1);
    if (__all_sync(0xffffffffu, ok)) return true;
    if ((threadIdx.x & 31) == 0) {
      set_error(err, kDevErrTimeout);
      for (int r = q + 1; r < issued; ++r) mbar_wait_bounded(&bars[r % ns], (r / ns) & 1);
    }
    __syncwarp();
    return false;
  }
};

// Walks the items one warp processes: chunk c of pass p of item i. Items are
// numbered (active expert, row run, K share); `per` items per expert, `sub`
// K shares per row run. The copy-issue cursor claims items (the first by the
// warp's position, later ones from a global counter) and records them in a
// per-warp queue that the compute cursor replays in the same order.
struct Cursor {
  int n_items, first, stride;
  int per, sub, nch;
  int* queue;
  int qpos;
  int i, ai, rr, ks, e, off, n, np, p, c;

  ES_DEV void load(const FfnArgs& a) {
    if (i >= n_items) return;
    ai = i / per;
    const int rem = i - ai * per;
    rr = rem / sub;
    ks = rem - rr * sub;
    e = a.act_e[ai];
    off = a.act_off[ai];
    n = a.act_n[ai];
    np = (n + kTiles * 8 - 1) / (kTiles * 8);
    p = 0;
    c = 0;
  }
  ES_DEV void claim(const FfnArgs& a, int* counter) {  // whole warp
    int v = 0;
    if ((threadIdx.x & 31) == 0) {
      v = qpos == 0 ? first : atomicAdd(counter, 1) + stride;
      queue[qpos & (kQueue - 1)] = v;
    }
    i = __shfl_sync(0xffffffffu, v, 0);
    ++qpos;
    load(a);
  }
  ES_DEV void replay(const FfnArgs& a) {  // whole warp
    __syncwarp();
    i = queue[qpos & (kQueue - 1)];
    ++qpos;
    load(a);
  }
  ES_DEV bool valid() const { return i < n_items; }
  template <bool kIssue>
  ES_DEV void advance(const FfnArgs& a, int* counter) {
    if (++c < nch) return;
    c = 0;
    if (++p < np) return;
    if (kIssue) claim(a, counter); else replay(a);
  }
};

// Warps that take part: enough per CTA that the items make whole rounds
// (a partial last round would leave most warps idle while a few finish).
// Returns the number of active warps per CTA.
ES_DEV int active_warps_per_cta(int n_items) {
  const long long total = (long long)gridDim.x * kWarps;
  const long long rounds = n_items > 0 ? (n_items + total - 1) / total : 1;
  const long long warps = (n_items + rounds - 1) / rounds;
  return (int)((warps + gridDim.x - 1) / gridDim.x);
}

ES_DEV void scale_bias(uint2 sb, float c0, float& s0, float& b0, float& s8, float& b8) {
  s0 = lo_half_f(sb.x);
  s8 = lo_half_f(sb.y);
  b0 = fmaf(-c0, s0, hi_half_f(sb.x));
  b8 = fmaf(-c0, s8, hi_half_f(sb.y));
}

// Split-K arrival: store this warp's partial (16 floats per lane) for K
// share `ks` of `slot`; true for the last of the KS warps, which then holds
// the fixed-order sum of all KS partials in `v`.
ES_DEV bool splitk_arrive(const FfnArgs& a, int slot, int KS, int ks, float (&v)[16]) {
  const int lane = threadIdx.x & 31;
  float4* part = reinterpret_cast<float4*>(a.partials) + ((size_t)slot * KS + ks) * 128;
#pragma unroll
  for (int q = 0; q < 4; ++q) part[lane * 4 + q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  __threadfence();
  __syncwarp();
  int old = 0;
  if (lane == 0) old = atomicAdd(&a.counters[slot], 1);
  old = __shfl_sync(0xffffffffu, old, 0);
  if (old != KS - 1) return false;
  __threadfence();
#pragma unroll
  for (int q = 0; q < 16; ++q) v[q] = 0.f;
  const float4* pp = reinterpret_cast<const float4*>(a.partials) + (size_t)slot * KS * 128;
  for (int k2 = 0; k2 < KS; ++k2) {  // fixed order: deterministic
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 t = __ldcg(pp + (size_t)k2 * 128 + lane * 4 + q);
      v[4 * q] += t.x; v[4 * q + 1] += t.y; v[4 * q + 2] += t.z; v[4 * q + 3] += t.w;
    }
  }
  if (lane == 0) a.counters[slot] = 0;
  return true;
}

// ---------------------------------------------------------------------------
// gate/up + SwiGLU -> h (fp16, fragment order)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kWarps * 32, 1) ffn_gateup_kernel(FfnArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_queue[kWarps][kQueue];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int GD = a.D / kGroup, RP = a.I / 32, KS = a.split_k;
  const int GPI = GD / KS;  // groups per item
  WarpRing ring{smem + (size_t)warp * kGUSlots * kGUChunk,
                reinterpret_cast<uint64_t*>(smem + (size_t)kWarps * kGUSlots * kGUChunk) + warp * kGUSlots,
                kGUChunk, kGUSlots, l2_evict_first_policy()};
  ring.init();
  pdl_wait();
  pdl_trigger();

  const int n_items = *a.n_active * RP * KS;
  const int per_cta = active_warps_per_cta(n_items);
  if (warp >= per_cta) return;
  Cursor ic{n_items, (int)blockIdx.x * per_cta + warp, (int)gridDim.x * per_cta, RP * KS, KS,
            GPI / kGUGroups, s_queue[warp], 0};
  ic.claim(a, &a.item_ctr[0]);
  Cursor cc = ic;
  cc.qpos = 0;
  cc.replay(a);
  if (!cc.valid()) return;
  auto src = [&](const Cursor& u) {
    return a.packed + (size_t)u.e * a.expert_bytes +
           gateup_tile_off(GD, 2 * u.rr, u.ks * GPI + u.c * kGUGroups, 0);
  };
  int issued = 0;
  for (; issued < kGUSlots && ic.valid(); ++issued) {
    if (lane == 0) ring.issue(issued, src(ic));
    ic.advance<true>(a, &a.item_ctr[0]);
  }

  float acc[kTiles][2][8];  // [token tile][row block of the pair][gate 4 | up 4]
  int tb[kTiles], tc0[kTiles], tc1[kTiles];
  int ntile = 0;
  for (int q = 0; cc.valid(); ++q) {
    if (cc.c == 0) {  // start of a pass over 16 tokens
      const int base = cc.p * kTiles * 8;
      ntile = min(kTiles, (cc.n - base + 7) / 8);
#pragma unroll
      for (int t = 0; t < kTiles; ++t) {
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int v = 0; v < 8; ++v) acc[t][j][v] = 0.f;
        const int cb = base + t * 8 + g, cq = base + t * 8 + 2 * c;
        tb[t] = cb < cc.n ? a.pair_tok[cc.off + cb] : -1;
        tc0[t] = cq < cc.n ? a.pair_tok[cc.off + cq] : -1;
        tc1[t] = cq + 1 < cc.n ? a.pair_tok[cc.off + cq + 1] : -1;
      }
    }
    if (!ring.wait(q, issued, a.err)) return;
    const uint8_t* st = ring.slot(q);
    const int G0 = cc.ks * GPI + cc.c * kGUGroups;
#pragma unroll
    for (int gi = 0; gi < kGUGroups; ++gi) {
      const int G = G0 + gi;
      uint32_t bw[kTiles][8];
      float xs0[kTiles], xs1[kTiles];
#pragma unroll
      for (int t = 0; t < kTiles; ++t) {
        uint4 xa = make_uint4(0, 0, 0, 0), xb = xa;
        if (t < ntile && tb[t] >= 0) {
          const uint4* xp = reinterpret_cast<const uint4*>(a.x_perm + ((size_t)tb[t] * GD + G) * kGroup + c * 16);
          xa = __ldg(xp);
          xb = __ldg(xp + 1);
        }
        bw[t][0] = xa.x; bw[t][1] = xa.y; bw[t][2] = xa.z; bw[t][3] = xa.w;
        bw[t][4] = xb.x; bw[t][5] = xb.y; bw[t][6] = xb.z; bw[t][7] = xb.w;
        xs0[t] = (t < ntile && tc0[t] >= 0) ? __ldg(a.xsum + (size_t)tc0[t] * GD + G) : 0.f;
        xs1[t] = (t < ntile && tc1[t] >= 0) ? __ldg(a.xsum + (size_t)tc1[t] * GD + G) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
#pragma unroll
        for (int proj = 0; proj < 2; ++proj) {
          const uint8_t* tile = st + (size_t)((gi * 2 + j) * 2 + proj) * kTileBytes;
          const uint4 cw = ld_shared16(tile + lane * 16);
          float s0, b0, s8, b8;
          scale_bias(ld_shared8(tile + kTileCodeBytes + g * 8), 128.f, s0, b0, s8, b8);
          uint32_t ao[4][4];
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            ao[s][0] = code_pair(cw.x, s); ao[s][1] = code_pair(cw.z, s);
            ao[s][2] = code_pair(cw.y, s); ao[s][3] = code_pair(cw.w, s);
          }
#pragma unroll
          for (int t = 0; t < kTiles; ++t) {
            if (t >= ntile) break;  // warp-uniform
            float tmp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int s = 0; s < 4; ++s)
              mma_bf16(tmp, ao[s][0], ao[s][1], ao[s][2], ao[s][3], bw[t][2 * s], bw[t][2 * s + 1], tmp);
            float* av = acc[t][j] + 4 * proj;
            av[0] = fmaf(s0, tmp[0], fmaf(b0, xs0[t], av[0]));
            av[1] = fmaf(s0, tmp[1], fmaf(b0, xs1[t], av[1]));
            av[2] = fmaf(s8, tmp[2], fmaf(b8, xs0[t], av[2]));
            av[3] = fmaf(s8, tmp[3], fmaf(b8, xs1[t], av[3]));
          }
        }
      }
    }
    __syncwarp();  // every lane is done with this slot: refill it
    if (ic.valid()) {
      if (lane == 0) ring.issue(issued, src(ic));
      ic.advance<true>(a, &a.item_ctr[0]);
      ++issued;
    }

    if (cc.c == cc.nch - 1) {  // end of the pass: SwiGLU -> h
      bool last = true;
      if (KS > 1) {  // batches of <= 8 tokens: one pass, one tile
        float v[16];
#pragma unroll
        for (int q2 = 0; q2 < 16; ++q2) v[q2] = acc[0][q2 >> 3][q2 & 7];
        last = splitk_arrive(a, cc.ai * RP + cc.rr, KS, cc.ks, v);
        if (last) {
#pragma unroll
          for (int q2 = 0; q2 < 16; ++q2) acc[0][q2 >> 3][q2 & 7] = v[q2];
        }
      }
      if (last) {
        const int base = cc.p * kTiles * 8;
#pragma unroll
        for (int t = 0; t < kTiles; ++t) {
          if (t >= ntile) break;
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int rb = 2 * cc.rr + j;
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const int row = (v < 2) ? g : g + 8;
              const int col = base + t * 8 + 2 * c + (v & 1);
              if (col < cc.n) {
                const float gv = acc[t][j][v];
                float h = gv / (1.f + expf(-gv)) * acc[t][j][4 + v];
                if (!(fabsf(h) <= 65504.f)) {  // outside fp16 (or NaN): saturate, flag
                  set_error(a.err, kDevErrRange);
                  h = h != h ? 0.f : copysignf(65504.f, h);
                }
                a.h16[(size_t)(cc.off + col) * a.I + frag_pos(rb * 16 + row)] =
                    __half_as_ushort(__float2half_rn(h));
              }
            }
          }
        }
      }
    }
    cc.advance<false>(a, nullptr);
  }
}

// ---------------------------------------------------------------------------
// down -> y per (token, slot)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kWarps * 32, 1) ffn_down_kernel(FfnArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_queue[kWarps][kQueue];
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int KG = a.I / kGroup, RQ = a.D / 64, KS = a.split_k_down;
  const int GPI = KG / KS;
  WarpRing ring{smem + (size_t)warp * kDNSlots * kDNChunk,
                reinterpret_cast<uint64_t*>(smem + (size_t)kWarps * kDNSlots * kDNChunk) + warp * kDNSlots,
                kDNChunk, kDNSlots, l2_evict_first_policy()};
  ring.init();
  // The expert list comes from the front-end kernel, which completed before
  // the gate/up kernel (this kernel's predecessor) passed its own
  // pdl_wait(), so the first weight copies can be in flight while gate/up
  // finishes; only h (written by gate/up) needs pdl_wait().
  const int n_items = *a.n_active * RQ * KS;
  const int per_cta = active_warps_per_cta(n_items);
  if (warp >= per_cta) {
    pdl_wait();
    pdl_trigger();
    return;
  }
  Cursor ic{n_items, (int)blockIdx.x * per_cta + warp, (int)gridDim.x * per_cta, RQ * KS, KS, GPI,
            s_queue[warp], 0};
  ic.claim(a, &a.item_ctr[1]);
  Cursor cc = ic;
  cc.qpos = 0;
  cc.replay(a);
  const bool any = cc.valid();
  auto src = [&](const Cursor& u) {
    return a.packed + (size_t)u.e * a.expert_bytes + down_tile_off(a.D, a.I, 4 * u.rr, u.ks * GPI + u.c);
  };
  int issued = 0;
  for (; any && issued < kDNSlots && ic.valid(); ++issued) {
    if (lane == 0) ring.issue(issued, src(ic));
    ic.advance<true>(a, &a.item_ctr[1]);
  }
  pdl_wait();
  pdl_trigger();
  if (!any) return;

  float acc[kTiles][4][4];  // [token tile][row block of the quad][c0..c3]
  int pb[kTiles];
  int ntile = 0;
  for (int q = 0; cc.valid(); ++q) {
    if (cc.c == 0) {
      const int base = cc.p * kTiles * 8;
      ntile = min(kTiles, (cc.n - base + 7) / 8);
#pragma unroll
      for (int t = 0; t < kTiles; ++t) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int v = 0; v < 4; ++v) acc[t][j][v] = 0.f;
        const int col = base + t * 8 + g;
        pb[t] = col < cc.n ? cc.off + col : -1;
      }
    }
    if (!ring.wait(q, issued, a.err)) return;
    const uint8_t* st = ring.slot(q);
    const int G = cc.ks * GPI + cc.c;
    uint32_t hw[kTiles][8];
    float hs0[kTiles], hs1[kTiles];
#pragma unroll
    for (int t = 0; t < kTiles; ++t) {
      uint4 h0 = make_uint4(0, 0, 0, 0), h1 = h0;
      if (t < ntile && pb[t] >= 0) {
        const uint4* hp = reinterpret_cast<const uint4*>(a.h16 + (size_t)pb[t] * a.I + G * kGroup + c * 16);
        h0 = hp[0];
        h1 = hp[1];
      }
      hw[t][0] = h0.x; hw[t][1] = h0.y; hw[t][2] = h0.z; hw[t][3] = h0.w;
      hw[t][4] = h1.x; hw[t][5] = h1.y; hw[t][6] = h1.z; hw[t][7] = h1.w;
      float hs = 0.f;
#pragma unroll
      for (int v = 0; v < 8; ++v) hs += lo_half_f(hw[t][v]) + hi_half_f(hw[t][v]);
      hs += __shfl_xor_sync(full, hs, 1);
      hs += __shfl_xor_sync(full, hs, 2);
      hs0[t] = __shfl_sync(full, hs, (2 * c) << 2);
      hs1[t] = __shfl_sync(full, hs, (2 * c + 1) << 2);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint8_t* tile = st + (size_t)j * kTileBytes;
      const uint4 cw = ld_shared16(tile + lane * 16);
      float s0, b0, s8, b8;
      scale_bias(ld_shared8(tile + kTileCodeBytes + g * 8), 1024.f, s0, b0, s8, b8);
      uint32_t ao[4][4];
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        ao[s][0] = code_pair_f16(cw.x, s); ao[s][1] = code_pair_f16(cw.z, s);
        ao[s][2] = code_pair_f16(cw.y, s); ao[s][3] = code_pair_f16(cw.w, s);
      }
#pragma unroll
      for (int t = 0; t < kTiles; ++t) {
        if (t >= ntile) break;  // warp-uniform
        float tmp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int s = 0; s < 4; ++s)
          mma_f16(tmp, ao[s][0], ao[s][1], ao[s][2], ao[s][3], hw[t][2 * s], hw[t][2 * s + 1], tmp);
        acc[t][j][0] = fmaf(s0, tmp[0], fmaf(b0, hs0[t], acc[t][j][0]));
        acc[t][j][1] = fmaf(s0, tmp[1], fmaf(b0, hs1[t], acc[t][j][1]));
        acc[t][j][2] = fmaf(s8, tmp[2], fmaf(b8, hs0[t], acc[t][j][2]));
        acc[t][j][3] = fmaf(s8, tmp[3], fmaf(b8, hs1[t], acc[t][j][3]));
      }
    }
    __syncwarp();
    if (ic.valid()) {
      if (lane == 0) ring.issue(issued, src(ic));
      ic.advance<true>(a, &a.item_ctr[1]);
      ++issued;
    }
    if (cc.c == cc.nch - 1) {  // end of the pass: store y rows
      bool last = true;
      if (KS > 1) {
        float v[16];
#pragma unroll
        for (int q2 = 0; q2 < 16; ++q2) v[q2] = acc[0][q2 >> 2][q2 & 3];
        last = splitk_arrive(a, cc.ai * RQ + cc.rr, KS, cc.ks, v);
        if (last) {
#pragma unroll
          for (int q2 = 0; q2 < 16; ++q2) acc[0][q2 >> 2][q2 & 3] = v[q2];
        }
      }
      if (last) {
        const int base = cc.p * kTiles * 8;
#pragma unroll
        for (int t = 0; t < kTiles; ++t) {
          if (t >= ntile) break;
          const int col = base + t * 8 + 2 * c;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float* y0 = a.y_pair + (size_t)(cc.off + col) * a.D + (4 * cc.rr + j) * 16;
            if (col < cc.n) { y0[g] = acc[t][j][0]; y0[g + 8] = acc[t][j][2]; }
            if (col + 1 < cc.n) { y0[a.D + g] = acc[t][j][1]; y0[a.D + g + 8] = acc[t][j][3]; }
          }
        }
      }
    }
    cc.advance<false>(a, nullptr);
  }
}

template <typename K>
cudaError_t launch_ring_kernel(K kernel, int slots, uint32_t chunk, int max_items,
                               const FfnArgs& a, cudaStream_t st) {
  const size_t smem = (size_t)kWarps * slots * (chunk + 8);
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  int grid = sm_count();
  const int need = (max_items + kWarps - 1) / kWarps;
  if (grid > need) grid = need;
  if (grid < 1) grid = 1;
  return launch_pdl(kernel, dim3(grid), dim3(kWarps * 32), smem, st, a);
}

}  // namespace

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!cached[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = v > 0 ? v : 148;
  }
  return cached[dev];
}

// Split of K over warps for tiny batches: grow while the item count is below
// the number of warps and each share keeps whole chunks.
int ffn_split_k(int T, int max_active, int D, int I) {
  if (T > kSplitKMaxTokens) return 1;
  const int GD = D / kGroup, RP = I / 32;
  const long long warps = (long long)sm_count() * kWarps;
  int ks = 1;
  while (ks < kMaxSplitK && GD % (ks * 2 * kGUGroups) == 0 && (long long)max_active * RP * ks < warps)
    ks *= 2;
  return ks;
}

int ffn_split_k_down(int T, int max_active, int D, int I) {
  if (T > kSplitKMaxTokens) return 1;
  const int KG = I / kGroup, RQ = D / 64;
  const long long warps = (long long)sm_count() * kWarps;
  int ks = 1;
  while (ks < kMaxSplitK && KG % (ks * 2) == 0 && (long long)max_active * RQ * ks < warps) ks *= 2;
  return ks;
}

cudaError_t launch_ffn_gateup(const FfnArgs& a, int max_active, cudaStream_t st) {
  if (max_active <= 0) return cudaSuccess;
  return launch_ring_kernel(ffn_gateup_kernel, kGUSlots, kGUChunk,
                            max_active * (a.I / 32) * a.split_k, a, st);
}

cudaError_t launch_ffn_down(const FfnArgs& a, int max_active, cudaStream_t st) {
  if (max_active <= 0) return cudaSuccess;
  return launch_ring_kernel(ffn_down_kernel, kDNSlots, kDNChunk,
                            max_active * (a.D / 64) * a.split_k_down, a, st);
}

}  // namespace es
