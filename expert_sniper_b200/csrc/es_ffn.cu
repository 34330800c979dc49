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
// Work. An item is (active expert, 16 rows of the output, share of K); one
// warp owns an item from start to finish: it streams the item's packed tiles
// in chunks of four 64-column groups through its own ring of shared-memory
// slots (bulk async copies + one mbarrier per slot, L2 evict-first), converts
// codes in registers (one LOP3 per pair) and runs m16n8k16 MMAs against up to
// 16 tokens at a time, looping over further tokens if an expert has more.
// Warps never wait for each other; items are claimed dynamically from a
// global counter (so experts with more tokens do not leave a tail), and the
// lane-0 copy issuer runs kSlots chunks ahead, across item boundaries. For very small batches the K dimension of
// gate/up is split over KS warps; each writes its partial sums and the last
// one to arrive (atomic counter, reset after use) adds the KS partials in
// fixed order before the SwiGLU, so results are deterministic.
#include "es_common.cuh"
#include "es_kernels.cuh"

namespace es {
namespace {

constexpr int kGPC = 4;    // 64-column groups per chunk
constexpr int kSlots = 2;  // ring slots per warp (power of two)
constexpr int kTiles = 2;  // n8 token tiles per pass: 16 tokens
constexpr int kGateupWarps = 16;
constexpr int kDownWarps = 16;
constexpr int kQueue = 8;  // per-warp queue of claimed items (> kSlots)
constexpr uint32_t kGateupChunk = kGPC * 2 * kTileBytes;  // gate + up tiles, 4608 B
constexpr uint32_t kDownChunk = kGPC * kTileBytes;        // 2304 B
constexpr uint32_t kDevErrTimeout = 0x8u;
constexpr uint32_t kDevErrRange = 0x10u;

// Per-warp ring of kSlots chunk buffers, one mbarrier each.
struct WarpRing {
  uint8_t* buf;
  uint64_t* bars;
  uint32_t bytes;
  uint64_t pol;

  ES_DEV void init() {
    if ((threadIdx.x & 31) == 0) {
      for (int s = 0; s < kSlots; ++s) mbar_init(&bars[s], 1);
      fence_mbar_init();
    }
    __syncwarp();
  }
  ES_DEV void issue(int q, const void* src) {  // one lane
    const int s = q & (kSlots - 1);
    mbar_arrive_expect_tx(&bars[s], bytes);
    bulk_copy_g2s(buf + (size_t)s * bytes, src, bytes, &bars[s], pol);
  }
  ES_DEV const uint8_t* slot(int q) const { return buf + (size_t)(q & (kSlots - 1)) * bytes; }
  // whole warp; false (after draining this warp's copies in flight) on timeout
  ES_DEV bool wait(int q, int issued, uint32_t* err) {
    const bool ok = mbar_wait_bounded(&bars[q & (kSlots - 1)], (q / kSlots) & 1);
    if (__all_sync(0xffffffffu, ok)) return true;
    if ((threadIdx.x & 31) == 0) {
      set_error(err, kDevErrTimeout);
      for (int r = q; r < issued; ++r) mbar_wait_bounded(&bars[r & (kSlots - 1)], (r / kSlots) & 1);
    }
    __syncwarp();
    return false;
  }
};

// Walks the items one warp claims: chunk c of pass p of item i.
// `per` = items per active expert. Items come from a global counter; the
// copy-issue cursor claims them (lane 0) and records them in a per-warp
// queue, which the compute cursor replays in the same order.
struct Cursor {
  int n_items;
  int per, sub;      // per = RB * KS (gate/up) or RBD (down); sub = KS or 1
  int nch;           // chunks per pass
  int* queue;        // [kQueue] per-warp claimed item ids (shared memory)
  int qpos;          // next queue slot this cursor reads or writes
  int i, ai, rb, ks, e, off, n, np, p, c;

  ES_DEV void load(const FfnArgs& a) {
    if (i >= n_items) return;
    ai = i / per;
    const int rem = i - ai * per;
    rb = rem / sub;
    ks = rem - rb * sub;
    e = a.act_e[ai];
    off = a.act_off[ai];
    n = a.act_n[ai];
    np = (n + kTiles * 8 - 1) / (kTiles * 8);
    p = 0;
    c = 0;
  }
  // issue side: claim the next item (whole warp)
  ES_DEV void claim(const FfnArgs& a, int* counter) {
    int v = 0;
    if ((threadIdx.x & 31) == 0) {
      v = atomicAdd(counter, 1);
      queue[qpos & (kQueue - 1)] = v;
    }
    i = __shfl_sync(0xffffffffu, v, 0);
    ++qpos;
    load(a);
  }
  // compute side: next item from the queue (whole warp)
  ES_DEV void replay(const FfnArgs& a) {
    __syncwarp();
    i = queue[qpos & (kQueue - 1)];
    ++qpos;
    load(a);
  }
  ES_DEV bool valid() const { return i < n_items; }
  // advance to the next chunk; at the end of an item, claim/replay the next
  template <bool kIssue>
  ES_DEV void advance(const FfnArgs& a, int* counter) {
    if (++c < nch) return;
    c = 0;
    if (++p < np) return;
    if (kIssue) claim(a, counter); else replay(a);
  }
};


// ---------------------------------------------------------------------------
// gate/up + SwiGLU -> h (fp16, fragment order)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kGateupWarps * 32, 1) ffn_gateup_kernel(FfnArgs a, int KS) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int GD = a.D / kGroup, RB = a.I / 16;
  const int GPI = GD / KS;  // groups per item
  WarpRing ring{smem + (size_t)warp * kSlots * kGateupChunk,
                reinterpret_cast<uint64_t*>(smem + (size_t)kGateupWarps * kSlots * kGateupChunk) +
                    warp * kSlots,
                kGateupChunk, l2_evict_first_policy()};
  ring.init();
  __shared__ int s_queue[kGateupWarps][kQueue];
  pdl_wait();
  pdl_trigger();

  const int n_items = *a.n_active * RB * KS;
  Cursor ic{n_items, RB * KS, KS, GPI / kGPC, s_queue[warp], 0};
  ic.claim(a, &a.item_ctr[0]);
  Cursor cc = ic;
  cc.qpos = 0;
  cc.replay(a);
  if (!cc.valid()) return;
  auto src = [&](const Cursor& u) {
    return a.packed + (size_t)u.e * a.expert_bytes +
           gateup_tile_off(GD, u.rb, u.ks * GPI + u.c * kGPC, 0);
  };
  int issued = 0;
  for (; issued < kSlots && ic.valid(); ++issued) {
    if (lane == 0) ring.issue(issued, src(ic));
    ic.advance<true>(a, &a.item_ctr[0]);
  }

  float acc[kTiles][8];
  int tb[kTiles], tc0[kTiles], tc1[kTiles];
  int ntile = 0;
  for (int q = 0; cc.valid(); ++q) {
    if (cc.c == 0) {  // start of a pass over 32 tokens
      const int base = cc.p * kTiles * 8;
      ntile = min(kTiles, (cc.n - base + 7) / 8);
#pragma unroll
      for (int t = 0; t < kTiles; ++t) {
#pragma unroll
        for (int v = 0; v < 8; ++v) acc[t][v] = 0.f;
        const int cb = base + t * 8 + g, cq = base + t * 8 + 2 * c;
        tb[t] = cb < cc.n ? a.pair_tok[cc.off + cb] : -1;
        tc0[t] = cq < cc.n ? a.pair_tok[cc.off + cq] : -1;
        tc1[t] = cq + 1 < cc.n ? a.pair_tok[cc.off + cq + 1] : -1;
      }
    }
    if (!ring.wait(q, issued, a.err)) return;
    const uint8_t* st = ring.slot(q);
    uint4 cg[kGPC], cu[kGPC];
    uint2 sgv[kGPC], suv[kGPC];
#pragma unroll
    for (int gi = 0; gi < kGPC; ++gi) {
      const uint8_t* tg = st + (size_t)(gi * 2) * kTileBytes;
      cg[gi] = ld_shared16(tg + lane * 16);
      cu[gi] = ld_shared16(tg + kTileBytes + lane * 16);
      sgv[gi] = ld_shared8(tg + kTileCodeBytes + g * 8);
      suv[gi] = ld_shared8(tg + kTileBytes + kTileCodeBytes + g * 8);
    }
    __syncwarp();  // slot consumed by every lane: refill it
    if (ic.valid()) {
      if (lane == 0) ring.issue(issued, src(ic));
      ic.advance<true>(a, &a.item_ctr[0]);
      ++issued;
    }
    const int G0 = cc.ks * GPI + cc.c * kGPC;
#pragma unroll
    for (int gi = 0; gi < kGPC; ++gi) {
      const int G = G0 + gi;
      const float gs0 = lo_half_f(sgv[gi].x), gs8 = lo_half_f(sgv[gi].y);
      const float gb0 = fmaf(-128.f, gs0, hi_half_f(sgv[gi].x));
      const float gb8 = fmaf(-128.f, gs8, hi_half_f(sgv[gi].y));
      const float us0 = lo_half_f(suv[gi].x), us8 = lo_half_f(suv[gi].y);
      const float ub0 = fmaf(-128.f, us0, hi_half_f(suv[gi].x));
      const float ub8 = fmaf(-128.f, us8, hi_half_f(suv[gi].y));
      // A operands of the four k-steps: rows g (words .x, .y) and g + 8 (.z, .w)
      uint32_t ag[4][4], au[4][4];
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        ag[s][0] = code_pair(cg[gi].x, s); ag[s][1] = code_pair(cg[gi].z, s);
        ag[s][2] = code_pair(cg[gi].y, s); ag[s][3] = code_pair(cg[gi].w, s);
        au[s][0] = code_pair(cu[gi].x, s); au[s][1] = code_pair(cu[gi].z, s);
        au[s][2] = code_pair(cu[gi].y, s); au[s][3] = code_pair(cu[gi].w, s);
      }
#pragma unroll
      for (int t = 0; t < kTiles; ++t) {
        if (t >= ntile) break;  // warp-uniform
        uint4 xa = make_uint4(0, 0, 0, 0), xb = xa;
        if (tb[t] >= 0) {
          const uint4* xp = reinterpret_cast<const uint4*>(a.x_perm + ((size_t)tb[t] * GD + G) * kGroup + c * 16);
          xa = __ldg(xp);
          xb = __ldg(xp + 1);
        }
        const float xs0 = tc0[t] >= 0 ? __ldg(a.xsum + (size_t)tc0[t] * GD + G) : 0.f;
        const float xs1 = tc1[t] >= 0 ? __ldg(a.xsum + (size_t)tc1[t] * GD + G) : 0.f;
        const uint32_t bw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
        float tg[4] = {0.f, 0.f, 0.f, 0.f}, tu[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          mma_bf16(tg, ag[s][0], ag[s][1], ag[s][2], ag[s][3], bw[2 * s], bw[2 * s + 1], tg);
          mma_bf16(tu, au[s][0], au[s][1], au[s][2], au[s][3], bw[2 * s], bw[2 * s + 1], tu);
        }
        acc[t][0] = fmaf(gs0, tg[0], fmaf(gb0, xs0, acc[t][0]));
        acc[t][1] = fmaf(gs0, tg[1], fmaf(gb0, xs1, acc[t][1]));
        acc[t][2] = fmaf(gs8, tg[2], fmaf(gb8, xs0, acc[t][2]));
        acc[t][3] = fmaf(gs8, tg[3], fmaf(gb8, xs1, acc[t][3]));
        acc[t][4] = fmaf(us0, tu[0], fmaf(ub0, xs0, acc[t][4]));
        acc[t][5] = fmaf(us0, tu[1], fmaf(ub0, xs1, acc[t][5]));
        acc[t][6] = fmaf(us8, tu[2], fmaf(ub8, xs0, acc[t][6]));
        acc[t][7] = fmaf(us8, tu[3], fmaf(ub8, xs1, acc[t][7]));
      }
    }

    if (cc.c == cc.nch - 1) {  // end of the pass: SwiGLU -> h
      bool last = true;
      if (KS > 1) {  // only for batches of <= 8 tokens: one pass, one tile
        const int slot = cc.ai * RB + cc.rb;
        float4* part = reinterpret_cast<float4*>(a.partials) + ((size_t)slot * KS + cc.ks) * 64;
        part[lane * 2] = make_float4(acc[0][0], acc[0][1], acc[0][2], acc[0][3]);
        part[lane * 2 + 1] = make_float4(acc[0][4], acc[0][5], acc[0][6], acc[0][7]);
        __threadfence();
        __syncwarp();
        int old = 0;
        if (lane == 0) old = atomicAdd(&a.counters[slot], 1);
        old = __shfl_sync(0xffffffffu, old, 0);
        last = old == KS - 1;
        if (last) {
          __threadfence();
#pragma unroll
          for (int v = 0; v < 8; ++v) acc[0][v] = 0.f;
          const float4* pp = reinterpret_cast<const float4*>(a.partials) + (size_t)slot * KS * 64;
          for (int k2 = 0; k2 < KS; ++k2) {  // fixed order: deterministic
            const float4 p0 = __ldcg(pp + (size_t)k2 * 64 + lane * 2);
            const float4 p1 = __ldcg(pp + (size_t)k2 * 64 + lane * 2 + 1);
            acc[0][0] += p0.x; acc[0][1] += p0.y; acc[0][2] += p0.z; acc[0][3] += p0.w;
            acc[0][4] += p1.x; acc[0][5] += p1.y; acc[0][6] += p1.z; acc[0][7] += p1.w;
          }
          if (lane == 0) a.counters[slot] = 0;
        }
      }
      if (last) {
        const int base = cc.p * kTiles * 8;
#pragma unroll
        for (int t = 0; t < kTiles; ++t) {
          if (t >= ntile) break;
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const int row = (v < 2) ? g : g + 8;
            const int col = base + t * 8 + 2 * c + (v & 1);
            if (col < cc.n) {
              const float gv = acc[t][v];
              float h = gv / (1.f + expf(-gv)) * acc[t][4 + v];
              if (!(fabsf(h) <= 65504.f)) {  // outside fp16 (or NaN): saturate, flag
                set_error(a.err, kDevErrRange);
                h = h != h ? 0.f : copysignf(65504.f, h);
              }
              a.h16[(size_t)(cc.off + col) * a.I + frag_pos(cc.rb * 16 + row)] =
                  __half_as_ushort(__float2half_rn(h));
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
__global__ void __launch_bounds__(kDownWarps * 32, 1) ffn_down_kernel(FfnArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int KG = a.I / kGroup, RBD = a.D / 16;
  WarpRing ring{smem + (size_t)warp * kSlots * kDownChunk,
                reinterpret_cast<uint64_t*>(smem + (size_t)kDownWarps * kSlots * kDownChunk) +
                    warp * kSlots,
                kDownChunk, l2_evict_first_policy()};
  ring.init();
  // The expert list comes from the front-end kernel, which completed before
  // the gate/up kernel (this kernel's predecessor) passed its own
  // pdl_wait(), so the first weight copies can be in flight while gate/up
  // finishes; only h (written by gate/up) needs pdl_wait().
  __shared__ int s_queue[kDownWarps][kQueue];
  const int n_items = *a.n_active * RBD;
  Cursor ic{n_items, RBD, 1, KG / kGPC, s_queue[warp], 0};
  ic.claim(a, &a.item_ctr[1]);
  Cursor cc = ic;
  cc.qpos = 0;
  cc.replay(a);
  const bool any = cc.valid();
  auto src = [&](const Cursor& u) {
    return a.packed + (size_t)u.e * a.expert_bytes + down_tile_off(a.D, a.I, u.rb, u.c * kGPC);
  };
  int issued = 0;
  for (; any && issued < kSlots && ic.valid(); ++issued) {
    if (lane == 0) ring.issue(issued, src(ic));
    ic.advance<true>(a, &a.item_ctr[1]);
  }
  pdl_wait();
  pdl_trigger();
  if (!any) return;

  float acc[kTiles][4];
  int pb[kTiles];
  int ntile = 0;
  for (int q = 0; cc.valid(); ++q) {
    if (cc.c == 0) {
      const int base = cc.p * kTiles * 8;
      ntile = min(kTiles, (cc.n - base + 7) / 8);
#pragma unroll
      for (int t = 0; t < kTiles; ++t) {
#pragma unroll
        for (int v = 0; v < 4; ++v) acc[t][v] = 0.f;
        const int col = base + t * 8 + g;
        pb[t] = col < cc.n ? cc.off + col : -1;
      }
    }
    if (!ring.wait(q, issued, a.err)) return;
    const uint8_t* st = ring.slot(q);
    uint4 cw[kGPC];
    uint2 sw[kGPC];
#pragma unroll
    for (int gi = 0; gi < kGPC; ++gi) {
      cw[gi] = ld_shared16(st + (size_t)gi * kTileBytes + lane * 16);
      sw[gi] = ld_shared8(st + (size_t)gi * kTileBytes + kTileCodeBytes + g * 8);
    }
    __syncwarp();
    if (ic.valid()) {
      if (lane == 0) ring.issue(issued, src(ic));
      ic.advance<true>(a, &a.item_ctr[1]);
      ++issued;
    }
    const int G0 = cc.c * kGPC;
#pragma unroll
    for (int gi = 0; gi < kGPC; ++gi) {
      const int G = G0 + gi;
      const float s0 = lo_half_f(sw[gi].x), s8 = lo_half_f(sw[gi].y);
      const float b0 = fmaf(-1024.f, s0, hi_half_f(sw[gi].x));
      const float b8 = fmaf(-1024.f, s8, hi_half_f(sw[gi].y));
      uint32_t ao[4][4];
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        ao[s][0] = code_pair_f16(cw[gi].x, s); ao[s][1] = code_pair_f16(cw[gi].z, s);
        ao[s][2] = code_pair_f16(cw[gi].y, s); ao[s][3] = code_pair_f16(cw[gi].w, s);
      }
#pragma unroll
      for (int t = 0; t < kTiles; ++t) {
        if (t >= ntile) break;  // warp-uniform
        uint4 h0 = make_uint4(0, 0, 0, 0), h1 = h0;
        if (pb[t] >= 0) {
          const uint4* hp = reinterpret_cast<const uint4*>(a.h16 + (size_t)pb[t] * a.I + G * kGroup + c * 16);
          h0 = hp[0];
          h1 = hp[1];
        }
        const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
        float hs = 0.f;
#pragma unroll
        for (int v = 0; v < 8; ++v) hs += lo_half_f(hw[v]) + hi_half_f(hw[v]);
        hs += __shfl_xor_sync(full, hs, 1);
        hs += __shfl_xor_sync(full, hs, 2);
        const float hs0 = __shfl_sync(full, hs, (2 * c) << 2);
        const float hs1 = __shfl_sync(full, hs, (2 * c + 1) << 2);
        float tmp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int s = 0; s < 4; ++s)
          mma_f16(tmp, ao[s][0], ao[s][1], ao[s][2], ao[s][3], hw[2 * s], hw[2 * s + 1], tmp);
        acc[t][0] = fmaf(s0, tmp[0], fmaf(b0, hs0, acc[t][0]));
        acc[t][1] = fmaf(s0, tmp[1], fmaf(b0, hs1, acc[t][1]));
        acc[t][2] = fmaf(s8, tmp[2], fmaf(b8, hs0, acc[t][2]));
        acc[t][3] = fmaf(s8, tmp[3], fmaf(b8, hs1, acc[t][3]));
      }
    }
    if (cc.c == cc.nch - 1) {  // end of the pass: store y rows
      const int base = cc.p * kTiles * 8;
#pragma unroll
      for (int t = 0; t < kTiles; ++t) {
        if (t >= ntile) break;
        const int col = base + t * 8 + 2 * c;
        float* y0 = a.y_pair + (size_t)(cc.off + col) * a.D + cc.rb * 16;
        if (col < cc.n) { y0[g] = acc[t][0]; y0[g + 8] = acc[t][2]; }
        if (col + 1 < cc.n) { y0[a.D + g] = acc[t][1]; y0[a.D + g + 8] = acc[t][3]; }
      }
    }
    cc.advance<false>(a, nullptr);
  }
}

template <typename K, typename... Args>
cudaError_t launch_ring_kernel(K kernel, int warps, uint32_t chunk, int max_items,
                               cudaStream_t st, Args... args) {
  const size_t smem = (size_t)warps * kSlots * (chunk + 8);
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  int grid = sm_count();
  const int need = (max_items + warps - 1) / warps;
  if (grid > need) grid = need;
  if (grid < 1) grid = 1;
  // items are claimed from a counter the front end zeroed
  return launch_pdl(kernel, dim3(grid), dim3(warps * 32), smem, st, args...);
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

int ffn_split_k(int T, int max_active, int D, int I) {
  const int GD = D / kGroup, RB = I / 16;
  if (T > kSplitKMaxTokens) return 1;
  const int warps = sm_count() * kGateupWarps;
  int ks = 1;
  while (ks < kMaxSplitK && GD % (ks * 2 * kGPC) == 0 && (long long)max_active * RB * ks < warps)
    ks *= 2;
  return ks;
}

cudaError_t launch_ffn_gateup(const FfnArgs& a, int max_active, cudaStream_t st) {
  if (max_active <= 0) return cudaSuccess;
  const int KS = a.split_k;
  return launch_ring_kernel(ffn_gateup_kernel, kGateupWarps, kGateupChunk,
                            max_active * (a.I / 16) * KS, st, a, KS);
}

cudaError_t launch_ffn_down(const FfnArgs& a, int max_active, cudaStream_t st) {
  if (max_active <= 0) return cudaSuccess;
  return launch_ring_kernel(ffn_down_kernel, kDownWarps, kDownChunk, max_active * (a.D / 16), st, a);
}

}  // namespace es
