// Decode expert FFN: 4-bit dequant-GEMV on register operands.
//
// Restates the three gather_qmm calls of run_expert_ffn
// (src/mlx_expert_sniper/engine.py:32-39) and the SwiGLU between them
// (engine.py:37) for every active expert, grouped by expert so each packed
// weight byte is read from HBM once per call no matter how many tokens chose
// the expert.
//
// Arithmetic. A code q becomes the exact bf16 value 128 + q (es_common.cuh),
// so the tensor core computes acc = sum_d (128 + q_d) x_d exactly in fp32
// from bf16 inputs, and per (row, 64-group)
//     sum_d w_d x_d = scale * acc + (bias - 128 * scale) * sum_d x_d ,
// which is the MLX dequantisation w = scale * q + bias with no rounding of
// the weights. The group sums of x are precomputed by the router kernel; the
// down projection takes h as bf16 hi + bf16 lo (two MMAs into one
// accumulator), keeping h to ~16 bits of mantissa.
//
// Work split. Every warp loads exactly four 64-column groups of one 16-row
// block (its whole weight share) up front into registers, so at decode sizes
// each SM has tens of KB of loads in flight. gate/up: a CTA owns (active
// expert, 16 rows of I); its warps split the D/64 groups and reduce through
// shared memory, then apply SwiGLU. down: a CTA owns (active expert, R blocks
// of 16 rows of D); I/256 warps split each block's groups. Tokens of an expert
// are taken 16 at a time (two n8 tiles) against the weights held in
// registers, so weights are read once however many tokens chose the expert.
#include "es_common.cuh"
#include "es_kernels.cuh"

namespace es {
namespace {

constexpr int kGPW = 4;        // gate/up: groups per warp
constexpr int kNT = 2;         // n8 token tiles per pass

// NWARP * 32 threads at <= 128 registers each (2 CTAs per SM at D = 2048)
template <int NWARP>
__global__ void __launch_bounds__(NWARP * 32, NWARP <= 8 ? 16 / NWARP : 1) ffn_gateup_kernel(FfnArgs a) {
  extern __shared__ __align__(16) float red[];  // [NWARP][kNT][32][8]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int GD = a.D / kGroup, RB = a.I / 16;
  const int ai = blockIdx.x / RB, rb = blockIdx.x - ai * RB;
  if (ai >= *a.n_active) return;  // block-uniform
  const int e = a.act_e[ai], off = a.act_off[ai], n = a.act_n[ai];
  const uint8_t* eb = a.packed + (size_t)e * a.expert_bytes;

  uint4 cg[kGPW], cu[kGPW];
  uint2 sgv[kGPW], suv[kGPW];
#pragma unroll
  for (int gi = 0; gi < kGPW; ++gi) {
    const int G = warp * kGPW + gi;
    const uint8_t* tg = eb + gateup_tile_off(GD, rb, G, 0);
    cg[gi] = ld_stream16(tg + lane * 16);
    cu[gi] = ld_stream16(tg + kTileBytes + lane * 16);
    sgv[gi] = ld_stream8(tg + kTileCodeBytes + g * 8);
    suv[gi] = ld_stream8(tg + kTileBytes + kTileCodeBytes + g * 8);
  }

  for (int base = 0; base < n; base += kNT * 8) {
    float ag[kNT][4], au[kNT][4];
    int tb[kNT], tc0[kNT], tc1[kNT];
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt) {
#pragma unroll
      for (int i = 0; i < 4; ++i) { ag[nt][i] = 0.f; au[nt][i] = 0.f; }
      const int colb = base + nt * 8 + g;
      const int colc = base + nt * 8 + 2 * c;
      tb[nt] = colb < n ? a.pair_tok[off + colb] : -1;
      tc0[nt] = colc < n ? a.pair_tok[off + colc] : -1;
      tc1[nt] = colc + 1 < n ? a.pair_tok[off + colc + 1] : -1;
    }
#pragma unroll
    for (int gi = 0; gi < kGPW; ++gi) {
      const int G = warp * kGPW + gi;
      const float gs0 = lo_half_f(sgv[gi].x), gs8 = lo_half_f(sgv[gi].y);
      const float gb0 = fmaf(-128.f, gs0, hi_half_f(sgv[gi].x));
      const float gb8 = fmaf(-128.f, gs8, hi_half_f(sgv[gi].y));
      const float us0 = lo_half_f(suv[gi].x), us8 = lo_half_f(suv[gi].y);
      const float ub0 = fmaf(-128.f, us0, hi_half_f(suv[gi].x));
      const float ub8 = fmaf(-128.f, us8, hi_half_f(suv[gi].y));
      // A operands of the four k-steps: rows g (words .x, .y) and g + 8 (.z, .w)
      uint32_t ag_op[4][4], au_op[4][4];
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        ag_op[s][0] = code_pair(cg[gi].x, s); ag_op[s][1] = code_pair(cg[gi].z, s);
        ag_op[s][2] = code_pair(cg[gi].y, s); ag_op[s][3] = code_pair(cg[gi].w, s);
        au_op[s][0] = code_pair(cu[gi].x, s); au_op[s][1] = code_pair(cu[gi].z, s);
        au_op[s][2] = code_pair(cu[gi].y, s); au_op[s][3] = code_pair(cu[gi].w, s);
      }
#pragma unroll
      for (int nt = 0; nt < kNT; ++nt) {
        uint4 xa = make_uint4(0, 0, 0, 0), xb = make_uint4(0, 0, 0, 0);
        if (tb[nt] >= 0) {
          const uint4* xp = reinterpret_cast<const uint4*>(a.x_perm + ((size_t)tb[nt] * GD + G) * kGroup + c * 16);
          xa = __ldg(xp);
          xb = __ldg(xp + 1);
        }
        const float xs0 = tc0[nt] >= 0 ? __ldg(a.xsum + (size_t)tc0[nt] * GD + G) : 0.f;
        const float xs1 = tc1[nt] >= 0 ? __ldg(a.xsum + (size_t)tc1[nt] * GD + G) : 0.f;
        const uint32_t bw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
        float tg[4] = {0.f, 0.f, 0.f, 0.f}, tu[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          mma_bf16(tg, ag_op[s][0], ag_op[s][1], ag_op[s][2], ag_op[s][3], bw[2 * s], bw[2 * s + 1], tg);
          mma_bf16(tu, au_op[s][0], au_op[s][1], au_op[s][2], au_op[s][3], bw[2 * s], bw[2 * s + 1], tu);
        }
        ag[nt][0] = fmaf(gs0, tg[0], fmaf(gb0, xs0, ag[nt][0]));
        ag[nt][1] = fmaf(gs0, tg[1], fmaf(gb0, xs1, ag[nt][1]));
        ag[nt][2] = fmaf(gs8, tg[2], fmaf(gb8, xs0, ag[nt][2]));
        ag[nt][3] = fmaf(gs8, tg[3], fmaf(gb8, xs1, ag[nt][3]));
        au[nt][0] = fmaf(us0, tu[0], fmaf(ub0, xs0, au[nt][0]));
        au[nt][1] = fmaf(us0, tu[1], fmaf(ub0, xs1, au[nt][1]));
        au[nt][2] = fmaf(us8, tu[2], fmaf(ub8, xs0, au[nt][2]));
        au[nt][3] = fmaf(us8, tu[3], fmaf(ub8, xs1, au[nt][3]));
      }
    }
    // cross-warp reduction of the K split
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt) {
      float4* r = reinterpret_cast<float4*>(red + (((size_t)warp * kNT + nt) * 32 + lane) * 8);
      r[0] = make_float4(ag[nt][0], ag[nt][1], ag[nt][2], ag[nt][3]);
      r[1] = make_float4(au[nt][0], au[nt][1], au[nt][2], au[nt][3]);
    }
    __syncthreads();
    if (threadIdx.x < kNT * 32) {
      const int nt = threadIdx.x >> 5, ln = threadIdx.x & 31;
      float gsum[4] = {0.f, 0.f, 0.f, 0.f}, usum[4] = {0.f, 0.f, 0.f, 0.f};
      for (int w = 0; w < NWARP; ++w) {
        const float4* q = reinterpret_cast<const float4*>(red + (((size_t)w * kNT + nt) * 32 + ln) * 8);
        const float4 q0 = q[0], q1 = q[1];
        gsum[0] += q0.x; gsum[1] += q0.y; gsum[2] += q0.z; gsum[3] += q0.w;
        usum[0] += q1.x; usum[1] += q1.y; usum[2] += q1.z; usum[3] += q1.w;
      }
      const int g2 = ln >> 2, c2 = ln & 3;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = (i < 2) ? g2 : g2 + 8;
        const int col = base + nt * 8 + 2 * c2 + (i & 1);
        if (col < n) {
          const float gv = gsum[i];
          const float h = gv / (1.f + expf(-gv)) * usum[i];
          const uint16_t hi = float_to_bf16_bits(h);
          const uint16_t lo = float_to_bf16_bits(h - bf16_bits_to_float(hi));
          const size_t idx = (size_t)(off + col) * a.I + frag_pos(rb * 16 + row);
          a.h_hi[idx] = hi;
          a.h_lo[idx] = lo;
        }
      }
    }
    __syncthreads();
  }
}

// down: R row blocks per CTA, KC warps per row block, each warp 4 groups of I.
template <int KC>
struct DownShape {
  static constexpr int R = KC <= 4 ? 4 : 2;
  static constexpr int WARPS = R * KC;
};

template <int KC>
__global__ void __launch_bounds__(DownShape<KC>::WARPS * 32) ffn_down_kernel(FfnArgs a) {
  constexpr int R = DownShape<KC>::R;
  extern __shared__ __align__(16) float red[];  // [R*KC][kNT][32][4]
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int rbl = warp / KC, kc = warp - rbl * KC;
  const int CPB = (a.D / 16) / R;  // CTAs per expert
  const int ai = blockIdx.x / CPB;
  const int rb = (blockIdx.x - ai * CPB) * R + rbl;
  if (ai >= *a.n_active) return;  // block-uniform
  const int e = a.act_e[ai], off = a.act_off[ai], n = a.act_n[ai];
  const uint8_t* tb = a.packed + (size_t)e * a.expert_bytes + down_tile_off(a.D, a.I, rb, kc * kGPW);

  uint4 cw[kGPW];
  uint2 sw[kGPW];
#pragma unroll
  for (int gi = 0; gi < kGPW; ++gi) {
    cw[gi] = ld_stream16(tb + (size_t)gi * kTileBytes + lane * 16);
    sw[gi] = ld_stream8(tb + (size_t)gi * kTileBytes + kTileCodeBytes + g * 8);
  }

  for (int base = 0; base < n; base += kNT * 8) {
    float acc[kNT][4];
    int pb[kNT];
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt) {
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[nt][i] = 0.f;
      const int col = base + nt * 8 + g;
      pb[nt] = col < n ? off + col : -1;
    }
#pragma unroll
    for (int gi = 0; gi < kGPW; ++gi) {
      const int G = kc * kGPW + gi;
      const float s0 = lo_half_f(sw[gi].x), s8 = lo_half_f(sw[gi].y);
      const float b0 = fmaf(-128.f, s0, hi_half_f(sw[gi].x));
      const float b8 = fmaf(-128.f, s8, hi_half_f(sw[gi].y));
      uint32_t a_op[4][4];
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        a_op[s][0] = code_pair(cw[gi].x, s); a_op[s][1] = code_pair(cw[gi].z, s);
        a_op[s][2] = code_pair(cw[gi].y, s); a_op[s][3] = code_pair(cw[gi].w, s);
      }
#pragma unroll
      for (int nt = 0; nt < kNT; ++nt) {
        uint4 h0 = make_uint4(0, 0, 0, 0), h1 = h0, l0 = h0, l1 = h0;
        if (pb[nt] >= 0) {
          const size_t o = (size_t)pb[nt] * a.I + G * kGroup + c * 16;
          const uint4* hp = reinterpret_cast<const uint4*>(a.h_hi + o);
          const uint4* lp = reinterpret_cast<const uint4*>(a.h_lo + o);
          h0 = hp[0]; h1 = hp[1]; l0 = lp[0]; l1 = lp[1];
        }
        const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
        const uint32_t lw[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
        float hs = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          hs += bf16_bits_to_float(hw[i] & 0xffffu) + bf16_bits_to_float(hw[i] >> 16);
          hs += bf16_bits_to_float(lw[i] & 0xffffu) + bf16_bits_to_float(lw[i] >> 16);
        }
        hs += __shfl_xor_sync(full, hs, 1);
        hs += __shfl_xor_sync(full, hs, 2);
        const float hs0 = __shfl_sync(full, hs, (2 * c) << 2);
        const float hs1 = __shfl_sync(full, hs, (2 * c + 1) << 2);
        float tmp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          mma_bf16(tmp, a_op[s][0], a_op[s][1], a_op[s][2], a_op[s][3], hw[2 * s], hw[2 * s + 1], tmp);
          mma_bf16(tmp, a_op[s][0], a_op[s][1], a_op[s][2], a_op[s][3], lw[2 * s], lw[2 * s + 1], tmp);
        }
        acc[nt][0] = fmaf(s0, tmp[0], fmaf(b0, hs0, acc[nt][0]));
        acc[nt][1] = fmaf(s0, tmp[1], fmaf(b0, hs1, acc[nt][1]));
        acc[nt][2] = fmaf(s8, tmp[2], fmaf(b8, hs0, acc[nt][2]));
        acc[nt][3] = fmaf(s8, tmp[3], fmaf(b8, hs1, acc[nt][3]));
      }
    }
    // reduce the KC partial sums of each row block, in kc order
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt)
      reinterpret_cast<float4*>(red)[((size_t)warp * kNT + nt) * 32 + lane] =
          make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]);
    __syncthreads();
    if (threadIdx.x < R * kNT * 32) {
      const int r2 = threadIdx.x / (kNT * 32);
      const int nt = (threadIdx.x >> 5) % kNT, ln = threadIdx.x & 31;
      float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int k2 = 0; k2 < KC; ++k2) {
        const float4 q = reinterpret_cast<const float4*>(red)[((size_t)(r2 * KC + k2) * kNT + nt) * 32 + ln];
        sum.x += q.x; sum.y += q.y; sum.z += q.z; sum.w += q.w;
      }
      const int g2 = ln >> 2, c2 = ln & 3;
      const int rbo = (blockIdx.x - ai * CPB) * R + r2;
      const int col = base + nt * 8 + 2 * c2;
      float* y0 = a.y_pair + (size_t)(off + col) * a.D + rbo * 16;
      if (col < n) { y0[g2] = sum.x; y0[g2 + 8] = sum.z; }
      if (col + 1 < n) { y0[a.D + g2] = sum.y; y0[a.D + g2 + 8] = sum.w; }
    }
    __syncthreads();
  }
}

template <int NWARP>
cudaError_t launch_gateup_nw(const FfnArgs& a, int max_active, cudaStream_t st) {
  const size_t smem = (size_t)NWARP * kNT * 32 * 8 * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(ffn_gateup_kernel<NWARP>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  ffn_gateup_kernel<NWARP><<<max_active * (a.I / 16), NWARP * 32, smem, st>>>(a);
  return cudaGetLastError();
}

template <int KC>
cudaError_t launch_down_kc(const FfnArgs& a, int max_active, cudaStream_t st) {
  constexpr int R = DownShape<KC>::R, WARPS = DownShape<KC>::WARPS;
  const int CPB = (a.D / 16) / R;
  const size_t smem = (size_t)WARPS * kNT * 32 * 4 * sizeof(float);
  ffn_down_kernel<KC><<<max_active * CPB, WARPS * 32, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_ffn_gateup(const FfnArgs& a, int max_active, cudaStream_t st) {
  if (max_active <= 0) return cudaSuccess;
  switch ((a.D / kGroup) / kGPW) {
    case 1: return launch_gateup_nw<1>(a, max_active, st);
    case 2: return launch_gateup_nw<2>(a, max_active, st);
    case 4: return launch_gateup_nw<4>(a, max_active, st);
    case 8: return launch_gateup_nw<8>(a, max_active, st);
    case 16: return launch_gateup_nw<16>(a, max_active, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_ffn_down(const FfnArgs& a, int max_active, cudaStream_t st) {
  if (max_active <= 0) return cudaSuccess;
  switch ((a.I / kGroup) / kGPW) {
    case 1: return launch_down_kc<1>(a, max_active, st);
    case 2: return launch_down_kc<2>(a, max_active, st);
    case 3: return launch_down_kc<3>(a, max_active, st);
    case 4: return launch_down_kc<4>(a, max_active, st);
    case 6: return launch_down_kc<6>(a, max_active, st);
    case 8: return launch_down_kc<8>(a, max_active, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace es
