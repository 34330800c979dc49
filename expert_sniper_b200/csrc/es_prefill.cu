// Tensor-core path of the MoE block: the expert FFN as a grouped GEMM on the
// 5th-generation tensor cores (tcgen05.mma, accumulators in tensor memory),
// with the 4-bit weights dequantised to fp16 on the way. Two variants of the
// GEMM share this file (template parameter TA):
//   large batches (prefill): 128-token tiles, the dequantised weights in
//     128-byte-swizzled shared memory;
//   small batches (from 4 pairs per routed expert): 32-token tiles, the
//     dequantised weights written straight into tensor memory and read
//     from there by the MMA (A operand in TMEM), several quantisation
//     groups per pipeline stage (2 for gate/up, 4 for down: 18 KB of codes
//     either way).
//
// Restates the same math as the decode kernels (engine.py:32-41 gather_qmm
// gate/up, SwiGLU, gather_qmm down; generate.py:173-178 shared expert), for
// batches where each expert sees enough tokens that one weight read feeds a
// tensor-core tile.
//
// Kernels, in launch order (one stream, programmatic dependent launches):
//   pf_front    router (generate.py:122-136) per token; per-expert slot
//               counters (atomicAdd -- the rank inside an expert's list is
//               arbitrary, which changes where a pair's rows live but not any
//               value: every GEMM column and the combine's expert-id-ordered
//               sum are independent of it); activations to fp16 with a
//               per-token power-of-two scale, in nibble order. The last CTA
//               scans the counts into expert offsets and the active list.
//   pf_scatter  slot -> pair index, pair -> token.
//   pf_gemm<1>  gate/up: per unit (expert, 128 rows of I, one token tile) two
//               accumulators [128 x N] in TMEM; epilogue SwiGLU -> fp16 h.
//   pf_gemm<0>  down: per unit (expert, 128 rows of D, one token tile) one
//               accumulator; epilogue -> fp16 per-pair rows (saturated
//               and flagged beyond the fp16 range, as h is).
//   combine     (es_combine.cu) fixed expert-id order, fp32.
//
// GEMM orientation: A = weights (M = 128 rows, K-major), B = activations of
// the unit's tokens (N = tokens rounded up to 16, K-major, gathered rows in
// 128-byte-swizzled shared memory), D = A * B^T in TMEM (lane = weight row,
// column = token). Weights are the large operand and are read from HBM
// exactly once per token tile.
//
// Warp roles of the persistent CTA (24 warps, one CTA per SM):
//   warp 0      copies the packed code tiles of each stage into a ring
//               (raw_full / raw_empty): one 5-D TMA load per stage, the
//               unit's runs of four 576-byte tiles for the stage's groups
//   warp 1      allocates TMEM; one lane issues tcgen05.mma and commits
//   warps 2-3   load the B rows into their ring: gate/up gathers token rows
//               of x16 with cp.async (completion tracked on the ring's
//               mbarrier), down copies consecutive pair rows of h16 with
//               one TMA tile load per quantisation group
//   warps 4-7   epilogue: tcgen05.ld from TMEM, math, global stores
//   warps 8-23  dequantise codes -> fp16 A: large tiles, gate/up all
//               sixteen warps on every stage, one per (16-row block,
//               projection), down two groups of eight warps taking alternate
//               stages, one 16-row block per warp (st.shared in the swizzled
//               layout); small tiles, one warp
//               per (TMEM lane quarter, quantisation group of the stage),
//               one weight row per thread (tcgen05.st) -- gate/up two groups
//               of eight warps taking alternate stages, down all sixteen
//               warps on every stage
// Every wait is bounded (ES_DEVERR_TIMEOUT); on a timeout each role stops,
// copies in flight are waited for, and TMEM is freed before returning.
#include <cudaTypedefs.h>

#include <mutex>

#include "es_common.cuh"
#include "es_kernels.cuh"
#include "es_route.cuh"

namespace es {
namespace {

// ---------------------------------------------------------------------------
// tcgen05 / async-copy primitives
// ---------------------------------------------------------------------------
ES_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
ES_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

ES_DEV void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                   smem_addr(dst)),
               "r"(ncols)
               : "memory");
}
ES_DEV void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
ES_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, fp16 inputs, fp32 accumulate
ES_DEV void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                     uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T: A is read from tensor memory (lane = row
// of A, each 32-bit column two consecutive K elements), B from shared memory
ES_DEV void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                        uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 TMEM lanes x 32 consecutive 32-bit columns from registers: thread i of
// the warp writes lane (base lane + i), columns col .. col + 31
ES_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// waits until this thread's tcgen05.st writes are done
ES_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

// mbarrier arrives once every tcgen05 op issued so far by this thread is done
ES_DEV void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
          smem_addr(bar))
      : "memory");
}

// 32 TMEM lanes x 16 consecutive 32-bit columns: thread i of the warp gets
// lane (base lane + i), columns col .. col + 15
ES_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// waits for this thread's tcgen05.ld; the registers pass through an empty
// volatile asm after the wait so no use of them is scheduled before it
ES_DEV void tmem_wait_ld(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) opaque(r[i]);
}

ES_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_addr(bar)) : "memory");
}

ES_DEV void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_addr(dst)), "l"(src)
               : "memory");
}
// the mbarrier's pending count is raised now and lowered when every
// cp.async issued so far by this thread has landed
ES_DEV void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.shared::cta.b64 [%0];\n" ::"r"(smem_addr(bar))
               : "memory");
}
ES_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }


// generic-proxy writes to shared memory -> visible to the tensor core's reads
ES_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

// Shared-memory matrix descriptor: K-major rows of 128 bytes (64 fp16),
// 128-byte swizzle (16-byte chunk c of row r stored at chunk c ^ (r & 7)),
// 8-row groups 1024 bytes apart. The tile base is 1024-byte aligned.
ES_DEV uint64_t sw128_desc(const void* p) {
  const uint32_t a = smem_addr(p);
  return (uint64_t)((a & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) |
         ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor: fp16 A and B (K-major), fp32 D, M = 128, N = n.
ES_DEV uint32_t idesc_f16_m128(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// ---------------------------------------------------------------------------
// Dequantisation of one packed word (8 codes of one row) to fp16 in nibble
// order: (q0,q4) (q1,q5) (q2,q6) (q3,q7) as four half2, w = scale * q + bias.
// 0x6400 | q is exactly 1024 + q in fp16, so the subtraction is exact and the
// fused multiply-add rounds once.
// ---------------------------------------------------------------------------
ES_DEV uint32_t nib_or(uint32_t w) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(r) : "r"(w), "r"(0x000F000Fu), "r"(0x64006400u));
  return r;
}
ES_DEV uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
ES_DEV __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

ES_DEV uint4 dequant_word(uint32_t w, __half2 s2, __half2 b2) {
  const __half2 k1024 = bits_h2(0x64006400u);
  uint4 o;
  o.x = h2_bits(__hfma2(__hsub2(bits_h2(nib_or(w)), k1024), s2, b2));
  o.y = h2_bits(__hfma2(__hsub2(bits_h2(nib_or(w >> 4)), k1024), s2, b2));
  o.z = h2_bits(__hfma2(__hsub2(bits_h2(nib_or(w >> 8)), k1024), s2, b2));
  o.w = h2_bits(__hfma2(__hsub2(bits_h2(nib_or(w >> 12)), k1024), s2, b2));
  return o;
}

ES_DEV void st_shared16(void* p, uint4 v) { *reinterpret_cast<uint4*>(p) = v; }

// ---------------------------------------------------------------------------
// Front end
// ---------------------------------------------------------------------------
constexpr int kFrontWarps = 16;
constexpr int kFrontThreads = kFrontWarps * 32;

// x row (bf16, or fp16 with x_f16) -> fp16 in nibble order, scaled by 2^s
// so that the row's largest magnitude lies in [2^14, 2^15): no overflow, and
// fp16's 11-bit significand holds every bf16 value of the row exactly down to
// 2^-28 of the maximum (fp16 input: every value down to 2^-25 of it). inv =
// 2^-s is undone exactly on the fp32 accumulators. Rows with a non-finite
// maximum keep s = 0 (NaN / inf propagate as in the reference).
ES_DEV float x_lo(uint32_t w, bool f16) {
  return f16 ? __half2float(__ushort_as_half((uint16_t)(w & 0xffffu))) : __uint_as_float(w << 16);
}
ES_DEV float x_hi(uint32_t w, bool f16) {
  return f16 ? __half2float(__ushort_as_half((uint16_t)(w >> 16))) : __uint_as_float(w & 0xffff0000u);
}

// One pass over the row: the lane's 16-byte chunks (D / 256 of them, at most
// kMaxRowChunks) are loaded once into registers, then reduced and converted.
constexpr int kMaxRowChunks = 16;  // D <= 4096

// the lane's chunks of row xr into registers (issued early, used later)
ES_DEV void x_row_load(const uint16_t* xr, int D, uint4 (&v)[kMaxRowChunks]) {
  const int lane = threadIdx.x & 31;
  const uint4* x4 = reinterpret_cast<const uint4*>(xr);
  const int nch = D / 8;
#pragma unroll
  for (int i = 0; i < kMaxRowChunks; ++i) {
    const int c = lane + 32 * i;
    v[i] = c < nch ? x4[c] : make_uint4(0, 0, 0, 0);
  }
}

ES_DEV void x_row_to_f16(const uint4 (&v)[kMaxRowChunks], uint16_t* outr, float* inv_out, int D,
                         bool f16) {
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const int nch = D / 8;
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxRowChunks; ++i) {
    const uint32_t ws[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      m = fmaxf(m, fabsf(x_lo(ws[q], f16)));
      m = fmaxf(m, fabsf(x_hi(ws[q], f16)));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(full, m, o));
  int s = 0;
  if (m > 0.f && m <= 3.4e38f) {
    const int e = (int)((__float_as_uint(m) >> 23) & 0xffu) - 127;
    s = 14 - e;
    s = s < -100 ? -100 : (s > 100 ? 100 : s);
  }
  const float scale = __uint_as_float((uint32_t)(127 + s) << 23);
  if (lane == 0) *inv_out = __uint_as_float((uint32_t)(127 - s) << 23);
  uint4* o4 = reinterpret_cast<uint4*>(outr);
#pragma unroll
  for (int i = 0; i < kMaxRowChunks; ++i) {
    const int c = lane + 32 * i;
    if (c >= nch) break;
    // elements e0..e7: v.x = (e0, e1), v.y = (e2, e3), v.z = (e4, e5), v.w = (e6, e7)
    const float e0 = x_lo(v[i].x, f16) * scale, e1 = x_hi(v[i].x, f16) * scale;
    const float e2 = x_lo(v[i].y, f16) * scale, e3 = x_hi(v[i].y, f16) * scale;
    const float e4 = x_lo(v[i].z, f16) * scale, e5 = x_hi(v[i].z, f16) * scale;
    const float e6 = x_lo(v[i].w, f16) * scale, e7 = x_hi(v[i].w, f16) * scale;
    uint4 o;
    o.x = h2_bits(__floats2half2_rn(e0, e4));
    o.y = h2_bits(__floats2half2_rn(e1, e5));
    o.z = h2_bits(__floats2half2_rn(e2, e6));
    o.w = h2_bits(__floats2half2_rn(e3, e7));
    o4[c] = o;
  }
}

template <int VPL>
__global__ void __launch_bounds__(kFrontThreads) pf_front_kernel(RouteArgs r, PfFrontArgs d) {
  __shared__ int s_off[kMaxExperts + 2];
  __shared__ int s_wc[kFrontWarps];
  __shared__ int s_wf[kFrontWarps];
  __shared__ int s_last;
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, tid = threadIdx.x;
  const int E = r.E, k = r.k;
  pdl_wait();
  pdl_trigger();

  for (int t = blockIdx.x * kFrontWarps + warp; t < r.T; t += gridDim.x * kFrontWarps) {
    // the token's activation row is loaded first so that its latency overlaps
    // the routing
    uint4 xv[kMaxRowChunks];
    x_row_load(r.x + (size_t)t * r.D, r.D, xv);
    int my_e = -1;
    float my_w = 0.f;
    if (r.logits) {
      route_token_warp<VPL>(r.logits, r.logits_f32, r.bias, t, E, k, r.renorm, r.err, my_e, my_w);
      if (lane < k && r.out_idx) {
        r.out_idx[(size_t)t * k + lane] = my_e;
        r.out_w[(size_t)t * k + lane] = my_w;
      }
    } else if (lane < k) {
      my_e = r.in_idx[(size_t)t * k + lane];
      my_w = r.in_w[(size_t)t * k + lane];
      if (my_e < -1 || my_e >= E) {
        set_error(r.err, 0x1u);
        my_e = -1;
      }
    }
    const int pos = sort_slots_warp(d.cs_pos, d.cs_w, k, t, my_e, my_w);
    if (lane < k && my_e >= 0) d.rank[(size_t)t * k + pos] = atomicAdd(&d.cnt[my_e], 1);
    if (r.has_shared) {
      const float gsg = shared_gate_warp(r.x + (size_t)t * r.D, r.sg_w, r.D, r.x_f16 != 0);
      if (lane == 0) r.sgate[t] = gsg;
    }
    x_row_to_f16(xv, r.x_perm + (size_t)t * r.D, r.xsum + t, r.D, r.x_f16 != 0);
  }

  // the last CTA turns the counts into offsets and the active list. The
  // block barrier orders every thread's writes before thread 0's fence and
  // ticket (one fence per CTA, as in a grid sync); the last CTA's thread 0
  // fences again before its threads read.
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    s_last = atomicAdd(d.ticket, 1) == (int)gridDim.x - 1;
    if (s_last) __threadfence();
  }
  __syncthreads();
  if (!s_last) return;
  const int E1 = E + (r.has_shared ? 1 : 0);
  for (int e = tid; e < E1; e += kFrontThreads) {
    s_off[e] = e < E ? __ldcg(d.cnt + e) : r.T;
    if (e < E) d.cnt[e] = 0;
  }
  __syncthreads();
  const int EPT = (E1 + kFrontThreads - 1) / kFrontThreads;
  const int e_lo = tid * EPT;
  int vc = 0, vf = 0;
  for (int q = 0; q < EPT; ++q)
    if (e_lo + q < E1) { vc += s_off[e_lo + q]; vf += s_off[e_lo + q] > 0; }
  const int my_c = vc, my_f = vf;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int nc = __shfl_up_sync(full, vc, o);
    const int nf = __shfl_up_sync(full, vf, o);
    if (lane >= o) { vc += nc; vf += nf; }
  }
  if (lane == 31) { s_wc[warp] = vc; s_wf[warp] = vf; }
  __syncthreads();
  if (warp == 0) {
    int wc = lane < kFrontWarps ? s_wc[lane] : 0, wf = lane < kFrontWarps ? s_wf[lane] : 0;
#pragma unroll
    for (int o = 1; o < kFrontWarps; o <<= 1) {
      const int nc = __shfl_up_sync(full, wc, o);
      const int nf = __shfl_up_sync(full, wf, o);
      if (lane >= o) { wc += nc; wf += nf; }
    }
    if (lane < kFrontWarps) { s_wc[lane] = wc; s_wf[lane] = wf; }
  }
  __syncthreads();
  int run_c = (warp > 0 ? s_wc[warp - 1] : 0) + vc - my_c;
  int run_f = (warp > 0 ? s_wf[warp - 1] : 0) + vf - my_f;
  for (int q = 0; q < EPT; ++q) {
    const int e = e_lo + q;
    if (e >= E1) break;
    const int cnt = s_off[e];
    d.off_e[e] = run_c;
    s_off[e] = run_c;  // the thread's own experts only: counts become offsets
    if (cnt > 0) {
      d.act_e[run_f] = e;
      d.act_off[run_f] = run_c;
      d.act_n[run_f] = cnt;
      ++run_f;
    }
    run_c += cnt;
  }
  if (tid == 0) {
    d.n_active[0] = s_wf[kFrontWarps - 1];
    d.item_ctr[0] = 0;
    d.item_ctr[1] = 0;
    *d.ticket = 0;
  }
  if (!d.fold_scatter) return;  // kernel-uniform
  // slot -> pair index, pair -> token (pf_scatter's work) from the offsets in
  // shared memory; the slots and their ranks come from every CTA
  __syncthreads();
  const int nk = r.T * k;
  for (int i = tid; i < nk; i += kFrontThreads) {
    const int e = __ldcg(d.cs_pos + i);
    if (e >= 0) {
      const int p = s_off[e] + __ldcg(d.rank + i);
      d.pair_tok[p] = i / k;
      d.cs_pos[i] = p;
    }
  }
  if (r.has_shared) {
    for (int t = tid; t < r.T; t += kFrontThreads) {
      const int p = s_off[E] + t;
      d.pair_tok[p] = t;
      d.pos_shared[t] = p;
    }
  }
}

__global__ void __launch_bounds__(256) pf_scatter_kernel(PfScatterArgs a) {
  pdl_wait();
  pdl_trigger();
  const int nk = a.T * a.k;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < nk) {
    const int e = a.cs_pos[i];
    if (e >= 0) {
      const int p = a.off_e[e] + a.rank[i];
      a.pair_tok[p] = i / a.k;
      a.cs_pos[i] = p;
    }
  } else if (a.has_shared && i < nk + a.T) {
    const int t = i - nk;
    const int p = a.off_e[a.E] + t;
    a.pair_tok[p] = t;
    a.pos_shared[t] = p;
  }
}

// ---------------------------------------------------------------------------
// Grouped GEMM
// ---------------------------------------------------------------------------
constexpr int kM = 128;           // weight rows per unit (UMMA M)
constexpr int kThreads = 768;
constexpr int kNumBThreads = 64;  // warps 2-3 (gate/up: cp.async gathers)
constexpr int kWarpLoad = 0, kWarpMma = 1, kWarpB = 2, kWarpEpi0 = 4, kWarpDq0 = 8,
              kDqWarps = 16;     // warps 8-23
constexpr int kRun = 4 * kTileBytes;  // four contiguous 576-byte tiles

// Two variants of the GEMM:
//   TA = false (large batches): token tiles of NT = 128; A is dequantised
//     into 128-byte-swizzled shared memory by eight warps per K-block (one
//     16-row block each), two groups taking alternate K-blocks;
//   TA = true (small batches): token tiles of NT = 32; A is dequantised
//     into TENSOR MEMORY (tcgen05.st, one weight row per thread: one warp
//     per TMEM lane quarter and quantisation group of the stage, kDqGroups
//     groups of such warps taking stages in turn) and the MMA reads it from
//     there, so no fp16 weights pass through shared memory.
// Rings: raw code tiles (TMA loads, HBM latency) and operand slots, each
// holding one stage of A (dequantised weights, written by the dequant
// warps) and of B (activation rows), completed on one barrier.
template <bool GU, int NT, bool TA>
struct PfCfg {
  static constexpr int kProj = GU ? 2 : 1;
  // quantisation groups (64 columns each) per pipeline stage: the small-tile
  // variant's stages are otherwise too small to cover the fixed cost of each
  // barrier hand-off -- 2 for gate/up (two projections per group already),
  // 4 for down, both 18 KB of codes per stage
  static constexpr int kKG = TA ? (GU ? 2 : 4) : 1;
  static constexpr int kTiles = 8 * kProj;  // 16-row tiles per group
  static constexpr int kRawBytes = kKG * kTiles * kTileBytes;
  static constexpr int kABytes = kM * 128;  // one projection (shared-memory A)
  static constexpr int kAStage = TA ? 0 : kProj * kABytes;
  static constexpr int kBStage = kKG * NT * 128;  // one 128-byte-swizzled [NT x 64] block per group
  static constexpr int kRawStages = TA ? 8 : (GU ? 3 : 6);
  static constexpr int kOpStages = TA ? 3 : (GU ? 4 : 6);  // A and B share barriers
  // projections each large-tile dequant warp converts: gate/up splits them
  // (one warp per (16-row block, projection)), down has one
  static constexpr int kPW = (!TA && GU) ? 1 : kProj;
  // warps per stage: small-tile variant, one per (TMEM lane quarter, group
  // of the stage); otherwise one per (16-row block, projection share)
  static constexpr int kNumDqWarps = TA ? 4 * kKG : 8 * (kProj / kPW);
  // groups of kNumDqWarps taking stages in turn (stage q goes to group
  // q mod kDqGroups). Two rules keep every parity wait of a group on the
  // phase it means:
  //   - operand slots: a group waits on a slot's empty barrier for the stage
  //     kOpStages before its own; with more groups than slots it could run
  //     two phases ahead of that barrier, where parity waits alias -- so at
  //     most kOpStages groups work;
  //   - raw slots: slot s is reused every kRawStages stages, and that reuse
  //     must stay inside one group (kRawStages a multiple of kDqGroups).
  //     Otherwise a group reaching stage q could test raw_full of a slot
  //     whose previous phase (stage q - kRawStages, another group's) has not
  //     landed yet; TMA loads of different slots may land out of order, so
  //     the parity test would pass on the old phase and read stale codes.
  // Resulting groups and slots: large gate/up 1 group of 16 warps (one per
  // 16-row block and projection), 3 raw and 4 operand slots; large down 2
  // groups of 8 (one 16-row block each), 6 raw slots
  // (0, 2, 4 / 1, 3, 5), 6 operand slots; small gate/up 2 groups of 8
  // (TMEM lane quarter x 2 quantisation groups of the stage), 8 raw slots
  // (even / odd), 3 operand slots; small down 1 group of 16 (lane quarter x
  // 4 quantisation groups), all 8 raw and 3 operand slots.
  static constexpr int kDqGroups =
      kDqWarps / kNumDqWarps < kOpStages ? kDqWarps / kNumDqWarps : kOpStages;
  static_assert(!TA || kNumDqWarps * kDqGroups <= kDqWarps, "dequant warps");
  static_assert(kDqGroups <= kOpStages && kDqGroups >= 1, "dequant groups vs operand slots");
  static_assert(kRawStages % kDqGroups == 0, "each raw slot is reused by one dequant group");
  static constexpr size_t kRawRing = (size_t)kRawStages * kRawBytes;
  static constexpr int kAccCols = kProj * NT;
  static constexpr int kACols = TA ? kKG * kProj * (kGroup / 2) : 0;  // TMEM A columns per slot
  static constexpr int kTmemCols = TA ? 512 : 2 * kAccCols;      // power of two >= 32
  static_assert(2 * kAccCols + kOpStages * kACols <= kTmemCols, "tensor memory budget");
  static_assert(NT % 32 == 0 && NT <= 128, "token tile");
  // the small-batch variant needs little shared memory; ask for more than
  // half an SM's so that one CTA (and one 512-column TMEM allocation) runs
  // per SM
  static constexpr size_t kSmemNeed = 1024 + (size_t)kOpStages * (kAStage + kBStage) + kRawRing;
  static constexpr size_t kSmem = (TA && kSmemNeed < 120 * 1024) ? 120 * 1024 : kSmemNeed;
};

ES_DEV void tma_tile2d(void* dst, const CUtensorMap* tm, int col, int row, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];\n" ::"r"(smem_addr(dst)),
      "l"(tm), "r"(col), "r"(row), "r"(smem_addr(bar))
      : "memory");
}

// One stage of a unit's code tiles (its 16-row tiles for kKG consecutive
// quantisation groups: runs of four contiguous 576-byte tiles) with one 5-D
// TMA load: 8-byte elements, dims {144, 2, group, run, expert}, box
// {144, 2, kKG, runs, 1}, x coordinate 0; lands run by run, each run's
// groups back to back.
ES_DEV void tma_codes5d(void* dst, const CUtensorMap* tm, int group, int run0, int expert,
                        uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4, %5, %6}], [%7], %8;\n" ::"r"(smem_addr(dst)),
      "l"(tm), "r"(0), "r"(0), "r"(group), "r"(run0), "r"(expert), "r"(smem_addr(bar)), "l"(pol)
      : "memory");
}

struct Unit {
  int e, rb, pair0, n;
};

// one lane of the (converged) warp is elected
ES_DEV bool elect_one() {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p;\n elect.sync _|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(r));
  return r != 0;
}

// bounded wait for a converged warp: lane 0 polls the barrier (one poller
// per warp keeps the barrier unit quiet), the warp barrier then orders the
// other lanes' accesses after lane 0's acquire
ES_DEV bool warp_wait(uint64_t* bar, uint32_t phase) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait_bounded(bar, phase);
  __syncwarp();
  return __shfl_sync(0xffffffffu, ok, 0);
}

// unit u -> (expert, row block, token tile of NT); s_ts = tile prefix over
// the active list (n_act + 1 entries)
template <int NT>
ES_DEV Unit decode_unit(const PfArgs& a, const int* s_ts, int n_act, int RB, int u) {
  const int t = u / RB;
  Unit r;
  r.rb = u - t * RB;
  int lo = 0, hi = n_act - 1;  // last a with s_ts[a] <= t
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (s_ts[mid] <= t) lo = mid; else hi = mid - 1;
  }
  const int ti = t - s_ts[lo];
  r.e = a.act_e[lo];
  r.pair0 = a.act_off[lo] + ti * NT;
  const int rem = a.act_n[lo] - ti * NT;
  r.n = rem < NT ? rem : NT;
  return r;
}

// First timed-out wait of a call: the error word gets ES_DEVERR_TIMEOUT and
// the next three words (reserved in the workspace's error block) record the
// wait site (1 loader raw_empty, 2 MMA acc_empty, 3 MMA op_full, 4 / 5 B
// loader op_empty, 6 epilogue acc_full, 7 / 8 dequant raw_full / op_empty,
// 9 drain), the CTA and the stage or unit.
ES_DEV void note_timeout(uint32_t* err, int site, int where) {
  set_error(err, 0x8u);
  if (atomicCAS(err + 1, 0u, (uint32_t)site) == 0u) {
    err[2] = blockIdx.x;
    err[3] = (uint32_t)where;
  }
}

// waits (bounded) for the last min(q, stages) phases armed on a ring of
// full barriers: copies still in flight land before the CTA exits
ES_DEV void drain_ring(uint64_t* full, int stages, int q, uint32_t* err) {
  const int first = q > stages ? q - stages : 0;
  for (int q2 = first; q2 < q; ++q2)
    if (!mbar_wait_bounded(&full[q2 % stages], (q2 / stages) & 1)) {
      note_timeout(err, 9, q2);
      break;
    }
}

template <bool GU, int NT, bool TA>
__global__ void __launch_bounds__(kThreads, 1) pf_gemm_kernel(const __grid_constant__ PfArgs a) {
  using C = PfCfg<GU, NT, TA>;
  constexpr int kNT = NT;
  extern __shared__ uint8_t dsmem[];
  __shared__ __align__(8) uint64_t raw_full[C::kRawStages], raw_empty[C::kRawStages];
  __shared__ __align__(8) uint64_t op_full[C::kOpStages], op_empty[C::kOpStages];
  __shared__ __align__(8) uint64_t acc_full[2], acc_empty[2], mma_done;
  __shared__ uint32_t s_tmem;
  __shared__ int s_ts[kMaxExperts + 2];
  __shared__ int s_wsum[kThreads / 32];
  __shared__ int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  auto aborted = [&]() { return *reinterpret_cast<volatile int*>(&s_abort) != 0; };
  auto set_abort = [&]() { *reinterpret_cast<volatile int*>(&s_abort) = 1; };
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(dsmem) + 1023) & ~(uintptr_t)1023);
  uint8_t* sa = base;
  uint8_t* sb = sa + (size_t)C::kOpStages * C::kAStage;
  uint8_t* raw = sb + (size_t)C::kOpStages * C::kBStage;

  if (tid == 0) {
    for (int i = 0; i < C::kRawStages; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], C::kNumDqWarps);
    }
    for (int i = 0; i < C::kOpStages; ++i) {
      // full: the 8 dequant warps of a K-block plus its B rows (64 cp.async
      // threads for gate/up, one TMA arrival for down); empty: the MMA commit
      mbar_init(&op_full[i], C::kNumDqWarps + (GU ? kNumBThreads : 1));
      mbar_init(&op_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(&mma_done, 1);
    s_abort = 0;
    fence_mbar_init();
  }
  if (warp == kWarpMma) {
    tmem_alloc(&s_tmem, C::kTmemCols);
    tmem_relinquish();
  }

  pdl_wait();
  // token-tile prefix over the active experts
  const int n_act = *a.n_active;
  {
    const int per = (n_act + kThreads - 1) / kThreads;
    const int lo = tid * per;
    int v = 0;
    for (int q = 0; q < per; ++q)
      if (lo + q < n_act) v += (a.act_n[lo + q] + kNT - 1) / kNT;
    const int mine = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int nv = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += nv;
    }
    if (lane == 31) s_wsum[warp] = v;
    __syncthreads();
    if (warp == 0) {
      int w = lane < kThreads / 32 ? s_wsum[lane] : 0;
#pragma unroll
      for (int o = 1; o < kThreads / 32; o <<= 1) {
        const int nw = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += nw;
      }
      if (lane < kThreads / 32) s_wsum[lane] = w;
    }
    __syncthreads();
    int run = (warp > 0 ? s_wsum[warp - 1] : 0) + v - mine;
    for (int q = 0; q < per; ++q) {
      if (lo + q >= n_act) break;
      s_ts[lo + q] = run;
      run += (a.act_n[lo + q] + kNT - 1) / kNT;
    }
    if (tid == kThreads - 1) s_ts[n_act] = s_wsum[kThreads / 32 - 1];
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_trigger();

  const uint32_t tmem = s_tmem;
  const int RB = (GU ? a.I : a.D) / kM;
  const int KB = (GU ? a.D : a.I) / (kGroup * C::kKG);  // stages per unit
  const int units = s_ts[n_act] * RB;

  if (warp == kWarpLoad) {
    // ---------------- packed code tiles -> raw ring ----------------
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      int q = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const Unit un = decode_unit<NT>(a, s_ts, n_act, RB, u);
        for (int kb = 0; kb < KB; ++kb, ++q) {
          const int s = q % C::kRawStages;
          if (!mbar_wait_bounded(&raw_empty[s], ((q / C::kRawStages) & 1) ^ 1)) {
            note_timeout(a.err, 1, q);
            ok = false;
            break;
          }
          if (aborted()) { ok = false; break; }
          mbar_arrive_expect_tx(&raw_full[s], C::kRawBytes);
          tma_codes5d(raw + (size_t)s * C::kRawBytes, &a.tm_a, kb * C::kKG,
                      (C::kRawBytes / (kRun * C::kKG)) * un.rb, un.e, &raw_full[s], pol);
        }
      }
      if (!ok) { set_error(a.err, 0x8u); set_abort(); }
      drain_ring(raw_full, C::kRawStages, q, a.err);
    }
  } else if (warp == kWarpMma) {
    // ---------------- tensor-core issue ----------------
    // The whole warp runs the loop (descriptors stay warp-uniform); one
    // elected lane issues each tcgen05 instruction.
    int iu = 0, so = 0;
    uint32_t ph = 0;  // operand ring slot and its phase parity
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++iu) {
      const Unit un = decode_unit<NT>(a, s_ts, n_act, RB, u);
      const uint32_t idesc = idesc_f16_m128((un.n + 15) & ~15);
      const int buf = iu & 1;
      if (!warp_wait(&acc_empty[buf], ((iu >> 1) & 1) ^ 1)) {
        if (lane == 0) note_timeout(a.err, 2, iu);
        ok = false;
        break;
      }
      if (aborted()) { ok = false; break; }
      tc_fence_after();
      const uint32_t d0 = tmem + buf * C::kAccCols;
      for (int kb = 0; kb < KB; ++kb) {
        if (!warp_wait(&op_full[so], ph)) {
          if (lane == 0) note_timeout(a.err, 3, iu * 1024 + kb);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t bdesc = sw128_desc(sb + (size_t)so * C::kBStage);
        if (TA) {
          // A slot so: columns [2 kAccCols + so kACols, + kACols): per
          // projection kKG groups of 32 columns, 8 per K = 16 step; B: one
          // [NT x 64] swizzled block per group (NT * 128 bytes = NT * 8
          // descriptor units apart)
          const uint32_t a0 = tmem + 2 * C::kAccCols + so * C::kACols;
          if (elect_one()) {
#pragma unroll
            for (int pj = 0; pj < C::kProj; ++pj)
#pragma unroll
              for (int g2 = 0; g2 < C::kKG; ++g2)
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                  umma_f16_ts(d0 + pj * kNT, a0 + (pj * C::kKG + g2) * (kGroup / 2) + 8 * kk,
                              bdesc + (uint64_t)g2 * (kNT * 8) + 2 * kk, idesc,
                              (kb > 0 || g2 > 0 || kk > 0) ? 1u : 0u);
            umma_commit(&op_empty[so]);
          }
        } else {
          const uint64_t adesc0 = sw128_desc(sa + (size_t)so * C::kAStage);
          if (elect_one()) {
#pragma unroll
            for (int pj = 0; pj < C::kProj; ++pj) {
              // projection pj's tile starts kABytes (16 KB = 1024 descriptor units) later
              const uint64_t adesc = adesc0 + (uint64_t)pj * (C::kABytes >> 4);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)  // K = 16 per instruction: +32 bytes
                umma_f16(d0 + pj * kNT, adesc + 2 * kk, bdesc + 2 * kk, idesc,
                         (kb > 0 || kk > 0) ? 1u : 0u);
            }
            umma_commit(&op_empty[so]);
          }
        }
        __syncwarp();
        if (++so == C::kOpStages) { so = 0; ph ^= 1u; }
      }
      if (!ok) break;
      if (elect_one()) umma_commit(&acc_full[buf]);
      __syncwarp();
    }
    if (!ok && lane == 0) { set_error(a.err, 0x8u); set_abort(); }
    __syncwarp();  // elect.sync needs the whole warp converged
    if (elect_one()) umma_commit(&mma_done);
    __syncwarp();
    warp_wait(&mma_done, 0);
  } else if (warp == kWarpB || warp == kWarpB + 1) {
    // ---------------- B rows (activations) -> B ring ----------------
    int q = 0;
    bool ok = true;
    if (GU) {
      // token rows of x16, gathered with 16-byte cp.async by 64 threads:
      // thread bt copies chunk bt % 8 of rows bt / 8 + 8 i; completion is
      // tracked on the slot's full barrier (cp.async.mbarrier.arrive), so no thread waits on
      // its copies
      const int bt = tid - kWarpB * 32, ch = bt & 7, r0 = bt >> 3;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const Unit un = decode_unit<NT>(a, s_ts, n_act, RB, u);
        const uint16_t* rows[kNT / 8];
#pragma unroll
        for (int i = 0; i < kNT / 8; ++i) {
          const int j = r0 + 8 * i;
          rows[i] = j < un.n ? a.x16 + (size_t)a.pair_tok[un.pair0 + j] * a.D + ch * 8 : nullptr;
        }
        for (int kb = 0; kb < KB; ++kb, ++q) {
          const int s = q % C::kOpStages;
          if (!warp_wait(&op_empty[s], ((q / C::kOpStages) & 1) ^ 1)) {
            if (lane == 0) note_timeout(a.err, 4, q);
            ok = false;
            break;
          }
          if (aborted()) { ok = false; break; }
          uint8_t* dst = sb + (size_t)s * C::kBStage;
#pragma unroll
          for (int g2 = 0; g2 < C::kKG; ++g2)
#pragma unroll
            for (int i = 0; i < kNT / 8; ++i) {
              const int j = r0 + 8 * i;
              if (rows[i])
                cp_async16(dst + g2 * (kNT * 128) + j * 128 + ((ch ^ (j & 7)) << 4),
                           rows[i] + (kb * C::kKG + g2) * kGroup);
            }
          cp_async_arrive(&op_full[s]);
          mbar_arrive(&op_full[s]);
        }
      }
      cp_async_wait_all();
    } else if (warp == kWarpB) {
      // NT consecutive pair rows of h16: one TMA tile per group
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const Unit un = decode_unit<NT>(a, s_ts, n_act, RB, u);
        for (int kb = 0; kb < KB; ++kb, ++q) {
          const int s = q % C::kOpStages;
          if (!warp_wait(&op_empty[s], ((q / C::kOpStages) & 1) ^ 1)) {
            if (lane == 0) note_timeout(a.err, 5, q);
            ok = false;
            break;
          }
          if (aborted()) { ok = false; break; }
          if (lane == 0) {
            mbar_arrive_expect_tx(&op_full[s], (uint32_t)C::kBStage);
#pragma unroll
            for (int g2 = 0; g2 < C::kKG; ++g2)
              tma_tile2d(sb + (size_t)s * C::kBStage + g2 * (kNT * 128), &a.tm_b,
                         (kb * C::kKG + g2) * kGroup, un.pair0, &op_full[s]);
          }
        }
      }
      if (lane == 0) drain_ring(op_full, C::kOpStages, q, a.err);
    }
    if (!ok && lane == 0) { set_error(a.err, 0x8u); set_abort(); }
  } else if (warp >= kWarpEpi0 && warp < kWarpEpi0 + 4) {
    // ---------------- epilogue ----------------
    const int ew = warp - kWarpEpi0;
    const int r = 32 * ew + lane;  // weight row inside the unit
    int iu = 0;
    bool ok = true;
    uint32_t range_err = 0;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++iu) {
      const Unit un = decode_unit<NT>(a, s_ts, n_act, RB, u);
      const int buf = iu & 1;
      // inverse token scales: lane holds tokens lane + 32 i, shuffled out per column
      float inv_r[kNT / 32];
#pragma unroll
      for (int i = 0; i < kNT / 32; ++i) {
        const int j = lane + 32 * i;
        inv_r[i] = (GU && j < un.n) ? a.xinv[a.pair_tok[un.pair0 + j]] : 0.f;
      }
      if (!warp_wait(&acc_full[buf], (iu >> 1) & 1)) {
        if (lane == 0) note_timeout(a.err, 6, iu);
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t tb = tmem + ((uint32_t)(32 * ew) << 16) + buf * C::kAccCols;
      const int npad = (un.n + 15) & ~15;
      for (int j0 = 0; j0 < npad; j0 += 16) {
        if (GU) {
          const int sel = j0 >> 5;
          float inv_sel = inv_r[0];
#pragma unroll
          for (int i = 1; i < kNT / 32; ++i)
            if (sel == i) inv_sel = inv_r[i];
          uint32_t g[16], v[16];
          tmem_ld16(tb + j0, g);
          tmem_ld16(tb + kNT + j0, v);
          tmem_wait_ld(g);
          tmem_wait_ld(v);
          const int col = un.rb * kM + nib_pos(r);
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            const int j = j0 + jj;
            const float inv = __shfl_sync(0xffffffffu, inv_sel, (j0 & 31) + jj);
            if (j < un.n) {
              const float gg = __uint_as_float(g[jj]) * inv;
              const float uu = __uint_as_float(v[jj]) * inv;
              float h = silu_f(gg) * uu;
              if (fabsf(h) > 65504.f) { range_err = 1; h = copysignf(65504.f, h); }
              a.h16[(size_t)(un.pair0 + j) * a.I + col] = __half_as_ushort(__float2half_rn(h));
            }
          }
        } else {
          uint32_t y[16];
          tmem_ld16(tb + j0, y);
          tmem_wait_ld(y);
          const int col = un.rb * kM + r;
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            const int j = j0 + jj;
            if (j < un.n) {
              float yv = __uint_as_float(y[jj]);
              if (fabsf(yv) > 65504.f) { range_err = 1; yv = copysignf(65504.f, yv); }
              a.y16[(size_t)(un.pair0 + j) * a.D + col] = __half_as_ushort(__float2half_rn(yv));
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
    if (range_err) set_error(a.err, 0x10u);
    if (!ok) { if (lane == 0) set_error(a.err, 0x8u); set_abort(); }
  } else if (TA && warp >= kWarpDq0) {
    // ---------------- codes -> fp16 A in tensor memory ----------------
    // warp 8 + kNumDqWarps grp + 4 sub + dw: TMEM lane quarter dw (warp % 4),
    // so thread `lane` owns weight row r = 32 dw + lane of the unit, and it
    // converts quantisation group `sub` of the stage; group grp of warps
    // takes stages q = grp mod kDqGroups (warps of groups >= kDqGroups idle)
    const int dw = (warp - kWarpDq0) & 3;
    const int sub = ((warp - kWarpDq0) >> 2) % C::kKG;
    const int grp = (warp - kWarpDq0) / C::kNumDqWarps;
    const int b16 = 2 * dw + (lane >> 4);  // 16-row tile of the row
    const int g = lane & 7, hf = (lane >> 3) & 1;  // row g + 8 hf of that tile
    constexpr int kRowBlocksPerRun = 4 / C::kProj;
    const int run = b16 / kRowBlocksPerRun, in_run = (b16 % kRowBlocksPerRun) * C::kProj;
    const uint32_t a_lane = tmem + ((uint32_t)(32 * dw) << 16) + 2 * C::kAccCols;
    int q = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok && grp < C::kDqGroups; u += gridDim.x) {
      for (int kb = 0; kb < KB; ++kb, ++q) {
        if (q % C::kDqGroups != grp) continue;
        const int sr = q % C::kRawStages, s_a = q % C::kOpStages;
        if (!warp_wait(&raw_full[sr], (q / C::kRawStages) & 1)) {
          if (lane == 0) note_timeout(a.err, 7, q);
          ok = false;
          break;
        }
        // group `sub` of the stage: the row's eight code words (words 2c,
        // 2c+1 sit in lane 4g + c's 16 bytes, row g + 8 in the upper half)
        // and its (scale, bias); the stage holds, per run of four tiles, the
        // kKG groups' runs back to back
        const uint8_t* slot = raw + (size_t)sr * C::kRawBytes + (size_t)(run * C::kKG + sub) * kRun;
        uint2 wv[C::kProj][4];
        uint32_t sbw[C::kProj];
#pragma unroll
        for (int pj = 0; pj < C::kProj; ++pj) {
          const uint8_t* tile = slot + (in_run + pj) * kTileBytes;
#pragma unroll
          for (int c = 0; c < 4; ++c) wv[pj][c] = ld_shared8(tile + (4 * g + c) * 16 + hf * 8);
          sbw[pj] = *reinterpret_cast<const uint32_t*>(tile + kTileCodeBytes + 8 * g + 4 * hf);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[sr]);
        if (!warp_wait(&op_empty[s_a], ((q / C::kOpStages) & 1) ^ 1)) {
          if (lane == 0) note_timeout(a.err, 8, q);
          ok = false;
          break;
        }
        if (__shfl_sync(0xffffffffu, aborted() ? 1 : 0, 0)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int pj = 0; pj < C::kProj; ++pj) {
          const __half2 s2 = __half2half2(__ushort_as_half((uint16_t)(sbw[pj] & 0xffffu)));
          const __half2 b2 = __half2half2(__ushort_as_half((uint16_t)(sbw[pj] >> 16)));
          uint32_t r[32];  // column 4j + s: elements (8j + s, 8j + s + 4), nibble order
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint4 o0 = dequant_word(wv[pj][c].x, s2, b2);
            const uint4 o1 = dequant_word(wv[pj][c].y, s2, b2);
            r[8 * c + 0] = o0.x; r[8 * c + 1] = o0.y; r[8 * c + 2] = o0.z; r[8 * c + 3] = o0.w;
            r[8 * c + 4] = o1.x; r[8 * c + 5] = o1.y; r[8 * c + 6] = o1.z; r[8 * c + 7] = o1.w;
          }
          tmem_st32(a_lane + s_a * C::kACols + (pj * C::kKG + sub) * (kGroup / 2), r);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&op_full[s_a]);
      }
    }
    if (!ok) { if (lane == 0) set_error(a.err, 0x8u); set_abort(); }
  } else if (!TA && warp >= kWarpDq0) {
    // ---------------- codes -> fp16 A tiles in shared memory ----------------
    const int dwi = (warp - kWarpDq0) % C::kNumDqWarps;
    const int dw = dwi % 8;                              // 16-row block of the unit
    const int pj0 = (dwi / 8) * C::kPW;                  // first projection it converts
    const int grp = (warp - kWarpDq0) / C::kNumDqWarps;  // takes K-blocks q = grp mod kDqGroups
    const int g = lane >> 2, c = lane & 3;
    int q = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      for (int kb = 0; kb < KB; ++kb, ++q) {
        if (q % C::kDqGroups != grp) continue;
        const int sr = q % C::kRawStages, s_a = q % C::kOpStages;
        if (!warp_wait(&raw_full[sr], (q / C::kRawStages) & 1)) {
          if (lane == 0) note_timeout(a.err, 7, q);
          ok = false;
          break;
        }
        uint4 cw[C::kPW];
        uint2 sbv[C::kPW];
#pragma unroll
        for (int pj = 0; pj < C::kPW; ++pj) {
          const uint8_t* tile =
              raw + (size_t)sr * C::kRawBytes + (dw * C::kProj + pj0 + pj) * kTileBytes;
          cw[pj] = ld_shared16(tile + 16 * lane);
          sbv[pj] = ld_shared8(tile + kTileCodeBytes + 8 * g);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[sr]);
        if (!warp_wait(&op_empty[s_a], ((q / C::kOpStages) & 1) ^ 1)) {
          if (lane == 0) note_timeout(a.err, 8, q);
          ok = false;
          break;
        }
        if (aborted()) { ok = false; break; }
#pragma unroll
        for (int pj = 0; pj < C::kPW; ++pj) {
          uint8_t* at = sa + (size_t)s_a * C::kAStage + (pj0 + pj) * C::kABytes;
          // rows g and g + 8 of this 16-row block; sbv = (scale, bias) of each
          const __half2 s_lo = __half2half2(__ushort_as_half((uint16_t)(sbv[pj].x & 0xffffu)));
          const __half2 b_lo = __half2half2(__ushort_as_half((uint16_t)(sbv[pj].x >> 16)));
          const __half2 s_hi = __half2half2(__ushort_as_half((uint16_t)(sbv[pj].y & 0xffffu)));
          const __half2 b_hi = __half2half2(__ushort_as_half((uint16_t)(sbv[pj].y >> 16)));
          const int row0 = dw * 16 + g, row1 = row0 + 8;
          // words 2c, 2c+1 of each row: chunks 2c and 2c+1 of the K-block
          st_shared16(at + row0 * 128 + (((2 * c) ^ g) << 4), dequant_word(cw[pj].x, s_lo, b_lo));
          st_shared16(at + row0 * 128 + (((2 * c + 1) ^ g) << 4), dequant_word(cw[pj].y, s_lo, b_lo));
          st_shared16(at + row1 * 128 + (((2 * c) ^ g) << 4), dequant_word(cw[pj].z, s_hi, b_hi));
          st_shared16(at + row1 * 128 + (((2 * c + 1) ^ g) << 4), dequant_word(cw[pj].w, s_hi, b_hi));
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&op_full[s_a]);
      }
    }
    if (!ok) { if (lane == 0) set_error(a.err, 0x8u); set_abort(); }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kWarpMma) tmem_dealloc(tmem, C::kTmemCols);
}

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D fp16 row-major [rows][cols] tensor map, 128-byte swizzle, box of 64
// columns (one K-block) x box_rows rows
cudaError_t encode_rows_f16(CUtensorMap* m, const void* base, int cols, long long rows,
                            int box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kGroup, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// 5-D map of one projection region's code tiles, 8-byte elements:
// {144, 2} = one 2304-byte run, then group (stride 2304 B), run (stride
// groups x 2304 B), expert (stride expert_bytes); box {144, 2, groups per
// stage, runs, 1}
cudaError_t encode_codes_map(CUtensorMap* m, const PfArgs& a, bool gu, int runs, int groups_per_box) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return cudaErrorNotSupported;
  const int groups = (gu ? a.D : a.I) / kGroup;
  const int nruns = gu ? a.I / 32 : a.D / 64;
  const uint8_t* base = a.packed + (gu ? 0 : gateup_region_bytes(a.D, a.I));
  const cuuint64_t dims[5] = {kRun / 16, 2, (cuuint64_t)groups, (cuuint64_t)nruns,
                              (cuuint64_t)a.E1};
  const cuuint64_t strides[4] = {kRun / 2, kRun, (cuuint64_t)groups * kRun,
                                 (cuuint64_t)a.expert_bytes};
  const cuuint32_t box[5] = {kRun / 16, 2, (cuuint32_t)groups_per_box, (cuuint32_t)runs, 1};
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 5, const_cast<uint8_t*>(base), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <bool GU, int NT, bool TA>
cudaError_t launch_pf_gemm(const PfArgs& a_in, long long b_rows, int max_units,
                           cudaStream_t st) {
  using C = PfCfg<GU, NT, TA>;
  int grid = sm_count();
  if (max_units < grid) grid = max_units;
  if (grid <= 0) return cudaSuccess;
  PfArgs a = a_in;
  // down loads 128 consecutive pair rows of h16 per TMA tile; gate/up
  // gathers token rows with cp.async and needs no tensor map
  cudaError_t e = GU ? cudaSuccess : encode_rows_f16(&a.tm_b, a.h16, a.I, b_rows, NT);
  if (e != cudaSuccess) return e;
  static_assert(C::kRawBytes % (kRun * C::kKG) == 0, "whole runs per stage");
  if (((GU ? a.D : a.I) / kGroup) % C::kKG != 0) return cudaErrorInvalidValue;
  e = encode_codes_map(&a.tm_a, a, GU, C::kRawBytes / (kRun * C::kKG), C::kKG);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(pf_gemm_kernel<GU, NT, TA>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kSmem);
  if (e != cudaSuccess) return e;
  return launch_pdl(pf_gemm_kernel<GU, NT, TA>, dim3(grid), dim3(kThreads), C::kSmem, st, a);
}

template <int VPL>
cudaError_t launch_pf_front_vpl(const RouteArgs& r, const PfFrontArgs& d, cudaStream_t st) {
  int blocks = (r.T + kFrontWarps - 1) / kFrontWarps;
  const int cap = 4 * sm_count();
  if (blocks > cap) blocks = cap;
  return launch_pdl(pf_front_kernel<VPL>, dim3(blocks), dim3(kFrontThreads), 0, st, r, d);
}

}  // namespace

cudaError_t launch_pf_front(const RouteArgs& r, const PfFrontArgs& d, cudaStream_t st) {
  if (r.T <= 0) return cudaSuccess;
  const int vpl = (r.E + 31) / 32;
  if (vpl <= 1) return launch_pf_front_vpl<1>(r, d, st);
  if (vpl <= 2) return launch_pf_front_vpl<2>(r, d, st);
  if (vpl <= 4) return launch_pf_front_vpl<4>(r, d, st);
  if (vpl <= 8) return launch_pf_front_vpl<8>(r, d, st);
  if (vpl <= 16) return launch_pf_front_vpl<16>(r, d, st);
  return launch_pf_front_vpl<32>(r, d, st);
}

cudaError_t launch_pf_scatter(const PfScatterArgs& a, cudaStream_t st) {
  const int n = a.T * a.k + (a.has_shared ? a.T : 0);
  if (n <= 0) return cudaSuccess;
  return launch_pdl(pf_scatter_kernel, dim3((n + 255) / 256), dim3(256), 0, st, a);
}

cudaError_t launch_pf_gateup(const PfArgs& a, long long tokens, int max_units, bool small,
                             cudaStream_t st) {
  return small ? launch_pf_gemm<true, kSmallTile, true>(a, tokens, max_units, st)
               : launch_pf_gemm<true, kLargeTile, false>(a, tokens, max_units, st);
}

cudaError_t launch_pf_down(const PfArgs& a, long long pairs, int max_units, bool small,
                           cudaStream_t st) {
  return small ? launch_pf_gemm<false, kSmallTile, true>(a, pairs, max_units, st)
               : launch_pf_gemm<false, kLargeTile, false>(a, pairs, max_units, st);
}

}  // namespace es
