// Front end of the MoE block, one launch: router, operand preparation and
// dispatch.
//
// Router: generate.py:122-136 restated per token (es_route.cuh), one warp per
// token, or given top-k ids (the run_expert_ffn entry, engine.py:15-20).
// Each routed (token, expert) pair sets bit t of the expert's token bitmap
// (atomicOr: the histogram is order-free and deterministic). The same CTA
// writes its tokens' activation rows in fragment order with 64-group sums
// and the shared-expert gate (generate.py:173-178).
//
// Dispatch: the last CTA to finish (ticket counter) turns the bitmaps into
// the token -> expert permutation -- counts by popcount, exclusive prefix
// offsets over experts, and a stable scatter: pair (t, e) goes to
// offset[e] + #{t' < t selecting e}, so tokens of an expert stay in ascending
// order (replacing the id -> local remap of engine.py:16-20 and the active
// set of generate.py:137-139). It also lists each token's slots in ascending
// expert id order for the combine, then returns the bitmap, the ticket and
// the FFN work counters to zero for the next call.
#include "es_common.cuh"
#include "es_kernels.cuh"
#include "es_route.cuh"

namespace es {
namespace {

constexpr int kFrontWarps = 16;
constexpr int kFrontThreads = kFrontWarps * 32;

// Dispatch by one CTA of kFrontThreads threads (the last to finish routing).
ES_DEV void dispatch_cta(const DispatchArgs& a, int* s_off) {
  __shared__ int s_wc[kFrontWarps];
  __shared__ int s_wf[kFrontWarps];
  const unsigned full = 0xffffffffu;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int E = a.E, E1 = a.E + (a.has_shared ? 1 : 0), W = a.W;

  // per-expert counts and per-word exclusive prefixes
  for (int e = tid; e < E1; e += kFrontThreads) {
    int cnt = 0;
    for (int w = 0; w < W; ++w) {
      a.wpre[(size_t)e * W + w] = cnt;
      cnt += __popc(__ldcg(a.bitmap + (size_t)e * W + w));
    }
    s_off[e] = cnt;
  }
  __syncthreads();

  // exclusive scan of counts and active flags: thread owns EPT consecutive experts
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
  if (lane == 31) { s_wc[wid] = vc; s_wf[wid] = vf; }
  __syncthreads();
  if (wid == 0) {
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
  int run_c = (wid > 0 ? s_wc[wid - 1] : 0) + vc - my_c;
  int run_f = (wid > 0 ? s_wf[wid - 1] : 0) + vf - my_f;
  const int total_f = s_wf[kFrontWarps - 1];
  __syncthreads();  // every thread has read its counts: s_off becomes offsets
  for (int q = 0; q < EPT; ++q) {
    const int e = e_lo + q;
    if (e >= E1) break;
    const int cnt = s_off[e];
    s_off[e] = run_c;
    if (cnt > 0) {
      a.act_e[run_f] = e;
      a.act_off[run_f] = run_c;
      a.act_n[run_f] = cnt;
      ++run_f;
    }
    run_c += cnt;
  }
  if (tid == 0) {
    a.n_active[0] = total_f;
    a.item_ctr[0] = 0;
    a.item_ctr[1] = 0;
  }
  __syncthreads();

  // stable scatter over (token, rank) in parallel: the routing pass stored
  // each token's experts in ascending id order (cs_pos holds the id there)
  const int k = a.k;
  for (int i = tid; i < a.T * k; i += kFrontThreads) {
    const int t = i / k;
    const int e = __ldcg(a.cs_pos + i);
    int p = -1;
    if (e >= 0) {
      const uint32_t word = __ldcg(a.bitmap + (size_t)e * W + (t >> 5));
      p = s_off[e] + a.wpre[(size_t)e * W + (t >> 5)] + __popc(word & ((1u << (t & 31)) - 1u));
      a.pair_tok[p] = t;
    }
    a.cs_pos[i] = p;
  }
  if (a.has_shared) {
    for (int t = tid; t < a.T; t += kFrontThreads) {
      const uint32_t word = __ldcg(a.bitmap + (size_t)E * W + (t >> 5));
      const int p = s_off[E] + a.wpre[(size_t)E * W + (t >> 5)] + __popc(word & ((1u << (t & 31)) - 1u));
      a.pair_tok[p] = t;
      a.pos_shared[t] = p;
    }
  }
}

template <int VPL>
__global__ void __launch_bounds__(kFrontThreads) front_kernel(RouteArgs r, DispatchArgs d) {
  __shared__ int s_off[kMaxExperts + 2];
  __shared__ int s_last;
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int E = r.E, k = r.k;
  pdl_wait();
  pdl_trigger();

  // routing, one warp per token
  for (int t = blockIdx.x * kFrontWarps + warp; t < r.T; t += gridDim.x * kFrontWarps) {
    int my_e = -1;
    float my_w = 0.f;
    if (r.logits) {
      route_token_warp<VPL>(r.logits, r.logits_f32, r.bias, t, E, k, r.renorm, r.err, my_e, my_w);
      if (lane < k) {
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
    if (!r.bitmap) continue;  // router only
    sort_slots_warp(d.cs_pos, d.cs_w, k, t, my_e, my_w);
    const uint32_t bit = 1u << (t & 31);
    if (lane < k && my_e >= 0) atomicOr(&r.bitmap[(size_t)my_e * r.W + (t >> 5)], bit);
    if (r.has_shared) {
      if (lane == 0) atomicOr(&r.bitmap[(size_t)E * r.W + (t >> 5)], bit);
      const float gsg = shared_gate_warp(r.x + (size_t)t * r.D, r.sg_w, r.D);
      if (lane == 0) r.sgate[t] = gsg;
    }
  }
  if (!r.bitmap) return;  // kernel-uniform

  // this CTA's activation rows -> fragment order + group sums
  const int chunks = r.D / 8, GD = r.D / kGroup;
  for (int tb = blockIdx.x * kFrontWarps; tb < r.T; tb += gridDim.x * kFrontWarps) {
    const int total = kFrontWarps * chunks;
    for (int c0 = 0; c0 < total; c0 += kFrontThreads) {
      const int c = c0 + threadIdx.x;
      const int tt = tb + c / chunks, q8 = c % chunks;
      const bool lv = c < total && tt < r.T;
      float sum = permute_chunk8(r.x + (size_t)tt * r.D, r.x_perm + (size_t)tt * r.D, q8, lv);
      sum += __shfl_xor_sync(full, sum, 1);
      sum += __shfl_xor_sync(full, sum, 2);
      sum += __shfl_xor_sync(full, sum, 4);
      if (lv && (q8 & 7) == 0) r.xsum[(size_t)tt * GD + (q8 >> 3)] = sum;
    }
  }

  // the last CTA dispatches. The block barrier orders every thread's writes
  // before thread 0's fence and ticket (one fence per CTA, as in a grid
  // sync); the last CTA's thread 0 fences again before its threads read.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicAdd(d.ticket, 1) == (int)gridDim.x - 1;
    if (s_last) __threadfence();
  }
  __syncthreads();
  if (!s_last) return;
  dispatch_cta(d, s_off);
  __syncthreads();
  const int words = (E + (r.has_shared ? 1 : 0)) * r.W;
  for (int i = threadIdx.x; i < words; i += kFrontThreads) r.bitmap[i] = 0u;
  if (threadIdx.x == 0) *d.ticket = 0;
}

template <int VPL>
cudaError_t launch_front_vpl(const RouteArgs& r, const DispatchArgs& d, cudaStream_t st) {
  int blocks = (r.T + kFrontWarps - 1) / kFrontWarps;
  const int cap = 4 * sm_count();
  if (blocks > cap) blocks = cap;
  return launch_pdl(front_kernel<VPL>, dim3(blocks), dim3(kFrontThreads), 0, st, r, d);
}

}  // namespace

cudaError_t launch_front(const RouteArgs& r, const DispatchArgs& d, cudaStream_t st) {
  if (r.T <= 0) return cudaSuccess;
  const int vpl = (r.E + 31) / 32;
  if (vpl <= 1) return launch_front_vpl<1>(r, d, st);
  if (vpl <= 2) return launch_front_vpl<2>(r, d, st);
  if (vpl <= 4) return launch_front_vpl<4>(r, d, st);
  if (vpl <= 8) return launch_front_vpl<8>(r, d, st);
  if (vpl <= 16) return launch_front_vpl<16>(r, d, st);
  return launch_front_vpl<32>(r, d, st);
}

}  // namespace es
