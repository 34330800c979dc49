// Token -> expert permutation: histogram (popcounts of the per-expert token
// bitmaps), exclusive prefix offsets, and a stable scatter.
//
// Replaces the host-side remap of run_expert_ffn
// (src/mlx_expert_sniper/engine.py:16-20: sorted active ids, id -> local
// index) and the active-set build of generate.py:137-139. The position of
// (token t, expert e) is offset[e] + #{t' < t selecting e}, read off the
// bitmap with one popcount, so the order inside an expert is ascending token
// id and the result does not depend on thread timing.
#include "es_common.cuh"
#include "es_kernels.cuh"

namespace es {
namespace {

constexpr int kThreads = 1024;

__global__ void __launch_bounds__(kThreads) dispatch_kernel(DispatchArgs a) {
  __shared__ int s_off[kMaxExperts + 2];
  __shared__ int s_wc[32];
  __shared__ int s_wf[32];
  const unsigned full = 0xffffffffu;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int E = a.E, E1 = a.E + (a.has_shared ? 1 : 0), W = a.W;

  // 1. per-expert counts and per-word exclusive prefixes
  for (int e = tid; e < E1; e += kThreads) {
    int c = 0;
    for (int w = 0; w < W; ++w) {
      a.wpre[(size_t)e * W + w] = c;
      c += __popc(a.bitmap[(size_t)e * W + w]);
    }
    s_off[e] = c;
  }
  __syncthreads();

  // 2. exclusive scan of the counts and of the "active" flags; each thread
  //    owns experts 2*tid and 2*tid + 1 (E1 <= 2048)
  const int e0 = 2 * tid, e1 = 2 * tid + 1;
  const int c0 = e0 < E1 ? s_off[e0] : 0;
  const int c1 = e1 < E1 ? s_off[e1] : 0;
  const int f0 = c0 > 0, f1 = c1 > 0;
  int vc = c0 + c1, vf = f0 + f1;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int nc = __shfl_up_sync(full, vc, o);
    const int nf = __shfl_up_sync(full, vf, o);
    if (lane >= o) { vc += nc; vf += nf; }
  }
  if (lane == 31) { s_wc[wid] = vc; s_wf[wid] = vf; }
  __syncthreads();
  if (wid == 0) {
    int wc = s_wc[lane], wf = s_wf[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int nc = __shfl_up_sync(full, wc, o);
      const int nf = __shfl_up_sync(full, wf, o);
      if (lane >= o) { wc += nc; wf += nf; }
    }
    s_wc[lane] = wc;
    s_wf[lane] = wf;
  }
  __syncthreads();
  const int ex_c = (wid > 0 ? s_wc[wid - 1] : 0) + vc - (c0 + c1);
  const int ex_f = (wid > 0 ? s_wf[wid - 1] : 0) + vf - (f0 + f1);
  if (e0 < E1) {
    s_off[e0] = ex_c;
    if (f0) { a.act_e[ex_f] = e0; a.act_off[ex_f] = ex_c; a.act_n[ex_f] = c0; }
  }
  if (e1 < E1) {
    s_off[e1] = ex_c + c0;
    if (f1) { a.act_e[ex_f + f0] = e1; a.act_off[ex_f + f0] = ex_c + c0; a.act_n[ex_f + f0] = c1; }
  }
  if (tid == 0) a.n_active[0] = s_wf[31];
  __syncthreads();

  // 3. stable scatter of (token, slot) pairs
  const int k = a.k, kk = k + (a.has_shared ? 1 : 0);
  const int total = a.T * kk;
  for (int i = tid; i < total; i += kThreads) {
    const int t = i / kk, j = i - t * kk;
    int e = (j < k) ? a.idx[(size_t)t * k + j] : E;
    if (j < k && (e < 0 || e >= E)) { a.pos[i] = -1; continue; }
    const uint32_t word = a.bitmap[(size_t)e * W + (t >> 5)];
    const int p = s_off[e] + a.wpre[(size_t)e * W + (t >> 5)] + __popc(word & ((1u << (t & 31)) - 1u));
    a.pair_tok[p] = t;
    a.pos[i] = p;
  }
}

}  // namespace

cudaError_t launch_dispatch(const DispatchArgs& a, cudaStream_t st) {
  if (a.T <= 0) return cudaSuccess;
  dispatch_kernel<<<1, kThreads, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace es
