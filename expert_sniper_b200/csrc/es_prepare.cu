// One-time repack of MLX-format expert tensors into the tiled layout of
// es_layout.h. Pure byte movement: every code, scale and bias is copied
// unchanged, so the packed blob has exactly the reference's bytes per expert
// (3*D*I*9/16). Counterpart of stack_proj (src/mlx_expert_sniper/engine.py:
// 22-30), which re-stacked the active experts on every call. The source is
// either stacked tensors or a streaming-format layer image (fixed-size expert
// blocks, src/mlx_expert_sniper/download.py:189-248), read in place.
#include "es_common.cuh"
#include "es_kernels.cuh"

namespace es {
namespace {

constexpr int kWarps = 8;

__global__ void __launch_bounds__(kWarps * 32) prepare_kernel(PrepareArgs a, long long total_tiles) {
  const int lane = threadIdx.x & 31;
  const long long wg = (long long)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (wg >= total_tiles) return;
  const int D = a.D, I = a.I, GD = D / kGroup, GI = I / kGroup;
  const long long gu_tiles = (long long)(I / 16) * GD * 2;
  const long long per_expert = gu_tiles + (long long)(D / 16) * GI;
  const int e = (int)(wg / per_expert);
  const long long t = wg - (long long)e * per_expert;
  int proj, rb, G, K;
  size_t dst_off;
  if (t < gu_tiles) {
    rb = (int)(t / (GD * 2));
    const int rem = (int)(t - (long long)rb * GD * 2);
    G = rem >> 1;
    proj = rem & 1;
    K = D;
    dst_off = gateup_tile_off(GD, rb, G, proj);
  } else {
    const long long t2 = t - gu_tiles;
    rb = (int)(t2 / GI);
    G = (int)(t2 - (long long)rb * GI);
    proj = 2;
    K = I;
    dst_off = down_tile_off(D, I, rb, G);
  }
  const bool shared = e >= a.E;
  const uint32_t* w = shared ? a.sw[proj]
                             : reinterpret_cast<const uint32_t*>(a.w[proj] + (size_t)e * a.ew[proj]);
  const uint16_t* s = shared ? a.ss[proj]
                             : reinterpret_cast<const uint16_t*>(a.s[proj] + (size_t)e * a.es[proj]);
  const uint16_t* b = shared ? a.sb[proj]
                             : reinterpret_cast<const uint16_t*>(a.b[proj] + (size_t)e * a.eb[proj]);
  uint8_t* dst = a.packed + (size_t)e * expert_bytes(D, I) + dst_off;

  const int g = lane >> 2, c = lane & 3;
  const size_t r0 = (size_t)(rb * 16 + g), r8 = r0 + 8;
  const size_t wcol = (size_t)G * 8 + 2 * c;
  uint4 v;
  v.x = w[r0 * (K / 8) + wcol];
  v.y = w[r0 * (K / 8) + wcol + 1];
  v.z = w[r8 * (K / 8) + wcol];
  v.w = w[r8 * (K / 8) + wcol + 1];
  reinterpret_cast<uint4*>(dst)[lane] = v;
  if (lane < 8) {
    const size_t q0 = (size_t)(rb * 16 + lane), q8 = q0 + 8;
    uint2 sb;
    sb.x = (uint32_t)s[q0 * (K / kGroup) + G] | ((uint32_t)b[q0 * (K / kGroup) + G] << 16);
    sb.y = (uint32_t)s[q8 * (K / kGroup) + G] | ((uint32_t)b[q8 * (K / kGroup) + G] << 16);
    reinterpret_cast<uint2*>(dst + kTileCodeBytes)[lane] = sb;
  }
}

}  // namespace

cudaError_t launch_prepare(const PrepareArgs& a, cudaStream_t st) {
  const int E1 = a.E + (a.has_shared ? 1 : 0);
  const long long per_expert = (long long)3 * a.D * a.I / 1024;
  const long long total = per_expert * E1;
  const long long blocks = (total + kWarps - 1) / kWarps;
  if (blocks <= 0) return cudaSuccess;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
  prepare_kernel<<<(unsigned)blocks, kWarps * 32, 0, st>>>(a, total);
  return cudaGetLastError();
}

}  // namespace es
