// Device helpers shared by the MoE block kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "es_layout.h"

#define ES_DEV __device__ __forceinline__

namespace es {

// ---------------------------------------------------------------------------
// 4-bit codes -> bf16 operands.
//
// A bf16 with bits 0x4300 | q (q < 128) is exactly 128 + q, so OR-ing a
// nibble into the mantissa of 128.0 converts it with one LOP3 and no
// rounding. For a packed word w (code n at bits 4n), pair s (0..3) gives
// the bf16x2 (128 + n_s, 128 + n_{s+4}): the low half holds nibble s, the
// high half nibble s + 4.
// ---------------------------------------------------------------------------
// (asm volatile keeps the compiler from hoisting all conversions of a warp's
// weights out of the token loop, which would need ~128 extra registers.)
ES_DEV uint32_t code_pair(uint32_t w, int s) {
  uint32_t r;
  asm volatile("lop3.b32 %0, %1, %2, %3, 0xEA;\n"
               : "=r"(r)
               : "r"(w >> (4 * s)), "r"(0x000F000Fu), "r"(0x43004300u));
  return r;
}

// D = A * B + C, m16n8k16, bf16 inputs, fp32 accumulate (register operands:
// the decode GEMV converts codes in registers and never stages them in
// shared memory).
ES_DEV void mma_bf16(float (&d)[4], const uint32_t a0, const uint32_t a1,
                     const uint32_t a2, const uint32_t a3, const uint32_t b0,
                     const uint32_t b1, const float (&c)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]),
        "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

// Streaming 16-byte load of packed weights: read once, keep out of L1.
ES_DEV uint4 ld_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

ES_DEV uint2 ld_stream8(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];\n"
               : "=r"(r.x), "=r"(r.y)
               : "l"(p));
  return r;
}

ES_DEV float bf16_bits_to_float(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

ES_DEV float half_bits_to_float(uint16_t b) {
  return __half2float(__ushort_as_half(b));
}

ES_DEV float lo_half_f(uint32_t v) { return half_bits_to_float(v & 0xFFFFu); }
ES_DEV float hi_half_f(uint32_t v) { return half_bits_to_float(v >> 16); }

// Round-to-nearest-even fp32 -> bf16 bits.
ES_DEV uint16_t float_to_bf16_bits(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// Orderable key of a float: larger float -> larger unsigned key. NaN maps to
// 0 (below -inf) so it is never selected.
ES_DEV uint32_t float_key(float f) {
  uint32_t u = __float_as_uint(f);
  if (f != f) return 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

ES_DEV float silu_f(float g) { return g / (1.0f + __expf(-g)); }

ES_DEV void set_error(uint32_t* err, uint32_t bit) {
  if (err) atomicOr(err, bit);
}

}  // namespace es
