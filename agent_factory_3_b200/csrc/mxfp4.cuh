// MXFP4 (e2m1 values, e8m0 scale per 32-element block) -> bf16, shared by the dequant kernel
// and the MXFP4 MoE GEMM.  Exact: every e2m1 value times a power of two is a bf16 value (or
// rounds like the fp32 product would at the ends of the range).
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

namespace af3 {

// e2m1 -> bf16 without a table.  For a nibble s|e1 e0|m, placing the three magnitude bits at
// bf16 bits 8..6 (exponent bits 1..0 and the top mantissa bit) and the sign at bit 15 gives
// the bf16 whose value is exactly e2m1(nibble) * 2^-126: e = 0 lands in the bf16 subnormal
// range (m * 2^-127) and e > 0 in the normal range (2^(e-127) * (1 + m/2)).  Two exact
// power-of-two multiplies (by 2^126 and by the block scale 2^(s-127)) then give the value.
// Four packed bytes (eight values, low nibble first) -> four bf16x2 words.
__device__ __forceinline__ uint32_t e2m1x2_to_bf16x2_unscaled(uint32_t byte) {
  const uint32_t t = byte * 0x1001u;  // low nibble at bits 0..3, high nibble at bits 16..19
  return ((t << 6) & 0x01C001C0u) | ((t << 12) & 0x80008000u);
}

// bf16 bits of 2^(s-127) (e8m0 scale): s = 0 is the subnormal 2^-127, s = 255 is +inf.
__device__ __forceinline__ uint32_t e8m0_to_bf16_bits(uint32_t s) {
  return s ? (s << 7) : 0x40u;
}

__device__ __forceinline__ uint4 e2m1x8_to_bf16x8(uint32_t w, uint32_t scale_bits) {
  const uint32_t k2p126 = 0x7E807E80u;  // bf16x2 (2^126, 2^126)
  const uint32_t sc2 = scale_bits | (scale_bits << 16);
  const __nv_bfloat162 c = *reinterpret_cast<const __nv_bfloat162*>(&k2p126);
  const __nv_bfloat162 sc = *reinterpret_cast<const __nv_bfloat162*>(&sc2);
  uint32_t r[4];
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    uint32_t x = e2m1x2_to_bf16x2_unscaled((w >> (8 * b)) & 0xFFu);
    __nv_bfloat162 v = __hmul2(__hmul2(*reinterpret_cast<__nv_bfloat162*>(&x), c), sc);
    r[b] = *reinterpret_cast<uint32_t*>(&v);
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}

// e2m1 -> f16 with the hardware converter (sm_100): four packed bytes (eight values, low
// nibble first) -> four f16x2 words scaled by the f16 bits of 2^(s-127).  Exact whenever the
// scaled values are f16 numbers, i.e. for s in [104, 140] (the caller checks the range).
__device__ __forceinline__ uint4 e2m1x8_to_f16x8(uint32_t w, uint32_t scale_f16_bits) {
  uint32_t r0, r1, r2, r3;
  asm("{\n"
      ".reg .b8 b0, b1, b2, b3;\n"
      "mov.b32 {b0, b1, b2, b3}, %4;\n"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n"
      "}\n"
      : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
      : "r"(w));
  const uint32_t sc2 = scale_f16_bits | (scale_f16_bits << 16);
  uint32_t o[4] = {r0, r1, r2, r3};
#pragma unroll
  for (int i = 0; i < 4; ++i)
    asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(o[i]) : "r"(sc2));
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// 16 packed bytes (32 e2m1 values, low nibble first) times one block scale -> 16 f16x2 words
__device__ __forceinline__ void e2m1x32_to_f16x32(uint4 w, uint32_t scale_f16_bits,
                                                  uint32_t (&v)[16]) {
  const uint32_t in[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint4 o = e2m1x8_to_f16x8(in[i], scale_f16_bits);
    v[4 * i] = o.x;
    v[4 * i + 1] = o.y;
    v[4 * i + 2] = o.z;
    v[4 * i + 3] = o.w;
  }
}

// 16 packed bytes (32 e2m1 values) -> 16 f16x2 words with integer operations only.  The three
// magnitude bits (e1 e0 m) of a nibble placed at f16 bits 11..9, with its sign at bit 15, encode
// exactly value * 2^-14 (exponent field e1e0 with bias 15; e = 0 gives the subnormal
// (m / 2) * 2^-14).  Per byte: one byte permute, two integer multiplies that place the low
// nibble at bits 9 / 15 and the high nibble at bits 25 / 31 (b * 0x1001 repeats the byte 12
// bits up), one lop3, then one f16x2 multiply by `scale2` = 2^(s-113) in both halves, which
// gives value * 2^(s-127) exactly whenever that is an f16 number.  Requires s in [99, 128].
__device__ __forceinline__ void e2m1x32_to_f16x32_int(uint4 w, uint32_t scale2, uint32_t (&v)[16]) {
  const uint32_t in[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t b = __byte_perm(in[i], 0u, 0x4440u + j);   // byte j, zero-extended
      const uint32_t d9 = b * 0x00200200u;                      // (b * 0x1001) << 9
      const uint32_t d12 = b * 0x01001000u;                     // (b * 0x1001) << 12
      uint32_t o = (d9 & 0x0E000E00u) | (d12 & 0x80008000u);
      asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(o) : "r"(scale2));
      v[4 * i + j] = o;
    }
  }
}

// f16x2 bits of 2^(s-113) in both halves (s in [99, 128]): the factor of the integer path.
__device__ __forceinline__ uint32_t e8m0_to_f16x2_int_scale(uint32_t s) {
  const uint32_t h = (s - 98u) << 10;
  return h | (h << 16);
}

// f16 bits of 2^(s-127): normal for s >= 113, subnormal 2^-24 * 2^(s-103) for s in [103, 112].
__device__ __forceinline__ uint32_t e8m0_to_f16_bits(uint32_t s) {
  return s >= 113 ? ((s - 112) << 10) : (1u << (s - 103));
}

// eight bf16 -> eight f16 (round to nearest; exact for values inside the f16 range)
__device__ __forceinline__ uint4 bf16x8_to_f16x8(uint4 v) {
  uint32_t in[4] = {v.x, v.y, v.z, v.w};
  uint32_t out[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float lo = __uint_as_float(in[i] << 16), hi = __uint_as_float(in[i] & 0xFFFF0000u);
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(out[i]) : "f"(hi), "f"(lo));
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

}  // namespace af3
