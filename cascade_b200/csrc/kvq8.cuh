// The reference's FP16 -> INT8 KV compression (KVCompressor,
// cascade_core.cpp:818-872) as device functions.
//
// The payload's 16-bit words are treated as int16 bit patterns (not as
// half-precision values).  Per block: int16 min/max -> scale = range/255
// (1 when range is 0), zero_point = (int8)(int)(min/scale) (wrapping modulo
// 256); codes = clamp(trunc(fma(v - min, 1/scale, 0.5)), 0, 255) - 128.
// Decompression: trunc(fma(code + 128, scale, zp*scale)) narrowed to int16
// modulo 2^16.  The reference's GCC build contracts both multiply-adds to
// FMA; the explicit __fmaf_rn / __fdiv_rn / __fmul_rn intrinsics below fix
// the rounding of every step so the device result is bit-identical.
//
// Header (8 bytes, little-endian, CompressionMeta of cascade.hpp:341-344):
//   [0..3] float scale, [4] int8 zero_point, [5..7] zero (the reference
//   leaves them uninitialised).
#pragma once

#include <stdint.h>

namespace cb {
namespace q8 {

struct Params {
  float scale;
  float inv;       // 1 / scale, correctly rounded
  float min_f;     // (float)min
  uint32_t mn_u;   // min as a 16-bit pattern, for modular differences
  int8_t zp;
};

// 2^23 as a float and its bit pattern: for 0 <= k < 2^23,
// __int_as_float(kMagicBits | k) == 2^23 + k exactly.
constexpr float kMagic = 8388608.0f;
constexpr uint32_t kMagicBits = 0x4B000000u;

__device__ __forceinline__ Params params_from_minmax(int mn, int mx,
                                                     bool empty) {
  Params p;
  if (empty) {  // no elements: defined here as scale 1, zp 0
    p.scale = 1.0f; p.inv = 1.0f; p.min_f = 0.0f; p.mn_u = 0; p.zp = 0;
    return p;
  }
  float range = __fsub_rn((float)mx, (float)mn);
  p.scale = (range > 0.0f) ? __fdiv_rn(range, 255.0f) : 1.0f;
  p.zp = (int8_t)(uint8_t)(uint32_t)__float2int_rz(
      __fdiv_rn((float)mn, p.scale));
  p.inv = __fdiv_rn(1.0f, p.scale);
  p.min_f = (float)mn;
  p.mn_u = (uint32_t)mn & 0xffffu;
  return p;
}

// The code of one value, given md = bits(2^23) | d with d = v - min
// (0 <= d <= 65535, v from the block the min was taken over), without
// integer/float conversion instructions (a quarter-rate pipe on this GPU):
//   x = 2^23 + d - 2^23           == (float)v - (float)min, exactly
//   r = fma(x, inv, 0.5)          the reference's rounding, one FMA
//   floor(r) = bits(RD(r + 2^23)) - bits(2^23), exact for 0 <= r < 2^23.
// The reference's clamp to [0, 255] never binds: r >= 0.5, and for every
// int16 range (checked for all 65 535) range * RN(1 / RN(range / 255)) + 0.5
// rounds below 256, which bounds r for every d <= range.  Returns the bits
// of RD(r + 2^23), whose low byte is q (0..255).
__device__ __forceinline__ uint32_t code_of_magic(uint32_t md,
                                                  const Params &p) {
  const float x = __fsub_rn(__uint_as_float(md), kMagic);
  const float r = __fmaf_rn(x, p.inv, 0.5f);
  return __float_as_uint(__fadd_rd(r, kMagic));
}

__device__ __forceinline__ uint32_t code(int v, const Params &p) {
  const uint32_t d = ((uint32_t)v - p.mn_u) & 0xffffu;
  return (code_of_magic(kMagicBits | d, p) & 0xffu) ^ 0x80u;  // q - 128
}

// Eight int16 values packed in a uint4 -> eight code bytes in a uint2.
__device__ __forceinline__ uint2 codes8(uint4 v, const Params &p) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  const uint32_t mhi = p.mn_u << 16;
  uint32_t c[8];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    c[2 * k] = code_of_magic(kMagicBits | ((w[k] - p.mn_u) & 0xffffu), p);
    c[2 * k + 1] = code_of_magic(kMagicBits | ((w[k] - mhi) >> 16), p);
  }
  // Low bytes of c[0..3] and c[4..7], then q - 128 on all four bytes.
  uint2 r;
  r.x = __byte_perm(__byte_perm(c[0], c[1], 0x0040),
                    __byte_perm(c[2], c[3], 0x0040), 0x5410) ^ 0x80808080u;
  r.y = __byte_perm(__byte_perm(c[4], c[5], 0x0040),
                    __byte_perm(c[6], c[7], 0x0040), 0x5410) ^ 0x80808080u;
  return r;
}

struct DeParams {
  float scale;
  float min_f;  // zp * scale, a rounded product
};

__device__ __forceinline__ DeParams deparams(uint32_t scale_bits, int8_t zp) {
  DeParams d;
  d.scale = __uint_as_float(scale_bits);
  d.min_f = __fmul_rn((float)zp, d.scale);
  return d;
}

// (float)code + 128 is the integer code ^ 0x80 (0..255), made exactly
// with the 2^23 pattern instead of a conversion instruction.
__device__ __forceinline__ uint32_t value(uint32_t code_byte,
                                          const DeParams &d) {
  const float x =
      __fsub_rn(__uint_as_float(kMagicBits | ((code_byte & 0xffu) ^ 0x80u)),
                kMagic);
  return (uint32_t)__float2int_rz(__fmaf_rn(x, d.scale, d.min_f)) & 0xffffu;
}

// Eight code bytes (uint2) -> eight int16 values (uint4).
__device__ __forceinline__ uint4 values8(uint2 c, const DeParams &d) {
  uint32_t b[8];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    b[k] = (c.x >> (8 * k)) & 0xffu;
    b[4 + k] = (c.y >> (8 * k)) & 0xffu;
  }
  uint4 r;
  r.x = value(b[0], d) | (value(b[1], d) << 16);
  r.y = value(b[2], d) | (value(b[3], d) << 16);
  r.z = value(b[4], d) | (value(b[5], d) << 16);
  r.w = value(b[6], d) | (value(b[7], d) << 16);
  return r;
}

}  // namespace q8
}  // namespace cb
