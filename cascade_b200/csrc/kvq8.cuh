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
  float inv;    // 1 / scale, correctly rounded
  float min_f;  // (float)min
  int8_t zp;
};

__device__ __forceinline__ Params params_from_minmax(int mn, int mx,
                                                     bool empty) {
  Params p;
  if (empty) {  // no elements: defined here as scale 1, zp 0
    p.scale = 1.0f; p.inv = 1.0f; p.min_f = 0.0f; p.zp = 0;
    return p;
  }
  float range = __fsub_rn((float)mx, (float)mn);
  p.scale = (range > 0.0f) ? __fdiv_rn(range, 255.0f) : 1.0f;
  p.zp = (int8_t)(uint8_t)(uint32_t)__float2int_rz(
      __fdiv_rn((float)mn, p.scale));
  p.inv = __fdiv_rn(1.0f, p.scale);
  p.min_f = (float)mn;
  return p;
}

__device__ __forceinline__ uint32_t code(int v, const Params &p) {
  int q = __float2int_rz(__fmaf_rn(__fsub_rn((float)v, p.min_f), p.inv, 0.5f));
  q = q < 0 ? 0 : (q > 255 ? 255 : q);
  return (uint32_t)(q - 128) & 0xffu;
}

// Eight int16 values packed in a uint4 -> eight code bytes in a uint2.
__device__ __forceinline__ uint2 codes8(uint4 v, const Params &p) {
  uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t c[8];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    c[2 * k] = code((int)(int16_t)(w[k] & 0xffffu), p);
    c[2 * k + 1] = code((int)(int16_t)(w[k] >> 16), p);
  }
  uint2 r;
  r.x = c[0] | (c[1] << 8) | (c[2] << 16) | (c[3] << 24);
  r.y = c[4] | (c[5] << 8) | (c[6] << 16) | (c[7] << 24);
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

__device__ __forceinline__ uint32_t value(uint32_t code_byte,
                                          const DeParams &d) {
  float x = __fadd_rn((float)(int8_t)(uint8_t)code_byte, 128.0f);
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
