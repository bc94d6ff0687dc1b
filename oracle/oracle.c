/*
 * ORACLE — test infrastructure only.  A plain-C CPU restatement of the
 * reference's block-ingest arithmetic, used by tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline leg as the checker.  The product never links,
 * loads or calls this file.
 *
 * Pinned against: (1) Python hashlib (OpenSSL 3.0.13 libcrypto, the library
 * the reference links for SHA-256 at cascade_core.cpp:20,45), (2) the
 * reference itself compiled by oracle/Makefile (oracle/_ref), and (3) the
 * committed fixtures under tests/golden/ that tests/golden/make_golden.py
 * generated from (2).
 *
 * Built by oracle/Makefile with -ffp-contract=off: every fused multiply-add
 * below is an explicit fmaf(), placed where GCC contracts the reference's
 * expression at -O3 -std=gnu++17 (the reference's build flags,
 * CMakeLists.txt:14 and CMAKE_CXX_STANDARD 17 with GNU extensions).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

/* ---------------------------------------------------------------------- */
/* SHA-256, FIPS 180-4 section 6.2.  The reference calls OpenSSL's one-shot
 * SHA256(data, size, hash) (cascade_core.cpp:45); this is the published
 * algorithm restated: big-endian words, 64 rounds per 64-byte chunk, padding
 * 0x80, zeros, 64-bit big-endian bit length. */

static const uint32_t K256[64] = {
    0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu,
    0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u, 0xd807aa98u, 0x12835b01u,
    0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u,
    0xc19bf174u, 0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu,
    0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau, 0x983e5152u,
    0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u,
    0x06ca6351u, 0x14292967u, 0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu,
    0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,
    0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u,
    0xd6990624u, 0xf40e3585u, 0x106aa070u, 0x19a4c116u, 0x1e376c08u,
    0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu,
    0x682e6ff3u, 0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u,
    0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u};

static uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

static void compress_chunk(uint32_t h[8], const uint8_t *p) {
  uint32_t w[64];
  for (int t = 0; t < 16; ++t)
    w[t] = ((uint32_t)p[4 * t] << 24) | ((uint32_t)p[4 * t + 1] << 16) |
           ((uint32_t)p[4 * t + 2] << 8) | (uint32_t)p[4 * t + 3];
  for (int t = 16; t < 64; ++t) {
    uint32_t s0 = rotr(w[t - 15], 7) ^ rotr(w[t - 15], 18) ^ (w[t - 15] >> 3);
    uint32_t s1 = rotr(w[t - 2], 17) ^ rotr(w[t - 2], 19) ^ (w[t - 2] >> 10);
    w[t] = w[t - 16] + s0 + w[t - 7] + s1;
  }
  uint32_t a = h[0], b = h[1], c = h[2], d = h[3];
  uint32_t e = h[4], f = h[5], g = h[6], hh = h[7];
  for (int t = 0; t < 64; ++t) {
    uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
    uint32_t ch = (e & f) ^ (~e & g);
    uint32_t t1 = hh + S1 + ch + K256[t] + w[t];
    uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
    uint32_t maj = (a & b) ^ (a & c) ^ (b & c);
    uint32_t t2 = S0 + maj;
    hh = g; g = f; f = e; e = d + t1;
    d = c; c = b; b = a; a = t1 + t2;
  }
  h[0] += a; h[1] += b; h[2] += c; h[3] += d;
  h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
}

void oracle_sha256(const uint8_t *data, size_t size, uint8_t out[32]) {
  uint32_t h[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                   0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
  size_t full = size / 64;
  for (size_t i = 0; i < full; ++i) compress_chunk(h, data + 64 * i);
  uint8_t tail[128];
  size_t rem = size - 64 * full;
  memset(tail, 0, sizeof(tail));
  if (rem) memcpy(tail, data + 64 * full, rem);
  tail[rem] = 0x80;
  size_t tail_len = (rem < 56) ? 64 : 128;
  uint64_t bits = (uint64_t)size * 8u;
  for (int i = 0; i < 8; ++i)
    tail[tail_len - 1 - i] = (uint8_t)(bits >> (8 * i));
  compress_chunk(h, tail);
  if (tail_len == 128) compress_chunk(h, tail + 64);
  for (int i = 0; i < 8; ++i) {
    out[4 * i] = (uint8_t)(h[i] >> 24);
    out[4 * i + 1] = (uint8_t)(h[i] >> 16);
    out[4 * i + 2] = (uint8_t)(h[i] >> 8);
    out[4 * i + 3] = (uint8_t)h[i];
  }
}

/* compute_block_id (cascade_core.cpp:43-53): digest bytes 0..15 as 32
 * lowercase hex characters plus a terminating NUL. */
void oracle_block_id(const uint8_t *data, size_t size, char out[33]) {
  static const char hexd[] = "0123456789abcdef";
  uint8_t d[32];
  oracle_sha256(data, size, d);
  for (int i = 0; i < 16; ++i) {
    out[2 * i] = hexd[d[i] >> 4];
    out[2 * i + 1] = hexd[d[i] & 15];
  }
  out[32] = '\0';
}

/* ---------------------------------------------------------------------- */
/* KVCompressor (cascade_core.cpp:818-872, cascade.hpp:341-365).
 * The FP16 payload is read as little-endian int16 bit patterns, not as
 * half-precision values. */

/* Per-block parameters from the int16 min and max
 * (cascade_core.cpp:830-832): scale = range/255 (or 1 when range is 0), and
 * zero_point = (int8)(int)(min/scale), which wraps modulo 256. */
void oracle_kv_params(int16_t mn, int16_t mx, float *scale, int8_t *zp) {
  float range = (float)mx - (float)mn;
  float s = (range > 0.0f) ? range / 255.0f : 1.0f;
  *scale = s;
  *zp = (int8_t)(uint8_t)(uint32_t)(int32_t)((float)mn / s);
}

/* One code (cascade_core.cpp:842-846): q = (int)((v - min)*inv + 0.5f)
 * with the multiply-add fused, clamped to [0,255], shifted by -128. */
int8_t oracle_kv_code(int16_t v, float min_f, float inv) {
  int q = (int)fmaf((float)v - min_f, inv, 0.5f);
  if (q < 0) q = 0;
  if (q > 255) q = 255;
  return (int8_t)(q - 128);
}

/* compress: writes the 8-byte header [float scale LE][int8 zp][3 zero bytes]
 * then size/2 codes; returns 8 + size/2.  An odd trailing byte is dropped, as
 * in the reference.  The reference reads element 0 even for size < 2 (an
 * out-of-bounds read); here size < 2 yields scale 1.0f, zp 0 and no codes. */
size_t oracle_kv_compress(const uint8_t *data, size_t size, uint8_t *out) {
  size_t n = size / 2;
  float scale = 1.0f;
  int8_t zp = 0;
  int16_t mn = 0, mx = 0;
  if (n) {
    memcpy(&mn, data, 2);
    mx = mn;
    for (size_t i = 1; i < n; ++i) {
      int16_t v;
      memcpy(&v, data + 2 * i, 2);
      if (v < mn) mn = v;
      if (v > mx) mx = v;
    }
    oracle_kv_params(mn, mx, &scale, &zp);
  }
  memcpy(out, &scale, 4);
  out[4] = (uint8_t)zp;
  out[5] = out[6] = out[7] = 0;
  float inv = 1.0f / scale;
  float min_f = (float)mn;
  for (size_t i = 0; i < n; ++i) {
    int16_t v;
    memcpy(&v, data + 2 * i, 2);
    out[8 + i] = (uint8_t)oracle_kv_code(v, min_f, inv);
  }
  return 8 + n;
}

/* decompress (cascade_core.cpp:851-872): min_f = zp*scale (a rounded
 * product), value = fmaf(code + 128, scale, min_f), truncated to int32 and
 * narrowed to int16 modulo 2^16.  Returns 0 when comp_size is too small. */
int oracle_kv_decompress(const uint8_t *comp, size_t comp_size, uint8_t *out,
                         size_t orig_size) {
  size_t n = orig_size / 2;
  if (comp_size < 8 + n) return 0;
  float scale;
  memcpy(&scale, comp, 4);
  int8_t zp = (int8_t)comp[4];
  float min_f = (float)zp * scale;
  for (size_t i = 0; i < n; ++i) {
    float x = (float)(int8_t)comp[8 + i] + 128.0f;
    int32_t w = (int32_t)fmaf(x, scale, min_f);
    uint16_t u = (uint16_t)(uint32_t)w;
    memcpy(out + 2 * i, &u, 2);
  }
  return 1;
}

/* Unfused variants, used only by the test that checks which form the
 * reference build takes. */
int8_t oracle_kv_code_unfused(int16_t v, float min_f, float inv) {
  volatile float p = ((float)v - min_f) * inv;
  int q = (int)(p + 0.5f);
  if (q < 0) q = 0;
  if (q > 255) q = 255;
  return (int8_t)(q - 128);
}

int16_t oracle_kv_value_unfused(int8_t code, float scale, float min_f) {
  volatile float p = ((float)code + 128.0f) * scale;
  return (int16_t)(uint16_t)(uint32_t)(int32_t)(p + min_f);
}
