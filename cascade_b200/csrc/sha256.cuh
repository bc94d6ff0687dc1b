// SHA-256 (FIPS 180-4) building blocks for sm_100a.
//
// The reference hashes a block with OpenSSL's one-shot SHA256()
// (cascade_core.cpp:45) and names it by the first 16 digest bytes
// (cascade_core.cpp:43-53).  Here the same function runs on the integer
// pipes: rotations are funnel shifts, the three-input XORs / Ch / Maj are
// single LOP3s after ptxas' logic folding, and big-endian word loads are one
// byte permute each.  Merkle-Damgard chaining makes each block one serial
// chain, so parallelism comes from hashing many blocks at once (one lane per
// block).
#pragma once

#include <stdint.h>

namespace cb {
namespace sha {

__device__ __forceinline__ uint32_t rotr(uint32_t x, int n) {
  return __funnelshift_r(x, x, n);
}

// Big-endian load of a little-endian-loaded word.
__device__ __forceinline__ uint32_t bswap(uint32_t x) {
  return __byte_perm(x, 0, 0x0123);
}

__device__ __forceinline__ uint32_t K(int t) {
  // FIPS 180-4 section 4.2.2: first 32 bits of the fractional parts of the
  // cube roots of the first 64 primes.  Indexed with a compile-time t inside
  // fully unrolled loops, so every use becomes an immediate operand.
  constexpr uint32_t k[64] = {
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
  return k[t];
}

// FIPS 180-4 section 5.3.3 initial hash value.
__device__ __forceinline__ void init(uint32_t st[8]) {
  st[0] = 0x6a09e667u; st[1] = 0xbb67ae85u; st[2] = 0x3c6ef372u;
  st[3] = 0xa54ff53au; st[4] = 0x510e527fu; st[5] = 0x9b05688cu;
  st[6] = 0x1f83d9abu; st[7] = 0x5be0cd19u;
}

__device__ __forceinline__ uint32_t sig0(uint32_t x) {
  return rotr(x, 7) ^ rotr(x, 18) ^ (x >> 3);
}
__device__ __forceinline__ uint32_t sig1(uint32_t x) {
  return rotr(x, 17) ^ rotr(x, 19) ^ (x >> 10);
}
__device__ __forceinline__ uint32_t Sig0(uint32_t x) {
  return rotr(x, 2) ^ rotr(x, 13) ^ rotr(x, 22);
}
__device__ __forceinline__ uint32_t Sig1(uint32_t x) {
  return rotr(x, 6) ^ rotr(x, 11) ^ rotr(x, 25);
}

// One 64-byte chunk: w[0..15] are the big-endian message words; the
// schedule is expanded in place in a rolling 16-word window.
__device__ __forceinline__ void compress(uint32_t st[8], uint32_t w[16]) {
  uint32_t a = st[0], b = st[1], c = st[2], d = st[3];
  uint32_t e = st[4], f = st[5], g = st[6], h = st[7];
#pragma unroll
  for (int t = 0; t < 64; ++t) {
    uint32_t wt;
    if (t < 16) {
      wt = w[t];
    } else {
      wt = w[t & 15] + sig0(w[(t - 15) & 15]) + w[(t - 7) & 15] +
           sig1(w[(t - 2) & 15]);
      w[t & 15] = wt;
    }
    uint32_t t1 = h + Sig1(e) + ((e & f) ^ (~e & g)) + K(t) + wt;
    uint32_t t2 = Sig0(a) + ((a & b) | (c & (a | b)));
    h = g; g = f; f = e; e = d + t1;
    d = c; c = b; b = a; a = t1 + t2;
  }
  st[0] += a; st[1] += b; st[2] += c; st[3] += d;
  st[4] += e; st[5] += f; st[6] += g; st[7] += h;
}

// x*m + y as one IMAD.  With m a run-time 1 (or -1) the compiler cannot
// fold the multiply away, so the add is issued to the FMA pipe instead of
// the integer ALU pipe, which the rotates and logic ops already fill.
__device__ __forceinline__ uint32_t mad(uint32_t x, uint32_t m, uint32_t y) {
  uint32_t r;
  asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(x), "r"(m), "r"(y));
  return r;
}

// One round given kw = K[t] + W[t], with the seven additions on the FMA
// pipe (10 ALU + 7 IMAD instructions) and arranged so the e-chain is three
// operations deep (rotate, LOP3, IMAD):
//   e' = Sig1(e) + (Ch(e,f,g) + (d + (h + kw)))
//   a' = e' + (Sig0(a) + (Maj(a,b,c) - d))          [= T1 + T2]
__device__ __forceinline__ void round_kw(uint32_t &a, uint32_t &b, uint32_t &c,
                                         uint32_t &d, uint32_t &e, uint32_t &f,
                                         uint32_t &g, uint32_t &h, uint32_t kw,
                                         uint32_t one, uint32_t neg_one) {
  const uint32_t hk = mad(h, one, kw);
  const uint32_t dhk = mad(d, one, hk);
  const uint32_t ch = (e & f) ^ (~e & g);
  const uint32_t dhkc = mad(ch, one, dhk);
  const uint32_t e_new = mad(Sig1(e), one, dhkc);
  const uint32_t maj = (a & b) | (c & (a | b));
  const uint32_t q = mad(d, neg_one, maj);
  const uint32_t u = mad(Sig0(a), one, q);
  const uint32_t a_new = mad(e_new, one, u);
  h = g; g = f; f = e; e = e_new;
  d = c; c = b; b = a; a = a_new;
}

// A round with both recurrences three operations deep (rotate, LOP3, add):
//   e' = Sig1(e) + Ch(e,f,g) + (d + h + kw)      [IMAD, IMAD]
//   a' = IADD3(e', Sig0(a), Maj(a,b,c) - d)      [one three-input ALU add]
// 11 ALU + 5 IMAD instructions.
__device__ __forceinline__ void round_kw3(uint32_t &a, uint32_t &b,
                                          uint32_t &c, uint32_t &d,
                                          uint32_t &e, uint32_t &f,
                                          uint32_t &g, uint32_t &h,
                                          uint32_t kw, uint32_t one,
                                          uint32_t neg_one) {
  const uint32_t hk = mad(h, one, kw);
  const uint32_t dhk = mad(d, one, hk);
  const uint32_t ch = (e & f) ^ (~e & g);
  const uint32_t dhkc = mad(ch, one, dhk);
  const uint32_t e_new = mad(Sig1(e), one, dhkc);
  const uint32_t maj = (a & b) | (c & (a | b));
  const uint32_t q = mad(d, neg_one, maj);
  const uint32_t a_new = e_new + Sig0(a) + q;
  h = g; g = f; f = e; e = e_new;
  d = c; c = b; b = a; a = a_new;
}

// round_kw3 with Ch added to d + h + kw on the integer ALU and the sum
// added to Sig1(e) by one IMAD: the e-recurrence carries one IMAD instead
// of two (12 ALU + 4 IMAD instructions).  With the K+W ring, 4096 chains:
// 1614 cycles per chunk against 1641 for round_kw3; from registers alone,
// 1602 against 1682.
//   e' = IMAD(Sig1(e), 1, Ch(e,f,g) + (d + (h + kw)))
//   a' = IADD3(e', Sig0(a), Maj(a,b,c) - d)
__device__ __forceinline__ void round_kw9(uint32_t &a, uint32_t &b,
                                          uint32_t &c, uint32_t &d,
                                          uint32_t &e, uint32_t &f,
                                          uint32_t &g, uint32_t &h,
                                          uint32_t kw, uint32_t one,
                                          uint32_t neg_one) {
  const uint32_t dhk = mad(d, one, mad(h, one, kw));
  const uint32_t ch = (e & f) ^ (~e & g);
  const uint32_t e_new = mad(Sig1(e), one, ch + dhk);
  const uint32_t q = mad(d, neg_one, (a & b) | (c & (a | b)));
  const uint32_t a_new = e_new + Sig0(a) + q;
  h = g; g = f; f = e; e = e_new;
  d = c; c = b; b = a; a = a_new;
}

}  // namespace sha
}  // namespace cb
