// Shared device helpers for the ecoint8 B200 library (sm_100a).
//
// Integer semantics follow PyTorch's int64 kernels, which the reference's
// strict path runs on (ecoint8/fixedpoint.py): products and sums wrap modulo
// 2^64, `a << s` is an unsigned shift that yields 0 for s >= 64, `a >> s` is
// arithmetic and saturates to the sign for s >= 64, and a floor division by
// 2^s is an arithmetic right shift.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/ecoint8_b200.h"

typedef long long i64;
typedef unsigned long long u64;

#define ECO_DEV __device__ __forceinline__

// ---------------------------------------------------------------- int64 wrap
ECO_DEV i64 mul64(i64 a, i64 b) { return (i64)((u64)a * (u64)b); }
ECO_DEV i64 add64(i64 a, i64 b) { return (i64)((u64)a + (u64)b); }
ECO_DEV i64 sub64(i64 a, i64 b) { return (i64)((u64)a - (u64)b); }
ECO_DEV i64 neg64(i64 a) { return (i64)(0ull - (u64)a); }
ECO_DEV i64 abs64(i64 a) { return a < 0 ? neg64(a) : a; }  // torch abs: INT64_MIN stays
ECO_DEV i64 shl64(i64 a, int s) { return s >= 64 ? 0 : (i64)((u64)a << s); }
ECO_DEV i64 sar64(i64 a, int s) { return a >> (s > 63 ? 63 : s); }
ECO_DEV int add32(int a, int b) { return (int)((unsigned)a + (unsigned)b); }
ECO_DEV int8_t sat8(i64 v) { return (int8_t)(v < -127 ? -127 : (v > 127 ? 127 : v)); }

// `apply_mult_shift` (fixedpoint.py:52-76) on one element: shift >= 0 rounds
// with `nudge` (either a U[0, 2^shift) draw or 2^(shift-1)); shift < 0 is a
// left shift with no draw.
ECO_DEV i64 ams(i64 x, i64 mult, int shift, i64 nudge) {
  i64 p = mul64(x, mult);
  return shift >= 0 ? sar64(add64(p, nudge), shift) : shl64(p, -shift);
}
ECO_DEV i64 half_nudge(int shift) { return shift > 0 ? (1ll << (shift - 1)) : 0; }
ECO_DEV i64 low_bits(u64 w, int n) { return n <= 0 ? 0 : (n >= 64 ? (i64)w : (i64)(w & ((1ull << n) - 1))); }

// 32x32 -> 64 products as single instructions (exact; two's complement sums).
ECO_DEV i64 mul_wide_s32(int a, int b) {
  i64 d;
  asm("mul.wide.s32 %0, %1, %2;" : "=l"(d) : "r"(a), "r"(b));
  return d;
}
ECO_DEV i64 mad_wide_s32(int a, int b, i64 c) {
  i64 d;
  asm("mad.wide.s32 %0, %1, %2, %3;" : "=l"(d) : "r"(a), "r"(b), "l"(c));
  return d;
}
ECO_DEV i64 mad_wide_u32(uint32_t a, uint32_t b, i64 c) {  // c + a * b modulo 2^64
  i64 d;
  asm("mad.wide.u32 %0, %1, %2, %3;" : "=l"(d) : "r"(a), "r"(b), "l"(c));
  return d;
}
ECO_DEV int hi32(i64 x) { return (int)(x >> 32); }
ECO_DEV uint32_t lo32(i64 x) { return (uint32_t)x; }
// (int)(x >> s) for 0 <= s < 32 when the result fits int32: one funnel shift.
ECO_DEV int shr_fit(i64 x, int s) { return (int)__funnelshift_r(lo32(x), (uint32_t)hi32(x), s); }

// Bytes of `w` that are > 0 as signed int8 -> 0xFF, others 0x00 (no carries cross bytes).
ECO_DEV uint32_t bytes_positive(uint32_t w) {
  const uint32_t t = (w & 0x7F7F7F7Fu) + 0x7F7F7F7Fu;  // bit 7: low seven bits nonzero
  const uint32_t k = t & ~w & 0x80808080u;            // ... and sign bit clear
  return (k >> 7) * 0xFFu;
}
// Byte k (0..3) of x, sign-extended: one byte permute whose upper selector nibbles
// replicate the byte's sign bit.
ECO_DEV int sbyte(uint32_t x, int k) {
  const uint32_t sel = (uint32_t)k | ((uint32_t)(k | 8) << 4) | ((uint32_t)(k | 8) << 8) | ((uint32_t)(k | 8) << 12);
  uint32_t d;
  asm("prmt.b32 %0, %1, 0, %2;" : "=r"(d) : "r"(x), "r"(sel));
  return (int)d;
}
// Low bytes of four ints packed into one word.
ECO_DEV uint32_t pack4(int a, int b, int c, int d) {
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}
// Four int32 saturated to [-128, 127] and packed into bytes (a lowest): two saturating
// pack conversions.
ECO_DEV uint32_t pack4_sat(int a, int b, int c, int d) {
  uint32_t hi, r;
  asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, 0;" : "=r"(hi) : "r"(d), "r"(c));
  asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(b), "r"(a), "r"(hi));
  return r;
}
// The same saturated to [-127, 127]: one per-byte max with -127 after the packs.
ECO_DEV uint32_t pack4_sat127(int a, int b, int c, int d) { return __vmaxs4(pack4_sat(a, b, c, d), 0x81818181u); }

// ---------------------------------------------------------------- Philox4x32-10
// Salmon et al., "Parallel random numbers: as easy as 1, 2, 3" (SC'11).
struct Philox4 {
  uint32_t x, y, z, w;
};
ECO_DEV Philox4 philox10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int i = 0; i < 10; ++i) {
    const u64 p0 = (u64)0xD2511F53u * c0;
    const u64 p1 = (u64)0xCD9E8D57u * c2;
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
    const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
    c1 = (uint32_t)p1;
    c3 = (uint32_t)p0;
    c0 = n0;
    c2 = n2;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return Philox4{c0, c1, c2, c3};
}

// The ten round keys of a Philox4x32-10 key (key + i * Weyl constants), computed
// once on the host.  Kernels keep them in their parameter block, so every round
// XORs a constant-bank operand instead of advancing two key registers.
struct PhiloxKeys {
  uint32_t k0[10], k1[10];
};
static inline __host__ __device__ PhiloxKeys philox_keys(u64 seed) {
  PhiloxKeys K;
  uint32_t a = (uint32_t)seed, b = (uint32_t)(seed >> 32);
  for (int i = 0; i < 10; ++i) {
    K.k0[i] = a;
    K.k1[i] = b;
    a += 0x9E3779B9u;
    b += 0xBB67AE85u;
  }
  return K;
}
ECO_DEV Philox4 philox10k(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, const PhiloxKeys& K) {
#pragma unroll
  for (int i = 0; i < 10; ++i) {
    const u64 p0 = (u64)0xD2511F53u * c0;
    const u64 p1 = (u64)0xCD9E8D57u * c2;
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ K.k0[i];
    const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ K.k1[i];
    c1 = (uint32_t)p1;
    c3 = (uint32_t)p0;
    c0 = n0;
    c2 = n2;
  }
  return Philox4{c0, c1, c2, c3};
}
// A site as a kernel uses it: ECO_SR_PHILOX_DEV becomes ECO_SR_PHILOX with the key
// read from device memory now (the launch may be a CUDA graph replay); `keys` gets the
// site's round keys (the host-computed ones of a plain Philox site).
ECO_DEV eco_sr_t sr_resolve(const eco_sr_t& in, const PhiloxKeys& host_keys, PhiloxKeys& keys) {
  eco_sr_t sr = in;
  if (sr.mode == ECO_SR_PHILOX_DEV) {
    sr.seed = *static_cast<const u64*>(in.nudge);
    sr.mode = ECO_SR_PHILOX;
    sr.nudge = nullptr;
    keys = philox_keys(sr.seed);
  } else {
    keys = host_keys;
  }
  return sr;
}
ECO_DEV eco_sr_t sr_resolve(const eco_sr_t& in) {
  PhiloxKeys unused;
  return sr_resolve(in, unused, unused);
}
// sr_quad with precomputed round keys (same bits).
ECO_DEV Philox4 sr_quad_k(const PhiloxKeys& K, u64 stream, uint32_t row, uint32_t quad) {
  return philox10k(quad, row, (uint32_t)stream, (uint32_t)(stream >> 32), K);
}

// The library's stochastic-rounding stream: 64 random bits for the column
// pair (2p, 2p+1) of row r at site `stream`: counter (p, r, stream_lo,
// stream_hi), key (seed_lo, seed_hi).  Even column -> (y:x), odd -> (w:z).
ECO_DEV void sr_pair(u64 seed, u64 stream, uint32_t row, uint32_t pair, u64& even, u64& odd) {
  const Philox4 o = philox10(pair, row, (uint32_t)stream, (uint32_t)(stream >> 32), (uint32_t)seed,
                             (uint32_t)(seed >> 32));
  even = ((u64)o.y << 32) | o.x;
  odd = ((u64)o.w << 32) | o.z;
}
ECO_DEV u64 sr_word(u64 seed, u64 stream, uint32_t row, uint32_t col) {
  u64 e, o;
  sr_pair(seed, stream, row, col >> 1, e, o);
  return (col & 1) ? o : e;
}

// The library's 32-bit stochastic-rounding field of element (row, col): word
// col & 3 of the Philox call with counter (col >> 2, row, stream_lo, stream_hi).
// One call serves four consecutive columns.
constexpr u64 kAltStream = 1ull << 63;  // a site's tie-break stream: its id with the top bit set
ECO_DEV Philox4 sr_quad(u64 seed, u64 stream, uint32_t row, uint32_t quad) {
  return philox10(quad, row, (uint32_t)stream, (uint32_t)(stream >> 32), (uint32_t)seed, (uint32_t)(seed >> 32));
}
ECO_DEV uint32_t quad_word(const Philox4& o, int k) { return k == 0 ? o.x : (k == 1 ? o.y : (k == 2 ? o.z : o.w)); }
ECO_DEV uint32_t sr_field(u64 seed, u64 stream, uint32_t row, uint32_t col) {
  return quad_word(sr_quad(seed, stream, row, col >> 2), col & 3);
}

// floor((p + u) / 2^c), 0 <= c <= 62, for the stream's nudge u of one element,
// with int64 wrap-around like the reference.  u's top bits are the element's
// field f; for c > 32 its low c-32 bits are the tie-break stream's field, which
// only matters when bits [c-32, c) of p + (f << (c-32)) are all ones (adding
// fewer than 2^(c-32) can only then carry into bit c): probability 2^-32.
static __device__ __noinline__ i64 sr_round_tie(i64 p2, int c, u64 seed, u64 stream, uint32_t row, uint32_t col) {
  const int lo = c - 32;
  const uint32_t t = sr_field(seed, stream | kAltStream, row, col);
  return sar64(add64(p2, (i64)(t & ((1u << lo) - 1u))), c);
}
ECO_DEV i64 sr_round(i64 p, int c, uint32_t f, u64 seed, u64 stream, uint32_t row, uint32_t col) {
  if (c <= 32) {
    const u64 u = c == 32 ? (u64)f : (u64)(f & ((1u << c) - 1u));
    return sar64(add64(p, (i64)u), c);
  }
  const int lo = c - 32;
  const i64 p2 = add64(p, (i64)((u64)f << lo));
  if ((uint32_t)((u64)p2 >> lo) != 0xFFFFFFFFu) return p2 >> c;
  return sr_round_tie(p2, c, seed, stream, row, col);
}

// The I8ECO step's momentum rounding: u's top 20 bits are bits 12..31 of the
// element's field (bits 0..11 are the weight nudge); for c > 20 the low c-20
// bits come from the tie-break stream's 64-bit word, needed only when bits
// [c-20, c) of p + (top << (c-20)) are all ones (probability 2^-20).
static __device__ __noinline__ i64 step_m_round_tie(i64 p2, int c, u64 seed, u64 stream, uint32_t row, uint32_t col) {
  const int lo = c - 20;
  const u64 t = sr_word(seed, stream | kAltStream, row, col);
  return sar64(add64(p2, (i64)(t & ((1ull << lo) - 1ull))), c);
}
ECO_DEV i64 step_m_round(i64 p, int c, uint32_t field, u64 seed, u64 stream, uint32_t row, uint32_t col) {
  const uint32_t top = field >> 12;
  if (c <= 20) return sar64(add64(p, (i64)(top & ((1u << c) - 1u))), c);
  const int lo = c - 20;
  const i64 p2 = add64(p, (i64)((u64)top << lo));
  if ((((u64)p2 >> lo) & 0xFFFFFull) != 0xFFFFFull) return sar64(p2, c);
  return step_m_round_tie(p2, c, seed, stream, row, col);
}

// Triton's tl.rand(seed, offset) for an int32 offset: Philox counter
// (offset, 0, 0, 0); first word as int32, folded to non-negative, times fp32
// 4.6566127342e-10 (triton/language/random.py, triton 3.6.0).
ECO_DEV float tl_rand(u64 seed, uint32_t offset) {
  const Philox4 o = philox10(offset, 0u, 0u, 0u, (uint32_t)seed, (uint32_t)(seed >> 32));
  int x = (int)o.x;
  x = x < 0 ? -x - 1 : x;
  return __fmul_rn(__int2float_rn(x), 4.6566127342e-10f);
}

// ---------------------------------------------------------------- fixed point
// quantize_multiplier (fixedpoint.py:26-37) in IEEE double: frexp is exact,
// mantissa * 2^31 is exact, and rint rounds half to even like Python's round.
ECO_DEV void qmult(double r, int& mult, int& shift) {
  if (r == 0.0) {
    mult = 0;
    shift = 0;
    return;
  }
  int e;
  const double mant = frexp(r, &e);
  i64 m = (i64)rint(__dmul_rn(mant, 2147483648.0));
  if (m == (1ll << 31)) {
    m >>= 1;
    e += 1;
  }
  mult = (int)m;
  shift = 31 - e;
}

// Error flags a kernel can raise in its error word (host turns them into exceptions).
enum : unsigned {
  ECO_FLAG_SHIFT_OVERFLOW = 1u,  // a requant shift beyond 62 (the reference raises)
  ECO_FLAG_BAD_RATIO = 2u,       // a zero / non-finite scale ratio
  ECO_FLAG_WAIT_TIMEOUT = 4u,    // a bounded device wait gave up
};

// ---------------------------------------------------------------- misc
static inline int eco_ceil_div(i64 a, i64 b) { return (int)((a + b - 1) / b); }
