// Memory-bound integer kernels of the strict path: int32 -> int8 requant with
// fused bias / ReLU / mask / square-sum, the general apply_mult_shift, column
// sums, max-abs and square-sum reductions.
#include <algorithm>

#include "abi.cuh"
#include "common.cuh"

namespace {

constexpr int kThreads = 256;

template <typename T>
ECO_DEV T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
ECO_DEV i64 warp_max64(i64 v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, (i64)__shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide reduction of one int64 into a global word (sum or max).
template <bool MAX>
ECO_DEV void block_reduce_to(i64 v, i64* out) {
  __shared__ i64 part[kThreads / 32];
  v = MAX ? warp_max64(v) : (i64)warp_sum((u64)v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) part[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < (int)(blockDim.x >> 5) ? part[lane] : (MAX ? (i64)INT64_MIN : 0);
    v = MAX ? warp_max64(v) : (i64)warp_sum((u64)v);
    if (lane == 0) {
      if (MAX)
        atomicMax(reinterpret_cast<long long*>(out), (long long)v);
      else
        atomicAdd(reinterpret_cast<unsigned long long*>(out), (unsigned long long)v);
    }
  }
}

ECO_DEV i64 replay_nudge(const eco_sr_t& sr, i64 r, i64 c) {
  const i64 idx = r * sr.nudge_ld + c;
  return sr.mode == ECO_SR_REPLAY32 ? (i64)(static_cast<const int32_t*>(sr.nudge)[idx])
                                    : static_cast<const i64*>(sr.nudge)[idx];
}

// floor((p + nudge) / 2^shift) (or p << -shift) for element (r, c) under the
// site's rounding mode; f is the element's Philox field (Philox mode only).
ECO_DEV i64 round_elem(const eco_sr_t& sr, int shift, i64 p, i64 r, i64 c, uint32_t f) {
  if (shift < 0) return shl64(p, -shift);
  if (sr.mode == ECO_SR_NEAREST) return sar64(add64(p, half_nudge(shift)), shift);
  if (sr.mode == ECO_SR_PHILOX)
    return sr_round(p, shift, f, sr.seed, sr.stream, (uint32_t)(sr.row_base + r), (uint32_t)c);
  return sar64(add64(p, replay_nudge(sr, r, c)), shift);
}

struct RequantArgs {
  const int32_t* src;
  i64 rows, cols, ld_src;
  const int32_t* bias;
  const int32_t* mult_col;
  i64 mult_scalar;
  int shift, relu;
  eco_sr_t sr;
  const int8_t* mask;
  i64 ld_mask;
  int8_t* dst;
  i64 ld_dst;
  i64* sumsq;
  int mult32;  // mult_scalar fits int32: 32x32->64 products
  PhiloxKeys keys;  // round keys of sr.seed (Philox mode)
  const i64* dparams;  // nullable: [_, mult, shift] on the device (eco_scale_from_amax) replace
                       // mult_scalar and shift; a shift beyond 62 stores zeros (already flagged)
};

// MODE: 0 round half up, 1 Philox, 2 replay.  One thread handles 16 consecutive
// columns of a row per iteration (one 64-byte load of int32, one 16-byte store).
template <bool VEC, int MODE>
__global__ void __launch_bounds__(kThreads) requant_kernel(const RequantArgs a) {
  PhiloxKeys keys;
  const eco_sr_t sr = sr_resolve(a.sr, a.keys, keys);
  const i64 cpr = (a.cols + 15) / 16;
  const i64 total = a.rows * cpr;
  const int shift = a.dparams ? (int)a.dparams[2] : a.shift;
  const i64 mult_scalar = a.dparams ? a.dparams[1] : a.mult_scalar;
  const bool mult32 = a.dparams ? true : a.mult32;
  const bool zero_out = shift > 62;
  const bool left = shift < 0;
  i64 sq = 0;
  for (i64 t = (i64)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (i64)gridDim.x * blockDim.x) {
    const i64 r = t / cpr;
    const i64 c0 = (t - r * cpr) * 16;
    int v[16];
    if (VEC) {
      const int4* p = reinterpret_cast<const int4*>(a.src + r * a.ld_src + c0);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int4 x = p[q];
        v[4 * q] = x.x; v[4 * q + 1] = x.y; v[4 * q + 2] = x.z; v[4 * q + 3] = x.w;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 16; ++e) v[e] = (c0 + e < a.cols) ? a.src[r * a.ld_src + c0 + e] : 0;
    }
    uint32_t packed[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      Philox4 rnd{0u, 0u, 0u, 0u};
      if (MODE == 1 && !left && !zero_out)
        rnd = sr_quad_k(keys, sr.stream, (uint32_t)(sr.row_base + r), (uint32_t)((c0 >> 2) + q));
      packed[q] = 0u;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int e = 4 * q + k;
        const i64 c = c0 + e;
        const bool in = VEC || c < a.cols;
        int x = v[e];
        if (a.bias && in) x = add32(x, a.bias[c]);
        const i64 prod = a.mult_col ? (i64)x * (i64)(in ? a.mult_col[c] : 0)
                                    : (mult32 ? (i64)x * (i64)(int)mult_scalar : mul64((i64)x, mult_scalar));
        i64 yv;
        if (zero_out)
          yv = 0;
        else if (left)
          yv = shl64(prod, -shift);
        else if (MODE == 0)
          yv = sar64(add64(prod, half_nudge(shift)), shift);
        else if (MODE == 1)
          yv = sr_round(prod, shift, quad_word(rnd, k), sr.seed, sr.stream, (uint32_t)(sr.row_base + r),
                        (uint32_t)c);
        else
          yv = in ? sar64(add64(prod, replay_nudge(sr, r, c)), shift) : 0;
        int8_t y = sat8(yv);
        if (a.relu && y < 0) y = 0;
        if (a.mask && in && a.mask[r * a.ld_mask + c] <= 0) y = 0;
        if (!in) y = 0;
        sq += (i64)y * y;
        packed[q] |= (uint32_t)(uint8_t)y << (8 * k);
      }
    }
    if (VEC) {
      *reinterpret_cast<int4*>(a.dst + r * a.ld_dst + c0) = make_int4(packed[0], packed[1], packed[2], packed[3]);
    } else {
#pragma unroll
      for (int e = 0; e < 16; ++e)
        if (c0 + e < a.cols) a.dst[r * a.ld_dst + c0 + e] = (int8_t)(packed[e / 4] >> (8 * (e % 4)));
    }
  }
  if (a.sumsq) block_reduce_to<false>(sq, a.sumsq);
}

// Philox requant of a 16-byte aligned, multiple-of-16-wide matrix, specialized at
// compile time: MASK (zero where mask <= 0), SUMSQ, COLM (per-column multipliers),
// BIAS, BIG (shift > 32).  A block walks rows (no index division); a thread takes 16
// columns per iteration: one 64-byte load, one 16-byte mask load, one 16-byte store,
// four Philox calls.  0 <= shift <= 62, and with |x * mult| < 2^62 every result of
// a shift > 32 fits int32, so the tail arithmetic is 32-bit.
template <bool MASK, bool SUMSQ, bool COLM, bool BIAS, bool BIG>
ECO_DEV void requant_philox_body(const RequantArgs& a, int sh) {
  PhiloxKeys keys;
  const eco_sr_t sr = sr_resolve(a.sr, a.keys, keys);
  const int cpr = (int)(a.cols >> 4);
  const bool zero_out = sh > 62;
  const int lo = sh - 32;  // BIG: bits of the tie-break draw
  const uint32_t pow2lo = BIG ? 1u << lo : 0u;
  const int32_t mult_s = (int32_t)(a.dparams ? a.dparams[1] : a.mult_scalar);
  long long sq = 0;
  // The block's work is the chunk sequence (row r, chunk j) with rows blockIdx.x +
  // k * gridDim.x; thread t takes every blockDim.x-th chunk of it, and the next
  // chunk's loads (possibly in the next row) are in flight while one computes.
  i64 r = blockIdx.x;
  int j = threadIdx.x;
  while (j >= cpr && r < a.rows) {
    j -= cpr;
    r += gridDim.x;
  }
  int4 nx[4], nm = make_int4(0, 0, 0, 0);
  if (r < a.rows) {
#pragma unroll
    for (int q = 0; q < 4; ++q) nx[q] = reinterpret_cast<const int4*>(a.src + r * a.ld_src + j * 16)[q];
    if (MASK) nm = *reinterpret_cast<const int4*>(a.mask + r * a.ld_mask + j * 16);
  }
  while (r < a.rows) {
    const i64 cr = r;
    const int c0 = j * 16;
    int v[16];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      v[4 * q] = nx[q].x; v[4 * q + 1] = nx[q].y; v[4 * q + 2] = nx[q].z; v[4 * q + 3] = nx[q].w;
    }
    const int4 mk = nm;
    j += blockDim.x;
    while (j >= cpr && r < a.rows) {
      j -= cpr;
      r += gridDim.x;
    }
    if (r < a.rows) {
#pragma unroll
      for (int q = 0; q < 4; ++q) nx[q] = reinterpret_cast<const int4*>(a.src + r * a.ld_src + j * 16)[q];
      if (MASK) nm = *reinterpret_cast<const int4*>(a.mask + r * a.ld_mask + j * 16);
    }
    const uint32_t grow = (uint32_t)(sr.row_base + cr);
    const uint32_t* mw = reinterpret_cast<const uint32_t*>(&mk);
    uint32_t packed[4];
    int sq32 = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const Philox4 rnd = sr_quad_k(keys, sr.stream, grow, (uint32_t)((c0 >> 2) + q));
      int y4[4];
      uint32_t tf[4] = {0u, 0u, 0u, 0u};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int e = 4 * q + k;
        const int c = c0 + e;
        int x = v[e];
        if (BIAS) x = add32(x, a.bias[c]);
        const i64 prod = mul_wide_s32(x, COLM ? a.mult_col[c] : mult_s);
        const uint32_t f = quad_word(rnd, k);
        int y;
        if (BIG) {
          const i64 p2 = mad_wide_u32(f, pow2lo, prod);  // prod + (f << lo)
          // the tie-break draw matters only when bits [lo, lo + 32) of p2 are all ones
          tf[k] = __funnelshift_r(lo32(p2), (uint32_t)hi32(p2), lo);
          y = hi32(p2) >> lo;  // (p2 >> shift) fits int32
        } else if (sh >= 0 && !zero_out) {
          const u64 u = sh == 32 ? (u64)f : (u64)(f & ((1u << sh) - 1u));
          const i64 t = sar64(prod + (i64)u, sh);
          y = t < -128 ? -128 : (t > 128 ? 128 : (int)t);
        } else if (!zero_out) {  // left shift: no draw
          const i64 t = shl64(prod, -sh);
          y = t < -128 ? -128 : (t > 128 ? 128 : (int)t);
        } else {
          y = 0;
        }
        y4[k] = y;
      }
      // rare (2^-32 per element): the tied elements take the exact draw
      if (BIG && __vimax3_u32(__vimax3_u32(tf[0], tf[1], tf[2]), tf[3], 0u) == 0xFFFFFFFFu) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (tf[k] != 0xFFFFFFFFu) continue;
          const int c = c0 + 4 * q + k;
          int x = v[4 * q + k];
          if (BIAS) x = add32(x, a.bias[c]);
          const i64 prod = mul_wide_s32(x, COLM ? a.mult_col[c] : mult_s);
          y4[k] = (int)max((i64)-128, min((i64)128, sr_round(prod, sh, quad_word(rnd, k), sr.seed, sr.stream,
                                                             grow, (uint32_t)c)));
        }
      }
      // saturate to [-128, 127] in the packs, then to [-127 or 0 (ReLU), 127] per byte
      packed[q] = __vmaxs4(pack4_sat(y4[0], y4[1], y4[2], y4[3]), a.relu ? 0u : 0x81818181u);
      if (MASK) packed[q] &= bytes_positive(mw[q]);
      if (SUMSQ) sq32 = __dp4a((int)packed[q], (int)packed[q], sq32);  // the four squares
    }
    if (SUMSQ) sq += sq32;
    *reinterpret_cast<int4*>(a.dst + cr * a.ld_dst + c0) = make_int4(packed[0], packed[1], packed[2], packed[3]);
  }
  if (SUMSQ) block_reduce_to<false>(sq, a.sumsq);
}

template <bool MASK, bool SUMSQ, bool COLM, bool BIAS, bool BIG>
__global__ void __launch_bounds__(kThreads) requant_philox_kernel(const RequantArgs a) {
  requant_philox_body<MASK, SUMSQ, COLM, BIAS, BIG>(a, a.shift);
}

// The requant whose multiplier and shift the device computed (eco_scale_from_amax):
// one launch that takes the wide (shift 33..62) or the narrow path by the shift it
// reads; a shift beyond 62 or below 0 is the narrow path's.
template <bool MASK, bool SUMSQ>
__global__ void __launch_bounds__(kThreads) requant_philox_dev_kernel(const RequantArgs a) {
  const int sh = (int)a.dparams[2];
  if (sh > 32 && sh <= 62)
    requant_philox_body<MASK, SUMSQ, false, false, true>(a, sh);
  else
    requant_philox_body<MASK, SUMSQ, false, false, false>(a, sh);
}

struct AmsArgs {
  const void* x;
  int x_bits;
  i64 rows, cols;
  const int32_t* mult;
  int mult_kind;
  i64 mult_scalar;
  int shift;
  eco_sr_t sr;
  i64* out;
};

__global__ void __launch_bounds__(kThreads) ams_kernel(const AmsArgs a) {
  const eco_sr_t sr = sr_resolve(a.sr);
  const i64 n = a.rows * a.cols;
  for (i64 i = (i64)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (i64)gridDim.x * blockDim.x) {
    const i64 r = i / a.cols, c = i - r * a.cols;
    i64 x = a.x_bits == 8 ? (i64)static_cast<const int8_t*>(a.x)[i]
            : a.x_bits == 32 ? (i64)static_cast<const int32_t*>(a.x)[i]
                             : static_cast<const i64*>(a.x)[i];
    const i64 m = a.mult_kind == 0 ? a.mult_scalar : (a.mult_kind == 1 ? a.mult[c] : a.mult[r]);
    const uint32_t f = (sr.mode == ECO_SR_PHILOX && a.shift >= 0)
                           ? sr_field(sr.seed, sr.stream, (uint32_t)(sr.row_base + r), (uint32_t)c)
                           : 0u;
    a.out[i] = round_elem(sr, a.shift, mul64(x, m), r, c, f);
  }
}

__global__ void __launch_bounds__(kThreads) colsum_kernel(const int8_t* g, i64 rows, i64 cols, i64 ld,
                                                          i64* out, i64 rows_per_block) {
  const i64 c = (i64)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  const i64 r0 = (i64)blockIdx.y * rows_per_block;
  const i64 r1 = min(rows, r0 + rows_per_block);
  i64 s = 0;
  for (i64 r = r0; r < r1; ++r) s += g[r * ld + c];
  atomicAdd(reinterpret_cast<unsigned long long*>(out + c), (unsigned long long)s);
}

// Column sums with 16 columns per thread (one 16-byte load per row; rows 16-byte aligned):
// the block's rows [r0, r1) summed in int32 (|sum| <= 127 * rows_per_block), then one int64
// atomic add per column and block.  Memory-bound: 1 B read per element.
__global__ void __launch_bounds__(kThreads) colsum16_kernel(const int8_t* __restrict__ g, i64 rows, i64 cols, i64 ld,
                                                            i64* out, i64 rows_per_block) {
  const i64 c0 = ((i64)blockIdx.x * blockDim.x + threadIdx.x) * 16;
  if (c0 >= cols) return;
  const i64 r0 = (i64)blockIdx.y * rows_per_block;
  const i64 r1 = min(rows, r0 + rows_per_block);
  int sum[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) sum[e] = 0;
  if (c0 + 16 <= cols) {
#pragma unroll 8
    for (i64 r = r0; r < r1; ++r) {  // eight rows' loads in flight per thread
      const int4 v = __ldg(reinterpret_cast<const int4*>(g + r * ld + c0));
      const uint32_t w[4] = {(uint32_t)v.x, (uint32_t)v.y, (uint32_t)v.z, (uint32_t)v.w};
#pragma unroll
      for (int e = 0; e < 16; ++e) sum[e] += sbyte(w[e >> 2], e & 3);
    }
  } else {
    for (i64 r = r0; r < r1; ++r)
#pragma unroll
      for (int e = 0; e < 16; ++e)
        if (c0 + e < cols) sum[e] += g[r * ld + c0 + e];
  }
#pragma unroll
  for (int e = 0; e < 16; ++e)
    if (c0 + e < cols) atomicAdd(reinterpret_cast<unsigned long long*>(out + c0 + e), (unsigned long long)(i64)sum[e]);
}

__global__ void __launch_bounds__(kThreads) amax_kernel(const void* x, int bits, i64 n, i64* out) {
  i64 m = INT64_MIN;
  for (i64 i = (i64)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (i64)gridDim.x * blockDim.x) {
    i64 v;
    if (bits == 32) {  // int32 abs wraps like torch: |INT32_MIN| stays negative
      const int xi = static_cast<const int32_t*>(x)[i];
      v = (i64)(int)(xi < 0 ? 0u - (unsigned)xi : (unsigned)xi);
    } else {
      v = abs64(static_cast<const i64*>(x)[i]);
    }
    m = max(m, v);
  }
  block_reduce_to<true>(m, out);
}

__global__ void __launch_bounds__(kThreads) sumsq_s8_kernel(const int8_t* x, i64 n, i64* out) {
  i64 s = 0;
  const i64 n16 = ((reinterpret_cast<uintptr_t>(x) & 15) == 0) ? n / 16 : 0;
  for (i64 i = (i64)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (i64)gridDim.x * blockDim.x) {
    const int4 q = reinterpret_cast<const int4*>(x)[i];
    const int8_t* b = reinterpret_cast<const int8_t*>(&q);
#pragma unroll
    for (int e = 0; e < 16; ++e) s += (i64)b[e] * b[e];
  }
  for (i64 i = n16 * 16 + (i64)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (i64)gridDim.x * blockDim.x)
    s += (i64)x[i] * x[i];
  block_reduce_to<false>(s, out);
}

__global__ void set_i64_kernel(i64* p, i64 v) { *p = v; }

int grid_for(i64 work, int per_sm = 8) {
  const i64 cap = (i64)eco_num_sms() * per_sm;
  return (int)std::max<i64>(1, std::min<i64>(cap, (work + kThreads - 1) / kThreads));
}

}  // namespace

// dX / dW requant whose scalar multiplier and shift were computed on the device
// (eco_scale_from_amax); Philox stochastic rounding only.
extern "C" int eco_requant_s32_s8_dev(const int32_t* src, int64_t rows, int64_t cols, int64_t ld_src,
                                      const int64_t* params, int relu, eco_sr_t sr, const int8_t* mask,
                                      int64_t ld_mask, int8_t* dst, int64_t ld_dst, int64_t* sumsq,
                                      eco_stream_t stream) {
  ECO_REQUIRE(src && dst && params && rows >= 0 && cols >= 0 && ld_src >= cols && ld_dst >= cols, ECO_ERR_ARG,
              "eco_requant_s32_s8_dev: bad arguments");
  ECO_REQUIRE(!mask || ld_mask >= cols, ECO_ERR_ARG, "eco_requant_s32_s8_dev: bad mask leading dim");
  ECO_REQUIRE(sr.mode == ECO_SR_PHILOX || sr.mode == ECO_SR_PHILOX_DEV, ECO_ERR_ARG,
              "eco_requant_s32_s8_dev: Philox rounding only");
  if (int rc = eco_check_sr(sr, 0, "eco_requant_s32_s8_dev")) return rc;
  cudaStream_t s = eco_stream(stream);
  if (sumsq && cudaMemsetAsync(sumsq, 0, sizeof(int64_t), s) != cudaSuccess)
    return eco_launch_check("eco_requant_s32_s8_dev memset");
  if (rows == 0 || cols == 0) return ECO_OK;
  RequantArgs a{src, rows, cols, ld_src, nullptr, nullptr, 0, 0, relu, sr,
                mask, ld_mask, dst, ld_dst, reinterpret_cast<i64*>(sumsq), 1,
                philox_keys(sr.mode == ECO_SR_PHILOX ? sr.seed : 0), reinterpret_cast<const i64*>(params)};
  const bool vec = cols % 16 == 0 && eco_aligned16(src) && ld_src % 4 == 0 && eco_aligned16(dst) &&
                   ld_dst % 16 == 0 && (!mask || (eco_aligned16(mask) && ld_mask % 16 == 0));
  if (vec) {
    const int gp = (int)std::max<i64>(1, std::min<i64>(rows, (i64)eco_num_sms() * 8));
#define ECO_RQD(M, Q) requant_philox_dev_kernel<M, Q><<<gp, kThreads, 0, s>>>(a)
    if (mask) {
      if (sumsq) ECO_RQD(true, true); else ECO_RQD(true, false);
    } else {
      if (sumsq) ECO_RQD(false, true); else ECO_RQD(false, false);
    }
#undef ECO_RQD
    return eco_launch_check("eco_requant_s32_s8_dev");
  }
  const int g = grid_for(rows * ((cols + 15) / 16));
  requant_kernel<false, 1><<<g, kThreads, 0, s>>>(a);
  return eco_launch_check("eco_requant_s32_s8_dev");
}

extern "C" int eco_requant_s32_s8(const int32_t* src, int64_t rows, int64_t cols, int64_t ld_src,
                                  const int32_t* bias_col, const int32_t* mult_col, int64_t mult_scalar,
                                  int shift, int relu, eco_sr_t sr, const int8_t* mask, int64_t ld_mask,
                                  int8_t* dst, int64_t ld_dst, int64_t* sumsq, eco_stream_t stream) {
  ECO_REQUIRE(src && dst && rows >= 0 && cols >= 0 && ld_src >= cols && ld_dst >= cols, ECO_ERR_ARG,
              "eco_requant_s32_s8: bad arguments");
  ECO_REQUIRE(!mask || ld_mask >= cols, ECO_ERR_ARG, "eco_requant_s32_s8: bad mask leading dim");
  if (int rc = eco_check_sr(sr, shift, "eco_requant_s32_s8")) return rc;
  cudaStream_t s = eco_stream(stream);
  if (sumsq && cudaMemsetAsync(sumsq, 0, sizeof(int64_t), s) != cudaSuccess)
    return eco_launch_check("eco_requant_s32_s8 memset");
  if (rows == 0 || cols == 0) return ECO_OK;
  RequantArgs a{src, rows, cols, ld_src, bias_col, mult_col, mult_scalar, shift, relu, sr,
                mask, ld_mask, dst, ld_dst, reinterpret_cast<i64*>(sumsq),
                mult_scalar >= INT32_MIN && mult_scalar <= INT32_MAX,
                philox_keys(sr.mode == ECO_SR_PHILOX ? sr.seed : 0), nullptr};
  const bool replay = sr.mode == ECO_SR_REPLAY32 || sr.mode == ECO_SR_REPLAY64;
  const bool vec = cols % 16 == 0 && eco_aligned16(src) && ld_src % 4 == 0 && eco_aligned16(dst) &&
                   ld_dst % 16 == 0 && (!mask || (eco_aligned16(mask) && ld_mask % 16 == 0)) &&
                   (!bias_col || eco_aligned16(bias_col)) && (!mult_col || eco_aligned16(mult_col));
  (void)replay;
  const i64 work = rows * ((cols + 15) / 16);
  const int mode =
      sr.mode == ECO_SR_NEAREST ? 0 : ((sr.mode == ECO_SR_PHILOX || sr.mode == ECO_SR_PHILOX_DEV) ? 1 : 2);
  const bool mult_ok = mult_col || (mult_scalar >= INT32_MIN && mult_scalar <= INT32_MAX);
  if (vec && mode == 1 && shift >= 0 && mult_ok) {
    const int gp = (int)std::max<i64>(1, std::min<i64>(rows, (i64)eco_num_sms() * 8));
    const bool big = shift > 32, m = mask != nullptr, q = sumsq != nullptr, cm = mult_col != nullptr,
               b = bias_col != nullptr;
#define ECO_RQP(M, Q, CM, B, BG) requant_philox_kernel<M, Q, CM, B, BG><<<gp, kThreads, 0, s>>>(a)
#define ECO_RQP_BIG(M, Q, CM, B) \
  do {                           \
    if (big) ECO_RQP(M, Q, CM, B, true); else ECO_RQP(M, Q, CM, B, false); \
  } while (0)
#define ECO_RQP_B(M, Q, CM) \
  do {                      \
    if (b) ECO_RQP_BIG(M, Q, CM, true); else ECO_RQP_BIG(M, Q, CM, false); \
  } while (0)
#define ECO_RQP_CM(M, Q) \
  do {                   \
    if (cm) ECO_RQP_B(M, Q, true); else ECO_RQP_B(M, Q, false); \
  } while (0)
    if (m) {
      if (q) ECO_RQP_CM(true, true); else ECO_RQP_CM(true, false);
    } else {
      if (q) ECO_RQP_CM(false, true); else ECO_RQP_CM(false, false);
    }
#undef ECO_RQP_CM
#undef ECO_RQP_B
#undef ECO_RQP_BIG
#undef ECO_RQP
    return eco_launch_check("eco_requant_s32_s8");
  }
  const int g = grid_for(work);
#define ECO_REQUANT_LAUNCH(V, M) requant_kernel<V, M><<<g, kThreads, 0, s>>>(a)
  if (vec) {
    if (mode == 0) ECO_REQUANT_LAUNCH(true, 0);
    else if (mode == 1) ECO_REQUANT_LAUNCH(true, 1);
    else ECO_REQUANT_LAUNCH(true, 2);
  } else {
    if (mode == 0) ECO_REQUANT_LAUNCH(false, 0);
    else if (mode == 1) ECO_REQUANT_LAUNCH(false, 1);
    else ECO_REQUANT_LAUNCH(false, 2);
  }
#undef ECO_REQUANT_LAUNCH
  return eco_launch_check("eco_requant_s32_s8");
}

extern "C" int eco_apply_mult_shift(const void* x, int x_bits, int64_t rows, int64_t cols,
                                    const int32_t* mult, int mult_kind, int64_t mult_scalar, int shift,
                                    eco_sr_t sr, int64_t* out, eco_stream_t stream) {
  ECO_REQUIRE(x && out && rows >= 0 && cols >= 0, ECO_ERR_ARG, "eco_apply_mult_shift: bad arguments");
  ECO_REQUIRE(x_bits == 8 || x_bits == 32 || x_bits == 64, ECO_ERR_ARG, "eco_apply_mult_shift: x_bits");
  ECO_REQUIRE(mult_kind >= 0 && mult_kind <= 2 && (mult_kind == 0 || mult), ECO_ERR_ARG,
              "eco_apply_mult_shift: mult_kind");
  if (int rc = eco_check_sr(sr, shift, "eco_apply_mult_shift")) return rc;
  if (rows * cols == 0) return ECO_OK;
  AmsArgs a{x, x_bits, rows, cols, mult, mult_kind, mult_scalar, shift, sr, reinterpret_cast<i64*>(out)};
  ams_kernel<<<grid_for(rows * cols), kThreads, 0, eco_stream(stream)>>>(a);
  return eco_launch_check("eco_apply_mult_shift");
}

extern "C" int eco_colsum_s8(const int8_t* g, int64_t rows, int64_t cols, int64_t ld, int64_t* out,
                             eco_stream_t stream) {
  ECO_REQUIRE(g && out && rows >= 0 && cols >= 0 && ld >= cols, ECO_ERR_ARG, "eco_colsum_s8: bad arguments");
  cudaStream_t s = eco_stream(stream);
  if (cudaMemsetAsync(out, 0, sizeof(int64_t) * (size_t)cols, s) != cudaSuccess)
    return eco_launch_check("eco_colsum_s8 memset");
  if (rows == 0 || cols == 0) return ECO_OK;
  if (eco_aligned16(g) && (ld % 16 == 0 || rows == 1)) {
    // about two blocks per SM: 16 columns per thread, the rows split between the blocks
    const i64 threads16 = (cols + 15) / 16;
    const int block = (int)std::min<i64>(kThreads, (threads16 + 31) / 32 * 32);
    const i64 gx = (threads16 + block - 1) / block;
    const i64 gy = std::min<i64>(rows, std::max<i64>(1, 2 * (i64)eco_num_sms() / gx));
    const i64 rpb = std::min<i64>((rows + gy - 1) / gy, 1 << 24);
    dim3 grid((unsigned)gx, (unsigned)((rows + rpb - 1) / rpb));
    colsum16_kernel<<<grid, block, 0, s>>>(g, rows, cols, ld, reinterpret_cast<i64*>(out), rpb);
    return eco_launch_check("eco_colsum_s8");
  }
  const i64 rpb = std::max<i64>(64, (rows + 65534) / 65535);
  dim3 grid((unsigned)((cols + kThreads - 1) / kThreads), (unsigned)((rows + rpb - 1) / rpb));
  colsum_kernel<<<grid, kThreads, 0, s>>>(g, rows, cols, ld, reinterpret_cast<i64*>(out), rpb);
  return eco_launch_check("eco_colsum_s8");
}

extern "C" int eco_amax(const void* x, int x_bits, int64_t n, int64_t* out, eco_stream_t stream) {
  ECO_REQUIRE(x && out && n >= 0 && (x_bits == 32 || x_bits == 64), ECO_ERR_ARG, "eco_amax: bad arguments");
  cudaStream_t s = eco_stream(stream);
  // start from INT64_MIN so an all-INT_MIN input keeps torch's wrapped value
  set_i64_kernel<<<1, 1, 0, s>>>(reinterpret_cast<i64*>(out), INT64_MIN);
  if (n == 0) return eco_launch_check("eco_amax init");
  amax_kernel<<<grid_for(n), kThreads, 0, s>>>(x, x_bits, n, reinterpret_cast<i64*>(out));
  return eco_launch_check("eco_amax");
}

extern "C" int eco_sumsq_s8(const int8_t* x, int64_t n, int64_t* out, eco_stream_t stream) {
  ECO_REQUIRE(x && out && n >= 0, ECO_ERR_ARG, "eco_sumsq_s8: bad arguments");
  cudaStream_t s = eco_stream(stream);
  if (cudaMemsetAsync(out, 0, sizeof(int64_t), s) != cudaSuccess) return eco_launch_check("eco_sumsq_s8 memset");
  if (n == 0) return ECO_OK;
  sumsq_s8_kernel<<<grid_for(n / 16 + 1), kThreads, 0, s>>>(x, n, reinterpret_cast<i64*>(out));
  return eco_launch_check("eco_sumsq_s8");
}
