// Fused single-pass integer ECO-SGDM step over many layers (I8ECO.step,
// ecoint8/strict/iopt.py:103-200), one launch, no host synchronisation.
//
// Layout: each layer's w, m, g are [rows, cols] int8 row-major in HBM.  The
// launch walks "tiles" of whole rows (rows_per_tile rows of one layer); a
// warp owns one row at a time and streams it with 16-byte loads, so the per-
// row fixed-point multipliers (iopt.py:134-148) are computed once per row in
// IEEE double and every element is one pass of int64 register arithmetic:
// read w, m, g (3 B) and write w, m (2 B).
//
// The common shift of a multiplier column is min over rows of the row shift;
// quantize_multiplier's shift is non-increasing in the ratio and each ratio is
// monotone in sw[o], so the common shift is the shift of the ratio at min(sw)
// (or max(sw) for the momentum requant column), computed per CTA in O(1).
//
// The new momentum scale (iopt.py:178-180) needs max over rows of
// rowmax_o * sw_o / 4096: every warp folds its rows into a CTA maximum, one
// atomicMax per CTA on the double's bits (non-negative doubles order like
// their bit patterns), and the last CTA to finish turns it into s_m and resets
// the accumulator and the completion counter for the next step.
#include <algorithm>

#include "abi.cuh"
#include "common.cuh"

namespace {

// One warp per block, twelve blocks per SM: the fast row path keeps ~166 registers per
// thread without spills (a 128-register cap spilled), and single-warp blocks walk their row
// tiles independently (64 x 4096^2: 3.58 ms against 3.89 ms with 256-thread blocks at two
// blocks per SM).
constexpr int kThreads = 32;
constexpr int kBlocksPerSM = 12;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxLayers = 80;  // per launch (kernel parameter space)

struct LayerDesc {
  eco_i8eco_layer_t L;
  i64 tile_begin;
  int rows_per_tile;
  int vec;  // cols % 16 == 0 and 16-byte aligned rows
};

struct StepParams {
  eco_i8eco_hyper_t H;
  PhiloxKeys keys;  // round keys of H.seed
  int n_layers;
  i64 total_tiles;
  LayerDesc layers[kMaxLayers];
};

struct LayerScalars {
  double s_m, sm4096, sg4096, lr_sgb;
  int com_m, com_g, com_mm, com_b;
  unsigned flags;
};

ECO_DEV double bits_to_double(i64 b) { return __longlong_as_double(b); }

ECO_DEV int shift_of(double r, unsigned& flags) {
  if (!(r >= 0.0) || r > 1.7e308) {  // NaN, negative or infinite ratio
    flags |= ECO_FLAG_BAD_RATIO;
    return 0;
  }
  int m, s;
  qmult(r, m, s);
  return s;
}

ECO_DEV LayerScalars layer_scalars(const eco_i8eco_layer_t& L, const eco_i8eco_hyper_t& H) {
  LayerScalars S;
  S.flags = 0;
  double s_g = L.s_g_dev ? __longlong_as_double(*L.s_g_dev) : L.s_g;
  if (H.grad_clip >= 0.0) {  // iopt.py:90-101
    const i64 sq = *L.gsq;
    const double n_real = __dmul_rn(__dsqrt_rn(__ll2double_rn(sq)), s_g);
    if (n_real > H.grad_clip) s_g = __dmul_rn(s_g, __ddiv_rn(H.grad_clip, n_real));
  }
  S.s_m = bits_to_double(L.state[0]);
  S.sm4096 = __dmul_rn(S.s_m, 4096.0);
  S.sg4096 = __dmul_rn(s_g, 4096.0);
  S.com_m = shift_of(__ddiv_rn(S.sm4096, L.sw_min), S.flags);
  S.com_g = shift_of(__ddiv_rn(S.sg4096, L.sw_min), S.flags);
  S.com_mm = S.s_m > 0.0 ? shift_of(__ddiv_rn(__ddiv_rn(L.sw_max, 4096.0), S.s_m), S.flags) : 0;
  S.lr_sgb = __dmul_rn(H.lr, L.s_gb_dev ? __longlong_as_double(*L.s_gb_dev) : L.s_gb);
  S.com_b = L.b_acc ? shift_of(__ddiv_rn(S.lr_sgb, __dmul_rn(L.sx, L.sw_min)), S.flags) : 0;
  if (S.com_m > 62 || S.com_g > 62 || S.com_mm > 62 || S.com_b > 62) S.flags |= ECO_FLAG_SHIFT_OVERFLOW;
  return S;
}

// Row multiplier m_o >> (s_o - com) (ilayer.py:68 / iopt.py:53).
ECO_DEV i64 row_mult(double r, int com, unsigned& flags) {
  if (!(r >= 0.0) || r > 1.7e308) {
    flags |= ECO_FLAG_BAD_RATIO;
    return 0;
  }
  int m, s;
  qmult(r, m, s);
  if (s < com) {
    flags |= ECO_FLAG_BAD_RATIO;
    return 0;
  }
  const int d = s - com;
  return d >= 31 ? 0 : (i64)(m >> d);
}

// s_m <- max_o(rowmax_o * sw_o / 4096) / 127 (or 1.0), clear the accumulator (iopt.py:178-180).
ECO_DEV void finalize_state(i64* st) {
  const i64 acc = atomicExch(reinterpret_cast<unsigned long long*>(&st[1]), 0ull);
  const u64 fl = atomicAdd(reinterpret_cast<unsigned long long*>(&st[2]), 0ull);
  if (fl) return;  // flagged layer keeps its scale
  const double amax_real = __longlong_as_double(acc);
  st[0] = __double_as_longlong(amax_real > 0.0 ? __ddiv_rn(amax_real, 127.0) : 1.0);
}

struct RowCtx {
  i64 mult_m, mult_g, mult_mm;
  int com_m, com_g, com_mm;
  i64 half_m, half_g;
  i64 b_q, nb_q, lr_q, a_q;
  bool fast;  // every intermediate of this row fits int32 (see row_is_fast)
};

// Conservative magnitude bounds of the step's intermediates for |w|,|m|,|g| <= 128
// (double arithmetic, far from its 2^53 limit at the 2^30 threshold).  When they
// all stay below 2^30 (|eU| below 2^26) the int32 path with 64-bit products is
// exactly the reference's int64 arithmetic.
ECO_DEV bool row_is_fast(const RowCtx& c) {
  if (c.com_m < 0 || c.com_g < 0 || c.com_mm < 0) return false;
  const double lim = 1073741824.0;  // 2^30
  if (c.b_q > INT32_MAX || c.b_q < INT32_MIN || c.nb_q > INT32_MAX || c.nb_q < INT32_MIN || c.lr_q > INT32_MAX ||
      c.lr_q < INT32_MIN || c.a_q > INT32_MAX || c.a_q < INT32_MIN || c.com_mm > 62)
    return false;
  const double bm = (128.0 * (double)c.mult_m + (double)c.half_m) * ldexp(1.0, -c.com_m) + 1.0;
  const double bg = (128.0 * (double)c.mult_g + (double)c.half_g) * ldexp(1.0, -c.com_g) + 1.0;
  const double bt = (bm * fabs((double)c.b_q) + bg * fabs((double)c.nb_q)) / 65536.0 + 1.0;
  const double bth = 128.0 * 4096.0 + bt * fabs((double)c.lr_q) / 65536.0 + 1.0;
  const double be = bth + 128.0 * 4096.0;
  const double bn = bt + be * fabs((double)c.a_q) / 65536.0 + 1.0;
  return bm < lim && bg < lim && bt < lim && bth + 4096.0 < lim && bn < lim && be < 67108864.0;
}

// One element of iopt.py:154-176 in exact int64 (the reference's arithmetic, wrap-around included).
ECO_DEV void eco_elem(const RowCtx& c, int w, int m, int g, i64 nw, i64& m_new_out, int8_t& w8, i64& rmax,
                      u64& rsum) {
  const i64 mU = ams(m, c.mult_m, c.com_m, c.half_m);
  const i64 gU = ams(g, c.mult_g, c.com_g, c.half_g);
  const i64 m_t = sar64(add64(mul64(mU, c.b_q), mul64(gU, c.nb_q)), 16);
  const i64 thU = sub64((i64)w << 12, sar64(mul64(m_t, c.lr_q), 16));
  i64 wn = sar64(add64(thU, nw), 12);
  wn = wn < -127 ? -127 : (wn > 127 ? 127 : wn);
  const i64 eU = sub64(thU, wn << 12);
  const i64 m_new = add64(m_t, sar64(mul64(eU, c.a_q), 16));
  rmax = max(rmax, abs64(m_new));
  rsum += (u64)abs64(eU);
  w8 = (int8_t)wn;
  m_new_out = m_new;
}

// Row constants of the int32 path (all fit int32 when row_is_fast holds).
struct FastRow {
  int mult_m, mult_g, mult_mm, half_m, half_g, b_q, nb_q, lr_q, a_q;
  int com_m, com_g, com_mm;
};

// (int)(x >> s) for 0 <= s <= 63 when the result fits int32: one funnel or one shift.
ECO_DEV int shr_to_int(i64 x, int s) {
  const int lo = (int)(uint32_t)x, hi = (int)(x >> 32);
  return s < 32 ? (int)__funnelshift_r((uint32_t)lo, (uint32_t)hi, s) : (hi >> (s - 32));
}

// The same element in int32 with 32x32->64 products (only when row_is_fast).
ECO_DEV void eco_elem_fast(const FastRow& c, int w, int m, int g, int nw, int& m_new_out, int8_t& w8, int& rmax,
                           int& rsum) {
  const int mU = shr_to_int((i64)m * c.mult_m + c.half_m, c.com_m);
  const int gU = shr_to_int((i64)g * c.mult_g + c.half_g, c.com_g);
  const int m_t = shr_to_int((i64)mU * c.b_q + (i64)gU * c.nb_q, 16);
  const int thU = (w << 12) - shr_to_int((i64)m_t * c.lr_q, 16);
  int wn = (thU + nw) >> 12;
  wn = wn < -127 ? -127 : (wn > 127 ? 127 : wn);
  const int eU = thU - (wn << 12);
  const int m_new = m_t + shr_to_int((i64)eU * c.a_q, 16);
  rmax = max(rmax, abs(m_new));
  rsum += abs(eU);
  w8 = (int8_t)wn;
  m_new_out = m_new;
}

// (x >> s) as int32 (the result fits): the high word shifted when s >= 32 (HI),
// else one funnel shift.
template <bool HI>
ECO_DEV int shr_sel(i64 x, int s) {
  return HI ? (hi32(x) >> (s - 32)) : shr_fit(x, s);
}

// One row of the step on the 32-bit path (row_is_fast holds, momentum shift in
// 32..51): single-instruction 32x32->64 products, one shift per requant, bytes
// unpacked and packed with byte permutes, and the momentum rounding's tie-break
// draw taken only on its 2^-20 ties.  Each lane takes every 32nd 16-byte chunk,
// with the next chunk's loads in flight.  Returns the row's max |m_new|; adds the
// row's sum |e| to rsum.
template <bool HM, bool HG>
ECO_DEV int fast32_row(const RowCtx& c, const PhiloxKeys& keys, u64 seed, u64 stream, uint32_t row, int8_t* wr,
                       int8_t* mr, const int8_t* gr, int nch, int lane, u64& rsum) {
  const int mmu = (int)c.mult_m, mgu = (int)c.mult_g, mmm = (int)c.mult_mm;
  const i64 hm = c.half_m, hg = c.half_g;
  const int cm = c.com_m, cg = c.com_g, lo = c.com_mm - 20, shm = c.com_mm - 32, lo12 = lo - 12;
  const uint32_t p2lo = 1u << lo;
  const int bq = (int)c.b_q, nbq = (int)c.nb_q, lrq = (int)c.lr_q, aq = (int)c.a_q;
  int rmx = 0, rmn = 0;
  int j = lane;
  int4 wn4 = make_int4(0, 0, 0, 0), mn4 = wn4, gn4 = wn4;
  if (j < nch) {
    wn4 = *reinterpret_cast<const int4*>(wr + 16 * j);
    mn4 = *reinterpret_cast<const int4*>(mr + 16 * j);
    gn4 = *reinterpret_cast<const int4*>(gr + 16 * j);
  }
  for (; j < nch; j += 32) {
    const int4 wv = wn4, mv = mn4, gv = gn4;
    if (j + 32 < nch) {  // the next chunk's loads fly while this one computes
      wn4 = *reinterpret_cast<const int4*>(wr + 16 * (j + 32));
      mn4 = *reinterpret_cast<const int4*>(mr + 16 * (j + 32));
      gn4 = *reinterpret_cast<const int4*>(gr + 16 * (j + 32));
    }
    const uint32_t* ww = reinterpret_cast<const uint32_t*>(&wv);
    const uint32_t* mw = reinterpret_cast<const uint32_t*>(&mv);
    const uint32_t* gw = reinterpret_cast<const uint32_t*>(&gv);
    uint32_t wo[4], mo[4];
    unsigned rsum32 = 0u;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const Philox4 rnd = sr_quad_k(keys, stream, row, (uint32_t)(4 * j + q));
      int wq[4], mq[4], mn[4];
      uint32_t tf[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t f = quad_word(rnd, k);
        const int w = sbyte(ww[q], k), m = sbyte(mw[q], k), g = sbyte(gw[q], k);
        const int mU = shr_sel<HM>(mad_wide_s32(m, mmu, hm), cm);
        const int gU = shr_sel<HG>(mad_wide_s32(g, mgu, hg), cg);
        const int m_t = shr_fit(mad_wide_s32(gU, nbq, mul_wide_s32(mU, bq)), 16);
        const int thU = w * 4096 - shr_fit(mul_wide_s32(m_t, lrq), 16);
        const int wn = max(min((thU + (int)(f & 0xFFFu)) >> 12, 127), -127);
        const int eU = thU - wn * 4096;
        const int m_new = m_t + shr_fit(mul_wide_s32(eU, aq), 16);
        mn[k] = m_new;
        rsum32 = __sad(eU, 0, rsum32);
        const i64 p2 = mad_wide_u32(f >> 12, p2lo, mul_wide_s32(m_new, mmm));
        // the tie-break draw matters only when bits [lo, lo + 20) of p2 are all ones;
        // they are the top 20 bits of tf
        tf[k] = __funnelshift_r(lo32(p2), (uint32_t)hi32(p2), lo12);
        wq[k] = wn;
        mq[k] = hi32(p2) >> shm;
      }
      rmx = __vimax3_s32(rmx, __vimax3_s32(mn[0], mn[1], mn[2]), mn[3]);
      rmn = __vimin3_s32(rmn, __vimin3_s32(mn[0], mn[1], mn[2]), mn[3]);
      if (__vimax3_u32(__vimax3_u32(tf[0], tf[1], tf[2]), tf[3], 0u) >= 0xFFFFF000u) {
        // rare (2^-20 per element): the tied elements take the exact draw
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (tf[k] < 0xFFFFF000u) continue;
          const uint32_t f = quad_word(rnd, k);
          const i64 p2 = mad_wide_u32(f >> 12, p2lo, mul_wide_s32(mn[k], mmm));
          mq[k] = (int)max((i64)-128, min((i64)127, step_m_round_tie(p2, c.com_mm, seed, stream, row,
                                                                    (uint32_t)(16 * j + 4 * q + k))));
        }
      }
      wo[q] = pack4_sat(wq[0], wq[1], wq[2], wq[3]);
      mo[q] = pack4_sat127(mq[0], mq[1], mq[2], mq[3]);
    }
    rsum += (u64)(unsigned)rsum32;
    *reinterpret_cast<int4*>(wr + 16 * j) = make_int4(wo[0], wo[1], wo[2], wo[3]);
    *reinterpret_cast<int4*>(mr + 16 * j) = make_int4(mo[0], mo[1], mo[2], mo[3]);
  }
  return max(rmx, -rmn);
}

ECO_DEV i64 replay(const void* p, int bits, i64 idx) {
  return bits == 32 ? (i64)static_cast<const int32_t*>(p)[idx] : static_cast<const i64*>(p)[idx];
}

// Momentum requant of one element: sat8(SR(m_new * mult_mm, com_mm)) with the site's draw.
ECO_DEV int8_t m_requant(const RowCtx& c, i64 m_new, bool philox, uint32_t field, i64 nm_replay, u64 seed,
                         u64 stream, uint32_t row, uint32_t col) {
  const i64 prod = mul64(m_new, c.mult_mm);
  if (c.com_mm < 0) return sat8(shl64(prod, -c.com_mm));
  if (philox) return sat8(step_m_round(prod, c.com_mm, field, seed, stream, row, col));
  return sat8(sar64(add64(prod, nm_replay), c.com_mm));
}

// The step's hyper-parameters and round keys as the launch sees them: the launch's
// copy or, when it names one, the device copy of the moment (a CUDA graph replay).
// Staged in shared memory by the block's first thread.
struct StepShared {
  eco_i8eco_hyper_t H;
  PhiloxKeys keys;
};
ECO_DEV void stage_hyper(const StepParams& P, StepShared& sh) {
  if (threadIdx.x == 0) {
    sh.H = P.H;
    if (P.H.dev) {
      const eco_i8eco_hyper_t& D = *P.H.dev;
      sh.H.lr = D.lr;
      sh.H.grad_clip = D.grad_clip;
      sh.H.b_q = D.b_q;
      sh.H.nb_q = D.nb_q;
      sh.H.lr_q = D.lr_q;
      sh.H.a_q = D.a_q;
      sh.H.seed = D.seed;
      sh.keys = philox_keys(D.seed);
    } else {
      sh.keys = P.keys;
    }
  }
  __syncthreads();
}

// Bias integer SGD of one row (iopt.py:187-197); r indexes the layer's arrays
// (global row r + row_base).
template <bool PHILOX>
ECO_DEV void bias_update(const eco_i8eco_layer_t& L, const eco_i8eco_hyper_t& H, const LayerScalars& S, i64 r,
                         double sw_o, unsigned& flags) {
  const i64 mb = row_mult(__ddiv_rn(S.lr_sgb, __dmul_rn(L.sx, sw_o)), S.com_b, flags);
  i64 nb = 0;
  if (S.com_b >= 0) {
    nb = PHILOX ? low_bits(sr_word(H.seed, L.stream_b, (uint32_t)(L.row_base + r), 0u), S.com_b)
                : replay(L.nudge_b, L.nudge_b_bits, r);
  }
  const int delta = (int)ams(L.gb_sum[r], mb, S.com_b, nb);
  L.b_acc[r] = (int)((unsigned)L.b_acc[r] - (unsigned)delta);
}

// The bias step of every global row [0, bias_rows) of the layers that ask for it
// (a data-parallel row shard), one thread per row; runs before the step kernel,
// which skips their biases.  A layer whose scalars are flagged is left alone
// (the step kernel records the flags).
template <bool PHILOX>
__global__ void i8eco_bias_kernel(const __grid_constant__ StepParams P) {
  __shared__ StepShared sh;
  stage_hyper(P, sh);
  const eco_i8eco_layer_t& L = P.layers[blockIdx.y].L;
  const i64 R = (i64)blockIdx.x * blockDim.x + threadIdx.x;
  if (!L.b_acc || R >= L.bias_rows) return;
  const LayerScalars S = layer_scalars(L, sh.H);
  if (S.flags) return;
  const i64 r = R - L.row_base;
  unsigned flags = 0;
  bias_update<PHILOX>(L, sh.H, S, r, L.sw[r], flags);
  if (flags) atomicOr(reinterpret_cast<unsigned long long*>(&L.state[2]), (u64)flags);
}

template <bool PHILOX>
__global__ void __launch_bounds__(kThreads, kBlocksPerSM) i8eco_step_kernel(const __grid_constant__ StepParams P) {
  __shared__ double s_wmax[kWarps];
  __shared__ int s_last;
  __shared__ StepShared sh;
  stage_hyper(P, sh);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const eco_i8eco_hyper_t& H = sh.H;
  for (i64 t = blockIdx.x; t < P.total_tiles; t += gridDim.x) {
    int li = 0;
    while (li + 1 < P.n_layers && P.layers[li + 1].tile_begin <= t) ++li;
    const LayerDesc& D = P.layers[li];
    const eco_i8eco_layer_t& L = D.L;
    const LayerScalars S = layer_scalars(L, H);
    if (S.flags) {  // the reference raises here: leave the layer untouched, flag it
      if (threadIdx.x == 0) atomicOr(reinterpret_cast<unsigned long long*>(&L.state[2]), (u64)S.flags);
      continue;
    }
    const i64 r0 = (t - D.tile_begin) * D.rows_per_tile;
    const i64 r1 = min((i64)L.rows, r0 + (i64)D.rows_per_tile);
    double wmax = 0.0;
    unsigned flags = 0;
    for (i64 r = r0 + warp; r < r1; r += kWarps) {
      const double sw_o = L.sw[r];
      RowCtx c;
      c.com_m = S.com_m;
      c.com_g = S.com_g;
      c.com_mm = S.com_mm;
      c.half_m = half_nudge(S.com_m);
      c.half_g = half_nudge(S.com_g);
      c.b_q = H.b_q;
      c.nb_q = H.nb_q;
      c.lr_q = H.lr_q;
      c.a_q = H.a_q;
      c.mult_m = row_mult(__ddiv_rn(S.sm4096, sw_o), S.com_m, flags);
      c.mult_g = row_mult(__ddiv_rn(S.sg4096, sw_o), S.com_g, flags);
      c.mult_mm = S.s_m > 0.0 ? row_mult(__ddiv_rn(__ddiv_rn(sw_o, 4096.0), S.s_m), S.com_mm, flags) : 0;
      c.fast = PHILOX && D.vec && row_is_fast(c);
      const uint32_t row = (uint32_t)(L.row_base + r);  // global row: shards draw what the whole layer would
      i64 rmax = INT64_MIN;
      u64 rsum = 0;
      int8_t* wr = L.w + r * L.cols;
      int8_t* mr = L.m + r * L.cols;
      const int8_t* gr = L.g + r * L.cols;
      const bool fast32 = c.fast && c.com_mm >= 32 && c.com_mm <= 51;
      if (fast32) {
        const bool hm = c.com_m >= 32, hg = c.com_g >= 32;
        int rmx;
        if (!hm && !hg)
          rmx = fast32_row<false, false>(c, sh.keys, H.seed, L.stream_w, row, wr, mr, gr, (int)(L.cols / 16), lane, rsum);
        else if (hm && !hg)
          rmx = fast32_row<true, false>(c, sh.keys, H.seed, L.stream_w, row, wr, mr, gr, (int)(L.cols / 16), lane, rsum);
        else if (!hm && hg)
          rmx = fast32_row<false, true>(c, sh.keys, H.seed, L.stream_w, row, wr, mr, gr, (int)(L.cols / 16), lane, rsum);
        else
          rmx = fast32_row<true, true>(c, sh.keys, H.seed, L.stream_w, row, wr, mr, gr, (int)(L.cols / 16), lane, rsum);
        rmax = rmx;
      } else if (c.fast) {
        FastRow fr;
        fr.mult_m = (int)c.mult_m; fr.mult_g = (int)c.mult_g; fr.mult_mm = (int)c.mult_mm;
        fr.half_m = (int)c.half_m; fr.half_g = (int)c.half_g;
        fr.b_q = (int)c.b_q; fr.nb_q = (int)c.nb_q; fr.lr_q = (int)c.lr_q; fr.a_q = (int)c.a_q;
        fr.com_m = c.com_m; fr.com_g = c.com_g; fr.com_mm = c.com_mm;
        int rmax32 = 0;
        for (i64 j = lane; j < L.cols / 16; j += 32) {
          const i64 c0 = j * 16;
          int4 wv = *reinterpret_cast<const int4*>(wr + c0);
          int4 mv = *reinterpret_cast<const int4*>(mr + c0);
          const int4 gv = *reinterpret_cast<const int4*>(gr + c0);
          int8_t* wb = reinterpret_cast<int8_t*>(&wv);
          int8_t* mb = reinterpret_cast<int8_t*>(&mv);
          const int8_t* gb = reinterpret_cast<const int8_t*>(&gv);
          int rsum32 = 0;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const Philox4 rnd = sr_quad_k(sh.keys, L.stream_w, row, (uint32_t)((c0 >> 2) + q));
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int e = 4 * q + k;
              const uint32_t f = quad_word(rnd, k);
              int m_new;
              int8_t w8;
              eco_elem_fast(fr, wb[e], mb[e], gb[e], (int)(f & 0xFFFu), m_new, w8, rmax32, rsum32);
              wb[e] = w8;
              mb[e] = sat8(step_m_round((i64)m_new * fr.mult_mm, fr.com_mm, f, H.seed, L.stream_w, row,
                                        (uint32_t)(c0 + e)));
            }
          }
          rsum += (u64)(unsigned)rsum32;
          *reinterpret_cast<int4*>(wr + c0) = wv;
          *reinterpret_cast<int4*>(mr + c0) = mv;
        }
        rmax = rmax32;
      } else {
        // exact int64 path: any shape, any alignment, replay mode, wide intermediates
        for (i64 c0 = 4 * lane; c0 < L.cols; c0 += 128) {
          Philox4 rnd{0u, 0u, 0u, 0u};
          if (PHILOX) rnd = sr_quad_k(sh.keys, L.stream_w, row, (uint32_t)(c0 >> 2));
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const i64 col = c0 + k;
            if (col >= L.cols) break;
            const i64 idx = r * L.cols + col;
            const uint32_t f = quad_word(rnd, k);
            const i64 nw = PHILOX ? (i64)(f & 0xFFFu) : replay(L.nudge_w, 32, idx);
            const i64 nm = (!PHILOX && S.com_mm >= 0) ? replay(L.nudge_m, L.nudge_m_bits, idx) : 0;
            i64 m_new;
            int8_t w8;
            eco_elem(c, wr[col], mr[col], gr[col], nw, m_new, w8, rmax, rsum);
            wr[col] = w8;
            mr[col] = m_requant(c, m_new, PHILOX, f, nm, H.seed, L.stream_w, row, (uint32_t)col);
          }
        }
      }
      // row reductions (torch: abs().amax(1), abs().sum(1) on int64)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        rmax = max(rmax, (i64)__shfl_xor_sync(0xffffffffu, rmax, o));
        rsum += __shfl_xor_sync(0xffffffffu, rsum, o);
      }
      if (lane == 0) {
        if (L.rowsum) L.rowsum[r] = (i64)rsum;
        // r * sw_o / 4096 (iopt.py:178); a negative row max can only come from INT64_MIN
        const double v = __ddiv_rn(__dmul_rn(__ll2double_rn(rmax), sw_o), 4096.0);
        wmax = fmax(wmax, v);
        if (L.b_acc && L.bias_rows == 0) bias_update<PHILOX>(L, H, S, r, sw_o, flags);
      }
    }
    if (flags && lane == 0) atomicOr(reinterpret_cast<unsigned long long*>(&L.state[2]), (u64)flags);
    if (lane == 0) s_wmax[warp] = wmax;
    __syncthreads();
    if (threadIdx.x == 0) {
      double v = 0.0;
      for (int w = 0; w < kWarps; ++w) v = fmax(v, s_wmax[w]);
      if (v > 0.0)
        atomicMax(reinterpret_cast<unsigned long long*>(&L.state[1]), (u64)__double_as_longlong(v));
    }
    __syncthreads();
  }
  // the last CTA to finish publishes the new momentum scales (iopt.py:178-180)
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(H.done_counter, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (H.finalize) {
    for (int li = threadIdx.x; li < P.n_layers; li += blockDim.x)
      finalize_state(reinterpret_cast<i64*>(P.layers[li].L.state));
  }
  if (threadIdx.x == 0) *H.done_counter = 0u;
}

__global__ void i8eco_finalize_kernel(i64* state, int n_layers) {
  for (int li = blockIdx.x * blockDim.x + threadIdx.x; li < n_layers; li += gridDim.x * blockDim.x)
    finalize_state(state + 4 * li);
}

}  // namespace

extern "C" int eco_i8eco_step(const eco_i8eco_layer_t* layers, int n_layers, const eco_i8eco_hyper_t* hyper,
                              eco_stream_t stream) {
  ECO_REQUIRE(layers && hyper && n_layers >= 0, ECO_ERR_ARG, "eco_i8eco_step: bad arguments");
  ECO_REQUIRE(hyper->done_counter, ECO_ERR_ARG, "eco_i8eco_step: done_counter is required");
  ECO_REQUIRE(hyper->sr_mode == ECO_SR_PHILOX || hyper->sr_mode == ECO_SR_REPLAY32 ||
                  hyper->sr_mode == ECO_SR_REPLAY64,
              ECO_ERR_ARG, "eco_i8eco_step: sr_mode must be Philox or replay");
  const bool replay = hyper->sr_mode != ECO_SR_PHILOX;
  for (int i = 0; i < n_layers; ++i) {
    const eco_i8eco_layer_t& L = layers[i];
    ECO_REQUIRE(L.w && L.m && L.g && L.sw && L.state && L.rows > 0 && L.cols > 0, ECO_ERR_ARG,
                "eco_i8eco_step: layer %d: null tensor or empty shape", i);
    ECO_REQUIRE(L.rows < (1ll << 31) && L.cols < (1ll << 31), ECO_ERR_ARG, "eco_i8eco_step: layer %d too large", i);
    ECO_REQUIRE(hyper->grad_clip < 0.0 || L.gsq, ECO_ERR_ARG, "eco_i8eco_step: layer %d: clipping needs gsq", i);
    ECO_REQUIRE(!L.b_acc || L.gb_sum, ECO_ERR_ARG, "eco_i8eco_step: layer %d: bias needs gb_sum", i);
    ECO_REQUIRE(!replay || (L.nudge_w && L.nudge_m && (!L.b_acc || L.nudge_b)), ECO_ERR_ARG,
                "eco_i8eco_step: layer %d: replay mode needs nudge tensors", i);
    ECO_REQUIRE(L.bias_rows == 0 || (L.bias_rows > 0 && L.bias_rows < (1ll << 31) && L.row_base >= 0 &&
                                      L.row_base + L.rows <= L.bias_rows),
                ECO_ERR_ARG, "eco_i8eco_step: layer %d: bias_rows must cover the stepped rows", i);
    ECO_REQUIRE(!replay || ((L.nudge_m_bits == 32 || L.nudge_m_bits == 64) &&
                            (!L.b_acc || L.nudge_b_bits == 32 || L.nudge_b_bits == 64)),
                ECO_ERR_ARG, "eco_i8eco_step: layer %d: nudge widths", i);
  }
  cudaStream_t s = eco_stream(stream);
  static_assert(sizeof(StepParams) < 30000, "kernel parameter space");
  for (int base = 0; base < n_layers; base += kMaxLayers) {
    StepParams P;
    P.H = *hyper;
    P.keys = philox_keys(hyper->seed);
    P.n_layers = std::min(kMaxLayers, n_layers - base);
    i64 tiles = 0;
    for (int i = 0; i < P.n_layers; ++i) {
      LayerDesc& D = P.layers[i];
      D.L = layers[base + i];
      const i64 target = std::max<i64>(kWarps, (64 * 1024) / D.L.cols);
      D.rows_per_tile = (int)std::min<i64>(D.L.rows, (target + kWarps - 1) / kWarps * kWarps);
      D.tile_begin = tiles;
      D.vec = (D.L.cols % 16 == 0) && eco_aligned16(D.L.w) && eco_aligned16(D.L.m) && eco_aligned16(D.L.g);
      tiles += (D.L.rows + D.rows_per_tile - 1) / D.rows_per_tile;
    }
    P.total_tiles = tiles;
    i64 bias_rows = 0;
    for (int i = 0; i < P.n_layers; ++i)
      if (P.layers[i].L.b_acc) bias_rows = std::max<i64>(bias_rows, P.layers[i].L.bias_rows);
    if (bias_rows > 0) {  // every bias of the data-parallel shards, before their weights
      const dim3 bgrid((unsigned)((bias_rows + 255) / 256), (unsigned)P.n_layers);
      if (replay)
        i8eco_bias_kernel<false><<<bgrid, 256, 0, s>>>(P);
      else
        i8eco_bias_kernel<true><<<bgrid, 256, 0, s>>>(P);
      if (int rc = eco_launch_check("eco_i8eco_step (bias)")) return rc;
    }
    int occ = 0;
    if (replay)
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, i8eco_step_kernel<false>, kThreads, 0);
    else
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, i8eco_step_kernel<true>, kThreads, 0);
    const i64 grid = std::max<i64>(1, std::min<i64>(tiles, (i64)eco_num_sms() * std::max(occ, 1)));
    if (replay)
      i8eco_step_kernel<false><<<(unsigned)grid, kThreads, 0, s>>>(P);
    else
      i8eco_step_kernel<true><<<(unsigned)grid, kThreads, 0, s>>>(P);
    if (int rc = eco_launch_check("eco_i8eco_step")) return rc;
  }
  return ECO_OK;
}

extern "C" int eco_i8eco_finalize(int64_t* state, int n_layers, eco_stream_t stream) {
  ECO_REQUIRE(state && n_layers >= 0, ECO_ERR_ARG, "eco_i8eco_finalize: bad arguments");
  if (n_layers == 0) return ECO_OK;
  i8eco_finalize_kernel<<<(n_layers + 127) / 128, 128, 0, eco_stream(stream)>>>(reinterpret_cast<i64*>(state),
                                                                               n_layers);
  return eco_launch_check("eco_i8eco_finalize");
}
