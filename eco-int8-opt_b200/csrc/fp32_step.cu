// The fp32-state ECO optimizers (ecoint8/eco.py:50-235: EcoSGDM, EcoAdam) as two
// multi-layer launches with no host synchronisation.
//
// Layout: per layer, int8 weights w [rows, cols], fp32 gradient g, fp32 moments m (and
// v for Adam) of the same shape, the layer's fp32 row scales s_w [rows] (for w_fp32())
// and the optimizer's frozen grid s_fixed [rows].  A launch walks "tiles" of kTile
// consecutive elements of one layer (tiles never straddle layers).
//
//   eco_fp32_gstats: per tile, sum g^2 in double and the count of non-finite g
//                    (eco.py:39-47 skips a layer with any; :97-100 clips by the norm),
//                    into the caller's scratch (one slot per tile, fixed order);
//   eco_fp32_step:   per tile, the layer's norm from its tiles' slots (summed in tile
//                    order, so every CTA sees the same bits), then one pass over the
//                    elements: read g, w, m (v), write w, m (v); per tile sum |e| in
//                    double into a second scratch slot for the statistics.
//
// Arithmetic: each fp32 operation of the reference's PyTorch expressions is one IEEE
// operation here, in the reference's order, with the semantics of PyTorch's CUDA kernels
// for those operations: a tensor times / plus a Python scalar rounds the scalar to fp32
// first; `a.add_(b, alpha=c)` is fma(c, b, a); a tensor divided by a Python scalar is a
// multiply by the scalar's reciprocal taken in double and rounded to fp32 (so
// v / (1 - 0.999) is v * 1000.0f, not v * 999.99994f); `scalar / tensor` is the tensor's reciprocal times
// the scalar; addcmul is a + (c * b) * b'.  The norm is sqrt of the double sum of
// squares, rounded to fp32 (PyTorch's fp32 reduction can differ from it in the last
// bit, which changes the clip factor only when clipping is active).
// Stochastic rounding u ~ U[0, 1): the library's Philox field of the element (24 bits),
// or an fp32 tensor of uniforms (a torch.rand_like draw, quant.py:25).
#include <algorithm>

#include "abi.cuh"
#include "common.cuh"

namespace {

constexpr int kThreads = 256;
constexpr i64 kTile = 64 * 1024;  // elements per tile
constexpr int kMaxLayers = 64;    // per launch (kernel parameter space)

struct TileMap {
  int n_layers;
  i64 total_tiles;
  i64 tile_begin[kMaxLayers + 1];
};

struct Fp32Params {
  eco_fp32_hyper_t H;
  PhiloxKeys keys;
  TileMap T;
  eco_fp32_layer_t L[kMaxLayers];
  double* gstats;  // [total_tiles][2]: sum g^2, non-finite count
  double* esum;    // [total_tiles]: sum |e|
  unsigned char vec[kMaxLayers];  // the layer takes 16-byte loads (cols % 4 == 0, aligned rows)
  // fp32 constants of the reference's expressions (host-rounded like PyTorch's scalars)
  float b_f, omb_f, lr_f, alpha_f, wd_f, eps_f, inv_bc1, inv_bc2, bc1_f, b2_f, omb2_f, adam_eps_f, cinj_f;
};

ECO_DEV int layer_of(const TileMap& T, i64 t) {
  int l = 0;
  while (l + 1 < T.n_layers && T.tile_begin[l + 1] <= t) ++l;
  return l;
}

template <typename T>
ECO_DEV T block_sum(T v, T* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  T s = 0;
  if (threadIdx.x == 0)
    for (int w = 0; w < kThreads / 32; ++w) s += sh[w];  // fixed order
  return s;  // valid in thread 0
}

__global__ void __launch_bounds__(kThreads) gstats_kernel(const __grid_constant__ Fp32Params P) {
  __shared__ double sh_s[kThreads / 32];
  __shared__ double sh_n[kThreads / 32];
  for (i64 t = blockIdx.x; t < P.T.total_tiles; t += gridDim.x) {
    const int l = layer_of(P.T, t);
    const eco_fp32_layer_t& L = P.L[l];
    const i64 n = L.rows * L.cols;
    const i64 e0 = (t - P.T.tile_begin[l]) * kTile, e1 = min(n, e0 + kTile);
    double s = 0.0, nf = 0.0;
    for (i64 i = e0 + threadIdx.x; i < e1; i += kThreads) {
      const float g = L.g[i];
      if (isfinite(g))
        s = __dadd_rn(s, __dmul_rn((double)g, (double)g));  // exact square, double sum
      else
        nf += 1.0;
    }
    const double S = block_sum(s, sh_s);
    const double N = block_sum(nf, sh_n);
    if (threadIdx.x == 0) {
      P.gstats[2 * t] = S;
      P.gstats[2 * t + 1] = N;
    }
  }
}

// The layer's gradient scale factor (1 when not clipping) and whether it is stepped.
ECO_DEV bool layer_clip(const Fp32Params& P, int l, float& factor, float* norm_out) {
  double S = 0.0, N = 0.0;
  for (i64 t = P.T.tile_begin[l]; t < P.T.tile_begin[l + 1]; ++t) {
    S = __dadd_rn(S, P.gstats[2 * t]);
    N += P.gstats[2 * t + 1];
  }
  const float n = __double2float_rn(__dsqrt_rn(S));  // g.norm() (fp32)
  if (norm_out) *norm_out = n;
  factor = 1.0f;
  if (P.H.grad_clip >= 0.0 && (double)n > P.H.grad_clip)  // eco.py:97-100 (Python double arithmetic)
    factor = __double2float_rn(__ddiv_rn(P.H.grad_clip, __dadd_rn((double)n, 1e-8)));
  return N == 0.0;
}

// One element of EcoSGDM.step / EcoAdam.step (eco.py:107-128, 196-226) in the reference's
// PyTorch fp32 operations: returns the new weight (as a float in [-127, 127]), momentum,
// second moment (Adam) and the error e.
template <bool ADAM>
ECO_DEV void step_elem(const Fp32Params& P, float w8, float m, float v_in, float g, float u, float sw, float s,
                       bool clip, float factor, float& q, float& m_n, float& v_n, float& e) {
  if (clip) g = __fmul_rn(g, factor);                         // g.mul_(clip / (n + EPS))
  const float wf = __fmul_rn(w8, sw);                         // layer.w_fp32()
  if (P.H.weight_decay != 0.0) g = __fmaf_rn(P.wd_f, wf, g);  // g.add_(w_fp32, alpha=wd)
  float th, m_t, eta = 0.0f;
  v_n = 0.0f;
  if (!ADAM) {
    m_t = __fadd_rn(__fmul_rn(m, P.b_f), __fmul_rn(g, P.omb_f));  // m * b + g * (1 - b)
    th = __fsub_rn(wf, __fmul_rn(P.lr_f, m_t));                   // w_fp32 - lr * m_tilde
  } else {
    m_t = __fmaf_rn(P.omb_f, g, __fmul_rn(m, P.b_f));                        // m.mul_(b1).add_(g, alpha=1-b1)
    v_n = __fmaf_rn(P.omb2_f, __fmul_rn(g, g), __fmul_rn(v_in, P.b2_f));    // v.mul_(b2).addcmul_(g, g, 1-b2)
    const float v_hat = __fadd_rn(__fsqrt_rn(__fmul_rn(v_n, P.inv_bc2)), P.adam_eps_f);
    eta = __fmul_rn(__frcp_rn(__fmul_rn(P.bc1_f, v_hat)), P.lr_f);          // lr / (bc1 * v_hat)
    th = __fsub_rn(wf, __fmul_rn(eta, __fmul_rn(m_t, P.inv_bc1)));         // w_fp32 - eta * (m / bc1)
  }
  const float x = __fdiv_rn(th, __fadd_rn(s, P.eps_f));    // quantize_symmetric: x / (s + EPS)
  q = fminf(fmaxf(floorf(__fadd_rn(x, u)), -127.0f), 127.0f);
  e = __fsub_rn(th, __fmul_rn(q, s));                      // th - w_new.float() * s_fixed
  if (!ADAM)
    m_n = __fadd_rn(m_t, __fmul_rn(P.alpha_f, e));  // m_tilde + alpha * e
  else
    m_n = __fadd_rn(m_t, __fmul_rn(e, __fmul_rn(__frcp_rn(eta), P.cinj_f)));  // m + e * (c / eta)
}

template <bool ADAM>
__global__ void __launch_bounds__(kThreads) fp32_step_kernel(const __grid_constant__ Fp32Params P) {
  __shared__ double sh_e[kThreads / 32];
  __shared__ float s_factor;
  __shared__ int s_ok;
  for (i64 t = blockIdx.x; t < P.T.total_tiles; t += gridDim.x) {
    const int l = layer_of(P.T, t);
    const eco_fp32_layer_t& L = P.L[l];
    __syncthreads();
    if (threadIdx.x == 0) {
      float f;
      s_ok = layer_clip(P, l, f, (t == P.T.tile_begin[l] && L.norm_out) ? L.norm_out : nullptr);
      s_factor = f;
      if (t == P.T.tile_begin[l] && L.stepped_out) *L.stepped_out = s_ok;
    }
    __syncthreads();
    if (!s_ok) {  // a non-finite gradient: the layer is left as it is (eco.py:44-46)
      if (threadIdx.x == 0) P.esum[t] = 0.0;
      continue;
    }
    const float factor = s_factor;
    const bool clip = P.H.grad_clip >= 0.0 && factor != 1.0f;
    const i64 n = L.rows * L.cols;
    const i64 e0 = (t - P.T.tile_begin[l]) * kTile, e1 = min(n, e0 + kTile);
    const bool philox = P.H.sr_mode == ECO_SR_PHILOX;
    double esum = 0.0;
    if (P.vec[l]) {
      // whole quads in one row: one 4-byte load of w, 16-byte loads of m, g (and v, u),
      // the row's scales once, the same operations per element in the same order
      const uint32_t cols = (uint32_t)L.cols;
      for (i64 q0 = e0 + 4 * (i64)threadIdx.x; q0 < e1; q0 += 4 * kThreads) {
        const uint32_t r = (uint32_t)q0 / cols;
        const uint32_t c0 = (uint32_t)q0 - r * cols;
        Philox4 rnd{0u, 0u, 0u, 0u};
        float4 u4 = make_float4(0.f, 0.f, 0.f, 0.f);
        if (philox)
          rnd = sr_quad_k(P.keys, L.stream, r, c0 >> 2);
        else
          u4 = *reinterpret_cast<const float4*>(L.u + q0);
        const uint32_t w4 = *reinterpret_cast<const uint32_t*>(L.w + q0);
        const float4 m4 = *reinterpret_cast<const float4*>(L.m + q0);
        const float4 g4 = *reinterpret_cast<const float4*>(L.g + q0);
        float4 v4 = make_float4(0.f, 0.f, 0.f, 0.f);
        if (ADAM) v4 = *reinterpret_cast<const float4*>(L.v + q0);
        const float sw = L.sw[r], sf = L.s_fixed[r];
        const float mi[4] = {m4.x, m4.y, m4.z, m4.w}, gi[4] = {g4.x, g4.y, g4.z, g4.w};
        const float vi[4] = {v4.x, v4.y, v4.z, v4.w}, ui[4] = {u4.x, u4.y, u4.z, u4.w};
        int qo[4];
        float mo[4], vo[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float u = philox ? __fmul_rn((float)(quad_word(rnd, k) >> 8), 0x1p-24f) : ui[k];
          float q, e;
          step_elem<ADAM>(P, (float)sbyte(w4, k), mi[k], vi[k], gi[k], u, sw, sf, clip, factor, q, mo[k], vo[k], e);
          qo[k] = (int)q;
          esum += (double)fabsf(e);
        }
        *reinterpret_cast<uint32_t*>(L.w + q0) = pack4(qo[0], qo[1], qo[2], qo[3]);
        *reinterpret_cast<float4*>(L.m + q0) = make_float4(mo[0], mo[1], mo[2], mo[3]);
        if (ADAM) *reinterpret_cast<float4*>(L.v + q0) = make_float4(vo[0], vo[1], vo[2], vo[3]);
      }
    } else {
      for (i64 q0 = e0 + 4 * (i64)threadIdx.x; q0 < e1; q0 += 4 * kThreads) {
        const i64 r = q0 / L.cols;
        const i64 c0 = q0 - r * L.cols;
        // four consecutive elements; a quad may cross a row end when cols % 4 != 0
        Philox4 rnd{0u, 0u, 0u, 0u};
        const bool one_row = c0 + 4 <= L.cols;
        if (philox && one_row && (c0 & 3) == 0) rnd = sr_quad_k(P.keys, L.stream, (uint32_t)r, (uint32_t)(c0 >> 2));
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const i64 i = q0 + k;
          if (i >= e1) break;
          const i64 row = one_row ? r : i / L.cols;
          const i64 col = i - row * L.cols;
          float u;
          if (philox) {
            const uint32_t f = (one_row && (c0 & 3) == 0) ? quad_word(rnd, k)
                                                            : sr_field(P.H.seed, L.stream, (uint32_t)row, (uint32_t)col);
            u = __fmul_rn((float)(f >> 8), 0x1p-24f);
          } else {
            u = L.u[i];
          }
          float q, m_n, v_n, e;
          step_elem<ADAM>(P, (float)L.w[i], L.m[i], ADAM ? L.v[i] : 0.0f, L.g[i], u, L.sw[row], L.s_fixed[row], clip,
                          factor, q, m_n, v_n, e);
          L.w[i] = (int8_t)q;
          L.m[i] = m_n;
          if (ADAM) L.v[i] = v_n;
          esum += (double)fabsf(e);
        }
      }
    }
    const double E = block_sum(esum, sh_e);
    if (threadIdx.x == 0) P.esum[t] = E;
  }
}

}  // namespace

extern "C" int eco_fp32_eco_step(const eco_fp32_layer_t* layers, int n_layers, const eco_fp32_hyper_t* hyper,
                                 double* scratch, int64_t scratch_len, eco_stream_t stream) {
  ECO_REQUIRE(layers && hyper && scratch && n_layers >= 1 && n_layers <= kMaxLayers, ECO_ERR_ARG,
              "eco_fp32_eco_step: bad arguments (1..%d layers)", kMaxLayers);
  ECO_REQUIRE(hyper->kind == 0 || hyper->kind == 1, ECO_ERR_ARG, "eco_fp32_eco_step: kind 0 (SGDM) or 1 (Adam)");
  ECO_REQUIRE(hyper->sr_mode == ECO_SR_PHILOX || hyper->sr_mode == ECO_SR_REPLAY_F32, ECO_ERR_ARG,
              "eco_fp32_eco_step: sr_mode must be Philox or fp32 replay");
  static_assert(sizeof(Fp32Params) < 30000, "kernel parameter space");
  Fp32Params P;
  P.H = *hyper;
  P.keys = philox_keys(hyper->seed);
  P.T.n_layers = n_layers;
  i64 tiles = 0;
  for (int l = 0; l < n_layers; ++l) {
    const eco_fp32_layer_t& L = layers[l];
    ECO_REQUIRE(L.w && L.m && L.g && L.sw && L.s_fixed && L.rows > 0 && L.cols > 0, ECO_ERR_ARG,
                "eco_fp32_eco_step: layer %d: null tensor or empty shape", l);
    ECO_REQUIRE(L.rows < (1ll << 31) && L.cols < (1ll << 31), ECO_ERR_ARG, "eco_fp32_eco_step: layer %d too large",
                l);
    ECO_REQUIRE(hyper->kind == 0 || L.v, ECO_ERR_ARG, "eco_fp32_eco_step: layer %d: Adam needs v", l);
    ECO_REQUIRE(hyper->sr_mode != ECO_SR_REPLAY_F32 || L.u, ECO_ERR_ARG,
                "eco_fp32_eco_step: layer %d: replay needs uniforms", l);
    P.L[l] = L;
    P.T.tile_begin[l] = tiles;
    tiles += (L.rows * L.cols + kTile - 1) / kTile;
  }
  P.T.tile_begin[n_layers] = tiles;
  P.T.total_tiles = tiles;
  ECO_REQUIRE(scratch_len >= 3 * tiles, ECO_ERR_ARG, "eco_fp32_eco_step: scratch needs %lld doubles",
              (long long)(3 * tiles));
  for (int l = 0; l < n_layers; ++l) {  // 16-byte loads need whole quads on aligned rows
    const eco_fp32_layer_t& L = P.L[l];
    const bool w_al = (reinterpret_cast<uintptr_t>(L.w) & 3) == 0;
    P.vec[l] = (unsigned char)(L.cols % 4 == 0 && L.rows * L.cols < (1ll << 32) && w_al &&
                               eco_aligned16(L.m) && eco_aligned16(L.g) && (hyper->kind == 0 || eco_aligned16(L.v)) &&
                               (hyper->sr_mode == ECO_SR_PHILOX || eco_aligned16(L.u)));
  }
  P.gstats = scratch;
  P.esum = scratch + 2 * tiles;
  const eco_fp32_hyper_t& H = *hyper;
  // PyTorch turns a Python scalar operand into the op's dtype (fp32), and divides by one
  // as a multiply by its reciprocal, computed in double and rounded to fp32
  P.b_f = (float)H.beta1;
  P.omb_f = (float)(1.0 - H.beta1);
  P.lr_f = (float)H.lr;
  P.alpha_f = (float)((1.0 / H.lr) * (1.0 - 1.0 / H.beta1));  // eco.py:89
  P.wd_f = (float)H.weight_decay;
  P.eps_f = (float)1e-8;  // quant.py:7 EPS
  P.b2_f = (float)H.beta2;
  P.omb2_f = (float)(1.0 - H.beta2);
  P.adam_eps_f = (float)H.eps;
  P.bc1_f = (float)H.bc1;
  P.inv_bc1 = (float)(1.0 / H.bc1);
  P.inv_bc2 = (float)(1.0 / H.bc2);
  P.cinj_f = (float)(1.0 - 1.0 / H.beta1);  // eco.py:223
  cudaStream_t s = eco_stream(stream);
  const unsigned grid = (unsigned)std::max<i64>(1, std::min<i64>(tiles, (i64)eco_num_sms() * 8));
  gstats_kernel<<<grid, kThreads, 0, s>>>(P);
  if (int rc = eco_launch_check("eco_fp32_eco_step (norm)")) return rc;
  if (H.kind == 0)
    fp32_step_kernel<false><<<grid, kThreads, 0, s>>>(P);
  else
    fp32_step_kernel<true><<<grid, kThreads, 0, s>>>(P);
  return eco_launch_check("eco_fp32_eco_step");
}

extern "C" int64_t eco_fp32_eco_scratch_len(const eco_fp32_layer_t* layers, int n_layers) {
  if (!layers || n_layers < 1) return 0;
  i64 tiles = 0;
  for (int l = 0; l < n_layers; ++l) tiles += (layers[l].rows * layers[l].cols + kTile - 1) / kTile;
  return 3 * tiles;
}
