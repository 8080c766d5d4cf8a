// The fp32 loss boundary at the end of the strict forward, fused: int8 logits
// -> fp32 logits -> mean cross-entropy gradient -> max |g| -> int8 gradient by
// stochastic rounding on the dynamic scale.  It replaces the four lines of the
// reference's training loop (examples/i8_demo.py:56-59) with quant.py:19-38:
//
//   logits_fp = logits_i8.float() * s_out
//   g = d CrossEntropy(logits_fp, y) / d logits_fp
//   s_g = calc_scale(max|g|);  g_i8 = clamp(floor(g / (s_g + EPS) + U[0,1)), +-127)
//
// The fp32 gradient never reaches HBM: the first launch computes each row's
// max and log-sum (one warp per row) and the global max |g|; the second
// recomputes the gradient in registers and writes int8.  The maximum is a
// device word, so a data-parallel caller takes the MAX over ranks between the
// two launches and nothing waits for the host.
//
// Arithmetic (fp32, one IEEE rounding per operation):
//   x_j = float(l_j) * s_out;  m = max_j x_j;  S = sum_j expf(x_j - m);  L = logf(S)
//   out_j = (x_j - m) - L  (log-softmax);  c = -1/count
//   g_j = -(expf(out_j) * c) for j != y,  g_y = fma(-expf(out_y), c, c)
// which is the log-softmax backward of the mean NLL loss.  The summation order
// of S is this kernel's own (lane-sequential, then a butterfly), so g agrees
// with PyTorch's CUDA cross-entropy gradient to within a few ulp; the
// quantization of a given g is PyTorch's own arithmetic bit for bit (division
// by the Python scalar s_g + EPS as a multiply by its reciprocal, taken in double
// and rounded to fp32).
#include <algorithm>

#include "abi.cuh"
#include "common.cuh"

namespace {

constexpr int kWarps = 8;

ECO_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
ECO_DEV float warp_sum(float v) {  // butterfly: every lane ends with the same bits
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

ECO_DEV float logit(const int8_t* row, int64_t j, float s) { return __fmul_rn((float)row[j], s); }

ECO_DEV float ce_grad(float x, float m, float logsum, bool target, float c) {
  const float e = expf(__fsub_rn(__fsub_rn(x, m), logsum));
  return target ? __fmaf_rn(-e, c, c) : -__fmul_rn(e, c);
}

// One warp per row; lane l owns columns 4 l + 128 k + (0..3).
__global__ void ce_rowstats_kernel(const int8_t* __restrict__ L, int64_t rows, int64_t cols, int64_t ld, float s,
                                   const int64_t* __restrict__ labels, float c, float2* __restrict__ stats,
                                   float* __restrict__ row_loss, unsigned* __restrict__ amax) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * kWarps + warp;
  if (r >= rows) return;  // whole warp
  const int8_t* row = L + r * ld;
  float m = -INFINITY;
  for (int64_t j0 = 4 * lane; j0 < cols; j0 += 128)
#pragma unroll
    for (int t = 0; t < 4; ++t)
      if (j0 + t < cols) m = fmaxf(m, logit(row, j0 + t, s));
  m = warp_max(m);
  float S = 0.0f;
  for (int64_t j0 = 4 * lane; j0 < cols; j0 += 128)
#pragma unroll
    for (int t = 0; t < 4; ++t)
      if (j0 + t < cols) S = __fadd_rn(S, expf(__fsub_rn(logit(row, j0 + t, s), m)));
  S = warp_sum(S);
  const float logsum = logf(S);
  const int64_t y = labels[r];
  float gmax = 0.0f;
  for (int64_t j0 = 4 * lane; j0 < cols; j0 += 128)
#pragma unroll
    for (int t = 0; t < 4; ++t)
      if (j0 + t < cols) gmax = fmaxf(gmax, fabsf(ce_grad(logit(row, j0 + t, s), m, logsum, j0 + t == y, c)));
  gmax = warp_max(gmax);
  if (lane == 0) {
    stats[r] = make_float2(m, logsum);
    if (row_loss) {  // NLL of the row: -log_softmax(x)_y (a label outside [0, cols) adds nothing)
      row_loss[r] = (y >= 0 && y < cols) ? -__fsub_rn(__fsub_rn(logit(row, y, s), m), logsum) : 0.0f;
    }
    if (gmax > 0.0f) atomicMax(amax, __float_as_uint(gmax));
  }
}

struct QuantArgs {
  const int8_t* L;
  int64_t rows, cols, ld;
  float s, c;
  const int64_t* labels;
  const float2* stats;
  const void* amax;
  int amax_bits;
  eco_sr_t sr;
  PhiloxKeys keys;
  int8_t* g;
  int64_t ld_g;
  float* g_fp;  // nullable: the fp32 gradient as well (tests)
  int64_t* scale_out;
  const float* row_loss;
  float* loss_out;
  int64_t count;
};

// s_g = calc_scale(max|g|) in double (quant.py:9-16), then PyTorch's division of an
// fp32 tensor by the Python scalar s_g + EPS: a multiply by its reciprocal, taken in
// double and rounded to fp32.
ECO_DEV double scale_of(const QuantArgs& A) {
  const uint32_t bits = A.amax_bits == 32 ? (uint32_t) * static_cast<const int32_t*>(A.amax)
                                          : (uint32_t) * static_cast<const int64_t*>(A.amax);
  const double a = (double)__uint_as_float(bits);
  return a < 1e-8 ? 1.0 : __ddiv_rn(a, 127.0);
}

__global__ void ce_quantize_kernel(const __grid_constant__ QuantArgs A) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * kWarps + warp;
  const double s_g = scale_of(A);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    A.scale_out[0] = __double_as_longlong(s_g);
    A.scale_out[1] = 0;
    A.scale_out[2] = 0;
  }
  if (blockIdx.x == 0 && A.loss_out) {  // the mean loss of these rows: a fixed-order sum
    __shared__ float part[kWarps * 32];
    float v = 0.0f;
    for (int64_t i = threadIdx.x; i < A.rows; i += blockDim.x) v = __fadd_rn(v, A.row_loss[i]);
    part[threadIdx.x] = v;
    __syncthreads();
    for (int w = blockDim.x / 2; w > 0; w >>= 1) {
      if ((int)threadIdx.x < w) part[threadIdx.x] = __fadd_rn(part[threadIdx.x], part[threadIdx.x + w]);
      __syncthreads();
    }
    if (threadIdx.x == 0) A.loss_out[0] = __fdiv_rn(part[0], (float)A.count);
  }
  if (r >= A.rows) return;
  const float inv = __double2float_rn(__ddiv_rn(1.0, __dadd_rn(s_g, 1e-8)));
  const int8_t* row = A.L + r * A.ld;
  const float2 st = A.stats[r];
  const int64_t y = A.labels[r];
  PhiloxKeys keys;
  const eco_sr_t sr = sr_resolve(A.sr, A.keys, keys);
  const bool philox = sr.mode == ECO_SR_PHILOX;
  const uint32_t grow = (uint32_t)(sr.row_base + r);
  int8_t* out = A.g + r * A.ld_g;
  for (int64_t j0 = 4 * lane; j0 < A.cols; j0 += 128) {
    Philox4 rnd{0u, 0u, 0u, 0u};
    if (philox) rnd = sr_quad_k(keys, sr.stream, grow, (uint32_t)(j0 >> 2));
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int64_t j = j0 + t;
      if (j >= A.cols) break;
      const float g = ce_grad(logit(row, j, A.s), st.x, st.y, j == y, A.c);
      if (A.g_fp) A.g_fp[r * A.cols + j] = g;
      const float u = philox ? __fmul_rn((float)(quad_word(rnd, t) >> 8), 0x1p-24f)
                             : static_cast<const float*>(sr.nudge)[r * sr.nudge_ld + j];
      const float q = floorf(__fadd_rn(__fmul_rn(g, inv), u));
      out[j] = (int8_t)fmaxf(-127.0f, fminf(127.0f, q));
    }
  }
}

}  // namespace

extern "C" int eco_ce_grad_rowstats(const int8_t* logits, int64_t rows, int64_t cols, int64_t ld, double s_out,
                                    const int64_t* labels, int64_t count, float* row_stats, float* row_loss,
                                    int32_t* amax, eco_stream_t stream) {
  ECO_REQUIRE(logits && labels && row_stats && amax && rows >= 0 && cols > 0 && ld >= cols && count > 0,
              ECO_ERR_ARG, "eco_ce_grad_rowstats: bad arguments");
  cudaStream_t s = eco_stream(stream);
  if (cudaMemsetAsync(amax, 0, sizeof(int32_t), s) != cudaSuccess) return eco_launch_check("ce amax memset");
  if (rows == 0) return ECO_OK;
  const float c = -(1.0f / (float)count);
  const int64_t grid = (rows + kWarps - 1) / kWarps;
  ce_rowstats_kernel<<<(unsigned)grid, 32 * kWarps, 0, s>>>(logits, rows, cols, ld, (float)s_out, labels, c,
                                                            reinterpret_cast<float2*>(row_stats), row_loss,
                                                            reinterpret_cast<unsigned*>(amax));
  return eco_launch_check("eco_ce_grad_rowstats");
}

extern "C" int eco_ce_grad_quantize(const int8_t* logits, int64_t rows, int64_t cols, int64_t ld, double s_out,
                                    const int64_t* labels, int64_t count, const float* row_stats,
                                    const void* amax, int amax_bits, eco_sr_t sr, int8_t* g, int64_t ld_g,
                                    float* g_fp, int64_t* scale_out, const float* row_loss, float* loss_out,
                                    eco_stream_t stream) {
  ECO_REQUIRE(logits && labels && row_stats && amax && g && scale_out && rows >= 0 && cols > 0 && ld >= cols &&
                  ld_g >= cols && count > 0 && (amax_bits == 32 || amax_bits == 64),
              ECO_ERR_ARG, "eco_ce_grad_quantize: bad arguments");
  ECO_REQUIRE(sr.mode == ECO_SR_PHILOX || (sr.mode == ECO_SR_PHILOX_DEV && sr.nudge) ||
                  (sr.mode == ECO_SR_REPLAY_F32 && sr.nudge && sr.nudge_ld >= cols),
              ECO_ERR_ARG, "eco_ce_grad_quantize: SR mode must be Philox or fp32 replay");
  ECO_REQUIRE(!loss_out || row_loss, ECO_ERR_ARG, "eco_ce_grad_quantize: the loss needs the row losses");
  QuantArgs A;
  A.L = logits;
  A.rows = rows;
  A.cols = cols;
  A.ld = ld;
  A.s = (float)s_out;
  A.c = -(1.0f / (float)count);
  A.labels = labels;
  A.stats = reinterpret_cast<const float2*>(row_stats);
  A.amax = amax;
  A.amax_bits = amax_bits;
  A.sr = sr;
  A.keys = philox_keys(sr.mode == ECO_SR_PHILOX ? sr.seed : 0);
  A.g = g;
  A.ld_g = ld_g;
  A.g_fp = g_fp;
  A.scale_out = scale_out;
  A.row_loss = row_loss;
  A.loss_out = loss_out;
  A.count = count;
  const int64_t grid = std::max<int64_t>(1, (rows + kWarps - 1) / kWarps);
  ce_quantize_kernel<<<(unsigned)grid, 32 * kWarps, 0, eco_stream(stream)>>>(A);
  return eco_launch_check("eco_ce_grad_quantize");
}
