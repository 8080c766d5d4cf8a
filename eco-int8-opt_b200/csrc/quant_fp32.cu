// Dynamic per-tensor int8 quantization of an fp32 matrix without a host round trip
// (quant.py:35-38, quantize_tensor_dynamic with stochastic=False), the input side of
// Int8LinearFunc (layers.py:47, :61):
//
//   a = max |x|;  s = calc_scale(a) = (a < 1e-8 ? 1 : a / 127)   (Python double arithmetic)
//   q = clamp(round(x / (s + 1e-8)), -127, 127)                     (quant.py:21-28)
//
// PyTorch divides a CUDA tensor by a Python scalar as a multiply by the scalar's
// reciprocal, taken in double and rounded to fp32, and torch.round rounds half to even;
// both are reproduced here, so q is the reference's bit for bit.  s goes to the device as
// double bits (scale_out[0]), where the dequantizing GEMM epilogue reads it.
#include <algorithm>

#include "abi.cuh"
#include "common.cuh"

namespace {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads) amax_f32_kernel(const float* __restrict__ x, int64_t rows, int64_t cols,
                                                            int64_t ld, unsigned* amax) {
  float m = 0.0f;
  const int64_t n = rows * cols;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kThreads) {
    const int64_t r = i / cols, c = i - r * cols;
    const float a = fabsf(x[r * ld + c]);
    m = (a > m || a != a) ? a : m;  // a NaN wins, as in torch.max
  }
  unsigned b = __float_as_uint(m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) b = max(b, __shfl_xor_sync(0xffffffffu, b, o));
  if ((threadIdx.x & 31) == 0 && b) atomicMax(amax, b);  // non-negative floats order like their bits
}

__global__ void __launch_bounds__(kThreads) quantize_f32_kernel(const float* __restrict__ x, int64_t rows,
                                                                int64_t cols, int64_t ld, const unsigned* amax,
                                                                int8_t* __restrict__ q, int64_t ld_q,
                                                                int64_t* scale_out) {
  const double a = (double)__uint_as_float(*amax);
  const double s = a < 1e-8 ? 1.0 : __ddiv_rn(a, 127.0);  // calc_scale (quant.py:9-16)
  const float inv = __double2float_rn(__ddiv_rn(1.0, __dadd_rn(s, 1e-8)));
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    scale_out[0] = __double_as_longlong(s);
    scale_out[1] = 0;
    scale_out[2] = 0;
  }
  const int64_t n = rows * cols;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kThreads) {
    const int64_t r = i / cols, c = i - r * cols;
    const float v = rintf(__fmul_rn(x[r * ld + c], inv));
    q[r * ld_q + c] = (int8_t)fminf(fmaxf(v, -127.0f), 127.0f);
  }
}

}  // namespace

extern "C" int eco_quantize_dynamic_f32(const float* x, int64_t rows, int64_t cols, int64_t ld, int32_t* amax,
                                        int8_t* q, int64_t ld_q, int64_t* scale_out, eco_stream_t stream) {
  ECO_REQUIRE(x && amax && q && scale_out && rows >= 0 && cols > 0 && ld >= cols && ld_q >= cols, ECO_ERR_ARG,
              "eco_quantize_dynamic_f32: bad arguments");
  cudaStream_t s = eco_stream(stream);
  if (cudaMemsetAsync(amax, 0, sizeof(int32_t), s) != cudaSuccess)
    return eco_launch_check("eco_quantize_dynamic_f32 memset");
  const int64_t cap = (int64_t)eco_num_sms() * 8;
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(cap, (rows * cols + kThreads - 1) / kThreads));
  amax_f32_kernel<<<grid, kThreads, 0, s>>>(x, rows, cols, ld, reinterpret_cast<unsigned*>(amax));
  quantize_f32_kernel<<<grid, kThreads, 0, s>>>(x, rows, cols, ld, reinterpret_cast<const unsigned*>(amax), q, ld_q,
                                                scale_out);
  return eco_launch_check("eco_quantize_dynamic_f32");
}
