// The backward's dynamic scales on the device, so a whole backward pass can be
// queued without a host round trip per layer.  Same IEEE double arithmetic, in
// the same order, as the reference's Python (fixedpoint.py:105-114 and :26-37):
//   gain = g0 * g1
//   s    = amax * gain / 127   (1.0 when amax * gain <= 0)
//   (mult, shift) = quantize_multiplier(gain / s)
#include "abi.cuh"
#include "common.cuh"

namespace {

__global__ void scale_kernel(const void* amax, int bits, const int64_t* g0_dev, double g0, double g1, int64_t* out,
                             uint32_t* flags) {
  if (threadIdx.x != 0) return;
  const i64 a = bits == 32 ? (i64) * static_cast<const int32_t*>(amax) : *static_cast<const i64*>(amax);
  const double ga = g0_dev ? __longlong_as_double(*g0_dev) : g0;
  const double gain = __dmul_rn(ga, g1);
  const double real = __dmul_rn(__ll2double_rn(a), gain);
  const double s = real <= 0.0 ? 1.0 : __ddiv_rn(real, 127.0);
  const double r = __ddiv_rn(gain, s);
  int m = 0, sh = 0;
  if (!(r >= 0.0) || r > 1.7e308) {
    if (flags) atomicOr(flags, (unsigned)ECO_FLAG_BAD_RATIO);
  } else {
    qmult(r, m, sh);
  }
  if (sh > 62 && flags) atomicOr(flags, (unsigned)ECO_FLAG_SHIFT_OVERFLOW);
  out[0] = __double_as_longlong(s);
  out[1] = m;
  out[2] = sh;
}

}  // namespace

extern "C" int eco_scale_from_amax(const void* amax, int amax_bits, const int64_t* gain0_dev, double gain0,
                                   double gain1, int64_t* out, uint32_t* flags, eco_stream_t stream) {
  ECO_REQUIRE(amax && out && (amax_bits == 32 || amax_bits == 64), ECO_ERR_ARG, "eco_scale_from_amax: bad arguments");
  scale_kernel<<<1, 32, 0, eco_stream(stream)>>>(amax, amax_bits, gain0_dev, gain0, gain1, out, flags);
  return eco_launch_check("eco_scale_from_amax");
}
