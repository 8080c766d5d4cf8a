// C-ABI housekeeping: version, last error, device support, shared checks.
#include "abi.cuh"

#include <cstring>
#include <mutex>

static thread_local char g_last_error[512] = "";

int eco_fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int eco_launch_check(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return eco_fail(ECO_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  return ECO_OK;
}

int eco_num_sms() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

int eco_check_sr(const eco_sr_t& sr, int shift, const char* who) {
  if (shift > 62)
    return eco_fail(ECO_ERR_RANGE, "%s: shift %d > 62 does not fit the int64 requant", who, shift);
  if (sr.mode < ECO_SR_NEAREST || sr.mode > ECO_SR_PHILOX_DEV || sr.mode == ECO_SR_REPLAY_F32)
    return eco_fail(ECO_ERR_ARG, "%s: unknown SR mode %d", who, sr.mode);
  if (sr.mode == ECO_SR_PHILOX_DEV && (sr.nudge == nullptr || (reinterpret_cast<uintptr_t>(sr.nudge) & 7) != 0))
    return eco_fail(ECO_ERR_ARG, "%s: ECO_SR_PHILOX_DEV needs an 8-byte aligned key word", who);
  if ((sr.mode == ECO_SR_REPLAY32 || sr.mode == ECO_SR_REPLAY64) && shift >= 0 && sr.nudge == nullptr)
    return eco_fail(ECO_ERR_ARG, "%s: replay SR mode without a nudge tensor", who);
  return ECO_OK;
}

extern "C" int eco_abi_version(void) { return ECO_ABI_VERSION; }

extern "C" const char* eco_last_error(void) { return g_last_error; }

extern "C" int eco_device_supported(int device) {
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess) {
    cudaGetLastError();
    return eco_fail(ECO_ERR_ARG, "eco_device_supported: no CUDA device %d", device);
  }
  return (major == 10 && minor == 0) ? 1 : 0;
}

extern "C" int eco_copy2d_s8(const int8_t* src, int64_t ld_src, int8_t* dst, int64_t ld_dst,
                             int64_t rows, int64_t cols, eco_stream_t stream) {
  ECO_REQUIRE(src && dst && rows >= 0 && cols >= 0 && ld_src >= cols && ld_dst >= cols, ECO_ERR_ARG,
              "eco_copy2d_s8: bad arguments");
  if (rows == 0 || cols == 0) return ECO_OK;
  cudaError_t e = cudaMemcpy2DAsync(dst, (size_t)ld_dst, src, (size_t)ld_src, (size_t)cols, (size_t)rows,
                                    cudaMemcpyDeviceToDevice, eco_stream(stream));
  if (e != cudaSuccess) return eco_fail(ECO_ERR_LAUNCH, "eco_copy2d_s8: %s", cudaGetErrorString(e));
  return ECO_OK;
}

namespace {
// dst[p][r][j] = src[r][p * c + j]: 16 bytes per thread when every row and block
// start is 16-byte aligned, else one byte per thread.
template <bool VEC>
__global__ void split_cols_kernel(const int8_t* __restrict__ src, int64_t ld, int64_t rows, int64_t c,
                                  int64_t parts, int8_t* __restrict__ dst) {
  const int64_t unit = VEC ? 16 : 1;
  const int64_t per_row = c / unit;
  const int64_t total = parts * rows * per_row;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < total; q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = q / (rows * per_row);
    const int64_t rem = q - p * rows * per_row;
    const int64_t r = rem / per_row;
    const int64_t j = rem - r * per_row;
    const int8_t* s = src + r * ld + p * c + j * unit;
    if (VEC)
      reinterpret_cast<int4*>(dst)[q] = *reinterpret_cast<const int4*>(s);
    else
      dst[q] = *s;
  }
}
}  // namespace

extern "C" int eco_split_cols_s8(const int8_t* src, int64_t ld_src, int64_t rows, int64_t cols, int64_t parts,
                                 int8_t* dst, eco_stream_t stream) {
  ECO_REQUIRE(src && dst && rows >= 0 && cols >= 0 && parts > 0 && cols % parts == 0 && ld_src >= cols,
              ECO_ERR_ARG, "eco_split_cols_s8: bad arguments (cols must divide into parts)");
  if (rows == 0 || cols == 0) return ECO_OK;
  const int64_t c = cols / parts;
  const bool vec = c % 16 == 0 && ld_src % 16 == 0 && eco_aligned16(src) && eco_aligned16(dst);
  const int64_t units = parts * rows * (vec ? c / 16 : c);
  const int64_t grid = std::min<int64_t>((units + 255) / 256, (int64_t)eco_num_sms() * 8);
  if (vec)
    split_cols_kernel<true><<<(unsigned)grid, 256, 0, eco_stream(stream)>>>(src, ld_src, rows, c, parts, dst);
  else
    split_cols_kernel<false><<<(unsigned)grid, 256, 0, eco_stream(stream)>>>(src, ld_src, rows, c, parts, dst);
  return eco_launch_check("eco_split_cols_s8");
}
