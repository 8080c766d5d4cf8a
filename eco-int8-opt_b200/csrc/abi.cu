// C-ABI housekeeping: version, last error, device support, shared checks.
#include "abi.cuh"

#include <algorithm>
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

namespace {
// Row copy into a destination whose rows start on 16-byte boundaries, from rows of any
// alignment (the relayout of an operand for the GEMM's TMA loads): a thread writes one
// 16-byte chunk, assembled by funnel shifts from the aligned 4-byte words that hold its
// 16 source bytes (every word read holds at least one byte of the row, so no read leaves
// the row's words); a row's last chunk, when shorter than 16 bytes, is copied bytewise.
__global__ void copy_rows_to_aligned_kernel(const int8_t* __restrict__ src, int64_t ld_src, int8_t* __restrict__ dst,
                                            int64_t ld_dst, int64_t rows, int64_t cols) {
  const int64_t nchunk = (cols + 15) / 16;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nchunk) return;
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
    const int8_t* s = src + r * ld_src + 16 * i;
    int8_t* d = dst + r * ld_dst + 16 * i;
    if (16 * i + 16 <= cols) {
      const uintptr_t a = reinterpret_cast<uintptr_t>(s);
      const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
      const uint32_t sh = (uint32_t)(a & 3) * 8;
      const uint32_t w0 = __ldg(w), w1 = __ldg(w + 1), w2 = __ldg(w + 2), w3 = __ldg(w + 3);
      const uint32_t w4 = sh ? __ldg(w + 4) : 0u;
      *reinterpret_cast<uint4*>(d) = make_uint4(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh),
                                                __funnelshift_r(w2, w3, sh), __funnelshift_r(w3, w4, sh));
    } else {
      for (int64_t b = 0; b < cols - 16 * i; ++b) d[b] = s[b];
    }
  }
}
}  // namespace

extern "C" int eco_copy2d_s8(const int8_t* src, int64_t ld_src, int8_t* dst, int64_t ld_dst,
                             int64_t rows, int64_t cols, eco_stream_t stream) {
  ECO_REQUIRE(src && dst && rows >= 0 && cols >= 0 && ld_src >= cols && ld_dst >= cols, ECO_ERR_ARG,
              "eco_copy2d_s8: bad arguments");
  if (rows == 0 || cols == 0) return ECO_OK;
  if (eco_aligned16(dst) && ld_dst % 16 == 0) {
    const int64_t nchunk = (cols + 15) / 16;
    const dim3 grid((unsigned)((nchunk + 127) / 128), (unsigned)std::min<int64_t>(rows, 32768));
    copy_rows_to_aligned_kernel<<<grid, 128, 0, eco_stream(stream)>>>(src, ld_src, dst, ld_dst, rows, cols);
    return eco_launch_check("eco_copy2d_s8");
  }
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
