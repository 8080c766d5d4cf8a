// eco_gemm_s8s32_noalloc: the int32 GEMM for callers that cannot allocate.
//
// The tensor-core GEMM reads its operands with TMA, which needs a 16-byte
// aligned base address and leading dimension.  An operand that breaks that
// rule (an odd width such as 10 or 1000 columns, or a view that starts at an
// odd offset) has to be copied into an aligned buffer first, and
// eco_gemm_s8s32 leaves that buffer to the caller.  Some callers cannot
// allocate device memory at all: code that runs while a CUDA graph is being
// captured, runtimes that plan all memory ahead and forbid allocator calls
// during execution, or plain C hosts that have no caching allocator and must
// not pay cudaMalloc's synchronisation inside a step.  This entry point copies
// misaligned operands into the file-scope buffer below instead, so it calls
// no cudaMalloc, cudaFree or allocating library routine.
//
// Limits and sharing:
//   * the buffer holds kNoAllocScratchBytes (32 MiB) on every GPU whose
//     process loads this part of the library, until the process exits; a call
//     whose relayout needs more (both operands, each rounded up to 256 bytes)
//     is rejected with ECO_ERR_ARG and a message;
//   * every call shares the one buffer: calls that overlap on the GPU (two
//     streams, or two host threads) race on it and must be serialised by the
//     caller; nothing in the buffer needs to start at zero, and each call
//     overwrites what the last one left;
//   * the first call on each device looks up the buffer's device address
//     (cudaGetSymbolAddress) with that device current; make that first call
//     before any stream capture.  The address is cached for the lifetime of
//     the device's primary context: a host that calls cudaDeviceReset (or
//     otherwise tears the primary context down) must not call this entry
//     point on that device again in the same process.
#include <mutex>

#include "abi.cuh"
#include "common.cuh"

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;
static __device__ __align__(256) int8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_mu;
int8_t* g_scratch_addr[kMaxDevices] = {};

// Device address of the buffer for the current device (looked up once per device).
int scratch_address(int8_t** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return eco_launch_check("eco_gemm_s8s32_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return eco_fail(ECO_ERR_ARG, "eco_gemm_s8s32_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess)
      return eco_fail(ECO_ERR_LAUNCH, "eco_gemm_s8s32_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_scratch_addr[dev] = static_cast<int8_t*>(p);
  }
  *out = g_scratch_addr[dev];
  return ECO_OK;
}

bool tma_ok(const int8_t* p, int64_t ld) { return eco_aligned16(p) && ld % 16 == 0; }
int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

}  // namespace

extern "C" int eco_gemm_s8s32_noalloc(const int8_t* A, int64_t lda, int a_layout, const int8_t* B, int64_t ldb,
                                      int b_layout, int64_t M, int64_t N, int64_t K, const int32_t* bias,
                                      int32_t* C, int64_t ldc, int32_t* amax, eco_stream_t stream) {
  // every check of the GEMM itself comes first, so a call that will be rejected queues no relayout
  ECO_REQUIRE(A && B && C && M > 0 && N > 0 && K > 0, ECO_ERR_ARG, "eco_gemm_s8s32_noalloc: bad arguments");
  ECO_REQUIRE(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), ECO_ERR_ARG,
              "eco_gemm_s8s32_noalloc: dims too large");
  ECO_REQUIRE(ldc >= N, ECO_ERR_ARG, "eco_gemm_s8s32_noalloc: ldc < N");
  ECO_REQUIRE((a_layout == 0 || a_layout == 1) && (b_layout == 0 || b_layout == 1), ECO_ERR_ARG,
              "eco_gemm_s8s32_noalloc: layout");
  // stored shapes: A is [M, K] (layout 0) or [K, M]; B is [N, K] (layout 0) or [K, N]
  const int64_t a_rows = a_layout ? K : M, a_cols = a_layout ? M : K;
  const int64_t b_rows = b_layout ? K : N, b_cols = b_layout ? N : K;
  ECO_REQUIRE(lda >= a_cols && ldb >= b_cols, ECO_ERR_ARG, "eco_gemm_s8s32_noalloc: leading dim too small");
  const bool move_a = !tma_ok(A, lda), move_b = !tma_ok(B, ldb);
  const int64_t lda16 = round_up(a_cols, 16), ldb16 = round_up(b_cols, 16);
  const int64_t bytes_a = move_a ? round_up(a_rows * lda16, 256) : 0;
  const int64_t bytes_b = move_b ? round_up(b_rows * ldb16, 256) : 0;
  if (bytes_a + bytes_b > (int64_t)kNoAllocScratchBytes)
    return eco_fail(ECO_ERR_ARG,
                    "eco_gemm_s8s32_noalloc: relayout needs %lld bytes of scratch; this entry point has %lld "
                    "(pass 16-byte aligned operands, or use eco_gemm_s8s32 with your own buffer)",
                    (long long)(bytes_a + bytes_b), (long long)kNoAllocScratchBytes);
  if (!move_a && !move_b)
    return eco_gemm_s8s32(A, lda, a_layout, B, ldb, b_layout, M, N, K, bias, C, ldc, amax, stream);
  int8_t* scratch = nullptr;
  if (int rc = scratch_address(&scratch)) return rc;
  cudaStream_t s = eco_stream(stream);
  const int8_t* a = A;
  const int8_t* b = B;
  if (move_a) {
    if (cudaMemcpy2DAsync(scratch, (size_t)lda16, A, (size_t)lda, (size_t)a_cols, (size_t)a_rows,
                          cudaMemcpyDeviceToDevice, s) != cudaSuccess)
      return eco_launch_check("eco_gemm_s8s32_noalloc: relayout A");
    a = scratch;
    lda = lda16;
  }
  if (move_b) {
    int8_t* dst = scratch + bytes_a;
    if (cudaMemcpy2DAsync(dst, (size_t)ldb16, B, (size_t)ldb, (size_t)b_cols, (size_t)b_rows,
                          cudaMemcpyDeviceToDevice, s) != cudaSuccess)
      return eco_launch_check("eco_gemm_s8s32_noalloc: relayout B");
    b = dst;
    ldb = ldb16;
  }
  return eco_gemm_s8s32(a, lda, a_layout, b, ldb, b_layout, M, N, K, bias, C, ldc, amax, stream);
}
