// EcoInt8SGDM fused step (ecoint8/eco.py:330-362 -> triton_kernels.py:127-170)
// as three stream-ordered kernels with no host synchronisation:
//   1. max |g| into scratch[0]                              (triton_kernels.py:156)
//   2. pass 1: recompute m_new, max |m_new| into scratch[1] (eco_amax_kernel, :67-90)
//   3. pass 2: same math with the pass-2 draws, store w, m;
//      the last CTA writes sm <- sm_new and clears scratch   (eco_fused_kernel :92-119, :169)
// Each element operation is one IEEE fp32 operation in the reference's order
// (no fused multiply-add).  The two divisions by 127 of the host glue follow
// PyTorch's CUDA kernel for a tensor divided by a Python scalar: a multiply
// by the reciprocal 1/127 (taken in double and rounded to fp32, which for 127
// is also the fp32 quotient 1.0f / 127.0f).
//
// Work per element: the reference draws five Philox4x32-10 words per element (two in
// pass 1, three in pass 2, each from its own counter), so the passes are bound by the
// integer issue rate, not by HBM.  The round keys are expanded once per launch (host)
// and kept in registers; threads walk the elements with an incremental (row, column)
// so no division by the row length is done per element.
#include <algorithm>

#include "abi.cuh"
#include "common.cuh"

namespace {

constexpr int kThreads = 256;

struct SgdmArgs {
  int8_t* w;
  int8_t* m;
  const float* g;
  i64 n, cols;
  const float* sw;
  float* sm;
  float lr, beta, wd, alpha;
  u64 seed;
  uint32_t* scratch;
  PhiloxKeys keys;  // round keys of seed
};

// Triton's tl.rand(seed, offset) (common.cuh: tl_rand) with the round keys given.
ECO_DEV float tl_rand_k(const PhiloxKeys& K, uint32_t offset) {
  const Philox4 o = philox10k(offset, 0u, 0u, 0u, K);
  int x = (int)o.x;
  x = x < 0 ? -x - 1 : x;
  return __fmul_rn(__int2float_rn(x), 4.6566127342e-10f);
}

// Element walk: thread t starts at element i0 = blockIdx.x * blockDim.x + t and steps by
// the grid size; (r, c) of the element are advanced without a division per step.
struct Walk {
  i64 i, r, c, step, dr, dc;
  ECO_DEV Walk(const SgdmArgs& a) {
    i = (i64)blockIdx.x * blockDim.x + threadIdx.x;
    step = (i64)gridDim.x * blockDim.x;
    r = i / a.cols;
    c = i - r * a.cols;
    dr = step / a.cols;
    dc = step - dr * a.cols;
  }
  ECO_DEV void next(i64 cols) {
    i += step;
    r += dr;
    c += dc;
    if (c >= cols) {
      c -= cols;
      ++r;
    }
  }
};

ECO_DEV float inv127() { return __fdiv_rn(1.0f, 127.0f); }

ECO_DEV void block_max_to(float v, uint32_t* out) {
  __shared__ float part[kThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) part[warp] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) b = fmaxf(b, part[i]);
    atomicMax(out, __float_as_uint(b));  // non-negative floats order like their bits
  }
}

// _eco_elem (triton_kernels.py:54-65)
ECO_DEV void eco_elem(float w, float m, float g, float sw, float sm, float sg, const SgdmArgs& a, float r_g,
                      float r_w, float& wq, float& m_new) {
  const float gv = __fdiv_rn(__fadd_rn(g, __fmul_rn(__fmul_rn(w, sw), a.wd)), sg);
  const float gq = fminf(fmaxf(floorf(__fadd_rn(gv, r_g)), -127.0f), 127.0f);
  const float g_hat = __fmul_rn(gq, sg);
  const float m_tilde =
      __fadd_rn(__fmul_rn(__fmul_rn(a.beta, m), sm), __fmul_rn(__fsub_rn(1.0f, a.beta), g_hat));
  const float th = __fsub_rn(__fmul_rn(w, sw), __fmul_rn(a.lr, m_tilde));
  wq = fminf(fmaxf(floorf(__fadd_rn(__fdiv_rn(th, sw), r_w)), -127.0f), 127.0f);
  const float e = __fsub_rn(th, __fmul_rn(wq, sw));
  m_new = __fadd_rn(m_tilde, __fmul_rn(a.alpha, e));
}

__global__ void __launch_bounds__(kThreads) gmax_kernel(const SgdmArgs a) {
  float v = 0.0f;
  for (i64 i = (i64)blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += (i64)gridDim.x * blockDim.x)
    v = fmaxf(v, fabsf(a.g[i]));
  block_max_to(v, &a.scratch[0]);
}

ECO_DEV float sg_of(const SgdmArgs& a) {
  return __fmul_rn(fmaxf(__uint_as_float(a.scratch[0]), 1e-12f), inv127());
}

__global__ void __launch_bounds__(kThreads) pass1_kernel(const SgdmArgs a) {
  const float sg = sg_of(a), sm = *a.sm;
  const PhiloxKeys K = a.keys;
  float v = 0.0f;
  for (Walk t(a); t.i < a.n; t.next(a.cols)) {
    const uint32_t b = (uint32_t)((u64)t.i * 2u);
    float wq, m_new;
    eco_elem((float)a.w[t.i], (float)a.m[t.i], a.g[t.i], a.sw[t.r], sm, sg, a, tl_rand_k(K, b), tl_rand_k(K, b + 1u),
             wq, m_new);
    v = fmaxf(v, fabsf(m_new));
  }
  block_max_to(v, &a.scratch[1]);
}

__global__ void __launch_bounds__(kThreads) pass2_kernel(const SgdmArgs a) {
  __shared__ int s_last;
  const float sg = sg_of(a), sm = *a.sm;
  const float sm_new = __fmul_rn(__uint_as_float(a.scratch[1]), inv127());
  const float smg = __fadd_rn(sm_new, 1e-8f);
  const PhiloxKeys K = a.keys;
  for (Walk t(a); t.i < a.n; t.next(a.cols)) {
    const uint32_t b = (uint32_t)((u64)t.i * 3u);
    float wq, m_new;
    eco_elem((float)a.w[t.i], (float)a.m[t.i], a.g[t.i], a.sw[t.r], sm, sg, a, tl_rand_k(K, b), tl_rand_k(K, b + 1u),
             wq, m_new);
    const float mq = fminf(fmaxf(floorf(__fadd_rn(__fdiv_rn(m_new, smg), tl_rand_k(K, b + 2u))), -127.0f), 127.0f);
    a.w[t.i] = (int8_t)wq;
    a.m[t.i] = (int8_t)mq;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&a.scratch[2], 1u) == gridDim.x - 1;
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    *a.sm = sm_new;  // sm_t.copy_(sm_new_t)
    a.scratch[0] = 0u;
    a.scratch[1] = 0u;
    a.scratch[2] = 0u;
  }
}

}  // namespace

extern "C" int eco_sgdm_step(int8_t* w, int8_t* m, const float* g, int64_t rows, int64_t cols, const float* sw,
                             float* sm, float lr, float beta, float wd, float alpha, uint64_t seed,
                             uint32_t* scratch, eco_stream_t stream) {
  ECO_REQUIRE(w && m && g && sw && sm && scratch && rows > 0 && cols > 0, ECO_ERR_ARG,
              "eco_sgdm_step: bad arguments");
  ECO_REQUIRE(rows * cols < (1ll << 31), ECO_ERR_ARG, "eco_sgdm_step: layer exceeds int32 element offsets");
  SgdmArgs a{w, m, g, rows * cols, cols, sw, sm, lr, beta, wd, alpha, seed, scratch, philox_keys(seed)};
  cudaStream_t s = eco_stream(stream);
  if (cudaMemsetAsync(scratch, 0, 4 * sizeof(uint32_t), s) != cudaSuccess) return eco_launch_check("eco_sgdm_step memset");
  const i64 cap = (i64)eco_num_sms() * 8;
  const unsigned grid = (unsigned)std::max<i64>(1, std::min<i64>(cap, (a.n + kThreads - 1) / kThreads));
  gmax_kernel<<<grid, kThreads, 0, s>>>(a);
  pass1_kernel<<<grid, kThreads, 0, s>>>(a);
  pass2_kernel<<<grid, kThreads, 0, s>>>(a);
  return eco_launch_check("eco_sgdm_step");
}
