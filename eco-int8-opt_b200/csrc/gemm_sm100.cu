// int8 x int8 -> int32 GEMM on sm_100a tensor cores (tcgen05.mma kind::i8).
//
// One CTA computes one 128 x BN output tile.  Warp roles (192 threads):
//   warp 0     TMA producer: one thread streams 128-deep K slices of A and B
//              into an S-stage shared-memory ring (128-byte swizzle);
//   warp 1     owns the TMEM accumulator (alloc / dealloc) and one thread issues
//              tcgen05.mma (M=128, N=BN, K=32) four times per slice;
//   warps 2-5  epilogue: tcgen05.ld the int32 accumulator (one row per thread),
//              then either store int32 + track max|C| (dX, dW, calibration) or
//              requantize in registers -- bias add, per-column multiplier,
//              stochastic rounding, ReLU, int8 saturation -- and store int8, so
//              the forward's int32 accumulator never reaches HBM.
// Both operand majors are native: a K-major tile is a [rows][128 B] TMA box,
// an MN-major tile is one or two [128 K rows][128 B] boxes, described to the
// MMA by the canonical SWIZZLE_128B K-major / MN-major shared-memory layouts.
// Every mbarrier wait is bounded by %globaltimer: on expiry the thread records
// ECO_FLAG_WAIT_TIMEOUT in a device word, in-flight copies are drained with a
// bounded wait, TMEM is freed and the CTA returns.
#include <cuda.h>

#include <algorithm>

#include "abi.cuh"
#include "common.cuh"

__device__ unsigned g_eco_device_errors;  // sticky error flags of bounded device waits

namespace {

constexpr int BM = 128;
constexpr int BK = 128;  // bytes = int8 elements per K slice (one 128-byte swizzle row)
constexpr int kThreads = 192;
constexpr unsigned long long kWaitNs = 4000000000ull;  // 4 s bound on any single wait

template <int BN>
struct Cfg {
  static constexpr int S = BN == 256 ? 4 : 6;
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = BN * BK;
  static constexpr int SMEM = S * (A_BYTES + B_BYTES) + 1024 /*barriers etc*/ + 2 * BN * 4 + 1024 /*align*/;
};

struct GemmParams {
  int M, N, K;
  int a_mn, b_mn;
  const int32_t* bias;
  // int32 epilogue
  int32_t* C;
  i64 ldc;
  int32_t* amax;
  // fused requant epilogue
  const int32_t* mult;
  int shift, relu;
  eco_sr_t sr;
  int8_t* Y;
  i64 ldy;
};

ECO_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
ECO_DEV unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
ECO_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
ECO_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
ECO_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the completion of phase `parity`; false (and a sticky flag) on timeout.
ECO_DEV bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kWaitNs) {
      atomicOr(&g_eco_device_errors, ECO_FLAG_WAIT_TIMEOUT);
      return false;
    }
  }
  return true;
}
ECO_DEV void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
ECO_DEV void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
ECO_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
ECO_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
ECO_DEV void umma_s8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
ECO_DEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
ECO_DEV void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor (tcgen05): start, leading / stride byte
// offsets (16-byte units), version 1, SWIZZLE_128B layout.
ECO_DEV uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor, kind::i8: D s32, A/B signed, majors, N >> 3, M >> 4.
ECO_DEV uint32_t idesc_s8(int n, int a_mn, int b_mn) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_s8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmParams p) {
  using C = Cfg<BN>;
  constexpr int S = C::S;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * C::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + S * C::B_BYTES);
  uint64_t* empty = full + S;
  uint64_t* accum = empty + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  volatile uint32_t* abort_flag = tmem_slot + 1;  // set when the producer or MMA thread timed out
  int32_t* s_mult = reinterpret_cast<int32_t*>(smem + S * (C::A_BYTES + C::B_BYTES) + 1024);
  int32_t* s_bias = s_mult + BN;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int num_kb = (p.K + BK - 1) / BK;

  if (warp == 0 && lane == 0) {
    *abort_flag = 0u;
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (warp >= 2) {
    for (int i = threadIdx.x - 64; i < BN; i += 128) {
      const int n = n0 + i;
      s_bias[i] = (p.bias && n < p.N) ? p.bias[n] : 0;
      s_mult[i] = (EPI == 1 && n < p.N) ? p.mult[n] : 0;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % S;
        const uint32_t ph = (uint32_t)(kb / S) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u)) {
          *abort_flag = 1u;
          break;
        }
        mbar_arrive_expect_tx(&full[s], C::A_BYTES + C::B_BYTES);
        const int k0 = kb * BK;
        uint8_t* a_dst = sA + s * C::A_BYTES;
        uint8_t* b_dst = sB + s * C::B_BYTES;
        if (p.a_mn)
          tma_load_2d(a_dst, &tmA, &full[s], m0, k0);
        else
          tma_load_2d(a_dst, &tmA, &full[s], k0, m0);
        if (p.b_mn) {
#pragma unroll
          for (int j = 0; j < BN / 128; ++j) tma_load_2d(b_dst + j * (128 * BK), &tmB, &full[s], n0 + 128 * j, k0);
        } else {
          tma_load_2d(b_dst, &tmB, &full[s], k0, n0);
        }
        ++issued;
      }
      // drain: every issued copy must land before the CTA can exit
      for (int kb = issued > S ? issued - S : 0; kb < issued; ++kb) mbar_wait(&full[kb % S], (uint32_t)(kb / S) & 1u);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_s8(BN, p.a_mn, p.b_mn);
      const uint32_t a_kstep = p.a_mn ? 32 * 128 : 32, b_kstep = p.b_mn ? 32 * 128 : 32;
      const uint32_t a_lbo = p.a_mn ? 128 * BK : 16, b_lbo = p.b_mn ? 128 * BK : 16;
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % S;
        if (!mbar_wait(&full[s], (uint32_t)(kb / S) & 1u)) {
          *abort_flag = 1u;
          break;
        }
        tc_fence_after();
        const uint32_t a_base = smem_u32(sA + s * C::A_BYTES), b_base = smem_u32(sB + s * C::B_BYTES);
#pragma unroll
        for (int kk = 0; kk < BK / 32; ++kk) {
          umma_s8(tmem, smem_desc(a_base + kk * a_kstep, a_lbo, 1024), smem_desc(b_base + kk * b_kstep, b_lbo, 1024),
                  idesc, (kb | kk) != 0);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(accum);  // also on an early exit: marks every issued MMA retired
    }
  } else {
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;
    const int m = m0 + row;
    const bool ok = mbar_wait(accum, 0) && *abort_flag == 0u;
    tc_fence_after();
    if (ok && num_kb > 0) {
      i64 amax = 0;
      for (int ch = 0; ch < BN / 32; ++ch) {
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(ch * 32), v);
        const int nb = n0 + ch * 32;
        if (nb >= p.N) continue;  // warp-uniform: whole chunk beyond N
        if (EPI == 0) {
          int o[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            o[e] = add32((int)v[e], s_bias[ch * 32 + e]);
            const int a = (int)(o[e] < 0 ? 0u - (unsigned)o[e] : (unsigned)o[e]);
            if (nb + e < p.N && m < p.M) amax = max(amax, (i64)a);
          }
          if (m < p.M) {
            int32_t* dst = p.C + (i64)m * p.ldc + nb;
            if (nb + 32 <= p.N && (p.ldc & 3) == 0 && (reinterpret_cast<uintptr_t>(p.C) & 15) == 0) {
#pragma unroll
              for (int e = 0; e < 32; e += 4) *reinterpret_cast<int4*>(dst + e) = make_int4(o[e], o[e + 1], o[e + 2], o[e + 3]);
            } else {
              for (int e = 0; e < 32 && nb + e < p.N; ++e) dst[e] = o[e];
            }
          }
        } else {
          uint32_t packed[8];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            i64 nud[2] = {0, 0};
            if (p.shift >= 0) {
              if (p.sr.mode == ECO_SR_NEAREST) {
                nud[0] = nud[1] = half_nudge(p.shift);
              } else if (p.sr.mode == ECO_SR_PHILOX) {
                u64 we, wo;
                sr_pair(p.sr.seed, p.sr.stream, (uint32_t)(p.sr.row_base + m), (uint32_t)((nb + e) >> 1), we, wo);
                nud[0] = low_bits(we, p.shift);
                nud[1] = low_bits(wo, p.shift);
              } else if (m < p.M) {
#pragma unroll
                for (int d = 0; d < 2; ++d) {
                  if (nb + e + d < p.N) {
                    const i64 idx = (i64)m * p.sr.nudge_ld + nb + e + d;
                    nud[d] = p.sr.mode == ECO_SR_REPLAY32 ? (i64) static_cast<const int32_t*>(p.sr.nudge)[idx]
                                                         : static_cast<const i64*>(p.sr.nudge)[idx];
                  }
                }
              }
            }
#pragma unroll
            for (int d = 0; d < 2; ++d) {
              const int x = add32((int)v[e + d], s_bias[ch * 32 + e + d]);
              int8_t y = sat8(ams((i64)x, (i64)s_mult[ch * 32 + e + d], p.shift, nud[d]));
              if (p.relu && y < 0) y = 0;
              const int byte = e + d;
              if (byte % 4 == 0) packed[byte / 4] = 0;
              packed[byte / 4] |= (uint32_t)(uint8_t)y << (8 * (byte % 4));
            }
          }
          if (m < p.M) {
            int8_t* dst = p.Y + (i64)m * p.ldy + nb;
            if (nb + 32 <= p.N && (p.ldy & 15) == 0 && (reinterpret_cast<uintptr_t>(p.Y) & 15) == 0) {
              *reinterpret_cast<int4*>(dst) = make_int4(packed[0], packed[1], packed[2], packed[3]);
              *reinterpret_cast<int4*>(dst + 16) = make_int4(packed[4], packed[5], packed[6], packed[7]);
            } else {
              for (int e = 0; e < 32 && nb + e < p.N; ++e) dst[e] = (int8_t)(packed[e / 4] >> (8 * (e % 4)));
            }
          }
        }
      }
      if (EPI == 0 && p.amax) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = max(amax, (i64)__shfl_xor_sync(0xffffffffu, amax, o));
        if (lane == 0) atomicMax(p.amax, (int)amax);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN));
  }
}

// ------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D int8 tensor map over [outer][inner] with leading dimension `ld` (bytes).
int make_tmap(CUtensorMap* map, const int8_t* base, i64 inner, i64 outer, i64 ld, int box_inner, int box_outer) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return eco_fail(ECO_ERR_LAUNCH, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  const cuuint64_t strides[1] = {(cuuint64_t)ld};
  const cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return eco_fail(ECO_ERR_LAUNCH, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return ECO_OK;
}

template <int BN, int EPI>
int launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, cudaStream_t s) {
  auto kern = gemm_s8_kernel<BN, EPI>;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<BN>::SMEM) != cudaSuccess)
      return eco_launch_check("gemm: cudaFuncSetAttribute");
    attr_set = true;
  }
  dim3 grid((unsigned)((p.N + BN - 1) / BN), (unsigned)((p.M + BM - 1) / BM));
  kern<<<grid, kThreads, Cfg<BN>::SMEM, s>>>(ta, tb, p);
  return eco_launch_check("gemm_s8_kernel");
}

int gemm_common(const int8_t* A, i64 lda, int a_layout, const int8_t* B, i64 ldb, int b_layout, i64 M, i64 N, i64 K,
                GemmParams& p, int epi, cudaStream_t s, const char* who) {
  ECO_REQUIRE(A && B && M > 0 && N > 0 && K > 0, ECO_ERR_ARG, "%s: null operand or empty shape", who);
  ECO_REQUIRE(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), ECO_ERR_ARG, "%s: dims too large", who);
  ECO_REQUIRE((a_layout == 0 || a_layout == 1) && (b_layout == 0 || b_layout == 1), ECO_ERR_ARG, "%s: layout", who);
  ECO_REQUIRE(lda >= (a_layout ? M : K) && ldb >= (b_layout ? N : K), ECO_ERR_ARG, "%s: leading dim too small", who);
  ECO_REQUIRE(eco_aligned16(A) && eco_aligned16(B) && lda % 16 == 0 && ldb % 16 == 0, ECO_ERR_MISALIGNED,
              "%s: operands need 16-byte aligned base and leading dims (lda=%lld ldb=%lld)", who, (long long)lda,
              (long long)ldb);
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.a_mn = a_layout;
  p.b_mn = b_layout;
  const int BN = N <= 128 ? 128 : 256;
  CUtensorMap ta, tb;
  if (int rc = a_layout ? make_tmap(&ta, A, M, K, lda, 128, BK) : make_tmap(&ta, A, K, M, lda, BK, BM)) return rc;
  if (int rc = b_layout ? make_tmap(&tb, B, N, K, ldb, 128, BK) : make_tmap(&tb, B, K, N, ldb, BK, BN)) return rc;
  if (BN == 128)
    return epi ? launch<128, 1>(ta, tb, p, s) : launch<128, 0>(ta, tb, p, s);
  return epi ? launch<256, 1>(ta, tb, p, s) : launch<256, 0>(ta, tb, p, s);
}

}  // namespace

extern "C" int eco_gemm_s8s32(const int8_t* A, int64_t lda, int a_layout, const int8_t* B, int64_t ldb, int b_layout,
                              int64_t M, int64_t N, int64_t K, const int32_t* bias, int32_t* C, int64_t ldc,
                              int32_t* amax, eco_stream_t stream) {
  ECO_REQUIRE(C && ldc >= N, ECO_ERR_ARG, "eco_gemm_s8s32: bad output");
  cudaStream_t s = eco_stream(stream);
  if (amax && cudaMemsetAsync(amax, 0, sizeof(int32_t), s) != cudaSuccess) return eco_launch_check("gemm amax memset");
  GemmParams p{};
  p.bias = bias;
  p.C = C;
  p.ldc = ldc;
  p.amax = amax;
  return gemm_common(A, lda, a_layout, B, ldb, b_layout, M, N, K, p, 0, s, "eco_gemm_s8s32");
}

extern "C" int eco_gemm_s8_requant(const int8_t* A, int64_t lda, int a_layout, const int8_t* B, int64_t ldb,
                                   int b_layout, int64_t M, int64_t N, int64_t K, const int32_t* bias,
                                   const int32_t* mult, int shift, int relu, eco_sr_t sr, int8_t* Y, int64_t ldy,
                                   eco_stream_t stream) {
  ECO_REQUIRE(Y && mult && ldy >= N, ECO_ERR_ARG, "eco_gemm_s8_requant: bad output or multipliers");
  if (int rc = eco_check_sr(sr, shift, "eco_gemm_s8_requant")) return rc;
  GemmParams p{};
  p.bias = bias;
  p.mult = mult;
  p.shift = shift;
  p.relu = relu;
  p.sr = sr;
  p.Y = Y;
  p.ldy = ldy;
  return gemm_common(A, lda, a_layout, B, ldb, b_layout, M, N, K, p, 1, eco_stream(stream), "eco_gemm_s8_requant");
}

extern "C" int eco_read_device_errors(uint32_t* flags) {
  ECO_REQUIRE(flags, ECO_ERR_ARG, "eco_read_device_errors: null output");
  unsigned v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_eco_device_errors, sizeof(v)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_eco_device_errors, &zero, sizeof(zero)) != cudaSuccess)
    return eco_launch_check("eco_read_device_errors");
  *flags = v;
  return ECO_OK;
}
