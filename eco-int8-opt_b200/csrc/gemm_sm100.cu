// int8 x int8 -> int32 GEMM on sm_100a tensor cores (tcgen05.mma kind::i8).
//
// Persistent kernel: one CTA per SM walks a grouped order of 128 x BN output
// tiles.  Warp roles (320 threads):
//   warp 0     TMA producer: one thread streams 128-deep K slices of A and B into
//              an S-stage shared-memory ring (128-byte swizzle), across tiles;
//   warp 1     owns TMEM (2 x BN columns: a double-buffered accumulator) and one
//              thread issues tcgen05.mma (M=128, N=BN, K=32) four times per slice
//              into the buffer the epilogue is not draining;
//   warps 2-9  epilogue: two warps per TMEM lane quarter, each on half of the
//              columns, tcgen05.ld the int32 accumulator (one row per thread) and
//              either store int32 + track max|C| (dX, dW, calibration) or
//              requantize in registers -- bias add, per-column multiplier,
//              stochastic rounding, ReLU, int8 saturation -- and store int8, so
//              the forward's int32 accumulator never reaches HBM.  Then they
//              release the buffer, and the epilogue of tile i overlaps the
//              MMAs of tile i+1.
// Both operand majors are native: a K-major tile is a [rows][128 B] TMA box,
// an MN-major tile is one or two [128 K rows][128 B] boxes, described to the
// MMA by the canonical SWIZZLE_128B K-major / MN-major shared-memory layouts.
// Every TMA load fills only the issuing CTA's own shared memory (the kernels also run in
// multi-GPU jobs).
// Every mbarrier wait is bounded by %globaltimer: on expiry the thread records
// ECO_FLAG_WAIT_TIMEOUT in a device word and raises the CTA's abort flag, the
// roles leave their loops, in-flight copies and MMAs are drained with bounded
// waits, TMEM is freed and the CTA returns.
#include <cuda.h>

#include <algorithm>
#include <cstdlib>

#include "abi.cuh"
#include "common.cuh"

__device__ unsigned g_eco_device_errors;  // sticky error flags of bounded device waits

namespace {

constexpr int BM = 128;
constexpr int BK = 128;  // bytes = int8 elements per K slice (one 128-byte swizzle row)
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr unsigned long long kWaitNs = 4000000000ull;  // 4 s bound on any single wait
constexpr int kGroupM = 16;                            // M tiles per raster group (L2 reuse)
constexpr int kStageBytes = kEpiWarps * 4096;          // epilogue row staging, 4 KB per warp

template <int BN>
struct Cfg {
  static constexpr int S = BN == 256 ? 4 : 6;
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = BN * BK;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM = S * (A_BYTES + B_BYTES) + 1024 /*barriers*/ + kStageBytes + 1024 /*align*/;
};

struct GemmParams {
  int M, N, K;
  int a_mn, b_mn;
  int tiles_m, tiles_n;
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
  PhiloxKeys keys;  // round keys of sr.seed
  // fp32 dequant epilogue: Yf = fp32(C) * fp32(sa * sb) * col_scale[n] + bias_f[n]
  float* Yf;
  i64 ldyf;
  const int64_t* sa_dev;  // nullable: sa as double bits on the device
  const int64_t* sb_dev;  // nullable: sb as double bits on the device
  double sa, sb;
  const float* col_scale;  // nullable
  const float* bias_f;     // nullable
};

// Tile t of the grouped raster: kGroupM M-tiles share each N column block in turn.
ECO_DEV void tile_coords(const GemmParams& p, int t, int& mb, int& nb) {
  const int per_group = kGroupM * p.tiles_n;
  const int g = t / per_group, r = t - g * per_group;
  const int m_first = g * kGroupM;
  const int gm = min(kGroupM, p.tiles_m - m_first);
  mb = m_first + r % gm;
  nb = r / gm;
}

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
ECO_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
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

// A warp's 32 x 32-word chunk (lane = row) written to rows that are not 16-byte aligned
// or that end inside the chunk: staged in the warp's 4 KB of shared memory, then stored
// one row per instruction (lane = column), so a store covers 128 contiguous bytes instead
// of 32 scattered words.  Row r's 16-byte group g sits at group g ^ (r & 7), which keeps
// both the 16-byte writes and the row reads free of bank conflicts.
ECO_DEV void stage_store_rows32(uint32_t* stage, const uint32_t (&w)[32], int lane, uint32_t* row0, i64 ld,
                                int rows_left, int cols_left) {
#pragma unroll
  for (int g = 0; g < 8; ++g)
    *reinterpret_cast<uint4*>(stage + lane * 32 + ((g ^ (lane & 7)) << 2)) =
        make_uint4(w[4 * g], w[4 * g + 1], w[4 * g + 2], w[4 * g + 3]);
  __syncwarp();
  const int rows = min(rows_left, 32);
#pragma unroll 4
  for (int r = 0; r < rows; ++r) {
    const uint32_t x = stage[r * 32 + ((((lane >> 2) ^ (r & 7)) << 2) | (lane & 3))];
    if (lane < cols_left) row0[r * ld + lane] = x;
  }
  __syncwarp();
}

// The same for a 32 x 32-byte chunk of int8 rows (lane = row holds 8 packed words).
// Row r's 16-byte halves sit at half h ^ ((r >> 2) & 1).
ECO_DEV void stage_store_rows8(uint32_t* stage, const uint32_t (&packed)[8], int lane, int8_t* row0, i64 ld,
                               int rows_left, int cols_left) {
  uint8_t* sb = reinterpret_cast<uint8_t*>(stage);
#pragma unroll
  for (int h = 0; h < 2; ++h)
    *reinterpret_cast<uint4*>(sb + lane * 32 + ((h ^ ((lane >> 2) & 1)) << 4)) =
        make_uint4(packed[4 * h], packed[4 * h + 1], packed[4 * h + 2], packed[4 * h + 3]);
  __syncwarp();
  const int rows = min(rows_left, 32);
#pragma unroll 4
  for (int r = 0; r < rows; ++r) {
    const uint8_t x = sb[r * 32 + ((((lane >> 4) ^ ((r >> 2) & 1))) << 4) + (lane & 15)];
    if (lane < cols_left) row0[r * ld + lane] = (int8_t)x;
  }
  __syncwarp();
}

// int32 epilogue for one 32-column chunk of one row: bias add, max|C|, store.
ECO_DEV void epi_store_s32(const GemmParams& p, const uint32_t (&v)[32], int m, int nb, int bias_lane, i64& amax,
                           uint32_t* stage, int lane) {
  uint32_t o[32];
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    const int x = add32((int)v[e], __shfl_sync(0xffffffffu, bias_lane, e));
    o[e] = (uint32_t)x;
    const int a = (int)(x < 0 ? 0u - (unsigned)x : (unsigned)x);
    if (nb + e < p.N && m < p.M) amax = max(amax, (i64)a);
  }
  if (nb + 32 <= p.N && (p.ldc & 3) == 0 && (reinterpret_cast<uintptr_t>(p.C) & 15) == 0) {  // warp-uniform
    if (m >= p.M) return;
    uint32_t* dst = reinterpret_cast<uint32_t*>(p.C + (i64)m * p.ldc + nb);
#pragma unroll
    for (int e = 0; e < 32; e += 4) *reinterpret_cast<uint4*>(dst + e) = make_uint4(o[e], o[e + 1], o[e + 2], o[e + 3]);
  } else {
    const int m0 = m - lane;
    stage_store_rows32(stage, o, lane, reinterpret_cast<uint32_t*>(p.C + (i64)m0 * p.ldc + nb), p.ldc, p.M - m0,
                       p.N - nb);
  }
}

// Fused requant epilogue for one 32-column chunk of one row: one Philox call per
// four columns (the element's 32-bit field; exact tie-break draws only when needed).
ECO_DEV void epi_store_requant(const GemmParams& p, const eco_sr_t& sr, const PhiloxKeys& keys,
                               const uint32_t (&v)[32], int m, int nb, int bias_lane, int mult_lane, uint32_t* stage,
                               int lane) {
  uint32_t packed[8];
  const uint32_t row = (uint32_t)(sr.row_base + m);
  const bool philox = sr.mode == ECO_SR_PHILOX && p.shift >= 0;
  if (philox && p.shift > 32 && p.shift <= 62) {
    // The usual forward case: single-instruction wide products, the 32-bit Philox field
    // added in place by a multiply-add, the 2^-32 tie test out of the per-element branch
    // (the warp redoes its tied elements together, so the shuffles stay convergent).
    const int sh = p.shift, lo = sh - 32;
    const uint32_t pow2lo = 1u << lo;
    const int lower = p.relu ? 0 : -127;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const Philox4 rnd = sr_quad_k(keys, sr.stream, row, (uint32_t)((nb >> 2) + q));
      int y4[4];
      unsigned ties = 0u;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int e = 4 * q + k;
        const int x = add32((int)v[e], __shfl_sync(0xffffffffu, bias_lane, e));
        const i64 p2 = mad_wide_u32(quad_word(rnd, k), pow2lo,
                                    mul_wide_s32(x, __shfl_sync(0xffffffffu, mult_lane, e)));
        ties |= (unsigned)(__funnelshift_r(lo32(p2), (uint32_t)hi32(p2), lo) == 0xFFFFFFFFu) << k;
        y4[k] = hi32(p2) >> lo;
      }
      if (__any_sync(0xffffffffu, ties != 0u)) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int e = 4 * q + k;
          const int x = add32((int)v[e], __shfl_sync(0xffffffffu, bias_lane, e));
          const i64 prod = mul_wide_s32(x, __shfl_sync(0xffffffffu, mult_lane, e));
          if ((ties >> k) & 1u)
            y4[k] = (int)max((i64)-128, min((i64)128, sr_round(prod, sh, quad_word(rnd, k), sr.seed,
                                                               sr.stream, row, (uint32_t)(nb + e))));
        }
      }
      packed[q] = pack4(max(min(y4[0], 127), lower), max(min(y4[1], 127), lower), max(min(y4[2], 127), lower),
                        max(min(y4[3], 127), lower));
    }
  } else {
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    Philox4 rnd{0u, 0u, 0u, 0u};
    if (philox) rnd = sr_quad_k(keys, sr.stream, row, (uint32_t)((nb >> 2) + q));
    packed[q] = 0u;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int e = 4 * q + k;
      const int x = add32((int)v[e], __shfl_sync(0xffffffffu, bias_lane, e));
      const i64 prod = (i64)x * (i64)__shfl_sync(0xffffffffu, mult_lane, e);  // 32x32->64, exact
      i64 yv;
      if (p.shift < 0) {
        yv = shl64(prod, -p.shift);
      } else if (philox) {
        yv = sr_round(prod, p.shift, quad_word(rnd, k), sr.seed, sr.stream, row, (uint32_t)(nb + e));
      } else if (sr.mode == ECO_SR_NEAREST) {
        yv = sar64(add64(prod, half_nudge(p.shift)), p.shift);
      } else {
        i64 nud = 0;
        if (m < p.M && nb + e < p.N) {
          const i64 idx = (i64)m * sr.nudge_ld + nb + e;
          nud = sr.mode == ECO_SR_REPLAY32 ? (i64) static_cast<const int32_t*>(sr.nudge)[idx]
                                            : static_cast<const i64*>(sr.nudge)[idx];
        }
        yv = sar64(add64(prod, nud), p.shift);
      }
      int8_t y = sat8(yv);
      if (p.relu && y < 0) y = 0;
      packed[q] |= (uint32_t)(uint8_t)y << (8 * k);
    }
  }
  }
  if (nb + 32 <= p.N && (p.ldy & 15) == 0 && (reinterpret_cast<uintptr_t>(p.Y) & 15) == 0) {  // warp-uniform
    if (m >= p.M) return;
    int8_t* dst = p.Y + (i64)m * p.ldy + nb;
    *reinterpret_cast<int4*>(dst) = make_int4(packed[0], packed[1], packed[2], packed[3]);
    *reinterpret_cast<int4*>(dst + 16) = make_int4(packed[4], packed[5], packed[6], packed[7]);
  } else {
    const int m0 = m - lane;
    stage_store_rows8(stage, packed, lane, p.Y + (i64)m0 * p.ldy + nb, p.ldy, p.M - m0, p.N - nb);
  }
}

// fp32 dequant epilogue for one 32-column chunk of one row (Int8LinearFunc, layers.py:
// 49-52, 64, 67): fp32(acc) * scalar, then * col_scale[n], then + bias[n], each one IEEE
// fp32 operation like PyTorch's kernels; the scalar is the fp32 rounding of the double
// product sa * sb (a Python float, or a product of two, in the reference).
ECO_DEV void epi_store_dequant(const GemmParams& p, float scalar, const uint32_t (&v)[32], int m, int nb,
                               float cs_lane, float bias_lane, uint32_t* stage, int lane) {
  uint32_t o[32];
#pragma unroll
  for (int e = 0; e < 32; ++e) {  // every lane shuffles (row m may be past the end)
    float y = __fmul_rn(__int2float_rn((int)v[e]), scalar);
    if (p.col_scale) y = __fmul_rn(y, __shfl_sync(0xffffffffu, cs_lane, e));
    if (p.bias_f) y = __fadd_rn(y, __shfl_sync(0xffffffffu, bias_lane, e));
    o[e] = __float_as_uint(y);
  }
  if (nb + 32 <= p.N && (p.ldyf & 3) == 0 && (reinterpret_cast<uintptr_t>(p.Yf) & 15) == 0) {  // warp-uniform
    if (m >= p.M) return;
    uint32_t* dst = reinterpret_cast<uint32_t*>(p.Yf + (i64)m * p.ldyf + nb);
#pragma unroll
    for (int e = 0; e < 32; e += 4) *reinterpret_cast<uint4*>(dst + e) = make_uint4(o[e], o[e + 1], o[e + 2], o[e + 3]);
  } else {
    const int m0 = m - lane;
    stage_store_rows32(stage, o, lane, reinterpret_cast<uint32_t*>(p.Yf + (i64)m0 * p.ldyf + nb), p.ldyf, p.M - m0,
                       p.N - nb);
  }
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
  uint64_t* tfull = empty + S;   // [2] accumulator buffer ready for the epilogue
  uint64_t* tempty = tfull + 2;  // [2] accumulator buffer drained by the epilogue
  uint64_t* drain = tempty + 2;  // every issued MMA retired
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile uint32_t* abort_flag = tmem_slot + 1;  // a role timed out: everyone leaves

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_kb = (p.K + BK - 1) / BK;
  const int num_tiles = p.tiles_m * p.tiles_n;

  if (warp == 0 && lane == 0) {
    *abort_flag = 0u;
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiWarps);
    }
    mbar_init(drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
        int mb, nb;
        tile_coords(p, t, mb, nb);
        const int m0 = mb * BM, n0 = nb * BN;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % S;
          if (!mbar_wait(&empty[s], ((uint32_t)(it / S) & 1u) ^ 1u)) {
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
            for (int j = 0; j < BN / 128; ++j)
              tma_load_2d(b_dst + j * (128 * BK), &tmB, &full[s], n0 + 128 * j, k0);
          } else {
            tma_load_2d(b_dst, &tmB, &full[s], k0, n0);
          }
        }
      }
      // drain: every issued copy must land before the CTA can exit
      for (int k = it > S ? it - S : 0; k < it; ++k) mbar_wait(&full[k % S], (uint32_t)(k / S) & 1u);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_s8(BN, p.a_mn, p.b_mn);
      const uint32_t a_kstep = p.a_mn ? 32 * 128 : 32, b_kstep = p.b_mn ? 32 * 128 : 32;
      const uint32_t a_lbo = p.a_mn ? 128 * BK : 16, b_lbo = p.b_mn ? 128 * BK : 16;
      int it = 0, j = 0;
      for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x, ++j) {
        const int b = j & 1;
        if (!mbar_wait(&tempty[b], ((uint32_t)(j >> 1) & 1u) ^ 1u)) {
          *abort_flag = 1u;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + (uint32_t)(b * BN);
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % S;
          if (!mbar_wait(&full[s], (uint32_t)(it / S) & 1u)) {
            *abort_flag = 1u;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + s * C::A_BYTES), b_base = smem_u32(sB + s * C::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk)
            umma_s8(d_tmem, smem_desc(a_base + kk * a_kstep, a_lbo, 1024),
                    smem_desc(b_base + kk * b_kstep, b_lbo, 1024), idesc, (kb | kk) != 0);
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&tfull[b]);
      }
      umma_commit(drain);  // arrives once every MMA issued above has retired
      mbar_wait(drain, 0);
    }
  } else {
    const int e = warp - 2;
    const int q = warp & 3;           // TMEM lane quarter this warp may access
    const int half = e >> 2;          // which half of the BN columns
    uint32_t* stage = reinterpret_cast<uint32_t*>(smem + S * (C::A_BYTES + C::B_BYTES) + 1024) + e * 1024;
    constexpr int kChunks = BN / 64;  // 32-column chunks per half
    i64 amax = 0;
    int j = 0;
    PhiloxKeys keys;
    const eco_sr_t sr = sr_resolve(p.sr, p.keys, keys);
    float scalar = 0.0f;
    if (EPI == 2) {
      const double a = p.sa_dev ? __longlong_as_double(*p.sa_dev) : p.sa;
      const double b = p.sb_dev ? __longlong_as_double(*p.sb_dev) : p.sb;
      scalar = __double2float_rn(__dmul_rn(a, b));
    }
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++j) {
      const int b = j & 1;
      if (!mbar_wait(&tfull[b], (uint32_t)(j >> 1) & 1u) || *abort_flag) {
        *abort_flag = 1u;
        break;
      }
      tc_fence_after();
      int mb, nb_t;
      tile_coords(p, t, mb, nb_t);
      const int m = mb * BM + q * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < kChunks; ++c) {
        const int col = half * (BN / 2) + c * 32;
        const int nb = nb_t * BN + col;
        uint32_t v[32];
        tmem_ld32(tmem + (uint32_t)(b * BN + col) + ((uint32_t)(q * 32) << 16), v);
        if (nb >= p.N) continue;  // warp-uniform
        const int n_lane = nb + lane;
        if (EPI == 2) {
          const float cs = (p.col_scale && n_lane < p.N) ? __ldg(p.col_scale + n_lane) : 0.0f;
          const float bf = (p.bias_f && n_lane < p.N) ? __ldg(p.bias_f + n_lane) : 0.0f;
          epi_store_dequant(p, scalar, v, m, nb, cs, bf, stage, lane);
          continue;
        }
        const int bias_lane = (p.bias && n_lane < p.N) ? __ldg(p.bias + n_lane) : 0;
        if (EPI == 0) {
          epi_store_s32(p, v, m, nb, bias_lane, amax, stage, lane);
        } else {
          const int mult_lane = n_lane < p.N ? __ldg(p.mult + n_lane) : 0;
          epi_store_requant(p, sr, keys, v, m, nb, bias_lane, mult_lane, stage, lane);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
    }
    if (EPI == 0 && p.amax) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = max(amax, (i64)__shfl_xor_sync(0xffffffffu, amax, o));
      if (lane == 0 && amax > 0) atomicMax(p.amax, (int)amax);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS));
  }
}

// ------------------------------------------------------------ CTA-pair kernel
// The same GEMM with 256 x 256 output tiles computed by a cluster of two CTAs on
// neighbouring SMs (tcgen05 cta_group::2).  CTA r of the pair loads rows [128 r, 128 r +
// 128) of the A tile and columns [128 r, 128 r + 128) of the B tile into its own shared
// memory (no multicast: every TMA load fills only the issuing CTA's memory); the even
// CTA issues tcgen05.mma.cta_group::2 (M = 256, N = 256), which reads both CTAs' halves
// and leaves each CTA's 128 rows of the accumulator in that CTA's TMEM.  Per SM and
// K slice this moves 32 KB from L2 instead of 48 KB.  Barriers: both CTAs' loads
// complete on the even CTA's `full` barrier (cp.async.bulk.tensor .cta_group::2); the
// MMA's commits arrive on both CTAs' `empty` / `tfull` barriers (multicast commit);
// both CTAs' epilogue warps arrive on the even CTA's `tempty` barrier.  Every wait is
// bounded as in the one-CTA kernel; both CTAs meet at cluster barriers after the
// barrier setup and before TMEM is freed (the even CTA's MMAs read the odd CTA's memory).
constexpr int PBN = 256;                         // tile N (both CTAs)
constexpr int PHALF_B = (PBN / 2) * BK;          // B bytes per CTA and stage
constexpr int PS = 6;                            // stages
constexpr int PSMEM = PS * (BM * BK + PHALF_B) + 1024 + kStageBytes + 1024;

ECO_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
ECO_DEV uint32_t map_to_rank0(const void* p) {  // the same shared variable in CTA 0 of the cluster
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(r) : "r"(smem_u32(p)));
  return r;
}
ECO_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
ECO_DEV void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}
ECO_DEV void umma_s8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
ECO_DEV void umma_commit_pair(uint64_t* bar) {  // arrive on `bar` in both CTAs of the pair
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}
ECO_DEV void umma_commit_pair_local(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
ECO_DEV void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
// Instruction descriptor of the pair MMA: as idesc_s8 with M = 256.
ECO_DEV uint32_t idesc_s8_pair(int n, int a_mn, int b_mn) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_s8_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const GemmParams p) {
  constexpr int S = PS;
  constexpr int A_BYTES = BM * BK, B_BYTES = PHALF_B;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + S * B_BYTES);  // used in CTA 0: both CTAs' bytes
  uint64_t* empty = full + S;                                        // each CTA: its stage is free
  uint64_t* tfull = empty + S;                                       // each CTA: accumulator ready
  uint64_t* tempty = tfull + 2;                                      // CTA 0: both CTAs drained it
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
  const int num_kb = (p.K + BK - 1) / BK;
  const int num_tiles = p.tiles_m * p.tiles_n;

  if (warp == 0 && lane == 0) {
    *abort_flag = 0u;
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * kEpiWarps);
    }
    mbar_init(drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(2 * PBN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before either CTA signals the other's
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int t = pair; t < num_tiles && !*abort_flag; t += n_pairs) {
        int mb, nb;
        tile_coords(p, t, mb, nb);
        const int m0 = mb * 2 * BM + (int)rank * BM, n0 = nb * PBN + (int)rank * (PBN / 2);
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % S;
          if (!mbar_wait(&empty[s], ((uint32_t)(it / S) & 1u) ^ 1u)) {
            *abort_flag = 1u;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * (A_BYTES + B_BYTES));
          const uint32_t bar = map_to_rank0(&full[s]);
          const int k0 = kb * BK;
          uint8_t* a_dst = sA + s * A_BYTES;
          uint8_t* b_dst = sB + s * B_BYTES;
          if (p.a_mn)
            tma_load_2d_pair(a_dst, &tmA, bar, m0, k0);
          else
            tma_load_2d_pair(a_dst, &tmA, bar, k0, m0);
          if (p.b_mn)
            tma_load_2d_pair(b_dst, &tmB, bar, n0, k0);
          else
            tma_load_2d_pair(b_dst, &tmB, bar, k0, n0);
        }
      }
      // drain: the MMAs released (consumed) the last stages this CTA filled
      for (int k = it > S ? it - S : 0; k < it; ++k) mbar_wait(&empty[k % S], (uint32_t)(k / S) & 1u);
    }
  } else if (warp == 1) {
    if (rank == 0 && lane == 0) {
      const uint32_t idesc = idesc_s8_pair(PBN, p.a_mn, p.b_mn);
      const uint32_t a_kstep = p.a_mn ? 32 * 128 : 32, b_kstep = p.b_mn ? 32 * 128 : 32;
      const uint32_t a_lbo = p.a_mn ? 128 * BK : 16, b_lbo = p.b_mn ? 128 * BK : 16;
      int it = 0, j = 0;
      for (int t = pair; t < num_tiles && !*abort_flag; t += n_pairs, ++j) {
        const int b = j & 1;
        if (!mbar_wait(&tempty[b], ((uint32_t)(j >> 1) & 1u) ^ 1u)) {
          *abort_flag = 1u;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + (uint32_t)(b * PBN);
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % S;
          if (!mbar_wait(&full[s], (uint32_t)(it / S) & 1u)) {
            *abort_flag = 1u;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + s * A_BYTES), b_base = smem_u32(sB + s * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk)
            umma_s8_pair(d_tmem, smem_desc(a_base + kk * a_kstep, a_lbo, 1024),
                         smem_desc(b_base + kk * b_kstep, b_lbo, 1024), idesc, (kb | kk) != 0);
          umma_commit_pair(&empty[s]);
        }
        if (!ok) break;
        umma_commit_pair(&tfull[b]);
      }
      umma_commit_pair_local(drain);  // arrives once every MMA issued above has retired
      mbar_wait(drain, 0);
    }
  } else {
    const int e = warp - 2;
    const int q = warp & 3;
    const int half = e >> 2;
    constexpr int kChunks = PBN / 64;
    uint32_t* stage = reinterpret_cast<uint32_t*>(smem + S * (A_BYTES + B_BYTES) + 1024) + e * 1024;
    PhiloxKeys keys;
    const eco_sr_t sr = sr_resolve(p.sr, p.keys, keys);
    float scalar = 0.0f;
    if (EPI == 2) {
      const double a = p.sa_dev ? __longlong_as_double(*p.sa_dev) : p.sa;
      const double b = p.sb_dev ? __longlong_as_double(*p.sb_dev) : p.sb;
      scalar = __double2float_rn(__dmul_rn(a, b));
    }
    const uint32_t tempty0 = map_to_rank0(&tempty[0]), tempty1 = map_to_rank0(&tempty[1]);
    i64 amax = 0;
    int j = 0;
    for (int t = pair; t < num_tiles; t += n_pairs, ++j) {
      const int b = j & 1;
      if (!mbar_wait(&tfull[b], (uint32_t)(j >> 1) & 1u) || *abort_flag) {
        *abort_flag = 1u;
        break;
      }
      tc_fence_after();
      int mb, nb_t;
      tile_coords(p, t, mb, nb_t);
      const int m = mb * 2 * BM + (int)rank * BM + q * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < kChunks; ++c) {
        const int col = half * (PBN / 2) + c * 32;
        const int nb = nb_t * PBN + col;
        uint32_t v[32];
        tmem_ld32(tmem + (uint32_t)(b * PBN + col) + ((uint32_t)(q * 32) << 16), v);
        if (nb >= p.N) continue;  // warp-uniform
        const int n_lane = nb + lane;
        if (EPI == 2) {
          const float cs = (p.col_scale && n_lane < p.N) ? __ldg(p.col_scale + n_lane) : 0.0f;
          const float bf = (p.bias_f && n_lane < p.N) ? __ldg(p.bias_f + n_lane) : 0.0f;
          epi_store_dequant(p, scalar, v, m, nb, cs, bf, stage, lane);
          continue;
        }
        const int bias_lane = (p.bias && n_lane < p.N) ? __ldg(p.bias + n_lane) : 0;
        if (EPI == 0) {
          epi_store_s32(p, v, m, nb, bias_lane, amax, stage, lane);
        } else {
          const int mult_lane = n_lane < p.N ? __ldg(p.mult + n_lane) : 0;
          epi_store_requant(p, sr, keys, v, m, nb, bias_lane, mult_lane, stage, lane);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(b ? tempty1 : tempty0);
    }
    if (EPI == 0 && p.amax) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = max(amax, (i64)__shfl_xor_sync(0xffffffffu, amax, o));
      if (lane == 0 && amax > 0) atomicMax(p.amax, (int)amax);
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the even CTA's MMAs are done with the odd CTA's memory
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * PBN));
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

// Upper bound on the persistent GEMM's CTAs (0 = one per SM).  A data-parallel
// caller lowers it so that NCCL's kernels find free SMs and overlap the GEMMs.
int g_gemm_sm_limit = 0;

// Whether a launch's epilogue can take the staged store path (an output whose rows are not
// 16-byte aligned, or a width that leaves a partial 32-column chunk).  Launches that never
// stage leave its 32 KB of shared memory out, so that the small kernels of other streams
// (requants, column sums) still fit on the SMs beside the persistent GEMM.
bool staging_needed(const GemmParams& p, int epi) {
  if (p.N % 32 != 0) return true;
  if (epi == 0) return (p.ldc & 3) != 0 || (reinterpret_cast<uintptr_t>(p.C) & 15) != 0;
  if (epi == 1) return (p.ldy & 15) != 0 || (reinterpret_cast<uintptr_t>(p.Y) & 15) != 0;
  return (p.ldyf & 3) != 0 || (reinterpret_cast<uintptr_t>(p.Yf) & 15) != 0;
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
  GemmParams q = p;
  q.tiles_m = (p.M + BM - 1) / BM;
  q.tiles_n = (p.N + BN - 1) / BN;
  const int tiles = q.tiles_m * q.tiles_n;
  int ctas = eco_num_sms();  // persistent: at most one CTA per SM
  if (g_gemm_sm_limit > 0) ctas = std::min(ctas, g_gemm_sm_limit);
  const int grid = std::min(tiles, ctas);
  kern<<<grid, kThreads, Cfg<BN>::SMEM - (staging_needed(p, EPI) ? 0 : kStageBytes), s>>>(ta, tb, q);
  return eco_launch_check("gemm_s8_kernel");
}

// CTA pairs for the large GEMMs: on unless ECO_GEMM_PAIRS=0 in the environment (read once;
// the one-CTA kernel then runs every shape).
bool pairs_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("ECO_GEMM_PAIRS");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

template <int EPI>
int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, cudaStream_t s) {
  auto kern = gemm_s8_pair_kernel<EPI>;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PSMEM) != cudaSuccess)
      return eco_launch_check("gemm (pairs): cudaFuncSetAttribute");
    attr_set = true;
  }
  GemmParams q = p;
  q.tiles_m = (p.M + 2 * BM - 1) / (2 * BM);
  q.tiles_n = (p.N + PBN - 1) / PBN;
  const int tiles = q.tiles_m * q.tiles_n;
  int ctas = eco_num_sms();
  if (g_gemm_sm_limit > 0) ctas = std::min(ctas, g_gemm_sm_limit);
  const int pairs = std::max(1, std::min(tiles, ctas / 2));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * pairs));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = PSMEM - (staging_needed(p, EPI) ? 0 : kStageBytes);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, ta, tb, q) != cudaSuccess) return eco_launch_check("gemm_s8_pair_kernel launch");
  return eco_launch_check("gemm_s8_pair_kernel");
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
  const bool pair = BN == 256 && M > BM && pairs_enabled() &&
                    (g_gemm_sm_limit == 0 || g_gemm_sm_limit >= 2) && eco_num_sms() >= 2;
  CUtensorMap ta, tb;
  if (pair) {  // each CTA of a pair loads a 128-row box of A and a 128-column box of B
    if (int rc = a_layout ? make_tmap(&ta, A, M, K, lda, 128, BK) : make_tmap(&ta, A, K, M, lda, BK, BM)) return rc;
    if (int rc = b_layout ? make_tmap(&tb, B, N, K, ldb, 128, BK) : make_tmap(&tb, B, K, N, ldb, BK, PBN / 2))
      return rc;
    return epi == 2 ? launch_pair<2>(ta, tb, p, s) : epi ? launch_pair<1>(ta, tb, p, s) : launch_pair<0>(ta, tb, p, s);
  }
  if (int rc = a_layout ? make_tmap(&ta, A, M, K, lda, 128, BK) : make_tmap(&ta, A, K, M, lda, BK, BM)) return rc;
  if (int rc = b_layout ? make_tmap(&tb, B, N, K, ldb, 128, BK) : make_tmap(&tb, B, K, N, ldb, BK, BN)) return rc;
  if (BN == 128)
    return epi == 2 ? launch<128, 2>(ta, tb, p, s) : epi ? launch<128, 1>(ta, tb, p, s) : launch<128, 0>(ta, tb, p, s);
  return epi == 2 ? launch<256, 2>(ta, tb, p, s) : epi ? launch<256, 1>(ta, tb, p, s) : launch<256, 0>(ta, tb, p, s);
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
  p.keys = philox_keys(sr.mode == ECO_SR_PHILOX ? sr.seed : 0);
  p.Y = Y;
  p.ldy = ldy;
  return gemm_common(A, lda, a_layout, B, ldb, b_layout, M, N, K, p, 1, eco_stream(stream), "eco_gemm_s8_requant");
}

extern "C" int eco_gemm_s8_dequant(const int8_t* A, int64_t lda, int a_layout, const int8_t* B, int64_t ldb,
                                   int b_layout, int64_t M, int64_t N, int64_t K, const int64_t* sa_dev, double sa,
                                   const int64_t* sb_dev, double sb, const float* col_scale, const float* bias,
                                   float* Y, int64_t ldy, eco_stream_t stream) {
  ECO_REQUIRE(Y && ldy >= N, ECO_ERR_ARG, "eco_gemm_s8_dequant: bad output");
  GemmParams p{};
  p.Yf = Y;
  p.ldyf = ldy;
  p.sa_dev = sa_dev;
  p.sb_dev = sb_dev;
  p.sa = sa;
  p.sb = sb;
  p.col_scale = col_scale;
  p.bias_f = bias;
  return gemm_common(A, lda, a_layout, B, ldb, b_layout, M, N, K, p, 2, eco_stream(stream), "eco_gemm_s8_dequant");
}

extern "C" int eco_set_gemm_sm_limit(int max_ctas) {
  ECO_REQUIRE(max_ctas >= 0, ECO_ERR_ARG, "eco_set_gemm_sm_limit: negative limit");
  g_gemm_sm_limit = max_ctas;
  return ECO_OK;
}

int eco_peer_errors_take(unsigned* out);  // peer.cu

extern "C" int eco_read_device_errors(uint32_t* flags) {
  ECO_REQUIRE(flags, ECO_ERR_ARG, "eco_read_device_errors: null output");
  unsigned v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_eco_device_errors, sizeof(v)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_eco_device_errors, &zero, sizeof(zero)) != cudaSuccess)
    return eco_launch_check("eco_read_device_errors");
  unsigned peer = 0;
  if (int rc = eco_peer_errors_take(&peer)) return rc;
  *flags = v | peer;
  return ECO_OK;
}
