// Data-parallel exchange over NVLink peer memory (one process per GPU).
//
// The buffers are allocated symmetrically on every rank and mapped into each
// process; a rank reaches a peer's copy through that peer's pointer.  Pushes are
// plain 16-byte stores into the peers' buffers (the SMs drive NVLink directly,
// without the per-channel copy loop of a collective library), and completion is
// published through per-rank flag words with release/acquire at system scope.
// Every wait is bounded: on expiry it records ECO_FLAG_WAIT_TIMEOUT in a sticky
// device word (read by eco_read_device_errors) and returns.
#include "abi.cuh"
#include "common.cuh"

#include <algorithm>
#include <type_traits>

namespace {

__device__ unsigned g_peer_errors;  // sticky flags of the bounded peer waits

constexpr unsigned long long kPeerWaitNs = 5ull * 1000 * 1000 * 1000;  // 5 s

struct PushArgs {
  const int8_t* src;
  int64_t ld_src, rows, cols;
  int8_t* dst[ECO_MAX_PEERS];
  int64_t ld_dst, dst_row0;
  int n, split;
  // optional completion signal (eco_peer_push_signal_s8): the last CTA publishes
  // `epoch` in entry (slot, rank) of every rank's flags
  int64_t* flags[ECO_MAX_PEERS];
  int n_ranks, rank, slot;
  int64_t epoch;
  const int64_t* epoch_dev;  // nullable: the epoch, read when the kernel runs
  unsigned* ticket;  // zero between launches; the last CTA resets it
};

// Broadcast: every destination receives all of src at rows dst_row0 + r.
// Split: destination p receives columns [p * c, (p + 1) * c), c = cols / n.
// A block copies kRows rows at a time (rows blockIdx.x + i * gridDim.x), each
// thread one unit of every row: all kRows loads are in flight before the stores,
// so a few CTAs keep enough bytes moving to fill NVLink.  VEC: 16-byte units
// (cols, c, ld_src, ld_dst multiples of 16 and aligned bases), else bytes.
ECO_DEV void st_release_sys(int64_t* p, int64_t v) {
  asm volatile("st.release.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

constexpr int kPushThreads = 512;
constexpr int kRows = 8;

template <bool VEC>
__global__ void __launch_bounds__(kPushThreads) peer_push_kernel(const __grid_constant__ PushArgs A) {
  typedef typename std::conditional<VEC, int4, int8_t>::type U;
  constexpr int unit = VEC ? 16 : 1;
  const int per_row = (int)(A.cols / unit);
  const int c_units = (int)((A.split ? A.cols / A.n : A.cols) / unit);
  for (int64_t r0 = blockIdx.x; r0 < A.rows; r0 += (int64_t)gridDim.x * kRows) {
    for (int j = threadIdx.x; j < per_row; j += kPushThreads) {
      U v[kRows];
#pragma unroll
      for (int i = 0; i < kRows; ++i) {
        const int64_t r = r0 + (int64_t)i * gridDim.x;
        if (r < A.rows) v[i] = reinterpret_cast<const U*>(A.src + r * A.ld_src)[j];
      }
      const int p0 = A.split ? j / c_units : 0;
      const int jd = j - p0 * c_units;
#pragma unroll
      for (int i = 0; i < kRows; ++i) {
        const int64_t r = r0 + (int64_t)i * gridDim.x;
        if (r >= A.rows) break;
        const int64_t drow = (A.dst_row0 + r) * A.ld_dst;
        if (A.split) {
          reinterpret_cast<U*>(A.dst[p0] + drow)[jd] = v[i];
        } else {
#pragma unroll 1
          for (int p = 0; p < A.n; ++p) reinterpret_cast<U*>(A.dst[p] + drow)[j] = v[i];
        }
      }
    }
  }
  if (A.ticket) {
    __threadfence_system();  // this thread's stores are visible to every GPU
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(A.ticket, 1u) == gridDim.x - 1) {  // every CTA has fenced
      *A.ticket = 0u;
      asm volatile("fence.sc.sys;" ::: "memory");
      const int64_t epoch = A.epoch_dev ? *A.epoch_dev : A.epoch;
      for (int p = 0; p < A.n_ranks; ++p)
        st_release_sys(A.flags[p] + (int64_t)A.slot * ECO_MAX_PEERS + A.rank, epoch);
    }
  }
}

struct FlagArgs {
  int64_t* peer_flags[ECO_MAX_PEERS];
};
ECO_DEV int64_t ld_acquire_sys(const int64_t* p) {
  int64_t v;
  asm volatile("ld.acquire.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
ECO_DEV unsigned long long peer_clock() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Thread p publishes `epoch` in slot (slot, rank) of rank p's flag array, after
// everything this stream did before (the previous kernels' stores included).
__global__ void peer_signal_kernel(const __grid_constant__ FlagArgs F, int n, int rank, int slot, int64_t epoch,
                                   const int64_t* epoch_dev) {
  const int p = threadIdx.x;
  if (p >= n) return;
  if (epoch_dev) epoch = *epoch_dev;
  asm volatile("fence.sc.sys;" ::: "memory");
  st_release_sys(F.peer_flags[p] + (int64_t)slot * ECO_MAX_PEERS + rank, epoch);
}

// Thread p waits until rank p's entry of `slot` in this rank's flags reaches `epoch`.
__global__ void peer_wait_kernel(const int64_t* flags, int n, int slot, int64_t epoch, const int64_t* epoch_dev,
                                 unsigned long long limit_ns) {
  const int p = threadIdx.x;
  if (p >= n) return;
  if (epoch_dev) epoch = *epoch_dev;
  const int64_t* f = flags + (int64_t)slot * ECO_MAX_PEERS + p;
  if (ld_acquire_sys(f) >= epoch) return;
  const unsigned long long t0 = peer_clock();
  while (ld_acquire_sys(f) < epoch) {
    if (peer_clock() - t0 > limit_ns) {
      atomicOr(&g_peer_errors, ECO_FLAG_WAIT_TIMEOUT);
      return;
    }
    __nanosleep(200);
  }
}

// All-reduce (MAX or SUM) of a short int64 vector through the ranks' exchange
// buffers: every rank stores its values into area (epoch & 1, rank) of every rank's
// buffer, fences, publishes `epoch` in flag entry (slot, rank) everywhere, waits for
// the n entries of its own slot, and reduces the n areas of its own buffer.  Two
// areas alternate: a rank can only write an area again after a later call has seen
// every rank's flag, i.e. after every rank finished reading it.
struct AllreduceArgs {
  const void* src;
  int src_bits, count, stride, op, n, rank, slot;
  int64_t epoch;
  const int64_t* epoch_dev;  // nullable: the epoch, read when the kernel runs
  int64_t* bufs[ECO_MAX_PEERS];
  int64_t* flags[ECO_MAX_PEERS];
  const int64_t* own_buf;
  const int64_t* own_flags;
  int64_t* out;
  unsigned long long limit_ns;
};

ECO_DEV int64_t ld_relaxed_sys(const int64_t* p) {
  int64_t v;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(256) peer_allreduce_kernel(const __grid_constant__ AllreduceArgs A) {
  const int64_t epoch = A.epoch_dev ? *A.epoch_dev : A.epoch;
  const int par = (int)(epoch & 1);
  for (int e = threadIdx.x; e < A.count; e += blockDim.x) {
    const int64_t v = A.src_bits == 32 ? (int64_t) static_cast<const int32_t*>(A.src)[e]
                                       : static_cast<const int64_t*>(A.src)[e];
    for (int p = 0; p < A.n; ++p) A.bufs[p][((int64_t)par * A.n + A.rank) * A.stride + e] = v;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < A.n) {
    asm volatile("fence.sc.sys;" ::: "memory");
    st_release_sys(A.flags[threadIdx.x] + (int64_t)A.slot * ECO_MAX_PEERS + A.rank, epoch);
  }
  __shared__ int s_late;
  if (threadIdx.x == 0) s_late = 0;
  __syncthreads();
  if (threadIdx.x < A.n) {
    const int64_t* f = A.own_flags + (int64_t)A.slot * ECO_MAX_PEERS + threadIdx.x;
    if (ld_acquire_sys(f) < epoch) {
      const unsigned long long t0 = peer_clock();
      while (ld_acquire_sys(f) < epoch) {
        if (peer_clock() - t0 > A.limit_ns) {
          atomicOr(&g_peer_errors, ECO_FLAG_WAIT_TIMEOUT);
          s_late = 1;
          break;
        }
        __nanosleep(200);
      }
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < A.count; e += blockDim.x) {
    int64_t acc = ld_relaxed_sys(A.own_buf + (int64_t)par * A.n * A.stride + e);
    for (int r = 1; r < A.n; ++r) {
      const int64_t v = ld_relaxed_sys(A.own_buf + ((int64_t)par * A.n + r) * A.stride + e);
      acc = A.op == 0 ? (v > acc ? v : acc) : (int64_t)((uint64_t)acc + (uint64_t)v);
    }
    A.out[e] = s_late ? 0 : acc;
  }
}

}  // namespace

// Sticky flags of the peer waits, cleared by the read (used by eco_read_device_errors).
int eco_peer_errors_take(unsigned* out) {
  unsigned zero = 0;
  if (cudaMemcpyFromSymbol(out, g_peer_errors, sizeof(*out)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_peer_errors, &zero, sizeof(zero)) != cudaSuccess)
    return eco_launch_check("eco_read_device_errors (peer)");
  return ECO_OK;
}

static int peer_push(const int8_t* src, int64_t ld_src, int64_t rows, int64_t cols, int8_t* const* dst, int n_dst,
                     int64_t ld_dst, int64_t dst_row0, int split, int ctas, int64_t* const* peer_flags, int n_ranks,
                     int rank, int slot, int64_t epoch, const int64_t* epoch_dev, unsigned* ticket,
                     eco_stream_t stream) {
  ECO_REQUIRE(src && dst && rows >= 0 && cols >= 0 && ld_src >= cols && dst_row0 >= 0, ECO_ERR_ARG,
              "eco_peer_push_s8: bad arguments");
  ECO_REQUIRE(n_dst >= 1 && n_dst <= ECO_MAX_PEERS, ECO_ERR_ARG, "eco_peer_push_s8: 1..%d destinations",
              ECO_MAX_PEERS);
  ECO_REQUIRE(!split || cols % n_dst == 0, ECO_ERR_ARG, "eco_peer_push_s8: split needs cols divisible by n_dst");
  ECO_REQUIRE(ld_dst >= (split ? cols / n_dst : cols), ECO_ERR_ARG, "eco_peer_push_s8: ld_dst too small");
  if ((rows == 0 || cols == 0) && !ticket) return ECO_OK;
  ECO_REQUIRE(rows > 0 && cols > 0, ECO_ERR_ARG, "eco_peer_push_signal_s8: empty matrix");
  PushArgs A{};
  A.src = src;
  A.ld_src = ld_src;
  A.rows = rows;
  A.cols = cols;
  A.ld_dst = ld_dst;
  A.dst_row0 = dst_row0;
  A.n = n_dst;
  A.split = split;
  bool vec = cols % 16 == 0 && ld_src % 16 == 0 && ld_dst % 16 == 0 && eco_aligned16(src) &&
             (!split || (cols / n_dst) % 16 == 0);
  for (int p = 0; p < ECO_MAX_PEERS; ++p) {
    A.dst[p] = p < n_dst ? dst[p] : nullptr;
    if (p < n_dst) {
      ECO_REQUIRE(dst[p], ECO_ERR_ARG, "eco_peer_push_s8: null destination %d", p);
      vec = vec && eco_aligned16(dst[p]);
    }
  }
  ECO_REQUIRE(cols < (1ll << 31), ECO_ERR_ARG, "eco_peer_push_s8: too many columns");
  A.ticket = ticket;
  if (ticket) {
    ECO_REQUIRE(peer_flags && n_ranks >= 1 && n_ranks <= ECO_MAX_PEERS && rank >= 0 && rank < n_ranks &&
                    slot >= 0 && (epoch > 0 || epoch_dev),
                ECO_ERR_ARG, "eco_peer_push_signal_s8: bad signal arguments");
    for (int p = 0; p < n_ranks; ++p) {
      ECO_REQUIRE(peer_flags[p], ECO_ERR_ARG, "eco_peer_push_signal_s8: null flag array %d", p);
      A.flags[p] = peer_flags[p];
    }
    A.n_ranks = n_ranks;
    A.rank = rank;
    A.slot = slot;
    A.epoch = epoch;
    A.epoch_dev = epoch_dev;
  }
  const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(rows, ctas > 0 ? ctas : eco_num_sms()));
  if (vec)
    peer_push_kernel<true><<<(unsigned)grid, kPushThreads, 0, eco_stream(stream)>>>(A);
  else
    peer_push_kernel<false><<<(unsigned)grid, kPushThreads, 0, eco_stream(stream)>>>(A);
  return eco_launch_check("eco_peer_push_s8");
}

extern "C" int eco_peer_push_s8(const int8_t* src, int64_t ld_src, int64_t rows, int64_t cols, int8_t* const* dst,
                                int n_dst, int64_t ld_dst, int64_t dst_row0, int split, int ctas,
                                eco_stream_t stream) {
  return peer_push(src, ld_src, rows, cols, dst, n_dst, ld_dst, dst_row0, split, ctas, nullptr, 0, 0, 0, 0, nullptr,
                   nullptr, stream);
}

extern "C" int eco_peer_push_signal_s8(const int8_t* src, int64_t ld_src, int64_t rows, int64_t cols,
                                       int8_t* const* dst, int n_dst, int64_t ld_dst, int64_t dst_row0, int split,
                                       int ctas, int64_t* const* peer_flags, int n_ranks, int rank, int slot,
                                       int64_t epoch, const int64_t* epoch_dev, uint32_t* ticket,
                                       eco_stream_t stream) {
  ECO_REQUIRE(ticket, ECO_ERR_ARG, "eco_peer_push_signal_s8: ticket word required");
  return peer_push(src, ld_src, rows, cols, dst, n_dst, ld_dst, dst_row0, split, ctas, peer_flags, n_ranks, rank,
                   slot, epoch, epoch_dev, ticket, stream);
}

extern "C" int eco_peer_signal(int64_t* const* peer_flags, int n, int rank, int slot, int64_t epoch,
                               const int64_t* epoch_dev, eco_stream_t stream) {
  ECO_REQUIRE(peer_flags && n >= 1 && n <= ECO_MAX_PEERS && rank >= 0 && rank < n && slot >= 0 &&
                  (epoch > 0 || epoch_dev),
              ECO_ERR_ARG, "eco_peer_signal: bad arguments");
  FlagArgs F;
  for (int p = 0; p < ECO_MAX_PEERS; ++p) {
    F.peer_flags[p] = p < n ? peer_flags[p] : nullptr;
    if (p < n) ECO_REQUIRE(peer_flags[p], ECO_ERR_ARG, "eco_peer_signal: null flag array %d", p);
  }
  peer_signal_kernel<<<1, 32, 0, eco_stream(stream)>>>(F, n, rank, slot, epoch, epoch_dev);
  return eco_launch_check("eco_peer_signal");
}

extern "C" int eco_peer_wait(const int64_t* flags, int n, int slot, int64_t epoch, const int64_t* epoch_dev,
                             int64_t timeout_us, eco_stream_t stream) {
  ECO_REQUIRE(flags && n >= 1 && n <= ECO_MAX_PEERS && slot >= 0 && (epoch > 0 || epoch_dev) && timeout_us >= 0,
              ECO_ERR_ARG,
              "eco_peer_wait: bad arguments");
  const unsigned long long limit = timeout_us > 0 ? std::min<unsigned long long>((unsigned long long)timeout_us * 1000ull,
                                                                                kPeerWaitNs)
                                                  : kPeerWaitNs;
  peer_wait_kernel<<<1, 32, 0, eco_stream(stream)>>>(flags, n, slot, epoch, epoch_dev, limit);
  return eco_launch_check("eco_peer_wait");
}

extern "C" int eco_peer_allreduce_i64(const void* src, int src_bits, int count, int op, int64_t* const* bufs,
                                      int stride, const int64_t* own_buf, int64_t* const* peer_flags,
                                      const int64_t* own_flags, int n, int rank, int slot, int64_t epoch,
                                      const int64_t* epoch_dev, int64_t* out, eco_stream_t stream) {
  ECO_REQUIRE(src && bufs && own_buf && peer_flags && own_flags && out && (src_bits == 32 || src_bits == 64) &&
                  count >= 1 && stride >= count && (op == 0 || op == 1) && n >= 1 && n <= ECO_MAX_PEERS &&
                  rank >= 0 && rank < n && slot >= 0 && (epoch > 0 || epoch_dev),
              ECO_ERR_ARG, "eco_peer_allreduce_i64: bad arguments");
  AllreduceArgs A{};
  A.src = src;
  A.src_bits = src_bits;
  A.count = count;
  A.stride = stride;
  A.op = op;
  A.n = n;
  A.rank = rank;
  A.slot = slot;
  A.epoch = epoch;
  A.epoch_dev = epoch_dev;
  for (int p = 0; p < n; ++p) {
    ECO_REQUIRE(bufs[p] && peer_flags[p], ECO_ERR_ARG, "eco_peer_allreduce_i64: null buffer %d", p);
    A.bufs[p] = bufs[p];
    A.flags[p] = peer_flags[p];
  }
  A.own_buf = own_buf;
  A.own_flags = own_flags;
  A.out = out;
  A.limit_ns = kPeerWaitNs;
  peer_allreduce_kernel<<<1, 256, 0, eco_stream(stream)>>>(A);
  return eco_launch_check("eco_peer_allreduce_i64");
}
