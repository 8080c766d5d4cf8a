/*
 * ecoint8_b200.h — C ABI of the B200 (sm_100a) library behind the ecoint8
 * strict int8 training path.
 *
 * Every entry point takes plain device pointers, sizes and a stream, returns
 * an int status (ECO_OK or a negative ECO_ERR_*), never synchronises the
 * host, and never allocates device memory: outputs, scratch words and
 * optimizer state are owned by the caller.  Work is enqueued on `stream`
 * (a cudaStream_t; NULL = the legacy default stream).  After a failure,
 * eco_last_error() returns a message for the calling thread.
 *
 * Process-wide state (everything else is per call):
 *   - the GEMM CTA cap set by eco_set_gemm_sm_limit (default 0: one CTA per SM);
 *   - a sticky device error word per GPU, set by bounded device waits that gave
 *     up and read-and-cleared by eco_read_device_errors;
 *   - the 32 MiB file-scope relayout buffer of eco_gemm_s8s32_noalloc (and its
 *     cached device address, one per device);
 *   - the IPC mappings a caller opened with eco_ipc_open, until eco_ipc_close.
 *
 * Matrices are row-major with an explicit leading dimension in elements.
 * Stochastic rounding (SR) draws follow the caller's eco_sr_t:
 *   ECO_SR_NEAREST  round half up: nudge = 2^(shift-1)      (fixedpoint.py:72-73)
 *   ECO_SR_PHILOX   nudge = low `shift` bits of the library's Philox4x32-10
 *                   word for (seed, stream, row_base + row, col)
 *   ECO_SR_REPLAY32 / ECO_SR_REPLAY64
 *                   nudge[row * nudge_ld + col], an int32 / int64 tensor such
 *                   as the reference's own torch.randint draw (fixedpoint.py:40-49)
 * Citations name files of the reference package ecoint8 v0.4.9.
 */
#ifndef ECOINT8_B200_H
#define ECOINT8_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ECO_API __attribute__((visibility("default")))
#else
#define ECO_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define ECO_ABI_VERSION 4

enum {
  ECO_OK = 0,
  ECO_ERR_ARG = -1,         /* bad pointer / size / layout argument */
  ECO_ERR_MISALIGNED = -2,  /* a TMA operand is not 16-byte aligned (address or leading dim) */
  ECO_ERR_ARCH = -3,        /* device is not sm_100 */
  ECO_ERR_LAUNCH = -4,      /* CUDA launch / driver error */
  ECO_ERR_RANGE = -5,       /* a requant shift outside [-63, 62] */
};

/* ECO_SR_REPLAY_F32: fp32 uniforms in [0, 1) at nudge[row * nudge_ld + col] (a
 * torch.rand_like draw, quant.py:25); only the loss-boundary entry point takes it.
 * ECO_SR_PHILOX_DEV: ECO_SR_PHILOX with the key read from device memory when the
 * kernel runs -- the uint64 word at `nudge` (8-byte aligned) instead of `seed` -- so a
 * captured CUDA graph replays the launch with whatever key that word holds then.
 * The requant, fused-GEMM and loss-boundary entry points take it. */
enum {
  ECO_SR_NEAREST = 0,
  ECO_SR_PHILOX = 1,
  ECO_SR_REPLAY32 = 2,
  ECO_SR_REPLAY64 = 3,
  ECO_SR_REPLAY_F32 = 4,
  ECO_SR_PHILOX_DEV = 5,
};

typedef void* eco_stream_t; /* cudaStream_t */

typedef struct {
  int32_t mode;        /* ECO_SR_* */
  int32_t pad_;
  const void* nudge;   /* replay modes: [rows, nudge_ld] int32 or int64 */
  int64_t nudge_ld;
  uint64_t seed;       /* Philox key */
  uint64_t stream;     /* Philox site id (unique per draw site) */
  int64_t row_base;    /* global row index of local row 0 (data parallel shards) */
} eco_sr_t;

ECO_API int eco_abi_version(void);
ECO_API const char* eco_last_error(void);
/* 1 when `device` is an sm_100 (B200-class) GPU, 0 otherwise, <0 on error. */
ECO_API int eco_device_supported(int device);

/* ---------------------------------------------------------------- GEMMs --
 * C[M,N] = A[M,K] . B[K,N] on int8 tcgen05 tensor cores, int32 accumulate.
 * a_layout 0: A stored [M, lda] (K contiguous);  1: A stored [K, lda] (M contiguous)
 * b_layout 0: B stored [N, ldb] (K contiguous);  1: B stored [K, ldb] (N contiguous)
 * Operands need 16-byte aligned base addresses and leading dims (ECO_ERR_MISALIGNED).
 */

/* C = A.B (+ bias[n], int32 wrap-around; bias nullable).  `amax` (nullable,
 * device int32) is overwritten with max |C|.
 * Replaces torch._int_mm at ecoint8/strict/ilayer.py:40-54 (called from :117,
 * :135, :152, :159), the `acc + b_acc` of :118-119 and the int_amax reductions
 * at :121, :153, :161. */
ECO_API int eco_gemm_s8s32(const int8_t* A, int64_t lda, int a_layout, const int8_t* B, int64_t ldb,
                   int b_layout, int64_t M, int64_t N, int64_t K, const int32_t* bias, int32_t* C,
                   int64_t ldc, int32_t* amax, eco_stream_t stream);

/* eco_gemm_s8s32 for callers that cannot allocate device memory (code running
 * under stream capture, runtimes that plan every buffer ahead, plain C hosts
 * without a caching allocator).  A and B need not follow the 16-byte rule: an
 * operand that breaks it is copied into a 32 MiB buffer the library keeps in
 * file-scope device memory (held by every GPU that loads it, until exit),
 * never into memory the call allocates.  A relayout larger than 32 MiB is
 * rejected with ECO_ERR_ARG.  All calls share that buffer, so calls that
 * overlap on the GPU race; the first call on a device looks the buffer up and
 * should come before any stream capture.  The looked-up address stays cached for
 * the lifetime of the device's primary context: after cudaDeviceReset on a device,
 * do not call this entry point on it again in that process.  No counterpart in the
 * reference (its torch._int_mm path pads into freshly allocated tensors). */
ECO_API int eco_gemm_s8s32_noalloc(const int8_t* A, int64_t lda, int a_layout, const int8_t* B,
                                   int64_t ldb, int b_layout, int64_t M, int64_t N, int64_t K,
                                   const int32_t* bias, int32_t* C, int64_t ldc, int32_t* amax,
                                   eco_stream_t stream);

/* Process-wide cap on the CTAs of the persistent GEMM kernels (0, the default: one
 * per SM).  A data-parallel caller sets it a little below the SM count so that the
 * collective kernels of NCCL, launched on other streams, find free SMs and overlap
 * the GEMMs.  No reference counterpart (the reference runs on one device). */
ECO_API int eco_set_gemm_sm_limit(int max_ctas);

/* Y = sat8(relu?( SR((C + bias[n]) * mult[n], shift) )) fused in the GEMM epilogue.
 * Replaces ilayer.py:135-141 (_int_mm + b_acc + _common_shift_requant :57-70) and,
 * with relu=1, the I8ReLU.apply_forward clamp that follows (:180-182). */
ECO_API int eco_gemm_s8_requant(const int8_t* A, int64_t lda, int a_layout, const int8_t* B, int64_t ldb,
                        int b_layout, int64_t M, int64_t N, int64_t K, const int32_t* bias,
                        const int32_t* mult, int shift, int relu, eco_sr_t sr, int8_t* Y,
                        int64_t ldy, eco_stream_t stream);

/* Int8LinearFunc's GEMMs with their fp32 epilogue fused (layers.py:45-75):
 * Y[m, n] = fp32(C[m, n]) * fp32(sa * sb), then * col_scale[n] (nullable), then
 * + bias[n] (nullable), each one IEEE fp32 operation like PyTorch's kernels; C = A.B as in
 * eco_gemm_s8s32 (int32, never stored).  sa / sb: doubles, each read from the device
 * (double bits at sa_dev / sb_dev, e.g. a scale from eco_quantize_dynamic_f32) when the
 * pointer is given, else the host value.  Replaces _int_mm + `acc.to(float32) * s_x *
 * s_w.t() + bias` (:48-52) and `dw_acc.float() * (s_g * s_x)`, `dx_acc.float() * (s_g *
 * s_w.mean())` (:63-67). */
ECO_API int eco_gemm_s8_dequant(const int8_t* A, int64_t lda, int a_layout, const int8_t* B, int64_t ldb,
                                int b_layout, int64_t M, int64_t N, int64_t K, const int64_t* sa_dev, double sa,
                                const int64_t* sb_dev, double sb, const float* col_scale, const float* bias,
                                float* Y, int64_t ldy, eco_stream_t stream);

/* ---------------------------------------------------------- elementwise --
 * dst = sat8(SR((src + bias[c]) * m, shift)), m = mult_col[c] or mult_scalar;
 * then dst = 0 where mask[r,c] <= 0 (mask nullable); relu clamps at 0;
 * sumsq (nullable, device int64) is overwritten with sum(dst^2).
 * Replaces the dX / dW requant of ilayer.py:155, :163, the relu mask of
 * :184-188 and the grad-clip square sum of iopt.py:96. */
ECO_API int eco_requant_s32_s8(const int32_t* src, int64_t rows, int64_t cols, int64_t ld_src,
                       const int32_t* bias_col, const int32_t* mult_col, int64_t mult_scalar,
                       int shift, int relu, eco_sr_t sr, const int8_t* mask, int64_t ld_mask,
                       int8_t* dst, int64_t ld_dst, int64_t* sumsq, eco_stream_t stream);

/* out = apply_mult_shift(x, mult, shift) as int64, no saturation.
 * x_bits 8/32/64; mult_kind 0 scalar, 1 per column [cols], 2 per row [rows].
 * Replaces fixedpoint.apply_mult_shift (fixedpoint.py:52-76) on CUDA tensors. */
ECO_API int eco_apply_mult_shift(const void* x, int x_bits, int64_t rows, int64_t cols, const int32_t* mult,
                         int mult_kind, int64_t mult_scalar, int shift, eco_sr_t sr, int64_t* out,
                         eco_stream_t stream);

/* out[c] = sum_r g[r, c] (int64).  Replaces ilayer.py:168 (g.int32.sum(0)). */
ECO_API int eco_colsum_s8(const int8_t* g, int64_t rows, int64_t cols, int64_t ld, int64_t* out,
                  eco_stream_t stream);

/* quantize_tensor_dynamic (quant.py:35-38, stochastic=False) of an fp32 [rows, cols]
 * matrix without a host round trip: *amax (overwritten) = the bits of max |x|;
 * s = calc_scale(max |x|) (quant.py:9-16) in double; q = clamp(round(x / (s + 1e-8)),
 * +-127) with PyTorch's CUDA arithmetic (a multiply by the fp32 reciprocal of the
 * scalar, round half to even).  scale_out: int64[3] = {double bits of s, 0, 0}. */
ECO_API int eco_quantize_dynamic_f32(const float* x, int64_t rows, int64_t cols, int64_t ld, int32_t* amax,
                                     int8_t* q, int64_t ld_q, int64_t* scale_out, eco_stream_t stream);

/* *out = max |x| over n int32/int64 elements (device int64 word, overwritten).
 * Replaces fixedpoint.int_amax's reduction (fixedpoint.py:85-88). */
ECO_API int eco_amax(const void* x, int x_bits, int64_t n, int64_t* out, eco_stream_t stream);

/* *out = sum x^2 over n int8 elements (device int64, overwritten).  iopt.py:96. */
ECO_API int eco_sumsq_s8(const int8_t* x, int64_t n, int64_t* out, eco_stream_t stream);

/* Reads and clears the sticky device error flags (bit 4: a bounded device wait
 * gave up, in a GEMM pipeline or a peer-exchange wait).  Synchronises the
 * device.  No reference counterpart: the reference has no device-side waits. */
ECO_API int eco_read_device_errors(uint32_t* flags);

/* 2-D strided int8 copy (relayout to a 16-byte aligned leading dimension). */
ECO_API int eco_copy2d_s8(const int8_t* src, int64_t ld_src, int8_t* dst, int64_t ld_dst, int64_t rows,
                  int64_t cols, eco_stream_t stream);

/* Splits the columns of a [rows, cols] int8 matrix into `parts` equal blocks and
 * stores block p as a contiguous [rows, cols / parts] matrix at dst + p * rows *
 * (cols / parts): the send buffer of the data-parallel all-to-all that hands
 * each rank its dY columns.  No reference counterpart (the reference has no
 * data parallelism). */
ECO_API int eco_split_cols_s8(const int8_t* src, int64_t ld_src, int64_t rows, int64_t cols, int64_t parts,
                      int8_t* dst, eco_stream_t stream);

/* ------------------------------------------------------------ loss boundary -----
 * The fp32 boundary at the end of the strict forward, fused into two launches with no
 * host synchronisation.  Replaces the training loop's loss lines (examples/i8_demo.py:
 * 56-59: logits_i8.float() * s_out, CrossEntropyLoss, its gradient) and the gradient's
 * quantize_tensor_dynamic(g, stochastic=True) (quant.py:19-38 with its .item() amax).
 * logits: [rows, cols] int8 (leading dim ld); labels: [rows] int64 in [0, cols); count:
 * the number of samples the mean runs over (the global batch under data parallelism).
 *
 * eco_ce_grad_rowstats: per row (max, log-sum-exp) into row_stats [rows, 2] fp32, the
 * row's NLL into row_loss [rows] (nullable), and *amax (overwritten) = the bit pattern
 * of max |g| as an int32 (non-negative floats order like their bits, so a MAX over
 * ranks of this word is the global maximum).
 *
 * eco_ce_grad_quantize: s_g = calc_scale(max|g|) with the maximum read from amax
 * (int32 or int64 word holding the float's bits); g_i8 = clamp(floor(g * fp32(1 /
 * (s_g + 1e-8)) + u), +-127) with u from sr (ECO_SR_PHILOX: 24 bits of the element's
 * Philox field, or ECO_SR_REPLAY_F32).  scale_out: int64[3] = {double bits of s_g, 0, 0}
 * (the layout of eco_scale_from_amax, so the queued backward reads it in place).
 * g_fp (nullable): the fp32 gradient [rows, cols] as well.  loss_out (nullable, needs
 * row_loss): sum of the row losses / count. */
ECO_API int eco_ce_grad_rowstats(const int8_t* logits, int64_t rows, int64_t cols, int64_t ld, double s_out,
                                 const int64_t* labels, int64_t count, float* row_stats, float* row_loss,
                                 int32_t* amax, eco_stream_t stream);
ECO_API int eco_ce_grad_quantize(const int8_t* logits, int64_t rows, int64_t cols, int64_t ld, double s_out,
                                 const int64_t* labels, int64_t count, const float* row_stats, const void* amax,
                                 int amax_bits, eco_sr_t sr, int8_t* g, int64_t ld_g, float* g_fp,
                                 int64_t* scale_out, const float* row_loss, float* loss_out, eco_stream_t stream);

/* ---------------------------------------------- device-side scales -----
 * The backward's dynamic scale chain without host round trips (used when a whole
 * backward pass is queued at once): the reference's dynamic_scale_from_int and
 * quantize_multiplier (fixedpoint.py:105-114, :26-37) in the same IEEE double
 * arithmetic, then the requant reads the multiplier and shift from the device.
 * Replaces the host scale lines of I8Linear.backward_i8 (ilayer.py:153-154 for dW,
 * :161-162 for dX) and the requants that follow them (:155, :163).
 *
 * eco_scale_from_amax: gain = (gain0_dev ? *gain0_dev (double bits) : gain0) * gain1;
 * s = amax * gain / 127 (1.0 when <= 0); (mult, shift) = quantize_multiplier(gain / s).
 * out: int64[3] = {double bits of s, mult, shift}.  A shift beyond 62 (the reference
 * raises) or a negative / non-finite ratio ORs ECO_FLAG_SHIFT_OVERFLOW /
 * ECO_FLAG_BAD_RATIO (1 / 2) into *flags (nullable). */
ECO_API int eco_scale_from_amax(const void* amax, int amax_bits, const int64_t* gain0_dev, double gain0,
                        double gain1, int64_t* out, uint32_t* flags, eco_stream_t stream);

/* eco_requant_s32_s8 with a scalar multiplier and shift read from params[1], params[2]
 * (the output of eco_scale_from_amax) and Philox rounding; no bias, no per-column
 * multipliers.  A shift beyond 62 stores zeros (the scale kernel flagged it). */
ECO_API int eco_requant_s32_s8_dev(const int32_t* src, int64_t rows, int64_t cols, int64_t ld_src,
                           const int64_t* params, int relu, eco_sr_t sr, const int8_t* mask, int64_t ld_mask,
                           int8_t* dst, int64_t ld_dst, int64_t* sumsq, eco_stream_t stream);

/* ------------------------------------------ data-parallel peer exchange -----
 * No reference counterpart (the reference has no data parallelism).  The buffers
 * are allocated on every rank and mapped into each process (each rank holds
 * device pointers to all ranks' copies); these calls move the exchange of the
 * data-parallel backward over NVLink with plain stores issued by a few CTAs,
 * and publish completion through flag words.  All waits are bounded (5 s): on
 * expiry the wait records bit 4 in the sticky device error flags
 * (eco_read_device_errors) and returns. */
#define ECO_MAX_PEERS 8

/* Pushes a [rows, cols] int8 matrix into n_dst destination buffers (device
 * pointers, host array) at rows dst_row0.. with leading dimension ld_dst.
 * split = 0: every destination receives the whole matrix (an all-gather of row
 * blocks); split = 1: destination p receives columns [p*c, (p+1)*c), c = cols /
 * n_dst (an all-to-all of column blocks).  ctas bounds the grid (0: one per SM). */
ECO_API int eco_peer_push_s8(const int8_t* src, int64_t ld_src, int64_t rows, int64_t cols, int8_t* const* dst,
                     int n_dst, int64_t ld_dst, int64_t dst_row0, int split, int ctas, eco_stream_t stream);

/* eco_peer_push_s8 that also publishes its completion: after every CTA's stores are
 * fenced at system scope, the last CTA writes epoch into entry (slot, rank) of the
 * n_ranks flag arrays (as eco_peer_signal; one launch instead of two).  ticket: a
 * device word, zero before the call (the kernel leaves it zero), one per call in
 * flight.
 * epoch_dev (here and in the calls below, nullable): a device word read when the kernel
 * runs, in place of `epoch` -- a captured CUDA graph replays the exchange with the
 * epochs of the moment. */
ECO_API int eco_peer_push_signal_s8(const int8_t* src, int64_t ld_src, int64_t rows, int64_t cols,
                            int8_t* const* dst, int n_dst, int64_t ld_dst, int64_t dst_row0, int split, int ctas,
                            int64_t* const* peer_flags, int n_ranks, int rank, int slot, int64_t epoch,
                            const int64_t* epoch_dev, uint32_t* ticket, eco_stream_t stream);

/* All-reduce (op 0: MAX, 1: SUM, int64 arithmetic) of count <= stride values (int32 or
 * int64 at src) over the n ranks, result int64[count] in out.  bufs: the n ranks'
 * exchange buffers, int64 [2][n][stride] each (own_buf: this rank's); flags as below,
 * one slot used by every call in order, epoch growing by one per call.  Bounded wait
 * (5 s; then out is zero and the error bit is set). */
ECO_API int eco_peer_allreduce_i64(const void* src, int src_bits, int count, int op, int64_t* const* bufs,
                           int stride, const int64_t* own_buf, int64_t* const* peer_flags,
                           const int64_t* own_flags, int n, int rank, int slot, int64_t epoch,
                           const int64_t* epoch_dev, int64_t* out, eco_stream_t stream);

/* Flag arrays are int64 [slots, ECO_MAX_PEERS], zero before first use.  signal:
 * after all prior work on the stream, writes epoch into entry (slot, rank) of
 * every rank's array (peer_flags: host array of the n ranks' flag pointers).
 * wait: the stream continues once entries (slot, 0..n-1) of this rank's array
 * all reach epoch (epochs only grow), or after timeout_us (0: the 5 s limit;
 * larger values are capped at it). */
ECO_API int eco_peer_signal(int64_t* const* peer_flags, int n, int rank, int slot, int64_t epoch,
                    const int64_t* epoch_dev, eco_stream_t stream);
ECO_API int eco_peer_wait(const int64_t* flags, int n, int slot, int64_t epoch, const int64_t* epoch_dev,
                  int64_t timeout_us, eco_stream_t stream);

/* Mapping the exchange buffers between the processes of one node (CUDA IPC).
 * export: the IPC handle (ECO_IPC_HANDLE_BYTES bytes at `handle`) of the device
 * allocation that contains `ptr`, and ptr's byte offset in it; the caller sends both
 * to the other ranks.  open: maps a peer's allocation into this process (unicast peer
 * mapping over NVLink; no multicast object is created) and returns its base; the
 * peer's buffer is base + offset.  close: unmaps a base returned by open.  The
 * exporting rank must keep its allocation alive until every peer has closed it. */
#define ECO_IPC_HANDLE_BYTES 64
ECO_API int eco_ipc_export(const void* ptr, void* handle, int64_t* offset);
ECO_API int eco_ipc_open(const void* handle, void** base);
ECO_API int eco_ipc_close(void* base);

/* -------------------------------------------------------- I8ECO step -----
 * One fused, single-pass integer ECO-SGDM step over a list of layers
 * (ecoint8/strict/iopt.py:103-200): per-row fixed-point multipliers and common
 * shifts are derived on the device from the scales (iopt.py:134-148), grad clip
 * from the device square sum (:90-101), weights and momentum are updated in
 * place, the momentum scale s_m is updated on the device from the row maxima
 * (:178-180), per-row sums of |e| are written for the statistics (:183), and
 * the bias takes its integer SGD step (:187-197).  No host synchronisation.
 */
typedef struct {
  int8_t* w;              /* [rows, cols] contiguous, updated in place */
  int8_t* m;              /* [rows, cols] contiguous momentum, updated in place */
  const int8_t* g;        /* [rows, cols] contiguous int8 weight gradient */
  const double* sw;       /* [rows] frozen per-row weight steps */
  int64_t* rowsum;        /* [rows] out: sum_j |e| (nullable) */
  const int64_t* gsq;     /* device sum g^2 (required when grad clipping) */
  int64_t* state;         /* device int64[4]: [0] s_m (double bits), [1] row-max
                             accumulator (double bits, zero between steps), [2] error flags */
  int32_t* b_acc;         /* [rows] int32 bias accumulator (nullable: no bias) */
  const int64_t* gb_sum;  /* [rows] int64 bias gradient column sums */
  const void* nudge_w;    /* replay: [rows, cols] int32 weight nudges */
  const void* nudge_m;    /* replay: [rows, cols] int32/int64 momentum nudges */
  const void* nudge_b;    /* replay: [rows] int32/int64 bias nudges */
  int64_t rows, cols;
  int64_t row_base;       /* global index of row 0 (a data-parallel row shard; else 0) */
  double sw_min, sw_max;  /* min / max of sw over ALL rows of the layer */
  double s_g;             /* layer._gw_s */
  double s_gb, sx;        /* layer._gb_s, layer.sx (bias step) */
  uint64_t stream_w;      /* Philox site of the weight / momentum nudges */
  uint64_t stream_b;      /* Philox site of the bias nudges */
  int32_t nudge_m_bits;   /* 32 or 64 */
  int32_t nudge_b_bits;   /* 32 or 64 */
  int64_t bias_rows;      /* 0: the bias of the stepped rows.  > 0: the bias of the layer's
                             global rows [0, bias_rows) instead, with b_acc, gb_sum, sw and
                             nudge_b indexed by (global row - row_base), so they must cover
                             those rows: a data-parallel row shard then updates every bias
                             (the bias step does not depend on the weights) and no rank has
                             to receive the others' biases */
  const int64_t* s_g_dev;  /* nullable: s_g as double bits on the device (a scale computed by
                              eco_scale_from_amax), used instead of s_g */
  const int64_t* s_gb_dev; /* nullable: likewise for s_gb */
} eco_i8eco_layer_t;

typedef struct eco_i8eco_hyper {
  double lr;
  double grad_clip;     /* < 0: no clipping (grad_clip=None) */
  int64_t b_q, nb_q, lr_q, a_q; /* iopt.py:107-110 */
  int32_t sr_mode;      /* ECO_SR_PHILOX or a replay mode (replay uses the layer nudges) */
  int32_t finalize;     /* 1: update s_m from the row maxima now; 0: leave the accumulator
                           (state[1]) for eco_i8eco_finalize, e.g. after a cross-rank max */
  uint64_t seed;
  uint32_t* done_counter; /* device word, zero between steps (reset by the kernel) */
  const struct eco_i8eco_hyper* dev; /* nullable: a copy of this struct in device memory whose
                             lr, grad_clip, b_q, nb_q, lr_q, a_q and seed the kernel reads when
                             it runs, in place of the values above (a captured CUDA graph then
                             replays the step with the learning rate and key of the moment) */
} eco_i8eco_hyper_t;

ECO_API int eco_i8eco_step(const eco_i8eco_layer_t* layers, int n_layers, const eco_i8eco_hyper_t* hyper,
                   eco_stream_t stream);

/* Turns each layer's row-max accumulator into its new momentum scale
 * (s_m = acc / 127, or 1.0 when the maximum is 0; iopt.py:178-180) and clears the
 * accumulator; layers with error flags keep their scale.  `state` is
 * [n_layers, 4] int64 as in eco_i8eco_layer_t.  Used after a step launched with
 * finalize = 0 once the accumulators hold the maximum over all row shards. */
ECO_API int eco_i8eco_finalize(int64_t* state, int n_layers, eco_stream_t stream);

/* --------------------------------------------------- EcoInt8SGDM step -----
 * The fused fp32-transient ECO step of EcoInt8SGDM (ecoint8/eco.py:330-362),
 * replacing the Triton kernels and their host glue (triton_kernels.py:127-170):
 * max|g|, pass 1 (max |m_new|), pass 2 (store w and m), sm <- sm_new.  `scratch`
 * is a device buffer of 4 uint32 words (cleared by the call). */
ECO_API int eco_sgdm_step(int8_t* w, int8_t* m, const float* g, int64_t rows, int64_t cols,
                  const float* sw, float* sm, float lr, float beta, float wd, float alpha,
                  uint64_t seed, uint32_t* scratch, eco_stream_t stream);

/* ------------------------------------------------- EcoSGDM / EcoAdam steps -----
 * The fp32-state ECO optimizers (ecoint8/eco.py:50-235) over a list of layers in two
 * launches, replacing the per-layer PyTorch loops of EcoSGDM.step (:94-131) and
 * EcoAdam.step (:182-228) with their .item() syncs (g.norm(), e.abs().mean()):
 *   1. per layer: the gradient norm (double sum of squares) and whether every
 *      gradient value is finite (_get_grad_w, :39-47);
 *   2. per element: clip, weight decay, moment update(s), stochastic rounding onto the
 *      frozen grid (quant.py:19-28), error injection; w and m (v) updated in place.
 * Each fp32 operation is the reference's PyTorch operation with PyTorch's CUDA
 * rounding (a Python scalar operand rounded to fp32; add with alpha and addcmul as a
 * fused multiply-add; division by a Python scalar as a multiply by the fp32
 * reciprocal; scalar / tensor as reciprocal times scalar).  The norm is the fp32
 * rounding of the square root of the double sum of squares.
 * scratch: device doubles, at least eco_fp32_eco_scratch_len() of them; on return
 * scratch[2*T + t] holds sum |e| of tile t of 65536 elements (layers in order, their
 * tiles in order), T = the number of tiles (the statistics' inputs). */
typedef struct {
  int8_t* w;             /* [rows, cols] int8 weights, updated in place */
  float* m;              /* [rows, cols] fp32 momentum / first moment, updated in place */
  float* v;              /* [rows, cols] fp32 second moment (Adam), updated in place; else NULL */
  const float* g;        /* [rows, cols] fp32 weight gradient (layer._grad_w) */
  const float* sw;       /* [rows] the layer's row scales s_w (w_fp32 = w * s_w) */
  const float* s_fixed;  /* [rows] the optimizer's frozen grid (the s_w clone taken at construction) */
  const float* u;        /* ECO_SR_REPLAY_F32: [rows, cols] uniforms in [0, 1); else NULL */
  int64_t rows, cols;
  uint64_t stream;       /* Philox site of the layer's rounding */
  float* norm_out;       /* nullable: the gradient norm, fp32 */
  int32_t* stepped_out;  /* nullable: 1 if the layer was stepped, 0 if skipped (non-finite gradient) */
} eco_fp32_layer_t;

typedef struct {
  int32_t kind;          /* 0: EcoSGDM, 1: EcoAdam */
  int32_t sr_mode;       /* ECO_SR_PHILOX or ECO_SR_REPLAY_F32 */
  double lr;
  double beta1;          /* EcoSGDM: momentum; EcoAdam: betas[0] */
  double beta2, eps;     /* EcoAdam */
  double weight_decay;
  double grad_clip;      /* < 0: no clipping (grad_clip=None) */
  double bc1, bc2;       /* EcoAdam: 1 - beta1^t, 1 - beta2^t (eco.py:184) */
  uint64_t seed;         /* Philox key (ECO_SR_PHILOX) */
} eco_fp32_hyper_t;

ECO_API int eco_fp32_eco_step(const eco_fp32_layer_t* layers, int n_layers, const eco_fp32_hyper_t* hyper,
                              double* scratch, int64_t scratch_len, eco_stream_t stream);
/* The scratch length (doubles) eco_fp32_eco_step needs for these layers (<= 0 on bad input). */
ECO_API int64_t eco_fp32_eco_scratch_len(const eco_fp32_layer_t* layers, int n_layers);

#ifdef __cplusplus
}
#endif
#endif /* ECOINT8_B200_H */
