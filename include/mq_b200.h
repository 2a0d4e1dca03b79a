/*
 * mq_b200 — B200 (sm_100a) quantized-linear engine behind a plain C ABI.
 *
 * Drop-in device path for mini_ai's quantized linear: y = x · Wᵀ over GGUF
 * Q8_0 / Q4_0 / Q4_1 weights. Every entry point takes plain pointers and
 * sizes, returns MQ_OK (0) or a negative MQ_ERR_* code, and leaves a message
 * in mq_last_error() for the calling thread. No C++ exception crosses this
 * boundary. Device pointers are CUDA device addresses on the handle's device;
 * `stream` is a cudaStream_t (NULL = the legacy default stream) and every
 * device call is stream-ordered and asynchronous unless stated otherwise.
 *
 * Reference interfaces replaced (paths in the mini_ai project):
 *   - QuantizeTensor / TensorFromQuantized / DequantizeTensor,
 *     include/mini_llama/quantized_tensor.h:21-24
 *   - QuantizedDotRow, include/mini_llama/quantized_tensor.h:25
 *   - LinearDispatch (quantized branch), include/mini_llama/matmul_dispatch.h:28
 *   - CudaModelState::UploadWeight + LinearKernel, src/cuda_backend.cu:94-110,275-283
 *   - CudaDeviceInfo, include/mini_llama/backend.h:10
 */
#ifndef MQ_B200_H_
#define MQ_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML block types; the numeric values are the reference's QuantType ids
 * (include/mini_llama/quantized_tensor.h:10 == gguf.h:15-17). */
enum {
  MQ_Q4_0 = 2, /* 18-byte block: fp16 d, 16 bytes of nibbles; w = d*(q-8)   */
  MQ_Q4_1 = 3, /* 20-byte block: fp16 d, fp16 m, 16 bytes;     w = d*q + m   */
  MQ_Q8_0 = 8  /* 34-byte block: fp16 d, 32 int8;              w = d*q       */
};

enum {
  MQ_OK = 0,
  MQ_ERR_INVALID = -1,     /* bad argument: type, shape, pointer, stride     */
  MQ_ERR_CUDA = -2,        /* a CUDA runtime call failed                     */
  MQ_ERR_SIZE = -3,        /* byte count does not match rows x cols x type   */
  MQ_ERR_NONFINITE = -4,   /* quantize input holds Inf/NaN                   */
  MQ_ERR_RANGE = -5,       /* quantize scale or min overflows fp16           */
  MQ_ERR_TIMEOUT = -6,     /* a bounded device wait on a peer ran out        */
  MQ_ERR_UNSUPPORTED = -7  /* not built for this device / configuration      */
};

typedef struct mq_weight mq_weight; /* opaque device-resident packed weight */

/* Message for the last failing call on this thread ("" if none). */
const char *mq_last_error(void);

/* Library version string. */
const char *mq_version(void);

/* Bytes of the GGUF block stream for a rows x cols matrix: rows *
 * ceil(cols/32) * {34|18|20}; 0 for an unknown type or a non-positive shape.
 * Mirrors the size rule of TensorFromQuantized, src/quantized_tensor.cc:88-96. */
size_t mq_quantized_bytes(int qtype, int rows, int cols);

/* Bit-exact host quantizer: packs a row-major F32 rows x cols matrix into
 * GGUF blocks exactly as QuantizeTensor does (src/quantized_tensor.cc:104-159),
 * using `threads` host threads (0 = all hardware threads). Errors:
 * MQ_ERR_NONFINITE for Inf/NaN input, MQ_ERR_RANGE when a scale or Q4_1 min
 * overflows fp16, MQ_ERR_SIZE when dst_bytes is not mq_quantized_bytes(). */
int mq_quantize(int qtype, const float *src, int rows, int cols, void *dst, size_t dst_bytes, int threads);

/* Host decoder, DequantizeTensor (src/quantized_tensor.cc:193-206). */
int mq_dequantize(int qtype, const void *blocks, size_t nbytes, int rows, int cols, float *dst);

/* Device quantizer: the same bit-exact packing as mq_quantize, run on the GPU
 * over a device F32 matrix into a device GGUF block buffer. Input errors
 * (non-finite values, fp16 overflow) are reported when the call returns, so
 * this call synchronizes `stream`. */
int mq_quantize_device(int device, int qtype, const float *d_src, int rows, int cols, void *d_dst,
                       size_t dst_bytes, void *stream);

/* Upload a packed weight. `blocks` is the GGUF block stream (host memory when
 * blocks_on_device == 0, a device pointer on `device` otherwise) of a rows x
 * cols matrix. The weight is re-laid out on the device for 16-byte vector
 * loads (quants and fp16 scales in separate, aligned planes); the number of
 * bytes per weight is unchanged. Replaces CudaModelState::UploadWeight
 * (src/cuda_backend.cu:275-283). Synchronizes `stream` before returning. */
int mq_weight_create(int device, int qtype, int rows, int cols, const void *blocks, size_t nbytes,
                     int blocks_on_device, void *stream, mq_weight **out);

/* Upload rows [row_begin, row_end) of a rows x cols packed weight as its own
 * handle: the output-row shard one GPU holds when a projection is split
 * across GPUs. `blocks` is the FULL matrix's block stream (host or device). */
int mq_weight_shard_create(int device, int qtype, int rows, int cols, int row_begin, int row_end,
                           const void *blocks, size_t nbytes, int blocks_on_device, void *stream,
                           mq_weight **out);

/* Release a handle and its device memory (NULL is a no-op). */
void mq_weight_destroy(mq_weight *w);

/* Shape, type, device and device bytes of a handle (any out-pointer may be NULL). */
int mq_weight_info(const mq_weight *w, int *qtype, int *rows, int *cols, int *device, size_t *device_bytes);

/* Write the handle's weight back as a GGUF block stream to host memory
 * (round-trip check of the device layout). Synchronous. */
int mq_weight_export(const mq_weight *w, void *dst, size_t dst_bytes);

/* y[i, n] = sum_k x[i, k] * W[n, k] (+ bias[n]) for i in [0, m).
 * x: device F32 [m, ldx] with ldx >= cols; y: device F32 [m, ldy] with
 * ldy >= rows; bias: device F32 [rows] or NULL. Small m runs a streaming
 * GEMV, larger m the tcgen05 tensor-core GEMMs (see mq_set_path). The tensor-
 * core paths keep per-(device, stream) scratch for the split activations,
 * allocated on first use and grown as needed (the growth synchronizes the
 * stream). A bounded wait that runs out inside a GEMM launch is reported as
 * MQ_ERR_TIMEOUT by the next mq_linear call on that device. Accumulation is
 * fp32; results
 * match the reference's sequential fp32 dot (QuantizedDotRow,
 * src/quantized_tensor.cc:161-191) to within accumulation-order rounding.
 * The quantized branch of LinearDispatch (src/matmul_optimized.cc:172-174)
 * and LinearKernel (src/cuda_backend.cu:94-110) accept m == 1 only; here any
 * m >= 0 works (m == 0 is a no-op). */
int mq_linear(const mq_weight *w, const float *x, int m, int ldx, const float *bias, float *y, int ldy,
              void *stream);

/* The gate/up half of the Llama FFN in one call: y = SwiGlu(x * W_gateᵀ,
 * x * W_upᵀ), i.e. y[i, n] = g / (1 + exp(-g)) * u with g, u the two products,
 * as FfnForward's `Linear(h, w_gate)`, `Linear(h, w_up)`, `SwiGlu(gate, up)`
 * (src/forward.cc:105-110; SwiGluKernel, src/cuda_backend.cu:241-245; Silu,
 * src/ops.cc:85-91). The gate product goes to a per-(device, stream) scratch
 * buffer and the up product's kernel applies the SwiGLU in its output write,
 * so the separate elementwise pass and one round trip of both outputs are
 * gone. Both weights must have the same shape and device; x, y as mq_linear. */
int mq_linear_swiglu(const mq_weight *w_gate, const mq_weight *w_up, const float *x, int m, int ldx, float *y,
                     int ldy, void *stream);

/* y = residual + (x * Wᵀ + bias): the linear followed by the residual add of
 * ForwardCuda (`AddKernel(x, o)` after the wo and w_down projections,
 * src/cuda_backend.cu:236-240), in the kernel's own output write. residual:
 * device F32 [m, ldy] with y's stride; it may be y itself (the usual
 * in-place residual stream). Otherwise as mq_linear. */
int mq_linear_residual(const mq_weight *w, const float *x, int m, int ldx, const float *bias, const float *residual,
                       float *y, int ldy, void *stream);

/* Same product for a ragged batch: `offsets` (host, n_seqs + 1 entries,
 * offsets[0] == 0, non-decreasing) delimits each request's rows inside the
 * contiguous [offsets[n_seqs], ldx] activation matrix. The rows are
 * independent, so the result equals mq_linear with m = offsets[n_seqs]; the
 * offsets are validated and kept for callers that need per-request slices. */
int mq_linear_ragged(const mq_weight *w, const float *x, const int *offsets, int n_seqs, int ldx,
                     const float *bias, float *y, int ldy, void *stream);

/* Same product as mq_linear for decode-sized batches, for callers that cannot
 * allocate device memory: they own every device byte through their own pool,
 * run under a fixed memory budget, or call from a hot loop where cudaMalloc's
 * device-wide synchronisation and latency are not acceptable. It has no
 * counterpart in the reference. This call allocates nothing: its scratch is a
 * fixed 3.6 MiB device array that every GPU loading the library holds until
 * the process exits. Limits: 1 <= m <= 16 (m == 0 is a no-op), weight cols
 * <= 16384 and rows <= 131072; larger requests fail with MQ_ERR_INVALID. The
 * first call on a device resolves the array's device address there, so make
 * that first call before any stream capture. All calls on a device share the
 * array, so calls that overlap on the GPU (other streams, other host threads)
 * race and must be serialised by the caller. A bounded device wait that runs
 * out writes NaN to the outputs. */
int mq_linear_noalloc(const mq_weight *w, const float *x, int m, int ldx, const float *bias, float *y, int ldy,
                      void *stream);

/* ---- Row-sharded linear across GPUs (one process or host thread per GPU).
 * A weight of N = G*R rows is split into G equal output-row shards
 * (mq_weight_shard_create with rows [r*R, (r+1)*R) on rank r). Each rank
 * computes its R outputs and an NCCL all-gather over NVLink assembles the
 * full [m, N] output on every rank. The result equals mq_linear on the whole
 * weight up to fp32 summation order: the kernels split each tile's K range
 * across CTAs by the launch's total work, so a shard may sum in another order
 * (bit-identical where both launches split alike, e.g. when neither has more
 * (128-row tile, K step) chunks than SMs). No counterpart in the reference, which runs every
 * linear on one device (`--device N`, src/main.cc:249-250); new surface for
 * the multi-GPU row of the hot path. NCCL is loaded at run time
 * (libnccl.so.2). */
typedef struct mq_comm mq_comm;
#define MQ_COMM_ID_BYTES 128

/* A fresh communicator id (rank 0 creates it and shares it with the other
 * ranks through the caller's own host channel). len >= MQ_COMM_ID_BYTES. */
int mq_comm_unique_id(void *id, size_t len);

/* Join the communicator of `nranks` ranks as `rank`, on `device`. Collective:
 * every rank must call it with the same id. With MQ_P2P_GATHER=1 in every
 * rank's environment (and 2..8 ranks) it also allocates a staging region of
 * 2 * nranks * 4 MiB on `device` and maps every peer's region through CUDA
 * IPC, so that mq_linear_sharded_allgather gathers over NVLink peer memory
 * instead of NCCL; if any rank cannot map every peer, all ranks use NCCL.
 * Destroy the communicators only after every rank's last gather completed
 * (for example after a barrier). */
int mq_comm_create(int device, int nranks, int rank, const void *id, size_t len, mq_comm **out);
void mq_comm_destroy(mq_comm *c);

/* 1 when the communicator gathers over NVLink peer memory (MQ_P2P_GATHER=1
 * and every rank mapped every peer), 0 when it uses NCCL's all-gather, a
 * negative code for a NULL handle. */
int mq_comm_uses_peer_gather(const mq_comm *c);

/* y[i, n] for all n in [0, N) on every rank: this rank's shard product
 * (+ bias[rank*R .. rank*R+R) when bias, the full [N] vector, is given) and
 * an all-gather of the slices. x: device F32 [m, ldx] (full K); y: device F32
 * [m, ldy] with ldy >= N. Stream-ordered on `stream`; every rank must call it
 * with the same m, in the same order relative to its other collectives. The
 * peer-memory gather (see mq_comm_create) takes outputs with m * R <= 2^20 and
 * may be captured in a CUDA graph. A peer that does not arrive within the wait
 * limit (MQ_P2P_WAIT_NS nanoseconds in the environment at mq_comm_create,
 * default 1 s) leaves NaN in that peer's output columns and poisons the
 * communicator: its next call and every later peer-memory gather on it fail
 * with MQ_ERR_TIMEOUT (replays of a captured graph write NaN without
 * waiting); destroy it and create a new one. */
int mq_linear_sharded_allgather(const mq_weight *shard, const float *x, int m, int ldx, const float *bias,
                                float *y, int ldy, mq_comm *comm, void *stream);

/* Kernel selection for the next mq_linear calls on this thread:
 * 0 = automatic (default): the tcgen05 int8 decode GEMV for m <= 4, the
 *     tcgen05 scale-folded decode GEMM for m <= 32 (the fp16 decode GEMM for
 *     weights whose block scales exceed the fold's fp16 range), the tcgen05
 *     prefill GEMM above;
 * 1 = force the stream-K SIMT GEMV, 2 = force the tcgen05 prefill GEMM,
 * 3 = force the tcgen05 int8 decode GEMV, 4 = force the tcgen05 fp16 decode
 * GEMM, 5 = force the SIMT dp4a decode GEMV, 6 = force the tcgen05
 * scale-folded decode GEMM (MQ_ERR_UNSUPPORTED for weights outside its
 * range), 7 = force the scale-folded decode GEMM on CTA pairs (tcgen05
 * cta_group::2; MQ_ERR_UNSUPPORTED for weights outside the fold's range or
 * with an odd number of 128-row tiles); other values are ignored. Returns the
 * previous mode. */
int mq_set_path(int mode);

/* Number of kernels this library has launched in this process (all devices,
 * all threads): the evidence a benchmark reports as its kernel count. */
uint64_t mq_kernel_launches(void);

/* Human-readable device list, like CudaDeviceInfo (src/cuda_backend.cu:355-369). */
int mq_device_info(char *buf, size_t len);

/* The bounded-wait error flag of `device` as its kernels see it: a device
 * pointer to an int in mapped host memory. A tensor-core kernel whose wait ran
 * out stores 1 there; the next tensor-core call on that device then returns
 * MQ_ERR_TIMEOUT and clears it. Exposed so that a monitor or a test can read
 * the flag or raise it from the device (cudaMemset, or a kernel's store). */
int mq_device_error_flag(int device, int **flag);

#ifdef __cplusplus
}
#endif
#endif /* MQ_B200_H_ */
