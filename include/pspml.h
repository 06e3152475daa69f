/*
 * pspml.h - C ABI of the B200 (sm_100a) backend for the cargo-psp-ml
 * TFLite inference path.
 *
 * The reference (saifk00/psp-ml) calls its kernels as plain Rust functions
 * from generated code:
 *   psp-ml/src/kernels/naive.rs:13-184   conv2d, conv2d_relu, max_pool2d,
 *                                        reshape, fully_connected(_relu)
 *   psp-ml/src/kernels/mod.rs:176-479    matmul_bt, matmul_bt_tiled, relu,
 *                                        im2col, im2col_padded, bias_add
 *   examples/mnist-bench/src/generated.rs:8-294
 *                                        forward / forward_timed (emitted by
 *                                        cargo-psp-ml/src/codegen/render.rs:14-73)
 * Every entry point below replaces one of those call sites; the comment on
 * each names the one it replaces.
 *
 * Conventions
 *  - Every function returns a pspml_status (0 = OK).  Nothing aborts or
 *    throws across this boundary.  pspml_last_error() returns a message for
 *    the last failing call made on the calling host thread.
 *  - Tensors are NHWC, row-major, batch outermost.  int8 activations carry a
 *    per-tensor zero point; weights are symmetric per output channel.
 *  - "dev" pointers are device memory on the context's GPU; "host" pointers
 *    are CPU memory (pinned memory from pspml_host_alloc gives full-speed
 *    copies).  The caller owns every buffer it passes in.
 *  - stream is a cudaStream_t passed as void* (NULL = legacy default stream).
 *  - A context belongs to one device.  Calls on one context are serialised
 *    by the caller; contexts on different devices may be driven from
 *    different host threads at the same time.
 */
#ifndef PSPML_H
#define PSPML_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PSPML_ABI_VERSION 2

typedef enum pspml_status {
  PSPML_OK = 0,
  PSPML_ERR_INVALID_ARG = 1,   /* bad shape, null pointer, bad offset      */
  PSPML_ERR_UNSUPPORTED = 2,   /* valid request this build does not cover  */
  PSPML_ERR_CUDA = 3,          /* a CUDA runtime/driver call failed        */
  PSPML_ERR_OOM = 4,           /* device or pinned-host allocation failed  */
  PSPML_ERR_TIMEOUT = 5,       /* host watchdog deadline passed            */
  PSPML_ERR_NO_DEVICE = 6,     /* no usable sm_100 device                  */
  PSPML_ERR_DEVICE_WAIT = 7    /* a kernel gave up on a bounded wait       */
} pspml_status;

/* Operator kinds.  The first five mirror the TFLite builtins the reference
 * lowers (cargo-psp-ml/src/parse/tflite/lowering.rs:92-104) plus the two it
 * rejects today (DEPTHWISE_CONV_2D, AVERAGE_POOL_2D; schema.fbs:260,263). */
typedef enum pspml_op_kind {
  PSPML_OP_CONV2D = 1,
  PSPML_OP_DEPTHWISE_CONV2D = 2,
  PSPML_OP_FULLY_CONNECTED = 3,
  PSPML_OP_MAX_POOL2D = 4,
  PSPML_OP_AVERAGE_POOL2D = 5,
  PSPML_OP_RESHAPE = 6
} pspml_op_kind;

/* One quantised operator.  Shapes are per sample (the batch is a call
 * argument).  This is the int8 counterpart of the reference's IR op
 * (cargo-psp-ml/src/ir/psp.rs:16-56) after codegen planning
 * (cargo-psp-ml/src/codegen/plan.rs:93-144): padding is explicit and may be
 * asymmetric (SAME padding per lowering.rs:341-364), and the quantisation
 * parameters TFLite stores per tensor are carried on the op.
 *
 *  CONV2D            filter [out_c][kernel_h][kernel_w][in_c] int8
 *  DEPTHWISE_CONV2D  filter [kernel_h][kernel_w][in_c] int8 (out_c == in_c)
 *  FULLY_CONNECTED   filter [out_c][in_h*in_w*in_c] int8
 *  conv / FC:        bias [out_c] int32, mult [out_c] int32 (Q31 multiplier),
 *                    shift [out_c] int32 (TFLite convention: >0 left shift)
 *  pools: zp_out must equal zp_in (TFLite keeps the input's quantisation).
 *  act_min/act_max clamp the requantised output (ReLU: act_min = zp_out).
 * Offsets are byte offsets into the weight blob, 16-byte aligned, or -1.
 * `flags` is 0 for the int8 ops; the f32 ops below read PSPML_F32_* bits
 * from it (their zp/act fields are ignored). */
typedef struct pspml_op_desc {
  int32_t kind;
  int32_t in_h, in_w, in_c;
  int32_t out_h, out_w, out_c;
  int32_t kernel_h, kernel_w;
  int32_t stride_h, stride_w;
  int32_t pad_top, pad_left, pad_bottom, pad_right;
  int32_t zp_in, zp_out;
  int32_t act_min, act_max;
  int32_t flags;
  int64_t filter_off, bias_off, mult_off, shift_off;
} pspml_op_desc;

typedef struct pspml_ctx pspml_ctx;
typedef struct pspml_model pspml_model;

/* Per-call timing filled by the host-buffer forward calls (may be NULL). */
typedef struct pspml_timing {
  double total_ms;        /* wall time of the whole call                   */
  double h2d_bytes;       /* bytes copied host -> device                   */
  double d2h_bytes;       /* bytes copied device -> host                   */
  int32_t micro_batches;  /* micro-batches the call was split into         */
  int32_t devices;        /* devices used                                  */
  int32_t rerun_shards;   /* pspml_forward_sharded: failed shards re-run on
                             the other devices                             */
} pspml_timing;

/* ------------------------------------------------------------------ misc */

/* Message for the last failing call on this host thread ("" if none). */
const char* pspml_last_error(void);
/* PSPML_ABI_VERSION of the loaded library. */
int32_t pspml_abi_version(void);
/* Number of sm_100 devices visible (0 when none). */
int pspml_device_count(int* count);

/* -------------------------------------------------------------- context */

/* Create a context on `device` with `workspace_bytes` of device scratch
 * (0 = default 64 MiB) used by the per-op calls below for folded biases.
 * Replaces the reference's static scratch buffers (render.rs:153-180). */
int pspml_ctx_create(int device, size_t workspace_bytes, pspml_ctx** out);
int pspml_ctx_destroy(pspml_ctx* ctx);
/* Host watchdog for synchronous calls (0 = no deadline).  A call that
 * passes the deadline returns PSPML_ERR_TIMEOUT while its device work may
 * still run: the caller keeps the buffers it passed valid until that work
 * ends (cudaDeviceSynchronize, or any later call on the same model, which
 * is ordered after it), and treats the outputs as not written. */
int pspml_ctx_set_timeout_ms(pspml_ctx* ctx, int64_t timeout_ms);
/* Reads and clears the device-side error word that kernels set when a
 * bounded wait expires; returns PSPML_ERR_DEVICE_WAIT if it was set.  The
 * tensor-core kernels bound every wait at 4 s; on expiry they record a code
 * here, stop, let issued copies land, free tensor memory and return. */
int pspml_ctx_check_device(pspml_ctx* ctx);
/* Diagnostic of the path above (no counterpart in the reference): one
 * thread waits, with the kernels' bounded wait, on a barrier that it
 * signals itself only when `signal` != 0; an unsignalled wait gives up after
 * limit_us (1 us .. 10 s) and sets the error word, so the next
 * pspml_ctx_check_device returns PSPML_ERR_DEVICE_WAIT.  Synchronous; the
 * context stays usable. */
int pspml_ctx_wait_selftest(pspml_ctx* ctx, int64_t limit_us, int32_t signal);

/* Pinned host memory for full-speed host<->device copies. */
int pspml_host_alloc(size_t bytes, void** out);
int pspml_host_free(void* p);

/* ---------------------------------------------------- per-op (int8) calls
 * All tensors are device pointers.  `batch` samples of shape d->in_* are
 * read from `in` and batch samples of shape d->out_* written to `out`.
 * The filter/bias/mult/shift offsets in `d` are ignored; the tensors are
 * passed directly.  These calls are asynchronous on `stream`. */

/* Replaces naive::conv2d / conv2d_relu (naive.rs:13-92) and the
 * im2col_padded -> matmul_bt_tiled -> bias_add -> relu chain
 * (mod.rs:215-479; generated.rs:76-91).  tcgen05 kind::i8 implicit GEMM
 * when in_c % 32 == 0 (1x1 or stride-1 convs), CUDA-core direct conv
 * otherwise. */
int pspml_conv2d_s8(pspml_ctx* ctx, const pspml_op_desc* d, int64_t batch,
                    const int8_t* in, const int8_t* filter,
                    const int32_t* bias, const int32_t* mult,
                    const int32_t* shift, int8_t* out, void* stream);

/* DEPTHWISE_CONV_2D (rejected by the reference at lowering.rs:98-103). */
int pspml_depthwise_conv2d_s8(pspml_ctx* ctx, const pspml_op_desc* d,
                              int64_t batch, const int8_t* in,
                              const int8_t* filter, const int32_t* bias,
                              const int32_t* mult, const int32_t* shift,
                              int8_t* out, void* stream);

/* Replaces naive::fully_connected / fully_connected_relu
 * (naive.rs:147-184), batched: out[b][o] for b < batch. */
int pspml_fully_connected_s8(pspml_ctx* ctx, const pspml_op_desc* d,
                             int64_t batch, const int8_t* in,
                             const int8_t* filter, const int32_t* bias,
                             const int32_t* mult, const int32_t* shift,
                             int8_t* out, void* stream);

/* pspml_fully_connected_s8 for callers that cannot allocate device memory
 * (no counterpart in the reference): code running under CUDA graph capture,
 * where cudaMalloc is not allowed; hosts whose device memory budget is fixed
 * at start-up; callers that pass only buffers they already own.  It takes no
 * context and allocates nothing: its scratch (folded biases, requantisation
 * table, error word) is a fixed 256 KiB array inside the library, held on
 * every device that loads the library until the process exits.
 *  - Ops needing more scratch than that (more than about 13000 output
 *    channels) are rejected with PSPML_ERR_INVALID_ARG and a message.
 *  - The first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress, which may load the library's device code);
 *    make that first call before any stream capture begins.
 *  - A kernel that gives up on a bounded wait sets an error word inside the
 *    same array; pspml_noalloc_check_device reads and clears it.
 *  - All calls on a device share the one array: calls whose GPU work
 *    overlaps (different streams, or host threads without ordering) race
 *    and may produce wrong results.  Order them on one stream.
 * Arguments and results are those of pspml_fully_connected_s8 (device
 * pointers, asynchronous on `stream`). */
int pspml_fully_connected_s8_noalloc(const pspml_op_desc* d, int64_t batch,
                                     const int8_t* in, const int8_t* filter,
                                     const int32_t* bias, const int32_t* mult,
                                     const int32_t* shift, int8_t* out,
                                     void* stream);
/* Reads and clears the error word of pspml_fully_connected_s8_noalloc on
 * the current device (the counterpart of pspml_ctx_check_device for that
 * entry point, which has no context): PSPML_ERR_DEVICE_WAIT if one of its
 * kernels gave up on a bounded wait since the last check.  Synchronous;
 * allocates nothing.  No counterpart in the reference. */
int pspml_noalloc_check_device(void);

/* Replaces naive::max_pool2d (naive.rs:98-132); any window and stride. */
int pspml_max_pool2d_s8(pspml_ctx* ctx, const pspml_op_desc* d, int64_t batch,
                        const int8_t* in, int8_t* out, void* stream);

/* AVERAGE_POOL_2D (rejected by the reference); global pooling is the
 * window == input case. */
int pspml_average_pool2d_s8(pspml_ctx* ctx, const pspml_op_desc* d,
                            int64_t batch, const int8_t* in, int8_t* out,
                            void* stream);

/* ---- f32 ops: the reference's own MNIST path, bit-identical to it ------
 * NHWC float tensors, device pointers, asynchronous on `stream`.  Every
 * output is one sequence of separately rounded products and sums in the
 * reference's order (no fused multiply-add), so results equal the
 * reference's exactly.  Bits of pspml_op_desc.flags: */
#define PSPML_F32_RELU 1       /* then `if (v < 0) v = 0` (keeps -0.0)      */
#define PSPML_F32_GEMM_ORDER 2 /* conv: im2col_padded -> matmul_bt_tiled ->
                                  bias_add order (psp-ml/src/kernels/
                                  mod.rs:176-479, what the reference's
                                  codegen emits): the sum starts at 0, runs
                                  over k in (ky, kx, ci) order including
                                  out-of-image taps (as 0) and the zero
                                  columns up to a multiple of 4, then adds
                                  the bias.  Without it: naive::conv2d
                                  (naive.rs:13-92), the sum starts at the
                                  bias and skips out-of-image taps.        */

/* Replaces the reference's conv lowering (mod.rs:176-479 with
 * PSPML_F32_GEMM_ORDER) or naive::conv2d[_relu] (naive.rs:13-92).
 * filter [out_c][kernel_h][kernel_w][in_c]; bias [out_c] or NULL. */
int pspml_conv2d_f32(pspml_ctx* ctx, const pspml_op_desc* d, int64_t batch,
                     const float* in, const float* filter, const float* bias,
                     float* out, void* stream);

/* Replaces naive::max_pool2d (naive.rs:98-132): -inf start, strict `>`. */
int pspml_max_pool2d_f32(pspml_ctx* ctx, const pspml_op_desc* d, int64_t batch,
                         const float* in, float* out, void* stream);

/* Replaces naive::fully_connected[_relu] (naive.rs:147-184): the sum starts
 * at bias[o] and adds the inputs in order.  filter [out_c][in_h*in_w*in_c]. */
int pspml_fully_connected_f32(pspml_ctx* ctx, const pspml_op_desc* d,
                              int64_t batch, const float* in,
                              const float* filter, const float* bias,
                              float* out, void* stream);

/* ------------------------------------------------------------ model level
 * The compiled-model counterpart of the generated forward()
 * (generated.rs:8-137): an op chain whose constants live at offsets in one
 * weight blob, as TensorKind::Constant{offset,len} does in the reference
 * (cargo-psp-ml/src/ir/graph.rs:22-31).  The model uploads and prepares the
 * weights once and plans one device arena for the intermediates by
 * liveness (the reference gives every intermediate its own static buffer,
 * render.rs:153-180). */

/* ops[0] consumes the model input, ops[i] consumes ops[i-1]'s output and the
 * last op produces the model output.  max_micro_batch bounds the arena. */
int pspml_model_create(pspml_ctx* ctx, const pspml_op_desc* ops, int32_t n_ops,
                       const void* blob, size_t blob_bytes,
                       int32_t max_micro_batch, pspml_model** out);
int pspml_model_destroy(pspml_model* m);
/* Bytes per sample of the model input and output; arena bytes in use. */
int pspml_model_info(const pspml_model* m, size_t* in_bytes_per_sample,
                     size_t* out_bytes_per_sample, size_t* arena_bytes);

/* How op `op` runs (no counterpart in the reference, whose ops are one call
 * each): *fused = 0 on its own, 1 if its kernel also computes op + 1 (a
 * depthwise conv fused with the 1x1 conv after it), 2 if op - 1's kernel
 * computes it.  Per-op times of pspml_forward_timed put a fused pair's time
 * on the first op. */
int pspml_model_op_fused(const pspml_model* m, int32_t op, int32_t* fused);

/* Device-resident forward: `batch` samples from dev_in to dev_out,
 * micro-batched, asynchronous on `stream`. */
int pspml_forward_device(pspml_model* m, const int8_t* dev_in, int8_t* dev_out,
                         int64_t batch, void* stream);

/* Host-buffer forward: copies in, runs and copies out with the three
 * overlapped per micro-batch; returns when host_out is complete.
 * Replaces generated::forward (generated.rs:8) for a batch. */
int pspml_forward(pspml_model* m, const int8_t* host_in, int8_t* host_out,
                  int64_t batch, pspml_timing* timing);

/* Host-buffer forward sharded by contiguous batch slices over several
 * models (one per device, one host thread each), no collective: every
 * device writes its disjoint slice of host_out.  A device whose shard fails
 * is dropped for the call and its slice re-run, split over the devices that
 * succeeded (timing->rerun_shards counts them); the call fails only when
 * no device succeeded, a re-run fails, or a shard timed out (its device may
 * still be writing its slice, so it is not re-run). */
int pspml_forward_sharded(pspml_model* const* models, int32_t n_models,
                          const int8_t* host_in, int8_t* host_out,
                          int64_t batch, pspml_timing* timing);

/* Host-side failure injection for testing the error paths (no
 * counterpart in the reference): the next `count` forward calls on `m`
 * return `status` (a PSPML_ERR_* code) without touching the GPU. */
int pspml_model_fail_next(pspml_model* m, int32_t count, int32_t status);

/* Timed variant, replacing generated::forward_timed (generated.rs:139-294):
 * a device-resident forward of `batch` samples (micro-batched like
 * pspml_forward_device) with CUDA events around every op; stores each op's
 * device time, summed over the micro-batches, in ms_per_op[n_ops].  Returns
 * when the work is done. */
int pspml_forward_timed(pspml_model* m, const int8_t* dev_in, int8_t* dev_out,
                        int64_t batch, float* ms_per_op, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PSPML_H */
