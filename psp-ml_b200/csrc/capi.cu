// capi.cu - C ABI: errors, contexts, pinned host memory, per-op int8 calls
// and TMA descriptor encoding.
#include <cudaTypedefs.h>

#include <chrono>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>

#include "kernels.h"
#include "ptx.cuh"
#include "runtime.h"

namespace pspml {

namespace {
thread_local std::string g_last_error;

// One thread waits, with the bounded wait every tensor-core kernel uses, on
// an mbarrier that it arrives on only when `signal` is set; an unsignalled
// wait runs out after limit_ns and records kDevErrSelfTest in the error
// word, exactly as a kernel whose TMA or MMA never completed would.
__global__ void k_wait_selftest(unsigned* err, uint64_t limit_ns, int32_t signal) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    if (signal) mbar_arrive(&bar);
    if (!mbar_wait(&bar, 0, nullptr, limit_ns)) atomicCAS(err, 0u, kDevErrSelfTest);
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
}  // namespace

int set_error(int status, const std::string& msg) {
  g_last_error = msg;
  return status;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return PSPML_OK;
  cudaGetLastError();  // clear sticky-free errors so the next call starts clean
  return set_error(e == cudaErrorMemoryAllocation ? PSPML_ERR_OOM : PSPML_ERR_CUDA,
                   std::string(what) + ": " + cudaGetErrorString(e));
}

void clear_error() { g_last_error.clear(); }

int validate_desc(const pspml_op_desc* d) {
  if (d == nullptr) return set_error(PSPML_ERR_INVALID_ARG, "null op descriptor");
  if (d->in_h <= 0 || d->in_w <= 0 || d->in_c <= 0 || d->out_h <= 0 || d->out_w <= 0 ||
      d->out_c <= 0)
    return set_error(PSPML_ERR_INVALID_ARG, "non-positive tensor dimension");
  if (d->zp_in < -128 || d->zp_in > 127 || d->zp_out < -128 || d->zp_out > 127)
    return set_error(PSPML_ERR_INVALID_ARG, "zero point outside int8");
  if (d->act_min < -128 || d->act_max > 127 || d->act_min > d->act_max)
    return set_error(PSPML_ERR_INVALID_ARG, "bad activation range");
  const bool windowed = d->kind == PSPML_OP_CONV2D || d->kind == PSPML_OP_DEPTHWISE_CONV2D ||
                        d->kind == PSPML_OP_MAX_POOL2D || d->kind == PSPML_OP_AVERAGE_POOL2D;
  if (windowed) {
    if (d->kernel_h <= 0 || d->kernel_w <= 0 || d->stride_h <= 0 || d->stride_w <= 0 ||
        d->pad_top < 0 || d->pad_left < 0 || d->pad_bottom < 0 || d->pad_right < 0)
      return set_error(PSPML_ERR_INVALID_ARG, "bad kernel / stride / padding");
    const int64_t eh = (static_cast<int64_t>(d->in_h) + d->pad_top + d->pad_bottom -
                        d->kernel_h) / d->stride_h + 1;
    const int64_t ew = (static_cast<int64_t>(d->in_w) + d->pad_left + d->pad_right -
                        d->kernel_w) / d->stride_w + 1;
    if (eh != d->out_h || ew != d->out_w)
      return set_error(PSPML_ERR_INVALID_ARG,
                       "output size does not match input, kernel, stride and padding");
  }
  switch (d->kind) {
    case PSPML_OP_CONV2D:
      break;
    case PSPML_OP_DEPTHWISE_CONV2D:
      if (d->out_c != d->in_c)
        return set_error(PSPML_ERR_UNSUPPORTED, "depthwise conv needs depth multiplier 1");
      break;
    case PSPML_OP_FULLY_CONNECTED:
      if (d->out_h != 1 || d->out_w != 1)
        return set_error(PSPML_ERR_INVALID_ARG, "fully connected output must be [1,1,N]");
      break;
    case PSPML_OP_MAX_POOL2D:
    case PSPML_OP_AVERAGE_POOL2D:
      if (d->out_c != d->in_c || d->zp_out != d->zp_in)
        return set_error(PSPML_ERR_INVALID_ARG, "pooling keeps channels and quantisation");
      // Padding narrower than the window on every side keeps at least one
      // input element in every window (an average over none is undefined).
      if (d->pad_top >= d->kernel_h || d->pad_bottom >= d->kernel_h ||
          d->pad_left >= d->kernel_w || d->pad_right >= d->kernel_w)
        return set_error(PSPML_ERR_INVALID_ARG, "pooling padding must be narrower than the window");
      break;
    case PSPML_OP_RESHAPE:
      if (static_cast<int64_t>(d->in_h) * d->in_w * d->in_c !=
          static_cast<int64_t>(d->out_h) * d->out_w * d->out_c)
        return set_error(PSPML_ERR_INVALID_ARG, "reshape changes the element count");
      break;
    default:
      return set_error(PSPML_ERR_INVALID_ARG, "unknown op kind");
  }
  return PSPML_OK;
}

int wait_event(pspml_ctx* ctx, cudaEvent_t ev) {
  if (ctx->timeout_ms <= 0) return cuda_status(cudaEventSynchronize(ev), "cudaEventSynchronize");
  const auto deadline =
      std::chrono::steady_clock::now() + std::chrono::milliseconds(ctx->timeout_ms);
  while (true) {
    const cudaError_t e = cudaEventQuery(ev);
    if (e == cudaSuccess) return PSPML_OK;
    if (e != cudaErrorNotReady) return cuda_status(e, "cudaEventQuery");
    if (std::chrono::steady_clock::now() > deadline)
      return set_error(PSPML_ERR_TIMEOUT, "device work did not finish before the deadline");
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

CUresult encode_tensor_map(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                           const uint64_t* strides_bytes, const uint32_t* box,
                           const uint32_t* elem_strides, CUtensorMapSwizzle swizzle) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  if (fn == nullptr) return CUDA_ERROR_NOT_FOUND;
  cuuint64_t d[5];
  cuuint64_t st[4];
  cuuint32_t b[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = elem_strides[i];
    if (i + 1 < rank) st[i] = strides_bytes[i];
  }
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, static_cast<cuuint32_t>(rank),
            const_cast<void*>(base), d, st, b, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

// Stateless op call: prepares the op's derived tables in the context
// workspace (ordered on `s` before the op itself) and launches it.
int run_op_stateless(pspml_ctx* ctx, const pspml_op_desc* d, int64_t batch, const int8_t* in,
                     const int8_t* filter, const int32_t* bias, const int32_t* mult,
                     const int32_t* shift, int8_t* out, cudaStream_t s) {
  const bool al = aligned16(in) && aligned16(out) && (filter == nullptr || aligned16(filter));
  OpPath path = choose_path(*d, al);
  size_t need = prepared_bytes(*d, path);
  if (path == OpPath::kTc4d && need == 0) {  // too many border classes for the tables
    path = OpPath::kDirect;
    need = prepared_bytes(*d, path);
  }
  if (need > ctx->workspace_bytes)
    return set_error(PSPML_ERR_OOM, "context workspace too small for this op's tables");
  PreparedOp p;
  int st = cuda_status(prepare_op(*d, path, filter, bias, mult, shift, ctx->workspace, &p, s),
                       "op preparation");
  if (st) return st;
  return cuda_status(launch_op(*d, p, batch, in, out, ctx->dev_err, ctx->num_sms, s),
                     "op launch");
}

int check_op_ptrs(const pspml_ctx* ctx, const void* in, const void* out, int64_t batch) {
  if (ctx == nullptr) return set_error(PSPML_ERR_INVALID_ARG, "null context");
  if (in == nullptr || out == nullptr) return set_error(PSPML_ERR_INVALID_ARG, "null tensor");
  if (batch < 0) return set_error(PSPML_ERR_INVALID_ARG, "negative batch");
  return PSPML_OK;
}

int check_weight_ptrs(const void* filter, const void* mult, const void* shift) {
  if (filter == nullptr || mult == nullptr || shift == nullptr)
    return set_error(PSPML_ERR_INVALID_ARG, "null filter / multiplier / shift");
  return PSPML_OK;
}

}  // namespace pspml

using namespace pspml;

extern "C" {

const char* pspml_last_error(void) { return g_last_error.c_str(); }

int32_t pspml_abi_version(void) { return PSPML_ABI_VERSION; }

int pspml_device_count(int* count) {
  if (count == nullptr) return set_error(PSPML_ERR_INVALID_ARG, "null count");
  *count = 0;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return PSPML_OK;
  }
  int ok = 0;
  for (int i = 0; i < n; ++i) {
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, i) == cudaSuccess && p.major == 10 && p.minor == 0) ++ok;
  }
  *count = ok;
  return PSPML_OK;
}

int pspml_ctx_create(int device, size_t workspace_bytes, pspml_ctx** out) {
  clear_error();
  if (out == nullptr) return set_error(PSPML_ERR_INVALID_ARG, "null output pointer");
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
    cudaGetLastError();
    return set_error(PSPML_ERR_NO_DEVICE, "no such CUDA device");
  }
  cudaDeviceProp prop;
  int st = cuda_status(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
  if (st) return st;
  if (prop.major != 10 || prop.minor != 0)
    return set_error(PSPML_ERR_NO_DEVICE, "device is not sm_100 (B200 class)");
  st = cuda_status(cudaSetDevice(device), "cudaSetDevice");
  if (st) return st;
  auto* ctx = new pspml_ctx();
  ctx->device = device;
  ctx->num_sms = prop.multiProcessorCount;
  ctx->workspace_bytes = workspace_bytes ? workspace_bytes : (64u << 20);
  st = cuda_status(cudaMalloc(&ctx->dev_err, 256), "cudaMalloc(error word)");
  if (!st)
    st = cuda_status(cudaMalloc(&ctx->workspace, ctx->workspace_bytes), "cudaMalloc(workspace)");
  if (!st)
    st = cuda_status(cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking),
                     "cudaStreamCreate");
  // Cleared on the context's own stream and waited for: a plain cudaMemset
  // runs on the legacy default stream, which non-blocking streams do not
  // wait for.
  if (!st) st = cuda_status(cudaMemsetAsync(ctx->dev_err, 0, 256, ctx->stream), "cudaMemset");
  if (!st) st = cuda_status(cudaStreamSynchronize(ctx->stream), "cudaMemset");
  if (st) {
    pspml_ctx_destroy(ctx);
    return st;
  }
  *out = ctx;
  return PSPML_OK;
}

int pspml_ctx_destroy(pspml_ctx* ctx) {
  if (ctx == nullptr) return PSPML_OK;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamDestroy(ctx->stream);
  if (ctx->workspace) cudaFree(ctx->workspace);
  if (ctx->dev_err) cudaFree(ctx->dev_err);
  delete ctx;
  return PSPML_OK;
}

int pspml_ctx_set_timeout_ms(pspml_ctx* ctx, int64_t timeout_ms) {
  if (ctx == nullptr || timeout_ms < 0) return set_error(PSPML_ERR_INVALID_ARG, "bad argument");
  ctx->timeout_ms = timeout_ms;
  return PSPML_OK;
}

int pspml_ctx_check_device(pspml_ctx* ctx) {
  if (ctx == nullptr) return set_error(PSPML_ERR_INVALID_ARG, "null context");
  cudaSetDevice(ctx->device);
  unsigned v = 0;
  int st = cuda_status(cudaMemcpy(&v, ctx->dev_err, sizeof(v), cudaMemcpyDeviceToHost),
                       "read device error word");
  if (st) return st;
  if (v != 0) {
    cudaMemsetAsync(ctx->dev_err, 0, sizeof(unsigned), ctx->stream);
    cudaStreamSynchronize(ctx->stream);
    char buf[96];
    std::snprintf(buf, sizeof(buf), "a kernel gave up on a bounded wait (code %u)", v);
    return set_error(PSPML_ERR_DEVICE_WAIT, buf);
  }
  return PSPML_OK;
}

int pspml_ctx_wait_selftest(pspml_ctx* ctx, int64_t limit_us, int32_t signal) {
  clear_error();
  if (ctx == nullptr) return set_error(PSPML_ERR_INVALID_ARG, "null context");
  if (limit_us < 1 || limit_us > 10000000)
    return set_error(PSPML_ERR_INVALID_ARG, "wait limit must be 1 us .. 10 s");
  int st = cuda_status(cudaSetDevice(ctx->device), "cudaSetDevice");
  if (st) return st;
  k_wait_selftest<<<1, 32, 0, ctx->stream>>>(ctx->dev_err, static_cast<uint64_t>(limit_us) * 1000u,
                                             signal);
  if ((st = cuda_status(cudaGetLastError(), "self-test launch"))) return st;
  return cuda_status(cudaStreamSynchronize(ctx->stream), "self-test");
}

int pspml_host_alloc(size_t bytes, void** out) {
  if (out == nullptr) return set_error(PSPML_ERR_INVALID_ARG, "null output pointer");
  *out = nullptr;
  if (bytes == 0) return PSPML_OK;
  return cuda_status(cudaMallocHost(out, bytes), "cudaMallocHost");
}

int pspml_host_free(void* p) {
  if (p == nullptr) return PSPML_OK;
  return cuda_status(cudaFreeHost(p), "cudaFreeHost");
}

int pspml_conv2d_s8(pspml_ctx* ctx, const pspml_op_desc* d, int64_t batch, const int8_t* in,
                    const int8_t* filter, const int32_t* bias, const int32_t* mult,
                    const int32_t* shift, int8_t* out, void* stream) {
  clear_error();
  int st = validate_desc(d);
  if (st) return st;
  if (d->kind != PSPML_OP_CONV2D) return set_error(PSPML_ERR_INVALID_ARG, "not a CONV2D op");
  if ((st = check_op_ptrs(ctx, in, out, batch)) || (st = check_weight_ptrs(filter, mult, shift)))
    return st;
  if (batch == 0) return PSPML_OK;
  cudaSetDevice(ctx->device);
  return run_op_stateless(ctx, d, batch, in, filter, bias, mult, shift, out,
                          static_cast<cudaStream_t>(stream));
}

int pspml_depthwise_conv2d_s8(pspml_ctx* ctx, const pspml_op_desc* d, int64_t batch,
                              const int8_t* in, const int8_t* filter, const int32_t* bias,
                              const int32_t* mult, const int32_t* shift, int8_t* out,
                              void* stream) {
  clear_error();
  int st = validate_desc(d);
  if (st) return st;
  if (d->kind != PSPML_OP_DEPTHWISE_CONV2D)
    return set_error(PSPML_ERR_INVALID_ARG, "not a DEPTHWISE_CONV2D op");
  if ((st = check_op_ptrs(ctx, in, out, batch)) || (st = check_weight_ptrs(filter, mult, shift)))
    return st;
  if (batch == 0) return PSPML_OK;
  cudaSetDevice(ctx->device);
  return run_op_stateless(ctx, d, batch, in, filter, bias, mult, shift, out,
                          static_cast<cudaStream_t>(stream));
}

int pspml_fully_connected_s8(pspml_ctx* ctx, const pspml_op_desc* d, int64_t batch,
                             const int8_t* in, const int8_t* filter, const int32_t* bias,
                             const int32_t* mult, const int32_t* shift, int8_t* out,
                             void* stream) {
  clear_error();
  int st = validate_desc(d);
  if (st) return st;
  if (d->kind != PSPML_OP_FULLY_CONNECTED)
    return set_error(PSPML_ERR_INVALID_ARG, "not a FULLY_CONNECTED op");
  if ((st = check_op_ptrs(ctx, in, out, batch)) || (st = check_weight_ptrs(filter, mult, shift)))
    return st;
  if (batch == 0) return PSPML_OK;
  cudaSetDevice(ctx->device);
  return run_op_stateless(ctx, d, batch, in, filter, bias, mult, shift, out,
                          static_cast<cudaStream_t>(stream));
}

int pspml_max_pool2d_s8(pspml_ctx* ctx, const pspml_op_desc* d, int64_t batch, const int8_t* in,
                        int8_t* out, void* stream) {
  clear_error();
  int st = validate_desc(d);
  if (st) return st;
  if (d->kind != PSPML_OP_MAX_POOL2D) return set_error(PSPML_ERR_INVALID_ARG, "not MAX_POOL2D");
  if ((st = check_op_ptrs(ctx, in, out, batch))) return st;
  if (batch == 0) return PSPML_OK;
  cudaSetDevice(ctx->device);
  return cuda_status(launch_maxpool(*d, batch, in, out, static_cast<cudaStream_t>(stream)),
                     "max pool");
}

int pspml_average_pool2d_s8(pspml_ctx* ctx, const pspml_op_desc* d, int64_t batch,
                            const int8_t* in, int8_t* out, void* stream) {
  clear_error();
  int st = validate_desc(d);
  if (st) return st;
  if (d->kind != PSPML_OP_AVERAGE_POOL2D)
    return set_error(PSPML_ERR_INVALID_ARG, "not AVERAGE_POOL2D");
  if ((st = check_op_ptrs(ctx, in, out, batch))) return st;
  if (batch == 0) return PSPML_OK;
  cudaSetDevice(ctx->device);
  return cuda_status(launch_avgpool(*d, batch, in, out, static_cast<cudaStream_t>(stream)),
                     "average pool");
}

// ---- f32 ops (the reference's own MNIST path)

int pspml_conv2d_f32(pspml_ctx* ctx, const pspml_op_desc* d, int64_t batch, const float* in,
                     const float* filter, const float* bias, float* out, void* stream) {
  clear_error();
  int st = validate_desc(d);
  if (st) return st;
  if (d->kind != PSPML_OP_CONV2D) return set_error(PSPML_ERR_INVALID_ARG, "not a CONV2D op");
  if ((st = check_op_ptrs(ctx, in, out, batch))) return st;
  if (filter == nullptr) return set_error(PSPML_ERR_INVALID_ARG, "null filter");
  if (batch == 0) return PSPML_OK;
  cudaSetDevice(ctx->device);
  return cuda_status(
      launch_conv2d_f32(*d, batch, in, filter, bias, out, static_cast<cudaStream_t>(stream)),
      "f32 conv");
}

int pspml_max_pool2d_f32(pspml_ctx* ctx, const pspml_op_desc* d, int64_t batch, const float* in,
                         float* out, void* stream) {
  clear_error();
  int st = validate_desc(d);
  if (st) return st;
  if (d->kind != PSPML_OP_MAX_POOL2D) return set_error(PSPML_ERR_INVALID_ARG, "not MAX_POOL2D");
  if ((st = check_op_ptrs(ctx, in, out, batch))) return st;
  if (batch == 0) return PSPML_OK;
  cudaSetDevice(ctx->device);
  return cuda_status(launch_max_pool2d_f32(*d, batch, in, out, static_cast<cudaStream_t>(stream)),
                     "f32 max pool");
}

int pspml_fully_connected_f32(pspml_ctx* ctx, const pspml_op_desc* d, int64_t batch,
                              const float* in, const float* filter, const float* bias,
                              float* out, void* stream) {
  clear_error();
  int st = validate_desc(d);
  if (st) return st;
  if (d->kind != PSPML_OP_FULLY_CONNECTED)
    return set_error(PSPML_ERR_INVALID_ARG, "not a FULLY_CONNECTED op");
  if ((st = check_op_ptrs(ctx, in, out, batch))) return st;
  if (filter == nullptr) return set_error(PSPML_ERR_INVALID_ARG, "null filter");
  if (batch == 0) return PSPML_OK;
  cudaSetDevice(ctx->device);
  return cuda_status(launch_fully_connected_f32(*d, batch, in, filter, bias, out,
                                                static_cast<cudaStream_t>(stream)),
                     "f32 fully connected");
}

}  // extern "C"
