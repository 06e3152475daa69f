// noalloc.cu - the fully-connected int8 op without any device allocation.
//
// Some callers cannot allocate device memory at all: code that runs while a
// CUDA graph is being captured (cudaMalloc is not a capturable operation),
// inference hosts whose memory budget is fixed when the process starts and
// may not grow (allocations can fail or block mid-serving), and callers
// that hand this library only pointers they already own (an allocator of
// their own, a pool shared with other work).  pspml_fully_connected_s8
// needs a context, and creating one allocates its workspace.  This entry
// point needs neither: its scratch (the folded biases, the requantisation
// table and the device error word) is a fixed array compiled into the
// library, present on every device that loads it until the process exits.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "kernels.h"
#include "runtime.h"

namespace pspml {
namespace {

// Scratch for one FC op's prepared tables: folded bias (4 B per output
// channel) and requantisation entries (16 B per channel plus one flag),
// each rounded up to 256 B.  256 KiB covers up to 13000 output channels.
constexpr size_t kNoAllocScratchBytes = 256 * 1024;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
static __device__ __align__(16) unsigned g_noalloc_err[4];

struct DeviceScratch {
  bool ready = false;
  uint8_t* scratch = nullptr;  // device address of g_noalloc_scratch on this device
  unsigned* err = nullptr;     // device address of g_noalloc_err
  int num_sms = 0;
};
constexpr int kMaxDevices = 64;
DeviceScratch g_devices[kMaxDevices];
std::mutex g_setup_mu;

// Looks the arrays' device addresses up once per device (the host-side
// names are only stand-ins, never device addresses).  Must run with `dev`
// current; it issues no allocation.  Nothing needs clearing here: a
// __device__ array starts at zero when the module loads, and
// pspml_noalloc_check_device clears the error word whenever it reads it.
int setup_device(int dev, DeviceScratch** out) {
  if (dev < 0 || dev >= kMaxDevices) return set_error(PSPML_ERR_NO_DEVICE, "device index too large");
  std::lock_guard<std::mutex> lock(g_setup_mu);
  DeviceScratch& d = g_devices[dev];
  if (!d.ready) {
    void* p = nullptr;
    int st = cuda_status(cudaGetSymbolAddress(&p, g_noalloc_scratch),
                         "cudaGetSymbolAddress(no-alloc scratch)");
    if (st) return st;
    d.scratch = static_cast<uint8_t*>(p);
    st = cuda_status(cudaGetSymbolAddress(&p, g_noalloc_err), "cudaGetSymbolAddress(error word)");
    if (st) return st;
    d.err = static_cast<unsigned*>(p);
    st = cuda_status(cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev),
                     "cudaDeviceGetAttribute");
    if (st) return st;
    d.ready = true;
  }
  *out = &d;
  return PSPML_OK;
}

}  // namespace
}  // namespace pspml

using namespace pspml;

extern "C" int pspml_fully_connected_s8_noalloc(const pspml_op_desc* d, int64_t batch,
                                                const int8_t* in, const int8_t* filter,
                                                const int32_t* bias, const int32_t* mult,
                                                const int32_t* shift, int8_t* out,
                                                void* stream) {
  clear_error();
  int st = validate_desc(d);
  if (st) return st;
  if (d->kind != PSPML_OP_FULLY_CONNECTED)
    return set_error(PSPML_ERR_INVALID_ARG, "not a FULLY_CONNECTED op");
  if (in == nullptr || out == nullptr || filter == nullptr || mult == nullptr ||
      shift == nullptr)
    return set_error(PSPML_ERR_INVALID_ARG, "null tensor");
  if (batch < 0) return set_error(PSPML_ERR_INVALID_ARG, "negative batch");
  const bool al = (reinterpret_cast<uintptr_t>(in) & 15u) == 0 &&
                  (reinterpret_cast<uintptr_t>(filter) & 15u) == 0;
  const OpPath path = choose_path(*d, al);
  const size_t need = prepared_bytes(*d, path);
  if (need > kNoAllocScratchBytes)
    return set_error(PSPML_ERR_INVALID_ARG,
                     "op needs " + std::to_string(need) + " bytes of scratch; the no-allocation "
                     "entry point has " + std::to_string(kNoAllocScratchBytes) +
                     " (about 13000 output channels at most)");
  if (batch == 0) return PSPML_OK;
  int dev = 0;
  st = cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
  if (st) return st;
  DeviceScratch* ds = nullptr;
  if ((st = setup_device(dev, &ds))) return st;
  auto s = static_cast<cudaStream_t>(stream);
  // prepare_op overwrites every table it uses (the all-fast flag is reset
  // with a memset on `s`), so nothing left by an earlier call is read.
  PreparedOp p;
  st = cuda_status(prepare_op(*d, path, filter, bias, mult, shift, ds->scratch, &p, s),
                   "op preparation");
  if (st) return st;
  return cuda_status(launch_op(*d, p, batch, in, out, ds->err, ds->num_sms, s), "op launch");
}

extern "C" int pspml_noalloc_check_device(void) {
  clear_error();
  unsigned v = 0;
  int st = cuda_status(cudaMemcpyFromSymbol(&v, g_noalloc_err, sizeof(v)),
                       "read no-allocation error word");
  if (st) return st;
  if (v == 0) return PSPML_OK;
  const unsigned zero = 0;
  st = cuda_status(cudaMemcpyToSymbol(g_noalloc_err, &zero, sizeof(zero)),
                   "clear no-allocation error word");
  // A copy from pageable memory may return before its DMA lands; wait for it
  // so that no later kernel's error code is cleared by it.
  if (!st)
    st = cuda_status(cudaStreamSynchronize(cudaStreamLegacy), "clear no-allocation error word");
  if (st) return st;
  return set_error(PSPML_ERR_DEVICE_WAIT,
                   "a no-allocation kernel gave up on a bounded wait (code " +
                       std::to_string(v) + ")");
}
