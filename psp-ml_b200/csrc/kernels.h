// kernels.h - launchers for the device kernels (host side, C++).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/pspml.h"

namespace pspml {

// Folded epilogue tables for a conv / FC layer on the device:
//   bias_eff[cls][n] = bias[n] - zp_in * sum of w[n][tap][ci] over the taps
//   that lie inside the image for border class cls.
// Class cls = ycls[y] * n_xcls + xcls[x] for an output pixel (x, y); a FC or
// unpadded layer has one class.
struct FoldedBias {
  int32_t* bias_eff = nullptr;  // [ncls][N]
  uint8_t* ycls = nullptr;      // [Ho] (null when ncls == 1)
  uint8_t* xcls = nullptr;      // [Wo]
  int32_t ncls = 1;
  int32_t n_xcls = 1;
};

// Host-side description of the border classes of a stride-1 conv.
struct BorderClasses {
  int32_t n_ycls = 1, n_xcls = 1;
  uint32_t ymask[64] = {0};  // valid-ky bit mask per row class
  uint32_t xmask[64] = {0};  // valid-kx bit mask per column class
  uint8_t ycls[4096];        // class of each output row
  uint8_t xcls[4096];        // class of each output column
};

// Fills `bc` for op `d` (stride must be 1 when more than one class is
// possible).  Returns false if the geometry has too many classes.
bool build_border_classes(const pspml_op_desc& d, BorderClasses* bc);

// Device prep: bias_eff[cls][n] from raw weights/bias (filter in
// [N][KH][KW][Ci] layout, or [N][K] for FC which is one tap).
cudaError_t launch_fold_bias(const pspml_op_desc& d, const int8_t* filter, const int32_t* bias,
                             const BorderClasses& bc, int32_t* bias_eff, cudaStream_t s);

// Which implementation runs a conv / FC.
enum class GemmPath { kTc2d, kTc4d, kDirect, kFcWarp };
GemmPath choose_conv_path(const pspml_op_desc& d);
GemmPath choose_fc_path(const pspml_op_desc& d);

// tcgen05 GEMM (2D: rows x K times N x K; 4D: implicit stride-1 conv).
// `rows` is batch*Ho*Wo for a conv, batch for FC.
cudaError_t launch_tc_gemm(const pspml_op_desc& d, GemmPath path, int64_t batch,
                           const int8_t* in, const int8_t* filter, const FoldedBias& fb,
                           const int32_t* mult, const int32_t* shift, int8_t* out,
                           unsigned* dev_err, int num_sms, cudaStream_t s);

// CUDA-core direct conv (any stride / padding / channel count).
cudaError_t launch_conv_direct(const pspml_op_desc& d, int64_t batch, const int8_t* in,
                               const int8_t* filter, const int32_t* bias, const int32_t* mult,
                               const int32_t* shift, int8_t* out, cudaStream_t s);

// CUDA-core FC (one warp per output), for K not a multiple of 16.
cudaError_t launch_fc_warp(const pspml_op_desc& d, int64_t batch, const int8_t* in,
                           const int8_t* filter, const int32_t* bias, const int32_t* mult,
                           const int32_t* shift, int8_t* out, cudaStream_t s);

cudaError_t launch_dwconv(const pspml_op_desc& d, int64_t batch, const int8_t* in,
                          const int8_t* filter, const int32_t* bias, const int32_t* mult,
                          const int32_t* shift, int8_t* out, cudaStream_t s);

cudaError_t launch_maxpool(const pspml_op_desc& d, int64_t batch, const int8_t* in,
                           int8_t* out, cudaStream_t s);

cudaError_t launch_avgpool(const pspml_op_desc& d, int64_t batch, const int8_t* in,
                           int8_t* out, cudaStream_t s);

// Encodes a tiled TMA descriptor through the driver entry point.
CUresult encode_tensor_map(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                           const uint64_t* strides_bytes, const uint32_t* box,
                           const uint32_t* elem_strides, CUtensorMapSwizzle swizzle);

}  // namespace pspml
