// f32.cu - the reference's own f32 kernels on the GPU, bit-exact.
//
// The reference runs one model itself: an f32 MNIST CNN (5x5 SAME convs with
// ReLU, 2x2 max pools, FC 784->64 ReLU, FC 64->10).  Its generated code
// lowers every conv to im2col_padded -> matmul_bt_tiled -> bias_add -> relu
// (psp-ml/src/kernels/mod.rs:176-479) and calls naive::max_pool2d and
// naive::fully_connected[_relu] (psp-ml/src/kernels/naive.rs:98-184); the
// naive conv (naive.rs:13-92) is its f32 semantic reference.  Each kernel
// here computes one output per thread in exactly the reference's summation
// order, with separately rounded multiplies and adds (no fused multiply-add),
// so the results are bit-identical to the reference's:
//   GEMM order   acc = 0; for k in [0, ceil4(KH*KW*Ci)): acc += a[k] * w[k]
//                (a = im2col row in (ky, kx, ci) order, 0 outside the image
//                and in the padding columns), then acc + bias, then ReLU
//   naive order  acc = bias; for (ky, kx) inside the image, ci: acc += x * w
//   max pool     m = -inf; for (ky, kx): if (v > m) m = v
//   FC           acc = bias; for i: acc += x[i] * w[o][i]; optional ReLU
// ReLU is `if (v < 0) v = 0`, which keeps -0.0.
#include <cuda_runtime.h>

#include <cmath>

#include "kernels.h"

namespace pspml {

namespace {

constexpr int kF32Block = 256;

struct F32Conv {
  int32_t H, W, Ci, Ho, Wo, Co, KH, KW, sh, sw, pt, pl;
  int32_t relu, gemm_order;
};

__device__ __forceinline__ float relu_keep_neg_zero(float v) { return v < 0.0f ? 0.0f : v; }

// One output (n, oy, ox, oc) per thread; weights [Co][KH][KW][Ci].
__global__ void k_conv2d_f32(const float* __restrict__ in, const float* __restrict__ w,
                             const float* __restrict__ bias, float* __restrict__ out,
                             const F32Conv g, int64_t total) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int oc = static_cast<int>(idx % g.Co);
  int64_t r = idx / g.Co;
  const int ox = static_cast<int>(r % g.Wo);
  r /= g.Wo;
  const int oy = static_cast<int>(r % g.Ho);
  const int64_t n = r / g.Ho;
  const float* img = in + n * static_cast<int64_t>(g.H) * g.W * g.Ci;
  const int K = g.KH * g.KW * g.Ci;
  const float* wo = w + static_cast<int64_t>(oc) * K;
  float acc;
  if (g.gemm_order) {
    // matmul_bt_tiled accumulates a zero-initialised tile over the padded K.
    acc = 0.0f;
    int k = 0;
    for (int ky = 0; ky < g.KH; ++ky) {
      const int iy = oy * g.sh + ky - g.pt;
      for (int kx = 0; kx < g.KW; ++kx) {
        const int ix = ox * g.sw + kx - g.pl;
        const bool inside = iy >= 0 && iy < g.H && ix >= 0 && ix < g.W;
        const float* px = img + (static_cast<int64_t>(inside ? iy : 0) * g.W + (inside ? ix : 0)) * g.Ci;
        for (int ci = 0; ci < g.Ci; ++ci, ++k) {
          const float a = inside ? px[ci] : 0.0f;
          acc = __fadd_rn(acc, __fmul_rn(a, wo[k]));
        }
      }
    }
    // Padding columns up to a multiple of 4: both operands are zero.
    for (; k < (K + 3) / 4 * 4; ++k) acc = __fadd_rn(acc, __fmul_rn(0.0f, 0.0f));
    if (bias != nullptr) acc = __fadd_rn(acc, bias[oc]);
  } else {
    acc = bias != nullptr ? bias[oc] : 0.0f;
    for (int ky = 0; ky < g.KH; ++ky) {
      const int iy = oy * g.sh + ky - g.pt;
      if (iy < 0 || iy >= g.H) continue;
      for (int kx = 0; kx < g.KW; ++kx) {
        const int ix = ox * g.sw + kx - g.pl;
        if (ix < 0 || ix >= g.W) continue;
        const float* px = img + (static_cast<int64_t>(iy) * g.W + ix) * g.Ci;
        const float* wk = wo + (ky * g.KW + kx) * g.Ci;
        for (int ci = 0; ci < g.Ci; ++ci) acc = __fadd_rn(acc, __fmul_rn(px[ci], wk[ci]));
      }
    }
  }
  out[idx] = g.relu ? relu_keep_neg_zero(acc) : acc;
}

__global__ void k_max_pool2d_f32(const float* __restrict__ in, float* __restrict__ out,
                                 const F32Conv g, int64_t total) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int c = static_cast<int>(idx % g.Co);
  int64_t r = idx / g.Co;
  const int ox = static_cast<int>(r % g.Wo);
  r /= g.Wo;
  const int oy = static_cast<int>(r % g.Ho);
  const int64_t n = r / g.Ho;
  const float* img = in + n * static_cast<int64_t>(g.H) * g.W * g.Ci;
  float m = -INFINITY;
  for (int ky = 0; ky < g.KH; ++ky) {
    const int iy = oy * g.sh + ky - g.pt;
    for (int kx = 0; kx < g.KW; ++kx) {
      const int ix = ox * g.sw + kx - g.pl;
      if (iy < 0 || iy >= g.H || ix < 0 || ix >= g.W) continue;
      const float v = img[(static_cast<int64_t>(iy) * g.W + ix) * g.Ci + c];
      if (v > m) m = v;
    }
  }
  out[idx] = m;
}

// One output (n, o) per thread: acc starts at bias[o], inputs in order.
__global__ void k_fully_connected_f32(const float* __restrict__ in, const float* __restrict__ w,
                                      const float* __restrict__ bias, float* __restrict__ out,
                                      int32_t K, int32_t N, int32_t relu, int64_t total) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int o = static_cast<int>(idx % N);
  const int64_t n = idx / N;
  const float* x = in + n * K;
  const float* wo = w + static_cast<int64_t>(o) * K;
  float acc = bias != nullptr ? bias[o] : 0.0f;
  for (int i = 0; i < K; ++i) acc = __fadd_rn(acc, __fmul_rn(x[i], wo[i]));
  out[idx] = relu ? relu_keep_neg_zero(acc) : acc;
}

F32Conv geom_f32(const pspml_op_desc& d) {
  F32Conv g;
  g.H = d.in_h;
  g.W = d.in_w;
  g.Ci = d.in_c;
  g.Ho = d.out_h;
  g.Wo = d.out_w;
  g.Co = d.out_c;
  g.KH = d.kernel_h;
  g.KW = d.kernel_w;
  g.sh = d.stride_h;
  g.sw = d.stride_w;
  g.pt = d.pad_top;
  g.pl = d.pad_left;
  g.relu = (d.flags & PSPML_F32_RELU) != 0;
  g.gemm_order = (d.flags & PSPML_F32_GEMM_ORDER) != 0;
  return g;
}

unsigned blocks_for(int64_t total) {
  return static_cast<unsigned>((total + kF32Block - 1) / kF32Block);
}

}  // namespace

cudaError_t launch_conv2d_f32(const pspml_op_desc& d, int64_t batch, const float* in,
                              const float* filter, const float* bias, float* out,
                              cudaStream_t s) {
  const int64_t total = batch * d.out_h * d.out_w * static_cast<int64_t>(d.out_c);
  if (total == 0) return cudaSuccess;
  if (blocks_for(total) > 0x7FFFFFFFu) return cudaErrorInvalidValue;
  k_conv2d_f32<<<blocks_for(total), kF32Block, 0, s>>>(in, filter, bias, out, geom_f32(d), total);
  return cudaGetLastError();
}

cudaError_t launch_max_pool2d_f32(const pspml_op_desc& d, int64_t batch, const float* in,
                                  float* out, cudaStream_t s) {
  const int64_t total = batch * d.out_h * d.out_w * static_cast<int64_t>(d.out_c);
  if (total == 0) return cudaSuccess;
  if (blocks_for(total) > 0x7FFFFFFFu) return cudaErrorInvalidValue;
  k_max_pool2d_f32<<<blocks_for(total), kF32Block, 0, s>>>(in, out, geom_f32(d), total);
  return cudaGetLastError();
}

cudaError_t launch_fully_connected_f32(const pspml_op_desc& d, int64_t batch, const float* in,
                                       const float* w, const float* bias, float* out,
                                       cudaStream_t s) {
  const int32_t K = d.in_h * d.in_w * d.in_c;
  const int64_t total = batch * static_cast<int64_t>(d.out_c);
  if (total == 0) return cudaSuccess;
  if (blocks_for(total) > 0x7FFFFFFFu) return cudaErrorInvalidValue;
  k_fully_connected_f32<<<blocks_for(total), kF32Block, 0, s>>>(
      in, w, bias, out, K, d.out_c, (d.flags & PSPML_F32_RELU) != 0, total);
  return cudaGetLastError();
}

}  // namespace pspml
