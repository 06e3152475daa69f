// cuda_core.cu - int8 kernels that run on the CUDA cores: depthwise conv,
// direct conv for channel counts the tensor-core path does not take, a
// warp-per-output FC, and max / average pooling.  All are NHWC with the
// TFLite requantisation fused in.
#include <algorithm>

#include "kernels.h"
#include "requant.cuh"

namespace pspml {

namespace {

constexpr int kBlock = 256;

struct Geom {
  int32_t H, W, C, Ho, Wo, Co, KH, KW, sh, sw, pt, pl;
  int32_t zp_in;
  ActParams ap;
};

Geom geom_of(const pspml_op_desc& d) {
  Geom g;
  g.H = d.in_h;
  g.W = d.in_w;
  g.C = d.in_c;
  g.Ho = d.out_h;
  g.Wo = d.out_w;
  g.Co = d.out_c;
  g.KH = d.kernel_h;
  g.KW = d.kernel_w;
  g.sh = d.stride_h;
  g.sw = d.stride_w;
  g.pt = d.pad_top;
  g.pl = d.pad_left;
  g.zp_in = d.zp_in;
  g.ap = ActParams{d.zp_out, d.act_min, d.act_max};
  return g;
}

unsigned grid_for(int64_t n) {
  return static_cast<unsigned>(std::max<int64_t>(1, (n + kBlock - 1) / kBlock));
}

// ----------------------------------------------------------- depthwise conv
// One thread per (sample, oy, ox, VEC channels).  Out-of-image taps are
// skipped (TFLite: padding is the real value zero).  filter [KH][KW][C].
template <int VEC>
__global__ void k_dwconv_s8(const int8_t* __restrict__ in, const int8_t* __restrict__ f,
                            const int32_t* __restrict__ bias, const int32_t* __restrict__ mult,
                            const int32_t* __restrict__ shift, int8_t* __restrict__ out,
                            const Geom g, int64_t total) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int cv = g.C / VEC;
  const int c0 = static_cast<int>(idx % cv) * VEC;
  const int64_t pix = idx / cv;
  const int ox = static_cast<int>(pix % g.Wo);
  const int oy = static_cast<int>((pix / g.Wo) % g.Ho);
  const int64_t n = pix / (static_cast<int64_t>(g.Wo) * g.Ho);
  int32_t acc[VEC];
#pragma unroll
  for (int j = 0; j < VEC; ++j) acc[j] = bias != nullptr ? __ldg(bias + c0 + j) : 0;
  const int iy0 = oy * g.sh - g.pt, ix0 = ox * g.sw - g.pl;
  const int8_t* img = in + n * g.H * g.W * static_cast<int64_t>(g.C);
  for (int ky = 0; ky < g.KH; ++ky) {
    const int iy = iy0 + ky;
    if (iy < 0 || iy >= g.H) continue;
    for (int kx = 0; kx < g.KW; ++kx) {
      const int ix = ix0 + kx;
      if (ix < 0 || ix >= g.W) continue;
      const int8_t* xp = img + (static_cast<int64_t>(iy) * g.W + ix) * g.C + c0;
      const int8_t* wp = f + (ky * g.KW + kx) * g.C + c0;
      if constexpr (VEC == 16) {
        const uint4 xv = __ldg(reinterpret_cast<const uint4*>(xp));
        const uint4 wv = __ldg(reinterpret_cast<const uint4*>(wp));
        const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
        const uint32_t ws[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int j = 0; j < 4; ++j)
            acc[4 * q + j] += (sbyte(xs[q], j) - g.zp_in) * sbyte(ws[q], j);
      } else if constexpr (VEC == 4) {
        const uint32_t xv = __ldg(reinterpret_cast<const uint32_t*>(xp));
        const uint32_t wv = __ldg(reinterpret_cast<const uint32_t*>(wp));
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[j] += (sbyte(xv, j) - g.zp_in) * sbyte(wv, j);
      } else {
        acc[0] += (static_cast<int32_t>(xp[0]) - g.zp_in) * static_cast<int32_t>(wp[0]);
      }
    }
  }
  int8_t* op = out + pix * g.C + c0;
  int32_t r[VEC];
#pragma unroll
  for (int j = 0; j < VEC; ++j)
    r[j] = finish_dev(acc[j], __ldg(mult + c0 + j), __ldg(shift + c0 + j), g.ap);
  if constexpr (VEC == 16) {
    *reinterpret_cast<uint4*>(op) =
        make_uint4(pack4_s8(r[0], r[1], r[2], r[3]), pack4_s8(r[4], r[5], r[6], r[7]),
                   pack4_s8(r[8], r[9], r[10], r[11]), pack4_s8(r[12], r[13], r[14], r[15]));
  } else if constexpr (VEC == 4) {
    *reinterpret_cast<uint32_t*>(op) = pack4_s8(r[0], r[1], r[2], r[3]);
  } else {
    op[0] = static_cast<int8_t>(r[0]);
  }
}

// ------------------------------------------------------------- direct conv
// One thread per (sample, oy, ox) and COB output channels (blockIdx.y picks
// the channel chunk).  The chunk's weights sit in shared memory as int32
// [K][COB] so the inner loop is a broadcast load and COB multiply-adds.
template <int COB>
__global__ void k_conv_direct_s8(const int8_t* __restrict__ in, const int8_t* __restrict__ f,
                                 const int32_t* __restrict__ bias,
                                 const int32_t* __restrict__ mult,
                                 const int32_t* __restrict__ shift, int8_t* __restrict__ out,
                                 const Geom g, int64_t pixels) {
  extern __shared__ int32_t sw[];
  const int K = g.KH * g.KW * g.C;
  const int co0 = blockIdx.y * COB;
  for (int i = threadIdx.x; i < K * COB; i += blockDim.x) {
    const int k = i / COB, j = i - (i / COB) * COB;
    const int co = co0 + j;
    sw[i] = co < g.Co ? static_cast<int32_t>(f[static_cast<int64_t>(co) * K + k]) : 0;
  }
  __syncthreads();
  const int64_t pix = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (pix >= pixels) return;
  const int ox = static_cast<int>(pix % g.Wo);
  const int oy = static_cast<int>((pix / g.Wo) % g.Ho);
  const int64_t n = pix / (static_cast<int64_t>(g.Wo) * g.Ho);
  int32_t acc[COB];
#pragma unroll
  for (int j = 0; j < COB; ++j)
    acc[j] = (bias != nullptr && co0 + j < g.Co) ? __ldg(bias + co0 + j) : 0;
  const int iy0 = oy * g.sh - g.pt, ix0 = ox * g.sw - g.pl;
  const int8_t* img = in + n * g.H * g.W * static_cast<int64_t>(g.C);
  for (int ky = 0; ky < g.KH; ++ky) {
    const int iy = iy0 + ky;
    if (iy < 0 || iy >= g.H) continue;
    for (int kx = 0; kx < g.KW; ++kx) {
      const int ix = ix0 + kx;
      if (ix < 0 || ix >= g.W) continue;
      const int8_t* xp = img + (static_cast<int64_t>(iy) * g.W + ix) * g.C;
      const int32_t* wr = sw + ((ky * g.KW + kx) * g.C) * COB;
      for (int ci = 0; ci < g.C; ++ci) {
        const int32_t x = static_cast<int32_t>(__ldg(xp + ci)) - g.zp_in;
#pragma unroll
        for (int j = 0; j < COB; ++j) acc[j] += x * wr[ci * COB + j];
      }
    }
  }
  int8_t* op = out + pix * g.Co + co0;
#pragma unroll
  for (int j = 0; j < COB; ++j)
    if (co0 + j < g.Co)
      op[j] = static_cast<int8_t>(
          finish_dev(acc[j], __ldg(mult + co0 + j), __ldg(shift + co0 + j), g.ap));
}

// --------------------------------------------------------------- FC (warp)
// One warp per (sample, output): strided dot product and a shuffle reduce.
__global__ void k_fc_warp_s8(const int8_t* __restrict__ in, const int8_t* __restrict__ f,
                             const int32_t* __restrict__ bias, const int32_t* __restrict__ mult,
                             const int32_t* __restrict__ shift, int8_t* __restrict__ out,
                             int64_t K, int32_t N, int64_t total, int32_t zp_in, ActParams ap) {
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= total) return;
  const int64_t b = w / N;
  const int32_t o = static_cast<int32_t>(w - b * N);
  const int8_t* x = in + b * K;
  const int8_t* wr = f + static_cast<int64_t>(o) * K;
  int32_t s = 0;
  for (int64_t k = lane; k < K; k += 32)
    s += (static_cast<int32_t>(x[k]) - zp_in) * static_cast<int32_t>(wr[k]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, off);
  if (lane == 0) {
    const int32_t acc = s + (bias != nullptr ? bias[o] : 0);
    out[b * N + o] = static_cast<int8_t>(finish_dev(acc, mult[o], shift[o], ap));
  }
}

// ----------------------------------------------------------------- pooling
// Max pool: one thread per (sample, oy, ox, VEC channels); the window is
// clipped to the image; the max starts at -128 and is then clamped.
template <int VEC>
__global__ void k_maxpool_s8(const int8_t* __restrict__ in, int8_t* __restrict__ out,
                             const Geom g, int64_t total) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int cv = g.C / VEC;
  const int c0 = static_cast<int>(idx % cv) * VEC;
  const int64_t pix = idx / cv;
  const int ox = static_cast<int>(pix % g.Wo);
  const int oy = static_cast<int>((pix / g.Wo) % g.Ho);
  const int64_t n = pix / (static_cast<int64_t>(g.Wo) * g.Ho);
  const int iy0 = oy * g.sh - g.pt, ix0 = ox * g.sw - g.pl;
  const int8_t* img = in + n * g.H * g.W * static_cast<int64_t>(g.C);
  constexpr int kWords = VEC >= 4 ? VEC / 4 : 1;
  uint32_t m[kWords];
  int32_t m1 = -128;
#pragma unroll
  for (int q = 0; q < kWords; ++q) m[q] = 0x80808080u;
  for (int ky = 0; ky < g.KH; ++ky) {
    const int iy = iy0 + ky;
    if (iy < 0 || iy >= g.H) continue;
    for (int kx = 0; kx < g.KW; ++kx) {
      const int ix = ix0 + kx;
      if (ix < 0 || ix >= g.W) continue;
      const int8_t* xp = img + (static_cast<int64_t>(iy) * g.W + ix) * g.C + c0;
      if constexpr (VEC == 16) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(xp));
        m[0] = __vmaxs4(m[0], v.x);
        m[1] = __vmaxs4(m[1], v.y);
        m[2] = __vmaxs4(m[2], v.z);
        m[3] = __vmaxs4(m[3], v.w);
      } else if constexpr (VEC == 4) {
        m[0] = __vmaxs4(m[0], __ldg(reinterpret_cast<const uint32_t*>(xp)));
      } else {
        m1 = max(m1, static_cast<int32_t>(xp[0]));
      }
    }
  }
  int8_t* op = out + pix * g.C + c0;
  if constexpr (VEC >= 4) {
    const uint32_t lo = (static_cast<uint32_t>(g.ap.act_min) & 0xFFu) * 0x01010101u;
    const uint32_t hi = (static_cast<uint32_t>(g.ap.act_max) & 0xFFu) * 0x01010101u;
#pragma unroll
    for (int q = 0; q < kWords; ++q) m[q] = __vmins4(__vmaxs4(m[q], lo), hi);
    if constexpr (VEC == 16)
      *reinterpret_cast<uint4*>(op) = make_uint4(m[0], m[1], m[2], m[3]);
    else
      *reinterpret_cast<uint32_t*>(op) = m[0];
  } else {
    m1 = max(m1, g.ap.act_min);
    m1 = min(m1, g.ap.act_max);
    op[0] = static_cast<int8_t>(m1);
  }
}

// Average pool: int32 sum of the in-image window, divided by the count with
// round-half-away-from-zero (TFLite), clamped.  One thread per (sample,
// oy, ox, 4 channels) or per channel when C % 4 != 0.
template <int VEC>
__global__ void k_avgpool_s8(const int8_t* __restrict__ in, int8_t* __restrict__ out,
                             const Geom g, int64_t total) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int cv = g.C / VEC;
  const int c0 = static_cast<int>(idx % cv) * VEC;
  const int64_t pix = idx / cv;
  const int ox = static_cast<int>(pix % g.Wo);
  const int oy = static_cast<int>((pix / g.Wo) % g.Ho);
  const int64_t n = pix / (static_cast<int64_t>(g.Wo) * g.Ho);
  const int iy0 = oy * g.sh - g.pt, ix0 = ox * g.sw - g.pl;
  const int8_t* img = in + n * g.H * g.W * static_cast<int64_t>(g.C);
  int32_t acc[VEC];
#pragma unroll
  for (int j = 0; j < VEC; ++j) acc[j] = 0;
  int32_t cnt = 0;
  for (int ky = 0; ky < g.KH; ++ky) {
    const int iy = iy0 + ky;
    if (iy < 0 || iy >= g.H) continue;
    for (int kx = 0; kx < g.KW; ++kx) {
      const int ix = ix0 + kx;
      if (ix < 0 || ix >= g.W) continue;
      const int8_t* xp = img + (static_cast<int64_t>(iy) * g.W + ix) * g.C + c0;
      if constexpr (VEC == 4) {
        const uint32_t v = __ldg(reinterpret_cast<const uint32_t*>(xp));
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[j] += sbyte(v, j);
      } else {
        acc[0] += xp[0];
      }
      ++cnt;
    }
  }
  int8_t* op = out + pix * g.C + c0;
  int32_t r[VEC];
#pragma unroll
  for (int j = 0; j < VEC; ++j) {
    int32_t a = acc[j];
    a = a > 0 ? (a + cnt / 2) / cnt : (a - cnt / 2) / cnt;
    a = max(a, g.ap.act_min);
    a = min(a, g.ap.act_max);
    r[j] = a;
  }
  if constexpr (VEC == 4)
    *reinterpret_cast<uint32_t*>(op) = pack4_s8(r[0], r[1], r[2], r[3]);
  else
    op[0] = static_cast<int8_t>(r[0]);
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

}  // namespace

cudaError_t launch_dwconv(const pspml_op_desc& d, int64_t batch, const int8_t* in,
                          const int8_t* filter, const int32_t* bias, const int32_t* mult,
                          const int32_t* shift, int8_t* out, cudaStream_t s) {
  const Geom g = geom_of(d);
  const int64_t pix = batch * g.Ho * g.Wo;
  if (g.C % 16 == 0 && aligned(in, 16) && aligned(out, 16) && aligned(filter, 16)) {
    const int64_t total = pix * (g.C / 16);
    k_dwconv_s8<16><<<grid_for(total), kBlock, 0, s>>>(in, filter, bias, mult, shift, out, g, total);
  } else if (g.C % 4 == 0 && aligned(in, 4) && aligned(out, 4) && aligned(filter, 4)) {
    const int64_t total = pix * (g.C / 4);
    k_dwconv_s8<4><<<grid_for(total), kBlock, 0, s>>>(in, filter, bias, mult, shift, out, g, total);
  } else {
    const int64_t total = pix * g.C;
    k_dwconv_s8<1><<<grid_for(total), kBlock, 0, s>>>(in, filter, bias, mult, shift, out, g, total);
  }
  return cudaGetLastError();
}

cudaError_t launch_conv_direct(const pspml_op_desc& d, int64_t batch, const int8_t* in,
                               const int8_t* filter, const int32_t* bias, const int32_t* mult,
                               const int32_t* shift, int8_t* out, cudaStream_t s) {
  const Geom g = geom_of(d);
  const int64_t pixels = batch * g.Ho * g.Wo;
  const int K = g.KH * g.KW * g.C;
  const int cob = g.Co >= 16 ? 16 : 8;
  const size_t smem = static_cast<size_t>(K) * cob * sizeof(int32_t);
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  const dim3 grid(grid_for(pixels), (g.Co + cob - 1) / cob);
  if (cob == 16) {
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(k_conv_direct_s8<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem));
    k_conv_direct_s8<16><<<grid, kBlock, smem, s>>>(in, filter, bias, mult, shift, out, g, pixels);
  } else {
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(k_conv_direct_s8<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem));
    k_conv_direct_s8<8><<<grid, kBlock, smem, s>>>(in, filter, bias, mult, shift, out, g, pixels);
  }
  return cudaGetLastError();
}

cudaError_t launch_fc_warp(const pspml_op_desc& d, int64_t batch, const int8_t* in,
                           const int8_t* filter, const int32_t* bias, const int32_t* mult,
                           const int32_t* shift, int8_t* out, cudaStream_t s) {
  const int64_t K = static_cast<int64_t>(d.in_h) * d.in_w * d.in_c;
  const int64_t total = batch * d.out_c;
  const int64_t threads = total * 32;
  k_fc_warp_s8<<<grid_for(threads), kBlock, 0, s>>>(in, filter, bias, mult, shift, out, K,
                                                   d.out_c, total, d.zp_in,
                                                   ActParams{d.zp_out, d.act_min, d.act_max});
  return cudaGetLastError();
}

cudaError_t launch_maxpool(const pspml_op_desc& d, int64_t batch, const int8_t* in,
                           int8_t* out, cudaStream_t s) {
  const Geom g = geom_of(d);
  const int64_t pix = batch * g.Ho * g.Wo;
  if (g.C % 16 == 0 && aligned(in, 16) && aligned(out, 16)) {
    const int64_t total = pix * (g.C / 16);
    k_maxpool_s8<16><<<grid_for(total), kBlock, 0, s>>>(in, out, g, total);
  } else if (g.C % 4 == 0 && aligned(in, 4) && aligned(out, 4)) {
    const int64_t total = pix * (g.C / 4);
    k_maxpool_s8<4><<<grid_for(total), kBlock, 0, s>>>(in, out, g, total);
  } else {
    const int64_t total = pix * g.C;
    k_maxpool_s8<1><<<grid_for(total), kBlock, 0, s>>>(in, out, g, total);
  }
  return cudaGetLastError();
}

cudaError_t launch_avgpool(const pspml_op_desc& d, int64_t batch, const int8_t* in,
                           int8_t* out, cudaStream_t s) {
  const Geom g = geom_of(d);
  const int64_t pix = batch * g.Ho * g.Wo;
  if (g.C % 4 == 0 && aligned(in, 4) && aligned(out, 4)) {
    const int64_t total = pix * (g.C / 4);
    k_avgpool_s8<4><<<grid_for(total), kBlock, 0, s>>>(in, out, g, total);
  } else {
    const int64_t total = pix * g.C;
    k_avgpool_s8<1><<<grid_for(total), kBlock, 0, s>>>(in, out, g, total);
  }
  return cudaGetLastError();
}

}  // namespace pspml
