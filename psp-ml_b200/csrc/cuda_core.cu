// cuda_core.cu - int8 kernels on the CUDA cores, NHWC, with the TFLite
// requantisation fused in:
//   k_dw3x3_s8       depthwise 3x3 (stride 1/2), dp4a over the three taps of a filter row
//   k_small_conv_s8  conv with few input channels (K <= 128) over packed patches
//   k_small_conv_tab_s8, k_stem_s2_s8  the 1 -> 32 channel 3x3 stem, constants
//                    as kernel-parameter operands / in registers
//   k_conv_direct_s8 any conv (fallback)
//   k_dw_generic_s8  any depthwise conv (fallback)
//   k_fc_warp_s8     FC with K % 16 != 0 (one warp per output)
//   k_maxpool_s8 / k_avgpool_s8
//
// The dp4a kernels accumulate sum(x * w) with out-of-image taps filled with
// the input zero point; the folded bias (bias - zp_in * sum(w)) makes that
// exactly TFLite's sum((x - zp_in) * w) + bias.
#include <algorithm>

#include "kernels.h"
#include "requant.cuh"

namespace pspml {

namespace {

constexpr int kBlock = 256;
constexpr int kMaxGridZ = 65535;

struct Geom {
  int32_t H, W, C, Ho, Wo, Co, KH, KW, sh, sw, pt, pl;
  int32_t zp_in;
  uint32_t lo4, hi4;
  int32_t clamp;
  int32_t act_min, act_max, zp_out;
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
  g.lo4 = splat4(d.act_min);
  g.hi4 = splat4(d.act_max);
  g.clamp = (d.act_min > -128 || d.act_max < 127) ? 1 : 0;
  g.act_min = d.act_min;
  g.act_max = d.act_max;
  g.zp_out = d.zp_out;
  return g;
}

unsigned grid_for(int64_t n) {
  return static_cast<unsigned>(std::max<int64_t>(1, (n + kBlock - 1) / kBlock));
}

template <int RQ = kRqGeneral>
__device__ __forceinline__ uint32_t finish4(int32_t a0, int32_t a1, int32_t a2, int32_t a3,
                                            const int4& b, const RqChannel& q0,
                                            const RqChannel& q1, const RqChannel& q2,
                                            const RqChannel& q3, const Geom& g) {
  uint32_t w = pack_sat4(rq_sel<RQ>(a0 + b.x, q0), rq_sel<RQ>(a1 + b.y, q1),
                         rq_sel<RQ>(a2 + b.z, q2), rq_sel<RQ>(a3 + b.w, q3));
  if (g.clamp) w = clamp4(w, g.lo4, g.hi4);
  return w;
}

__device__ __forceinline__ int8_t finish1(int32_t a, const RqChannel& q, const Geom& g) {
  int32_t r = rq_apply(a, q);
  r = max(r, -128);
  r = min(r, 127);
  uint32_t w = static_cast<uint32_t>(r) & 0xFFu;
  if (g.clamp) w = clamp4(w * 0x01010101u, g.lo4, g.hi4) & 0xFFu;
  return static_cast<int8_t>(w);
}

// ------------------------------------------------------ depthwise 3x3 (dp4a)
// Thread: 4 channels (one word) x PX consecutive output pixels x a strip of
// output rows (blockIdx.y).  Each input row the thread needs (NIN pixels of
// its 4 channels) is transposed once, with byte permutes, into per-channel
// words of 4 consecutive pixels; a dp4a of such a word (funnel-shifted to
// the output pixel's first tap) against the channel's packed row weights
// [w(ky,0), w(ky,1), w(ky,2), 0] is the three taps of one filter row, so an
// output costs three dp4a.  The thread keeps the three transposed rows of
// the current output row in registers and loads the S new rows of the next
// output row while it computes.  Block: 128 threads over (pixel group,
// channel word) pairs of one image (blockIdx.z + n_base).  Weights [9][C];
// out-of-image taps read zp_in.
template <int S, int PX, int RQ>
__global__ void __launch_bounds__(128)
    k_dw3x3_s8(const uint32_t* __restrict__ in, const uint32_t* __restrict__ f,
               const int32_t* __restrict__ bias_eff, const RqChannel* __restrict__ rq,
               uint32_t* __restrict__ out, const Geom g, int32_t rows_per, int64_t n_base) {
  constexpr int NIN = (PX - 1) * S + 3;  // input pixels of a row
  constexpr int NT = (NIN + 3) / 4;      // transposed words per channel
  const int cwn = g.C >> 2;
  const int pair = blockIdx.x * 128 + threadIdx.x;
  const int groups = (g.Wo + PX - 1) / PX;
  if (pair >= groups * cwn) return;
  const int cw = pair % cwn;
  const int pg = pair / cwn;
  const int oy0 = blockIdx.y * rows_per;
  const int oy1 = min(oy0 + rows_per, g.Ho);
  const int64_t n = n_base + blockIdx.z;
  const int ox0 = pg * PX;

  // wr[ky][c]: the three taps of filter row ky for channel c, byte kx.
  uint32_t wr[3][4];
#pragma unroll
  for (int ky = 0; ky < 3; ++ky) {
    const uint32_t t0 = __ldg(f + (3 * ky) * cwn + cw);
    const uint32_t t1 = __ldg(f + (3 * ky + 1) * cwn + cw);
    const uint32_t t2 = __ldg(f + (3 * ky + 2) * cwn + cw);
    const uint32_t lo01 = __byte_perm(t0, t1, 0x5140);  // t0.c0 t1.c0 t0.c1 t1.c1
    const uint32_t hi01 = __byte_perm(t0, t1, 0x7362);  // t0.c2 t1.c2 t0.c3 t1.c3
    wr[ky][0] = __byte_perm(lo01, t2, 0x0410) & 0x00FFFFFFu;
    wr[ky][1] = __byte_perm(lo01, t2, 0x0532) & 0x00FFFFFFu;
    wr[ky][2] = __byte_perm(hi01, t2, 0x0610) & 0x00FFFFFFu;
    wr[ky][3] = __byte_perm(hi01, t2, 0x0732) & 0x00FFFFFFu;
  }
  const int4 b = __ldg(reinterpret_cast<const int4*>(bias_eff) + cw);
  const RqChannel q0 = load_rq(rq + 4 * cw), q1 = load_rq(rq + 4 * cw + 1),
                  q2 = load_rq(rq + 4 * cw + 2), q3 = load_rq(rq + 4 * cw + 3);
  // Floor form with the bias and the rounding one folded into a 64-bit
  // addend per channel (the same integer as (acc + bias) * M + C + 2^32):
  // an output is one wide multiply-add and one shift, and the addend sits in
  // an aligned register pair for the whole strip.
  int64_t fd[4] = {0, 0, 0, 0};
  if constexpr (RQ == kRqFloor) {
    fd[0] = floor_addend(b.x, q0);
    fd[1] = floor_addend(b.y, q1);
    fd[2] = floor_addend(b.z, q2);
    fd[3] = floor_addend(b.w, q3);
  }

  const uint32_t zpw = splat4(g.zp_in);
  const int ix0 = ox0 * S - g.pl;
  const uint32_t* img = in + n * static_cast<int64_t>(g.H) * g.W * cwn + cw;
  auto load_row = [&](int iy, uint32_t (&x)[NIN]) {
    const bool row_ok = iy >= 0 && iy < g.H;
    const uint32_t* rowp = img + static_cast<int64_t>(row_ok ? iy : 0) * g.W * cwn;
#pragma unroll
    for (int c = 0; c < NIN; ++c) {
      const int ix = ix0 + c;
      x[c] = (row_ok && ix >= 0 && ix < g.W) ? __ldg(rowp + ix * cwn) : zpw;
    }
  };
  // Pixel-major words (4 channels each) -> channel-major words (4 pixels).
  auto transpose = [&](const uint32_t (&x)[NIN], uint32_t (&t)[4][NT]) {
#pragma unroll
    for (int k = 0; k < NT; ++k) {
      const uint32_t a = x[4 * k];
      const uint32_t bb = 4 * k + 1 < NIN ? x[4 * k + 1] : zpw;
      const uint32_t c = 4 * k + 2 < NIN ? x[4 * k + 2] : zpw;
      const uint32_t d = 4 * k + 3 < NIN ? x[4 * k + 3] : zpw;
      const uint32_t ab_lo = __byte_perm(a, bb, 0x5140);
      const uint32_t ab_hi = __byte_perm(a, bb, 0x7362);
      const uint32_t cd_lo = __byte_perm(c, d, 0x5140);
      const uint32_t cd_hi = __byte_perm(c, d, 0x7362);
      t[0][k] = __byte_perm(ab_lo, cd_lo, 0x5410);
      t[1][k] = __byte_perm(ab_lo, cd_lo, 0x7632);
      t[2][k] = __byte_perm(ab_hi, cd_hi, 0x5410);
      t[3][k] = __byte_perm(ab_hi, cd_hi, 0x7632);
    }
  };
  uint32_t t0[4][NT], t1[4][NT], t2[4][NT];
  {
    uint32_t x[NIN];
    const int iy0 = oy0 * S - g.pt;
    load_row(iy0, x);
    transpose(x, t0);
    load_row(iy0 + 1, x);
    transpose(x, t1);
    load_row(iy0 + 2, x);
    transpose(x, t2);
  }
  uint32_t* obase = out + (n * g.Ho) * static_cast<int64_t>(g.Wo) * cwn + cw;
#pragma unroll 1
  for (int oy = oy0; oy < oy1; ++oy) {
    // Rows of the next output row: input rows (oy+1)*S - pt + {0,1,2}, of
    // which the first 3 - S are already held.
    uint32_t p0[NIN], p1[NIN];
    const int niy = (oy + 1) * S - g.pt;
#pragma unroll
    for (int c = 0; c < NIN; ++c) p0[c] = p1[c] = zpw;
    if (oy + 1 < oy1) {
      if (S == 1) {
        load_row(niy + 2, p0);
      } else {
        load_row(niy + 1, p0);
        load_row(niy + 2, p1);
      }
    }
    uint32_t* orow = obase + static_cast<int64_t>(oy) * g.Wo * cwn;
#pragma unroll
    for (int p = 0; p < PX; ++p) {
      // Bytes S*p .. S*p+3 of a channel's transposed row.
      auto tap = [&](const uint32_t (&t)[NT]) -> uint32_t {
        const int off = S * p;
        if (off % 4 == 0) return t[off / 4];
        return __funnelshift_r(t[off / 4], t[off / 4 + 1], 8 * (off % 4));
      };
      int32_t acc[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        int32_t a = __dp4a(static_cast<int>(tap(t0[c])), static_cast<int>(wr[0][c]), 0);
        a = __dp4a(static_cast<int>(tap(t1[c])), static_cast<int>(wr[1][c]), a);
        acc[c] = __dp4a(static_cast<int>(tap(t2[c])), static_cast<int>(wr[2][c]), a);
      }
      if (ox0 + p < g.Wo) {
        uint32_t w;
        if constexpr (RQ == kRqFloor) {
          w = pack_sat4(rq_floor_folded(acc[0], q0.m, fd[0], q0.sr),
                        rq_floor_folded(acc[1], q1.m, fd[1], q1.sr),
                        rq_floor_folded(acc[2], q2.m, fd[2], q2.sr),
                        rq_floor_folded(acc[3], q3.m, fd[3], q3.sr));
          if (g.clamp) w = clamp4(w, g.lo4, g.hi4);
        } else {
          w = finish4<RQ>(acc[0], acc[1], acc[2], acc[3], b, q0, q1, q2, q3, g);
        }
        orow[static_cast<int64_t>(ox0 + p) * cwn] = w;
      }
    }
    if (S == 1) {
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int k = 0; k < NT; ++k) {
          t0[c][k] = t1[c][k];
          t1[c][k] = t2[c][k];
        }
      transpose(p0, t2);
    } else {
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int k = 0; k < NT; ++k) t0[c][k] = t2[c][k];
      transpose(p0, t1);
      transpose(p1, t2);
    }
  }
}

// --------------------------------------------------- small-channel conv (dp4a)
// Thread: one output pixel x COB output channels (blockIdx.y picks the chunk).
// The KHxKWxCI patch is packed into NW words in TFLite filter order
// (ky, kx, ci); out-of-image taps hold the input zero point.  Weights of the
// chunk sit in shared memory as [COB][NW] words (16-byte rows).
template <int KH, int KW, int CI, int COB, int RQ>
__global__ void __launch_bounds__(128)
    k_small_conv_s8(const int8_t* __restrict__ in, const uint32_t* __restrict__ wpack,
                    int32_t nw_stride, const int32_t* __restrict__ bias_eff,
                    const RqChannel* __restrict__ rq, int8_t* __restrict__ out, const Geom g,
                    int64_t n_base, uint32_t total, const FastDiv per_img) {
  constexpr int K = KH * KW * CI;
  constexpr int NW = (K + 3) / 4;
  constexpr int NW4 = (NW + 3) / 4;
  __shared__ uint4 sw[COB][NW4];
  const int co0 = blockIdx.y * COB;
  for (int i = threadIdx.x; i < COB * NW4; i += blockDim.x) {
    const int co = i / NW4, w4 = i - (i / NW4) * NW4;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (co0 + co < g.Co)
      v = __ldg(reinterpret_cast<const uint4*>(wpack + static_cast<int64_t>(co0 + co) * nw_stride) +
                w4);
    sw[co][w4] = v;
  }
  __syncthreads();
  // Flat loop over (image, pixel): a block loads its weights once and no
  // thread idles on a partial last block of an image.
  for (uint32_t idx = blockIdx.x * 128 + threadIdx.x; idx < total; idx += gridDim.x * 128) {
  const uint32_t nl = per_img.div(idx);
  const int pix = static_cast<int>(idx - nl * per_img.d);
  const int oy = pix / g.Wo, ox = pix - (pix / g.Wo) * g.Wo;
  const int64_t n = n_base + nl;
  const int8_t* img = in + n * static_cast<int64_t>(g.H) * g.W * CI;

  uint32_t x[NW4 * 4];
#pragma unroll
  for (int i = 0; i < NW4 * 4; ++i) x[i] = 0;
  const uint32_t zpb = static_cast<uint32_t>(g.zp_in) & 0xFFu;
#pragma unroll
  for (int ky = 0; ky < KH; ++ky) {
    const int iy = oy * g.sh - g.pt + ky;
#pragma unroll
    for (int kx = 0; kx < KW; ++kx) {
      const int ix = ox * g.sw - g.pl + kx;
      const bool ok = iy >= 0 && iy < g.H && ix >= 0 && ix < g.W;
      const int8_t* px = img + (static_cast<int64_t>(ok ? iy : 0) * g.W + (ok ? ix : 0)) * CI;
      if constexpr (CI % 4 == 0) {
#pragma unroll
        for (int c4 = 0; c4 < CI / 4; ++c4) {
          const uint32_t v = ok ? __ldg(reinterpret_cast<const uint32_t*>(px) + c4)
                                : zpb * 0x01010101u;
          x[((ky * KW + kx) * CI) / 4 + c4] = v;
        }
      } else {
#pragma unroll
        for (int ci = 0; ci < CI; ++ci) {
          const int k = (ky * KW + kx) * CI + ci;
          const uint32_t b = ok ? static_cast<uint32_t>(static_cast<uint8_t>(__ldg(px + ci))) : zpb;
          x[k >> 2] |= b << (8 * (k & 3));
        }
      }
    }
  }

  const int cnt = min(COB, g.Co - co0);
  int8_t* op = out + ((n * g.Ho + oy) * static_cast<int64_t>(g.Wo) + ox) * g.Co + co0;
  const bool vec = (g.Co % 4 == 0) && cnt == COB &&
                   (reinterpret_cast<uintptr_t>(op) & 3u) == 0;
#pragma unroll
  for (int c4 = 0; c4 < COB / 4; ++c4) {
    int32_t a[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int co = c4 * 4 + j;
      int32_t s = 0;
#pragma unroll
      for (int w4 = 0; w4 < NW4; ++w4) {
        const uint4 wv = sw[co][w4];
        s = __dp4a(static_cast<int>(x[4 * w4 + 0]), static_cast<int>(wv.x), s);
        s = __dp4a(static_cast<int>(x[4 * w4 + 1]), static_cast<int>(wv.y), s);
        s = __dp4a(static_cast<int>(x[4 * w4 + 2]), static_cast<int>(wv.z), s);
        s = __dp4a(static_cast<int>(x[4 * w4 + 3]), static_cast<int>(wv.w), s);
      }
      a[j] = s;
    }
    if (vec) {
      const int4 b = __ldg(reinterpret_cast<const int4*>(bias_eff + co0) + c4);
      const int cb = co0 + 4 * c4;
      reinterpret_cast<uint32_t*>(op)[c4] =
          finish4<RQ>(a[0], a[1], a[2], a[3], b, load_rq(rq + cb), load_rq(rq + cb + 1),
                  load_rq(rq + cb + 2), load_rq(rq + cb + 3), g);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int co = c4 * 4 + j;
        if (co < cnt)
          op[co] = finish1(a[j] + __ldg(bias_eff + co0 + co), load_rq(rq + co0 + co), g);
      }
    }
  }
}
}

// Conv + ReLU + 2x2 / stride-2 max pool (TFLite CONV_2D then MAX_POOL_2D):
// a thread computes the four conv pixels of one pooled output pixel for COB
// output channels as k_small_conv_s8 does, requantises each and keeps the
// byte-wise signed max, so only the pooled tensor reaches memory.  TFLite
// pools the requantised int8 outputs, so the result is exact.  Needs 4 | Co
// (whole words) and even Ho, Wo; the pooled output is [Ho/2][Wo/2][Co].
template <int KH, int KW, int CI, int COB, int RQ>
__global__ void __launch_bounds__(128)
    k_small_conv_pool_s8(const int8_t* __restrict__ in, const uint32_t* __restrict__ wpack,
                         int32_t nw_stride, const int32_t* __restrict__ bias_eff,
                         const RqChannel* __restrict__ rq, int8_t* __restrict__ out,
                         const Geom g, int64_t n_base, uint32_t total, const FastDiv per_img) {
  constexpr int K = KH * KW * CI;
  constexpr int NW = (K + 3) / 4;
  constexpr int NW4 = (NW + 3) / 4;
  __shared__ uint4 sw[COB][NW4];
  const int co0 = blockIdx.y * COB;
  for (int i = threadIdx.x; i < COB * NW4; i += blockDim.x) {
    const int co = i / NW4, w4 = i - (i / NW4) * NW4;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (co0 + co < g.Co)
      v = __ldg(reinterpret_cast<const uint4*>(wpack + static_cast<int64_t>(co0 + co) * nw_stride) +
                w4);
    sw[co][w4] = v;
  }
  __syncthreads();
  const int Hp = g.Ho >> 1, Wp = g.Wo >> 1;
  for (uint32_t idx = blockIdx.x * 128 + threadIdx.x; idx < total; idx += gridDim.x * 128) {
  const uint32_t nl = per_img.div(idx);
  const int pix = static_cast<int>(idx - nl * per_img.d);
  const int py = pix / Wp, px = pix - (pix / Wp) * Wp;
  const int64_t n = n_base + nl;
  const int8_t* img = in + n * static_cast<int64_t>(g.H) * g.W * CI;
  const uint32_t zpb = static_cast<uint32_t>(g.zp_in) & 0xFFu;
  const int cnt = min(COB, g.Co - co0);
  uint32_t best[COB / 4];
#pragma unroll 1
  for (int sub = 0; sub < 4; ++sub) {
    const int oy = 2 * py + (sub >> 1), ox = 2 * px + (sub & 1);
    uint32_t x[NW4 * 4];
#pragma unroll
    for (int i = 0; i < NW4 * 4; ++i) x[i] = 0;
#pragma unroll
    for (int ky = 0; ky < KH; ++ky) {
      const int iy = oy * g.sh - g.pt + ky;
#pragma unroll
      for (int kx = 0; kx < KW; ++kx) {
        const int ix = ox * g.sw - g.pl + kx;
        const bool ok = iy >= 0 && iy < g.H && ix >= 0 && ix < g.W;
        const int8_t* pxp = img + (static_cast<int64_t>(ok ? iy : 0) * g.W + (ok ? ix : 0)) * CI;
        if constexpr (CI % 4 == 0) {
#pragma unroll
          for (int c4 = 0; c4 < CI / 4; ++c4)
            x[((ky * KW + kx) * CI) / 4 + c4] =
                ok ? __ldg(reinterpret_cast<const uint32_t*>(pxp) + c4) : zpb * 0x01010101u;
        } else {
#pragma unroll
          for (int ci = 0; ci < CI; ++ci) {
            const int k = (ky * KW + kx) * CI + ci;
            const uint32_t b =
                ok ? static_cast<uint32_t>(static_cast<uint8_t>(__ldg(pxp + ci))) : zpb;
            x[k >> 2] |= b << (8 * (k & 3));
          }
        }
      }
    }
#pragma unroll
    for (int c4 = 0; c4 < COB / 4; ++c4) {
      int32_t a[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int co = c4 * 4 + j;
        int32_t acc = 0;
#pragma unroll
        for (int w4 = 0; w4 < NW4; ++w4) {
          const uint4 wv = sw[co][w4];
          acc = __dp4a(static_cast<int>(x[4 * w4 + 0]), static_cast<int>(wv.x), acc);
          acc = __dp4a(static_cast<int>(x[4 * w4 + 1]), static_cast<int>(wv.y), acc);
          acc = __dp4a(static_cast<int>(x[4 * w4 + 2]), static_cast<int>(wv.z), acc);
          acc = __dp4a(static_cast<int>(x[4 * w4 + 3]), static_cast<int>(wv.w), acc);
        }
        a[j] = acc;
      }
      const int cb = min(co0 + 4 * c4, g.Co - 4);  // channels past Co are never stored
      const int4 b = __ldg(reinterpret_cast<const int4*>(bias_eff + cb));
      const uint32_t w = finish4<RQ>(a[0], a[1], a[2], a[3], b, load_rq(rq + cb),
                                     load_rq(rq + cb + 1), load_rq(rq + cb + 2),
                                     load_rq(rq + cb + 3), g);
      best[c4] = sub == 0 ? w : __vmaxs4(best[c4], w);
    }
  }
  uint32_t* op = reinterpret_cast<uint32_t*>(
      out + ((n * Hp + py) * static_cast<int64_t>(Wp) + px) * g.Co + co0);
#pragma unroll
  for (int c4 = 0; c4 < COB / 4; ++c4)
    if (4 * c4 < cnt) op[c4] = best[c4];
}
}

// 3x3 stride-1 conv with few input channels (CI in {1, 2, 3, 4, 8}): a
// thread computes a 2x2 block of output pixels x COB channels from the 4x4
// input window it loads once (zero point outside the image), so every
// weight word read from shared memory and every requantisation constant
// serves four pixels (one pixel per thread re-read each weight per pixel
// and loaded its nine taps separately).  For CI % 4 == 0 the patch words
// are the window's pixel words themselves; for CI < 4 they are assembled
// from the window bytes.  POOL: the block is the 2x2 window of the max pool
// after the conv and only its max is stored ([Ho/2][Wo/2][Co]); otherwise
// the block's pixels inside the image are stored.  Needs 4 | Co.
template <int CI, int COB, int RQ, bool POOL>
__global__ void __launch_bounds__(128)
    k_small_conv_2x2_s8(const int8_t* __restrict__ in, const uint32_t* __restrict__ wpack,
                        int32_t nw_stride, const int32_t* __restrict__ bias_eff,
                        const RqChannel* __restrict__ rq, int8_t* __restrict__ out,
                        const Geom g, int64_t n_base, uint32_t total, const FastDiv per_img,
                        const FastDiv per_row) {
  constexpr int K = 9 * CI;
  constexpr int NW = (K + 3) / 4;
  constexpr int NW4 = (NW + 3) / 4;
  constexpr int CW = CI % 4 == 0 ? CI / 4 : 0;  // words per pixel when whole words
  __shared__ uint4 sw[COB][NW4];
  const int co0 = blockIdx.y * COB;
  for (int i = threadIdx.x; i < COB * NW4; i += blockDim.x) {
    const int co = i / NW4, w4 = i - (i / NW4) * NW4;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (co0 + co < g.Co)
      v = __ldg(reinterpret_cast<const uint4*>(wpack + static_cast<int64_t>(co0 + co) * nw_stride) +
                w4);
    sw[co][w4] = v;
  }
  __syncthreads();
  const int Bw = static_cast<int>(per_row.d);
  const uint32_t zp4 = (static_cast<uint32_t>(g.zp_in) & 0xFFu) * 0x01010101u;
  const int Hp = g.Ho >> 1, Wp = g.Wo >> 1;
  for (uint32_t idx = blockIdx.x * 128 + threadIdx.x; idx < total; idx += gridDim.x * 128) {
    const uint32_t nl = per_img.div(idx);
    const uint32_t blk = idx - nl * per_img.d;
    const int by = static_cast<int>(per_row.div(blk));
    const int bx = static_cast<int>(blk) - by * Bw;
    const int oy0 = 2 * by, ox0 = 2 * bx;
    const int64_t n = n_base + nl;
    const int8_t* img = in + n * static_cast<int64_t>(g.H) * g.W * CI;
    const int iy0 = oy0 - g.pt, ix0 = ox0 - g.pl;

    // The 4x4 window: words of CI % 4 == 0 pixels, or bytes.
    uint32_t win[4][4][CW > 0 ? CW : CI];
#pragma unroll
    for (int wy = 0; wy < 4; ++wy) {
      const int iy = iy0 + wy;
#pragma unroll
      for (int wx = 0; wx < 4; ++wx) {
        const int ix = ix0 + wx;
        const bool ok = iy >= 0 && iy < g.H && ix >= 0 && ix < g.W;
        const int8_t* pxp = img + (static_cast<int64_t>(ok ? iy : 0) * g.W + (ok ? ix : 0)) * CI;
        if constexpr (CW == 2) {
          const uint2 v = ok ? __ldg(reinterpret_cast<const uint2*>(pxp)) : make_uint2(zp4, zp4);
          win[wy][wx][0] = v.x;
          win[wy][wx][1] = v.y;
        } else if constexpr (CW == 1) {
          win[wy][wx][0] = ok ? __ldg(reinterpret_cast<const uint32_t*>(pxp)) : zp4;
        } else {
#pragma unroll
          for (int ci = 0; ci < CI; ++ci)
            win[wy][wx][ci] = ok ? static_cast<uint32_t>(static_cast<uint8_t>(__ldg(pxp + ci)))
                                 : (zp4 & 0xFFu);
        }
      }
    }
    // Patch words of the four pixels (sub = dy * 2 + dx), filter order
    // (ky, kx, ci), zero beyond the K bytes.
    uint32_t x[4][NW4 * 4];
#pragma unroll
    for (int sub = 0; sub < 4; ++sub) {
      const int dy = sub >> 1, dx = sub & 1;
#pragma unroll
      for (int wi = 0; wi < NW4 * 4; ++wi) x[sub][wi] = 0;
      if constexpr (CW > 0) {
#pragma unroll
        for (int t = 0; t < 9; ++t)
#pragma unroll
          for (int c = 0; c < CW; ++c) x[sub][t * CW + c] = win[dy + t / 3][dx + t % 3][c];
      } else {
#pragma unroll
        for (int t = 0; t < 9; ++t)
#pragma unroll
          for (int ci = 0; ci < CI; ++ci) {
            const int k = t * CI + ci;
            x[sub][k >> 2] |= win[dy + t / 3][dx + t % 3][ci] << (8 * (k & 3));
          }
      }
    }
    const int cnt = min(COB, g.Co - co0);
    uint32_t* prow = nullptr;  // pooled output word row
    uint32_t* orow[4];         // the block's output word rows (null outside the image)
    if constexpr (POOL) {
      prow = reinterpret_cast<uint32_t*>(
          out + ((n * Hp + by) * static_cast<int64_t>(Wp) + bx) * g.Co + co0);
    } else {
#pragma unroll
      for (int sub = 0; sub < 4; ++sub) {
        const int oy = oy0 + (sub >> 1), ox = ox0 + (sub & 1);
        orow[sub] = (oy < g.Ho && ox < g.Wo)
                        ? reinterpret_cast<uint32_t*>(
                              out + ((n * g.Ho + oy) * static_cast<int64_t>(g.Wo) + ox) * g.Co + co0)
                        : nullptr;
      }
    }
#pragma unroll
    for (int c4 = 0; c4 < COB / 4; ++c4) {
      int32_t a[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int sub = 0; sub < 4; ++sub) a[sub][j] = 0;
#pragma unroll
        for (int w4 = 0; w4 < NW4; ++w4) {
          const uint4 wv = sw[c4 * 4 + j][w4];
          const uint32_t wq[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
          for (int sub = 0; sub < 4; ++sub) {
            int32_t acc = a[sub][j];
#pragma unroll
            for (int q = 0; q < 4; ++q)  // the patch's padding words are zero: skipped
              if (4 * w4 + q < NW)
                acc = __dp4a(static_cast<int>(x[sub][4 * w4 + q]), static_cast<int>(wq[q]), acc);
            a[sub][j] = acc;
          }
        }
      }
      const int cb = min(co0 + 4 * c4, g.Co - 4);  // channels past Co are never stored
      const int4 b = __ldg(reinterpret_cast<const int4*>(bias_eff + cb));
      const RqChannel q0 = load_rq(rq + cb), q1 = load_rq(rq + cb + 1),
                      q2 = load_rq(rq + cb + 2), q3 = load_rq(rq + cb + 3);
      uint32_t r4[4];
#pragma unroll
      for (int sub = 0; sub < 4; ++sub)
        r4[sub] = finish4<RQ>(a[sub][0], a[sub][1], a[sub][2], a[sub][3], b, q0, q1, q2, q3, g);
      if (4 * c4 < cnt) {
        if constexpr (POOL) {
          prow[c4] = __vmaxs4(__vmaxs4(r4[0], r4[1]), __vmaxs4(r4[2], r4[3]));
        } else {
#pragma unroll
          for (int sub = 0; sub < 4; ++sub)
            if (orow[sub] != nullptr) orow[sub][c4] = r4[sub];
        }
      }
    }
  }
}

// Constant-table variant for 32 output channels and a patch of at most 16
// bytes (the stem conv): weights and requant constants are kernel-parameter
// operands at compile-time offsets, so the only loads are the input patch
// (the smem/global tables made the L1 pipe the bottleneck).
template <int KH, int KW, int CI, int Q>
__global__ void __launch_bounds__(128)
    k_small_conv_tab_s8(const int8_t* __restrict__ in, int8_t* __restrict__ out, const Geom g,
                        int64_t n_base, const __grid_constant__ SmallConvTable tab) {
  constexpr int K = KH * KW * CI;
  constexpr int NW = (K + 3) / 4;
  static_assert(NW <= 4, "patch of at most 16 bytes");
  const int pix = blockIdx.x * 128 + threadIdx.x;
  if (pix >= g.Ho * g.Wo) return;
  const int oy = pix / g.Wo, ox = pix - (pix / g.Wo) * g.Wo;
  const int64_t n = n_base + blockIdx.z;
  const int8_t* img = in + n * static_cast<int64_t>(g.H) * g.W * CI;
  uint32_t x[NW];
#pragma unroll
  for (int i = 0; i < NW; ++i) x[i] = 0;
  const uint32_t zpb = static_cast<uint32_t>(g.zp_in) & 0xFFu;
#pragma unroll
  for (int ky = 0; ky < KH; ++ky) {
    const int iy = oy * g.sh - g.pt + ky;
#pragma unroll
    for (int kx = 0; kx < KW; ++kx) {
      const int ix = ox * g.sw - g.pl + kx;
      const bool ok = iy >= 0 && iy < g.H && ix >= 0 && ix < g.W;
      const int8_t* px = img + (static_cast<int64_t>(ok ? iy : 0) * g.W + (ok ? ix : 0)) * CI;
#pragma unroll
      for (int ci = 0; ci < CI; ++ci) {
        const int k = (ky * KW + kx) * CI + ci;
        const uint32_t b = ok ? static_cast<uint32_t>(static_cast<uint8_t>(__ldg(px + ci))) : zpb;
        x[k >> 2] |= b << (8 * (k & 3));
      }
    }
  }
  uint32_t words[8];
#pragma unroll
  for (int c4 = 0; c4 < 8; ++c4) {
    int32_t r[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int co = 4 * c4 + j;
      int32_t acc = 0;
#pragma unroll
      for (int w = 0; w < NW; ++w)
        acc = __dp4a(static_cast<int>(x[w]), static_cast<int>(tab.w[co][w]), acc);
      if constexpr ((Q & kEpFloor) != 0) {
        r[j] = rq_tab_q<Q>(static_cast<uint32_t>(acc), tab.mh[co], tab.bs[co]);
      } else {
        const int2 bs = tab.bs[co];
        r[j] = rq_tab(acc + bs.x, tab.mh[co], bs.y);
      }
    }
    uint32_t w4 = pack_sat4(r[0], r[1], r[2], r[3]);
    if constexpr ((Q & kEpClamp) != 0) w4 = clamp4(w4, g.lo4, g.hi4);
    words[c4] = w4;
  }
  uint4* op = reinterpret_cast<uint4*>(out + ((n * g.Ho + oy) * static_cast<int64_t>(g.Wo) + ox) * 32);
  op[0] = make_uint4(words[0], words[1], words[2], words[3]);
  op[1] = make_uint4(words[4], words[5], words[6], words[7]);
}

// Stride-2 variant of the constant-table stem for rows whose width is a
// multiple of 8 and no left padding (the config-3 stem, 96x512 -> 48x256):
// a thread keeps the weights and requant constants of 8 output channels in
// registers and computes 4 consecutive pixels x 8 channels per output row,
// for a strip of up to kStemRows rows.  Lane = pixel group (lane >> 2) x
// channel group (lane & 3); a warp covers 32 consecutive pixels, a block
// 128.  The block first copies the strip's 2 * rows + 1 input rows (257
// bytes each, zero point outside the image) into shared memory with 8-byte
// loads, so the row loop reads shared memory only; each pixel's patch words
// come from its 9 bytes per row with funnel shifts and byte permutes.  The
// weight words and per-channel constants are register operands, so an
// output costs three dp4a, one wide multiply-add and a shift (floor form).
constexpr int kStemRows = 16;
constexpr int kStemRowBytes = 264;  // 257 used, 8-byte multiple

template <int Q>
__global__ void __launch_bounds__(128)
    k_stem_s2_s8(const int8_t* __restrict__ in, int8_t* __restrict__ out, const Geom g,
                 int64_t n_base, const __grid_constant__ SmallConvTable tab) {
  __shared__ __align__(16) uint8_t srow[2 * kStemRows + 1][kStemRowBytes];
  const int oy0 = blockIdx.y * kStemRows;
  const int oy1 = min(oy0 + kStemRows, g.Ho);
  const int64_t n = n_base + blockIdx.z;
  const int xb = blockIdx.x * 256;  // first input column of the block
  const int nrows = 2 * (oy1 - oy0) + 1;
  const int iy0 = 2 * oy0 - g.pt;
  const uint32_t zpw = splat4(g.zp_in);
  {
    const int8_t* img = in + n * static_cast<int64_t>(g.H) * g.W;
    constexpr int kChunks = kStemRowBytes / 8;  // 33 chunks of 8 bytes per row
    for (int c = threadIdx.x; c < nrows * kChunks; c += 128) {
      const int rr = c / kChunks;
      const int k = c - rr * kChunks;
      const int iy = iy0 + rr;
      const int x = xb + 8 * k;
      uint2 v = make_uint2(zpw, zpw);
      // W % 8 == 0: a chunk is wholly inside or outside the row.
      if (iy >= 0 && iy < g.H && x < g.W)
        v = __ldg(reinterpret_cast<const uint2*>(img + static_cast<int64_t>(iy) * g.W + x));
      *reinterpret_cast<uint2*>(&srow[rr][8 * k]) = v;
    }
  }

  const int lane = threadIdx.x & 31;
  const int cg = lane & 3;
  const int px = (threadIdx.x >> 5) * 32 + (lane >> 2) * 4;  // first pixel within the block
  const int ox0 = blockIdx.x * 128 + px;
  uint32_t w[8][3];
  // The 64-bit addend of each channel is held as one int64 (an aligned
  // register pair) so the wide multiply-add of an output needs no moves.
  int32_t m[8], sr[8], bias[8];
  int64_t cd[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int co = cg * 8 + k;
#pragma unroll
    for (int j = 0; j < 3; ++j) w[k][j] = tab.w[co][j];
    const int2 mh = tab.mh[co];
    const int2 bs = tab.bs[co];
    sr[k] = bs.y;
    if constexpr ((Q & kEpFloor) != 0) {
      // D with the bias folded in (floor_entry).
      m[k] = bs.x;
      cd[k] = floor_d(mh);
      bias[k] = 0;
    } else {
      // C - 2^32 ({2^30, high word}); the bias goes onto the accumulator.
      m[k] = mh.x;
      cd[k] = static_cast<int64_t>(
          (static_cast<uint64_t>(static_cast<uint32_t>(mh.y)) << 32) | 0x40000000u);
      bias[k] = bs.x;
    }
  }
  __syncthreads();
  if (ox0 >= g.Wo) return;

  // Bytes 2 * px .. 2 * px + 8 of shared row rr: {lo, hi, byte 8}.
  auto row = [&](int rr, uint32_t& lo, uint32_t& hi, uint32_t& b8) {
    const uint2 v = *reinterpret_cast<const uint2*>(&srow[rr][2 * px]);
    lo = v.x;
    hi = v.y;
    b8 = srow[rr][2 * px + 8];
  };
  uint32_t r0l, r0h, r0b, r1l, r1h, r1b, r2l, r2h, r2b;
  row(0, r0l, r0h, r0b);
  int8_t* obase = out + (n * g.Ho) * static_cast<int64_t>(g.Wo) * 32 + cg * 8;
#pragma unroll 1
  for (int oy = oy0; oy < oy1; ++oy) {
    const int rr = 2 * (oy - oy0);
    row(rr + 1, r1l, r1h, r1b);
    row(rr + 2, r2l, r2h, r2b);
    int8_t* orow = obase + (static_cast<int64_t>(oy) * g.Wo + ox0) * 32;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      // Bytes 2j .. 2j+3 of each row.
      const uint32_t s0 = j == 0 ? r0l : j == 1 ? __funnelshift_r(r0l, r0h, 16)
                                       : j == 2 ? r0h : __funnelshift_r(r0h, r0b, 16);
      const uint32_t s1 = j == 0 ? r1l : j == 1 ? __funnelshift_r(r1l, r1h, 16)
                                       : j == 2 ? r1h : __funnelshift_r(r1h, r1b, 16);
      const uint32_t s2 = j == 0 ? r2l : j == 1 ? __funnelshift_r(r2l, r2h, 16)
                                       : j == 2 ? r2h : __funnelshift_r(r2h, r2b, 16);
      // Patch words in filter order (ky, kx): taps 0-3, 4-7, 8.
      const uint32_t p0 = __byte_perm(s0, s1, 0x4210);
      const uint32_t p1 = __byte_perm(s1, s2, 0x5421);
      const uint32_t p2 = s2 >> 16;
      int32_t r[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        int32_t acc = __dp4a(static_cast<int>(p0), static_cast<int>(w[k][0]), 0);
        acc = __dp4a(static_cast<int>(p1), static_cast<int>(w[k][1]), acc);
        acc = __dp4a(static_cast<int>(p2), static_cast<int>(w[k][2]), acc);
        const int64_t c = cd[k];
        if constexpr ((Q & kEpFloor) != 0) {
          const int64_t t = static_cast<int64_t>(acc) * m[k] + c;
          r[k] = static_cast<int32_t>(t >> 32) >> sr[k];
        } else {
          const int32_t a = acc + bias[k];
          const int64_t t = static_cast<int64_t>(a) * m[k] + c;
          const uint32_t lo = static_cast<uint32_t>(t);
          const int32_t hi = static_cast<int32_t>(t >> 32);
          r[k] = (hi + static_cast<int32_t>((~static_cast<uint32_t>(a) | lo) >> 31)) >> sr[k];
        }
      }
      uint32_t w0 = pack_sat4(r[0], r[1], r[2], r[3]);
      uint32_t w1 = pack_sat4(r[4], r[5], r[6], r[7]);
      if constexpr ((Q & kEpClamp) != 0) {
        w0 = clamp4(w0, g.lo4, g.hi4);
        w1 = clamp4(w1, g.lo4, g.hi4);
      }
      *reinterpret_cast<uint2*>(orow + j * 32) = make_uint2(w0, w1);
    }
    r0l = r2l;
    r0h = r2h;
    r0b = r2b;
  }
}

// ------------------------------------------------------------- direct conv
// Fallback for any conv: one thread per (sample, oy, ox) and COB output
// channels; weights of the chunk in shared memory as int32 [K][COB].
template <int COB>
__global__ void k_conv_direct_s8(const int8_t* __restrict__ in, const int8_t* __restrict__ f,
                                 const int32_t* __restrict__ bias,
                                 const RqChannel* __restrict__ rq, int8_t* __restrict__ out,
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
    if (co0 + j < g.Co) op[j] = finish1(acc[j], load_rq(rq + co0 + j), g);
}

// --------------------------------------------------- depthwise (fallback)
__global__ void k_dw_generic_s8(const int8_t* __restrict__ in, const int8_t* __restrict__ f,
                                const int32_t* __restrict__ bias,
                                const RqChannel* __restrict__ rq, int8_t* __restrict__ out,
                                const Geom g, int64_t total) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int c = static_cast<int>(idx % g.C);
  const int64_t pix = idx / g.C;
  const int ox = static_cast<int>(pix % g.Wo);
  const int oy = static_cast<int>((pix / g.Wo) % g.Ho);
  const int64_t n = pix / (static_cast<int64_t>(g.Wo) * g.Ho);
  int32_t acc = bias != nullptr ? __ldg(bias + c) : 0;
  const int iy0 = oy * g.sh - g.pt, ix0 = ox * g.sw - g.pl;
  const int8_t* img = in + n * g.H * g.W * static_cast<int64_t>(g.C);
  for (int ky = 0; ky < g.KH; ++ky) {
    const int iy = iy0 + ky;
    if (iy < 0 || iy >= g.H) continue;
    for (int kx = 0; kx < g.KW; ++kx) {
      const int ix = ix0 + kx;
      if (ix < 0 || ix >= g.W) continue;
      acc += (static_cast<int32_t>(img[(static_cast<int64_t>(iy) * g.W + ix) * g.C + c]) -
              g.zp_in) *
             static_cast<int32_t>(f[(ky * g.KW + kx) * g.C + c]);
    }
  }
  out[pix * g.C + c] = finish1(acc, load_rq(rq + c), g);
}

// --------------------------------------------------------------- FC (warp)
__global__ void k_fc_warp_s8(const int8_t* __restrict__ in, const int8_t* __restrict__ f,
                             const int32_t* __restrict__ bias, const RqChannel* __restrict__ rq,
                             int8_t* __restrict__ out, int64_t K, int32_t N, int64_t total,
                             const Geom g) {
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= total) return;
  const int64_t b = w / N;
  const int32_t o = static_cast<int32_t>(w - b * N);
  const int8_t* x = in + b * K;
  const int8_t* wr = f + static_cast<int64_t>(o) * K;
  int32_t s = 0;
  for (int64_t k = lane; k < K; k += 32)
    s += (static_cast<int32_t>(x[k]) - g.zp_in) * static_cast<int32_t>(wr[k]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, off);
  if (lane == 0) out[b * N + o] = finish1(s + (bias != nullptr ? bias[o] : 0), load_rq(rq + o), g);
}

// ------------------------------------------------ small-batch FC (GEMV)
// FC over B <= 4 samples with K % 16 == 0: a GEMV, bound by reading the
// weights once.  A warp takes one output channel at a time (grid-stride
// over channels, every SM busy); each lane streams 16-byte chunks of the
// weight row, four in flight, and dots them with the same chunks of every
// sample (the B x K activations stay in L1 / L2).  The sums start from the
// folded bias (bias - zp_in * sum(w)), so sum(x * w) + bias_eff is TFLite's
// sum((x - zp_in) * w) + bias; any requantisation form.
// Streaming (evict-first) 16-byte load through the intrinsic, which the
// compiler schedules freely: a lane's eight weight loads issue back to back,
// ahead of the dot products (inline assembly was kept in order and left
// one load in flight).
__device__ __forceinline__ uint4 ld_stream16(const uint4* p) { return __ldcs(p); }

__device__ __forceinline__ int32_t dot16(const uint4 a, const uint4 b, int32_t s) {
  s = __dp4a(static_cast<int>(a.x), static_cast<int>(b.x), s);
  s = __dp4a(static_cast<int>(a.y), static_cast<int>(b.y), s);
  s = __dp4a(static_cast<int>(a.z), static_cast<int>(b.z), s);
  return __dp4a(static_cast<int>(a.w), static_cast<int>(b.w), s);
}

template <int B>
__global__ void __launch_bounds__(256)
    k_fc_gemv_s8(const int8_t* __restrict__ in, const int8_t* __restrict__ f,
                 const int32_t* __restrict__ bias_eff, const RqChannel* __restrict__ rq,
                 int8_t* __restrict__ out, int32_t K, int32_t N, const Geom g) {
  const int lane = threadIdx.x & 31;
  const int32_t warps = static_cast<int32_t>(gridDim.x * (blockDim.x >> 5));
  const int32_t chunks = K >> 4;
  for (int32_t o = static_cast<int32_t>(blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5));
       o < N; o += warps) {
    const uint4* wr = reinterpret_cast<const uint4*>(f + static_cast<int64_t>(o) * K);
    int32_t acc[B];
#pragma unroll
    for (int b = 0; b < B; ++b) acc[b] = 0;
    int32_t c = lane;
    // Eight 16-byte weight loads per lane in flight (4 KB per warp).
    for (; c + 224 < chunks; c += 256) {
      uint4 w[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) w[u] = ld_stream16(wr + c + 32 * u);
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const uint4* xr = reinterpret_cast<const uint4*>(in + static_cast<int64_t>(b) * K);
#pragma unroll
        for (int u = 0; u < 8; ++u) acc[b] = dot16(w[u], __ldg(xr + c + 32 * u), acc[b]);
      }
    }
#pragma unroll 4
    for (; c < chunks; c += 32) {
      const uint4 w0 = ld_stream16(wr + c);
#pragma unroll
      for (int b = 0; b < B; ++b)
        acc[b] = dot16(w0, __ldg(reinterpret_cast<const uint4*>(in + static_cast<int64_t>(b) * K) + c),
                       acc[b]);
    }
#pragma unroll
    for (int b = 0; b < B; ++b)
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) acc[b] += __shfl_xor_sync(0xFFFFFFFFu, acc[b], off);
    if (lane < B) {
      int32_t a = acc[0];
#pragma unroll
      for (int b = 1; b < B; ++b)
        if (lane == b) a = acc[b];
      int32_t r = rq_apply(a + __ldg(bias_eff + o), load_rq(rq + o));
      r = min(max(r, g.act_min), g.act_max);
      out[static_cast<int64_t>(lane) * N + o] = static_cast<int8_t>(r);
    }
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
#pragma unroll
    for (int q = 0; q < kWords; ++q) m[q] = clamp4(m[q], g.lo4, g.hi4);
    if constexpr (VEC == 16)
      *reinterpret_cast<uint4*>(op) = make_uint4(m[0], m[1], m[2], m[3]);
    else
      *reinterpret_cast<uint32_t*>(op) = m[0];
  } else {
    op[0] = static_cast<int8_t>(clamp4(static_cast<uint32_t>(m1) & 0xFFu, g.lo4, g.hi4) & 0xFFu);
  }
}

// Average pool: int32 sum of the in-image window, divided by the count with
// round-half-away-from-zero (TFLite), clamped.
template <int VEC>
__global__ void k_avgpool_s8(const int8_t* __restrict__ in, int8_t* __restrict__ out,
                             const Geom g, int32_t act_min, int32_t act_max, int64_t total) {
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
      if constexpr (VEC == 16) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(xp));
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[4 * q + j] += sbyte(w[q], j);
      } else if constexpr (VEC == 4) {
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
    a = max(a, act_min);
    a = min(a, act_max);
    r[j] = a;
  }
  if constexpr (VEC == 16)
    *reinterpret_cast<uint4*>(op) =
        make_uint4(pack4_s8(r[0], r[1], r[2], r[3]), pack4_s8(r[4], r[5], r[6], r[7]),
                   pack4_s8(r[8], r[9], r[10], r[11]), pack4_s8(r[12], r[13], r[14], r[15]));
  else if constexpr (VEC == 4)
    *reinterpret_cast<uint32_t*>(op) = pack4_s8(r[0], r[1], r[2], r[3]);
  else
    op[0] = static_cast<int8_t>(r[0]);
}

// Global average pool (the window is the whole image, no padding): a thread
// sums 16 channels of one sample over every pixel with eight 16-byte loads
// in flight (the windowed kernel above keeps one load in flight per thread,
// too few to cover HBM latency), then divides as k_avgpool_s8 does.
__global__ void k_gap_s8(const int8_t* __restrict__ in, int8_t* __restrict__ out, int32_t hw,
                         int32_t C, int32_t act_min, int32_t act_max, int64_t total) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int cv = C / 16;
  const int64_t n = idx / cv;
  const int c0 = static_cast<int>(idx - n * cv) * 16;
  const int8_t* px = in + n * hw * static_cast<int64_t>(C) + c0;
  int32_t acc[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) acc[j] = 0;
  auto add16 = [&](const uint4 v) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[4 * q + j] += sbyte(w[q], j);
  };
  int i = 0;
  for (; i + 8 <= hw; i += 8) {
    uint4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      v[u] = __ldg(reinterpret_cast<const uint4*>(px + static_cast<int64_t>(i + u) * C));
#pragma unroll
    for (int u = 0; u < 8; ++u) add16(v[u]);
  }
  for (; i < hw; ++i) add16(__ldg(reinterpret_cast<const uint4*>(px + static_cast<int64_t>(i) * C)));
  int32_t r[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    int32_t a = acc[j];
    a = a > 0 ? (a + hw / 2) / hw : (a - hw / 2) / hw;
    a = max(a, act_min);
    a = min(a, act_max);
    r[j] = a;
  }
  *reinterpret_cast<uint4*>(out + n * C + c0) =
      make_uint4(pack4_s8(r[0], r[1], r[2], r[3]), pack4_s8(r[4], r[5], r[6], r[7]),
                 pack4_s8(r[8], r[9], r[10], r[11]), pack4_s8(r[12], r[13], r[14], r[15]));
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

template <int KH, int KW, int CI, int RQ>
cudaError_t small_conv_cob(const Geom& g, const PreparedOp& p, int64_t batch, const int8_t* in,
                           int8_t* out, cudaStream_t s, bool pool) {
  const int cob = g.Co <= 8 ? 8 : g.Co <= 16 ? 16 : 32;
  const int64_t pix = pool ? static_cast<int64_t>(g.Ho / 2) * (g.Wo / 2)
                           : static_cast<int64_t>(g.Ho) * g.Wo;
  // Launches over batch slices of fewer than 2^31 (image, pixel) pairs;
  // each block loops over the pairs (at most 16 blocks of 128 threads per
  // SM per channel chunk).
  const int64_t per_launch = std::max<int64_t>(1, ((1ll << 31) - 1) / pix);
  const FastDiv fd(static_cast<uint32_t>(pix));
  for (int64_t n0 = 0; n0 < batch; n0 += per_launch) {
    const int64_t nimg = std::min<int64_t>(per_launch, batch - n0);
    const uint32_t total = static_cast<uint32_t>(nimg * pix);
    const dim3 grid(static_cast<unsigned>(std::min<int64_t>((total + 127) / 128, 148 * 16)),
                    (g.Co + cob - 1) / cob, 1);
    if (pool) {
      if (cob == 8)
        k_small_conv_pool_s8<KH, KW, CI, 8, RQ><<<grid, 128, 0, s>>>(
            in, p.wpack, p.nw, p.bias_eff, p.rq, out, g, n0, total, fd);
      else if (cob == 16)
        k_small_conv_pool_s8<KH, KW, CI, 16, RQ><<<grid, 128, 0, s>>>(
            in, p.wpack, p.nw, p.bias_eff, p.rq, out, g, n0, total, fd);
      else
        k_small_conv_pool_s8<KH, KW, CI, 32, RQ><<<grid, 128, 0, s>>>(
            in, p.wpack, p.nw, p.bias_eff, p.rq, out, g, n0, total, fd);
      continue;
    }
    if (cob == 8)
      k_small_conv_s8<KH, KW, CI, 8, RQ><<<grid, 128, 0, s>>>(in, p.wpack, p.nw, p.bias_eff,
                                                              p.rq, out, g, n0, total, fd);
    else if (cob == 16)
      k_small_conv_s8<KH, KW, CI, 16, RQ><<<grid, 128, 0, s>>>(in, p.wpack, p.nw, p.bias_eff,
                                                               p.rq, out, g, n0, total, fd);
    else
      k_small_conv_s8<KH, KW, CI, 32, RQ><<<grid, 128, 0, s>>>(in, p.wpack, p.nw, p.bias_eff,
                                                               p.rq, out, g, n0, total, fd);
  }
  return cudaGetLastError();
}

// The 2x2-block kernel (3x3, stride 1, 4 | Co, 4-byte aligned output).
template <int CI, int RQ>
cudaError_t small_conv_2x2(const Geom& g, const PreparedOp& p, int64_t batch, const int8_t* in,
                           int8_t* out, cudaStream_t s, bool pool) {
  const int cob = g.Co <= 8 ? 8 : g.Co <= 16 ? 16 : 32;
  const int bh = pool ? g.Ho / 2 : (g.Ho + 1) / 2;
  const int bw = pool ? g.Wo / 2 : (g.Wo + 1) / 2;
  const int64_t per = static_cast<int64_t>(bh) * bw;
  const int64_t per_launch = std::max<int64_t>(1, ((1ll << 31) - 1) / per);
  const FastDiv fd(static_cast<uint32_t>(per)), fr(static_cast<uint32_t>(bw));
  for (int64_t n0 = 0; n0 < batch; n0 += per_launch) {
    const int64_t nimg = std::min<int64_t>(per_launch, batch - n0);
    const uint32_t total = static_cast<uint32_t>(nimg * per);
    const dim3 grid(static_cast<unsigned>(std::min<int64_t>((total + 127) / 128, 148 * 16)),
                    (g.Co + cob - 1) / cob, 1);
#define PSPML_SC2(COB, POOLV)                                                              \
  k_small_conv_2x2_s8<CI, COB, RQ, POOLV><<<grid, 128, 0, s>>>(in, p.wpack, p.nw, p.bias_eff, \
                                                                p.rq, out, g, n0, total, fd, fr)
    if (pool) {
      if (cob == 8) PSPML_SC2(8, true);
      else if (cob == 16) PSPML_SC2(16, true);
      else PSPML_SC2(32, true);
    } else {
      if (cob == 8) PSPML_SC2(8, false);
      else if (cob == 16) PSPML_SC2(16, false);
      else PSPML_SC2(32, false);
    }
#undef PSPML_SC2
  }
  return cudaGetLastError();
}

template <int KH, int KW, int CI>
cudaError_t small_conv_cob(const Geom& g, const PreparedOp& p, int64_t batch, const int8_t* in,
                           int8_t* out, cudaStream_t s, bool pool) {
  if (KH == 3 && KW == 3 && g.sh == 1 && g.sw == 1 && g.Co % 4 == 0 &&
      (reinterpret_cast<uintptr_t>(out) & 3u) == 0 &&
      (CI % 4 != 0 || (reinterpret_cast<uintptr_t>(in) & (4u * (CI / 4) - 1)) == 0)) {
    switch (rq_form(p.all_fast_known, g.act_min, g.zp_out)) {
      case kRqFloor: return small_conv_2x2<CI, kRqFloor>(g, p, batch, in, out, s, pool);
      case kRqFast: return small_conv_2x2<CI, kRqFast>(g, p, batch, in, out, s, pool);
      default: return small_conv_2x2<CI, kRqGeneral>(g, p, batch, in, out, s, pool);
    }
  }
  switch (rq_form(p.all_fast_known, g.act_min, g.zp_out)) {
    case kRqFloor: return small_conv_cob<KH, KW, CI, kRqFloor>(g, p, batch, in, out, s, pool);
    case kRqFast: return small_conv_cob<KH, KW, CI, kRqFast>(g, p, batch, in, out, s, pool);
    default: return small_conv_cob<KH, KW, CI, kRqGeneral>(g, p, batch, in, out, s, pool);
  }
}

}  // namespace

bool small_conv_supported(const pspml_op_desc& d) {
  if (d.kernel_h != 3 || d.kernel_w != 3) return false;
  return d.in_c == 1 || d.in_c == 2 || d.in_c == 3 || d.in_c == 4 || d.in_c == 8;
}

template <int CI>
cudaError_t small_conv_tab(const Geom& g, const PreparedOp& p, int64_t batch, const int8_t* in,
                           int8_t* out, cudaStream_t s) {
  for (int64_t n0 = 0; n0 < batch; n0 += kMaxGridZ) {
    const unsigned nz = static_cast<unsigned>(std::min<int64_t>(kMaxGridZ, batch - n0));
    const dim3 grid((g.Ho * g.Wo + 127) / 128, 1, nz);
    const SmallConvTable& t = *p.sc_table;
    switch (ep_flags(g.act_min, g.act_max, g.zp_out)) {
      case 0: k_small_conv_tab_s8<3, 3, CI, 0><<<grid, 128, 0, s>>>(in, out, g, n0, t); break;
      case 1: k_small_conv_tab_s8<3, 3, CI, 1><<<grid, 128, 0, s>>>(in, out, g, n0, t); break;
      case 2: k_small_conv_tab_s8<3, 3, CI, 2><<<grid, 128, 0, s>>>(in, out, g, n0, t); break;
      default: k_small_conv_tab_s8<3, 3, CI, 3><<<grid, 128, 0, s>>>(in, out, g, n0, t); break;
    }
  }
  return cudaGetLastError();
}

// Shapes of k_stem_s2_s8: the table kernel's shapes with stride 2, no left
// padding, rows of a multiple of 8 bytes and 4 | out_w <= in_w / 2.
static bool stem_s2_ok(const pspml_op_desc& d, const int8_t* in, const int8_t* out) {
  return d.stride_h == 2 && d.stride_w == 2 && d.pad_left == 0 && d.pad_top >= 0 &&
         d.pad_top <= 2 && d.in_w % 8 == 0 && d.out_w % 4 == 0 && 2 * d.out_w <= d.in_w &&
         (reinterpret_cast<uintptr_t>(in) & 7u) == 0 && (reinterpret_cast<uintptr_t>(out) & 7u) == 0;
}

static cudaError_t stem_s2(const Geom& g, const PreparedOp& p, int64_t batch, const int8_t* in,
                    int8_t* out, cudaStream_t s) {
  for (int64_t n0 = 0; n0 < batch; n0 += kMaxGridZ) {
    const unsigned nz = static_cast<unsigned>(std::min<int64_t>(kMaxGridZ, batch - n0));
    const dim3 grid((g.Wo + 127) / 128, (g.Ho + kStemRows - 1) / kStemRows, nz);
    const SmallConvTable& t = *p.sc_table;
    switch (ep_flags(g.act_min, g.act_max, g.zp_out)) {
      case 0: k_stem_s2_s8<0><<<grid, 128, 0, s>>>(in, out, g, n0, t); break;
      case 1: k_stem_s2_s8<1><<<grid, 128, 0, s>>>(in, out, g, n0, t); break;
      case 2: k_stem_s2_s8<2><<<grid, 128, 0, s>>>(in, out, g, n0, t); break;
      default: k_stem_s2_s8<3><<<grid, 128, 0, s>>>(in, out, g, n0, t); break;
    }
  }
  return cudaGetLastError();
}

cudaError_t launch_small_conv(const pspml_op_desc& d, const PreparedOp& p, int64_t batch,
                              const int8_t* in, int8_t* out, cudaStream_t s, bool pool) {
  const Geom g = geom_of(d);
  if (pool) {
    if (d.out_c % 4 != 0 || d.out_h % 2 != 0 || d.out_w % 2 != 0 ||
        (reinterpret_cast<uintptr_t>(out) & 3u) != 0)
      return cudaErrorInvalidValue;
    switch (d.in_c) {
      case 1: return small_conv_cob<3, 3, 1>(g, p, batch, in, out, s, true);
      case 2: return small_conv_cob<3, 3, 2>(g, p, batch, in, out, s, true);
      case 3: return small_conv_cob<3, 3, 3>(g, p, batch, in, out, s, true);
      case 4: return small_conv_cob<3, 3, 4>(g, p, batch, in, out, s, true);
      case 8: return small_conv_cob<3, 3, 8>(g, p, batch, in, out, s, true);
      default: return cudaErrorInvalidValue;
    }
  }
  if (p.sc_table != nullptr && p.all_fast_known && d.out_c == 32 && d.in_c == 1 &&
      d.kernel_h == 3 && d.kernel_w == 3 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0) {
    if (stem_s2_ok(d, in, out)) return stem_s2(g, p, batch, in, out, s);
    return small_conv_tab<1>(g, p, batch, in, out, s);
  }
  switch (d.in_c) {
    case 1: return small_conv_cob<3, 3, 1>(g, p, batch, in, out, s, false);
    case 2: return small_conv_cob<3, 3, 2>(g, p, batch, in, out, s, false);
    case 3: return small_conv_cob<3, 3, 3>(g, p, batch, in, out, s, false);
    case 4: return small_conv_cob<3, 3, 4>(g, p, batch, in, out, s, false);
    case 8: return small_conv_cob<3, 3, 8>(g, p, batch, in, out, s, false);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_dw3x3(const pspml_op_desc& d, const PreparedOp& p, int64_t batch,
                         const int8_t* in, int8_t* out, cudaStream_t s) {
  const Geom g = geom_of(d);
  constexpr int PX = 4;
  const int groups = (g.Wo + PX - 1) / PX;
  const int pairs = groups * (g.C / 4);
  const int rows_per = std::min(g.Ho, 16);
  const unsigned strips = static_cast<unsigned>((g.Ho + rows_per - 1) / rows_per);
  for (int64_t n0 = 0; n0 < batch; n0 += kMaxGridZ) {
    const unsigned nz = static_cast<unsigned>(std::min<int64_t>(kMaxGridZ, batch - n0));
    const dim3 grid((pairs + 127) / 128, strips, nz);
    const auto* i32 = reinterpret_cast<const uint32_t*>(in);
    const auto* f32 = reinterpret_cast<const uint32_t*>(p.filter);
    auto* o32 = reinterpret_cast<uint32_t*>(out);
    const int form = rq_form(p.all_fast_known, g.act_min, g.zp_out);
    if (g.sh == 1) {
      if (form == kRqFloor)
        k_dw3x3_s8<1, PX, kRqFloor>
            <<<grid, 128, 0, s>>>(i32, f32, p.bias_eff, p.rq, o32, g, rows_per, n0);
      else if (form == kRqFast)
        k_dw3x3_s8<1, PX, kRqFast>
            <<<grid, 128, 0, s>>>(i32, f32, p.bias_eff, p.rq, o32, g, rows_per, n0);
      else
        k_dw3x3_s8<1, PX, kRqGeneral>
            <<<grid, 128, 0, s>>>(i32, f32, p.bias_eff, p.rq, o32, g, rows_per, n0);
    } else {
      if (form == kRqFloor)
        k_dw3x3_s8<2, PX, kRqFloor>
            <<<grid, 128, 0, s>>>(i32, f32, p.bias_eff, p.rq, o32, g, rows_per, n0);
      else if (form == kRqFast)
        k_dw3x3_s8<2, PX, kRqFast>
            <<<grid, 128, 0, s>>>(i32, f32, p.bias_eff, p.rq, o32, g, rows_per, n0);
      else
        k_dw3x3_s8<2, PX, kRqGeneral>
            <<<grid, 128, 0, s>>>(i32, f32, p.bias_eff, p.rq, o32, g, rows_per, n0);
    }
  }
  return cudaGetLastError();
}

cudaError_t launch_dw_generic(const pspml_op_desc& d, const PreparedOp& p, int64_t batch,
                              const int8_t* in, int8_t* out, cudaStream_t s) {
  const Geom g = geom_of(d);
  const int64_t total = batch * g.Ho * g.Wo * g.C;
  k_dw_generic_s8<<<grid_for(total), kBlock, 0, s>>>(in, p.filter, p.bias, p.rq, out, g, total);
  return cudaGetLastError();
}

cudaError_t launch_conv_direct(const pspml_op_desc& d, const PreparedOp& p, int64_t batch,
                               const int8_t* in, int8_t* out, cudaStream_t s) {
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
    k_conv_direct_s8<16><<<grid, kBlock, smem, s>>>(in, p.filter, p.bias, p.rq, out, g, pixels);
  } else {
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(k_conv_direct_s8<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem));
    k_conv_direct_s8<8><<<grid, kBlock, smem, s>>>(in, p.filter, p.bias, p.rq, out, g, pixels);
  }
  return cudaGetLastError();
}

cudaError_t launch_fc_warp(const pspml_op_desc& d, const PreparedOp& p, int64_t batch,
                           const int8_t* in, int8_t* out, cudaStream_t s) {
  const Geom g = geom_of(d);
  const int64_t K = static_cast<int64_t>(d.in_h) * d.in_w * d.in_c;
  const int64_t total = batch * d.out_c;
  k_fc_warp_s8<<<grid_for(total * 32), kBlock, 0, s>>>(in, p.filter, p.bias, p.rq, out, K,
                                                       d.out_c, total, g);
  return cudaGetLastError();
}

cudaError_t launch_fc_gemv(const pspml_op_desc& d, const PreparedOp& p, int64_t batch,
                           const int8_t* in, int8_t* out, int num_sms, cudaStream_t s) {
  const Geom g = geom_of(d);
  const int64_t K = static_cast<int64_t>(d.in_h) * d.in_w * d.in_c;
  if (batch < 1 || batch > kGemvMaxBatch || K % 16 != 0 || K >= (1ll << 31) ||
      (reinterpret_cast<uintptr_t>(in) & 15u) != 0 ||
      (reinterpret_cast<uintptr_t>(p.filter) & 15u) != 0)
    return cudaErrorInvalidValue;
  const int64_t warps = std::min<int64_t>(d.out_c, static_cast<int64_t>(num_sms) * 64);
  const unsigned grid = static_cast<unsigned>((warps + 7) / 8);
  const int32_t k32 = static_cast<int32_t>(K);
  switch (batch) {
    case 1: k_fc_gemv_s8<1><<<grid, 256, 0, s>>>(in, p.filter, p.bias_eff, p.rq, out, k32, d.out_c, g); break;
    case 2: k_fc_gemv_s8<2><<<grid, 256, 0, s>>>(in, p.filter, p.bias_eff, p.rq, out, k32, d.out_c, g); break;
    case 3: k_fc_gemv_s8<3><<<grid, 256, 0, s>>>(in, p.filter, p.bias_eff, p.rq, out, k32, d.out_c, g); break;
    default: k_fc_gemv_s8<4><<<grid, 256, 0, s>>>(in, p.filter, p.bias_eff, p.rq, out, k32, d.out_c, g); break;
  }
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
  const bool global = g.Ho == 1 && g.Wo == 1 && g.KH == g.H && g.KW == g.W && g.pt == 0 &&
                      g.pl == 0;
  if (global && g.C % 16 == 0 && aligned(in, 16) && aligned(out, 16)) {
    const int64_t total = batch * (g.C / 16);
    k_gap_s8<<<grid_for(total), kBlock, 0, s>>>(in, out, g.H * g.W, g.C, d.act_min, d.act_max,
                                                total);
  } else if (g.C % 16 == 0 && aligned(in, 16) && aligned(out, 16)) {
    // 16 channels a thread: a warp reads 512 contiguous bytes per pixel.
    const int64_t total = pix * (g.C / 16);
    k_avgpool_s8<16><<<grid_for(total), kBlock, 0, s>>>(in, out, g, d.act_min, d.act_max, total);
  } else if (g.C % 4 == 0 && aligned(in, 4) && aligned(out, 4)) {
    const int64_t total = pix * (g.C / 4);
    k_avgpool_s8<4><<<grid_for(total), kBlock, 0, s>>>(in, out, g, d.act_min, d.act_max, total);
  } else {
    const int64_t total = pix * g.C;
    k_avgpool_s8<1><<<grid_for(total), kBlock, 0, s>>>(in, out, g, d.act_min, d.act_max, total);
  }
  return cudaGetLastError();
}

}  // namespace pspml
