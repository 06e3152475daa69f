/*
 * pspml_oracle.c - CPU oracle for the psp-ml inference path.
 *
 * TEST INFRASTRUCTURE ONLY (see pspml_oracle.h).  Only the test suite, the
 * smoke check and the benchmark's CPU-baseline leg load this library; the
 * product path never does.
 *
 * Build: oracle/Makefile (gcc -O3 -fopenmp -ffp-contract=off).
 */
#include "pspml_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ======================================================================
 * f32: restatement of psp-ml/src/kernels/{naive.rs,mod.rs} host paths.
 * Loop nests and summation order follow the cited lines exactly; the file
 * is compiled with -ffp-contract=off so products and sums round separately
 * as in the Rust build.
 * ==================================================================== */

/* naive.rs:13-66 - direct NHWC conv; the sum starts at bias[oc] (or 0) and
 * adds x*w in ky, kx, ic order; taps in the zero padding are skipped. */
void orc_f32_conv2d(const float* in, const int64_t in_shape[4],
                    const float* filter, const int64_t f_shape[4],
                    const float* bias, const int64_t stride[2],
                    const int64_t padding[2], float* out,
                    const int64_t out_shape[4]) {
  const int64_t n = in_shape[0], h = in_shape[1], w = in_shape[2],
                ci = in_shape[3];
  const int64_t co = f_shape[0], kh = f_shape[1], kw = f_shape[2];
  const int64_t ho = out_shape[1], wo = out_shape[2];
  for (int64_t b = 0; b < n; ++b)
    for (int64_t oy = 0; oy < ho; ++oy)
      for (int64_t ox = 0; ox < wo; ++ox)
        for (int64_t oc = 0; oc < co; ++oc) {
          float sum = bias ? bias[oc] : 0.0f;
          for (int64_t ky = 0; ky < kh; ++ky)
            for (int64_t kx = 0; kx < kw; ++kx) {
              const int64_t iyp = oy * stride[0] + ky;
              const int64_t ixp = ox * stride[1] + kx;
              if (iyp < padding[0] || ixp < padding[1]) continue;
              const int64_t iy = iyp - padding[0], ix = ixp - padding[1];
              if (iy >= h || ix >= w) continue;
              for (int64_t ic = 0; ic < ci; ++ic) {
                const float xv = in[b * (h * w * ci) + iy * (w * ci) + ix * ci + ic];
                const float wv = filter[oc * (kh * kw * ci) + ky * (kw * ci) + kx * ci + ic];
                const float prod = xv * wv;
                sum = sum + prod;
              }
            }
          out[b * (ho * wo * co) + oy * (wo * co) + ox * co + oc] = sum;
        }
}

/* naive.rs:75-92 - conv2d followed by `if v < 0 { v = 0 }` (keeps -0.0). */
void orc_f32_conv2d_relu(const float* in, const int64_t in_shape[4],
                         const float* filter, const int64_t f_shape[4],
                         const float* bias, const int64_t stride[2],
                         const int64_t padding[2], float* out,
                         const int64_t out_shape[4]) {
  orc_f32_conv2d(in, in_shape, filter, f_shape, bias, stride, padding, out,
                 out_shape);
  const int64_t total = out_shape[0] * out_shape[1] * out_shape[2] * out_shape[3];
  for (int64_t i = 0; i < total; ++i)
    if (out[i] < 0.0f) out[i] = 0.0f;
}

/* naive.rs:98-132 - max over the window starting from -inf, strict `>`. */
void orc_f32_max_pool2d(const float* in, const int64_t in_shape[4],
                        const int64_t kernel[2], const int64_t stride[2],
                        float* out, const int64_t out_shape[4]) {
  const int64_t n = in_shape[0], h = in_shape[1], w = in_shape[2],
                c = in_shape[3];
  const int64_t ho = out_shape[1], wo = out_shape[2];
  for (int64_t b = 0; b < n; ++b)
    for (int64_t oy = 0; oy < ho; ++oy)
      for (int64_t ox = 0; ox < wo; ++ox)
        for (int64_t ch = 0; ch < c; ++ch) {
          float m = -INFINITY;
          for (int64_t ky = 0; ky < kernel[0]; ++ky)
            for (int64_t kx = 0; kx < kernel[1]; ++kx) {
              const int64_t iy = oy * stride[0] + ky, ix = ox * stride[1] + kx;
              const float v = in[b * (h * w * c) + iy * (w * c) + ix * c + ch];
              if (v > m) m = v;
            }
          out[b * (ho * wo * c) + oy * (wo * c) + ox * c + ch] = m;
        }
}

/* naive.rs:135-139 */
void orc_f32_reshape(const float* in, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = in[i];
}

/* naive.rs:147-162 - the sum starts at bias[o], inputs in order. */
void orc_f32_fully_connected(const float* in, int64_t in_features,
                             const float* w, const float* b, float* out,
                             int64_t out_features) {
  for (int64_t o = 0; o < out_features; ++o) {
    float sum = b[o];
    for (int64_t i = 0; i < in_features; ++i) {
      const float prod = in[i] * w[o * in_features + i];
      sum = sum + prod;
    }
    out[o] = sum;
  }
}

/* naive.rs:170-184 */
void orc_f32_fully_connected_relu(const float* in, int64_t in_features,
                                  const float* w, const float* b, float* out,
                                  int64_t out_features) {
  orc_f32_fully_connected(in, in_features, w, b, out, out_features);
  for (int64_t o = 0; o < out_features; ++o)
    if (out[o] < 0.0f) out[o] = 0.0f;
}

/* mod.rs:176-198 with load_tile/store_tile (mod.rs:25-79) and the host
 * vfpu_mul_acc_bt (mod.rs:127-135): 4x4 tiles, zero-padded at the edges,
 * acc[i][j] += a[i][k] * b[j][k] for k in tile order. */
void orc_f32_matmul_bt(const float* a, const float* b, float* c, int64_t m,
                       int64_t k, int64_t n) {
  const int64_t Q = 4;
  const int64_t tm = (m + Q - 1) / Q, tn = (n + Q - 1) / Q, tk = (k + Q - 1) / Q;
  for (int64_t ti = 0; ti < tm; ++ti)
    for (int64_t tj = 0; tj < tn; ++tj) {
      float acc[16] = {0};
      for (int64_t t = 0; t < tk; ++t) {
        float at[16] = {0}, bt[16] = {0};
        for (int64_t r = 0; r < Q; ++r)
          for (int64_t cc = 0; cc < Q; ++cc) {
            const int64_t ar = ti * Q + r, br = tj * Q + r, col = t * Q + cc;
            if (ar < m && col < k) at[r * Q + cc] = a[ar * k + col];
            if (br < n && col < k) bt[r * Q + cc] = b[br * k + col];
          }
        for (int64_t i = 0; i < Q; ++i)
          for (int64_t j = 0; j < Q; ++j)
            for (int64_t kk = 0; kk < Q; ++kk) {
              const float prod = at[i * Q + kk] * bt[j * Q + kk];
              acc[i * Q + j] = acc[i * Q + j] + prod;
            }
      }
      for (int64_t r = 0; r < Q; ++r)
        for (int64_t cc = 0; cc < Q; ++cc) {
          const int64_t row = ti * Q + r, col = tj * Q + cc;
          if (row < m && col < n) c[row * n + col] = acc[r * Q + cc];
        }
    }
}

/* mod.rs:310-344 (host build of matmul_bt_tiled): pre-padded operands. */
void orc_f32_matmul_bt_tiled(const float* a, const float* b, float* c,
                             int64_t m_tiles, int64_t k_tiles,
                             int64_t n_tiles) {
  const int64_t Q = 4, k = k_tiles * Q, n = n_tiles * Q;
  for (int64_t ti = 0; ti < m_tiles; ++ti)
    for (int64_t tj = 0; tj < n_tiles; ++tj) {
      float acc[16] = {0};
      for (int64_t t = 0; t < k_tiles; ++t)
        for (int64_t r = 0; r < Q; ++r)
          for (int64_t cc = 0; cc < Q; ++cc)
            for (int64_t kk = 0; kk < Q; ++kk) {
              const float av = a[(ti * Q + r) * k + t * Q + kk];
              const float bv = b[(tj * Q + cc) * k + t * Q + kk];
              const float prod = av * bv;
              acc[r * Q + cc] = acc[r * Q + cc] + prod;
            }
      for (int64_t r = 0; r < Q; ++r)
        for (int64_t cc = 0; cc < Q; ++cc)
          c[(ti * Q + r) * n + tj * Q + cc] = acc[r * Q + cc];
    }
}

/* mod.rs:347-364 (host vfpu_relu4 + scalar tail): `if x < 0 { x = 0 }`. */
void orc_f32_relu(float* data, int64_t n) {
  for (int64_t i = 0; i < n; ++i)
    if (data[i] < 0.0f) data[i] = 0.0f;
}

/* mod.rs:374-415 */
void orc_f32_im2col(const float* in, const int64_t in_shape[4],
                    const int64_t kernel[2], const int64_t stride[2],
                    const int64_t padding[2], const int64_t out_hw[2],
                    float* col) {
  const int64_t n = in_shape[0], h = in_shape[1], w = in_shape[2],
                ci = in_shape[3];
  const int64_t kh = kernel[0], kw = kernel[1], k = kh * kw * ci;
  for (int64_t b = 0; b < n; ++b)
    for (int64_t oy = 0; oy < out_hw[0]; ++oy)
      for (int64_t ox = 0; ox < out_hw[1]; ++ox) {
        const int64_t row = b * (out_hw[0] * out_hw[1]) + oy * out_hw[1] + ox;
        for (int64_t ky = 0; ky < kh; ++ky)
          for (int64_t kx = 0; kx < kw; ++kx) {
            const int64_t iy = oy * stride[0] + ky - padding[0];
            const int64_t ix = ox * stride[1] + kx - padding[1];
            for (int64_t ic = 0; ic < ci; ++ic) {
              const int64_t ci_idx = ky * (kw * ci) + kx * ci + ic;
              const int inside = iy >= 0 && iy < h && ix >= 0 && ix < w;
              col[row * k + ci_idx] =
                  inside ? in[b * (h * w * ci) + iy * (w * ci) + ix * ci + ic] : 0.0f;
            }
          }
      }
}

/* mod.rs:427-467 - stride 1, row pitch ceil4(K); pad columns untouched. */
void orc_f32_im2col_padded(const float* in, const int64_t in_shape[4],
                           const int64_t kernel[2], const int64_t padding[2],
                           const int64_t out_hw[2], float* col) {
  const int64_t n = in_shape[0], h = in_shape[1], w = in_shape[2],
                ci = in_shape[3];
  const int64_t kh = kernel[0], kw = kernel[1], k = kh * kw * ci;
  const int64_t kp = (k + 3) / 4 * 4;
  for (int64_t b = 0; b < n; ++b)
    for (int64_t oy = 0; oy < out_hw[0]; ++oy)
      for (int64_t ox = 0; ox < out_hw[1]; ++ox) {
        const int64_t row = b * (out_hw[0] * out_hw[1]) + oy * out_hw[1] + ox;
        for (int64_t ky = 0; ky < kh; ++ky)
          for (int64_t kx = 0; kx < kw; ++kx) {
            const int64_t iy = oy + ky - padding[0];
            const int64_t ix = ox + kx - padding[1];
            for (int64_t ic = 0; ic < ci; ++ic) {
              const int64_t ci_idx = ky * (kw * ci) + kx * ci + ic;
              const int inside = iy >= 0 && iy < h && ix >= 0 && ix < w;
              col[row * kp + ci_idx] =
                  inside ? in[b * (h * w * ci) + iy * (w * ci) + ix * ci + ic] : 0.0f;
            }
          }
      }
}

/* mod.rs:473-479 */
void orc_f32_bias_add(float* data, const float* bias, int64_t rows,
                      int64_t cols) {
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < cols; ++c)
      data[r * cols + c] = data[r * cols + c] + bias[c];
}

/* cargo-psp-ml/src/parse/tflite/lowering.rs:341-364 */
void orc_same_padding(int64_t in_h, int64_t in_w, int64_t k_h, int64_t k_w,
                      int64_t s_h, int64_t s_w, int64_t out[4]) {
  const int64_t oh = (in_h + s_h - 1) / s_h, ow = (in_w + s_w - 1) / s_w;
  int64_t th = (oh - 1) * s_h + k_h - in_h;
  int64_t tw = (ow - 1) * s_w + k_w - in_w;
  if (th < 0) th = 0;
  if (tw < 0) tw = 0;
  out[0] = th / 2;
  out[1] = th - th / 2;
  out[2] = tw / 2;
  out[3] = tw - tw / 2;
}

/* ======================================================================
 * int8: TFLite int8 reference semantics, written from the published
 * fixed-point method (gemmlowp fixedpoint.h; TFLite common.h /
 * quantization_util.cc; reference_integer_ops conv / depthwise_conv /
 * fully_connected / pooling).  Third-party spec, not vendored by the
 * reference and not exercised by it: parity UNPINNED against the reference.
 * ==================================================================== */

/* gemmlowp SaturatingRoundingDoublingHighMul: (a*b + nudge) / 2^31 with the
 * quotient truncated toward zero; nudge = 2^30 for a non-negative product,
 * 1 - 2^30 otherwise; INT32_MIN * INT32_MIN saturates to INT32_MAX. */
int32_t orc_srdhm(int32_t a, int32_t b) {
  if (a == INT32_MIN && b == INT32_MIN) return INT32_MAX;
  const int64_t ab = (int64_t)a * (int64_t)b;
  const int64_t nudge = ab >= 0 ? (INT64_C(1) << 30) : (INT64_C(1) - (INT64_C(1) << 30));
  const int64_t q = (ab + nudge) / (INT64_C(1) << 31); /* C division truncates */
  return (int32_t)q;
}

/* gemmlowp RoundingDivideByPOT: arithmetic shift right by `exponent` with
 * round-half-away-from-zero. */
int32_t orc_rdbpot(int32_t x, int32_t exponent) {
  const int32_t mask = (int32_t)((UINT32_C(1) << exponent) - 1);
  const int32_t remainder = x & mask;
  const int32_t threshold = (mask >> 1) + (x < 0 ? 1 : 0);
  return (x >> exponent) + (remainder > threshold ? 1 : 0);
}

/* TFLite MultiplyByQuantizedMultiplier (double-rounding form).  The left
 * shift of x is done in unsigned arithmetic (wraps instead of being C UB). */
int32_t orc_mbqm(int32_t x, int32_t multiplier, int32_t shift) {
  const int32_t left = shift > 0 ? shift : 0;
  const int32_t right = shift > 0 ? 0 : -shift;
  const int32_t xs = (int32_t)((uint32_t)x << left);
  return orc_rdbpot(orc_srdhm(xs, multiplier), right);
}

/* TFLite QuantizeMultiplier: real = M * 2^(shift-31), M in [2^30, 2^31). */
void orc_quantize_multiplier(double real, int32_t* multiplier, int32_t* shift) {
  if (real == 0.0) {
    *multiplier = 0;
    *shift = 0;
    return;
  }
  int e = 0;
  const double q = frexp(real, &e);
  int64_t q_fixed = (int64_t)round(q * (double)(INT64_C(1) << 31));
  if (q_fixed == (INT64_C(1) << 31)) {
    q_fixed /= 2;
    ++e;
  }
  if (e < -31) {
    e = 0;
    q_fixed = 0;
  }
  if (e > 30) {
    e = 30;
    q_fixed = (INT64_C(1) << 31) - 1;
  }
  *multiplier = (int32_t)q_fixed;
  *shift = e;
}

static inline int8_t orc_finish(int32_t acc, int32_t mult, int32_t shift,
                                const pspml_op_desc* d) {
  int32_t v = orc_mbqm(acc, mult, shift) + d->zp_out;
  if (v < d->act_min) v = d->act_min;
  if (v > d->act_max) v = d->act_max;
  return (int8_t)v;
}

/* reference_integer_ops::ConvPerChannel (dilation 1): taps outside the
 * image are skipped, i.e. padding is the real value 0 (quantised zp_in). */
static void orc_conv_one(const pspml_op_desc* d, const int8_t* in,
                         const int8_t* f, const int32_t* bias,
                         const int32_t* mult, const int32_t* shift,
                         int8_t* out) {
  const int32_t H = d->in_h, W = d->in_w, C = d->in_c;
  const int32_t Ho = d->out_h, Wo = d->out_w, Co = d->out_c;
  const int32_t KH = d->kernel_h, KW = d->kernel_w;
  for (int32_t oy = 0; oy < Ho; ++oy)
    for (int32_t ox = 0; ox < Wo; ++ox)
      for (int32_t oc = 0; oc < Co; ++oc) {
        const int32_t iy0 = oy * d->stride_h - d->pad_top;
        const int32_t ix0 = ox * d->stride_w - d->pad_left;
        int32_t acc = 0;
        for (int32_t ky = 0; ky < KH; ++ky)
          for (int32_t kx = 0; kx < KW; ++kx) {
            const int32_t iy = iy0 + ky, ix = ix0 + kx;
            if (iy < 0 || iy >= H || ix < 0 || ix >= W) continue;
            for (int32_t ic = 0; ic < C; ++ic) {
              const int32_t xv = in[((int64_t)iy * W + ix) * C + ic];
              const int32_t wv = f[(((int64_t)oc * KH + ky) * KW + kx) * C + ic];
              acc += wv * (xv - d->zp_in);
            }
          }
        if (bias) acc += bias[oc];
        out[((int64_t)oy * Wo + ox) * Co + oc] = orc_finish(acc, mult[oc], shift[oc], d);
      }
}

/* reference_integer_ops::DepthwiseConvPerChannel, depth multiplier 1;
 * filter [KH][KW][C]. */
static void orc_dw_one(const pspml_op_desc* d, const int8_t* in,
                       const int8_t* f, const int32_t* bias,
                       const int32_t* mult, const int32_t* shift,
                       int8_t* out) {
  const int32_t H = d->in_h, W = d->in_w, C = d->in_c;
  const int32_t Ho = d->out_h, Wo = d->out_w;
  const int32_t KH = d->kernel_h, KW = d->kernel_w;
  for (int32_t oy = 0; oy < Ho; ++oy)
    for (int32_t ox = 0; ox < Wo; ++ox)
      for (int32_t c = 0; c < C; ++c) {
        const int32_t iy0 = oy * d->stride_h - d->pad_top;
        const int32_t ix0 = ox * d->stride_w - d->pad_left;
        int32_t acc = 0;
        for (int32_t ky = 0; ky < KH; ++ky)
          for (int32_t kx = 0; kx < KW; ++kx) {
            const int32_t iy = iy0 + ky, ix = ix0 + kx;
            if (iy < 0 || iy >= H || ix < 0 || ix >= W) continue;
            const int32_t xv = in[((int64_t)iy * W + ix) * C + c];
            const int32_t wv = f[((int64_t)ky * KW + kx) * C + c];
            acc += wv * (xv - d->zp_in);
          }
        if (bias) acc += bias[c];
        out[((int64_t)oy * Wo + ox) * C + c] = orc_finish(acc, mult[c], shift[c], d);
      }
}

/* reference_integer_ops::FullyConnectedPerChannel (filter offset 0). */
static void orc_fc_one(const pspml_op_desc* d, const int8_t* in,
                       const int8_t* f, const int32_t* bias,
                       const int32_t* mult, const int32_t* shift,
                       int8_t* out) {
  const int64_t K = (int64_t)d->in_h * d->in_w * d->in_c;
  const int32_t N = d->out_c;
  for (int32_t o = 0; o < N; ++o) {
    int32_t acc = 0;
    for (int64_t k = 0; k < K; ++k)
      acc += (int32_t)f[(int64_t)o * K + k] * ((int32_t)in[k] - d->zp_in);
    if (bias) acc += bias[o];
    out[o] = orc_finish(acc, mult[o], shift[o], d);
  }
}

/* reference_integer_ops::MaxPool: window clipped to the image, max starts
 * at the lowest int8, then clamped to the activation range. */
static void orc_maxpool_one(const pspml_op_desc* d, const int8_t* in,
                            int8_t* out) {
  const int32_t H = d->in_h, W = d->in_w, C = d->in_c;
  for (int32_t oy = 0; oy < d->out_h; ++oy)
    for (int32_t ox = 0; ox < d->out_w; ++ox)
      for (int32_t c = 0; c < C; ++c) {
        const int32_t iy0 = oy * d->stride_h - d->pad_top;
        const int32_t ix0 = ox * d->stride_w - d->pad_left;
        int32_t m = -128;
        for (int32_t ky = 0; ky < d->kernel_h; ++ky)
          for (int32_t kx = 0; kx < d->kernel_w; ++kx) {
            const int32_t iy = iy0 + ky, ix = ix0 + kx;
            if (iy < 0 || iy >= H || ix < 0 || ix >= W) continue;
            const int32_t v = in[((int64_t)iy * W + ix) * C + c];
            if (v > m) m = v;
          }
        if (m < d->act_min) m = d->act_min;
        if (m > d->act_max) m = d->act_max;
        out[((int64_t)oy * d->out_w + ox) * C + c] = (int8_t)m;
      }
}

/* reference_integer_ops::AveragePool: sum of the in-image window, divided
 * by the count with round-half-away-from-zero, clamped. */
static int orc_avgpool_one(const pspml_op_desc* d, const int8_t* in,
                           int8_t* out) {
  const int32_t H = d->in_h, W = d->in_w, C = d->in_c;
  for (int32_t oy = 0; oy < d->out_h; ++oy)
    for (int32_t ox = 0; ox < d->out_w; ++ox)
      for (int32_t c = 0; c < C; ++c) {
        const int32_t iy0 = oy * d->stride_h - d->pad_top;
        const int32_t ix0 = ox * d->stride_w - d->pad_left;
        int32_t acc = 0, cnt = 0;
        for (int32_t ky = 0; ky < d->kernel_h; ++ky)
          for (int32_t kx = 0; kx < d->kernel_w; ++kx) {
            const int32_t iy = iy0 + ky, ix = ix0 + kx;
            if (iy < 0 || iy >= H || ix < 0 || ix >= W) continue;
            acc += in[((int64_t)iy * W + ix) * C + c];
            ++cnt;
          }
        if (cnt == 0) return -1;
        acc = acc > 0 ? (acc + cnt / 2) / cnt : (acc - cnt / 2) / cnt;
        if (acc < d->act_min) acc = d->act_min;
        if (acc > d->act_max) acc = d->act_max;
        out[((int64_t)oy * d->out_w + ox) * C + c] = (int8_t)acc;
      }
  return 0;
}

static int64_t desc_in_elems(const pspml_op_desc* d) {
  return (int64_t)d->in_h * d->in_w * d->in_c;
}
static int64_t desc_out_elems(const pspml_op_desc* d) {
  return (int64_t)d->out_h * d->out_w * d->out_c;
}

static int orc_op_one(const pspml_op_desc* d, const int8_t* in,
                      const int8_t* f, const int32_t* bias,
                      const int32_t* mult, const int32_t* shift,
                      int8_t* out) {
  switch (d->kind) {
    case PSPML_OP_CONV2D:
      orc_conv_one(d, in, f, bias, mult, shift, out);
      return 0;
    case PSPML_OP_DEPTHWISE_CONV2D:
      orc_dw_one(d, in, f, bias, mult, shift, out);
      return 0;
    case PSPML_OP_FULLY_CONNECTED:
      orc_fc_one(d, in, f, bias, mult, shift, out);
      return 0;
    case PSPML_OP_MAX_POOL2D:
      orc_maxpool_one(d, in, out);
      return 0;
    case PSPML_OP_AVERAGE_POOL2D:
      return orc_avgpool_one(d, in, out);
    case PSPML_OP_RESHAPE:
      memcpy(out, in, (size_t)desc_in_elems(d));
      return 0;
    default:
      return -1;
  }
}

int orc_op_s8(const pspml_op_desc* d, int64_t batch, const int8_t* in,
              const int8_t* filter, const int32_t* bias, const int32_t* mult,
              const int32_t* shift, int8_t* out) {
  const int64_t ie = desc_in_elems(d), oe = desc_out_elems(d);
  int bad = 0;
#pragma omp parallel for schedule(static) reduction(| : bad)
  for (int64_t b = 0; b < batch; ++b)
    bad |= orc_op_one(d, in + b * ie, filter, bias, mult, shift, out + b * oe) != 0;
  return bad ? -1 : 0;
}

static const void* blob_at(const uint8_t* blob, int64_t off) {
  return off < 0 ? NULL : (const void*)(blob + off);
}

int orc_net_forward_s8(const pspml_op_desc* ops, int32_t n_ops,
                       const uint8_t* blob, int64_t batch, const int8_t* in,
                       int8_t* out, int32_t threads) {
  if (n_ops <= 0) return -1;
  int64_t max_elems = desc_in_elems(&ops[0]);
  for (int32_t i = 0; i < n_ops; ++i) {
    if (desc_in_elems(&ops[i]) > max_elems) max_elems = desc_in_elems(&ops[i]);
    if (desc_out_elems(&ops[i]) > max_elems) max_elems = desc_out_elems(&ops[i]);
  }
  const int64_t in_elems = desc_in_elems(&ops[0]);
  const int64_t out_elems = desc_out_elems(&ops[n_ops - 1]);
  int bad = 0;
#ifdef _OPENMP
  if (threads <= 0) threads = omp_get_max_threads();
#else
  (void)threads;
#endif
#pragma omp parallel num_threads(threads) reduction(| : bad)
  {
    int8_t* a = (int8_t*)malloc((size_t)max_elems);
    int8_t* b = (int8_t*)malloc((size_t)max_elems);
    if (!a || !b) {
      bad = 1;
    } else {
#pragma omp for schedule(dynamic, 1)
      for (int64_t s = 0; s < batch; ++s) {
        const int8_t* cur = in + s * in_elems;
        int8_t* dst = a;
        for (int32_t i = 0; i < n_ops; ++i) {
          const pspml_op_desc* d = &ops[i];
          int8_t* o = (i == n_ops - 1) ? out + s * out_elems : dst;
          bad |= orc_op_one(d, cur, (const int8_t*)blob_at(blob, d->filter_off),
                            (const int32_t*)blob_at(blob, d->bias_off),
                            (const int32_t*)blob_at(blob, d->mult_off),
                            (const int32_t*)blob_at(blob, d->shift_off), o) != 0;
          cur = o;
          dst = (dst == a) ? b : a;
        }
      }
    }
    free(a);
    free(b);
  }
  return bad ? -1 : 0;
}
