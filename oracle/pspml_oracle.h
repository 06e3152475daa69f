/*
 * pspml_oracle.h - CPU oracle for the psp-ml inference path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the checker the parity tests, the
 * smoke check and the CPU-baseline leg of the benchmark compare against.
 * The product library never links, loads or calls it.
 *
 * Two families:
 *  - f32: a restatement of the reference's own kernels, same loop nests and
 *    summation order (psp-ml/src/kernels/naive.rs, psp-ml/src/kernels/mod.rs
 *    host paths).  Compiled with -ffp-contract=off so a*b+c is never fused,
 *    matching rustc's default.  Pinned by the reference's known-answer tests
 *    (psp-ml/src/bin/test-kernels.rs:47-390).
 *  - int8: TFLite's int8 reference semantics (per-channel conv / depthwise /
 *    fully-connected with gemmlowp fixed-point requantisation, max / average
 *    pooling).  The reference has no int8 kernels, so these are written from
 *    the published fixed-point method (gemmlowp SaturatingRoundingDoubling-
 *    HighMul + RoundingDivideByPOT, TFLite MultiplyByQuantizedMultiplier and
 *    QuantizeMultiplier).  Parity for int8 is therefore UNPINNED against the
 *    reference; it is pinned against hand-computed known answers instead.
 */
#ifndef PSPML_ORACLE_H
#define PSPML_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#include "../include/pspml.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- f32 */
void orc_f32_conv2d(const float* in, const int64_t in_shape[4],
                    const float* filter, const int64_t f_shape[4],
                    const float* bias, const int64_t stride[2],
                    const int64_t padding[2], float* out,
                    const int64_t out_shape[4]);
void orc_f32_conv2d_relu(const float* in, const int64_t in_shape[4],
                         const float* filter, const int64_t f_shape[4],
                         const float* bias, const int64_t stride[2],
                         const int64_t padding[2], float* out,
                         const int64_t out_shape[4]);
void orc_f32_max_pool2d(const float* in, const int64_t in_shape[4],
                        const int64_t kernel[2], const int64_t stride[2],
                        float* out, const int64_t out_shape[4]);
void orc_f32_reshape(const float* in, float* out, int64_t n);
void orc_f32_fully_connected(const float* in, int64_t in_features,
                             const float* w, const float* b, float* out,
                             int64_t out_features);
void orc_f32_fully_connected_relu(const float* in, int64_t in_features,
                                  const float* w, const float* b, float* out,
                                  int64_t out_features);
void orc_f32_matmul_bt(const float* a, const float* b, float* c, int64_t m,
                       int64_t k, int64_t n);
void orc_f32_matmul_bt_tiled(const float* a, const float* b, float* c,
                             int64_t m_tiles, int64_t k_tiles,
                             int64_t n_tiles);
void orc_f32_relu(float* data, int64_t n);
void orc_f32_im2col(const float* in, const int64_t in_shape[4],
                    const int64_t kernel[2], const int64_t stride[2],
                    const int64_t padding[2], const int64_t out_hw[2],
                    float* col);
void orc_f32_im2col_padded(const float* in, const int64_t in_shape[4],
                           const int64_t kernel[2], const int64_t padding[2],
                           const int64_t out_hw[2], float* col);
void orc_f32_bias_add(float* data, const float* bias, int64_t rows,
                      int64_t cols);
/* SAME padding split (cargo-psp-ml/src/parse/tflite/lowering.rs:341-364):
 * out = {top, bottom, left, right}. */
void orc_same_padding(int64_t in_h, int64_t in_w, int64_t k_h, int64_t k_w,
                      int64_t s_h, int64_t s_w, int64_t out[4]);

/* --------------------------------------------------------------- int8 */
int32_t orc_srdhm(int32_t a, int32_t b);
int32_t orc_rdbpot(int32_t x, int32_t exponent);
int32_t orc_mbqm(int32_t x, int32_t multiplier, int32_t shift);
void orc_quantize_multiplier(double real, int32_t* multiplier, int32_t* shift);

/* One op over `batch` samples (tensors passed directly). */
int orc_op_s8(const pspml_op_desc* d, int64_t batch, const int8_t* in,
              const int8_t* filter, const int32_t* bias, const int32_t* mult,
              const int32_t* shift, int8_t* out);

/* Whole chain (ops index a weight blob as in pspml_model_create), OpenMP
 * over the batch with `threads` threads (<= 0: all). */
int orc_net_forward_s8(const pspml_op_desc* ops, int32_t n_ops,
                       const uint8_t* blob, int64_t batch, const int8_t* in,
                       int8_t* out, int32_t threads);

#ifdef __cplusplus
}
#endif

#endif
