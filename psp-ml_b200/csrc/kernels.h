// kernels.h - device-side preparation and launch of the int8 ops (host C++).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/pspml.h"
#include "requant.cuh"

namespace pspml {

// Which kernel runs an op.
enum class OpPath {
  kTc2d,       // tcgen05 GEMM, A = [rows][K] (FC, 1x1 stride-1 conv)
  kTc4d,       // tcgen05 implicit GEMM over NHWC (stride-1 conv, in_c % 16 == 0)
  kSmallConv,  // CUDA-core dp4a conv over packed patches (small in_c)
  kDirect,     // CUDA-core conv, any shape (fallback)
  kFcWarp,     // CUDA-core FC, one warp per output (K % 16 != 0)
  kDwTc,       // tcgen05 depthwise 3x3 stride 1 (block-diagonal), C % 32 == 0
  kDw3x3,      // CUDA-core dp4a depthwise 3x3, C % 4 == 0
  kDwGeneric,  // CUDA-core depthwise, any shape (fallback)
  kMaxPool,
  kAvgPool,
  kReshape
};

// Border classes of a conv with padding: output row y has class ycls[y],
// column x has class xcls[x]; ymask/xmask give the in-image filter taps of
// each class.
struct BorderClasses {
  int32_t n_ycls = 1, n_xcls = 1;
  uint32_t ymask[64] = {0};
  uint32_t xmask[64] = {0};
  uint8_t ycls[4096];
  uint8_t xcls[4096];
};
bool build_border_classes(const pspml_op_desc& d, BorderClasses* bc);

// Requantisation constants and folded biases of one op passed to the GEMM
// kernel as a __grid_constant__ parameter: the epilogue's per-channel
// reads are warp-uniform, and the constant bank serves them without
// occupying the L1 data pipe (staging them in shared memory made that pipe
// the bottleneck: every lane reloads the same 20 bytes per output).
// Per channel {M, C_hi} and {bias of the base border class, shift}; the
// other border classes add a per-(class, channel) bias difference.  The low
// word of C is 2^30 for every channel whose right shift is >= 2, which the
// host checks before it builds a table.  When a kernel's channel block is
// fixed, the table offsets are compile-time constants and the epilogue reads
// the entries as constant-bank operands with no load instruction at all.
constexpr int kTabRq = 512;
constexpr int kTabDelta = 4608;  // 9 border classes x 512 channels
struct EpiTable {
  // Fast form: mh = {M, high word of C - 2^32}, bs = {folded bias of class
  // base_cls, right shift - 1}; floor form (floor_entry): the bias folded
  // into D, mh = D as one 64-bit word {low, high}, bs = {M, right shift - 1}.
  int2 mh[kTabRq];
  int2 bs[kTabRq];
  int32_t dbias[kTabDelta];  // [ncls][N]: folded bias of the class - that of base_cls
};

// Fast requant with the table's split constants (C low word = 2^30); `a` is
// the accumulator plus the folded bias.
__device__ __forceinline__ int32_t rq_tab(int32_t a, const int2 mh, int32_t sr) {
  const int64_t c =
      static_cast<int64_t>((static_cast<uint64_t>(static_cast<uint32_t>(mh.y)) << 32) |
                           0x40000000u);
  const int64_t t = static_cast<int64_t>(a) * mh.x + c;
  const uint32_t lo = static_cast<uint32_t>(t);
  const int32_t hi = static_cast<int32_t>(t >> 32);
  return (hi + static_cast<int32_t>((~static_cast<uint32_t>(a) | lo) >> 31)) >> sr;
}

// Epilogue variants of the table kernels: bit 0 clamps to the activation
// range (narrower than int8), bit 1 takes the floor form.
constexpr int kEpClamp = 1;
constexpr int kEpFloor = 2;
inline int ep_flags(int32_t act_min, int32_t act_max, int32_t zp_out) {
  return ((act_min > -128 || act_max < 127) ? kEpClamp : 0) |
         (act_min >= zp_out ? kEpFloor : 0);
}

// Floor-form table entry (ops with act_min >= zp_out, rq_fast_floor): the
// folded bias moves into the 64-bit addend, D = bias * M + C with the full
// C = 2^30 + 2^(30+r) + zp_out * 2^(31+r); the entry is
// mh = D as one 64-bit word (low word first), bs = {M, r - 1}, and
//   out + zp_out = high word of (acc * M + D) >> (r - 1).
// One wide multiply-add and one shift per output.  D is stored whole so the
// multiply-add reads it as one 64-bit operand: assembling it from two
// separate words cost two register moves per output (14.4 against 18.0
// outputs per clock per SM on B200, measured in a requantisation
// microbenchmark).  The table builder makes
// these entries for exactly the ops whose ep_flags have kEpFloor, so every
// kernel reading an op's table agrees on its form.
__host__ inline void floor_entry(int32_t m, uint32_t c_lo, int32_t c_hi, int32_t sr,
                                 int32_t bias, int2* mh, int2* bs) {
  const int64_t c =
      static_cast<int64_t>((static_cast<uint64_t>(static_cast<uint32_t>(c_hi)) << 32) | c_lo) +
      (int64_t{1} << 32);
  const int64_t d = static_cast<int64_t>(bias) * m + c;
  *mh = make_int2(static_cast<int32_t>(static_cast<uint32_t>(static_cast<uint64_t>(d))),
                  static_cast<int32_t>(d >> 32));
  *bs = make_int2(m, sr);
}

// The 64-bit addend D of a floor-form entry (mh of floor_entry).
__device__ __forceinline__ int64_t floor_d(const int2& mh) {
  return *reinterpret_cast<const long long*>(&mh);
}

// Floor-form requantisation of an accumulator with entry (mh, bs).
__device__ __forceinline__ int32_t rq_floor_entry(uint32_t acc, const int2& mh, const int2& bs) {
  const int64_t t = static_cast<int64_t>(static_cast<int32_t>(acc)) * bs.x + floor_d(mh);
  return static_cast<int32_t>(t >> 32) >> bs.y;
}

// Table requantisation of an accumulator (plus any border-class bias
// difference) in the op's form.
template <int Q>
__device__ __forceinline__ int32_t rq_tab_q(uint32_t acc, const int2& mh, const int2& bs) {
  if constexpr ((Q & kEpFloor) != 0) {
    return rq_floor_entry(acc, mh, bs);
  } else {
    return rq_tab(static_cast<int32_t>(acc) + bs.x, mh, bs.y);
  }
}

// Requantises 16 accumulators of channels ch .. ch+15 (table entries, bias
// of the base class) into 16 packed bytes; Q: the op's ep_flags.
template <int Q>
__device__ __forceinline__ uint4 requant16_tab(const uint32_t* v, const EpiTable& tab, int ch,
                                               uint32_t lo4, uint32_t hi4) {
  uint32_t packed[4];
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    int32_t r[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = ch + 4 * g + k;
      if constexpr ((Q & kEpFloor) != 0) {
        r[k] = rq_tab_q<Q>(v[4 * g + k], tab.mh[c], tab.bs[c]);
      } else {
        const int2 bs = tab.bs[c];
        r[k] = rq_tab(static_cast<int32_t>(v[4 * g + k]) + bs.x, tab.mh[c], bs.y);
      }
    }
    uint32_t w = pack_sat4(r[0], r[1], r[2], r[3]);
    if constexpr ((Q & kEpClamp) != 0) w = clamp4(w, lo4, hi4);
    packed[g] = w;
  }
  return make_uint4(packed[0], packed[1], packed[2], packed[3]);
}

// Adds the bias difference of a non-base border class (table offset `off`
// = class * N + first channel) to the first `cnt` of 16 accumulators.
__device__ __forceinline__ void add_class_delta(uint32_t* v, const EpiTable& tab, int off,
                                                int cnt) {
#pragma unroll
  for (int j = 0; j < 16; ++j)
    if (j < cnt) v[j] += static_cast<uint32_t>(tab.dbias[off + j]);
}

// Constant table of a depthwise conv and the pointwise conv fused after it
// (dwpw_tc.cu, dwrs_tc.cu): the depthwise op's split constants and
// per-class bias differences (up to 9 border classes x 256 channels), the
// pointwise op's split constants.
constexpr int kDwTabC = 512;
struct DwPwTable {
  int2 dw_mh[kDwTabC];
  int2 dw_bs[kDwTabC];
  int32_t dw_dbias[9 * kDwTabC];
  int2 pw_mh[256];
  int2 pw_bs[256];
};

// Constant table of a small-channel conv with 32 output channels and a
// patch of at most 16 bytes (the stem): split requant constants, folded
// bias (all taps, zp-filled halo) and the patch-order weight words.
struct SmallConvTable {
  int2 mh[32];
  int2 bs[32];  // {folded bias, right shift - 1}
  uint32_t w[32][4];
};

// Unsigned division by a divisor fixed at launch, for numerators below 2^31:
// q = (umulhi(n, m) + n) >> l with l = ceil(log2 d) and
// m = floor(2^32 (2^l - d) / d) + 1 (the round-up multiplier method of
// Granlund and Montgomery, "Division by invariant integers using
// multiplication", 1994).
struct FastDiv {
  uint32_t d = 1, m = 1;
  int32_t l = 0;
  FastDiv() = default;
  explicit FastDiv(uint32_t div) : d(div) {
    while ((1ull << l) < div) ++l;
    m = static_cast<uint32_t>((((1ull << 32) * ((1ull << l) - div)) / div) + 1);
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const {
    return (__umulhi(n, m) + n) >> l;
  }
};

// Everything a kernel needs beyond the activations, on the device.
struct PreparedOp {
  const EpiTable* table = nullptr;  // host copy for the constant-table epilogue (or null)
  OpPath path = OpPath::kDirect;
  const int8_t* filter = nullptr;   // TFLite-layout filter
  const int32_t* bias = nullptr;    // raw bias (fallback kernels)
  const int32_t* mult = nullptr;
  const int32_t* shift = nullptr;
  const uint32_t* wpack = nullptr;  // kSmallConv: [N][nw] patch-order words
  int32_t nw = 0;
  int32_t* bias_eff = nullptr;      // [ncls][N]: bias - zp_in * (in-image weight sum)
  RqChannel* rq = nullptr;          // [N]
  int32_t* rq_all_fast = nullptr;   // -1 when every channel has a fast-form entry, else 0
  bool all_fast_known = false;      // host knows every channel takes the fast form
  uint8_t* ycls = nullptr;          // [out_h] (tensor-core conv with ncls > 1)
  uint8_t* xcls = nullptr;          // [out_w]
  int32_t ncls = 1, n_xcls = 1;
  int32_t base_cls = 0;             // border class of an interior pixel (the table's base)
  const SmallConvTable* sc_table = nullptr;  // host copy (kSmallConv with 32 outputs)
};

// Input-channel / kernel shapes k_small_conv_s8 is instantiated for.
bool small_conv_supported(const pspml_op_desc& d);

// Depthwise shapes the tensor-core depthwise kernel takes (dw_tc.cu).
bool dw_tc_supported(const pspml_op_desc& d);
// Packs the block-diagonal weights ([C/32][9][2][32][16] bytes, 9216 per
// group) and folds the per-class bias; masks_dev holds 128 words.
cudaError_t prepare_dw_tc(const pspml_op_desc& d, const int8_t* filter, const int32_t* bias,
                          const BorderClasses& bc, uint8_t* wpack, int32_t* bias_eff,
                          uint32_t* masks_dev, cudaStream_t s);
cudaError_t launch_dw_tc(const pspml_op_desc& d, const PreparedOp& p, int64_t batch,
                         const int8_t* in, int8_t* out, unsigned* dev_err, int num_sms,
                         cudaStream_t s);

// Fused depthwise 3x3 + pointwise 1x1 pair (dwpw_tc.cu).
bool dwpw_pair_supported(const pspml_op_desc& dw, const pspml_op_desc& pw);
size_t dwpw_packed_bytes(const pspml_op_desc& pw);
// [N][C] pointwise filter -> [C/16][N][16] (K-major core-matrix order).
cudaError_t pack_pw_kmajor(const int8_t* filter, int32_t N, int32_t C, uint8_t* out,
                           cudaStream_t s);
cudaError_t launch_dwpw(const pspml_op_desc& dw, const PreparedOp& pdw, const pspml_op_desc& pw,
                        const uint8_t* wpw_packed, const DwPwTable& tab, int64_t batch,
                        const int8_t* in, int8_t* out, unsigned* dev_err, int num_sms,
                        cudaStream_t s);

// Row-streaming depthwise 3x3 (dwrs_tc.cu): every input row is one A
// operand whose MMA updates all the output rows it feeds.  Stride 1 or 2,
// rows of >= 64 output pixels, C in {32, 64} or a multiple of 64 up to 256;
// fused with a 64-output 1x1 conv for stride 1, C = 64, rows >= 128 px.
bool dwrs_dw_supported(const pspml_op_desc& d);
bool dwrs_pair_supported(const pspml_op_desc& dw, const pspml_op_desc& pw);
cudaError_t launch_dwrs_dw(const pspml_op_desc& d, const PreparedOp& p, int64_t batch,
                           const int8_t* in, int8_t* out, unsigned* dev_err, int num_sms,
                           cudaStream_t s);
cudaError_t launch_dwrs_pair(const pspml_op_desc& dw, const PreparedOp& pdw,
                             const pspml_op_desc& pw, const uint8_t* wpw_packed,
                             const DwPwTable& tab, int64_t batch, const int8_t* in, int8_t* out,
                             unsigned* dev_err, int num_sms, cudaStream_t s);

// A 3x3 stride-1 conv of 32 -> 32, 32 -> 64 or 64 -> 64 channels prepared
// for the implicit GEMM (kTc4d, constant table) run on the row-streaming
// kernel with dense weight blocks (dwrs_tc.cu): every input row is loaded
// once instead of once per filter tap.  pack_conv_rs writes the
// conv_rs_packed_bytes packed weights.  pool: the 2x2 / stride-2 max pool
// after the conv runs in its epilogue (out is then the pool's output; the
// pool descriptor must pass conv_pool_supported).
bool dense_rs_supported(const pspml_op_desc& conv, const PreparedOp& p);
size_t conv_rs_packed_bytes(const pspml_op_desc& conv);
cudaError_t pack_conv_rs(const pspml_op_desc& conv, const int8_t* filter, uint8_t* out,
                         cudaStream_t s);
cudaError_t launch_dense_rs(const pspml_op_desc& conv, const PreparedOp& p,
                            const uint8_t* wpack, int64_t batch, const int8_t* in, int8_t* out,
                            unsigned* dev_err, int num_sms, cudaStream_t s, bool pool = false);

// 3x3 convs with 1, 2, 3, 4 or 8 input channels and 16, 32 or 64 outputs
// on the tensor cores (im2col_tc.cu): patches gathered into a shared-memory
// A tile per 128 output pixels, requantised from tensor memory with the
// op's constant table.
bool im2col_conv_supported(const pspml_op_desc& d, const PreparedOp& p, const int8_t* in,
                           const int8_t* out);
cudaError_t launch_im2col_conv(const pspml_op_desc& d, const PreparedOp& p, int64_t batch,
                               const int8_t* in, int8_t* out, unsigned* dev_err, int num_sms,
                               cudaStream_t s);

// Path for op `d` given operand alignment (16-byte aligned pointers allow the
// TMA / vector paths).
OpPath choose_path(const pspml_op_desc& d, bool aligned16);

// Device bytes prepare_op needs for `d` on `path`.
size_t prepared_bytes(const pspml_op_desc& d, OpPath path);

// Fills `out` using `mem` (device, prepared_bytes(d, path) bytes, 256-byte
// aligned) for derived tables; kernels on `s`.  Returns a cudaError_t.
cudaError_t prepare_op(const pspml_op_desc& d, OpPath path, const int8_t* filter,
                       const int32_t* bias, const int32_t* mult, const int32_t* shift,
                       uint8_t* mem, PreparedOp* out, cudaStream_t s);

// True when every channel's (multiplier, shift) takes the fast requant form
// (host copies of the arrays).
bool host_all_fast(const int32_t* mult, const int32_t* shift, int32_t n);

// Launches op `d` over `batch` samples.
cudaError_t launch_op(const pspml_op_desc& d, const PreparedOp& p, int64_t batch,
                      const int8_t* in, int8_t* out, unsigned* dev_err, int num_sms,
                      cudaStream_t s);

// ---- individual launchers (gemm_tc.cu, cuda_core.cu)
// pool: a 2x2 / stride-2 max pool after the conv is fused into its
// epilogue and `out` is the pooled tensor (conv_pool_supported).
cudaError_t launch_tc_gemm(const pspml_op_desc& d, const PreparedOp& p, int64_t batch,
                           const int8_t* in, int8_t* out, unsigned* dev_err, int num_sms,
                           cudaStream_t s, bool pool = false);
cudaError_t launch_small_conv(const pspml_op_desc& d, const PreparedOp& p, int64_t batch,
                              const int8_t* in, int8_t* out, cudaStream_t s, bool pool = false);

// Whether conv `conv` (prepared as `p`) can run with the max pool `pool`
// after it fused into its epilogue: a 2x2 / stride-2 unpadded pool over the
// whole conv output, a pool clamp no narrower than the conv's, and a conv
// path with a pooled epilogue (tensor-core implicit GEMM with a constant
// table and N % 16 == 0, or the small-channel conv with 4 | N).
bool conv_pool_supported(const pspml_op_desc& conv, const PreparedOp& p,
                         const pspml_op_desc& pool);
// Launches the conv with the pool fused; `out` is the pool's output.
cudaError_t launch_conv_pool(const pspml_op_desc& d, const PreparedOp& p, int64_t batch,
                             const int8_t* in, int8_t* out, unsigned* dev_err, int num_sms,
                             cudaStream_t s);
cudaError_t launch_conv_direct(const pspml_op_desc& d, const PreparedOp& p, int64_t batch,
                               const int8_t* in, int8_t* out, cudaStream_t s);
cudaError_t launch_fc_warp(const pspml_op_desc& d, const PreparedOp& p, int64_t batch,
                           const int8_t* in, int8_t* out, cudaStream_t s);
// FC over at most kGemvMaxBatch samples on a kTc2d-prepared op (folded bias
// and requant tables), K % 16 == 0, 16-byte aligned input and filter: a
// weight-streaming GEMV on the CUDA cores (the tensor-core tiles would hold
// one valid row of 128).
constexpr int64_t kGemvMaxBatch = 4;
cudaError_t launch_fc_gemv(const pspml_op_desc& d, const PreparedOp& p, int64_t batch,
                           const int8_t* in, int8_t* out, int num_sms, cudaStream_t s);
cudaError_t launch_dw3x3(const pspml_op_desc& d, const PreparedOp& p, int64_t batch,
                         const int8_t* in, int8_t* out, cudaStream_t s);
cudaError_t launch_dw_generic(const pspml_op_desc& d, const PreparedOp& p, int64_t batch,
                              const int8_t* in, int8_t* out, cudaStream_t s);
cudaError_t launch_maxpool(const pspml_op_desc& d, int64_t batch, const int8_t* in,
                           int8_t* out, cudaStream_t s);
cudaError_t launch_avgpool(const pspml_op_desc& d, int64_t batch, const int8_t* in,
                           int8_t* out, cudaStream_t s);

// ---- f32 kernels of the reference's own MNIST path (f32.cu)
cudaError_t launch_conv2d_f32(const pspml_op_desc& d, int64_t batch, const float* in,
                              const float* filter, const float* bias, float* out,
                              cudaStream_t s);
cudaError_t launch_max_pool2d_f32(const pspml_op_desc& d, int64_t batch, const float* in,
                                  float* out, cudaStream_t s);
cudaError_t launch_fully_connected_f32(const pspml_op_desc& d, int64_t batch, const float* in,
                                       const float* w, const float* bias, float* out,
                                       cudaStream_t s);

// ---- preparation kernels (prep.cu)
cudaError_t launch_fold_bias(const pspml_op_desc& d, const int8_t* filter, const int32_t* bias,
                             const BorderClasses& bc, int32_t* bias_eff, cudaStream_t s);
cudaError_t launch_build_rq(const int32_t* mult, const int32_t* shift, int32_t zp_out, int32_t n,
                            RqChannel* rq, int32_t* all_fast, cudaStream_t s);
cudaError_t launch_pack_patch_weights(const int8_t* filter, int32_t n, int32_t k, int32_t nw,
                                      uint32_t* out, cudaStream_t s);

// Encodes a tiled TMA descriptor through the driver entry point.
CUresult encode_tensor_map(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                           const uint64_t* strides_bytes, const uint32_t* box,
                           const uint32_t* elem_strides, CUtensorMapSwizzle swizzle);

inline size_t align256(size_t v) { return (v + 255) / 256 * 256; }

}  // namespace pspml
