// prep.cu - per-op preparation (done once per model op, or per call for the
// stateless per-op C-ABI entry points) and the launch dispatcher.
//
// Preparation folds the input zero point into the bias, builds the
// per-channel requantisation constants and repacks small-conv weights:
//   bias_eff[cls][n] = bias[n] - zp_in * sum(w[n][tap][ci]) over the taps
//                      that lie inside the image for border class cls
// so that kernels can accumulate sum(x * w) directly (out-of-image taps
// filled with 0 by TMA, or with zp_in by the CUDA-core kernels, are then
// exact), as TFLite's sum((x - zp_in) * w) + bias.
#include <algorithm>

#include "kernels.h"

namespace pspml {

namespace {

constexpr int kMaxSmallConvWords = 32;  // patch words (K <= 128) for kSmallConv

struct FoldArgs {
  int32_t N, taps, kw, Kc;
  int32_t n_ycls, n_xcls;
  int32_t zp_in;
  uint32_t ymask[64];
  uint32_t xmask[64];
};

// One warp per output channel: per-tap weight sums, then one folded bias per
// border class.  Filter [N][taps][Kc].
__global__ void k_fold_bias(const int8_t* __restrict__ filter, const int32_t* __restrict__ bias,
                            int32_t* __restrict__ bias_eff, const FoldArgs a) {
  __shared__ int32_t wsum_s[8][64];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x * 8 + w;
  if (n >= a.N) return;
  int32_t* wsum = wsum_s[w];
  const int8_t* fr = filter + static_cast<int64_t>(n) * a.taps * a.Kc;
  for (int tap = 0; tap < a.taps; ++tap) {
    int32_t s = 0;
    for (int c = lane; c < a.Kc; c += 32) s += fr[static_cast<int64_t>(tap) * a.Kc + c];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
    if (lane == 0) wsum[tap] = s;
  }
  __syncwarp();
  const int32_t b = bias != nullptr ? bias[n] : 0;
  const int ncls = a.n_ycls * a.n_xcls;
  for (int cls = lane; cls < ncls; cls += 32) {
    const uint32_t ym = a.ymask[cls / a.n_xcls];
    const uint32_t xm = a.xmask[cls % a.n_xcls];
    int32_t s = 0;
    for (int tap = 0; tap < a.taps; ++tap) {
      const int ky = tap / a.kw, kx = tap - (tap / a.kw) * a.kw;
      if (((ym >> ky) & 1u) && ((xm >> kx) & 1u)) s += wsum[tap];
    }
    bias_eff[static_cast<int64_t>(cls) * a.N + n] = static_cast<int32_t>(
        static_cast<uint32_t>(b) - static_cast<uint32_t>(a.zp_in) * static_cast<uint32_t>(s));
  }
}

// Depthwise filter [taps][C]: bias_eff[c] = bias[c] - zp_in * sum_t w[t][c].
__global__ void k_fold_dw(const int8_t* __restrict__ filter, const int32_t* __restrict__ bias,
                          int32_t* __restrict__ bias_eff, int32_t C, int32_t taps,
                          int32_t zp_in) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  int32_t s = 0;
  for (int t = 0; t < taps; ++t) s += filter[static_cast<int64_t>(t) * C + c];
  const int32_t b = bias != nullptr ? bias[c] : 0;
  bias_eff[c] = static_cast<int32_t>(static_cast<uint32_t>(b) -
                                     static_cast<uint32_t>(zp_in) * static_cast<uint32_t>(s));
}

__global__ void k_build_rq(const int32_t* __restrict__ mult, const int32_t* __restrict__ shift,
                           int32_t zp_out, int32_t n, RqChannel* __restrict__ rq,
                           int32_t* __restrict__ all_fast) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const RqChannel q = make_rq(mult[i], shift[i], zp_out);
    rq[i] = q;
    if (q.sr < 0) atomicAnd(all_fast, 0);
  }
}

// [N][K] int8 -> [N][nw] words, zero padded past K.
__global__ void k_pack_patch_weights(const int8_t* __restrict__ f, int32_t n, int32_t k,
                                     int32_t nw, uint32_t* __restrict__ out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(n) * nw) return;
  const int64_t row = i / nw;
  const int word = static_cast<int>(i - row * nw);
  uint32_t v = 0;
  for (int j = 0; j < 4; ++j) {
    const int kk = word * 4 + j;
    if (kk < k) v |= (static_cast<uint32_t>(static_cast<uint8_t>(f[row * k + kk]))) << (8 * j);
  }
  out[i] = v;
}

bool is_1x1_same(const pspml_op_desc& d) {
  return d.kernel_h == 1 && d.kernel_w == 1 && d.stride_h == 1 && d.stride_w == 1 &&
         d.pad_top == 0 && d.pad_left == 0 && d.out_h == d.in_h && d.out_w == d.in_w;
}

int small_conv_words(const pspml_op_desc& d) {
  const int k = d.kernel_h * d.kernel_w * d.in_c;
  return ((k + 3) / 4 + 3) / 4 * 4;  // words, padded to a multiple of 4 (16-byte rows)
}

struct Carve {
  uint8_t* base;
  size_t off = 0;
  template <class T>
  T* take(size_t bytes) {
    T* p = reinterpret_cast<T*>(base ? base + off : nullptr);
    off += align256(bytes);
    return p;
  }
};

}  // namespace

bool build_border_classes(const pspml_op_desc& d, BorderClasses* bc) {
  const int kh = d.kernel_h, kw = d.kernel_w;
  if (d.out_h > 4096 || d.out_w > 4096 || kh > 32 || kw > 32) return false;
  auto classify = [](int out, int in, int k, int stride, int pad, uint32_t* masks, int* nmask,
                     uint8_t* cls) {
    *nmask = 0;
    for (int o = 0; o < out; ++o) {
      uint32_t m = 0;
      for (int t = 0; t < k; ++t) {
        const int i = o * stride + t - pad;
        if (i >= 0 && i < in) m |= 1u << t;
      }
      int found = -1;
      for (int j = 0; j < *nmask; ++j)
        if (masks[j] == m) found = j;
      if (found < 0) {
        if (*nmask >= 64) return false;
        masks[*nmask] = m;
        found = (*nmask)++;
      }
      cls[o] = static_cast<uint8_t>(found);
    }
    return true;
  };
  if (!classify(d.out_h, d.in_h, kh, d.stride_h, d.pad_top, bc->ymask, &bc->n_ycls, bc->ycls))
    return false;
  if (!classify(d.out_w, d.in_w, kw, d.stride_w, d.pad_left, bc->xmask, &bc->n_xcls, bc->xcls))
    return false;
  return true;
}

OpPath choose_path(const pspml_op_desc& d, bool aligned16) {
  switch (d.kind) {
    case PSPML_OP_CONV2D: {
      if (aligned16 && d.in_c % 16 == 0) {
        if (is_1x1_same(d)) return OpPath::kTc2d;
        if (d.stride_h == 1 && d.stride_w == 1 && d.kernel_h * d.kernel_w <= 64 &&
            d.kernel_h <= 32 && d.kernel_w <= 32 && d.out_w <= 4096 && d.out_h <= 4096)
          return OpPath::kTc4d;
      }
      if (aligned16 && small_conv_supported(d) && small_conv_words(d) <= kMaxSmallConvWords)
        return OpPath::kSmallConv;
      return OpPath::kDirect;
    }
    case PSPML_OP_DEPTHWISE_CONV2D:
      if (aligned16 && (dw_tc_supported(d) || dwrs_dw_supported(d))) return OpPath::kDwTc;
      if (d.in_c % 4 == 0 && d.kernel_h == 3 && d.kernel_w == 3 &&
          (d.stride_h == 1 || d.stride_h == 2) && d.stride_w == d.stride_h && aligned16)
        return OpPath::kDw3x3;
      return OpPath::kDwGeneric;
    case PSPML_OP_FULLY_CONNECTED: {
      const int64_t k = static_cast<int64_t>(d.in_h) * d.in_w * d.in_c;
      return (aligned16 && k % 16 == 0) ? OpPath::kTc2d : OpPath::kFcWarp;
    }
    case PSPML_OP_MAX_POOL2D:
      return OpPath::kMaxPool;
    case PSPML_OP_AVERAGE_POOL2D:
      return OpPath::kAvgPool;
    default:
      return OpPath::kReshape;
  }
}

size_t prepared_bytes(const pspml_op_desc& d, OpPath path) {
  const size_t n = static_cast<size_t>(d.out_c);
  Carve c{nullptr};
  switch (path) {
    case OpPath::kTc2d:
      c.take<int32_t>(n * 4);
      c.take<RqChannel>((n + 1) * sizeof(RqChannel));
      break;
    case OpPath::kTc4d: {
      BorderClasses bc;
      if (!build_border_classes(d, &bc)) return 0;
      c.take<int32_t>(static_cast<size_t>(bc.n_ycls) * bc.n_xcls * n * 4);
      c.take<RqChannel>((n + 1) * sizeof(RqChannel));
      c.take<uint8_t>(d.out_h);
      c.take<uint8_t>(d.out_w);
      break;
    }
    case OpPath::kSmallConv:
      c.take<int32_t>(n * 4);
      c.take<RqChannel>((n + 1) * sizeof(RqChannel));
      c.take<uint32_t>(n * small_conv_words(d) * 4);
      break;
    case OpPath::kDw3x3:
      c.take<int32_t>(n * 4);
      c.take<RqChannel>((n + 1) * sizeof(RqChannel));
      break;
    case OpPath::kDwTc: {
      BorderClasses bc;
      if (!build_border_classes(d, &bc)) return 0;
      c.take<int32_t>(static_cast<size_t>(bc.n_ycls) * bc.n_xcls * n * 4);
      c.take<RqChannel>((n + 1) * sizeof(RqChannel));
      c.take<uint8_t>(d.out_h);
      c.take<uint8_t>(d.out_w);
      c.take<uint8_t>(n / 32 * 9216);
      c.take<uint32_t>(128 * 4);
      break;
    }
    case OpPath::kDirect:
    case OpPath::kFcWarp:
    case OpPath::kDwGeneric:
      c.take<RqChannel>((n + 1) * sizeof(RqChannel));
      break;
    default:
      break;
  }
  return c.off;
}

cudaError_t prepare_op(const pspml_op_desc& d, OpPath path, const int8_t* filter,
                       const int32_t* bias, const int32_t* mult, const int32_t* shift,
                       uint8_t* mem, PreparedOp* out, cudaStream_t s) {
  PreparedOp p;
  p.path = path;
  p.filter = filter;
  p.bias = bias;
  p.mult = mult;
  p.shift = shift;
  const int32_t n = d.out_c;
  Carve c{mem};
  cudaError_t e = cudaSuccess;
  BorderClasses* bc = nullptr;
  static thread_local BorderClasses bc_store;
  auto rq_and = [&]() {
    p.rq = c.take<RqChannel>((static_cast<size_t>(n) + 1) * sizeof(RqChannel));
    p.rq_all_fast = reinterpret_cast<int32_t*>(p.rq + n);
    return launch_build_rq(mult, shift, d.zp_out, n, p.rq, p.rq_all_fast, s);
  };
  switch (path) {
    case OpPath::kTc2d:
    case OpPath::kSmallConv: {
      bc_store.n_ycls = bc_store.n_xcls = 1;
      bc_store.ymask[0] = bc_store.xmask[0] = 0xFFFFFFFFu;
      bc = &bc_store;
      p.bias_eff = c.take<int32_t>(static_cast<size_t>(n) * 4);
      if ((e = rq_and()) != cudaSuccess) break;
      if (path == OpPath::kSmallConv) {
        p.nw = small_conv_words(d);
        uint32_t* wp = c.take<uint32_t>(static_cast<size_t>(n) * p.nw * 4);
        p.wpack = wp;
        e = launch_pack_patch_weights(filter, n, d.kernel_h * d.kernel_w * d.in_c, p.nw, wp, s);
        if (e != cudaSuccess) break;
      }
      e = launch_fold_bias(d, filter, bias, *bc, p.bias_eff, s);
      break;
    }
    case OpPath::kTc4d: {
      if (!build_border_classes(d, &bc_store)) return cudaErrorInvalidValue;
      bc = &bc_store;
      p.ncls = bc->n_ycls * bc->n_xcls;
      p.n_xcls = bc->n_xcls;
      p.base_cls = bc->ycls[d.out_h / 2] * bc->n_xcls + bc->xcls[d.out_w / 2];
      p.bias_eff = c.take<int32_t>(static_cast<size_t>(p.ncls) * n * 4);
      if ((e = rq_and()) != cudaSuccess) break;
      p.ycls = c.take<uint8_t>(d.out_h);
      p.xcls = c.take<uint8_t>(d.out_w);
      if (p.ncls > 1) {
        if ((e = cudaMemcpyAsync(p.ycls, bc->ycls, d.out_h, cudaMemcpyHostToDevice, s)) !=
            cudaSuccess)
          break;
        if ((e = cudaMemcpyAsync(p.xcls, bc->xcls, d.out_w, cudaMemcpyHostToDevice, s)) !=
            cudaSuccess)
          break;
      }
      e = launch_fold_bias(d, filter, bias, *bc, p.bias_eff, s);
      break;
    }
    case OpPath::kDwTc: {
      if (!build_border_classes(d, &bc_store)) return cudaErrorInvalidValue;
      bc = &bc_store;
      p.ncls = bc->n_ycls * bc->n_xcls;
      p.n_xcls = bc->n_xcls;
      p.base_cls = bc->ycls[d.out_h / 2] * bc->n_xcls + bc->xcls[d.out_w / 2];
      p.bias_eff = c.take<int32_t>(static_cast<size_t>(p.ncls) * n * 4);
      if ((e = rq_and()) != cudaSuccess) break;
      p.ycls = c.take<uint8_t>(d.out_h);
      p.xcls = c.take<uint8_t>(d.out_w);
      if ((e = cudaMemcpyAsync(p.ycls, bc->ycls, d.out_h, cudaMemcpyHostToDevice, s)) !=
          cudaSuccess)
        break;
      if ((e = cudaMemcpyAsync(p.xcls, bc->xcls, d.out_w, cudaMemcpyHostToDevice, s)) !=
          cudaSuccess)
        break;
      uint8_t* wp = c.take<uint8_t>(static_cast<size_t>(n) / 32 * 9216);
      p.wpack = reinterpret_cast<const uint32_t*>(wp);
      uint32_t* masks = c.take<uint32_t>(128 * 4);
      e = prepare_dw_tc(d, filter, bias, *bc, wp, p.bias_eff, masks, s);
      break;
    }
    case OpPath::kDw3x3: {
      p.bias_eff = c.take<int32_t>(static_cast<size_t>(n) * 4);
      if ((e = rq_and()) != cudaSuccess) break;
      k_fold_dw<<<(n + 127) / 128, 128, 0, s>>>(filter, bias, p.bias_eff, n,
                                                d.kernel_h * d.kernel_w, d.zp_in);
      e = cudaGetLastError();
      break;
    }
    case OpPath::kDirect:
    case OpPath::kFcWarp:
    case OpPath::kDwGeneric:
      e = rq_and();
      break;
    default:
      break;
  }
  *out = p;
  return e;
}

bool host_all_fast(const int32_t* mult, const int32_t* shift, int32_t n) {
  for (int32_t i = 0; i < n; ++i)
    if (make_rq(mult[i], shift[i], 0).sr < 0) return false;
  return true;
}

bool conv_pool_supported(const pspml_op_desc& conv, const PreparedOp& p,
                         const pspml_op_desc& pool) {
  if (conv.kind != PSPML_OP_CONV2D || pool.kind != PSPML_OP_MAX_POOL2D) return false;
  if (pool.kernel_h != 2 || pool.kernel_w != 2 || pool.stride_h != 2 || pool.stride_w != 2 ||
      pool.pad_top != 0 || pool.pad_left != 0 || pool.pad_bottom != 0 || pool.pad_right != 0)
    return false;
  if (pool.in_h != conv.out_h || pool.in_w != conv.out_w || pool.in_c != conv.out_c ||
      conv.out_h % 2 != 0 || conv.out_w % 2 != 0)
    return false;
  // The pool clamps to its own activation range; a range no narrower than
  // the conv's makes that clamp a no-op on the conv's outputs.
  if (pool.act_min > conv.act_min || pool.act_max < conv.act_max) return false;
  if (p.path == OpPath::kTc4d)
    return p.all_fast_known && p.table != nullptr && conv.out_c % 16 == 0;
  if (p.path == OpPath::kSmallConv) return conv.out_c % 4 == 0 && small_conv_supported(conv);
  return false;
}

cudaError_t launch_conv_pool(const pspml_op_desc& d, const PreparedOp& p, int64_t batch,
                             const int8_t* in, int8_t* out, unsigned* dev_err, int num_sms,
                             cudaStream_t s) {
  if (batch <= 0) return cudaSuccess;
  if (p.path == OpPath::kTc4d)
    return launch_tc_gemm(d, p, batch, in, out, dev_err, num_sms, s, true);
  if (p.path == OpPath::kSmallConv) return launch_small_conv(d, p, batch, in, out, s, true);
  return cudaErrorInvalidValue;
}

cudaError_t launch_op(const pspml_op_desc& d, const PreparedOp& p, int64_t batch,
                      const int8_t* in, int8_t* out, unsigned* dev_err, int num_sms,
                      cudaStream_t s) {
  if (batch <= 0) return cudaSuccess;
  switch (p.path) {
    case OpPath::kTc2d:
      if (d.kind == PSPML_OP_FULLY_CONNECTED && batch <= kGemvMaxBatch &&
          (reinterpret_cast<uintptr_t>(in) & 15u) == 0)
        return launch_fc_gemv(d, p, batch, in, out, num_sms, s);
      return launch_tc_gemm(d, p, batch, in, out, dev_err, num_sms, s);
    case OpPath::kTc4d:
      return launch_tc_gemm(d, p, batch, in, out, dev_err, num_sms, s);
    case OpPath::kSmallConv:
      if (im2col_conv_supported(d, p, in, out))
        return launch_im2col_conv(d, p, batch, in, out, dev_err, num_sms, s);
      return launch_small_conv(d, p, batch, in, out, s);
    case OpPath::kDirect:
      return launch_conv_direct(d, p, batch, in, out, s);
    case OpPath::kFcWarp:
      return launch_fc_warp(d, p, batch, in, out, s);
    case OpPath::kDwTc:
      return launch_dw_tc(d, p, batch, in, out, dev_err, num_sms, s);
    case OpPath::kDw3x3:
      return launch_dw3x3(d, p, batch, in, out, s);
    case OpPath::kDwGeneric:
      return launch_dw_generic(d, p, batch, in, out, s);
    case OpPath::kMaxPool:
      return launch_maxpool(d, batch, in, out, s);
    case OpPath::kAvgPool:
      return launch_avgpool(d, batch, in, out, s);
    case OpPath::kReshape: {
      const size_t bytes = static_cast<size_t>(batch) * d.out_h * d.out_w * d.out_c;
      if (out == in) return cudaSuccess;
      return cudaMemcpyAsync(out, in, bytes, cudaMemcpyDeviceToDevice, s);
    }
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_fold_bias(const pspml_op_desc& d, const int8_t* filter, const int32_t* bias,
                             const BorderClasses& bc, int32_t* bias_eff, cudaStream_t s) {
  FoldArgs a{};
  a.N = d.out_c;
  if (d.kind == PSPML_OP_FULLY_CONNECTED) {
    a.taps = 1;
    a.kw = 1;
    a.Kc = d.in_h * d.in_w * d.in_c;
  } else {
    a.taps = d.kernel_h * d.kernel_w;
    a.kw = d.kernel_w;
    a.Kc = d.in_c;
  }
  a.n_ycls = bc.n_ycls;
  a.n_xcls = bc.n_xcls;
  for (int i = 0; i < 64; ++i) {
    a.ymask[i] = bc.ymask[i];
    a.xmask[i] = bc.xmask[i];
  }
  if (a.taps > 64) return cudaErrorInvalidValue;
  a.zp_in = d.zp_in;
  k_fold_bias<<<(a.N + 7) / 8, 256, 0, s>>>(filter, bias, bias_eff, a);
  return cudaGetLastError();
}

cudaError_t launch_build_rq(const int32_t* mult, const int32_t* shift, int32_t zp_out, int32_t n,
                            RqChannel* rq, int32_t* all_fast, cudaStream_t s) {
  cudaError_t e = cudaMemsetAsync(all_fast, 0xFF, sizeof(int32_t), s);
  if (e != cudaSuccess) return e;
  k_build_rq<<<(n + 127) / 128, 128, 0, s>>>(mult, shift, zp_out, n, rq, all_fast);
  return cudaGetLastError();
}

cudaError_t launch_pack_patch_weights(const int8_t* filter, int32_t n, int32_t k, int32_t nw,
                                      uint32_t* out, cudaStream_t s) {
  const int64_t total = static_cast<int64_t>(n) * nw;
  k_pack_patch_weights<<<static_cast<unsigned>((total + 255) / 256), 256, 0, s>>>(filter, n, k,
                                                                                 nw, out);
  return cudaGetLastError();
}

}  // namespace pspml
