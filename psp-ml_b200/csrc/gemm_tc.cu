// gemm_tc.cu - int8 GEMM / implicit-GEMM conv on the 5th-generation tensor
// cores (tcgen05.mma kind::i8, int32 accumulators in tensor memory), with
// TFLite per-channel requantisation fused into the epilogue.
//
// Replaces the reference's im2col_padded -> matmul_bt_tiled -> bias_add ->
// relu chain (psp-ml/src/kernels/mod.rs:215-479) and its FC loop
// (psp-ml/src/kernels/naive.rs:147-184) for int8 tensors.
//
// Operands (both K-major, int8):
//   A  activations.  2D: [rows][K] (FC rows = samples, 1x1 conv rows = pixels)
//                    4D: the NHWC input itself; for filter tap (ky,kx) the
//                    A tile of 128 output pixels is one TMA box at the
//                    shifted position.  Out-of-image taps are zero-filled
//                    by TMA; the folded bias of the pixel's border class
//                    corrects for the input zero point there.
//   B  weights [N][taps*Kc] exactly as TFLite stores them ([Co][KH][KW][Ci]).
//
// Persistent kernel, one CTA per SM:
//   warp 0           TMA producer (one thread), STAGES-deep smem ring
//   warp 1           tensor-memory allocator + MMA issuer (one thread)
//   warps 2..2+4G-1  G epilogue groups of 4 warps (one per tensor-memory
//                    lane quarter).  The groups take the CTA's tiles in
//                    turn; NB accumulator buffers in tensor memory let the
//                    MMAs run ahead of the epilogues.
// The epilogue is the critical path for the small-K layers of these
// networks (K = 32..512), so it gets up to 16 warps.  Tiles of 256 rows (two
// M = 128 MMAs per k step) halve the per-tile handoffs for narrow outputs.
#include "gemm_tc.cuh"

namespace pspml {

namespace tcg {

// Instantiated in gemm_tc_bk{32,64,128}.cu.
extern template cudaError_t run_tc_bn<32>(int, int, const CUtensorMap&, const CUtensorMap&,
                                          const TcGemmArgs&, const EpiTable*, int, cudaStream_t);
extern template cudaError_t run_tc_bn<64>(int, int, const CUtensorMap&, const CUtensorMap&,
                                          const TcGemmArgs&, const EpiTable*, int, cudaStream_t);
extern template cudaError_t run_tc_bn<128>(int, int, const CUtensorMap&, const CUtensorMap&,
                                           const TcGemmArgs&, const EpiTable*, int, cudaStream_t);

cudaError_t launch_tc_gemm_once(const pspml_op_desc& d, const PreparedOp& pp, int64_t batch,
                                const int8_t* in, int8_t* out, unsigned* dev_err, int num_sms,
                                cudaStream_t s, bool pool) {
  const int N = d.out_c;
  const bool is_fc = d.kind == PSPML_OP_FULLY_CONNECTED;
  const int Kc = is_fc ? d.in_h * d.in_w * d.in_c : d.in_c;
  const int taps = is_fc ? 1 : d.kernel_h * d.kernel_w;
  // With a constant table, N = 257..512 runs as up to four 128-column tiles
  // (each CTA on one): an epilogue warp then reads 2 KB of the table per
  // tile, which stays in the constant cache, and B stays resident.  (Two
  // 256-column tiles measured slower at N = 512: b6/b7 pointwise 17.8/22.8
  // against 18.8/37.9 ms per config-4 step.  For N <= 256 one 256-column
  // tile is faster: splitting it makes every CTA pair read A twice.)
  const bool tab = pp.all_fast_known && pp.table != nullptr;
  int bn = N <= 32 ? 32 : N <= 64 ? 64 : (N <= 128 || (tab && N > 256 && N <= 512)) ? 128 : 256;
  // A 2D GEMM with few row tiles (an FC over a small batch) would leave
  // most SMs idle with wide N tiles: narrow them until the grid covers the
  // SMs (each CTA then streams a narrower slice of the weights).
  bool narrowed = false;
  if (pp.path == OpPath::kTc2d) {
    const int64_t rows2d = is_fc ? batch : batch * d.out_h * d.out_w;
    const int64_t tiles_m = (rows2d + kBM - 1) / kBM;
    while (bn > 32 && tiles_m * ((N + bn - 1) / bn) < num_sms) {
      bn /= 2;
      narrowed = true;
    }
  }
  const int bk = Kc >= 128 ? 128 : (Kc > 32 ? 64 : 32);

  TcGemmArgs a{};
  a.tiles_n = (N + bn - 1) / bn;
  a.kblocks = (Kc + bk - 1) / bk;
  a.taps = taps;
  a.kw = is_fc ? 1 : d.kernel_w;
  a.pad_t = is_fc ? 0 : d.pad_top;
  a.pad_l = is_fc ? 0 : d.pad_left;
  a.N = N;
  a.Kc = Kc;
  a.out = out;
  a.bias = pp.bias_eff;
  a.ycls = pp.ncls > 1 ? pp.ycls : nullptr;
  a.xcls = pp.ncls > 1 ? pp.xcls : nullptr;
  a.n_xcls = pp.n_xcls;
  a.rq = pp.rq;
  a.all_fast = pp.rq_all_fast;
  a.ncls = pp.ncls;
  a.base_cls = pp.base_cls;
  a.param_smem = static_cast<int32_t>(param_smem_bytes(N, pp.ncls));
  a.lo4 = splat4(d.act_min);
  a.hi4 = splat4(d.act_max);
  a.clamp = (d.act_min > -128 || d.act_max < 127) ? 1 : 0;
  a.ep = ep_flags(d.act_min, d.act_max, d.zp_out);
  a.err = dev_err;

  int mt = 1;
  const CUtensorMapSwizzle swz = bk == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                 : bk == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                            : CU_TENSOR_MAP_SWIZZLE_32B;
  CUtensorMap ma, mb;
  const uint32_t estr[4] = {1, 1, 1, 1};
  if (pool && (pp.path != OpPath::kTc4d || !pp.all_fast_known || pp.table == nullptr ||
               N % 16 != 0 || d.out_h % 2 != 0 || d.out_w % 2 != 0))
    return cudaErrorInvalidValue;
  a.pool = pool ? 1 : 0;
  a.Hp = d.out_h / 2;
  a.Wp = d.out_w / 2;
  if (pp.path == OpPath::kTc4d) {
    // A pooled epilogue needs a window's pixels in one warp: tiles of at
    // most 16 pixels per row.
    const int bw = std::min(pow2_ceil(d.out_w), pool ? 16 : 128);
    const int bh = std::min(pow2_ceil(d.out_h), 128 / bw);
    const int bi = 128 / (bw * bh);
    a.conv4d = 1;
    a.bw_log2 = ilog2_exact(bw);
    a.bh_log2 = ilog2_exact(bh);
    a.bi = bi;
    a.tiles_x = (d.out_w + bw - 1) / bw;
    a.tiles_y = (d.out_h + bh - 1) / bh;
    a.Wo = d.out_w;
    a.Ho = d.out_h;
    a.nimg = batch;
    const int64_t tiles_img = (batch + bi - 1) / bi;
    const int64_t tiles_m = tiles_img * a.tiles_x * a.tiles_y;
    a.tiles_total = tiles_m * a.tiles_n;
    a.fd_per_img = FastDiv(static_cast<uint32_t>(a.tiles_x * a.tiles_y));
    a.fd_tiles_x = FastDiv(static_cast<uint32_t>(a.tiles_x));
    const uint64_t dims[4] = {static_cast<uint64_t>(d.in_c), static_cast<uint64_t>(d.in_w),
                              static_cast<uint64_t>(d.in_h), static_cast<uint64_t>(batch)};
    const uint64_t strides[3] = {static_cast<uint64_t>(d.in_c),
                                 static_cast<uint64_t>(d.in_w) * d.in_c,
                                 static_cast<uint64_t>(d.in_h) * d.in_w * d.in_c};
    const uint32_t box[4] = {static_cast<uint32_t>(bk), static_cast<uint32_t>(bw),
                             static_cast<uint32_t>(bh), static_cast<uint32_t>(bi)};
    if (encode_tensor_map(&ma, in, 4, dims, strides, box, estr, swz) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  } else {
    const int64_t rows = is_fc ? batch : batch * d.out_h * d.out_w;
    if (rows >= (1ll << 31) - 2 * kBM) return cudaErrorInvalidValue;
    mt = bn <= 64 && !narrowed && rows > kBM && pp.all_fast_known && pp.table != nullptr ? 2 : 1;
    a.conv4d = 0;
    a.rows = rows;
    a.ldo = N;
    a.tiles_total = ((rows + kBM * mt - 1) / (kBM * mt)) * a.tiles_n;
    const uint64_t dims[2] = {static_cast<uint64_t>(Kc), static_cast<uint64_t>(rows)};
    const uint64_t strides[1] = {static_cast<uint64_t>(Kc)};
    const uint32_t box[2] = {static_cast<uint32_t>(bk), static_cast<uint32_t>(kBM * mt)};
    if (encode_tensor_map(&ma, in, 2, dims, strides, box, estr, swz) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(taps) * Kc, static_cast<uint64_t>(N)};
    const uint64_t strides[1] = {static_cast<uint64_t>(taps) * Kc};
    const uint32_t box[2] = {static_cast<uint32_t>(bk), static_cast<uint32_t>(bn)};
    if (encode_tensor_map(&mb, pp.filter, 2, dims, strides, box, estr, swz) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  if (a.tiles_total >= (1ll << 31)) return cudaErrorInvalidValue;
  a.fd_tiles_n = FastDiv(static_cast<uint32_t>(a.tiles_n));
  const EpiTable* table = pp.all_fast_known ? pp.table : nullptr;
  switch (bk) {
    case 128: return run_tc_bn<128>(bn, mt, ma, mb, a, table, num_sms, s);
    case 64: return run_tc_bn<64>(bn, mt, ma, mb, a, table, num_sms, s);
    default: return run_tc_bn<32>(bn, mt, ma, mb, a, table, num_sms, s);
  }
}

}  // namespace tcg

using tcg::launch_tc_gemm_once;

// Tile indices are 32-bit in the kernel: batches with 2^31 or more tiles
// (or A rows) run as several launches over batch slices.
cudaError_t launch_tc_gemm(const pspml_op_desc& d, const PreparedOp& pp, int64_t batch,
                           const int8_t* in, int8_t* out, unsigned* dev_err, int num_sms,
                           cudaStream_t s, bool pool) {
  const bool is_fc = d.kind == PSPML_OP_FULLY_CONNECTED;
  const int64_t rows_per = is_fc ? 1 : static_cast<int64_t>(d.out_h) * d.out_w;
  // Rows bound the 2D tile count; a 4D tile holds at least one output row
  // segment, so rows also bound the 4D count.  (2^31 - 2^12) / 32 N tiles.
  const int64_t max_rows = ((1ll << 31) - 4096) / std::max(1, (d.out_c + 31) / 32);
  const int64_t chunk = std::max<int64_t>(1, max_rows / rows_per);
  const int64_t in_per = static_cast<int64_t>(d.in_h) * d.in_w * d.in_c;
  const int64_t out_per = pool ? static_cast<int64_t>(d.out_h / 2) * (d.out_w / 2) * d.out_c
                              : static_cast<int64_t>(d.out_h) * d.out_w * d.out_c;
  for (int64_t b0 = 0; b0 < batch; b0 += chunk) {
    const cudaError_t e =
        launch_tc_gemm_once(d, pp, std::min(chunk, batch - b0), in + b0 * in_per,
                            out + b0 * out_per, dev_err, num_sms, s, pool);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace pspml
