// gemm_tc.cuh - the tcgen05 int8 GEMM kernel and its launch templates,
// shared by gemm_tc.cu (operand set-up and dispatch) and the gemm_tc_bk*.cu
// files, each of which instantiates the kernels of one K-block width (the
// instantiations compile in parallel).
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
#pragma once

#include <algorithm>
#include <atomic>

#include "kernels.h"
#include "ptx.cuh"
#include "requant.cuh"

namespace pspml {

namespace tcg {

constexpr int kBM = 128;
constexpr int kMaxStages = 8;
constexpr int kSmemLimit = 232448;  // 227 KB opt-in per block

struct TcGemmArgs {
  int64_t tiles_total;
  int32_t tiles_n;
  int32_t kblocks;     // channel blocks per tap
  int32_t taps, kw;    // filter taps, filter width
  int32_t pad_t, pad_l;
  int32_t conv4d;
  int32_t bw_log2, bh_log2, bi;
  int32_t tiles_x, tiles_y;
  int64_t rows;        // 2D: number of A rows
  int32_t N;
  int32_t Wo, Ho;
  int64_t nimg;
  int32_t Kc;          // channels per tap (column stride of a tap in B)
  int8_t* out;
  int64_t ldo;
  const int32_t* bias;  // [ncls][N] folded bias
  const uint8_t* ycls;
  const uint8_t* xcls;
  int32_t n_xcls;
  const RqChannel* rq;
  const int32_t* all_fast;  // -1: every channel has a fast-form requant entry
  int32_t ncls;             // rows of the folded-bias table
  int32_t base_cls;         // border class whose bias the constant table holds
  FastDiv fd_tiles_n, fd_per_img, fd_tiles_x;  // tile index -> (n tile, m tile), origin
  int32_t param_smem;       // bytes of requant + bias tables staged in smem (0: read global)
  uint32_t lo4, hi4;    // activation clamp, bytes replicated
  int32_t clamp;        // act range narrower than int8
  int32_t ep;           // ep_flags of the op (table epilogues)
  unsigned* err;
  int32_t stages;
  int32_t group;  // k-iterations per pipeline stage (divides taps * kblocks): one
                  // TMA barrier and one MMA commit cover `group` filter taps
  int32_t b_res;  // the CTA's N tile of B stays in smem, loaded once (the grid is a
                  // multiple of tiles_n, so CTA b always works on N tile b % tiles_n)
  // 2x2 / stride-2 max pool fused into the 4D epilogue: `out` is the pooled
  // [nimg][Hp][Wp][N] tensor (Hp = Ho / 2, Wp = Wo / 2).  Tiles are at most
  // 16 pixels wide, so a window's four pixels are lanes l, l ^ 1, l ^ bw,
  // l ^ bw ^ 1 of one epilogue warp.
  int32_t pool;
  int32_t Hp, Wp;
  // kEpiConvStatic: bytes of shared memory holding the border-class bias
  // differences, rows of BN + 1 words (0: no border classes).  Lanes of one
  // warp hold pixels of up to nine classes; read from the constant bank at
  // per-lane offsets those loads serialise, from shared memory the padded
  // rows put each class on its own bank.
  int32_t dbias_smem;
};

// Signed byte-wise max of a 16-byte chunk with the same chunk of lane ^ m.
__device__ __forceinline__ uint4 vmax_xor(const uint4 w, int m) {
  return make_uint4(__vmaxs4(w.x, __shfl_xor_sync(0xFFFFFFFFu, w.x, m)),
                    __vmaxs4(w.y, __shfl_xor_sync(0xFFFFFFFFu, w.y, m)),
                    __vmaxs4(w.z, __shfl_xor_sync(0xFFFFFFFFu, w.z, m)),
                    __vmaxs4(w.w, __shfl_xor_sync(0xFFFFFFFFu, w.w, m)));
}

constexpr int kParamSmemMax = 32 * 1024;

inline size_t param_smem_bytes(int n, int ncls) {
  const size_t b = static_cast<size_t>(n) * sizeof(RqChannel) +
                   (static_cast<size_t>(ncls) * n * 4 + 15) / 16 * 16;
  return b <= static_cast<size_t>(kParamSmemMax) ? b : 0;
}

template <int BK>
struct SwizzleFor;
template <>
struct SwizzleFor<128> {
  static constexpr uint32_t kLayout = 2;  // 128B swizzle
};
template <>
struct SwizzleFor<64> {
  static constexpr uint32_t kLayout = 4;  // 64B swizzle
};
template <>
struct SwizzleFor<32> {
  static constexpr uint32_t kLayout = 6;  // 32B swizzle
};

// Epilogue variants of k_gemm_s8.
enum : int {
  kEpiGeneral = 0,  // tables in smem or global, runtime fast/general requant
  kEpiTable = 1,    // fast requant, tables a kernel parameter, runtime offsets
  kEpiStatic = 2,   // as kEpiTable with every offset a compile-time constant:
                    // 2D A, one N tile (N == BN), 16-byte aligned rows
  kEpiConvStatic = 3  // 4D (implicit-GEMM conv) A with N == BN (one N tile):
                      // compile-time table offsets, border-class bias
                      // differences and the fused max pool as in kEpiTable
};

// Tensor-memory accumulator buffers and epilogue groups per tile width.
// MT accumulators of 128 rows x BN columns per tile (a tile has 128 * MT
// rows: one TMA box, MT MMAs per k step, one handoff).
template <int BN, int MT, int MODE>
struct EpiShape {
  static constexpr int kCols = BN * MT;  // tensor-memory columns per buffer
  static constexpr int kBufs = (512 / kCols) >= 8 ? 8 : (512 / kCols);
  // 256-column tiles of the table epilogues: two groups drain each tile,
  // one 128-column half each, so four groups work over the two buffers
  // (with one group per tile these kernels had half the epilogue warps of
  // the 128-column ones).
  static constexpr int kSplit =
      (BN == 256 && MT == 1 && (MODE == kEpiStatic || MODE == kEpiTable)) ? 2 : 1;
  // Three groups for 256-row tiles: 14 warps leave 128 registers a thread
  // (an SM sub-partition holds at most four of them).
  static constexpr int kGroups = (MT == 2 ? 3 : (kBufs >= 4 ? 4 : kBufs)) * kSplit;
  static constexpr int kThreads = 64 + 128 * kGroups;
  static constexpr uint32_t kTmemCols = kBufs * kCols;
};

__device__ __forceinline__ void record_error(unsigned* err, volatile int* abort_flag,
                                             unsigned code) {
  *abort_flag = 1;
  if (err != nullptr) atomicCAS(err, 0u, code);
}

struct TileOrigin {
  int32_t x0, y0;
  int64_t n0;
};
// Tile indices stay below 2^31 (the host splits larger batches).
__device__ __forceinline__ TileOrigin tile_origin(const TcGemmArgs& p, uint32_t tm) {
  const uint32_t ti = p.fd_per_img.div(tm);
  const int32_t rem = static_cast<int32_t>(tm - ti * p.fd_per_img.d);
  const int32_t ty = static_cast<int32_t>(p.fd_tiles_x.div(static_cast<uint32_t>(rem)));
  const int32_t tx = rem - ty * p.tiles_x;
  TileOrigin o;
  o.x0 = tx << p.bw_log2;
  o.y0 = ty << p.bh_log2;
  o.n0 = static_cast<int64_t>(ti) * p.bi;
  return o;
}

// Requantises 32 accumulators of one output row and stores them.  bias / rq
// point into shared memory when the tables are staged there, else global.
// Sixteen requantised, clamped outputs of channels bias[0..15] / rq[0..15]
// as four packed words.
template <bool FAST>
__device__ __forceinline__ void requant_chunk16(const uint32_t (&v)[16], const int32_t* bias,
                                                const RqChannel* rq, const TcGemmArgs& p,
                                                uint32_t (&packed)[4]) {
  const bool bvec = (reinterpret_cast<uintptr_t>(bias) & 15u) == 0;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    int4 b4;
    if (bvec) {
      b4 = reinterpret_cast<const int4*>(bias)[g];
    } else {
      b4 = make_int4(bias[4 * g], bias[4 * g + 1], bias[4 * g + 2], bias[4 * g + 3]);
    }
    const RqChannel q0 = rq[4 * g], q1 = rq[4 * g + 1], q2 = rq[4 * g + 2], q3 = rq[4 * g + 3];
    const int32_t r0 = rq_sel<FAST>(static_cast<int32_t>(v[4 * g + 0]) + b4.x, q0);
    const int32_t r1 = rq_sel<FAST>(static_cast<int32_t>(v[4 * g + 1]) + b4.y, q1);
    const int32_t r2 = rq_sel<FAST>(static_cast<int32_t>(v[4 * g + 2]) + b4.z, q2);
    const int32_t r3 = rq_sel<FAST>(static_cast<int32_t>(v[4 * g + 3]) + b4.w, q3);
    uint32_t w = pack_sat4(r0, r1, r2, r3);
    if (p.clamp) w = clamp4(w, p.lo4, p.hi4);
    packed[g] = w;
  }
}

template <bool FAST>
__device__ __forceinline__ void epilogue_chunk(const uint32_t (&v)[16], int8_t* dst,
                                               const int32_t* bias, const RqChannel* rq, int cnt,
                                               const TcGemmArgs& p) {
  if (cnt == 16) {
    uint32_t packed[4];
    requant_chunk16<FAST>(v, bias, rq, p, packed);
    if ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
      *reinterpret_cast<uint4*>(dst) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    } else if ((reinterpret_cast<uintptr_t>(dst) & 3u) == 0) {
      uint32_t* d1 = reinterpret_cast<uint32_t*>(dst);
#pragma unroll
      for (int g = 0; g < 4; ++g) d1[g] = packed[g];
    } else {
#pragma unroll
      for (int g = 0; g < 4; ++g)
#pragma unroll
        for (int j = 0; j < 4; ++j) dst[4 * g + j] = static_cast<int8_t>(packed[g] >> (8 * j));
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (j < cnt) {
        int32_t r = rq_sel<FAST>(static_cast<int32_t>(v[j]) + bias[j], rq[j]);
        r = max(r, -128);
        r = min(r, 127);
        uint32_t w = static_cast<uint32_t>(r) & 0xFFu;
        if (p.clamp) w = clamp4(w * 0x01010101u, p.lo4, p.hi4) & 0xFFu;
        dst[j] = static_cast<int8_t>(w);
      }
    }
  }
}

struct NoTable {
  int32_t unused;
};

template <int MODE>
struct TabOf {
  using type = EpiTable;
};
template <>
struct TabOf<kEpiGeneral> {
  using type = NoTable;
};

__device__ __forceinline__ void store16(int8_t* dst, const uint4 w) {
  if ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
    *reinterpret_cast<uint4*>(dst) = w;
  } else {
    const uint32_t packed[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int g = 0; g < 4; ++g)
#pragma unroll
      for (int j = 0; j < 4; ++j) dst[4 * g + j] = static_cast<int8_t>(packed[g] >> (8 * j));
  }
}

// Constant-table version of epilogue_chunk (fast requant only), channel
// offset known at run time.  `border`: the row's class is not the table's
// base class; its bias difference sits at dbias[cls_off + channel].  QF:
// kEpFloor for floor-form tables, else 0; the clamp is chosen at run time.
template <int QF>
__device__ __forceinline__ void epilogue_chunk_tab(uint32_t (&v)[16], int8_t* dst,
                                                   const EpiTable& tab, bool border, int cls_off,
                                                   int nc, int cnt, const TcGemmArgs& p) {
  if (border) add_class_delta(v, tab, cls_off + nc, cnt);
  if (cnt == 16) {
    store16(dst, p.clamp ? requant16_tab<QF | kEpClamp>(v, tab, nc, p.lo4, p.hi4)
                         : requant16_tab<QF>(v, tab, nc, p.lo4, p.hi4));
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (j < cnt) {
        int32_t r = rq_tab_q<QF>(v[j], tab.mh[nc + j], tab.bs[nc + j]);
        r = max(r, -128);
        r = min(r, 127);
        uint32_t w = static_cast<uint32_t>(r) & 0xFFu;
        if (p.clamp) w = clamp4(w * 0x01010101u, p.lo4, p.hi4) & 0xFFu;
        dst[j] = static_cast<int8_t>(w);
      }
    }
  }
}

// One output row of BN channels with compile-time table offsets: every
// per-channel constant is a constant-bank operand of the instruction using
// it.  Tensor-memory loads run one 16-column chunk ahead of the arithmetic;
// for tiles of up to 128 columns each 32-column pair of chunks leaves as one
// 32-byte store (rows of N bytes, N a multiple of 32, 32-byte aligned
// output).  Q: the op's ep_flags.
template <int BN, int NOFF, int Q>
__device__ __forceinline__ void epilogue_row_static(const EpiTable& tab, uint32_t taddr,
                                                    int8_t* orow, bool valid,
                                                    const TcGemmArgs& p) {
  orow += NOFF;
  uint32_t v0[16], v1[16];
  tmem_ld16_nowait(taddr, v0);
  static_assert(BN % 32 == 0, "32-byte stores");
#pragma unroll
  for (int c = 0; c < BN; c += 32) {
    tmem_wait_ld(v0);
    tmem_ld16_nowait(taddr + c + 16, v1);
    const uint4 w0 = requant16_tab<Q>(v0, tab, NOFF + c, p.lo4, p.hi4);
    if constexpr (BN > 128) {
      // (Measured: 256-column rows lose with the paired store.)
      if (valid) *reinterpret_cast<uint4*>(orow + c) = w0;
    }
    tmem_wait_ld(v1);
    if (c + 32 < BN) tmem_ld16_nowait(taddr + c + 32, v0);
    const uint4 w1 = requant16_tab<Q>(v1, tab, NOFF + c + 16, p.lo4, p.hi4);
    if constexpr (BN > 128) {
      if (valid) *reinterpret_cast<uint4*>(orow + c + 16) = w1;
    } else {
      if (valid) st_global_v8(orow + c, w0, w1);
    }
  }
}

// One output row of a 2D tile at a run-time table offset n0 (kEpiTable, the
// group's columns inside N, 32-byte aligned rows): as epilogue_row_static,
// but the loop over 32-column pairs is not unrolled and the constants are
// loaded at run-time offsets, so one small body serves every N tile of the
// grid.  Q: the op's ep_flags.
template <int BN, int Q>
__device__ __forceinline__ void epilogue_row_tab(const EpiTable& tab, uint32_t taddr,
                                                 int8_t* orow, int n0, bool valid,
                                                 const TcGemmArgs& p) {
  static_assert(BN % 32 == 0, "32-byte stores");
  orow += n0;
  uint32_t v0[16], v1[16];
  tmem_ld16_nowait(taddr, v0);
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    tmem_wait_ld(v0);
    tmem_ld16_nowait(taddr + c + 16, v1);
    const uint4 w0 = requant16_tab<Q>(v0, tab, n0 + c, p.lo4, p.hi4);
    tmem_wait_ld(v1);
    if (c + 32 < BN) tmem_ld16_nowait(taddr + c + 32, v0);
    const uint4 w1 = requant16_tab<Q>(v1, tab, n0 + c + 16, p.lo4, p.hi4);
    if (valid) st_global_v8(orow + c, w0, w1);
  }
}

// One output pixel of a conv tile whose N is the tile width, every
// requantisation constant at a compile-time table offset (a constant-bank
// operand, no load): the run-time-offset loop of kEpiTable loads two table
// words per output.  Tensor-memory loads run one 16-column chunk ahead.
// `border`: the pixel's class is not the table's base class (its bias
// differences are drow[channel], the class's row in shared memory).  POOL: the 2x2 max
// over lanes l, l ^ 1, l ^ vert (see the pooled branch of the kernel); the
// window's top-left lane stores the pooled chunk at `orow`.  Q: the op's
// ep_flags.
template <int BN, int Q, bool POOL>
__device__ __forceinline__ void epilogue_row_conv(const EpiTable& tab, uint32_t taddr,
                                                  int8_t* orow, bool store, bool border,
                                                  const int32_t* drow, int vert,
                                                  const TcGemmArgs& p) {
  uint32_t v0[16], v1[16];
  tmem_ld16_nowait(taddr, v0);
#pragma unroll
  for (int c = 0; c < BN; c += 32) {
    tmem_wait_ld(v0);
    tmem_ld16_nowait(taddr + c + 16, v1);
    if (border)
#pragma unroll
      for (int j = 0; j < 16; ++j) v0[j] += static_cast<uint32_t>(drow[c + j]);
    uint4 w0 = requant16_tab<Q>(v0, tab, c, p.lo4, p.hi4);
    if constexpr (POOL) w0 = vmax_xor(vmax_xor(w0, 1), vert);
    if (store) store16(orow + c, w0);
    tmem_wait_ld(v1);
    if (c + 32 < BN) tmem_ld16_nowait(taddr + c + 32, v0);
    if (border)
#pragma unroll
      for (int j = 0; j < 16; ++j) v1[j] += static_cast<uint32_t>(drow[c + 16 + j]);
    uint4 w1 = requant16_tab<Q>(v1, tab, c + 16, p.lo4, p.hi4);
    if constexpr (POOL) w1 = vmax_xor(vmax_xor(w1, 1), vert);
    if (store) store16(orow + c + 16, w1);
  }
}

template <int BN, int BK, int MT, int MODE, int Q>
__global__ void __launch_bounds__(EpiShape<BN, MT, MODE>::kThreads, 1)
    k_gemm_s8(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const TcGemmArgs p, const __grid_constant__ typename TabOf<MODE>::type tab) {
  constexpr int TM = kBM * MT;  // rows per tile
  constexpr int A_BYTES = TM * BK;
  constexpr int B_BYTES = BN * BK;
  constexpr uint32_t kLayout = SwizzleFor<BK>::kLayout;
  constexpr uint32_t kSbo = 8 * BK;  // bytes between 8-row groups
  using Shape = EpiShape<BN, MT, MODE>;
  constexpr int NB = Shape::kBufs;
  constexpr int G = Shape::kGroups;
  constexpr int SPL = Shape::kSplit;  // epilogue groups per tile
  constexpr int W = BN / SPL;         // columns a group drains
  constexpr int kCols = Shape::kCols;
  constexpr uint32_t kTmemCols = Shape::kTmemCols;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int stages = p.stages;
  const int kiters = p.taps * p.kblocks;
  const int grp = p.group;  // k-iterations per stage
  uint8_t* sA = smem;
  uint8_t* sB = smem + stages * grp * A_BYTES;  // B ring, or all of B when b_res
  uint8_t* sP = sB + (p.b_res ? kiters : stages * grp) * B_BYTES;  // staged requant + bias tables
  RqChannel* srq = reinterpret_cast<RqChannel*>(sP);
  int32_t* sbias = reinterpret_cast<int32_t*>(sP + static_cast<size_t>(p.N) * sizeof(RqChannel));
  int32_t* sdb = reinterpret_cast<int32_t*>(sP + p.param_smem);  // [ncls][BN + 1]
  uint64_t* full = reinterpret_cast<uint64_t*>(sP + p.param_smem + p.dbias_smem);
  uint64_t* empty = full + stages;
  uint64_t* tfull = empty + stages;
  uint64_t* tempty = tfull + NB;
  uint64_t* mma_done = tempty + NB;
  uint64_t* bres_full = mma_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bres_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < NB; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4 * SPL);
    }
    mbar_init(mma_done, 1);
    mbar_init(bres_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (p.param_smem) {
    for (int i = threadIdx.x; i < p.N; i += blockDim.x) srq[i] = p.rq[i];
    for (int i = threadIdx.x; i < p.ncls * p.N; i += blockDim.x) sbias[i] = p.bias[i];
  }
  if constexpr (MODE == kEpiConvStatic) {
    if (p.dbias_smem)
      for (int i = threadIdx.x; i < p.ncls * BN; i += blockDim.x)
        sdb[(i / BN) * (BN + 1) + i % BN] = tab.dbias[i];
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    // One thread; the loop body is kept short (no divisions, incremental
    // coordinates): at small K it issues a tile every few hundred cycles
    // and its own latency sets the pace.
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int64_t issued = 0;
      bool ok = true;
      const uint32_t a_tx = static_cast<uint32_t>(grp) * (p.b_res ? A_BYTES : A_BYTES + B_BYTES);
      if (p.b_res) {
        // Every SM would otherwise fetch the same few KB of weights from the
        // same L2 slices for every tile.
        mbar_arrive_expect_tx(bres_full, static_cast<uint32_t>(kiters * B_BYTES));
        for (int it = 0; it < kiters; ++it) {
          const int tap = it / p.kblocks;
          const int kb = it - tap * p.kblocks;
          tma_load_2d(sB + it * B_BYTES, &tmB, bres_full, tap * p.Kc + kb * BK,
                      static_cast<int32_t>(blockIdx.x % p.tiles_n) * BN);
        }
      }
      // Tile t = tm * tiles_n + tn, advanced by gridDim.x per step.
      const int32_t tiles_n = p.tiles_n;
      const int32_t step_m = static_cast<int32_t>(gridDim.x) / tiles_n;
      const int32_t step_n = static_cast<int32_t>(gridDim.x) - step_m * tiles_n;
      int32_t tm = static_cast<int32_t>(blockIdx.x) / tiles_n;
      int32_t tn = static_cast<int32_t>(blockIdx.x) - tm * tiles_n;
      const int32_t kblocks = p.kblocks;
      for (int64_t t = blockIdx.x; t < p.tiles_total; t += gridDim.x) {
        TileOrigin o{0, 0, 0};
        if (p.conv4d) o = tile_origin(p, static_cast<uint32_t>(tm));
        int tap = 0, kb = 0, ky = 0, kx = 0;
        // (The static 2D epilogue only runs 1x1 GEMMs, whose stages are one
        // k-block: those kernels carry only this loop.)
        if (MODE == kEpiStatic || grp == 1) {
        // One k-block per stage (the loop of the 1x1 GEMMs, whose tiles are
        // short enough that this thread's own instructions set the pace).
        for (int it = 0; it < kiters; ++it) {
          if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag)) {
            record_error(p.err, abort_flag, kDevErrTmaWait);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], a_tx);
          if (p.conv4d)
            tma_load_4d(sA + s * A_BYTES, &tmA, &full[s], kb * BK, o.x0 + kx - p.pad_l,
                        o.y0 + ky - p.pad_t, static_cast<int32_t>(o.n0));
          else
            tma_load_2d(sA + s * A_BYTES, &tmA, &full[s], kb * BK, tm * TM);
          if (!p.b_res)
            tma_load_2d(sB + s * B_BYTES, &tmB, &full[s], tap * p.Kc + kb * BK, tn * BN);
          ++issued;
          if (++s == stages) {
            s = 0;
            ph ^= 1u;
          }
          if (++kb == kblocks) {
            kb = 0;
            ++tap;
            if (++kx == p.kw) {
              kx = 0;
              ++ky;
            }
          }
        }
        } else if constexpr (MODE != kEpiStatic)
        for (int it = 0; it < kiters; it += grp) {
          if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag)) {
            record_error(p.err, abort_flag, kDevErrTmaWait);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], a_tx);
          for (int g = 0; g < grp; ++g) {
            const int slot = s * grp + g;
            if (p.conv4d)
              tma_load_4d(sA + slot * A_BYTES, &tmA, &full[s], kb * BK, o.x0 + kx - p.pad_l,
                          o.y0 + ky - p.pad_t, static_cast<int32_t>(o.n0));
            else
              tma_load_2d(sA + slot * A_BYTES, &tmA, &full[s], kb * BK, tm * TM);
            if (!p.b_res)
              tma_load_2d(sB + slot * B_BYTES, &tmB, &full[s], tap * p.Kc + kb * BK, tn * BN);
            if (++kb == kblocks) {
              kb = 0;
              ++tap;
              if (++kx == p.kw) {
                kx = 0;
                ++ky;
              }
            }
          }
          ++issued;
          if (++s == stages) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        tm += step_m;
        tn += step_n;
        if (tn >= tiles_n) {
          tn -= tiles_n;
          ++tm;
        }
      }
      if (!ok) {
        // Let the copies already issued land before the CTA's smem goes away.
        const int64_t first = issued > stages ? issued - stages : 0;
        for (int64_t g = first; g < issued; ++g)
          mbar_wait(&full[g % stages], static_cast<uint32_t>((g / stages) & 1), nullptr);
      }
      if (p.b_res) mbar_wait(bres_full, 0, nullptr);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc_s8(kBM, BN);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      if (p.b_res && !mbar_wait(bres_full, 0, abort_flag)) {
        record_error(p.err, abort_flag, kDevErrMmaWait);
        ok = false;
      }
      const uint32_t a_base = smem_u32(sA);
      const uint32_t b_base = smem_u32(sB);
      int b = 0;
      uint32_t use_par = 0;  // parity of the current pass over the NB buffers
      for (int64_t t = blockIdx.x; ok && t < p.tiles_total; t += gridDim.x) {
        if (!mbar_wait(&tempty[b], use_par ^ 1u, abort_flag)) {
          record_error(p.err, abort_flag, kDevErrMmaWait);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(b * kCols);
        if (MODE == kEpiStatic || grp == 1) {
        for (int it = 0; it < kiters; ++it) {
          if (!mbar_wait(&full[s], ph, abort_flag)) {
            record_error(p.err, abort_flag, kDevErrMmaWait);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = a_base + static_cast<uint32_t>(s * A_BYTES);
          const uint32_t b0 = b_base + static_cast<uint32_t>((p.b_res ? it : s) * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk) {
            const uint64_t bd = make_sdesc(b0 + kk * 32, 16, kSbo, kLayout);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
              const uint64_t ad = make_sdesc(a0 + mt * kBM * BK + kk * 32, 16, kSbo, kLayout);
              umma_i8(d_tmem + mt * BN, ad, bd, idesc, (it > 0 || kk > 0) ? 1u : 0u);
            }
          }
          umma_commit(&empty[s]);
          if (++s == stages) {
            s = 0;
            ph ^= 1u;
          }
        }
        } else if constexpr (MODE != kEpiStatic)
        for (int it = 0; it < kiters; it += grp) {
          if (!mbar_wait(&full[s], ph, abort_flag)) {
            record_error(p.err, abort_flag, kDevErrMmaWait);
            ok = false;
            break;
          }
          tc_fence_after();
          for (int g = 0; g < grp; ++g) {
            const int slot = s * grp + g;
            const uint32_t a0 = a_base + static_cast<uint32_t>(slot * A_BYTES);
            const uint32_t b0 =
                b_base + static_cast<uint32_t>((p.b_res ? it + g : slot) * B_BYTES);
#pragma unroll
            for (int kk = 0; kk < BK / 32; ++kk) {
              const uint64_t bd = make_sdesc(b0 + kk * 32, 16, kSbo, kLayout);
#pragma unroll
              for (int mt = 0; mt < MT; ++mt) {
                const uint64_t ad = make_sdesc(a0 + mt * kBM * BK + kk * 32, 16, kSbo, kLayout);
                umma_i8(d_tmem + mt * BN, ad, bd, idesc, (it + g > 0 || kk > 0) ? 1u : 0u);
              }
            }
          }
          umma_commit(&empty[s]);
          if (++s == stages) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[b]);
        if (++b == NB) {
          b = 0;
          use_par ^= 1u;
        }
      }
      // All MMAs issued by this thread complete before tensor memory is freed.
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, nullptr);
    }
  } else {
    // --------------------------------------------------------- epilogue
    const int grp = (warp - 2) >> 2;
    const int gt = grp / SPL;                // tile slot of this group
    const int c_lo = (grp - gt * SPL) * W;   // its first column in the tile
    const int q = warp & 3;  // tensor-memory lane quarter this warp may read
    const int row = q * 32 + lane;
    const uint32_t tlane = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    const bool fast = MODE != kEpiGeneral || *p.all_fast != 0;
    const RqChannel* rqb = p.param_smem ? srq : p.rq;
    const int32_t* bb = p.param_smem ? sbias : p.bias;
    int64_t i = gt;
    for (int64_t t = blockIdx.x + static_cast<int64_t>(gt) * gridDim.x; t < p.tiles_total;
         t += static_cast<int64_t>(G / SPL) * gridDim.x, i += G / SPL) {
      const int b = static_cast<int>(i % NB);
      const uint32_t use = static_cast<uint32_t>(i / NB);
      int ready = 0;
      if (lane == 0) {
        ready = mbar_wait(&tfull[b], use & 1u, abort_flag) ? 1 : 0;
        if (!ready) record_error(p.err, abort_flag, kDevErrEpiWait);
      }
      ready = __shfl_sync(0xFFFFFFFFu, ready, 0);
      if (!ready) break;
      tc_fence_after();
      const uint32_t tb0 = tlane + static_cast<uint32_t>(b * kCols);

      if constexpr (MODE == kEpiStatic) {
        // One N tile (the host picks this variant only then).
        const uint32_t tm = static_cast<uint32_t>(t);
#pragma unroll 1
        for (int mt = 0; mt < MT; ++mt) {
          const int64_t r = static_cast<int64_t>(tm) * TM + mt * kBM + row;
          int8_t* orow = p.out + r * p.ldo;
          const uint32_t ta = tb0 + static_cast<uint32_t>(mt * BN);
          if constexpr (SPL == 1)
            epilogue_row_static<BN, 0, Q>(tab, ta, orow, r < p.rows, p);
          else if (c_lo == 0)
            epilogue_row_static<W, 0, Q>(tab, ta, orow, r < p.rows, p);
          else
            epilogue_row_static<W, W, Q>(tab, ta + W, orow, r < p.rows, p);
        }
      } else if constexpr (MODE == kEpiConvStatic) {
        // Implicit-GEMM conv, one N tile: pixel (x, y) of image n.
        const uint32_t tm = static_cast<uint32_t>(t);
        const TileOrigin o = tile_origin(p, tm);
        const int32_t x = o.x0 + (row & ((1 << p.bw_log2) - 1));
        const int32_t y = o.y0 + ((row >> p.bw_log2) & ((1 << p.bh_log2) - 1));
        const int64_t n = o.n0 + (row >> (p.bw_log2 + p.bh_log2));
        const bool valid = x < p.Wo && y < p.Ho && n < p.nimg;
        const int32_t* drow = sdb;
        bool border = false;
        if (valid && p.ycls != nullptr) {
          const int cls = p.ycls[y] * p.n_xcls + p.xcls[x];
          drow = sdb + cls * (BN + 1);
          border = cls != p.base_cls;
        }
        if (p.pool) {
          int8_t* prow =
              p.out + ((n * p.Hp + (y >> 1)) * p.Wp + (x >> 1)) * static_cast<int64_t>(BN);
          epilogue_row_conv<BN, Q, true>(tab, tb0, prow, valid && ((x | y) & 1) == 0, border,
                                         drow, 1 << p.bw_log2, p);
        } else {
          int8_t* orow = p.out + ((n * p.Ho + y) * p.Wo + x) * static_cast<int64_t>(BN);
          epilogue_row_conv<BN, Q, false>(tab, tb0, orow, valid, border, drow, 0, p);
        }
      } else {
#pragma unroll 1
      for (int mt = 0; mt < MT; ++mt) {
        const uint32_t tb = tb0 + static_cast<uint32_t>(mt * BN);
        const uint32_t tm = p.fd_tiles_n.div(static_cast<uint32_t>(t));
        const int32_t tn = static_cast<int32_t>(t - static_cast<int64_t>(tm) * p.tiles_n);
        bool valid;
        int8_t* orow;
        const int32_t* brow = bb;
        int cls_off = 0;
        bool border = false;
        if (p.conv4d) {
          const TileOrigin o = tile_origin(p, tm);
          const int32_t x = o.x0 + (row & ((1 << p.bw_log2) - 1));
          const int32_t y = o.y0 + ((row >> p.bw_log2) & ((1 << p.bh_log2) - 1));
          const int64_t n = o.n0 + (row >> (p.bw_log2 + p.bh_log2));
          valid = x < p.Wo && y < p.Ho && n < p.nimg;
          orow = p.out + ((n * p.Ho + y) * p.Wo + x) * static_cast<int64_t>(p.N);
          if (valid && p.ycls != nullptr) {
            const int cls = p.ycls[y] * p.n_xcls + p.xcls[x];
            cls_off = cls * p.N;
            border = cls != p.base_cls;
            brow = bb + cls_off;
          }
          if constexpr (MODE == kEpiTable) {
            if (p.pool) {
              // Conv + ReLU + 2x2 max pool: requantise this pixel's 16
              // channels, take the max with the window's other three lanes
              // (horizontal neighbour lane ^ 1, vertical lane ^ bw) and let
              // the window's top-left lane store the pooled chunk.  TFLite
              // pools the requantised int8 outputs, so this is exact.  The
              // host fuses only N % 16 == 0 and even Ho, Wo: a window's
              // lanes are all valid or all invalid, and every lane joins
              // the shuffles.
              int8_t* prow =
                  p.out + ((n * p.Hp + (y >> 1)) * p.Wp + (x >> 1)) * static_cast<int64_t>(p.N);
              const bool store = valid && ((x | y) & 1) == 0;
              const int vert = 1 << p.bw_log2;
#pragma unroll 1
              for (int c = c_lo; c < c_lo + W; c += 16) {
                uint32_t v[16];
                tmem_ld16(tb + static_cast<uint32_t>(c), v);
                const int32_t nc = tn * BN + c;
                if (nc < p.N) {
                  if (border) add_class_delta(v, tab, cls_off + nc, 16);
                  uint4 w = p.clamp
                                ? requant16_tab<(Q & kEpFloor) | kEpClamp>(v, tab, nc, p.lo4, p.hi4)
                                : requant16_tab<Q & kEpFloor>(v, tab, nc, p.lo4, p.hi4);
                  w = vmax_xor(vmax_xor(w, 1), vert);
                  if (store) store16(prow + nc, w);
                }
              }
              continue;
            }
          }
        } else {
          const int64_t r = static_cast<int64_t>(tm) * TM + mt * kBM + row;
          valid = r < p.rows;
          orow = p.out + r * p.ldo;
        }
        const int32_t n0 = tn * BN;
        if constexpr (MODE == kEpiTable && W <= 128) {
          if (!p.conv4d && n0 + c_lo + W <= p.N &&
              ((reinterpret_cast<uintptr_t>(p.out) | static_cast<uintptr_t>(p.ldo)) & 31u) == 0) {
            const uint32_t th = tb + static_cast<uint32_t>(c_lo);
            if (p.clamp)
              epilogue_row_tab<W, (Q & kEpFloor) | kEpClamp>(tab, th, orow, n0 + c_lo, valid, p);
            else
              epilogue_row_tab<W, Q & kEpFloor>(tab, th, orow, n0 + c_lo, valid, p);
            continue;
          }
        }
        // (256-column tiles only: the tile the host picks for odd N > 256
        // without a constant table; narrower variants keep their registers.)
        if constexpr (MODE == kEpiGeneral && BN == 256)
        if (!p.conv4d && (p.ldo & 3) != 0 && n0 + BN <= p.N) {
          // Rows whose starts are not 4-byte aligned (an odd row length such
          // as 3337 logits), full N tile: this thread writes the row segment
          // [n0, n0 + BN) in order, so each 16-byte chunk leaves as four
          // 4-byte-aligned words, funnel-shifted against the previous
          // chunk's last word; only the s = start % 4 head and tail bytes
          // are single-byte stores.  (Sixteen byte stores per chunk, each
          // touching 32 rows, had made this epilogue store-bound.)
          int8_t* d0 = orow + n0;
          const uint32_t sa = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(d0) & 3u);
          uint32_t* aw = reinterpret_cast<uint32_t*>(d0 - sa);
          const uint32_t sh = 8u * (4u - sa);
          uint32_t carry = 0;
#pragma unroll 1
          for (int c = 0; c < BN; c += 16) {
            uint32_t v[16];
            tmem_ld16(tb + static_cast<uint32_t>(c), v);
            if (valid) {
              uint32_t w[4];
              if (fast)
                requant_chunk16<true>(v, brow + n0 + c, rqb + n0 + c, p, w);
              else
                requant_chunk16<false>(v, brow + n0 + c, rqb + n0 + c, p, w);
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const int j = c / 4 + k;  // aligned word: segment bytes 4j - sa .. 4j + 3 - sa
                if (j == 0 && sa != 0) {
#pragma unroll
                  for (int t = 0; t < 3; ++t)
                    if (t < static_cast<int>(4u - sa)) d0[t] = static_cast<int8_t>(w[0] >> (8 * t));
                } else {
                  aw[j] = __funnelshift_rc(carry, w[k], sh);
                }
                carry = w[k];
              }
            }
          }
          if (valid && sa != 0) {
#pragma unroll
            for (int t = 0; t < 3; ++t)
              if (t < static_cast<int>(sa))
                d0[BN - static_cast<int>(sa) + t] =
                    static_cast<int8_t>(carry >> (8 * (4 - static_cast<int>(sa) + t)));
          }
          continue;
        }
#pragma unroll 1
        for (int c = c_lo; c < c_lo + W; c += 16) {
          uint32_t v[16];
          tmem_ld16(tb + static_cast<uint32_t>(c), v);
          const int32_t nc = n0 + c;
          if (valid && nc < p.N) {
            const int cnt = min(16, p.N - nc);
            if constexpr (MODE == kEpiTable) {
              epilogue_chunk_tab<Q & kEpFloor>(v, orow + nc, tab, border, cls_off, nc, cnt, p);
            } else {
              if (fast)
                epilogue_chunk<true>(v, orow + nc, brow + nc, rqb + nc, cnt, p);
              else
                epilogue_chunk<false>(v, orow + nc, brow + nc, rqb + nc, cnt, p);
            }
          }
        }
      }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

inline int ilog2_exact(int v) {
  int l = 0;
  while ((1 << l) < v) ++l;
  return l;
}

inline int pow2_ceil(int v) {
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}

// Sets the dynamic shared memory limit of one kernel variant, once per
// device.
template <int BN, int BK, int MT, int MODE, int Q>
cudaError_t ensure_smem_attr() {
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if ((done.load() & bit) != 0) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(k_gemm_s8<BN, BK, MT, MODE, Q>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kSmemLimit);
  if (e == cudaSuccess) done.fetch_or(bit);
  return e;
}

template <int BN, int BK, int MT, int MODE, int Q>
cudaError_t launch_variant(const CUtensorMap& ma, const CUtensorMap& mb, const TcGemmArgs& args,
                           const typename TabOf<MODE>::type& tab, int64_t grid, int smem,
                           cudaStream_t s) {
  const cudaError_t e = ensure_smem_attr<BN, BK, MT, MODE, Q>();
  if (e != cudaSuccess) return e;
  k_gemm_s8<BN, BK, MT, MODE, Q>
      <<<static_cast<unsigned>(grid), EpiShape<BN, MT, MODE>::kThreads, smem, s>>>(ma, mb, args, tab);
  return cudaGetLastError();
}

// Epilogue variant per op: the static constant-table epilogue for 2D
// operands with one N tile, the run-time-offset table epilogue for other
// ops whose host holds a table, the general one (tables in smem or global,
// runtime fast/general flag) otherwise.  (With four N tiles the static
// epilogue ran four compile-time bodies side by side, one per tile, and its
// warps stalled on instruction fetch: 4.1-4.5 cycles per issue against 0.26
// for the same kernel with one N tile.)
template <int BN, int BK, int MT>
cudaError_t run_tc(const CUtensorMap& ma, const CUtensorMap& mb, TcGemmArgs args,
                   const EpiTable* table, int num_sms, cudaStream_t s) {
  constexpr int A_BYTES = kBM * MT * BK;
  if (table != nullptr) args.param_smem = 0;
  // A grid that is a multiple of tiles_n (or one tile per CTA) keeps every
  // CTA on one N tile; its weights then stay resident when they fit next to
  // >= 4 A stages.
  int64_t grid = std::min<int64_t>(args.tiles_total, num_sms);
  if (grid < args.tiles_total && args.tiles_n > 1 && num_sms >= args.tiles_n)
    grid = num_sms / args.tiles_n * args.tiles_n;
  const bool fixed_n = grid % args.tiles_n == 0 || grid == args.tiles_total;
  const int kiters = args.taps * args.kblocks;
  const int bres_bytes = kiters * BN * BK;
  // The conv epilogue with compile-time table offsets (N == BN, one N tile)
  // stages the border-class bias differences in shared memory.
  const bool conv_static = MT == 1 && table != nullptr && args.conv4d && args.tiles_n == 1 &&
                           args.N == BN;
  args.dbias_smem = conv_static && args.ycls != nullptr
                        ? (args.ncls * (BN + 1) * 4 + 15) / 16 * 16
                        : 0;
  const int base_overhead = 1024 + 64 * 8 + 64 + args.param_smem + args.dbias_smem;
  args.b_res = fixed_n && base_overhead + bres_bytes + 4 * A_BYTES <= kSmemLimit;
  const int iter_bytes = args.b_res ? A_BYTES : A_BYTES + BN * BK;
  const int overhead = base_overhead + (args.b_res ? bres_bytes : 0);
  // Stages of `group` k-iterations for convs with several filter taps: the
  // largest divisor of the tile's k-iterations (at most 9) that still
  // leaves three stages.  Small-channel 3x3 convs (9 taps of one K block
  // each) then take one or three barrier hand-offs per tile instead of nine.
  // (1x1 GEMMs keep one k-block per stage: grouping their 2-4 K blocks
  // measured slower.)
  int group = 1;
  for (int g = std::min(kiters, 9); args.taps > 1 && g > 1; --g)
    if (kiters % g == 0 && 3 * g * iter_bytes <= kSmemLimit - overhead) {
      group = g;
      break;
    }
  const int stage_bytes = group * iter_bytes;
  int stages = (kSmemLimit - overhead) / stage_bytes;
  stages = std::min(stages, kMaxStages);
  // At least 120 KB so that a second CTA never shares the SM: the grid is
  // one persistent CTA per SM.
  const int smem = std::max(overhead + stages * stage_bytes, 120 * 1024);
  args.stages = stages;
  args.group = group;
  if (grid <= 0) return cudaSuccess;
  if (table == nullptr) {
    // 256-row tiles only run with a constant table (the host picks MT).
    if constexpr (MT == 1)
      return launch_variant<BN, BK, MT, kEpiGeneral, 0>(ma, mb, args, NoTable{0}, grid, smem,
                                                        s);
    else
      return cudaErrorInvalidValue;
  }
  if constexpr (MT == 1) {
    if (args.conv4d && args.tiles_n == 1 && args.N == BN) {
      switch (args.ep) {
        case 0: return launch_variant<BN, BK, 1, kEpiConvStatic, 0>(ma, mb, args, *table, grid, smem, s);
        case 1: return launch_variant<BN, BK, 1, kEpiConvStatic, 1>(ma, mb, args, *table, grid, smem, s);
        case 2: return launch_variant<BN, BK, 1, kEpiConvStatic, 2>(ma, mb, args, *table, grid, smem, s);
        default: return launch_variant<BN, BK, 1, kEpiConvStatic, 3>(ma, mb, args, *table, grid, smem, s);
      }
    }
  }
  const bool is_static = !args.conv4d && fixed_n && args.tiles_n == 1 &&
                         args.N == args.tiles_n * BN && args.ldo == args.N &&
                         (reinterpret_cast<uintptr_t>(args.out) & 31u) == 0;
  if (!is_static) {
    if (args.ep & kEpFloor)
      return launch_variant<BN, BK, MT, kEpiTable, kEpFloor>(ma, mb, args, *table, grid, smem, s);
    return launch_variant<BN, BK, MT, kEpiTable, 0>(ma, mb, args, *table, grid, smem, s);
  }
  switch (args.ep) {
    case 0: return launch_variant<BN, BK, MT, kEpiStatic, 0>(ma, mb, args, *table, grid, smem, s);
    case 1: return launch_variant<BN, BK, MT, kEpiStatic, 1>(ma, mb, args, *table, grid, smem, s);
    case 2: return launch_variant<BN, BK, MT, kEpiStatic, 2>(ma, mb, args, *table, grid, smem, s);
    default: return launch_variant<BN, BK, MT, kEpiStatic, 3>(ma, mb, args, *table, grid, smem, s);
  }
}

// 256-row tiles (MT = 2) for narrow 2D GEMMs, whose per-tile handoff cost
// would otherwise dominate; 128-row tiles elsewhere.
template <int BK>
cudaError_t run_tc_bn(int bn, int mt, const CUtensorMap& ma, const CUtensorMap& mb,
                      const TcGemmArgs& args, const EpiTable* table, int num_sms,
                      cudaStream_t s) {
  if (mt == 2) {
    if (bn == 32) return run_tc<32, BK, 2>(ma, mb, args, table, num_sms, s);
    return run_tc<64, BK, 2>(ma, mb, args, table, num_sms, s);
  }
  switch (bn) {
    case 32: return run_tc<32, BK, 1>(ma, mb, args, table, num_sms, s);
    case 64: return run_tc<64, BK, 1>(ma, mb, args, table, num_sms, s);
    case 128: return run_tc<128, BK, 1>(ma, mb, args, table, num_sms, s);
    default: return run_tc<256, BK, 1>(ma, mb, args, table, num_sms, s);
  }
}

}  // namespace tcg

}  // namespace pspml
