// dwrs_tc.cu - int8 depthwise 3x3 conv (stride 1 or 2) streamed by rows
// on the tensor cores, alone or fused with the 1x1 conv after it.
//
// Block-diagonal weights turn the depthwise conv of a 32-channel group
// into GEMMs (see dw_tc.cu).  This kernel makes every input row a single
// A operand: input row y feeds the output rows r with S*r - pad_top + ky = y
// (ky = 0..2), so one MMA whose N covers those rows (32 columns of
// block-diagonal weights per row, each with its ky) updates all of them at
// once.  Per input row and group that is 3 MMAs, one per horizontal tap kx
// (the tap is a 16-byte move of the A descriptor start in the no-swizzle
// layout), and every input row is loaded once.
//
// Stride 1: an input row feeds three output rows; accumulators sit in a
// ring of R 32-column tensor-memory blocks per group (row r in block r % R).
// R = 4 for the depthwise (or dense) conv alone: the block a new row takes
// was freed by the row completed two input rows earlier, so the MMA thread
// runs a row ahead of the epilogue; an input row's blocks form one or two
// runs of consecutive blocks, one MMA per run against a window of the
// weights kept as ky blocks [2 1 0].  R = 3 for the fused pair: the three
// blocks are always all live, which weight block meets which accumulator
// block rotates with y % 3, so the weights of each kx are kept as five ky
// blocks [2 1 0 2 1] and the MMA takes the three-block window that starts
// at (1, 0, 2)[y % 3].
// Stride 2: an input row feeds one (ky = 1) or two (ky = 2 and 0) output
// rows; a ring of two blocks, weights as [2 0 2 1].  The input is viewed as
// [C][parity][W/2][N][H], so that tap kx's pixels 2j + kx - pad_left are
// one box of consecutive pairs of one parity (each tap its own box).
//
// A block must hold zeros before its row takes its first contribution, so
// the epilogue zeroes it right after reading the finished row, before the
// requantisation arithmetic; every MMA accumulates.  Output rows outside
// the image get no MMA.
//
// Work unit: a strip = one sample x one 128-pixel column tile (x one
// 64-channel block when the channels come in blocks) x all rows.  Two
// slots run independent strips so that one slot's MMAs overlap the other's
// epilogue.  Per slot: one TMA thread (16-channel boxes of 130 pixels, zero
// filled outside the image), one MMA thread and two epilogue sets of four
// warps (one per tensor-memory lane quarter) that take the slot's rows in
// turn.  Every epilogue warp handles all channels of its 32 pixels, so all
// of them run one code path: with a path per channel range the unrolled
// requantisation code of four paths interleaved on each scheduler and
// instruction fetch stalled.  Rows narrower than 128 pixels leave lanes of
// the tile idle; warps whose 32 pixels are all outside the row skip the
// arithmetic.
//
// Fused pointwise (stride 1, 64 channels): one epilogue set writes every
// requantised depthwise row into a shared-memory A tile [C/16][128][16 B]
// (two buffers, rows alternating); the MMA thread runs C/32 MMAs (M=128,
// N=NPW, K=32) against the resident 1x1 weights into a pointwise
// accumulator; the other set requantises that and stores NHWC.  The
// depthwise output never reaches global memory.
//
// Requantisation constants come from a kernel-parameter table: at
// compile-time offsets for a single channel block, at warp-uniform run-time
// offsets when the channels come in blocks.
//
// Zero points: the TMA zero fill stands for the padding, so the folded bias
// depends on the pixel's border class (in-image taps); the epilogue adds the
// class's bias difference for border pixels (tables from the model's
// preparation, as in dw_tc.cu).
//
// Every wait is bounded; on expiry the kernel records an error, stops its
// roles, drains its copies and MMAs, frees tensor memory and exits.
#include <algorithm>
#include <atomic>
#include <cstring>

#include "kernels.h"
#include "ptx.cuh"
#include "requant.cuh"

namespace pspml {

namespace {

constexpr int kRsSmemLimit = 232448;
constexpr int kRsMaxStages = 8;
constexpr int kRsMaxSets = 4;
constexpr int kRsMaxRing = 4;  // accumulator blocks per group

struct RsArgs {
  int32_t strips;  // batch * tiles_x, or batch / P rounded up (per channel block)
  int32_t tiles_x, batch;
  int32_t Hin, Ho, Wo;  // input rows, output rows and width
  int32_t pad_t, pad_l;
  FastDiv fd_tiles_x;
  const uint8_t* wdw;  // [C/32][9][2][32][16] (dw_tc packing)
  const uint8_t* wpw;  // [C/16][NPW][16] (pointwise, K-major core matrices)
  int8_t* out;         // [B][Ho][Wo][out channels]
  const uint8_t* ycls;
  const uint8_t* xcls;
  int32_t n_xcls, base_cls;
  uint32_t dw_lo4, dw_hi4, pw_lo4, pw_hi4;
  unsigned* err;
  int32_t stages;
  int32_t borders;  // 0: every border class has the base class's folded bias (an
                    // input zero point of 0), so no pixel needs a difference
};

// Barriers of one slot.  Rows are numbered per slot across its strips; row
// g belongs to epilogue set g % RS and lives in accumulator block r % R (r:
// output row).  Every barrier that a set waits on completes only for that
// set's rows, in order, and its next completion needs the set's previous
// one consumed, so no parity wait can fall two phases behind.
struct RsBars {
  uint64_t in_full[kRsMaxStages];
  uint64_t in_empty[kRsMaxStages];
  uint64_t dw_full[kRsMaxSets * kRsMaxRing];  // MMA -> set: row complete, [set][block]
  uint64_t dw_free[kRsMaxRing];               // set -> MMA: block read and zeroed
  uint64_t apw_full[kRsMaxSets];     // set -> MMA: its pointwise A tile written
  uint64_t pw_full[kRsMaxSets];      // MMA -> set: its row's pointwise accumulator complete
  uint64_t pw_empty;                 // set -> MMA: pointwise accumulator read
};

// CG: 32-channel groups per strip; NPW: pointwise outputs (0: depthwise
// only); S: stride; NCB: channel blocks of the op (CTA b takes block
// b % NCB, so all its warps use compile-time table offsets of one block);
// NS: slots; RS: epilogue sets per slot (four warps each, one per
// tensor-memory lane quarter, taking rows in turn); P: samples packed into
// the 128 tile rows (rows of at most 128 / P pixels).
// GI: 0 for the depthwise conv; for a dense 3x3 conv the number of
// 32-channel input groups (every output group then accumulates every input
// group: weights [output group][input group][tap]).
template <int CG, int NPW, int S, int NCB, int P, int GI = 0, int POOL = 0>
struct RsShape {
  static constexpr int NS = 2;
  static constexpr int RS = 2;
  static constexpr int C = CG * 32;                    // channels of a strip
  // Accumulator ring blocks.  Stride 1: an input row reaches three output
  // rows; with four blocks (the depthwise or dense conv alone) the block a
  // new row takes was read one input row earlier, so the MMAs of one row
  // never wait for the epilogue of the row completed just before.  The
  // fused pair keeps three (its pointwise accumulator needs the rest).
  static constexpr int R = S == 1 ? (NPW == 0 ? 4 : 3) : 2;
  static constexpr int NBB = S == 1 ? (R == 4 ? 3 : 5) : 4;  // weight blocks per kx
  static constexpr int kHalf = NBB * 32 * 16;          // one K-half of a kx's weights
  static constexpr int kTap = 2 * kHalf;               // weights of one (group, kx)
  static constexpr int Wt = 128 / P;                   // tile columns per sample
  // TMA boxes per input row: one (stride 1), an even and an odd one
  // (stride 2), or with packed samples one per tap kx, each already shifted
  // by its tap (a 16-byte move of the descriptor would cross into the next
  // sample's pixels).  Full rows: a box holds every 16-channel chunk of the
  // row's input groups as [chunk][pixel][16 B] (the K-major A layout
  // without swizzle, one chunk per K-half).  Packed samples: a box is
  // [sample][pixel][32 B per input group] in the 32- or 64-byte swizzled
  // K-major layout (group gi's MMA starts 32 B into the swizzle row), so
  // the copy moves whole 32-byte sectors: 16-byte rows cost one L2 request
  // and a 32-byte sector each.
  static constexpr int GIN = GI > 0 ? GI : CG;        // input groups per row
  static constexpr bool kSwz = P > 1 || S == 2;  // pre-shifted swizzled boxes
  static constexpr int kBoxes = kSwz ? 3 : 1;
  static constexpr int kBoxPx = kSwz ? 128 : 130;  // pixels per chunk
  static constexpr int kRegion = kBoxPx * 16;         // one chunk: the K-half stride
  static constexpr int kBoxBytes = GIN * 2 * kRegion;
  // Swizzled boxes start on 1024-byte boundaries, the others on 128.
  static constexpr int kBoxStride =
      kSwz ? (kBoxBytes + 1023) / 1024 * 1024 : (kBoxBytes + 127) / 128 * 128;
  static constexpr uint32_t kALayout = !kSwz ? 0u : (GIN == 1 ? 6u : 4u);  // none, 32B, 64B
  static constexpr uint32_t kALbo = kSwz ? 16u : static_cast<uint32_t>(kRegion);
  static constexpr uint32_t kASbo = kSwz ? 256u * GIN : 128u;  // between 8-row groups
  static constexpr int kInRow = kBoxes * kBoxStride;
  // Per (slot, set): the pointwise A tile, or with the pool the window's
  // first row (both [C/16][128 rows][16 B]).
  static constexpr int kApw = NPW > 0 || POOL != 0 ? 128 * C : 0;
  static constexpr int kSlotCols = 512 / NS;
  static constexpr int kThreads = 128 + NS * RS * 128;
  static_assert(CG * R * 32 + NPW <= kSlotCols, "tensor memory per slot");
  static constexpr int kBdw = CG * (GI > 0 ? GI : 1) * 3 * kTap;  // resident weights of one block
  static_assert(NCB == 1 || NPW == 0, "channel blocks are for the depthwise conv alone");
  static_assert(NCB == 1 || NCB == 2 || NCB == 4 || NCB == 8, "channel blocks");
  static_assert(P == 1 || P == 2 || P == 4, "packed samples");
  static_assert(P == 1 || NPW == 0, "packed samples are for a depthwise (or dense) conv alone");
  static_assert(NPW == 0 || S == 1, "fused pointwise after a stride-1 depthwise conv");
  static_assert(RS <= kRsMaxSets, "epilogue sets");
  static_assert(R <= kRsMaxRing, "accumulator ring");
  static_assert(GI == 0 || (NCB == 1 && NPW == 0), "dense conv: one channel block, no pair");
  static_assert(POOL == 0 || (NPW == 0 && NCB == 1 && S == 1), "pool after a dense conv");
};

// Weight block order per kx: ky of each 32-row block.  Stride 1, 3-block
// ring: [2 1 0 2 1] (every rotation of [2 1 0] is a window); 4-block ring:
// [2 1 0] (a run of consecutive blocks holds consecutive rows, so its
// windows are pieces of [2 1 0]); stride 2: [2 0 2 1].
__host__ __device__ constexpr int rs_block_ky(int S, int nbb, int blk) {
  return S == 1 ? (nbb == 3 ? 2 - blk : (blk == 2 ? 0 : ((blk == 1 || blk == 4) ? 1 : 2)))
                : (blk == 1 ? 0 : (blk == 3 ? 1 : 2));
}

__device__ __forceinline__ void rs_record_error(unsigned* err, volatile int* abort_flag,
                                                unsigned code) {
  *abort_flag = 1;
  if (err != nullptr) atomicCAS(err, 0u, code);
}

__device__ __forceinline__ void rs_fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Lane 0 waits, the warp learns the outcome.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int lane) {
  int ok = 0;
  if (lane == 0) ok = mbar_wait(bar, parity, abort_flag) ? 1 : 0;
  return __shfl_sync(0xFFFFFFFFu, ok, 0) != 0;
}

template <int Q>
__device__ __forceinline__ uint4 rs_requant16(const uint32_t* v, const int2* mh, const int2* bs,
                                              int ch, uint32_t lo4, uint32_t hi4) {
  uint32_t packed[4];
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    int32_t r[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = ch + 4 * g + k;
      if constexpr ((Q & kEpFloor) != 0) {
        r[k] = rq_floor_entry(v[4 * g + k], mh[c], bs[c]);
      } else {
        const int2 b = bs[c];
        r[k] = rq_tab(static_cast<int32_t>(v[4 * g + k]) + b.x, mh[c], b.y);
      }
    }
    uint32_t w = pack_sat4(r[0], r[1], r[2], r[3]);
    if constexpr ((Q & kEpClamp) != 0) w = clamp4(w, lo4, hi4);
    packed[g] = w;
  }
  return make_uint4(packed[0], packed[1], packed[2], packed[3]);
}

// Strip i -> (first sample, column tile).
struct RsStrip {
  uint32_t n;
  int tx;
};
template <int P>
__device__ __forceinline__ RsStrip rs_strip(const RsArgs& p, int i) {
  RsStrip st;
  if constexpr (P > 1) {
    st.n = static_cast<uint32_t>(i) * P;
    st.tx = 0;
  } else {
    st.n = p.fd_tiles_x.div(static_cast<uint32_t>(i));
    st.tx = i - static_cast<int>(st.n) * p.tiles_x;
  }
  return st;
}

// Strips of slot k of this CTA: the CTAs of one channel block share its
// strips.
__device__ __forceinline__ void rs_strip_range(int ncb, int k, int ns, int* first, int* step) {
  const int per_block = static_cast<int>(gridDim.x) / ncb;
  *first = static_cast<int>(blockIdx.x) / ncb + k * per_block;
  *step = ns * per_block;
}

// Epilogue of one warp: set `set` of slot `k`, lane quarter q, every
// channel of the strip.  All epilogue warps of a kernel run this one code
// path.
template <int CG, int NPW, int S, int NCB, int P, int CB, int DWQ, int PWQ, int GI, int POOL>
__device__ __forceinline__ void rs_epilogue(const RsArgs& p, const DwPwTable& tab, RsBars& bars,
                                            uint8_t* sA, uint32_t tm_slot, int k, int set, int q,
                                            int lane, volatile int* abort_flag) {
  using Sh = RsShape<CG, NPW, S, NCB, P, GI, POOL>;
  constexpr int C = Sh::C;
  constexpr int R = Sh::R;
  constexpr int RS = Sh::RS;
  constexpr int NV = C / 16;
  constexpr int Cop = NCB * C;   // channels of the op
  constexpr int cbase = CB * C;  // this CTA's channel block
  constexpr int NP = NPW / 16;
  const int row = q * 32 + lane;
  const uint32_t tl = tm_slot + (static_cast<uint32_t>(q * 32) << 16);

  // The accumulator blocks start zeroed (set 0 covers every lane).
  if (set == 0) {
#pragma unroll
    for (int g = 0; g < CG; ++g)
#pragma unroll
      for (int j = 0; j < R; ++j) {
        tmem_st16_zero(tl + g * R * 32 + j * 32);
        tmem_st16_zero(tl + g * R * 32 + j * 32 + 16);
      }
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0)
#pragma unroll
      for (int j = 0; j < R; ++j) mbar_arrive(&bars.dw_free[j]);
  }

  int first, step;
  rs_strip_range(NCB, k, Sh::NS, &first, &step);
  const int Ho = p.Ho;

  if constexpr (NPW > 0) {
    // Fused pair: set 0 requantises every row's depthwise output into the
    // pointwise A tile of buffer g % RS, set 1 every row's pointwise output,
    // so neither set waits for the other half of its own row.  Barriers:
    // dw_full[g % RS][r % R] (rows of one barrier complete in row order and
    // set 0 frees a block only after waiting for its previous row), apw_full
    // and pw_full per A buffer, pw_empty for the one pointwise accumulator.
    // Set 0 rewrites buffer b only after the pointwise MMAs of row g - RS
    // that read it have completed.
    uint32_t full_ph = 0;  // bit (b * R + rb): parity of the next wait on dw_full[b][rb]
    uint32_t g = 0;        // row number within the slot
    for (int i = first; i < p.strips; i += step) {
      const RsStrip st = rs_strip<P>(p, i);
      const int x = st.tx * 128 + row;
      const bool valid = x < p.Wo;
      int cls_top = p.base_cls, cls_mid = p.base_cls, cls_bot = p.base_cls;
      if (set == 0 && valid && p.borders) {
        const int xc = p.xcls[x];
        cls_top = p.ycls[0] * p.n_xcls + xc;
        cls_mid = p.ycls[Ho > 1 ? 1 : 0] * p.n_xcls + xc;
        cls_bot = p.ycls[Ho - 1] * p.n_xcls + xc;
      }
      const int64_t pix0 = (static_cast<int64_t>(st.n) * Ho) * p.Wo + x;
      for (int r = 0; r < Ho; ++r, ++g) {
        const int b = static_cast<int>(g % RS);
        if (set == 0) {
          const int rb = r % R;
          const int bit = b * R + rb;
          if (!warp_wait(&bars.dw_full[b * kRsMaxRing + rb], (full_ph >> bit) & 1u, abort_flag,
                         lane)) {
            if (lane == 0) rs_record_error(p.err, abort_flag, kDevErrEpiWait);
            return;
          }
          full_ph ^= 1u << bit;
          tc_fence_after();
          uint32_t v[NV][16];
#pragma unroll
          for (int h = 0; h < NV; ++h)
            tmem_ld16_nowait(
                tl + static_cast<uint32_t>((h / 2) * R * 32 + rb * 32 + (h % 2) * 16), v[h]);
#pragma unroll
          for (int h = 0; h < NV; ++h) tmem_wait_ld(v[h]);
#pragma unroll
          for (int h = 0; h < NV; ++h)
            tmem_st16_zero(tl + static_cast<uint32_t>((h / 2) * R * 32 + rb * 32 + (h % 2) * 16));
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars.dw_free[rb]);
          const int cls = r == 0 ? cls_top : (r == Ho - 1 ? cls_bot : cls_mid);
          if (valid && cls != p.base_cls) {
            const int off = cls * C;
#pragma unroll
            for (int h = 0; h < NV; ++h)
#pragma unroll
              for (int j = 0; j < 16; ++j)
                v[h][j] += static_cast<uint32_t>(tab.dw_dbias[off + h * 16 + j]);
          }
          if (g >= static_cast<uint32_t>(RS) &&
              !warp_wait(&bars.pw_full[b], ((g / RS) - 1u) & 1u, abort_flag, lane)) {
            if (lane == 0) rs_record_error(p.err, abort_flag, kDevErrEpiWait);
            return;
          }
          uint8_t* atile = sA + b * Sh::kApw + row * 16;
#pragma unroll
          for (int h = 0; h < NV; ++h)
            *reinterpret_cast<uint4*>(atile + h * 2048) =
                rs_requant16<DWQ>(v[h], tab.dw_mh, tab.dw_bs, h * 16, p.dw_lo4, p.dw_hi4);
          rs_fence_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars.apw_full[b]);
        } else {
          if (!warp_wait(&bars.pw_full[b], (g / RS) & 1u, abort_flag, lane)) {
            if (lane == 0) rs_record_error(p.err, abort_flag, kDevErrEpiWait);
            return;
          }
          tc_fence_after();
          uint32_t u[NP][16];
          const uint32_t tp = tl + static_cast<uint32_t>(CG * R * 32);
#pragma unroll
          for (int h = 0; h < NP; ++h) tmem_ld16_nowait(tp + h * 16, u[h]);
#pragma unroll
          for (int h = 0; h < NP; ++h) tmem_wait_ld(u[h]);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars.pw_empty);
          if (valid) {
            int8_t* o = p.out + (pix0 + static_cast<int64_t>(r) * p.Wo) * NPW;
            static_assert(NP % 2 == 0, "32-byte stores");
#pragma unroll
            for (int h = 0; h < NP; h += 2)
              st_global_v8(o + 16 * h,
                           rs_requant16<PWQ>(u[h], tab.pw_mh, tab.pw_bs, h * 16, p.pw_lo4,
                                             p.pw_hi4),
                           rs_requant16<PWQ>(u[h + 1], tab.pw_mh, tab.pw_bs, h * 16 + 16,
                                             p.pw_lo4, p.pw_hi4));
          }
        }
      }
    }
    return;
  }

  uint32_t full_ph = 0;  // bit j: parity of the next wait on dw_full[set][j]
  uint8_t* atile = sA + set * Sh::kApw + row * 16;
  uint32_t g = 0;  // row number within the slot
  for (int i = first; i < p.strips; i += step) {
    const RsStrip st = rs_strip<P>(p, i);
    // Tile row -> (sample, pixel): with packed samples, sample row / Wt.
    const uint32_t n = st.n + static_cast<uint32_t>(row / Sh::Wt);
    const int x = st.tx * 128 + (P > 1 ? row % Sh::Wt : row);
    const bool valid = x < p.Wo && (P == 1 || static_cast<int>(n) < p.batch);
    const bool any_valid = __any_sync(0xFFFFFFFFu, valid);
    // Border classes: the first, the last and the interior output rows.
    int cls_top = p.base_cls, cls_mid = p.base_cls, cls_bot = p.base_cls;
    if (valid && p.borders) {
      const int xc = p.xcls[x];
      cls_top = p.ycls[0] * p.n_xcls + xc;
      cls_mid = p.ycls[Ho > 1 ? 1 : 0] * p.n_xcls + xc;
      cls_bot = p.ycls[Ho - 1] * p.n_xcls + xc;
    }
    const int64_t pix0 = (static_cast<int64_t>(n) * Ho) * p.Wo + x;
    for (int r = 0; r < Ho; ++r, ++g) {
      // With the pool, a set takes output rows in pairs (both rows of a
      // pooling window).
      if (static_cast<int>((POOL ? g >> 1 : g) % RS) != set) continue;
      const int rb = r % R;
      if (!warp_wait(&bars.dw_full[set * kRsMaxRing + rb], (full_ph >> rb) & 1u, abort_flag,
                     lane)) {
        if (lane == 0) rs_record_error(p.err, abort_flag, kDevErrEpiWait);
        return;
      }
      full_ph ^= 1u << rb;
      tc_fence_after();
      const bool load = any_valid;
      uint32_t v[NV][16];
      if (load) {
#pragma unroll
        for (int h = 0; h < NV; ++h)
          tmem_ld16_nowait(tl + static_cast<uint32_t>((h / 2) * R * 32 + rb * 32 + (h % 2) * 16),
                           v[h]);
#pragma unroll
        for (int h = 0; h < NV; ++h) tmem_wait_ld(v[h]);
#pragma unroll
        for (int h = 0; h < NV; ++h)
          tmem_st16_zero(tl + static_cast<uint32_t>((h / 2) * R * 32 + rb * 32 + (h % 2) * 16));
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.dw_free[rb]);

      const int64_t pix = pix0 + static_cast<int64_t>(r) * p.Wo;
      if constexpr (POOL != 0) {
        // 2x2 max pool: every lane requantises its pixel (the window's
        // other column is lane row ^ 1, its other row the set's previous
        // row), even columns of odd rows store the window's maximum.
        if (valid) {
          const int cls = r == 0 ? cls_top : (r == Ho - 1 ? cls_bot : cls_mid);
          if (cls != p.base_cls) {
            const int off = cls * Cop + cbase;
#pragma unroll
            for (int h = 0; h < NV; ++h)
#pragma unroll
              for (int j = 0; j < 16; ++j)
                v[h][j] += static_cast<uint32_t>(tab.dw_dbias[off + h * 16 + j]);
          }
        }
        const int2* mh = tab.dw_mh + cbase;
        const int2* bs = tab.dw_bs + cbase;
        const bool first = (r & 1) == 0;
        const bool store = !first && valid && (x & 1) == 0;
        int8_t* o = p.out +
                    ((static_cast<int64_t>(n) * (Ho / 2) + (r >> 1)) * (p.Wo / 2) + (x >> 1)) *
                        Cop +
                    cbase;
        static_assert(NV % 2 == 0, "32-byte stores");
        // 32 channels at a time; the set's shared-memory row buffer keeps
        // the first row (each thread rereads only what it wrote).
#pragma unroll
        for (int h = 0; h < NV; h += 2) {
          uint4 wv[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            uint4 a = rs_requant16<DWQ>(v[h + e], mh, bs, (h + e) * 16, p.dw_lo4, p.dw_hi4);
            a.x = __vmaxs4(a.x, __shfl_xor_sync(0xFFFFFFFFu, a.x, 1));
            a.y = __vmaxs4(a.y, __shfl_xor_sync(0xFFFFFFFFu, a.y, 1));
            a.z = __vmaxs4(a.z, __shfl_xor_sync(0xFFFFFFFFu, a.z, 1));
            a.w = __vmaxs4(a.w, __shfl_xor_sync(0xFFFFFFFFu, a.w, 1));
            uint4* keep = reinterpret_cast<uint4*>(atile + (h + e) * 2048);
            if (first) {
              *keep = a;
            } else {
              const uint4 k0 = *keep;
              a.x = __vmaxs4(a.x, k0.x);
              a.y = __vmaxs4(a.y, k0.y);
              a.z = __vmaxs4(a.z, k0.z);
              a.w = __vmaxs4(a.w, k0.w);
            }
            wv[e] = a;
          }
          if (store) st_global_v8(o + 16 * h, wv[0], wv[1]);
        }
      } else {
        if (valid) {
          const int cls = r == 0 ? cls_top : (r == Ho - 1 ? cls_bot : cls_mid);
          if (cls != p.base_cls) {
            const int off = cls * Cop + cbase;
#pragma unroll
            for (int h = 0; h < NV; ++h)
#pragma unroll
              for (int j = 0; j < 16; ++j)
                v[h][j] += static_cast<uint32_t>(tab.dw_dbias[off + h * 16 + j]);
          }
          int8_t* o = p.out + pix * Cop + cbase;
          const int2* mh = tab.dw_mh + cbase;
          const int2* bs = tab.dw_bs + cbase;
          static_assert(NV % 2 == 0, "32-byte stores");
#pragma unroll
          for (int h = 0; h < NV; h += 2)
            st_global_v8(o + 16 * h, rs_requant16<DWQ>(v[h], mh, bs, h * 16, p.dw_lo4, p.dw_hi4),
                         rs_requant16<DWQ>(v[h + 1], mh, bs, h * 16 + 16, p.dw_lo4, p.dw_hi4));
        }
      }
    }
  }
}

template <int CG, int NPW, int S, int NCB, int P, int DWQ, int PWQ, int GI = 0, int POOL = 0>
__global__ void __launch_bounds__(RsShape<CG, NPW, S, NCB, P, GI, POOL>::kThreads, 1)
    k_dwrs_s8(const __grid_constant__ CUtensorMap tmIn, const RsArgs p,
              const __grid_constant__ DwPwTable tab) {
  using Sh = RsShape<CG, NPW, S, NCB, P, GI, POOL>;
  static_assert(Sh::Wt * P == 128, "tile rows");
  constexpr int C = Sh::C;
  constexpr int NS = Sh::NS;
  constexpr int RS = Sh::RS;
  constexpr int R = Sh::R;
  constexpr int NBB = Sh::NBB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int stages = p.stages;
  const int cb = NCB == 1 ? 0 : static_cast<int>(blockIdx.x) % NCB;  // this CTA's channel block
  uint8_t* sBdw = smem;
  uint8_t* sBpw = sBdw + Sh::kBdw;
  uint8_t* sApw = sBpw + NPW * C;             // [slot][set][C/16][128][16]
  uint8_t* sIn = sApw + NS * RS * Sh::kApw;   // [slot][stage][box][group][half][kRegion]
  RsBars* bars = reinterpret_cast<RsBars*>(sIn + NS * stages * Sh::kInRow);
  uint64_t* mma_done = reinterpret_cast<uint64_t*>(bars + NS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + NS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Resident weights: the depthwise weights of each (group, kx) of the
  // channel block as NBB ky blocks (two K-halves of NBB*32 rows x 16 B);
  // the pointwise weights as packed.
  {
    constexpr int nB = CG * (GI > 0 ? GI : 1) * 3 * 2 * NBB * 32;  // 16-byte rows
    for (int i = threadIdx.x; i < nB; i += blockDim.x) {
      int t = i;
      const int rr = t % 32;
      t /= 32;
      const int blk = t % NBB;
      t /= NBB;
      const int h = t % 2;
      t /= 2;
      const int kx = t % 3;
      const int gg = t / 3;
      const int ky = rs_block_ky(S, NBB, blk);
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(
          p.wdw + ((cb * CG + gg) * 9 + ky * 3 + kx) * 1024 + h * 512 + rr * 16));
      *reinterpret_cast<uint4*>(sBdw + (gg * 3 + kx) * Sh::kTap + h * Sh::kHalf +
                                (blk * 32 + rr) * 16) = v;
    }
    if constexpr (NPW > 0) {
      for (int i = threadIdx.x; i < NPW * C / 16; i += blockDim.x)
        reinterpret_cast<uint4*>(sBpw)[i] = __ldg(reinterpret_cast<const uint4*>(p.wpw) + i);
    }
  }
  rs_fence_async_smem();

  if (threadIdx.x == 0) {
    for (int k = 0; k < NS; ++k) {
      RsBars& b = bars[k];
      for (int s = 0; s < stages; ++s) {
        mbar_init(&b.in_full[s], 1);
        mbar_init(&b.in_empty[s], 1);
      }
      for (int j = 0; j < RS * kRsMaxRing; ++j) mbar_init(&b.dw_full[j], 1);
      for (int j = 0; j < kRsMaxRing; ++j) mbar_init(&b.dw_free[j], 4);
      for (int j = 0; j < RS; ++j) {
        mbar_init(&b.apw_full[j], 4);
        mbar_init(&b.pw_full[j], 1);
      }
      mbar_init(&b.pw_empty, 4);
      mbar_init(&mma_done[k], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int Hin = p.Hin;
  const int Ho = p.Ho;

  if (warp < 2) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0 && warp < NS) {
      const int k = warp;
      RsBars& b = bars[k];
      tma_prefetch_desc(&tmIn);
      uint8_t* in_k = sIn + k * stages * Sh::kInRow;
      int first, step;
      rs_strip_range(NCB, k, NS, &first, &step);
      const int c0 = cb * C;
      int s = 0;
      uint32_t ph = 0;
      int64_t issued = 0;
      bool ok = true;
      for (int i = first; ok && i < p.strips; i += step) {
        const RsStrip st = rs_strip<P>(p, i);
        for (int y = 0; y < Hin; ++y) {
          if (!mbar_wait(&b.in_empty[s], ph ^ 1u, abort_flag)) {
            rs_record_error(p.err, abort_flag, kDevErrTmaWait);
            ok = false;
            break;
          }
          uint8_t* a = in_k + s * Sh::kInRow;
          if constexpr (Sh::kSwz) {
            // Per tap kx one box of Wt pixels x P samples, already shifted
            // (column tile tx starts at output pixel 128 tx):
            // stride 1 over [C][W][N][H] (box {32 x groups, Wt, P, 1}),
            // stride 2 over [C][parity][W/2][N][H] (box {32 x groups, 1,
            // Wt, P, 1}: input pixel 2j + kx - pad_l is pair j + ((kx -
            // pad_l) >> 1) of parity (kx - pad_l) & 1).
            mbar_arrive_expect_tx(&b.in_full[s], 3 * Sh::kBoxBytes);
            const int x0 = st.tx * 128;
#pragma unroll
            for (int kx = 0; kx < 3; ++kx) {
              if constexpr (S == 1) {
                tma_load_4d(a + kx * Sh::kBoxStride, &tmIn, &b.in_full[s], c0,
                            x0 + kx - p.pad_l, static_cast<int>(st.n), y);
              } else {
                const int t = kx - p.pad_l;
                tma_load_5d(a + kx * Sh::kBoxStride, &tmIn, &b.in_full[s], c0, t & 1,
                            x0 + (t >> 1), static_cast<int>(st.n), y);
              }
            }
          } else {
            // Full stride-1 rows: one box over [16 ch][W][N][C/16 chunks][H]
            // holding every 16-channel chunk of the strip's input groups.
            mbar_arrive_expect_tx(&b.in_full[s], Sh::kBoxBytes);
            tma_load_5d(a, &tmIn, &b.in_full[s], 0, st.tx * 128 - p.pad_l,
                        static_cast<int>(st.n), c0 / 16, y);
          }
          ++issued;
          if (++s == stages) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok) {
        // Copies already issued land before the kernel exits.
        const int64_t from = issued > stages ? issued - stages : 0;
        for (int64_t gi = from; gi < issued; ++gi)
          mbar_wait(&b.in_full[gi % stages], static_cast<uint32_t>((gi / stages) & 1),
                         nullptr);
      }
    }
  } else if (warp < 4) {
    // -------------------------------------------------------- MMA issuer
    if (lane == 0 && warp - 2 < NS) {
      const int k = warp - 2;
      RsBars& b = bars[k];
      const uint32_t tm_slot = tmem_base + static_cast<uint32_t>(k * Sh::kSlotCols);
      const uint32_t in0 = smem_u32(sIn + k * stages * Sh::kInRow);
      const uint32_t bpw0 = smem_u32(sBpw);
      const uint32_t apw0 = smem_u32(sApw + k * RS * Sh::kApw);
      int first, step;
      rs_strip_range(NCB, k, NS, &first, &step);
      const int pt = p.pad_t;
      int s = 0;
      uint32_t ph = 0;
      uint32_t free_ph = 0;  // bit j: parity of the next wait on dw_free[j]
      uint32_t gbase = 0;    // slot row number of the strip's first output row
      uint32_t gp = 0;       // next row for the pointwise MMAs
      bool ok = true;
      auto pointwise = [&]() -> bool {
        if constexpr (NPW > 0) {
          const uint32_t set = gp % RS;
          if (!mbar_wait(&b.apw_full[set], (gp / RS) & 1u, abort_flag)) return false;
          if (!mbar_wait(&b.pw_empty, (gp & 1u) ^ 1u, abort_flag)) return false;
          tc_fence_after();
          const uint32_t a_t = apw0 + set * static_cast<uint32_t>(Sh::kApw);
          const uint32_t d_t = tm_slot + static_cast<uint32_t>(CG * R * 32);
          const uint32_t idesc_pw = make_idesc_s8(128, NPW);
#pragma unroll
          for (int kc = 0; kc < C / 32; ++kc) {
            const uint64_t ad = make_sdesc(a_t + kc * 2 * 2048, 2048, 128, 0);
            const uint64_t bd = make_sdesc(bpw0 + kc * 2 * (NPW * 16), NPW * 16, 128, 0);
            umma_i8(d_t, ad, bd, idesc_pw, kc > 0 ? 1u : 0u);
          }
          umma_commit(&b.pw_full[set]);
          ++gp;
        }
        return true;
      };
      // Descriptor templates: an operand's descriptor differs from these only
      // in the start-address field (address >> 4, below 2^14 for shared
      // memory), so each MMA adds an offset to one 64-bit value.
      const uint64_t adesc0 = make_sdesc(in0, Sh::kALbo, Sh::kASbo, Sh::kALayout);
      const uint64_t bdesc_smem = make_sdesc(smem_u32(sBdw), Sh::kHalf, 128, 0);
      uint32_t aoff[3];  // A start of tap kx within a stage, group 0 (16-byte units)
#pragma unroll
      for (int kx = 0; kx < 3; ++kx) {
        if constexpr (Sh::kSwz) {
          aoff[kx] = static_cast<uint32_t>((kx * Sh::kBoxStride) / 16);
        } else {
          aoff[kx] = static_cast<uint32_t>(kx);  // a one-pixel (16-byte) move
        }
      }
      // Input group stride in a box (16-byte units).
      constexpr uint32_t kGroupA = Sh::kSwz ? 2u : (2 * Sh::kRegion) / 16;
      const uint32_t idesc1 = make_idesc_s8(128, 32);
      const uint32_t idesc2 = make_idesc_s8(128, 64);
      const uint32_t idesc3 = make_idesc_s8(128, 96);
      const uint64_t bdesc0 = bdesc_smem;
      for (int i = first; ok && i < p.strips; i += step) {
        int pw_next = 0;
        // Output rows [nc, nn) have started and are not complete: exactly the
        // rows the current input row reaches.  first(r) = max(0, S r - pt),
        // last(r) = min(Hin - 1, S r - pt + 2).
        int nn = 0, nc = 0, nn_blk = 0, nc_blk = 0;
        int ym = (pt + 2) % 3;  // (y + pt - 1) mod 3: the ky of row y is 1 - pt
        for (int y = 0; y < Hin; ++y) {
          while (ok && nn < Ho && S * nn - pt <= y) {
            ok = mbar_wait(&b.dw_free[nn_blk], (free_ph >> nn_blk) & 1u, abort_flag);
            free_ph ^= 1u << nn_blk;
            ++nn;
            if (++nn_blk == R) nn_blk = 0;
          }
          if (ok) ok = mbar_wait(&b.in_full[s], ph, abort_flag);
          if (!ok) break;
          tc_fence_after();
          uint32_t live = 0;
          {
            int jb = nc_blk;
            for (int r = nc; r < nn; ++r) {
              live |= 1u << jb;
              if (++jb == R) jb = 0;
            }
          }
          int o;
          if constexpr (S == 1) {
            o = ym == 0 ? 1 : (ym == 1 ? 0 : 2);
          } else {
            // u even: rows u/2 - 1 (ky 2) and u/2 (ky 0); u odd: (u-1)/2 (ky 1).
            const int u = y + pt;
            o = (u & 1) == 0 ? ((((u >> 1) - 1) & 1) == 0 ? 0 : 1) : 3 - (((u - 1) >> 1) & 1);
          }
          const uint64_t astage = adesc0 + static_cast<uint64_t>((s * Sh::kInRow) / 16);
          int j = 0;
          while (j < R) {
            if (((live >> j) & 1u) == 0) {
              ++j;
              continue;
            }
            int j1 = j + 1;
            while (j1 < R && ((live >> j1) & 1u) != 0) ++j1;
            const uint32_t idesc = j1 - j == 1 ? idesc1 : (j1 - j == 2 ? idesc2 : idesc3);
            // Weight window of the run: its first block j holds row
            // nc + (j - nc_blk) mod R, whose tap is ky = y + pt - row.
            int wb = o + j;
            if constexpr (R == 4) wb = 2 - (y + pt - (nc + ((j - nc_blk + R) & 3)));
            const uint64_t bwin = bdesc0 + static_cast<uint64_t>(wb * 32);
            if constexpr (GI == 0) {
#pragma unroll
              for (int gq = 0; gq < CG; ++gq) {
#pragma unroll
                for (int kx = 0; kx < 3; ++kx) {
                  umma_i8(tm_slot + static_cast<uint32_t>(gq * R * 32 + j * 32),
                          astage + gq * kGroupA + aoff[kx],
                          bwin + static_cast<uint64_t>(((gq * 3 + kx) * Sh::kTap) / 16), idesc,
                          1u);
                }
              }
            } else {
              // Dense: output group go sums every input group gi.
#pragma unroll
              for (int go = 0; go < CG; ++go)
#pragma unroll
                for (int gi = 0; gi < GI; ++gi)
#pragma unroll
                  for (int kx = 0; kx < 3; ++kx)
                    umma_i8(tm_slot + static_cast<uint32_t>(go * R * 32 + j * 32),
                            astage + gi * kGroupA + aoff[kx],
                            bwin + static_cast<uint64_t>((((go * GI + gi) * 3 + kx) * Sh::kTap) /
                                                         16),
                            idesc, 1u);
            }
            j = j1;
          }
          umma_commit(&b.in_empty[s]);
          if (++s == stages) {
            s = 0;
            ph ^= 1u;
          }
          // Rows whose last input row this is are complete.
          while (nc < Ho && (S * nc - pt + 2 <= y || y == Hin - 1)) {
            const uint32_t gr = gbase + static_cast<uint32_t>(nc);
            umma_commit(&b.dw_full[((POOL ? gr >> 1 : gr) % RS) * kRsMaxRing + nc_blk]);
            ++nc;
            if (++nc_blk == R) nc_blk = 0;
          }
          if (++ym == 3) ym = 0;
          if constexpr (NPW > 0) {
            while (ok && pw_next <= y - 2) {
              ok = pointwise();
              ++pw_next;
            }
          }
        }
        if constexpr (NPW > 0) {
          while (ok && pw_next < Ho) {
            ok = pointwise();
            ++pw_next;
          }
        }
        gbase += static_cast<uint32_t>(Ho);
      }
      if (!ok) rs_record_error(p.err, abort_flag, kDevErrMmaWait);
      // Every MMA of this thread completes before tensor memory is freed.
      umma_commit(&mma_done[k]);
      mbar_wait(&mma_done[k], 0, nullptr);
    }
  } else {
    // ---------------------------------------------------------- epilogue
    const int ew = warp - 4;
    const int k = ew / (RS * 4);
    const int set = (ew / 4) % RS;
    const int q = warp & 3;
    uint8_t* sA = sApw + k * RS * Sh::kApw;
    const uint32_t tm = tmem_base + static_cast<uint32_t>(k * Sh::kSlotCols);
    // One code path per CTA: its channel block's table offsets are
    // compile-time constants.
    if (cb == 0) {
      rs_epilogue<CG, NPW, S, NCB, P, 0, DWQ, PWQ, GI, POOL>(p, tab, bars[k], sA, tm, k, set, q, lane,
                                                        abort_flag);
    } else if constexpr (NCB >= 2) {
      if (cb == 1) {
        rs_epilogue<CG, NPW, S, NCB, P, 1, DWQ, PWQ, GI, POOL>(p, tab, bars[k], sA, tm, k, set, q,
                                                          lane, abort_flag);
      } else if constexpr (NCB >= 4) {
        if (cb == 2) {
          rs_epilogue<CG, NPW, S, NCB, P, 2, DWQ, PWQ, GI, POOL>(p, tab, bars[k], sA, tm, k, set, q,
                                                            lane, abort_flag);
        } else if (cb == 3) {
          rs_epilogue<CG, NPW, S, NCB, P, 3, DWQ, PWQ, GI, POOL>(p, tab, bars[k], sA, tm, k, set, q,
                                                            lane, abort_flag);
        } else if constexpr (NCB >= 8) {
          if (cb == 4)
            rs_epilogue<CG, NPW, S, NCB, P, 4, DWQ, PWQ, GI, POOL>(p, tab, bars[k], sA, tm, k, set, q,
                                                              lane, abort_flag);
          else if (cb == 5)
            rs_epilogue<CG, NPW, S, NCB, P, 5, DWQ, PWQ, GI, POOL>(p, tab, bars[k], sA, tm, k, set, q,
                                                              lane, abort_flag);
          else if (cb == 6)
            rs_epilogue<CG, NPW, S, NCB, P, 6, DWQ, PWQ, GI, POOL>(p, tab, bars[k], sA, tm, k, set, q,
                                                              lane, abort_flag);
          else
            rs_epilogue<CG, NPW, S, NCB, P, 7, DWQ, PWQ, GI, POOL>(p, tab, bars[k], sA, tm, k, set, q,
                                                              lane, abort_flag);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

template <int CG, int NPW, int S, int NCB, int P, int DWC, int PWC, int GI = 0, int POOL = 0>
cudaError_t rs_launch(const CUtensorMap& m, const RsArgs& a, const DwPwTable& tab, int grid,
                      int smem, cudaStream_t s) {
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if ((done.load() & bit) == 0) {
    const cudaError_t e = cudaFuncSetAttribute(k_dwrs_s8<CG, NPW, S, NCB, P, DWC, PWC, GI, POOL>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               kRsSmemLimit);
    if (e != cudaSuccess) return e;
    done.fetch_or(bit);
  }
  k_dwrs_s8<CG, NPW, S, NCB, P, DWC, PWC, GI, POOL>
      <<<grid, RsShape<CG, NPW, S, NCB, P, GI>::kThreads, smem, s>>>(m, a, tab);
  return cudaGetLastError();
}

// The pointwise epilogue variant (ep_flags of the pointwise op).
template <int CG, int NPW, int S, int NCB, int P, int DWQ, int GI = 0, int POOL = 0>
cudaError_t rs_launch_pw(const CUtensorMap& m, const RsArgs& a, const DwPwTable& tab, int pwq,
                         int grid, int smem, cudaStream_t s) {
  if constexpr (NPW == 0) {
    return rs_launch<CG, NPW, S, NCB, P, DWQ, 0, GI, POOL>(m, a, tab, grid, smem, s);
  } else {
    switch (pwq) {
      case 0: return rs_launch<CG, NPW, S, NCB, P, DWQ, 0>(m, a, tab, grid, smem, s);
      case 1: return rs_launch<CG, NPW, S, NCB, P, DWQ, 1>(m, a, tab, grid, smem, s);
      case 2: return rs_launch<CG, NPW, S, NCB, P, DWQ, 2>(m, a, tab, grid, smem, s);
      default: return rs_launch<CG, NPW, S, NCB, P, DWQ, 3>(m, a, tab, grid, smem, s);
    }
  }
}

// Shared memory of one launch (bytes) and its input stages.
template <int CG, int NPW, int S, int NCB, int P, int GI = 0, int POOL = 0>
bool rs_smem(int* smem, int* stages) {
  using Sh = RsShape<CG, NPW, S, NCB, P, GI, POOL>;
  const int fixed = Sh::kBdw + NPW * Sh::C + Sh::NS * Sh::RS * Sh::kApw;
  const int overhead = 1024 + fixed + Sh::NS * static_cast<int>(sizeof(RsBars)) + 64;
  const int st = std::min(kRsMaxStages, (kRsSmemLimit - overhead) / (Sh::NS * Sh::kInRow));
  if (st < 3) return false;
  *stages = st;
  *smem = std::max(overhead + Sh::NS * st * Sh::kInRow, 120 * 1024);
  return true;
}

template <int CG, int NPW, int S, int NCB, int P, int GI = 0, int POOL = 0>
cudaError_t rs_shape(const CUtensorMap& m, RsArgs a, const DwPwTable& tab, int dwq, int pwq,
                     int num_sms, cudaStream_t s) {
  using Sh = RsShape<CG, NPW, S, NCB, P, GI, POOL>;
  int smem = 0;
  if (!rs_smem<CG, NPW, S, NCB, P, GI, POOL>(&smem, &a.stages)) return cudaErrorInvalidValue;
  // NCB CTAs per group of strips, one per channel block.
  const int per_block = static_cast<int>(std::min<int64_t>(
      (static_cast<int64_t>(a.strips) + Sh::NS - 1) / Sh::NS, std::max(1, num_sms / NCB)));
  const int grid = per_block * NCB;
  if (a.strips <= 0) return cudaSuccess;
  switch (dwq) {
    case 0: return rs_launch_pw<CG, NPW, S, NCB, P, 0, GI, POOL>(m, a, tab, pwq, grid, smem, s);
    case 1: return rs_launch_pw<CG, NPW, S, NCB, P, 1, GI, POOL>(m, a, tab, pwq, grid, smem, s);
    case 2: return rs_launch_pw<CG, NPW, S, NCB, P, 2, GI, POOL>(m, a, tab, pwq, grid, smem, s);
    default: return rs_launch_pw<CG, NPW, S, NCB, P, 3, GI, POOL>(m, a, tab, pwq, grid, smem, s);
  }
}

// Shapes the kernel takes: 3x3 depthwise, stride 1 or 2 (square), at most
// one row/column of top/left padding, 64 or more output pixels per row; C
// in {32, 64} or a multiple of 64 up to 256 (channel blocks), or 512 for
// stride-1 rows of at most 32 pixels (four samples per tile); stride 2
// needs an even input width (the [C][parity][W/2] pixel view).
bool rs_geometry_ok(const pspml_op_desc& d) {
  if (d.kind != PSPML_OP_DEPTHWISE_CONV2D || d.kernel_h != 3 || d.kernel_w != 3 ||
      d.stride_h != d.stride_w || d.in_c != d.out_c)
    return false;
  const int S = d.stride_h;
  if (S != 1 && S != 2) return false;
  if (d.pad_top < 0 || d.pad_top > 1 || d.pad_left < 0 || d.pad_left > 1) return false;
  // The interior output rows share one border class (the epilogue reads the
  // classes of the first, second and last rows only).
  if (d.pad_bottom < 0 || d.pad_bottom > (S == 1 ? 1 : 2)) return false;
  if (S == 2 && (d.in_w % 2 != 0)) return false;
  if (d.out_w < 1 || d.out_w > 65535 || d.out_h > 4096 || d.in_h > 65535) return false;
  const int C = d.in_c;
  if (!(C == 32 || C == 64 || C == 128 || C == 256 || C == 512)) return false;
  // 512 channels (eight blocks) only with four samples per tile: stride 1,
  // rows of at most 32 pixels.
  if (C == 512 && (S != 1 || d.out_w > 32)) return false;
  // Every output row takes at least one input row: S*r - pad_top + 2 >= 0
  // and S*(out_h-1) - pad_top <= in_h - 1.
  if (S * (d.out_h - 1) - d.pad_top > d.in_h - 1) return false;
  return true;
}

// Samples per 128-row tile: 1 for rows of more than 64 pixels, 2 for
// 33..64, 4 for up to 32 (stride 1, C >= 64, depthwise alone).
// Set in the depthwise-shaped descriptor of a dense 32 -> 32 conv
// (launch_dense_rs): its 64-pixel rows pack two samples per tile too.
constexpr int32_t kRsDenseFlag = 1 << 16;

int rs_packing(const pspml_op_desc& d, int npw) {
  if (npw != 0 || d.out_w > 64) return 1;
  if ((d.flags & kRsDenseFlag) != 0) {
    if (d.stride_h != 1) return 1;
    if (d.out_c == 32) return d.out_w > 32 ? 2 : 1;  // 32 -> 32: one or two samples per tile
    return d.out_w > 32 ? 2 : 4;
  }
  if (d.in_c < 64) return 1;
  return d.out_w > 32 ? 2 : 4;
}

// One launch over `batch` samples (strip count below 2^31).
cudaError_t rs_once(const pspml_op_desc& dw, const PreparedOp& pdw, int npw,
                    const uint8_t* wpw_packed, const DwPwTable& tab, int pwq, int32_t pw_min,
                    int32_t pw_max, int64_t batch, const int8_t* in, int8_t* out,
                    unsigned* dev_err, int num_sms, cudaStream_t s, bool pool) {
  const int C = dw.in_c;
  const int S = dw.stride_h;
  // Samples packed per 128-row tile: rows of at most 32 or 64 pixels share
  // a tile.
  const int P = rs_packing(dw, npw);
  RsArgs a{};
  a.tiles_x = (dw.out_w + 127) / 128;
  a.batch = static_cast<int32_t>(batch);
  a.strips = static_cast<int32_t>(P > 1 ? (batch + P - 1) / P : batch * a.tiles_x);
  a.fd_tiles_x = FastDiv(static_cast<uint32_t>(a.tiles_x));
  a.Hin = dw.in_h;
  a.Ho = dw.out_h;
  a.Wo = dw.out_w;
  a.pad_t = dw.pad_top;
  a.pad_l = dw.pad_left;
  a.wdw = reinterpret_cast<const uint8_t*>(pdw.wpack);
  a.wpw = wpw_packed;
  a.out = out;
  a.ycls = pdw.ycls;
  a.xcls = pdw.xcls;
  a.n_xcls = pdw.n_xcls;
  a.base_cls = pdw.base_cls;
  // With an input zero point of 0 the zero fill at the borders is the real
  // zero: every class's bias difference is 0 and the epilogue skips them.
  a.borders = 0;
  for (int i = 0; i < pdw.ncls * C && !a.borders; ++i) a.borders = tab.dw_dbias[i] != 0;
  a.dw_lo4 = splat4(dw.act_min);
  a.dw_hi4 = splat4(dw.act_max);
  a.pw_lo4 = splat4(pw_min);
  a.pw_hi4 = splat4(pw_max);
  a.err = dev_err;
  const int dwq = ep_flags(dw.act_min, dw.act_max, dw.zp_out);

  // Full stride-1 rows: a view whose box holds every 16-channel chunk of a
  // row's input groups (the chunk is a dimension of stride 16 bytes),
  // [16 ch][W][N][C/16][H], box {16, 130, 1, chunks, 1}.  Packed samples and
  // stride 2: one pre-shifted box per tap with rows of 32 x groups channels
  // in the 32- or 64-byte swizzled layout.  chunks = 2 x the input groups of
  // a strip (the depthwise channel block, or every input channel of a dense
  // conv).
  const int gin = (dw.flags & kRsDenseFlag) != 0 ? C / 32 : (C == 32 ? 1 : 2);
  const uint32_t chunks = static_cast<uint32_t>(2 * gin);
  const uint64_t W = static_cast<uint64_t>(dw.in_w), H = static_cast<uint64_t>(dw.in_h);
  const uint64_t Cu = static_cast<uint64_t>(C);
  CUtensorMap m;
  const uint32_t estr[5] = {1, 1, 1, 1, 1};
  if (S == 1 && P > 1) {
    // Packed samples: [C][W][N][H], box {32 x groups, 128/P, P, 1}, 32- or
    // 64-byte swizzle.
    const uint64_t dims[4] = {Cu, W, static_cast<uint64_t>(batch), H};
    const uint64_t strides[3] = {Cu, H * W * Cu, W * Cu};
    const uint32_t box[4] = {16 * chunks, static_cast<uint32_t>(128 / P),
                             static_cast<uint32_t>(P), 1};
    if (encode_tensor_map(&m, in, 4, dims, strides, box, estr,
                          gin == 1 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B) !=
        CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  } else if (S == 2) {
    // Stride 2: [C][parity][W/2][N][H], box {32 x groups, 1, 128/P, P, 1},
    // 32- or 64-byte swizzle.
    const uint64_t dims[5] = {Cu, 2, W / 2, static_cast<uint64_t>(batch), H};
    const uint64_t strides[4] = {Cu, 2 * Cu, H * W * Cu, W * Cu};
    const uint32_t box[5] = {16 * chunks, 1, static_cast<uint32_t>(128 / P),
                             static_cast<uint32_t>(P), 1};
    if (encode_tensor_map(&m, in, 5, dims, strides, box, estr,
                          gin == 1 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B) !=
        CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  } else {
    const uint64_t dims[5] = {16, W, static_cast<uint64_t>(batch), Cu / 16, H};
    const uint64_t strides[4] = {Cu, H * W * Cu, 16, W * Cu};
    const uint32_t box[5] = {16, 130, 1, chunks, 1};
    if (encode_tensor_map(&m, in, 5, dims, strides, box, estr, CU_TENSOR_MAP_SWIZZLE_NONE) !=
        CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  if (pool) {
    // A dense conv with the 2x2 max pool after it in its epilogue.
    if ((dw.flags & kRsDenseFlag) == 0 || S != 1 || npw != 0) return cudaErrorInvalidValue;
    if (dw.out_c == 32 && C == 32) {
      if (P == 1) return rs_shape<1, 0, 1, 1, 1, 0, 1>(m, a, tab, dwq, 0, num_sms, s);
      if (P == 2) return rs_shape<1, 0, 1, 1, 2, 0, 1>(m, a, tab, dwq, 0, num_sms, s);
    } else if (dw.out_c == 64 && C == 32) {
      if (P == 1) return rs_shape<2, 0, 1, 1, 1, 1, 1>(m, a, tab, dwq, 0, num_sms, s);
      if (P == 2) return rs_shape<2, 0, 1, 1, 2, 1, 1>(m, a, tab, dwq, 0, num_sms, s);
      return rs_shape<2, 0, 1, 1, 4, 1, 1>(m, a, tab, dwq, 0, num_sms, s);
    } else if (dw.out_c == 64 && C == 64) {
      if (P == 1) return rs_shape<2, 0, 1, 1, 1, 2, 1>(m, a, tab, dwq, 0, num_sms, s);
      if (P == 2) return rs_shape<2, 0, 1, 1, 2, 2, 1>(m, a, tab, dwq, 0, num_sms, s);
      return rs_shape<2, 0, 1, 1, 4, 2, 1>(m, a, tab, dwq, 0, num_sms, s);
    }
    return cudaErrorInvalidValue;
  }
  if ((dw.flags & kRsDenseFlag) != 0 && dw.out_c != 32) {
    // Dense 32 -> 64 (one input group) and 64 -> 64 (two), stride 1.
    if (S != 1 || dw.out_c != 64 || npw != 0) return cudaErrorInvalidValue;
    if (C == 32) {
      if (P == 1) return rs_shape<2, 0, 1, 1, 1, 1>(m, a, tab, dwq, 0, num_sms, s);
      if (P == 2) return rs_shape<2, 0, 1, 1, 2, 1>(m, a, tab, dwq, 0, num_sms, s);
      return rs_shape<2, 0, 1, 1, 4, 1>(m, a, tab, dwq, 0, num_sms, s);
    }
    if (C == 64) {
      if (P == 1) return rs_shape<2, 0, 1, 1, 1, 2>(m, a, tab, dwq, 0, num_sms, s);
      if (P == 2) return rs_shape<2, 0, 1, 1, 2, 2>(m, a, tab, dwq, 0, num_sms, s);
      return rs_shape<2, 0, 1, 1, 4, 2>(m, a, tab, dwq, 0, num_sms, s);
    }
    return cudaErrorInvalidValue;
  }
  if (npw == 64 && C == 64 && S == 1 && P == 1)
    return rs_shape<2, 64, 1, 1, 1>(m, a, tab, dwq, pwq, num_sms, s);
  if (npw != 0) return cudaErrorInvalidValue;
  if (P == 1) {
    if (S == 1) {
      if (C == 32) return rs_shape<1, 0, 1, 1, 1>(m, a, tab, dwq, 0, num_sms, s);
      if (C == 64) return rs_shape<2, 0, 1, 1, 1>(m, a, tab, dwq, 0, num_sms, s);
      if (C == 128) return rs_shape<2, 0, 1, 2, 1>(m, a, tab, dwq, 0, num_sms, s);
      if (C == 256) return rs_shape<2, 0, 1, 4, 1>(m, a, tab, dwq, 0, num_sms, s);
    } else {
      if (C == 32) return rs_shape<1, 0, 2, 1, 1>(m, a, tab, dwq, 0, num_sms, s);
      if (C == 64) return rs_shape<2, 0, 2, 1, 1>(m, a, tab, dwq, 0, num_sms, s);
      if (C == 128) return rs_shape<2, 0, 2, 2, 1>(m, a, tab, dwq, 0, num_sms, s);
      if (C == 256) return rs_shape<2, 0, 2, 4, 1>(m, a, tab, dwq, 0, num_sms, s);
    }
  } else if (S == 2) {
    if (P == 2) {
      if (C == 64) return rs_shape<2, 0, 2, 1, 2>(m, a, tab, dwq, 0, num_sms, s);
      if (C == 128) return rs_shape<2, 0, 2, 2, 2>(m, a, tab, dwq, 0, num_sms, s);
      if (C == 256) return rs_shape<2, 0, 2, 4, 2>(m, a, tab, dwq, 0, num_sms, s);
    } else {
      if (C == 64) return rs_shape<2, 0, 2, 1, 4>(m, a, tab, dwq, 0, num_sms, s);
      if (C == 128) return rs_shape<2, 0, 2, 2, 4>(m, a, tab, dwq, 0, num_sms, s);
      if (C == 256) return rs_shape<2, 0, 2, 4, 4>(m, a, tab, dwq, 0, num_sms, s);
    }
  } else if (S == 1) {
    if (P == 2) {
      if (C == 32) return rs_shape<1, 0, 1, 1, 2>(m, a, tab, dwq, 0, num_sms, s);
      if (C == 64) return rs_shape<2, 0, 1, 1, 2>(m, a, tab, dwq, 0, num_sms, s);
      if (C == 128) return rs_shape<2, 0, 1, 2, 2>(m, a, tab, dwq, 0, num_sms, s);
      if (C == 256) return rs_shape<2, 0, 1, 4, 2>(m, a, tab, dwq, 0, num_sms, s);
    } else {
      if (C == 64) return rs_shape<2, 0, 1, 1, 4>(m, a, tab, dwq, 0, num_sms, s);
      if (C == 128) return rs_shape<2, 0, 1, 2, 4>(m, a, tab, dwq, 0, num_sms, s);
      if (C == 256) return rs_shape<2, 0, 1, 4, 4>(m, a, tab, dwq, 0, num_sms, s);
      if (C == 512) return rs_shape<2, 0, 1, 8, 4>(m, a, tab, dwq, 0, num_sms, s);
    }
  }
  return cudaErrorInvalidValue;
}

cudaError_t rs_run(const pspml_op_desc& dw, const PreparedOp& pdw, int npw,
                   const uint8_t* wpw_packed, const DwPwTable& tab, int pwq, int32_t pw_min,
                   int32_t pw_max, int64_t out_per, int64_t batch, const int8_t* in, int8_t* out,
                   unsigned* dev_err, int num_sms, cudaStream_t s, bool pool = false) {
  const int64_t per_sample = static_cast<int64_t>((dw.out_w + 127) / 128);
  // Whole packed groups per launch.
  const int64_t chunk = std::max<int64_t>(4, ((1ll << 31) - 1) / per_sample) / 4 * 4;
  const int64_t in_per = static_cast<int64_t>(dw.in_h) * dw.in_w * dw.in_c;
  for (int64_t b0 = 0; b0 < batch; b0 += chunk) {
    const cudaError_t e =
        rs_once(dw, pdw, npw, wpw_packed, tab, pwq, pw_min, pw_max, std::min(chunk, batch - b0),
                in + b0 * in_per, out + b0 * out_per, dev_err, num_sms, s, pool);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace

// Rows of 65..127 pixels leave tile lanes idle; narrower rows pack several
// samples per tile (C >= 64, stride 1 or 2).  (Packed stride-2 rows had
// measured slower than the CUDA-core kernel while their boxes had 16-byte
// rows; with 64-byte swizzled rows they take config 3's blocks 4 and 6 at
// 0.90-0.94 of HBM.)
bool dwrs_dw_supported(const pspml_op_desc& d) {
  if (!rs_geometry_ok(d)) return false;
  if (d.out_w >= 128) return true;
  return d.out_w <= 64 && d.in_c >= 64;
}

// The 32-channel pair measured faster on the tile-per-row kernel
// (dwpw_tc.cu, 141 against 164 ms per config-4 step, and 129 against 150
// with the later epilogues): with half the
// depthwise channels a row carries less work and this kernel's per-row
// chain (MMA, commit, block release) sets the pace, while that kernel
// keeps four independent tiles in flight.
bool dwrs_pair_supported(const pspml_op_desc& dw, const pspml_op_desc& pw) {
  return rs_geometry_ok(dw) && dw.stride_h == 1 && dw.out_w >= 128 && pw.out_c == 64 &&
         dw.in_c == 64;
}

cudaError_t launch_dwrs_dw(const pspml_op_desc& d, const PreparedOp& p, int64_t batch,
                           const int8_t* in, int8_t* out, unsigned* dev_err, int num_sms,
                           cudaStream_t s) {
  const int C = d.in_c;
  if (p.table == nullptr || !p.all_fast_known || p.ncls > 9 || C > kDwTabC)
    return cudaErrorInvalidValue;
  static thread_local DwPwTable tab;
  std::memset(&tab, 0, sizeof(tab));
  for (int c = 0; c < C; ++c) {
    tab.dw_mh[c] = p.table->mh[c];
    tab.dw_bs[c] = p.table->bs[c];
  }
  for (int k = 0; k < p.ncls; ++k)
    for (int c = 0; c < C; ++c) tab.dw_dbias[k * C + c] = p.table->dbias[k * C + c];
  const int64_t out_per = static_cast<int64_t>(d.out_h) * d.out_w * d.out_c;
  return rs_run(d, p, 0, nullptr, tab, 0, -128, 127, out_per, batch, in, out, dev_err,
                num_sms, s);
}

cudaError_t launch_dwrs_pair(const pspml_op_desc& dw, const PreparedOp& pdw,
                             const pspml_op_desc& pw, const uint8_t* wpw_packed,
                             const DwPwTable& tab, int64_t batch, const int8_t* in, int8_t* out,
                             unsigned* dev_err, int num_sms, cudaStream_t s) {
  const int pwq = ep_flags(pw.act_min, pw.act_max, pw.zp_out);
  const int64_t out_per = static_cast<int64_t>(pw.out_h) * pw.out_w * pw.out_c;
  return rs_run(dw, pdw, pw.out_c, wpw_packed, tab, pwq, pw.act_min, pw.act_max, out_per, batch,
                in, out, dev_err, num_sms, s);
}

// ---- dense 3x3 conv on the row-streaming kernel
// A 3x3 stride-1 conv with 32 or 64 input and output channels is the
// depthwise kernel with full 32x32 weight blocks in place of the
// block-diagonal ones: per input row, tap kx and (output group, input
// group) one MMA (K = 32 input channels, N = the group's 32 output
// channels of each output row the input row feeds) accumulates every
// (ky, kx) tap, and every input row crosses into shared memory once (the
// implicit-GEMM conv loads each input pixel once per filter tap).  The
// border-class folded biases are the conv's own (every class sums over the
// input channels of its in-image taps).

// [Co/32 x Ci/32 blocks (output group major)][9 taps][2 K-halves]
// [32 output channels][16 input-channel bytes]: the layout of the depthwise
// packing with dense blocks.
__global__ void k_pack_conv_rs(const int8_t* __restrict__ f, int32_t ci, int32_t co,
                               uint8_t* __restrict__ out) {
  const int i = static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x);
  const int gi_n = ci / 32;
  if (i >= (co / 32) * gi_n * 9 * 1024) return;
  const int blk = i / (9 * 1024);
  const int go = blk / gi_n, gi = blk % gi_n;
  const int r = i % (9 * 1024);
  const int tap = r / 1024;
  const int half = (r % 1024) / 512;
  const int row = (r % 512) / 16;
  const int j = r % 16;
  out[i] = static_cast<uint8_t>(f[((go * 32 + row) * 9 + tap) * ci + gi * 32 + half * 16 + j]);
}

namespace {
pspml_op_desc dense_as_depthwise(const pspml_op_desc& conv) {
  pspml_op_desc dw = conv;
  dw.kind = PSPML_OP_DEPTHWISE_CONV2D;
  dw.flags |= kRsDenseFlag;
  return dw;
}
}  // namespace

bool dense_rs_supported(const pspml_op_desc& conv, const PreparedOp& p) {
  if (conv.kind != PSPML_OP_CONV2D || conv.kernel_h != 3 || conv.kernel_w != 3 ||
      conv.stride_h != 1 || conv.stride_w != 1)
    return false;
  const bool shape = (conv.in_c == 32 && (conv.out_c == 32 || conv.out_c == 64)) ||
                     (conv.in_c == 64 && conv.out_c == 64);
  if (!shape) return false;
  if (p.path != OpPath::kTc4d || p.table == nullptr || !p.all_fast_known || p.ncls > 9)
    return false;
  pspml_op_desc g = dense_as_depthwise(conv);
  g.in_c = g.out_c;  // the geometry check of the depthwise shapes
  return rs_geometry_ok(g);
}

size_t conv_rs_packed_bytes(const pspml_op_desc& conv) {
  return static_cast<size_t>(conv.out_c / 32) * (conv.in_c / 32) * 9 * 1024;
}

cudaError_t pack_conv_rs(const pspml_op_desc& conv, const int8_t* filter, uint8_t* out,
                         cudaStream_t s) {
  const int total = static_cast<int>(conv_rs_packed_bytes(conv));
  k_pack_conv_rs<<<(total + 255) / 256, 256, 0, s>>>(filter, conv.in_c, conv.out_c, out);
  return cudaGetLastError();
}

cudaError_t launch_dense_rs(const pspml_op_desc& conv, const PreparedOp& p,
                            const uint8_t* wpack, int64_t batch, const int8_t* in, int8_t* out,
                            unsigned* dev_err, int num_sms, cudaStream_t s, bool pool) {
  const int N = conv.out_c;
  if (p.table == nullptr || !p.all_fast_known || p.ncls > 9 || N > kDwTabC)
    return cudaErrorInvalidValue;
  static thread_local DwPwTable tab;
  std::memset(&tab, 0, sizeof(tab));
  for (int c = 0; c < N; ++c) {
    tab.dw_mh[c] = p.table->mh[c];
    tab.dw_bs[c] = p.table->bs[c];
  }
  for (int k = 0; k < p.ncls; ++k)
    for (int c = 0; c < N; ++c) tab.dw_dbias[k * N + c] = p.table->dbias[k * N + c];
  PreparedOp q = p;
  q.wpack = reinterpret_cast<const uint32_t*>(wpack);
  if (pool && (conv.out_h % 2 != 0 || conv.out_w % 2 != 0)) return cudaErrorInvalidValue;
  const int64_t out_per = pool ? static_cast<int64_t>(conv.out_h / 2) * (conv.out_w / 2) * N
                               : static_cast<int64_t>(conv.out_h) * conv.out_w * N;
  return rs_run(dense_as_depthwise(conv), q, 0, nullptr, tab, 0, -128, 127, out_per, batch, in,
                out, dev_err, num_sms, s, pool);
}

}  // namespace pspml
