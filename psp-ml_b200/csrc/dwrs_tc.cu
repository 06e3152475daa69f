// dwrs_tc.cu - int8 depthwise 3x3 stride-1 conv streamed by rows on the
// tensor cores, alone or fused with the 1x1 conv after it.
//
// Block-diagonal weights turn the depthwise conv of a 32-channel group
// into GEMMs (see dw_tc.cu).  This kernel makes every input row a single
// A operand: input row y feeds output rows y-1, y and y+1 through the
// vertical taps ky = 2, 1, 0, so one MMA with N = 96 (three 32-column
// blocks of block-diagonal weights, one per ky) updates all three output
// rows at once.  Per input row and group that is 3 MMAs (one per
// horizontal tap kx; the tap shift is a 16-byte move of the A descriptor
// start in the no-swizzle layout) instead of 9 per output row, and every
// input row is loaded once instead of three times.
//
// Tensor memory: per group, a ring of three 32-column accumulator blocks;
// output row r lives in block r % 3.  Which weight block meets which
// accumulator block rotates with y % 3: the kernel keeps the weights of each
// kx as five ky blocks [2 1 0 2 1] and takes the three-block window that
// starts at block (1, 0, 2)[y % 3].  A block must hold zeros before its row
// takes its first contribution, so the epilogue zeroes it right after
// reading the finished row, before the requantisation arithmetic; every MMA
// accumulates.  The first and last input rows of a strip skip the output
// rows outside the image (a narrower N).
//
// Work unit: a strip = one sample x one 128-pixel column tile x all rows.
// Two slots run independent strips so that one slot's MMAs overlap the
// other's epilogue.  Per slot: one TMA thread (input rows, 16-channel boxes
// of 130 pixels, zero filled outside the image), one MMA thread and two
// epilogue sets of four warps (one per tensor-memory lane quarter) that
// take the slot's rows in turn.  Every epilogue warp handles all channels
// of its 32 pixels, so all of them run one code path: with a path per
// channel range the unrolled requantisation code of four paths interleaved
// on each scheduler and instruction fetch stalled.
//
// Fused pointwise: the epilogue writes the requantised depthwise row into a
// shared-memory A tile [C/16][128][16 B]; the MMA thread runs C/32 MMAs
// (M=128, N=NPW, K=32) against the resident 1x1 weights into a pointwise
// accumulator; the epilogue requantises that and stores NHWC.  The
// depthwise output never reaches global memory.
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

constexpr int kRsRegion = 2176;           // one input row of 16 channels: 130 px x 16 B, padded
constexpr int kRsHalf = 5 * 32 * 16;      // one K-half of a five-block weight column (2560 B)
constexpr int kRsTap = 2 * kRsHalf;       // weights of one (group, kx)
constexpr int kRsSmemLimit = 232448;
constexpr int kRsMaxStages = 8;
constexpr int kRsMaxSets = 4;

struct RsArgs {
  int32_t strips;  // batch * tiles_x
  int32_t tiles_x, H, W;
  int32_t pad_l;
  FastDiv fd_tiles_x;
  const uint8_t* wdw;  // [C/32][9][2][32][16] (dw_tc packing)
  const uint8_t* wpw;  // [C/16][NPW][16] (pointwise, K-major core matrices)
  int8_t* out;         // [B][H][W][out channels]
  const uint8_t* ycls;
  const uint8_t* xcls;
  int32_t n_xcls, base_cls;
  uint32_t dw_lo4, dw_hi4, pw_lo4, pw_hi4;
  unsigned* err;
  int32_t stages;
};

// Barriers of one slot.  Rows are numbered per slot across its strips; row
// g belongs to epilogue set g % RS and lives in accumulator block r % 3 (r:
// row within the image).  Every barrier that a set waits on completes only
// for that set's rows, in order, and its next completion needs the set's
// previous one consumed, so no parity wait can fall two phases behind.
struct RsBars {
  uint64_t in_full[kRsMaxStages];
  uint64_t in_empty[kRsMaxStages];
  uint64_t dw_full[kRsMaxSets * 3];  // MMA -> set: row complete, [set][block]
  uint64_t dw_free[3];               // set -> MMA: block read and zeroed
  uint64_t apw_full[kRsMaxSets];     // set -> MMA: its pointwise A tile written
  uint64_t pw_full[kRsMaxSets];      // MMA -> set: its row's pointwise accumulator complete
  uint64_t pw_empty;                 // set -> MMA: pointwise accumulator read
};

// CG: 32-channel groups (C = 32 CG); NPW: pointwise outputs (0: depthwise
// only); NS: slots (independent strips); RS: epilogue sets per slot (four
// warps each, one per tensor-memory lane quarter, taking rows in turn).
template <int CG, int NPW, int NS, int RS>
struct RsShape {
  static constexpr int C = CG * 32;
  static constexpr int kInRow = CG * 2 * kRsRegion;
  static constexpr int kBdw = CG * 3 * kRsTap;
  static constexpr int kBpw = NPW * C;
  static constexpr int kApw = NPW > 0 ? 128 * C : 0;
  static constexpr int kFixed = kBdw + kBpw + NS * RS * kApw;
  static constexpr int kSlotCols = 512 / NS;
  static constexpr int kThreads = 128 + NS * RS * 128;
  static_assert(CG * 96 + NPW <= kSlotCols, "tensor memory per slot");
  static_assert(NS == 1 || NS == 2, "slots");
  static_assert(RS == 2 || RS == 4, "epilogue sets");
  static_assert(RS <= kRsMaxSets, "epilogue sets");
};

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
  if (lane == 0) ok = mbar_wait_poll(bar, parity, abort_flag) ? 1 : 0;
  return __shfl_sync(0xFFFFFFFFu, ok, 0) != 0;
}

template <bool CLAMP>
__device__ __forceinline__ uint4 rs_requant16(const uint32_t* v, const int2* mh, const int2* bs,
                                              int ch, uint32_t lo4, uint32_t hi4) {
  uint32_t packed[4];
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    int32_t r[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = ch + 4 * g + k;
      const int2 b = bs[c];
      r[k] = rq_tab(static_cast<int32_t>(v[4 * g + k]) + b.x, mh[c], b.y);
    }
    uint32_t w = pack_sat4(r[0], r[1], r[2], r[3]);
    if constexpr (CLAMP) w = clamp4(w, lo4, hi4);
    packed[g] = w;
  }
  return make_uint4(packed[0], packed[1], packed[2], packed[3]);
}

// Epilogue of one warp: set `set` of slot `k`, lane quarter q, every
// channel.  All epilogue warps of a kernel run this one code path.
template <int CG, int NPW, int NS, int RS, bool DWCLAMP, bool PWCLAMP>
__device__ __forceinline__ void rs_epilogue(const RsArgs& p, const DwPwTable& tab, RsBars& bars,
                                            uint8_t* sA, uint32_t tm_slot, int k, int set, int q,
                                            int lane, volatile int* abort_flag) {
  using S = RsShape<CG, NPW, NS, RS>;
  constexpr int C = S::C;
  constexpr int NV = C / 16;
  constexpr int NP = NPW / 16;
  const int row = q * 32 + lane;
  const uint32_t tl = tm_slot + (static_cast<uint32_t>(q * 32) << 16);

  // The accumulator blocks start zeroed (set 0 covers every lane).
  if (set == 0) {
#pragma unroll
    for (int g = 0; g < CG; ++g)
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        tmem_st16_zero(tl + g * 96 + j * 32);
        tmem_st16_zero(tl + g * 96 + j * 32 + 16);
      }
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0)
#pragma unroll
      for (int j = 0; j < 3; ++j) mbar_arrive(&bars.dw_free[j]);
  }

  uint32_t full_ph = 0;  // bit j: parity of the next wait on dw_full[set][j]
  uint32_t pw_ph = 0;
  uint8_t* atile = sA + set * S::kApw + row * 16;
  const int first = static_cast<int>(blockIdx.x) + k * static_cast<int>(gridDim.x);
  const int step = NS * static_cast<int>(gridDim.x);
  const int H = p.H;
  uint32_t g = 0;  // row number within the slot
  for (int i = first; i < p.strips; i += step) {
    const uint32_t n = p.fd_tiles_x.div(static_cast<uint32_t>(i));
    const int tx = i - static_cast<int>(n) * p.tiles_x;
    const int x = tx * 128 + row;
    const bool valid = x < p.W;
    // Border classes: rows 0 and H-1 and the interior rows (SAME 3x3).
    int cls_top = 0, cls_mid = 0, cls_bot = 0;
    if (valid) {
      const int xc = p.xcls[x];
      cls_top = p.ycls[0] * p.n_xcls + xc;
      cls_mid = p.ycls[H > 1 ? 1 : 0] * p.n_xcls + xc;
      cls_bot = p.ycls[H - 1] * p.n_xcls + xc;
    }
    const int64_t pix0 = (static_cast<int64_t>(n) * H) * p.W + x;
    for (int r = 0; r < H; ++r, ++g) {
      if (static_cast<int>(g % RS) != set) continue;
      const int rb = r % 3;
      if (!warp_wait(&bars.dw_full[set * 3 + rb], (full_ph >> rb) & 1u, abort_flag, lane)) {
        if (lane == 0) rs_record_error(p.err, abort_flag, kDevErrEpiWait);
        return;
      }
      full_ph ^= 1u << rb;
      tc_fence_after();
      uint32_t v[NV][16];
#pragma unroll
      for (int h = 0; h < NV; ++h)
        tmem_ld16_nowait(tl + static_cast<uint32_t>((h / 2) * 96 + rb * 32 + (h % 2) * 16), v[h]);
#pragma unroll
      for (int h = 0; h < NV; ++h) tmem_wait_ld(v[h]);
#pragma unroll
      for (int h = 0; h < NV; ++h)
        tmem_st16_zero(tl + static_cast<uint32_t>((h / 2) * 96 + rb * 32 + (h % 2) * 16));
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.dw_free[rb]);

      const int cls = r == 0 ? cls_top : (r == H - 1 ? cls_bot : cls_mid);
      if (valid && cls != p.base_cls) {
        const int off = cls * C;
#pragma unroll
        for (int h = 0; h < NV; ++h)
#pragma unroll
          for (int j = 0; j < 16; ++j)
            v[h][j] += static_cast<uint32_t>(tab.dw_dbias[off + h * 16 + j]);
      }
      const int64_t pix = pix0 + static_cast<int64_t>(r) * p.W;
      if constexpr (NPW > 0) {
#pragma unroll
        for (int h = 0; h < NV; ++h)
          *reinterpret_cast<uint4*>(atile + h * 2048) =
              rs_requant16<DWCLAMP>(v[h], tab.dw_mh, tab.dw_bs, h * 16, p.dw_lo4, p.dw_hi4);
        rs_fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars.apw_full[set]);
        // This row's pointwise accumulator.
        if (!warp_wait(&bars.pw_full[set], pw_ph, abort_flag, lane)) {
          if (lane == 0) rs_record_error(p.err, abort_flag, kDevErrEpiWait);
          return;
        }
        pw_ph ^= 1u;
        tc_fence_after();
        uint32_t u[NP][16];
        const uint32_t tp = tl + static_cast<uint32_t>(CG * 96);
#pragma unroll
        for (int h = 0; h < NP; ++h) tmem_ld16_nowait(tp + h * 16, u[h]);
#pragma unroll
        for (int h = 0; h < NP; ++h) tmem_wait_ld(u[h]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars.pw_empty);
        if (valid) {
          int8_t* o = p.out + pix * NPW;
#pragma unroll
          for (int h = 0; h < NP; ++h)
            reinterpret_cast<uint4*>(o)[h] =
                rs_requant16<PWCLAMP>(u[h], tab.pw_mh, tab.pw_bs, h * 16, p.pw_lo4, p.pw_hi4);
        }
      } else {
        if (valid) {
          int8_t* o = p.out + pix * C;
#pragma unroll
          for (int h = 0; h < NV; ++h)
            reinterpret_cast<uint4*>(o)[h] =
                rs_requant16<DWCLAMP>(v[h], tab.dw_mh, tab.dw_bs, h * 16, p.dw_lo4, p.dw_hi4);
        }
      }
    }
  }
}

template <int CG, int NPW, int NS, int RS, bool DWCLAMP, bool PWCLAMP>
__global__ void __launch_bounds__(RsShape<CG, NPW, NS, RS>::kThreads, 1)
    k_dwrs_s8(const __grid_constant__ CUtensorMap tmIn, const RsArgs p,
              const __grid_constant__ DwPwTable tab) {
  using S = RsShape<CG, NPW, NS, RS>;
  constexpr int C = S::C;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int stages = p.stages;
  uint8_t* sBdw = smem;
  uint8_t* sBpw = sBdw + S::kBdw;
  uint8_t* sApw = sBpw + S::kBpw;           // [slot][set][C/16][128][16]
  uint8_t* sIn = sApw + NS * RS * S::kApw;  // [slot][stage][CG*2][kRsRegion]
  RsBars* bars = reinterpret_cast<RsBars*>(sIn + NS * stages * S::kInRow);
  uint64_t* mma_done = reinterpret_cast<uint64_t*>(bars + NS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + NS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Resident weights: the depthwise weights of each (group, kx) as five ky
  // blocks [2 1 0 2 1] (two K-halves of 160 rows x 16 B); the pointwise
  // weights as packed.
  {
    constexpr int nB = CG * 3 * 2 * 5 * 32;  // 16-byte rows
    for (int i = threadIdx.x; i < nB; i += blockDim.x) {
      int t = i;
      const int rr = t % 32;
      t /= 32;
      const int blk = t % 5;
      t /= 5;
      const int h = t % 2;
      t /= 2;
      const int kx = t % 3;
      const int g = t / 3;
      const int ky = blk == 2 ? 0 : ((blk == 1 || blk == 4) ? 1 : 2);
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(
          p.wdw + (g * 9 + ky * 3 + kx) * 1024 + h * 512 + rr * 16));
      *reinterpret_cast<uint4*>(sBdw + (g * 3 + kx) * kRsTap + h * kRsHalf + (blk * 32 + rr) * 16) =
          v;
    }
    if constexpr (NPW > 0) {
      for (int i = threadIdx.x; i < S::kBpw / 16; i += blockDim.x)
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
      for (int j = 0; j < RS * 3; ++j) mbar_init(&b.dw_full[j], 1);
      for (int j = 0; j < 3; ++j) mbar_init(&b.dw_free[j], 4);
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
  const int H = p.H;

  if (warp < 2) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0 && warp < NS) {
      const int k = warp;
      RsBars& b = bars[k];
      tma_prefetch_desc(&tmIn);
      uint8_t* in_k = sIn + k * stages * S::kInRow;
      const int first = static_cast<int>(blockIdx.x) + k * static_cast<int>(gridDim.x);
      const int step = NS * static_cast<int>(gridDim.x);
      int s = 0;
      uint32_t ph = 0;
      int64_t issued = 0;
      bool ok = true;
      for (int i = first; ok && i < p.strips; i += step) {
        const uint32_t n = p.fd_tiles_x.div(static_cast<uint32_t>(i));
        const int tx = i - static_cast<int>(n) * p.tiles_x;
        const int x0 = tx * 128 - p.pad_l;
        for (int y = 0; y < H; ++y) {
          if (!mbar_wait_poll(&b.in_empty[s], ph ^ 1u, abort_flag)) {
            rs_record_error(p.err, abort_flag, kDevErrTmaWait);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&b.in_full[s], CG * 2 * 16 * 130);
          uint8_t* a = in_k + s * S::kInRow;
#pragma unroll
          for (int g = 0; g < CG; ++g)
#pragma unroll
            for (int h = 0; h < 2; ++h)
              tma_load_4d(a + (g * 2 + h) * kRsRegion, &tmIn, &b.in_full[s], g * 32 + h * 16, x0,
                          y, static_cast<int>(n));
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
        for (int64_t g = from; g < issued; ++g)
          mbar_wait_poll(&b.in_full[g % stages], static_cast<uint32_t>((g / stages) & 1), nullptr);
      }
    }
  } else if (warp < 4) {
    // -------------------------------------------------------- MMA issuer
    if (lane == 0 && warp - 2 < NS) {
      const int k = warp - 2;
      RsBars& b = bars[k];
      const uint32_t tm_slot = tmem_base + static_cast<uint32_t>(k * S::kSlotCols);
      const uint32_t in0 = smem_u32(sIn + k * stages * S::kInRow);
      const uint32_t bdw0 = smem_u32(sBdw);
      const uint32_t bpw0 = smem_u32(sBpw);
      const uint32_t apw0 = smem_u32(sApw + k * RS * S::kApw);
      const int first = static_cast<int>(blockIdx.x) + k * static_cast<int>(gridDim.x);
      const int step = NS * static_cast<int>(gridDim.x);
      int s = 0;
      uint32_t ph = 0;
      uint32_t free_ph = 0;  // bit j: parity of the next wait on dw_free[j]
      uint32_t gbase = 0;    // slot row number of the strip's first row
      uint32_t gp = 0;       // next row for the pointwise MMAs
      bool ok = true;
      auto need = [&](int r) -> bool {
        const int j = r % 3;
        const bool o = mbar_wait_poll(&b.dw_free[j], (free_ph >> j) & 1u, abort_flag);
        free_ph ^= 1u << j;
        return o;
      };
      auto pointwise = [&]() -> bool {
        if constexpr (NPW > 0) {
          const uint32_t set = gp % RS;
          if (!mbar_wait_poll(&b.apw_full[set], (gp / RS) & 1u, abort_flag)) return false;
          if (!mbar_wait_poll(&b.pw_empty, (gp & 1u) ^ 1u, abort_flag)) return false;
          tc_fence_after();
          const uint32_t a_t = apw0 + set * static_cast<uint32_t>(S::kApw);
          const uint32_t d_t = tm_slot + static_cast<uint32_t>(CG * 96);
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
      for (int i = first; ok && i < p.strips; i += step) {
        int pw_next = 0;
        for (int y = 0; y < H; ++y) {
          if (y == 0) {
            ok = need(0) && (H < 2 || need(1));
          } else if (y + 1 < H) {
            ok = need(y + 1);
          }
          if (ok) ok = mbar_wait_poll(&b.in_full[s], ph, abort_flag);
          if (!ok) break;
          tc_fence_after();
          // Block j holds the output row of y-1 .. y+1 that is j mod 3; bit j
          // of `live` says that row is inside the image.
          uint32_t live = 0;
#pragma unroll
          for (int j = 0; j < 3; ++j) {
            const int rj = y - 1 + (((j - y + 1) % 3) + 3) % 3;
            if (rj >= 0 && rj < H) live |= 1u << j;
          }
          const int ym = y % 3;
          const int o = ym == 0 ? 1 : (ym == 1 ? 0 : 2);
          const uint32_t a_row = in0 + static_cast<uint32_t>(s * S::kInRow);
          int j = 0;
          while (j < 3) {
            if (((live >> j) & 1u) == 0) {
              ++j;
              continue;
            }
            int j1 = j + 1;
            while (j1 < 3 && ((live >> j1) & 1u) != 0) ++j1;
            const uint32_t idesc = make_idesc_s8(128, 32 * (j1 - j));
#pragma unroll
            for (int g = 0; g < CG; ++g) {
#pragma unroll
              for (int kx = 0; kx < 3; ++kx) {
                const uint64_t ad =
                    make_sdesc(a_row + (g * 2) * kRsRegion + kx * 16, kRsRegion, 128, 0);
                const uint64_t bd =
                    make_sdesc(bdw0 + (g * 3 + kx) * kRsTap + (o + j) * 512, kRsHalf, 128, 0);
                umma_i8(tm_slot + static_cast<uint32_t>(g * 96 + j * 32), ad, bd, idesc, 1u);
              }
            }
            j = j1;
          }
          umma_commit(&b.in_empty[s]);
          if (++s == stages) {
            s = 0;
            ph ^= 1u;
          }
          // Row y-1 is complete after input row y; the last input row also
          // completes its own row.
          if (y >= 1) {
            const uint32_t gr = gbase + static_cast<uint32_t>(y - 1);
            umma_commit(&b.dw_full[(gr % RS) * 3 + (y - 1) % 3]);
          }
          if (y == H - 1) {
            const uint32_t gr = gbase + static_cast<uint32_t>(y);
            umma_commit(&b.dw_full[(gr % RS) * 3 + y % 3]);
          }
          while (ok && pw_next <= y - 2) {
            ok = pointwise();
            ++pw_next;
          }
        }
        while (ok && NPW > 0 && pw_next < H) {
          ok = pointwise();
          ++pw_next;
        }
        gbase += static_cast<uint32_t>(H);
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
    rs_epilogue<CG, NPW, NS, RS, DWCLAMP, PWCLAMP>(
        p, tab, bars[k], sApw + k * RS * S::kApw,
        tmem_base + static_cast<uint32_t>(k * S::kSlotCols), k, set, q, lane, abort_flag);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

template <int CG, int NPW, int NS, int RS, bool DWC, bool PWC>
cudaError_t rs_launch(const CUtensorMap& m, const RsArgs& a, const DwPwTable& tab, int grid,
                      int smem, cudaStream_t s) {
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if ((done.load() & bit) == 0) {
    const cudaError_t e = cudaFuncSetAttribute(k_dwrs_s8<CG, NPW, NS, RS, DWC, PWC>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               kRsSmemLimit);
    if (e != cudaSuccess) return e;
    done.fetch_or(bit);
  }
  k_dwrs_s8<CG, NPW, NS, RS, DWC, PWC>
      <<<grid, RsShape<CG, NPW, NS, RS>::kThreads, smem, s>>>(m, a, tab);
  return cudaGetLastError();
}

template <int CG, int NPW, int NS, int RS>
cudaError_t rs_shape(const CUtensorMap& m, RsArgs a, const DwPwTable& tab, bool dwc, bool pwc,
                     int num_sms, cudaStream_t s) {
  using S = RsShape<CG, NPW, NS, RS>;
  const int overhead = 1024 + S::kFixed + NS * static_cast<int>(sizeof(RsBars)) + 64;
  a.stages = std::min(kRsMaxStages, (kRsSmemLimit - overhead) / (NS * S::kInRow));
  if (a.stages < 2) return cudaErrorInvalidValue;
  const int smem = std::max(overhead + NS * a.stages * S::kInRow, 120 * 1024);
  const int grid = static_cast<int>(
      std::min<int64_t>((static_cast<int64_t>(a.strips) + NS - 1) / NS, num_sms));
  if (grid <= 0) return cudaSuccess;
  if (dwc)
    return pwc ? rs_launch<CG, NPW, NS, RS, true, true>(m, a, tab, grid, smem, s)
               : rs_launch<CG, NPW, NS, RS, true, false>(m, a, tab, grid, smem, s);
  return pwc ? rs_launch<CG, NPW, NS, RS, false, true>(m, a, tab, grid, smem, s)
             : rs_launch<CG, NPW, NS, RS, false, false>(m, a, tab, grid, smem, s);
}

bool rs_geometry_ok(const pspml_op_desc& d) {
  return d.kind == PSPML_OP_DEPTHWISE_CONV2D && d.kernel_h == 3 && d.kernel_w == 3 &&
         d.stride_h == 1 && d.stride_w == 1 && d.pad_top == 1 && d.pad_bottom == 1 &&
         d.pad_left <= 1 && d.out_h == d.in_h && d.out_w >= 128 && d.out_w <= 65535 &&
         d.out_h <= 4096 && d.in_c == d.out_c;
}

// One launch over `batch` samples (strip count below 2^31).
cudaError_t rs_once(const pspml_op_desc& dw, const PreparedOp& pdw, int npw,
                    const uint8_t* wpw_packed, const DwPwTable& tab, bool pwc, int32_t pw_min,
                    int32_t pw_max, int64_t batch, const int8_t* in, int8_t* out,
                    unsigned* dev_err, int num_sms, cudaStream_t s) {
  RsArgs a{};
  a.tiles_x = (dw.out_w + 127) / 128;
  a.strips = static_cast<int32_t>(batch * a.tiles_x);
  a.fd_tiles_x = FastDiv(static_cast<uint32_t>(a.tiles_x));
  a.H = dw.out_h;
  a.W = dw.out_w;
  a.pad_l = dw.pad_left;
  a.wdw = reinterpret_cast<const uint8_t*>(pdw.wpack);
  a.wpw = wpw_packed;
  a.out = out;
  a.ycls = pdw.ycls;
  a.xcls = pdw.xcls;
  a.n_xcls = pdw.n_xcls;
  a.base_cls = pdw.base_cls;
  a.dw_lo4 = splat4(dw.act_min);
  a.dw_hi4 = splat4(dw.act_max);
  a.pw_lo4 = splat4(pw_min);
  a.pw_hi4 = splat4(pw_max);
  a.err = dev_err;
  const bool dwc = dw.act_min > -128 || dw.act_max < 127;

  const int C = dw.in_c;
  CUtensorMap m;
  const uint64_t dims[4] = {static_cast<uint64_t>(C), static_cast<uint64_t>(dw.in_w),
                            static_cast<uint64_t>(dw.in_h), static_cast<uint64_t>(batch)};
  const uint64_t strides[3] = {static_cast<uint64_t>(C), static_cast<uint64_t>(dw.in_w) * C,
                               static_cast<uint64_t>(dw.in_h) * dw.in_w * C};
  const uint32_t box[4] = {16, 130, 1, 1};
  const uint32_t estr[4] = {1, 1, 1, 1};
  if (encode_tensor_map(&m, in, 4, dims, strides, box, estr, CU_TENSOR_MAP_SWIZZLE_NONE) !=
      CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  if (npw == 64 && C == 32) return rs_shape<1, 64, 2, 2>(m, a, tab, dwc, pwc, num_sms, s);
  if (npw == 64 && C == 64) return rs_shape<2, 64, 2, 2>(m, a, tab, dwc, pwc, num_sms, s);
  if (npw == 0 && C == 32) return rs_shape<1, 0, 2, 2>(m, a, tab, dwc, false, num_sms, s);
  if (npw == 0 && C == 64) return rs_shape<2, 0, 2, 2>(m, a, tab, dwc, false, num_sms, s);
  return cudaErrorInvalidValue;
}

cudaError_t rs_run(const pspml_op_desc& dw, const PreparedOp& pdw, int npw,
                   const uint8_t* wpw_packed, const DwPwTable& tab, bool pwc, int32_t pw_min,
                   int32_t pw_max, int64_t out_per, int64_t batch, const int8_t* in, int8_t* out,
                   unsigned* dev_err, int num_sms, cudaStream_t s) {
  const int64_t tiles_x = (dw.out_w + 127) / 128;
  const int64_t chunk = std::max<int64_t>(1, ((1ll << 31) - 1) / tiles_x);
  const int64_t in_per = static_cast<int64_t>(dw.in_h) * dw.in_w * dw.in_c;
  for (int64_t b0 = 0; b0 < batch; b0 += chunk) {
    const cudaError_t e =
        rs_once(dw, pdw, npw, wpw_packed, tab, pwc, pw_min, pw_max, std::min(chunk, batch - b0),
                in + b0 * in_per, out + b0 * out_per, dev_err, num_sms, s);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace

bool dwrs_dw_supported(const pspml_op_desc& d) {
  return rs_geometry_ok(d) && (d.in_c == 32 || d.in_c == 64);
}

// The 32-channel pair measured faster on the tile-per-row kernel
// (dwpw_tc.cu): with a third of the channels its depthwise MMAs are cheap
// there, and its epilogue keeps four tiles in flight.
bool dwrs_pair_supported(const pspml_op_desc& dw, const pspml_op_desc& pw) {
  return rs_geometry_ok(dw) && pw.out_c == 64 && dw.in_c == 64;
}

cudaError_t launch_dwrs_dw(const pspml_op_desc& d, const PreparedOp& p, int64_t batch,
                           const int8_t* in, int8_t* out, unsigned* dev_err, int num_sms,
                           cudaStream_t s) {
  if (p.table == nullptr || !p.all_fast_known || p.ncls > 9) return cudaErrorInvalidValue;
  DwPwTable tab;
  std::memset(&tab, 0, sizeof(tab));
  const int C = d.in_c;
  for (int c = 0; c < C; ++c) {
    tab.dw_mh[c] = p.table->mh[c];
    tab.dw_bs[c] = p.table->bs[c];
  }
  for (int k = 0; k < p.ncls; ++k)
    for (int c = 0; c < C; ++c) tab.dw_dbias[k * C + c] = p.table->dbias[k * C + c];
  const int64_t out_per = static_cast<int64_t>(d.out_h) * d.out_w * d.out_c;
  return rs_run(d, p, 0, nullptr, tab, false, -128, 127, out_per, batch, in, out, dev_err,
                num_sms, s);
}

cudaError_t launch_dwrs_pair(const pspml_op_desc& dw, const PreparedOp& pdw,
                             const pspml_op_desc& pw, const uint8_t* wpw_packed,
                             const DwPwTable& tab, int64_t batch, const int8_t* in, int8_t* out,
                             unsigned* dev_err, int num_sms, cudaStream_t s) {
  const bool pwc = pw.act_min > -128 || pw.act_max < 127;
  const int64_t out_per = static_cast<int64_t>(pw.out_h) * pw.out_w * pw.out_c;
  return rs_run(dw, pdw, pw.out_c, wpw_packed, tab, pwc, pw.act_min, pw.act_max, out_per, batch,
                in, out, dev_err, num_sms, s);
}

}  // namespace pspml
