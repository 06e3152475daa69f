// im2col_tc.cu - int8 3x3 convs with 2, 3, 4 or 8 input channels on the
// tensor cores (the config-2 first conv, 3 -> 32 channels).
//
// With so few input channels a conv is one small GEMM per output pixel: its
// patch (3 filter rows of 3 * in_c bytes) against the [out_c][patch]
// weights.  The CUDA-core kernels spend about three dp4a per output there;
// here the tensor core does the products and the CUDA cores gather patches
// and requantise.
//
// Work unit: a tile of 128 output pixels (whole output rows when a row has
// at most 128 pixels, else 128 pixels of one row).  A CTA is one worker of
// four warps (one tensor-memory lane quarter each); several share an SM.
// Its tiles flow through a two-deep pipeline (two staging buffers, A tiles
// and accumulators); in the iteration of tile i it
//   1. waits for tile i's input rows, which cp.async copied into shared
//      memory two iterations earlier (rows outside the image: the input
//      zero point; the left/right padding columns hold it from the start);
//   2. lets every thread gather its pixel's patch into one row of a K-major
//      A tile [K/16][128][16 B] (no swizzle): filter row ky contributes
//      QW = ceil(3 in_c / 4) words, funnel-shifted out of the staged row,
//      whose bytes beyond the 3 in_c real ones meet zero weights;
//   3. starts the copies of tile i + 2 into the staging buffer just read;
//   4. issues tile i's 1-3 MMAs (M = 128, N = out_c, K = 32 each) from one
//      thread against the weights, resident in shared memory in the same
//      patch order, with a commit to the buffer's barrier;
//   5. while they run, requantises tile i - 1's accumulator and stores it.
//
// Epilogue: tcgen05.ld in the 16x256b shape gives a thread columns 2k and
// 2k + 1 (k = lane % 4) of every 8-column block for four pixels, so a thread
// only ever meets out_c / 4 channels and keeps their requantisation
// constants in registers for the whole kernel (the floor form is then one
// wide multiply-add and a shift per output, with no constant-bank moves).
// Pairs of packed channel bytes are exchanged within each group of four
// lanes so that every lane ends with 8 consecutive channels of a pixel, and
// the four lanes of a group store the pixel's 32 bytes together.  The
// folded bias covers all taps: the staged padding holds the zero point, so
// there are no border classes.
//
// Every wait is bounded; on expiry the kernel records an error, waits for
// its own copies and MMAs, frees tensor memory and exits.
#include <algorithm>
#include <atomic>

#include "kernels.h"
#include "ptx.cuh"
#include "requant.cuh"

namespace pspml {

namespace {

constexpr int kIcLead = 16;  // staged row: bytes before input column 0
constexpr int kIcTail = 48;  // staged row: padding + over-read after the last column
constexpr int kIcSmemLimit = 96 * 1024;  // dynamic shared memory of one CTA
constexpr int kSmSmem = 233472;          // shared memory of an SM (bytes)

struct IcArgs {
  int32_t H, W, Ho, Wo;
  int32_t pt, pl;
  int32_t R;         // output rows per tile (1 when rows are wider than 128 px)
  int32_t tiles_x;   // 128-pixel tiles per output row (1 when R > 1)
  int32_t nr;        // input rows staged per tile: (R - 1) * S + 3
  int32_t rb;        // staged row stride (bytes, multiple of 16)
  int32_t tiles;     // over the batch
  FastDiv fd_tps;    // tiles per sample
  FastDiv fd_tx;     // tiles_x
  FastDiv fd_vpr;    // copy units per staged row
  int32_t vpr;
  uint32_t zp4;      // input zero point in every byte
  int32_t v16;       // staged rows copied in 16-byte units (row bytes, base 16-aligned)
  uint32_t lo4, hi4;
  const int8_t* in;
  const int8_t* filter;  // TFLite [out_c][3][3][in_c]
  int8_t* out;
  unsigned* err;
};

template <int CI, int S, int N>
struct IcShape {
  static constexpr int QW = (3 * CI + 3) / 4;              // words per filter row
  static constexpr int KW = 3 * QW;                        // patch words
  static constexpr int KB = (KW * 4 + 31) / 32;            // 32-byte K blocks (MMAs)
  static constexpr int KH16 = 2 * KB;                      // 16-byte K halves
  static constexpr bool kAligned = CI % 4 == 0;            // patch rows start on words
  static constexpr int kA = KH16 * 2048;                   // one A tile
  static constexpr int kB = KH16 * N * 16;                 // resident weights
  static constexpr int kCols = N;                          // columns of one accumulator
  static constexpr int NC = N / 4;                         // channels a thread requantises
  static constexpr int kMaxCtas = 512 / (2 * kCols);       // CTAs an SM's tensor memory holds
  static_assert(KB <= 3, "patch of at most 96 bytes");
  static_assert(N == 32 || N == 64, "output channels");
};

__device__ __forceinline__ void ic_record_error(unsigned* err, volatile int* abort_flag,
                                                unsigned code) {
  *abort_flag = 1;
  if (err != nullptr) atomicCAS(err, 0u, code);
}

// Ampere-style asynchronous global -> shared copies (16 or 4 bytes),
// grouped per tile.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait1() {
  asm volatile("cp.async.wait_group 1;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

__device__ __forceinline__ void ic_fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// The four lanes k of a group hold, for one pixel, 16-bit channel pairs
// P_k[g] (channels 8g + 2k and 8g + 2k + 1) as w01 = P_k[0] | P_k[1] << 16
// and w23 = P_k[2] | P_k[3] << 16.  Afterwards lane k holds 8-channel
// block k: o0 = P_0[k] | P_1[k] << 16, o1 = P_2[k] | P_3[k] << 16.
__device__ __forceinline__ void quad_transpose(uint32_t w01, uint32_t w23, int k, uint32_t* o0,
                                               uint32_t* o1) {
  // Lanes 0, 1 want blocks 0, 1 (everyone's w01), lanes 2, 3 blocks 2, 3.
  const bool hi = (k & 2) != 0;
  const uint32_t keep = hi ? w23 : w01;
  const uint32_t x = __shfl_xor_sync(0xFFFFFFFFu, hi ? w01 : w23, 2);
  // keep = P_k[b..b+1], x = P_(k^2)[b..b+1] (b = 0 or 2).  Lane k wants
  // element k & 1 of every lane's pair: it keeps its own two and swaps the
  // other element of both with lane k ^ 1.
  const bool odd = (k & 1) != 0;
  const uint32_t y = __shfl_xor_sync(0xFFFFFFFFu, prmt(keep, x, odd ? 0x5410u : 0x7632u), 1);
  uint32_t a, b;
  if (!odd) {
    a = prmt(keep, y, 0x5410u);  // P_k[b] | P_(k^1)[b] << 16
    b = prmt(x, y, 0x7610u);     // P_(k^2)[b] | P_(k^3)[b] << 16
  } else {
    a = prmt(y, keep, 0x7610u);  // P_(k^1)[b+1] | P_k[b+1] << 16
    b = prmt(y, x, 0x7632u);     // P_(k^3)[b+1] | P_(k^2)[b+1] << 16
  }
  // Lanes 0, 1 own P_0, P_1 in a; lanes 2, 3 own P_2, P_3 in a.
  *o0 = hi ? b : a;
  *o1 = hi ? a : b;
}

// CI: input channels; S: stride; N: output channels; Q: ep_flags.
template <int CI, int S, int N, int Q>
__global__ void __launch_bounds__(128) k_im2col_s8(const IcArgs p,
                                                   const __grid_constant__ EpiTable tab) {
  using Sh = IcShape<CI, S, N>;
  constexpr int QW = Sh::QW;
  constexpr int KH16 = Sh::KH16;
  constexpr int NC = Sh::NC;
  constexpr int kBPad = (Sh::kB + 1023) / 1024 * 1024;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int stage = p.nr * p.rb;
  uint8_t* sB = smem;                  // [KH16][N][16]
  uint8_t* sA = sB + kBPad;            // [2][KH16][128][16]
  uint8_t* sIn = sA + 2 * Sh::kA;      // [2][nr][rb]
  uint64_t* bars = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(sIn + 2 * stage) + 7) & ~static_cast<uintptr_t>(7));
  uint64_t* acc_full = bars;           // [2]: MMA -> warps
  uint64_t* done = bars + 2;           // final drain
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int px = threadIdx.x;  // tile row
  const int q = px >> 5;       // lane quarter
  const int lane = px & 31;
  const int k4 = lane & 3;     // column pair within an 8-column block
  // Resident weights in patch order: word j of K half h for output n holds
  // patch bytes 4 (4h + j) .. +3; patch word k = ky * QW + i covers bytes
  // 4i .. 4i+3 of filter row ky, byte b = kx * CI + c (zero past 3 CI).
  for (int i = px; i < KH16 * N * 4; i += 128) {
    const int j = i & 3;
    const int nrow = (i >> 2) % N;
    const int h = (i >> 2) / N;
    const int k = 4 * h + j;
    const int ky = k / QW;
    uint32_t wd = 0;
    if (ky < 3) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int b = 4 * (k - ky * QW) + e;
        if (b < 3 * CI) {
          const int kx = b / CI, c = b - (b / CI) * CI;
          const uint32_t v = static_cast<uint8_t>(p.filter[((nrow * 3 + ky) * 3 + kx) * CI + c]);
          wd |= v << (8 * e);
        }
      }
    }
    reinterpret_cast<uint32_t*>(sB)[(h * N + nrow) * 4 + j] = wd;
  }
  // A tiles start zeroed (K halves past the patch stay zero); staged rows
  // start as the input zero point (the padding columns keep it).
  for (int i = px; i < 2 * Sh::kA / 16; i += 128)
    reinterpret_cast<uint4*>(sA)[i] = make_uint4(0, 0, 0, 0);
  for (int i = px; i < 2 * stage / 16; i += 128)
    reinterpret_cast<uint4*>(sIn)[i] = make_uint4(p.zp4, p.zp4, p.zp4, p.zp4);
  ic_fence_async_smem();
  if (px == 0) {
    mbar_init(&acc_full[0], 1);
    mbar_init(&acc_full[1], 1);
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (q == 0) {
    tmem_alloc(tmem_slot, 2 * Sh::kCols);
    tmem_relinquish();
  }
  // This thread's requantisation constants: channels 8g + 2 k4 + e of
  // every 8-column block g, entry 2g + e.
  int2 cmh[NC], cbs[NC];
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = 8 * (i >> 1) + 2 * k4 + (i & 1);
    cmh[i] = tab.mh[c];
    cbs[i] = tab.bs[c];
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // The patch this thread gathers: tile row px.
  int r_g = 0, ox_g = px;
  if (p.R > 1) {
    r_g = px / p.Wo;
    ox_g = px - r_g * p.Wo;
  }
  const bool gather_ok = r_g < p.R;
  // The four pixels this thread requantises: tile rows 32q + 16h + 8r + lane/4.
  int r_e[4], ox_e[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = 32 * q + 16 * (i >> 1) + 8 * (i & 1) + (lane >> 2);
    r_e[i] = p.R > 1 ? row / p.Wo : 0;
    ox_e[i] = p.R > 1 ? row - r_e[i] * p.Wo : row;
  }
  const int tps = p.tiles_x * ((p.Ho + p.R - 1) / p.R);
  const int row_bytes = p.W * CI;
  const int nt = static_cast<int>(blockIdx.x) < p.tiles
                     ? (p.tiles - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                     : 0;  // this CTA's tiles

  // Tile -> (sample, tile row, tile column).
  auto tile_pos = [&](int i, uint32_t* n, int* ty, int* tx) {
    const uint32_t t = static_cast<uint32_t>(static_cast<int>(blockIdx.x) + i * static_cast<int>(gridDim.x));
    *n = p.fd_tps.div(t);
    const uint32_t rem = t - *n * static_cast<uint32_t>(tps);
    const uint32_t tyu = p.fd_tx.div(rem);
    *ty = static_cast<int>(tyu);
    *tx = static_cast<int>(rem - tyu * static_cast<uint32_t>(p.tiles_x));
  };
  // Copies the input rows of local tile i into staging buffer b as one
  // cp.async group (empty past the last tile); rows outside the image get
  // the zero point.
  auto stage_tile = [&](int i, int b) {
    if (i < nt) {
      uint32_t n;
      int ty, tx;
      tile_pos(i, &n, &ty, &tx);
      const int iy0 = ty * p.R * S - p.pt;
      uint8_t* base = sIn + b * stage + kIcLead;
      const int unit = p.v16 ? 16 : 4;
      for (int e = px; e < p.nr * p.vpr; e += 128) {
        const int j = static_cast<int>(p.fd_vpr.div(static_cast<uint32_t>(e)));
        const int u = e - j * p.vpr;
        const int iy = iy0 + j;
        uint8_t* dst = base + j * p.rb + u * unit;
        if (iy >= 0 && iy < p.H) {
          const int8_t* src =
              p.in + (static_cast<int64_t>(n) * p.H + iy) * row_bytes + u * unit;
          if (p.v16)
            cp_async16(dst, src);
          else
            cp_async4(dst, src);
        } else if (p.v16) {
          *reinterpret_cast<uint4*>(dst) = make_uint4(p.zp4, p.zp4, p.zp4, p.zp4);
        } else {
          *reinterpret_cast<uint32_t*>(dst) = p.zp4;
        }
      }
    }
    cp_async_commit();
  };

  stage_tile(0, 0);
  stage_tile(1, 1);
  bool failed = false;
  uint32_t pn = 0;  // sample and tile row / column of the previous tile
  int pty = 0, ptx = 0;
  for (int i = 0; i <= nt; ++i) {
    uint32_t n = 0;
    int ty = 0, tx = 0;
    if (i < nt) {
      tile_pos(i, &n, &ty, &tx);
      cp_async_wait1();  // this thread's copies of tile i
    }
    // Tile i's rows are staged, and the tensor-memory loads of tile i - 2
    // (same accumulator) are done.
    tc_fence_before();
    if (__syncthreads_or(failed ? 1 : 0) != 0) break;
    tc_fence_after();
    if (i < nt) {
      const int b = i & 1;
      // This thread's patch -> its row of the A tile.
      uint8_t* atile = sA + b * Sh::kA;
      const uint8_t* stg = sIn + b * stage;
      const int oy = ty * p.R + r_g;
      const int ox = tx * 128 + ox_g;
      uint32_t wv[KH16 * 4];
#pragma unroll
      for (int k = 0; k < KH16 * 4; ++k) wv[k] = 0;
      if (gather_ok && oy < p.Ho && ox < p.Wo) {
        const int b0 = (ox * S - p.pl) * CI;  // >= -16: inside the row's lead bytes
#pragma unroll
        for (int ky = 0; ky < 3; ++ky) {
          const uint8_t* row = stg + (r_g * S + ky) * p.rb + kIcLead;
          if constexpr (Sh::kAligned) {
            const uint32_t* src = reinterpret_cast<const uint32_t*>(row + b0);
#pragma unroll
            for (int k = 0; k < QW; ++k) wv[ky * QW + k] = src[k];
          } else {
            const uint32_t* src = reinterpret_cast<const uint32_t*>(row + (b0 & ~3));
            const uint32_t sh = static_cast<uint32_t>(b0 & 3) * 8u;
            uint32_t x[QW + 1];
#pragma unroll
            for (int k = 0; k <= QW; ++k) x[k] = src[k];
#pragma unroll
            for (int k = 0; k < QW; ++k) wv[ky * QW + k] = __funnelshift_r(x[k], x[k + 1], sh);
          }
        }
      }
#pragma unroll
      for (int h = 0; h < KH16; ++h)
        if (4 * h < Sh::KW)
          *reinterpret_cast<uint4*>(atile + h * 2048 + px * 16) =
              make_uint4(wv[4 * h], wv[4 * h + 1], wv[4 * h + 2], wv[4 * h + 3]);
      ic_fence_async_smem();
      __syncthreads();

      // Staging buffer b is free: tile i + 2's rows.
      stage_tile(i + 2, b);
      // The MMAs of tile i.
      if (px == 0) {
        tc_fence_after();
        const uint32_t a0 = smem_u32(atile), b0s = smem_u32(sB);
        const uint32_t idesc = make_idesc_s8(128, N);
#pragma unroll
        for (int kb = 0; kb < Sh::KB; ++kb) {
          const uint64_t ad = make_sdesc(a0 + kb * 2 * 2048, 2048, 128, 0);
          const uint64_t bd = make_sdesc(b0s + kb * 2 * (N * 16), N * 16, 128, 0);
          umma_i8(tmem_base + static_cast<uint32_t>(b * Sh::kCols), ad, bd, idesc,
                  kb > 0 ? 1u : 0u);
        }
        umma_commit(&acc_full[b]);
      }
    }

    // The epilogue of tile i - 1 (its MMAs overlapped the work above).
    if (i > 0) {
      const int j = i - 1, b = j & 1;
      int ok = 0;
      if (lane == 0)
        ok = mbar_wait(&acc_full[b], static_cast<uint32_t>((j >> 1) & 1), abort_flag) ? 1 : 0;
      ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
      if (!ok) {
        if (lane == 0) ic_record_error(p.err, abort_flag, kDevErrEpiWait);
        failed = true;
      } else {
        tc_fence_after();
        const uint32_t tq = tmem_base + static_cast<uint32_t>(b * Sh::kCols) +
                            (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t acc[N / 16][8];
#pragma unroll
          for (int u = 0; u < N / 16; ++u)
            tmem_ld_16x256b_x2(tq + (static_cast<uint32_t>(16 * h) << 16) +
                                   static_cast<uint32_t>(16 * u),
                               acc[u]);
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            const int pi = 2 * h + r;
            int32_t y[NC];
#pragma unroll
            for (int c = 0; c < NC; ++c) {
              // Entry c: block g = c / 2, column 2 k4 + (c & 1); the load's
              // registers of block g: 4 (g % 2) + 2 r + (c & 1).
              const uint32_t v = acc[c >> 2][4 * ((c >> 1) & 1) + 2 * r + (c & 1)];
              if constexpr ((Q & kEpFloor) != 0)
                y[c] = rq_floor_entry(v, cmh[c], cbs[c]);
              else
                y[c] = rq_tab(static_cast<int32_t>(v) + cbs[c].x, cmh[c], cbs[c].y);
            }
            const int oy = pty * p.R + r_e[pi];
            const int ox = ptx * 128 + ox_e[pi];
            const bool valid = r_e[pi] < p.R && oy < p.Ho && ox < p.Wo;
            int8_t* o = p.out + ((static_cast<int64_t>(pn) * p.Ho + oy) * p.Wo + ox) * N + 8 * k4;
#pragma unroll
            for (int hb = 0; hb < N / 32; ++hb) {
              uint32_t w01 = pack_sat4(y[8 * hb], y[8 * hb + 1], y[8 * hb + 2], y[8 * hb + 3]);
              uint32_t w23 =
                  pack_sat4(y[8 * hb + 4], y[8 * hb + 5], y[8 * hb + 6], y[8 * hb + 7]);
              if constexpr ((Q & kEpClamp) != 0) {
                w01 = clamp4(w01, p.lo4, p.hi4);
                w23 = clamp4(w23, p.lo4, p.hi4);
              }
              uint32_t o0, o1;
              quad_transpose(w01, w23, k4, &o0, &o1);
              if (valid) *reinterpret_cast<uint2*>(o + 32 * hb) = make_uint2(o0, o1);
            }
          }
        }
      }
    }
    pn = n;
    pty = ty;
    ptx = tx;
  }
  cp_async_wait_all();  // no copy lands after the CTA exits

  // Every MMA completes before tensor memory is freed.
  if (px == 0) {
    umma_commit(done);
    mbar_wait(done, 0, nullptr);
  }
  tc_fence_before();
  __syncthreads();
  if (q == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * Sh::kCols);
  }
}

}  // namespace

namespace {

// Tile geometry of a conv: output rows per tile, staged input rows and the
// staged row stride.
void ic_geometry(const pspml_op_desc& d, int* R, int* nr, int* rb) {
  *R = d.out_w <= 128 ? 128 / d.out_w : 1;
  *nr = (*R - 1) * d.stride_h + 3;
  *rb = (kIcLead + d.in_w * d.in_c + kIcTail + 15) / 16 * 16;
}

// Dynamic shared memory one CTA needs.
int ic_smem_need(const pspml_op_desc& d) {
  int R, nr, rb;
  ic_geometry(d, &R, &nr, &rb);
  const int qw = (3 * d.in_c + 3) / 4;
  const int kb = (3 * qw * 4 + 31) / 32;
  const int b_pad = (2 * kb * d.out_c * 16 + 1023) / 1024 * 1024;
  return 1024 + b_pad + 2 * (2 * kb * 2048) + 2 * nr * rb + 8 + 3 * 8 + 16;
}

template <int CI, int S, int N, int Q>
cudaError_t ic_launch(const IcArgs& a, const EpiTable& tab, int need, int num_sms,
                      cudaStream_t s) {
  using Sh = IcShape<CI, S, N>;
  static std::atomic<uint64_t> attr_done{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  // At most kMaxCtas CTAs per SM (their accumulators fill tensor memory):
  // each asks for more than an SM's shared memory / (kMaxCtas + 1).
  const int floor_req = kSmSmem / (Sh::kMaxCtas + 1) - 1024 + 128;
  const int smem = std::max(need, floor_req);
  static std::atomic<int> regs{0};
  if ((attr_done.load() & bit) == 0) {
    cudaError_t e = cudaFuncSetAttribute(
        k_im2col_s8<CI, S, N, Q>, cudaFuncAttributeMaxDynamicSharedMemorySize, kIcSmemLimit);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(k_im2col_s8<CI, S, N, Q>,
                               cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    cudaFuncAttributes fa{};
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, k_im2col_s8<CI, S, N, Q>);
    if (e != cudaSuccess) return e;
    regs.store(fa.numRegs);
    attr_done.fetch_or(bit);
  }
  // CTAs per SM: registers (allocated per warp in units of 256), shared
  // memory (1 KB reserved per CTA) and tensor memory.
  const int warp_regs = (regs.load() * 32 + 255) / 256 * 256;
  const int by_regs = 65536 / (4 * warp_regs);
  const int by_smem = kSmSmem / (smem + 1024);
  const int occ = std::max(1, std::min({by_regs, by_smem, Sh::kMaxCtas}));
  const int grid =
      static_cast<int>(std::min<int64_t>(a.tiles, static_cast<int64_t>(num_sms) * occ));
  k_im2col_s8<CI, S, N, Q><<<grid, 128, smem, s>>>(a, tab);
  return cudaGetLastError();
}

template <int CI, int S, int N>
cudaError_t ic_form(const IcArgs& a, const EpiTable& tab, int q, int need, int num_sms,
                    cudaStream_t s) {
  switch (q) {
    case 0: return ic_launch<CI, S, N, 0>(a, tab, need, num_sms, s);
    case 1: return ic_launch<CI, S, N, 1>(a, tab, need, num_sms, s);
    case 2: return ic_launch<CI, S, N, 2>(a, tab, need, num_sms, s);
    default: return ic_launch<CI, S, N, 3>(a, tab, need, num_sms, s);
  }
}

template <int CI>
cudaError_t ic_shape(const IcArgs& a, const EpiTable& tab, int stride, int n, int q, int need,
                     int num_sms, cudaStream_t s) {
  if (stride == 1)
    return n == 32 ? ic_form<CI, 1, 32>(a, tab, q, need, num_sms, s)
                   : ic_form<CI, 1, 64>(a, tab, q, need, num_sms, s);
  return n == 32 ? ic_form<CI, 2, 32>(a, tab, q, need, num_sms, s)
                 : ic_form<CI, 2, 64>(a, tab, q, need, num_sms, s);
}

}  // namespace

// 3x3 convs, stride 1 or 2, with 2, 3, 4 or 8 input channels and 32 or 64
// outputs, every channel in the fast requantisation form (constant table),
// padding of at most 2 per side, input rows of a multiple of 4 bytes,
// 32-byte aligned outputs and staged rows that fit one CTA's shared memory.
// (One input channel stays on the CUDA cores: three dp4a per output with
// register-resident constants beat this kernel's patch gathering there.)
bool im2col_conv_supported(const pspml_op_desc& d, const PreparedOp& p, const int8_t* in,
                           const int8_t* out) {
  if (d.kind != PSPML_OP_CONV2D || d.kernel_h != 3 || d.kernel_w != 3) return false;
  if (d.stride_h != d.stride_w || (d.stride_h != 1 && d.stride_h != 2)) return false;
  const int ci = d.in_c;
  if (!(ci == 2 || ci == 3 || ci == 4 || ci == 8)) return false;
  if (!(d.out_c == 32 || d.out_c == 64)) return false;
  if (p.table == nullptr || !p.all_fast_known || p.ncls != 1) return false;
  if (d.pad_top < 0 || d.pad_top > 2 || d.pad_left < 0 || d.pad_left > 2 || d.pad_bottom < 0 ||
      d.pad_bottom > 2 || d.pad_right < 0 || d.pad_right > 2)
    return false;
  if ((static_cast<int64_t>(d.in_w) * ci) % 4 != 0 || d.in_w > 4096) return false;
  if ((reinterpret_cast<uintptr_t>(in) & 3u) != 0) return false;
  if ((reinterpret_cast<uintptr_t>(out) & 31u) != 0) return false;
  return ic_smem_need(d) <= kIcSmemLimit;
}

cudaError_t launch_im2col_conv(const pspml_op_desc& d, const PreparedOp& p, int64_t batch,
                               const int8_t* in, int8_t* out, unsigned* dev_err, int num_sms,
                               cudaStream_t s) {
  if (batch <= 0) return cudaSuccess;
  if (!im2col_conv_supported(d, p, in, out)) return cudaErrorInvalidValue;
  const int S = d.stride_h;
  IcArgs a{};
  a.H = d.in_h;
  a.W = d.in_w;
  a.Ho = d.out_h;
  a.Wo = d.out_w;
  a.pt = d.pad_top;
  a.pl = d.pad_left;
  ic_geometry(d, &a.R, &a.nr, &a.rb);
  a.tiles_x = d.out_w <= 128 ? 1 : (d.out_w + 127) / 128;
  const int64_t tps = static_cast<int64_t>(a.tiles_x) * ((d.out_h + a.R - 1) / a.R);
  a.fd_tps = FastDiv(static_cast<uint32_t>(tps));
  a.fd_tx = FastDiv(static_cast<uint32_t>(a.tiles_x));
  a.zp4 = splat4(d.zp_in);
  const int64_t row_bytes = static_cast<int64_t>(d.in_w) * d.in_c;
  a.v16 = (row_bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(in) & 15u) == 0) ? 1 : 0;
  a.vpr = static_cast<int32_t>(row_bytes / (a.v16 ? 16 : 4));
  a.fd_vpr = FastDiv(static_cast<uint32_t>(a.vpr));
  a.lo4 = splat4(d.act_min);
  a.hi4 = splat4(d.act_max);
  a.filter = p.filter;
  a.err = dev_err;
  const int q = ep_flags(d.act_min, d.act_max, d.zp_out);
  const int need = ic_smem_need(d);
  const int64_t in_per = static_cast<int64_t>(d.in_h) * d.in_w * d.in_c;
  const int64_t out_per = static_cast<int64_t>(d.out_h) * d.out_w * d.out_c;
  // Tile indices are 32-bit: larger batches run as several launches.
  const int64_t chunk = std::max<int64_t>(1, ((1ll << 31) - 1) / tps);
  for (int64_t b0 = 0; b0 < batch; b0 += chunk) {
    const int64_t nb = std::min(chunk, batch - b0);
    a.tiles = static_cast<int32_t>(nb * tps);
    a.in = in + b0 * in_per;
    a.out = out + b0 * out_per;
    cudaError_t e = cudaErrorInvalidValue;
    switch (d.in_c) {
      case 2: e = ic_shape<2>(a, *p.table, S, d.out_c, q, need, num_sms, s); break;
      case 3: e = ic_shape<3>(a, *p.table, S, d.out_c, q, need, num_sms, s); break;
      case 4: e = ic_shape<4>(a, *p.table, S, d.out_c, q, need, num_sms, s); break;
      case 8: e = ic_shape<8>(a, *p.table, S, d.out_c, q, need, num_sms, s); break;
      default: break;
    }
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace pspml
