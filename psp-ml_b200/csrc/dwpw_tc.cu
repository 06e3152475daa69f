// dwpw_tc.cu - a depthwise 3x3 stride-1 conv and the 1x1 conv after it as
// one tensor-core kernel (the depthwise-separable block of the config-3
// network).
//
// The pair runs as two chained GEMMs per tile of 128 output pixels of one
// row, over all C channels:
//   1. depthwise: per 32-channel group, 9 MMAs (M=128, N=32, K=32) with
//      block-diagonal weights over the three halo input rows, exactly as in
//      dw_tc.cu;
//   2. the epilogue warps requantise those accumulators (folded bias per
//      border class, TFLite requant, clamp) straight into a shared-memory A
//      tile [C/16][128 rows][16 B] (K-major, no swizzle);
//   3. pointwise: C/32 MMAs (M=128, N=N, K=32) of that tile against the
//      resident 1x1 weights; the epilogue requantises and stores NHWC.
// The depthwise output never reaches HBM, and one pipeline serves both
// convs.  Two MMA threads take the even and the odd tiles; each issues the
// pointwise MMAs of its previous tile after the depthwise MMAs of the next,
// so the tensor pipe has work while the epilogue builds the A tile.
//
// Roles: warp 0 TMA (halo rows, weights once), warps 1 and 2 + 4G MMA, G
// groups of 4 epilogue warps (one per tensor-memory lane quarter) taking
// tiles in turn.
// Every wait is bounded; on expiry the kernel records an error, drains its
// copies and MMAs, frees tensor memory and exits.
#include <algorithm>
#include <atomic>

#include "kernels.h"
#include "ptx.cuh"
#include "requant.cuh"

namespace pspml {

namespace {

constexpr int kRegionF = 2176;  // one halo row half: 130 px x 16 B, padded to 128 B
constexpr int kSmemLimitF = 232448;
constexpr int kDwGroupBytes = 9 * 2 * 32 * 16;  // block-diagonal weights of one group

struct DwPwArgs {
  int64_t tiles;  // batch * Ho * tiles_x, below 2^31
  FastDiv fd_tiles_x, fd_ho;
  int32_t tiles_x, Ho, Wo;
  int32_t pad_t, pad_l;
  const uint8_t* wdw;  // [CG][9][2][32][16]
  const uint8_t* wpw;  // [C/16][N][16]
  int8_t* out;         // [B][Ho][Wo][N]
  const uint8_t* ycls;
  const uint8_t* xcls;
  int32_t n_xcls, base_cls;
  uint32_t dw_lo4, dw_hi4, pw_lo4, pw_hi4;
  unsigned* err;
  int32_t stages;
};

template <int CG, int N>
struct DwPwShape {
  static constexpr int C = CG * 32;
  static constexpr int kCols = C + N;  // tensor-memory columns per tile
  static constexpr int kBufs = (512 / kCols) >= 8 ? 8 : (512 / kCols);
  static constexpr int kGroups = kBufs >= 4 ? 4 : kBufs;
  static constexpr int kMma2 = 2 + 4 * kGroups;  // second MMA-issuing warp (odd tiles)
  static constexpr int kThreads = 64 + 128 * kGroups + 32;
  static constexpr int kStage = 6 * CG * kRegionF;  // 3 rows x CG groups x 2 halves
  static constexpr int kApw = 128 * C;              // one pointwise A tile
  static constexpr int kFixed = CG * kDwGroupBytes + C * N + kBufs * kApw;
};

__device__ __forceinline__ void fused_record_error(unsigned* err, volatile int* abort_flag,
                                                   unsigned code) {
  *abort_flag = 1;
  if (err != nullptr) atomicCAS(err, 0u, code);
}

__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 16 outputs of channels ch..ch+15 with the pair table's split constants.
template <int Q>
__device__ __forceinline__ uint4 requant16_pair(const uint32_t* v, const int2* mh, const int2* bs,
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

template <int CG, int N, int DWQ, int PWQ>
__global__ void __launch_bounds__(DwPwShape<CG, N>::kThreads, 1)
    k_dwpw_s8(const __grid_constant__ CUtensorMap tmIn, const DwPwArgs p,
              const __grid_constant__ DwPwTable tab) {
  using S = DwPwShape<CG, N>;
  constexpr int C = S::C;
  constexpr int NB = S::kBufs;
  constexpr int G = S::kGroups;
  constexpr int kCols = S::kCols;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int stages = p.stages;
  uint8_t* sBdw = smem;
  uint8_t* sBpw = sBdw + CG * kDwGroupBytes;
  uint8_t* sApw = sBpw + C * N;
  uint8_t* sIn = sApw + NB * S::kApw;
  uint64_t* in_full = reinterpret_cast<uint64_t*>(sIn + stages * S::kStage);
  uint64_t* in_empty = in_full + stages;
  uint64_t* dw_full = in_empty + stages;
  uint64_t* apw_full = dw_full + NB;
  uint64_t* pw_full = apw_full + NB;
  uint64_t* tmem_empty = pw_full + NB;
  uint64_t* wfull = tmem_empty + NB;
  uint64_t* mma_done = wfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&in_full[s], 1);
      mbar_init(&in_empty[s], 1);
    }
    for (int a = 0; a < NB; ++a) {
      mbar_init(&dw_full[a], 1);
      mbar_init(&apw_full[a], 4);
      mbar_init(&pw_full[a], 1);
      mbar_init(&tmem_empty[a], 4);
    }
    mbar_init(wfull, 1);
    mbar_init(mma_done, 2);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmIn);
      mbar_arrive_expect_tx(wfull, CG * kDwGroupBytes + C * N);
      bulk_load(sBdw, p.wdw, CG * kDwGroupBytes, wfull);
      bulk_load(sBpw, p.wpw, C * N, wfull);
      int s = 0;
      uint32_t ph = 0;
      int64_t issued = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < p.tiles; t += gridDim.x) {
        const uint32_t rest = p.fd_tiles_x.div(static_cast<uint32_t>(t));
        const int tx = static_cast<int>(static_cast<uint32_t>(t) - rest * p.tiles_x);
        const uint32_t n = p.fd_ho.div(rest);
        const int y = static_cast<int>(rest - n * p.Ho);
        if (!mbar_wait(&in_empty[s], ph ^ 1u, abort_flag)) {
          fused_record_error(p.err, abort_flag, kDevErrTmaWait);
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&in_full[s], 6 * CG * 16 * 130);
        uint8_t* a = sIn + s * S::kStage;
#pragma unroll
        for (int ky = 0; ky < 3; ++ky)
#pragma unroll
          for (int g = 0; g < CG; ++g)
#pragma unroll
            for (int h = 0; h < 2; ++h)
              tma_load_4d(a + ((ky * CG + g) * 2 + h) * kRegionF, &tmIn, &in_full[s],
                          g * 32 + h * 16, tx * 128 - p.pad_l, y - p.pad_t + ky,
                          static_cast<int>(n));
        ++issued;
        if (++s == stages) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (!ok) {
        const int64_t first = issued > stages ? issued - stages : 0;
        for (int64_t g = first; g < issued; ++g)
          mbar_wait(&in_full[g % stages], static_cast<uint32_t>((g / stages) & 1), nullptr);
      }
      mbar_wait(wfull, 0, nullptr);
    }
  } else if (warp == 1 || warp == S::kMma2) {
    // ------------------------------------------------------- MMA issuers
    // Two threads, one for the even and one for the odd local tiles (each
    // issues and commits the MMAs of its own tiles): a single issuing thread
    // set the pace.
    if (lane == 0) {
      const uint32_t idesc_dw = make_idesc_s8(128, 32);
      const uint32_t idesc_pw = make_idesc_s8(128, N);
      bool ok = mbar_wait(wfull, 0, abort_flag);
      if (!ok) fused_record_error(p.err, abort_flag, kDevErrMmaWait);
      const uint32_t bdw0 = smem_u32(sBdw);
      const uint32_t bpw0 = smem_u32(sBpw);
      const uint32_t apw0 = smem_u32(sApw);
      const uint32_t in0 = smem_u32(sIn);
      int pb = 0;           // buffer of this thread's previous tile
      uint32_t ppar = 0;    // its use parity
      bool have_prev = false;
      // Pointwise MMAs of the tile in buffer `bb` (its A tile built by the
      // epilogue).
      auto pointwise = [&](int bb, uint32_t pr) -> bool {
        if (!mbar_wait(&apw_full[bb], pr, abort_flag)) return false;
        tc_fence_after();
        const uint32_t a_t = apw0 + static_cast<uint32_t>(bb * S::kApw);
        const uint32_t d_t = tmem_base + static_cast<uint32_t>(bb * kCols + C);
#pragma unroll
        for (int kc = 0; kc < C / 32; ++kc) {
          const uint64_t ad = make_sdesc(a_t + kc * 2 * 2048, 2048, 128, 0);
          const uint64_t bd = make_sdesc(bpw0 + kc * 2 * (N * 16), N * 16, 128, 0);
          umma_i8(d_t, ad, bd, idesc_pw, kc > 0 ? 1u : 0u);
        }
        umma_commit(&pw_full[bb]);
        return true;
      };
      int64_t i = warp == 1 ? 0 : 1;  // local tile index
      for (int64_t t = blockIdx.x + i * gridDim.x; ok && t < p.tiles;
           t += 2 * static_cast<int64_t>(gridDim.x), i += 2) {
        const int s = static_cast<int>(i % stages);
        const uint32_t ph = static_cast<uint32_t>((i / stages) & 1);
        const int b = static_cast<int>(i % NB);
        const uint32_t par = static_cast<uint32_t>((i / NB) & 1);
        if (!mbar_wait(&tmem_empty[b], par ^ 1u, abort_flag) ||
            !mbar_wait(&in_full[s], ph, abort_flag)) {
          fused_record_error(p.err, abort_flag, kDevErrMmaWait);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = in0 + static_cast<uint32_t>(s * S::kStage);
        const uint32_t d_t = tmem_base + static_cast<uint32_t>(b * kCols);
#pragma unroll
        for (int g = 0; g < CG; ++g) {
#pragma unroll
          for (int tap = 0; tap < 9; ++tap) {
            const int ky = tap / 3, kx = tap % 3;
            const uint64_t ad =
                make_sdesc(a0 + ((ky * CG + g) * 2) * kRegionF + kx * 16, kRegionF, 128, 0);
            const uint64_t bd = make_sdesc(bdw0 + g * kDwGroupBytes + tap * 1024, 512, 128, 0);
            umma_i8(d_t + g * 32, ad, bd, idesc_dw, tap > 0 ? 1u : 0u);
          }
        }
        umma_commit(&in_empty[s]);
        umma_commit(&dw_full[b]);
        if (have_prev && !pointwise(pb, ppar)) {
          fused_record_error(p.err, abort_flag, kDevErrMmaWait);
          ok = false;
          break;
        }
        have_prev = true;
        pb = b;
        ppar = par;
      }
      if (ok && have_prev && !pointwise(pb, ppar))
        fused_record_error(p.err, abort_flag, kDevErrMmaWait);
      // All MMAs issued by this thread complete before tensor memory is freed.
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, nullptr);
    }
  } else {
    // --------------------------------------------------------- epilogue
    const int grp = (warp - 2) >> 2;
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t tlane = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    int b = grp % NB;
    uint32_t par = static_cast<uint32_t>((grp / NB) & 1);
    for (int64_t t = blockIdx.x + static_cast<int64_t>(grp) * gridDim.x; t < p.tiles;
         t += static_cast<int64_t>(G) * gridDim.x) {
      // ---- depthwise accumulators -> int8 A tile in shared memory
      int ready = 0;
      if (lane == 0) {
        ready = mbar_wait(&dw_full[b], par, abort_flag) ? 1 : 0;
        if (!ready) fused_record_error(p.err, abort_flag, kDevErrEpiWait);
      }
      ready = __shfl_sync(0xFFFFFFFFu, ready, 0);
      if (!ready) break;
      tc_fence_after();
      const uint32_t rest = p.fd_tiles_x.div(static_cast<uint32_t>(t));
      const int tx = static_cast<int>(static_cast<uint32_t>(t) - rest * p.tiles_x);
      const uint32_t n = p.fd_ho.div(rest);
      const int y = static_cast<int>(rest - n * p.Ho);
      const int x = tx * 128 + row;
      const bool valid = x < p.Wo;
      const int cls = valid ? p.ycls[y] * p.n_xcls + p.xcls[x] : p.base_cls;
      const bool border = cls != p.base_cls;
      const int cls_off = cls * C;
      const uint32_t tb = tlane + static_cast<uint32_t>(b * kCols);
      uint8_t* arow = sApw + b * S::kApw + row * 16;
#pragma unroll
      for (int g = 0; g < CG; ++g) {
        uint32_t v0[16], v1[16];
        tmem_ld16_nowait(tb + static_cast<uint32_t>(g * 32), v0);
        tmem_ld16_nowait(tb + static_cast<uint32_t>(g * 32 + 16), v1);
        tmem_wait_ld(v0);
        tmem_wait_ld(v1);
        if (border) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            v0[j] += static_cast<uint32_t>(tab.dw_dbias[cls_off + g * 32 + j]);
            v1[j] += static_cast<uint32_t>(tab.dw_dbias[cls_off + g * 32 + 16 + j]);
          }
        }
        const uint4 w0 =
            requant16_pair<DWQ>(v0, tab.dw_mh, tab.dw_bs, g * 32, p.dw_lo4, p.dw_hi4);
        const uint4 w1 =
            requant16_pair<DWQ>(v1, tab.dw_mh, tab.dw_bs, g * 32 + 16, p.dw_lo4, p.dw_hi4);
        *reinterpret_cast<uint4*>(arow + (2 * g) * 2048) = w0;
        *reinterpret_cast<uint4*>(arow + (2 * g + 1) * 2048) = w1;
      }
      // The tensor core reads the tile through the async proxy.
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&apw_full[b]);

      // ---- pointwise accumulators -> int8 output
      if (lane == 0) {
        ready = mbar_wait(&pw_full[b], par, abort_flag) ? 1 : 0;
        if (!ready) fused_record_error(p.err, abort_flag, kDevErrEpiWait);
      }
      ready = __shfl_sync(0xFFFFFFFFu, ready, 0);
      if (!ready) break;
      tc_fence_after();
      int8_t* orow = p.out + (static_cast<int64_t>(rest) * p.Wo + x) * N;
      const uint32_t tp = tb + static_cast<uint32_t>(C);
      uint32_t u0[16], u1[16];
      tmem_ld16_nowait(tp, u0);
      static_assert(N % 32 == 0, "32-byte stores");
#pragma unroll
      for (int c = 0; c < N; c += 32) {
        tmem_wait_ld(u0);
        tmem_ld16_nowait(tp + static_cast<uint32_t>(c + 16), u1);
        const uint4 o0 = requant16_pair<PWQ>(u0, tab.pw_mh, tab.pw_bs, c, p.pw_lo4, p.pw_hi4);
        tmem_wait_ld(u1);
        if (c + 32 < N) tmem_ld16_nowait(tp + static_cast<uint32_t>(c + 32), u0);
        const uint4 o1 =
            requant16_pair<PWQ>(u1, tab.pw_mh, tab.pw_bs, c + 16, p.pw_lo4, p.pw_hi4);
        // 32-byte aligned: rows of N bytes, arena or checked output base.
        if (valid) st_global_v8(orow + c, o0, o1);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_empty[b]);
      b += G;
      while (b >= NB) {
        b -= NB;
        par ^= 1u;
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// [N][C] int8 -> [C/16][N][16] (K-major core-matrix order, no swizzle).
__global__ void k_pack_pw_kmajor(const int8_t* __restrict__ f, int32_t N, int32_t C,
                                 uint8_t* __restrict__ out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(N) * C) return;
  const int j = static_cast<int>(i % 16);
  const int64_t r = i / 16;
  const int n = static_cast<int>(r % N);
  const int kc = static_cast<int>(r / N);
  out[i] = static_cast<uint8_t>(f[static_cast<int64_t>(n) * C + kc * 16 + j]);
}

template <int CG, int N, int DWC, int PWC>
cudaError_t launch_pair(const CUtensorMap& m, const DwPwArgs& a, const DwPwTable& tab,
                        int grid, int smem, cudaStream_t s) {
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if ((done.load() & bit) == 0) {
    const cudaError_t e = cudaFuncSetAttribute(
        k_dwpw_s8<CG, N, DWC, PWC>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimitF);
    if (e != cudaSuccess) return e;
    done.fetch_or(bit);
  }
  k_dwpw_s8<CG, N, DWC, PWC><<<grid, DwPwShape<CG, N>::kThreads, smem, s>>>(m, a, tab);
  return cudaGetLastError();
}

template <int CG, int N, int DWQ>
cudaError_t launch_pair_pw(const CUtensorMap& m, const DwPwArgs& a, const DwPwTable& tab,
                           int pwq, int grid, int smem, cudaStream_t s) {
  switch (pwq) {
    case 0: return launch_pair<CG, N, DWQ, 0>(m, a, tab, grid, smem, s);
    case 1: return launch_pair<CG, N, DWQ, 1>(m, a, tab, grid, smem, s);
    case 2: return launch_pair<CG, N, DWQ, 2>(m, a, tab, grid, smem, s);
    default: return launch_pair<CG, N, DWQ, 3>(m, a, tab, grid, smem, s);
  }
}

template <int CG, int N>
cudaError_t launch_shape(const CUtensorMap& m, DwPwArgs a, const DwPwTable& tab, int dwq,
                         int pwq, int num_sms, cudaStream_t s) {
  using S = DwPwShape<CG, N>;
  const int overhead = 1024 + S::kFixed + 64 * 8 + 64;
  // An even count (4 for both shapes): the two MMA threads take alternate
  // tiles, so each input stage is then always read by the same thread and
  // its parity waits on the stage run in order.
  a.stages = std::min(4, (kSmemLimitF - overhead) / S::kStage) & ~1;
  if (a.stages < 2) return cudaErrorInvalidValue;
  const int smem = std::max(overhead + a.stages * S::kStage, 120 * 1024);
  const int grid = static_cast<int>(std::min<int64_t>(a.tiles, num_sms));
  if (grid <= 0) return cudaSuccess;
  switch (dwq) {
    case 0: return launch_pair_pw<CG, N, 0>(m, a, tab, pwq, grid, smem, s);
    case 1: return launch_pair_pw<CG, N, 1>(m, a, tab, pwq, grid, smem, s);
    case 2: return launch_pair_pw<CG, N, 2>(m, a, tab, pwq, grid, smem, s);
    default: return launch_pair_pw<CG, N, 3>(m, a, tab, pwq, grid, smem, s);
  }
}

}  // namespace

bool dwpw_pair_supported(const pspml_op_desc& dw, const pspml_op_desc& pw) {
  if (!dw_tc_supported(dw)) return false;
  if (pw.kind != PSPML_OP_CONV2D || pw.kernel_h != 1 || pw.kernel_w != 1 || pw.stride_h != 1 ||
      pw.stride_w != 1 || pw.pad_top != 0 || pw.pad_left != 0 || pw.pad_bottom != 0 ||
      pw.pad_right != 0)
    return false;
  if (pw.in_c != dw.out_c || pw.in_h != dw.out_h || pw.in_w != dw.out_w) return false;
  const int C = dw.in_c, N = pw.out_c;
  // Instantiated shapes (the config-3 blocks 0 and 1): C + N <= 128 keeps
  // four or more accumulator buffers (and four epilogue groups) in tensor
  // memory.  The C = N = 128 pair (two buffers, two groups, two input
  // stages) measured slower fused than as two kernels, so it is not fused.
  return (C == 32 && N == 64) || (C == 64 && N == 64);
}

size_t dwpw_packed_bytes(const pspml_op_desc& pw) {
  return static_cast<size_t>(pw.out_c) * pw.in_c;
}

cudaError_t pack_pw_kmajor(const int8_t* filter, int32_t N, int32_t C, uint8_t* out,
                           cudaStream_t s) {
  const int64_t total = static_cast<int64_t>(N) * C;
  k_pack_pw_kmajor<<<static_cast<unsigned>((total + 255) / 256), 256, 0, s>>>(filter, N, C, out);
  return cudaGetLastError();
}

cudaError_t launch_dwpw_once(const pspml_op_desc& dw, const PreparedOp& pdw,
                             const pspml_op_desc& pw, const uint8_t* wpw_packed,
                             const DwPwTable& tab, int64_t batch, const int8_t* in, int8_t* out,
                             unsigned* dev_err, int num_sms, cudaStream_t s) {
  DwPwArgs a{};
  a.tiles_x = (dw.out_w + 127) / 128;
  a.Ho = dw.out_h;
  a.Wo = dw.out_w;
  a.pad_t = dw.pad_top;
  a.pad_l = dw.pad_left;
  a.tiles = batch * dw.out_h * a.tiles_x;
  if (a.tiles >= (1ll << 31)) return cudaErrorInvalidValue;
  a.fd_tiles_x = FastDiv(static_cast<uint32_t>(a.tiles_x));
  a.fd_ho = FastDiv(static_cast<uint32_t>(a.Ho));
  a.wdw = reinterpret_cast<const uint8_t*>(pdw.wpack);
  a.wpw = wpw_packed;
  a.out = out;
  a.ycls = pdw.ycls;
  a.xcls = pdw.xcls;
  a.n_xcls = pdw.n_xcls;
  a.base_cls = pdw.base_cls;
  a.dw_lo4 = splat4(dw.act_min);
  a.dw_hi4 = splat4(dw.act_max);
  a.pw_lo4 = splat4(pw.act_min);
  a.pw_hi4 = splat4(pw.act_max);
  a.err = dev_err;
  const int dwq = ep_flags(dw.act_min, dw.act_max, dw.zp_out);
  const int pwq = ep_flags(pw.act_min, pw.act_max, pw.zp_out);

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
  const int N = pw.out_c;
  if (C == 32 && N == 64) return launch_shape<1, 64>(m, a, tab, dwq, pwq, num_sms, s);
  if (C == 64 && N == 64) return launch_shape<2, 64>(m, a, tab, dwq, pwq, num_sms, s);
  return cudaErrorInvalidValue;
}

// Tile indices are 32-bit in the kernel: larger batches run as several
// launches over batch slices.
cudaError_t launch_dwpw(const pspml_op_desc& dw, const PreparedOp& pdw, const pspml_op_desc& pw,
                        const uint8_t* wpw_packed, const DwPwTable& tab, int64_t batch,
                        const int8_t* in, int8_t* out, unsigned* dev_err, int num_sms,
                        cudaStream_t s) {
  if (dwrs_pair_supported(dw, pw))
    return launch_dwrs_pair(dw, pdw, pw, wpw_packed, tab, batch, in, out, dev_err, num_sms, s);
  const int64_t tiles_per = static_cast<int64_t>(dw.out_h) * ((dw.out_w + 127) / 128);
  const int64_t chunk = std::max<int64_t>(1, ((1ll << 31) - 1) / tiles_per);
  const int64_t in_per = static_cast<int64_t>(dw.in_h) * dw.in_w * dw.in_c;
  const int64_t out_per = static_cast<int64_t>(pw.out_h) * pw.out_w * pw.out_c;
  for (int64_t b0 = 0; b0 < batch; b0 += chunk) {
    const cudaError_t e =
        launch_dwpw_once(dw, pdw, pw, wpw_packed, tab, std::min(chunk, batch - b0),
                         in + b0 * in_per, out + b0 * out_per, dev_err, num_sms, s);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace pspml
