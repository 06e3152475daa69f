// requant_forms.cu - throughput of the requantisation forms the epilogues use.
//
//   make -C psp-ml_b200 microbench && psp-ml_b200/_build/requant_forms
//
// Every thread requantises 16 channels per loop iteration (accumulators from
// a per-thread LCG, constants from a __grid_constant__ table at
// compile-time offsets, exactly as the tensor-core epilogues read theirs),
// packs them to int8 and folds the words into a sink.  The table kernels'
// forms are measured as the library's own helpers (kernels.h):
//   floor_split   floor form, 64-bit addend assembled from two table words
//                 ({M, D high}, {D low, shift}: the earlier entry layout)
//   floor_entry   floor form, floor_entry layout (D stored whole)
//   floor_2px     floor_entry, two accumulators per constant read
//   fast          fast form (rq_tab: bias add, sign term)
//   fast_fma_bias fast form with the bias added by a multiply-add with a
//                 run-time one (moves that add from the ALU to the FMA pipe)
// Before timing, a check kernel compares every form with TFLite's literal
// MultiplyByQuantizedMultiplier (mbqm_dev) on 2^24 accumulators x 16
// channels: the fast forms exactly, the floor forms after the clamp at the
// output zero point they are used with.
#include <cstdint>
#include <cstdio>

#include "../csrc/kernels.h"

using namespace pspml;

namespace {

constexpr int kCh = 16;

struct FormTable {
  int2 split_mh[kCh], split_bs[kCh];  // {M, D high}, {D low, shift}
  int2 fl_mh[kCh], fl_bs[kCh];        // floor_entry
  int2 fa_mh[kCh], fa_bs[kCh];        // fast: {M, C high}, {bias, shift}
  int32_t m[kCh], shift[kCh], zp[kCh], bias[kCh];  // TFLite parameters
};

enum Form { kOverhead, kFloorSplit, kFloorEntry, kFloor2px, kFast, kFastFmaBias, kForms };
const char* kNames[kForms] = {"overhead", "floor_split", "floor_entry", "floor_2px", "fast",
                              "fast_fma_bias"};

__device__ __forceinline__ int32_t floor_split(uint32_t acc, const int2& mh, const int2& bs) {
  const int64_t d = static_cast<int64_t>(
      (static_cast<uint64_t>(static_cast<uint32_t>(mh.y)) << 32) | static_cast<uint32_t>(bs.x));
  const int64_t t = static_cast<int64_t>(static_cast<int32_t>(acc)) * mh.x + d;
  return static_cast<int32_t>(t >> 32) >> bs.y;
}

__device__ __forceinline__ int32_t fast_fma_bias(int32_t acc, const int2& mh, const int2& bs,
                                                 int32_t one) {
  int32_t a;
  asm("mad.lo.s32 %0, %1, %2, %3;" : "=r"(a) : "r"(acc), "r"(one), "r"(bs.x));
  return rq_tab(a, mh, bs.y);
}

template <int F>
__device__ __forceinline__ int32_t form(int32_t acc, const FormTable& t, int c, int32_t one) {
  if constexpr (F == kOverhead) return acc;
  if constexpr (F == kFloorSplit) return floor_split(static_cast<uint32_t>(acc), t.split_mh[c], t.split_bs[c]);
  if constexpr (F == kFloorEntry || F == kFloor2px)
    return rq_floor_entry(static_cast<uint32_t>(acc), t.fl_mh[c], t.fl_bs[c]);
  if constexpr (F == kFast) return rq_tab(acc + t.fa_bs[c].x, t.fa_mh[c], t.fa_bs[c].y);
  if constexpr (F == kFastFmaBias) return fast_fma_bias(acc, t.fa_mh[c], t.fa_bs[c], one);
  return 0;
}

template <int F>
__global__ void __launch_bounds__(256) k_forms(const __grid_constant__ FormTable t, int iters,
                                               int32_t one, uint32_t* sink) {
  uint32_t x = blockIdx.x * 256 + threadIdx.x;
  uint32_t acc = 0;
  constexpr int kPx = F == kFloor2px ? 2 : 1;
  for (int it = 0; it < iters / kPx; ++it) {
    x = x * 1664525u + 1013904223u;
    const int32_t base = static_cast<int32_t>(x) >> 12;
#pragma unroll
    for (int p = 0; p < kPx; ++p) {
#pragma unroll
      for (int g = 0; g < kCh / 4; ++g) {
        int32_t r[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int c = 4 * g + k;
          r[k] = form<F>((base ^ (p * 0x5555)) + c * 977, t, c, one);
        }
        acc ^= pack_sat4(r[0], r[1], r[2], r[3]);
      }
    }
  }
  sink[blockIdx.x * 256 + threadIdx.x] = acc;
}

__global__ void k_check(const __grid_constant__ FormTable t, int n, int32_t one,
                        unsigned long long* bad) {
  unsigned long long nb[4] = {0, 0, 0, 0};
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    uint32_t h = static_cast<uint32_t>(i) * 2654435761u;
    h ^= h >> 15;
    h *= 2246822519u;
    h ^= h >> 13;
    const int32_t acc = static_cast<int32_t>(h % (1u << 22)) - (1 << 21);
    for (int c = 0; c < kCh; ++c) {
      const int32_t tfl = mbqm_dev(acc + t.bias[c], t.m[c], t.shift[c]) + t.zp[c];
      const int32_t tfl_relu = max(tfl, t.zp[c]);
      nb[0] += max(form<kFloorSplit>(acc, t, c, one), t.zp[c]) != tfl_relu;
      nb[1] += max(form<kFloorEntry>(acc, t, c, one), t.zp[c]) != tfl_relu;
      nb[2] += form<kFast>(acc, t, c, one) != tfl;
      nb[3] += form<kFastFmaBias>(acc, t, c, one) != tfl;
    }
  }
  for (int k = 0; k < 4; ++k)
    if (nb[k] != 0) atomicAdd(&bad[k], nb[k]);
}

uint64_t g_state = 0x243F6A8885A308D3ull;
uint64_t next_u64() {
  uint64_t z = (g_state += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

int check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    std::fprintf(stderr, "%s: %s\n", what, cudaGetErrorString(e));
    return 1;
  }
  return 0;
}

}  // namespace

int main() {
  FormTable t{};
  for (int c = 0; c < kCh; ++c) {
    // TFLite multipliers in [2^30, 2^31), right shifts 2..21 (fast-form
    // tables need a C low word of 2^30), any output zero point.
    const int32_t m = static_cast<int32_t>((1u << 30) + next_u64() % (1u << 30));
    const int32_t shift = -static_cast<int32_t>(2 + next_u64() % 20);
    const int32_t zp = static_cast<int32_t>(next_u64() % 256) - 128;
    const int32_t bias = static_cast<int32_t>(next_u64() % 200001) - 100000;
    const RqChannel q = make_rq(m, shift, zp);
    t.m[c] = m;
    t.shift[c] = shift;
    t.zp[c] = zp;
    t.bias[c] = bias;
    int2 mh, bs;
    floor_entry(q.m, q.c_lo, q.c_hi, q.sr, bias, &mh, &bs);
    t.fl_mh[c] = mh;
    t.fl_bs[c] = bs;
    t.split_mh[c] = make_int2(bs.x, mh.y);  // {M, D high}
    t.split_bs[c] = make_int2(mh.x, bs.y);  // {D low, shift}
    t.fa_mh[c] = make_int2(q.m, q.c_hi);
    t.fa_bs[c] = make_int2(bias, q.sr);
  }
  const int blocks = 148 * 8, iters = 2048;
  uint32_t* sink = nullptr;
  unsigned long long* bad = nullptr;
  if (check(cudaMalloc(&sink, static_cast<size_t>(blocks) * 256 * 4), "cudaMalloc") ||
      check(cudaMalloc(&bad, 4 * sizeof(unsigned long long)), "cudaMalloc") ||
      check(cudaMemset(bad, 0, 4 * sizeof(unsigned long long)), "cudaMemset"))
    return 1;
  const int n_check = 1 << 24;
  k_check<<<blocks, 256>>>(t, n_check, 1, bad);
  unsigned long long hb[4];
  if (check(cudaMemcpy(hb, bad, sizeof(hb), cudaMemcpyDeviceToHost), "check")) return 1;
  std::printf("mismatches against TFLite over %d accumulators x %d channels: floor_split %llu "
              "floor_entry %llu fast %llu fast_fma_bias %llu\n",
              n_check, kCh, hb[0], hb[1], hb[2], hb[3]);
  int sm_mhz = 0;
  cudaDeviceGetAttribute(&sm_mhz, cudaDevAttrClockRate, 0);
  sm_mhz /= 1000;
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  for (int f = 0; f < kForms; ++f) {
    float ms = 0.f;
    for (int rep = 0; rep < 3; ++rep) {
      cudaEventRecord(e0);
      switch (f) {
        case kOverhead: k_forms<kOverhead><<<blocks, 256>>>(t, iters, 1, sink); break;
        case kFloorSplit: k_forms<kFloorSplit><<<blocks, 256>>>(t, iters, 1, sink); break;
        case kFloorEntry: k_forms<kFloorEntry><<<blocks, 256>>>(t, iters, 1, sink); break;
        case kFloor2px: k_forms<kFloor2px><<<blocks, 256>>>(t, iters, 1, sink); break;
        case kFast: k_forms<kFast><<<blocks, 256>>>(t, iters, 1, sink); break;
        case kFastFmaBias: k_forms<kFastFmaBias><<<blocks, 256>>>(t, iters, 1, sink); break;
      }
      cudaEventRecord(e1);
      if (check(cudaEventSynchronize(e1), kNames[f])) return 1;
      cudaEventElapsedTime(&ms, e0, e1);
    }
    const double outs = static_cast<double>(blocks) * 256 * iters * kCh;
    std::printf("%-14s %8.3f ms  %8.1f Gout/s  %6.2f outputs/clock/SM (%d SMs, %d MHz max)\n",
                kNames[f], ms, outs / ms / 1e6, outs / (ms * 1e-3) / sms / (sm_mhz * 1e6), sms,
                sm_mhz);
  }
  const cudaError_t e = cudaDeviceSynchronize();
  std::printf("status %s\n", cudaGetErrorString(e));
  cudaFree(sink);
  cudaFree(bad);
  return e == cudaSuccess && hb[0] + hb[1] + hb[2] + hb[3] == 0 ? 0 : 1;
}
