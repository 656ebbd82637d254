// LSE-weighted combine of split-KV partial outputs (no reference counterpart;
// the reference has no split-KV path). For every (batch, row, head):
//   M = max_g LSE_g,  w_g = exp(LSE_g - M),  W = sum_g w_g
//   O = sum_g w_g O_g / W,  LSE = M + log(W)
// Slices whose LSE_g is -inf (the row saw no key of that slice) get w_g = 0.
// HBM/NVLink bound: one warp reads the 256-byte BF16 row of every part with
// coalesced 8-byte loads; partial buffers may sit on peer GPUs (plain loads).
#pragma once
#include <cuda_bf16.h>
#include <cstdint>
#include <type_traits>

namespace fav4 {

constexpr int kMaxCombineParts = 16;   // parts accepted by the public combine entry point
constexpr int kCombineCapacity = 32;   // parts the kernel handles (the one-launch split-KV uses up to 32)

struct CombineParams {
  const __nv_bfloat16* o[kCombineCapacity];
  const float* lse[kCombineCapacity];
  int parts;
  __nv_bfloat16* out;
  float* lse_out;
  int batch, heads, sq;
};

// MaxParts: compile-time bound on p.parts (2, 4, 8, 16 or 32; the host picks
// the smallest that fits). Every LSE value and the first 8 O pieces of a row
// are loaded before any is used, the rest 8 at a time, so the loads (L2, HBM
// or a peer GPU's memory) overlap instead of queueing one round trip per part;
// a small bound keeps the registers low enough for many warps per SM. Row
// indices are 32-bit when the row count allows (the host's Idx64 otherwise).
// LoadAll: every O piece of a row in one batch too (for launches with no
// more rows than warps, where a row's latency is the whole kernel).
template <int MaxParts, bool Idx64, bool LoadAll = false>
__global__ void __launch_bounds__(256) combine_kernel(const __grid_constant__ CombineParams p) {
  // Launched as a programmatic dependent of the split kernel: wait until its
  // partials are written (returns at once for an ordinary launch).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  using Idx = typename std::conditional<Idx64, int64_t, uint32_t>::type;
  constexpr int kBatch = (LoadAll || MaxParts < 8) ? MaxParts : 8;
  const int lane = threadIdx.x % 32;
  const Idx total = static_cast<Idx>(p.batch) * p.sq * p.heads;
  const Idx warps = static_cast<Idx>(gridDim.x) * (blockDim.x / 32);
  const int parts = p.parts;
  for (Idx idx = (static_cast<Idx>(blockIdx.x) * blockDim.x + threadIdx.x) / 32; idx < total; idx += warps) {
    const Idx heads = static_cast<Idx>(p.heads), sq = static_cast<Idx>(p.sq);
    const Idx br = idx / heads;  // b * sq + r
    const Idx h = idx - br * heads;
    const Idx b = br / sq;
    const Idx r = br - b * sq;
    const int64_t lse_idx = (static_cast<int64_t>(b) * p.heads + static_cast<int64_t>(h)) * p.sq + static_cast<int64_t>(r);
    const int64_t o_off = static_cast<int64_t>(idx) * 128 + lane * 4;
    float lg[MaxParts];
    uint2 raw[kBatch];
#pragma unroll
    for (int g = 0; g < MaxParts; ++g)
      if (g < parts) lg[g] = p.lse[g][lse_idx];
#pragma unroll
    for (int u = 0; u < kBatch; ++u)
      if (u < parts) raw[u] = *reinterpret_cast<const uint2*>(p.o[u] + o_off);
    float mx = -INFINITY;
#pragma unroll
    for (int g = 0; g < MaxParts; ++g)
      if (g < parts) mx = fmaxf(mx, lg[g]);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    float wsum = 0.f;
    if (mx != -INFINITY) {
#pragma unroll
      for (int g0 = 0; g0 < MaxParts; g0 += kBatch) {
        if (g0 >= parts) break;
        if (g0 > 0) {
#pragma unroll
          for (int u = 0; u < kBatch; ++u)
            if (g0 + u < parts) raw[u] = *reinterpret_cast<const uint2*>(p.o[g0 + u] + o_off);
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          const int g = g0 + u;
          if (g < parts && lg[g] != -INFINITY) {
            const float w = expf(lg[g] - mx);
            wsum += w;
            const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&raw[u].x);
            const __nv_bfloat162 c = *reinterpret_cast<const __nv_bfloat162*>(&raw[u].y);
            acc[0] = fmaf(w, __low2float(a), acc[0]);
            acc[1] = fmaf(w, __high2float(a), acc[1]);
            acc[2] = fmaf(w, __low2float(c), acc[2]);
            acc[3] = fmaf(w, __high2float(c), acc[3]);
          }
        }
      }
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    __nv_bfloat162 lo = __floats2bfloat162_rn(acc[0] * inv, acc[1] * inv);
    __nv_bfloat162 hi = __floats2bfloat162_rn(acc[2] * inv, acc[3] * inv);
    uint2 outw;
    outw.x = *reinterpret_cast<uint32_t*>(&lo);
    outw.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(p.out + o_off) = outw;
    if (p.lse_out != nullptr && lane == 0) p.lse_out[lse_idx] = wsum > 0.f ? mx + logf(wsum) : -INFINITY;
  }
}

}  // namespace fav4
