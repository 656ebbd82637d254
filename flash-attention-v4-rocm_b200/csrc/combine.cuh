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

__global__ void __launch_bounds__(256) combine_kernel(const __grid_constant__ CombineParams p) {
  // Launched as a programmatic dependent of the split kernel: wait until its
  // partials are written (returns at once for an ordinary launch).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane = threadIdx.x % 32;
  const int64_t total = static_cast<int64_t>(p.batch) * p.sq * p.heads;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  for (int64_t idx = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32; idx < total;
       idx += warps) {
    const int h = static_cast<int>(idx % p.heads);
    const int64_t br = idx / p.heads;  // b * sq + r
    const int r = static_cast<int>(br % p.sq);
    const int b = static_cast<int>(br / p.sq);
    const int64_t lse_idx = (static_cast<int64_t>(b) * p.heads + h) * p.sq + r;
    float mx = -INFINITY;
    float lg[kCombineCapacity];
#pragma unroll
    for (int g = 0; g < kCombineCapacity; ++g) {
      if (g < p.parts) {
        lg[g] = p.lse[g][lse_idx];
        mx = fmaxf(mx, lg[g]);
      }
    }
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    float wsum = 0.f;
    if (mx != -INFINITY) {
#pragma unroll
      for (int g = 0; g < kCombineCapacity; ++g) {
        if (g < p.parts && lg[g] != -INFINITY) {
          const float w = expf(lg[g] - mx);
          wsum += w;
          const uint2 raw = *reinterpret_cast<const uint2*>(p.o[g] + idx * 128 + lane * 4);
          const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
          const __nv_bfloat162 c = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
          acc[0] = fmaf(w, __low2float(a), acc[0]);
          acc[1] = fmaf(w, __high2float(a), acc[1]);
          acc[2] = fmaf(w, __low2float(c), acc[2]);
          acc[3] = fmaf(w, __high2float(c), acc[3]);
        }
      }
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    __nv_bfloat162 lo = __floats2bfloat162_rn(acc[0] * inv, acc[1] * inv);
    __nv_bfloat162 hi = __floats2bfloat162_rn(acc[2] * inv, acc[3] * inv);
    uint2 outw;
    outw.x = *reinterpret_cast<uint32_t*>(&lo);
    outw.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(p.out + idx * 128 + lane * 4) = outw;
    if (p.lse_out != nullptr && lane == 0) p.lse_out[lse_idx] = wsum > 0.f ? mx + logf(wsum) : -INFINITY;
  }
}

}  // namespace fav4
