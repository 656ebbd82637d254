// Test-only probe library (libfav4_probe.so). Each probe exercises one sm_100a
// building block of the attention kernel in isolation so a layout mistake is
// caught by a small exact test instead of a wrong attention output:
//
//  fav4_probe_tma_load   one 128-row BSHD tile through the same TMA map and
//                        128-byte swizzle as the kernel, un-swizzled to global.
//                        The B200 counterpart of the reference's TDM load test
//                        (tests/bshd_tdm.hip:8-45): head offset, row stride
//                        H*128 and zero fill of rows past the end.
//  fav4_probe_gemm_qk    D = A B^T with A, B K-major in shared memory: the
//                        descriptors the kernel uses for S = Q K^T.
//  fav4_probe_gemm_pv    D = P V with P in TMEM (written by tcgen05.st) and V
//                        MN-major in shared memory: the O += P V step.
//  fav4_probe_bounded_wait  waits on an mbarrier that nothing arrives on; the
//                        bounded wait must give up, set the status word and
//                        let the kernel finish (failure detection test).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "attn_fwd_sm100.cuh"
#include "sm100.cuh"
#include "tensor_map.h"

namespace fav4 {
namespace probe {

__device__ uint32_t g_probe_status;

constexpr int kProbeSmem = 3 * kTileBytes + 1024 + 64;

// Shared tile -> row-major global [128][128] bf16, undoing the 128B swizzle:
// row r, 16-byte chunk c of a half lives at r*128 + ((c ^ (r % 8)) * 16).
__device__ void unswizzle_tile(const uint8_t* tile, __nv_bfloat16* out) {
  for (int idx = threadIdx.x; idx < 128 * 16; idx += blockDim.x) {
    const int r = idx / 16, c16 = idx % 16;  // 16 chunks of 8 bf16 per row
    const int half = c16 / 8, c = c16 % 8;
    const uint4 v = *reinterpret_cast<const uint4*>(tile + half * kBoxBytes + r * 128 + ((c ^ (r % 8)) * 16));
    *reinterpret_cast<uint4*>(out + r * 128 + c16 * 8) = v;
  }
}

__global__ void __launch_bounds__(128) tma_load_kernel(const __grid_constant__ CUtensorMap map, int head,
                                                       __nv_bfloat16* out, uint64_t limit_ns) {
  extern __shared__ uint8_t raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  const uint32_t bar = smem_addr(smem + 3 * kTileBytes);
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + 3 * kTileBytes + 16);
  if (threadIdx.x == 0) {
    *abort_flag = 0;
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  WaitCtl ctl{abort_flag, &g_probe_status, limit_ns};
  bool ok = true;
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(bar, kTileBytes);
    const uint64_t pol = policy_evict_first();
    tma_load_4d(smem_addr(smem), &map, bar, 0, head, 0, 0, pol);
    tma_load_4d(smem_addr(smem) + kBoxBytes, &map, bar, 64, head, 0, 0, pol);
  }
  ok = mbar_wait(bar, 0, ctl, kStatusTimeoutProbe);
  __syncthreads();
  if (ok) unswizzle_tile(smem, out);
}

// Loads a 128x128 bf16 tile (rows of 128 contiguous elements) as a BSHD
// tensor [1, 128, 1, 128] with the kernel's TMA map.
__device__ void load_tile(uint8_t* smem, uint32_t dst, const CUtensorMap* map, uint32_t bar) {
  tma_load_4d(dst, map, bar, 0, 0, 0, 0, policy_evict_first());
  tma_load_4d(dst + kBoxBytes, map, bar, 64, 0, 0, 0, policy_evict_first());
}

// mode 0: D = A B^T (SS, both K-major). mode 1: D = P V (TS, P from TMEM, V MN-major).
__global__ void __launch_bounds__(128) gemm_kernel(const __grid_constant__ CUtensorMap ma,
                                                   const __grid_constant__ CUtensorMap mb, int mode,
                                                   const __nv_bfloat16* p_rows, float* d, uint64_t limit_ns) {
  extern __shared__ uint8_t raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sa = smem_addr(smem), sb = sa + kTileBytes;
  const uint32_t bar_load = smem_addr(smem + 3 * kTileBytes);
  const uint32_t bar_mma = bar_load + 8;
  uint32_t* holder = reinterpret_cast<uint32_t*>(smem + 3 * kTileBytes + 16);
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + 3 * kTileBytes + 20);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    *abort_flag = 0;
    mbar_init(bar_load, 1);
    mbar_init(bar_mma, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_addr(holder), 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *holder;  // D at [0,128), P at [128,192)
  WaitCtl ctl{abort_flag, &g_probe_status, limit_ns};
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  if (mode == 1) {
    // P row r (= TMEM lane r) as 64 packed bf16 pairs.
    const int r = threadIdx.x;
    uint32_t pk[2][32];
#pragma unroll
    for (int c = 0; c < 64; ++c) {
      const __nv_bfloat16 lo = p_rows[r * 128 + 2 * c], hi = p_rows[r * 128 + 2 * c + 1];
      pk[c / 32][c % 32] = static_cast<uint32_t>(__bfloat16_as_ushort(lo)) |
                           (static_cast<uint32_t>(__bfloat16_as_ushort(hi)) << 16);
    }
    tmem_st32(tmem + lane_off + 128, pk[0]);
    tmem_st32(tmem + lane_off + 160, pk[1]);
    tmem_st_wait();
  }
  tc_fence_before();
  __syncthreads();
  bool ok = true;
  if (threadIdx.x == 0) {
    tc_fence_after();
    mbar_arrive_expect_tx(bar_load, mode == 0 ? 2 * kTileBytes : kTileBytes);
    if (mode == 0) load_tile(smem, sa, &ma, bar_load);
    load_tile(smem, sb, &mb, bar_load);
    ok = mbar_wait(bar_load, 0, ctl, kStatusTimeoutProbe);
    if (ok) {
      if (mode == 0) {
        constexpr uint32_t idesc = make_idesc_bf16(128, 128, false);
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = (k / 4) * kBoxBytes + (k % 4) * 32;
          umma_ss(tmem, make_sdesc_sw128(sa + off, 16, 1024), make_sdesc_sw128(sb + off, 16, 1024), idesc,
                  k > 0 ? 1u : 0u);
        }
      } else {
        constexpr uint32_t idesc = make_idesc_bf16(128, 128, true);
        for (int k = 0; k < 8; ++k)
          umma_ts(tmem, tmem + 128 + k * 8, make_sdesc_sw128(sb + k * 2048, kBoxBytes, 1024), idesc,
                  k > 0 ? 1u : 0u);
      }
    }
    tc_commit(bar_mma);
  }
  __syncthreads();
  volatile uint32_t no_abort = 0;
  WaitCtl drain{&no_abort, &g_probe_status, limit_ns};
  ok = warp_wait(bar_mma, 0, drain, kStatusTimeoutProbe) && !*abort_flag;
  tc_fence_after();
  if (ok) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t r[32];
      tmem_ld32(tmem + lane_off + c * 32, r);
      tmem_ld_wait();
      for (int e = 0; e < 32; ++e) d[threadIdx.x * 128 + c * 32 + e] = __uint_as_float(r[e]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// One thread waits on a barrier that is initialised for one arrival that
// never comes; the bounded wait must return false within `limit_ns`.
__global__ void bounded_wait_kernel(uint64_t limit_ns, int* waited_out) {
  __shared__ __align__(8) uint64_t bar_storage;
  __shared__ uint32_t abort_word;
  if (threadIdx.x == 0) {
    abort_word = 0;
    mbar_init(smem_addr(&bar_storage), 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    WaitCtl ctl{&abort_word, &g_probe_status, limit_ns};
    const uint64_t t0 = global_timer_ns();
    const bool ok = mbar_wait(smem_addr(&bar_storage), 0, ctl, kStatusTimeoutProbe);
    waited_out[0] = ok ? 1 : 0;
    waited_out[1] = static_cast<int>((global_timer_ns() - t0) / 1000);  // microseconds
    waited_out[2] = static_cast<int>(abort_word);
  }
}

uint64_t limit_ns() { return 2000ull * 1000000ull; }

}  // namespace probe
}  // namespace fav4

using namespace fav4;

extern "C" int fav4_probe_tma_load(const void* input, void* output, int rows, int heads, int head,
                                   cudaStream_t stream) {
  if (!input || !output || rows <= 0 || heads <= 0 || head < 0 || head >= heads) return cudaErrorInvalidValue;
  CUtensorMap map;
  if (!encode_bshd(&map, input, 1, rows, heads)) return cudaErrorInvalidValue;
  cudaError_t e =
      cudaFuncSetAttribute(probe::tma_load_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, probe::kProbeSmem);
  if (e != cudaSuccess) return e;
  probe::tma_load_kernel<<<1, 128, probe::kProbeSmem, stream>>>(map, head, static_cast<__nv_bfloat16*>(output),
                                                                probe::limit_ns());
  return cudaGetLastError();
}

static int gemm_probe(const void* a, const void* b, float* d, int mode, cudaStream_t stream) {
  CUtensorMap ma, mb;
  if (!encode_bshd(&ma, a, 1, 128, 1) || !encode_bshd(&mb, b, 1, 128, 1)) return cudaErrorInvalidValue;
  cudaError_t e =
      cudaFuncSetAttribute(probe::gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, probe::kProbeSmem);
  if (e != cudaSuccess) return e;
  probe::gemm_kernel<<<1, 128, probe::kProbeSmem, stream>>>(ma, mb, mode, static_cast<const __nv_bfloat16*>(a), d,
                                                            probe::limit_ns());
  return cudaGetLastError();
}

// a: [128 rows][128 k] bf16, b: [128 cols][128 k] bf16 -> d[128][128] = a b^T (fp32)
extern "C" int fav4_probe_gemm_qk(const void* a, const void* b, float* d, cudaStream_t stream) {
  if (!a || !b || !d) return cudaErrorInvalidValue;
  return gemm_probe(a, b, d, 0, stream);
}

// p: [128 rows][128 k] bf16, v: [128 k][128 n] bf16 -> d[128][128] = p v (fp32)
extern "C" int fav4_probe_gemm_pv(const void* p, const void* v, float* d, cudaStream_t stream) {
  if (!p || !v || !d) return cudaErrorInvalidValue;
  return gemm_probe(p, v, d, 1, stream);
}

// out (device int[3]): {wait succeeded, microseconds waited, abort flag}
extern "C" int fav4_probe_bounded_wait(int limit_us, int* out, cudaStream_t stream) {
  if (!out || limit_us <= 0) return cudaErrorInvalidValue;
  probe::bounded_wait_kernel<<<1, 32, 0, stream>>>(static_cast<uint64_t>(limit_us) * 1000ull, out);
  return cudaGetLastError();
}

extern "C" int fav4_probe_status(int clear) {
  uint32_t v = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  if (cudaMemcpyFromSymbol(&v, probe::g_probe_status, sizeof(v)) != cudaSuccess) return -1;
  if (clear) {
    const uint32_t zero = 0;
    if (cudaMemcpyToSymbol(probe::g_probe_status, &zero, sizeof(zero)) != cudaSuccess) return -1;
  }
  return static_cast<int>(v & 0x7fffffffu);
}
