// Host side of the C ABI declared in include/fav4_bshd.h.
//
// fav4_bshd_forward keeps the reference's argument checks one for one
// (src/bshd.hip:27-34), its Auto rule (src/bshd.hip:23-25) and its return
// convention (invalid -> cudaErrorInvalidValue, else the launch status,
// src/bshd.hip:17-19), then encodes TMA tensor maps for the BSHD tensors and
// launches the persistent sm_100a kernel on the caller's stream. Nothing is
// allocated and the host never synchronises.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <climits>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <mutex>

#include "attn_fwd_sm100.cuh"
#include "attn_fwd_wide_sm100.cuh"
#include "attn_bwd_sm100.cuh"
#include "attn_bwd_fused_sm100.cuh"
#include "combine.cuh"
#include "tensor_map.h"
#include "fav4_bshd.h"

namespace fav4 {

__device__ uint32_t g_status;  // per-device pipeline status word (see fav4_bshd_pipeline_status)

namespace {

constexpr int kMaxDevices = 64;

uint64_t wait_limit_ns() {
  static uint64_t limit = [] {
    const char* env = std::getenv("FAV4_WAIT_LIMIT_MS");
    long ms = env ? std::strtol(env, nullptr, 10) : 0;
    if (ms <= 0) ms = 2000;
    return static_cast<uint64_t>(ms) * 1000000ull;
  }();
  return limit;
}

size_t round256(size_t n) { return (n + 255) & ~size_t(255); }

struct DeviceInfo {
  int sms = 0;
  uint32_t* status = nullptr;
};

// Per-device facts fetched once: SM count and the device address of g_status.
bool device_info(int dev, DeviceInfo* out) {
  static std::mutex mu;
  static DeviceInfo cache[kMaxDevices];
  static bool ready[kMaxDevices] = {};
  if (dev < 0 || dev >= kMaxDevices) return false;
  std::lock_guard<std::mutex> lock(mu);
  if (!ready[dev]) {
    DeviceInfo d;
    if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return false;
    void* addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_status) != cudaSuccess) return false;
    d.status = static_cast<uint32_t*>(addr);
    cache[dev] = d;
    ready[dev] = true;
  }
  *out = cache[dev];
  return true;
}

// The reference's argument checks (src/bshd.hip:27-34).
bool args_valid(const Fav4Args* a, int causal, int config) {
  if (!a || !a->q || !a->k || !a->v || !a->o || a->batch <= 0 || a->heads <= 0 || a->sq <= 0 || a->sk <= 0 ||
      (causal != 0 && causal != 1) || config < 0 || config > 3 || !std::isfinite(a->scale) || a->scale <= 0)
    return false;
  if (a->batch > INT_MAX / a->heads || a->heads > INT_MAX / 128 || a->sq > INT_MAX / (a->heads * 128) ||
      a->sk > INT_MAX / (a->heads * 128) ||
      ((reinterpret_cast<uintptr_t>(a->q) | reinterpret_cast<uintptr_t>(a->k) | reinterpret_cast<uintptr_t>(a->v) |
        reinterpret_cast<uintptr_t>(a->o)) &
       15))
    return false;
  // LSE is written with 4-byte stores: a misaligned pointer would fault on the GPU
  if (reinterpret_cast<uintptr_t>(a->lse) & 3) return false;
  return true;
}

// Causal work-tile schedule (see sched_tile in attn_fwd_sm100.cuh): the number
// of head-pair work items when pairing gives the shorter estimated makespan
// on `sms` persistent CTAs, else 0 (plain stride). A tile costs its K/V steps
// plus one for its fill and drain. Both schedules are simulated (tile costs
// depend only on the query block); decisions are cached per shape.
int paired_items(int batch, int heads, int sq, int sk, int qtiles, int sms) {
  const int rows = qtiles * kBlockM;
  const int nm = (sq + rows - 1) / rows;
  const int64_t tiles = static_cast<int64_t>(batch) * heads * nm;
  const int64_t items = static_cast<int64_t>(batch) * heads * ((nm + 1) / 2);
  if (nm < 2 || items > INT_MAX || sms <= 0) return 0;
  struct Entry {
    int batch, heads, sq, sk, qtiles, sms, items;
  };
  constexpr int kCache = 32;
  static std::mutex mu;
  static Entry cache[kCache];
  static int used = 0, next = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    for (int e = 0; e < used; ++e) {
      const Entry& c = cache[e];
      if (c.batch == batch && c.heads == heads && c.sq == sq && c.sk == sk && c.qtiles == qtiles && c.sms == sms)
        return c.items;
    }
  }
  auto cost = [&](int mb) -> int64_t {  // K/V steps of the work tile at query block mb, + 1
    int n = 0;
    for (int i = 0; i < qtiles; ++i) {
      const int r0 = mb * rows + i * kBlockM;
      if (r0 >= sq) continue;
      const int hi = r0 + kBlockM < sk ? r0 + kBlockM : sk;
      const int ni = (hi + kBlockN - 1) / kBlockN;
      n = ni > n ? ni : n;
    }
    return n > 0 ? n + 1 : 0;
  };
  constexpr int kMaxGrid = 1024;
  int64_t load[kMaxGrid];
  // plain stride: tile t has query block nm - 1 - (t % (heads * nm)) / heads
  const int g1 = static_cast<int>(tiles < sms ? tiles : sms);
  const int g2 = static_cast<int>(items < sms ? items : sms);
  if (g1 > kMaxGrid || g2 > kMaxGrid) return 0;
  int64_t span_stride = 0, span_pairs = 0;
  for (int c = 0; c < g1; ++c) load[c] = 0;
  for (int64_t t = 0; t < tiles; ++t) load[t % g1] += cost(nm - 1 - static_cast<int>(t % (heads * nm)) / heads);
  for (int c = 0; c < g1; ++c) span_stride = load[c] > span_stride ? load[c] : span_stride;
  for (int c = 0; c < g2; ++c) load[c] = 0;
  const int per_b = ((nm + 1) / 2) * heads;
  for (int64_t it = 0; it < items; ++it) {
    const int q = static_cast<int>(it % per_b) / heads;
    load[it % g2] += cost(nm - 1 - q) + (nm - 1 - q != q ? cost(q) : 0);
  }
  for (int c = 0; c < g2; ++c) span_pairs = load[c] > span_pairs ? load[c] : span_pairs;
  // a CTA lists at most kMaxListTiles paired tiles (two per item)
  const bool fits = 2 * ((items + g2 - 1) / g2) <= kMaxListTiles;
  const int result = (fits && span_pairs < span_stride) ? static_cast<int>(items) : 0;
  std::lock_guard<std::mutex> lock(mu);
  cache[next] = Entry{batch, heads, sq, sk, qtiles, sms, result};
  next = (next + 1) % kCache;
  used = used < kCache ? used + 1 : used;
  return result;
}

// B200 tilings behind the reference's config ids (include/fav4_bshd.h:17-18):
//   1: one 128-row Q tile per CTA, 2 K/V ring slots, MUFU exp2 only
//   2: two 128-row Q tiles per CTA sharing each K/V tile (ping-pong),
//      2 ring slots, 1/4 of exp2 on the FMA polynomial (Auto for sq >= 128)
//   3: as 2 with every exp2 on MUFU (no polynomial)
// Varlen: a.sq / a.sk are the packed row counts, a.batch the number of
// sequences, cu_q / cu_k their device offsets and max_sq the longest query
// sequence (it sizes the tile grid).
template <bool Causal, int QTiles, int Slots, int PolyPer8, bool Split, bool Varlen = false>
int launch_fwd(const Fav4Args& a, int kv_heads, int kv_begin, int kv_end, int splits, cudaStream_t stream,
               const int* cu_q = nullptr, const int* cu_k = nullptr, int max_sq = 0) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  DeviceInfo info;
  if (!device_info(dev, &info)) return cudaErrorInvalidDevice;
  constexpr int smem = SmemLayout<QTiles, Slots>::kAlloc;
  constexpr bool kPairable = Causal && !Split && !Varlen;
  const int items = kPairable ? paired_items(a.batch, a.heads, a.sq, a.sk, QTiles, info.sms) : 0;
  // [0]: plain schedule, [1]: paired schedule (the same kernel where it does not apply)
  decltype(&attn_fwd_sm100_kernel<Causal, QTiles, Slots, PolyPer8, Split, Varlen, false>) variants[2] = {
      attn_fwd_sm100_kernel<Causal, QTiles, Slots, PolyPer8, Split, Varlen, false>,
      attn_fwd_sm100_kernel<Causal, QTiles, Slots, PolyPer8, Split, Varlen, kPairable>};
  auto kernel = variants[items > 0 ? 1 : 0];
  {
    // both variants get their attribute on the first call, so later calls set
    // nothing whichever schedule they pick
    static std::mutex mu;
    static bool attr_set[kMaxDevices] = {};
    std::lock_guard<std::mutex> lock(mu);
    if (!attr_set[dev]) {
      for (auto fn : variants) {
        e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
      }
      attr_set[dev] = true;
    }
  }
  CUtensorMap tq, tk, tv, to;
  const int mb = Varlen ? 1 : a.batch;  // packed sequences: one batch entry of sq / sk rows
  if (!encode_bshd(&tq, a.q, mb, a.sq, a.heads) || !encode_bshd(&tk, a.k, mb, a.sk, kv_heads) ||
      !encode_bshd(&tv, a.v, mb, a.sk, kv_heads) || !encode_bshd(&to, a.o, mb * splits, a.sq, a.heads))
    return cudaErrorInvalidValue;
  FwdParams p;
  p.o = static_cast<__nv_bfloat16*>(a.o);
  p.lse = a.lse;
  p.batch = a.batch;
  p.heads = a.heads;
  p.sq = a.sq;
  p.sk = a.sk;
  p.kv_group = a.heads / kv_heads;
  p.kv_begin = kv_begin;
  p.kv_end = kv_end;
  p.splits = splits;
  // whole 128-key tiles per split
  p.kv_chunk = ((kv_end - kv_begin + splits - 1) / splits + kBlockN - 1) / kBlockN * kBlockN;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.num_mblocks = ((Varlen ? max_sq : a.sq) + QTiles * kBlockM - 1) / (QTiles * kBlockM);
  p.cu_q = cu_q;
  p.cu_k = cu_k;
  const int64_t base = static_cast<int64_t>(a.batch) * a.heads * p.num_mblocks;
  const int64_t tiles = base * splits;
  if (tiles > INT_MAX) return cudaErrorInvalidValue;
  p.num_base_tiles = static_cast<int>(base);
  p.num_tiles = static_cast<int>(tiles);
  p.num_items = items;
  p.status = info.status;
  p.wait_limit_ns = wait_limit_ns();
  const int64_t work = p.num_items > 0 ? p.num_items : tiles;
  const int grid = static_cast<int>(work < info.sms ? work : info.sms);
  kernel<<<grid, 384, smem, stream>>>(tq, tk, tv, to, p);
  return cudaGetLastError();
}

// Wide-step kernel (attn_fwd_wide_sm100.cuh): one 128-row Q tile per CTA,
// 256 keys per step; whole key range, no splits, no packed sequences; dense
// only (Auto never picks it for causal launches).
template <bool Causal>
int launch_fwd_wide(const Fav4Args& a, int kv_heads, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  DeviceInfo info;
  if (!device_info(dev, &info)) return cudaErrorInvalidDevice;
  constexpr int smem = WideLayout::kAlloc;
  auto kernel = attn_fwd_wide_kernel<Causal, 2>;  // 2 of 8 exp2 columns on the polynomial, as config 2
  {
    static std::mutex mu;
    static bool attr_set[kMaxDevices] = {};
    std::lock_guard<std::mutex> lock(mu);
    if (!attr_set[dev]) {
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
      attr_set[dev] = true;
    }
  }
  CUtensorMap tq, tk, tv;
  if (!encode_bshd(&tq, a.q, a.batch, a.sq, a.heads) || !encode_bshd(&tk, a.k, a.batch, a.sk, kv_heads, kWideN) ||
      !encode_bshd(&tv, a.v, a.batch, a.sk, kv_heads, kWideN))
    return cudaErrorInvalidValue;
  FwdParams p = {};
  p.o = static_cast<__nv_bfloat16*>(a.o);
  p.lse = a.lse;
  p.batch = a.batch;
  p.heads = a.heads;
  p.sq = a.sq;
  p.sk = a.sk;
  p.kv_group = a.heads / kv_heads;
  p.kv_begin = 0;
  p.kv_end = a.sk;
  p.splits = 1;
  p.kv_chunk = a.sk;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.num_mblocks = (a.sq + kBlockM - 1) / kBlockM;
  const int64_t tiles = static_cast<int64_t>(a.batch) * a.heads * p.num_mblocks;
  if (tiles > INT_MAX) return cudaErrorInvalidValue;
  p.num_base_tiles = static_cast<int>(tiles);
  p.num_tiles = static_cast<int>(tiles);
  p.num_items = 0;
  p.status = info.status;
  p.wait_limit_ns = wait_limit_ns();
  const int grid = static_cast<int>(tiles < info.sms ? tiles : info.sms);
  kernel<<<grid, 384, smem, stream>>>(tq, tk, tv, p);
  return cudaGetLastError();
}

template <bool Causal>
int dispatch(const Fav4Args& a, int config, int kv_begin, int kv_end, cudaStream_t stream, int kv_heads = 0,
             int splits = 1) {
  if (kv_heads == 0) kv_heads = a.heads;
  if (splits > 1) {  // the work tiles carry a key-range index
    switch (config) {
      case 1: return launch_fwd<Causal, 1, 2, 0, true, false>(a, kv_heads, kv_begin, kv_end, splits, stream);
      case 2: return launch_fwd<Causal, 2, 2, 2, true, false>(a, kv_heads, kv_begin, kv_end, splits, stream);
      case 3: return launch_fwd<Causal, 2, 2, 0, true, false>(a, kv_heads, kv_begin, kv_end, splits, stream);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (config) {
    case 1: return launch_fwd<Causal, 1, 2, 0, false, false>(a, kv_heads, kv_begin, kv_end, 1, stream);
    case 2: return launch_fwd<Causal, 2, 2, 2, false, false>(a, kv_heads, kv_begin, kv_end, 1, stream);
    case 3: return launch_fwd<Causal, 2, 2, 0, false, false>(a, kv_heads, kv_begin, kv_end, 1, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace
}  // namespace fav4

extern "C" int fav4_bshd_select_config(const Fav4Args* a) { return a->sq < 128 ? 1 : 2; }

namespace fav4 {
// Auto of the whole-key-range entries (fav4_bshd_forward, _gqa, _host and the
// one-launch split-KV ones): the reference's rule, then one-Q-tile work tiles
// when two-tile ones (without key splits) would occupy at most half of the SMs.
// With so few tiles the SMs would idle anyway, and twice as many 128-row tiles
// spread the work wider (measured +8-15 % at B4 S512 and B8 S256, while at 0.86
// of the SMs (B4 S1024) two-tile tiles are still faster dense); decode shapes
// with Sq = 128 get the double-buffered one-tile kernel instead of a two-tile
// one whose second tile is empty.
//
// Dense launches of the full key range (allow_wide: fav4_bshd_forward, _gqa,
// _host) then take the wide-step kernel (kConfigWide) when its 128-row tiles
// fill the last wave so much better that its 0.92x per-tile speed (B32 S4096)
// still wins: waves(128-row tiles) < 1.84 x waves(256-row tiles), with Sk >=
// 2048 (shorter key ranges favour the two-tile kernel). Measured: B4 S4096
// 1.05x, B2 S8192 1.08x, B1 S16384 1.08x, B5 S4096 1.02x; B3 S4096 and B4
// S3072, where the rule keeps config 2, would lose 3-5 %.
constexpr int kConfigWide = 4;  // internal: never accepted from callers
int auto_config(const Fav4Args* a, bool causal = true, bool allow_wide = false) {
  const int c = fav4_bshd_select_config(a);
  int dev = 0;
  DeviceInfo info;
  if (c != 2 || cudaGetDevice(&dev) != cudaSuccess || !device_info(dev, &info)) return c;
  const int64_t tiles = static_cast<int64_t>(a->batch) * a->heads * ((a->sq + 2 * kBlockM - 1) / (2 * kBlockM));
  if (2 * tiles <= info.sms) return 1;
  if (allow_wide && !causal && a->sk >= 2048) {
    const int64_t tiles_w = static_cast<int64_t>(a->batch) * a->heads * ((a->sq + kBlockM - 1) / kBlockM);
    const int64_t waves = (tiles + info.sms - 1) / info.sms, waves_w = (tiles_w + info.sms - 1) / info.sms;
    if (waves_w * 25 < waves * 46) return kConfigWide;
  }
  return c;
}
}  // namespace fav4

namespace fav4 {
namespace {

template <bool Causal>
int dispatch_varlen(const Fav4Args& a, int config, int kv_heads, const int* cu_q, const int* cu_k, int max_sq,
                    cudaStream_t stream) {
  switch (config) {
    case 1: return launch_fwd<Causal, 1, 2, 0, false, true>(a, kv_heads, 0, a.sk, 1, stream, cu_q, cu_k, max_sq);
    case 2: return launch_fwd<Causal, 2, 2, 2, false, true>(a, kv_heads, 0, a.sk, 1, stream, cu_q, cu_k, max_sq);
    case 3: return launch_fwd<Causal, 2, 2, 0, false, true>(a, kv_heads, 0, a.sk, 1, stream, cu_q, cu_k, max_sq);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace
}  // namespace fav4

extern "C" int fav4_bshd_forward_varlen(const Fav4VarlenArgs* v, int causal, int config, cudaStream_t stream) {
  if (!v || !v->cu_seqlens_q || !v->cu_seqlens_k || v->max_sq <= 0 || v->max_sq > v->total_q || v->kv_heads < 1 ||
      v->heads < 1 || v->kv_heads > v->heads || v->heads % v->kv_heads ||
      (reinterpret_cast<uintptr_t>(v->cu_seqlens_q) & 3) || (reinterpret_cast<uintptr_t>(v->cu_seqlens_k) & 3))
    return cudaErrorInvalidValue;
  Fav4Args a;
  a.q = v->q;
  a.k = v->k;
  a.v = v->v;
  a.o = v->o;
  a.lse = v->lse;
  a.batch = v->batch;
  a.heads = v->heads;
  a.sq = v->total_q;
  a.sk = v->total_k;
  a.scale = v->scale;
  if (!fav4::args_valid(&a, causal, config) || (v->lse && (reinterpret_cast<uintptr_t>(v->lse) & 3)))
    return cudaErrorInvalidValue;
  if (config == 0) config = v->max_sq < 128 ? 1 : 2;
  return causal ? fav4::dispatch_varlen<true>(a, config, v->kv_heads, v->cu_seqlens_q, v->cu_seqlens_k, v->max_sq,
                                              stream)
                : fav4::dispatch_varlen<false>(a, config, v->kv_heads, v->cu_seqlens_q, v->cu_seqlens_k, v->max_sq,
                                               stream);
}

extern "C" int fav4_bshd_forward(const Fav4Args* a, int causal, int config, cudaStream_t stream) {
  if (!fav4::args_valid(a, causal, config)) return cudaErrorInvalidValue;
  if (config == 0) config = fav4::auto_config(a, causal != 0, true);
  if (config == fav4::kConfigWide) return fav4::launch_fwd_wide<false>(*a, a->heads, stream);
  return causal ? fav4::dispatch<true>(*a, config, 0, a->sk, stream)
                : fav4::dispatch<false>(*a, config, 0, a->sk, stream);
}

extern "C" int fav4_bshd_forward_wide(const Fav4Args* a, cudaStream_t stream) {
  if (!fav4::args_valid(a, 0, 0)) return cudaErrorInvalidValue;
  return fav4::launch_fwd_wide<false>(*a, a->heads, stream);
}

extern "C" int fav4_bshd_forward_gqa(const Fav4Args* a, int kv_heads, int causal, int config,
                                     cudaStream_t stream) {
  if (!fav4::args_valid(a, causal, config) || kv_heads < 1 || kv_heads > a->heads || a->heads % kv_heads)
    return cudaErrorInvalidValue;
  if (config == 0) config = fav4::auto_config(a, causal != 0, true);
  if (config == fav4::kConfigWide) return fav4::launch_fwd_wide<false>(*a, kv_heads, stream);
  return causal ? fav4::dispatch<true>(*a, config, 0, a->sk, stream, kv_heads)
                : fav4::dispatch<false>(*a, config, 0, a->sk, stream, kv_heads);
}

extern "C" int fav4_bshd_forward_partial(const Fav4Args* a, int causal, int config, int kv_begin, int kv_end,
                                         cudaStream_t stream) {
  if (!fav4::args_valid(a, causal, config) || !a->lse || kv_begin < 0 || kv_end <= kv_begin || kv_end > a->sk ||
      (reinterpret_cast<uintptr_t>(a->lse) & 3))
    return cudaErrorInvalidValue;
  if (config == 0) config = fav4_bshd_select_config(a);
  return causal ? fav4::dispatch<true>(*a, config, kv_begin, kv_end, stream)
                : fav4::dispatch<false>(*a, config, kv_begin, kv_end, stream);
}

namespace fav4 {
namespace {

// The combine launch for 1..kCombineCapacity parts (arguments validated as fav4_bshd_combine does).
// after_split: the launch directly follows the one-launch split kernel on the
// same stream, so it goes out as a programmatic dependent launch: it is
// scheduled while the split kernel's last CTAs run and waits in
// griddepcontrol.wait until that kernel's writes are visible.
int combine_parts(const void* const* o_parts, const float* const* lse_parts, int parts, void* o, float* lse,
                  int batch, int heads, int sq, cudaStream_t stream, bool after_split = false) {
  if (!o_parts || !lse_parts || !o || parts < 1 || parts > kCombineCapacity || batch <= 0 || heads <= 0 ||
      sq <= 0 || batch > INT_MAX / heads || heads > INT_MAX / 128 || sq > INT_MAX / (heads * 128) ||
      (reinterpret_cast<uintptr_t>(o) & 15) || (reinterpret_cast<uintptr_t>(lse) & 3))
    return cudaErrorInvalidValue;
  CombineParams p = {};
  for (int g = 0; g < parts; ++g) {
    if (!o_parts[g] || !lse_parts[g] || (reinterpret_cast<uintptr_t>(o_parts[g]) & 15) ||
        (reinterpret_cast<uintptr_t>(lse_parts[g]) & 3))
      return cudaErrorInvalidValue;
    p.o[g] = static_cast<const __nv_bfloat16*>(o_parts[g]);
    p.lse[g] = lse_parts[g];
  }
  p.parts = parts;
  p.out = static_cast<__nv_bfloat16*>(o);
  p.lse_out = lse;
  p.batch = batch;
  p.heads = heads;
  p.sq = sq;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  DeviceInfo info;
  if (!device_info(dev, &info)) return cudaErrorInvalidDevice;
  const int64_t rows = static_cast<int64_t>(batch) * sq * heads;
  const int64_t want = (rows + 7) / 8;  // 8 warps per block, one row per warp per pass
  const int64_t cap = static_cast<int64_t>(info.sms) * 8;
  const int grid = static_cast<int>(want < cap ? want : cap);
  // the smallest compile-time part bound that fits, 32-bit row indices when they suffice
  void (*kernel)(CombineParams);
  const bool idx64 = rows > static_cast<int64_t>(INT32_MAX);
  if (parts <= 2) kernel = idx64 ? combine_kernel<2, true> : combine_kernel<2, false>;
  else if (parts <= 4) kernel = idx64 ? combine_kernel<4, true> : combine_kernel<4, false>;
  else if (parts <= 8) kernel = idx64 ? combine_kernel<8, true> : combine_kernel<8, false>;
  else if (parts <= 16) kernel = idx64 ? combine_kernel<16, true> : combine_kernel<16, false>;
  else kernel = idx64 ? combine_kernel<32, true> : combine_kernel<32, false>;
  if (parts > 8 && rows <= static_cast<int64_t>(grid) * 8)  // one row per warp: all loads at once
    kernel = parts <= 16 ? combine_kernel<16, false, true> : combine_kernel<32, false, true>;
  if (!after_split) {
    kernel<<<grid, 256, 0, stream>>>(p);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, p);
}

}  // namespace
}  // namespace fav4

extern "C" int fav4_bshd_combine(const void* const* o_parts, const float* const* lse_parts, int parts, void* o,
                                 float* lse, int batch, int heads, int sq, cudaStream_t stream) {
  if (parts > fav4::kMaxCombineParts) return cudaErrorInvalidValue;
  return fav4::combine_parts(o_parts, lse_parts, parts, o, lse, batch, heads, sq, stream);
}

// --------------------------------------------------------------------------
// Forward from host buffers, pipelined over batch chunks: the copy of chunk
// c+1 to the device, the forwards of chunk c and the copy of chunk c-1 back
// to the host run at the same time (two copy streams beside the caller's
// stream; PCIe copies in both directions overlap each other and the kernels).
namespace fav4 {
namespace {

constexpr int kMaxHostOuts = 8;

struct HostLayout {
  int chunk_batch = 0, chunks = 0, slots = 0;
  size_t q = 0, kv = 0, o = 0, lse = 0;  // bytes of one chunk's tensors (rounded to 256)
  size_t slot = 0;                       // bytes of one staging slot
};

bool host_layout(const Fav4Args* a, const Fav4HostOut* outs, int n_outs, int chunks, HostLayout* l) {
  if (!a || a->batch <= 0 || a->heads <= 0 || a->sq <= 0 || a->sk <= 0 || n_outs < 1 || n_outs > kMaxHostOuts ||
      chunks < 1 || a->batch > INT_MAX / a->heads || a->heads > INT_MAX / 128 || a->sq > INT_MAX / (a->heads * 128) ||
      a->sk > INT_MAX / (a->heads * 128))
    return false;
  l->chunks = chunks < a->batch ? chunks : a->batch;
  l->chunk_batch = (a->batch + l->chunks - 1) / l->chunks;
  l->chunks = (a->batch + l->chunk_batch - 1) / l->chunk_batch;
  l->slots = l->chunks > 1 ? 2 : 1;
  const size_t row = static_cast<size_t>(a->heads) * kHeadDim * 2;
  l->q = round256(static_cast<size_t>(l->chunk_batch) * a->sq * row);
  l->kv = round256(static_cast<size_t>(l->chunk_batch) * a->sk * row);
  l->o = l->q;
  l->lse = round256(static_cast<size_t>(l->chunk_batch) * a->heads * a->sq * 4);
  l->slot = l->q + 2 * l->kv;
  for (int j = 0; j < n_outs; ++j) l->slot += l->o + ((outs && outs[j].lse) ? l->lse : 0);
  return true;
}

// Copy streams and events of fav4_bshd_forward_host, created on a device's
// first call (with that device current) and kept until the process exits, so
// a call creates nothing. A call holds its device's mutex while it enqueues:
// host threads that call at the same time take turns (enqueueing only; the
// GPU work of consecutive calls is ordered through the callers' streams).
struct HostPipe {
  cudaStream_t up = nullptr, down = nullptr;
  cudaEvent_t fork = nullptr, uploaded[2] = {}, computed[2] = {}, downloaded[2] = {};
  cudaError_t create() {
    cudaError_t e = cudaStreamCreateWithFlags(&up, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&down, cudaStreamNonBlocking);
    cudaEvent_t* all[] = {&fork, &uploaded[0], &uploaded[1], &computed[0], &computed[1], &downloaded[0],
                          &downloaded[1]};
    for (cudaEvent_t* ev : all)
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(ev, cudaEventDisableTiming);
    if (e != cudaSuccess) release();
    return e;
  }
  void release() {
    cudaEvent_t* all[] = {&fork, &uploaded[0], &uploaded[1], &computed[0], &computed[1], &downloaded[0],
                          &downloaded[1]};
    for (cudaEvent_t* ev : all) {
      if (*ev) cudaEventDestroy(*ev);
      *ev = nullptr;
    }
    if (up) cudaStreamDestroy(up);
    if (down) cudaStreamDestroy(down);
    up = down = nullptr;
  }
};

struct HostPipeSlot {
  std::mutex mu;
  HostPipe pipe;
  bool ready = false;
};

HostPipeSlot* host_pipe_slot(int dev) {
  static HostPipeSlot slots[kMaxDevices];
  return (dev >= 0 && dev < kMaxDevices) ? &slots[dev] : nullptr;
}

}  // namespace
}  // namespace fav4

extern "C" size_t fav4_bshd_host_workspace_bytes(const Fav4Args* a, const Fav4HostOut* outs, int n_outs,
                                                  int chunks) {
  fav4::HostLayout l;
  if (!outs || !fav4::host_layout(a, outs, n_outs, chunks, &l)) return 0;
  return static_cast<size_t>(l.slots) * l.slot;
}

extern "C" int fav4_bshd_forward_host(const Fav4Args* a, const Fav4HostOut* outs, int n_outs, int chunks,
                                      void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  fav4::HostLayout l;
  if (!outs || !fav4::host_layout(a, outs, n_outs, chunks, &l) || !a->q || !a->k || !a->v ||
      !std::isfinite(a->scale) || a->scale <= 0 || !workspace || (reinterpret_cast<uintptr_t>(workspace) & 255) ||
      workspace_bytes < static_cast<size_t>(l.slots) * l.slot)
    return cudaErrorInvalidValue;
  for (int j = 0; j < n_outs; ++j)
    if (!outs[j].o || (outs[j].causal != 0 && outs[j].causal != 1) || outs[j].config < 0 || outs[j].config > 3)
      return cudaErrorInvalidValue;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  fav4::HostPipeSlot* slot_of_dev = fav4::host_pipe_slot(dev);
  if (!slot_of_dev) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> pipe_lock(slot_of_dev->mu);
  if (!slot_of_dev->ready) {
    e = slot_of_dev->pipe.create();
    if (e != cudaSuccess) return e;
    slot_of_dev->ready = true;
  }
  fav4::HostPipe& pipe = slot_of_dev->pipe;
  // The copy streams start behind everything already queued on the caller's stream.
  e = cudaEventRecord(pipe.fork, stream);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(pipe.up, pipe.fork, 0);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(pipe.down, pipe.fork, 0);
  if (e != cudaSuccess) return e;
  const size_t row = static_cast<size_t>(a->heads) * fav4::kHeadDim * 2;  // bytes of one (token) row
  const size_t lse_row = static_cast<size_t>(a->heads) * a->sq * 4;        // LSE bytes of one batch entry
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  int last = 0;
  for (int c = 0; c < l.chunks && e == cudaSuccess; ++c) {
    const int s = c % l.slots;
    last = s;
    const int b0 = c * l.chunk_batch;
    const int nb = b0 + l.chunk_batch <= a->batch ? l.chunk_batch : a->batch - b0;
    unsigned char* slot = ws + s * l.slot;
    unsigned char *dq = slot, *dk = slot + l.q, *dv = slot + l.q + l.kv;
    const size_t q_bytes = static_cast<size_t>(nb) * a->sq * row, kv_bytes = static_cast<size_t>(nb) * a->sk * row;
    // upload: the slot's inputs are free once the forwards of chunk c-2 ran
    if (c >= l.slots) e = cudaStreamWaitEvent(pipe.up, pipe.computed[s], 0);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(dq, static_cast<const unsigned char*>(a->q) + static_cast<size_t>(b0) * a->sq * row, q_bytes,
                          cudaMemcpyHostToDevice, pipe.up);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(dk, static_cast<const unsigned char*>(a->k) + static_cast<size_t>(b0) * a->sk * row, kv_bytes,
                          cudaMemcpyHostToDevice, pipe.up);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(dv, static_cast<const unsigned char*>(a->v) + static_cast<size_t>(b0) * a->sk * row, kv_bytes,
                          cudaMemcpyHostToDevice, pipe.up);
    if (e == cudaSuccess) e = cudaEventRecord(pipe.uploaded[s], pipe.up);
    // forwards on the caller's stream, once the slot's outputs were copied out
    if (e == cudaSuccess) e = cudaStreamWaitEvent(stream, pipe.uploaded[s], 0);
    if (e == cudaSuccess && c >= l.slots) e = cudaStreamWaitEvent(stream, pipe.downloaded[s], 0);
    unsigned char* out = slot + l.q + 2 * l.kv;
    unsigned char* dst[fav4::kMaxHostOuts];
    float* dst_lse[fav4::kMaxHostOuts];
    for (int j = 0; j < n_outs && e == cudaSuccess; ++j) {
      Fav4Args ca = *a;
      ca.q = dq;
      ca.k = dk;
      ca.v = dv;
      ca.batch = nb;
      ca.o = dst[j] = out;
      out += l.o;
      ca.lse = dst_lse[j] = outs[j].lse ? reinterpret_cast<float*>(out) : nullptr;
      if (outs[j].lse) out += l.lse;
      // Auto is resolved on the whole batch, so chunking never changes the numbers.
      const int cfg = outs[j].config ? outs[j].config : fav4::auto_config(a, outs[j].causal != 0, true);
      e = static_cast<cudaError_t>(cfg == fav4::kConfigWide ? fav4::launch_fwd_wide<false>(ca, ca.heads, stream)
                                                             : fav4_bshd_forward(&ca, outs[j].causal, cfg, stream));
    }
    if (e == cudaSuccess) e = cudaEventRecord(pipe.computed[s], stream);
    // download
    if (e == cudaSuccess) e = cudaStreamWaitEvent(pipe.down, pipe.computed[s], 0);
    for (int j = 0; j < n_outs && e == cudaSuccess; ++j) {
      e = cudaMemcpyAsync(static_cast<unsigned char*>(outs[j].o) + static_cast<size_t>(b0) * a->sq * row, dst[j], q_bytes,
                          cudaMemcpyDeviceToHost, pipe.down);
      if (e == cudaSuccess && outs[j].lse)
        e = cudaMemcpyAsync(reinterpret_cast<unsigned char*>(outs[j].lse) + static_cast<size_t>(b0) * lse_row, dst_lse[j], static_cast<size_t>(nb) * lse_row,
                            cudaMemcpyDeviceToHost, pipe.down);
    }
    if (e == cudaSuccess) e = cudaEventRecord(pipe.downloaded[s], pipe.down);
  }
  // Join: the caller's stream continues after the last copy back (copies on
  // one stream complete in order, so the last one covers the others).
  const cudaError_t j = cudaStreamWaitEvent(stream, pipe.downloaded[last], 0);
  return e != cudaSuccess ? e : j;
}

// --------------------------------------------------------------------------
// Split-KV in one launch, for shapes with few query tiles (decoding: Sq much
// smaller than Sk). The kernel's work tiles gain a split index; split s
// writes its partial O (normalised within the split) and LSE to slice s of a
// caller-provided workspace, and the LSE-weighted combine kernel merges the
// slices into O and LSE.
namespace fav4 {
namespace {

struct SplitLayout {
  size_t o_slice = 0, lse_slice = 0;  // bytes of one split's partial O / LSE (rounded to 256)
};

SplitLayout split_layout(const Fav4Args* a) {
  SplitLayout l;
  const size_t rows = static_cast<size_t>(a->batch) * a->sq * a->heads;
  l.o_slice = round256(rows * kHeadDim * 2);
  l.lse_slice = round256(rows * 4);
  return l;
}

// Query tiles of the work decomposition the config uses.
int64_t base_tiles(const Fav4Args* a, int config) {
  const int rows = config == 1 ? kBlockM : 2 * kBlockM;
  return static_cast<int64_t>(a->batch) * a->heads * ((a->sq + rows - 1) / rows);
}

}  // namespace
}  // namespace fav4

extern "C" int fav4_bshd_splitkv_splits(const Fav4Args* a, int causal, int config) {
  if (!fav4::args_valid(a, causal, config)) return -1;
  if (config == 0) config = fav4::auto_config(a);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  fav4::DeviceInfo info;
  if (!fav4::device_info(dev, &info)) return -1;
  const int64_t base = fav4::base_tiles(a, config);
  // keys any query row can see (top-left causal: rows < sq see keys < sq)
  const int keys = causal ? (a->sq < a->sk ? a->sq : a->sk) : a->sk;
  const int64_t kv_tiles = (keys + fav4::kBlockN - 1) / fav4::kBlockN;
  // as many work tiles as fit one wave over the SMs, at least 4 K/V tiles (512 keys) per split, at most 32
  int64_t splits = info.sms / base;
  if (splits > kv_tiles / 4) splits = kv_tiles / 4;
  if (splits > fav4::kCombineCapacity) splits = fav4::kCombineCapacity;
  return splits < 1 ? 1 : static_cast<int>(splits);
}

extern "C" size_t fav4_bshd_splitkv_workspace_bytes(const Fav4Args* a, int splits) {
  if (!a || a->batch <= 0 || a->heads <= 0 || a->sq <= 0 || splits < 1 || splits > fav4::kCombineCapacity ||
      a->batch > INT_MAX / a->heads || a->heads > INT_MAX / 128 || a->sq > INT_MAX / (a->heads * 128))
    return 0;
  if (splits == 1) return 0;
  const fav4::SplitLayout l = fav4::split_layout(a);
  return static_cast<size_t>(splits) * (l.o_slice + l.lse_slice);
}

namespace fav4 {
namespace {

// Keys [kv_begin, kv_end) in `splits` ranges inside one launch, then the LSE
// combine into a->o / a->lse (args already validated, config resolved).
int splitkv_range(const Fav4Args* a, int causal, int config, int kv_begin, int kv_end, int splits, void* workspace,
                  size_t workspace_bytes, cudaStream_t stream) {
  if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255) ||
      workspace_bytes < fav4_bshd_splitkv_workspace_bytes(a, splits))
    return cudaErrorInvalidValue;
  const SplitLayout l = split_layout(a);
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  Fav4Args pa = *a;
  pa.o = ws;                                                   // [splits][B][Sq][H][128] BF16
  pa.lse = reinterpret_cast<float*>(ws + splits * l.o_slice);  // [splits][B][H][Sq] FP32
  // The kernel indexes the slices densely: O slice s starts s * B*Sq*H*128 elements in (exactly
  // o_slice bytes, a multiple of 256), LSE slice s starts s * B*H*Sq values into the LSE region.
  const size_t o_elems = static_cast<size_t>(a->batch) * a->sq * a->heads * kHeadDim;
  const size_t lse_elems = static_cast<size_t>(a->batch) * a->heads * a->sq;
  const void* o_parts[kCombineCapacity];
  const float* lse_parts[kCombineCapacity];
  for (int s = 0; s < splits; ++s) {
    o_parts[s] = ws + s * o_elems * 2;
    lse_parts[s] = reinterpret_cast<const float*>(ws + splits * l.o_slice) + s * lse_elems;
  }
  const int e = causal ? dispatch<true>(pa, config, kv_begin, kv_end, stream, 0, splits)
                       : dispatch<false>(pa, config, kv_begin, kv_end, stream, 0, splits);
  if (e != cudaSuccess) return e;
  return combine_parts(o_parts, lse_parts, splits, a->o, a->lse, a->batch, a->heads, a->sq, stream, true);
}

}  // namespace
}  // namespace fav4

extern "C" int fav4_bshd_forward_splitkv(const Fav4Args* a, int causal, int config, int splits, void* workspace,
                                         size_t workspace_bytes, cudaStream_t stream) {
  if (!fav4::args_valid(a, causal, config) || splits < 0 || splits > fav4::kCombineCapacity)
    return cudaErrorInvalidValue;
  if (config == 0) config = fav4::auto_config(a);
  if (splits == 0) splits = fav4_bshd_splitkv_splits(a, causal, config);
  if (splits < 1) return cudaErrorInvalidValue;
  if (splits == 1) return fav4_bshd_forward(a, causal, config, stream);
  return fav4::splitkv_range(a, causal, config, 0, a->sk, splits, workspace, workspace_bytes, stream);
}

extern "C" int fav4_bshd_forward_partial_splitkv(const Fav4Args* a, int causal, int config, int kv_begin,
                                                 int kv_end, int splits, void* workspace, size_t workspace_bytes,
                                                 cudaStream_t stream) {
  if (!fav4::args_valid(a, causal, config) || !a->lse || kv_begin < 0 || kv_end <= kv_begin || kv_end > a->sk ||
      (reinterpret_cast<uintptr_t>(a->lse) & 3) || splits < 1 || splits > fav4::kCombineCapacity)
    return cudaErrorInvalidValue;
  if (config == 0) config = fav4_bshd_select_config(a);
  if (splits == 1) return fav4_bshd_forward_partial(a, causal, config, kv_begin, kv_end, stream);
  return fav4::splitkv_range(a, causal, config, kv_begin, kv_end, splits, workspace, workspace_bytes, stream);
}

// --------------------------------------------------------------------------
// Split-KV forward with its partials in a fixed device array (no cudaMalloc),
// for callers that cannot allocate device memory. One array per device,
// shared by every call: overlapping calls race (see include/fav4_bshd.h).
// The slices run as one launch of the key-range kernel (splitkv_range), the
// array standing in for the caller's workspace.
namespace fav4 {
namespace {

constexpr size_t kStaticScratchBytes = size_t(64) << 20;  // 64 MiB
static __device__ __align__(256) unsigned char g_splitkv_scratch[kStaticScratchBytes];

// Device address of g_splitkv_scratch on the current device, looked up once
// per device with that device current (host code cannot use the symbol itself).
cudaError_t static_scratch(int dev, unsigned char** out) {
  static std::mutex mu;
  static unsigned char* addr[kMaxDevices] = {};
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_splitkv_scratch);
    if (e != cudaSuccess) return e;
    addr[dev] = static_cast<unsigned char*>(p);
  }
  *out = addr[dev];
  return cudaSuccess;
}

}  // namespace
}  // namespace fav4

extern "C" int fav4_bshd_forward_splitkv_static(const Fav4Args* a, int causal, int config, int splits,
                                                cudaStream_t stream) {
  if (!fav4::args_valid(a, causal, config) || splits < 1 || splits > fav4::kMaxCombineParts)
    return cudaErrorInvalidValue;
  if (config == 0) config = fav4::auto_config(a);
  if (splits == 1) return fav4_bshd_forward(a, causal, config, stream);  // one slice: no partials
  const size_t need = fav4_bshd_splitkv_workspace_bytes(a, splits);
  if (need == 0 || need > fav4::kStaticScratchBytes) return cudaErrorMemoryAllocation;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  unsigned char* scratch = nullptr;
  e = fav4::static_scratch(dev, &scratch);
  if (e != cudaSuccess) return e;
  return fav4::splitkv_range(a, causal, config, 0, a->sk, splits, scratch, fav4::kStaticScratchBytes, stream);
}

// --------------------------------------------------------------------------
// Backward pass (no reference counterpart), all on the caller's stream:
// D = rowsum(dO * O), then either the fused kernel (dK, dV and FP32 dQ partial
// sums by reduction, then the dQ conversion) or, deterministic, the KV kernel
// (dK, dV) and the Q kernel (dQ).
namespace fav4 {
namespace {

bool bwd_args_valid(const Fav4BwdArgs* a, int kv_heads, int causal) {
  if (!a || !a->q || !a->k || !a->v || !a->o || !a->dout || !a->lse || !a->dq || !a->dk || !a->dv ||
      a->batch <= 0 || a->heads <= 0 || a->sq <= 0 || a->sk <= 0 || (causal != 0 && causal != 1) ||
      !std::isfinite(a->scale) || a->scale <= 0 || kv_heads <= 0 || a->heads % kv_heads != 0)
    return false;
  if (a->batch > INT_MAX / a->heads || a->heads > INT_MAX / 128 || a->sq > INT_MAX / (a->heads * 128) ||
      a->sk > INT_MAX / (a->heads * 128))
    return false;
  const uintptr_t al = reinterpret_cast<uintptr_t>(a->q) | reinterpret_cast<uintptr_t>(a->k) |
                       reinterpret_cast<uintptr_t>(a->v) | reinterpret_cast<uintptr_t>(a->o) |
                       reinterpret_cast<uintptr_t>(a->dout) | reinterpret_cast<uintptr_t>(a->dq) |
                       reinterpret_cast<uintptr_t>(a->dk) | reinterpret_cast<uintptr_t>(a->dv);
  return (al & 15) == 0 && (reinterpret_cast<uintptr_t>(a->lse) & 3) == 0;
}

template <bool KV, bool Causal>
int launch_bwd(const BwdParams& base, const CUtensorMap& o0, const CUtensorMap& o1, const CUtensorMap& i0,
               const CUtensorMap& i1, int outer_len, const DeviceInfo& info, int dev, cudaStream_t stream) {
  auto kernel = attn_bwd_sm100_kernel<KV, Causal>;
  constexpr int smem = BwdSmem::kAlloc;
  {
    static std::mutex mu;
    static bool attr_set[kMaxDevices] = {};
    std::lock_guard<std::mutex> lock(mu);
    if (!attr_set[dev]) {
      const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
      attr_set[dev] = true;
    }
  }
  BwdParams p = base;
  p.num_outer = (outer_len + kBlockM - 1) / kBlockM;
  const int64_t tiles = static_cast<int64_t>(p.batch) * (KV ? p.kv_heads : p.heads) * p.num_outer;
  if (tiles > INT_MAX) return cudaErrorInvalidValue;
  p.num_tiles = static_cast<int>(tiles);
  const int grid = static_cast<int>(tiles < info.sms ? tiles : info.sms);
  kernel<<<grid, 192, smem, stream>>>(o0, o1, i0, i1, p);
  return cudaGetLastError();
}

// Causal backward schedule (see bwd_sched in attn_bwd_fused_sm100.cuh): the
// number of head-pair work items when pairing gives the shorter estimated
// makespan on `sms` CTAs, else 0. A key tile k walks the query tiles k..nq-1
// of each query head of its group; it costs those steps plus one.
int bwd_paired_items(int batch, int kv_heads, int group, int sq, int sk, int sms) {
  const int nq = (sq + kBlockM - 1) / kBlockM, nk = (sk + kBlockN - 1) / kBlockN;
  const int64_t tiles = static_cast<int64_t>(batch) * kv_heads * nk;
  const int64_t items = static_cast<int64_t>(batch) * kv_heads * ((nk + 1) / 2);
  if (nk < 2 || items > INT_MAX / 2 || sms <= 0) return 0;
  auto cost = [&](int k) -> int64_t {
    const int o0 = k * kBlockN;
    if (o0 >= sk || o0 >= sq) return 1;
    return static_cast<int64_t>(nq - o0 / kBlockM) * group + 1;
  };
  constexpr int kMaxGrid = 1024;
  int64_t load[kMaxGrid];
  const int g1 = static_cast<int>(tiles < sms ? tiles : sms);
  const int g2 = static_cast<int>(items < sms ? items : sms);
  if (g1 > kMaxGrid || g2 > kMaxGrid || tiles > (int64_t(1) << 22)) return 0;
  int64_t span_stride = 0, span_pairs = 0;
  for (int c = 0; c < g1; ++c) load[c] = 0;
  for (int64_t t = 0; t < tiles; ++t) load[t % g1] += cost(static_cast<int>(t % (int64_t(kv_heads) * nk)) / kv_heads);
  for (int c = 0; c < g1; ++c) span_stride = load[c] > span_stride ? load[c] : span_stride;
  for (int c = 0; c < g2; ++c) load[c] = 0;
  const int per_b = ((nk + 1) / 2) * kv_heads;
  for (int64_t it = 0; it < items; ++it) {
    const int q = static_cast<int>(it % per_b) / kv_heads;
    load[it % g2] += cost(q) + (nk - 1 - q != q ? cost(nk - 1 - q) : 0);
  }
  for (int c = 0; c < g2; ++c) span_pairs = load[c] > span_pairs ? load[c] : span_pairs;
  return span_pairs < span_stride ? static_cast<int>(items) : 0;
}

template <bool Causal, bool Varlen>
int launch_bwd_fused(const BwdFusedParams& base, const CUtensorMap& tk, const CUtensorMap& tv,
                     const CUtensorMap& tq, const CUtensorMap& tdo, const DeviceInfo& info, int dev,
                     cudaStream_t stream) {
  auto kernel = attn_bwd_fused_kernel<Causal, Varlen>;
  constexpr int smem = BwdFusedSmem::kBytes;
  {
    static std::mutex mu;
    static bool attr_set[kMaxDevices] = {};
    std::lock_guard<std::mutex> lock(mu);
    if (!attr_set[dev]) {
      const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
      attr_set[dev] = true;
    }
  }
  BwdFusedParams p = base;
  p.num_outer = ((Varlen ? p.max_sk : p.sk) + kBlockN - 1) / kBlockN;
  const int64_t tiles = static_cast<int64_t>(p.batch) * p.kv_heads * p.num_outer;
  if (tiles > INT_MAX) return cudaErrorInvalidValue;
  p.num_tiles = static_cast<int>(tiles);
  p.num_items = (Causal && !Varlen) ? bwd_paired_items(p.batch, p.kv_heads, p.group, p.sq, p.sk, info.sms) : 0;
  const int64_t work = p.num_items > 0 ? p.num_items : tiles;
  const int grid = static_cast<int>(work < info.sms ? work : info.sms);
  p.num_slots = p.num_items > 0 ? 2 * grid * ((p.num_items + grid - 1) / grid) : p.num_tiles;
  kernel<<<grid, 512, smem, stream>>>(tk, tv, tq, tdo, p);
  return cudaGetLastError();
}

// Workspace: D and LSE * log2(e) as [B, H, q tiles * 128] (rows past Sq zero), then the
// FP32 dQ accumulator [B, H, q tiles, 128, 128] (fused path only).
size_t bwd_stat_bytes(const Fav4BwdArgs* a) {
  const size_t nq = (static_cast<size_t>(a->sq) + kBlockM - 1) / kBlockM;
  return round256(static_cast<size_t>(a->batch) * a->heads * nq * kBlockM * 4);
}
size_t bwd_acc_bytes(const Fav4BwdArgs* a) {
  const size_t nq = (static_cast<size_t>(a->sq) + kBlockM - 1) / kBlockM;
  return round256(static_cast<size_t>(a->batch) * a->heads * nq * kBlockM * kHeadDim * 4);
}

int launch_dq_convert(const float* acc, void* dq, int batch, int heads, int sq, int nq, float scale, const int* cu_q,
                      int max_sq, const DeviceInfo& info, cudaStream_t stream) {
  const int64_t threads = static_cast<int64_t>(batch) * heads * nq * kBlockM * 4;
  const int64_t want = (threads + 255) / 256;
  const int64_t cap = static_cast<int64_t>(info.sms) * 16;
  attn_bwd_dq_convert_kernel<<<static_cast<int>(want < cap ? want : cap), 256, 0, stream>>>(
      acc, static_cast<__nv_bfloat16*>(dq), batch, heads, sq, nq, scale, cu_q, max_sq);
  return cudaGetLastError();
}

struct BwdSetup {
  DeviceInfo info;
  int dev = 0;
  CUtensorMap tq, tk, tv, tdo;
  float* dsum = nullptr;
  float* lse2 = nullptr;
  int stat_stride = 0;
};

// Validation, tensor maps and the preprocess (D, LSE * log2(e)) shared by both paths.
int bwd_prepare(const Fav4BwdArgs* a, int kv_heads, int causal, void* workspace, size_t workspace_bytes,
                cudaStream_t stream, BwdSetup* st) {
  if (!bwd_args_valid(a, kv_heads, causal) || !workspace || (reinterpret_cast<uintptr_t>(workspace) & 255) ||
      workspace_bytes < fav4_bshd_backward_workspace_bytes(a))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaGetDevice(&st->dev);
  if (e != cudaSuccess) return e;
  if (!device_info(st->dev, &st->info)) return cudaErrorInvalidDevice;
  if (!encode_bshd(&st->tq, a->q, a->batch, a->sq, a->heads) || !encode_bshd(&st->tk, a->k, a->batch, a->sk, kv_heads) ||
      !encode_bshd(&st->tv, a->v, a->batch, a->sk, kv_heads) ||
      !encode_bshd(&st->tdo, a->dout, a->batch, a->sq, a->heads))
    return cudaErrorInvalidValue;
  st->stat_stride = (a->sq + kBlockM - 1) / kBlockM * kBlockM;
  st->dsum = static_cast<float*>(workspace);
  st->lse2 = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + bwd_stat_bytes(a));
  const int64_t rows = static_cast<int64_t>(a->batch) * a->sq * a->heads;
  const int64_t want = (rows + 15) / 16;  // two rows per warp, eight warps per block
  const int64_t cap = static_cast<int64_t>(st->info.sms) * 16;
  attn_bwd_dsum_kernel<<<static_cast<int>(want < cap ? want : cap), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(a->o), static_cast<const __nv_bfloat16*>(a->dout), a->lse, st->dsum,
      st->lse2, a->batch, a->sq, a->heads, st->stat_stride);
  return cudaGetLastError();
}

}  // namespace
}  // namespace fav4

extern "C" size_t fav4_bshd_backward_workspace_bytes(const Fav4BwdArgs* a) {
  if (!a || a->batch <= 0 || a->heads <= 0 || a->sq <= 0 || a->batch > INT_MAX / a->heads ||
      a->heads > INT_MAX / 128 || a->sq > INT_MAX / (a->heads * 128))
    return 0;
  return 2 * fav4::bwd_stat_bytes(a) + fav4::bwd_acc_bytes(a);
}

namespace fav4 {
namespace {

int backward_fused(const Fav4BwdArgs* a, int kv_heads, int causal, void* workspace, size_t workspace_bytes,
                   cudaStream_t stream) {
  fav4::BwdSetup st;
  cudaError_t e =
      static_cast<cudaError_t>(fav4::bwd_prepare(a, kv_heads, causal, workspace, workspace_bytes, stream, &st));
  if (e != cudaSuccess) return e;
  float* acc = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + 2 * fav4::bwd_stat_bytes(a));
  const int nq = st.stat_stride / fav4::kBlockM;
  e = cudaMemsetAsync(acc, 0, static_cast<size_t>(a->batch) * a->heads * nq * fav4::kBlockM * fav4::kHeadDim * 4,
                      stream);
  if (e != cudaSuccess) return e;
  fav4::BwdFusedParams p = {};
  p.lse2 = st.lse2;
  p.dsum = st.dsum;
  p.dq_acc = acc;
  p.dk = static_cast<__nv_bfloat16*>(a->dk);
  p.dv = static_cast<__nv_bfloat16*>(a->dv);
  p.batch = a->batch;
  p.heads = a->heads;
  p.sq = a->sq;
  p.sk = a->sk;
  p.kv_heads = kv_heads;
  p.group = a->heads / kv_heads;
  p.stat_stride = st.stat_stride;
  p.scale = a->scale;
  p.scale_log2 = a->scale * 1.4426950408889634f;
  p.status = st.info.status;
  p.wait_limit_ns = fav4::wait_limit_ns();
  e = static_cast<cudaError_t>(
      causal ? fav4::launch_bwd_fused<true, false>(p, st.tk, st.tv, st.tq, st.tdo, st.info, st.dev, stream)
             : fav4::launch_bwd_fused<false, false>(p, st.tk, st.tv, st.tq, st.tdo, st.info, st.dev, stream));
  if (e != cudaSuccess) return e;
  return launch_dq_convert(acc, a->dq, a->batch, a->heads, a->sq, nq, a->scale, nullptr, 0, st.info, stream);
}

int backward_deterministic(const Fav4BwdArgs* a, int kv_heads, int causal, void* workspace,
                           size_t workspace_bytes, cudaStream_t stream) {
  fav4::BwdSetup st;
  cudaError_t e =
      static_cast<cudaError_t>(fav4::bwd_prepare(a, kv_heads, causal, workspace, workspace_bytes, stream, &st));
  if (e != cudaSuccess) return e;
  const fav4::DeviceInfo& info = st.info;
  const int dev = st.dev;
  const CUtensorMap &tq = st.tq, &tk = st.tk, &tv = st.tv, &tdo = st.tdo;
  float* dsum = st.dsum;
  float* lse2 = st.lse2;
  fav4::BwdParams p = {};
  p.lse2 = lse2;
  p.dsum = dsum;
  p.stat_stride = st.stat_stride;
  p.batch = a->batch;
  p.heads = a->heads;
  p.sq = a->sq;
  p.sk = a->sk;
  p.kv_heads = kv_heads;
  p.group = a->heads / kv_heads;
  p.scale = a->scale;
  p.scale_log2 = a->scale * 1.4426950408889634f;
  p.status = info.status;
  p.wait_limit_ns = fav4::wait_limit_ns();
  // KV kernel: dK, dV
  fav4::BwdParams pk = p;
  pk.g0 = static_cast<__nv_bfloat16*>(a->dk);
  pk.g1 = static_cast<__nv_bfloat16*>(a->dv);
  e = static_cast<cudaError_t>(causal ? fav4::launch_bwd<true, true>(pk, tk, tv, tq, tdo, a->sk, info, dev, stream)
                                      : fav4::launch_bwd<true, false>(pk, tk, tv, tq, tdo, a->sk, info, dev, stream));
  if (e != cudaSuccess) return e;
  // Q kernel: dQ
  fav4::BwdParams pq = p;
  pq.g0 = static_cast<__nv_bfloat16*>(a->dq);
  pq.g1 = nullptr;
  return causal ? fav4::launch_bwd<false, true>(pq, tq, tdo, tk, tv, a->sq, info, dev, stream)
                : fav4::launch_bwd<false, false>(pq, tq, tdo, tk, tv, a->sq, info, dev, stream);
}

}  // namespace
}  // namespace fav4

extern "C" int fav4_bshd_backward(const Fav4BwdArgs* a, int causal, void* workspace, size_t workspace_bytes,
                                  cudaStream_t stream) {
  if (!a) return cudaErrorInvalidValue;
  return fav4::backward_fused(a, a->heads, causal, workspace, workspace_bytes, stream);
}

extern "C" int fav4_bshd_backward_deterministic(const Fav4BwdArgs* a, int causal, void* workspace,
                                                size_t workspace_bytes, cudaStream_t stream) {
  if (!a) return cudaErrorInvalidValue;
  return fav4::backward_deterministic(a, a->heads, causal, workspace, workspace_bytes, stream);
}

extern "C" int fav4_bshd_backward_gqa(const Fav4BwdArgs* a, int kv_heads, int causal, int deterministic,
                                      void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (!a || (deterministic != 0 && deterministic != 1)) return cudaErrorInvalidValue;
  return deterministic ? fav4::backward_deterministic(a, kv_heads, causal, workspace, workspace_bytes, stream)
                       : fav4::backward_fused(a, kv_heads, causal, workspace, workspace_bytes, stream);
}

namespace fav4 {
namespace {

bool varlen_bwd_valid(const Fav4VarlenBwdArgs* a, int causal) {
  if (!a || !a->q || !a->k || !a->v || !a->o || !a->dout || !a->lse || !a->dq || !a->dk || !a->dv ||
      !a->cu_seqlens_q || !a->cu_seqlens_k || a->batch <= 0 || a->heads <= 0 || a->kv_heads <= 0 ||
      a->heads % a->kv_heads != 0 || a->total_q <= 0 || a->total_k <= 0 || a->max_sq <= 0 || a->max_sk <= 0 ||
      a->max_sq > a->total_q || a->max_sk > a->total_k || (causal != 0 && causal != 1) || !std::isfinite(a->scale) ||
      a->scale <= 0)
    return false;
  if (a->heads > INT_MAX / 128 || a->total_q > INT_MAX / (a->heads * 128) ||
      a->total_k > INT_MAX / (a->kv_heads * 128) || a->batch > INT_MAX / a->heads - 1)
    return false;
  const uintptr_t al = reinterpret_cast<uintptr_t>(a->q) | reinterpret_cast<uintptr_t>(a->k) |
                       reinterpret_cast<uintptr_t>(a->v) | reinterpret_cast<uintptr_t>(a->o) |
                       reinterpret_cast<uintptr_t>(a->dout) | reinterpret_cast<uintptr_t>(a->dq) |
                       reinterpret_cast<uintptr_t>(a->dk) | reinterpret_cast<uintptr_t>(a->dv);
  const uintptr_t al4 = reinterpret_cast<uintptr_t>(a->lse) | reinterpret_cast<uintptr_t>(a->cu_seqlens_q) |
                        reinterpret_cast<uintptr_t>(a->cu_seqlens_k);
  return (al & 15) == 0 && (al4 & 3) == 0;
}

size_t varlen_stat_bytes(const Fav4VarlenBwdArgs* a) {
  const size_t nq = (static_cast<size_t>(a->max_sq) + kBlockM - 1) / kBlockM;
  return round256(static_cast<size_t>(a->batch) * a->heads * nq * kBlockM * 4);
}
size_t varlen_acc_bytes(const Fav4VarlenBwdArgs* a) {
  const size_t nq = (static_cast<size_t>(a->max_sq) + kBlockM - 1) / kBlockM;
  return round256(static_cast<size_t>(a->batch) * a->heads * nq * kBlockM * kHeadDim * 4);
}

}  // namespace
}  // namespace fav4

extern "C" size_t fav4_bshd_backward_varlen_workspace_bytes(const Fav4VarlenBwdArgs* a) {
  if (!fav4::varlen_bwd_valid(a, 0)) return 0;
  return 2 * fav4::varlen_stat_bytes(a) + fav4::varlen_acc_bytes(a);
}

extern "C" int fav4_bshd_backward_varlen(const Fav4VarlenBwdArgs* a, int causal, void* workspace,
                                         size_t workspace_bytes, cudaStream_t stream) {
  if (!fav4::varlen_bwd_valid(a, causal) || !workspace || (reinterpret_cast<uintptr_t>(workspace) & 255) ||
      workspace_bytes < fav4_bshd_backward_varlen_workspace_bytes(a))
    return cudaErrorInvalidValue;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  fav4::DeviceInfo info;
  if (!fav4::device_info(dev, &info)) return cudaErrorInvalidDevice;
  CUtensorMap tq, tk, tv, tdo;
  if (!fav4::encode_bshd(&tq, a->q, 1, a->total_q, a->heads) || !fav4::encode_bshd(&tk, a->k, 1, a->total_k, a->kv_heads) ||
      !fav4::encode_bshd(&tv, a->v, 1, a->total_k, a->kv_heads) ||
      !fav4::encode_bshd(&tdo, a->dout, 1, a->total_q, a->heads))
    return cudaErrorInvalidValue;
  const int nq = (a->max_sq + fav4::kBlockM - 1) / fav4::kBlockM;
  const int stat_stride = nq * fav4::kBlockM;
  float* dsum = static_cast<float*>(workspace);
  float* lse2 = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + fav4::varlen_stat_bytes(a));
  float* acc = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + 2 * fav4::varlen_stat_bytes(a));
  {
    const int64_t slots = static_cast<int64_t>(a->batch) * stat_stride * a->heads;
    const int64_t want = (slots + 15) / 16;  // two slots per warp, eight warps per block
    const int64_t cap = static_cast<int64_t>(info.sms) * 16;
    fav4::attn_bwd_dsum_varlen_kernel<<<static_cast<int>(want < cap ? want : cap), 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(a->o), static_cast<const __nv_bfloat16*>(a->dout), a->lse, dsum, lse2,
        a->cu_seqlens_q, a->batch, a->heads, a->total_q, a->max_sq, stat_stride);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  e = cudaMemsetAsync(acc, 0, static_cast<size_t>(a->batch) * a->heads * nq * fav4::kBlockM * fav4::kHeadDim * 4,
                      stream);
  if (e != cudaSuccess) return e;
  fav4::BwdFusedParams p = {};
  p.lse2 = lse2;
  p.dsum = dsum;
  p.dq_acc = acc;
  p.dk = static_cast<__nv_bfloat16*>(a->dk);
  p.dv = static_cast<__nv_bfloat16*>(a->dv);
  p.batch = a->batch;
  p.heads = a->heads;
  p.sq = a->total_q;
  p.sk = a->total_k;
  p.kv_heads = a->kv_heads;
  p.group = a->heads / a->kv_heads;
  p.cu_q = a->cu_seqlens_q;
  p.cu_k = a->cu_seqlens_k;
  p.max_sq = a->max_sq;
  p.max_sk = a->max_sk;
  p.stat_stride = stat_stride;
  p.scale = a->scale;
  p.scale_log2 = a->scale * 1.4426950408889634f;
  p.status = info.status;
  p.wait_limit_ns = fav4::wait_limit_ns();
  e = static_cast<cudaError_t>(causal ? fav4::launch_bwd_fused<true, true>(p, tk, tv, tq, tdo, info, dev, stream)
                                      : fav4::launch_bwd_fused<false, true>(p, tk, tv, tq, tdo, info, dev, stream));
  if (e != cudaSuccess) return e;
  return fav4::launch_dq_convert(acc, a->dq, a->batch, a->heads, a->total_q, nq, a->scale, a->cu_seqlens_q,
                                 a->max_sq, info, stream);
}

extern "C" int fav4_bshd_pipeline_status(int clear) {
  uint32_t v = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  if (cudaMemcpyFromSymbol(&v, fav4::g_status, sizeof(v)) != cudaSuccess) return -1;
  if (clear) {
    const uint32_t zero = 0;
    if (cudaMemcpyToSymbol(fav4::g_status, &zero, sizeof(zero)) != cudaSuccess) return -1;
  }
  return static_cast<int>(v & 0x7fffffffu);
}
