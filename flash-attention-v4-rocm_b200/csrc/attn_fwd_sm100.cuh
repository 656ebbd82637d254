// BF16 attention forward for B200 (sm_100a), native BSHD layout, head dim 128.
//
// Replaces the reference's single fused kernel `bshd_kernel`
// (src/bshd_kernel.hpp:50-211) with a warp-specialised tcgen05 pipeline:
//
//   warp 8  (load)     TMA: Q tiles once per work tile, then a ring of 64 KiB
//                      slots holding the groups {K0}, {V0,K1}, {V1,K2}, ...
//   warp 9  (mma)      one thread issues tcgen05.mma: S_i = Q_i K^T into TMEM,
//                      O_i += P_i V with P_i read back from TMEM.
//   warps 0-3 / 4-7    softmax for Q tile 0 / Q tile 1: one TMEM lane (= one
//                      query row) per thread; exp2 online softmax with the lazy
//                      rescale of bshd_kernel.hpp:155-164 (threshold 8 base-2
//                      units); the rare O correction is done in TMEM by the row
//                      owner; epilogue O/l -> BF16 and LSE (bshd_kernel.hpp:195-210):
//                      each 64-column half of the O tile goes through a 16 KiB
//                      shared-memory stage and one TMA store (whole 128-byte row
//                      pieces instead of 16-byte stores to 32 rows per
//                      instruction; rows past Sq are clipped by the store).
//
// TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512).
// P_i (BF16 pairs, 64 columns) overwrites the first half of S_i.
//
// A CTA is persistent and walks work tiles (batch, head, block of QTILES*128
// query rows) with a static stride of gridDim.x. Causal work tiles are ordered
// batch by batch, heads interleaved, longest first (the order of
// bshd_kernel.hpp:56-59); dense work tiles keep the query blocks of one head
// adjacent so the K/V stream of that head is shared through L2.
#pragma once
#include <cuda_bf16.h>
#include <cstdint>
#include "sm100.cuh"

namespace fav4 {

constexpr int kHeadDim = 128;
constexpr int kBlockM = 128;  // query rows per Q tile (= TMEM lanes)
constexpr int kBlockN = 128;  // keys per K/V tile
constexpr int kBoxBytes = 128 * 64 * 2;          // one TMA box: 128 rows x 64 bf16
constexpr int kTileBytes = 2 * kBoxBytes;        // a 128 x 128 bf16 tile = 32 KiB
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;        // base-2 units, bshd_kernel.hpp:157
constexpr uint32_t kLaunchRegs = 168;            // 65536 / 384 rounded down to a multiple of 8
constexpr uint32_t kSoftmaxRegs = 216;
constexpr uint32_t kOtherRegs = 72;
// One Q tile (warps 4-7 idle at kOtherRegs): the softmax warpgroup and the
// load/MMA warpgroup take the freed registers, 128 * (232 + 72 + 136) <= 384 * 168.
constexpr uint32_t kSoftmaxRegs1 = 232;
constexpr uint32_t kOtherRegs1 = 136;

struct FwdParams {
  __nv_bfloat16* o;
  float* lse;
  int batch, heads, sq, sk;
  int kv_group;          // query heads per K/V head (1 unless grouped-query attention)
  int kv_begin, kv_end;  // keys [kv_begin, kv_end) are attended (split-KV slices)
  int splits;            // KV splits inside this launch (1 = none): split s attends
  int kv_chunk;          //   [kv_begin + s*kv_chunk, min(kv_end, kv_begin + (s+1)*kv_chunk)) and
                         //   writes its partial O / LSE to slice s of o / lse
  float scale_log2;      // scale * log2(e)
  int num_mblocks;       // query blocks of QTILES*128 rows per (batch, head)
  int num_base_tiles;    // batch * heads * num_mblocks
  int num_tiles;         // num_base_tiles * splits
  int num_items;         // paired causal schedule: work items (0 = plain stride over the tiles)
  const int* cu_q;        // packed sequences (Varlen): batch + 1 row offsets into Q / O (sq = total rows)
  const int* cu_k;        //   and into K / V (sk = total keys)
  uint32_t* status;
  uint64_t wait_limit_ns;
};

struct TileCoord {
  int b, h, m0;          // m0 = first query row of the work tile (within its sequence)
  int split;             // KV split of the work tile
  int kv_begin, kv_end;  // keys it attends (within its sequence)
  int sq;                // query rows of its sequence
  int q0, k0;            // first row of its sequence in Q / O and in K / V (packed sequences)
  int tb, ob;            // batch coordinate of Q/K/V and of O / LSE (split slices, packed: 0)
};

// Split: the launch has a key-range index (p.splits > 1); without it every
// work tile attends [p.kv_begin, p.kv_end) and the index is a constant 0.
// Varlen: batch entry b is the packed sequence [cu_q[b], cu_q[b+1]) of Q / O
// against [cu_k[b], cu_k[b+1]) of K / V; offsets are clamped to the tensors,
// so malformed offsets cannot move an access outside them.
template <bool Causal, int QTiles, bool Split = false, bool Varlen = false>
__device__ __forceinline__ TileCoord tile_coord(const FwdParams& p, int t) {
  TileCoord c;
  if (Split) {
    c.split = t / p.num_base_tiles;  // splits outermost
    t -= c.split * p.num_base_tiles;
    c.kv_begin = p.kv_begin + c.split * p.kv_chunk;
    c.kv_end = min(p.kv_end, c.kv_begin + p.kv_chunk);
  } else {
    c.split = 0;
    c.kv_begin = p.kv_begin;
    c.kv_end = p.kv_end;
  }
  if (Causal) {
    const int per_batch = p.heads * p.num_mblocks;
    c.b = t / per_batch;
    const int w = t - c.b * per_batch;
    c.h = w % p.heads;
    c.m0 = (p.num_mblocks - 1 - w / p.heads) * (QTiles * kBlockM);
  } else {
    const int bh = t / p.num_mblocks;
    c.b = bh / p.heads;
    c.h = bh - c.b * p.heads;
    c.m0 = (t - bh * p.num_mblocks) * (QTiles * kBlockM);
  }
  if (Varlen) {
    const int qa = min(max(__ldg(p.cu_q + c.b), 0), p.sq), qe = min(max(__ldg(p.cu_q + c.b + 1), qa), p.sq);
    const int ka = min(max(__ldg(p.cu_k + c.b), 0), p.sk), ke = min(max(__ldg(p.cu_k + c.b + 1), ka), p.sk);
    c.q0 = qa;
    c.sq = qe - qa;
    c.k0 = ka;
    c.kv_begin = 0;
    c.kv_end = ke - ka;
    c.tb = 0;
    c.ob = 0;
  } else {
    c.q0 = 0;
    c.k0 = 0;
    c.sq = p.sq;
    c.tb = c.b;
    c.ob = c.split * p.batch + c.b;
  }
  return c;
}

// Number of K/V tiles the Q tile at row r0 of work tile `c` needs (0 = tile skipped).
template <bool Causal>
__device__ __forceinline__ int kv_tiles_for(const FwdParams& p, const TileCoord& c, int r0) {
  if (r0 >= c.sq) return 0;  // no real query row in this Q tile
  int hi = c.kv_end;
  if (Causal) hi = min(hi, r0 + kBlockM);  // top-left causal: key c visible to row r iff c <= r
  if (hi <= c.kv_begin) return 0;
  return (hi - c.kv_begin + kBlockN - 1) / kBlockN;
}

// Work-tile schedules (the loops of all three roles walk the same one).
//
// Plain: tiles blockIdx.x, blockIdx.x + gridDim.x, ... of the order tile_coord
// defines. Paired (the Paired instantiation, causal without split or packed
// sequences; the host picks it when it balances better): a work item is the
// longest and the shortest query block of one (batch, head) -- m-blocks
// nm-1-q and q -- run back to back by one CTA, so every item has the same
// number of K/V steps (a middle block without a partner runs alone) and both
// tiles read the same head's K/V. Items go batch by batch, pairs outermost,
// heads interleaved, and CTAs take them with a stride of gridDim.x. A CTA's
// paired tiles are listed once in shared memory at kernel start
// (build_pair_list); the host keeps the list within kMaxListTiles.
constexpr int kMaxListTiles = 127;  // + their count: 512 bytes

// This CTA's paired tiles in tile_coord's causal order (w = (nm - 1 -
// m-block) * heads + head); returns how many.
__device__ __forceinline__ int build_pair_list(const FwdParams& p, int* list) {
  const int nm = p.num_mblocks, per_b = ((nm + 1) >> 1) * p.heads;
  int n = 0;
  for (int item = blockIdx.x; item < p.num_items && n + 2 <= kMaxListTiles; item += gridDim.x) {
    const int b = item / per_b, r = item - b * per_b;
    const int q = r / p.heads, h = r - q * p.heads;
    list[n++] = b * p.heads * nm + r;  // the long tile: m-block nm - 1 - q, w = q * heads + h = r
    if (nm - 1 - q != q) list[n++] = b * p.heads * nm + (nm - 1 - q) * p.heads + h;
  }
  return n;
}

// Phase parities the MMA thread waits on: q_full, p_full[i], o_empty[i]. The
// packed form keeps them as bits of one register, which the split-KV
// instantiations need to stay within the load/MMA warpgroup's registers
// (72); the others keep one register each, measured 2-3 % faster there.
template <bool Packed>
struct MmaParities {
  uint32_t q = 0, pp[2] = {0, 0}, oe[2] = {1, 1};
  __device__ __forceinline__ uint32_t q_full() const { return q; }
  __device__ __forceinline__ void flip_q_full() { q ^= 1u; }
  __device__ __forceinline__ uint32_t p_full(int i) const { return pp[i]; }
  __device__ __forceinline__ void flip_p_full(int i) { pp[i] ^= 1u; }
  __device__ __forceinline__ uint32_t o_empty(int i) const { return oe[i]; }
  __device__ __forceinline__ void flip_o_empty(int i) { oe[i] ^= 1u; }
};
template <>
struct MmaParities<true> {
  uint32_t bits = 0x18u;  // bit 0 q_full, bits 1-2 p_full[i], bits 3-4 o_empty[i]
  __device__ __forceinline__ uint32_t q_full() const { return bits & 1u; }
  __device__ __forceinline__ void flip_q_full() { bits ^= 1u; }
  __device__ __forceinline__ uint32_t p_full(int i) const { return (bits >> (1 + i)) & 1u; }
  __device__ __forceinline__ void flip_p_full(int i) { bits ^= 2u << i; }
  __device__ __forceinline__ uint32_t o_empty(int i) const { return (bits >> (3 + i)) & 1u; }
  __device__ __forceinline__ void flip_o_empty(int i) { bits ^= 8u << i; }
};

// The load warp's q_empty parity and, per ring stage, whether it was armed
// and with which parity (for the drain on abort); packed or not as above.
template <bool Packed>
struct LoadState {
  uint32_t q = 1, armed = 0, armed_par = 0;
  __device__ __forceinline__ uint32_t q_empty() const { return q; }
  __device__ __forceinline__ void flip_q_empty() { q ^= 1u; }
  __device__ __forceinline__ void arm(int stage, uint32_t phase) {
    armed |= 1u << stage;
    armed_par = (armed_par & ~(1u << stage)) | (phase << stage);
  }
  __device__ __forceinline__ bool was_armed(int stage) const { return (armed >> stage) & 1u; }
  __device__ __forceinline__ uint32_t armed_parity(int stage) const { return (armed_par >> stage) & 1u; }
};
template <>
struct LoadState<true> {
  uint32_t bits = 1u;  // bit 0 q_empty, bit 8 + s armed, bit 16 + s its parity
  __device__ __forceinline__ uint32_t q_empty() const { return bits & 1u; }
  __device__ __forceinline__ void flip_q_empty() { bits ^= 1u; }
  __device__ __forceinline__ void arm(int stage, uint32_t phase) {
    bits = (bits & ~(1u << (16 + stage))) | (1u << (8 + stage)) | (phase << (16 + stage));
  }
  __device__ __forceinline__ bool was_armed(int stage) const { return (bits >> (8 + stage)) & 1u; }
  __device__ __forceinline__ uint32_t armed_parity(int stage) const { return (bits >> (16 + stage)) & 1u; }
};

// Shared memory: Q tiles, then a ring of 64 KiB slots, then barriers. Per work
// tile the load warp fills the ring with the groups G(-1) = {K0},
// G(j) = {V_j, K_j+1} (j = 0..N-2) and G(N-1) = {V_N-1}: exactly what the MMA
// warp consumes in its prologue (S(0)) and in step j (PV(j), S(j+1)). V sits
// at +0 and K at +32 KiB of a slot; one full and one empty barrier per slot.
template <int QTiles, int Slots>
struct SmemLayout {
  static constexpr int kSlotBytes = 2 * kTileBytes;
  static constexpr int kQ = 0;                                // QTiles x 32 KiB
  static constexpr int kKV = QTiles * kTileBytes;             // Slots x 64 KiB
  static constexpr int kBar = kKV + Slots * kSlotBytes;       // mbarriers
  // barrier slots (8 bytes each)
  static constexpr int kQFull = 0, kQEmpty = 1, kKVFull = 2, kKVEmpty = 2 + Slots;
  static constexpr int kSFull = 2 + 2 * Slots, kPFull = kSFull + 2, kOFull = kPFull + 2, kOEmpty = kOFull + 2;
  static constexpr int kNumBars = kOEmpty + 2 + 1;            // + teardown barrier
  static constexpr int kTeardown = kNumBars - 1;
  static constexpr int kTmemHolder = kBar + kNumBars * 8;
  static constexpr int kAbort = kTmemHolder + 4;
  static constexpr int kList = (kAbort + 4 + 15) & ~15;         // paired schedule: this CTA's tiles
  static constexpr int kStage = (kList + 4 * (kMaxListTiles + 1) + 1023) & ~1023;  // [Q tile] O store stage: 128 rows x 128 B
  static constexpr int kBytes = kStage + QTiles * kBoxBytes;
  static constexpr int kAlloc = kBytes + 1024;                // slack for 1 KiB alignment
  static_assert(kAlloc <= 227 * 1024, "shared memory budget");
};

// Ring position shared by the producer (load warp) and consumer (mma warp).
struct Ring {
  int stage = 0;
  uint32_t phase = 0;
  template <int Slots>
  __device__ __forceinline__ void advance() {
    if (++stage == Slots) { stage = 0; phase ^= 1u; }
  }
};

// ---------------------------------------------------------------------------
// exp2 split between MUFU and an FMA polynomial.
// The polynomial path: 2^x = 2^j * 2^f with j = round-to-nearest(x) taken from
// the mantissa of x + 1.5*2^23, f = x - j in [-0.5, 0.5], and
// 2^f ~ 1 + c1 f + c2 f^2 + c3 f^3, a minimax fit of the relative error with
// the constant term pinned to 1 (so x = 0, the row maximum, is exact; max
// relative error 1.01e-4), computed for this library by a linear program
// (fav4_bshd/exp2_poly.py). 2^j is added into the exponent field with an
// integer add. x is clamped at -126 so the exponent never borrows into the
// sign bit, and anything below -126 (masked keys are -inf) returns exactly 0.
// ---------------------------------------------------------------------------
constexpr float kPolyC1 = 0.6932829022407532f;
constexpr float kPolyC2 = 0.2422109693288803f;
constexpr float kPolyC3 = 0.055009059607982635f;

__device__ __forceinline__ float ex2_poly(float x) {
  const float t = fmaxf(x, -126.0f);
  const float r = __fadd_rn(t, 12582912.0f);  // 1.5 * 2^23: integer part lands in the low mantissa bits
  const float j = __fsub_rn(r, 12582912.0f);
  const float f = __fsub_rn(t, j);
  float q = __fmaf_rn(kPolyC3, f, kPolyC2);
  q = __fmaf_rn(q, f, kPolyC1);
  q = __fmaf_rn(q, f, 1.0f);
  const float y = __uint_as_float(__float_as_uint(q) + (__float_as_uint(r) << 23));
  return x < -126.0f ? 0.0f : y;
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// The polynomial exp2 on a pair, with packed FP32x2 FMA-pipe arithmetic.
// Exact0: inputs below -126 (masked keys are -inf) give exactly 0; without it
// they give ~2^-126 * p(f) (only reachable from logits 126 base-2 units under
// the row maximum, where the true value is 0 to FP32 precision anyway).
template <bool Exact0>
__device__ __forceinline__ float2 ex2_poly2(float2 x) {
  const float2 t = make_float2(fmaxf(x.x, -126.0f), fmaxf(x.y, -126.0f));
  const float2 r = __fadd2_rn(t, make_float2(12582912.0f, 12582912.0f));
  const float2 j = __fadd2_rn(r, make_float2(-12582912.0f, -12582912.0f));
  const float2 f = __ffma2_rn(j, make_float2(-1.0f, -1.0f), t);  // t - j, exact
  float2 q = __ffma2_rn(make_float2(kPolyC3, kPolyC3), f, make_float2(kPolyC2, kPolyC2));
  q = __ffma2_rn(q, f, make_float2(kPolyC1, kPolyC1));
  q = __ffma2_rn(q, f, make_float2(1.0f, 1.0f));
  float2 y;
  y.x = __uint_as_float(__float_as_uint(q.x) + (__float_as_uint(r.x) << 23));
  y.y = __uint_as_float(__float_as_uint(q.y) + (__float_as_uint(r.y) << 23));
  if (Exact0) {
    y.x = x.x < -126.0f ? 0.0f : y.x;
    y.y = x.y < -126.0f ? 0.0f : y.y;
  }
  return y;
}

// P = exp2(S * scale_log2 - mb) for one row of 128 scores: columns c with
// (c % 8) < PolyPer8 use the polynomial, the rest MUFU ex2. P is rounded to
// BF16 pairs and stored to TMEM at t_p (64 columns); the return value is the
// row sum of the unrounded FP32 probabilities (bshd_kernel.hpp:165-181).
template <int PolyPer8, bool Masked>
__device__ __forceinline__ float exp_pack_store(const float (&s)[128], float scale_log2, float mb, uint32_t t_p) {
  const float2 sc = make_float2(scale_log2, scale_log2);
  const float2 nb = make_float2(-mb, -mb);
  float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    uint32_t pk[32];
#pragma unroll
    for (int cc = 0; cc < 64; cc += 2) {
      const int c = half * 64 + cc;
      const float2 x = __ffma2_rn(make_float2(s[c], s[c + 1]), sc, nb);
      float2 e;
      if (PolyPer8 > 0 && (c % 8) < PolyPer8) {
        e = ex2_poly2<Masked>(x);
      } else {
        e = make_float2(ex2_mufu(x.x), ex2_mufu(x.y));
      }
      acc[(cc / 2) % 4] = __fadd2_rn(acc[(cc / 2) % 4], e);
      pk[cc / 2] = pack_bf16x2(e.x, e.y);
    }
    tmem_st32(t_p + half * 32, pk);
  }
  const float2 a = __fadd2_rn(__fadd2_rn(acc[0], acc[1]), __fadd2_rn(acc[2], acc[3]));
  return a.x + a.y;
}

// ---------------------------------------------------------------------------
template <bool Causal, int QTiles, int Slots, int PolyPer8, bool Split, bool Varlen, bool Paired = false>
__global__ void __launch_bounds__(384, 1)
    attn_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                          const FwdParams p) {
  using L = SmemLayout<QTiles, Slots>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_addr(smem);
  const uint32_t bar0 = sbase + L::kBar;
  auto bar = [&](int slot) -> uint32_t { return bar0 + 8u * slot; };
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + L::kAbort);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::kTmemHolder);
  int* tile_list = reinterpret_cast<int*>(smem + L::kList);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  WaitCtl ctl{abort_flag, p.status, p.wait_limit_ns};

  if (threadIdx.x == 0) {
    *abort_flag = 0u;
    mbar_init(bar(L::kQFull), 1);
    mbar_init(bar(L::kQEmpty), 1);
    for (int s = 0; s < Slots; ++s) {
      mbar_init(bar(L::kKVFull + s), 1);
      mbar_init(bar(L::kKVEmpty + s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(L::kSFull + i), 1);
      mbar_init(bar(L::kPFull + i), 4);   // one arrival per softmax warp
      mbar_init(bar(L::kOFull + i), 1);
      mbar_init(bar(L::kOEmpty + i), 4);
    }
    mbar_init(bar(L::kTeardown), 1);
    fence_mbar_init();
    if (Paired) tile_list[kMaxListTiles] = build_pair_list(p, tile_list);
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_o);
  }
  if (warp == 9) {
    tmem_alloc(smem_addr(tmem_holder), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  // Split launches are followed by the combine as a programmatic dependent
  // launch: let it be scheduled now (it waits for this grid's writes itself).
  if (Split) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int list_len = Paired ? tile_list[kMaxListTiles] : 0;  // paired schedule: this CTA's tiles

  // 384 threads launched with kLaunchRegs registers each (ptxas must report
  // exactly that: __launch_bounds__(384, 1) caps it at 168). Softmax
  // warpgroups take kSoftmaxRegs, the load/MMA warpgroup keeps kOtherRegs:
  // 128 * (2 * 216 + 72) = 64512 = 384 * 168.
  static_assert(128 * (2 * kSoftmaxRegs + kOtherRegs) <= 384 * kLaunchRegs, "register split exceeds the launch");
  static_assert(128 * (kSoftmaxRegs1 + kOtherRegs + kOtherRegs1) <= 384 * kLaunchRegs, "one-tile split exceeds the launch");
  static_assert(!Paired || (Causal && !Split && !Varlen), "the paired schedule is for causal tiles of one launch");
  // One Q tile per CTA (config 1): S is double-buffered in TMEM (the second Q
  // tile's columns are free), so S is computed two K/V steps ahead of PV and
  // the softmax of step j overlaps the MMAs of steps j-1 and j+1. Two Q tiles:
  // one S buffer per tile, the tiles ping-pong, S one step ahead.
  constexpr int KA = QTiles == 1 ? 2 : 1;

  if (warp >= 8) {
    regs_release<(QTiles == 1 ? kOtherRegs1 : kOtherRegs)>();
    if (warp == 8) {
    // ============================ TMA producer ============================
    if (lane == 0) {
      const uint64_t pol_kv = policy_evict_last();
      const uint64_t pol_q = policy_evict_first();
      Ring ring;
      LoadState<Split || Varlen || QTiles == 1> st;
      bool ok = true;
      for (int v = Paired ? 0 : blockIdx.x; v < (Paired ? list_len : p.num_tiles) && ok; v += Paired ? 1 : gridDim.x) {
        const int t = Paired ? tile_list[v] : v;
        const TileCoord tc = tile_coord<Causal, QTiles, Split, Varlen>(p, t);
        const int n0 = kv_tiles_for<Causal>(p, tc, tc.m0);
        const int n1 = QTiles > 1 ? kv_tiles_for<Causal>(p, tc, tc.m0 + kBlockM) : 0;
        const int N = max(n0, n1);
        if (N == 0) continue;
        if (!mbar_wait(bar(L::kQEmpty), st.q_empty(), ctl, kStatusTimeoutLoad)) { ok = false; break; }
        st.flip_q_empty();
        const int nq = (n0 > 0 ? 1 : 0) + (n1 > 0 ? 1 : 0);
        const int kvh = tc.h / p.kv_group;  // K/V head shared by this query head's group
        mbar_arrive_expect_tx(bar(L::kQFull), nq * kTileBytes);
        for (int i = 0; i < QTiles; ++i) {
          if ((i == 0 ? n0 : n1) == 0) continue;
          const uint32_t dst = sbase + L::kQ + i * kTileBytes;
          tma_load_4d(dst, &tm_q, bar(L::kQFull), 0, tc.h, tc.q0 + tc.m0 + i * kBlockM, tc.tb, pol_q);
          tma_load_4d(dst + kBoxBytes, &tm_q, bar(L::kQFull), 64, tc.h, tc.q0 + tc.m0 + i * kBlockM, tc.tb, pol_q);
        }
        // Groups G(g) = {V_g, K_(g+KA)} for g = -KA .. N-1 (empty ones skipped):
        // the MMA thread computes S KA steps ahead of PV (see the MMA issuer).
        for (int g = -KA; g < N && ok; ++g) {
          const bool has_v = g >= 0, has_k = g + KA < N;
          if (KA > 1 && !has_v && !has_k) continue;
          if (!mbar_wait(bar(L::kKVEmpty + ring.stage), ring.phase ^ 1u, ctl, kStatusTimeoutLoad)) {
            ok = false;
            break;
          }
          const uint32_t fb = bar(L::kKVFull + ring.stage);
          mbar_arrive_expect_tx(fb, (has_v ? kTileBytes : 0) + (has_k ? kTileBytes : 0));
          st.arm(ring.stage, ring.phase);
          const uint32_t dst = sbase + L::kKV + ring.stage * L::kSlotBytes;
          if (has_v) {
            const int sv = tc.k0 + tc.kv_begin + g * kBlockN;
            tma_load_4d(dst, &tm_v, fb, 0, kvh, sv, tc.tb, pol_kv);
            tma_load_4d(dst + kBoxBytes, &tm_v, fb, 64, kvh, sv, tc.tb, pol_kv);
          }
          if (has_k) {
            const int sk0 = tc.k0 + tc.kv_begin + (g + KA) * kBlockN;
            tma_load_4d(dst + kTileBytes, &tm_k, fb, 0, kvh, sk0, tc.tb, pol_kv);
            tma_load_4d(dst + kTileBytes + kBoxBytes, &tm_k, fb, 64, kvh, sk0, tc.tb, pol_kv);
          }
          ring.advance<Slots>();
        }
      }
      if (!ok) {
        // Let every copy this warp issued land before the CTA exits.
        WaitCtl drain{abort_flag, p.status, p.wait_limit_ns};
        volatile uint32_t no_abort = 0;
        drain.abort = &no_abort;
        for (int s = 0; s < Slots; ++s)
          if (st.was_armed(s)) mbar_wait(bar(L::kKVFull + s), st.armed_parity(s), drain, kStatusTimeoutDrain);
      }
    }
    __syncwarp();
  } else if (warp == 9) {
    // ============================= MMA issuer =============================
    // One thread issues every MMA, in the order S0(0) S1(0), then per K/V
    // pair j: PV0(j) S0(j+1) PV1(j) S1(j+1). That order makes the two Q tiles
    // ping-pong (softmax of one tile overlaps the other tile's MMAs), and since
    // tcgen05 ops of one thread execute in issue order, S_i(j+1) overwrites
    // P_i only after PV_i(j) has read it.
    if (lane == 0) {
      constexpr uint32_t idesc_qk = make_idesc_bf16(kBlockM, kBlockN, false);
      constexpr uint32_t idesc_pv = make_idesc_bf16(kBlockM, kHeadDim, true);
      Ring ring;
      MmaParities<Split || Varlen || QTiles == 1> par;
      bool ok = true;
      // Descriptor words, computed once: K-major (Q, K) and MN-major (V),
      // 128-byte swizzle, 8-row groups 1024 bytes apart; V's two 64-column
      // halves are one box (16 KiB) apart. Per MMA only the address word moves.
      const uint64_t dk = make_sdesc_sw128(sbase, 16, 1024);
      const uint64_t dv = make_sdesc_sw128(sbase, kBoxBytes, 1024);
      const uint32_t k_lo = static_cast<uint32_t>(dk), k_hi = static_cast<uint32_t>(dk >> 32);
      const uint32_t v_lo = static_cast<uint32_t>(dv), v_hi = static_cast<uint32_t>(dv >> 32);
      auto issue_s = [&](int i, int slot) {  // K of the group in `slot`
        const uint32_t qa = k_lo + ((L::kQ + i * kTileBytes) >> 4);
        const uint32_t ka = k_lo + ((L::kKV + slot * L::kSlotBytes + kTileBytes) >> 4);
        const uint32_t d = tmem + i * 128;
#pragma unroll
        for (int k = 0; k < kHeadDim / 16; ++k) {
          const uint32_t off = ((k / 4) * kBoxBytes + (k % 4) * 32) >> 4;
          umma_ss_w(d, qa + off, k_hi, ka + off, k_hi, idesc_qk, k > 0 ? 1u : 0u);
        }
        tc_commit(bar(L::kSFull + i));
      };
      auto issue_pv = [&](int i, int slot, bool acc) {  // V of the group in `slot`
        const uint32_t va = v_lo + ((L::kKV + slot * L::kSlotBytes) >> 4);
        const uint32_t d = tmem + 256 + i * 128;
        const uint32_t pa = tmem + i * 128;
        umma_ts_w(d, pa, va, v_hi, idesc_pv, acc ? 1u : 0u);
#pragma unroll
        for (int k = 1; k < kBlockN / 16; ++k) umma_ts_w(d, pa + k * 8, va + ((k * 2048) >> 4), v_hi, idesc_pv, 1u);
      };
      // One Q tile (QTiles == 1): S buffer b at TMEM columns 128 b, O at 256.
      auto issue_s_buf = [&](int b, int slot) {
        const uint32_t qa = k_lo + (L::kQ >> 4);
        const uint32_t ka = k_lo + ((L::kKV + slot * L::kSlotBytes + kTileBytes) >> 4);
        const uint32_t d = tmem + b * 128;
#pragma unroll
        for (int k = 0; k < kHeadDim / 16; ++k) {
          const uint32_t off = ((k / 4) * kBoxBytes + (k % 4) * 32) >> 4;
          umma_ss_w(d, qa + off, k_hi, ka + off, k_hi, idesc_qk, k > 0 ? 1u : 0u);
        }
        tc_commit(bar(L::kSFull + b));
      };
      auto issue_pv_buf = [&](int b, int slot, bool acc) {
        const uint32_t va = v_lo + ((L::kKV + slot * L::kSlotBytes) >> 4);
        const uint32_t d = tmem + 256;
        const uint32_t pa = tmem + b * 128;
        umma_ts_w(d, pa, va, v_hi, idesc_pv, acc ? 1u : 0u);
#pragma unroll
        for (int k = 1; k < kBlockN / 16; ++k) umma_ts_w(d, pa + k * 8, va + ((k * 2048) >> 4), v_hi, idesc_pv, 1u);
      };
      for (int v = Paired ? 0 : blockIdx.x; v < (Paired ? list_len : p.num_tiles) && ok; v += Paired ? 1 : gridDim.x) {
        const int t = Paired ? tile_list[v] : v;
        const TileCoord tc = tile_coord<Causal, QTiles, Split, Varlen>(p, t);
        const int n0 = kv_tiles_for<Causal>(p, tc, tc.m0);
        const int n1 = QTiles > 1 ? kv_tiles_for<Causal>(p, tc, tc.m0 + kBlockM) : 0;
        const int N = max(n0, n1);
        if (N == 0) continue;
        if (!mbar_wait(bar(L::kQFull), par.q_full(), ctl, kStatusTimeoutMma)) { ok = false; break; }
        par.flip_q_full();
        if constexpr (QTiles == 1) {
          // S buffer b = j % 2 (TMEM columns 128 b). Prologue: S(0) from G(-2) = {K0}
          // and S(1) from G(-1) = {K1}; step j: PV(j) from buffer j % 2, then S(j+2)
          // into the same buffer (after PV(j) has read P(j), in issue order), both
          // from G(j) = {V_j, K_j+2}. Every PV is committed to pv_done (the o_full
          // barrier of the unused second tile) so the softmax can wait for PV(j-1)
          // before it rescales O.
          for (int pb = 0; pb < 2 && pb < N && ok; ++pb) {
            if (!mbar_wait(bar(L::kKVFull + ring.stage), ring.phase, ctl, kStatusTimeoutMma)) { ok = false; break; }
            tc_fence_after();
            issue_s_buf(pb, ring.stage);
            tc_commit(bar(L::kKVEmpty + ring.stage));
            ring.advance<Slots>();
          }
          if (N <= 2 && ok) tc_commit(bar(L::kQEmpty));
          if (ok && !mbar_wait(bar(L::kKVFull + ring.stage), ring.phase, ctl, kStatusTimeoutMma)) ok = false;
          for (int j = 0; j < N && ok; ++j) {
            const int b = j & 1;
            const int cur = ring.stage;
            Ring nxt = ring;
            nxt.advance<Slots>();
            if (!mbar_wait(bar(L::kPFull + b), par.p_full(b), ctl, kStatusTimeoutMma)) { ok = false; break; }
            par.flip_p_full(b);
            if (j == 0) {
              if (!mbar_wait(bar(L::kOEmpty), par.o_empty(0), ctl, kStatusTimeoutMma)) { ok = false; break; }
              par.flip_o_empty(0);
            }
            tc_fence_after();
            issue_pv_buf(b, cur, j > 0);
            tc_commit(bar(L::kOFull + 1));  // pv_done
            if (j + 1 == N) tc_commit(bar(L::kOFull));
            if (j + 2 < N) issue_s_buf(b, cur);
            tc_commit(bar(L::kKVEmpty + cur));  // V_j and K_j+2 are no longer read
            if (j + 3 == N) tc_commit(bar(L::kQEmpty));
            ring = nxt;
            if (j + 1 < N && !mbar_wait(bar(L::kKVFull + ring.stage), ring.phase, ctl, kStatusTimeoutMma)) {
              ok = false;
              break;
            }
          }
          continue;
        }
        // group G(-1) = {K0}
        if (!mbar_wait(bar(L::kKVFull + ring.stage), ring.phase, ctl, kStatusTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        if (n0 > 0) issue_s(0, ring.stage);
        if (n1 > 0) issue_s(1, ring.stage);
        tc_commit(bar(L::kKVEmpty + ring.stage));
        if (N == 1) tc_commit(bar(L::kQEmpty));
        ring.advance<Slots>();
        // G(0) is awaited while the S MMAs above drain.
        if (!mbar_wait(bar(L::kKVFull + ring.stage), ring.phase, ctl, kStatusTimeoutMma)) { ok = false; break; }
        for (int j = 0; j < N && ok; ++j) {
          // group G(j) = {V_j, K_j+1} is resident (awaited one step earlier).
          // Between the last MMA of one batch and the first of the next only
          // a commit, a P wait and a fence remain: everything else sits in the
          // shadow of MMAs the tensor pipe is still working through.
          const int cur = ring.stage;
          Ring nxt = ring;
          nxt.advance<Slots>();
#pragma unroll
          for (int i = 0; i < QTiles; ++i) {
            const int ni = i == 0 ? n0 : n1;
            if (j < ni && ok) {
              if (!mbar_wait(bar(L::kPFull + i), par.p_full(i), ctl, kStatusTimeoutMma)) { ok = false; continue; }
              par.flip_p_full(i);
              if (j == 0) {
                if (!mbar_wait(bar(L::kOEmpty + i), par.o_empty(i), ctl, kStatusTimeoutMma)) { ok = false; continue; }
                par.flip_o_empty(i);
              }
              tc_fence_after();
              issue_pv(i, cur, j > 0);
              if (j + 1 == ni) tc_commit(bar(L::kOFull + i));
            }
            if (i == QTiles - 1 && j + 1 < N && ok) {
              // next group, awaited behind this tile's PV MMAs
              if (!mbar_wait(bar(L::kKVFull + nxt.stage), nxt.phase, ctl, kStatusTimeoutMma)) { ok = false; continue; }
            }
            if (j + 1 < ni && ok) issue_s(i, cur);
          }
          if (!ok) break;
          tc_commit(bar(L::kKVEmpty + cur));  // V_j and K_j+1 are no longer read
          if (j + 2 == N) tc_commit(bar(L::kQEmpty));
          ring = nxt;
        }
      }
      // Every MMA this thread issued has finished once this barrier flips.
      tc_commit(bar(L::kTeardown));
      WaitCtl drain{abort_flag, p.status, p.wait_limit_ns};
      volatile uint32_t no_abort = 0;
      drain.abort = &no_abort;
      mbar_wait(bar(L::kTeardown), 0, drain, kStatusTimeoutDrain);
    }
    __syncwarp();
    }  // warps 10-11: idle
  } else if (warp < 4 * QTiles) {
    // ============================== softmax ===============================
    regs_claim<(QTiles == 1 ? kSoftmaxRegs1 : kSoftmaxRegs)>();
    const int i = warp / 4;                  // Q tile served by this warpgroup
    const int row = (warp % 4) * 32 + lane;  // TMEM lane = row within the Q tile
    const uint32_t lane_off = static_cast<uint32_t>((warp % 4) * 32) << 16;
    const uint32_t t_s0 = tmem + lane_off + i * 128;  // one Q tile: S buffer j % 2 at t_s0 + 128 (j % 2)
    const uint32_t t_o = tmem + lane_off + 256 + i * 128;
    // O store stage of this Q tile: 16-byte chunk c of a row at (c ^ (row % 8)), the TMA 128-byte swizzle
    uint8_t* stage_row = smem + L::kStage + i * kBoxBytes + row * 128;
    const uint32_t stage = sbase + L::kStage + i * kBoxBytes;
    const bool issuer = warp % 4 == 0 && lane == 0;  // issues this warpgroup's O stores
    uint32_t s_par = 0, o_full_par = 0;  // one Q tile: s_par bit b for S buffer b
    uint32_t pv_seen = 0;                 // one Q tile: PVs of earlier work tiles (pv_done phases)
    const float scale_log2 = p.scale_log2;
    bool ok = true;
    for (int v = Paired ? 0 : blockIdx.x; v < (Paired ? list_len : p.num_tiles) && ok; v += Paired ? 1 : gridDim.x) {
      const int t = Paired ? tile_list[v] : v;
      const TileCoord tc = tile_coord<Causal, QTiles, Split, Varlen>(p, t);
      const int r0 = tc.m0 + i * kBlockM;
      const int ni = kv_tiles_for<Causal>(p, tc, r0);
      const int grow = r0 + row;  // query row (global within the sequence)
      float m = -INFINITY, l = 0.f;
      if (ni == 0) {
        if (r0 >= tc.sq) continue;  // padding-only Q tile: nothing to write
      }
      for (int j = 0; j < ni; ++j) {
        const int sb = QTiles == 1 ? (j & 1) : i;  // S buffer / barrier of this step
        const uint32_t t_s = t_s0 + (QTiles == 1 ? sb * 128 : 0);
        const uint32_t s_bit = QTiles == 1 ? 1u << sb : 1u;
        if (!warp_wait(bar(L::kSFull + sb), (s_par & s_bit) ? 1u : 0u, ctl, kStatusTimeoutSoftmax)) { ok = false; break; }
        s_par ^= s_bit;
        tc_fence_after();
        uint32_t sr[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(t_s + c * 32, sr[c]);
        tmem_ld_wait();
        float s[128];
#pragma unroll
        for (int c = 0; c < 128; ++c) s[c] = __uint_as_float(sr[c / 32][c % 32]);
        const int col0 = tc.kv_begin + j * kBlockN;
        // Mask keys past kv_end, and (causal) keys after this row.
        const bool masked = (col0 + kBlockN > tc.kv_end) || (Causal && (col0 + kBlockN - 1 > r0));
        if (masked) {
          int lim = tc.kv_end - 1 - col0;  // last visible column index within the tile
          if (Causal) lim = min(lim, grow - col0);
#pragma unroll
          for (int c = 0; c < 128; ++c) s[c] = c > lim ? -INFINITY : s[c];
        }
        // four independent max chains (the latency of one 64-long chain shows)
        float mx0 = fmax3(s[0], s[1], s[2]), mx1 = fmax3(s[3], s[4], s[5]);
        float mx2 = fmax3(s[6], s[7], s[8]), mx3 = fmax3(s[9], s[10], s[11]);
#pragma unroll
        for (int c = 12; c < 124; c += 8) {
          mx0 = fmax3(mx0, s[c], s[c + 1]);
          mx1 = fmax3(mx1, s[c + 2], s[c + 3]);
          mx2 = fmax3(mx2, s[c + 4], s[c + 5]);
          mx3 = fmax3(mx3, s[c + 6], s[c + 7]);
        }
        mx0 = fmax3(mx0, s[124], s[125]);
        mx1 = fmax3(mx1, s[126], s[127]);
        const float mx = fmax3(fmaxf(mx0, mx1), mx2, mx3) * scale_log2;
        const float cand = fmaxf(m, mx);
        const bool update = (j == 0) || (cand > m + kRescaleThreshold);
        const float m_new = update ? cand : m;
        const bool rescale = (j > 0) && __any_sync(0xffffffffu, update);
        const float alpha = rescale ? ((m_new == -INFINITY) ? 1.f : ex2_mufu(m - m_new)) : 1.f;
        m = m_new;
        const float mb = (m == -INFINITY) ? 0.f : m;
        const float rowsum = masked ? exp_pack_store<PolyPer8, true>(s, scale_log2, mb, t_s)
                                    : exp_pack_store<PolyPer8, false>(s, scale_log2, mb, t_s);
        l = l * alpha + rowsum;
        if (rescale) {
          // Lazy correction: the row owner rescales O_i in TMEM before PV of
          // this tile is issued. O_i must hold P V of all previous tiles: with
          // two Q tiles the S commit that released this tile covers PV(j-1);
          // with one (S two steps ahead) it covers only PV(j-2), so wait for
          // pv_done's completion of PV(j-1) (phases count every PV of the CTA).
          if (QTiles == 1) {
            const uint32_t ph = (pv_seen + j - 1) & 1u;
            if (!warp_wait(bar(L::kOFull + 1), ph, ctl, kStatusTimeoutSoftmax)) { ok = false; break; }
            tc_fence_after();
          }
          const float2 a2 = make_float2(alpha, alpha);
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t orow[32];
            tmem_ld32(t_o + c * 32, orow);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              const float2 v = __fmul2_rn(make_float2(__uint_as_float(orow[e]), __uint_as_float(orow[e + 1])), a2);
              orow[e] = __float_as_uint(v.x);
              orow[e + 1] = __float_as_uint(v.y);
            }
            tmem_st32(t_o + c * 32, orow);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();  // every lane's P / O stores are complete
        if (lane == 0) mbar_arrive(bar(L::kPFull + sb));
      }
      pv_seen += ni;
      // ------------------------------ epilogue ------------------------------
      const bool live = grow < tc.sq;
      // O row of this thread: [ob][q0 + grow] in a tensor of sq rows per batch entry
      const int64_t orow = (static_cast<int64_t>(tc.ob) * p.sq + tc.q0 + grow) * p.heads + tc.h;
      if (ni > 0) {
        // The four warps of this warpgroup meet at 128-thread AND-barriers
        // (id 1 + i); a warp that gave up on a wait above arrives with
        // `false`, so all four leave together.
        const bool got = ok && warp_wait(bar(L::kOFull + i), o_full_par, ctl, kStatusTimeoutSoftmax);
        if (issuer) tma_store_wait_read_all();  // the previous tile's stores have read the stage
        if (!pair_all(1 + i, 128, got)) { ok = false; break; }
        o_full_par ^= 1u;
        tc_fence_after();
        const float inv = l > 0.f ? __frcp_rn(l) : 0.f;
        // The ragged last Q tile of a packed sequence is stored row by row: a 128-row TMA box would
        // also write the next sequence's rows. Tile-uniform, so all four warps take the same path.
        const bool direct = Varlen && r0 + kBlockM > tc.sq;
        // All 128 columns of the O row in one batch of TMEM loads and one wait:
        // loads issued one by one each wait behind the other tile's MMAs.
        // O_i is free for the next work tile as soon as it is in registers.
        uint32_t oall[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(t_o + c * 32, oall[c]);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();  // every lane has read its row of O_i
        if (lane == 0) mbar_arrive(bar(L::kOEmpty + i));
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t pk[32];
#pragma unroll
          for (int c = 0; c < 2; ++c) {
#pragma unroll
            for (int e = 0; e < 16; ++e)
              pk[c * 16 + e] = pack_bf16x2(__uint_as_float(oall[half * 2 + c][2 * e]) * inv,
                                           __uint_as_float(oall[half * 2 + c][2 * e + 1]) * inv);
          }
          if (half == 1 && !direct) pair_all(1 + i, 128, true);  // the store of columns 0-63 has read the stage
          if (direct) {
            if (live) {
              uint4* dst = reinterpret_cast<uint4*>(p.o + orow * kHeadDim + half * 64);
#pragma unroll
              for (int c = 0; c < 8; ++c) dst[c] = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
            }
            continue;
          }
#pragma unroll
          for (int c = 0; c < 8; ++c)
            *reinterpret_cast<uint4*>(stage_row + ((c ^ (row & 7)) * 16)) =
                make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
          fence_proxy_async_smem();
          pair_all(1 + i, 128, true);  // every row of this half is staged
          if (issuer) {
            tma_store_4d(&tm_o, stage, half * 64, tc.h, tc.q0 + r0, tc.ob);  // O map: batch = splits x batch
            tma_store_commit();
            if (half == 0) tma_store_wait_read_all();
          }
        }
      } else if (live) {
        // no key visible to this Q tile (a split-KV slice, an empty key sequence): O = 0
        uint4* dst = reinterpret_cast<uint4*>(p.o + orow * kHeadDim);
#pragma unroll
        for (int v = 0; v < 16; ++v) dst[v] = make_uint4(0u, 0u, 0u, 0u);
      }
      if (!ok) break;
      if (live && p.lse != nullptr) {
        p.lse[(static_cast<int64_t>(tc.ob) * p.heads + tc.h) * p.sq + tc.q0 + grow] =
            l > 0.f ? m * kLn2 + logf(l) : -INFINITY;
      }
    }
    if (issuer) tma_store_wait_all();  // every O store is complete before the CTA exits
  } else {
    regs_release<kOtherRegs>();  // warps 4-7 when QTiles == 1: Q tile 1 unused
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace fav4
