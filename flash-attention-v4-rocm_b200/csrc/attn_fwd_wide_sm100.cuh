// BF16 attention forward for B200 (sm_100a), wide-step variant: one 128-row Q
// tile per CTA against 256 keys per step.
//
// The two-tile kernel (attn_fwd_sm100.cuh) issues 16 MMAs of 128x128x16 per
// 128x128 block of scores; each takes as long to issue (~61 cycles) as to run
// (64), so the single issuing thread paces the tensor pipe. Here S is one
// 128x256 product (N = 256: 128 cycles per MMA for the same issue cost) and P
// has TMEM columns of its own, so S(j+1) runs while the softmax of step j is
// still working and PV(j) follows P(j):
//
//   TMEM (512 columns): S [0,256) FP32, P [256,384) BF16 pairs, O [384,512).
//   warp 8  (load)     TMA: Q once per work tile, then K0, K1, V0, K2, V1, ...
//                      in a ring of three 64 KiB slots (256 keys x 128 each).
//   warp 9  (mma)      S(j+1) = Q K_j+1^T once the softmax has read S(j);
//                      O += P(j) V_j once P(j) is stored.
//   warps 0-3 / 4-7    softmax, keys 0-127 / 128-255 of each step for all 128
//                      rows (a TMEM lane quarter per warp): the two warps of a
//                      row exchange their row maxima through shared memory, so
//                      both make the same lazy-rescale decision
//                      (bshd_kernel.hpp:155-164, threshold 8 base-2 units);
//                      each keeps its part of the row sum and of O.
//   epilogue           O / l -> BF16 with 16-byte stores, LSE (bshd_kernel.hpp:195-210).
//
// Plain launches only (no key splits, no packed sequences); grouped-query K/V
// heads as in the two-tile kernel.
#pragma once
#include "attn_fwd_sm100.cuh"

namespace fav4 {

constexpr int kWideN = 256;                          // keys per step
constexpr int kWideBoxBytes = kWideN * 64 * 2;       // one K/V TMA box: 256 rows x 64 bf16 = 32 KiB
constexpr int kWideSlotBytes = 2 * kWideBoxBytes;    // one K or V block: 64 KiB
constexpr int kWideSlots = 3;

struct WideLayout {
  static constexpr int kQ = 0;                                     // 32 KiB
  static constexpr int kRing = kTileBytes;                         // 3 x 64 KiB
  static constexpr int kXchg = kRing + kWideSlots * kWideSlotBytes;  // [2 parities][2 halves][128 rows] FP32
  static constexpr int kBar = kXchg + 2 * 2 * kBlockM * 4;
  static constexpr int kQFull = 0, kQEmpty = 1, kKVFull = 2, kKVEmpty = 2 + kWideSlots;
  static constexpr int kSFull = 2 + 2 * kWideSlots, kSLoad = kSFull + 1, kPFull = kSLoad + 1,
                       kPVDone = kPFull + 1, kOEmpty = kPVDone + 1, kTeardown = kOEmpty + 1;
  static constexpr int kXchgBar = kTeardown + 1;  // one per TMEM lane quarter: its two softmax warps
  static constexpr int kNumBars = kXchgBar + 4;
  static constexpr int kTmemHolder = kBar + kNumBars * 8;
  static constexpr int kAbort = kTmemHolder + 4;
  static constexpr int kBytes = kAbort + 4;
  // The 1 KiB-aligned layout must start at the dynamic shared memory base: the
  // kernel checks that and otherwise reports kStatusSmemAlign and does nothing.
  static constexpr int kAlloc = kBytes;
  static_assert(kAlloc <= 227 * 1024, "shared memory budget");
};

// Ring position of item `i` (the producer and the MMA thread count items).
struct WideRing {
  uint32_t item = 0;
  __device__ __forceinline__ int stage() const { return static_cast<int>(item % kWideSlots); }
  __device__ __forceinline__ uint32_t phase() const { return (item / kWideSlots) & 1u; }
};

// P = exp2(S * scale_log2 - mb) for 128 scores of a row, packed to BF16 pairs
// in registers (the split between MUFU and the polynomial and the row sum as
// exp_pack_store); the caller stores pk once the previous PV has read P.
template <int PolyPer8, bool Masked>
__device__ __forceinline__ float exp_pack_regs(const float (&s)[128], float scale_log2, float mb, uint32_t (&pk)[64]) {
  const float2 sc = make_float2(scale_log2, scale_log2);
  const float2 nb = make_float2(-mb, -mb);
  float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
  for (int c = 0; c < 128; c += 2) {
    const float2 x = __ffma2_rn(make_float2(s[c], s[c + 1]), sc, nb);
    float2 e;
    if (PolyPer8 > 0 && (c % 8) < PolyPer8) {
      e = ex2_poly2<Masked>(x);
    } else {
      e = make_float2(ex2_mufu(x.x), ex2_mufu(x.y));
    }
    acc[(c / 2) % 4] = __fadd2_rn(acc[(c / 2) % 4], e);
    pk[c / 2] = pack_bf16x2(e.x, e.y);
  }
  const float2 a = __fadd2_rn(__fadd2_rn(acc[0], acc[1]), __fadd2_rn(acc[2], acc[3]));
  return a.x + a.y;
}

// Steps (256-key blocks) of work tile `c`: keys [kv_begin, hi), hi clipped to
// the last row of the tile under the top-left causal mask; 0 for a tile of
// padding rows only.
template <bool Causal>
__device__ __forceinline__ int wide_steps(const TileCoord& c) {
  if (c.m0 >= c.sq) return 0;
  int hi = c.kv_end;
  if (Causal) hi = min(hi, c.m0 + kBlockM);
  if (hi <= c.kv_begin) return 0;
  return (hi - c.kv_begin + kWideN - 1) / kWideN;
}

// Item `it` of a work tile of n steps in the order the MMA thread reads them:
// K0, then per step j: K_j+1 (while j+1 < n), V_j.
__device__ __forceinline__ void wide_item(int it, int n, bool* is_k, int* block) {
  if (it == 0) {
    *is_k = true;
    *block = 0;
  } else if (it == 2 * n - 1) {
    *is_k = false;
    *block = n - 1;
  } else {
    const int j = (it - 1) >> 1;
    *is_k = ((it - 1) & 1) == 0;
    *block = *is_k ? j + 1 : j;
  }
}

template <bool Causal, int PolyPer8>
__global__ void __launch_bounds__(384, 1)
    attn_fwd_wide_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const FwdParams p) {
  using L = WideLayout;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_addr(smem);
  if (sbase & 1023u) {  // the layout needs a 1 KiB-aligned base (uniform: every thread returns)
    if (threadIdx.x == 0) atomicOr(p.status, kStatusSmemAlign);
    return;
  }
  const uint32_t bar0 = sbase + L::kBar;
  auto bar = [&](int slot) -> uint32_t { return bar0 + 8u * slot; };
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + L::kAbort);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::kTmemHolder);
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  WaitCtl ctl{abort_flag, p.status, p.wait_limit_ns};

  if (threadIdx.x == 0) {
    *abort_flag = 0u;
    mbar_init(bar(L::kQFull), 1);
    mbar_init(bar(L::kQEmpty), 1);
    for (int s = 0; s < kWideSlots; ++s) {
      mbar_init(bar(L::kKVFull + s), 1);
      mbar_init(bar(L::kKVEmpty + s), 1);
    }
    mbar_init(bar(L::kSFull), 1);
    mbar_init(bar(L::kSLoad), 8);   // every softmax warp has read its half of S
    mbar_init(bar(L::kPFull), 8);   // every softmax warp has stored its half of P
    mbar_init(bar(L::kPVDone), 1);
    mbar_init(bar(L::kOEmpty), 8);
    mbar_init(bar(L::kTeardown), 1);
    for (int q = 0; q < 4; ++q) mbar_init(bar(L::kXchgBar + q), 2);
    fence_mbar_init();
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  if (warp == 9) {
    tmem_alloc(smem_addr(tmem_holder), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  static_assert(128 * (2 * kSoftmaxRegs + kOtherRegs) <= 384 * kLaunchRegs, "register split exceeds the launch");

  if (warp >= 8) {
    regs_release<kOtherRegs>();
    if (warp == 8 && lane == 0) {
      // ============================ TMA producer ============================
      const uint64_t pol_kv = policy_evict_last();
      const uint64_t pol_q = policy_evict_first();
      WideRing ring;
      uint32_t q_empty = 1, q_arms = 0, armed = 0, armed_par = 0;
      bool ok = true;
      for (int v = blockIdx.x; v < p.num_tiles && ok; v += gridDim.x) {
        const TileCoord tc = tile_coord<Causal, 1, false, false>(p, v);
        const int n = wide_steps<Causal>(tc);
        if (n == 0) continue;
        if (!mbar_wait(bar(L::kQEmpty), q_empty, ctl, kStatusTimeoutLoad)) { ok = false; break; }
        q_empty ^= 1u;
        const int kvh = tc.h / p.kv_group;
        mbar_arrive_expect_tx(bar(L::kQFull), kTileBytes);
        ++q_arms;
        tma_load_4d(sbase + L::kQ, &tm_q, bar(L::kQFull), 0, tc.h, tc.q0 + tc.m0, tc.tb, pol_q);
        tma_load_4d(sbase + L::kQ + kBoxBytes, &tm_q, bar(L::kQFull), 64, tc.h, tc.q0 + tc.m0, tc.tb, pol_q);
        for (int it = 0; it < 2 * n && ok; ++it) {
          bool is_k;
          int blk;
          wide_item(it, n, &is_k, &blk);
          const int st = ring.stage();
          if (!mbar_wait(bar(L::kKVEmpty + st), ring.phase() ^ 1u, ctl, kStatusTimeoutLoad)) {
            ok = false;
            break;
          }
          const uint32_t fb = bar(L::kKVFull + st);
          mbar_arrive_expect_tx(fb, kWideSlotBytes);
          armed |= 1u << st;
          armed_par = (armed_par & ~(1u << st)) | (ring.phase() << st);
          const uint32_t dst = sbase + L::kRing + st * kWideSlotBytes;
          const int row = tc.k0 + tc.kv_begin + blk * kWideN;
          const CUtensorMap* map = is_k ? &tm_k : &tm_v;
          tma_load_4d(dst, map, fb, 0, kvh, row, tc.tb, pol_kv);
          tma_load_4d(dst + kWideBoxBytes, map, fb, 64, kvh, row, tc.tb, pol_kv);
          ++ring.item;
        }
      }
      if (!ok) {
        // Let every copy this warp issued land before the CTA exits.
        WaitCtl drain{abort_flag, p.status, p.wait_limit_ns};
        volatile uint32_t no_abort = 0;
        drain.abort = &no_abort;
        for (int s = 0; s < kWideSlots; ++s)
          if ((armed >> s) & 1u) mbar_wait(bar(L::kKVFull + s), (armed_par >> s) & 1u, drain, kStatusTimeoutDrain);
        if (q_arms > 0) mbar_wait(bar(L::kQFull), (q_arms - 1) & 1u, drain, kStatusTimeoutDrain);
      }
    } else if (warp == 9 && lane == 0) {
      // ============================= MMA issuer =============================
      // Per work tile: S(0), then per step j: S(j+1) once the softmax has read
      // S(j), PV(j) once P(j) is stored. Each MMA reads one ring item and
      // releases its slot by a commit.
      constexpr uint32_t idesc_s = make_idesc_bf16(kBlockM, kWideN, false);
      constexpr uint32_t idesc_pv = make_idesc_bf16(kBlockM, kHeadDim, true);
      const uint64_t dk = make_sdesc_sw128(sbase, 16, 1024);
      const uint64_t dv = make_sdesc_sw128(sbase, kWideBoxBytes, 1024);
      const uint32_t k_lo = static_cast<uint32_t>(dk), k_hi = static_cast<uint32_t>(dk >> 32);
      const uint32_t v_lo = static_cast<uint32_t>(dv), v_hi = static_cast<uint32_t>(dv >> 32);
      auto issue_s = [&](int slot) {  // S = Q K^T, 128 x 256, into TMEM columns 0-255
        const uint32_t qa = k_lo + (L::kQ >> 4);
        const uint32_t ka = k_lo + ((L::kRing + slot * kWideSlotBytes) >> 4);
#pragma unroll
        for (int k = 0; k < kHeadDim / 16; ++k) {
          const uint32_t oq = ((k / 4) * kBoxBytes + (k % 4) * 32) >> 4;
          const uint32_t ok_ = ((k / 4) * kWideBoxBytes + (k % 4) * 32) >> 4;
          umma_ss_w(tmem, qa + oq, k_hi, ka + ok_, k_hi, idesc_s, k > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](int slot, bool acc) {  // O += P V over 256 keys, P from TMEM columns 256-383
        const uint32_t va = v_lo + ((L::kRing + slot * kWideSlotBytes) >> 4);
#pragma unroll
        for (int k = 0; k < kWideN / 16; ++k)
          umma_ts_w(tmem + 384, tmem + 256 + k * 8, va + ((k * 2048) >> 4), v_hi, idesc_pv,
                    (acc || k > 0) ? 1u : 0u);
      };
      WideRing ring;
      uint32_t q_full = 0, s_load = 0, p_full = 0, o_empty = 1;
      bool ok = true;
      for (int v = blockIdx.x; v < p.num_tiles && ok; v += gridDim.x) {
        const TileCoord tc = tile_coord<Causal, 1, false, false>(p, v);
        const int n = wide_steps<Causal>(tc);
        if (n == 0) continue;
        if (!mbar_wait(bar(L::kQFull), q_full, ctl, kStatusTimeoutMma)) { ok = false; break; }
        q_full ^= 1u;
        // S(0): the softmax has read the previous tile's last S (awaited in its last step)
        if (!mbar_wait(bar(L::kKVFull + ring.stage()), ring.phase(), ctl, kStatusTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        issue_s(ring.stage());
        tc_commit(bar(L::kKVEmpty + ring.stage()));
        tc_commit(bar(L::kSFull));
        if (n == 1) tc_commit(bar(L::kQEmpty));
        ++ring.item;
        for (int j = 0; j < n && ok; ++j) {
          if (!mbar_wait(bar(L::kSLoad), s_load, ctl, kStatusTimeoutMma)) { ok = false; break; }
          s_load ^= 1u;
          if (j + 1 < n) {
            if (!mbar_wait(bar(L::kKVFull + ring.stage()), ring.phase(), ctl, kStatusTimeoutMma)) { ok = false; break; }
            tc_fence_after();
            issue_s(ring.stage());
            tc_commit(bar(L::kKVEmpty + ring.stage()));
            tc_commit(bar(L::kSFull));
            if (j + 2 == n) tc_commit(bar(L::kQEmpty));
            ++ring.item;
          }
          if (!mbar_wait(bar(L::kPFull), p_full, ctl, kStatusTimeoutMma)) { ok = false; break; }
          p_full ^= 1u;
          if (j == 0) {
            if (!mbar_wait(bar(L::kOEmpty), o_empty, ctl, kStatusTimeoutMma)) { ok = false; break; }
            o_empty ^= 1u;
          }
          if (!mbar_wait(bar(L::kKVFull + ring.stage()), ring.phase(), ctl, kStatusTimeoutMma)) { ok = false; break; }
          tc_fence_after();
          issue_pv(ring.stage(), j > 0);
          tc_commit(bar(L::kKVEmpty + ring.stage()));
          tc_commit(bar(L::kPVDone));
          ++ring.item;
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
  } else {
    // ============================== softmax ===============================
    regs_claim<kSoftmaxRegs>();
    const int half = warp / 4;       // keys 128 * half .. 128 * half + 127 of every step
    const int rq = warp % 4;         // TMEM lane quarter of this warp
    const int row = rq * 32 + lane;  // TMEM lane = query row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(rq * 32) << 16;
    const uint32_t t_s = tmem + lane_off + half * 128;
    const uint32_t t_p = tmem + lane_off + 256 + half * 64;
    const uint32_t t_o = tmem + lane_off + 384 + half * 64;
    float* xchg = reinterpret_cast<float*>(smem + L::kXchg);
    const uint32_t xbar = bar(L::kXchgBar + rq);
    const float scale_log2 = p.scale_log2;
    uint32_t s_par = 0, pv_cnt = 0, x_cnt = 0;
    bool ok = true;
    // The two warps of a lane quarter trade one value per row: each writes
    // its own, both arrive on the quarter's barrier, each reads the other's.
    // Buffers alternate, so a warp writes a buffer again only after its
    // partner has passed the exchange in between, i.e. has read it.
    auto exchange = [&](float val, float* other) -> bool {
      float* buf = xchg + (x_cnt & 1u) * 2 * kBlockM;
      buf[half * kBlockM + row] = val;
      __syncwarp();
      if (lane == 0) mbar_arrive(xbar);
      const bool got = warp_wait(xbar, x_cnt & 1u, ctl, kStatusTimeoutSoftmax);
      *other = buf[(1 - half) * kBlockM + row];
      ++x_cnt;
      return got;
    };
    for (int v = blockIdx.x; v < p.num_tiles && ok; v += gridDim.x) {
      const TileCoord tc = tile_coord<Causal, 1, false, false>(p, v);
      const int n = wide_steps<Causal>(tc);
      const int r0 = tc.m0;
      const int grow = r0 + row;  // query row within its sequence
      const bool live = grow < tc.sq;
      const int64_t orow = (static_cast<int64_t>(tc.ob) * p.sq + tc.q0 + grow) * p.heads + tc.h;
      if (n == 0) {
        if (live) {  // no key visible to these rows: O = 0
          uint4* dst = reinterpret_cast<uint4*>(p.o + orow * kHeadDim + half * 64);
#pragma unroll
          for (int c = 0; c < 8; ++c) dst[c] = make_uint4(0u, 0u, 0u, 0u);
          if (half == 0 && p.lse != nullptr)
            p.lse[(static_cast<int64_t>(tc.ob) * p.heads + tc.h) * p.sq + tc.q0 + grow] = -INFINITY;
        }
        continue;
      }
      float m = -INFINITY, l = 0.f;  // l: this warp's half of the row sum
      for (int j = 0; j < n; ++j) {
        if (!warp_wait(bar(L::kSFull), s_par, ctl, kStatusTimeoutSoftmax)) { ok = false; break; }
        s_par ^= 1u;
        tc_fence_after();
        uint32_t sr[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(t_s + c * 32, sr[c]);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(L::kSLoad));  // S(j+1) may overwrite S now
        float s[128];
#pragma unroll
        for (int c = 0; c < 128; ++c) s[c] = __uint_as_float(sr[c / 32][c % 32]);
        const int col0 = tc.kv_begin + j * kWideN + half * 128;
        // Mask keys past kv_end, and (causal) keys after this row.
        const bool masked = (col0 + 128 > tc.kv_end) || (Causal && (col0 + 127 > r0));
        if (masked) {
          int lim = tc.kv_end - 1 - col0;  // last visible column index within this half
          if (Causal) lim = min(lim, grow - col0);
#pragma unroll
          for (int c = 0; c < 128; ++c) s[c] = c > lim ? -INFINITY : s[c];
        }
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
        float mx_other;
        if (!exchange(mx, &mx_other)) { ok = false; break; }
        // Both warps of the row see the same two maxima, so they take the
        // same decisions below.
        const float cand = fmaxf(m, fmaxf(mx, mx_other));
        const bool update = (j == 0) || (cand > m + kRescaleThreshold);
        const float m_new = update ? cand : m;
        const bool rescale = (j > 0) && __any_sync(0xffffffffu, update);
        const float alpha = rescale ? ((m_new == -INFINITY) ? 1.f : ex2_mufu(m - m_new)) : 1.f;
        m = m_new;
        const float mb = (m == -INFINITY) ? 0.f : m;
        // P(j) in registers while PV(j-1) still reads P(j-1) from TMEM.
        uint32_t pk[64];
        const float rowsum = masked ? exp_pack_regs<PolyPer8, true>(s, scale_log2, mb, pk)
                                    : exp_pack_regs<PolyPer8, false>(s, scale_log2, mb, pk);
        l = l * alpha + rowsum;
        if (j > 0) {
          // PV(j-1) has read P(j-1) and added into O: P(j) and a rescale of O may go ahead.
          if (!warp_wait(bar(L::kPVDone), pv_cnt & 1u, ctl, kStatusTimeoutSoftmax)) { ok = false; break; }
          ++pv_cnt;
          tc_fence_after();
        }
        if (rescale) {
          const float2 a2 = make_float2(alpha, alpha);
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            uint32_t orw[32];
            tmem_ld32(t_o + c * 32, orw);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              const float2 x = __fmul2_rn(make_float2(__uint_as_float(orw[e]), __uint_as_float(orw[e + 1])), a2);
              orw[e] = __float_as_uint(x.x);
              orw[e + 1] = __float_as_uint(x.y);
            }
            tmem_st32(t_o + c * 32, orw);
          }
        }
        {
          uint32_t (&p0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&pk[0]);
          uint32_t (&p1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&pk[32]);
          tmem_st32(t_p, p0);
          tmem_st32(t_p + 32, p1);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();  // every lane's P / O stores are complete
        if (lane == 0) mbar_arrive(bar(L::kPFull));
      }
      if (!ok) break;
      // ------------------------------ epilogue ------------------------------
      // PV(n-1) has finished: this warp's 64 columns of O are final.
      if (!warp_wait(bar(L::kPVDone), pv_cnt & 1u, ctl, kStatusTimeoutSoftmax)) { ok = false; break; }
      ++pv_cnt;
      tc_fence_after();
      uint32_t oh[2][32];
      tmem_ld32(t_o, oh[0]);
      tmem_ld32(t_o + 32, oh[1]);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(L::kOEmpty));  // O may take the next tile's PV
      float l_other;
      if (!exchange(l, &l_other)) { ok = false; break; }
      const float lt = l + l_other;  // the same sum in both warps (addition commutes)
      const float inv = lt > 0.f ? __frcp_rn(lt) : 0.f;
      if (live) {
        uint32_t pk[32];
#pragma unroll
        for (int e = 0; e < 32; ++e)
          pk[e] = pack_bf16x2(__uint_as_float(oh[e / 16][2 * (e % 16)]) * inv,
                              __uint_as_float(oh[e / 16][2 * (e % 16) + 1]) * inv);
        uint4* dst = reinterpret_cast<uint4*>(p.o + orow * kHeadDim + half * 64);
#pragma unroll
        for (int c = 0; c < 8; ++c) dst[c] = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        if (half == 0 && p.lse != nullptr)
          p.lse[(static_cast<int64_t>(tc.ob) * p.heads + tc.h) * p.sq + tc.q0 + grow] =
              lt > 0.f ? m * kLn2 + logf(lt) : -INFINITY;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace fav4
