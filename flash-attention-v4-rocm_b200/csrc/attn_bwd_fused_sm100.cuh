// Fused BF16 attention backward for B200 (sm_100a): dK, dV and the dQ
// partial sums of one key tile in a single pass over the query tiles.
//
// A work tile is (batch, K/V head, 128 keys). K_j and V_j stay in shared
// memory; for every query head of the K/V head's group (one head without
// grouped-query attention) and every query tile i that sees them (Q_i, dO_i
// and the tile's LSE*log2(e) and D rows arrive by TMA in a two-stage ring)
// the kernel computes
//
//   S^T = K_j Q_i^T          dP^T = V_j dO_i^T                 (TMEM)
//   P^T = exp2(S^T scale log2e - LSE2)   dS^T = P^T (dP^T - D)  (registers)
//   dV += P^T dO_i           dK += dS^T Q_i                    (TMEM, whole loop)
//   dQ_i(j) = dS K_j                                           (TMEM, per step)
//
// and adds dQ_i(j) into an FP32 accumulator with vector reductions
// (`red.global.add.v4.f32`); a separate pass scales and converts the
// accumulator to BF16. Five GEMMs per (i, j) pair, one exponential pass.
//
// dS goes to shared memory once, keys as rows and queries contiguous (128-byte
// swizzle, two 64-query boxes): the K-major A operand of dK = dS^T Q_i and the
// MN-major A operand of dQ = dS K_j.
//
// Roles (16 warps, 512 threads):
//   warps 0-7   elementwise. Warp w serves TMEM lanes 32 (w % 4) .. +31 (keys)
//               and query columns 64 (w / 4) .. +63 of S^T / dP^T.
//   warps 8-11  dQ drain: copy dQ_i(j) out of TMEM into registers (which frees
//               the columns for the next dP^T at once), then issue the
//               reductions; at the end of a work tile, the dK / dV epilogue.
//   warp 12     TMA producer. warp 13: one thread issues every MMA and owns
//               TMEM. warps 14-15 idle.
//
// TMEM (512 columns): T0 = S^T, T1 = dP^T, T2 = dV, T3 = dK. P^T (BF16 pairs)
// overwrites, for the query half h, columns [64 h, 64 h + 32) of T0: columns
// that only that half's warps read. dQ_i(j) reuses all of T1 once the
// elementwise warps have read dP^T.
//
// Issue order for step i (one thread, so the tensor pipe runs it in order):
//   dV(i)  S^T(i+1)  dK(i)  dQ(i)  [the drain has read dQ(i)]  dP^T(i+1)
// S^T(i+1) only waits for P^T(i) (the first elementwise phase), so the
// exponentials of step i+1 overlap dK(i), dQ(i), the drain and dP^T(i+1).
#pragma once
#include "attn_bwd_sm100.cuh"

namespace fav4 {

struct BwdFusedParams {
  const float* lse2;  // LSE * log2(e), [B, H, stat_stride] (rows past Sq are 0)
  const float* dsum;  // D = rowsum(dO * O), same layout
  float* dq_acc;      // [B, H, q tiles, 32 column quads, 128 rows, 4] FP32, zeroed before the launch
  __nv_bfloat16* dk;  // [B, Sk, H_kv, 128]
  __nv_bfloat16* dv;
  int batch, heads, sq, sk;
  int kv_heads, group;  // K/V heads, heads / kv_heads
  // Packed sequences (Varlen): batch entry b is rows [cu_q[b], cu_q[b+1]) of Q, O, dO, dQ against
  // [cu_k[b], cu_k[b+1]) of K, V, dK, dV; sq / sk are then the packed totals and max_sq / max_sk
  // bound every sequence (longer ones are cut to them).
  const int* cu_q;
  const int* cu_k;
  int max_sq, max_sk;
  int stat_stride;    // q tiles * 128 (q tiles of max_sq for packed sequences)
  float scale, scale_log2;
  int num_outer;      // key tiles per (batch, head)
  int num_tiles;      // batch * kv_heads * num_outer
  int num_items;      // causal head-pair schedule: work items (0 = plain stride over the tiles)
  int num_slots;      // loop positions the CTAs stride over (num_tiles, or 2 gridDim.x ceil(items / gridDim.x))
  uint32_t* status;
  uint64_t wait_limit_ns;
};

struct BwdFusedSmem {
  static constexpr int kK = 0;                        // K_j, 32 KiB (two 64-column boxes)
  static constexpr int kV = kTileBytes;               // V_j
  static constexpr int kQ = 2 * kTileBytes;           // [2 stages] Q_i
  static constexpr int kDO = 4 * kTileBytes;          // [2 stages] dO_i
  static constexpr int kDS = 6 * kTileBytes;          // dS, MN-major (two 64-query boxes)
  static constexpr int kStat = 7 * kTileBytes;        // [2 stages] LSE2[128], D[128]
  static constexpr int kStatBytes = 2 * kBlockM * 4;
  static constexpr int kBar = kStat + 2 * kStatBytes;
  static constexpr int kKVFull = 0, kKVEmpty = 1, kInFull = 2, kInEmpty = 4;
  static constexpr int kSFull = 6, kDPFull = 7, kPFull = 8, kDSFull = 9, kDQFull = 10, kDQEmpty = 11;
  static constexpr int kAccFull = 12, kAccEmpty = 13, kTeardown = 14;
  static constexpr int kNumBars = 15;
  static constexpr int kTmemHolder = kBar + kNumBars * 8;
  static constexpr int kAbort = kTmemHolder + 4;
  // No alignment slack fits: the kernel requires a 1 KiB-aligned dynamic
  // shared-memory base and reports kStatusSmemAlign otherwise.
  static constexpr int kBytes = kAbort + 4;
  static_assert(kBytes <= 227 * 1024, "shared memory budget");
};

// Register split: elementwise warpgroups, drain warpgroup, TMA/MMA warpgroup.
// (88 for the TMA/MMA warpgroup: with fewer the MMA issue loop spills to local memory.)
constexpr uint32_t kBwdLaunchRegs = 128, kBwdElemRegs = 144, kBwdDrainRegs = 136, kBwdOtherRegs = 88;
static_assert(128 * (2 * kBwdElemRegs + kBwdDrainRegs + kBwdOtherRegs) <= 512 * kBwdLaunchRegs,
              "register split exceeds the launch");
static_assert(kBwdElemRegs > kBwdLaunchRegs && kBwdDrainRegs > kBwdLaunchRegs && kBwdOtherRegs < kBwdLaunchRegs,
              "setmaxnreg.inc must raise and setmaxnreg.dec must lower the count");

// 1-D bulk copy global -> shared, completing on `bar` (16-byte aligned, size a multiple of 16).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

// One batch entry: its first query row and key in the (packed) tensors and its lengths.
struct BwdSeq {
  int q0, sq, k0, sk;
};
template <bool Varlen>
__device__ __forceinline__ BwdSeq bwd_seq(const BwdFusedParams& p, int b) {
  if (!Varlen) return BwdSeq{0, p.sq, 0, p.sk};
  // offsets clamped to the tensors and lengths to max_sq / max_sk: malformed offsets cannot move
  // an access outside the tensors, the statistics or the accumulator
  const int qa = min(max(__ldg(p.cu_q + b), 0), p.sq), qe = min(max(__ldg(p.cu_q + b + 1), qa), p.sq);
  const int ka = min(max(__ldg(p.cu_k + b), 0), p.sk), ke = min(max(__ldg(p.cu_k + b + 1), ka), p.sk);
  return BwdSeq{qa, min(qe - qa, p.max_sq), ka, min(ke - ka, p.max_sk)};
}

// Work tile at loop position v; every role walks v = blockIdx.x, + gridDim.x, ...
// below p.num_slots. Plain schedule: tile v of bwd_tile's order. Head-pair
// schedule (causal, p.num_items > 0; the host picks it when it balances
// better): a work item is the key tile q with the most query tiles to walk and
// the key tile nk-1-q with the fewest, of one (batch, K/V head), so all items
// cost the same and both read the same head's Q and dO. The long tile runs at
// position (2 (item / G)) G + item % G and the short one a wave later, on the
// same CTA (G = gridDim.x). -1: an empty position (past the last item, or the
// missing partner of a middle key tile).
__device__ __forceinline__ int bwd_sched(const BwdFusedParams& p, int v) {
  if (p.num_items == 0) return v;
  const int g = gridDim.x;
  const int w = v / g;
  const int item = (w >> 1) * g + (v - w * g);
  if (item >= p.num_items) return -1;
  const int nk = p.num_outer, per_b = ((nk + 1) >> 1) * p.kv_heads;
  const int b = item / per_b, r = item - b * per_b;
  const int q = r / p.kv_heads, h = r - q * p.kv_heads;
  if ((w & 1) && nk - 1 - q == q) return -1;
  const int k = (w & 1) ? nk - 1 - q : q;
  return (b * nk + k) * p.kv_heads + h;  // bwd_tile: w = k * kv_heads + h within batch entry b
}

template <bool Causal, bool Varlen>
__global__ void __launch_bounds__(512, 1)
    attn_bwd_fused_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                          const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                          const BwdFusedParams p) {
  using L = BwdFusedSmem;
  extern __shared__ __align__(1024) uint8_t fused_smem[];
  uint8_t* smem = fused_smem;
  const uint32_t sbase = smem_addr(smem);
  if (sbase & 1023u) {  // every thread leaves before any barrier or TMEM use
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
  BwdParams rp = {};  // the fields bwd_range / bwd_tile / bwd_step read
  rp.sq = p.sq;
  rp.sk = p.sk;
  rp.heads = p.heads;
  rp.kv_heads = p.kv_heads;
  rp.group = p.group;
  rp.num_outer = p.num_outer;

  if (threadIdx.x == 0) {
    *abort_flag = 0u;
    mbar_init(bar(L::kKVFull), 1);
    mbar_init(bar(L::kKVEmpty), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(L::kInFull + s), 1);
      mbar_init(bar(L::kInEmpty + s), 1 + 8);  // the MMA commit and every elementwise warp (statistics read)
    }
    mbar_init(bar(L::kSFull), 1);
    mbar_init(bar(L::kDPFull), 1);
    mbar_init(bar(L::kPFull), 8);
    mbar_init(bar(L::kDSFull), 8);
    mbar_init(bar(L::kDQFull), 1);
    mbar_init(bar(L::kDQEmpty), 4);
    mbar_init(bar(L::kAccFull), 1);
    mbar_init(bar(L::kAccEmpty), 4);
    mbar_init(bar(L::kTeardown), 1);
    fence_mbar_init();
  }
  if (warp == 12 && lane == 0) {
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_do);
  }
  if (warp == 13) {
    tmem_alloc(smem_addr(tmem_holder), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int nq = p.stat_stride / kBlockM;  // query tiles per (batch entry, head) in the accumulator

  if (warp >= 12) {
    regs_release<kBwdOtherRegs>();
    if (warp == 12 && lane == 0) {
      // ============================ TMA producer ============================
      const uint64_t pol = policy_evict_last();
      Ring ring;
      uint32_t kv_empty_par = 1;
      uint32_t armed = 0, armed_par = 0;  // stages (bits 0-1) and the K/V pair (bit 2) in flight
      bool ok = true;
      for (int v = blockIdx.x; v < p.num_slots && ok; v += gridDim.x) {
      const int t = bwd_sched(p, v);
      if (t < 0) continue;
        int b, h, idx, lo, hi;
        bwd_tile<Causal>(rp, t, b, h, idx, true);
        const int o0 = idx * kBlockN;
        const BwdSeq sq = bwd_seq<Varlen>(p, b);
        BwdParams rt = rp;
        rt.sq = sq.sq;
        rt.sk = sq.sk;
        bwd_range<true, Causal>(rt, o0, lo, hi);
        if (hi <= lo) continue;
        const int tb = Varlen ? 0 : b;  // batch coordinate of the tensor maps
        if (!mbar_wait(bar(L::kKVEmpty), kv_empty_par, ctl, kStatusTimeoutLoad)) { ok = false; break; }
        kv_empty_par ^= 1u;
        mbar_arrive_expect_tx(bar(L::kKVFull), 2 * kTileBytes);
        armed |= 4u;
        armed_par = (armed_par & ~4u) | (kv_empty_par << 2);
        for (int c = 0; c < 2; ++c) {
          tma_load_4d(sbase + L::kK + c * kBoxBytes, &tm_k, bar(L::kKVFull), c * 64, h, sq.k0 + o0, tb, pol);
          tma_load_4d(sbase + L::kV + c * kBoxBytes, &tm_v, bar(L::kKVFull), c * 64, h, sq.k0 + o0, tb, pol);
        }
        const int steps = bwd_steps<true>(rt, lo, hi);
        for (int st = 0; st < steps && ok; ++st) {
          int hq, i;
          bwd_step<true>(rt, h, lo, hi, st, hq, i);
          const int64_t stat_bh = (static_cast<int64_t>(b) * p.heads + hq) * p.stat_stride;
          if (!mbar_wait(bar(L::kInEmpty + ring.stage), ring.phase ^ 1u, ctl, kStatusTimeoutLoad)) {
            ok = false;
            break;
          }
          const uint32_t fb = bar(L::kInFull + ring.stage);
          mbar_arrive_expect_tx(fb, 2 * kTileBytes + L::kStatBytes);
          armed |= 1u << ring.stage;
          armed_par = (armed_par & ~(1u << ring.stage)) | (ring.phase << ring.stage);
          const int row = i * kBlockM;
          for (int c = 0; c < 2; ++c) {
            tma_load_4d(sbase + L::kQ + ring.stage * kTileBytes + c * kBoxBytes, &tm_q, fb, c * 64, hq, sq.q0 + row,
                        tb, pol);
            tma_load_4d(sbase + L::kDO + ring.stage * kTileBytes + c * kBoxBytes, &tm_do, fb, c * 64, hq,
                        sq.q0 + row, tb, pol);
          }
          const uint32_t sa = sbase + L::kStat + ring.stage * L::kStatBytes;
          bulk_load(sa, p.lse2 + stat_bh + row, kBlockM * 4, fb);
          bulk_load(sa + kBlockM * 4, p.dsum + stat_bh + row, kBlockM * 4, fb);
          ring.advance<2>();
        }
      }
      if (!ok) {
        // Let every copy this thread issued land before the CTA exits.
        WaitCtl drain{abort_flag, p.status, p.wait_limit_ns};
        volatile uint32_t no_abort = 0;
        drain.abort = &no_abort;
        for (int s = 0; s < 2; ++s)
          if (armed & (1u << s)) mbar_wait(bar(L::kInFull + s), (armed_par >> s) & 1u, drain, kStatusTimeoutDrain);
        if (armed & 4u) mbar_wait(bar(L::kKVFull), (armed_par >> 2) & 1u, drain, kStatusTimeoutDrain);
      }
    } else if (warp == 13 && lane == 0) {
      // ============================= MMA issuer =============================
      constexpr uint32_t idesc_ss = make_idesc_bf16(kBlockM, kBlockN, false);              // A, B K-major
      constexpr uint32_t idesc_ts = make_idesc_bf16(kBlockM, kHeadDim, true);              // A TMEM, B MN-major
      constexpr uint32_t idesc_dq = make_idesc_bf16(kBlockM, kHeadDim, true) | (1u << 15);  // A, B MN-major
      constexpr uint32_t idesc_dk = make_idesc_bf16(kBlockN, kHeadDim, true);               // A K-major, B MN-major
      const uint64_t dk = make_sdesc_sw128(sbase, 16, 1024);
      const uint64_t dv = make_sdesc_sw128(sbase, kBoxBytes, 1024);
      const uint32_t k_lo = static_cast<uint32_t>(dk), k_hi = static_cast<uint32_t>(dk >> 32);
      const uint32_t v_lo = static_cast<uint32_t>(dv), v_hi = static_cast<uint32_t>(dv >> 32);
      Ring ring;
      uint32_t kv_full_par = 0, p_par = 0, ds_par = 0, dq_empty_par = 1, acc_empty_par = 1;
      bool ok = true;
      // D (tmem column d) = A (shared tile a) B (shared tile b)^T over the head dimension, both K-major
      auto mma_ss = [&](uint32_t d, int a_off, int b_off) {
        const uint32_t aa = k_lo + (a_off >> 4), ba = k_lo + (b_off >> 4);
#pragma unroll
        for (int k = 0; k < kHeadDim / 16; ++k) {
          const uint32_t off = ((k / 4) * kBoxBytes + (k % 4) * 32) >> 4;
          umma_ss_w(tmem + d, aa + off, k_hi, ba + off, k_hi, idesc_ss, k > 0 ? 1u : 0u);
        }
      };
      // D (tmem column d) (+)= A (BF16 pairs in tmem column a: queries 0-63 at +0, 64-127 at +64)
      //                        B (shared tile b, MN-major) over the 128 queries
      auto mma_ts = [&](uint32_t d, uint32_t a, int b_off, bool acc) {
        const uint32_t ba = v_lo + (b_off >> 4);
#pragma unroll
        for (int k = 0; k < kBlockM / 16; ++k)
          umma_ts_w(tmem + d, tmem + a + k * 8 + (k >= 4 ? 32 : 0), ba + ((k * 2048) >> 4), v_hi, idesc_ts,
                    (acc || k > 0) ? 1u : 0u);
      };
      // T3 += dS^T Q_i over the 128 queries: A = dS (K-major: keys as rows), B = Q_i (MN-major)
      auto mma_dk = [&](int q_off, bool acc) {
#pragma unroll
        for (int k = 0; k < kBlockM / 16; ++k)
          umma_ss_w(tmem + 384, k_lo + ((L::kDS + (k / 4) * kBoxBytes + (k % 4) * 32) >> 4), k_hi,
                    v_lo + ((q_off + k * 2048) >> 4), v_hi, idesc_dk, (acc || k > 0) ? 1u : 0u);
      };
      // T1 = dS K_j over the 128 keys: A = dS (MN-major, queries contiguous), B = K_j (MN-major)
      auto mma_dq = [&]() {
#pragma unroll
        for (int k = 0; k < kBlockN / 16; ++k)
          umma_ss_w(tmem + 128, v_lo + ((L::kDS + k * 2048) >> 4), v_hi, v_lo + ((L::kK + k * 2048) >> 4), v_hi,
                    idesc_dq, k > 0 ? 1u : 0u);
      };
      for (int v = blockIdx.x; v < p.num_slots && ok; v += gridDim.x) {
      const int t = bwd_sched(p, v);
      if (t < 0) continue;
        int b, h, idx, lo, hi;
        bwd_tile<Causal>(rp, t, b, h, idx, true);
        const BwdSeq sq = bwd_seq<Varlen>(p, b);
        BwdParams rt = rp;
        rt.sq = sq.sq;
        rt.sk = sq.sk;
        bwd_range<true, Causal>(rt, idx * kBlockN, lo, hi);
        if (hi <= lo) continue;
        if (!mbar_wait(bar(L::kKVFull), kv_full_par, ctl, kStatusTimeoutMma)) { ok = false; break; }
        kv_full_par ^= 1u;
        if (!mbar_wait(bar(L::kInFull + ring.stage), ring.phase, ctl, kStatusTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        mma_ss(0, L::kK, L::kQ + ring.stage * kTileBytes);  // S^T(lo)
        tc_commit(bar(L::kSFull));
        if (!mbar_wait(bar(L::kDQEmpty), dq_empty_par, ctl, kStatusTimeoutMma)) { ok = false; break; }
        dq_empty_par ^= 1u;
        tc_fence_after();
        mma_ss(128, L::kV, L::kDO + ring.stage * kTileBytes);  // dP^T(lo)
        tc_commit(bar(L::kDPFull));
        const int steps = bwd_steps<true>(rt, lo, hi);
        for (int st = 0; st < steps && ok; ++st) {
          const int cur = ring.stage;
          Ring nxt = ring;
          nxt.advance<2>();
          const bool more = st + 1 < steps;
          if (!mbar_wait(bar(L::kPFull), p_par, ctl, kStatusTimeoutMma)) { ok = false; break; }
          p_par ^= 1u;
          if (st == 0) {
            if (!mbar_wait(bar(L::kAccEmpty), acc_empty_par, ctl, kStatusTimeoutMma)) { ok = false; break; }
            acc_empty_par ^= 1u;
          }
          tc_fence_after();
          mma_ts(256, 0, L::kDO + cur * kTileBytes, st > 0);  // dV += P^T dO_i
          if (more) {
            // S^T(i+1) overwrites T0 after dV has read P^T(i) (same thread, issue order)
            if (!mbar_wait(bar(L::kInFull + nxt.stage), nxt.phase, ctl, kStatusTimeoutMma)) { ok = false; break; }
            tc_fence_after();
            mma_ss(0, L::kK, L::kQ + nxt.stage * kTileBytes);
            tc_commit(bar(L::kSFull));
          }
          if (!mbar_wait(bar(L::kDSFull), ds_par, ctl, kStatusTimeoutMma)) { ok = false; break; }
          ds_par ^= 1u;
          tc_fence_after();
          mma_dk(L::kQ + cur * kTileBytes, st > 0);  // dK += dS^T Q_i
          tc_commit(bar(L::kInEmpty + cur));         // Q_i, dO_i read for the last time
          mma_dq();                                  // T1 = dS K_j
          tc_commit(bar(L::kDQFull));
          if (more) {
            if (!mbar_wait(bar(L::kDQEmpty), dq_empty_par, ctl, kStatusTimeoutMma)) { ok = false; break; }
            dq_empty_par ^= 1u;
            tc_fence_after();
            mma_ss(128, L::kV, L::kDO + nxt.stage * kTileBytes);  // dP^T(i+1)
            tc_commit(bar(L::kDPFull));
          }
          ring = nxt;
        }
        if (!ok) break;
        tc_commit(bar(L::kKVEmpty));
        tc_commit(bar(L::kAccFull));
      }
      tc_commit(bar(L::kTeardown));
      WaitCtl drain{abort_flag, p.status, p.wait_limit_ns};
      volatile uint32_t no_abort = 0;
      drain.abort = &no_abort;
      mbar_wait(bar(L::kTeardown), 0, drain, kStatusTimeoutDrain);
    }
    __syncwarp();
  } else if (warp >= 8) {
    // ====================== dQ drain and dK / dV epilogue =====================
    regs_claim<kBwdDrainRegs>();
    const int row = (warp % 4) * 32 + lane;  // TMEM lane: a query row (dQ) or a key (dK, dV)
    const uint32_t lane_off = static_cast<uint32_t>((warp % 4) * 32) << 16;
    uint32_t dq_par = 0, acc_full_par = 0;
    bool ok = true;
    for (int v = blockIdx.x; v < p.num_slots && ok; v += gridDim.x) {
      const int t = bwd_sched(p, v);
      if (t < 0) continue;
      int b, h, idx, lo, hi;
      bwd_tile<Causal>(rp, t, b, h, idx, true);
      const int o0 = idx * kBlockN;
      const BwdSeq sq = bwd_seq<Varlen>(p, b);
      BwdParams rt = rp;
      rt.sq = sq.sq;
      rt.sk = sq.sk;
      bwd_range<true, Causal>(rt, o0, lo, hi);
      const int key = o0 + row;
      // this key's row of dK / dV: [B, Sk, H_kv, 128] or packed [total_k, H_kv, 128]
      const int64_t krow = Varlen ? static_cast<int64_t>(sq.k0) + key : static_cast<int64_t>(b) * p.sk + key;
      const int steps = bwd_steps<true>(rt, lo, hi);
      for (int st = 0; st < steps; ++st) {
        int hq, i;
        bwd_step<true>(rt, h, lo, hi, st, hq, i);
        if (!warp_wait(bar(L::kDQFull), dq_par, ctl, kStatusTimeoutSoftmax)) { ok = false; break; }
        dq_par ^= 1u;
        tc_fence_after();
        uint32_t v[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tmem + lane_off + 128 + c * 32, v[c]);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(L::kDQEmpty));  // T1 may take dP^T(i+1)
        // tile (b, h, i) of the accumulator: [32 column quads][128 rows][4]; a warp's reduction
        // covers 32 consecutive rows of one quad, 512 contiguous bytes
        float* acc = p.dq_acc + ((static_cast<int64_t>(b) * p.heads + hq) * nq + i) * (kBlockM * kHeadDim) + row * 4;
#pragma unroll
        for (int q4 = 0; q4 < 32; ++q4) {
          const uint32_t* s = &v[q4 / 8][(q4 % 8) * 4];
          red_add_v4(acc + q4 * (kBlockM * 4), __uint_as_float(s[0]), __uint_as_float(s[1]), __uint_as_float(s[2]),
                     __uint_as_float(s[3]));
        }
      }
      if (!ok) break;
      if (hi <= lo) {
        // no query row sees these keys (causal, Sk > Sq): zero gradients
        if (key < sq.sk) {
          const int64_t off = (krow * p.kv_heads + h) * kHeadDim;
          uint4* d0 = reinterpret_cast<uint4*>(p.dk + off);
          uint4* d1 = reinterpret_cast<uint4*>(p.dv + off);
#pragma unroll
          for (int w = 0; w < 16; ++w) {
            d0[w] = make_uint4(0u, 0u, 0u, 0u);
            d1[w] = make_uint4(0u, 0u, 0u, 0u);
          }
        }
        continue;
      }
      if (!warp_wait(bar(L::kAccFull), acc_full_par, ctl, kStatusTimeoutSoftmax)) { ok = false; break; }
      acc_full_par ^= 1u;
      tc_fence_after();
      const int64_t off = (krow * p.kv_heads + h) * kHeadDim;
#pragma unroll 1
      for (int g = 0; g < 2; ++g) {
        // g = 0: dK (T3, times scale); g = 1: dV (T2)
        const uint32_t col = g == 0 ? 384u : 256u;
        const float mul = g == 0 ? p.scale : 1.f;
        __nv_bfloat16* dst_row = (g == 0 ? p.dk : p.dv) + off;
#pragma unroll 1
        for (int ch = 0; ch < 4; ++ch) {
          uint32_t a[32];
          tmem_ld32(tmem + lane_off + col + ch * 32, a);
          tmem_ld_wait();
          if (key < sq.sk) {
            uint4* dst = reinterpret_cast<uint4*>(dst_row + ch * 32);
#pragma unroll
            for (int w = 0; w < 4; ++w) {
              uint4 x;
              x.x = pack_bf16x2(__uint_as_float(a[8 * w + 0]) * mul, __uint_as_float(a[8 * w + 1]) * mul);
              x.y = pack_bf16x2(__uint_as_float(a[8 * w + 2]) * mul, __uint_as_float(a[8 * w + 3]) * mul);
              x.z = pack_bf16x2(__uint_as_float(a[8 * w + 4]) * mul, __uint_as_float(a[8 * w + 5]) * mul);
              x.w = pack_bf16x2(__uint_as_float(a[8 * w + 6]) * mul, __uint_as_float(a[8 * w + 7]) * mul);
              dst[w] = x;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(L::kAccEmpty));
    }
  } else {
    // ============================ elementwise =============================
    regs_claim<kBwdElemRegs>();
    const int half = warp / 4;                    // query columns 64 half .. +63
    const int key_lane = (warp % 4) * 32 + lane;  // TMEM lane = key within the tile
    const uint32_t lane_off = static_cast<uint32_t>((warp % 4) * 32) << 16;
    const uint32_t t_s = tmem + lane_off + half * 64;        // this half's S^T columns; P^T at +0..31
    const uint32_t t_dp = tmem + lane_off + 128 + half * 64;  // dP^T
    // dS row of this key in the MN-major A tile: box `half`, 128 bytes per key, 16-byte chunks swizzled
    uint8_t* ds_row = smem + L::kDS + half * kBoxBytes + key_lane * 128;
    const int sw = key_lane & 7;
    Ring ring;
    uint32_t s_par = 0, dp_par = 0;
    bool ok = true;
    const float2 sc = make_float2(p.scale_log2, p.scale_log2);
    for (int v = blockIdx.x; v < p.num_slots && ok; v += gridDim.x) {
      const int t = bwd_sched(p, v);
      if (t < 0) continue;
      int b, h, idx, lo, hi;
      bwd_tile<Causal>(rp, t, b, h, idx, true);
      const int o0 = idx * kBlockN;
      const BwdSeq sq = bwd_seq<Varlen>(p, b);
      BwdParams rt = rp;
      rt.sq = sq.sq;
      rt.sk = sq.sk;
      bwd_range<true, Causal>(rt, o0, lo, hi);
      const int key = o0 + key_lane;
      const int steps = bwd_steps<true>(rt, lo, hi);
      for (int st = 0; st < steps; ++st) {
        int hq, i;
        bwd_step<true>(rt, h, lo, hi, st, hq, i);
        const float* stat = reinterpret_cast<const float*>(smem + L::kStat + ring.stage * L::kStatBytes);
        if (!warp_wait(bar(L::kInFull + ring.stage), ring.phase, ctl, kStatusTimeoutSoftmax)) { ok = false; break; }
        if (!warp_wait(bar(L::kSFull), s_par, ctl, kStatusTimeoutSoftmax)) { ok = false; break; }
        s_par ^= 1u;
        tc_fence_after();
        const int q0 = i * kBlockM + half * 64;  // first query column of this half
        // masks only on boundary tiles: the causal diagonal and tails past Sq / Sk
        // (packed sequences: rows and keys past the sequence's end belong to the next one)
        const bool masked = (Causal && o0 + kBlockN - 1 > i * kBlockM) || i * kBlockM + kBlockM > sq.sq ||
                            o0 + kBlockN > sq.sk;
        // ---- phase A: P^T = exp2(S^T scale log2e - LSE2) ----
        float pr[64];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t sr[32];
          tmem_ld32(t_s + c * 32, sr);
          tmem_ld_wait();
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            const float4 l4 = *reinterpret_cast<const float4*>(stat + half * 64 + c * 32 + e);
#pragma unroll
            for (int u = 0; u < 4; u += 2) {
              const float2 nl = make_float2(-(u == 0 ? l4.x : l4.z), -(u == 0 ? l4.y : l4.w));
              const float2 x = __ffma2_rn(make_float2(__uint_as_float(sr[e + u]), __uint_as_float(sr[e + u + 1])), sc, nl);
              float2 v2 = make_float2(ex2_mufu(x.x), ex2_mufu(x.y));
              if (masked) {
                const int qa = q0 + c * 32 + e + u;
                if (!(qa < sq.sq && key < sq.sk && (!Causal || key <= qa))) v2.x = 0.f;
                if (!(qa + 1 < sq.sq && key < sq.sk && (!Causal || key <= qa + 1))) v2.y = 0.f;
              }
              pr[c * 32 + e + u] = v2.x;
              pr[c * 32 + e + u + 1] = v2.y;
              pk[(e + u) / 2] = pack_bf16x2(v2.x, v2.y);
            }
          }
          tmem_st16(t_s + c * 16, pk);  // over S^T columns this thread has read
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(L::kPFull));
        // ---- phase B: dS^T = P^T (dP^T - D) -> shared memory (dK, dQ) ----
        if (!warp_wait(bar(L::kDPFull), dp_par, ctl, kStatusTimeoutSoftmax)) { ok = false; break; }
        dp_par ^= 1u;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t dr[32];
          tmem_ld32(t_dp + c * 32, dr);
          tmem_ld_wait();
          uint32_t dk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            const float4 d4 = *reinterpret_cast<const float4*>(stat + kBlockM + half * 64 + c * 32 + e);
            const float2 da = __fadd2_rn(make_float2(__uint_as_float(dr[e]), __uint_as_float(dr[e + 1])),
                                         make_float2(-d4.x, -d4.y));
            const float2 db = __fadd2_rn(make_float2(__uint_as_float(dr[e + 2]), __uint_as_float(dr[e + 3])),
                                         make_float2(-d4.z, -d4.w));
            const float2 sa = __fmul2_rn(make_float2(pr[c * 32 + e], pr[c * 32 + e + 1]), da);
            const float2 sb = __fmul2_rn(make_float2(pr[c * 32 + e + 2], pr[c * 32 + e + 3]), db);
            dk[e / 2] = pack_bf16x2(sa.x, sa.y);
            dk[e / 2 + 1] = pack_bf16x2(sb.x, sb.y);
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int chunk = c * 4 + j;  // 8 queries per 16-byte chunk
            *reinterpret_cast<uint4*>(ds_row + ((chunk ^ sw) << 4)) =
                make_uint4(dk[4 * j], dk[4 * j + 1], dk[4 * j + 2], dk[4 * j + 3]);
          }
        }
        fence_proxy_async_smem();  // dS visible to the tensor core
        tc_fence_before();         // dP^T reads done: T1 may take dQ
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(bar(L::kDSFull));
          mbar_arrive(bar(L::kInEmpty + ring.stage));  // this stage's statistics are read
        }
        ring.advance<2>();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 13) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// dQ = scale * accumulator, BF16 [B, Sq, H, 128] (packed [total_q, H, 128] when cu_q is
// given: batch entry b's rows go to cu_q[b] + r, at most max_sq of them). nq query tiles per
// (batch entry, head) in the accumulator. One thread per (tile row, 32 columns): eight 16-byte
// accumulator loads (a warp reads 512 contiguous bytes per load) and four 16-byte stores.
__global__ void __launch_bounds__(256) attn_bwd_dq_convert_kernel(const float* __restrict__ acc,
                                                                  __nv_bfloat16* __restrict__ dq, int batch,
                                                                  int heads, int sq, int nq, float scale,
                                                                  const int* __restrict__ cu_q, int max_sq) {
  const int64_t total = static_cast<int64_t>(batch) * heads * nq * kBlockM * 4;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(t % kBlockM);
    const int64_t rest = t / kBlockM;
    const int oct = static_cast<int>(rest % 4);  // columns 32 oct .. +31
    const int64_t tile = rest / 4;               // (b * heads + h) * nq + i
    const int i = static_cast<int>(tile % nq);
    const int64_t bh = tile / nq;
    const int h = static_cast<int>(bh % heads);
    const int64_t b = bh / heads;
    const int q = i * kBlockM + r;
    int64_t orow;  // row of dQ
    if (cu_q) {
      const int qa = min(max(__ldg(cu_q + b), 0), sq), qe = min(max(__ldg(cu_q + b + 1), qa), sq);
      if (q >= min(qe - qa, max_sq)) continue;
      orow = qa + q;
    } else {
      if (q >= sq) continue;
      orow = b * sq + q;
    }
    const float4* src = reinterpret_cast<const float4*>(acc + tile * (kBlockM * kHeadDim)) + oct * 8 * kBlockM + r;
    uint4* dst = reinterpret_cast<uint4*>(dq + (orow * heads + h) * kHeadDim + oct * 32);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float4 x = src[(2 * w) * kBlockM], y = src[(2 * w + 1) * kBlockM];
      dst[w] = make_uint4(pack_bf16x2(x.x * scale, x.y * scale), pack_bf16x2(x.z * scale, x.w * scale),
                          pack_bf16x2(y.x * scale, y.y * scale), pack_bf16x2(y.z * scale, y.w * scale));
    }
  }
}

// Packed sequences: D = rowsum(dO * O) and LSE * log2(e) into [B, H, stat_stride] (batch entry b's
// row r from packed row cu_q[b] + r; 0 past the entry's length, at most max_sq), from O, dO
// [total_q, H, 128] and the forward's LSE [H, total_q]. Two (b, r, h) slots per warp, half a warp
// each, with the same per-row arithmetic as attn_bwd_dsum_kernel (row_dot_half).
__global__ void __launch_bounds__(256) attn_bwd_dsum_varlen_kernel(
    const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout, const float* __restrict__ lse,
    float* __restrict__ dsum, float* __restrict__ lse2, const int* __restrict__ cu_q, int batch, int heads,
    int total_q, int max_sq, int stat_stride) {
  const int64_t slots = static_cast<int64_t>(batch) * stat_stride * heads;
  const int lane = threadIdx.x % 32;
  const int half = lane / 16, sub = lane % 16;
  for (int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32; 2 * w < slots;
       w += static_cast<int64_t>(gridDim.x) * blockDim.x / 32) {
    const int64_t slot = 2 * w + half;  // (b * stat_stride + r) * heads + h
    const bool in = slot < slots;
    const int h = static_cast<int>(slot % heads);
    const int64_t br = slot / heads;
    const int r = static_cast<int>(br % stat_stride);
    const int b = static_cast<int>(min(br / stat_stride, static_cast<int64_t>(batch - 1)));
    const int qa = min(max(__ldg(cu_q + b), 0), total_q), qe = min(max(__ldg(cu_q + b + 1), qa), total_q);
    const bool live = in && r < min(qe - qa, max_sq);
    const int64_t row = live ? (static_cast<int64_t>(qa) + r) * heads + h : 0;
    const float s = row_dot_half(o + row * kHeadDim, dout + row * kHeadDim, sub, live);
    if (sub == 0 && in) {
      const int64_t at = (static_cast<int64_t>(b) * heads + h) * stat_stride + r;
      dsum[at] = s;
      lse2[at] = live ? lse[static_cast<int64_t>(h) * total_q + qa + r] * 1.4426950408889634f : 0.f;
    }
  }
}

}  // namespace fav4
