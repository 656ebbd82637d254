// BF16 attention backward for B200 (sm_100a), BSHD layout, head dim 128.
//
// The reference implements only the forward pass (README.md:24). These
// kernels are the deterministic backward path (fav4_bshd_backward_deterministic;
// the fused kernel in attn_bwd_fused_sm100.cuh is the default). They compute
// dQ, dK, dV of O = softmax(Q K^T * scale) V (top-left causal or dense) from
// Q, K, V, O, dO and the forward's LSE, with the standard recomputation
// formulas (no attention matrix in HBM, no atomics, results deterministic):
//
//   P = exp(S - LSE), S = scale Q K^T     D = rowsum(dO * O)   (preprocess)
//   dV = P^T dO     dP = dO V^T     dS = P * (dP - D)
//   dK = scale dS^T Q                   dQ = scale dS K
//
// One kernel template, two modes:
//   KV mode: a work tile is (batch, K/V head, 128 keys); K_j and V_j stay in
//            shared memory while the loop runs over each query head of the
//            K/V head's group and the query tiles i that see them
//            (bwd_step): S^T = K_j Q_i^T and dP^T = V_j dO_i^T (TMEM), then per
//            key (TMEM lane) P^T and dS^T, then dV += P^T dO_i and
//            dK += dS^T Q_i, accumulated in TMEM for the whole loop.
//   Q mode:  a work tile is (batch, head, 128 query rows); Q_i and dO_i stay,
//            the loop runs over the key tiles j: S, dP, dS per row, then
//            dQ += dS K_j.
// Every MMA form is the forward's: A and B K-major in shared memory for S and
// dP, A (P^T, dS^T or dS as BF16 pairs) from TMEM with B MN-major for the
// accumulations.
//
//   warps 0-3  elementwise: one TMEM lane per thread, 32 columns at a time
//   warp 4     TMA: the outer tile pair once per work tile, then a ring of two
//              stages of the inner tile pair
//   warp 5     one thread issues every MMA and allocates TMEM
//
// TMEM (512 columns): T0 S^T / S, T1 dP^T / dP (their first 64 columns are
// overwritten by P^T and dS^T / dS), T2 dV / dQ, T3 dK.
#pragma once
#include "attn_fwd_sm100.cuh"

namespace fav4 {

struct BwdParams {
  const float* lse2;  // forward LSE * log2(e) [B, H, stat_stride] (written by the preprocess)
  const float* dsum;  // D = rowsum(dO * O) [B, H, stat_stride]
  __nv_bfloat16* g0;  // KV mode: dK, Q mode: dQ  ([B, S, H, 128])
  __nv_bfloat16* g1;  // KV mode: dV
  int batch, heads, sq, sk;
  int kv_heads;       // K / V heads (a divisor of heads: grouped-query attention)
  int group;          // heads / kv_heads
  int stat_stride;    // row stride of lse2 / dsum (>= sq)
  float scale;        // softmax scale
  float scale_log2;   // scale * log2(e)
  int num_outer;      // outer tiles per (batch, head)
  int num_tiles;      // batch * (KV mode: kv_heads, Q mode: heads) * num_outer
  uint32_t* status;
  uint64_t wait_limit_ns;
};

struct BwdSmem {
  static constexpr int kOuter = 0;                   // 2 x 32 KiB
  static constexpr int kInner = 2 * kTileBytes;      // 2 stages x 2 x 32 KiB
  static constexpr int kBar = kInner + 4 * kTileBytes;
  static constexpr int kOuterFull = 0, kOuterEmpty = 1, kInFull = 2, kInEmpty = 4;
  static constexpr int kSFull = 6, kPFull = 7;  // kPFull: [4] one per 32-column chunk of P^T / dS^T
  static constexpr int kAccFull = 11, kAccEmpty = 12, kTeardown = 13;
  static constexpr int kNumBars = 14;
  static constexpr int kTmemHolder = kBar + kNumBars * 8;
  static constexpr int kAbort = kTmemHolder + 4;
  static constexpr int kBytes = kAbort + 4;
  static constexpr int kAlloc = kBytes + 1024;
  static_assert(kAlloc <= 227 * 1024, "shared memory budget");
};

// Inner-loop range of a work tile: KV mode, query tiles [lo, hi) that see keys
// [o0, o0+128); Q mode, key tiles [lo, hi) that rows [o0, o0+128) see.
template <bool KV, bool Causal>
__device__ __forceinline__ void bwd_range(const BwdParams& p, int o0, int& lo, int& hi) {
  const int nq = (p.sq + kBlockM - 1) / kBlockM, nk = (p.sk + kBlockN - 1) / kBlockN;
  if (KV) {
    lo = Causal ? o0 / kBlockM : 0;  // a query row r sees key c iff c <= r
    hi = (o0 < p.sk && (!Causal || o0 < p.sq)) ? nq : lo;
  } else {
    lo = 0;
    hi = o0 < p.sq ? (Causal ? min(nk, o0 / kBlockN + 1) : nk) : 0;
  }
}

// Work tile t: batch b, head h (KV mode: a K / V head, Q mode: a query head), outer tile idx.
template <bool Causal>
__device__ __forceinline__ void bwd_tile(const BwdParams& p, int t, int& b, int& h, int& idx, bool kv) {
  const int th = kv ? p.kv_heads : p.heads;
  const int per_batch = th * p.num_outer;
  b = t / per_batch;
  const int w = t - b * per_batch;
  h = w % th;
  const int k = w / th;
  // causal: the longest loops first (low key tiles in KV mode, high row tiles in Q mode)
  idx = (Causal && !kv) ? p.num_outer - 1 - k : k;
}

// Inner steps of a work tile. KV mode walks the query tiles [lo, hi) of each
// query head of the K / V head's group in turn (dK, dV sum over the group);
// Q mode walks the key tiles [lo, hi).
template <bool KV>
__device__ __forceinline__ int bwd_steps(const BwdParams& p, int lo, int hi) {
  return KV ? (hi - lo) * p.group : hi - lo;
}
// Step s: the query head hq of the inner tile and the inner tile index n.
template <bool KV>
__device__ __forceinline__ void bwd_step(const BwdParams& p, int h, int lo, int hi, int s, int& hq, int& n) {
  if (KV) {
    const int len = hi - lo;
    hq = h * p.group + s / len;
    n = lo + s % len;
  } else {
    hq = h;
    n = lo + s;
  }
}

template <bool KV, bool Causal>
__global__ void __launch_bounds__(192, 1)
    attn_bwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_o0, const __grid_constant__ CUtensorMap tm_o1,
                          const __grid_constant__ CUtensorMap tm_i0, const __grid_constant__ CUtensorMap tm_i1,
                          const BwdParams p) {
  using L = BwdSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_addr(smem);
  const uint32_t bar0 = sbase + L::kBar;
  auto bar = [&](int slot) -> uint32_t { return bar0 + 8u * slot; };
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + L::kAbort);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::kTmemHolder);
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  WaitCtl ctl{abort_flag, p.status, p.wait_limit_ns};

  if (threadIdx.x == 0) {
    *abort_flag = 0u;
    mbar_init(bar(L::kOuterFull), 1);
    mbar_init(bar(L::kOuterEmpty), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(L::kInFull + s), 1);
      mbar_init(bar(L::kInEmpty + s), 1);
    }
    mbar_init(bar(L::kSFull), 1);
    for (int c = 0; c < 4; ++c) mbar_init(bar(L::kPFull + c), 4);  // elementwise warps, per chunk
    mbar_init(bar(L::kAccFull), 1);
    mbar_init(bar(L::kAccEmpty), 4);  // elementwise warps, after the epilogue read
    mbar_init(bar(L::kTeardown), 1);
    fence_mbar_init();
  }
  if (warp == 4 && lane == 0) {
    tma_prefetch_desc(&tm_o0);
    tma_prefetch_desc(&tm_o1);
    tma_prefetch_desc(&tm_i0);
    tma_prefetch_desc(&tm_i1);
  }
  if (warp == 5) {
    tmem_alloc(smem_addr(tmem_holder), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 4) {
    // ============================ TMA producer ============================
    if (lane == 0) {
      const uint64_t pol = policy_evict_last();
      Ring ring;
      uint32_t outer_empty_par = 1;
      uint32_t armed = 0, armed_par = 0;  // inner stages (bits 0-1) and the outer pair (bit 2) in flight
      bool ok = true;
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        int b, h, idx, lo, hi;
        bwd_tile<Causal>(p, t, b, h, idx, KV);
        const int o0 = idx * kBlockM;
        bwd_range<KV, Causal>(p, o0, lo, hi);
        if (hi <= lo) continue;
        if (!mbar_wait(bar(L::kOuterEmpty), outer_empty_par, ctl, kStatusTimeoutLoad)) { ok = false; break; }
        outer_empty_par ^= 1u;
        mbar_arrive_expect_tx(bar(L::kOuterFull), 2 * kTileBytes);
        armed |= 4u;
        armed_par = (armed_par & ~4u) | (outer_empty_par << 2);  // parity of this fill
        for (int c = 0; c < 2; ++c) {
          tma_load_4d(sbase + L::kOuter + c * kBoxBytes, &tm_o0, bar(L::kOuterFull), c * 64, h, o0, b, pol);
          tma_load_4d(sbase + L::kOuter + kTileBytes + c * kBoxBytes, &tm_o1, bar(L::kOuterFull), c * 64, h, o0, b,
                      pol);
        }
        const int steps = bwd_steps<KV>(p, lo, hi);
        for (int st = 0; st < steps && ok; ++st) {
          int hq, n;
          bwd_step<KV>(p, h, lo, hi, st, hq, n);
          const int hi_head = KV ? hq : h / p.group;  // head of the inner tensors (Q, dO or K, V)
          if (!mbar_wait(bar(L::kInEmpty + ring.stage), ring.phase ^ 1u, ctl, kStatusTimeoutLoad)) {
            ok = false;
            break;
          }
          const uint32_t fb = bar(L::kInFull + ring.stage);
          mbar_arrive_expect_tx(fb, 2 * kTileBytes);
          armed |= 1u << ring.stage;
          armed_par = (armed_par & ~(1u << ring.stage)) | (ring.phase << ring.stage);
          const uint32_t dst = sbase + L::kInner + ring.stage * 2 * kTileBytes;
          const int row = n * kBlockM;
          for (int c = 0; c < 2; ++c) {
            tma_load_4d(dst + c * kBoxBytes, &tm_i0, fb, c * 64, hi_head, row, b, pol);
            tma_load_4d(dst + kTileBytes + c * kBoxBytes, &tm_i1, fb, c * 64, hi_head, row, b, pol);
          }
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
        if (armed & 4u) mbar_wait(bar(L::kOuterFull), (armed_par >> 2) & 1u, drain, kStatusTimeoutDrain);
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    // ============================= MMA issuer =============================
    if (lane == 0) {
      constexpr uint32_t idesc_ss = make_idesc_bf16(kBlockM, kBlockN, false);
      constexpr uint32_t idesc_ts = make_idesc_bf16(kBlockM, kHeadDim, true);
      const uint64_t dk = make_sdesc_sw128(sbase, 16, 1024);
      const uint64_t dv = make_sdesc_sw128(sbase, kBoxBytes, 1024);
      const uint32_t k_lo = static_cast<uint32_t>(dk), k_hi = static_cast<uint32_t>(dk >> 32);
      const uint32_t v_lo = static_cast<uint32_t>(dv), v_hi = static_cast<uint32_t>(dv >> 32);
      Ring ring;
      uint32_t outer_full_par = 0, p_par = 0, acc_empty_par = 1;
      bool ok = true;
      // D (tmem column d) = A (shared tile a) * B (shared tile bt)^T, both K-major
      auto mma_ss = [&](uint32_t d, int a_off, int b_off) {
        const uint32_t aa = k_lo + (a_off >> 4), ba = k_lo + (b_off >> 4);
#pragma unroll
        for (int k = 0; k < kHeadDim / 16; ++k) {
          const uint32_t off = ((k / 4) * kBoxBytes + (k % 4) * 32) >> 4;
          umma_ss_w(tmem + d, aa + off, k_hi, ba + off, k_hi, idesc_ss, k > 0 ? 1u : 0u);
        }
      };
      // D (tmem column d) (+)= A (tmem column a, BF16 pairs) * B (shared tile b, MN-major), K steps
      // [2 ch, 2 ch + 2): the 32 columns of chunk ch
      auto mma_ts = [&](uint32_t d, uint32_t a, int b_off, bool acc, int ch) {
        const uint32_t ba = v_lo + (b_off >> 4);
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const int k = 2 * ch + kk;
          umma_ts_w(tmem + d, tmem + a + k * 8, ba + ((k * 2048) >> 4), v_hi, idesc_ts, (acc || k > 0) ? 1u : 0u);
        }
      };
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        int b, h, idx, lo, hi;
        bwd_tile<Causal>(p, t, b, h, idx, KV);
        bwd_range<KV, Causal>(p, idx * kBlockM, lo, hi);
        if (hi <= lo) continue;
        if (!mbar_wait(bar(L::kOuterFull), outer_full_par, ctl, kStatusTimeoutMma)) { ok = false; break; }
        outer_full_par ^= 1u;
        if (!mbar_wait(bar(L::kAccEmpty), acc_empty_par, ctl, kStatusTimeoutMma)) { ok = false; break; }
        acc_empty_par ^= 1u;
        const int steps = bwd_steps<KV>(p, lo, hi);
        for (int st = 0; st < steps && ok; ++st) {
          if (!mbar_wait(bar(L::kInFull + ring.stage), ring.phase, ctl, kStatusTimeoutMma)) { ok = false; break; }
          tc_fence_after();
          const int in0 = L::kInner + ring.stage * 2 * kTileBytes, in1 = in0 + kTileBytes;
          mma_ss(0, L::kOuter, in0);                // T0 = outer0 inner0^T
          mma_ss(128, L::kOuter + kTileBytes, in1);  // T1 = outer1 inner1^T
          tc_commit(bar(L::kSFull));
          // the accumulating MMAs of each 32-column chunk as soon as it is stored
#pragma unroll 1
          for (int ch = 0; ch < 4 && ok; ++ch) {
            if (!mbar_wait(bar(L::kPFull + ch), p_par, ctl, kStatusTimeoutMma)) { ok = false; break; }
            tc_fence_after();
            if (KV) {
              mma_ts(256, 0, in1, st > 0, ch);    // dV += P^T dO_i
              mma_ts(384, 128, in0, st > 0, ch);  // dK += dS^T Q_i
            } else {
              mma_ts(256, 128, in0, st > 0, ch);  // dQ += dS K_j
            }
          }
          if (!ok) break;
          p_par ^= 1u;
          tc_commit(bar(L::kInEmpty + ring.stage));
          ring.advance<2>();
        }
        if (!ok) break;
        tc_commit(bar(L::kOuterEmpty));
        tc_commit(bar(L::kAccFull));
      }
      tc_commit(bar(L::kTeardown));
      WaitCtl drain{abort_flag, p.status, p.wait_limit_ns};
      volatile uint32_t no_abort = 0;
      drain.abort = &no_abort;
      mbar_wait(bar(L::kTeardown), 0, drain, kStatusTimeoutDrain);
    }
    __syncwarp();
  } else {
    // ============================ elementwise =============================
    const int row = warp * 32 + lane;  // TMEM lane: a key (KV mode) or a query row (Q mode)
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    uint32_t s_par = 0, acc_full_par = 0;
    bool ok = true;
    const float2 sc = make_float2(p.scale_log2, p.scale_log2);
    for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
      int b, h, idx, lo, hi;
      bwd_tile<Causal>(p, t, b, h, idx, KV);
      const int o0 = idx * kBlockM;
      bwd_range<KV, Causal>(p, o0, lo, hi);
      const int mine = o0 + row;  // this thread's key (KV) or query row (Q)
      // LSE / D row base (Q mode: this work tile's head; KV mode: set per step below)
      int64_t stat0 = (static_cast<int64_t>(b) * p.heads + h) * p.stat_stride;
      // Q mode: this row's statistics (rows past Sq read row Sq-1 and are not stored)
      float2 lse2_row = make_float2(0.f, 0.f), d_row = make_float2(0.f, 0.f);
      if (!KV) {
        const int r = min(mine, p.sq - 1);
        lse2_row.x = lse2_row.y = -p.lse2[stat0 + r];
        d_row.x = d_row.y = -p.dsum[stat0 + r];
      }
      const int steps = bwd_steps<KV>(p, lo, hi);
      for (int st = 0; st < steps; ++st) {
        int hq, n;
        bwd_step<KV>(p, h, lo, hi, st, hq, n);
        if (KV) stat0 = (static_cast<int64_t>(b) * p.heads + hq) * p.stat_stride;
        if (!warp_wait(bar(L::kSFull), s_par, ctl, kStatusTimeoutSoftmax)) { ok = false; break; }
        s_par ^= 1u;
        tc_fence_after();
        const int c0 = n * kBlockN;  // first column: a query row (KV) or a key (Q)
        // Masks only on boundary tiles: the causal diagonal and tails past Sq / Sk (rows and keys past
        // the ends read zeros from TMA, which contribute nothing; the mask keeps exp2 finite there).
        const int r_lo = KV ? c0 : o0, k_lo = KV ? o0 : c0;
        const bool masked = (Causal && k_lo + kBlockN - 1 > r_lo) || r_lo + kBlockM > p.sq || k_lo + kBlockN > p.sk;
#pragma unroll 1
        for (int ch = 0; ch < 4; ++ch) {
          uint32_t sr[32], dr[32];
          tmem_ld32(tmem + lane_off + ch * 32, sr);
          tmem_ld32(tmem + lane_off + 128 + ch * 32, dr);
          // KV mode: the chunk's 32 query rows' statistics (the same for every lane), negated
          float nl[32], nd[32];
          if (KV) {
            const int r0c = c0 + ch * 32;
            if (r0c + 32 <= p.sq && ((stat0 + r0c) & 3) == 0) {  // whole chunk, 16-byte aligned
              const float4* l4 = reinterpret_cast<const float4*>(p.lse2 + stat0 + r0c);
              const float4* d4 = reinterpret_cast<const float4*>(p.dsum + stat0 + r0c);
#pragma unroll
              for (int v = 0; v < 8; ++v) {
                const float4 x = l4[v], y = d4[v];
                nl[4 * v] = -x.x, nl[4 * v + 1] = -x.y, nl[4 * v + 2] = -x.z, nl[4 * v + 3] = -x.w;
                nd[4 * v] = -y.x, nd[4 * v + 1] = -y.y, nd[4 * v + 2] = -y.z, nd[4 * v + 3] = -y.w;
              }
            } else {
#pragma unroll
              for (int c = 0; c < 32; ++c) {
                const int rc = min(r0c + c, p.sq - 1);
                nl[c] = -p.lse2[stat0 + rc];
                nd[c] = -p.dsum[stat0 + rc];
              }
            }
          }
          tmem_ld_wait();
          uint32_t pk[16], dk[16];
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const float2 nl2 = KV ? make_float2(nl[c], nl[c + 1]) : lse2_row;
            const float2 nd2 = KV ? make_float2(nd[c], nd[c + 1]) : d_row;
            const float2 x = __ffma2_rn(make_float2(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])), sc, nl2);
            float2 pr = make_float2(ex2_mufu(x.x), ex2_mufu(x.y));
            if (masked) {
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const int col = c0 + ch * 32 + c + e;
                const int r = KV ? col : mine, key = KV ? mine : col;
                const bool valid = r < p.sq && key < p.sk && (!Causal || key <= r);
                if (!valid) (e == 0 ? pr.x : pr.y) = 0.f;
              }
            }
            const float2 dp = __fadd2_rn(make_float2(__uint_as_float(dr[c]), __uint_as_float(dr[c + 1])), nd2);
            const float2 ds = __fmul2_rn(pr, dp);
            pk[c / 2] = pack_bf16x2(pr.x, pr.y);
            dk[c / 2] = pack_bf16x2(ds.x, ds.y);
          }
          // column chunk ch of P^T / dS^T (BF16 pairs) lands in columns [16 ch, 16 ch + 16),
          // S / dP columns this thread has already read; the MMAs of the chunk may start
          if (KV) tmem_st16(tmem + lane_off + ch * 16, pk);
          tmem_st16(tmem + lane_off + 128 + ch * 16, dk);
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(L::kPFull + ch));
        }
      }
      if (!ok) break;
      // ------------------------------ epilogue ------------------------------
      if (hi <= lo) {
        // nothing attends this tile (KV mode: keys no query row sees): zero gradients
        if (KV && mine < p.sk) {
          const int64_t off = ((static_cast<int64_t>(b) * p.sk + mine) * p.kv_heads + h) * kHeadDim;
          uint4* d0 = reinterpret_cast<uint4*>(p.g0 + off);
          uint4* d1 = reinterpret_cast<uint4*>(p.g1 + off);
#pragma unroll
          for (int v = 0; v < 16; ++v) {
            d0[v] = make_uint4(0u, 0u, 0u, 0u);
            d1[v] = make_uint4(0u, 0u, 0u, 0u);
          }
        }
        continue;
      }
      if (!warp_wait(bar(L::kAccFull), acc_full_par, ctl, kStatusTimeoutSoftmax)) { ok = false; break; }
      acc_full_par ^= 1u;
      tc_fence_after();
      const int limit = KV ? p.sk : p.sq;
      const int64_t off = ((static_cast<int64_t>(b) * limit + mine) * (KV ? p.kv_heads : p.heads) + h) * kHeadDim;
#pragma unroll 1
      for (int g = 0; g < (KV ? 2 : 1); ++g) {
        // KV: g = 0 dK (column 384, times scale), g = 1 dV (column 256); Q: dQ (column 256, times scale)
        const uint32_t col = KV ? (g == 0 ? 384u : 256u) : 256u;
        const float mul = (KV && g == 1) ? 1.f : p.scale;
        __nv_bfloat16* dst_row = (g == 0 ? p.g0 : p.g1) + off;
#pragma unroll 1
        for (int ch = 0; ch < 4; ++ch) {
          uint32_t acc[32];
          tmem_ld32(tmem + lane_off + col + ch * 32, acc);
          tmem_ld_wait();
          if (mine < limit) {
            uint4* dst = reinterpret_cast<uint4*>(dst_row + ch * 32);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 w;
              w.x = pack_bf16x2(__uint_as_float(acc[8 * v + 0]) * mul, __uint_as_float(acc[8 * v + 1]) * mul);
              w.y = pack_bf16x2(__uint_as_float(acc[8 * v + 2]) * mul, __uint_as_float(acc[8 * v + 3]) * mul);
              w.z = pack_bf16x2(__uint_as_float(acc[8 * v + 4]) * mul, __uint_as_float(acc[8 * v + 5]) * mul);
              w.w = pack_bf16x2(__uint_as_float(acc[8 * v + 6]) * mul, __uint_as_float(acc[8 * v + 7]) * mul);
              dst[v] = w;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(L::kAccEmpty));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// D of one row (128 BF16 of O and of dO) over half a warp: lane `sub` (0-15) of the half takes
// elements 8 sub .. 8 sub + 7 (nothing when `live` is false); every lane of the half ends with the
// sum. All 32 lanes must call it together. Both preprocess kernels use it, so D is bit-identical
// between the padded-batch and the packed-sequence layouts.
__device__ __forceinline__ float row_dot_half(const __nv_bfloat16* o_row, const __nv_bfloat16* g_row, int sub,
                                              bool live) {
  float s = 0.f;
  if (live) {
    const uint4 a = reinterpret_cast<const uint4*>(o_row)[sub];
    const uint4 g = reinterpret_cast<const uint4*>(g_row)[sub];
    const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&g);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 x = __bfloat1622float2(a2[e]), y = __bfloat1622float2(g2[e]);
      s = fmaf(x.x, y.x, fmaf(x.y, y.y, s));
    }
  }
#pragma unroll
  for (int d = 8; d > 0; d >>= 1) s += __shfl_xor_sync(0xffffffffu, s, d);  // within each half
  return s;
}

// D = rowsum(dO * O) in FP32 and LSE * log2(e), stored [B, H, stat_stride]; entries of rows
// sq .. stat_stride-1 are set to 0. Rows are (batch, query row, head) in memory order, 256 bytes
// each; a warp takes two adjacent rows per iteration, 16 bytes of O and dO per lane (half a warp
// per row), so one load instruction covers 512 contiguous bytes.
__global__ void __launch_bounds__(256) attn_bwd_dsum_kernel(const __nv_bfloat16* __restrict__ o,
                                                            const __nv_bfloat16* __restrict__ dout,
                                                            const float* __restrict__ lse, float* __restrict__ dsum,
                                                            float* __restrict__ lse2, int batch, int sq, int heads,
                                                            int stat_stride) {
  const int pad = stat_stride - sq;
  const int64_t pads = static_cast<int64_t>(batch) * heads * pad;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < pads;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t at = (t / pad) * stat_stride + sq + t % pad;
    dsum[at] = 0.f;
    lse2[at] = 0.f;
  }
  const int64_t rows = static_cast<int64_t>(batch) * sq * heads;
  const int lane = threadIdx.x % 32;
  const int half = lane / 16, sub = lane % 16;
  for (int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32; 2 * w < rows;
       w += static_cast<int64_t>(gridDim.x) * blockDim.x / 32) {
    const int64_t row = 2 * w + half;  // (b * sq + r) * heads + h
    const bool live = row < rows;
    const float s = row_dot_half(o + (live ? row : 0) * kHeadDim, dout + (live ? row : 0) * kHeadDim, sub, live);
    if (sub == 0 && live) {
      const int h = static_cast<int>(row % heads);
      const int64_t br = row / heads;
      const int r = static_cast<int>(br % sq);
      const int64_t bb = br / sq;
      const int64_t at = (bb * heads + h) * stat_stride + r;  // padded statistics row
      dsum[at] = s;
      lse2[at] = lse[(bb * heads + h) * sq + r] * 1.4426950408889634f;  // the forward's LSE is [B, H, Sq]
    }
  }
}

}  // namespace fav4
