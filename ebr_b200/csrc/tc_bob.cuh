// tc_bob.cuh: the tensor-core double backward for N > 128 at D = 64, with the score products of one step overlapping
// the pointwise work of the previous one.
//
// Three passes, as in the reference's _bob_row_kernel / _bob_col_kernel (triton_kernels.py:347-551) restated with the
// closed form of reference.py:80-90: a row pass for the per-row statistics D, E, T; a row pass for hQ and hdO; a
// column pass for hK and hV. Per 64-key (or 64-query) step the MMA warp forms four score tiles of M = 128, N = 64 --
// S = Q K^T, dP = dO V^T, G = gQ K^T + Q gK^T, R = dO gV^T (their transposes in the column pass) -- and the output
// passes accumulate from 16-bit tiles the compute warps derive from them.
//
// Roles (320 threads, one persistent CTA per SM):
//   warps 0-7  compute: warp w owns TMEM lanes [32 (w % 4), 32 (w % 4) + 32) -- one query (key) row per thread -- and
//              warpgroup w / 4 the columns [32 (w / 4), 32 (w / 4) + 32) of every step, so both warpgroups work on
//              the same step and a row's sums are split in two halves, added at the end of the item;
//   warp 8     TMA producer: the item's 128-row tiles (two buffers), the streamed 64-row tiles (a three-stage ring)
//              and, in the column pass, each step's lse / D / E / T;
//   warp 9     MMA issuer (one thread).
// Score products that share an operand run as one N = 128 product over two adjacent ring tiles: Q [K; gK]^T gives S
// and Q gK^T side by side, gQ K^T accumulates onto the second half (G), dO [V; gV]^T gives dP and R (the column pass:
// K [Q; gQ]^T, then gK Q^T onto G^T; V dO^T and gV dO^T). This reads each 128-row operand from shared memory once
// instead of twice, which is what limits the N = 64 products.
// Tensor memory (512 columns):
//   statistics pass: two score buffers of 256 columns (S, G, dP, R at +0, +64, +128, +192); step g uses buffer g % 2,
//     so the products of step g + 1 run while the compute warps read step g;
//   output passes: one score buffer [0, 256), the 16-bit tiles [256, 384) (four of 32 columns: 64 keys as pairs), the
//     two accumulators in [384, 448) and [448, 512). A step's scores are released as soon as the compute warps have
//     loaded them, so the tensor pipe runs the next step's score products, then this step's accumulating products
//     (issued once the 16-bit tiles are written), while the compute warps work.
#pragma once

#include "tc_attn.cuh"

namespace ebr {

// kPass: 0 statistics, 1 row outputs, 2 column outputs.
template <int kPass>
struct BobSplitLayout {
  static constexpr bool kCol = kPass == 2;
  static constexpr uint32_t kBig = kHalfBytes;   // [128 x 64] 16-bit tile
  static constexpr uint32_t kSmall = 64u * 128u;  // [64 x 64] 16-bit tile
  static constexpr int kItemBufs = 2;
  static constexpr int kStages = kCol ? 3 : 4;
  static constexpr int kItemTiles = kCol ? 4 : 3;  // row passes: Q, dO, gQ; column pass: K, V, gK, gV
  static constexpr int kRingTiles = kCol ? 3 : 4;  // row passes: K, gK, V, gV; column pass: Q, gQ, dO
  static constexpr uint32_t kItemBytes = kItemTiles * kBig;
  static constexpr uint32_t kStageBytes = kRingTiles * kSmall;
  static constexpr uint32_t kRing = kItemBufs * kItemBytes;
  // Column pass: each stage's per-query (lse, D, E, T), [stage][64 queries][4] floats. (The statistics pass exchanges
  // its partial row sums through the item's spent gQ tile.)
  static constexpr uint32_t kAux = kRing + kStages * kStageBytes;
  static constexpr uint32_t kAuxBytes = kCol ? kStages * 64 * 4 * 4 : 0;
  static constexpr uint32_t kBytes = kAux + kAuxBytes;
  static constexpr uint32_t kSmem = kBytes + 1024;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr int kThreads = 320;
};

// The score products of one step into S, G, dP, R = t0 + 0, 64, 128, 192 (M = 128, K = 64, all K-major), from SW128
// descriptors of the tiles' first K columns (K step kk adds 32 bytes, 2 in the descriptor's address field).
// Row passes: a = Q, dO, gQ (128-row item tiles); bk / bv = the ring tiles K and V, each followed by gK / gV.
__device__ __forceinline__ void bob_scores_rows(uint32_t t0, uint64_t aq, uint64_t ado, uint64_t agq, uint64_t bk,
                                                uint64_t bv, bool has_gq, bool has_gk, bool has_gv, bool bf16) {
  const uint32_t id64 = idesc_f16(bf16, 0, 0, 128, 64), id128 = idesc_f16(bf16, 0, 0, 128, 128);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const uint32_t acc = kk > 0 ? 1u : 0u;
    const uint64_t o = static_cast<uint64_t>(2 * kk);
    mma_ss(t0, aq + o, bk + o, has_gk ? id128 : id64, acc);           // [S | Q gK^T] = Q [K; gK]^T
    if (has_gq) mma_ss(t0 + 64, agq + o, bk + o, id64, (has_gk || kk > 0) ? 1u : 0u);  // G += gQ K^T
    mma_ss(t0 + 128, ado + o, bv + o, has_gv ? id128 : id64, acc);   // [dP | R] = dO [V; gV]^T
  }
}
// Column pass: a = K, V, gK, gV (item tiles); bq = the ring tile Q, followed by gQ; bdo = dO.
__device__ __forceinline__ void bob_scores_cols(uint32_t t0, uint64_t ak, uint64_t av, uint64_t agk, uint64_t agv,
                                                uint64_t bq, uint64_t bdo, bool has_gq, bool has_gk, bool has_gv,
                                                bool bf16) {
  const uint32_t id64 = idesc_f16(bf16, 0, 0, 128, 64), id128 = idesc_f16(bf16, 0, 0, 128, 128);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const uint32_t acc = kk > 0 ? 1u : 0u;
    const uint64_t o = static_cast<uint64_t>(2 * kk);
    mma_ss(t0, ak + o, bq + o, has_gq ? id128 : id64, acc);           // [S^T | K gQ^T] = K [Q; gQ]^T
    if (has_gk) mma_ss(t0 + 64, agk + o, bq + o, id64, (has_gq || kk > 0) ? 1u : 0u);  // G^T += gK Q^T
    mma_ss(t0 + 128, av + o, bdo + o, id64, acc);                     // dP^T = V dO^T
    if (has_gv) mma_ss(t0 + 192, agv + o, bdo + o, id64, acc);        // R^T = gV dO^T
  }
}

// ------------------------------------------------------------------------------------------------ statistics pass

// Per query row: D = <dO, O>, E = sum_j P G (G scaled), T = sum_j P (dP - D) G - E sum_j P dP + sum_j P R, written to
// `stats` ([3][B H N]). An item is 128 query rows of one slice; the keys stream in 64-key steps.
template <typename T>
__global__ void __launch_bounds__(320, 1)
    tc_bob_stats_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tdo,
                        const __grid_constant__ CUtensorMap tgq, const __grid_constant__ CUtensorMap tk64,
                        const __grid_constant__ CUtensorMap tv64, const __grid_constant__ CUtensorMap tgk64,
                        const __grid_constant__ CUtensorMap tgv64, const T* __restrict__ o,
                        const float* __restrict__ lse, float* __restrict__ stats, int BH, int H, int N, float scale,
                        uint32_t flags) {
  using L = BobSplitLayout<0>;
  constexpr int NS = L::kStages, NI = L::kItemBufs;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = align1024(smem_raw);
  __shared__ uint64_t it_full[NI], it_empty[NI], rg_full[NS], rg_empty[NS], s_full[2], s_free[2], part_full[NI];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_qt = (N + kTile - 1) / kTile, n_ks = (N + 63) / 64;
  const int64_t items = static_cast<int64_t>(BH) * n_qt;
  const int64_t rows_total = static_cast<int64_t>(BH) * N;
  const bool has_gq = flags & 1u, has_gk = flags & 2u, has_gv = flags & 4u;
  auto item = [&](int b, int i) { return smem + b * L::kItemBytes + i * L::kBig; };                // 0 Q 1 dO 2 gQ
  auto ring = [&](int s, int i) { return smem + L::kRing + s * L::kStageBytes + i * L::kSmall; };  // 0 K 1 gK 2 V 3 gV

  if (tid == 0) {
    for (int i = 0; i < NI; ++i) {
      mbar_init(&it_full[i], 1);
      // The MMA warp's commit + every compute thread once the item's partial sums have been exchanged.
      mbar_init(&it_empty[i], 1 + 256);
      mbar_init(&part_full[i], 128);
    }
    for (int i = 0; i < NS; ++i) {
      mbar_init(&rg_full[i], 1);
      mbar_init(&rg_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 256);
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  volatile int* abort = &abort_flag;

  if (warp == 8) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      uint32_t g = 0;
      bool ok = true;
      const uint32_t item_bytes = (2u + (has_gq ? 1u : 0u)) * L::kBig;
      const uint32_t ring_bytes = (2u + (has_gk ? 1u : 0u) + (has_gv ? 1u : 0u)) * L::kSmall;
      int64_t li = 0;
      for (int64_t it = blockIdx.x; it < items && ok; it += gridDim.x, ++li) {
        const int bh = static_cast<int>(it / n_qt), qt = static_cast<int>(it - static_cast<int64_t>(bh) * n_qt);
        const int b = bh / H, h = bh - (bh / H) * H;
        const int ib = static_cast<int>(li % NI);
        ok = mbar_wait_or_abort(&it_empty[ib], (static_cast<uint32_t>(li / NI) & 1) ^ 1, 511, abort);
        if (!ok) break;
        mbar_arrive_expect_tx(&it_full[ib], item_bytes);
        tma_load_4d(item(ib, 0), &tq, &it_full[ib], 0, qt * kTile, h, b);
        tma_load_4d(item(ib, 1), &tdo, &it_full[ib], 0, qt * kTile, h, b);
        if (has_gq) tma_load_4d(item(ib, 2), &tgq, &it_full[ib], 0, qt * kTile, h, b);
        for (int j = 0; j < n_ks && ok; ++j, ++g) {
          const int s = static_cast<int>(g % NS);
          ok = mbar_wait_or_abort(&rg_empty[s], ((g / NS) & 1) ^ 1, 512, abort);
          if (!ok) break;
          mbar_arrive_expect_tx(&rg_full[s], ring_bytes);
          tma_load_4d(ring(s, 0), &tk64, &rg_full[s], 0, j * 64, h, b);
          if (has_gk) tma_load_4d(ring(s, 1), &tgk64, &rg_full[s], 0, j * 64, h, b);
          tma_load_4d(ring(s, 2), &tv64, &rg_full[s], 0, j * 64, h, b);
          if (has_gv) tma_load_4d(ring(s, 3), &tgv64, &rg_full[s], 0, j * 64, h, b);
        }
      }
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      // K-major descriptor of a tile at byte offset `off` of the aligned shared block.
      const uint64_t d0 = sw128_desc(smem_u32(smem), 16u, 1024u);
      auto da = [&](int b, int i) { return d0 + ((b * L::kItemBytes + i * L::kBig) >> 4); };
      auto db = [&](int s, int i) { return d0 + ((L::kRing + s * L::kStageBytes + i * L::kSmall) >> 4); };
      uint32_t g = 0;
      bool ok = true;
      int64_t li = 0;
      for (int64_t it = blockIdx.x; it < items && ok; it += gridDim.x, ++li) {
        const int ib = static_cast<int>(li % NI);
        ok = mbar_wait_or_abort(&it_full[ib], static_cast<uint32_t>(li / NI) & 1, 521, abort);
        const uint64_t aq = da(ib, 0), ado = da(ib, 1), agq = da(ib, 2);
        for (int j = 0; j < n_ks && ok; ++j, ++g) {
          const int s = static_cast<int>(g % NS), b = static_cast<int>(g & 1);
          // Buffer b is free once the compute warps have read its previous step (the first use passes at once).
          ok = mbar_wait_or_abort(&s_free[b], ((g >> 1) & 1) ^ 1, 522, abort);
          if (ok) ok = mbar_wait_or_abort(&rg_full[s], (g / NS) & 1, 523, abort);
          if (!ok) break;
          tc_fence_after();
          bob_scores_rows(tmem + 256 * b, aq, ado, agq, db(s, 0), db(s, 2), has_gq, has_gk, has_gv, is_bf16<T>());
          mma_commit(&s_full[b]);
          mma_commit(&rg_empty[s]);
          if (j == n_ks - 1) mma_commit(&it_empty[ib]);
        }
      }
    }
  } else if (warp < 8) {
    // ---------------------------------------------------------------- compute warps
    const int w = warp >> 2, wq = warp & 3, lrow = wq * 32 + lane, col0 = 32 * w;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    uint32_t g = 0;
    bool ok = true;
    int64_t li = 0;
    for (int64_t it = blockIdx.x; it < items && ok; it += gridDim.x, ++li) {
      const int bh = static_cast<int>(it / n_qt), qt = static_cast<int>(it - static_cast<int64_t>(bh) * n_qt);
      const int ib = static_cast<int>(li % NI);
      const int row = qt * kTile + lrow;
      const bool row_ok = row < N;
      const int64_t grow = static_cast<int64_t>(bh) * N + row;
      const float Li = row_ok ? lse[grow] : 0.f;
      ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&it_full[ib], static_cast<uint32_t>(li / NI) & 1, 531, abort));
      if (!ok) break;
      const float Di = row_ok ? row_delta<T, 64>(item(ib, 1), lrow, o + grow * 64) : 0.f;
      float e_ = 0.f, c1 = 0.f, c2 = 0.f, c3 = 0.f;
      for (int j = 0; j < n_ks; ++j, ++g) {
        const int b = static_cast<int>(g & 1);
        ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&s_full[b], (g >> 1) & 1, 532, abort));
        if (!ok) break;
        tc_fence_after();
        const uint32_t t0 = tmem + lane_off + 256 * b + col0;
        uint32_t rs[32], rp[32], rg[32], rr[32];
        tmem_ld32(t0, rs);
        if (has_gq || has_gk) tmem_ld32(t0 + 64, rg);
        tmem_ld32(t0 + 128, rp);
        if (has_gv) tmem_ld32(t0 + 192, rr);
        tmem_wait_ld_regs(rs);
        tmem_wait_ld_regs(rp);
        if (has_gq || has_gk) tmem_wait_ld_regs(rg);
        if (has_gv) tmem_wait_ld_regs(rr);
        tc_fence_before();
        mbar_arrive(&s_free[b]);
        const int valid = N - j * 64 - col0;  // keys of this half that exist
#pragma unroll
        for (int u = 0; u < 32; ++u) {
          float p = exp_nat(fmaf(__uint_as_float(rs[u]), scale, -Li));
          if (u >= valid) p = 0.f;
          const float gg = (has_gq || has_gk) ? __uint_as_float(rg[u]) * scale : 0.f;
          const float dp = __uint_as_float(rp[u]);
          e_ += p * gg;
          c1 += p * (dp - Di) * gg;
          c2 += p * dp;
          if (has_gv) c3 += p * __uint_as_float(rr[u]);
        }
      }
      if (!ok) break;
      // The two halves of each row meet in the item's gQ tile, which no product reads any more (the last step's scores
      // have completed): warpgroup 1 writes its sums, warpgroup 0 adds them; both then release the item buffer.
      float* ps = reinterpret_cast<float*>(item(ib, 2));
      if (w == 1) {
        ps[lrow] = e_;
        ps[128 + lrow] = c1;
        ps[256 + lrow] = c2;
        ps[384 + lrow] = c3;
        mbar_arrive(&part_full[ib]);
      } else {
        ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&part_full[ib], static_cast<uint32_t>(li / NI) & 1, 534, abort));
        if (!ok) break;
        e_ += ps[lrow];
        c1 += ps[128 + lrow];
        c2 += ps[256 + lrow];
        c3 += ps[384 + lrow];
        if (row_ok) {
          stats[grow] = Di;
          stats[rows_total + grow] = e_;
          stats[2 * rows_total + grow] = c1 - e_ * c2 + c3;
        }
      }
      // The generic-proxy accesses above come before the next TMA write into this buffer.
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&it_empty[ib]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, L::kTmemCols);
}

// ------------------------------------------------------------------------------------------------ output passes

// Row pass: hQ = scale (gS K + dS gK) and hdO = A V + P gV, with dS = P (dP - D), A = P (G - E), gS = P (gp - T),
// gp = (dP - D) G - E dP + R from the statistics pass. Column pass (kCol): hK = scale (gS^T Q + dS^T gQ) and
// hV = A^T dO over the transposed tiles, with each query's lse / D / E / T staged per step. An item is 128 query
// (key) rows of one slice; the other side streams in 64-row steps.
template <typename T, bool kCol>
__global__ void __launch_bounds__(320, 1)
    tc_bob_out_kernel(const __grid_constant__ CUtensorMap ta0, const __grid_constant__ CUtensorMap ta1,
                      const __grid_constant__ CUtensorMap ta2, const __grid_constant__ CUtensorMap ta3,
                      const __grid_constant__ CUtensorMap tb0, const __grid_constant__ CUtensorMap tb1,
                      const __grid_constant__ CUtensorMap tb2, const __grid_constant__ CUtensorMap tb3,
                      const float* __restrict__ lse, const float* __restrict__ stats, T* __restrict__ out0,
                      T* __restrict__ out1, int BH, int H, int N, float scale, uint32_t flags) {
  using L = BobSplitLayout<kCol ? 2 : 1>;
  constexpr int NS = L::kStages, NI = L::kItemBufs;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = align1024(smem_raw);
  __shared__ uint64_t it_full[NI], it_empty[NI], rg_full[NS], rg_empty[NS], s_full, s_free, p_full, pk_free, o_done,
      acc_free;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_it = (N + kTile - 1) / kTile, n_st = (N + 63) / 64;
  const int64_t items = static_cast<int64_t>(BH) * n_it;
  const int64_t rows_total = static_cast<int64_t>(BH) * N;
  const bool has_gq = flags & 1u, has_gk = flags & 2u, has_gv = flags & 4u;
  // Which optional tiles exist: row pass items (Q, dO, gQ) and ring (K, gK, V, gV); column pass items (K, V, gK, gV)
  // and ring (Q, gQ, dO).
  const bool item_has[4] = {true, true, kCol ? has_gk : has_gq, kCol ? has_gv : false};
  const bool ring_has[4] = {true, kCol ? has_gq : has_gk, true, kCol ? false : has_gv};
  auto item = [&](int b, int i) { return smem + b * L::kItemBytes + i * L::kBig; };
  auto ring = [&](int s, int i) { return smem + L::kRing + s * L::kStageBytes + i * L::kSmall; };
  float* stg = reinterpret_cast<float*>(smem + L::kAux);  // column pass: [stage][64][lse, D, E, T]

  if (tid == 0) {
    for (int i = 0; i < NI; ++i) {
      mbar_init(&it_full[i], 1);
      mbar_init(&it_empty[i], 1);
    }
    for (int i = 0; i < NS; ++i) {
      mbar_init(&rg_full[i], kCol ? 33 : 1);  // column pass: + one arrive per producer lane after its stats writes
      mbar_init(&rg_empty[i], 1);
    }
    mbar_init(&s_full, 1);
    mbar_init(&s_free, 256);
    mbar_init(&p_full, 256);
    mbar_init(&pk_free, 1);
    mbar_init(&o_done, 1);
    mbar_init(&acc_free, 256);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  volatile int* abort = &abort_flag;

  if (warp == 8) {
    // ---------------------------------------------------------------- producer (lane 0: TMA; column pass: all lanes
    // also stage the step's per-query statistics)
    uint32_t g = 0;
    bool ok = true;
    uint32_t item_bytes = 0, ring_bytes = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (i < L::kItemTiles && item_has[i]) item_bytes += L::kBig;
      if (i < L::kRingTiles && ring_has[i]) ring_bytes += L::kSmall;
    }
    const CUtensorMap* amap[4] = {&ta0, &ta1, &ta2, &ta3};
    const CUtensorMap* bmap[4] = {&tb0, &tb1, &tb2, &tb3};
    // Column pass: this lane's (lse, D, E, T) of queries lane and lane + 32 of a step, loaded while the previous
    // step is staged. Queries past N get zeros: with their zero Q / dO / gQ rows every derived value is 0.
    auto load_stats = [&](int64_t base_, int j_, float4 (&v)[2]) {
#pragma unroll
      for (int k2 = 0; k2 < 2; ++k2) {
        const int qi = j_ * 64 + lane + 32 * k2;
        v[k2] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (qi < N) {
          v[k2].x = __ldg(lse + base_ + qi);
          v[k2].y = __ldg(stats + base_ + qi);
          v[k2].z = __ldg(stats + rows_total + base_ + qi);
          v[k2].w = __ldg(stats + 2 * rows_total + base_ + qi);
        }
      }
    };
    int64_t li = 0;
    for (int64_t it = blockIdx.x; it < items && ok; it += gridDim.x, ++li) {
      const int bh = static_cast<int>(it / n_it), t = static_cast<int>(it - static_cast<int64_t>(bh) * n_it);
      const int b = bh / H, h = bh - (bh / H) * H;
      const int64_t base = static_cast<int64_t>(bh) * N;
      const int ib = static_cast<int>(li % NI);
      float4 cur[2];
      if (kCol) load_stats(base, 0, cur);
      if (lane == 0) {
        ok = mbar_wait_or_abort(&it_empty[ib], (static_cast<uint32_t>(li / NI) & 1) ^ 1, 541, abort);
        if (ok) {
          mbar_arrive_expect_tx(&it_full[ib], item_bytes);
#pragma unroll
          for (int i = 0; i < L::kItemTiles; ++i)
            if (item_has[i]) tma_load_4d(item(ib, i), amap[i], &it_full[ib], 0, t * kTile, h, b);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      for (int j = 0; j < n_st && ok; ++j, ++g) {
        const int s = static_cast<int>(g % NS);
        float4 nxt[2];
        if (kCol && j + 1 < n_st) load_stats(base, j + 1, nxt);
        ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&rg_empty[s], ((g / NS) & 1) ^ 1, 542, abort));
        if (!ok) break;
        if (lane == 0) {
          mbar_arrive_expect_tx(&rg_full[s], ring_bytes);
#pragma unroll
          for (int i = 0; i < L::kRingTiles; ++i)
            if (ring_has[i]) tma_load_4d(ring(s, i), bmap[i], &rg_full[s], 0, j * 64, h, b);
        }
        if (kCol) {
          float4* st = reinterpret_cast<float4*>(stg) + s * 64;
#pragma unroll
          for (int k2 = 0; k2 < 2; ++k2) {
            st[lane + 32 * k2] = cur[k2];
            cur[k2] = nxt[k2];
          }
          mbar_arrive(&rg_full[s]);
        }
      }
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdKM = idesc_f16(is_bf16<T>(), 0, 1, 128, 64);
      const uint32_t tPk = tmem + 256, tAcc0 = tmem + 384, tAcc1 = tmem + 448;
      // Descriptors of a tile at byte offset `off` of the aligned shared block: K-major (score products) and MN-major
      // (accumulating products, B = the ring tile read with its 64 columns as N; K step kk = 16 rows = 2048 bytes).
      const uint64_t d0 = sw128_desc(smem_u32(smem), 16u, 1024u);
      const uint64_t m0 = sw128_desc(smem_u32(smem), L::kSmall, 1024u);
      auto da = [&](int b, int i) { return d0 + ((b * L::kItemBytes + i * L::kBig) >> 4); };
      auto rof = [&](int s, int i) { return static_cast<uint64_t>((L::kRing + s * L::kStageBytes + i * L::kSmall) >> 4); };
      uint32_t g = 0;
      bool ok = true;
      // The accumulating products of step g are issued after the score products of step g + 1: the step waiting for
      // them (its index, ring stage, position in its item, item) is held here.
      bool pend = false;
      uint32_t pg = 0;
      int ps = 0, pj = 0;
      bool plast = false;
      int64_t pli = 0;
      auto accumulate = [&]() -> bool {
        if (!mbar_wait_or_abort(&p_full, pg & 1, 553, abort)) return false;
        // The first step of an item overwrites the accumulators: the previous item's must have been stored.
        if (pj == 0 && pli > 0 && !mbar_wait_or_abort(&acc_free, static_cast<uint32_t>(pli - 1) & 1, 554, abort))
          return false;
        tc_fence_after();
        const uint64_t b0 = m0 + rof(ps, 0), b1 = m0 + rof(ps, 1), b2 = m0 + rof(ps, 2), b3 = m0 + rof(ps, 3);
        const uint32_t first = pj > 0 ? 1u : 0u;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t acc0 = kk > 0 ? 1u : first;
          const uint32_t a = tPk + kk * 8;
          const uint64_t o = static_cast<uint64_t>(128 * kk);
          // Row pass: hQ += gS K (+ dS gK), hdO += A V (+ P gV). Column pass: hK += gS^T Q (+ dS^T gQ), hV += A^T dO.
          mma_ts(tAcc0, a, b0 + o, kIdKM, acc0);
          if (kCol ? has_gq : has_gk) mma_ts(tAcc0, a + 32, b1 + o, kIdKM, 1u);
          mma_ts(tAcc1, a + 64, b2 + o, kIdKM, acc0);
          if (!kCol && has_gv) mma_ts(tAcc1, a + 96, b3 + o, kIdKM, 1u);
        }
        mma_commit(&pk_free);
        mma_commit(&rg_empty[ps]);
        if (plast) mma_commit(&o_done);
        return true;
      };
      int64_t li = 0;
      for (int64_t it = blockIdx.x; it < items && ok; it += gridDim.x, ++li) {
        const int ib = static_cast<int>(li % NI);
        ok = mbar_wait_or_abort(&it_full[ib], static_cast<uint32_t>(li / NI) & 1, 551, abort);
        for (int j = 0; j < n_st && ok; ++j, ++g) {
          const int s = static_cast<int>(g % NS);
          ok = mbar_wait_or_abort(&rg_full[s], (g / NS) & 1, 552, abort);
          // The score buffer is free once the compute warps have loaded the previous step.
          if (ok) ok = mbar_wait_or_abort(&s_free, (g & 1) ^ 1, 555, abort);
          if (!ok) break;
          tc_fence_after();
          const uint64_t a0 = da(ib, 0), a1 = da(ib, 1), a2 = da(ib, 2), a3 = da(ib, 3);
          const uint64_t r0 = d0 + rof(s, 0), r2 = d0 + rof(s, 2);
          if (!kCol)
            bob_scores_rows(tmem, a0, a1, a2, r0, r2, has_gq, has_gk, has_gv, is_bf16<T>());
          else
            bob_scores_cols(tmem, a0, a1, a2, a3, r0, r2, has_gq, has_gk, has_gv, is_bf16<T>());
          mma_commit(&s_full);
          if (j == n_st - 1) mma_commit(&it_empty[ib]);
          if (pend) ok = accumulate();
          pend = true;
          pg = g;
          ps = s;
          pj = j;
          plast = j == n_st - 1;
          pli = li;
        }
      }
      if (ok && pend) accumulate();
    }
  } else if (warp < 8) {
    // ---------------------------------------------------------------- compute warps
    const int w = warp >> 2, wq = warp & 3, lrow = wq * 32 + lane, col0 = 32 * w;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t t0 = tmem + lane_off + col0;              // this thread's 32 score columns
    const uint32_t tp = tmem + lane_off + 256 + (col0 >> 1);  // its 16 columns of each 16-bit tile
    uint32_t g = 0;
    bool ok = true;
    int64_t li = 0;
    for (int64_t it = blockIdx.x; it < items && ok; it += gridDim.x, ++li) {
      const int bh = static_cast<int>(it / n_it), t = static_cast<int>(it - static_cast<int64_t>(bh) * n_it);
      const int row = t * kTile + lrow;
      const bool row_ok = row < N;
      const int64_t grow = static_cast<int64_t>(bh) * N + row;
      // Row pass: this row's statistics (rows past N: 0, and their zero Q / dO / gQ make every product 0 but P V).
      float Li = 0.f, Di = 0.f, Ei = 0.f, Ti = 0.f;
      if (!kCol && row_ok) {
        Li = lse[grow];
        Di = stats[grow];
        Ei = stats[rows_total + grow];
        Ti = stats[2 * rows_total + grow];
      }
      for (int j = 0; j < n_st; ++j, ++g) {
        ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&s_full, g & 1, 561, abort));
        if (!ok) break;
        tc_fence_after();
        uint32_t rs[32], rp[32], rg[32], rr[32];
        const bool load_g = has_gq || has_gk, load_r = has_gv;
        tmem_ld32(t0, rs);
        if (load_g) tmem_ld32(t0 + 64, rg);
        tmem_ld32(t0 + 128, rp);
        if (load_r) tmem_ld32(t0 + 192, rr);
        tmem_wait_ld_regs(rs);
        tmem_wait_ld_regs(rp);
        if (load_g) tmem_wait_ld_regs(rg);
        if (load_r) tmem_wait_ld_regs(rr);
        tc_fence_before();
        mbar_arrive(&s_free);
        // The previous step's accumulating products must have read the 16-bit tiles before they are rewritten.
        ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&pk_free, (g & 1) ^ 1, 562, abort));
        if (!ok) break;
        tc_fence_after();
        const int valid = kCol ? 64 : N - j * 64 - col0;  // row pass: keys of this half that exist
        const float4* st = reinterpret_cast<const float4*>(stg) + (g % NS) * 64 + col0;
#pragma unroll
        for (int c = 0; c < 32; c += 16) {
          uint32_t pgs[8], pds[8], pa[8], pp[8];
#pragma unroll
          for (int u = 0; u < 16; u += 2) {
            float v_gs[2], v_ds[2], v_a[2], v_p[2];
#pragma unroll
            for (int x = 0; x < 2; ++x) {
              const int e = c + u + x;
              float Lr = Li, Dr = Di, Er = Ei, Tr = Ti;
              if (kCol) {
                const float4 q4 = st[e];
                Lr = q4.x;
                Dr = q4.y;
                Er = q4.z;
                Tr = q4.w;
              }
              float p = exp_nat(fmaf(__uint_as_float(rs[e]), scale, -Lr));
              if (!kCol && e >= valid) p = 0.f;
              const float gg = load_g ? __uint_as_float(rg[e]) * scale : 0.f;
              const float dp = __uint_as_float(rp[e]);
              const float r = load_r ? __uint_as_float(rr[e]) : 0.f;
              const float gp = (dp - Dr) * gg - Er * dp + r;
              v_p[x] = p;
              v_ds[x] = p * (dp - Dr);
              v_a[x] = p * (gg - Er);
              v_gs[x] = p * (gp - Tr);
            }
            pgs[u >> 1] = pack2<T>(v_gs[0], v_gs[1]);
            pds[u >> 1] = pack2<T>(v_ds[0], v_ds[1]);
            pa[u >> 1] = pack2<T>(v_a[0], v_a[1]);
            pp[u >> 1] = pack2<T>(v_p[0], v_p[1]);
          }
          tmem_st8(tp + (c >> 1), pgs);
          tmem_st8(tp + 32 + (c >> 1), pds);
          tmem_st8(tp + 64 + (c >> 1), pa);
          if (!kCol) tmem_st8(tp + 96 + (c >> 1), pp);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full);
      }
      if (!ok) break;
      ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&o_done, static_cast<uint32_t>(li) & 1, 563, abort));
      if (!ok) break;
      tc_fence_after();
      // Warpgroup 0 stores the first output (hQ / hK, times scale), warpgroup 1 the second (hdO / hV).
      T* dst = row_ok ? (w == 0 ? out0 : out1) + grow * 64 : nullptr;
      store_cols_from_tmem<T, 64>(tmem + lane_off + (w == 0 ? 384 : 448), 0, w == 0 ? scale : 1.f, dst);
      tc_fence_before();
      mbar_arrive(&acc_free);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, L::kTmemCols);
}

}  // namespace ebr
