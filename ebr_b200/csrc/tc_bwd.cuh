// tc_bwd.cuh: the tensor-core backward for N > 128 with multi-buffered score tiles (row pass for dQ, column pass for
// dK / dV), each with separate MMA issuers for the score products and for the accumulating products.
#pragma once

#include "tc_attn.cuh"

namespace ebr {

// Row pass: one persistent CTA per SM; an item is 128 query rows of one (b, h) slice (Q and dO staged per item), and
// the keys stream in 64-key steps. Tensor memory (512 columns): score buffer b in {0, 1, 2} holds S = Q K^T in
// [128 b, 128 b + 64) and dP = dO V^T in [128 b + 64, 128 b + 128); dQ accumulates in [384, 384 + D). Steps are
// numbered across items; step g uses buffer g % 3 and compute warpgroup g % 2, so the scores of the group's next step
// are computed (their buffer freed by an earlier step) while it works on the current one. Roles:
//   warps 0-3 / 4-7  compute warpgroup 0 / 1, taking the even / odd steps: thread t owns query row t
//                    (TMEM lane t) and all 64 keys of its step; it forms dS = P (dP - D_i) with
//                    P = exp(fma(s, scale, -lse_i)) and writes dS as 16-bit pairs over its S columns (keys
//                    [16 m, 16 m + 16) in columns [8 m, 8 m + 8));
//   warp 8           TMA producer: Q and dO per item, 64-key K / V tiles into a 4-stage ring;
//   warp 9           S / dP issuer: S(g), dP(g) into buffer g % 3 once dQ += dS(g - 3) K has completed;
//   warp 10          dQ issuer: dQ += dS(j) K_j (dS from TMEM, K read MN-major) once step j's dS is written.
// Each compute warpgroup also computes D_i = <dO_i, O_i> of its rows from the stored O at the start of an item (group
// 0 writes it to `di_out` for the column pass), and at the end stores half of dQ's columns. While one group works on a
// step, the tensor pipe runs the other buffer's products. The reference's _bwd_dq_kernel + _rowdot_kernel
// (triton_kernels.py:277-339, :171-181).
template <int D>
struct BwdRowLayout {
  static constexpr uint32_t kBig = (D / 64) * kHalfBytes;  // [128 x D] tile (Q, dO)
  static constexpr uint32_t kHalf64 = 64u * 128u;          // [64 x 64] 16-bit half
  static constexpr uint32_t kSmall = (D / 64) * kHalf64;   // [64 x D] tile (K, V)
  static constexpr int kQBufs = D == 64 ? 2 : 1;
  static constexpr int kStages = 4;
  static constexpr uint32_t kQ = 0;                     // buffer b: Q at kQ + 3 b kBig, dO at + kBig, O at + 2 kBig
  static constexpr uint32_t kRing = 3 * kQBufs * kBig;  // stage s: K at kRing + 2 s kSmall, V at + kSmall
  static constexpr uint32_t kBytes = kRing + kStages * 2 * kSmall;
  static constexpr uint32_t kSmem = kBytes + 1024;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr int kThreads = 352;
  static constexpr int kSBufs = 3;  // score buffers of 128 columns; dQ after them
  // dQ accumulators: two at D = 64 (3 x 128 + 2 x 64 = 512 columns), so an item's first dQ products need not wait
  // until the previous item's dQ has been read out; one at D = 128.
  static constexpr int kDqBufs = D == 64 ? 2 : 1;
};

template <typename T, int D>
__global__ void __launch_bounds__(352, 1)
    tc_bwd_dq_split_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk64,
                           const __grid_constant__ CUtensorMap tv64, const __grid_constant__ CUtensorMap tdo,
                           const __grid_constant__ CUtensorMap to, const float* __restrict__ lse,
                           float* __restrict__ di_out,
                           T* __restrict__ dq, int BH, int H, int N, float scale) {
  using L = BwdRowLayout<D>;
  constexpr int NS = L::kStages, QB = L::kQBufs, NB = L::kSBufs;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = align1024(smem_raw);
  constexpr int DB = L::kDqBufs;
  __shared__ uint64_t q_full[QB], q_empty[QB], kv_full[NS], kv_empty[NS], s_full[NB], p_full[NB], ds_free[NB],
      dq_done[DB], dq_free[DB];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_qt = (N + kTile - 1) / kTile, n_ks = (N + 63) / 64;
  const int64_t items = static_cast<int64_t>(BH) * n_qt;
  constexpr bool kB = is_bf16<T>();
  auto sQ = [&](int b) { return smem + L::kQ + b * 3 * L::kBig; };
  auto sDO = [&](int b) { return smem + L::kQ + b * 3 * L::kBig + L::kBig; };
  auto sO = [&](int b) { return smem + L::kQ + b * 3 * L::kBig + 2 * L::kBig; };
  auto sK = [&](int s) { return smem + L::kRing + s * 2 * L::kSmall; };
  auto sV = [&](int s) { return smem + L::kRing + s * 2 * L::kSmall + L::kSmall; };

  if (tid == 0) {
    for (int i = 0; i < QB; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < NS; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 2);  // the S / dP issuer's and the dQ issuer's commits
    }
    for (int b = 0; b < NB; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 128);
      mbar_init(&ds_free[b], 1);
    }
    for (int i = 0; i < DB; ++i) {
      mbar_init(&dq_done[i], 1);
      mbar_init(&dq_free[i], 256);
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
  const uint32_t tDQ = tmem + NB * 128;
  volatile int* abort = &abort_flag;

  if (warp == 8) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk64);
      tma_prefetch_desc(&tv64);
      tma_prefetch_desc(&tdo);
      tma_prefetch_desc(&to);
      uint32_t kv_use = 0, quse = 0;
      bool ok = true;
      for (int64_t it = blockIdx.x; it < items && ok; it += gridDim.x, ++quse) {
        const int bh = static_cast<int>(it / n_qt), qt = static_cast<int>(it - static_cast<int64_t>(bh) * n_qt);
        const int b = bh / H, h = bh - (bh / H) * H;
        const int qb = static_cast<int>(quse % QB);
        ok = mbar_wait_or_abort(&q_empty[qb], ((quse / QB) & 1) ^ 1, 311, abort);
        if (!ok) break;
        mbar_arrive_expect_tx(&q_full[qb], 3 * L::kBig);
        for (int hh = 0; hh < D / 64; ++hh) {
          tma_load_4d(sQ(qb) + hh * kHalfBytes, &tq, &q_full[qb], hh * 64, qt * kTile, h, b);
          tma_load_4d(sDO(qb) + hh * kHalfBytes, &tdo, &q_full[qb], hh * 64, qt * kTile, h, b);
          tma_load_4d(sO(qb) + hh * kHalfBytes, &to, &q_full[qb], hh * 64, qt * kTile, h, b);
        }
        for (int j = 0; j < n_ks && ok; ++j, ++kv_use) {
          const int s = static_cast<int>(kv_use % NS);
          ok = mbar_wait_or_abort(&kv_empty[s], ((kv_use / NS) & 1) ^ 1, 312, abort);
          if (!ok) break;
          mbar_arrive_expect_tx(&kv_full[s], 2 * L::kSmall);
          for (int hh = 0; hh < D / 64; ++hh) {
            tma_load_4d(sK(s) + hh * L::kHalf64, &tk64, &kv_full[s], hh * 64, j * 64, h, b);
            tma_load_4d(sV(s) + hh * L::kHalf64, &tv64, &kv_full[s], hh * 64, j * 64, h, b);
          }
        }
      }
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------------- S / dP issuer
    if (lane == 0) {
      uint32_t kv_use = 0, quse = 0;  // kv_use: global step counter (buffer kv_use % NB, its use kv_use / NB)
      bool ok = true;
      const uint64_t dQ0 = sw128_desc(smem_u32(sQ(0)), 16u, 1024u);
      const uint64_t dK0 = sw128_desc(smem_u32(sK(0)), 16u, 1024u);
      const uint32_t idNN = idesc_f16(kB, 0, 0, 128, 64);
      for (int64_t it = blockIdx.x; it < items && ok; it += gridDim.x, ++quse) {
        const int qb = static_cast<int>(quse % QB);
        ok = mbar_wait_or_abort(&q_full[qb], (quse / QB) & 1, 321, abort);
        const uint64_t aq = dQ0 + static_cast<uint64_t>(qb * ((3 * L::kBig) >> 4));
        const uint64_t ado = aq + (L::kBig >> 4);
        for (int j = 0; j < n_ks && ok; ++j, ++kv_use) {
          const int b = static_cast<int>(kv_use % NB), s = static_cast<int>(kv_use % NS);
          // Buffer b is free once the dQ product of its previous use has completed (the first use passes at once).
          ok = mbar_wait_or_abort(&ds_free[b], ((kv_use / NB) & 1) ^ 1, 322, abort);
          if (ok) ok = mbar_wait_or_abort(&kv_full[s], (kv_use / NS) & 1, 323, abort);
          if (!ok) break;
          tc_fence_after();
          const uint64_t bk = dK0 + static_cast<uint64_t>(s * ((2 * L::kSmall) >> 4));
          const uint64_t bv = bk + (L::kSmall >> 4);
          const uint32_t tS = tmem + b * 128, tDP = tS + 64;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t oa = ((kk >> 2) * kHalfBytes + (kk & 3) * 32) >> 4;
            const uint32_t ob = ((kk >> 2) * L::kHalf64 + (kk & 3) * 32) >> 4;
            mma_ss(tS, aq + oa, bk + ob, idNN, kk > 0 ? 1u : 0u);
            mma_ss(tDP, ado + oa, bv + ob, idNN, kk > 0 ? 1u : 0u);
          }
          mma_commit(&s_full[b]);
          mma_commit(&kv_empty[s]);
          if (j == n_ks - 1) mma_commit(&q_empty[qb]);
        }
      }
    }
  } else if (warp == 10) {
    // ---------------------------------------------------------------- dQ issuer
    if (lane == 0) {
      uint32_t kv_use = 0, icnt = 0;
      bool ok = true;
      const uint64_t dK0 = sw128_desc(smem_u32(sK(0)), L::kHalf64, 1024u);
      const uint32_t idKM = idesc_f16(kB, 0, 1, 128, D);
      for (int64_t it = blockIdx.x; it < items && ok; it += gridDim.x, ++icnt) {
        // The dQ buffer's previous item must have been read out before this item's first product overwrites it.
        const int db = static_cast<int>(icnt % DB);
        const uint32_t tDQb = tDQ + db * D;
        ok = mbar_wait_or_abort(&dq_free[db], ((icnt / DB) & 1) ^ 1, 331, abort);
        for (int j = 0; j < n_ks && ok; ++j, ++kv_use) {
          const int b = static_cast<int>(kv_use % NB), s = static_cast<int>(kv_use % NS);
          ok = mbar_wait_or_abort(&p_full[b], (kv_use / NB) & 1, 332, abort);
          if (!ok) break;
          tc_fence_after();
          const uint64_t bk = dK0 + static_cast<uint64_t>(s * ((2 * L::kSmall) >> 4));
          const uint32_t tA = tmem + b * 128;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_ts(tDQb, tA + kk * 8, bk + ((kk * 2048) >> 4), idKM, (j > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&ds_free[b]);
          mma_commit(&kv_empty[s]);
        }
        if (ok) mma_commit(&dq_done[db]);
      }
    }
  } else if (warp < 8) {
    // ---------------------------------------------------------------- compute warpgroups
    const int w = warp >> 2, wq = warp & 3, lrow = wq * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    uint32_t g0 = 0, icnt = 0, quse = 0;  // global step of the item's first step, items
    bool ok = true;
    // This thread's lse of the next item is loaded while the current item runs (O and dO arrive by TMA with Q).
    float l_nx = 0.f;
    auto prefetch = [&](int64_t it_) {
      if (it_ >= items) return;
      const int bh_ = static_cast<int>(it_ / n_qt);
      const int row_ = static_cast<int>(it_ - static_cast<int64_t>(bh_) * n_qt) * kTile + lrow;
      if (row_ < N) l_nx = __ldg(lse + static_cast<int64_t>(bh_) * N + row_);
    };
    prefetch(blockIdx.x);
    for (int64_t it = blockIdx.x; it < items && ok; it += gridDim.x, ++icnt, ++quse, g0 += n_ks) {
      const int bh = static_cast<int>(it / n_qt), qt = static_cast<int>(it - static_cast<int64_t>(bh) * n_qt);
      const int qb = static_cast<int>(quse % QB);
      const int row = qt * kTile + lrow;
      const bool row_ok = row < N;
      const int64_t grow = static_cast<int64_t>(bh) * N + row;
      const float Li = row_ok ? l_nx : 0.f;
      prefetch(it + gridDim.x);
      ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&q_full[qb], (quse / QB) & 1, 341, abort));
      if (!ok) break;
      float Di = 0.f;
      if (row_ok) {
        Di = row_delta_smem<T, D>(sDO(qb), sO(qb), lrow);
        if (w == 0) di_out[grow] = Di;
      }
      // This group takes the steps whose global index has its parity (so the groups alternate across items too).
      for (int j = static_cast<int>((w + 2 - (g0 & 1)) & 1); j < n_ks; j += 2) {
        const uint32_t g = g0 + j;
        const int b = static_cast<int>(g % NB);
        const uint32_t tS = tmem + lane_off + b * 128, tDP = tS + 64;
        ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&s_full[b], (g / NB) & 1, 342, abort));
        if (!ok) break;
        tc_fence_after();
        // Query rows past N have zero Q / dO (TMA fill) and Li = Di = 0, so their dS is exactly 0 without a mask;
        // keys past N (the last step only) are masked so exp(-Li) cannot reach dQ.
        const int valid = N - j * 64;
        const int nch = valid > 32 ? 2 : 1;
        // The second 32 keys' scores are requested before the first 32 are turned into dS, so that load's latency
        // hides behind the exponentials.
        uint32_t rs[2][32], rp[2][32];
        tmem_ld32(tS, rs[0]);
        tmem_ld32(tDP, rp[0]);
        tmem_wait_ld_regs(rs[0]);
        tmem_wait_ld_regs(rp[0]);
        if (nch > 1) {
          tmem_ld32(tS + 32, rs[1]);
          tmem_ld32(tDP + 32, rp[1]);
        }
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t pk[16];
          if (c < nch) {
            if (c == 1) {
              tmem_wait_ld_regs(rs[1]);
              tmem_wait_ld_regs(rp[1]);
            }
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              float ds[2];
#pragma unroll
              for (int u = 0; u < 2; ++u) {
                float p = exp_nat(fmaf(__uint_as_float(rs[c][e + u]), scale, -Li));
                if (valid < 64 && 32 * c + e + u >= valid) p = 0.f;
                ds[u] = p * (__uint_as_float(rp[c][e + u]) - Di);
              }
              pk[e >> 1] = pack2<T>(ds[0], ds[1]);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) pk[e] = 0u;  // keys past N: dS = 0
          }
          tmem_st16(tS + 16 * c, pk);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[b]);
      }
      if (!ok) break;
      const int db = static_cast<int>(icnt % DB);
      ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&dq_done[db], (icnt / DB) & 1, 343, abort));
      if (!ok) break;
      tc_fence_after();
      T* dst = row_ok ? dq + grow * D : nullptr;
      store_cols_from_tmem<T, D / 2>(tDQ + db * D + lane_off, w * (D / 2), scale, dst);
      tc_fence_before();
      mbar_arrive(&dq_free[db]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, L::kTmemCols);
}

// Column pass: an item is 128 keys of one slice (K and V staged per item), the queries stream in 64-query steps (Q,
// dO, and each step's lse and D_i staged by the producer warp). Tensor memory: score buffer b (three at D = 64, two at
// D = 128; step g uses buffer g % NB) holds S^T = K Q^T in [128 b, 128 b + 64) and dP^T = V dO^T in
// [128 b + 64, 128 b + 128); dK and dV accumulate in the D + D columns after the buffers. Roles:
//   warps 0-3 / 4-7  compute warpgroups for the even / odd steps: thread t owns key row t (TMEM lane t) and all 64
//                    queries of its step; it writes P^T = exp(fma(s, scale, -lse_q)) and dS^T = P^T (dP^T - D_q) as
//                    16-bit pairs over the S^T / dP^T columns (queries [16 m, 16 m + 16) in columns [8 m, 8 m + 8));
//   warp 8           producer: K, V per item; Q, dO 64-row tiles into a 4-stage ring; lse / D of each step in shared
//                    memory (all 32 lanes);
//   warp 9           S^T / dP^T issuer, into buffer g % NB once the dK / dV products of its previous use have
//                    completed;
//   warp 10          dK / dV issuer: dV += P^T dO, dK += dS^T Q (A from TMEM, B read MN-major).
// At the end of an item warpgroup 0 stores dK (times scale), warpgroup 1 dV. The reference's _bwd_col_kernel
// (triton_kernels.py:184-274, two-kernel mode).
template <int D>
struct BwdColLayout {
  static constexpr uint32_t kBig = (D / 64) * kHalfBytes;  // [128 x D] tile (K, V)
  static constexpr uint32_t kHalf64 = 64u * 128u;
  static constexpr uint32_t kSmall = (D / 64) * kHalf64;  // [64 x D] tile (Q, dO)
  static constexpr int kKBufs = D == 64 ? 2 : 1;
  static constexpr int kStages = 4;
  static constexpr uint32_t kK = 0;                                 // buffer b: K at kK + 2 b kBig, V at + kBig
  static constexpr uint32_t kRing = 2 * kKBufs * kBig;              // stage s: Q at kRing + 2 s kSmall, dO at + kSmall
  static constexpr uint32_t kStats = kRing + kStages * 2 * kSmall;  // [stage][lse 64 | D 64] floats
  static constexpr uint32_t kBytes = kStats + kStages * 128 * 4;
  static constexpr uint32_t kSmem = kBytes + 1024;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr int kThreads = 352;
  static constexpr int kSBufs = D == 64 ? 3 : 2;  // score buffers of 128 columns; dK, dV after them
};

template <typename T, int D>
__global__ void __launch_bounds__(352, 1)
    tc_bwd_dkdv_split_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                             const __grid_constant__ CUtensorMap tq64, const __grid_constant__ CUtensorMap tdo64,
                             const float* __restrict__ lse, const float* __restrict__ di, T* __restrict__ dk,
                             T* __restrict__ dv, int BH, int H, int N, float scale) {
  using L = BwdColLayout<D>;
  constexpr int NS = L::kStages, KB = L::kKBufs, NB = L::kSBufs;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = align1024(smem_raw);
  __shared__ uint64_t k_full[KB], k_empty[KB], q_full[NS], q_empty[NS], s_full[NB], p_full[NB], ds_free[NB], kv_done,
      kv_free;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_kt = (N + kTile - 1) / kTile, n_qs = (N + 63) / 64;
  const int64_t items = static_cast<int64_t>(BH) * n_kt;
  constexpr bool kB = is_bf16<T>();
  auto sK = [&](int b) { return smem + L::kK + b * 2 * L::kBig; };
  auto sV = [&](int b) { return smem + L::kK + b * 2 * L::kBig + L::kBig; };
  auto sQ = [&](int s) { return smem + L::kRing + s * 2 * L::kSmall; };
  auto sDO = [&](int s) { return smem + L::kRing + s * 2 * L::kSmall + L::kSmall; };
  float* stats = reinterpret_cast<float*>(smem + L::kStats);

  if (tid == 0) {
    for (int i = 0; i < KB; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < NS; ++i) {
      mbar_init(&q_full[i], 33);  // the TMA transaction arrive + one arrive per producer lane after its lse / D writes
      mbar_init(&q_empty[i], 2);  // the two issuers' commits
    }
    for (int b = 0; b < NB; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 128);
      mbar_init(&ds_free[b], 1);
    }
    mbar_init(&kv_done, 1);
    mbar_init(&kv_free, 256);
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
  const uint32_t tDK = tmem + NB * 128, tDV = tmem + NB * 128 + D;
  volatile int* abort = &abort_flag;

  if (warp == 8) {
    // ---------------------------------------------------------------- producer (lane 0: TMA; all lanes: lse / D)
    uint32_t q_use = 0, kuse = 0;
    bool ok = true;
    // This lane's lse / D of a query step (queries lane and lane + 32). Queries past N get lse = D = 0: with their
    // zero Q / dO rows this makes P^T = 1 and dS^T = 0 there, and dO = 0 keeps them out of dV, so the compute warps
    // need no mask. A step's values are loaded while the previous step is staged, so their latency stays off the ring.
    auto load_stats = [&](int64_t base_, int i_, float (&l)[2], float (&d)[2]) {
#pragma unroll
      for (int k2 = 0; k2 < 2; ++k2) {
        const int qi = i_ * 64 + lane + 32 * k2;
        l[k2] = qi < N ? __ldg(lse + base_ + qi) : 0.f;
        d[k2] = qi < N ? __ldg(di + base_ + qi) : 0.f;
      }
    };
    for (int64_t it = blockIdx.x; it < items && ok; it += gridDim.x, ++kuse) {
      const int bh = static_cast<int>(it / n_kt), kt = static_cast<int>(it - static_cast<int64_t>(bh) * n_kt);
      const int b = bh / H, h = bh - (bh / H) * H;
      const int64_t base = static_cast<int64_t>(bh) * N;
      const int kb = static_cast<int>(kuse % KB);
      float cl[2], cd[2];
      load_stats(base, 0, cl, cd);
      if (lane == 0) {
        ok = mbar_wait_or_abort(&k_empty[kb], ((kuse / KB) & 1) ^ 1, 411, abort);
        if (ok) {
          mbar_arrive_expect_tx(&k_full[kb], 2 * L::kBig);
          for (int hh = 0; hh < D / 64; ++hh) {
            tma_load_4d(sK(kb) + hh * kHalfBytes, &tk, &k_full[kb], hh * 64, kt * kTile, h, b);
            tma_load_4d(sV(kb) + hh * kHalfBytes, &tv, &k_full[kb], hh * 64, kt * kTile, h, b);
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      for (int i = 0; i < n_qs && ok; ++i, ++q_use) {
        const int s = static_cast<int>(q_use % NS);
        float nl[2] = {0.f, 0.f}, nd[2] = {0.f, 0.f};
        if (i + 1 < n_qs) load_stats(base, i + 1, nl, nd);
        ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&q_empty[s], ((q_use / NS) & 1) ^ 1, 412, abort));
        if (!ok) break;
        if (lane == 0) {
          mbar_arrive_expect_tx(&q_full[s], 2 * L::kSmall);
          for (int hh = 0; hh < D / 64; ++hh) {
            tma_load_4d(sQ(s) + hh * L::kHalf64, &tq64, &q_full[s], hh * 64, i * 64, h, b);
            tma_load_4d(sDO(s) + hh * L::kHalf64, &tdo64, &q_full[s], hh * 64, i * 64, h, b);
          }
        }
        float* st = stats + s * 128;
#pragma unroll
        for (int k2 = 0; k2 < 2; ++k2) {
          st[lane + 32 * k2] = cl[k2];
          st[64 + lane + 32 * k2] = cd[k2];
          cl[k2] = nl[k2];
          cd[k2] = nd[k2];
        }
        mbar_arrive(&q_full[s]);
      }
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------------- S^T / dP^T issuer
    if (lane == 0) {
      uint32_t q_use = 0, kuse = 0;  // q_use: global step counter (buffer q_use % NB, its use q_use / NB)
      bool ok = true;
      const uint64_t dK0 = sw128_desc(smem_u32(sK(0)), 16u, 1024u);
      const uint64_t dQ0 = sw128_desc(smem_u32(sQ(0)), 16u, 1024u);
      const uint32_t idNN = idesc_f16(kB, 0, 0, 128, 64);
      for (int64_t it = blockIdx.x; it < items && ok; it += gridDim.x, ++kuse) {
        const int kb = static_cast<int>(kuse % KB);
        ok = mbar_wait_or_abort(&k_full[kb], (kuse / KB) & 1, 421, abort);
        const uint64_t ak = dK0 + static_cast<uint64_t>(kb * ((2 * L::kBig) >> 4));
        const uint64_t av = ak + (L::kBig >> 4);
        for (int i = 0; i < n_qs && ok; ++i, ++q_use) {
          const int b = static_cast<int>(q_use % NB), s = static_cast<int>(q_use % NS);
          ok = mbar_wait_or_abort(&ds_free[b], ((q_use / NB) & 1) ^ 1, 422, abort);
          if (ok) ok = mbar_wait_or_abort(&q_full[s], (q_use / NS) & 1, 423, abort);
          if (!ok) break;
          tc_fence_after();
          const uint64_t bq = dQ0 + static_cast<uint64_t>(s * ((2 * L::kSmall) >> 4));
          const uint64_t bdo = bq + (L::kSmall >> 4);
          const uint32_t tS = tmem + b * 128, tDP = tS + 64;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t oa = ((kk >> 2) * kHalfBytes + (kk & 3) * 32) >> 4;
            const uint32_t ob = ((kk >> 2) * L::kHalf64 + (kk & 3) * 32) >> 4;
            mma_ss(tS, ak + oa, bq + ob, idNN, kk > 0 ? 1u : 0u);
            mma_ss(tDP, av + oa, bdo + ob, idNN, kk > 0 ? 1u : 0u);
          }
          mma_commit(&s_full[b]);
          mma_commit(&q_empty[s]);
          if (i == n_qs - 1) mma_commit(&k_empty[kb]);
        }
      }
    }
  } else if (warp == 10) {
    // ---------------------------------------------------------------- dK / dV issuer
    if (lane == 0) {
      uint32_t q_use = 0, icnt = 0;
      bool ok = true;
      const uint64_t dQ0 = sw128_desc(smem_u32(sQ(0)), L::kHalf64, 1024u);
      const uint32_t idKM = idesc_f16(kB, 0, 1, 128, D);
      for (int64_t it = blockIdx.x; it < items && ok; it += gridDim.x, ++icnt) {
        ok = mbar_wait_or_abort(&kv_free, (icnt & 1) ^ 1, 431, abort);
        for (int i = 0; i < n_qs && ok; ++i, ++q_use) {
          const int b = static_cast<int>(q_use % NB), s = static_cast<int>(q_use % NS);
          ok = mbar_wait_or_abort(&p_full[b], (q_use / NB) & 1, 432, abort);
          if (!ok) break;
          tc_fence_after();
          const uint64_t bq = dQ0 + static_cast<uint64_t>(s * ((2 * L::kSmall) >> 4));
          const uint64_t bdo = bq + (L::kSmall >> 4);
          const uint32_t tP = tmem + b * 128, tD = tP + 64;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t step = (kk * 2048) >> 4;
            mma_ts(tDV, tP + kk * 8, bdo + step, idKM, (i > 0 || kk > 0) ? 1u : 0u);
            mma_ts(tDK, tD + kk * 8, bq + step, idKM, (i > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&ds_free[b]);
          mma_commit(&q_empty[s]);
        }
        if (ok) mma_commit(&kv_done);
      }
    }
  } else if (warp < 8) {
    // ---------------------------------------------------------------- compute warpgroups
    const int w = warp >> 2, wq = warp & 3, lkey = wq * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    uint32_t icnt = 0, q_base = 0;  // items, global step of the item's first step
    bool ok = true;
    for (int64_t it = blockIdx.x; it < items && ok; it += gridDim.x, ++icnt, q_base += n_qs) {
      const int bh = static_cast<int>(it / n_kt), kt = static_cast<int>(it - static_cast<int64_t>(bh) * n_kt);
      // This group takes the steps whose global index has its parity.
      for (int i = static_cast<int>((w + 2 - (q_base & 1)) & 1); i < n_qs; i += 2) {
        const uint32_t g = q_base + i;
        const int s = static_cast<int>(g % NS), b = static_cast<int>(g % NB);
        const uint32_t tS = tmem + lane_off + b * 128, tDP = tS + 64;
        ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&s_full[b], (g / NB) & 1, 441, abort));
        if (!ok) break;
        tc_fence_after();
        // The stage's lse / D were written before q_full completed, and S^T was computed after it.
        const float* st = stats + s * 128;
        // The second 32 queries' scores are requested before the first 32 are processed (latency hidden).
        uint32_t rs[2][32], rp[2][32];
        tmem_ld32(tS, rs[0]);
        tmem_ld32(tDP, rp[0]);
        tmem_wait_ld_regs(rs[0]);
        tmem_wait_ld_regs(rp[0]);
        tmem_ld32(tS + 32, rs[1]);
        tmem_ld32(tDP + 32, rp[1]);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          if (c == 1) {
            tmem_wait_ld_regs(rs[1]);
            tmem_wait_ld_regs(rp[1]);
          }
          uint32_t pp[16], pd[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            float p[2], ds[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int qc = 32 * c + e + u;
              p[u] = exp_nat(fmaf(__uint_as_float(rs[c][e + u]), scale, -st[qc]));
              ds[u] = p[u] * (__uint_as_float(rp[c][e + u]) - st[64 + qc]);
            }
            pp[e >> 1] = pack2<T>(p[0], p[1]);
            pd[e >> 1] = pack2<T>(ds[0], ds[1]);
          }
          tmem_st16(tS + 16 * c, pp);
          tmem_st16(tDP + 16 * c, pd);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[b]);
      }
      if (!ok) break;
      ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&kv_done, icnt & 1, 442, abort));
      if (!ok) break;
      tc_fence_after();
      const int key = kt * kTile + lkey;
      const int64_t gk = static_cast<int64_t>(bh) * N + key;
      // Warpgroup 0 writes dK, warpgroup 1 writes dV.
      T* dst = key < N ? (w == 0 ? dk : dv) + gk * D : nullptr;
      store_cols_from_tmem<T, D>((w == 0 ? tDK : tDV) + lane_off, 0, w == 0 ? scale : 1.f, dst);
      tc_fence_before();
      mbar_arrive(&kv_free);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, L::kTmemCols);
}

}  // namespace ebr
