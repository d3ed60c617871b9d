// tc_fwd.cuh: the tensor-core forward for N > 128: two query tiles of one (b, h) slice per CTA in ping-pong, keys
// in 64-key tiles with the scores double-buffered in tensor memory.
//
// One persistent CTA per SM; an item is a pair of 128-row query tiles (2p, 2p + 1) of one slice, which share every
// K / V tile the producer stages. Tensor memory (512 columns): the S / P columns of tile A are [0, 128), of tile B
// [128, 256), each split into two 64-column halves used by alternate key tiles; O of A is [256, 256 + D), of B
// [256 + D, 256 + 2 D). While the softmax works on key tile j in one half, the tensor core computes S(j + 1) into the
// other, so the softmax warps never wait for a Q K^T product except at the start of an item. Roles:
//   warps 0-3  softmax of tile A, warps 4-7 softmax of tile B: thread t owns query row t of its tile (TMEM lane t)
//              and the whole 64-key row of S, so the row max and row sum need no exchange between threads;
//   warp 8     TMA producer: the pair's two Q tiles (double-buffered at D = 64), 64-key K / V tiles into a ring;
//   warp 9     MMA issuer: per key tile j, O += P V for A and B (P read from TMEM), then S(j + 2) = Q K^T for A and
//              B into the half P(j) occupied, once that P V has completed;
//   warp 10    (D = 64) V converter: each V tile transposed and widened to fp32 for the tf32 P V product.
// Per key tile a softmax thread loads its 64 scores (two tcgen05.ld of 32 columns), takes the row max with the
// three-input max, and forms P = 2^(s * scale * log2 e - m * log2 e) with one ex2 per element. O and the row sum are
// rescaled only when the max grows past the one in use by more than 8 (log2 units) -- a warp-uniform decision, since
// tcgen05.ld / st are warp-collective -- after waiting for the previous P V to land in O. P is written back over S:
// in fp32 at D = 64 (the P V product runs in tf32, so P keeps 10 mantissa bits and is never rounded to 16 bits), as a
// 16-bit hi / lo pair at D = 128 (for keys [16 k, 16 k + 16): P_hi in columns [16 k, 16 k + 8), P_lo in
// [16 k + 8, 16 k + 16); O += P_hi V + P_lo V). A ragged last key tile is computed over ceil(n / 32) * 32 keys, and
// warps whose 32 query rows all lie past N skip their softmax work.
// Same math as the reference's _fwd_kernel (triton_kernels.py:98-163) with P carried more accurately.
#pragma once

#include "tc_attn.cuh"

namespace ebr {

constexpr int kKeyTile = 64;  // keys per K / V tile of the paired forward

template <int D>
struct FwdPairLayout {
  static constexpr bool kTf32 = D == 64;                   // P V in tf32 (else 16-bit hi / lo)
  static constexpr uint32_t kOp = (D / 64) * kHalfBytes;   // one [128 x D] 16-bit tile (Q)
  static constexpr uint32_t kKv = (D / 64) * 64u * 128u;   // one [64 x D] 16-bit tile (K or V)
  static constexpr uint32_t kVt = kTf32 ? 2u * kKv : 0u;   // the fp32 transposed V tile
  static constexpr int kQBufs = D == 64 ? 2 : 1;           // Q buffers per tile of the pair
  static constexpr int kStages = 4;                        // K / V ring depth
  static constexpr uint32_t kQ = 0;                        // Q of tile t, buffer b: kQ + (t * kQBufs + b) * kOp
  static constexpr uint32_t kStage = 2 * kKv + kVt;        // stage s: K, V, fp32 V^T
  static constexpr uint32_t kKV = 2 * kQBufs * kOp;
  static constexpr uint32_t kBytes = kKV + kStages * kStage;
  static constexpr uint32_t kSmem = kBytes + 1024;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr int kThreads = kTf32 ? 384 : 352;  // 8 softmax + producer + 2 MMA (+ converter) warps
  // S / P buffers of 64 columns per query tile: three at D = 64 (3 x 64 + 64 columns of O per tile), two at D = 128.
  static constexpr int kSBufs = D == 64 ? 3 : 2;
  static constexpr uint32_t kOCol = 2 * kSBufs * 64;  // first O column (O of tile t at kOCol + t D)
};

// Key columns computed in key tile j of n_kt (all 64 but in a ragged last tile: a multiple of 32).
__device__ __forceinline__ int fwd_cols(int j, int n_kt, int N) {
  if (j < n_kt - 1) return kKeyTile;
  const int valid = N - j * kKeyTile;
  return ((valid + 31) >> 5) << 5;
}

// The fp32 V tile is stored transposed, as the K-major B operand of the tf32 P V product (tf32 takes K-major
// operands in the plain 128-byte swizzle): rows = the 64 head-dim columns, K = the 64 keys in two 32-key blocks of
// [64 rows x 128 B] (8 KiB apart), 8-row swizzle atoms of 1 KiB. K-step kk (8 keys, 32 bytes) of the descriptor:
__device__ __forceinline__ uint64_t desc_vt32(const unsigned char* tile, int kk) {
  return sw128_desc(smem_u32(tile) + (kk >> 2) * 8192u + (kk & 3) * 32u, 16u, 1024u);
}

// Transpose-and-widen keys [0, keys) (a multiple of 32) of a TMA-written [64 keys x 64] 16-bit SW128 V tile into
// that layout. One warp: lane l < keys / 4 owns keys [4 l, 4 l + 4) and walks the eight 8-column chunks; per chunk it
// reads four 16-byte rows and writes eight 16-byte rows (4 keys of one head-dim column each); the eight lanes of one
// key block write eight different 16-byte slots of a row.
template <typename T>
__device__ __forceinline__ void widen_vt_tile(const unsigned char* src, unsigned char* dst, int keys, int lane) {
  if (4 * lane >= keys) return;
  const int slot = lane & 7;
  unsigned char* out = dst + (lane >> 3) * 8192;
#pragma unroll 2
  for (int c = 0; c < 8; ++c) {
    float f[4][8];
#pragma unroll
    for (int kq = 0; kq < 4; ++kq) {
      const uint4 u = *reinterpret_cast<const uint4*>(src + sw128_off(4 * lane + kq, c));
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        f[kq][2 * q] = unpack_lo<T>(w[q]);
        f[kq][2 * q + 1] = unpack_hi<T>(w[q]);
      }
    }
#pragma unroll
    for (int d = 0; d < 8; ++d) {
      const int row = 8 * c + d;
      *reinterpret_cast<float4*>(out + sw128_off(row, slot)) = make_float4(f[0][d], f[1][d], f[2][d], f[3][d]);
    }
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(D == 64 ? 384 : 352, 1)
    tc_fwd_pair_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                       const __grid_constant__ CUtensorMap tv, T* __restrict__ out, float* __restrict__ lse, int BH,
                       int H, int N, float scale) {
  using L = FwdPairLayout<D>;
  constexpr int NS = L::kStages, QB = L::kQBufs;
  constexpr bool TF = L::kTf32;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = align1024(smem_raw);
  constexpr int NB = L::kSBufs;
  // s_full / p_full / o_done per query tile and per S buffer: several key tiles of one query tile are in flight at
  // once, and an mbarrier's parity only tells one phase from the next.
  __shared__ uint64_t q_full[2][QB], q_empty[2][QB], kv_full[NS], kv_empty[NS], vt_full[NS], s_full[2][NB],
      p_full[2][NB], o_done[2][NB];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_qt = (N + kTile - 1) / kTile, n_kt = (N + kKeyTile - 1) / kKeyTile;
  const int n_pairs = (n_qt + 1) >> 1;
  const int64_t items = static_cast<int64_t>(BH) * n_pairs;
  constexpr bool kB = is_bf16<T>();
  constexpr uint32_t kIdPV = TF ? idesc_tf32(0, 0, 128, D) : idesc_f16(kB, 0, 1, 128, D);
  constexpr float kLog2e = 1.4426950408889634f;
  constexpr float kTau = 5.545177444479562f;  // 8 ln 2: lazy-rescale threshold in natural units
  auto sQ = [&](int t, int b) { return smem + L::kQ + (t * QB + b) * L::kOp; };
  auto sK = [&](int s) { return smem + L::kKV + s * L::kStage; };
  auto sV = [&](int s) { return smem + L::kKV + s * L::kStage + L::kKv; };
  auto sVt = [&](int s) { return smem + L::kKV + s * L::kStage + 2 * L::kKv; };

  if (tid == 0) {
    for (int t = 0; t < 2; ++t) {
      for (int b = 0; b < QB; ++b) {
        mbar_init(&q_full[t][b], 1);
        mbar_init(&q_empty[t][b], 1);
      }
      for (int h = 0; h < NB; ++h) {
        mbar_init(&s_full[t][h], 1);
        mbar_init(&p_full[t][h], 128);
        mbar_init(&o_done[t][h], 1);
      }
    }
    for (int i = 0; i < NS; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 2);  // one commit from each tile's MMA warp
      mbar_init(&vt_full[i], 1);
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
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      uint32_t kv_use = 0, quse[2] = {0, 0};
      bool ok = true;
      for (int64_t it = blockIdx.x; it < items && ok; it += gridDim.x) {
        const int bh = static_cast<int>(it / n_pairs), pr = static_cast<int>(it - static_cast<int64_t>(bh) * n_pairs);
        const int b = bh / H, h = bh - (bh / H) * H;
        for (int t = 0; t < 2 && ok; ++t) {
          const int qt = 2 * pr + t;
          if (qt >= n_qt) break;
          const int qb = static_cast<int>(quse[t] % QB);
          ok = mbar_wait_or_abort(&q_empty[t][qb], ((quse[t] / QB) & 1) ^ 1, 211, abort);
          if (!ok) break;
          mbar_arrive_expect_tx(&q_full[t][qb], L::kOp);
          for (int hh = 0; hh < D / 64; ++hh)
            tma_load_4d(sQ(t, qb) + hh * kHalfBytes, &tq, &q_full[t][qb], hh * 64, qt * kTile, h, b);
          ++quse[t];
        }
        for (int j = 0; j < n_kt && ok; ++j, ++kv_use) {
          const int s = static_cast<int>(kv_use % NS);
          ok = mbar_wait_or_abort(&kv_empty[s], ((kv_use / NS) & 1) ^ 1, 212, abort);
          if (!ok) break;
          mbar_arrive_expect_tx(&kv_full[s], 2 * L::kKv);
          for (int hh = 0; hh < D / 64; ++hh) {
            tma_load_4d(sK(s) + hh * (64 * 128), &tk, &kv_full[s], hh * 64, j * kKeyTile, h, b);
            tma_load_4d(sV(s) + hh * (64 * 128), &tv, &kv_full[s], hh * 64, j * kKeyTile, h, b);
          }
        }
      }
    }
  } else if (warp == 11) {
    // ---------------------------------------------------------------- V transpose + widening (tf32 P V only)
    if constexpr (TF) {
      uint32_t kv_use = 0;
      bool ok = true;
      for (int64_t it = blockIdx.x; it < items && ok; it += gridDim.x) {
        for (int j = 0; j < n_kt && ok; ++j, ++kv_use) {
          const int s = static_cast<int>(kv_use % NS);
          ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&kv_full[s], (kv_use / NS) & 1, 241, abort));
          if (!ok) break;
          widen_vt_tile<T>(sV(s), sVt(s), fwd_cols(j, n_kt, N), lane);
          fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core
          __syncwarp();
          if (lane == 0) mbar_arrive(&vt_full[s]);
        }
      }
    }
  } else if (warp == 9 || warp == 10) {
    // ---------------------------------------------------------------- MMA issuers, one per query tile of the pair
    // Warp 9 issues tile A's products, warp 10 tile B's; the tensor pipe interleaves the two streams. Per key tile j:
    // O_t += P_t(j) V_j once P_t(j) is written (and at D = 64 V_j widened), then S_t(j + 2) = Q_t K_{j+2}^T into
    // buffer (j + 2) % NB once the P V product that last used it (tile j + 2 - NB) has completed. Phase parities
    // are kept as bit masks (bit b: buffer b) so the loop state stays in registers.
    const int t = warp - 9;
    if (lane == 0) {
      uint32_t kv_use = 0, quse = 0, pbits = 0, obits = 0;  // obits: parity of the NEXT o_done commit per buffer
      bool ok = true;
      const uint64_t dQ = sw128_desc(smem_u32(sQ(t, 0)), 16u, 1024u);
      const uint64_t dK = sw128_desc(smem_u32(sK(0)), 16u, 1024u);
      const uint64_t dV = TF ? sw128_desc(smem_u32(sVt(0)), 16u, 1024u) : sw128_desc(smem_u32(sV(0)), 64u * 128u, 1024u);
      constexpr uint64_t kStageD = L::kStage >> 4;
      const uint32_t idS = idesc_f16(kB, 0, 0, 128, kKeyTile);
      const uint32_t idS_last = idesc_f16(kB, 0, 0, 128, fwd_cols(n_kt - 1, n_kt, N));
      const int nc_last = fwd_cols(n_kt - 1, n_kt, N);
      const uint32_t tS0 = tmem + t * (NB * 64), tO = tmem + L::kOCol + t * D;
      // S(j) = Q K_j^T into buffer b. A: the [128 x D] Q tile (64-column halves 16 KiB apart); B: the [64 x D] K tile
      // in stage s (halves 8 KiB apart).
      auto issue_s = [&](int qb, int b, uint32_t s, bool last) {
        const uint64_t a0 = dQ + static_cast<uint64_t>(qb * (L::kOp >> 4));
        const uint64_t b0 = dK + s * kStageD;
        const uint32_t id = last ? idS_last : idS;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          mma_ss(tS0 + b * 64, a0 + (((kk >> 2) * kHalfBytes + (kk & 3) * 32) >> 4),
                 b0 + (((kk >> 2) * 8192 + (kk & 3) * 32) >> 4), id, kk > 0 ? 1u : 0u);
      };
      // O += P(j) V_j, P from buffer b, V (or V^T in fp32) from stage s.
      auto issue_pv = [&](int b, uint32_t s, bool first, bool last) {
        const uint32_t tP = tS0 + b * 64;
        const uint64_t v0 = dV + s * kStageD;
        const int nsteps = (last ? nc_last : kKeyTile) / (TF ? 8 : 16);
        if constexpr (TF) {
#pragma unroll
          for (int kk = 0; kk < kKeyTile / 8; ++kk)
            if (kk < nsteps)
              mma_ts_tf32(tO, tP + kk * 8, v0 + (((kk >> 2) * 8192 + (kk & 3) * 32) >> 4), kIdPV,
                          (!first || kk > 0) ? 1u : 0u);
        } else {
#pragma unroll
          for (int kk = 0; kk < kKeyTile / 16; ++kk) {
            if (kk < nsteps) {
              const uint64_t bd = v0 + ((kk * 2048) >> 4);
              mma_ts(tO, tP + kk * 16, bd, kIdPV, (!first || kk > 0) ? 1u : 0u);
              mma_ts(tO, tP + kk * 16 + 8, bd, kIdPV, 1u);
            }
          }
        }
      };
      for (int64_t it = blockIdx.x; it < items && ok; it += gridDim.x) {
        const int bh = static_cast<int>(it / n_pairs), pr = static_cast<int>(it - static_cast<int64_t>(bh) * n_pairs);
        const bool active = 2 * pr + t < n_qt;
        if (!active) {
          // No tile B in this pair: still release each K / V stage once it has been filled (in order, so an
          // arrival never runs ahead of the stage's use by the other warp).
          for (int j = 0; j < n_kt && ok; ++j, ++kv_use) {
            ok = mbar_wait_or_abort(&kv_full[kv_use % NS], (kv_use / NS) & 1, 229, abort);
            if (ok) mbar_arrive(&kv_empty[kv_use % NS]);
          }
          continue;
        }
        const int qb = static_cast<int>(quse % QB);
        ok = mbar_wait_or_abort(&q_full[t][qb], (quse / QB) & 1, 221, abort);
        // S(0) and S(1) (the previous item's P V products have all completed: waited at its end).
        for (int jj = 0; jj < 2 && jj < n_kt && ok; ++jj) {
          const uint32_t u = kv_use + jj;
          ok = mbar_wait_or_abort(&kv_full[u % NS], (u / NS) & 1, 222, abort);
          if (!ok) break;
          tc_fence_after();
          issue_s(qb, jj, u % NS, jj == n_kt - 1);
          mma_commit(&s_full[t][jj]);
          if (jj == n_kt - 1) mma_commit(&q_empty[t][qb]);
        }
        int b = 0;  // buffer of tile j (j % NB)
        for (int j = 0; j < n_kt && ok; ++j, ++kv_use) {
          const uint32_t s = kv_use % NS;
          if constexpr (TF) {
            ok = mbar_wait_or_abort(&vt_full[s], (kv_use / NS) & 1, 227, abort);
            if (!ok) break;
          }
          ok = mbar_wait_or_abort(&p_full[t][b], (pbits >> b) & 1, 224, abort);
          if (!ok) break;
          pbits ^= 1u << b;
          tc_fence_after();
          issue_pv(b, s, j == 0, j == n_kt - 1);
          mma_commit(&o_done[t][b]);
          obits ^= 1u << b;
          mma_commit(&kv_empty[s]);
          if (j + 2 < n_kt) {
            // S(j + 2) into buffer (j + 2) % NB, last used by tile j + 2 - NB: wait for that P V to complete.
            const int b2 = (b + 2) % NB;
            const uint32_t u2 = kv_use + 2;
            ok = mbar_wait_or_abort(&kv_full[u2 % NS], (u2 / NS) & 1, 223, abort);
            if (ok) ok = mbar_wait_or_abort(&o_done[t][b2], ((obits >> b2) & 1) ^ 1, 225, abort);
            if (!ok) break;
            tc_fence_after();
            issue_s(qb, b2, u2 % NS, j + 2 == n_kt - 1);
            mma_commit(&s_full[t][b2]);
            if (j + 2 == n_kt - 1) mma_commit(&q_empty[t][qb]);
          }
          b = (b + 1 == NB) ? 0 : b + 1;
        }
        // The next item's S(0) / S(1) overwrite these buffers: its last P V (and so every earlier one) must have
        // completed.
        const int bl = (n_kt - 1) % NB;
        if (ok) ok = mbar_wait_or_abort(&o_done[t][bl], ((obits >> bl) & 1) ^ 1, 226, abort);
        ++quse;
      }
    }
  } else if (warp < 8) {
    // ---------------------------------------------------------------- softmax / epilogue (warps 0-7)
    const int t = warp >> 2, wq = warp & 3, lrow = wq * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t tSt = tmem + lane_off + t * (NB * 64), tO = tmem + lane_off + L::kOCol + t * D;
    const bool pos = scale >= 0.f;
    const float c1 = scale * kLog2e;
    const float fill = pos ? -INFINITY : INFINITY;
    uint32_t hcnt[NB] = {};  // key tiles processed in each S buffer (= phases of its s_full / p_full / o_done)
    bool ok = true;
    for (int64_t it = blockIdx.x; it < items && ok; it += gridDim.x) {
      const int bh = static_cast<int>(it / n_pairs), pr = static_cast<int>(it - static_cast<int64_t>(bh) * n_pairs);
      const int qt = 2 * pr + t;
      if (qt >= n_qt) continue;  // tile B of an odd tile count: nothing for this warpgroup
      const int row = qt * kTile + lrow;
      const bool warp_rows = qt * kTile + wq * 32 < N;  // warp-uniform: any of this warp's rows inside [0, N)
      float m_used = -INFINITY, l_run = 0.f;
      for (int j = 0; j < n_kt; ++j) {
        const int hf = j % NB;
        ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&s_full[t][hf], hcnt[hf] & 1, 231, abort));
        if (!ok) break;
        tc_fence_after();
        if (warp_rows) {
          const uint32_t tS = tSt + hf * 64;
          const int nc = fwd_cols(j, n_kt, N), nch = nc >> 5;
          const int valid = N - j * kKeyTile;  // keys of this tile inside [0, N) (>= nc - 31)
          uint32_t r[2][32];
          tmem_ld32(tS, r[0]);
          if (nch > 1) tmem_ld32(tS + 32, r[1]);
          tmem_wait_ld_regs(r[0]);
          tmem_wait_ld_regs(r[1]);
          // Row max of the raw scores (the min for a negative scale), masked keys excluded.
          float m0 = fill, m1 = fill;
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            if (c < nch) {
              if (valid < nc) {  // ragged last tile only (warp-uniform)
#pragma unroll
                for (int e = 0; e < 32; ++e)
                  if (32 * c + e >= valid) r[c][e] = __float_as_uint(fill);
              }
              if (pos) {
#pragma unroll
                for (int e = 0; e < 32; e += 4) {
                  m0 = fmax3(m0, __uint_as_float(r[c][e]), __uint_as_float(r[c][e + 1]));
                  m1 = fmax3(m1, __uint_as_float(r[c][e + 2]), __uint_as_float(r[c][e + 3]));
                }
              } else {
#pragma unroll
                for (int e = 0; e < 32; e += 4) {
                  m0 = fmin3(m0, __uint_as_float(r[c][e]), __uint_as_float(r[c][e + 1]));
                  m1 = fmin3(m1, __uint_as_float(r[c][e + 2]), __uint_as_float(r[c][e + 3]));
                }
              }
            }
          }
          const float mx = (pos ? fmaxf(m0, m1) : fminf(m0, m1)) * scale;
          const bool need = (j == 0) || (mx > m_used + kTau);
          float alpha = 1.f;
          if (need) {
            alpha = (j == 0) ? 0.f : exp_nat(m_used - mx);
            l_run *= alpha;
            m_used = mx;
          }
          // P = 2^(s * scale log2 e - m log2 e), 32 key columns per TMEM store.
          const float negm = -m_used * kLog2e;
          float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            if (c < nch) {
              uint32_t pk[32];
#pragma unroll
              for (int g = 0; g < 2; ++g) {  // 16 keys (hi / lo layout: hi -> pk[16 g .. + 8), lo -> + 8)
#pragma unroll
                for (int e = 0; e < 16; e += 2) {
                  const int ke = 16 * g + e;
                  // Masked keys hold -inf / +inf: fma gives -inf (the scale's sign matches the fill), 2^-inf = 0.
                  const float p0 = exp2_approx(fmaf(__uint_as_float(r[c][ke]), c1, negm));
                  const float p1 = exp2_approx(fmaf(__uint_as_float(r[c][ke + 1]), c1, negm));
                  if (e & 2) {
                    acc2 += p0;
                    acc3 += p1;
                  } else {
                    acc0 += p0;
                    acc1 += p1;
                  }
                  if constexpr (TF) {
                    pk[ke] = __float_as_uint(p0);
                    pk[ke + 1] = __float_as_uint(p1);
                  } else {
                    const uint32_t ph = pack2<T>(p0, p1);
                    pk[16 * g + (e >> 1)] = ph;
                    pk[16 * g + 8 + (e >> 1)] = pack2<T>(p0 - unpack_lo<T>(ph), p1 - unpack_hi<T>(ph));
                  }
                }
              }
              tmem_st32(tS + 32 * c, pk);
            }
          }
          l_run += (acc0 + acc1) + (acc2 + acc3);
          // Lazy rescale of O, once the previous P V (S(j) may have been computed before it) has landed.
          if (j > 0 && __any_sync(0xffffffffu, need)) {
            const int hp = (j - 1) % NB;
            ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&o_done[t][hp], (hcnt[hp] - 1) & 1, 233, abort));
            tc_fence_after();
            if (ok) {
#pragma unroll 1
              for (int c = 0; c < D; c += 32) {
                uint32_t o[32];
                tmem_ld32(tO + c, o);
                tmem_wait_ld_regs(o);
#pragma unroll
                for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
                tmem_st32(tO + c, o);
              }
            }
          }
          tmem_wait_st();
        }
        tc_fence_before();
        mbar_arrive(&p_full[t][hf]);
        ++hcnt[hf];
        if (!ok) break;
      }
      if (!ok) break;
      const int hl = (n_kt - 1) % NB;  // the last P V of the item (its completion implies the earlier ones')
      ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&o_done[t][hl], (hcnt[hl] - 1) & 1, 232, abort));
      if (!ok) break;
      tc_fence_after();
      if (warp_rows) {
        const bool row_ok = row < N;
        const int64_t grow = static_cast<int64_t>(bh) * N + row;
        store_cols_from_tmem<T, D>(tO, 0, 1.f / l_run, row_ok ? out + grow * D : nullptr);
        if (row_ok) lse[grow] = m_used + logf(l_run);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, L::kTmemCols);
}

}  // namespace ebr
