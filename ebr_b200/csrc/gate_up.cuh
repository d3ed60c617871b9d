// gate_up.cuh: the MLP's gate / up projection as a tensor-core GEMM whose epilogue also applies the SwiGLU activation:
// h = x W^T ([rows, 2 I]: gate columns [0, I), up columns [I, 2 I)) and act = round(round(silu(gate)) * up), both
// written once, so the activation never re-reads h from memory (h is kept for the backward).
//
// One persistent CTA per SM; a tile is 128 rows of x by 128 gate columns [j0, j0 + 128) and the matching 128 up
// columns [I + j0, I + j0 + 128): the W tile of a K block is two 128-row TMA boxes stacked into one [256 x 64] operand,
// so one M128 N256 K16 instruction forms both halves. A CTA takes whole m-tiles (all I / 128 column tiles). Roles as in
// the qkv projection (qkv_rope.cuh): producer warp (16), MMA warp (17), sixteen epilogue warps -- warp w owns TMEM
// lanes [32 (w % 4), +32) (one row per thread) and the gate / up column pairs [16 g, +16) and [16 (g + 4), +16) of the
// tile, g = w / 4. The epilogue
// rounds gate and up to the I/O type (the values the unfused GEMM writes), stores them to h, and forms the activation
// as ebr_swiglu_fwd does (silu(g) = g / (1 + exp(-g)) in fp32, rounded; times up, rounded).
// The reference's F.silu(gate) * up after gate_up_proj(x).chunk(2) (models/layers.py:82-84).
#pragma once

#include "qkv_rope.cuh"

namespace ebr {

// 128 x 256 tiles, 64-wide K blocks, two TMEM accumulators as the qkv projection; a 4-stage ring and, after it, two
// [32 rows x 16 columns] staging boxes per epilogue warp (1 KB each, 32-byte swizzle). A warp writes each output chunk
// into one box and one lane stores it with a tiled TMA store, alternating the two boxes: the stores leave the warp at
// once and the async proxy writes whole 32-byte row pieces, where per-lane global stores of the same pieces held the
// epilogue warps behind the SM's store path (0.36 of 1.13 ms at 262k tokens).
// Sixteen epilogue warps (four per TMEM lane quarter) keep enough exponentials and divisions in flight to stay ahead of
// the tensor pipe; 576 threads leave 96 registers a thread.
struct GateUpLayout {
  static constexpr int kBM = 128, kBN = 256, kBK = 64;
  static constexpr uint32_t kATile = kBM * kBK * 2;
  static constexpr uint32_t kBTile = kBN * kBK * 2;
  static constexpr int kStages = 4;
  static constexpr uint32_t kStage = kATile + kBTile;
  static constexpr int kEpiWarps = 16;
  static constexpr uint32_t kBox = 32 * 16 * 2;  // one [32 x 16] output chunk
  static constexpr uint32_t kStaging = kStages * kStage;
  static constexpr uint32_t kBytes = kStaging + kEpiWarps * 2 * kBox;
  static constexpr uint32_t kSmem = kBytes + 1024;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr int kThreads = (kEpiWarps + 2) * 32;
};

// x: [M, C] (TMA map, box 64 x 128); w: [2 I, C] (TMA map, box 64 x 128); th: h [M, 2 I] and ta: act [M, I] (TMA
// store maps, box 16 x 32, 32-byte swizzle).
template <typename T>
__global__ void __launch_bounds__(GateUpLayout::kThreads, 1)
    tc_gate_up_swiglu_kernel(const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap tw,
                             const __grid_constant__ CUtensorMap th, const __grid_constant__ CUtensorMap ta, int64_t M,
                             int C, int I) {
  using L = GateUpLayout;
  constexpr int NS = L::kStages;
  constexpr uint32_t kHalfB = L::kBTile / 2;  // one 128-row W box
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = align1024(smem_raw);
  __shared__ uint64_t full[NS], empty[NS], acc_full[2], acc_empty[2];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_nt = I / 128, n_kb = C / L::kBK;
  const int64_t n_mt = (M + L::kBM - 1) / L::kBM;

  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], L::kEpiWarps * 32);
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

  if (warp == L::kEpiWarps) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tx);
      tma_prefetch_desc(&tw);
      uint32_t use = 0;
      bool ok = true;
      for (int64_t j = 0; ok; ++j) {
        const int64_t mt = blockIdx.x + (j / n_nt) * gridDim.x;
        if (mt >= n_mt) break;
        const int nt = static_cast<int>(j % n_nt);
        for (int kb = 0; kb < n_kb; ++kb, ++use) {
          const int s = static_cast<int>(use % NS);
          ok = mbar_wait_or_abort(&empty[s], ((use / NS) & 1) ^ 1, 911, abort);
          if (!ok) break;
          unsigned char* st = smem + s * L::kStage;
          mbar_arrive_expect_tx(&full[s], L::kStage);
          tma_load_2d(st, &tx, &full[s], kb * L::kBK, static_cast<int>(mt * L::kBM));
          tma_load_2d(st + L::kATile, &tw, &full[s], kb * L::kBK, nt * 128);              // gate rows
          tma_load_2d(st + L::kATile + kHalfB, &tw, &full[s], kb * L::kBK, I + nt * 128);  // up rows
        }
      }
    }
  } else if (warp == L::kEpiWarps + 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t id = idesc_f16(is_bf16<T>(), 0, 0, 128, 256);
      const uint64_t d0 = sw128_desc(smem_u32(smem), 16u, 1024u);
      uint32_t use = 0, lt = 0;
      bool ok = true;
      for (int64_t j = 0; ok && blockIdx.x + (j / n_nt) * gridDim.x < n_mt; ++j, ++lt) {
        const uint32_t ab = lt & 1;
        ok = mbar_wait_or_abort(&acc_empty[ab], ((lt >> 1) & 1) ^ 1, 921, abort);
        for (int kb = 0; kb < n_kb && ok; ++kb, ++use) {
          const int s = static_cast<int>(use % NS);
          ok = mbar_wait_or_abort(&full[s], (use / NS) & 1, 922, abort);
          if (!ok) break;
          tc_fence_after();
          const uint64_t da = d0 + ((s * L::kStage) >> 4), db = da + (L::kATile >> 4);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_ss(tmem + ab * 256, da + 2 * kk, db + 2 * kk, id, (kb > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&empty[s]);
        }
        if (ok) mma_commit(&acc_full[ab]);
      }
    }
  } else if (warp < L::kEpiWarps) {
    // ---------------------------------------------------------------- epilogue
    using layers::mul_rn;
    using layers::rnd;
    const int wq = warp & 3, grp = warp >> 2;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    unsigned char* stage = smem + L::kStaging + warp * 2 * L::kBox;
    if (lane == 0) {
      tma_prefetch_desc(&th);
      tma_prefetch_desc(&ta);
    }
    uint32_t chunk = 0;  // chunks this warp has stored (the staging box alternates)
    // Store a [32 rows x 16 columns] chunk at (row_base, col) of the map's matrix. Lane r writes row r's 32 bytes,
    // its two 16-byte halves swapped on rows with bit 2 set (the 32-byte swizzle: address bit 4 ^= bit 7), so that the
    // eight lanes of each shared-memory phase hit distinct banks. Before a box is rewritten, the store issued from it
    // two chunks ago must have finished reading it.
    auto store_chunk = [&](const uint32_t (&w)[8], const CUtensorMap* map, int64_t row_base, int col) {
      unsigned char* box = stage + (chunk & 1) * L::kBox;
      if (lane == 0) tma_store_wait_read_1();
      __syncwarp();
      uint4* sr = reinterpret_cast<uint4*>(box + lane * 32);
      const int sw = (lane >> 2) & 1;
      sr[sw] = make_uint4(w[0], w[1], w[2], w[3]);
      sr[sw ^ 1] = make_uint4(w[4], w[5], w[6], w[7]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && row_base < M) {  // a box wholly past the last row is not issued
        tma_store_2d(map, box, col, static_cast<int>(row_base));
        tma_store_commit();
      }
      ++chunk;
    };
    uint32_t lt = 0;
    for (int64_t j = 0;; ++j, ++lt) {
      const int64_t mt = blockIdx.x + (j / n_nt) * gridDim.x;
      if (mt >= n_mt) break;
      const int nt = static_cast<int>(j % n_nt);
      const int64_t row_base = mt * L::kBM + wq * 32;  // this warp's first row
      const uint32_t ab = lt & 1;
      if (!__all_sync(0xffffffffu, mbar_wait_or_abort(&acc_full[ab], (lt >> 1) & 1, 931, abort))) break;
      tc_fence_after();
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        const int cc = 16 * (grp + 4 * part);  // gate / up column pair offset within the tile
        const uint32_t tg = tmem + lane_off + ab * 256 + cc, tu = tg + 128;
        uint32_t rg[16], ru[16];
        tmem_ld16(tg, rg);
        tmem_ld16(tu, ru);
        tmem_wait_ld();
        if (part == 1) {  // the accumulator is read out: the MMA warp may refill it while this tile is stored
          tc_fence_before();
          mbar_arrive(&acc_empty[ab]);
        }
        uint32_t wg[8], wu[8], wa[8];
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          wg[p] = pack2<T>(__uint_as_float(rg[2 * p]), __uint_as_float(rg[2 * p + 1]));
          wu[p] = pack2<T>(__uint_as_float(ru[2 * p]), __uint_as_float(ru[2 * p + 1]));
          float a2[2];
#pragma unroll
          for (int x = 0; x < 2; ++x) {
            const float g = x == 0 ? unpack_lo<T>(wg[p]) : unpack_hi<T>(wg[p]);
            const float u = x == 0 ? unpack_lo<T>(wu[p]) : unpack_hi<T>(wu[p]);
            a2[x] = mul_rn(rnd<T>(g / (1.f + expf(-g))), u);
          }
          wa[p] = pack2<T>(a2[0], a2[1]);
        }
        const int c0 = nt * 128 + cc;
        store_chunk(wg, &th, row_base, c0);
        store_chunk(wu, &th, row_base, I + c0);
        store_chunk(wa, &ta, row_base, c0);
      }
    }
    if (lane == 0) tma_store_wait_all();  // the staging boxes stay valid until every store has completed
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, L::kTmemCols);
}

}  // namespace ebr
