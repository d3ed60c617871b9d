// o_proj.cuh: the attention's output projection as a tensor-core GEMM that reads the attention output in its
// head-major [B, H, N, D] layout, y[b, n, :] = sum_h O[b, h, n, :] W[:, h D : (h + 1) D]^T, so the [B, H, N, D] ->
// [B, N, H D] transpose copy in front of the projection is never made.
//
// One persistent CTA per SM; an m-tile is 128 tokens of one batch item (rows n0 .. n0 + 127 of every head; a last,
// partial block of a sample reads zeros past N and stores only its valid rows), an n-tile 256 output columns. A CTA
// takes whole m-tiles (all of their n-tiles): m-tiles blockIdx.x, blockIdx.x + gridDim.x, ... Roles (320 threads):
//   warp 8     TMA producer: per 64-wide K block (head h, columns [64 c, 64 c + 64) of it) the O tile [128 x 64] (a
//              4-D box of one (b, h)) and the W tile [256 x 64], both K-major with 128-byte swizzle, into a 3-stage
//              ring;
//   warp 9     MMA issuer: 4 x tcgen05.mma M128 N256 K16 per K block into one of two 256-column TMEM accumulators;
//   warps 0-7  epilogue: warp w owns TMEM lanes [32 (w % 4), +32) (one token per thread) and columns
//              [128 (w / 4), +128) of the tile; it rounds the fp32 sums to the I/O type and stores them to y through
//              its shared-memory staging buffer (eight 64-byte row segments per store instruction).
// The reference's self.o(y.transpose(1, 2).reshape(b, n, h d)) in EnergyAttention (models/attention.py:241-242).
#pragma once

#include "qkv_rope.cuh"

namespace ebr {

// 128 x 256 tiles, 64-wide K blocks, a 3-stage ring, two TMEM accumulators and, after the ring, one [32 rows x 80 B]
// staging buffer per epilogue warp (a 32-column chunk is re-read from it so that four consecutive lanes store one row's
// 64 bytes: eight whole row segments per store instruction).
struct OProjLayout {
  static constexpr int kBM = 128, kBN = 256, kBK = 64;
  static constexpr uint32_t kATile = kBM * kBK * 2;
  static constexpr uint32_t kBTile = kBN * kBK * 2;
  static constexpr int kStages = 3;
  static constexpr uint32_t kStage = kATile + kBTile;
  static constexpr uint32_t kStagePitch = 80;
  static constexpr uint32_t kStaging = kStages * kStage;
  static constexpr uint32_t kBytes = kStaging + 8 * 32 * kStagePitch;
  static constexpr uint32_t kSmem = kBytes + 1024;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr int kThreads = 320;
};

// o: 4-D TMA map over O (D, N, H, B), box 64 x 128; w: [C_out, H D] (TMA map, box 64 x 256); y: [B, N, C_out].
template <typename T, int D>
__global__ void __launch_bounds__(320, 1)
    tc_o_proj_kernel(const __grid_constant__ CUtensorMap to, const __grid_constant__ CUtensorMap tw, int B, int H,
                     int N, int C_out, T* __restrict__ y) {
  using L = OProjLayout;
  constexpr int NS = L::kStages;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = align1024(smem_raw);
  __shared__ uint64_t full[NS], empty[NS], acc_full[2], acc_empty[2];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_nb = (N + L::kBM - 1) / L::kBM;  // 128-token blocks per sample
  const int n_nt = C_out / L::kBN, n_kb = H * (D / L::kBK);
  const int64_t n_mt = static_cast<int64_t>(B) * n_nb;

  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 256);
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
      tma_prefetch_desc(&to);
      tma_prefetch_desc(&tw);
      uint32_t use = 0;
      bool ok = true;
      for (int64_t j = 0; ok; ++j) {
        const int64_t mt = blockIdx.x + (j / n_nt) * gridDim.x;
        if (mt >= n_mt) break;
        const int nt = static_cast<int>(j % n_nt);
        const int b = static_cast<int>(mt / n_nb), nb = static_cast<int>(mt - static_cast<int64_t>(b) * n_nb);
        for (int kb = 0; kb < n_kb; ++kb, ++use) {
          const int s = static_cast<int>(use % NS);
          ok = mbar_wait_or_abort(&empty[s], ((use / NS) & 1) ^ 1, 811, abort);
          if (!ok) break;
          unsigned char* st = smem + s * L::kStage;
          mbar_arrive_expect_tx(&full[s], L::kStage);
          const int h = kb / (D / L::kBK), c = kb - h * (D / L::kBK);
          tma_load_4d(st, &to, &full[s], c * L::kBK, nb * L::kBM, h, b);
          tma_load_2d(st + L::kATile, &tw, &full[s], kb * L::kBK, nt * L::kBN);
        }
      }
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t id = idesc_f16(is_bf16<T>(), 0, 0, 128, 256);
      const uint64_t d0 = sw128_desc(smem_u32(smem), 16u, 1024u);
      uint32_t use = 0, lt = 0;
      bool ok = true;
      for (int64_t j = 0; ok && blockIdx.x + (j / n_nt) * gridDim.x < n_mt; ++j, ++lt) {
        const uint32_t ab = lt & 1;
        ok = mbar_wait_or_abort(&acc_empty[ab], ((lt >> 1) & 1) ^ 1, 821, abort);
        for (int kb = 0; kb < n_kb && ok; ++kb, ++use) {
          const int s = static_cast<int>(use % NS);
          ok = mbar_wait_or_abort(&full[s], (use / NS) & 1, 822, abort);
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
  } else if (warp < 8) {
    // ---------------------------------------------------------------- epilogue
    const int wq = warp & 3, grp = warp >> 2;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    unsigned char* stage = smem + L::kStaging + warp * 32 * L::kStagePitch;
    uint32_t lt = 0;
    for (int64_t j = 0;; ++j, ++lt) {
      const int64_t mt = blockIdx.x + (j / n_nt) * gridDim.x;
      if (mt >= n_mt) break;
      const int nt = static_cast<int>(j % n_nt);
      const int b = static_cast<int>(mt / n_nb), nb = static_cast<int>(mt - static_cast<int64_t>(b) * n_nb);
      const int n0 = nb * L::kBM + wq * 32;  // this warp's first token
      T* dst = y + static_cast<int64_t>(b) * N * C_out + nt * L::kBN + grp * 128;
      const uint32_t ab = lt & 1;
      if (!__all_sync(0xffffffffu, mbar_wait_or_abort(&acc_full[ab], (lt >> 1) & 1, 831, abort))) break;
      tc_fence_after();
      const uint32_t tacc = tmem + lane_off + ab * 256 + grp * 128;
      // Two 32-column loads in flight: the next one is requested before the current one is rounded and stored.
      uint32_t r[2][32];
      tmem_ld32(tacc, r[0]);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        tmem_wait_ld_regs(r[c & 1]);
        if (c < 3) tmem_ld32(tacc + 32 * (c + 1), r[(c + 1) & 1]);
        // The row's 32 columns go to the warp's staging buffer; lane l then stores 16 bytes (l % 4) of token
        // n0 + l / 4 + 8 k, so each store instruction writes eight whole 64-byte row segments.
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const uint32_t* v = &r[c & 1][8 * q4];
          *reinterpret_cast<uint4*>(stage + lane * L::kStagePitch + 16 * q4) =
              make_uint4(pack2<T>(__uint_as_float(v[0]), __uint_as_float(v[1])),
                         pack2<T>(__uint_as_float(v[2]), __uint_as_float(v[3])),
                         pack2<T>(__uint_as_float(v[4]), __uint_as_float(v[5])),
                         pack2<T>(__uint_as_float(v[6]), __uint_as_float(v[7])));
        }
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int rr = lane / 4 + 8 * k;
          const uint4 val = *reinterpret_cast<const uint4*>(stage + rr * L::kStagePitch + 16 * (lane % 4));
          if (n0 + rr < N)
            *reinterpret_cast<uint4*>(dst + static_cast<int64_t>(n0 + rr) * C_out + 32 * c + 8 * (lane % 4)) = val;
        }
        __syncwarp();
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[ab]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, L::kTmemCols);
}

}  // namespace ebr
