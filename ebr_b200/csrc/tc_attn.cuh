// tc_attn.cuh: tcgen05 tensor-core kernels of the three attention passes for 16-bit inputs (bf16 / fp16).
//
// Layout. Every operand tile is a [128 rows x 64 cols] 16-bit tile in the 128-byte-swizzled layout that a TMA load
// with CU_TENSOR_MAP_SWIZZLE_128B writes (rows of 128 B, 8-row atoms of 1 KiB, 16-byte chunk c of row r stored at
// chunk c ^ (r % 8)); D = 128 uses two such tiles side by side (the "halves"). The same tile serves as a K-major
// operand (K = the 64 columns) and, read the other way, as an MN-major operand (K = the 128 rows), so Q, K, V, dO and
// the derived [query x key] tiles P / dS / A / gS are staged once and used in both orientations.
//
// Roles. 128 threads; thread t owns TMEM lane t, which is query row t of the tile (or key row t for the key-major
// accumulators). Thread 0 issues the TMA loads and the tcgen05.mma instructions; all threads do the softmax and row
// statistics on registers loaded from TMEM and write the derived 16-bit tiles to shared memory.
//
// Numerics follow the reference's Triton kernels (models/fused_attn/triton_kernels.py): 16-bit operands and fp32
// accumulation in every dot; P and dS (and the second-order tiles) rounded to the input type before they enter a
// dot (:576-586); exp applied as exp2 after subtracting in natural units (:48-56); P = exp(fma(q.k, scale, -lse))
// (:87-88); D = rowsum(dO * O) from the stored O; the fp32 scale is shared by logits and gradients (:689-693).
#pragma once

#include <type_traits>

#include "sm100.cuh"

namespace ebr {

constexpr int kTile = 128;                    // rows of a tile (queries or keys)
constexpr uint32_t kHalfBytes = 128u * 64u * 2u;  // one [128 x 64] 16-bit SW128 tile

template <typename T>
__host__ __device__ constexpr bool is_bf16() {
  return sizeof(T) == 2 && !std::is_same<T, __half>::value;
}

__device__ __forceinline__ unsigned char* align1024(unsigned char* p) {
  const uint32_t a = smem_u32(p);
  return p + ((1024u - (a & 1023u)) & 1023u);
}

// Descriptor of a K-major operand: a [128 x (64 * halves)] tile, K-step kk (16 elements) of the K = columns axis.
__device__ __forceinline__ uint64_t desc_kmajor(const unsigned char* tile, int kk) {
  return sw128_desc(smem_u32(tile) + (kk >> 2) * kHalfBytes + (kk & 3) * 32u, 16u, 1024u);
}
// Descriptor of an MN-major operand read from the same tile: MN = the columns (64 per half, halves kHalfBytes apart),
// K-step kk covers rows [16 kk, 16 kk + 16).
__device__ __forceinline__ uint64_t desc_mnmajor(const unsigned char* tile, int kk) {
  return sw128_desc(smem_u32(tile) + kk * 2048u, kHalfBytes, 1024u);
}

// Byte offset of 16-byte chunk `chunk` (0..7 within a 64-column half) of row `row` in a SW128 tile.
__device__ __forceinline__ uint32_t sw128_off(int row, int chunk) {
  return static_cast<uint32_t>(row) * 128u + ((static_cast<uint32_t>(chunk) ^ (static_cast<uint32_t>(row) & 7u)) << 4);
}

// Store 32 consecutive columns [c, c + 32) of row `row` (16 packed pairs) into a [128 x 128] 16-bit SW128 tile.
__device__ __forceinline__ void st_row32(unsigned char* tile, int row, int c, const uint32_t (&pk)[16]) {
  unsigned char* half = tile + (c >> 6) * kHalfBytes;
  const int c0 = (c & 63) >> 3;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    *reinterpret_cast<uint4*>(half + sw128_off(row, c0 + q)) =
        make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
  }
}

// Load 8 consecutive columns [8 chunk, 8 chunk + 8) of row `row` of a TMA-written SW128 operand tile, widened.
template <typename T>
__device__ __forceinline__ void ld_row8(const unsigned char* tile, int row, int chunk, float (&x)[8]) {
  const unsigned char* half = tile + (chunk >> 3) * kHalfBytes;
  const uint4 u = *reinterpret_cast<const uint4*>(half + sw128_off(row, chunk & 7));
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = static_cast<float>(e[i]);
}

template <typename T>
__device__ __forceinline__ void ld_global8(const T* p, float (&x)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = static_cast<float>(e[i]);
}

// Write one output row of D values (fp32 in TMEM columns [col, col + D) of this thread's lane) times `mul`.
template <typename T, int D>
__device__ __forceinline__ void store_row_from_tmem(uint32_t taddr, float mul, T* dst) {
#pragma unroll
  for (int c = 0; c < D; c += 32) {
    uint32_t r[32];
    tmem_ld32(taddr + c, r);
    tmem_wait_ld();
    if (dst) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 u;
        u.x = pack2<T>(__uint_as_float(r[8 * q + 0]) * mul, __uint_as_float(r[8 * q + 1]) * mul);
        u.y = pack2<T>(__uint_as_float(r[8 * q + 2]) * mul, __uint_as_float(r[8 * q + 3]) * mul);
        u.z = pack2<T>(__uint_as_float(r[8 * q + 4]) * mul, __uint_as_float(r[8 * q + 5]) * mul);
        u.w = pack2<T>(__uint_as_float(r[8 * q + 6]) * mul, __uint_as_float(r[8 * q + 7]) * mul);
        *reinterpret_cast<uint4*>(dst + c + 8 * q) = u;
      }
    }
  }
}

// Store columns [col0, col0 + NC) of this thread's TMEM lane (fp32) times `mul` to dst[col0 .. col0 + NC).
template <typename T, int NC>
__device__ __forceinline__ void store_cols_from_tmem(uint32_t taddr, int col0, float mul, T* dst) {
#pragma unroll
  for (int c = 0; c < NC; c += 32) {
    uint32_t r[32];
    tmem_ld32(taddr + col0 + c, r);
    tmem_wait_ld();
    if (dst) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 u;
        u.x = pack2<T>(__uint_as_float(r[8 * q + 0]) * mul, __uint_as_float(r[8 * q + 1]) * mul);
        u.y = pack2<T>(__uint_as_float(r[8 * q + 2]) * mul, __uint_as_float(r[8 * q + 3]) * mul);
        u.z = pack2<T>(__uint_as_float(r[8 * q + 4]) * mul, __uint_as_float(r[8 * q + 5]) * mul);
        u.w = pack2<T>(__uint_as_float(r[8 * q + 6]) * mul, __uint_as_float(r[8 * q + 7]) * mul);
        *reinterpret_cast<uint4*>(dst + col0 + c + 8 * q) = u;
      }
    }
  }
}

// Issue the K-major x K-major product over the head dim: D[tmem] (+)= A[128 x D] * B[128 x D]^T (M = N = 128).
template <int D>
__device__ __forceinline__ void mma_rows_x_rows(uint32_t d_tmem, const unsigned char* a, const unsigned char* b,
                                                uint32_t idesc, bool accumulate_first) {
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) mma_ss(d_tmem, desc_kmajor(a, kk), desc_kmajor(b, kk), idesc, (kk > 0 || accumulate_first) ? 1u : 0u);
}
// D[tmem] (+)= A[128 x 128 keys/queries] (K-major) * B (MN-major over the 128 rows of a [128 x D] tile).
__device__ __forceinline__ void mma_tile_x_rows(uint32_t d_tmem, const unsigned char* a, const unsigned char* b,
                                                uint32_t idesc, bool accumulate_first) {
#pragma unroll
  for (int kk = 0; kk < kTile / 16; ++kk)
    mma_ss(d_tmem, desc_kmajor(a, kk), desc_mnmajor(b, kk), idesc, (kk > 0 || accumulate_first) ? 1u : 0u);
}
// D[tmem] (+)= A^T (A a [128 q x 128 k] tile read MN-major: M = keys) * B (MN-major [128 q x D] tile).
__device__ __forceinline__ void mma_tileT_x_rows(uint32_t d_tmem, const unsigned char* a, const unsigned char* b,
                                                 uint32_t idesc, bool accumulate_first) {
#pragma unroll
  for (int kk = 0; kk < kTile / 16; ++kk)
    mma_ss(d_tmem, desc_mnmajor(a, kk), desc_mnmajor(b, kk), idesc, (kk > 0 || accumulate_first) ? 1u : 0u);
}

// ================================================================================================ backward helpers

// Shared helper: thread `row`'s D_i = <dO_i, O_i> from the TMA-staged dO tile and the stored (contiguous) O.
template <typename T, int D>
__device__ __forceinline__ float row_delta(const unsigned char* sDO, int row, const T* orow) {
  float di = 0.f;
#pragma unroll
  for (int c = 0; c < D / 8; ++c) {
    float x[8], y[8];
    ld_row8<T>(sDO, row, c, x);
    ld_global8<T>(orow + 8 * c, y);
#pragma unroll
    for (int i = 0; i < 8; ++i) di += x[i] * y[i];
  }
  return di;
}

// row_delta with both rows in shared memory ([128 x D] SW128 tiles of dO and O).
template <typename T, int D>
__device__ __forceinline__ float row_delta_smem(const unsigned char* sDO, const unsigned char* sO, int row) {
  float di = 0.f;
#pragma unroll
  for (int c = 0; c < D / 8; ++c) {
    float x[8], y[8];
    ld_row8<T>(sDO, row, c, x);
    ld_row8<T>(sO, row, c, y);
#pragma unroll
    for (int i = 0; i < 8; ++i) di += x[i] * y[i];
  }
  return di;
}

// ================================================================================================ tile descriptors for 64- and 128-row tiles

// Descriptors for tiles of `rows` rows (64 or 128): the 64-column halves of a D = 128 tile are rows * 128 B apart.
__device__ __forceinline__ uint64_t desc_kmajor_r(const unsigned char* tile, int kk, uint32_t half_bytes) {
  return sw128_desc(smem_u32(tile) + (kk >> 2) * half_bytes + (kk & 3) * 32u, 16u, 1024u);
}
__device__ __forceinline__ uint64_t desc_mnmajor_r(const unsigned char* tile, int kk, uint32_t half_bytes) {
  return sw128_desc(smem_u32(tile) + kk * 2048u, half_bytes, 1024u);
}

// ================================================================================================ double backward (pipelined)

template <int D>
struct BobPipeLayout {
  static constexpr uint32_t kHalf64 = 64u * 128u;
  static constexpr uint32_t kBig = (D / 64) * kHalfBytes;  // [128 x D]
  static constexpr uint32_t kSmall = (D / 64) * kHalf64;   // [64 x D]
  static constexpr int kItemBufs = D == 64 ? 2 : 1;
  static constexpr int kStages = D == 64 ? 2 : 1;
  // Item tiles: 3 (row passes: Q, dO, gQ) or 4 (column pass: K, V, gK, gV) big tiles per buffer.
  // Ring tiles: 4 (row passes: K, V, gK, gV) or 3 (column pass: Q, dO, gQ) small tiles per stage.
  static constexpr uint32_t kItemBytes = 4 * kBig;
  static constexpr uint32_t kStageBytes = 4 * kSmall;
  static constexpr uint32_t kRing = kItemBufs * kItemBytes;
  static constexpr uint32_t kStats = kRing + kStages * kStageBytes;  // column pass: [stage][L | D | E | T][64]
  static constexpr uint32_t kBytes = kStats + kStages * 4 * 64 * 4;
  static constexpr uint32_t kSmem = kBytes + 1024;
  static constexpr int kThreads = 192;
};

// Row passes of the double backward at D = 128 (D = 64 uses tc_bob.cuh) (the reference's _bob_row_kernel,
// triton_kernels.py:347-445, restated with the closed form of reference.py:80-90). An item is 128 query rows of one
// slice (Q, dO, gQ per item); the key-side tiles K, V, gK, gV stream in steps of 64 keys. Per step the MMA warp forms
// S = Q K^T, dP = dO V^T, G = gQ K^T + Q gK^T and R = dO gV^T (M = 128, N = 64) in TMEM.
//   kPhase 0 (statistics): the compute warps accumulate e = sum P G, and sum dS G, sum P dP, sum P R per row, and write
//     D = <dO, O>, E = e and T = sum P gp = sum dS G - E sum P dP + sum P R to `stats` ([3][B H N]).
//   kPhase 1 (outputs): with D, E, T known they form dS = P (dP - D), A = P (G - E), gS = P (gp - T) with
//     gp = (dP - D) G - E dP + R, pack gS, dS, A, P to 16 bits over the columns they read, and the MMA warp
//     accumulates hQ += gS K + dS gK and hdO += A V + P gV from TMEM. hQ is scaled at the end.
// `flags`: bit 0 gQ, bit 1 gK, bit 2 gV present (an absent cotangent is zero: its loads and products are skipped).
// TMEM: S [0,64), dP [64,128), G [128,192), R [192,256); phase 1 adds hQ [256, 256 + D), hdO after it.
template <typename T, int D, int kPhase>
__global__ void __launch_bounds__(192, 1)
    tc_bob_row_pipe_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tdo,
                           const __grid_constant__ CUtensorMap tgq, const __grid_constant__ CUtensorMap tk64,
                           const __grid_constant__ CUtensorMap tv64, const __grid_constant__ CUtensorMap tgk64,
                           const __grid_constant__ CUtensorMap tgv64, const T* __restrict__ o,
                           const float* __restrict__ lse, float* __restrict__ stats, T* __restrict__ hq,
                           T* __restrict__ hdo, int BH, int H, int N, float scale, uint32_t flags) {
  using L = BobPipeLayout<D>;
  constexpr int NS = L::kStages, NB = L::kItemBufs;
  constexpr uint32_t kCols = kPhase == 0 ? 256 : 512;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = align1024(smem_raw);
  __shared__ uint64_t it_full[2], it_empty[2], rg_full[2], rg_empty[2], s_full, p_full, o_done;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_qt = (N + kTile - 1) / kTile, n_ks = (N + 63) / 64;
  const int64_t items = static_cast<int64_t>(BH) * n_qt;
  const int64_t rows_total = static_cast<int64_t>(BH) * N;
  const bool has_gq = flags & 1u, has_gk = flags & 2u, has_gv = flags & 4u;
  constexpr bool kB = is_bf16<T>();
  constexpr uint32_t kIdNN = idesc_f16(kB, 0, 0, 128, 64);
  constexpr uint32_t kIdKM = idesc_f16(kB, 0, 1, 128, D);
  auto item = [&](int b, int i) { return smem + b * L::kItemBytes + i * L::kBig; };          // 0 Q, 1 dO, 2 gQ
  auto ring = [&](int s, int i) { return smem + L::kRing + s * L::kStageBytes + i * L::kSmall; };  // 0 K 1 V 2 gK 3 gV

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&it_full[i], 1);
      // Phase 0's compute warps read dO from the item tiles (for D): they release the buffer too.
      mbar_init(&it_empty[i], kPhase == 0 ? 129 : 1);
      mbar_init(&rg_full[i], 1);
      mbar_init(&rg_empty[i], 1);
    }
    mbar_init(&s_full, 1);
    mbar_init(&p_full, 128);
    mbar_init(&o_done, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  volatile int* abort = &abort_flag;

  if (warp == 4) {
    if (lane == 0) {
      uint32_t r_use = 0;
      int64_t li = 0;
      bool ok = true;
      const uint32_t item_bytes = (2u + (has_gq ? 1u : 0u)) * L::kBig;
      const uint32_t ring_bytes = (2u + (has_gk ? 1u : 0u) + (has_gv ? 1u : 0u)) * L::kSmall;
      for (int64_t it = blockIdx.x; it < items && ok; it += gridDim.x, ++li) {
        const int bh = static_cast<int>(it / n_qt), qt = static_cast<int>(it - static_cast<int64_t>(bh) * n_qt);
        const int b = bh / H, h = bh - (bh / H) * H;
        const int ib = static_cast<int>(li % NB);
        const uint32_t iu = static_cast<uint32_t>(li / NB);
        ok = mbar_wait_or_abort(&it_empty[ib], (iu & 1) ^ 1, 311, abort);
        if (!ok) break;
        mbar_arrive_expect_tx(&it_full[ib], item_bytes);
        for (int hh = 0; hh < D / 64; ++hh) {
          tma_load_4d(item(ib, 0) + hh * kHalfBytes, &tq, &it_full[ib], hh * 64, qt * kTile, h, b);
          tma_load_4d(item(ib, 1) + hh * kHalfBytes, &tdo, &it_full[ib], hh * 64, qt * kTile, h, b);
          if (has_gq) tma_load_4d(item(ib, 2) + hh * kHalfBytes, &tgq, &it_full[ib], hh * 64, qt * kTile, h, b);
        }
        for (int j = 0; j < n_ks; ++j, ++r_use) {
          const int s = static_cast<int>(r_use % NS);
          ok = mbar_wait_or_abort(&rg_empty[s], ((r_use / NS) & 1) ^ 1, 312, abort);
          if (!ok) break;
          mbar_arrive_expect_tx(&rg_full[s], ring_bytes);
          for (int hh = 0; hh < D / 64; ++hh) {
            tma_load_4d(ring(s, 0) + hh * L::kHalf64, &tk64, &rg_full[s], hh * 64, j * 64, h, b);
            tma_load_4d(ring(s, 1) + hh * L::kHalf64, &tv64, &rg_full[s], hh * 64, j * 64, h, b);
            if (has_gk) tma_load_4d(ring(s, 2) + hh * L::kHalf64, &tgk64, &rg_full[s], hh * 64, j * 64, h, b);
            if (has_gv) tma_load_4d(ring(s, 3) + hh * L::kHalf64, &tgv64, &rg_full[s], hh * 64, j * 64, h, b);
          }
        }
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      const uint32_t tS = tmem, tDP = tmem + 64, tG = tmem + 128, tR = tmem + 192;
      const uint32_t tHQ = tmem + 256, tHDO = tmem + 256 + D;
      uint32_t r_use = 0, t = 0;
      int64_t li = 0;
      bool ok = true;
      for (int64_t it = blockIdx.x; it < items && ok; it += gridDim.x, ++li) {
        const int ib = static_cast<int>(li % NB);
        ok = mbar_wait_or_abort(&it_full[ib], static_cast<uint32_t>(li / NB) & 1, 321, abort);
        for (int j = 0; j < n_ks && ok; ++j, ++r_use, ++t) {
          const int s = static_cast<int>(r_use % NS);
          ok = mbar_wait_or_abort(&rg_full[s], (r_use / NS) & 1, 322, abort);
          // The previous step's accumulators (phase 0) or 16-bit tiles (phase 1) must be consumed first.
          if (ok && t > 0)
            ok = kPhase == 0 ? mbar_wait_or_abort(&p_full, (t - 1) & 1, 323, abort)
                             : mbar_wait_or_abort(&o_done, (t - 1) & 1, 323, abort);
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t acc = kk > 0 ? 1u : 0u;
            const uint64_t dk = desc_kmajor_r(ring(s, 0), kk, L::kHalf64);
            mma_ss(tS, desc_kmajor(item(ib, 0), kk), dk, kIdNN, acc);
            mma_ss(tDP, desc_kmajor(item(ib, 1), kk), desc_kmajor_r(ring(s, 1), kk, L::kHalf64), kIdNN, acc);
            if (has_gq) mma_ss(tG, desc_kmajor(item(ib, 2), kk), dk, kIdNN, acc);
            if (has_gk)
              mma_ss(tG, desc_kmajor(item(ib, 0), kk), desc_kmajor_r(ring(s, 2), kk, L::kHalf64), kIdNN,
                     (has_gq || kk > 0) ? 1u : 0u);
            if (has_gv)
              mma_ss(tR, desc_kmajor(item(ib, 1), kk), desc_kmajor_r(ring(s, 3), kk, L::kHalf64), kIdNN, acc);
          }
          mma_commit(&s_full);
          if (kPhase == 0) {
            mma_commit(&rg_empty[s]);
            if (j == n_ks - 1) mma_commit(&it_empty[ib]);
          } else {
            ok = mbar_wait_or_abort(&p_full, t & 1, 324, abort);
            if (!ok) break;
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint32_t acc0 = (j > 0 || kk > 0) ? 1u : 0u;
              mma_ts(tHQ, tS + kk * 8, desc_mnmajor_r(ring(s, 0), kk, L::kHalf64), kIdKM, acc0);
              if (has_gk) mma_ts(tHQ, tDP + kk * 8, desc_mnmajor_r(ring(s, 2), kk, L::kHalf64), kIdKM, 1u);
              mma_ts(tHDO, tG + kk * 8, desc_mnmajor_r(ring(s, 1), kk, L::kHalf64), kIdKM, acc0);
              if (has_gv) mma_ts(tHDO, tR + kk * 8, desc_mnmajor_r(ring(s, 3), kk, L::kHalf64), kIdKM, 1u);
            }
            mma_commit(&o_done);
            mma_commit(&rg_empty[s]);
            if (j == n_ks - 1) mma_commit(&it_empty[ib]);
          }
        }
      }
    }
  } else {
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t tS = tmem + lane_off, tDP = tmem + 64 + lane_off, tG = tmem + 128 + lane_off,
                   tR = tmem + 192 + lane_off;
    uint32_t t = 0;
    int64_t li = 0;
    bool ok = true;
    for (int64_t it = blockIdx.x; it < items && ok; it += gridDim.x, ++li) {
      const int bh = static_cast<int>(it / n_qt), qt = static_cast<int>(it - static_cast<int64_t>(bh) * n_qt);
      const int ib = static_cast<int>(li % NB);
      const int row = qt * kTile + tid;
      const bool row_ok = row < N;
      const int64_t grow = static_cast<int64_t>(bh) * N + row;
      const float Li = row_ok ? lse[grow] : 0.f;
      float Di = 0.f, Ei = 0.f, Ti = 0.f;
      if (kPhase == 0) {
        ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&it_full[ib], static_cast<uint32_t>(li / NB) & 1, 331, abort));
        if (!ok) break;
        if (row_ok) Di = row_delta<T, D>(item(ib, 1), tid, o + grow * D);
        mbar_arrive(&it_empty[ib]);
      } else if (row_ok) {
        Di = stats[grow];
        Ei = stats[rows_total + grow];
        Ti = stats[2 * rows_total + grow];
      }
      float e_ = 0.f, c1 = 0.f, c2 = 0.f, c3 = 0.f;
      for (int j = 0; j < n_ks; ++j, ++t) {
        ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&s_full, t & 1, 332, abort));
        if (!ok) break;
        tc_fence_after();
        const int valid = N - j * 64;
#pragma unroll 1
        for (int c = 0; c < 64; c += 16) {
          uint32_t rs[16], rp[16], rg[16], rr[16];
          tmem_ld16(tS + c, rs);
          tmem_ld16(tDP + c, rp);
          if (has_gq || has_gk) tmem_ld16(tG + c, rg);
          if (has_gv) tmem_ld16(tR + c, rr);
          tmem_wait_ld();
          if (kPhase == 0) {
#pragma unroll
            for (int u = 0; u < 16; ++u) {
              float p = exp_nat(fmaf(__uint_as_float(rs[u]), scale, -Li));
              if (valid < 64 && c + u >= valid) p = 0.f;
              const float g = (has_gq || has_gk) ? __uint_as_float(rg[u]) * scale : 0.f;
              const float dp = __uint_as_float(rp[u]);
              e_ += p * g;
              c1 += p * (dp - Di) * g;
              c2 += p * dp;
              if (has_gv) c3 += p * __uint_as_float(rr[u]);
            }
          } else {
            uint32_t pgs[8], pds[8], pa[8], pp[8];
#pragma unroll
            for (int u = 0; u < 16; u += 2) {
              float v_gs[2], v_ds[2], v_a[2], v_p[2];
#pragma unroll
              for (int w = 0; w < 2; ++w) {
                float p = exp_nat(fmaf(__uint_as_float(rs[u + w]), scale, -Li));
                if (valid < 64 && c + u + w >= valid) p = 0.f;
                const float g = (has_gq || has_gk) ? __uint_as_float(rg[u + w]) * scale : 0.f;
                const float dp = __uint_as_float(rp[u + w]);
                const float r = has_gv ? __uint_as_float(rr[u + w]) : 0.f;
                const float gp = (dp - Di) * g - Ei * dp + r;
                v_p[w] = p;
                v_ds[w] = p * (dp - Di);
                v_a[w] = p * (g - Ei);
                v_gs[w] = p * (gp - Ti);
              }
              pgs[u >> 1] = pack2<T>(v_gs[0], v_gs[1]);
              pds[u >> 1] = pack2<T>(v_ds[0], v_ds[1]);
              pa[u >> 1] = pack2<T>(v_a[0], v_a[1]);
              pp[u >> 1] = pack2<T>(v_p[0], v_p[1]);
            }
            tmem_st8(tS + (c >> 1), pgs);
            tmem_st8(tDP + (c >> 1), pds);
            tmem_st8(tG + (c >> 1), pa);
            tmem_st8(tR + (c >> 1), pp);
          }
        }
        if (kPhase == 1) tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full);
      }
      if (!ok) break;
      if (kPhase == 0) {
        if (row_ok) {
          stats[grow] = Di;
          stats[rows_total + grow] = e_;
          stats[2 * rows_total + grow] = c1 - e_ * c2 + c3;
        }
      } else {
        ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&o_done, (t - 1) & 1, 333, abort));
        if (!ok) break;
        tc_fence_after();
        T* none = nullptr;
        store_row_from_tmem<T, D>(tmem + 256 + lane_off, scale, row_ok ? hq + grow * D : none);
        store_row_from_tmem<T, D>(tmem + 256 + D + lane_off, 1.f, row_ok ? hdo + grow * D : none);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kCols);
}

// Column pass of the double backward at D = 128 (D = 64 uses tc_bob.cuh) (the reference's _bob_col_kernel,
// triton_kernels.py:448-551): an item is 128 keys of one slice (K, V, gK, gV per item); the query-side tiles Q, dO,
// gQ stream in steps of 64 queries, with each step's lse, D, E, T staged in shared memory by the producer warp.
// Per step: S^T, dP^T, G^T = K gQ^T + gK Q^T, R^T = gV dO^T (M = 128 keys, N = 64 queries); the compute warps
// (thread t = key t) form gS^T, dS^T, A^T as in the row pass and the MMA warp accumulates hK += gS^T Q + dS^T gQ and
// hV += A^T dO from TMEM. TMEM: S^T [0,64), dP^T [64,128), G^T [128,192), R^T [192,256), hK [256, 256 + D), hV after.
template <typename T, int D>
__global__ void __launch_bounds__(192, 1)
    tc_bob_col_pipe_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                           const __grid_constant__ CUtensorMap tgk, const __grid_constant__ CUtensorMap tgv,
                           const __grid_constant__ CUtensorMap tq64, const __grid_constant__ CUtensorMap tdo64,
                           const __grid_constant__ CUtensorMap tgq64, const float* __restrict__ lse,
                           const float* __restrict__ stats, T* __restrict__ hk, T* __restrict__ hv, int BH, int H,
                           int N, float scale, uint32_t flags) {
  using L = BobPipeLayout<D>;
  constexpr int NS = L::kStages, NB = L::kItemBufs;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = align1024(smem_raw);
  __shared__ uint64_t it_full[2], it_empty[2], rg_full[2], rg_empty[2], s_full, p_full, o_done;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_kt = (N + kTile - 1) / kTile, n_qs = (N + 63) / 64;
  const int64_t items = static_cast<int64_t>(BH) * n_kt;
  const int64_t rows_total = static_cast<int64_t>(BH) * N;
  const bool has_gq = flags & 1u, has_gk = flags & 2u, has_gv = flags & 4u;
  constexpr bool kB = is_bf16<T>();
  constexpr uint32_t kIdNN = idesc_f16(kB, 0, 0, 128, 64);
  constexpr uint32_t kIdKM = idesc_f16(kB, 0, 1, 128, D);
  auto item = [&](int b, int i) { return smem + b * L::kItemBytes + i * L::kBig; };          // 0 K 1 V 2 gK 3 gV
  auto ring = [&](int s, int i) { return smem + L::kRing + s * L::kStageBytes + i * L::kSmall; };  // 0 Q 1 dO 2 gQ
  float* stg = reinterpret_cast<float*>(smem + L::kStats);  // [stage][L 64 | D 64 | E 64 | T 64]

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&it_full[i], 1);
      mbar_init(&it_empty[i], 1);
      mbar_init(&rg_full[i], 33);  // TMA transaction arrive + one arrive per producer lane after its scalar writes
      mbar_init(&rg_empty[i], 1);
    }
    mbar_init(&s_full, 1);
    mbar_init(&p_full, 128);
    mbar_init(&o_done, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  volatile int* abort = &abort_flag;

  if (warp == 4) {
    uint32_t r_use = 0;
    int64_t li = 0;
    bool ok = true;
    const uint32_t item_bytes = (2u + (has_gk ? 1u : 0u) + (has_gv ? 1u : 0u)) * L::kBig;
    const uint32_t ring_bytes = (2u + (has_gq ? 1u : 0u)) * L::kSmall;
    for (int64_t it = blockIdx.x; it < items && ok; it += gridDim.x, ++li) {
      const int bh = static_cast<int>(it / n_kt), kt = static_cast<int>(it - static_cast<int64_t>(bh) * n_kt);
      const int b = bh / H, h = bh - (bh / H) * H;
      const int64_t base = static_cast<int64_t>(bh) * N;
      const int ib = static_cast<int>(li % NB);
      if (lane == 0) {
        ok = mbar_wait_or_abort(&it_empty[ib], (static_cast<uint32_t>(li / NB) & 1) ^ 1, 341, abort);
        if (ok) {
          mbar_arrive_expect_tx(&it_full[ib], item_bytes);
          for (int hh = 0; hh < D / 64; ++hh) {
            tma_load_4d(item(ib, 0) + hh * kHalfBytes, &tk, &it_full[ib], hh * 64, kt * kTile, h, b);
            tma_load_4d(item(ib, 1) + hh * kHalfBytes, &tv, &it_full[ib], hh * 64, kt * kTile, h, b);
            if (has_gk) tma_load_4d(item(ib, 2) + hh * kHalfBytes, &tgk, &it_full[ib], hh * 64, kt * kTile, h, b);
            if (has_gv) tma_load_4d(item(ib, 3) + hh * kHalfBytes, &tgv, &it_full[ib], hh * 64, kt * kTile, h, b);
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      for (int i = 0; i < n_qs && ok; ++i, ++r_use) {
        const int s = static_cast<int>(r_use % NS);
        ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&rg_empty[s], ((r_use / NS) & 1) ^ 1, 342, abort));
        if (!ok) break;
        if (lane == 0) {
          mbar_arrive_expect_tx(&rg_full[s], ring_bytes);
          for (int hh = 0; hh < D / 64; ++hh) {
            tma_load_4d(ring(s, 0) + hh * L::kHalf64, &tq64, &rg_full[s], hh * 64, i * 64, h, b);
            tma_load_4d(ring(s, 1) + hh * L::kHalf64, &tdo64, &rg_full[s], hh * 64, i * 64, h, b);
            if (has_gq) tma_load_4d(ring(s, 2) + hh * L::kHalf64, &tgq64, &rg_full[s], hh * 64, i * 64, h, b);
          }
        }
        // Queries past N get L = D = E = T = 0: with their zero Q / dO / gQ rows every derived value there is 0.
        float* st = stg + s * 256;
#pragma unroll
        for (int k2 = lane; k2 < 64; k2 += 32) {
          const int qi = i * 64 + k2;
          const bool in = qi < N;
          st[k2] = in ? lse[base + qi] : 0.f;
          st[64 + k2] = in ? stats[base + qi] : 0.f;
          st[128 + k2] = in ? stats[rows_total + base + qi] : 0.f;
          st[192 + k2] = in ? stats[2 * rows_total + base + qi] : 0.f;
        }
        mbar_arrive(&rg_full[s]);
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      const uint32_t tS = tmem, tDP = tmem + 64, tG = tmem + 128, tR = tmem + 192;
      const uint32_t tHK = tmem + 256, tHV = tmem + 256 + D;
      uint32_t r_use = 0, t = 0;
      int64_t li = 0;
      bool ok = true;
      for (int64_t it = blockIdx.x; it < items && ok; it += gridDim.x, ++li) {
        const int ib = static_cast<int>(li % NB);
        ok = mbar_wait_or_abort(&it_full[ib], static_cast<uint32_t>(li / NB) & 1, 351, abort);
        for (int i = 0; i < n_qs && ok; ++i, ++r_use, ++t) {
          const int s = static_cast<int>(r_use % NS);
          ok = mbar_wait_or_abort(&rg_full[s], (r_use / NS) & 1, 352, abort);
          if (ok && t > 0) ok = mbar_wait_or_abort(&o_done, (t - 1) & 1, 353, abort);
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t acc = kk > 0 ? 1u : 0u;
            const uint64_t dq_ = desc_kmajor_r(ring(s, 0), kk, L::kHalf64);
            mma_ss(tS, desc_kmajor(item(ib, 0), kk), dq_, kIdNN, acc);
            mma_ss(tDP, desc_kmajor(item(ib, 1), kk), desc_kmajor_r(ring(s, 1), kk, L::kHalf64), kIdNN, acc);
            if (has_gq) mma_ss(tG, desc_kmajor(item(ib, 0), kk), desc_kmajor_r(ring(s, 2), kk, L::kHalf64), kIdNN, acc);
            if (has_gk) mma_ss(tG, desc_kmajor(item(ib, 2), kk), dq_, kIdNN, (has_gq || kk > 0) ? 1u : 0u);
            if (has_gv)
              mma_ss(tR, desc_kmajor(item(ib, 3), kk), desc_kmajor_r(ring(s, 1), kk, L::kHalf64), kIdNN, acc);
          }
          mma_commit(&s_full);
          ok = mbar_wait_or_abort(&p_full, t & 1, 354, abort);
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t acc0 = (i > 0 || kk > 0) ? 1u : 0u;
            mma_ts(tHK, tS + kk * 8, desc_mnmajor_r(ring(s, 0), kk, L::kHalf64), kIdKM, acc0);
            if (has_gq) mma_ts(tHK, tDP + kk * 8, desc_mnmajor_r(ring(s, 2), kk, L::kHalf64), kIdKM, 1u);
            mma_ts(tHV, tG + kk * 8, desc_mnmajor_r(ring(s, 1), kk, L::kHalf64), kIdKM, acc0);
          }
          mma_commit(&o_done);
          mma_commit(&rg_empty[s]);
          if (i == n_qs - 1) mma_commit(&it_empty[ib]);
        }
      }
    }
  } else {
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t tS = tmem + lane_off, tDP = tmem + 64 + lane_off, tG = tmem + 128 + lane_off,
                   tR = tmem + 192 + lane_off;
    uint32_t t = 0;
    bool ok = true;
    for (int64_t it = blockIdx.x; it < items && ok; it += gridDim.x) {
      const int bh = static_cast<int>(it / n_kt), kt = static_cast<int>(it - static_cast<int64_t>(bh) * n_kt);
      for (int i = 0; i < n_qs; ++i, ++t) {
        const int s = static_cast<int>(t % NS);
        ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&rg_full[s], (t / NS) & 1, 361, abort));
        if (!ok) break;
        const float* st = stg + s * 256;
        ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&s_full, t & 1, 362, abort));
        if (!ok) break;
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 64; c += 16) {
          uint32_t rs[16], rp[16], rg[16], rr[16];
          tmem_ld16(tS + c, rs);
          tmem_ld16(tDP + c, rp);
          if (has_gq || has_gk) tmem_ld16(tG + c, rg);
          if (has_gv) tmem_ld16(tR + c, rr);
          tmem_wait_ld();
          uint32_t pgs[8], pds[8], pa[8];
#pragma unroll
          for (int u = 0; u < 16; u += 2) {
            float v_gs[2], v_ds[2], v_a[2];
#pragma unroll
            for (int w = 0; w < 2; ++w) {
              const int qc = c + u + w;
              const float Lq = st[qc], Dq = st[64 + qc], Eq = st[128 + qc], Tq = st[192 + qc];
              const float p = exp_nat(fmaf(__uint_as_float(rs[u + w]), scale, -Lq));
              const float g = (has_gq || has_gk) ? __uint_as_float(rg[u + w]) * scale : 0.f;
              const float dp = __uint_as_float(rp[u + w]);
              const float r = has_gv ? __uint_as_float(rr[u + w]) : 0.f;
              const float gp = (dp - Dq) * g - Eq * dp + r;
              v_ds[w] = p * (dp - Dq);
              v_a[w] = p * (g - Eq);
              v_gs[w] = p * (gp - Tq);
            }
            pgs[u >> 1] = pack2<T>(v_gs[0], v_gs[1]);
            pds[u >> 1] = pack2<T>(v_ds[0], v_ds[1]);
            pa[u >> 1] = pack2<T>(v_a[0], v_a[1]);
          }
          tmem_st8(tS + (c >> 1), pgs);
          tmem_st8(tDP + (c >> 1), pds);
          tmem_st8(tG + (c >> 1), pa);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full);
      }
      if (!ok) break;
      ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&o_done, (t - 1) & 1, 363, abort));
      if (!ok) break;
      tc_fence_after();
      const int key = kt * kTile + tid;
      const int64_t gk = static_cast<int64_t>(bh) * N + key;
      T* none = nullptr;
      store_row_from_tmem<T, D>(tmem + 256 + lane_off, scale, key < N ? hk + gk * D : none);
      store_row_from_tmem<T, D>(tmem + 256 + D + lane_off, 1.f, key < N ? hv + gk * D : none);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

}  // namespace ebr
