// qkv_rope.cuh: the qkv projection of the energy network's attention as a tensor-core GEMM whose epilogue is the 2D-RoPE
// split: q, k, v = split(x W^T) with the rotation, the per-head temperature and the head-major layout applied to each
// accumulator tile on its way out, so the [B, N, 3 H D] projection never reaches memory.
//
// One persistent CTA per SM; a tile is 128 rows of x (tokens) by 256 output columns (4 heads at D = 64, 2 at D = 128,
// all of one of q / k / v since H D is a multiple of 256). A CTA takes whole m-tiles (128 rows, all 3 H D / 256 column
// tiles in order q, k, v): m-tiles blockIdx.x, blockIdx.x + gridDim.x, ... Roles (320 threads):
//   warp 8     TMA producer: per 64-wide K block, the x tile [128 x 64] and the W tile [256 x 64] (both K-major,
//              128-byte swizzle) into a 4-stage ring;
//   warp 9     MMA issuer: 4 x tcgen05.mma M128 N256 K16 per K block into one of two 256-column accumulators in TMEM,
//              so the epilogue of a tile overlaps the products of the next;
//   warps 0-7  epilogue: warp w owns TMEM lanes [32 (w % 4), +32) (one token row per thread) and, in every head of
//              the tile, the half of the columns that warpgroup w / 4 rotates together (see qkv_slot_start). It rounds
//              the fp32 accumulators to the I/O type (the value the unfused GEMM writes), rotates q and k as
//              ebr_rope_split does -- t' = round(t cos + quarter_swap(t) sin), multiplies and adds rounded separately;
//              q' = round(q' qscale[h]) when a temperature is given -- and stores to q / k / v [B, H, N, D]
//              (32-byte runs of a head row).
// The GEMM sums in fp32 in K-steps of 16 where cuBLAS may order the sum differently, so a projection value can differ
// from the unfused path's in the last bit of the I/O type; the rotation on equal inputs is bit-identical.
// The reference's F.linear + rope_split (models/attention.py:233-242, models/fused_attn/rope_split.py:31-50, :77-82).
#pragma once

#include "layers.cuh"
#include "tc_attn.cuh"

namespace ebr {

struct QkvRopeLayout {
  static constexpr int kBM = 128, kBN = 256, kBK = 64;
  static constexpr uint32_t kATile = kBM * kBK * 2;  // 16 KB
  static constexpr uint32_t kBTile = kBN * kBK * 2;  // 32 KB
  static constexpr int kStages = 4;
  static constexpr uint32_t kStage = kATile + kBTile;
  static constexpr uint32_t kStagePitch = 80;  // bytes per staged row of an epilogue warp (64 of data)
  static constexpr uint32_t kStaging = kStages * kStage;
  static constexpr uint32_t kBytes = kStaging + 8 * 32 * kStagePitch;
  static constexpr uint32_t kSmem = kBytes + 1024;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr int kThreads = 320;
};

// The four token rows one epilogue lane stores for its warp (rows l / 4 + 8 k of the warp's 32, k = 0 .. 3): the
// offset of each row in a [B, H, N, D] tensor at head 0 (-1 for rows past M). A staged chunk of the warp's 32 rows is
// stored 16 bytes per lane, four lanes per row: eight rows per store instruction.
struct StoreRows {
  int64_t off[4];
};

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
          "r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// 2-D tiled TMA store of one box from shared memory (laid out as the map's swizzle says) to (column c0, row c1); rows
// past the tensor's end are not written. Tracked by this thread's bulk async-groups (tma_store_commit, wait below).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
               : "memory");
}
// 3-D tiled TMA store of one box (coordinates c0 innermost); elements past the tensor's extents are not written.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* smem_src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
// Wait until at most the most recent committed bulk store group of this thread may still be reading shared memory.
__device__ __forceinline__ void tma_store_wait_read_1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}

// Epilogue slots: the 32 columns of a head that one rotation pairs with each other, elements [da, da + 16) and
// [da + D / 4, da + D / 4 + 16) (quarter_swap (a, b, c, d) -> (b, a, d, c) pairs element e with e +- D / 4). At D = 64 a
// head has two slots (da = 0, 32), at D = 128 four (da = 0, 16, 64, 80). Warpgroup g of the epilogue takes slots
// [S g, S g + S) of every head of the tile (S = 1 at D = 64, 2 at D = 128), so a thread loads its token's table values
// for a slot once per tile and applies them to every head.
template <int D>
__device__ __forceinline__ int qkv_slot_start(int slot) {
  return (slot / (D / 64)) * (D / 2) + (slot % (D / 64)) * 16;
}

// The 16-bit pair of a rounded fp32 pair, and the pair widened back as an f32x2 operand.
template <typename T>
__device__ __forceinline__ uint64_t widen2(uint32_t w) {
  return f2_pack(unpack_lo<T>(w), unpack_hi<T>(w));
}
template <typename T>
__device__ __forceinline__ uint32_t narrow2(uint64_t v) {
  float lo, hi;
  f2_unpack(v, lo, hi);
  return pack2<T>(lo, hi);
}

// One slot of two heads of a token row: accumulators (fp32) at TMEM columns ta0 / ta1 + da and + da + D / 4. `tab`:
// the slot's table values as f32x2 pairs -- cos of the first 16 elements [0, 8), their sin [8, 16), cos of the
// partners [16, 24), their sin [24, 32). Each rounding of the scalar formula happens at the same place here: products
// and the sum in f32x2 (round to nearest per lane), the result rounded to the I/O type once, the temperature product
// rounded to fp32 and then to the I/O type by the store.
template <typename T, int D>
__device__ __forceinline__ void qkv_rope_slot2(uint32_t ta0, uint32_t ta1, int da, bool rotate, bool scale_q,
                                               float qs0, float qs1, const uint64_t (&tab)[32], unsigned char* stage,
                                               const StoreRows& rows, T* head0, T* head1, int lane) {
  constexpr int kQ = D / 4;
  uint32_t r[4][16];
  tmem_ld16(ta0 + da, r[0]);
  tmem_ld16(ta0 + da + kQ, r[1]);
  tmem_ld16(ta1 + da, r[2]);
  tmem_ld16(ta1 + da + kQ, r[3]);
  tmem_wait_ld();
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    uint32_t wa[8], wb[8];  // the head's outputs as 16-bit pairs: elements [da, da + 16) and their partners
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      wa[i] = pack2<T>(__uint_as_float(r[2 * hh][2 * i]), __uint_as_float(r[2 * hh][2 * i + 1]));
      wb[i] = pack2<T>(__uint_as_float(r[2 * hh + 1][2 * i]), __uint_as_float(r[2 * hh + 1][2 * i + 1]));
    }
    if (rotate) {
      const float qsf = hh == 0 ? qs0 : qs1;
      const uint64_t qs = f2_pack(qsf, qsf);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint64_t a = widen2<T>(wa[i]), b = widen2<T>(wb[i]);
        uint32_t oa = narrow2<T>(f2_add(f2_mul(a, tab[i]), f2_mul(b, tab[8 + i])));
        uint32_t ob = narrow2<T>(f2_add(f2_mul(b, tab[16 + i]), f2_mul(a, tab[24 + i])));
        if (scale_q) {
          oa = narrow2<T>(f2_mul(widen2<T>(oa), qs));
          ob = narrow2<T>(f2_mul(widen2<T>(ob), qs));
        }
        wa[i] = oa;
        wb[i] = ob;
      }
    }
    // Stage the row's 64 bytes (elements [da, da + 16) then [da + D / 4, ...)), then store four rows' pieces.
    uint4* sr = reinterpret_cast<uint4*>(stage + lane * QkvRopeLayout::kStagePitch);
    sr[0] = make_uint4(wa[0], wa[1], wa[2], wa[3]);
    sr[1] = make_uint4(wa[4], wa[5], wa[6], wa[7]);
    sr[2] = make_uint4(wb[0], wb[1], wb[2], wb[3]);
    sr[3] = make_uint4(wb[4], wb[5], wb[6], wb[7]);
    __syncwarp();
    T* head = hh == 0 ? head0 : head1;
    const int p = lane & 3, col = da + (p < 2 ? 8 * p : kQ + 8 * (p - 2));
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int rr = (lane >> 2) + 8 * k;
      const uint4 v = *reinterpret_cast<const uint4*>(stage + rr * QkvRopeLayout::kStagePitch + 16 * p);
      if (rows.off[k] >= 0) *reinterpret_cast<uint4*>(head + rows.off[k] + col) = v;
    }
    __syncwarp();
  }
}

// x: [M, C] (TMA map, box 64 x 128), w: [3 H D, C] (TMA map, box 64 x 256); M = B N tokens, C % 64 == 0,
// (H D) % 256 == 0. cos / sin: fp32 [N, D]; qscale: NULL or fp32 [H].
template <typename T, int D>
__global__ void __launch_bounds__(320, 1)
    tc_qkv_rope_kernel(const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap tw, int64_t M,
                       int C, int N, int H, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                       const float* __restrict__ qscale, T* __restrict__ q, T* __restrict__ k, T* __restrict__ v) {
  using L = QkvRopeLayout;
  constexpr int NS = L::kStages;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = align1024(smem_raw);
  __shared__ uint64_t full[NS], empty[NS], acc_full[2], acc_empty[2];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int HD = H * D, n_nt = 3 * HD / L::kBN, n_kb = C / L::kBK;
  const int64_t n_mt = (M + L::kBM - 1) / L::kBM;

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
          ok = mbar_wait_or_abort(&empty[s], ((use / NS) & 1) ^ 1, 611, abort);
          if (!ok) break;
          unsigned char* st = smem + s * L::kStage;
          mbar_arrive_expect_tx(&full[s], L::kStage);
          tma_load_2d(st, &tx, &full[s], kb * L::kBK, mt * L::kBM);
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
        ok = mbar_wait_or_abort(&acc_empty[ab], ((lt >> 1) & 1) ^ 1, 621, abort);
        for (int kb = 0; kb < n_kb && ok; ++kb, ++use) {
          const int s = static_cast<int>(use % NS);
          ok = mbar_wait_or_abort(&full[s], (use / NS) & 1, 622, abort);
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
    constexpr int kSlots = D / 64;          // slots per head this warpgroup takes
    constexpr int kHeads = L::kBN / D;      // heads per tile
    const int wq = warp & 3, grp = warp >> 2;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    unsigned char* stage = smem + L::kStaging + warp * 32 * L::kStagePitch;
    // tab: this thread's table values for one slot of its token row, as f32x2 pairs (see qkv_rope_slot2). At D = 64
    // (one slot) they serve every q / k tile of the m-tile and the next m-tile's are requested during its v tiles,
    // which do not rotate; at D = 128 each slot's are loaded before its use.
    uint64_t tab[32];
    auto load_tab = [&](int64_t mt_, int slot) {
      const int64_t row_ = mt_ * L::kBM + wq * 32 + lane;
      const int64_t n_ = row_ < M ? row_ % N : 0;
      const int da = qkv_slot_start<D>(grp * kSlots + slot);
      const float* src[4] = {cos_t + n_ * D + da, sin_t + n_ * D + da, cos_t + n_ * D + da + D / 4,
                             sin_t + n_ * D + da + D / 4};
#pragma unroll
      for (int part = 0; part < 4; ++part) {
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
          const float4 f = __ldg(reinterpret_cast<const float4*>(src[part] + i));
          tab[part * 8 + i / 2] = f2_pack(f.x, f.y);
          tab[part * 8 + i / 2 + 1] = f2_pack(f.z, f.w);
        }
      }
    };
    if (kSlots == 1 && blockIdx.x < n_mt) load_tab(blockIdx.x, 0);
    uint32_t lt = 0;
    for (int64_t j = 0;; ++j, ++lt) {
      const int64_t mt = blockIdx.x + (j / n_nt) * gridDim.x;
      if (mt >= n_mt) break;
      const int nt = static_cast<int>(j % n_nt);
      const uint32_t ab = lt & 1;
      const int sec = (nt * L::kBN) / HD, h0 = (nt * L::kBN - sec * HD) / D;  // the tile's part and first head
      const bool rotate = sec != 2, scale_q = sec == 0 && qscale != nullptr;
      const int64_t head_stride = static_cast<int64_t>(N) * D;
      T* base = (sec == 0 ? q : sec == 1 ? k : v) + h0 * head_stride;
      StoreRows rows;
#pragma unroll
      for (int kq = 0; kq < 4; ++kq) {
        const int64_t tok = mt * L::kBM + wq * 32 + (lane >> 2) + 8 * kq;
        const int64_t bq = tok / N;
        rows.off[kq] = tok < M ? (bq * H * N + (tok - bq * N)) * D : -1;
      }
      if (kSlots == 1 && sec == 2 && h0 == 0 && mt + gridDim.x < n_mt) load_tab(mt + gridDim.x, 0);
      if (!__all_sync(0xffffffffu, mbar_wait_or_abort(&acc_full[ab], (lt >> 1) & 1, 631, abort))) break;
      tc_fence_after();
      const uint32_t tacc = tmem + lane_off + ab * 256;
#pragma unroll
      for (int slot = 0; slot < kSlots; ++slot) {
        if (kSlots > 1 && rotate) load_tab(mt, slot);
        const int da = qkv_slot_start<D>(grp * kSlots + slot);
#pragma unroll
        for (int hl = 0; hl < kHeads; hl += 2) {
          const float qs0 = scale_q ? __ldg(qscale + h0 + hl) : 1.f;
          const float qs1 = scale_q ? __ldg(qscale + h0 + hl + 1) : 1.f;
          qkv_rope_slot2<T, D>(tacc + hl * D, tacc + (hl + 1) * D, da, rotate, scale_q, qs0, qs1, tab, stage, rows,
                               base + hl * head_stride, base + (hl + 1) * head_stride, lane);
        }
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
