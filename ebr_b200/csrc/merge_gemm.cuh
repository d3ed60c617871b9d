// merge_gemm.cuh: the input gradient of the qkv projection with the 2D-RoPE merge folded into the GEMM's A operand:
// dx = merge(dq, dk, dv) W, where merge is the adjoint of the split (g' = g cos + quarter_swap(g sin), dq first rounded
// times the per-head temperature) and W is the [3 H D, C] projection weight. The merged [tokens, 3 H D] gradient never
// reaches memory: each A tile is read head-major from dq / dk / dv and rotated in shared memory on its way to the
// tensor core.
//
// D = 64, C = 512 (one m-tile covers all C output columns as two 256-column TMEM accumulators). An m-tile is 128
// tokens of one sample (head-major rows do not cross samples); m-tiles of a sample are ceil(N / 128), the last one
// partial. One persistent CTA per SM over m-tiles. Per m-tile the K loop walks the 3 H blocks of 64 columns, block kb
// = (part kb / H, head kb % H). Roles (320 threads):
//   warp 8     TMA producer: per block, the A tile [128 tokens x 64] of dq / dk / dv (4-D box, K-major, 128-byte
//              swizzle) into a 4-stage A ring, and W rows [64 kb, 64 kb + 64) as two [64 x 256] MN-major halves into a
//              4-stage B ring;
//   warp 9     MMA issuer: per block, once its A tile is rotated, 4 x M128 N256 K16 into each accumulator half;
//   warps 0-7  rotation, then epilogue. Thread (row r = tid % 128, half f = tid / 128) owns the 16-byte chunks
//              c = f, f + 2, f + 4, f + 6 of row r: every quarter_swap partner (chunk c ^ 2) is in the same set, so a
//              thread rotates its 32 elements alone, with its row's 32 cos / sin values held in registers for the
//              m-tile. dv blocks need no rotation. At the m-tile's end warps w, w + 4 drain TMEM lanes
//              [32 (w % 4), +32), columns [256 (w / 4), +256), into dx: each [32 x 32] chunk is written to one of
//              the warp's two shared-memory boxes (64-byte swizzle) and leaves by a 3-D TMA store, which clips the
//              rows past N; the addend's row piece of the next chunk is loaded while the current one is drained.
// Rounding as ebr_rope_merge (the merged value is the same 16-bit number the unfused path writes, multiplies and adds
// rounded separately); the GEMM sums in fp32 in K-steps of 16, where cuBLAS may order the sum differently.
// The reference's rope_merge + the linear layer's input gradient (models/fused_attn/rope_split.py:52-67, :84-96).
#pragma once

#include "layers.cuh"
#include "qkv_rope.cuh"
#include "tc_attn.cuh"

namespace ebr {

struct MergeGemmLayout {
  static constexpr int kBM = 128, kBN = 256, kBK = 64, kC = 512;
  static constexpr uint32_t kATile = kBM * kBK * 2;  // 16 KB
  static constexpr uint32_t kBHalf = kBK * kBN * 2;  // 32 KB: W rows [64 kb, +64) x columns [256 h, +256)
  static constexpr int kAStages = 4, kBStages = 4;
  static constexpr uint32_t kBRing = kAStages * kATile;
  static constexpr uint32_t kEpiBox = 32 * 32 * 2;  // one epilogue warp's [32 rows x 32 columns] output chunk
  static constexpr uint32_t kEpi = kBRing + kBStages * kBHalf;  // 192 KB of rings, then two boxes per epilogue warp
  static constexpr uint32_t kBytes = kEpi + 8 * 2 * kEpiBox;
  static constexpr uint32_t kSmem = kBytes + 1024;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr int kThreads = 320;
};

// Rotate this thread's four chunks of row r of an A tile in place (16-bit T, D = 64: quarters of 16 elements, the
// partner of chunk c is chunk c ^ 2). cs[i][e] / sn[i][e]: cos / sin of element 8 (f + 2 i) + e of the row's token.
template <typename T>
__device__ __forceinline__ void merge_rotate_row(unsigned char* tile, int r, int f, const float (&cs)[4][8],
                                                 const float (&sn)[4][8], bool scale, float qs) {
  uint4 w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = *reinterpret_cast<const uint4*>(tile + sw128_off(r, f + 2 * i));
  float g[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t u[4] = {w[i].x, w[i].y, w[i].z, w[i].w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      g[i][2 * q] = unpack_lo<T>(u[q]);
      g[i][2 * q + 1] = unpack_hi<T>(u[q]);
    }
    if (scale) {
#pragma unroll
      for (int e = 0; e < 8; ++e) g[i][e] = static_cast<float>(layers::rnd<T>(layers::mul_rn(g[i][e], qs)));
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int p = i ^ 1;  // chunk f + 2 i has partner chunk (f + 2 i) ^ 2 = f + 2 (i ^ 1)
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float a = layers::add_rn(layers::mul_rn(g[i][2 * q], cs[i][2 * q]),
                                     layers::mul_rn(g[p][2 * q], sn[p][2 * q]));
      const float b = layers::add_rn(layers::mul_rn(g[i][2 * q + 1], cs[i][2 * q + 1]),
                                     layers::mul_rn(g[p][2 * q + 1], sn[p][2 * q + 1]));
      o[q] = pack2<T>(a, b);
    }
    *reinterpret_cast<uint4*>(tile + sw128_off(r, f + 2 * i)) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// tq / tk / tv: 4-D TMA maps over dq / dk / dv (D, N, H, B), box 64 x 128; tw: W [3 H D, C] (box 64 columns x 64
// rows); tdx: 3-D TMA store map over dx [B, N, C] (box 32 x 32 x 1, 64-byte swizzle). cos / sin: fp32 [N, D]; qscale:
// NULL or fp32 [H]. addend: NULL or [B, N, C]: then
// dx = round(round(merge W) + addend), the value a separate add of the two 16-bit tensors gives (a block input's
// residual gradient joined to its qkv-projection gradient).
template <typename T>
__global__ void __launch_bounds__(320, 1)
    tc_merge_gemm_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                         const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tw, int B, int H,
                         int N, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                         const float* __restrict__ qscale, const T* __restrict__ addend,
                         const __grid_constant__ CUtensorMap tdx) {
  using L = MergeGemmLayout;
  constexpr int NA = L::kAStages, NB = L::kBStages, D = 64;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = align1024(smem_raw);
  __shared__ uint64_t a_full[NA], a_ready[NA], a_empty[NA], b_full[NB], b_empty[NB], acc_full, acc_empty[2];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_nb = (N + L::kBM - 1) / L::kBM;  // 128-token blocks per sample
  const int n_kb = 3 * H;                     // 64-column blocks of the merged gradient (D = 64: one per head)
  const int64_t n_mt = static_cast<int64_t>(B) * n_nb;

  if (tid == 0) {
    for (int i = 0; i < NA; ++i) {
      mbar_init(&a_full[i], 1);
      mbar_init(&a_ready[i], 256);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < NB; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    mbar_init(&acc_full, 1);
    mbar_init(&acc_empty[0], 128);
    mbar_init(&acc_empty[1], 128);
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
  auto a_tile = [&](int s) { return smem + s * L::kATile; };
  auto b_half = [&](int s) { return smem + L::kBRing + s * L::kBHalf; };

  if (warp == 8) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      tma_prefetch_desc(&tw);
      uint32_t ause = 0, buse = 0;
      bool ok = true;
      for (int64_t mt = blockIdx.x; mt < n_mt && ok; mt += gridDim.x) {
        const int b = static_cast<int>(mt / n_nb), nb = static_cast<int>(mt - static_cast<int64_t>(b) * n_nb);
        for (int kb = 0; kb < n_kb && ok; ++kb, ++ause) {
          const int s = static_cast<int>(ause % NA);
          ok = mbar_wait_or_abort(&a_empty[s], ((ause / NA) & 1) ^ 1, 911, abort);
          if (!ok) break;
          const int part = kb / H, h = kb - part * H;
          mbar_arrive_expect_tx(&a_full[s], L::kATile);
          tma_load_4d(a_tile(s), part == 0 ? &tq : part == 1 ? &tk : &tv, &a_full[s], 0, nb * L::kBM, h, b);
          for (int nh = 0; nh < 2 && ok; ++nh, ++buse) {
            const int sb = static_cast<int>(buse % NB);
            ok = mbar_wait_or_abort(&b_empty[sb], ((buse / NB) & 1) ^ 1, 912, abort);
            if (!ok) break;
            mbar_arrive_expect_tx(&b_full[sb], L::kBHalf);
            for (int c = 0; c < 4; ++c)
              tma_load_2d(b_half(sb) + c * (L::kBK * 128), &tw, &b_full[sb], nh * L::kBN + 64 * c, kb * L::kBK);
          }
        }
      }
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t id = idesc_f16(is_bf16<T>(), 0, 1, 128, 256);  // A K-major (tokens x K), B MN-major (W rows)
      uint32_t ause = 0, buse = 0, lt = 0;
      bool ok = true;
      for (int64_t mt = blockIdx.x; mt < n_mt && ok; mt += gridDim.x, ++lt) {
        for (int kb = 0; kb < n_kb && ok; ++kb, ++ause) {
          const int s = static_cast<int>(ause % NA);
          ok = mbar_wait_or_abort(&a_ready[s], (ause / NA) & 1, 921, abort);
          if (!ok) break;
          const uint64_t da = sw128_desc(smem_u32(a_tile(s)), 16u, 1024u);
          for (int nh = 0; nh < 2 && ok; ++nh, ++buse) {
            if (kb == 0) ok = mbar_wait_or_abort(&acc_empty[nh], (lt & 1) ^ 1, 923, abort);
            const int sb = static_cast<int>(buse % NB);
            if (ok) ok = mbar_wait_or_abort(&b_full[sb], (buse / NB) & 1, 922, abort);
            if (!ok) break;
            tc_fence_after();
            const uint32_t base = smem_u32(b_half(sb));
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_ss(tmem + nh * 256, da + 2 * kk, sw128_desc(base + kk * 2048u, 64u * 128u, 1024u), id,
                     (kb > 0 || kk > 0) ? 1u : 0u);
            mma_commit(&b_empty[sb]);
          }
          if (ok) mma_commit(&a_empty[s]);
        }
        if (ok) mma_commit(&acc_full);
      }
    }
  } else if (warp < 8) {
    // ---------------------------------------------------------------- rotation, then epilogue
    const int r = tid & 127, f = tid >> 7;
    const int wq = warp & 3, half = warp >> 2;
    unsigned char* boxes = smem + L::kEpi + warp * 2 * L::kEpiBox;
    if (lane == 0) tma_prefetch_desc(&tdx);
    uint32_t ause = 0, lt = 0, chunk = 0;
    bool ok = true;
    for (int64_t mt = blockIdx.x; mt < n_mt && ok; mt += gridDim.x, ++lt) {
      const int b = static_cast<int>(mt / n_nb), nb = static_cast<int>(mt - static_cast<int64_t>(b) * n_nb);
      const int n_row = nb * L::kBM + r;  // this thread's token in the sample (rows past N are zero: any table row)
      const int nt = n_row < N ? n_row : 0;
      float cs[4][8], sn[4][8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int e0 = 8 * (f + 2 * i);
        layers::load_table_v<8>(cos_t + static_cast<int64_t>(nt) * D + e0, cs[i]);
        layers::load_table_v<8>(sin_t + static_cast<int64_t>(nt) * D + e0, sn[i]);
      }
      for (int kb = 0; kb < n_kb; ++kb, ++ause) {
        const int s = static_cast<int>(ause % NA);
        ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&a_full[s], (ause / NA) & 1, 931, abort));
        if (!ok) break;
        const int part = kb / H;
        if (part < 2) {
          const bool sc = part == 0 && qscale != nullptr;
          merge_rotate_row<T>(a_tile(s), r, f, cs, sn, sc, sc ? __ldg(qscale + (kb - part * H)) : 1.f);
          fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core
        }
        mbar_arrive(&a_ready[s]);
      }
      if (!ok) break;
      // Epilogue: this warp's 32 rows, columns [256 half, +256), as eight [32 x 32] chunks.
      const int row0 = nb * L::kBM + wq * 32, row = row0 + lane;
      const T* add = (row < N && addend) ? addend + (static_cast<int64_t>(b) * N + row) * L::kC + half * L::kBN
                                         : nullptr;
      uint4 an[4] = {};  // the addend's row piece of the next chunk
      if (add) {
#pragma unroll
        for (int q = 0; q < 4; ++q) an[q] = __ldg(reinterpret_cast<const uint4*>(add) + q);
      }
      ok = __all_sync(0xffffffffu, mbar_wait_or_abort(&acc_full, lt & 1, 932, abort));
      if (!ok) break;
      tc_fence_after();
      const uint32_t tacc = tmem + (static_cast<uint32_t>(wq * 32) << 16) + half * 256;
#pragma unroll 1
      for (int c = 0; c < L::kBN; c += 32, ++chunk) {
        uint32_t v[32];
        tmem_ld32(tacc + c, v);
        uint4 ac[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) ac[q] = an[q];
        if (add && c + 32 < L::kBN) {
#pragma unroll
          for (int q = 0; q < 4; ++q) an[q] = __ldg(reinterpret_cast<const uint4*>(add + c + 32) + q);
        }
        tmem_wait_ld_regs(v);
        if (c + 32 == L::kBN) {  // the accumulator half is read out: the next m-tile's products may start
          tc_fence_before();
          mbar_arrive(&acc_empty[half]);
        }
        unsigned char* box = boxes + (chunk & 1) * L::kEpiBox;
        if (lane == 0) tma_store_wait_read_1();  // the store issued from this box two chunks ago has read it
        __syncwarp();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) w[e] = pack2<T>(__uint_as_float(v[8 * q + 2 * e]), __uint_as_float(v[8 * q + 2 * e + 1]));
          if (add) {
            const uint32_t aw[4] = {ac[q].x, ac[q].y, ac[q].z, ac[q].w};
#pragma unroll
            for (int e = 0; e < 4; ++e)
              w[e] = pack2<T>(layers::add_rn(unpack_lo<T>(w[e]), unpack_lo<T>(aw[e])),
                              layers::add_rn(unpack_hi<T>(w[e]), unpack_hi<T>(aw[e])));
          }
          // 64-byte swizzle: the 16-byte piece q of row `lane` sits at piece q ^ ((lane >> 1) & 3)
          *reinterpret_cast<uint4*>(box + lane * 64 + 16 * (q ^ ((lane >> 1) & 3))) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && row0 < N) {  // a box wholly past the sample's last row is not issued
          tma_store_3d(&tdx, box, half * L::kBN + c, row0, b);
          tma_store_commit();
        }
      }
    }
    if (lane == 0) tma_store_wait_all();  // the boxes stay valid until every store has completed
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, L::kTmemCols);
}

}  // namespace ebr
