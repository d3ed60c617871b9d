// tc_short.cuh: short-sequence (N <= 128) tensor-core kernels.
//
// At N <= 128 a whole (b, h) slice fits one 128-row tile, so the passes are bound by HBM, not by the tensor pipe
// (4 N^2 D FLOP against 8 N D bytes in the forward: about N / 2 FLOP per byte, far below the B200's ~250). What
// decides their speed is how many bytes each SM keeps in flight and how little each tile waits on the previous one.
// So these kernels are persistent (one CTA per SM), keep a ring of input stages loading ahead, double-buffer every
// tensor-memory accumulator so the tensor pipe works on tile t + 1 while tile t is in the pointwise code, and write
// their outputs through shared memory with TMA stores.
//
// Packing. ``per`` = floor(128 / N) slices are stacked in one 128-row tile when their rows sit at a uniform stride
// (B * H slices read as one axis of the tensor map; otherwise ``per`` divides H and the tile stays inside one batch
// row). Row r of a tile belongs to slice r / N and attends only to the keys of that slice: the score tile is
// block-diagonal and every other column is masked. Rows and key columns at or beyond per * N are zero in shared
// memory (the stages are cleared once; the TMA boxes never reach them).
//
// Geometry. The 4-D tensor maps are (D, N, Hs, Bs) with boxes (64, N, per, 1): Hs = B * H and Bs = 1 when the
// slices are packed along one axis, else Hs = H and Bs = B. Tile t covers Hs-indices [h0, h0 + per) of Bs-index b'
// with h0 = (t mod ceil(Hs / per)) * per; its slice r / N is b' * Hs + h0 + r / N, valid while h0 + r / N < Hs (the
// boxes read zeros past the end and the stores clip there).
#pragma once

#include "tc_attn.cuh"

namespace ebr {

struct ShortGeom {
  int N;            // rows of a slice
  int per;          // slices per tile
  int hs;           // extent of the tensor maps' third axis (H, or B * H when packed along one axis)
  int tiles_per_b;  // ceil(hs / per)
  int tiles;        // tiles_per_b * Bs
};

__device__ __forceinline__ void short_tile_coords(const ShortGeom& g, int t, int& hb, int& h0) {
  hb = t / g.tiles_per_b;
  h0 = (t - hb * g.tiles_per_b) * g.per;
}

// ================================================================================================ forward

template <int D>
struct FwdShortLayout {
  static constexpr uint32_t kOp = (D / 64) * kHalfBytes;    // one [128 x D] 16-bit tile
  static constexpr uint32_t kBytes = 3 * kOp;               // Q, K, V (O is staged over the spent V)
  static constexpr uint32_t kSmem = kBytes + 1024;
  static constexpr uint32_t kTmemCols = D == 64 ? 128 : 256;  // S, then P (fp16) in [0, 64) and O in [64, 64 + D)
  static constexpr int kCtasPerSm = D == 64 ? 4 : 2;
  static constexpr int kThreads = 128;
};

// Forward for N <= 128. Each CTA is one 4-warp pipeline over its tiles (blockIdx.x, blockIdx.x + gridDim.x, ...),
// and kCtasPerSm of them share an SM, so several tiles are always in different phases on one SM: the pass is bound by
// HBM, and a single tile's chain (scores -> softmax -> P V -> store) is long, so overlap between tiles is what keeps
// the memory system busy. Thread r owns row r of the tile (tensor-memory lane r); thread 0 also issues the TMA
// loads, the tcgen05 products and the TMA store. Per tile:
//   S = Q K^T into tensor memory; once it is done the next tile's Q and K are loaded over the spent ones;
//   row max m of s scale over the row's slice; P = 2^(s scale log2 e - m log2 e) (0 outside the slice) written back as
//   fp16 pairs into columns [0, kc / 2) (columns already read);
//   V converted in place to fp16 times 2^e, e the one power of two that puts the tile's max |v| in [2^14, 2^15)
//   (exact: a 16-bit input has at most 11 significant bits; nothing overflows, and entries below 2^-28 of the
//   largest lose relative precision only); fp16 inputs are used as they are;
//   O = P V (tcgen05 kind::f16, P from tensor memory) into columns [64, 64 + D); O 2^-e / l rounded over the spent V,
//   one TMA store, lse = m + log l; the next tile's V is loaded once the store has read the buffer.
// P keeps fp16's 11 significant bits in the P V product (the reference's kernels round P to the 16-bit input type,
// models/fused_attn/triton_kernels.py:576-586); otherwise the math of the reference's _fwd_kernel (:98-163) with the
// whole key range in one tile.
template <typename T, int D>
__global__ void __launch_bounds__(128, D == 64 ? 4 : 2)
    tc_fwd_short_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap to,
                        float* __restrict__ lse, const ShortGeom geo, float scale) {
  using L = FwdShortLayout<D>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = align1024(smem_raw);
  unsigned char* sq = smem;
  unsigned char* sk = smem + L::kOp;
  unsigned char* sv = smem + 2 * L::kOp;
  __shared__ uint64_t qk_full, v_full, s_full, o_full;
  __shared__ uint32_t tmem_slot, vmax_slot[4];
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int N = geo.N, rows = geo.per * geo.N;
  const int kc = (rows + 31) & ~31;  // key columns computed (the S product's N; the P V product's K)
  constexpr bool kB = is_bf16<T>();
  const uint32_t id_s = idesc_f16(kB, 0, 0, 128, kc);
  constexpr uint32_t kIdPV = idesc_f16(false, 0, 1, 128, D);  // fp16 P (tensor memory) x fp16 V (shared, MN-major)
  const int n_local = geo.tiles > static_cast<int>(blockIdx.x)
                          ? (geo.tiles - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                          : 0;
  const uint32_t box_bytes = 128u * static_cast<uint32_t>(rows);  // one 64-column box of `rows` rows

  // Clear the tiles once: rows at or beyond `rows` (never written by the boxes) must be finite for the products.
  for (uint32_t i = tid * 16u; i < L::kBytes; i += L::kThreads * 16u)
    *reinterpret_cast<uint4*>(smem + i) = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async_smem();
  if (tid == 0) {
    mbar_init(&qk_full, 1);
    mbar_init(&v_full, 1);
    mbar_init(&s_full, 1);
    mbar_init(&o_full, 1);
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
  const bool leader = tid == 0;
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  const uint32_t tS = tmem + lane_off, tO = tmem + 64 + lane_off;
  const int r = tid;
  const bool row_ok = r < rows;
  const int j0_row = row_ok ? (r / N) * N : 0;  // this row's key columns: [j0_row, j1_row)
  const int j1_row = row_ok ? j0_row + N : 0;
  const int wlo = __reduce_min_sync(0xffffffffu, row_ok ? j0_row : 1 << 20);
  const int whi = __reduce_max_sync(0xffffffffu, j1_row);
  bool chunk_any[4], chunk_all[4];  // the warp's 32-column chunks: reached by some row / wholly inside every row's
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    chunk_any[c] = 32 * c < kc && 32 * c < whi && 32 * c + 32 > wlo;
    chunk_all[c] = __all_sync(0xffffffffu, row_ok && j0_row <= 32 * c && 32 * c + 32 <= j1_row);
  }
  const float sl2 = scale * 1.4426950408889634f;  // exp(s scale - m) = 2^(s sl2 - m log2 e)

  auto coords = [&](int li, int& hb, int& h0) {
    short_tile_coords(geo, static_cast<int>(blockIdx.x) + li * static_cast<int>(gridDim.x), hb, h0);
  };
  auto load_qk = [&](int li) {
    int hb, h0;
    coords(li, hb, h0);
    mbar_arrive_expect_tx(&qk_full, 2u * (D / 64) * box_bytes);
    for (int hh = 0; hh < D / 64; ++hh) {
      tma_load_4d(sq + hh * kHalfBytes, &tq, &qk_full, hh * 64, 0, h0, hb);
      tma_load_4d(sk + hh * kHalfBytes, &tk, &qk_full, hh * 64, 0, h0, hb);
    }
  };
  auto load_v = [&](int li) {
    int hb, h0;
    coords(li, hb, h0);
    mbar_arrive_expect_tx(&v_full, (D / 64) * box_bytes);
    for (int hh = 0; hh < D / 64; ++hh) tma_load_4d(sv + hh * kHalfBytes, &tv, &v_full, hh * 64, 0, h0, hb);
  };
  if (leader && n_local > 0) {
    tma_prefetch_desc(&tq), tma_prefetch_desc(&tk), tma_prefetch_desc(&tv), tma_prefetch_desc(&to);
    load_qk(0);
    load_v(0);
  }

  bool ok = true;
  for (int li = 0; li < n_local && ok; ++li) {
    int hb, h0;
    coords(li, hb, h0);
    const uint32_t par = static_cast<uint32_t>(li) & 1u;
    // ---- S = Q K^T
    if (leader) {
      ok = mbar_wait_or_abort(&qk_full, par, 441, abort);
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          mma_ss(tmem, desc_kmajor(sq, kk), desc_kmajor(sk, kk), id_s, kk > 0 ? 1u : 0u);
        mma_commit(&s_full);
      }
    }
    ok = __all_sync(0xffffffffu, ok && mbar_wait_or_abort(&s_full, par, 444, abort));
    if (!ok) break;
    tc_fence_after();
    // Q and K are spent: the next tile's Q and K go in now.
    if (leader && li + 1 < n_local) load_qk(li + 1);
    int j0, j1;  // re-read per tile through an opaque move: keeps per-column masks from being hoisted and held
    asm volatile("mov.b32 %0, %1;" : "=r"(j0) : "r"(j0_row));
    asm volatile("mov.b32 %0, %1;" : "=r"(j1) : "r"(j1_row));
    // ---- pass 1: row max of y = s scale log2(e) (any sign of scale), one chunk per tensor-memory round trip
    float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      if (!chunk_any[cc]) continue;
      uint32_t x[32];
      tmem_ld32(tS + 32 * cc, x);
      tmem_wait_ld_regs(x);
      if (chunk_all[cc]) {
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          mx[0] = fmax3(mx[0], __uint_as_float(x[e]) * sl2, __uint_as_float(x[e + 1]) * sl2);
          mx[1] = fmax3(mx[1], __uint_as_float(x[e + 2]) * sl2, __uint_as_float(x[e + 3]) * sl2);
          mx[2] = fmax3(mx[2], __uint_as_float(x[e + 4]) * sl2, __uint_as_float(x[e + 5]) * sl2);
          mx[3] = fmax3(mx[3], __uint_as_float(x[e + 6]) * sl2, __uint_as_float(x[e + 7]) * sl2);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const bool in = 32 * cc + e >= j0 && 32 * cc + e < j1;
          mx[e & 3] = in ? fmaxf(mx[e & 3], __uint_as_float(x[e]) * sl2) : mx[e & 3];
        }
      }
      asm volatile("" : "+f"(mx[0]), "+f"(mx[1]), "+f"(mx[2]), "+f"(mx[3]));  // finish this chunk first
    }
    const float m2 = row_ok ? fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) : 0.f;  // max of y
    // ---- pass 2: P = 2^(y - m2) as fp16 pairs: keys [32 c, 32 c + 32) into columns [16 c, 16 c + 16), which hold
    // scores that are already read (chunk c writes over chunk c / 2)
    float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      if (32 * cc >= kc) continue;
      uint32_t pk[16];
      if (!chunk_any[cc]) {
#pragma unroll
        for (int e = 0; e < 16; ++e) pk[e] = 0u;
      } else {
        uint32_t x[32];
        tmem_ld32(tS + 32 * cc, x);
        tmem_wait_ld_regs(x);
        if (chunk_all[cc]) {
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const float p0 = exp2_approx(fmaf(__uint_as_float(x[e]), sl2, -m2));
            const float p1 = exp2_approx(fmaf(__uint_as_float(x[e + 1]), sl2, -m2));
            ls[(e >> 1) & 3] += p0 + p1;
            pk[e >> 1] = pack_f16(p0, p1);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const bool in0 = 32 * cc + e >= j0 && 32 * cc + e < j1;
            const bool in1 = 32 * cc + e + 1 >= j0 && 32 * cc + e + 1 < j1;
            const float p0 = in0 ? exp2_approx(fmaf(__uint_as_float(x[e]), sl2, -m2)) : 0.f;
            const float p1 = in1 ? exp2_approx(fmaf(__uint_as_float(x[e + 1]), sl2, -m2)) : 0.f;
            ls[(e >> 1) & 3] += p0 + p1;
            pk[e >> 1] = pack_f16(p0, p1);
          }
        }
      }
      tmem_st16(tS + 16 * cc, pk);
    }
    const float l = (ls[0] + ls[1]) + (ls[2] + ls[3]);
    tmem_wait_st();
    tc_fence_before();
    // ---- V to fp16 times 2^e, in place (bf16 inputs; fp16 inputs are used as they are)
    ok = __all_sync(0xffffffffu, ok && mbar_wait_or_abort(&v_full, par, 443, abort));
    if (!ok) break;
    float vscale_inv = 1.f;
    if (kB) {
      // max |v| over the tile (16-bit magnitudes order like their bit patterns)
      uint32_t vm = 0;
      if (row_ok) {
#pragma unroll
        for (int c = 0; c < D / 8; ++c) {
          const uint4 u = *reinterpret_cast<const uint4*>(sv + (c >> 3) * kHalfBytes + sw128_off(r, c & 7));
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) vm = max(vm, max(w[q] & 0x7FFFu, (w[q] >> 16) & 0x7FFFu));
        }
      }
      vm = __reduce_max_sync(0xffffffffu, vm);
      if (lane == 0) vmax_slot[warp] = vm;
      __syncthreads();
      const uint32_t vmax = max(max(vmax_slot[0], vmax_slot[1]), max(vmax_slot[2], vmax_slot[3]));
      int e = 14 - (static_cast<int>(vmax >> 7) - 127);  // bf16 exponent of the largest |v|
      e = max(-100, min(100, e));
      const float vs = exp2f(static_cast<float>(e));
      vscale_inv = exp2f(static_cast<float>(-e));
      if (row_ok) {
#pragma unroll
        for (int c = 0; c < D / 8; ++c) {
          uint4* a = reinterpret_cast<uint4*>(sv + (c >> 3) * kHalfBytes + sw128_off(r, c & 7));
          const uint4 u = *a;
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
          uint32_t h[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) h[q] = pack_f16(unpack_lo<T>(w[q]) * vs, unpack_hi<T>(w[q]) * vs);
          *a = make_uint4(h[0], h[1], h[2], h[3]);
        }
      }
      fence_proxy_async_smem();
    }
    __syncthreads();  // P stored by every thread; V converted
    // ---- O = P V
    if (leader) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        if (kk < kc / 16) mma_ts(tmem + 64, tmem + kk * 8, desc_mnmajor(sv, kk), kIdPV, kk > 0 ? 1u : 0u);
      mma_commit(&o_full);
    }
    ok = __all_sync(0xffffffffu, ok && mbar_wait_or_abort(&o_full, par, 445, abort));
    if (!ok) break;
    tc_fence_after();
    // ---- epilogue: O 2^-e / l over the spent V, rows >= `rows` as zeros; lse
    const float inv = (row_ok && l > 0.f) ? vscale_inv / l : 0.f;
    int rt;  // the row, re-read here so the staging addresses are formed here
    asm volatile("mov.b32 %0, %1;" : "=r"(rt) : "r"(r));
#pragma unroll
    for (int c = 0; c < D; c += 32) {
      uint32_t v[32];
      tmem_ld32(tO + c, v);
      tmem_wait_ld_regs(v);
      unsigned char* half = sv + (c >> 6) * kHalfBytes;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 u = make_uint4(0u, 0u, 0u, 0u);
        if (row_ok) {
          u.x = pack2<T>(__uint_as_float(v[8 * q + 0]) * inv, __uint_as_float(v[8 * q + 1]) * inv);
          u.y = pack2<T>(__uint_as_float(v[8 * q + 2]) * inv, __uint_as_float(v[8 * q + 3]) * inv);
          u.z = pack2<T>(__uint_as_float(v[8 * q + 4]) * inv, __uint_as_float(v[8 * q + 5]) * inv);
          u.w = pack2<T>(__uint_as_float(v[8 * q + 6]) * inv, __uint_as_float(v[8 * q + 7]) * inv);
        }
        *reinterpret_cast<uint4*>(half + sw128_off(rt, ((c & 63) >> 3) + q)) = u;
      }
    }
    if (row_ok && h0 + r / N < geo.hs) {
      const int64_t slice = static_cast<int64_t>(hb) * geo.hs + h0 + r / N;
      lse[slice * N + (r - j0_row)] = m2 * 0.6931471805599453f + logf(l);  // natural units: ln 2 * max of y
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (leader) {
      for (int hh = 0; hh < D / 64; ++hh) tma_store_4d(&to, sv + hh * kHalfBytes, hh * 64, 0, h0, hb);
      tma_store_commit();
      tma_store_wait_read();  // V's buffer is free again
      if (li + 1 < n_local) load_v(li + 1);
    }
  }
  if (leader) tma_store_wait_all();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, L::kTmemCols);
}

// ================================================================================================ backward

template <int D>
struct BwdShortLayout {
  static constexpr uint32_t kOp = (D / 64) * kHalfBytes;  // one [128 x D] 16-bit tile
  // Q, K, V, dO; then P over the spent V (its first 64-key half; the second half has its own buffer at D = 64) and
  // dS in its own [128 x 128] tile.
  static constexpr uint32_t kQ = 0, kK = kOp, kV = 2 * kOp, kDO = 3 * kOp;
  static constexpr uint32_t kP1 = 4 * kOp;                              // P keys [64, 128) (D = 64 only)
  static constexpr uint32_t kDS = D == 64 ? kP1 + kHalfBytes : 4 * kOp;
  static constexpr uint32_t kBytes = kDS + 2 * kHalfBytes;
  // The barriers live after the tiles and there is no static shared memory, so the dynamic block starts on the
  // CTA's shared-memory base (1024-byte aligned; checked at run time) and needs no alignment slack: two CTAs of
  // 112 KiB + 64 B then fit one SM's 228 KiB.
  static constexpr uint32_t kSmem = kBytes + 64;
  static constexpr uint32_t kTmemCols = D == 64 ? 256 : 512;
  // S [0, 128), dP [128, 256); then dV [0, D), dK [D, 2 D), dQ [2 D, 3 D) over them.
  static constexpr uint32_t cS = 0, cDP = 128, cDV = 0, cDK = D, cDQ = 2 * D;
  static constexpr int kCtasPerSm = D == 64 ? 2 : 1;
  static constexpr int kThreads = 128;
};

// Backward for N <= 128 (packed tiles as in the forward), persistent; kCtasPerSm CTAs share an SM so that one tile's
// loads and products overlap another's pointwise work. Thread r owns row r of the tile: query row r for S, dP and dQ,
// key row r for dK and dV; thread 0 also issues the TMA loads and the tcgen05 products. Per tile:
//   S = Q K^T and dP = dO V^T into tensor memory; meanwhile each thread reads lse and D = <dO, O> of its row (O, the
//   stored forward output, from global memory);
//   P = exp(s scale - lse) (0 outside the row's slice) and dS = P (dP - D), rounded to the input type, written as
//   [query x key] tiles to shared memory (P over the spent V);
//   dV = P^T dO, dK = dS^T Q, dQ = dS K into tensor memory over the spent S and dP; once they are done the next tile's
//   inputs are loaded, and the three gradients (dK and dQ times scale) are rounded into the spent dS and P tiles and
//   written with TMA stores at D = 64, or go to global memory row by row at D = 128.
// The reference's SINGLE mode (models/fused_attn/triton_kernels.py:250-264, :742-768): D from the stored O
// (reference.py:44-45), P and dS rounded to the input type before their products (:576-586).
template <typename T, int D>
__global__ void __launch_bounds__(128, D == 64 ? 2 : 1)
    tc_bwd_short_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                        const __grid_constant__ CUtensorMap tdq, const __grid_constant__ CUtensorMap tdk,
                        const __grid_constant__ CUtensorMap tdv, const T* __restrict__ o,
                        const float* __restrict__ lse, T* __restrict__ dq, T* __restrict__ dk, T* __restrict__ dv,
                        const ShortGeom geo, float scale) {
  using L = BwdShortLayout<D>;
  extern __shared__ __align__(1024) unsigned char smem[];
  unsigned char* sQ = smem + L::kQ;
  unsigned char* sK = smem + L::kK;
  unsigned char* sV = smem + L::kV;
  unsigned char* sDO = smem + L::kDO;
  unsigned char* sDS = smem + L::kDS;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBytes);
  uint64_t& in_full = bars[0];
  uint64_t& s_full = bars[1];
  uint64_t& g_full = bars[2];
  uint32_t& tmem_slot = *reinterpret_cast<uint32_t*>(smem + L::kBytes + 24);
  int& abort_flag = *reinterpret_cast<int*>(smem + L::kBytes + 28);
  if (smem_u32(smem) & 1023u) {  // the swizzled tiles need a 1024-byte-aligned base
    if (threadIdx.x == 0) atomicExch(&g_device_error, 460);
    return;
  }

  const int tid = threadIdx.x, warp = tid >> 5;
  const int N = geo.N, rows = geo.per * geo.N;
  const int kc = (rows + 31) & ~31;   // key columns computed (S / dP N; the dQ product's K)
  const int kr = (rows + 15) & ~15;   // query rows reduced over (the dV / dK products' K)
  constexpr bool kB = is_bf16<T>();
  const uint32_t id_nn = idesc_f16(kB, 0, 0, 128, kc);      // S, dP
  constexpr uint32_t kIdKM = idesc_f16(kB, 0, 1, 128, D);   // dQ = dS K
  constexpr uint32_t kIdMM = idesc_f16(kB, 1, 1, 128, D);   // dK = dS^T Q, dV = P^T dO
  const int n_local = geo.tiles > static_cast<int>(blockIdx.x)
                          ? (geo.tiles - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                          : 0;
  const uint32_t box_bytes = 128u * static_cast<uint32_t>(rows);
  // P's two 64-key halves: the spent V (and at D = 64 its own buffer for the second half).
  auto p_half = [&](int hh) -> unsigned char* { return (D == 64 && hh == 1) ? smem + L::kP1 : sV + hh * kHalfBytes; };

  for (uint32_t i = tid * 16u; i < L::kBytes; i += L::kThreads * 16u)
    *reinterpret_cast<uint4*>(smem + i) = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async_smem();
  if (tid == 0) {
    mbar_init(&in_full, 1);
    mbar_init(&s_full, 1);
    mbar_init(&g_full, 1);
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
  const bool leader = tid == 0;
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  const int r = tid;
  const bool row_ok = r < rows;
  const int j0_row = row_ok ? (r / N) * N : 0;
  const int j1_row = row_ok ? j0_row + N : 0;

  auto coords = [&](int li, int& hb, int& h0) {
    short_tile_coords(geo, static_cast<int>(blockIdx.x) + li * static_cast<int>(gridDim.x), hb, h0);
  };
  auto load = [&](int li) {
    int hb, h0;
    coords(li, hb, h0);
    mbar_arrive_expect_tx(&in_full, 4u * (D / 64) * box_bytes);
    for (int hh = 0; hh < D / 64; ++hh) {
      tma_load_4d(sQ + hh * kHalfBytes, &tq, &in_full, hh * 64, 0, h0, hb);
      tma_load_4d(sK + hh * kHalfBytes, &tk, &in_full, hh * 64, 0, h0, hb);
      tma_load_4d(sV + hh * kHalfBytes, &tv, &in_full, hh * 64, 0, h0, hb);
      tma_load_4d(sDO + hh * kHalfBytes, &tdo, &in_full, hh * 64, 0, h0, hb);
    }
  };
  if (leader && n_local > 0) {
    tma_prefetch_desc(&tq), tma_prefetch_desc(&tk), tma_prefetch_desc(&tv), tma_prefetch_desc(&tdo);
    load(0);
  }

  constexpr bool kStaged = D == 64;  // gradients leave through TMA stores from the spent dS and P tiles
  bool ok = true;
  for (int li = 0; li < n_local && ok; ++li) {
    int hb, h0;
    coords(li, hb, h0);
    const uint32_t par = static_cast<uint32_t>(li) & 1u;
    const bool mine = row_ok && h0 + r / N < geo.hs;  // this row is a real row of a real slice
    const int64_t grow = mine ? (static_cast<int64_t>(hb) * geo.hs + h0 + r / N) * N + (r - j0_row) : 0;
    // Row statistics while the inputs land and the products run: lse, and O's row for D = <dO, O>.
    const float Li = mine ? lse[grow] : 0.f;
    uint4 orow[D / 8];
#pragma unroll
    for (int c = 0; c < D / 8; ++c)
      orow[c] = mine ? *reinterpret_cast<const uint4*>(o + grow * D + 8 * c) : make_uint4(0u, 0u, 0u, 0u);
    if (leader) {
      ok = mbar_wait_or_abort(&in_full, par, 451, abort);
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          mma_ss(tmem + L::cS, desc_kmajor(sQ, kk), desc_kmajor(sK, kk), id_nn, kk > 0 ? 1u : 0u);
          mma_ss(tmem + L::cDP, desc_kmajor(sDO, kk), desc_kmajor(sV, kk), id_nn, kk > 0 ? 1u : 0u);
        }
        mma_commit(&s_full);
      }
    }
    ok = __all_sync(0xffffffffu, ok && mbar_wait_or_abort(&in_full, par, 452, abort));
    if (!ok) break;
    float Di = 0.f;
#pragma unroll
    for (int c = 0; c < D / 8; ++c) {
      float x[8];
      ld_row8<T>(sDO, r, c, x);
      const uint32_t w[4] = {orow[c].x, orow[c].y, orow[c].z, orow[c].w};
#pragma unroll
      for (int q = 0; q < 4; ++q) Di += x[2 * q] * unpack_lo<T>(w[q]) + x[2 * q + 1] * unpack_hi<T>(w[q]);
    }
    ok = __all_sync(0xffffffffu, ok && mbar_wait_or_abort(&s_full, par, 453, abort));
    if (!ok) break;
    if (kStaged && li > 0) {  // the previous tile's gradient stores must have read the dS and P tiles
      if (leader) tma_store_wait_read();
      __syncthreads();
    }
    tc_fence_after();
    int j0, j1;  // re-read per tile through an opaque move: keeps per-column masks from being hoisted and held
    asm volatile("mov.b32 %0, %1;" : "=r"(j0) : "r"(j0_row));
    asm volatile("mov.b32 %0, %1;" : "=r"(j1) : "r"(j1_row));
    // P and dS, 32 key columns at a time, as 16-bit [query x key] tiles (every row written: zeros where masked).
#pragma unroll
    for (int c = 0; c < 128; c += 32) {
      uint32_t pk[16], dk16[16];
      if (c < kc) {
        uint32_t rs[32], rp[32];
        tmem_ld32(tmem + L::cS + lane_off + c, rs);
        tmem_ld32(tmem + L::cDP + lane_off + c, rp);
        tmem_wait_ld_regs(rs);
        tmem_wait_ld_regs(rp);
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float pp[2], ds[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const bool in = c + e + u >= j0 && c + e + u < j1;
            pp[u] = in ? exp_nat(fmaf(__uint_as_float(rs[e + u]), scale, -Li)) : 0.f;
            ds[u] = pp[u] * (__uint_as_float(rp[e + u]) - Di);
          }
          pk[e >> 1] = pack2<T>(pp[0], pp[1]);
          dk16[e >> 1] = pack2<T>(ds[0], ds[1]);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) pk[e] = dk16[e] = 0u;
      }
      unsigned char* ph = p_half(c >> 6);
      unsigned char* dh = sDS + (c >> 6) * kHalfBytes;
      const int c0 = (c & 63) >> 3;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        *reinterpret_cast<uint4*>(ph + sw128_off(r, c0 + q)) = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2],
                                                                           pk[4 * q + 3]);
        *reinterpret_cast<uint4*>(dh + sw128_off(r, c0 + q)) = make_uint4(dk16[4 * q], dk16[4 * q + 1],
                                                                           dk16[4 * q + 2], dk16[4 * q + 3]);
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (leader) {
      tc_fence_after();
      // dV = P^T dO and dK = dS^T Q (M = keys, K = queries), dQ = dS K (M = queries, K = keys).
      for (int kk = 0; kk < kr / 16; ++kk) {
        const uint32_t acc = kk > 0 ? 1u : 0u;
        const uint32_t pa = smem_u32(p_half(0)) + kk * 2048u;  // P read MN-major: M = keys, K-step kk = queries
        const uint64_t pdesc = sw128_desc(pa, D == 64 ? (smem_u32(p_half(1)) - smem_u32(p_half(0))) : kHalfBytes,
                                          1024u);
        mma_ss(tmem + L::cDV, pdesc, desc_mnmajor(sDO, kk), kIdMM, acc);
        mma_ss(tmem + L::cDK, desc_mnmajor(sDS, kk), desc_mnmajor(sQ, kk), kIdMM, acc);
      }
      for (int kk = 0; kk < kc / 16; ++kk)
        mma_ss(tmem + L::cDQ, desc_kmajor(sDS, kk), desc_mnmajor(sK, kk), kIdKM, kk > 0 ? 1u : 0u);
      mma_commit(&g_full);
    }
    ok = __all_sync(0xffffffffu, ok && mbar_wait_or_abort(&g_full, par, 454, abort));
    if (!ok) break;
    tc_fence_after();
    if (leader && li + 1 < n_local) load(li + 1);  // every input buffer is spent
    if constexpr (kStaged) {
      // Gradients rounded into the spent tiles (dQ, dK over the two dS halves, dV over P's second half), rows
      // >= `rows` as zeros, then one TMA store each: key row r of dK and dV, query row r of dQ.
      int rt;  // the row, re-read here so the staging addresses are formed here
      asm volatile("mov.b32 %0, %1;" : "=r"(rt) : "r"(r));
      unsigned char* const dst[3] = {sDS, sDS + kHalfBytes, smem + L::kP1};
      const uint32_t col[3] = {L::cDQ, L::cDK, L::cDV};
      const float mul[3] = {scale, scale, 1.f};
#pragma unroll
      for (int g = 0; g < 3; ++g) {
#pragma unroll
        for (int c = 0; c < 64; c += 32) {
          uint32_t v[32];
          tmem_ld32(tmem + col[g] + lane_off + c, v);
          tmem_wait_ld_regs(v);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 u = make_uint4(0u, 0u, 0u, 0u);
            if (row_ok) {
              u.x = pack2<T>(__uint_as_float(v[8 * q + 0]) * mul[g], __uint_as_float(v[8 * q + 1]) * mul[g]);
              u.y = pack2<T>(__uint_as_float(v[8 * q + 2]) * mul[g], __uint_as_float(v[8 * q + 3]) * mul[g]);
              u.z = pack2<T>(__uint_as_float(v[8 * q + 4]) * mul[g], __uint_as_float(v[8 * q + 5]) * mul[g]);
              u.w = pack2<T>(__uint_as_float(v[8 * q + 6]) * mul[g], __uint_as_float(v[8 * q + 7]) * mul[g]);
            }
            *reinterpret_cast<uint4*>(dst[g] + sw128_off(rt, (c >> 3) + q)) = u;
          }
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncthreads();  // staged, and tensor memory read out before the next tile's products overwrite it
      if (leader) {
        tma_store_4d(&tdq, dst[0], 0, 0, h0, hb);
        tma_store_4d(&tdk, dst[1], 0, 0, h0, hb);
        tma_store_4d(&tdv, dst[2], 0, 0, h0, hb);
        tma_store_commit();
      }
    } else {
      // Gradients to global memory: key row r of dK and dV, query row r of dQ.
      store_row_from_tmem<T, D>(tmem + L::cDV + lane_off, 1.f, mine ? dv + grow * D : nullptr);
      store_row_from_tmem<T, D>(tmem + L::cDK + lane_off, scale, mine ? dk + grow * D : nullptr);
      store_row_from_tmem<T, D>(tmem + L::cDQ + lane_off, scale, mine ? dq + grow * D : nullptr);
      tc_fence_before();
      __syncthreads();  // tensor memory read out before the next tile's products overwrite it
    }
  }
  if (kStaged && leader) tma_store_wait_all();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, L::kTmemCols);
}

// ================================================================================================ double backward

struct BobShortLayout {  // D = 64
  static constexpr uint32_t kOp = kHalfBytes;
  static constexpr uint32_t kQ = 0, kK = kOp, kV = 2 * kOp, kDO = 3 * kOp, kGQ = 4 * kOp, kGK = 5 * kOp,
                            kGV = 6 * kOp;
  static constexpr uint32_t kGS = 7 * kOp, kDS = kGS + 2 * kHalfBytes, kA = kDS + 2 * kHalfBytes;
  static constexpr uint32_t kBytes = kA + 2 * kHalfBytes;  // 7 * 16 KiB + 3 * 32 KiB = 208 KiB
  static constexpr uint32_t kSmem = kBytes + 64;           // barriers after the tiles; no static shared memory
  static constexpr uint32_t kTmemCols = 512;
  // Scores: S [0,128), dP [128,256), G [256,384), R [384,512). Outputs: packed 16-bit P in [0,64) (over S, once read),
  // hQ [256,320), hdO [320,384), hK [384,448), hV [448,512).
  static constexpr uint32_t cS = 0, cDP = 128, cG = 256, cR = 384;
  static constexpr uint32_t cP16 = 0, cHQ = 256, cHDO = 320, cHK = 384, cHV = 448;
};

// Double backward for N <= 128 at D = 64 (packed tiles as in the forward), persistent, one CTA per SM (its four
// score products fill the SM's tensor memory). Per tile, the closed form of reference.py:61-91:
//   S = Q K^T, dP = dO V^T, G = scale (gQ K^T + Q gK^T), R = dO gV^T           (tcgen05, tensor memory)
//   per query row (masked to its slice): D = <dO, O>, e = sum P G, t = sum P gp with gp = (dP - D) G - e dP + R;
//   then P, dS = P (dP - D), A = P (G - e), gS = P (gp - t) rounded to the input type (gS, dS, A to shared memory,
//   P to tensor memory);
//   hQ = scale (gS K + dS gK), hdO = A V + P gV, hK = scale (gS^T Q + dS^T gQ), hV = A^T dO
// Once the second products are done the next tile's inputs are loaded, while the outputs are rounded into the spent
// gS and dS tiles and leave through TMA stores. A zero cotangent (bit 0 gq, 1 gk, 2 gv of zero_mask) is never
// loaded: its tile stays cleared. The reference's Triton kernels do this as a SINGLE column pass
// (models/fused_attn/triton_kernels.py:448-551, :878-909).
template <typename T>
__global__ void __launch_bounds__(128, 1)
    tc_bob_short_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                        const __grid_constant__ CUtensorMap tgq, const __grid_constant__ CUtensorMap tgk,
                        const __grid_constant__ CUtensorMap tgv, const __grid_constant__ CUtensorMap thq,
                        const __grid_constant__ CUtensorMap thk, const __grid_constant__ CUtensorMap thv,
                        const __grid_constant__ CUtensorMap thdo, const T* __restrict__ o,
                        const float* __restrict__ lse, const ShortGeom geo, float scale, uint32_t zero_mask) {
  constexpr int D = 64;
  using L = BobShortLayout;
  extern __shared__ __align__(1024) unsigned char smem[];
  unsigned char* sQ = smem + L::kQ;
  unsigned char* sK = smem + L::kK;
  unsigned char* sV = smem + L::kV;
  unsigned char* sDO = smem + L::kDO;
  unsigned char* sGQ = smem + L::kGQ;
  unsigned char* sGK = smem + L::kGK;
  unsigned char* sGV = smem + L::kGV;
  unsigned char* sGS = smem + L::kGS;
  unsigned char* sDS = smem + L::kDS;
  unsigned char* sA = smem + L::kA;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBytes);
  uint64_t& in_full = bars[0];
  uint64_t& s_full = bars[1];
  uint64_t& g_full = bars[2];
  uint32_t& tmem_slot = *reinterpret_cast<uint32_t*>(smem + L::kBytes + 24);
  int& abort_flag = *reinterpret_cast<int*>(smem + L::kBytes + 28);
  if (smem_u32(smem) & 1023u) {  // the swizzled tiles need a 1024-byte-aligned base
    if (threadIdx.x == 0) atomicExch(&g_device_error, 470);
    return;
  }

  const int tid = threadIdx.x, warp = tid >> 5;
  const int N = geo.N, rows = geo.per * geo.N;
  const int kc = (rows + 31) & ~31;  // key columns of the score products (and K of the key-side sums)
  const int kr = (rows + 15) & ~15;  // query rows reduced over (K of hK, hV)
  constexpr bool kB = is_bf16<T>();
  const uint32_t id_nn = idesc_f16(kB, 0, 0, 128, kc);
  constexpr uint32_t kIdKM = idesc_f16(kB, 0, 1, 128, D);
  constexpr uint32_t kIdMM = idesc_f16(kB, 1, 1, 128, D);
  const int n_local = geo.tiles > static_cast<int>(blockIdx.x)
                          ? (geo.tiles - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                          : 0;
  const uint32_t box_bytes = 128u * static_cast<uint32_t>(rows);
  const uint32_t n_loaded = 7u - static_cast<uint32_t>(__popc(zero_mask & 7u));

  for (uint32_t i = tid * 16u; i < L::kBytes; i += 128u * 16u)
    *reinterpret_cast<uint4*>(smem + i) = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async_smem();
  if (tid == 0) {
    mbar_init(&in_full, 1);
    mbar_init(&s_full, 1);
    mbar_init(&g_full, 1);
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
  const bool leader = tid == 0;
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  const int r = tid;
  const bool row_ok = r < rows;
  const int j0_row = row_ok ? (r / N) * N : 0;
  const int j1_row = row_ok ? j0_row + N : 0;

  auto coords = [&](int li, int& hb, int& h0) {
    short_tile_coords(geo, static_cast<int>(blockIdx.x) + li * static_cast<int>(gridDim.x), hb, h0);
  };
  auto load = [&](int li) {
    int hb, h0;
    coords(li, hb, h0);
    mbar_arrive_expect_tx(&in_full, n_loaded * box_bytes);
    tma_load_4d(sQ, &tq, &in_full, 0, 0, h0, hb);
    tma_load_4d(sK, &tk, &in_full, 0, 0, h0, hb);
    tma_load_4d(sV, &tv, &in_full, 0, 0, h0, hb);
    tma_load_4d(sDO, &tdo, &in_full, 0, 0, h0, hb);
    if (!(zero_mask & 1u)) tma_load_4d(sGQ, &tgq, &in_full, 0, 0, h0, hb);
    if (!(zero_mask & 2u)) tma_load_4d(sGK, &tgk, &in_full, 0, 0, h0, hb);
    if (!(zero_mask & 4u)) tma_load_4d(sGV, &tgv, &in_full, 0, 0, h0, hb);
  };
  if (leader && n_local > 0) load(0);

  bool ok = true;
  for (int li = 0; li < n_local && ok; ++li) {
    int hb, h0;
    coords(li, hb, h0);
    const uint32_t par = static_cast<uint32_t>(li) & 1u;
    const bool mine = row_ok && h0 + r / N < geo.hs;
    const int64_t grow = mine ? (static_cast<int64_t>(hb) * geo.hs + h0 + r / N) * N + (r - j0_row) : 0;
    const float Li = mine ? lse[grow] : 0.f;
    uint4 orow[D / 8];
#pragma unroll
    for (int c = 0; c < D / 8; ++c)
      orow[c] = mine ? *reinterpret_cast<const uint4*>(o + grow * D + 8 * c) : make_uint4(0u, 0u, 0u, 0u);
    if (leader) {
      ok = mbar_wait_or_abort(&in_full, par, 471, abort);
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t acc = kk > 0 ? 1u : 0u;
          mma_ss(tmem + L::cS, desc_kmajor(sQ, kk), desc_kmajor(sK, kk), id_nn, acc);
          mma_ss(tmem + L::cDP, desc_kmajor(sDO, kk), desc_kmajor(sV, kk), id_nn, acc);
          mma_ss(tmem + L::cG, desc_kmajor(sGQ, kk), desc_kmajor(sK, kk), id_nn, acc);
          mma_ss(tmem + L::cR, desc_kmajor(sDO, kk), desc_kmajor(sGV, kk), id_nn, acc);
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          mma_ss(tmem + L::cG, desc_kmajor(sQ, kk), desc_kmajor(sGK, kk), id_nn, 1u);
        mma_commit(&s_full);
      }
    }
    ok = __all_sync(0xffffffffu, ok && mbar_wait_or_abort(&in_full, par, 472, abort));
    if (!ok) break;
    float Di = 0.f;
#pragma unroll
    for (int c = 0; c < D / 8; ++c) {
      float x[8];
      ld_row8<T>(sDO, r, c, x);
      const uint32_t w[4] = {orow[c].x, orow[c].y, orow[c].z, orow[c].w};
#pragma unroll
      for (int q = 0; q < 4; ++q) Di += x[2 * q] * unpack_lo<T>(w[q]) + x[2 * q + 1] * unpack_hi<T>(w[q]);
    }
    ok = __all_sync(0xffffffffu, ok && mbar_wait_or_abort(&s_full, par, 473, abort));
    if (!ok) break;
    if (li > 0) {  // the previous tile's output stores must have read the gS and dS tiles
      if (leader) tma_store_wait_read();
      __syncthreads();
    }
    tc_fence_after();
    int j0, j1;  // re-read per tile through an opaque move: keeps per-column masks from being hoisted and held
    asm volatile("mov.b32 %0, %1;" : "=r"(j0) : "r"(j0_row));
    asm volatile("mov.b32 %0, %1;" : "=r"(j1) : "r"(j1_row));
    // Pass 1: e = sum P G, and sum P gp = sum dS G - e sum P dP + sum P R.
    float e_ = 0.f, c1 = 0.f, c2 = 0.f, c3 = 0.f;
#pragma unroll
    for (int c = 0; c < 128; c += 32) {
      if (c >= kc) continue;
      uint32_t rs[32], rp[32], rg[32], rr[32];
      tmem_ld32(tmem + L::cS + lane_off + c, rs);
      tmem_ld32(tmem + L::cDP + lane_off + c, rp);
      tmem_ld32(tmem + L::cG + lane_off + c, rg);
      tmem_ld32(tmem + L::cR + lane_off + c, rr);
      tmem_wait_ld_regs(rs);
      tmem_wait_ld_regs(rp);
      tmem_wait_ld_regs(rg);
      tmem_wait_ld_regs(rr);
#pragma unroll
      for (int u = 0; u < 32; ++u) {
        const bool in = c + u >= j0 && c + u < j1;
        const float p = in ? exp_nat(fmaf(__uint_as_float(rs[u]), scale, -Li)) : 0.f;
        const float g = __uint_as_float(rg[u]) * scale;
        const float dp = __uint_as_float(rp[u]);
        e_ += p * g;
        c1 += p * (dp - Di) * g;
        c2 += p * dp;
        c3 += p * __uint_as_float(rr[u]);
      }
    }
    const float t_ = c1 - e_ * c2 + c3;
    // Pass 2: the derived tiles (every row and column written: zeros where masked); P packed to 16 bits into
    // tensor-memory columns [c / 2, c / 2 + 16), over S columns this thread has already read.
#pragma unroll
    for (int c = 0; c < 128; c += 32) {
      uint32_t pk_p[16], pk_gs[16], pk_ds[16], pk_a[16];
      if (c < kc) {
        uint32_t rs[32], rp[32], rg[32], rr[32];
        tmem_ld32(tmem + L::cS + lane_off + c, rs);
        tmem_ld32(tmem + L::cDP + lane_off + c, rp);
        tmem_ld32(tmem + L::cG + lane_off + c, rg);
        tmem_ld32(tmem + L::cR + lane_off + c, rr);
        tmem_wait_ld_regs(rs);
        tmem_wait_ld_regs(rp);
        tmem_wait_ld_regs(rg);
        tmem_wait_ld_regs(rr);
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float pv[2], gs[2], ds[2], a[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const bool in = c + e + u >= j0 && c + e + u < j1;
            const float pp = in ? exp_nat(fmaf(__uint_as_float(rs[e + u]), scale, -Li)) : 0.f;
            const float g = __uint_as_float(rg[e + u]) * scale;
            const float dp = __uint_as_float(rp[e + u]);
            const float gp = (dp - Di) * g - e_ * dp + __uint_as_float(rr[e + u]);
            pv[u] = pp;
            ds[u] = pp * (dp - Di);
            a[u] = pp * (g - e_);
            gs[u] = pp * (gp - t_);
          }
          pk_p[e >> 1] = pack2<T>(pv[0], pv[1]);
          pk_gs[e >> 1] = pack2<T>(gs[0], gs[1]);
          pk_ds[e >> 1] = pack2<T>(ds[0], ds[1]);
          pk_a[e >> 1] = pack2<T>(a[0], a[1]);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) pk_p[e] = pk_gs[e] = pk_ds[e] = pk_a[e] = 0u;
      }
      st_row32(sGS, r, c, pk_gs);
      st_row32(sDS, r, c, pk_ds);
      st_row32(sA, r, c, pk_a);
      uint32_t lo[8], hi[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        lo[i] = pk_p[i];
        hi[i] = pk_p[8 + i];
      }
      tmem_st8(tmem + L::cP16 + lane_off + (c >> 1), lo);
      tmem_st8(tmem + L::cP16 + lane_off + (c >> 1) + 8, hi);
    }
    tmem_wait_st();
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (leader) {
      tc_fence_after();
      for (int kk = 0; kk < kc / 16; ++kk) {  // K = keys
        const uint32_t acc = kk > 0 ? 1u : 0u;
        mma_ss(tmem + L::cHQ, desc_kmajor(sGS, kk), desc_mnmajor(sK, kk), kIdKM, acc);
        mma_ss(tmem + L::cHQ, desc_kmajor(sDS, kk), desc_mnmajor(sGK, kk), kIdKM, 1u);
        mma_ss(tmem + L::cHDO, desc_kmajor(sA, kk), desc_mnmajor(sV, kk), kIdKM, acc);
        mma_ts(tmem + L::cHDO, tmem + L::cP16 + kk * 8, desc_mnmajor(sGV, kk), kIdKM, 1u);
      }
      for (int kk = 0; kk < kr / 16; ++kk) {  // K = queries
        const uint32_t acc = kk > 0 ? 1u : 0u;
        mma_ss(tmem + L::cHK, desc_mnmajor(sGS, kk), desc_mnmajor(sQ, kk), kIdMM, acc);
        mma_ss(tmem + L::cHK, desc_mnmajor(sDS, kk), desc_mnmajor(sGQ, kk), kIdMM, 1u);
        mma_ss(tmem + L::cHV, desc_mnmajor(sA, kk), desc_mnmajor(sDO, kk), kIdMM, acc);
      }
      mma_commit(&g_full);
    }
    ok = __all_sync(0xffffffffu, ok && mbar_wait_or_abort(&g_full, par, 474, abort));
    if (!ok) break;
    tc_fence_after();
    if (leader && li + 1 < n_local) load(li + 1);  // every input tile is spent
    // Outputs rounded into the spent gS (hQ, hdO) and dS (hK, hV) tiles, rows >= `rows` as zeros; TMA stores.
    int rt;  // the row, re-read here so the staging addresses are formed here
    asm volatile("mov.b32 %0, %1;" : "=r"(rt) : "r"(r));
    unsigned char* const dst[4] = {sGS, sGS + kHalfBytes, sDS, sDS + kHalfBytes};
    const uint32_t col[4] = {L::cHQ, L::cHDO, L::cHK, L::cHV};
    const float mul[4] = {scale, 1.f, scale, 1.f};
#pragma unroll
    for (int g = 0; g < 4; ++g) {
#pragma unroll
      for (int c = 0; c < 64; c += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + col[g] + lane_off + c, v);
        tmem_wait_ld_regs(v);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 u = make_uint4(0u, 0u, 0u, 0u);
          if (row_ok) {
            u.x = pack2<T>(__uint_as_float(v[8 * q + 0]) * mul[g], __uint_as_float(v[8 * q + 1]) * mul[g]);
            u.y = pack2<T>(__uint_as_float(v[8 * q + 2]) * mul[g], __uint_as_float(v[8 * q + 3]) * mul[g]);
            u.z = pack2<T>(__uint_as_float(v[8 * q + 4]) * mul[g], __uint_as_float(v[8 * q + 5]) * mul[g]);
            u.w = pack2<T>(__uint_as_float(v[8 * q + 6]) * mul[g], __uint_as_float(v[8 * q + 7]) * mul[g]);
          }
          *reinterpret_cast<uint4*>(dst[g] + sw128_off(rt, (c >> 3) + q)) = u;
        }
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();  // staged, and tensor memory read out before the next tile's products overwrite it
    if (leader) {
      tma_store_4d(&thq, dst[0], 0, 0, h0, hb);
      tma_store_4d(&thdo, dst[1], 0, 0, h0, hb);
      tma_store_4d(&thk, dst[2], 0, 0, h0, hb);
      tma_store_4d(&thv, dst[3], 0, 0, h0, hb);
      tma_store_commit();
    }
  }
  if (leader) tma_store_wait_all();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, L::kTmemCols);
}

}  // namespace ebr
