// layers.cuh: the fused pointwise / row kernels on either side of the attention in the energy network (2D-RoPE split
// and merge, residual + rms_norm and its backward, the SwiGLU activation and its backward, the descent step with its
// sphere projection). All are HBM-bound: each reads its inputs once and writes its outputs once, 16 bytes per thread
// access where the pointers and row lengths allow it (V elements of the I/O type), else one element per access.
//
// Rounding follows the reference's eager code operation by operation (multiplies and adds rounded separately with the
// _rn intrinsics, so the compiler does not contract them into fused multiply-adds, and one rounding to the I/O type
// where the eager code converts), so outputs equal the eager ones except where a row sum is taken in another order.
#pragma once

#include "sm100.cuh"

namespace ebr {
namespace layers {

constexpr int kThreads = 256;

// ------------------------------------------------------------------------------------------------ arithmetic

__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ double mul_rn(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ double add_rn(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ float sub_rn(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ double sub_rn(double a, double b) { return __dsub_rn(a, b); }
__device__ __forceinline__ float div_rn(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ double div_rn(double a, double b) { return __ddiv_rn(a, b); }
__device__ __forceinline__ float rsqrt_c(float x) { return rsqrtf(x); }
__device__ __forceinline__ double rsqrt_c(double x) { return rsqrt(x); }
__device__ __forceinline__ float sqrt_c(float x) { return sqrtf(x); }
__device__ __forceinline__ double sqrt_c(double x) { return sqrt(x); }
__device__ __forceinline__ float exp_c(float x) { return expf(x); }
__device__ __forceinline__ double exp_c(double x) { return exp(x); }

// Round a compute-type value to the I/O type and back.
template <typename T>
__device__ __forceinline__ typename Elem<T>::C rnd(typename Elem<T>::C x) {
  return static_cast<typename Elem<T>::C>(Elem<T>::to(x));
}

// V elements of T moved as one access (16 bytes when V * sizeof(T) == 16).
template <typename T, int V>
struct alignas(sizeof(T) * V) Pack {
  T e[V];
};

template <typename T, int V>
__device__ __forceinline__ void load_c(const T* p, typename Elem<T>::C (&out)[V]) {
  const Pack<T, V> pk = *reinterpret_cast<const Pack<T, V>*>(p);
#pragma unroll
  for (int i = 0; i < V; ++i) out[i] = static_cast<typename Elem<T>::C>(pk.e[i]);
}

template <typename T, int V>
__device__ __forceinline__ void store_c(T* p, const typename Elem<T>::C (&in)[V]) {
  Pack<T, V> pk;
#pragma unroll
  for (int i = 0; i < V; ++i) pk.e[i] = Elem<T>::to(in[i]);
  *reinterpret_cast<Pack<T, V>*>(p) = pk;
}

template <int V>
__device__ __forceinline__ void load_table(const float* p, float (&out)[V]) {
#pragma unroll
  for (int i = 0; i < V; ++i) out[i] = __ldg(p + i);
}

template <typename C>
__device__ __forceinline__ C warp_sum(C v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ int64_t grid_stride() { return static_cast<int64_t>(gridDim.x) * blockDim.x; }
__device__ __forceinline__ int64_t global_tid() { return static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; }

// ------------------------------------------------------------------------------------------------ 2D RoPE split

// quarter_swap's source index for element d of a head row of D = 4 Q elements: (a, b, c, d) -> (b, a, d, c).
__device__ __forceinline__ int swap_index(int d, int Q) { return ((d / Q) ^ 1) * Q + (d % Q); }

template <int V>
__device__ __forceinline__ void load_table_v(const float* p, float (&out)[V]) {
  if constexpr (V % 4 == 0) {
#pragma unroll
    for (int i = 0; i < V; i += 4) {
      const float4 t = __ldg(reinterpret_cast<const float4*>(p + i));
      out[i] = t.x;
      out[i + 1] = t.y;
      out[i + 2] = t.z;
      out[i + 3] = t.w;
    }
  } else {
    load_table<V>(p, out);
  }
}

// A token's qkv row is 3 H D / V "slots" of V elements (slot = (part * H + h) * (D / V) + chunk, part 0 / 1 / 2 for
// q / k / v). A block is one token's slots wide (blockDim.x >= slots: each thread keeps one slot for every token it
// visits) and walks tokens blockIdx.x, blockIdx.x + gridDim.x, ...; a warp reads a contiguous stretch of the row.
// Chunks never straddle a quarter of D (Q % V == 0), so a chunk's quarter_swap partner is the contiguous chunk at
// swap_index(d0). The tables are float32 [N, D] rows (16-byte aligned when D % 4 == 0).
struct RopeSlot {
  int part, h, d0;
};

__device__ __forceinline__ RopeSlot rope_slot(int slot, int H, int cpr, int V) {
  const int c = slot % cpr, r = slot / cpr;
  return RopeSlot{r / H, r % H, c * V};
}

template <typename T, int V>
__device__ __forceinline__ void rope_split_one(const T* __restrict__ qkv, int64_t sb, int64_t sn, int64_t b,
                                               int64_t n, int64_t N, int H, int D, RopeSlot sl,
                                               const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                               const float* __restrict__ qscale, T* __restrict__ q,
                                               T* __restrict__ k, T* __restrict__ v) {
  using C = typename Elem<T>::C;
  const T* row = qkv + b * sb + n * sn + static_cast<int64_t>(sl.part * H + sl.h) * D;
  T* dst = (sl.part == 0 ? q : sl.part == 1 ? k : v) + ((b * H + sl.h) * N + n) * D + sl.d0;
  C own[V];
  load_c<T, V>(row + sl.d0, own);
  if (sl.part == 2) {
    store_c<T, V>(dst, own);
    return;
  }
  C partner[V];
  float cs[V], sn_[V];
  load_c<T, V>(row + swap_index(sl.d0, D / 4), partner);
  load_table_v<V>(cos_t + n * D + sl.d0, cs);
  load_table_v<V>(sin_t + n * D + sl.d0, sn_);
  C out[V];
#pragma unroll
  for (int e = 0; e < V; ++e) {
    out[e] = rnd<T>(add_rn(mul_rn(own[e], static_cast<C>(cs[e])), mul_rn(partner[e], static_cast<C>(sn_[e]))));
    if (sl.part == 0 && qscale) out[e] = mul_rn(out[e], static_cast<C>(__ldg(qscale + sl.h)));
  }
  store_c<T, V>(dst, out);
}

template <typename T, int V>
__global__ void rope_split_kernel(const T* __restrict__ qkv, int64_t sb, int64_t sn, int64_t N, int H, int D,
                                  int64_t tokens, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                  const float* __restrict__ qscale, T* __restrict__ q, T* __restrict__ k,
                                  T* __restrict__ v) {
  const int cpr = D / V, slots = 3 * H * cpr;
  if (static_cast<int>(blockDim.x) >= slots) {
    if (static_cast<int>(threadIdx.x) >= slots) return;
    const RopeSlot sl = rope_slot(threadIdx.x, H, cpr, V);
    for (int64_t tok = blockIdx.x; tok < tokens; tok += gridDim.x) {
      const int64_t b = tok / N;
      rope_split_one<T, V>(qkv, sb, sn, b, tok - b * N, N, H, D, sl, cos_t, sin_t, qscale, q, k, v);
    }
  } else {
    for (int64_t tok = blockIdx.x; tok < tokens; tok += gridDim.x) {
      const int64_t b = tok / N;
      for (int s = threadIdx.x; s < slots; s += blockDim.x)
        rope_split_one<T, V>(qkv, sb, sn, b, tok - b * N, N, H, D, rope_slot(s, H, cpr, V), cos_t, sin_t, qscale,
                             q, k, v);
    }
  }
}

// The adjoint, same slots and token walk (so the dqkv writes are contiguous): g' = g * cos + quarter_swap(g * sin)
// for dq (after its qscale rounding) and dk; dv copied.
template <typename T, int V>
__device__ __forceinline__ void rope_merge_one(const ebr_operand& dq, const ebr_operand& dk, const ebr_operand& dv,
                                               int64_t tok, int64_t b, int64_t n, int H, int D, RopeSlot sl,
                                               const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                               const float* __restrict__ qscale, T* __restrict__ out) {
  using C = typename Elem<T>::C;
  const ebr_operand& op = sl.part == 0 ? dq : sl.part == 1 ? dk : dv;
  const T* row = static_cast<const T*>(op.data) + b * op.stride_b + sl.h * op.stride_h + n * op.stride_n;
  T* dst = out + tok * (3 * static_cast<int64_t>(H) * D) + static_cast<int64_t>(sl.part * H + sl.h) * D + sl.d0;
  C own[V];
  load_c<T, V>(row + sl.d0, own);
  if (sl.part == 2) {
    store_c<T, V>(dst, own);
    return;
  }
  const int p0 = swap_index(sl.d0, D / 4);
  C partner[V];
  float cs[V], sp[V];
  load_c<T, V>(row + p0, partner);
  load_table_v<V>(cos_t + n * D + sl.d0, cs);
  load_table_v<V>(sin_t + n * D + p0, sp);
  if (sl.part == 0 && qscale) {
    const C s = static_cast<C>(__ldg(qscale + sl.h));
#pragma unroll
    for (int e = 0; e < V; ++e) {
      own[e] = rnd<T>(mul_rn(own[e], s));
      partner[e] = rnd<T>(mul_rn(partner[e], s));
    }
  }
  C res[V];
#pragma unroll
  for (int e = 0; e < V; ++e)
    res[e] = add_rn(mul_rn(own[e], static_cast<C>(cs[e])), mul_rn(partner[e], static_cast<C>(sp[e])));
  store_c<T, V>(dst, res);
}

template <typename T, int V>
__global__ void rope_merge_kernel(ebr_operand dq, ebr_operand dk, ebr_operand dv, int64_t N, int H, int D,
                                  int64_t tokens, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                  const float* __restrict__ qscale, T* __restrict__ out) {
  const int cpr = D / V, slots = 3 * H * cpr;
  if (static_cast<int>(blockDim.x) >= slots) {
    if (static_cast<int>(threadIdx.x) >= slots) return;
    const RopeSlot sl = rope_slot(threadIdx.x, H, cpr, V);
    for (int64_t tok = blockIdx.x; tok < tokens; tok += gridDim.x) {
      const int64_t b = tok / N;
      rope_merge_one<T, V>(dq, dk, dv, tok, b, tok - b * N, H, D, sl, cos_t, sin_t, qscale, out);
    }
  } else {
    for (int64_t tok = blockIdx.x; tok < tokens; tok += gridDim.x) {
      const int64_t b = tok / N;
      for (int s = threadIdx.x; s < slots; s += blockDim.x)
        rope_merge_one<T, V>(dq, dk, dv, tok, b, tok - b * N, H, D, rope_slot(s, H, cpr, V), cos_t, sin_t, qscale,
                             out);
    }
  }
}

// The merge for 16-byte slots (V * sizeof(T) == 16) whose quarter partner lies in the same warp (D / V divides 32
// and D >= 4 V): slot = threadIdx.x, the partner slot is slot ^ (D / 4 V). Each thread loads only its own 16 bytes
// per token -- the partner's arrive by a shuffle -- and issues the loads of kTok tokens (blockIdx.x + u gridDim.x)
// before it computes or stores any, so each SM keeps kTok times the bytes of the one-token walk in flight (the merge
// is bound by the latency of its loads, not by HBM bandwidth, with one token in flight). Same arithmetic as
// rope_merge_one.
template <typename T, int V, int kTok>
__global__ void rope_merge_wide_kernel(ebr_operand dq, ebr_operand dk, ebr_operand dv, int64_t N, int H, int D,
                                       int64_t tokens, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                       const float* __restrict__ qscale, T* __restrict__ out) {
  static_assert(V * sizeof(T) == 16, "one 16-byte access per slot");
  using C = typename Elem<T>::C;
  const int cpr = D / V, slots = 3 * H * cpr;
  const int slot = static_cast<int>(threadIdx.x);
  const bool live = slot < slots;  // the block is rounded up to whole warps
  const RopeSlot sl = rope_slot(live ? slot : 0, H, cpr, V);
  const ebr_operand op = sl.part == 0 ? dq : sl.part == 1 ? dk : dv;
  const T* src = static_cast<const T*>(op.data) + sl.h * op.stride_h + sl.d0;
  const int64_t row3 = 3 * static_cast<int64_t>(H) * D;
  const int64_t col = static_cast<int64_t>(sl.part * H + sl.h) * D + sl.d0;
  const int lane_off = D / (4 * V);
  const int p0 = swap_index(sl.d0, D / 4);
  const bool scaled = sl.part == 0 && qscale != nullptr;
  const C s = scaled ? static_cast<C>(__ldg(qscale + sl.h)) : C(1);
  for (int64_t tok0 = blockIdx.x; tok0 < tokens; tok0 += kTok * static_cast<int64_t>(gridDim.x)) {
    Pack<T, V> raw[kTok];
#pragma unroll
    for (int u = 0; u < kTok; ++u) {
      const int64_t tok = tok0 + u * static_cast<int64_t>(gridDim.x);
      if (live && tok < tokens) {
        const int64_t b = tok / N, n = tok - b * N;
        raw[u] = *reinterpret_cast<const Pack<T, V>*>(src + b * op.stride_b + n * op.stride_n);
      } else {
#pragma unroll
        for (int i = 0; i < V; ++i) raw[u].e[i] = T();
      }
    }
#pragma unroll
    for (int u = 0; u < kTok; ++u) {
      const int64_t tok = tok0 + u * static_cast<int64_t>(gridDim.x);
      uint4 w = *reinterpret_cast<const uint4*>(&raw[u]);  // every lane shuffles (the partner may be any live lane)
      w.x = __shfl_xor_sync(0xffffffffu, w.x, lane_off);
      w.y = __shfl_xor_sync(0xffffffffu, w.y, lane_off);
      w.z = __shfl_xor_sync(0xffffffffu, w.z, lane_off);
      w.w = __shfl_xor_sync(0xffffffffu, w.w, lane_off);
      if (!live || tok >= tokens) continue;
      T* dst = out + tok * row3 + col;
      if (sl.part == 2) {
        *reinterpret_cast<Pack<T, V>*>(dst) = raw[u];
        continue;
      }
      const Pack<T, V> pw = *reinterpret_cast<const Pack<T, V>*>(&w);
      const int64_t n = tok - (tok / N) * N;
      float cs[V], sp[V];
      load_table_v<V>(cos_t + n * D + sl.d0, cs);
      load_table_v<V>(sin_t + n * D + p0, sp);
      C res[V];
#pragma unroll
      for (int e = 0; e < V; ++e) {
        C own = static_cast<C>(raw[u].e[e]), partner = static_cast<C>(pw.e[e]);
        if (scaled) {
          own = rnd<T>(mul_rn(own, s));
          partner = rnd<T>(mul_rn(partner, s));
        }
        res[e] = add_rn(mul_rn(own, static_cast<C>(cs[e])), mul_rn(partner, static_cast<C>(sp[e])));
      }
      store_c<T, V>(dst, res);
    }
  }
}

// ------------------------------------------------------------------------------------------------ residual + rms_norm

// One warp per row of C elements, two passes over the row (the second hits L1 / L2): the sum of squares of
// s = round(x + a), then y = round(s * rstd) (+ round(post * post_scale), rounded again).
template <typename T, int V>
__global__ void __launch_bounds__(kThreads) add_rms_norm_kernel(int64_t rows, int C_, float eps,
                                                                const T* __restrict__ x, const T* __restrict__ a,
                                                                T* __restrict__ sum_out, T* __restrict__ y,
                                                                float* __restrict__ rstd_out,
                                                                const T* __restrict__ post, float post_scale) {
  using C = typename Elem<T>::C;
  const int lane = threadIdx.x & 31;
  const int64_t warps = grid_stride() >> 5;
  for (int64_t row = global_tid() >> 5; row < rows; row += warps) {
    const int64_t base = row * C_;
    C ss = 0;
    for (int c = lane * V; c < C_; c += 32 * V) {
      C xs[V];
      load_c<T, V>(x + base + c, xs);
      if (a) {
        C as[V];
        load_c<T, V>(a + base + c, as);
#pragma unroll
        for (int e = 0; e < V; ++e) xs[e] = rnd<T>(add_rn(xs[e], as[e]));
        if (sum_out) store_c<T, V>(sum_out + base + c, xs);
      }
#pragma unroll
      for (int e = 0; e < V; ++e) ss += xs[e] * xs[e];
    }
    ss = warp_sum(ss);
    const C r = rsqrt_c(add_rn(div_rn(ss, static_cast<C>(C_)), static_cast<C>(eps)));
    for (int c = lane * V; c < C_; c += 32 * V) {
      C xs[V];
      load_c<T, V>(x + base + c, xs);
      if (a) {
        C as[V];
        load_c<T, V>(a + base + c, as);
#pragma unroll
        for (int e = 0; e < V; ++e) xs[e] = rnd<T>(add_rn(xs[e], as[e]));
      }
      C out[V];
#pragma unroll
      for (int e = 0; e < V; ++e) out[e] = mul_rn(xs[e], r);
      if (post) {
        C ps[V];
        load_c<T, V>(post + base + c, ps);
#pragma unroll
        for (int e = 0; e < V; ++e)
          out[e] = add_rn(rnd<T>(out[e]), rnd<T>(mul_rn(ps[e], static_cast<C>(post_scale))));
      }
      store_c<T, V>(y + base + c, out);
    }
    if (rstd_out && lane == 0) rstd_out[row] = static_cast<float>(r);
  }
}

// gs = round(rstd * (g - xh * mean(g * xh))), xh = s * rstd; one warp per row, two passes.
template <typename T, int V>
__global__ void __launch_bounds__(kThreads) rms_norm_bwd_kernel(int64_t rows, int C_, const T* __restrict__ s,
                                                                const float* __restrict__ rstd,
                                                                const T* __restrict__ gy, T* __restrict__ gs) {
  using C = typename Elem<T>::C;
  const int lane = threadIdx.x & 31;
  const int64_t warps = grid_stride() >> 5;
  for (int64_t row = global_tid() >> 5; row < rows; row += warps) {
    const int64_t base = row * C_;
    const C r = static_cast<C>(rstd[row]);
    C dot = 0;
    for (int c = lane * V; c < C_; c += 32 * V) {
      C xs[V], gs_[V];
      load_c<T, V>(s + base + c, xs);
      load_c<T, V>(gy + base + c, gs_);
#pragma unroll
      for (int e = 0; e < V; ++e) dot += gs_[e] * (xs[e] * r);
    }
    const C mean = warp_sum(dot) / static_cast<C>(C_);
    for (int c = lane * V; c < C_; c += 32 * V) {
      C xs[V], g[V], out[V];
      load_c<T, V>(s + base + c, xs);
      load_c<T, V>(gy + base + c, g);
#pragma unroll
      for (int e = 0; e < V; ++e) out[e] = r * (g[e] - (xs[e] * r) * mean);
      store_c<T, V>(gs + base + c, out);
    }
  }
}

// The double backward of rms_norm, for a graph built through the backward above (second-order training). With
// n = C, r = rstd (a function of s: dr/ds_k = -r^3 s_k / n), gs = r (g - xh mean(g xh)), xh = s r, and the
// upstream gradient u = dL/dgs, the row sums U_g = sum u g, U_s = sum u s, G = sum g s give
//   dL/dg_k = r u_k - (r^3 / n) s_k U_s,
//   dL/ds_k = (r^3 / n) (-s_k U_g + 3 r^2 s_k G U_s / n - G u_k - g_k U_s).
// One warp per row, two passes; fp32 throughout and one rounding to the I/O type per output.
template <typename T, int V>
__global__ void __launch_bounds__(kThreads) rms_norm_bwd2_kernel(int64_t rows, int C_, const T* __restrict__ s,
                                                                 const float* __restrict__ rstd,
                                                                 const T* __restrict__ gy, const T* __restrict__ u,
                                                                 T* __restrict__ ds, T* __restrict__ dgy) {
  using C = typename Elem<T>::C;
  const int lane = threadIdx.x & 31;
  const int64_t warps = grid_stride() >> 5;
  for (int64_t row = global_tid() >> 5; row < rows; row += warps) {
    const int64_t base = row * C_;
    const C r = static_cast<C>(rstd[row]);
    C ug = 0, us = 0, gs_ = 0;
    for (int c = lane * V; c < C_; c += 32 * V) {
      C xs[V], g[V], uu[V];
      load_c<T, V>(s + base + c, xs);
      load_c<T, V>(gy + base + c, g);
      load_c<T, V>(u + base + c, uu);
#pragma unroll
      for (int e = 0; e < V; ++e) {
        ug += uu[e] * g[e];
        us += uu[e] * xs[e];
        gs_ += g[e] * xs[e];
      }
    }
    ug = warp_sum(ug);
    us = warp_sum(us);
    gs_ = warp_sum(gs_);
    const C n = static_cast<C>(C_);
    const C r3n = r * r * r / n;
    const C k3 = C(3) * r * r * gs_ * us / n;
    for (int c = lane * V; c < C_; c += 32 * V) {
      C xs[V], g[V], uu[V], o_s[V], o_g[V];
      load_c<T, V>(s + base + c, xs);
      load_c<T, V>(gy + base + c, g);
      load_c<T, V>(u + base + c, uu);
#pragma unroll
      for (int e = 0; e < V; ++e) {
        o_s[e] = r3n * (xs[e] * (k3 - ug) - gs_ * uu[e] - g[e] * us);
        o_g[e] = r * uu[e] - r3n * xs[e] * us;
      }
      store_c<T, V>(ds + base + c, o_s);
      store_c<T, V>(dgy + base + c, o_g);
    }
  }
}

// ------------------------------------------------------------------------------------------------ SwiGLU

template <typename C>
__device__ __forceinline__ C silu_c(C x) {
  return x / (C(1) + exp_c(-x));
}

// out[r, j] = round(round(silu(h[r, j])) * h[r, I + j]); one thread per V-element chunk.
template <typename T, int V>
__global__ void __launch_bounds__(kThreads) swiglu_fwd_kernel(int64_t rows, int64_t I, const T* __restrict__ h,
                                                              T* __restrict__ out) {
  using C = typename Elem<T>::C;
  const int64_t cpr = I / V, total = rows * cpr;
  for (int64_t i = global_tid(); i < total; i += grid_stride()) {
    const int64_t r = i / cpr, j = (i - r * cpr) * V;
    C g[V], u[V], o[V];
    load_c<T, V>(h + r * 2 * I + j, g);
    load_c<T, V>(h + r * 2 * I + I + j, u);
#pragma unroll
    for (int e = 0; e < V; ++e) o[e] = mul_rn(rnd<T>(silu_c(g[e])), u[e]);
    store_c<T, V>(out + r * I + j, o);
  }
}

// gh[r, j] = silu'(gate) * round(gout * up), gh[r, I + j] = round(gout * round(silu(gate))).
template <typename T, int V>
__global__ void __launch_bounds__(kThreads) swiglu_bwd_kernel(int64_t rows, int64_t I, const T* __restrict__ h,
                                                              const T* __restrict__ gout, T* __restrict__ gh) {
  using C = typename Elem<T>::C;
  const int64_t cpr = I / V, total = rows * cpr;
  for (int64_t i = global_tid(); i < total; i += grid_stride()) {
    const int64_t r = i / cpr, j = (i - r * cpr) * V;
    C g[V], u[V], go[V], dg[V], du[V];
    load_c<T, V>(h + r * 2 * I + j, g);
    load_c<T, V>(h + r * 2 * I + I + j, u);
    load_c<T, V>(gout + r * I + j, go);
#pragma unroll
    for (int e = 0; e < V; ++e) {
      const C sg = C(1) / (C(1) + exp_c(-g[e]));
      const C act = rnd<T>(silu_c(g[e]));
      du[e] = mul_rn(go[e], act);
      const C da = rnd<T>(mul_rn(go[e], u[e]));
      dg[e] = da * sg * (C(1) + g[e] * (C(1) - sg));
    }
    store_c<T, V>(gh + r * 2 * I + j, dg);
    store_c<T, V>(gh + r * 2 * I + I + j, du);
  }
}

// The double backward of swiglu_bwd, for a graph built through it (second-order training). swiglu_bwd gives
// dg = da s1 (da = round(gout up), s1 = silu'(g) = sg (1 + g (1 - sg)), sg = sigmoid(g)) and du = gout act
// (act = round(silu(g))); with the upstream gradients ug = dL/d(dg), uu = dL/d(du) and s2 = silu''(g) =
// sg (1 - sg) (2 + g (1 - 2 sg)):
//   dL/dgout = ug up s1 + uu act,   dL/dup = ug gout s1,   dL/dg = ug da s2 + uu gout s1.
// The roundings of da and act are taken as the identity in the derivative, as autograd does for a cast.
template <typename T, int V>
__global__ void __launch_bounds__(kThreads) swiglu_bwd2_kernel(int64_t rows, int64_t I, const T* __restrict__ h,
                                                               const T* __restrict__ gout, const T* __restrict__ u,
                                                               T* __restrict__ dh, T* __restrict__ dgout) {
  using C = typename Elem<T>::C;
  const int64_t cpr = I / V, total = rows * cpr;
  for (int64_t i = global_tid(); i < total; i += grid_stride()) {
    const int64_t r = i / cpr, j = (i - r * cpr) * V;
    C g[V], up[V], go[V], ug[V], uu[V], o_g[V], o_u[V], o_go[V];
    load_c<T, V>(h + r * 2 * I + j, g);
    load_c<T, V>(h + r * 2 * I + I + j, up);
    load_c<T, V>(gout + r * I + j, go);
    load_c<T, V>(u + r * 2 * I + j, ug);
    load_c<T, V>(u + r * 2 * I + I + j, uu);
#pragma unroll
    for (int e = 0; e < V; ++e) {
      const C sg = C(1) / (C(1) + exp_c(-g[e]));
      const C s1 = sg * (C(1) + g[e] * (C(1) - sg));
      const C s2 = sg * (C(1) - sg) * (C(2) + g[e] * (C(1) - C(2) * sg));
      const C act = rnd<T>(silu_c(g[e]));
      const C da = rnd<T>(mul_rn(go[e], up[e]));
      o_go[e] = ug[e] * up[e] * s1 + uu[e] * act;
      o_u[e] = ug[e] * go[e] * s1;
      o_g[e] = ug[e] * da * s2 + uu[e] * go[e] * s1;
    }
    store_c<T, V>(dh + r * 2 * I + j, o_g);
    store_c<T, V>(dh + r * 2 * I + I + j, o_u);
    store_c<T, V>(dgout + r * I + j, o_go);
  }
}

// ------------------------------------------------------------------------------------------------ descent step

constexpr int kStepChunk = kThreads * 32;  // elements of one row handled by one block

// Block (chunk, row): u = round(v - round(alpha * g)) into z_next, and the block's sum of u^2 into partial.
template <typename T, int V>
__global__ void __launch_bounds__(kThreads) descent_step_kernel(int64_t row_elems, int chunks, double alpha,
                                                                const T* __restrict__ v, const T* __restrict__ g,
                                                                T* __restrict__ z_next, float* __restrict__ partial) {
  using C = typename Elem<T>::C;
  __shared__ float red[kThreads / 32];
  const int64_t row = blockIdx.y;
  const int64_t lo = static_cast<int64_t>(blockIdx.x) * kStepChunk;
  const int64_t hi = min(lo + kStepChunk, row_elems);
  const int64_t base = row * row_elems;
  float ss = 0.f;
  for (int64_t c = lo + threadIdx.x * V; c < hi; c += kThreads * V) {
    C vs[V], gs[V], u[V];
    load_c<T, V>(v + base + c, vs);
    load_c<T, V>(g + base + c, gs);
#pragma unroll
    for (int e = 0; e < V; ++e) {
      u[e] = rnd<T>(sub_rn(vs[e], rnd<T>(mul_rn(static_cast<C>(alpha), gs[e]))));
      ss += static_cast<float>(u[e] * u[e]);
    }
    store_c<T, V>(z_next + base + c, u);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < kThreads / 32; ++w) t += red[w];
    partial[row * chunks + blockIdx.x] = t;
  }
}

// Block (chunk, row): rms of the row from its partial sums (every block adds them in the same order), then
// z_next = round(u / max(rms, eps)) in place.
template <typename T, int V>
__global__ void __launch_bounds__(kThreads) sphere_kernel(int64_t row_elems, int chunks, float eps,
                                                          T* __restrict__ z_next, const float* __restrict__ partial) {
  using C = typename Elem<T>::C;
  __shared__ float rms_s;
  const int64_t row = blockIdx.y;
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < chunks; ++i) t += partial[row * chunks + i];
    rms_s = fmaxf(sqrtf(__fdiv_rn(t, static_cast<float>(row_elems))), eps);
  }
  __syncthreads();
  const C rms = static_cast<C>(rms_s);
  const int64_t lo = static_cast<int64_t>(blockIdx.x) * kStepChunk;
  const int64_t hi = min(lo + kStepChunk, row_elems);
  const int64_t base = row * row_elems;
  for (int64_t c = lo + threadIdx.x * V; c < hi; c += kThreads * V) {
    C u[V];
    load_c<T, V>(z_next + base + c, u);
#pragma unroll
    for (int e = 0; e < V; ++e) u[e] = div_rn(u[e], rms);
    store_c<T, V>(z_next + base + c, u);
  }
}

}  // namespace layers
}  // namespace ebr
