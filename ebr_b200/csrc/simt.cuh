// simt.cuh: CUDA-core kernels of the three attention passes, for every dtype and any D <= 256.
//
// These carry the float32 / float64 calls (the reference's IEEE and fp64 modes, triton_kernels.py:9-15, :33-37, used
// by its second-order self-test and gradcheck-style checks) and half-type calls whose shape or strides the tcgen05
// kernels do not take. They compute in float64 for float64 and float32 otherwise, one thread block per query row
// (row passes) or key row (column passes), with the same row / column split and row scalars as the reference's
// two-kernel mode (triton_kernels.py:171-339, :347-551). The math of each pass is the dense formula of
// reference.py:23-91; the double backward uses the closed form of reference.py:80-90 directly.
#pragma once

#include "sm100.cuh"

namespace ebr {

constexpr int kSimtThreads = 128;

template <typename T>
struct Strided {
  const T* p;
  int64_t sb, sh, sn;
  __device__ __forceinline__ const T* row(int64_t b, int64_t h, int64_t n) const { return p + b * sb + h * sh + n * sn; }
};

template <typename C>
__device__ __forceinline__ C warp_sum(C x) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  return x;
}
template <typename C>
__device__ __forceinline__ C warp_max(C x) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) x = max(x, __shfl_xor_sync(0xffffffffu, x, off));
  return x;
}

// Block-wide sum / max in a fixed order (deterministic). `red` holds kSimtThreads/32 values.
template <typename C>
__device__ C block_sum(C x, C* red) {
  x = warp_sum(x);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = x;
  __syncthreads();
  C t = 0;
#pragma unroll
  for (int w = 0; w < kSimtThreads / 32; ++w) t += red[w];
  return t;
}
template <typename C>
__device__ C block_max(C x, C* red) {
  x = warp_max(x);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = x;
  __syncthreads();
  C t = red[0];
#pragma unroll
  for (int w = 1; w < kSimtThreads / 32; ++w) t = max(t, red[w]);
  return t;
}

// <x (shared, compute type), row (global, storage type)> over D.
template <typename T, typename C>
__device__ __forceinline__ C dot_row(const C* x, const T* row, int D) {
  C acc = 0;
  for (int d = 0; d < D; ++d) acc += x[d] * static_cast<C>(Elem<T>::load(row + d));
  return acc;
}

template <typename T, typename C>
__device__ __forceinline__ void load_row(C* dst, const T* row, int D) {
  for (int d = threadIdx.x; d < D; d += kSimtThreads) dst[d] = row ? static_cast<C>(Elem<T>::load(row + d)) : C(0);
}

// ------------------------------------------------------------------------------------------------ forward

// One block per (b, h, query row i): three sweeps over the keys (row max, row sum, then P V), matching
// reference.attn_fwd: lse = logsumexp(scale q k^T), o = exp(s - lse) v.
template <typename T>
__global__ void __launch_bounds__(kSimtThreads) simt_fwd(int64_t rows, int H, int N, int D, double scale_d,
                                                         Strided<T> q, Strided<T> k, Strided<T> v, T* o,
                                                         typename Elem<T>::C* lse) {
  using C = typename Elem<T>::C;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  C* qs = reinterpret_cast<C*>(smem_raw);
  C* ps = qs + D;
  C* red = ps + kSimtThreads;
  const C scale = static_cast<C>(scale_d);
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const int64_t bh = row / N;
    const int i = static_cast<int>(row - bh * N);
    const int64_t b = bh / H, h = bh - b * H;
    __syncthreads();
    load_row(qs, q.row(b, h, i), D);
    __syncthreads();
    C mx = -INFINITY;
    for (int j = threadIdx.x; j < N; j += kSimtThreads) mx = max(mx, scale * dot_row(qs, k.row(b, h, j), D));
    mx = block_max(mx, red);
    C sum = 0;
    for (int j = threadIdx.x; j < N; j += kSimtThreads) sum += exp(scale * dot_row(qs, k.row(b, h, j), D) - mx);
    sum = block_sum(sum, red);
    const C L = mx + log(sum);
    C acc0 = 0, acc1 = 0;
    const int d0 = threadIdx.x, d1 = threadIdx.x + kSimtThreads;
    for (int j0 = 0; j0 < N; j0 += kSimtThreads) {
      const int j = j0 + threadIdx.x;
      __syncthreads();
      ps[threadIdx.x] = (j < N) ? exp(scale * dot_row(qs, k.row(b, h, j), D) - L) : C(0);
      __syncthreads();
      const int cnt = min(kSimtThreads, N - j0);
      for (int jj = 0; jj < cnt; ++jj) {
        const T* vr = v.row(b, h, j0 + jj);
        if (d0 < D) acc0 += ps[jj] * static_cast<C>(Elem<T>::load(vr + d0));
        if (d1 < D) acc1 += ps[jj] * static_cast<C>(Elem<T>::load(vr + d1));
      }
    }
    T* orow = o + row * D;
    if (d0 < D) orow[d0] = Elem<T>::to(acc0);
    if (d1 < D) orow[d1] = Elem<T>::to(acc1);
    if (threadIdx.x == 0) lse[row] = L;
  }
}

// ------------------------------------------------------------------------------------------------ backward

// Row pass: D_i = <dO_i, O_i> (stored O), dQ_i = scale * sum_j dS_ij k_j. Writes D_i to di[row].
template <typename T>
__global__ void __launch_bounds__(kSimtThreads) simt_bwd_row(int64_t rows, int H, int N, int D, double scale_d,
                                                             Strided<T> q, Strided<T> k, Strided<T> v, const T* o,
                                                             const typename Elem<T>::C* lse, Strided<T> dout, T* dq,
                                                             typename Elem<T>::C* di) {
  using C = typename Elem<T>::C;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  C* qs = reinterpret_cast<C*>(smem_raw);
  C* dos = qs + D;
  C* dss = dos + D;
  C* red = dss + kSimtThreads;
  const C scale = static_cast<C>(scale_d);
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const int64_t bh = row / N;
    const int i = static_cast<int>(row - bh * N);
    const int64_t b = bh / H, h = bh - b * H;
    __syncthreads();
    load_row(qs, q.row(b, h, i), D);
    load_row(dos, dout.row(b, h, i), D);
    __syncthreads();
    C part = 0;
    for (int d = threadIdx.x; d < D; d += kSimtThreads) part += dos[d] * static_cast<C>(Elem<T>::load(o + row * D + d));
    const C Di = block_sum(part, red);
    const C Li = lse[row];
    C acc0 = 0, acc1 = 0;
    const int d0 = threadIdx.x, d1 = threadIdx.x + kSimtThreads;
    for (int j0 = 0; j0 < N; j0 += kSimtThreads) {
      const int j = j0 + threadIdx.x;
      C ds = 0;
      if (j < N) {
        const C p = exp(scale * dot_row(qs, k.row(b, h, j), D) - Li);
        const C dp = dot_row(dos, v.row(b, h, j), D);
        ds = p * (dp - Di);
      }
      __syncthreads();
      dss[threadIdx.x] = ds;
      __syncthreads();
      const int cnt = min(kSimtThreads, N - j0);
      for (int jj = 0; jj < cnt; ++jj) {
        const T* kr = k.row(b, h, j0 + jj);
        if (d0 < D) acc0 += dss[jj] * static_cast<C>(Elem<T>::load(kr + d0));
        if (d1 < D) acc1 += dss[jj] * static_cast<C>(Elem<T>::load(kr + d1));
      }
    }
    T* r = dq + row * D;
    if (d0 < D) r[d0] = Elem<T>::to(acc0 * scale);
    if (d1 < D) r[d1] = Elem<T>::to(acc1 * scale);
    if (threadIdx.x == 0) di[row] = Di;
  }
}

// Column pass: dK_j = scale * sum_i dS_ij q_i, dV_j = sum_i P_ij dO_i, with D_i from the row pass.
template <typename T>
__global__ void __launch_bounds__(kSimtThreads) simt_bwd_col(int64_t rows, int H, int N, int D, double scale_d,
                                                             Strided<T> q, Strided<T> k, Strided<T> v,
                                                             const typename Elem<T>::C* lse, Strided<T> dout,
                                                             const typename Elem<T>::C* di, T* dk, T* dv) {
  using C = typename Elem<T>::C;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  C* ks = reinterpret_cast<C*>(smem_raw);
  C* vs = ks + D;
  C* ps = vs + D;
  C* dss = ps + kSimtThreads;
  const C scale = static_cast<C>(scale_d);
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const int64_t bh = row / N;
    const int j = static_cast<int>(row - bh * N);
    const int64_t b = bh / H, h = bh - b * H;
    __syncthreads();
    load_row(ks, k.row(b, h, j), D);
    load_row(vs, v.row(b, h, j), D);
    __syncthreads();
    C dk0 = 0, dk1 = 0, dv0 = 0, dv1 = 0;
    const int d0 = threadIdx.x, d1 = threadIdx.x + kSimtThreads;
    for (int i0 = 0; i0 < N; i0 += kSimtThreads) {
      const int i = i0 + threadIdx.x;
      C p = 0, ds = 0;
      if (i < N) {
        const int64_t ri = bh * N + i;
        p = exp(scale * dot_row(ks, q.row(b, h, i), D) - lse[ri]);
        const C dp = dot_row(vs, dout.row(b, h, i), D);
        ds = p * (dp - di[ri]);
      }
      __syncthreads();
      ps[threadIdx.x] = p;
      dss[threadIdx.x] = ds;
      __syncthreads();
      const int cnt = min(kSimtThreads, N - i0);
      for (int ii = 0; ii < cnt; ++ii) {
        const T* qr = q.row(b, h, i0 + ii);
        const T* dr = dout.row(b, h, i0 + ii);
        if (d0 < D) {
          dk0 += dss[ii] * static_cast<C>(Elem<T>::load(qr + d0));
          dv0 += ps[ii] * static_cast<C>(Elem<T>::load(dr + d0));
        }
        if (d1 < D) {
          dk1 += dss[ii] * static_cast<C>(Elem<T>::load(qr + d1));
          dv1 += ps[ii] * static_cast<C>(Elem<T>::load(dr + d1));
        }
      }
    }
    if (d0 < D) {
      dk[row * D + d0] = Elem<T>::to(dk0 * scale);
      dv[row * D + d0] = Elem<T>::to(dv0);
    }
    if (d1 < D) {
      dk[row * D + d1] = Elem<T>::to(dk1 * scale);
      dv[row * D + d1] = Elem<T>::to(dv1);
    }
  }
}

// ------------------------------------------------------------------------------------------------ backward of backward

template <typename T, typename C>
__device__ __forceinline__ C dot_row_opt(const C* x, const T* row, int D) {
  return row ? dot_row(x, row, D) : C(0);
}
template <typename T>
__device__ __forceinline__ const T* row_opt(const Strided<T>& s, int64_t b, int64_t h, int64_t n) {
  return s.p ? s.row(b, h, n) : nullptr;
}
template <typename T>
__device__ __forceinline__ float load_opt(const T* row, int d) {
  return row ? static_cast<float>(Elem<T>::load(row + d)) : 0.f;
}
__device__ __forceinline__ double load_opt(const double* row, int d) { return row ? row[d] : 0.0; }

// Per (query i, key j): the quantities of reference.py:80-88 given the row scalars D_i, E_i, T_i.
template <typename C>
struct BobTerms {
  C p, ds, a, gs;
};
template <typename C>
__device__ __forceinline__ BobTerms<C> bob_terms(C s_scaled, C Li, C g, C dp, C r, C Di, C Ei, C Ti) {
  BobTerms<C> t;
  t.p = exp(s_scaled - Li);
  t.ds = t.p * (dp - Di);
  t.a = t.p * (g - Ei);
  const C gp = (dp - Di) * g - Ei * dp + r;
  t.gs = t.p * (gp - Ti);
  return t;
}

// Row pass: D_i, E_i = sum_j P g, T_i = sum_j P gp (as sum ds g - E sum P dP + sum P r), then
// hQ_i = scale * sum_j (gS k_j + dS gk_j), hdO_i = sum_j (A v_j + P gv_j). Writes D, E, T to stats[0..2][row].
template <typename T>
__global__ void __launch_bounds__(kSimtThreads) simt_bob_row(int64_t rows, int H, int N, int D, double scale_d,
                                                             Strided<T> q, Strided<T> k, Strided<T> v, const T* o,
                                                             const typename Elem<T>::C* lse, Strided<T> dout,
                                                             Strided<T> gq, Strided<T> gk, Strided<T> gv, T* hq,
                                                             T* hdo, typename Elem<T>::C* stats) {
  using C = typename Elem<T>::C;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  C* qs = reinterpret_cast<C*>(smem_raw);
  C* gqs = qs + D;
  C* dos = gqs + D;
  C* s_gs = dos + D;
  C* s_ds = s_gs + kSimtThreads;
  C* s_a = s_ds + kSimtThreads;
  C* s_p = s_a + kSimtThreads;
  C* red = s_p + kSimtThreads;
  const C scale = static_cast<C>(scale_d);
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const int64_t bh = row / N;
    const int i = static_cast<int>(row - bh * N);
    const int64_t b = bh / H, h = bh - b * H;
    __syncthreads();
    load_row(qs, q.row(b, h, i), D);
    load_row(gqs, row_opt(gq, b, h, i), D);
    load_row(dos, dout.row(b, h, i), D);
    __syncthreads();
    C part = 0;
    for (int d = threadIdx.x; d < D; d += kSimtThreads) part += dos[d] * static_cast<C>(Elem<T>::load(o + row * D + d));
    const C Di = block_sum(part, red);
    const C Li = lse[row];
    C e = 0, c1 = 0, c2 = 0, c3 = 0;
    for (int j = threadIdx.x; j < N; j += kSimtThreads) {
      const T* kr = k.row(b, h, j);
      const C p = exp(scale * dot_row(qs, kr, D) - Li);
      const C g = (dot_row(gqs, kr, D) + dot_row_opt(qs, row_opt(gk, b, h, j), D)) * scale;
      const C dp = dot_row(dos, v.row(b, h, j), D);
      const C r = dot_row_opt(dos, row_opt(gv, b, h, j), D);
      e += p * g;
      c1 += p * (dp - Di) * g;
      c2 += p * dp;
      c3 += p * r;
    }
    const C E = block_sum(e, red);
    const C C1 = block_sum(c1, red);
    const C C2 = block_sum(c2, red);
    const C C3 = block_sum(c3, red);
    const C Tt = C1 - E * C2 + C3;
    C hq0 = 0, hq1 = 0, ho0 = 0, ho1 = 0;
    const int d0 = threadIdx.x, d1 = threadIdx.x + kSimtThreads;
    for (int j0 = 0; j0 < N; j0 += kSimtThreads) {
      const int j = j0 + threadIdx.x;
      BobTerms<C> t{0, 0, 0, 0};
      if (j < N) {
        const T* kr = k.row(b, h, j);
        const C g = (dot_row(gqs, kr, D) + dot_row_opt(qs, row_opt(gk, b, h, j), D)) * scale;
        const C dp = dot_row(dos, v.row(b, h, j), D);
        const C r = dot_row_opt(dos, row_opt(gv, b, h, j), D);
        t = bob_terms<C>(scale * dot_row(qs, kr, D), Li, g, dp, r, Di, E, Tt);
      }
      __syncthreads();
      s_gs[threadIdx.x] = t.gs;
      s_ds[threadIdx.x] = t.ds;
      s_a[threadIdx.x] = t.a;
      s_p[threadIdx.x] = t.p;
      __syncthreads();
      const int cnt = min(kSimtThreads, N - j0);
      for (int jj = 0; jj < cnt; ++jj) {
        const int jn = j0 + jj;
        const T* kr = k.row(b, h, jn);
        const T* vr = v.row(b, h, jn);
        const T* gkr = row_opt(gk, b, h, jn);
        const T* gvr = row_opt(gv, b, h, jn);
        if (d0 < D) {
          hq0 += s_gs[jj] * static_cast<C>(Elem<T>::load(kr + d0)) + s_ds[jj] * static_cast<C>(load_opt(gkr, d0));
          ho0 += s_a[jj] * static_cast<C>(Elem<T>::load(vr + d0)) + s_p[jj] * static_cast<C>(load_opt(gvr, d0));
        }
        if (d1 < D) {
          hq1 += s_gs[jj] * static_cast<C>(Elem<T>::load(kr + d1)) + s_ds[jj] * static_cast<C>(load_opt(gkr, d1));
          ho1 += s_a[jj] * static_cast<C>(Elem<T>::load(vr + d1)) + s_p[jj] * static_cast<C>(load_opt(gvr, d1));
        }
      }
    }
    if (d0 < D) {
      hq[row * D + d0] = Elem<T>::to(hq0 * scale);
      hdo[row * D + d0] = Elem<T>::to(ho0);
    }
    if (d1 < D) {
      hq[row * D + d1] = Elem<T>::to(hq1 * scale);
      hdo[row * D + d1] = Elem<T>::to(ho1);
    }
    if (threadIdx.x == 0) {
      stats[row] = Di;
      stats[rows + row] = E;
      stats[2 * rows + row] = Tt;
    }
  }
}

// Column pass: hK_j = scale * sum_i (gS q_i + dS gq_i), hV_j = sum_i A dO_i, with D, E, T from the row pass.
template <typename T>
__global__ void __launch_bounds__(kSimtThreads) simt_bob_col(int64_t rows, int H, int N, int D, double scale_d,
                                                             Strided<T> q, Strided<T> k, Strided<T> v,
                                                             const typename Elem<T>::C* lse, Strided<T> dout,
                                                             Strided<T> gq, Strided<T> gk, Strided<T> gv, T* hk,
                                                             T* hv, const typename Elem<T>::C* stats) {
  using C = typename Elem<T>::C;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  C* ks = reinterpret_cast<C*>(smem_raw);
  C* gks = ks + D;
  C* vs = gks + D;
  C* gvs = vs + D;
  C* s_gs = gvs + D;
  C* s_ds = s_gs + kSimtThreads;
  C* s_a = s_ds + kSimtThreads;
  const C scale = static_cast<C>(scale_d);
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const int64_t bh = row / N;
    const int j = static_cast<int>(row - bh * N);
    const int64_t b = bh / H, h = bh - b * H;
    __syncthreads();
    load_row(ks, k.row(b, h, j), D);
    load_row(gks, row_opt(gk, b, h, j), D);
    load_row(vs, v.row(b, h, j), D);
    load_row(gvs, row_opt(gv, b, h, j), D);
    __syncthreads();
    C hk0 = 0, hk1 = 0, hv0 = 0, hv1 = 0;
    const int d0 = threadIdx.x, d1 = threadIdx.x + kSimtThreads;
    for (int i0 = 0; i0 < N; i0 += kSimtThreads) {
      const int i = i0 + threadIdx.x;
      BobTerms<C> t{0, 0, 0, 0};
      if (i < N) {
        const int64_t ri = bh * N + i;
        const T* qr = q.row(b, h, i);
        const T* dr = dout.row(b, h, i);
        const C g = (dot_row_opt(ks, row_opt(gq, b, h, i), D) + dot_row(gks, qr, D)) * scale;
        const C dp = dot_row(vs, dr, D);
        const C r = dot_row(gvs, dr, D);
        t = bob_terms<C>(scale * dot_row(ks, qr, D), lse[ri], g, dp, r, stats[ri], stats[rows + ri],
                         stats[2 * rows + ri]);
      }
      __syncthreads();
      s_gs[threadIdx.x] = t.gs;
      s_ds[threadIdx.x] = t.ds;
      s_a[threadIdx.x] = t.a;
      __syncthreads();
      const int cnt = min(kSimtThreads, N - i0);
      for (int ii = 0; ii < cnt; ++ii) {
        const int in = i0 + ii;
        const T* qr = q.row(b, h, in);
        const T* dr = dout.row(b, h, in);
        const T* gqr = row_opt(gq, b, h, in);
        if (d0 < D) {
          hk0 += s_gs[ii] * static_cast<C>(Elem<T>::load(qr + d0)) + s_ds[ii] * static_cast<C>(load_opt(gqr, d0));
          hv0 += s_a[ii] * static_cast<C>(Elem<T>::load(dr + d0));
        }
        if (d1 < D) {
          hk1 += s_gs[ii] * static_cast<C>(Elem<T>::load(qr + d1)) + s_ds[ii] * static_cast<C>(load_opt(gqr, d1));
          hv1 += s_a[ii] * static_cast<C>(Elem<T>::load(dr + d1));
        }
      }
    }
    if (d0 < D) {
      hk[row * D + d0] = Elem<T>::to(hk0 * scale);
      hv[row * D + d0] = Elem<T>::to(hv0);
    }
    if (d1 < D) {
      hk[row * D + d1] = Elem<T>::to(hk1 * scale);
      hv[row * D + d1] = Elem<T>::to(hv1);
    }
  }
}

}  // namespace ebr
