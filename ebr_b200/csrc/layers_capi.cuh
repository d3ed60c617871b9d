// layers_capi.cuh: the C ABI of include/ebr_layers.h (included at the end of capi.cu, which owns the error state,
// the device check and the launch counter). Validates arguments, picks the 16-byte vector width when the pointers and
// row lengths allow it, and launches the kernels of layers.cuh on the caller's stream.
#pragma once

#include <algorithm>
#include <initializer_list>
#include <type_traits>

#include "../../include/ebr_layers.h"
#include "layers.cuh"
#include "gate_up.cuh"
#include "o_proj.cuh"
#include "merge_gemm.cuh"
#include "qkv_rope.cuh"

namespace {

using ebr::layers::kThreads;

// Grid for a grid-stride kernel over `work` thread-items.
dim3 flat_grid(int device, int64_t work) {
  const int64_t want = (work + kThreads - 1) / kThreads;
  const int64_t cap = static_cast<int64_t>(sm_count(device)) * 16;
  return dim3(static_cast<unsigned>(std::max<int64_t>(1, std::min(want, cap))));
}

template <typename T>
constexpr int vec_width() {
  return static_cast<int>(16 / sizeof(T));
}

bool all_aligned16(std::initializer_list<const void*> ps) {
  for (const void* p : ps)
    if (p && !aligned16(p)) return false;
  return true;
}

int check_layer_dtype(int dtype, bool allow_f64) {
  if (dtype == EBR_FLOAT32 || dtype == EBR_FLOAT16 || dtype == EBR_BFLOAT16) return EBR_OK;
  if (dtype == EBR_FLOAT64 && allow_f64) return EBR_OK;
  return set_error(EBR_ERR_DTYPE, "unsupported dtype for this layer kernel%s%s");
}

// Run fn.template operator()<T>() for the I/O type of `dtype`.
template <typename Fn>
int with_type(int dtype, Fn&& fn) {
  switch (dtype) {
    case EBR_FLOAT32: return fn(static_cast<float*>(nullptr));
    case EBR_FLOAT16: return fn(static_cast<__half*>(nullptr));
    case EBR_BFLOAT16: return fn(static_cast<__nv_bfloat16*>(nullptr));
    case EBR_FLOAT64: return fn(static_cast<double*>(nullptr));
    default: return set_error(EBR_ERR_DTYPE, "unknown dtype%s%s");
  }
}

// RoPE launch shape: one token's slots per block (rounded up to whole warps, at most 1024 threads; wider rows loop),
// enough blocks to fill the SMs, each walking tokens with a stride of the grid.
struct RopeGrid {
  dim3 blocks, threads;
};

RopeGrid rope_grid(int device, int64_t slots, int64_t tokens) {
  const int threads = static_cast<int>(std::min<int64_t>(1024, (slots + 31) / 32 * 32));
  const int64_t per_sm = std::max<int64_t>(1, 2048 / threads);
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>(tokens, per_sm * sm_count(device) * 4));
  return RopeGrid{dim3(static_cast<unsigned>(blocks)), dim3(static_cast<unsigned>(threads))};
}

int check_rope_shape(int64_t B, int64_t N, int64_t H, int64_t D) {
  if (B < 0 || N < 0 || H < 0) return set_error(EBR_ERR_SHAPE, "negative size%s%s");
  if (D < 4 || D % 4 != 0 || D > 4096) return set_error(EBR_ERR_SHAPE, "head dim must be a multiple of 4 in [4, 4096]%s%s");
  if (H > (1 << 20) || N > (int64_t{1} << 31) || B > (int64_t{1} << 31))
    return set_error(EBR_ERR_SHAPE, "size too large%s%s");
  return EBR_OK;
}

// 2-D TMA map over a row-major [rows, cols] 16-bit matrix (row stride in elements), 64-column x box_rows boxes,
// 128-byte swizzle; rows past the end read as zeros.
int make_matrix_map(CUtensorMap* map, const void* ptr, int dtype, int64_t rows, int64_t cols, int64_t row_stride,
                    uint32_t box_rows) {
  EncodeTiled enc = encode_fn();
  if (!enc) return set_error(EBR_ERR_CUDA, "cuTensorMapEncodeTiled unavailable%s%s");
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride * 2)};
  const cuuint32_t box[2] = {64, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dtype == EBR_BFLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                   const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(EBR_ERR_CUDA, "cuTensorMapEncodeTiled failed%s%s");
  return EBR_OK;
}

// 2-D TMA store map over a row-major [rows, cols] 16-bit matrix: boxes of 16 columns x 32 rows with the 32-byte
// swizzle (one epilogue warp's output chunk); rows past the end are not written.
int make_chunk_store_map(CUtensorMap* map, void* ptr, int dtype, int64_t rows, int64_t cols, int64_t row_stride) {
  EncodeTiled enc = encode_fn();
  if (!enc) return set_error(EBR_ERR_CUDA, "cuTensorMapEncodeTiled unavailable%s%s");
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride * 2)};
  const cuuint32_t box[2] = {16, 32};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dtype == EBR_BFLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                   ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B,
                   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(EBR_ERR_CUDA, "cuTensorMapEncodeTiled failed%s%s");
  return EBR_OK;
}

// 3-D TMA store map over a contiguous [B, N, C] 16-bit tensor: boxes of 32 columns x 32 rows of one sample with the
// 64-byte swizzle (one epilogue warp's output chunk); rows past N are not written, so a box never spills into the next
// sample.
int make_sample_store_map(CUtensorMap* map, void* ptr, int dtype, int64_t B, int64_t N, int64_t C) {
  EncodeTiled enc = encode_fn();
  if (!enc) return set_error(EBR_ERR_CUDA, "cuTensorMapEncodeTiled unavailable%s%s");
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(B)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(C * 2), static_cast<cuuint64_t>(N * C * 2)};
  const cuuint32_t box[3] = {32, 32, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, dtype == EBR_BFLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                   ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(EBR_ERR_CUDA, "cuTensorMapEncodeTiled failed%s%s");
  return EBR_OK;
}

}  // namespace

extern "C" {

int ebr_rope_split(int dtype, int64_t B, int64_t N, int64_t H, int64_t D, const void* qkv, int64_t stride_b,
                   int64_t stride_n, const float* cos_table, const float* sin_table, const float* qscale, void* q,
                   void* k, void* v, void* stream) {
  int rc = check_layer_dtype(dtype, true);
  if (rc == EBR_OK) rc = check_rope_shape(B, N, H, D);
  if (rc != EBR_OK) return rc;
  if (B * N * H == 0) return EBR_OK;
  if (!qkv || !cos_table || !sin_table || !q || !k || !v) return set_error(EBR_ERR_NULL, "rope_split: NULL pointer%s%s");
  if (stride_b < 0 || stride_n < 0) return set_error(EBR_ERR_STRIDE, "rope_split: negative stride%s%s");
  int device = 0;
  if ((rc = check_device(&device)) != EBR_OK) return rc;
  auto st = static_cast<cudaStream_t>(stream);
  return with_type(dtype, [&](auto* tag) -> int {
    using T = std::remove_pointer_t<decltype(tag)>;
    constexpr int V = vec_width<T>();
    const bool vec = (D / 4) % V == 0 && stride_b % V == 0 && stride_n % V == 0 &&
                     all_aligned16({qkv, q, k, v, cos_table, sin_table});
    const T* src = static_cast<const T*>(qkv);
    const int64_t tokens = B * N;
    if (vec) {
      const RopeGrid g = rope_grid(device, 3 * H * (D / V), tokens);
      ebr::layers::rope_split_kernel<T, V><<<g.blocks, g.threads, 0, st>>>(
          src, stride_b, stride_n, N, static_cast<int>(H), static_cast<int>(D), tokens, cos_table, sin_table, qscale,
          static_cast<T*>(q), static_cast<T*>(k), static_cast<T*>(v));
    } else {
      const RopeGrid g = rope_grid(device, 3 * H * D, tokens);
      ebr::layers::rope_split_kernel<T, 1><<<g.blocks, g.threads, 0, st>>>(
          src, stride_b, stride_n, N, static_cast<int>(H), static_cast<int>(D), tokens, cos_table, sin_table, qscale,
          static_cast<T*>(q), static_cast<T*>(k), static_cast<T*>(v));
    }
    return check_launch("rope_split");
  });
}

int ebr_rope_merge(int dtype, int64_t B, int64_t N, int64_t H, int64_t D, const ebr_operand* dq,
                   const ebr_operand* dk, const ebr_operand* dv, const float* cos_table, const float* sin_table,
                   const float* qscale, void* dqkv, void* stream) {
  int rc = check_layer_dtype(dtype, true);
  if (rc == EBR_OK) rc = check_rope_shape(B, N, H, D);
  if (rc == EBR_OK) rc = check_operand(dq, "dq");
  if (rc == EBR_OK) rc = check_operand(dk, "dk");
  if (rc == EBR_OK) rc = check_operand(dv, "dv");
  if (rc != EBR_OK) return rc;
  if (B * N * H == 0) return EBR_OK;
  if (!cos_table || !sin_table || !dqkv) return set_error(EBR_ERR_NULL, "rope_merge: NULL pointer%s%s");
  int device = 0;
  if ((rc = check_device(&device)) != EBR_OK) return rc;
  auto st = static_cast<cudaStream_t>(stream);
  return with_type(dtype, [&](auto* tag) -> int {
    using T = std::remove_pointer_t<decltype(tag)>;
    constexpr int V = vec_width<T>();
    bool vec = (D / 4) % V == 0 && all_aligned16({dqkv, cos_table, sin_table});
    for (const ebr_operand* op : {dq, dk, dv})
      vec = vec && aligned16(op->data) && op->stride_b % V == 0 && op->stride_h % V == 0 && op->stride_n % V == 0;
    const int Vr = vec ? V : 1;
    const int64_t tokens = B * N;
    if constexpr (V * sizeof(T) == 16) {
      // Partner slot in the same warp: D / V divides 32 and the partner offset D / 4 V is a power of two.
      const int64_t cpr = D / V, off = D / (4 * V);
      constexpr int kTok = 4;
      if (vec && off >= 1 && 32 % cpr == 0 && (off & (off - 1)) == 0 && 3 * H * cpr <= 1024) {
        const RopeGrid g = rope_grid(device, 3 * H * cpr, (tokens + kTok - 1) / kTok);
        ebr::layers::rope_merge_wide_kernel<T, V, kTok><<<g.blocks, g.threads, 0, st>>>(
            *dq, *dk, *dv, N, static_cast<int>(H), static_cast<int>(D), tokens, cos_table, sin_table, qscale,
            static_cast<T*>(dqkv));
        return check_launch("rope_merge");
      }
    }
    const RopeGrid g = rope_grid(device, 3 * H * (D / Vr), tokens);
    if (vec)
      ebr::layers::rope_merge_kernel<T, V><<<g.blocks, g.threads, 0, st>>>(
          *dq, *dk, *dv, N, static_cast<int>(H), static_cast<int>(D), tokens, cos_table, sin_table, qscale,
          static_cast<T*>(dqkv));
    else
      ebr::layers::rope_merge_kernel<T, 1><<<g.blocks, g.threads, 0, st>>>(
          *dq, *dk, *dv, N, static_cast<int>(H), static_cast<int>(D), tokens, cos_table, sin_table, qscale,
          static_cast<T*>(dqkv));
    return check_launch("rope_merge");
  });
}

int ebr_add_rms_norm(int dtype, int64_t rows, int64_t C, double eps, const void* x, const void* a, void* sum_out,
                     void* y, float* rstd_out, const void* post, double post_scale, void* stream) {
  int rc = check_layer_dtype(dtype, false);
  if (rc != EBR_OK) return rc;
  if (rows < 0 || C < 1 || C > (1 << 20)) return set_error(EBR_ERR_SHAPE, "add_rms_norm: bad rows / row length%s%s");
  if (rows == 0) return EBR_OK;
  if (!x || !y) return set_error(EBR_ERR_NULL, "add_rms_norm: NULL pointer%s%s");
  int device = 0;
  if ((rc = check_device(&device)) != EBR_OK) return rc;
  auto st = static_cast<cudaStream_t>(stream);
  return with_type(dtype, [&](auto* tag) -> int {
    using T = std::remove_pointer_t<decltype(tag)>;
    constexpr int V = vec_width<T>();
    const bool vec = C % V == 0 && all_aligned16({x, a, sum_out, y, post});
    const dim3 grid = flat_grid(device, rows * 32);
    if (vec)
      ebr::layers::add_rms_norm_kernel<T, V><<<grid, kThreads, 0, st>>>(
          rows, static_cast<int>(C), static_cast<float>(eps), static_cast<const T*>(x), static_cast<const T*>(a),
          static_cast<T*>(sum_out), static_cast<T*>(y), rstd_out, static_cast<const T*>(post),
          static_cast<float>(post_scale));
    else
      ebr::layers::add_rms_norm_kernel<T, 1><<<grid, kThreads, 0, st>>>(
          rows, static_cast<int>(C), static_cast<float>(eps), static_cast<const T*>(x), static_cast<const T*>(a),
          static_cast<T*>(sum_out), static_cast<T*>(y), rstd_out, static_cast<const T*>(post),
          static_cast<float>(post_scale));
    return check_launch("add_rms_norm");
  });
}

int ebr_rms_norm_bwd(int dtype, int64_t rows, int64_t C, const void* s, const float* rstd, const void* gy, void* gs,
                     void* stream) {
  int rc = check_layer_dtype(dtype, false);
  if (rc != EBR_OK) return rc;
  if (rows < 0 || C < 1 || C > (1 << 20)) return set_error(EBR_ERR_SHAPE, "rms_norm_bwd: bad rows / row length%s%s");
  if (rows == 0) return EBR_OK;
  if (!s || !rstd || !gy || !gs) return set_error(EBR_ERR_NULL, "rms_norm_bwd: NULL pointer%s%s");
  int device = 0;
  if ((rc = check_device(&device)) != EBR_OK) return rc;
  auto st = static_cast<cudaStream_t>(stream);
  return with_type(dtype, [&](auto* tag) -> int {
    using T = std::remove_pointer_t<decltype(tag)>;
    constexpr int V = vec_width<T>();
    const bool vec = C % V == 0 && all_aligned16({s, gy, gs});
    const dim3 grid = flat_grid(device, rows * 32);
    if (vec)
      ebr::layers::rms_norm_bwd_kernel<T, V><<<grid, kThreads, 0, st>>>(
          rows, static_cast<int>(C), static_cast<const T*>(s), rstd, static_cast<const T*>(gy), static_cast<T*>(gs));
    else
      ebr::layers::rms_norm_bwd_kernel<T, 1><<<grid, kThreads, 0, st>>>(
          rows, static_cast<int>(C), static_cast<const T*>(s), rstd, static_cast<const T*>(gy), static_cast<T*>(gs));
    return check_launch("rms_norm_bwd");
  });
}

int ebr_swiglu_fwd(int dtype, int64_t rows, int64_t I, const void* h, void* out, void* stream) {
  int rc = check_layer_dtype(dtype, false);
  if (rc != EBR_OK) return rc;
  if (rows < 0 || I < 1) return set_error(EBR_ERR_SHAPE, "swiglu: bad rows / width%s%s");
  if (rows == 0) return EBR_OK;
  if (!h || !out) return set_error(EBR_ERR_NULL, "swiglu: NULL pointer%s%s");
  int device = 0;
  if ((rc = check_device(&device)) != EBR_OK) return rc;
  auto st = static_cast<cudaStream_t>(stream);
  return with_type(dtype, [&](auto* tag) -> int {
    using T = std::remove_pointer_t<decltype(tag)>;
    constexpr int V = vec_width<T>();
    if (I % V == 0 && all_aligned16({h, out}))
      ebr::layers::swiglu_fwd_kernel<T, V><<<flat_grid(device, rows * (I / V)), kThreads, 0, st>>>(
          rows, I, static_cast<const T*>(h), static_cast<T*>(out));
    else
      ebr::layers::swiglu_fwd_kernel<T, 1><<<flat_grid(device, rows * I), kThreads, 0, st>>>(
          rows, I, static_cast<const T*>(h), static_cast<T*>(out));
    return check_launch("swiglu_fwd");
  });
}

int ebr_rms_norm_bwd2(int dtype, int64_t rows, int64_t C, const void* s, const float* rstd, const void* gy,
                      const void* u, void* ds, void* dgy, void* stream) {
  int rc = check_layer_dtype(dtype, false);
  if (rc != EBR_OK) return rc;
  if (rows < 0 || C < 1 || C > (1 << 20)) return set_error(EBR_ERR_SHAPE, "rms_norm_bwd2: bad rows / row length%s%s");
  if (rows == 0) return EBR_OK;
  if (!s || !rstd || !gy || !u || !ds || !dgy) return set_error(EBR_ERR_NULL, "rms_norm_bwd2: NULL pointer%s%s");
  int device = 0;
  if ((rc = check_device(&device)) != EBR_OK) return rc;
  auto st = static_cast<cudaStream_t>(stream);
  return with_type(dtype, [&](auto* tag) -> int {
    using T = std::remove_pointer_t<decltype(tag)>;
    constexpr int V = vec_width<T>();
    const dim3 grid = flat_grid(device, rows * 32);
    auto go = [&](auto kernel) {
      kernel<<<grid, kThreads, 0, st>>>(rows, static_cast<int>(C), static_cast<const T*>(s), rstd,
                                        static_cast<const T*>(gy), static_cast<const T*>(u), static_cast<T*>(ds),
                                        static_cast<T*>(dgy));
    };
    if (C % V == 0 && all_aligned16({s, gy, u, ds, dgy}))
      go(ebr::layers::rms_norm_bwd2_kernel<T, V>);
    else
      go(ebr::layers::rms_norm_bwd2_kernel<T, 1>);
    return check_launch("rms_norm_bwd2");
  });
}

int ebr_swiglu_bwd2(int dtype, int64_t rows, int64_t I, const void* h, const void* gout, const void* u, void* dh,
                    void* dgout, void* stream) {
  int rc = check_layer_dtype(dtype, false);
  if (rc != EBR_OK) return rc;
  if (rows < 0 || I < 1) return set_error(EBR_ERR_SHAPE, "swiglu_bwd2: bad rows / width%s%s");
  if (rows == 0) return EBR_OK;
  if (!h || !gout || !u || !dh || !dgout) return set_error(EBR_ERR_NULL, "swiglu_bwd2: NULL pointer%s%s");
  int device = 0;
  if ((rc = check_device(&device)) != EBR_OK) return rc;
  auto st = static_cast<cudaStream_t>(stream);
  return with_type(dtype, [&](auto* tag) -> int {
    using T = std::remove_pointer_t<decltype(tag)>;
    constexpr int V = vec_width<T>();
    if (I % V == 0 && all_aligned16({h, gout, u, dh, dgout}))
      ebr::layers::swiglu_bwd2_kernel<T, V><<<flat_grid(device, rows * (I / V)), kThreads, 0, st>>>(
          rows, I, static_cast<const T*>(h), static_cast<const T*>(gout), static_cast<const T*>(u),
          static_cast<T*>(dh), static_cast<T*>(dgout));
    else
      ebr::layers::swiglu_bwd2_kernel<T, 1><<<flat_grid(device, rows * I), kThreads, 0, st>>>(
          rows, I, static_cast<const T*>(h), static_cast<const T*>(gout), static_cast<const T*>(u),
          static_cast<T*>(dh), static_cast<T*>(dgout));
    return check_launch("swiglu_bwd2");
  });
}

int ebr_swiglu_bwd(int dtype, int64_t rows, int64_t I, const void* h, const void* gout, void* gh, void* stream) {
  int rc = check_layer_dtype(dtype, false);
  if (rc != EBR_OK) return rc;
  if (rows < 0 || I < 1) return set_error(EBR_ERR_SHAPE, "swiglu_bwd: bad rows / width%s%s");
  if (rows == 0) return EBR_OK;
  if (!h || !gout || !gh) return set_error(EBR_ERR_NULL, "swiglu_bwd: NULL pointer%s%s");
  int device = 0;
  if ((rc = check_device(&device)) != EBR_OK) return rc;
  auto st = static_cast<cudaStream_t>(stream);
  return with_type(dtype, [&](auto* tag) -> int {
    using T = std::remove_pointer_t<decltype(tag)>;
    constexpr int V = vec_width<T>();
    if (I % V == 0 && all_aligned16({h, gout, gh}))
      ebr::layers::swiglu_bwd_kernel<T, V><<<flat_grid(device, rows * (I / V)), kThreads, 0, st>>>(
          rows, I, static_cast<const T*>(h), static_cast<const T*>(gout), static_cast<T*>(gh));
    else
      ebr::layers::swiglu_bwd_kernel<T, 1><<<flat_grid(device, rows * I), kThreads, 0, st>>>(
          rows, I, static_cast<const T*>(h), static_cast<const T*>(gout), static_cast<T*>(gh));
    return check_launch("swiglu_bwd");
  });
}

size_t ebr_descent_step_scratch_floats(int64_t rows, int64_t row_elems) {
  if (rows <= 0 || row_elems <= 0) return 0;
  const int64_t chunks = (row_elems + ebr::layers::kStepChunk - 1) / ebr::layers::kStepChunk;
  return static_cast<size_t>(rows * chunks);
}

int ebr_descent_step(int dtype, int64_t rows, int64_t row_elems, double alpha, double eps, const void* v,
                     const void* g, void* z_next, float* partial, size_t partial_floats, void* stream) {
  int rc = check_layer_dtype(dtype, false);
  if (rc != EBR_OK) return rc;
  if (rows < 0 || row_elems < 1 || rows > 65535) return set_error(EBR_ERR_SHAPE, "descent_step: bad rows / row length%s%s");
  if (rows == 0) return EBR_OK;
  if (!v || !g || !z_next) return set_error(EBR_ERR_NULL, "descent_step: NULL pointer%s%s");
  if (!partial || partial_floats < ebr_descent_step_scratch_floats(rows, row_elems))
    return set_error(EBR_ERR_SCRATCH, "descent_step: partial-sum scratch missing or too small%s%s");
  int device = 0;
  if ((rc = check_device(&device)) != EBR_OK) return rc;
  auto st = static_cast<cudaStream_t>(stream);
  const int chunks = static_cast<int>((row_elems + ebr::layers::kStepChunk - 1) / ebr::layers::kStepChunk);
  const dim3 grid(static_cast<unsigned>(chunks), static_cast<unsigned>(rows));
  return with_type(dtype, [&](auto* tag) -> int {
    using T = std::remove_pointer_t<decltype(tag)>;
    constexpr int V = vec_width<T>();
    const bool vec = row_elems % V == 0 && all_aligned16({v, g, z_next});
    if (vec) {
      ebr::layers::descent_step_kernel<T, V><<<grid, kThreads, 0, st>>>(
          row_elems, chunks, alpha, static_cast<const T*>(v), static_cast<const T*>(g), static_cast<T*>(z_next),
          partial);
      rc = check_launch("descent_step");
      if (rc != EBR_OK) return rc;
      ebr::layers::sphere_kernel<T, V><<<grid, kThreads, 0, st>>>(row_elems, chunks, static_cast<float>(eps),
                                                                  static_cast<T*>(z_next), partial);
    } else {
      ebr::layers::descent_step_kernel<T, 1><<<grid, kThreads, 0, st>>>(
          row_elems, chunks, alpha, static_cast<const T*>(v), static_cast<const T*>(g), static_cast<T*>(z_next),
          partial);
      rc = check_launch("descent_step");
      if (rc != EBR_OK) return rc;
      ebr::layers::sphere_kernel<T, 1><<<grid, kThreads, 0, st>>>(row_elems, chunks, static_cast<float>(eps),
                                                                  static_cast<T*>(z_next), partial);
    }
    return check_launch("sphere");
  });
}

int ebr_qkv_rope_split(int dtype, int64_t B, int64_t N, int64_t H, int64_t D, int64_t C, const void* x,
                       int64_t x_stride, const void* w, const float* cos_table, const float* sin_table,
                       const float* qscale, void* q, void* k, void* v, void* stream) {
  if (dtype != EBR_BFLOAT16 && dtype != EBR_FLOAT16)
    return set_error(EBR_ERR_DTYPE, "qkv_rope_split: bfloat16 or float16 only%s%s");
  if (B < 0 || N < 0 || H < 1 || C < 1 || (D != 64 && D != 128) || (H * D) % 256 != 0 || C % 64 != 0 ||
      N > INT32_MAX || H * D > (INT32_MAX / 3) || C > INT32_MAX)
    return set_error(EBR_ERR_SHAPE, "qkv_rope_split: needs D = 64 or 128, H D a multiple of 256, C a multiple of 64%s%s");
  if (B * N == 0) return EBR_OK;
  if (!x || !w || !cos_table || !sin_table || !q || !k || !v)
    return set_error(EBR_ERR_NULL, "qkv_rope_split: NULL pointer%s%s");
  if (x_stride < C || x_stride % 8 != 0 || !all_aligned16({x, w, q, k, v, cos_table, sin_table}))
    return set_error(EBR_ERR_STRIDE, "qkv_rope_split: x rows need a stride >= C, a multiple of 8 elements, and 16-byte "
                                     "aligned pointers%s%s");
  int device = 0;
  int rc = check_device(&device);
  if (rc != EBR_OK) return rc;
  auto st = static_cast<cudaStream_t>(stream);
  using L = ebr::QkvRopeLayout;
  const int64_t M = B * N;
  CUtensorMap tx, tw;
  if ((rc = make_matrix_map(&tx, x, dtype, M, C, x_stride, L::kBM)) != EBR_OK) return rc;
  if ((rc = make_matrix_map(&tw, w, dtype, 3 * H * D, C, C, L::kBN)) != EBR_OK) return rc;
  const int64_t m_tiles = (M + L::kBM - 1) / L::kBM;  // a CTA takes whole 128-row m-tiles
  const int64_t cap = sm_count(device);
  const unsigned grid = static_cast<unsigned>(m_tiles < cap ? m_tiles : cap);
  auto launch = [&](auto kernel, auto* out_tag) -> int {
    using T = std::remove_pointer_t<decltype(out_tag)>;
    if ((rc = prepare_tc_kernel(reinterpret_cast<const void*>(kernel), device, L::kSmem, L::kTmemCols, L::kThreads)))
      return rc;
    kernel<<<grid, L::kThreads, L::kSmem, st>>>(tx, tw, M, static_cast<int>(C), static_cast<int>(N), static_cast<int>(H),
                                                cos_table, sin_table, qscale, static_cast<T*>(q), static_cast<T*>(k),
                                                static_cast<T*>(v));
    return check_launch("tc_qkv_rope_kernel");
  };
  if (dtype == EBR_BFLOAT16)
    return D == 64 ? launch(ebr::tc_qkv_rope_kernel<__nv_bfloat16, 64>, static_cast<__nv_bfloat16*>(nullptr))
                   : launch(ebr::tc_qkv_rope_kernel<__nv_bfloat16, 128>, static_cast<__nv_bfloat16*>(nullptr));
  return D == 64 ? launch(ebr::tc_qkv_rope_kernel<__half, 64>, static_cast<__half*>(nullptr))
                 : launch(ebr::tc_qkv_rope_kernel<__half, 128>, static_cast<__half*>(nullptr));
}

int ebr_o_proj(int dtype, int64_t B, int64_t H, int64_t N, int64_t D, int64_t C_out, const ebr_operand* o,
               const void* w, void* y, void* stream) {
  if (dtype != EBR_BFLOAT16 && dtype != EBR_FLOAT16)
    return set_error(EBR_ERR_DTYPE, "o_proj: bfloat16 or float16 only%s%s");
  if (B < 0 || N < 0 || H < 1 || (D != 64 && D != 128) || C_out < 256 || C_out % 256 != 0 || B > INT32_MAX ||
      N > INT32_MAX || H * D > INT32_MAX || C_out > INT32_MAX)
    return set_error(EBR_ERR_SHAPE, "o_proj: needs D = 64 or 128 and C_out a positive multiple of 256%s%s");
  if (B * N == 0) return EBR_OK;
  int rc = check_operand(o, "o");
  if (rc != EBR_OK) return rc;
  if (!w || !y) return set_error(EBR_ERR_NULL, "o_proj: NULL pointer%s%s");
  if (!tc_operand_ok(o, B, H, N) || !all_aligned16({w, y}))
    return set_error(EBR_ERR_STRIDE, "o_proj: o needs 16-byte aligned data and strides, w / y 16-byte alignment%s%s");
  int device = 0;
  if ((rc = check_device(&device)) != EBR_OK) return rc;
  auto st = static_cast<cudaStream_t>(stream);
  using L = ebr::OProjLayout;
  CUtensorMap to, tw;
  if (make_tile_map(&to, o, dtype, B, H, N, D)) return set_error(EBR_ERR_CUDA, "o_proj: tensor map for o%s%s");
  if ((rc = make_matrix_map(&tw, w, dtype, C_out, H * D, H * D, L::kBN)) != EBR_OK) return rc;
  const int64_t m_tiles = B * ((N + L::kBM - 1) / L::kBM);
  const int64_t cap = sm_count(device);
  const unsigned grid = static_cast<unsigned>(m_tiles < cap ? m_tiles : cap);
  auto launch = [&](auto kernel, auto* out_tag) -> int {
    using T = std::remove_pointer_t<decltype(out_tag)>;
    if ((rc = prepare_tc_kernel(reinterpret_cast<const void*>(kernel), device, L::kSmem, L::kTmemCols, L::kThreads)))
      return rc;
    kernel<<<grid, L::kThreads, L::kSmem, st>>>(to, tw, static_cast<int>(B), static_cast<int>(H), static_cast<int>(N),
                                                static_cast<int>(C_out), static_cast<T*>(y));
    return check_launch("tc_o_proj_kernel");
  };
  if (dtype == EBR_BFLOAT16)
    return D == 64 ? launch(ebr::tc_o_proj_kernel<__nv_bfloat16, 64>, static_cast<__nv_bfloat16*>(nullptr))
                   : launch(ebr::tc_o_proj_kernel<__nv_bfloat16, 128>, static_cast<__nv_bfloat16*>(nullptr));
  return D == 64 ? launch(ebr::tc_o_proj_kernel<__half, 64>, static_cast<__half*>(nullptr))
                 : launch(ebr::tc_o_proj_kernel<__half, 128>, static_cast<__half*>(nullptr));
}

int ebr_qkv_rope_merge_dx(int dtype, int64_t B, int64_t N, int64_t H, int64_t D, int64_t C, const ebr_operand* dq,
                          const ebr_operand* dk, const ebr_operand* dv, const void* w, const float* cos_table,
                          const float* sin_table, const float* qscale, const void* addend, void* dx, void* stream) {
  using L = ebr::MergeGemmLayout;
  if (dtype != EBR_BFLOAT16 && dtype != EBR_FLOAT16)
    return set_error(EBR_ERR_DTYPE, "qkv_rope_merge_dx: bfloat16 or float16 only%s%s");
  if (B < 0 || N < 0 || H < 1 || D != 64 || C != L::kC || B > INT32_MAX || N > INT32_MAX || H > 4096)
    return set_error(EBR_ERR_SHAPE, "qkv_rope_merge_dx: needs D = 64 and C = 512%s%s");
  if (B * N == 0) return EBR_OK;
  int rc = check_operand(dq, "dq");
  if (rc == EBR_OK) rc = check_operand(dk, "dk");
  if (rc == EBR_OK) rc = check_operand(dv, "dv");
  if (rc != EBR_OK) return rc;
  if (!w || !dx || !cos_table || !sin_table) return set_error(EBR_ERR_NULL, "qkv_rope_merge_dx: NULL pointer%s%s");
  if (!tc_operand_ok(dq, B, H, N) || !tc_operand_ok(dk, B, H, N) || !tc_operand_ok(dv, B, H, N) ||
      !all_aligned16({w, dx, cos_table, sin_table, addend}))
    return set_error(EBR_ERR_STRIDE, "qkv_rope_merge_dx: 16-byte aligned data and strides needed%s%s");
  int device = 0;
  if ((rc = check_device(&device)) != EBR_OK) return rc;
  auto st = static_cast<cudaStream_t>(stream);
  CUtensorMap tq, tk, tv, tw, tdx;
  if (make_tile_map(&tq, dq, dtype, B, H, N, D) || make_tile_map(&tk, dk, dtype, B, H, N, D) ||
      make_tile_map(&tv, dv, dtype, B, H, N, D))
    return set_error(EBR_ERR_CUDA, "qkv_rope_merge_dx: tensor map for dq / dk / dv%s%s");
  if ((rc = make_matrix_map(&tw, w, dtype, 3 * H * D, C, C, L::kBK)) != EBR_OK) return rc;
  if ((rc = make_sample_store_map(&tdx, dx, dtype, B, N, C)) != EBR_OK) return rc;
  const int64_t m_tiles = B * ((N + L::kBM - 1) / L::kBM);
  const int64_t cap = sm_count(device);
  const unsigned grid = static_cast<unsigned>(m_tiles < cap ? m_tiles : cap);
  auto launch = [&](auto kernel, auto* out_tag) -> int {
    using T = std::remove_pointer_t<decltype(out_tag)>;
    if ((rc = prepare_tc_kernel(reinterpret_cast<const void*>(kernel), device, L::kSmem, L::kTmemCols, L::kThreads)))
      return rc;
    kernel<<<grid, L::kThreads, L::kSmem, st>>>(tq, tk, tv, tw, static_cast<int>(B), static_cast<int>(H),
                                                static_cast<int>(N), cos_table, sin_table, qscale,
                                                static_cast<const T*>(addend), tdx);
    return check_launch("tc_merge_gemm_kernel");
  };
  if (dtype == EBR_BFLOAT16)
    return launch(ebr::tc_merge_gemm_kernel<__nv_bfloat16>, static_cast<__nv_bfloat16*>(nullptr));
  return launch(ebr::tc_merge_gemm_kernel<__half>, static_cast<__half*>(nullptr));
}

int ebr_gate_up_swiglu(int dtype, int64_t rows, int64_t C, int64_t I, const void* x, int64_t x_stride, const void* w,
                       void* h, void* act, void* stream) {
  if (dtype != EBR_BFLOAT16 && dtype != EBR_FLOAT16)
    return set_error(EBR_ERR_DTYPE, "gate_up_swiglu: bfloat16 or float16 only%s%s");
  if (rows < 0 || C < 1 || I < 1 || C % 64 != 0 || I % 128 != 0 || rows > INT32_MAX || C > INT32_MAX ||
      I > INT32_MAX / 2)
    return set_error(EBR_ERR_SHAPE, "gate_up_swiglu: needs C a multiple of 64, I a multiple of 128 and rows < 2^31%s%s");
  if (rows == 0) return EBR_OK;
  if (!x || !w || !h || !act) return set_error(EBR_ERR_NULL, "gate_up_swiglu: NULL pointer%s%s");
  if (x_stride < C || x_stride % 8 != 0 || !all_aligned16({x, w, h, act}))
    return set_error(EBR_ERR_STRIDE, "gate_up_swiglu: x rows need a stride >= C, a multiple of 8 elements, and "
                                     "16-byte aligned pointers%s%s");
  int device = 0;
  int rc = check_device(&device);
  if (rc != EBR_OK) return rc;
  auto st = static_cast<cudaStream_t>(stream);
  using L = ebr::GateUpLayout;
  CUtensorMap tx, tw, th, ta;
  if ((rc = make_matrix_map(&tx, x, dtype, rows, C, x_stride, L::kBM)) != EBR_OK) return rc;
  if ((rc = make_matrix_map(&tw, w, dtype, 2 * I, C, C, 128)) != EBR_OK) return rc;
  if ((rc = make_chunk_store_map(&th, h, dtype, rows, 2 * I, 2 * I)) != EBR_OK) return rc;
  if ((rc = make_chunk_store_map(&ta, act, dtype, rows, I, I)) != EBR_OK) return rc;
  const int64_t m_tiles = (rows + L::kBM - 1) / L::kBM;
  const int64_t cap = sm_count(device);
  const unsigned grid = static_cast<unsigned>(m_tiles < cap ? m_tiles : cap);
  auto launch = [&](auto kernel) -> int {
    if ((rc = prepare_tc_kernel(reinterpret_cast<const void*>(kernel), device, L::kSmem, L::kTmemCols, L::kThreads)))
      return rc;
    kernel<<<grid, L::kThreads, L::kSmem, st>>>(tx, tw, th, ta, rows, static_cast<int>(C), static_cast<int>(I));
    return check_launch("tc_gate_up_swiglu_kernel");
  };
  if (dtype == EBR_BFLOAT16) return launch(ebr::tc_gate_up_swiglu_kernel<__nv_bfloat16>);
  return launch(ebr::tc_gate_up_swiglu_kernel<__half>);
}

}  // extern "C"
