// capi.cu: the C ABI of include/ebr_attn.h. Validates arguments on the host, picks the kernel family for the call's
// dtype / shape / strides (the counterpart of the reference's launch plans, triton_kernels.py:612-676), builds the TMA
// tensor maps and launches on the caller's stream. Never allocates device memory and never traps.
#include <atomic>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>

#include "../../include/ebr_attn.h"
#include "simt.cuh"
#include "tc_attn.cuh"
#include "tc_bob.cuh"
#include "tc_bwd.cuh"
#include "tc_fwd.cuh"
#include "tc_short.cuh"

namespace {

using namespace ebr;

thread_local char g_last_error[512] = "";
std::atomic<uint64_t> g_launch_count{0};

int set_error(int status, const char* fmt, const char* a = "", const char* b = "") {
  std::snprintf(g_last_error, sizeof(g_last_error), fmt, a, b);
  return status;
}

int cuda_error(cudaError_t e, const char* what) {
  return set_error(EBR_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// ------------------------------------------------------------------------------------------------ device checks

constexpr int kMaxDevices = 64;
constexpr int kBoundedWaitTestSite = 9001;  // the site ebr_attn_test_bounded_wait's wait records

int check_device(int* device_out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  static std::atomic<int> arch[kMaxDevices];  // 0 unknown, else major * 10 + minor
  int a = (dev < kMaxDevices) ? arch[dev].load() : 0;
  if (a == 0) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    a = major * 10 + minor;
    if (dev < kMaxDevices) arch[dev].store(a);
  }
  if (a != 100) return set_error(EBR_ERR_DEVICE, "ebr_attn needs an sm_100 (B200) device%s%s");
  *device_out = dev;
  return EBR_OK;
}

// Raise a kernel's dynamic shared memory limit once per device, and refuse a launch shape under which more CTAs
// could share an SM than its tensor memory (512 columns) can serve: tcgen05.alloc would then block.
int prepare_tc_kernel(const void* kernel, int device, uint32_t smem, uint32_t tmem_cols, int threads = 128) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> verdicts;
  std::lock_guard<std::mutex> lock(mu);
  auto it = verdicts.find({kernel, device});
  if (it != verdicts.end()) return it->second;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute");
  int blocks = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, threads, smem);
  if (e != cudaSuccess) return cuda_error(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
  const int verdict = (blocks >= 1 && static_cast<uint32_t>(blocks) * tmem_cols <= 512u)
                          ? EBR_OK
                          : set_error(EBR_ERR_CUDA, "tensor-memory budget check failed%s%s");
  verdicts[{kernel, device}] = verdict;
  return verdict;
}

int check_launch(const char* what) {
  g_launch_count.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? EBR_OK : cuda_error(e, what);
}

// ------------------------------------------------------------------------------------------------ argument checks

size_t elem_size(int dtype) {
  switch (dtype) {
    case EBR_FLOAT32: return 4;
    case EBR_FLOAT16:
    case EBR_BFLOAT16: return 2;
    case EBR_FLOAT64: return 8;
    default: return 0;
  }
}
size_t stat_size(int dtype) { return dtype == EBR_FLOAT64 ? 8 : 4; }

int check_shape(int dtype, int64_t B, int64_t H, int64_t N, int64_t D) {
  if (elem_size(dtype) == 0) return set_error(EBR_ERR_DTYPE, "unknown dtype%s%s");
  if (B < 0 || H < 0 || N < 0) return set_error(EBR_ERR_SHAPE, "negative size%s%s");
  if (D < 1 || D > 256) return set_error(EBR_ERR_SHAPE, "head dim must be in [1, 256]%s%s");
  if (N > (int64_t{1} << 30) || H > (int64_t{1} << 30) || B > (int64_t{1} << 30))
    return set_error(EBR_ERR_SHAPE, "size too large%s%s");
  // Bound the products before any size arithmetic: the kernels index slices with 32-bit B * H, and rows / scratch
  // sizes are B * H * N (each factor <= 2^30, so B * H fits and (B * H) * N cannot overflow once B * H < 2^31).
  if (B * H >= (int64_t{1} << 31) || B * H * N >= (int64_t{1} << 40))
    return set_error(EBR_ERR_SHAPE, "B * H or B * H * N too large%s%s");
  return EBR_OK;
}

int check_operand(const ebr_operand* op, const char* name, bool optional = false) {
  if (!op) return optional ? EBR_OK : set_error(EBR_ERR_NULL, "operand %s is NULL%s", name);
  if (!op->data && !optional) return set_error(EBR_ERR_NULL, "operand %s has no data%s", name);
  if (op->stride_b < 0 || op->stride_h < 0 || op->stride_n < 0)
    return set_error(EBR_ERR_STRIDE, "operand %s has a negative stride%s", name);
  return EBR_OK;
}

template <typename T>
Strided<T> strided(const ebr_operand* op) {
  if (!op || !op->data) return Strided<T>{nullptr, 0, 0, 0};
  return Strided<T>{static_cast<const T*>(op->data), op->stride_b, op->stride_h, op->stride_n};
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Internal: a TMA tensor map could not be encoded for these operands; the CUDA-core kernels take the call instead.
constexpr int kNoTensorMap = -1;

// ------------------------------------------------------------------------------------------------ TMA tensor maps

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
  static EncodeTiled fn = []() -> EncodeTiled {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiled>(p);
  }();
  return fn;
}

// A stride the tensor-core path can take: 16-byte multiple (TMA), or irrelevant because the dim has size 1.
bool tma_stride_ok(int64_t stride_elems, int64_t extent) {
  return extent <= 1 || ((stride_elems * 2) % 16 == 0 && stride_elems * 2 < (int64_t{1} << 40));
}

bool tc_operand_ok(const ebr_operand* op, int64_t B, int64_t H, int64_t N) {
  if (!op || !op->data) return true;  // a zero operand is not loaded
  return aligned16(op->data) && tma_stride_ok(op->stride_n, N) && tma_stride_ok(op->stride_h, H) &&
         tma_stride_ok(op->stride_b, B) && (op->stride_n > 0 || N <= 1);
}

// [B, H, N, D] 16-bit operand -> 4-D tensor map (D, N, H, B), box 64 x box_rows x 1 x 1, 128-byte swizzle, zero
// fill outside the tensor.
int make_tile_map(CUtensorMap* map, const ebr_operand* op, int dtype, int64_t B, int64_t H, int64_t N, int64_t D,
                  uint32_t box_rows = 128) {
  EncodeTiled enc = encode_fn();
  if (!enc) return set_error(EBR_ERR_CUDA, "cuTensorMapEncodeTiled unavailable%s%s");
  auto fix = [](int64_t stride, int64_t extent) -> cuuint64_t {
    return static_cast<cuuint64_t>(extent <= 1 ? 16 : stride * 2);
  };
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(H),
                              static_cast<cuuint64_t>(B)};
  const cuuint64_t strides[3] = {fix(op->stride_n, N), fix(op->stride_h, H), fix(op->stride_b, B)};
  const cuuint32_t box[4] = {64, box_rows, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, dtype == EBR_BFLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                   const_cast<void*>(op->data), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(EBR_ERR_CUDA, "cuTensorMapEncodeTiled failed%s%s");
  return EBR_OK;
}

// 16-bit 4-D tensor map with an explicit box: dims (D, N, hs, bs) with element strides (sn, sh, sb), box
// (64, box_n, box_h, 1), 128-byte swizzle, zero fill outside the tensor (the short-sequence kernels' tiles).
int make_box_map(CUtensorMap* map, const void* data, int dtype, int64_t D, int64_t N, int64_t hs, int64_t bs,
                 int64_t sn, int64_t sh, int64_t sb, uint32_t box_n, uint32_t box_h) {
  EncodeTiled enc = encode_fn();
  if (!enc) return set_error(EBR_ERR_CUDA, "cuTensorMapEncodeTiled unavailable%s%s");
  auto fix = [](int64_t stride, int64_t extent) -> cuuint64_t {
    return static_cast<cuuint64_t>(extent <= 1 ? 16 : stride * 2);
  };
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(hs),
                              static_cast<cuuint64_t>(bs)};
  const cuuint64_t strides[3] = {fix(sn, N), fix(sh, hs), fix(sb, bs)};
  const cuuint32_t box[4] = {64, box_n, box_h, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, dtype == EBR_BFLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                   const_cast<void*>(data), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(EBR_ERR_CUDA, "cuTensorMapEncodeTiled failed%s%s");
  return EBR_OK;
}

// Tile geometry of a short-sequence (N <= 128) launch. Slices are packed floor(128 / N) per tile along one axis of
// B * H when every operand reaches slice (b, h) at b * stride_b + h * stride_h with stride_b = H * stride_h (any
// contiguous or head-major tensor); otherwise the tile holds a divisor of H slices of one batch row.
struct ShortPlan {
  ShortGeom geo;
  int64_t hs, bs;  // tensor-map extents of the slice axes
  bool flat;       // B * H slices read as one axis
};

ShortPlan short_plan(int64_t B, int64_t H, int64_t N, std::initializer_list<const ebr_operand*> ops) {
  bool flat = true;
  for (const ebr_operand* op : ops)
    if (op && op->data && B > 1 && op->stride_b != H * op->stride_h) flat = false;
  ShortPlan p{};
  p.flat = flat;
  p.hs = flat ? B * H : H;
  p.bs = flat ? 1 : B;
  int64_t per = kTile / N;
  if (per > p.hs) per = p.hs;
  if (!flat)
    while (per > 1 && H % per) --per;
  if (per < 1) per = 1;
  p.geo.N = static_cast<int>(N);
  p.geo.per = static_cast<int>(per);
  p.geo.hs = static_cast<int>(p.hs);
  p.geo.tiles_per_b = static_cast<int>((p.hs + per - 1) / per);
  p.geo.tiles = static_cast<int>(p.geo.tiles_per_b * p.bs);
  return p;
}

// An input operand's short-sequence map under `plan`.
int make_short_map(CUtensorMap* map, const ebr_operand* op, int dtype, const ShortPlan& plan, int64_t D) {
  return make_box_map(map, op->data, dtype, D, plan.geo.N, plan.hs, plan.bs, op->stride_n, op->stride_h,
                      op->stride_b, static_cast<uint32_t>(plan.geo.N), static_cast<uint32_t>(plan.geo.per));
}
// A contiguous [B, H, N, D] output's map under `plan`.
int make_short_out_map(CUtensorMap* map, void* data, int dtype, const ShortPlan& plan, int64_t H, int64_t D) {
  const int64_t N = plan.geo.N;
  return make_box_map(map, data, dtype, D, N, plan.hs, plan.bs, D, N * D, H * N * D, static_cast<uint32_t>(N),
                      static_cast<uint32_t>(plan.geo.per));
}

bool tc_eligible(int dtype, int64_t D, std::initializer_list<const ebr_operand*> ops, int64_t B, int64_t H, int64_t N) {
  if (dtype != EBR_BFLOAT16 && dtype != EBR_FLOAT16) return false;
  if (D != 64 && D != 128) return false;
  for (const ebr_operand* op : ops)
    if (!tc_operand_ok(op, B, H, N)) return false;
  return true;
}

int simt_grid(int64_t rows) {
  const int64_t cap = 148 * 32;
  return static_cast<int>(rows < cap ? rows : cap);
}

// ------------------------------------------------------------------------------------------------ forward

template <typename T>
int launch_simt_fwd(int64_t B, int64_t H, int64_t N, int64_t D, double scale, const ebr_operand* q,
                    const ebr_operand* k, const ebr_operand* v, void* o, void* lse, cudaStream_t st) {
  using C = typename Elem<T>::C;
  const int64_t rows = B * H * N;
  const size_t smem = (D + kSimtThreads + 8) * sizeof(C);
  simt_fwd<T><<<simt_grid(rows), kSimtThreads, smem, st>>>(rows, static_cast<int>(H), static_cast<int>(N),
                                                             static_cast<int>(D), scale, strided<T>(q), strided<T>(k),
                                                             strided<T>(v), static_cast<T*>(o), static_cast<C*>(lse));
  return check_launch("simt_fwd");
}

int sm_count(int device) {
  static std::atomic<int> counts[kMaxDevices];
  int c = counts[device].load();
  if (c == 0) {
    cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, device);
    if (c <= 0) c = 148;
    counts[device].store(c);
  }
  return c;
}

template <typename T, int D>
int launch_tc_fwd_short(int device, int dtype, int64_t B, int64_t H, int64_t N, double scale, const ebr_operand* q,
                        const ebr_operand* k, const ebr_operand* v, void* o, void* lse, cudaStream_t st) {
  using L = FwdShortLayout<D>;
  const ShortPlan plan = short_plan(B, H, N, {q, k, v});
  CUtensorMap tq, tk, tv, to;
  if (make_short_map(&tq, q, dtype, plan, D) || make_short_map(&tk, k, dtype, plan, D) ||
      make_short_map(&tv, v, dtype, plan, D) || make_short_out_map(&to, o, dtype, plan, H, D))
    return kNoTensorMap;
  const void* fn = reinterpret_cast<const void*>(tc_fwd_short_kernel<T, D>);
  int s = prepare_tc_kernel(fn, device, L::kSmem, L::kTmemCols, L::kThreads);
  if (s) return s;
  const int cap = L::kCtasPerSm * sm_count(device);
  const unsigned grid = static_cast<unsigned>(plan.geo.tiles < cap ? plan.geo.tiles : cap);
  tc_fwd_short_kernel<T, D><<<grid, L::kThreads, L::kSmem, st>>>(tq, tk, tv, to, static_cast<float*>(lse), plan.geo,
                                                                  static_cast<float>(scale));
  return check_launch("tc_fwd_short_kernel");
}

template <typename T, int D>
int launch_tc_fwd_pair(int device, int dtype, int64_t B, int64_t H, int64_t N, double scale, const ebr_operand* q,
                       const ebr_operand* k, const ebr_operand* v, void* o, void* lse, cudaStream_t st) {
  using L = FwdPairLayout<D>;
  CUtensorMap tq, tk, tv;  // Q in 128-row boxes, K / V in 64-row boxes (kKeyTile)
  if (make_tile_map(&tq, q, dtype, B, H, N, D) || make_tile_map(&tk, k, dtype, B, H, N, D, kKeyTile) ||
      make_tile_map(&tv, v, dtype, B, H, N, D, kKeyTile))
    return kNoTensorMap;
  const void* fn = reinterpret_cast<const void*>(tc_fwd_pair_kernel<T, D>);
  int s = prepare_tc_kernel(fn, device, L::kSmem, L::kTmemCols, L::kThreads);
  if (s) return s;
  const int64_t n_qt = (N + kTile - 1) / kTile;
  const int64_t items = B * H * ((n_qt + 1) / 2);
  const int64_t cap = sm_count(device);
  const unsigned grid = static_cast<unsigned>(items < cap ? items : cap);
  tc_fwd_pair_kernel<T, D><<<grid, L::kThreads, L::kSmem, st>>>(tq, tk, tv, static_cast<T*>(o),
                                                                 static_cast<float*>(lse), static_cast<int>(B * H),
                                                                 static_cast<int>(H), static_cast<int>(N),
                                                                 static_cast<float>(scale));
  return check_launch("tc_fwd_pair_kernel");
}

// ------------------------------------------------------------------------------------------------ backward

template <typename T>
int launch_simt_bwd(int64_t B, int64_t H, int64_t N, int64_t D, double scale, const ebr_operand* q,
                    const ebr_operand* k, const ebr_operand* v, const void* o, const void* lse,
                    const ebr_operand* dout, void* dq, void* dk, void* dv, void* scratch, cudaStream_t st) {
  using C = typename Elem<T>::C;
  const int64_t rows = B * H * N;
  C* di = static_cast<C*>(scratch);
  simt_bwd_row<T><<<simt_grid(rows), kSimtThreads, (2 * D + kSimtThreads + 8) * sizeof(C), st>>>(
      rows, static_cast<int>(H), static_cast<int>(N), static_cast<int>(D), scale, strided<T>(q), strided<T>(k),
      strided<T>(v), static_cast<const T*>(o), static_cast<const C*>(lse), strided<T>(dout), static_cast<T*>(dq), di);
  int s = check_launch("simt_bwd_row");
  if (s) return s;
  simt_bwd_col<T><<<simt_grid(rows), kSimtThreads, (2 * D + 2 * kSimtThreads) * sizeof(C), st>>>(
      rows, static_cast<int>(H), static_cast<int>(N), static_cast<int>(D), scale, strided<T>(q), strided<T>(k),
      strided<T>(v), static_cast<const C*>(lse), strided<T>(dout), di, static_cast<T*>(dk), static_cast<T*>(dv));
  return check_launch("simt_bwd_col");
}

template <typename T, int D>
int launch_tc_bwd_short(int device, int dtype, int64_t B, int64_t H, int64_t N, double scale, const ebr_operand* q,
                        const ebr_operand* k, const ebr_operand* v, const void* o, const void* lse,
                        const ebr_operand* dout, void* dq, void* dk, void* dv, cudaStream_t st) {
  using L = BwdShortLayout<D>;
  const ShortPlan plan = short_plan(B, H, N, {q, k, v, dout});
  CUtensorMap tq, tk, tv, tdo, tdq, tdk, tdv;
  if (make_short_map(&tq, q, dtype, plan, D) || make_short_map(&tk, k, dtype, plan, D) ||
      make_short_map(&tv, v, dtype, plan, D) || make_short_map(&tdo, dout, dtype, plan, D) ||
      make_short_out_map(&tdq, dq, dtype, plan, H, D) || make_short_out_map(&tdk, dk, dtype, plan, H, D) ||
      make_short_out_map(&tdv, dv, dtype, plan, H, D))
    return kNoTensorMap;
  int s = prepare_tc_kernel(reinterpret_cast<const void*>(tc_bwd_short_kernel<T, D>), device, L::kSmem,
                            L::kTmemCols, L::kThreads);
  if (s) return s;
  const int cap = L::kCtasPerSm * sm_count(device);
  const unsigned grid = static_cast<unsigned>(plan.geo.tiles < cap ? plan.geo.tiles : cap);
  tc_bwd_short_kernel<T, D><<<grid, L::kThreads, L::kSmem, st>>>(
      tq, tk, tv, tdo, tdq, tdk, tdv, static_cast<const T*>(o), static_cast<const float*>(lse), static_cast<T*>(dq),
      static_cast<T*>(dk), static_cast<T*>(dv), plan.geo, static_cast<float>(scale));
  return check_launch("tc_bwd_short_kernel");
}

template <typename T, int D>
int launch_tc_bwd_pipe(int device, int dtype, int64_t B, int64_t H, int64_t N, double scale, const ebr_operand* q,
                       const ebr_operand* k, const ebr_operand* v, const void* o, const void* lse,
                       const ebr_operand* dout, void* dq, void* dk, void* dv, void* scratch, cudaStream_t st) {
  CUtensorMap tq, tk, tv, tdo, tq64, tk64, tv64, tdo64;
  if (make_tile_map(&tq, q, dtype, B, H, N, D) || make_tile_map(&tk, k, dtype, B, H, N, D) ||
      make_tile_map(&tv, v, dtype, B, H, N, D) || make_tile_map(&tdo, dout, dtype, B, H, N, D) ||
      make_tile_map(&tq64, q, dtype, B, H, N, D, 64) || make_tile_map(&tk64, k, dtype, B, H, N, D, 64) ||
      make_tile_map(&tv64, v, dtype, B, H, N, D, 64) || make_tile_map(&tdo64, dout, dtype, B, H, N, D, 64))
    return kNoTensorMap;
  using LR = BwdRowLayout<D>;
  using LC = BwdColLayout<D>;
  const void* fq = reinterpret_cast<const void*>(tc_bwd_dq_split_kernel<T, D>);
  const void* fk = reinterpret_cast<const void*>(tc_bwd_dkdv_split_kernel<T, D>);
  int s = prepare_tc_kernel(fq, device, LR::kSmem, LR::kTmemCols, LR::kThreads);
  if (s) return s;
  s = prepare_tc_kernel(fk, device, LC::kSmem, LC::kTmemCols, LC::kThreads);
  if (s) return s;
  const int64_t items = B * H * ((N + kTile - 1) / kTile);  // 128-row query tiles (row pass) = key tiles (column)
  const int64_t cap = sm_count(device);
  const unsigned grid = static_cast<unsigned>(items < cap ? items : cap);
  float* di = static_cast<float*>(scratch);
  const int BH = static_cast<int>(B * H), Hi = static_cast<int>(H), Ni = static_cast<int>(N);
  // O is contiguous [B, H, N, D]: the row pass stages it by TMA with Q and dO (for D_i = <dO_i, O_i>).
  const ebr_operand oo{o, H * N * D, N * D, D};
  CUtensorMap to;
  if (make_tile_map(&to, &oo, dtype, B, H, N, D)) return kNoTensorMap;
  tc_bwd_dq_split_kernel<T, D><<<grid, LR::kThreads, LR::kSmem, st>>>(
      tq, tk64, tv64, tdo, to, static_cast<const float*>(lse), di, static_cast<T*>(dq), BH, Hi, Ni,
      static_cast<float>(scale));
  if ((s = check_launch("tc_bwd_dq_split_kernel"))) return s;
  tc_bwd_dkdv_split_kernel<T, D><<<grid, LC::kThreads, LC::kSmem, st>>>(
      tk, tv, tq64, tdo64, static_cast<const float*>(lse), di, static_cast<T*>(dk), static_cast<T*>(dv), BH, Hi, Ni,
      static_cast<float>(scale));
  return check_launch("tc_bwd_dkdv_split_kernel");
}

// ------------------------------------------------------------------------------------------------ double backward

template <typename T>
int launch_simt_bob(int64_t B, int64_t H, int64_t N, int64_t D, double scale, const ebr_operand* q,
                    const ebr_operand* k, const ebr_operand* v, const void* o, const void* lse,
                    const ebr_operand* dout, const ebr_operand* gq, const ebr_operand* gk, const ebr_operand* gv,
                    void* hq, void* hk, void* hv, void* hdo, void* scratch, cudaStream_t st) {
  using C = typename Elem<T>::C;
  const int64_t rows = B * H * N;
  C* stats = static_cast<C*>(scratch);
  simt_bob_row<T><<<simt_grid(rows), kSimtThreads, (3 * D + 4 * kSimtThreads + 8) * sizeof(C), st>>>(
      rows, static_cast<int>(H), static_cast<int>(N), static_cast<int>(D), scale, strided<T>(q), strided<T>(k),
      strided<T>(v), static_cast<const T*>(o), static_cast<const C*>(lse), strided<T>(dout), strided<T>(gq),
      strided<T>(gk), strided<T>(gv), static_cast<T*>(hq), static_cast<T*>(hdo), stats);
  int s = check_launch("simt_bob_row");
  if (s) return s;
  simt_bob_col<T><<<simt_grid(rows), kSimtThreads, (4 * D + 3 * kSimtThreads) * sizeof(C), st>>>(
      rows, static_cast<int>(H), static_cast<int>(N), static_cast<int>(D), scale, strided<T>(q), strided<T>(k),
      strided<T>(v), static_cast<const C*>(lse), strided<T>(dout), strided<T>(gq), strided<T>(gk), strided<T>(gv),
      static_cast<T*>(hk), static_cast<T*>(hv), stats);
  return check_launch("simt_bob_col");
}

template <typename T, int D>
int launch_tc_bob_pipe(int device, int dtype, int64_t B, int64_t H, int64_t N, double scale, const ebr_operand* q,
                       const ebr_operand* k, const ebr_operand* v, const void* o, const void* lse,
                       const ebr_operand* dout, const ebr_operand* gq, const ebr_operand* gk, const ebr_operand* gv,
                       void* hq, void* hk, void* hv, void* hdo, void* scratch, cudaStream_t st) {
  using L = BobPipeLayout<D>;
  const bool has[3] = {gq && gq->data, gk && gk->data, gv && gv->data};
  const uint32_t flags = (has[0] ? 1u : 0u) | (has[1] ? 2u : 0u) | (has[2] ? 4u : 0u);
  CUtensorMap tq, tdo, tgq, tk, tv, tgk, tgv, tq64, tdo64, tgq64, tk64, tv64, tgk64, tgv64;
  if (make_tile_map(&tq, q, dtype, B, H, N, D) || make_tile_map(&tdo, dout, dtype, B, H, N, D) ||
      make_tile_map(&tk, k, dtype, B, H, N, D) || make_tile_map(&tv, v, dtype, B, H, N, D) ||
      make_tile_map(&tq64, q, dtype, B, H, N, D, 64) || make_tile_map(&tdo64, dout, dtype, B, H, N, D, 64) ||
      make_tile_map(&tk64, k, dtype, B, H, N, D, 64) || make_tile_map(&tv64, v, dtype, B, H, N, D, 64))
    return kNoTensorMap;
  // An absent cotangent's maps are never read (its loads and products are skipped); any valid map fills the slot.
  const ebr_operand* gs[3] = {gq, gk, gv};
  CUtensorMap* big[3] = {&tgq, &tgk, &tgv};
  CUtensorMap* small[3] = {&tgq64, &tgk64, &tgv64};
  for (int i = 0; i < 3; ++i) {
    if (!has[i]) {
      *big[i] = tq;
      *small[i] = tq64;
    } else if (make_tile_map(big[i], gs[i], dtype, B, H, N, D) || make_tile_map(small[i], gs[i], dtype, B, H, N, D, 64)) {
      return kNoTensorMap;
    }
  }
  const void* f0 = reinterpret_cast<const void*>(tc_bob_row_pipe_kernel<T, D, 0>);
  const void* f1 = reinterpret_cast<const void*>(tc_bob_row_pipe_kernel<T, D, 1>);
  const void* f2 = reinterpret_cast<const void*>(tc_bob_col_pipe_kernel<T, D>);
  int s = prepare_tc_kernel(f0, device, L::kSmem, 256, L::kThreads);
  if (s || (s = prepare_tc_kernel(f1, device, L::kSmem, 512, L::kThreads)) ||
      (s = prepare_tc_kernel(f2, device, L::kSmem, 512, L::kThreads)))
    return s;
  const int64_t items = B * H * ((N + kTile - 1) / kTile);
  const int64_t cap = sm_count(device);
  const unsigned grid = static_cast<unsigned>(items < cap ? items : cap);
  float* stats = static_cast<float*>(scratch);
  const int BH = static_cast<int>(B * H), Hi = static_cast<int>(H), Ni = static_cast<int>(N);
  const float sc = static_cast<float>(scale);
  tc_bob_row_pipe_kernel<T, D, 0><<<grid, L::kThreads, L::kSmem, st>>>(
      tq, tdo, tgq, tk64, tv64, tgk64, tgv64, static_cast<const T*>(o), static_cast<const float*>(lse), stats,
      nullptr, nullptr, BH, Hi, Ni, sc, flags);
  if ((s = check_launch("tc_bob_row_pipe_kernel<0>"))) return s;
  tc_bob_row_pipe_kernel<T, D, 1><<<grid, L::kThreads, L::kSmem, st>>>(
      tq, tdo, tgq, tk64, tv64, tgk64, tgv64, static_cast<const T*>(o), static_cast<const float*>(lse), stats,
      static_cast<T*>(hq), static_cast<T*>(hdo), BH, Hi, Ni, sc, flags);
  if ((s = check_launch("tc_bob_row_pipe_kernel<1>"))) return s;
  tc_bob_col_pipe_kernel<T, D><<<grid, L::kThreads, L::kSmem, st>>>(
      tk, tv, tgk, tgv, tq64, tdo64, tgq64, static_cast<const float*>(lse), stats, static_cast<T*>(hk),
      static_cast<T*>(hv), BH, Hi, Ni, sc, flags);
  return check_launch("tc_bob_col_pipe_kernel");
}

// D = 64: the statistics pass and the two output passes of tc_bob.cuh.
template <typename T>
int launch_tc_bob_split(int device, int dtype, int64_t B, int64_t H, int64_t N, double scale, const ebr_operand* q,
                        const ebr_operand* k, const ebr_operand* v, const void* o, const void* lse,
                        const ebr_operand* dout, const ebr_operand* gq, const ebr_operand* gk, const ebr_operand* gv,
                        void* hq, void* hk, void* hv, void* hdo, void* scratch, cudaStream_t st) {
  constexpr int D = 64;
  using L0 = BobSplitLayout<0>;
  using LR = BobSplitLayout<1>;
  using LC = BobSplitLayout<2>;
  const bool has[3] = {gq && gq->data, gk && gk->data, gv && gv->data};
  const uint32_t flags = (has[0] ? 1u : 0u) | (has[1] ? 2u : 0u) | (has[2] ? 4u : 0u);
  CUtensorMap tq, tdo, tgq, tk, tv, tgk, tgv, tq64, tdo64, tgq64, tk64, tv64, tgk64, tgv64;
  if (make_tile_map(&tq, q, dtype, B, H, N, D) || make_tile_map(&tdo, dout, dtype, B, H, N, D) ||
      make_tile_map(&tk, k, dtype, B, H, N, D) || make_tile_map(&tv, v, dtype, B, H, N, D) ||
      make_tile_map(&tq64, q, dtype, B, H, N, D, 64) || make_tile_map(&tdo64, dout, dtype, B, H, N, D, 64) ||
      make_tile_map(&tk64, k, dtype, B, H, N, D, 64) || make_tile_map(&tv64, v, dtype, B, H, N, D, 64))
    return kNoTensorMap;
  // An absent cotangent's maps are never read (its loads and products are skipped); any valid map fills the slot.
  const ebr_operand* gs[3] = {gq, gk, gv};
  CUtensorMap* big[3] = {&tgq, &tgk, &tgv};
  CUtensorMap* small[3] = {&tgq64, &tgk64, &tgv64};
  for (int i = 0; i < 3; ++i) {
    if (!has[i]) {
      *big[i] = tq;
      *small[i] = tq64;
    } else if (make_tile_map(big[i], gs[i], dtype, B, H, N, D) || make_tile_map(small[i], gs[i], dtype, B, H, N, D, 64)) {
      return kNoTensorMap;
    }
  }
  const void* f0 = reinterpret_cast<const void*>(tc_bob_stats_kernel<T>);
  const void* f1 = reinterpret_cast<const void*>(tc_bob_out_kernel<T, false>);
  const void* f2 = reinterpret_cast<const void*>(tc_bob_out_kernel<T, true>);
  int s = prepare_tc_kernel(f0, device, L0::kSmem, L0::kTmemCols, L0::kThreads);
  if (s || (s = prepare_tc_kernel(f1, device, LR::kSmem, LR::kTmemCols, LR::kThreads)) ||
      (s = prepare_tc_kernel(f2, device, LC::kSmem, LC::kTmemCols, LC::kThreads)))
    return s;
  const int64_t items = B * H * ((N + kTile - 1) / kTile);
  const int64_t cap = sm_count(device);
  const unsigned grid = static_cast<unsigned>(items < cap ? items : cap);
  float* stats = static_cast<float*>(scratch);
  const int BH = static_cast<int>(B * H), Hi = static_cast<int>(H), Ni = static_cast<int>(N);
  const float sc = static_cast<float>(scale);
  const float* lsef = static_cast<const float*>(lse);
  tc_bob_stats_kernel<T><<<grid, L0::kThreads, L0::kSmem, st>>>(tq, tdo, tgq, tk64, tv64, tgk64, tgv64,
                                                                 static_cast<const T*>(o), lsef, stats, BH, Hi, Ni, sc,
                                                                 flags);
  if ((s = check_launch("tc_bob_stats_kernel"))) return s;
  tc_bob_out_kernel<T, false><<<grid, LR::kThreads, LR::kSmem, st>>>(tq, tdo, tgq, tq, tk64, tgk64, tv64, tgv64, lsef,
                                                                     stats, static_cast<T*>(hq), static_cast<T*>(hdo),
                                                                     BH, Hi, Ni, sc, flags);
  if ((s = check_launch("tc_bob_out_kernel<rows>"))) return s;
  tc_bob_out_kernel<T, true><<<grid, LC::kThreads, LC::kSmem, st>>>(tk, tv, tgk, tgv, tq64, tgq64, tdo64, tq64, lsef,
                                                                    stats, static_cast<T*>(hk), static_cast<T*>(hv),
                                                                    BH, Hi, Ni, sc, flags);
  return check_launch("tc_bob_out_kernel<cols>");
}

template <typename T>
int launch_tc_bob_short(int device, int dtype, int64_t B, int64_t H, int64_t N, double scale, const ebr_operand* q,
                        const ebr_operand* k, const ebr_operand* v, const void* o, const void* lse,
                        const ebr_operand* dout, const ebr_operand* gq, const ebr_operand* gk, const ebr_operand* gv,
                        void* hq, void* hk, void* hv, void* hdo, cudaStream_t st) {
  using L = BobShortLayout;
  constexpr int D = 64;
  const ShortPlan plan = short_plan(B, H, N, {q, k, v, dout, gq, gk, gv});
  CUtensorMap tq, tk, tv, tdo, tgq, tgk, tgv, thq, thk, thv, thdo;
  uint32_t zero_mask = 0;
  const ebr_operand* gs[3] = {gq, gk, gv};
  CUtensorMap* gm[3] = {&tgq, &tgk, &tgv};
  if (make_short_map(&tq, q, dtype, plan, D) || make_short_map(&tk, k, dtype, plan, D) ||
      make_short_map(&tv, v, dtype, plan, D) || make_short_map(&tdo, dout, dtype, plan, D) ||
      make_short_out_map(&thq, hq, dtype, plan, H, D) || make_short_out_map(&thk, hk, dtype, plan, H, D) ||
      make_short_out_map(&thv, hv, dtype, plan, H, D) || make_short_out_map(&thdo, hdo, dtype, plan, H, D))
    return kNoTensorMap;
  for (int i = 0; i < 3; ++i) {
    if (!gs[i] || !gs[i]->data) {
      zero_mask |= 1u << i;
      *gm[i] = tq;  // never read
    } else if (make_short_map(gm[i], gs[i], dtype, plan, D)) {
      return kNoTensorMap;
    }
  }
  int s = prepare_tc_kernel(reinterpret_cast<const void*>(tc_bob_short_kernel<T>), device, L::kSmem, L::kTmemCols);
  if (s) return s;
  const int cap = sm_count(device);
  const unsigned grid = static_cast<unsigned>(plan.geo.tiles < cap ? plan.geo.tiles : cap);
  tc_bob_short_kernel<T><<<grid, 128, L::kSmem, st>>>(tq, tk, tv, tdo, tgq, tgk, tgv, thq, thk, thv, thdo,
                                                      static_cast<const T*>(o), static_cast<const float*>(lse),
                                                      plan.geo, static_cast<float>(scale), zero_mask);
  return check_launch("tc_bob_short_kernel");
}

// Built-in row scratch of ebr_attn_bwd_noalloc (see include/ebr_attn.h). Host code must not pass the symbol itself
// to a kernel: it names a host-side stand-in. noalloc_scratch() returns this device's address of it.
static __device__ __align__(256) unsigned char g_bwd_noalloc_scratch[EBR_ATTN_NOALLOC_SCRATCH_BYTES];

using CtxGetCurrent = CUresult (*)(CUcontext*);

CtxGetCurrent ctx_get_current_fn() {
  static CtxGetCurrent fn = []() -> CtxGetCurrent {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<CtxGetCurrent>(p);
  }();
  return fn;
}

// The address of g_bwd_noalloc_scratch in the calling thread's current CUDA context, looked up with
// cudaGetSymbolAddress once per context (a symbol has one address per context: the primary context of each device,
// or a context the caller created with the driver API). Up to kMaxScratchContexts contexts are remembered at once.
int noalloc_scratch(void** out) {
  constexpr int kMaxScratchContexts = 64;
  static std::mutex mu;
  static CUcontext ctxs[kMaxScratchContexts] = {};
  static void* ptrs[kMaxScratchContexts] = {};
  static int next = 0;
  CtxGetCurrent get_ctx = ctx_get_current_fn();
  if (!get_ctx) return set_error(EBR_ERR_CUDA, "cuCtxGetCurrent is unavailable%s%s");
  std::lock_guard<std::mutex> lock(mu);
  CUcontext ctx = nullptr;
  if (get_ctx(&ctx) != CUDA_SUCCESS) return set_error(EBR_ERR_CUDA, "cuCtxGetCurrent failed%s%s");
  for (int i = 0; ctx && i < kMaxScratchContexts; ++i)
    if (ctxs[i] == ctx) {
      *out = ptrs[i];
      return EBR_OK;
    }
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_bwd_noalloc_scratch);  // makes the device's primary context current
  if (e != cudaSuccess || !p) return cuda_error(e, "cudaGetSymbolAddress(g_bwd_noalloc_scratch)");
  if (!ctx && (get_ctx(&ctx) != CUDA_SUCCESS || !ctx)) return set_error(EBR_ERR_CUDA, "no current CUDA context%s%s");
  ctxs[next] = ctx;
  ptrs[next] = p;
  next = (next + 1) % kMaxScratchContexts;
  *out = p;
  return EBR_OK;
}

// One thread waits, with a limit of `limit_ns`, on an mbarrier that nothing completes (ebr_attn_test_bounded_wait).
__global__ void bounded_wait_test_kernel(uint64_t limit_ns, int site) {
  __shared__ __align__(8) uint64_t bar;
  mbar_init(&bar, 1);
  fence_barrier_init();
  mbar_wait_limited(&bar, 0, site, limit_ns);
}

}  // namespace

// ================================================================================================ C ABI

extern "C" {

int ebr_attn_uses_tensor_cores(int dtype, int64_t D, const ebr_operand* q, const ebr_operand* k,
                               const ebr_operand* v) {
  // Shape-independent part of the choice; N only decides between the single-tile and multi-tile kernels.
  return tc_eligible(dtype, D, {q, k, v}, 2, 2, 2) ? 1 : 0;
}

int ebr_attn_fwd(int dtype, int64_t B, int64_t H, int64_t N, int64_t D, double scale, const ebr_operand* q,
                 const ebr_operand* k, const ebr_operand* v, void* o, void* lse, void* stream) {
  int s;
  if ((s = check_shape(dtype, B, H, N, D)) || (s = check_operand(q, "q")) || (s = check_operand(k, "k")) ||
      (s = check_operand(v, "v")))
    return s;
  if (!o || !lse) return set_error(EBR_ERR_NULL, "output pointer is NULL%s%s");
  if (B * H * N == 0) return EBR_OK;
  int device = 0;
  if ((s = check_device(&device))) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (tc_eligible(dtype, D, {q, k, v}, B, H, N) && aligned16(o)) {
    // N > 128: two query tiles per CTA in ping-pong; N <= 128 (one tile per slice): two CTAs per SM.
    const bool pair = N > kTile;
    if (dtype == EBR_BFLOAT16) {
      if (pair)
        s = D == 64 ? launch_tc_fwd_pair<__nv_bfloat16, 64>(device, dtype, B, H, N, scale, q, k, v, o, lse, st)
                    : launch_tc_fwd_pair<__nv_bfloat16, 128>(device, dtype, B, H, N, scale, q, k, v, o, lse, st);
      else
        s = D == 64 ? launch_tc_fwd_short<__nv_bfloat16, 64>(device, dtype, B, H, N, scale, q, k, v, o, lse, st)
                    : launch_tc_fwd_short<__nv_bfloat16, 128>(device, dtype, B, H, N, scale, q, k, v, o, lse, st);
    } else {
      if (pair)
        s = D == 64 ? launch_tc_fwd_pair<__half, 64>(device, dtype, B, H, N, scale, q, k, v, o, lse, st)
                    : launch_tc_fwd_pair<__half, 128>(device, dtype, B, H, N, scale, q, k, v, o, lse, st);
      else
        s = D == 64 ? launch_tc_fwd_short<__half, 64>(device, dtype, B, H, N, scale, q, k, v, o, lse, st)
                    : launch_tc_fwd_short<__half, 128>(device, dtype, B, H, N, scale, q, k, v, o, lse, st);
    }
    if (s != kNoTensorMap) return s;
  }
  switch (dtype) {
    case EBR_FLOAT32: return launch_simt_fwd<float>(B, H, N, D, scale, q, k, v, o, lse, st);
    case EBR_FLOAT64: return launch_simt_fwd<double>(B, H, N, D, scale, q, k, v, o, lse, st);
    case EBR_BFLOAT16: return launch_simt_fwd<__nv_bfloat16>(B, H, N, D, scale, q, k, v, o, lse, st);
    default: return launch_simt_fwd<__half>(B, H, N, D, scale, q, k, v, o, lse, st);
  }
}

size_t ebr_attn_bwd_scratch_bytes(int dtype, int64_t B, int64_t H, int64_t N, int64_t D) {
  (void)D;
  if (elem_size(dtype) == 0 || B < 0 || H < 0 || N < 0) return 0;
  return static_cast<size_t>(B * H * N) * stat_size(dtype);
}

int ebr_attn_bwd(int dtype, int64_t B, int64_t H, int64_t N, int64_t D, double scale, const ebr_operand* q,
                 const ebr_operand* k, const ebr_operand* v, const void* o, const void* lse,
                 const ebr_operand* dout, void* dq, void* dk, void* dv, void* scratch, size_t scratch_bytes,
                 void* stream) {
  int s;
  if ((s = check_shape(dtype, B, H, N, D)) || (s = check_operand(q, "q")) || (s = check_operand(k, "k")) ||
      (s = check_operand(v, "v")) || (s = check_operand(dout, "dout")))
    return s;
  if (!o || !lse || !dq || !dk || !dv) return set_error(EBR_ERR_NULL, "o / lse / output pointer is NULL%s%s");
  if (B * H * N == 0) return EBR_OK;
  int device = 0;
  if ((s = check_device(&device))) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool outs_ok = aligned16(o) && aligned16(dq) && aligned16(dk) && aligned16(dv);
  const bool scratch_ok = scratch && scratch_bytes >= ebr_attn_bwd_scratch_bytes(dtype, B, H, N, D);
  if (N > kTile && scratch_ok && outs_ok && tc_eligible(dtype, D, {q, k, v, dout}, B, H, N)) {
    if (dtype == EBR_BFLOAT16)
      s = D == 64 ? launch_tc_bwd_pipe<__nv_bfloat16, 64>(device, dtype, B, H, N, scale, q, k, v, o, lse, dout, dq,
                                                           dk, dv, scratch, st)
                  : launch_tc_bwd_pipe<__nv_bfloat16, 128>(device, dtype, B, H, N, scale, q, k, v, o, lse, dout, dq,
                                                            dk, dv, scratch, st);
    else
      s = D == 64 ? launch_tc_bwd_pipe<__half, 64>(device, dtype, B, H, N, scale, q, k, v, o, lse, dout, dq, dk, dv,
                                                   scratch, st)
                  : launch_tc_bwd_pipe<__half, 128>(device, dtype, B, H, N, scale, q, k, v, o, lse, dout, dq, dk,
                                                    dv, scratch, st);
    if (s != kNoTensorMap) return s;
  }
  if (N <= kTile && outs_ok && tc_eligible(dtype, D, {q, k, v, dout}, B, H, N)) {
    if (dtype == EBR_BFLOAT16)
      s = D == 64 ? launch_tc_bwd_short<__nv_bfloat16, 64>(device, dtype, B, H, N, scale, q, k, v, o, lse, dout, dq,
                                                             dk, dv, st)
                  : launch_tc_bwd_short<__nv_bfloat16, 128>(device, dtype, B, H, N, scale, q, k, v, o, lse, dout,
                                                              dq, dk, dv, st);
    else
      s = D == 64 ? launch_tc_bwd_short<__half, 64>(device, dtype, B, H, N, scale, q, k, v, o, lse, dout, dq, dk,
                                                     dv, st)
                  : launch_tc_bwd_short<__half, 128>(device, dtype, B, H, N, scale, q, k, v, o, lse, dout, dq, dk,
                                                      dv, st);
    if (s != kNoTensorMap) return s;
  }
  if (!scratch || scratch_bytes < ebr_attn_bwd_scratch_bytes(dtype, B, H, N, D))
    return set_error(EBR_ERR_SCRATCH, "scratch missing or too small%s%s");
  switch (dtype) {
    case EBR_FLOAT32: return launch_simt_bwd<float>(B, H, N, D, scale, q, k, v, o, lse, dout, dq, dk, dv, scratch, st);
    case EBR_FLOAT64:
      return launch_simt_bwd<double>(B, H, N, D, scale, q, k, v, o, lse, dout, dq, dk, dv, scratch, st);
    case EBR_BFLOAT16:
      return launch_simt_bwd<__nv_bfloat16>(B, H, N, D, scale, q, k, v, o, lse, dout, dq, dk, dv, scratch, st);
    default: return launch_simt_bwd<__half>(B, H, N, D, scale, q, k, v, o, lse, dout, dq, dk, dv, scratch, st);
  }
}

size_t ebr_attn_bwd_bwd_scratch_bytes(int dtype, int64_t B, int64_t H, int64_t N, int64_t D) {
  (void)D;
  if (elem_size(dtype) == 0 || B < 0 || H < 0 || N < 0) return 0;
  return 3 * static_cast<size_t>(B * H * N) * stat_size(dtype);
}

int ebr_attn_bwd_bwd(int dtype, int64_t B, int64_t H, int64_t N, int64_t D, double scale, const ebr_operand* q,
                     const ebr_operand* k, const ebr_operand* v, const void* o, const void* lse,
                     const ebr_operand* dout, const void* dq, const ebr_operand* gq, const ebr_operand* gk,
                     const ebr_operand* gv, void* hq, void* hk, void* hv, void* hdout, void* scratch,
                     size_t scratch_bytes, void* stream) {
  (void)dq;  // accepted for the op contract, not read (reference.py:74)
  int s;
  if ((s = check_shape(dtype, B, H, N, D)) || (s = check_operand(q, "q")) || (s = check_operand(k, "k")) ||
      (s = check_operand(v, "v")) || (s = check_operand(dout, "dout")) || (s = check_operand(gq, "gq", true)) ||
      (s = check_operand(gk, "gk", true)) || (s = check_operand(gv, "gv", true)))
    return s;
  if (!o || !lse || !hq || !hk || !hv || !hdout)
    return set_error(EBR_ERR_NULL, "o / lse / output pointer is NULL%s%s");
  if (B * H * N == 0) return EBR_OK;
  int device = 0;
  if ((s = check_device(&device))) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool outs_ok = aligned16(o) && aligned16(hq) && aligned16(hk) && aligned16(hv) && aligned16(hdout);
  if (N <= kTile && D == 64 && outs_ok && tc_eligible(dtype, D, {q, k, v, dout, gq, gk, gv}, B, H, N)) {
    if (dtype == EBR_BFLOAT16)
      s = launch_tc_bob_short<__nv_bfloat16>(device, dtype, B, H, N, scale, q, k, v, o, lse, dout, gq, gk, gv, hq,
                                              hk, hv, hdout, st);
    else
      s = launch_tc_bob_short<__half>(device, dtype, B, H, N, scale, q, k, v, o, lse, dout, gq, gk, gv, hq, hk, hv,
                                       hdout, st);
    if (s != kNoTensorMap) return s;
  }
  if (!scratch || scratch_bytes < ebr_attn_bwd_bwd_scratch_bytes(dtype, B, H, N, D))
    return set_error(EBR_ERR_SCRATCH, "scratch missing or too small%s%s");
  if (outs_ok && tc_eligible(dtype, D, {q, k, v, dout, gq, gk, gv}, B, H, N)) {
    if (dtype == EBR_BFLOAT16)
      s = D == 64 ? launch_tc_bob_split<__nv_bfloat16>(device, dtype, B, H, N, scale, q, k, v, o, lse, dout, gq, gk,
                                                        gv, hq, hk, hv, hdout, scratch, st)
                  : launch_tc_bob_pipe<__nv_bfloat16, 128>(device, dtype, B, H, N, scale, q, k, v, o, lse, dout, gq,
                                                            gk, gv, hq, hk, hv, hdout, scratch, st);
    else
      s = D == 64 ? launch_tc_bob_split<__half>(device, dtype, B, H, N, scale, q, k, v, o, lse, dout, gq, gk, gv, hq,
                                                hk, hv, hdout, scratch, st)
                  : launch_tc_bob_pipe<__half, 128>(device, dtype, B, H, N, scale, q, k, v, o, lse, dout, gq, gk, gv,
                                                    hq, hk, hv, hdout, scratch, st);
    if (s != kNoTensorMap) return s;
  }
  switch (dtype) {
    case EBR_FLOAT32:
      return launch_simt_bob<float>(B, H, N, D, scale, q, k, v, o, lse, dout, gq, gk, gv, hq, hk, hv, hdout, scratch,
                                    st);
    case EBR_FLOAT64:
      return launch_simt_bob<double>(B, H, N, D, scale, q, k, v, o, lse, dout, gq, gk, gv, hq, hk, hv, hdout,
                                     scratch, st);
    case EBR_BFLOAT16:
      return launch_simt_bob<__nv_bfloat16>(B, H, N, D, scale, q, k, v, o, lse, dout, gq, gk, gv, hq, hk, hv, hdout,
                                            scratch, st);
    default:
      return launch_simt_bob<__half>(B, H, N, D, scale, q, k, v, o, lse, dout, gq, gk, gv, hq, hk, hv, hdout, scratch,
                                     st);
  }
}

int ebr_attn_bwd_noalloc(int dtype, int64_t B, int64_t H, int64_t N, int64_t D, double scale,
                         const ebr_operand* q, const ebr_operand* k, const ebr_operand* v, const void* o,
                         const void* lse, const ebr_operand* dout, void* dq, void* dk, void* dv, void* stream) {
  int s;
  if ((s = check_shape(dtype, B, H, N, D)) || (s = check_operand(q, "q")) || (s = check_operand(k, "k")) ||
      (s = check_operand(v, "v")) || (s = check_operand(dout, "dout")))
    return s;
  if (!o || !lse || !dq || !dk || !dv) return set_error(EBR_ERR_NULL, "o / lse / output pointer is NULL%s%s");
  if (B * H * N == 0) return EBR_OK;
  const size_t need = ebr_attn_bwd_scratch_bytes(dtype, B, H, N, D);
  if (need > EBR_ATTN_NOALLOC_SCRATCH_BYTES) {
    std::snprintf(g_last_error, sizeof(g_last_error),
                  "ebr_attn_bwd_noalloc: B*H*N = %lld rows need %zu bytes of row scratch; the built-in buffer holds "
                  "%zu bytes (use ebr_attn_bwd with a caller-provided buffer)",
                  static_cast<long long>(B * H * N), need, static_cast<size_t>(EBR_ATTN_NOALLOC_SCRATCH_BYTES));
    return EBR_ERR_SCRATCH;
  }
  int device = 0;
  if ((s = check_device(&device))) return s;
  void* scratch = nullptr;
  if ((s = noalloc_scratch(&scratch))) return s;
  return ebr_attn_bwd(dtype, B, H, N, D, scale, q, k, v, o, lse, dout, dq, dk, dv, scratch,
                      EBR_ATTN_NOALLOC_SCRATCH_BYTES, stream);
}

int ebr_attn_device_status(void) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_error(e, "cudaDeviceSynchronize");
  int flag = 0;
  e = cudaMemcpyFromSymbol(&flag, ebr::g_device_error, sizeof(int));
  if (e != cudaSuccess) return cuda_error(e, "cudaMemcpyFromSymbol");
  if (flag != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(ebr::g_device_error, &zero, sizeof(int));
    std::snprintf(g_last_error, sizeof(g_last_error), "bounded device wait ran out at site %d", flag);
    return EBR_ERR_DEVICE_TIMEOUT;
  }
  return EBR_OK;
}

int ebr_attn_test_bounded_wait(int64_t limit_ns, void* stream) {
  if (limit_ns < 1000 || limit_ns > 1000000000) return set_error(EBR_ERR_SHAPE, "limit_ns must be in [1 us, 1 s]%s%s");
  int device = 0, s;
  if ((s = check_device(&device))) return s;
  bounded_wait_test_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<uint64_t>(limit_ns),
                                                                          kBoundedWaitTestSite);
  return check_launch("bounded_wait_test_kernel");
}

const char* ebr_attn_status_string(int status) {
  switch (status) {
    case EBR_OK: return "ok";
    case EBR_ERR_NULL: return "null pointer";
    case EBR_ERR_SHAPE: return "bad shape";
    case EBR_ERR_DTYPE: return "unsupported dtype";
    case EBR_ERR_STRIDE: return "bad stride";
    case EBR_ERR_SCRATCH: return "scratch missing or too small";
    case EBR_ERR_CUDA: return "CUDA error";
    case EBR_ERR_DEVICE: return "unsupported device";
    case EBR_ERR_DEVICE_TIMEOUT: return "device wait timed out";
    default: return "unknown status";
  }
}

const char* ebr_attn_last_error(void) { return g_last_error; }

uint64_t ebr_attn_launch_count(void) { return g_launch_count.load(); }

}  // extern "C"

// The fused kernels on either side of the attention (include/ebr_layers.h).
#include "layers_capi.cuh"
