// bq4_api.cu -- the extern "C" boundary of libbq4 (include/bq4.h).
//
// Host-side validation mirrors the reference's eligibility rules and error
// behaviour (patches/burn-cubecl-0.21.0/src/ops/qtensor.rs:303-368), except
// that failures return a status instead of panicking.  Nothing here computes
// on the CPU: every numeric result comes from a CUDA kernel, and calls fail
// with BQ4_EUNSUPPORTED on devices without the sm_100a kernels.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <vector>

#include "bq4_internal.h"

namespace bq4 {

static thread_local char g_err[512] = "no error";
static thread_local uint64_t g_launches = 0;

bq4_status set_error(bq4_status code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

bq4_status check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return BQ4_OK;
  return set_error(BQ4_ECUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

void note_launch(uint64_t n) { g_launches += n; }

bq4_status poll_device_error();

namespace {

bool valid_block(int32_t b) { return b == 8 || b == 16 || b == 32 || b == 64 || b == 128; }

bq4_status check_geometry(int64_t K, int64_t N, int32_t block, int32_t layout) {
  if (layout != BQ4_LAYOUT_COL && layout != BQ4_LAYOUT_ROW && layout != BQ4_LAYOUT_NPACKED)
    return set_error(BQ4_EINVAL_ARG, "layout %d is not BQ4_LAYOUT_COL/ROW/NPACKED", layout);
  if (!valid_block(block))
    return set_error(BQ4_EINVAL_BLOCK, "block %d not in {8,16,32,64,128}", block);
  if (K <= 0 || N <= 0)
    return set_error(BQ4_EINVAL_SHAPE, "K=%lld N=%lld must be positive", (long long)K, (long long)N);
  if (layout == BQ4_LAYOUT_NPACKED) {
    // packed and blocked along N (the last axis of a plain [K,N] tensor)
    if (N % 8 != 0) return set_error(BQ4_EINVAL_SHAPE, "N=%lld is not a multiple of 8", (long long)N);
    if (N % block != 0)
      return set_error(BQ4_EINVAL_BLOCK, "block %d does not divide N=%lld", block, (long long)N);
    if (K > (int64_t)1 << 24 || N > (int64_t)1 << 24)
      return set_error(BQ4_EINVAL_SHAPE, "K or N above 2^24");
    return BQ4_OK;
  }
  if (K % 8 != 0) return set_error(BQ4_EINVAL_SHAPE, "K=%lld is not a multiple of 8", (long long)K);
  if (K % block != 0)
    return set_error(BQ4_EINVAL_BLOCK, "block %d does not divide K=%lld", block, (long long)K);
  if (K > (int64_t)1 << 24 || N > (int64_t)1 << 24)
    return set_error(BQ4_EINVAL_SHAPE, "K or N above 2^24");
  return BQ4_OK;
}

bool is_device_ptr(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

bq4_status require_sm100(int device) {
  if (!device_is_sm100(device))
    return set_error(BQ4_EUNSUPPORTED,
                     "device %d is not sm_100 (B200); libbq4 has no kernels for it", device);
  return BQ4_OK;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Build a prepared weight for the (n0..n0+N, k0..k0+K) window of a source
// tensor of extents src_N x src_K.
bq4_status prepare_window(const uint32_t* words, const float* scales, int64_t src_K, int64_t src_N,
                          int32_t block, int32_t layout, int64_t n0, int64_t N, int64_t k0,
                          int64_t K, int32_t device, bq4_weight** out) {
  if (!out) return set_error(BQ4_EINVAL_ARG, "out is NULL");
  *out = nullptr;
  if (!words || !scales) return set_error(BQ4_EINVAL_ARG, "packed_words/scales is NULL");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
    cudaGetLastError();
    return set_error(BQ4_EINVAL_ARG, "device %d not present", device);
  }
  bq4_status st = require_sm100(device);
  if (st) return st;
  DeviceGuard guard(device);

  bq4_weight* w = new (std::nothrow) bq4_weight();
  if (!w) return set_error(BQ4_ECUDA, "host allocation failed");
  w->K = K;
  w->N = N;
  w->block = block;
  w->layout = layout;
  w->device = device;
  w->Kp = (K + kStageK - 1) / kStageK * kStageK;
  w->nkc = w->Kp / kChunkK;
  w->nkb = w->Kp / block;
  w->ntiles = (N + kTileN - 1) / kTileN;
  w->Np = w->ntiles * kTileN;
  w->q_bytes = (size_t)w->ntiles * w->nkc * 1024 * sizeof(uint32_t);
  w->s_bytes = (size_t)w->ntiles * w->nkb * 128 * sizeof(float);

  const bool pre = layout == BQ4_LAYOUT_NPACKED;
  if (pre) {
    w->q_bytes = w->s_bytes = 0;
    w->h_bytes = (size_t)w->ntiles * w->nkc * 128 * 64 * sizeof(uint16_t);
  }
  const size_t src_words = pre ? (size_t)src_K * (size_t)(src_N / 8) : (size_t)src_N * (size_t)(src_K / 8);
  const size_t src_scales = pre ? (size_t)src_K * (size_t)(src_N / block) : (size_t)src_N * (size_t)(src_K / block);
  const uint32_t* dwords = words;
  const float* dscales = scales;
  void* tmp_w = nullptr;
  void* tmp_s = nullptr;
  cudaError_t e = cudaSuccess;
  if (!is_device_ptr(words)) {
    e = cudaMalloc(&tmp_w, src_words * 4);
    if (e == cudaSuccess) e = cudaMemcpy(tmp_w, words, src_words * 4, cudaMemcpyHostToDevice);
    dwords = static_cast<const uint32_t*>(tmp_w);
  }
  if (e == cudaSuccess && !is_device_ptr(scales)) {
    e = cudaMalloc(&tmp_s, src_scales * 4);
    if (e == cudaSuccess) e = cudaMemcpy(tmp_s, scales, src_scales * 4, cudaMemcpyHostToDevice);
    dscales = static_cast<const float*>(tmp_s);
  }
  if (pre) {
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&w->h), w->h_bytes);
    if (e == cudaSuccess)
      e = launch_prepare_pre(dwords, dscales, K, N, block, n0, k0, src_N, src_K, w, nullptr);
  } else {
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&w->q), w->q_bytes);
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&w->s), w->s_bytes);
    if (e == cudaSuccess)
      e = launch_prepare(dwords, dscales, K, N, block, layout, n0, k0, src_N, src_K, w, nullptr);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(nullptr);
  if (tmp_w) cudaFree(tmp_w);
  if (tmp_s) cudaFree(tmp_s);
  if (e != cudaSuccess) {
    if (w->q) cudaFree(w->q);
    if (w->s) cudaFree(w->s);
    if (w->h) cudaFree(w->h);
    delete w;
    return check_cuda(e, "bq4_weight_prepare");
  }
  *out = w;
  return BQ4_OK;
}

bq4_status check_weight(const bq4_weight* w, const char* name) {
  if (!w || !((w->q && w->s) || w->h)) return set_error(BQ4_EINVAL_ARG, "%s is NULL or freed", name);
  return BQ4_OK;
}

bq4_status check_compute_args(const bq4_weight* w, const float* x, int64_t M, int64_t ldx,
                              const float* y, void* workspace) {
  if (!x || !y) return set_error(BQ4_EINVAL_ARG, "x/y is NULL");
  if (M <= 0) return set_error(BQ4_EINVAL_SHAPE, "M=%lld must be positive", (long long)M);
  if (ldx < w->K)
    return set_error(BQ4_EINVAL_SHAPE, "ldx=%lld < K=%lld", (long long)ldx, (long long)w->K);
  if (!aligned(x, 4) || !aligned(y, 4)) return set_error(BQ4_EALIGN, "x/y not 4-byte aligned");
  if (!workspace) return set_error(BQ4_EWORKSPACE, "workspace is NULL");
  if (!aligned(workspace, 256)) return set_error(BQ4_EALIGN, "workspace not 256-byte aligned");
  return BQ4_OK;
}

}  // namespace
}  // namespace bq4

using namespace bq4;

extern "C" {

const char* bq4_version(void) { return "bq4 0.1.0 (sm_100a tcgen05)"; }

const char* bq4_last_error_string(void) { return g_err; }

uint64_t bq4_launch_count(void) { return g_launches; }
void bq4_launch_count_reset(void) { g_launches = 0; }

bq4_status bq4_poll_device_error(void) { return poll_device_error(); }

bq4_status bq4_set_numerics(bq4_numerics mode) {
  if (mode != BQ4_NUMERICS_AUTO && mode != BQ4_NUMERICS_EXACT && mode != BQ4_NUMERICS_FOLDED)
    return set_error(BQ4_EINVAL_ARG, "numerics mode %d unknown", (int)mode);
  set_numerics_mode((int)mode);
  return BQ4_OK;
}

bq4_status bq4_weight_prepare(const uint32_t* packed_words, const float* scales, int64_t K,
                              int64_t N, int32_t block, bq4_layout layout, int32_t device,
                              bq4_weight** out) {
  bq4_status st = check_geometry(K, N, block, layout);
  if (st) return st;
  return prepare_window(packed_words, scales, K, N, block, layout, 0, N, 0, K, device, out);
}

bq4_status bq4_weight_prepare_shard(const uint32_t* packed_words, const float* scales, int64_t K,
                                    int64_t N, int32_t block, bq4_layout layout, int32_t kind,
                                    int32_t rank, int32_t size, int32_t device, bq4_weight** out) {
  bq4_status st = check_geometry(K, N, block, layout);
  if (st) return st;
  if (size <= 0 || rank < 0 || rank >= size)
    return set_error(BQ4_EINVAL_ARG, "rank %d / size %d invalid", rank, size);
  if (kind == 0) {
    if (N % size != 0)
      return set_error(BQ4_EINVAL_SHAPE, "column shard: N=%lld not divisible by %d", (long long)N, size);
    if (layout == BQ4_LAYOUT_NPACKED && ((N / size) % block != 0 || (N / size) % 8 != 0))
      return set_error(BQ4_EINVAL_BLOCK, "column shard of an N-packed weight must fall on block boundaries");
    const int64_t n = N / size;
    return prepare_window(packed_words, scales, K, N, block, layout, rank * n, n, 0, K, device, out);
  }
  if (kind == 1) {
    if (layout == BQ4_LAYOUT_NPACKED && K % size == 0) {
      const int64_t k = K / size;
      return prepare_window(packed_words, scales, K, N, block, layout, 0, N, rank * k, k, device, out);
    }
    if (K % size != 0 || (K / size) % block != 0 || (K / size) % 8 != 0)
      return set_error(BQ4_EINVAL_BLOCK,
                       "row shard: K=%lld over %d parts does not fall on block-%d boundaries",
                       (long long)K, size, block);
    const int64_t k = K / size;
    return prepare_window(packed_words, scales, K, N, block, layout, 0, N, rank * k, k, device, out);
  }
  return set_error(BQ4_EINVAL_ARG, "shard kind %d not 0 (column) or 1 (row)", kind);
}

bq4_status bq4_weight_free(bq4_weight* w) {
  if (!w) return BQ4_OK;
  DeviceGuard guard(w->device);
  cudaError_t e1 = w->q ? cudaFree(w->q) : cudaSuccess;
  cudaError_t e2 = w->s ? cudaFree(w->s) : cudaSuccess;
  cudaError_t e3 = w->h ? cudaFree(w->h) : cudaSuccess;
  if (e2 == cudaSuccess) e2 = e3;
  w->q = nullptr;
  w->s = nullptr;
  w->h = nullptr;
  delete w;
  if (e1 != cudaSuccess) return check_cuda(e1, "bq4_weight_free");
  return check_cuda(e2, "bq4_weight_free");
}

bq4_status bq4_weight_info(const bq4_weight* w, int64_t* K, int64_t* N, int32_t* block,
                           int32_t* layout, size_t* device_bytes) {
  bq4_status st = check_weight(w, "w");
  if (st) return st;
  if (K) *K = w->K;
  if (N) *N = w->N;
  if (block) *block = w->block;
  if (layout) *layout = w->layout;
  if (device_bytes) *device_bytes = w->q_bytes + w->s_bytes + w->h_bytes;
  return BQ4_OK;
}

bq4_status bq4_linear_workspace_size(const bq4_weight* w, int64_t M, size_t* bytes) {
  bq4_status st = check_weight(w, "w");
  if (st) return st;
  if (!bytes) return set_error(BQ4_EINVAL_ARG, "bytes is NULL");
  GemmPlan plan;
  st = plan_gemm(w, 1, M, w->device, &plan);
  if (st) return st;
  *bytes = plan.workspace_bytes;
  return BQ4_OK;
}

bq4_status bq4_linear_plan_info(const bq4_weight* w, int64_t M, int32_t gated, int32_t* info, int32_t n) {
  bq4_status st = check_weight(w, "w");
  if (st) return st;
  if (!info || n < 0) return set_error(BQ4_EINVAL_ARG, "info is NULL or n < 0");
  DeviceGuard guard(w->device);
  GemmPlan plan;
  st = plan_gemm(w, gated ? 2 : 1, M, w->device, &plan);
  if (st) return st;
  const int32_t v[13] = {plan.bt, plan.ksplit, plan.grid, plan.exact, plan.ta, plan.stages, plan.sk_tiles,
                         plan.dp_tiles, (int32_t)(plan.workspace_bytes / 256), plan.wide, plan.tail_tiles,
                         plan.tail_split, plan.skinny};
  for (int32_t i = 0; i < n && i < 13; ++i) info[i] = v[i];
  return BQ4_OK;
}

bq4_status bq4_linear(const bq4_weight* w, const float* x, int64_t M, int64_t ldx,
                      const float* bias, bq4_act act, const float* aux, float* y, void* workspace,
                      size_t workspace_bytes, bq4_stream_t stream) {
  bq4_status st = check_weight(w, "w");
  if (st) return st;
  if (act != BQ4_ACT_NONE && act != BQ4_ACT_GELU_TANH && act != BQ4_ACT_SILU)
    return set_error(BQ4_EINVAL_ARG, "act %d unknown", (int)act);
  st = check_compute_args(w, x, M, ldx, y, workspace);
  if (st) return st;
  GemmPlan plan;
  st = plan_gemm(w, 1, M, w->device, &plan);
  if (st) return st;
  if (workspace_bytes < plan.workspace_bytes)
    return set_error(BQ4_EWORKSPACE, "workspace %zu < required %zu bytes", workspace_bytes,
                     plan.workspace_bytes);
  DeviceGuard guard(w->device);
  const bq4_weight* ws[1] = {w};
  const float* b[1] = {bias};
  return run_gemm(plan, ws, x, M, ldx, b, (int)act, aux, y, workspace,
                  reinterpret_cast<cudaStream_t>(stream));
}

static bq4_status select_rows(const uint32_t* values, const float* scales, int64_t rows, int64_t cols, int32_t block,
                              const void* ids, int32_t ids_i64, int64_t n, uint32_t* out_values, float* out_scales,
                              float* out_f32, bq4_stream_t stream) {
  if (!values || !scales || !ids) return set_error(BQ4_EINVAL_ARG, "values/scales/ids is NULL");
  if (block != 8 && block != 16 && block != 32 && block != 64 && block != 128)
    return set_error(BQ4_EINVAL_BLOCK, "block %d not in {8,16,32,64,128}", (int)block);
  if (rows <= 0 || cols <= 0 || n < 0 || cols % block)
    return set_error(BQ4_EINVAL_SHAPE, "rows=%lld cols=%lld n=%lld block=%d", (long long)rows, (long long)cols,
                     (long long)n, (int)block);
  if (!aligned(values, 4) || !aligned(scales, 4) || !aligned(ids, ids_i64 ? 8 : 4))
    return set_error(BQ4_EALIGN, "values/scales/ids misaligned");
  if (out_f32 && !aligned(out_f32, 16)) return set_error(BQ4_EALIGN, "out not 16-byte aligned");
  if (n == 0) return BQ4_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  bq4_status st = require_sm100(dev);
  if (st) return st;
  int* err = device_error_word();
  if (!err) return set_error(BQ4_ECUDA, "device error word unavailable");
  cudaError_t e = launch_select_rows(values, scales, rows, cols, block, ids, ids_i64 ? 1 : 0, n, out_values,
                                     out_scales, out_f32, err, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? BQ4_OK : check_cuda(e, "select_rows launch");
}

bq4_status bq4_q_select_rows(const uint32_t* values, const float* scales, int64_t rows, int64_t cols, int32_t block,
                             const void* ids, int32_t ids_i64, int64_t n, uint32_t* out_values, float* out_scales,
                             bq4_stream_t stream) {
  if (!out_values || !out_scales) return set_error(BQ4_EINVAL_ARG, "out_values/out_scales is NULL");
  if (!aligned(out_values, 4) || !aligned(out_scales, 4)) return set_error(BQ4_EALIGN, "outputs misaligned");
  return select_rows(values, scales, rows, cols, block, ids, ids_i64, n, out_values, out_scales, nullptr, stream);
}

bq4_status bq4_q_select_rows_dequant(const uint32_t* values, const float* scales, int64_t rows, int64_t cols,
                                     int32_t block, const void* ids, int32_t ids_i64, int64_t n, float* out,
                                     bq4_stream_t stream) {
  if (!out) return set_error(BQ4_EINVAL_ARG, "out is NULL");
  return select_rows(values, scales, rows, cols, block, ids, ids_i64, n, nullptr, nullptr, out, stream);
}

bq4_status bq4_parse_stored_dtype(const char* stored_dtype, int32_t* block, int32_t* axis) {
  if (!stored_dtype || !block || !axis) return set_error(BQ4_EINVAL_ARG, "NULL argument");
  int b = 0, n = 0;
  int ax = -1;
  if (sscanf(stored_dtype, "q4s-block%dx1-f32-packed-axis1%n", &b, &n) == 1 && stored_dtype[n] == '\0') {
    ax = 1;
  } else if (sscanf(stored_dtype, "q4s-block%d-f32-packed-axis0%n", &b, &n) == 1 && stored_dtype[n] == '\0') {
    ax = 0;
  }
  if (ax < 0 || !(b == 8 || b == 16 || b == 32 || b == 64 || b == 128))
    return set_error(BQ4_EINVAL_ARG, "stored dtype '%s' is not a packed-Q4 (Q4S, F32 scales) spelling",
                     stored_dtype);
  // the parse must round-trip to the exact spelling (no leading zeros or signs)
  char canon[64];
  snprintf(canon, sizeof(canon), ax ? "q4s-block%dx1-f32-packed-axis1" : "q4s-block%d-f32-packed-axis0", b);
  if (strcmp(canon, stored_dtype) != 0)
    return set_error(BQ4_EINVAL_ARG, "stored dtype '%s' is not in canonical form", stored_dtype);
  *block = b;
  *axis = ax;
  return BQ4_OK;
}

bq4_status bq4_weight_prepare_payload(const void* payload, size_t nbytes, int64_t rows, int64_t cols,
                                      const char* stored_dtype, int32_t transposed_view, int32_t device,
                                      bq4_weight** out) {
  int32_t block = 0, axis = 0;
  bq4_status st = bq4_parse_stored_dtype(stored_dtype, &block, &axis);
  if (st) return st;
  if (!payload || !out) return set_error(BQ4_EINVAL_ARG, "payload/out is NULL");
  if (rows <= 0 || cols <= 0) return set_error(BQ4_EINVAL_SHAPE, "shape [%lld, %lld]", (long long)rows, (long long)cols);
  const int64_t elems = rows * cols;
  if (elems % block || elems % 8 || elems / rows != cols)
    return set_error(BQ4_EINVAL_SHAPE, "shape [%lld, %lld] does not hold whole blocks of %d", (long long)rows,
                     (long long)cols, (int)block);
  const size_t words_bytes = (size_t)(elems / 2), want = words_bytes + (size_t)(elems / block) * 4;
  if (nbytes != want)
    return set_error(BQ4_EINVAL_SHAPE, "payload of %zu bytes; shape [%lld, %lld] block %d needs %zu", nbytes,
                     (long long)rows, (long long)cols, (int)block, want);
  int64_t K, N;
  bq4_layout layout;
  if (axis == 1) {
    K = rows; N = cols; layout = BQ4_LAYOUT_ROW;          // stored [K, N], packed along K
  } else if (transposed_view) {
    K = cols; N = rows; layout = BQ4_LAYOUT_COL;          // stored [N, K] seen as [K, N]
  } else {
    K = rows; N = cols; layout = BQ4_LAYOUT_NPACKED;      // plain stored [K, N], packed along N
  }
  const uint8_t* p8 = static_cast<const uint8_t*>(payload);
  // a host payload may sit at any byte offset of a file buffer: copy it to
  // 4-byte alignment first (device payloads must already be aligned)
  std::vector<uint32_t> aligned_copy;
  if (!is_device_ptr(payload) && !aligned(payload, 4)) {
    aligned_copy.resize((nbytes + 3) / 4);
    memcpy(aligned_copy.data(), payload, nbytes);
    p8 = reinterpret_cast<const uint8_t*>(aligned_copy.data());
  } else if (!aligned(payload, 4)) {
    return set_error(BQ4_EALIGN, "device payload not 4-byte aligned");
  }
  return bq4_weight_prepare(reinterpret_cast<const uint32_t*>(p8), reinterpret_cast<const float*>(p8 + words_bytes),
                            K, N, block, layout, device, out);
}

bq4_status bq4_set_sm_budget(int32_t sms) {
  if (sms < 0) return set_error(BQ4_EINVAL_ARG, "sm budget %d is negative", (int)sms);
  set_sm_budget(sms);
  return BQ4_OK;
}

bq4_status bq4_rms_renorm(const void* x, bq4_dtype x_dtype, int64_t M, int64_t H, int64_t ldx, void* out,
                          bq4_dtype out_dtype, int64_t ldo, float eps, bq4_stream_t stream) {
  if ((x_dtype != BQ4_DTYPE_F32 && x_dtype != BQ4_DTYPE_F16) ||
      (out_dtype != BQ4_DTYPE_F32 && out_dtype != BQ4_DTYPE_F16))
    return set_error(BQ4_EINVAL_ARG, "dtype unknown");
  if (!x || !out) return set_error(BQ4_EINVAL_ARG, "x/out is NULL");
  if (M <= 0 || H <= 0 || M > 0x7fffffff || ldx < H || ldo < H)
    return set_error(BQ4_EINVAL_SHAPE, "M=%lld H=%lld ldx=%lld ldo=%lld", (long long)M, (long long)H,
                     (long long)ldx, (long long)ldo);
  if (!(eps > 0.0f)) return set_error(BQ4_EINVAL_ARG, "eps must be positive");
  const size_t ax = x_dtype == BQ4_DTYPE_F16 ? 2 : 4, ao = out_dtype == BQ4_DTYPE_F16 ? 2 : 4;
  if (!aligned(x, ax) || !aligned(out, ao)) return set_error(BQ4_EALIGN, "x/out misaligned");
  cudaError_t e = launch_rms_renorm(x, x_dtype == BQ4_DTYPE_F16, M, H, ldx, out, out_dtype == BQ4_DTYPE_F16, ldo,
                                    eps, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? BQ4_OK : check_cuda(e, "rms_renorm launch");
}

bq4_status bq4_qk_norm_rope(const void* x, bq4_dtype x_dtype, int64_t M, int64_t heads, int64_t head_dim,
                            int64_t ldx, const float* gamma, float eps, const float* cos_t, const float* sin_t,
                            int64_t ld_rope, void* y, bq4_dtype y_dtype, int64_t ldy, bq4_stream_t stream) {
  if ((x_dtype != BQ4_DTYPE_F32 && x_dtype != BQ4_DTYPE_F16) || (y_dtype != BQ4_DTYPE_F32 && y_dtype != BQ4_DTYPE_F16))
    return set_error(BQ4_EINVAL_ARG, "dtype unknown");
  if (!x || !y) return set_error(BQ4_EINVAL_ARG, "x/y is NULL");
  if ((cos_t == nullptr) != (sin_t == nullptr)) return set_error(BQ4_EINVAL_ARG, "cos and sin must both be given");
  if (M <= 0 || heads <= 0 || head_dim <= 0 || head_dim % 2 || head_dim > 256 || M * heads > 0x7fffffffLL ||
      ldx < heads * head_dim || ldy < heads * head_dim || (cos_t && ld_rope < head_dim))
    return set_error(BQ4_EINVAL_SHAPE, "M=%lld heads=%lld head_dim=%lld (even, <= 256) ldx=%lld ldy=%lld ld_rope=%lld",
                     (long long)M, (long long)heads, (long long)head_dim, (long long)ldx, (long long)ldy,
                     (long long)ld_rope);
  if (!(eps > 0.0f)) return set_error(BQ4_EINVAL_ARG, "eps must be positive");
  if (x == y && (x_dtype != y_dtype || ldx != ldy))
    return set_error(BQ4_EINVAL_ARG, "in place needs the same dtype and pitch");
  const size_t ax = x_dtype == BQ4_DTYPE_F16 ? 2 : 4, ay = y_dtype == BQ4_DTYPE_F16 ? 2 : 4;
  if (!aligned(x, ax) || !aligned(y, ay) || (gamma && !aligned(gamma, 4)) || (cos_t && (!aligned(cos_t, 4) ||
                                                                                      !aligned(sin_t, 4))))
    return set_error(BQ4_EALIGN, "x/y/gamma/cos/sin misaligned");
  cudaError_t e = launch_qk_norm_rope(x, x_dtype == BQ4_DTYPE_F16, M, (int)heads, (int)head_dim, ldx, gamma, eps,
                                      cos_t, sin_t, ld_rope, y, y_dtype == BQ4_DTYPE_F16, ldy,
                                      reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? BQ4_OK : check_cuda(e, "qk_norm_rope launch");
}

static bool qk_fused(const bq4_weight* w, int64_t head_dim) { return head_dim == 128 && w->N % 128 == 0; }

bq4_status bq4_linear_qk_norm_rope_workspace_size(const bq4_weight* w, int64_t M, bq4_dtype x_dtype,
                                                  int64_t head_dim, size_t* bytes) {
  if (x_dtype != BQ4_DTYPE_F32 && x_dtype != BQ4_DTYPE_F16)
    return set_error(BQ4_EINVAL_ARG, "x_dtype %d unknown", (int)x_dtype);
  bq4_status st = check_weight(w, "w");
  if (st) return st;
  if (!bytes) return set_error(BQ4_EINVAL_ARG, "bytes is NULL");
  GemmPlan plan;
  st = plan_gemm(w, 1, M, w->device, &plan, true, qk_fused(w, head_dim));
  if (st) return st;
  *bytes = x_dtype == BQ4_DTYPE_F16 ? plan.sk_bytes + plan.partial_bytes : plan.workspace_bytes;
  return BQ4_OK;
}

bq4_status bq4_linear_qk_norm_rope(const bq4_weight* w, const void* x, bq4_dtype x_dtype, int64_t M, int64_t ldx,
                                   const float* bias, int64_t q_heads, int64_t k_heads, int64_t head_dim,
                                   const float* gamma_q, const float* gamma_k, float eps, const float* cos_t,
                                   const float* sin_t, int64_t ld_rope, void* y, bq4_dtype y_dtype, int64_t ldy,
                                   void* workspace, size_t workspace_bytes, bq4_stream_t stream) {
  bq4_status st = check_weight(w, "w");
  if (st) return st;
  if (head_dim <= 0 || head_dim % 2 || head_dim > 256 || q_heads < 0 || k_heads < 0 || w->N % head_dim ||
      (q_heads + k_heads) * head_dim > w->N)
    return set_error(BQ4_EINVAL_SHAPE, "heads %lld + %lld of %lld (even, <= 256) do not fit N=%lld",
                     (long long)q_heads, (long long)k_heads, (long long)head_dim, (long long)w->N);
  if ((cos_t == nullptr) != (sin_t == nullptr)) return set_error(BQ4_EINVAL_ARG, "cos and sin must both be given");
  if (cos_t && ld_rope < head_dim) return set_error(BQ4_EINVAL_SHAPE, "ld_rope < head_dim");
  if (!(eps > 0.0f)) return set_error(BQ4_EINVAL_ARG, "eps must be positive");
  if (ldy == 0) ldy = w->N;
  if (!qk_fused(w, head_dim)) {
    // the linear, then the norm and rotation in place on its q and k sections
    st = bq4_linear_ex(w, x, x_dtype, M, ldx, bias, BQ4_ACT_NONE, nullptr, y, y_dtype, ldy, workspace,
                       workspace_bytes, stream);
    if (st) return st;
    DeviceGuard guard(w->device);
    const size_t es = y_dtype == BQ4_DTYPE_F16 ? 2 : 4;
    if (q_heads > 0) {
      st = bq4_qk_norm_rope(y, y_dtype, M, q_heads, head_dim, ldy, gamma_q, eps, cos_t, sin_t, ld_rope, y, y_dtype,
                            ldy, stream);
      if (st) return st;
    }
    if (k_heads > 0) {
      void* yk = static_cast<uint8_t*>(y) + (size_t)q_heads * head_dim * es;
      st = bq4_qk_norm_rope(yk, y_dtype, M, k_heads, head_dim, ldy, gamma_k, eps, cos_t, sin_t, ld_rope, yk,
                            y_dtype, ldy, stream);
    }
    return st;
  }
  // fused: every 128-feature tile is one head
  if ((x_dtype != BQ4_DTYPE_F32 && x_dtype != BQ4_DTYPE_F16) || (y_dtype != BQ4_DTYPE_F32 && y_dtype != BQ4_DTYPE_F16))
    return set_error(BQ4_EINVAL_ARG, "x_dtype %d / y_dtype %d unknown", (int)x_dtype, (int)y_dtype);
  if (!x || !y) return set_error(BQ4_EINVAL_ARG, "x/y is NULL");
  if (M <= 0 || M > 0x7fffffff) return set_error(BQ4_EINVAL_SHAPE, "M=%lld", (long long)M);
  if (ldx < w->K) return set_error(BQ4_EINVAL_SHAPE, "ldx=%lld < K=%lld", (long long)ldx, (long long)w->K);
  if (ldy < w->N) return set_error(BQ4_EINVAL_SHAPE, "ldy=%lld < N=%lld", (long long)ldy, (long long)w->N);
  const int x16 = x_dtype == BQ4_DTYPE_F16, y16 = y_dtype == BQ4_DTYPE_F16;
  if (x16) {
    if (w->K != w->Kp)
      return set_error(BQ4_EINVAL_SHAPE, "f16 x needs K %% 128 == 0 (K=%lld)", (long long)w->K);
    if (!aligned(x, 16) || ldx % 8)
      return set_error(BQ4_EALIGN, "f16 x needs a 16-byte aligned base and ldx %% 8 == 0");
  } else if (!aligned(x, 4)) {
    return set_error(BQ4_EALIGN, "x not 4-byte aligned");
  }
  if (!aligned(y, y16 ? 2 : 4)) return set_error(BQ4_EALIGN, "y misaligned");
  GemmPlan plan;
  st = plan_gemm(w, 1, M, w->device, &plan, true, true);
  if (st) return st;
  const size_t need = x16 ? plan.sk_bytes + plan.partial_bytes : plan.workspace_bytes;
  if (need) {
    if (!workspace) return set_error(BQ4_EWORKSPACE, "workspace is NULL");
    if (!aligned(workspace, 256)) return set_error(BQ4_EALIGN, "workspace not 256-byte aligned");
    if (workspace_bytes < need)
      return set_error(BQ4_EWORKSPACE, "workspace %zu < required %zu bytes", workspace_bytes, need);
  }
  DeviceGuard guard(w->device);
  QkParams qk;
  qk.q_heads = (int)q_heads;
  qk.k_heads = (int)k_heads;
  qk.eps = eps;
  qk.gamma_q = gamma_q;
  qk.gamma_k = gamma_k;
  qk.cos_t = cos_t;
  qk.sin_t = sin_t;
  qk.ld_rope = cos_t ? ld_rope : 128;
  const bq4_weight* ws[1] = {w};
  const float* b[1] = {bias};
  GemmIo io;
  io.x_f16 = x16;
  io.y_f16 = y16;
  io.ldy = ldy;
  io.qk = &qk;
  return run_gemm(plan, ws, x, M, ldx, b, (int)BQ4_ACT_NONE, nullptr, y, workspace,
                  reinterpret_cast<cudaStream_t>(stream), io);
}

// ---------------------------------------------------------------- peer exchange

bq4_status bq4_peer_buffer_alloc(size_t bytes, int32_t device, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return set_error(BQ4_EINVAL_ARG, "ptr/handle is NULL or bytes is 0");
  DeviceGuard guard(device);
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return check_cuda(e, "cudaMalloc (peer buffer)");
  e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return check_cuda(e, "peer buffer set-up");
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == BQ4_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return BQ4_OK;
}

bq4_status bq4_peer_buffer_open(const void* handle, int32_t device, void** ptr) {
  if (!ptr || !handle) return set_error(BQ4_EINVAL_ARG, "ptr/handle is NULL");
  DeviceGuard guard(device);
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? BQ4_OK : check_cuda(e, "cudaIpcOpenMemHandle");
}

bq4_status bq4_peer_buffer_close(void* ptr) {
  if (!ptr) return BQ4_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? BQ4_OK : check_cuda(e, "cudaIpcCloseMemHandle");
}

bq4_status bq4_peer_buffer_free(void* ptr, int32_t device) {
  if (!ptr) return BQ4_OK;
  DeviceGuard guard(device);
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? BQ4_OK : check_cuda(e, "cudaFree (peer buffer)");
}

bq4_status bq4_peer_signal_wait(uint32_t* flags, uint32_t* const* peer_flags, int32_t nranks, int32_t rank,
                                uint32_t epoch, bq4_stream_t stream) {
  if (!flags || !peer_flags) return set_error(BQ4_EINVAL_ARG, "flags is NULL");
  if (nranks < 1 || nranks > BQ4_MAX_PEERS || rank < 0 || rank >= nranks)
    return set_error(BQ4_EINVAL_ARG, "rank %d of %d ranks (at most %d)", (int)rank, (int)nranks, BQ4_MAX_PEERS);
  for (int r = 0; r < nranks; ++r)
    if (r != rank && !peer_flags[r]) return set_error(BQ4_EINVAL_ARG, "peer_flags[%d] is NULL", r);
  if (nranks == 1) return BQ4_OK;
  cudaError_t e = launch_peer_signal_wait(flags, peer_flags, nranks, rank, epoch, device_error_word(),
                                          reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? BQ4_OK : check_cuda(e, "peer signal/wait launch");
}

bq4_status bq4_set_peer_wait_timeout_ns(uint64_t ns) {
  set_peer_wait_ns(ns);
  return BQ4_OK;
}

bq4_status bq4_reduce_slices(const float* recv, int32_t nranks, int64_t rows, int64_t H, int64_t ld, int32_t renorm,
                             float eps, void* out, bq4_dtype out_dtype, int64_t ldo, bq4_stream_t stream) {
  if (!recv || !out) return set_error(BQ4_EINVAL_ARG, "recv/out is NULL");
  if (out_dtype != BQ4_DTYPE_F32 && out_dtype != BQ4_DTYPE_F16) return set_error(BQ4_EINVAL_ARG, "dtype unknown");
  if (nranks < 1 || nranks > BQ4_MAX_PEERS || rows <= 0 || H <= 0 || H % 4 || H > 8192 || ld < H || ld % 4 ||
      ldo < H || ldo % 4)
    return set_error(BQ4_EINVAL_SHAPE, "nranks=%d rows=%lld H=%lld (H %% 4 == 0, <= 8192) ld=%lld ldo=%lld",
                     (int)nranks, (long long)rows, (long long)H, (long long)ld, (long long)ldo);
  if (renorm && !(eps > 0.0f)) return set_error(BQ4_EINVAL_ARG, "eps must be positive");
  if (!aligned(recv, 16) || !aligned(out, out_dtype == BQ4_DTYPE_F16 ? 8 : 16))
    return set_error(BQ4_EALIGN, "recv/out misaligned");
  cudaError_t e = launch_reduce_slices(recv, nranks, rows, H, ld, renorm, eps, out, out_dtype == BQ4_DTYPE_F16, ldo,
                                       reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? BQ4_OK : check_cuda(e, "reduce_slices launch");
}

bq4_status bq4_reduce_slices_peer(const float* const* src_ranks, int32_t nranks, int64_t row0, int64_t rows,
                                  int64_t H, int64_t ld, int32_t renorm, float eps, void* out, bq4_dtype out_dtype,
                                  int64_t ldo, bq4_stream_t stream) {
  if (!src_ranks || !out) return set_error(BQ4_EINVAL_ARG, "src_ranks/out is NULL");
  if (out_dtype != BQ4_DTYPE_F32 && out_dtype != BQ4_DTYPE_F16) return set_error(BQ4_EINVAL_ARG, "dtype unknown");
  if (nranks < 1 || nranks > BQ4_MAX_PEERS || row0 < 0 || rows <= 0 || H <= 0 || H % 4 || H > 8192 || ld < H ||
      ld % 4 || ldo < H || ldo % 4)
    return set_error(BQ4_EINVAL_SHAPE, "nranks=%d row0=%lld rows=%lld H=%lld (H %% 4 == 0, <= 8192) ld=%lld ldo=%lld",
                     (int)nranks, (long long)row0, (long long)rows, (long long)H, (long long)ld, (long long)ldo);
  if (renorm && !(eps > 0.0f)) return set_error(BQ4_EINVAL_ARG, "eps must be positive");
  for (int r = 0; r < nranks; ++r)
    if (!src_ranks[r] || !aligned(src_ranks[r], 16))
      return set_error(BQ4_EALIGN, "src_ranks[%d] is NULL or not 16-byte aligned", r);
  if (!aligned(out, out_dtype == BQ4_DTYPE_F16 ? 8 : 16)) return set_error(BQ4_EALIGN, "out misaligned");
  cudaError_t e = launch_reduce_slices_peer(src_ranks, nranks, row0, rows, H, ld, renorm, eps, out, nullptr,
                                            out_dtype == BQ4_DTYPE_F16, ldo, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? BQ4_OK : check_cuda(e, "reduce_slices_peer launch");
}

bq4_status bq4_reduce_slices_peer_bcast(const float* const* src_ranks, int32_t nranks, int64_t row0, int64_t rows,
                                        int64_t H, int64_t ld, int32_t renorm, float eps, void* const* out_ranks,
                                        bq4_dtype out_dtype, int64_t ldo, bq4_stream_t stream) {
  if (!src_ranks || !out_ranks) return set_error(BQ4_EINVAL_ARG, "src_ranks/out_ranks is NULL");
  if (out_dtype != BQ4_DTYPE_F32 && out_dtype != BQ4_DTYPE_F16) return set_error(BQ4_EINVAL_ARG, "dtype unknown");
  if (nranks < 1 || nranks > BQ4_MAX_PEERS || row0 < 0 || rows <= 0 || H <= 0 || H % 4 || H > 8192 || ld < H ||
      ld % 4 || ldo < H || ldo % 4)
    return set_error(BQ4_EINVAL_SHAPE, "nranks=%d row0=%lld rows=%lld H=%lld (H %% 4 == 0, <= 8192) ld=%lld ldo=%lld",
                     (int)nranks, (long long)row0, (long long)rows, (long long)H, (long long)ld, (long long)ldo);
  if (renorm && !(eps > 0.0f)) return set_error(BQ4_EINVAL_ARG, "eps must be positive");
  for (int r = 0; r < nranks; ++r) {
    if (!src_ranks[r] || !aligned(src_ranks[r], 16))
      return set_error(BQ4_EALIGN, "src_ranks[%d] is NULL or not 16-byte aligned", r);
    if (!out_ranks[r] || !aligned(out_ranks[r], out_dtype == BQ4_DTYPE_F16 ? 8 : 16))
      return set_error(BQ4_EALIGN, "out_ranks[%d] is NULL or misaligned", r);
  }
  cudaError_t e = launch_reduce_slices_peer(src_ranks, nranks, row0, rows, H, ld, renorm, eps, out_ranks[0],
                                            out_ranks, out_dtype == BQ4_DTYPE_F16, ldo,
                                            reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? BQ4_OK : check_cuda(e, "reduce_slices_peer_bcast launch");
}

bq4_status bq4_linear_rowscatter(const bq4_weight* w, const void* x, bq4_dtype x_dtype, int64_t M, int64_t ldx,
                                 const float* bias, bq4_act act, float* const* y_ranks, int32_t nranks, int32_t rank,
                                 int64_t ldy, void* workspace, size_t workspace_bytes, bq4_stream_t stream) {
  bq4_status st = check_weight(w, "w");
  if (st) return st;
  if (act != BQ4_ACT_NONE && act != BQ4_ACT_GELU_TANH && act != BQ4_ACT_SILU)
    return set_error(BQ4_EINVAL_ARG, "act %d unknown", (int)act);
  if (x_dtype != BQ4_DTYPE_F32 && x_dtype != BQ4_DTYPE_F16) return set_error(BQ4_EINVAL_ARG, "x_dtype unknown");
  if (!x || !y_ranks) return set_error(BQ4_EINVAL_ARG, "x/y_ranks is NULL");
  if (nranks < 1 || nranks > BQ4_MAX_PEERS || rank < 0 || rank >= nranks)
    return set_error(BQ4_EINVAL_ARG, "rank %d of %d ranks (at most %d)", (int)rank, (int)nranks, BQ4_MAX_PEERS);
  for (int r = 0; r < nranks; ++r)
    if (!y_ranks[r] || !aligned(y_ranks[r], 4)) return set_error(BQ4_EINVAL_ARG, "y_ranks[%d] is NULL or misaligned", r);
  if (M <= 0 || M % nranks || M > 0x7fffffff)
    return set_error(BQ4_EINVAL_SHAPE, "M=%lld must be a positive multiple of nranks=%d", (long long)M, (int)nranks);
  if (ldx < w->K) return set_error(BQ4_EINVAL_SHAPE, "ldx=%lld < K=%lld", (long long)ldx, (long long)w->K);
  if (ldy == 0) ldy = w->N;
  if (ldy < w->N) return set_error(BQ4_EINVAL_SHAPE, "ldy=%lld < N=%lld", (long long)ldy, (long long)w->N);
  const int x16 = x_dtype == BQ4_DTYPE_F16;
  if (x16) {
    if (w->K != w->Kp) return set_error(BQ4_EINVAL_SHAPE, "f16 x needs K %% 128 == 0 (K=%lld)", (long long)w->K);
    if (!aligned(x, 16) || ldx % 8) return set_error(BQ4_EALIGN, "f16 x needs a 16-byte aligned base and ldx %% 8 == 0");
  } else if (!aligned(x, 4)) {
    return set_error(BQ4_EALIGN, "x not 4-byte aligned");
  }
  GemmPlan plan;
  st = plan_gemm(w, 1, M, w->device, &plan);
  if (st) return st;
  const size_t need = x16 ? plan.sk_bytes + plan.partial_bytes : plan.workspace_bytes;
  if (need) {
    if (!workspace) return set_error(BQ4_EWORKSPACE, "workspace is NULL");
    if (!aligned(workspace, 256)) return set_error(BQ4_EALIGN, "workspace not 256-byte aligned");
    if (workspace_bytes < need)
      return set_error(BQ4_EWORKSPACE, "workspace %zu < required %zu bytes", workspace_bytes, need);
  }
  DeviceGuard guard(w->device);
  const bq4_weight* ws[1] = {w};
  const float* b[1] = {bias};
  GemmIo io;
  io.x_f16 = x16;
  io.y_f16 = 0;
  io.ldy = ldy;
  io.sc_rows = (int)(M / nranks);
  io.sc_rank = rank;
  io.sc_nranks = nranks;
  io.sc_y = y_ranks;
  return run_gemm(plan, ws, x, M, ldx, b, (int)act, nullptr, y_ranks[rank], workspace,
                  reinterpret_cast<cudaStream_t>(stream), io);
}

bq4_status bq4_linear_ex_workspace_size(const bq4_weight* w, int64_t M, bq4_dtype x_dtype, size_t* bytes) {
  if (x_dtype != BQ4_DTYPE_F32 && x_dtype != BQ4_DTYPE_F16)
    return set_error(BQ4_EINVAL_ARG, "x_dtype %d unknown", (int)x_dtype);
  bq4_status st = check_weight(w, "w");
  if (st) return st;
  if (!bytes) return set_error(BQ4_EINVAL_ARG, "bytes is NULL");
  GemmPlan plan;
  st = plan_gemm(w, 1, M, w->device, &plan);
  if (st) return st;
  *bytes = x_dtype == BQ4_DTYPE_F16 ? plan.sk_bytes + plan.partial_bytes : plan.workspace_bytes;
  return BQ4_OK;
}

bq4_status bq4_linear_ex(const bq4_weight* w, const void* x, bq4_dtype x_dtype, int64_t M, int64_t ldx,
                         const float* bias, bq4_act act, const float* aux, void* y, bq4_dtype y_dtype,
                         int64_t ldy, void* workspace, size_t workspace_bytes, bq4_stream_t stream) {
  bq4_status st = check_weight(w, "w");
  if (st) return st;
  if (act != BQ4_ACT_NONE && act != BQ4_ACT_GELU_TANH && act != BQ4_ACT_SILU)
    return set_error(BQ4_EINVAL_ARG, "act %d unknown", (int)act);
  if ((x_dtype != BQ4_DTYPE_F32 && x_dtype != BQ4_DTYPE_F16) ||
      (y_dtype != BQ4_DTYPE_F32 && y_dtype != BQ4_DTYPE_F16))
    return set_error(BQ4_EINVAL_ARG, "x_dtype %d / y_dtype %d unknown", (int)x_dtype, (int)y_dtype);
  if (!x || !y) return set_error(BQ4_EINVAL_ARG, "x/y is NULL");
  if (M <= 0) return set_error(BQ4_EINVAL_SHAPE, "M=%lld must be positive", (long long)M);
  if (ldx < w->K) return set_error(BQ4_EINVAL_SHAPE, "ldx=%lld < K=%lld", (long long)ldx, (long long)w->K);
  if (ldy == 0) ldy = w->N;
  if (ldy < w->N) return set_error(BQ4_EINVAL_SHAPE, "ldy=%lld < N=%lld", (long long)ldy, (long long)w->N);
  const int x16 = x_dtype == BQ4_DTYPE_F16, y16 = y_dtype == BQ4_DTYPE_F16;
  if (x16) {
    if (w->K != w->Kp)
      return set_error(BQ4_EINVAL_SHAPE, "f16 x needs K %% 128 == 0 (K=%lld)", (long long)w->K);
    if (!aligned(x, 16) || ldx % 8)
      return set_error(BQ4_EALIGN, "f16 x needs a 16-byte aligned base and ldx %% 8 == 0");
  } else if (!aligned(x, 4)) {
    return set_error(BQ4_EALIGN, "x not 4-byte aligned");
  }
  if (!aligned(y, y16 ? 2 : 4)) return set_error(BQ4_EALIGN, "y misaligned");
  GemmPlan plan;
  st = plan_gemm(w, 1, M, w->device, &plan);
  if (st) return st;
  const size_t need = x16 ? plan.sk_bytes + plan.partial_bytes : plan.workspace_bytes;
  if (need) {
    if (!workspace) return set_error(BQ4_EWORKSPACE, "workspace is NULL");
    if (!aligned(workspace, 256)) return set_error(BQ4_EALIGN, "workspace not 256-byte aligned");
    if (workspace_bytes < need)
      return set_error(BQ4_EWORKSPACE, "workspace %zu < required %zu bytes", workspace_bytes, need);
  }
  DeviceGuard guard(w->device);
  const bq4_weight* ws[1] = {w};
  const float* b[1] = {bias};
  GemmIo io;
  io.x_f16 = x16;
  io.y_f16 = y16;
  io.ldy = ldy;
  return run_gemm(plan, ws, x, M, ldx, b, (int)act, aux, y, workspace, reinterpret_cast<cudaStream_t>(stream),
                  io);
}

bq4_status bq4_linear_gated_workspace_size(const bq4_weight* gate, const bq4_weight* up, int64_t M,
                                           size_t* bytes) {
  bq4_status st = check_weight(gate, "gate");
  if (st) return st;
  st = check_weight(up, "up");
  if (st) return st;
  if (!bytes) return set_error(BQ4_EINVAL_ARG, "bytes is NULL");
  GemmPlan plan;
  st = plan_gemm(gate, 2, M, gate->device, &plan);
  if (st) return st;
  *bytes = plan.workspace_bytes;
  return BQ4_OK;
}

bq4_status bq4_linear_gated(const bq4_weight* gate, const bq4_weight* up, const float* x,
                            int64_t M, int64_t ldx, const float* gate_bias, const float* up_bias,
                            float* y, void* workspace, size_t workspace_bytes,
                            bq4_stream_t stream) {
  bq4_status st = check_weight(gate, "gate");
  if (st) return st;
  st = check_weight(up, "up");
  if (st) return st;
  if (gate->K != up->K || gate->N != up->N || gate->block != up->block || gate->device != up->device)
    return set_error(BQ4_EINVAL_SHAPE, "gate and up weights differ in K/N/block/device");
  // one kernel streams both weights: the same prepared form (pre-expanded
  // N-packed tiles, or nibbles + scales), and packed-Q4 weights only
  if ((gate->h != nullptr) != (up->h != nullptr) || gate->tf32 || up->tf32)
    return set_error(BQ4_EINVAL_ARG, "gate and up must both be packed-Q4 weights of the same prepared form");
  st = check_compute_args(gate, x, M, ldx, y, workspace);
  if (st) return st;
  GemmPlan plan;
  st = plan_gemm(gate, 2, M, gate->device, &plan);
  if (st) return st;
  if (workspace_bytes < plan.workspace_bytes)
    return set_error(BQ4_EWORKSPACE, "workspace %zu < required %zu bytes", workspace_bytes,
                     plan.workspace_bytes);
  DeviceGuard guard(gate->device);
  const bq4_weight* ws[2] = {gate, up};
  const float* b[2] = {gate_bias, up_bias};
  return run_gemm(plan, ws, x, M, ldx, b, BQ4_ACT_NONE, nullptr, y, workspace,
                  reinterpret_cast<cudaStream_t>(stream));
}

bq4_status bq4_dequant(const bq4_weight* w, float* out, bq4_layout out_layout, bq4_stream_t stream) {
  bq4_status st = check_weight(w, "w");
  if (st) return st;
  if (!out) return set_error(BQ4_EINVAL_ARG, "out is NULL");
  if (out_layout != BQ4_LAYOUT_COL && out_layout != BQ4_LAYOUT_ROW)
    return set_error(BQ4_EINVAL_ARG, "out_layout %d", (int)out_layout);
  if (w->tf32)
    return set_error(BQ4_EUNSUPPORTED,
                     "a packed-F16 weight holds no Q4 values; widen its source with bq4_packed_f16_to_f32");
  if (w->h)
    return set_error(BQ4_EUNSUPPORTED,
                     "weight was prepared from BQ4_LAYOUT_NPACKED (pre-expanded f16); use bq4_dequant_raw");
  DeviceGuard guard(w->device);
  return check_cuda(launch_dequant_prepared(w, out, out_layout, reinterpret_cast<cudaStream_t>(stream)),
                    "bq4_dequant");
}

bq4_status bq4_dequant_raw(const uint32_t* packed_words, const float* scales, int64_t K, int64_t N,
                           int32_t block, bq4_layout layout, float* out, bq4_layout out_layout,
                           bq4_stream_t stream) {
  bq4_status st = check_geometry(K, N, block, layout);
  if (st) return st;
  if (!packed_words || !scales || !out) return set_error(BQ4_EINVAL_ARG, "NULL pointer");
  if (out_layout != BQ4_LAYOUT_COL && out_layout != BQ4_LAYOUT_ROW)
    return set_error(BQ4_EINVAL_ARG, "out_layout %d", (int)out_layout);
  int dev = 0;
  cudaGetDevice(&dev);
  st = require_sm100(dev);
  if (st) return st;
  return check_cuda(launch_dequant_raw(packed_words, scales, K, N, block, layout, out, out_layout,
                                       reinterpret_cast<cudaStream_t>(stream)),
                    "bq4_dequant_raw");
}

// ------------------------------------------------------------ q_matmul mirror

static bq4_status check_scheme(const bq4_quant_scheme* s) {
  // patches/burn-cubecl-0.21.0/src/ops/qtensor.rs:304-323
  if (!s) return set_error(BQ4_EINVAL_ARG, "scheme is NULL");
  if (s->value != 0) return set_error(BQ4_EINVAL_ARG, "scheme value is not Q4S");
  if (s->mode != 0) return set_error(BQ4_EINVAL_ARG, "scheme mode is not Symmetric");
  if (s->param != 0) return set_error(BQ4_EINVAL_ARG, "scheme param is not F32");
  if (s->store_packed_dim != 0 && s->store_packed_dim != 1)
    return set_error(BQ4_EINVAL_ARG, "scheme store is not PackedU32(0|1)");
  if (s->block_rank != 1 && s->block_rank != 2)
    return set_error(BQ4_EINVAL_ARG, "scheme level is not Block([b]) or Block([b,1])");
  if (!valid_block(s->block)) return set_error(BQ4_EINVAL_BLOCK, "block %d unsupported", s->block);
  return BQ4_OK;
}

static void q_matmul_view(int64_t K, int64_t N, int32_t block, int32_t layout, bq4_weight* w) {
  memset(w, 0, sizeof(*w));
  w->layout = layout;
  w->K = K;
  w->N = N;
  w->block = block;
  w->Kp = (K + kStageK - 1) / kStageK * kStageK;
  w->nkc = w->Kp / kChunkK;
  w->nkb = w->Kp / block;
  w->ntiles = (N + kTileN - 1) / kTileN;
  w->Np = w->ntiles * kTileN;
  if (layout == BQ4_LAYOUT_NPACKED) {
    w->h_bytes = (size_t)w->ntiles * w->nkc * 128 * 64 * 2;
  } else {
    w->q_bytes = (size_t)w->ntiles * w->nkc * 1024 * 4;
    w->s_bytes = (size_t)w->ntiles * w->nkb * 128 * 4;
  }
}

static size_t q_matmul_weight_bytes(const bq4_weight& w) {
  return (w.q_bytes + 255) / 256 * 256 + (w.s_bytes + 255) / 256 * 256 + (w.h_bytes + 255) / 256 * 256;
}

bq4_status bq4_q_matmul_workspace_size(int64_t M, int64_t K, int64_t N, const bq4_quant_scheme* scheme,
                                       size_t* bytes) {
  bq4_status st = check_scheme(scheme);
  if (st) return st;
  const int32_t layout = scheme->store_packed_dim == 1 ? BQ4_LAYOUT_ROW
                         : (scheme->rhs_transposed_view ? BQ4_LAYOUT_COL : BQ4_LAYOUT_NPACKED);
  st = check_geometry(K, N, scheme->block, layout);
  if (st) return st;
  if (!bytes) return set_error(BQ4_EINVAL_ARG, "bytes is NULL");
  bq4_weight w;
  q_matmul_view(K, N, scheme->block, layout, &w);
  int dev = 0;
  cudaGetDevice(&dev);
  GemmPlan plan;
  st = plan_gemm(&w, 1, M, dev, &plan);
  if (st) return st;
  *bytes = q_matmul_weight_bytes(w) + plan.workspace_bytes;
  return BQ4_OK;
}

bq4_status bq4_q_matmul(const float* lhs, int64_t M, int64_t K, const uint32_t* rhs_values,
                        const float* rhs_scales, int64_t N, const bq4_quant_scheme* scheme,
                        float* out, void* workspace, size_t workspace_bytes, bq4_stream_t stream) {
  bq4_status st = check_scheme(scheme);
  if (st) return st;
  // PackedU32(1): the stored [K,N] tensor is packed along K (Boogu row
  // layout).  PackedU32(0): packed along the stored tensor's last axis -- K
  // when rhs is the transposed view of a stored [N,K] tensor (Qwen), N when
  // rhs is stored as a plain [K,N] tensor.
  const int32_t layout = scheme->store_packed_dim == 1 ? BQ4_LAYOUT_ROW
                         : (scheme->rhs_transposed_view ? BQ4_LAYOUT_COL : BQ4_LAYOUT_NPACKED);
  st = check_geometry(K, N, scheme->block, layout);
  if (st) return st;
  if (!rhs_values || !rhs_scales || !lhs || !out) return set_error(BQ4_EINVAL_ARG, "NULL pointer");
  int dev = 0;
  cudaGetDevice(&dev);
  st = require_sm100(dev);
  if (st) return st;
  bq4_weight w;
  q_matmul_view(K, N, scheme->block, layout, &w);
  w.device = dev;
  size_t need = 0;
  st = bq4_q_matmul_workspace_size(M, K, N, scheme, &need);
  if (st) return st;
  if (!workspace || workspace_bytes < need)
    return set_error(BQ4_EWORKSPACE, "workspace %zu < required %zu bytes", workspace_bytes, need);
  if (!aligned(workspace, 256)) return set_error(BQ4_EALIGN, "workspace not 256-byte aligned");
  uint8_t* p = static_cast<uint8_t*>(workspace);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (layout == BQ4_LAYOUT_NPACKED) {
    w.h = reinterpret_cast<uint16_t*>(p);
    p += (w.h_bytes + 255) / 256 * 256;
    e = launch_prepare_pre(rhs_values, rhs_scales, K, N, scheme->block, 0, 0, N, K, &w, s);
  } else {
    w.q = reinterpret_cast<uint32_t*>(p);
    p += (w.q_bytes + 255) / 256 * 256;
    w.s = reinterpret_cast<float*>(p);
    p += (w.s_bytes + 255) / 256 * 256;
    e = launch_prepare(rhs_values, rhs_scales, K, N, scheme->block, layout, 0, 0, N, K, &w, s);
  }
  if (e != cudaSuccess) return check_cuda(e, "q_matmul prepare");
  GemmPlan plan;
  st = plan_gemm(&w, 1, M, dev, &plan);
  if (st) return st;
  const bq4_weight* ws[1] = {&w};
  const float* b[1] = {nullptr};
  return run_gemm(plan, ws, lhs, M, K, b, BQ4_ACT_NONE, nullptr, out, p, s);
}

// ------------------------------------------------------------ host packers

int32_t bq4_row_block_for(int64_t input) {
  static const int32_t groups[5] = {128, 64, 32, 16, 8};
  for (int i = 0; i < 5; ++i)
    if (input > 0 && input % groups[i] == 0) return groups[i];
  return 0;
}

static inline int8_t q4_quantize(float v, float inverse) {
  float q = std::round(v * inverse);  // f32::round: half away from zero
  if (q < -7.0f) q = -7.0f;
  if (q > 7.0f) q = 7.0f;
  return static_cast<int8_t>(q);
}

static inline float q4_scale(float alpha) {
  return alpha == 0.0f ? 1.17549435e-38f /* f32::MIN_POSITIVE */ : alpha / 7.0f;
}

bq4_status bq4_quantize_col_block128(const float* values, int64_t rows, int64_t inner,
                                     uint32_t* words, float* scales) {
  // crates/burn_qwen3_vl/src/artifacts.rs:1301-1366
  if (!values || !words || !scales) return set_error(BQ4_EINVAL_ARG, "NULL pointer");
  if (rows <= 0 || inner <= 0 || inner % 128 != 0)
    return set_error(BQ4_EINVAL_SHAPE, "inner dimension %lld is not divisible by 128", (long long)inner);
  const int64_t total = rows * inner;
  for (int64_t i = 0; i < total; ++i)
    if (!std::isfinite(values[i])) return set_error(BQ4_ENONFINITE, "non-finite value at %lld", (long long)i);
  for (int64_t blk = 0; blk < total / 128; ++blk) {
    const float* v = values + blk * 128;
    float alpha = 0.0f;
    for (int i = 0; i < 128; ++i) alpha = std::fmax(alpha, std::fabs(v[i]));
    const float sc = q4_scale(alpha);
    scales[blk] = sc;
    const float inverse = 1.0f / sc;
    for (int wi = 0; wi < 16; ++wi) {
      uint32_t word = 0;
      for (int lane = 0; lane < 8; ++lane)
        word |= (uint32_t)((uint8_t)q4_quantize(v[wi * 8 + lane], inverse) & 0x0f) << (lane * 4);
      words[blk * 16 + wi] = word;
    }
  }
  return BQ4_OK;
}

bq4_status bq4_quantize_row_up_to128(const float* values, int64_t input, int64_t output,
                                     uint32_t* words, float* scales, int32_t* block_out) {
  // crates/burn_boogu/src/artifacts.rs:7296-7385
  if (!values || !words || !scales || !block_out) return set_error(BQ4_EINVAL_ARG, "NULL pointer");
  if (input <= 0 || output <= 0 || output % 8 != 0)
    return set_error(BQ4_EINVAL_SHAPE, "output width %lld is not divisible by 8", (long long)output);
  const int32_t block = bq4_row_block_for(input);
  if (!block)
    return set_error(BQ4_EINVAL_BLOCK, "input width %lld has no supported exact block", (long long)input);
  for (int64_t i = 0; i < input * output; ++i)
    if (!std::isfinite(values[i])) return set_error(BQ4_ENONFINITE, "non-finite value at %lld", (long long)i);
  std::vector<int8_t> q((size_t)(input * output));
  for (int64_t kb = 0; kb < input / block; ++kb) {
    const int64_t k0 = kb * block;
    for (int64_t n = 0; n < output; ++n) {
      float alpha = 0.0f;
      for (int64_t k = k0; k < k0 + block; ++k) alpha = std::fmax(alpha, std::fabs(values[k * output + n]));
      const float sc = q4_scale(alpha);
      scales[kb * output + n] = sc;
      const float inverse = 1.0f / sc;
      for (int64_t k = k0; k < k0 + block; ++k) q[k * output + n] = q4_quantize(values[k * output + n], inverse);
    }
  }
  for (int64_t kw = 0; kw < input / 8; ++kw)
    for (int64_t n = 0; n < output; ++n) {
      uint32_t word = 0;
      for (int lane = 0; lane < 8; ++lane)
        word |= (uint32_t)((uint8_t)q[(kw * 8 + lane) * output + n] & 0x0f) << (lane * 4);
      words[kw * output + n] = word;
    }
  *block_out = block;
  return BQ4_OK;
}

}  // extern "C"
