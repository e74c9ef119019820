// bq4_noalloc.cu -- bq4_linear for callers that cannot allocate device memory.
//
// bq4_linear needs a caller-provided workspace (the f16 copy of the
// activations, the split-K partial tiles and the stream-K slots).  Some
// callers have no way to provide one: a host runtime whose allocator owns
// all device memory and offers no hook to hand a foreign op a scratch
// buffer, code that must not call cudaMalloc because it synchronizes the
// device, or a process that is not permitted to grow its device footprint
// after start-up.  For them
// bq4_linear_noalloc runs the same GEMM with its scratch in a fixed-size
// static device array that every GPU loading this library holds until the
// process exits (BQ4_NOALLOC_SCRATCH_BYTES per device).
//
// The array's host-side name is only a stand-in; its device address is
// looked up with cudaGetSymbolAddress once per device (with that device
// current) on the first call there, and cached.  Calls on one device share
// the array: two calls that overlap on the GPU (different streams, or
// different host threads without ordering) race on it.  It holds the f16
// copy of the activations, the split-K partial tiles and the stream-K
// partial slots, which every call writes in full before anything reads
// them, and the stream-K flags, which the call zeroes first -- so nothing in
// it needs to start at zero.
#include <cuda_runtime.h>

#include <mutex>

#include "bq4_internal.h"

namespace bq4 {
namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[BQ4_NOALLOC_SCRATCH_BYTES];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {nullptr};

// Device address of the scratch array on `device` (which must be current).
bq4_status noalloc_scratch(int device, void** out) {
  if (device < 0 || device >= 64) return set_error(BQ4_EINVAL_ARG, "device %d out of range", device);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) return check_cuda(e != cudaSuccess ? e : cudaErrorInvalidSymbol,
                                                  "cudaGetSymbolAddress(no-alloc scratch)");
    g_noalloc_ptr[device] = p;
  }
  *out = g_noalloc_ptr[device];
  return BQ4_OK;
}

}  // namespace
}  // namespace bq4

using namespace bq4;

extern "C" bq4_status bq4_linear_noalloc(const bq4_weight* w, const float* x, int64_t M, int64_t ldx,
                                         const float* bias, bq4_act act, const float* aux, float* y,
                                         bq4_stream_t stream) {
  if (!w || !((w->q && w->s) || w->h)) return set_error(BQ4_EINVAL_ARG, "w is NULL or freed");
  if (act != BQ4_ACT_NONE && act != BQ4_ACT_GELU_TANH && act != BQ4_ACT_SILU)
    return set_error(BQ4_EINVAL_ARG, "act %d unknown", (int)act);
  if (!x || !y) return set_error(BQ4_EINVAL_ARG, "x/y is NULL");
  if (M <= 0) return set_error(BQ4_EINVAL_SHAPE, "M=%lld must be positive", (long long)M);
  if (ldx < w->K)
    return set_error(BQ4_EINVAL_SHAPE, "ldx=%lld < K=%lld", (long long)ldx, (long long)w->K);
  if ((reinterpret_cast<uintptr_t>(x) & 3) || (reinterpret_cast<uintptr_t>(y) & 3))
    return set_error(BQ4_EALIGN, "x/y not 4-byte aligned");
  GemmPlan plan;
  bq4_status st = plan_gemm(w, 1, M, w->device, &plan);
  if (st == BQ4_OK && plan.sk_tiles && plan.workspace_bytes > (size_t)BQ4_NOALLOC_SCRATCH_BYTES)
    st = plan_gemm(w, 1, M, w->device, &plan, false);  // whole tiles need no stream-K slots
  if (st) return st;
  if (plan.workspace_bytes > (size_t)BQ4_NOALLOC_SCRATCH_BYTES)
    return set_error(BQ4_EWORKSPACE,
                     "bq4_linear_noalloc: M=%lld K=%lld needs %zu bytes of scratch, above its static "
                     "limit of %zu bytes; use bq4_linear with a workspace",
                     (long long)M, (long long)w->K, plan.workspace_bytes,
                     (size_t)BQ4_NOALLOC_SCRATCH_BYTES);
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != w->device) {
    cudaError_t e = cudaSetDevice(w->device);
    if (e != cudaSuccess) return check_cuda(e, "cudaSetDevice");
  }
  void* scratch = nullptr;
  st = noalloc_scratch(w->device, &scratch);
  if (st == BQ4_OK) {
    const bq4_weight* ws[1] = {w};
    const float* b[1] = {bias};
    st = run_gemm(plan, ws, x, M, ldx, b, (int)act, aux, y, scratch,
                  reinterpret_cast<cudaStream_t>(stream));
  }
  if (prev >= 0 && prev != w->device) cudaSetDevice(prev);
  return st;
}
