// bq4_peer.cu -- the pieces of the tensor-parallel exchange that run over
// NVLink peer memory between the GPUs of one node (one process per GPU).
//
// A row-parallel linear's partial products are written by its GEMM
// epilogue straight into the buffer of the rank that owns each output row
// (bq4_linear_rowscatter); ranks then pass a cross-GPU signal/wait
// (bq4_peer_signal_wait) and each owner sums the partials of its rows in
// rank order, optionally RMS-renormalising them (bq4_reduce_slices).  In the
// pull form each rank's GEMM writes its whole partial product into its own
// shared buffer, and after the signal/wait each owner reads its rows from
// every rank's buffer (bq4_reduce_slices_peer).  The shared buffers are
// plain cudaMalloc allocations exported with CUDA IPC handles
// (bq4_peer_buffer_*): plain peer loads and stores between GPUs.
//
// Every wait is bounded: a signal/wait that times out records BQ4_ETIMEOUT
// in the device error word and returns.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstring>

#include "bq4_internal.h"
#include "sm100_ptx.cuh"

namespace bq4 {
namespace {

constexpr uint64_t kPeerWaitNs = 10000000000ull;  // default 10 s: ranks enqueue at their own pace
std::atomic<uint64_t> g_peer_wait_ns{kPeerWaitNs};

__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void st4(__half* p, float4 v) {  // round to nearest even, as the staging kernel
  const __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
  *reinterpret_cast<uint2*>(p) = make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
}

struct PeerFlags {
  unsigned* p[BQ4_MAX_PEERS];
};

// One thread: publish `epoch` into slot `rank` of every peer's flag array
// (release at system scope, so everything this rank wrote before -- the
// kernels ahead of this one on its stream -- is visible to a peer that
// reads the flag with acquire), then wait until every peer has published
// `epoch` into this rank's own array.
__global__ void peer_signal_wait_kernel(unsigned* local, PeerFlags peers, int nranks, int rank, unsigned epoch,
                                        uint64_t limit_ns, int* err) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  __threadfence_system();
  for (int r = 0; r < nranks; ++r)
    if (r != rank)
      asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(peers.p[r] + rank), "r"(epoch) : "memory");
  const uint64_t t0 = ptx::globaltimer();
  for (int r = 0; r < nranks; ++r) {
    if (r == rank) continue;
    while (true) {
      unsigned v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(local + r) : "memory");
      if ((int)(v - epoch) >= 0) break;
      if (ptx::globaltimer() - t0 > limit_ns) {
        if (err) atomicExch(err, (int)BQ4_ETIMEOUT);
        return;
      }
      __nanosleep(256);
    }
  }
}

// The P partial slices of a reduction: slice s, row r is src.p[s] + (row0 + r) * ld.
struct SliceSrc {
  const float* p[BQ4_MAX_PEERS];
};
// Where the reduced rows go: n == 0: out + r * ldo; else row r of the result
// to p[q] + (row0 + r) * ldo for every q < n (every rank's copy of the
// activations, over peer memory).
struct RowDst {
  void* p[BQ4_MAX_PEERS];
  int n;
  int64_t row0;
};

// out[r] = sum over s = 0..P-1 (in that order) of slice s, row r, for the R
// rows this rank owns (rows of H floats at pitch ld), then optionally the
// per-row RMS renorm with the thread mapping and arithmetic of
// rms_renorm_vec4_kernel (so the result matches an all-reduce followed by
// that kernel bit for bit when the summation orders agree).  H % 4 == 0.
// The slices are one local receive buffer (the push exchange: [P][R] rows)
// or the ranks' own partial buffers read over peer memory (the pull
// exchange: rank s's full [M] rows, this rank's R starting at row0); a
// thread issues the loads of all P slices of its columns before adding, so
// P remote reads are in flight together.
template <typename TO, bool kRenorm>
__global__ void reduce_slices_kernel(const SliceSrc src, int P, int64_t row0, int64_t R, int64_t H, int64_t ld,
                                     float eps, TO* __restrict__ out, int64_t ldo, const RowDst dst) {
  constexpr int kMaxVec = 8;  // H <= 8 * 4 * blockDim.x
  __shared__ float part[32];
  for (int64_t r = blockIdx.x; r < R; r += gridDim.x) {
    float4 v[kMaxVec];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
      const int64_t h = ((int64_t)threadIdx.x + (int64_t)i * blockDim.x) * 4;
      v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (h < H) {
        for (int s = 0; s < P; ++s) {
          const float4 t = *reinterpret_cast<const float4*>(src.p[s] + (row0 + r) * ld + h);
          v[i].x += t.x; v[i].y += t.y; v[i].z += t.z; v[i].w += t.w;
        }
        ss = fmaf(v[i].x, v[i].x, ss); ss = fmaf(v[i].y, v[i].y, ss);
        ss = fmaf(v[i].z, v[i].z, ss); ss = fmaf(v[i].w, v[i].w, ss);
      }
    }
    float rs = 1.0f;
    if (kRenorm) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
      __syncthreads();
      if (threadIdx.x < 32) {
        float t = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (threadIdx.x == 0) part[0] = t;
      }
      __syncthreads();
      rs = rsqrtf(part[0] / (float)H + eps);
      __syncthreads();  // part[] is rewritten by the next row
    }
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
      const int64_t h = ((int64_t)threadIdx.x + (int64_t)i * blockDim.x) * 4;
      if (h >= H) continue;
      const float4 o = make_float4(v[i].x * rs, v[i].y * rs, v[i].z * rs, v[i].w * rs);
      if (dst.n == 0) {
        st4(out + r * ldo + h, o);
      } else {
        for (int q = 0; q < dst.n; ++q) st4(static_cast<TO*>(dst.p[q]) + (dst.row0 + r) * ldo + h, o);
      }
    }
  }
}

}  // namespace

void set_peer_wait_ns(uint64_t ns) { g_peer_wait_ns.store(ns ? ns : kPeerWaitNs, std::memory_order_relaxed); }

cudaError_t launch_peer_signal_wait(unsigned* local, unsigned* const* peers, int nranks, int rank, unsigned epoch,
                                    int* err, cudaStream_t s) {
  PeerFlags pf;
  memset(&pf, 0, sizeof(pf));
  for (int r = 0; r < nranks && r < BQ4_MAX_PEERS; ++r) pf.p[r] = peers[r];
  peer_signal_wait_kernel<<<1, 32, 0, s>>>(local, pf, nranks, rank, epoch,
                                           g_peer_wait_ns.load(std::memory_order_relaxed), err);
  note_launch();
  return cudaGetLastError();
}

namespace {
cudaError_t launch_reduce(const SliceSrc& src, int P, int64_t row0, int64_t R, int64_t H, int64_t ld, int renorm,
                          float eps, void* out, int out_f16, int64_t ldo, const RowDst& dst, cudaStream_t s) {
  const int grid = R < 148 * 8 ? (int)R : 148 * 8;
  if (out_f16) {
    __half* o = static_cast<__half*>(out);
    if (renorm)
      reduce_slices_kernel<__half, true><<<grid, 256, 0, s>>>(src, P, row0, R, H, ld, eps, o, ldo, dst);
    else
      reduce_slices_kernel<__half, false><<<grid, 256, 0, s>>>(src, P, row0, R, H, ld, eps, o, ldo, dst);
  } else {
    float* o = static_cast<float*>(out);
    if (renorm)
      reduce_slices_kernel<float, true><<<grid, 256, 0, s>>>(src, P, row0, R, H, ld, eps, o, ldo, dst);
    else
      reduce_slices_kernel<float, false><<<grid, 256, 0, s>>>(src, P, row0, R, H, ld, eps, o, ldo, dst);
  }
  note_launch();
  return cudaGetLastError();
}
}  // namespace

cudaError_t launch_reduce_slices(const float* recv, int P, int64_t R, int64_t H, int64_t ld, int renorm, float eps,
                                 void* out, int out_f16, int64_t ldo, cudaStream_t s) {
  SliceSrc src;
  memset(&src, 0, sizeof(src));
  for (int r = 0; r < P && r < BQ4_MAX_PEERS; ++r) src.p[r] = recv + (int64_t)r * R * ld;
  RowDst dst;
  memset(&dst, 0, sizeof(dst));
  return launch_reduce(src, P, 0, R, H, ld, renorm, eps, out, out_f16, ldo, dst, s);
}

cudaError_t launch_reduce_slices_peer(const float* const* src_ranks, int P, int64_t row0, int64_t R, int64_t H,
                                      int64_t ld, int renorm, float eps, void* out, void* const* out_ranks,
                                      int out_f16, int64_t ldo, cudaStream_t s) {
  SliceSrc src;
  memset(&src, 0, sizeof(src));
  for (int r = 0; r < P && r < BQ4_MAX_PEERS; ++r) src.p[r] = src_ranks[r];
  RowDst dst;
  memset(&dst, 0, sizeof(dst));
  if (out_ranks) {
    for (int r = 0; r < P && r < BQ4_MAX_PEERS; ++r) dst.p[r] = out_ranks[r];
    dst.n = P;
    dst.row0 = row0;
  }
  return launch_reduce(src, P, row0, R, H, ld, renorm, eps, out, out_f16, ldo, dst, s);
}

}  // namespace bq4
