// bq4_kernels.cu -- load-time re-layout, bit-exact dequantization and the
// activation f32 -> f16 staging pass.  All HBM-bound byte work: 128-bit
// accesses where the layout allows, grids sized in multiples of the SM count.
#include <cuda_fp16.h>

#include "bq4_internal.h"

namespace bq4 {
namespace {

// Logical lane stored at nibble position p of a prepared word.
__device__ __constant__ int kPermLane[8] = {0, 2, 4, 6, 1, 3, 5, 7};

__device__ __forceinline__ int32_t nibble_s4(uint32_t word, int lane) {
  // Sign-extend the 4-bit two's-complement value at bits [4*lane, 4*lane+3].
  return static_cast<int32_t>(word << (28 - 4 * lane)) >> 28;
}

__device__ __forceinline__ uint32_t raw_word(const uint32_t* words, int32_t layout, int64_t n,
                                             int64_t kw, int64_t src_N, int64_t src_KW) {
  return layout == BQ4_LAYOUT_COL ? words[n * src_KW + kw] : words[kw * src_N + n];
}

__device__ __forceinline__ float raw_scale(const float* scales, int32_t layout, int64_t n,
                                           int64_t kb, int64_t src_N, int64_t src_KB) {
  return layout == BQ4_LAYOUT_COL ? scales[n * src_KB + kb] : scales[kb * src_N + n];
}

// One thread per prepared word.  The shard is rows [n0, n0+N) and K range
// [k0, k0+K) of a source weight whose full extents are src_N x src_K.
__global__ void prepare_q_kernel(const uint32_t* __restrict__ words, int32_t layout, int64_t N,
                                 int64_t K, int64_t n0, int64_t k0, int64_t src_N, int64_t src_K,
                                 int64_t nkc, int64_t total, uint32_t* __restrict__ out) {
  const int64_t src_KW = src_K / 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = i & 3;
    const int64_t r = (i >> 2) & 127;
    const int64_t h = (i >> 9) & 1;
    const int64_t kc = (i >> 10) % nkc;
    const int64_t tile = (i >> 10) / nkc;
    const int64_t n = tile * 128 + r;
    const int64_t kw = kc * 8 + h * 4 + j;  // word index inside the shard
    uint32_t v = 0;
    if (n < N && kw * 8 < K) {
      const uint32_t src = raw_word(words, layout, n0 + n, k0 / 8 + kw, src_N, src_KW);
#pragma unroll
      for (int p = 0; p < 8; ++p) v |= ((src >> (4 * kPermLane[p])) & 0xFu) << (4 * p);
    }
    out[i] = v;
  }
}

__global__ void prepare_s_kernel(const float* __restrict__ scales, int32_t layout, int64_t N,
                                 int64_t K, int32_t block, int64_t n0, int64_t k0, int64_t src_N,
                                 int64_t src_K, int64_t nkb, int64_t total, float* __restrict__ out) {
  const int64_t src_KB = src_K / block;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i & 127;
    const int64_t kb = (i >> 7) % nkb;
    const int64_t tile = (i >> 7) / nkb;
    const int64_t n = tile * 128 + r;
    float v = 0.0f;
    if (n < N && kb * block < K) v = raw_scale(scales, layout, n0 + n, k0 / block + kb, src_N, src_KB);
    out[i] = v;
  }
}

// Dequantize from the prepared layout.  One thread per output element of
// the logical tensor: out_layout ROW -> [K][N], COL -> [N][K].
__global__ void dequant_prepared_kernel(const uint32_t* __restrict__ q, const float* __restrict__ s,
                                        int64_t K, int64_t N, int64_t nkc, int64_t nkb,
                                        int32_t block, int32_t out_layout,
                                        float* __restrict__ out) {
  const int64_t total = K * N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t k, n;
    if (out_layout == BQ4_LAYOUT_ROW) {
      k = i / N;
      n = i - k * N;
    } else {
      n = i / K;
      k = i - n * K;
    }
    const int64_t tile = n >> 7, r = n & 127;
    const int64_t kc = k >> 6, within = k & 63;
    const int64_t h = within >> 5, j = (within >> 3) & 3, lane = k & 7;
    const uint32_t word = q[((((tile * nkc + kc) * 2 + h) * 128 + r) << 2) + j];
    // logical lane -> stored position: pos = {0,4,1,5,2,6,3,7}[lane]
    const int pos = (lane >> 1) + ((lane & 1) << 2);
    const int32_t qv = nibble_s4(word, pos);
    const float sc = s[(tile * nkb + k / block) * 128 + r];
    out[i] = static_cast<float>(qv) * sc;
  }
}

// Pre-expanded tiles from an N-packed source (words [K][N/8], scales
// [K][N/block], blocks along N).  One thread per 16-byte chunk = 8 K values
// of one row n; stored at its 128-byte-swizzled position.
__global__ void prepare_pre_kernel(const uint32_t* __restrict__ words, const float* __restrict__ scales,
                                   int64_t N, int64_t K, int32_t block, int64_t n0, int64_t k0,
                                   int64_t src_N, int64_t nkc, int64_t total, uint16_t* __restrict__ out) {
  const int64_t NW8 = src_N / 8, NB = src_N / block;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = i & 7;
    const int64_t r = (i >> 3) & 127;
    const int64_t kc = (i >> 10) % nkc;
    const int64_t tile = (i >> 10) / nkc;
    const int64_t n = tile * 128 + r;
    __align__(16) __half v[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const int64_t k = kc * 64 + j * 8 + t;
      float val = 0.0f;
      if (n < N && k < K) {
        const int64_t sn = n0 + n, sk = k0 + k;
        const uint32_t word = words[sk * NW8 + sn / 8];
        val = static_cast<float>(nibble_s4(word, static_cast<int>(sn & 7))) * scales[sk * NB + sn / block];
      }
      v[t] = __float2half_rn(val);
    }
    uint16_t* dst = out + ((tile * nkc + kc) * 128 + r) * 64 + ((j ^ (r & 7)) * 8);
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(v);
  }
}

__global__ void dequant_raw_kernel(const uint32_t* __restrict__ words, const float* __restrict__ scales,
                                   int64_t K, int64_t N, int32_t block, int32_t layout,
                                   int32_t out_layout, float* __restrict__ out) {
  const int64_t total = K * N;
  const int64_t KW = K / 8, KB = K / block;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t k, n;
    if (out_layout == BQ4_LAYOUT_ROW) {
      k = i / N;
      n = i - k * N;
    } else {
      n = i / K;
      k = i - n * K;
    }
    if (layout == BQ4_LAYOUT_NPACKED) {
      const uint32_t word = words[k * (N / 8) + (n >> 3)];
      const float sc = scales[k * (N / block) + n / block];
      out[i] = static_cast<float>(nibble_s4(word, static_cast<int>(n & 7))) * sc;
    } else {
      const uint32_t word = raw_word(words, layout, n, k >> 3, N, KW);
      const float sc = raw_scale(scales, layout, n, k / block, N, KB);
      out[i] = static_cast<float>(nibble_s4(word, static_cast<int>(k & 7))) * sc;
    }
  }
}

// x f32 [M][ldx] -> xh f16 [M][Kp] with round-to-nearest-even, zero padding
// K..Kp-1.  Each thread converts 8 consecutive K values into one 16-byte
// store.  Block 0 also zeroes the GEMM's stream-K flags (nflags words).
__global__ void convert_x_kernel(const float* __restrict__ x, int64_t M, int64_t K, int64_t ldx,
                                 int64_t Kp, uint4* __restrict__ xh, int vec4, unsigned* __restrict__ flags,
                                 int nflags) {
  // The GEMM that consumes xh is launched as a programmatic dependent: it may
  // start its weight-side prologue now and waits for this grid's completion
  // before it reads xh or touches the flags.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < nflags; i += blockDim.x) flags[i] = 0u;
  const int64_t per_row = Kp / 8;
  const int64_t total = M * per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / per_row;
    const int64_t k = (i - m * per_row) * 8;
    float v[8];
    const float* src = x + m * ldx + k;
    if (k + 8 <= K && vec4) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(src));
      const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 1);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
      for (int t = 0; t < 8; ++t) v[t] = (k + t < K) ? __ldg(src + t) : 0.0f;
    }
    uint4 o;
    __half2 h0 = __floats2half2_rn(v[0], v[1]);
    __half2 h1 = __floats2half2_rn(v[2], v[3]);
    __half2 h2 = __floats2half2_rn(v[4], v[5]);
    __half2 h3 = __floats2half2_rn(v[6], v[7]);
    o.x = *reinterpret_cast<uint32_t*>(&h0);
    o.y = *reinterpret_cast<uint32_t*>(&h1);
    o.z = *reinterpret_cast<uint32_t*>(&h2);
    o.w = *reinterpret_cast<uint32_t*>(&h3);
    xh[i] = o;
  }
}

int grid_for(int64_t total, int threads, int device) {
  const int sms = device_sm_count(device);
  int64_t blocks = (total + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sms) * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

}  // namespace

cudaError_t launch_prepare(const uint32_t* words, const float* scales, int64_t K, int64_t N,
                           int32_t block, int32_t layout, int64_t n0, int64_t k0, int64_t src_N,
                           int64_t src_K, const bq4_weight* w, cudaStream_t s) {
  const int dev = current_device();
  const int64_t qtotal = w->ntiles * w->nkc * 1024;
  prepare_q_kernel<<<grid_for(qtotal, 256, dev), 256, 0, s>>>(words, layout, N, K, n0, k0, src_N,
                                                               src_K, w->nkc, qtotal, w->q);
  note_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int64_t stotal = w->ntiles * w->nkb * 128;
  prepare_s_kernel<<<grid_for(stotal, 256, dev), 256, 0, s>>>(scales, layout, N, K, block, n0, k0,
                                                               src_N, src_K, w->nkb, stotal, w->s);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_prepare_pre(const uint32_t* words, const float* scales, int64_t K, int64_t N,
                               int32_t block, int64_t n0, int64_t k0, int64_t src_N, int64_t src_K,
                               const bq4_weight* w, cudaStream_t s) {
  (void)src_K;
  const int64_t total = w->ntiles * w->nkc * 1024;
  prepare_pre_kernel<<<grid_for(total, 256, current_device()), 256, 0, s>>>(
      words, scales, N, K, block, n0, k0, src_N, w->nkc, total, w->h);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_dequant_prepared(const bq4_weight* w, float* out, int32_t out_layout,
                                    cudaStream_t s) {
  const int64_t total = w->K * w->N;
  dequant_prepared_kernel<<<grid_for(total, 256, w->device), 256, 0, s>>>(
      w->q, w->s, w->K, w->N, w->nkc, w->nkb, w->block, out_layout, out);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_dequant_raw(const uint32_t* words, const float* scales, int64_t K, int64_t N,
                               int32_t block, int32_t layout, float* out, int32_t out_layout,
                               cudaStream_t s) {
  const int64_t total = K * N;
  dequant_raw_kernel<<<grid_for(total, 256, current_device()), 256, 0, s>>>(
      words, scales, K, N, block, layout, out_layout, out);
  note_launch();
  return cudaGetLastError();
}

// Row selection from a packed Q4S matrix [rows][cols] (PackedU32(0): words
// [rows][wpr], scales [rows][spr], blocks along the row).  One thread per
// output word: copies it (out_values) and/or writes its 8 dequantized values
// (out_f32); one thread per output scale copies it (out_scales).  An index
// outside [0, rows) gives a zero row and records BQ4_EINVAL_ARG in *err.
__global__ void select_rows_kernel(const uint32_t* __restrict__ values, const float* __restrict__ scales,
                                   int64_t rows, int64_t wpr, int64_t spr, int block, const void* __restrict__ ids,
                                   int ids64, int64_t n, uint32_t* __restrict__ out_values,
                                   float* __restrict__ out_scales, float* __restrict__ out_f32, int* err) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (int64_t i = t0; i < n * wpr; i += stride) {
    const int64_t r = i / wpr, w = i - r * wpr;
    const int64_t id = ids64 ? reinterpret_cast<const int64_t*>(ids)[r] : reinterpret_cast<const int32_t*>(ids)[r];
    const bool ok = id >= 0 && id < rows;
    if (!ok && w == 0) atomicCAS(err, 0, (int)BQ4_EINVAL_ARG);
    const uint32_t word = ok ? __ldg(values + id * wpr + w) : 0u;
    if (out_values) out_values[i] = word;
    if (out_f32) {
      const float sc = ok ? __ldg(scales + id * spr + (w * 8) / block) : 0.0f;
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int q = (int)((word >> (4 * j)) & 0xFu);
        v[j] = (float)(q >= 8 ? q - 16 : q) * sc;
      }
      float4* dst = reinterpret_cast<float4*>(out_f32 + r * wpr * 8 + w * 8);
      dst[0] = make_float4(v[0], v[1], v[2], v[3]);
      dst[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
  }
  if (out_scales) {
    for (int64_t i = t0; i < n * spr; i += stride) {
      const int64_t r = i / spr, c = i - r * spr;
      const int64_t id = ids64 ? reinterpret_cast<const int64_t*>(ids)[r] : reinterpret_cast<const int32_t*>(ids)[r];
      out_scales[i] = (id >= 0 && id < rows) ? __ldg(scales + id * spr + c) : 0.0f;
    }
  }
}

cudaError_t launch_select_rows(const uint32_t* values, const float* scales, int64_t rows, int64_t cols, int block,
                               const void* ids, int ids64, int64_t n, uint32_t* out_values, float* out_scales,
                               float* out_f32, int* err, cudaStream_t s) {
  const int64_t wpr = cols / 8, spr = cols / block;
  const int64_t work = n * wpr > n * spr ? n * wpr : n * spr;
  select_rows_kernel<<<grid_for(work, 256, current_device()), 256, 0, s>>>(
      values, scales, rows, wpr, spr, block, ids, ids64, n, out_values, out_scales, out_f32, err);
  note_launch();
  return cudaGetLastError();
}

// One block of 256 threads per row: out[m,:] = x[m,:] * rsqrt(mean(x[m,:]^2)
// + eps), f32 arithmetic, f32 or f16 in and out.
__global__ void rms_renorm_kernel(const void* __restrict__ x, int x_f16, int64_t H, int64_t ldx,
                                  void* __restrict__ out, int out_f16, int64_t ldo, float eps) {
  const int64_t m = blockIdx.x;
  const __half* xh = reinterpret_cast<const __half*>(x) + m * ldx;
  const float* xf = reinterpret_cast<const float*>(x) + m * ldx;
  float ss = 0.0f;
  for (int64_t h = threadIdx.x; h < H; h += blockDim.x) {
    const float v = x_f16 ? __half2float(xh[h]) : xf[h];
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  __shared__ float part[32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) part[0] = t;
  }
  __syncthreads();
  const float r = rsqrtf(part[0] / (float)H + eps);
  __half* oh = reinterpret_cast<__half*>(out) + m * ldo;
  float* of = reinterpret_cast<float*>(out) + m * ldo;
  for (int64_t h = threadIdx.x; h < H; h += blockDim.x) {
    const float v = (x_f16 ? __half2float(xh[h]) : xf[h]) * r;
    if (out_f16)
      oh[h] = __float2half_rn(v);
    else
      of[h] = v;
  }
}

// Four values per access (16-byte f32 / 8-byte f16 loads and stores), for
// rows whose width, pitches and bases allow it: more bytes in flight per
// thread than the scalar kernel, which is latency-bound at this size.
__device__ __forceinline__ float4 load4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 load4(const __half* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ void store4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void store4(__half* p, float4 v) {
  const __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
  *reinterpret_cast<uint2*>(p) = make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
}

template <typename TI, typename TO>
__global__ void rms_renorm_vec4_kernel(const TI* __restrict__ x, int64_t H, int64_t ldx, TO* __restrict__ out,
                                       int64_t ldo, float eps) {
  const int64_t m = blockIdx.x;
  const TI* xr = x + m * ldx;
  TO* orow = out + m * ldo;
  float ss = 0.0f;
  for (int64_t h = (int64_t)threadIdx.x * 4; h < H; h += (int64_t)blockDim.x * 4) {
    const float4 v = load4(xr + h);
    ss = fmaf(v.x, v.x, ss); ss = fmaf(v.y, v.y, ss); ss = fmaf(v.z, v.z, ss); ss = fmaf(v.w, v.w, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  __shared__ float part[32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) part[0] = t;
  }
  __syncthreads();
  const float r = rsqrtf(part[0] / (float)H + eps);
  for (int64_t h = (int64_t)threadIdx.x * 4; h < H; h += (int64_t)blockDim.x * 4) {
    const float4 v = load4(xr + h);
    store4(orow + h, make_float4(v.x * r, v.y * r, v.z * r, v.w * r));
  }
}

cudaError_t launch_rms_renorm(const void* x, int x_f16, int64_t M, int64_t H, int64_t ldx, void* out,
                              int out_f16, int64_t ldo, float eps, cudaStream_t s) {
  const uintptr_t ax = x_f16 ? 7 : 15, ao = out_f16 ? 7 : 15;
  const bool vec = H % 4 == 0 && ldx % 4 == 0 && ldo % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & ax) == 0 &&
                   (reinterpret_cast<uintptr_t>(out) & ao) == 0;
  if (!vec) {
    rms_renorm_kernel<<<(unsigned)M, 256, 0, s>>>(x, x_f16, H, ldx, out, out_f16, ldo, eps);
  } else if (x_f16) {
    if (out_f16)
      rms_renorm_vec4_kernel<__half, __half><<<(unsigned)M, 256, 0, s>>>(
          static_cast<const __half*>(x), H, ldx, static_cast<__half*>(out), ldo, eps);
    else
      rms_renorm_vec4_kernel<__half, float><<<(unsigned)M, 256, 0, s>>>(
          static_cast<const __half*>(x), H, ldx, static_cast<float*>(out), ldo, eps);
  } else {
    if (out_f16)
      rms_renorm_vec4_kernel<float, __half><<<(unsigned)M, 256, 0, s>>>(
          static_cast<const float*>(x), H, ldx, static_cast<__half*>(out), ldo, eps);
    else
      rms_renorm_vec4_kernel<float, float><<<(unsigned)M, 256, 0, s>>>(
          static_cast<const float*>(x), H, ldx, static_cast<float*>(out), ldo, eps);
  }
  note_launch();
  return cudaGetLastError();
}

// QK-norm + RoPE on the q or k section of a projection output
// (crates/burn_boogu/src/model/attention.rs:114-133, 916-928): one warp per
// (token, head); lane l holds the pairs l, l+32, ... of the head, so the
// interleaved rotation needs no exchange.  Every pair is loaded before any
// is stored (in place is allowed).  The divide and sqrt are IEEE
// (x / sqrt(mean(x^2) + eps) * gamma, the reference's order).
template <typename TI, typename TO>
__global__ void qk_norm_rope_kernel(const TI* __restrict__ x, int64_t M, int heads, int hd, int64_t ldx,
                                    const float* __restrict__ gamma, float eps, const float* __restrict__ cos_t,
                                    const float* __restrict__ sin_t, int64_t ldr, TO* __restrict__ y, int64_t ldy) {
  constexpr int kMaxPairs = 4;  // head_dim <= 256
  const int lane = threadIdx.x & 31;
  const int64_t rows = M * heads;
  const int npairs = hd >> 1;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
       r += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const int64_t m = r / heads;
    const int h = (int)(r - m * heads);
    const TI* xr = x + m * ldx + (int64_t)h * hd;
    float a[kMaxPairs], b[kMaxPairs];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < kMaxPairs; ++i) {
      const int p = lane + 32 * i;
      a[i] = b[i] = 0.0f;
      if (p < npairs) {
        a[i] = static_cast<float>(xr[2 * p]);
        b[i] = static_cast<float>(xr[2 * p + 1]);
        ss += a[i] * a[i] + b[i] * b[i];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rms = sqrtf(ss / (float)hd + eps);
    TO* yr = y + m * ldy + (int64_t)h * hd;
#pragma unroll
    for (int i = 0; i < kMaxPairs; ++i) {
      const int p = lane + 32 * i;
      if (p < npairs) {
        float v0 = a[i] / rms, v1 = b[i] / rms;
        if (gamma) {
          v0 *= __ldg(gamma + 2 * p);
          v1 *= __ldg(gamma + 2 * p + 1);
        }
        float o0 = v0, o1 = v1;
        if (cos_t) {
          const float* cr = cos_t + m * ldr + 2 * p;
          const float* sr = sin_t + m * ldr + 2 * p;
          o0 = v0 * __ldg(cr) - v1 * __ldg(sr);
          o1 = v1 * __ldg(cr + 1) + v0 * __ldg(sr + 1);
        }
        yr[2 * p] = static_cast<TO>(o0);
        yr[2 * p + 1] = static_cast<TO>(o1);
      }
    }
  }
}

// The same with 16-byte accesses, token-major: head_dim a multiple of 4 and
// at most 128.  One warp per token keeps the token's cos/sin (and gamma) in
// registers and walks its heads kHeads at a time, all of a group's loads
// issued first; lane l holds values 4l..4l+3 (two rotation pairs).  Reading
// the tables once per token instead of once per (token, head) takes them
// off the L2-to-SM path, where they were two thirds of the bytes.  Values
// are scaled by one reciprocal of the RMS (within an ulp of the division).
template <typename TI, typename TO>
__global__ void qk_norm_rope_vec4_kernel(const TI* __restrict__ x, int64_t M, int heads, int hd, int64_t ldx,
                                         const float* __restrict__ gamma, float eps, const float* __restrict__ cos_t,
                                         const float* __restrict__ sin_t, int64_t ldr, TO* __restrict__ y,
                                         int64_t ldy) {
  constexpr int kHeads = 8;
  const int lane = threadIdx.x & 31;
  const bool on = lane * 4 < hd;
  const float4 g = (on && gamma) ? *reinterpret_cast<const float4*>(gamma + 4 * lane) : make_float4(1.f, 1.f, 1.f, 1.f);
  for (int64_t m = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); m < M;
       m += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    float4 c = make_float4(1.f, 1.f, 1.f, 1.f), sn = make_float4(0.f, 0.f, 0.f, 0.f);
    if (on && cos_t) {
      c = *reinterpret_cast<const float4*>(cos_t + m * ldr + 4 * lane);
      sn = *reinterpret_cast<const float4*>(sin_t + m * ldr + 4 * lane);
    }
    const TI* xr = x + m * ldx + 4 * lane;
    TO* yr = y + m * ldy + 4 * lane;
    for (int h0 = 0; h0 < heads; h0 += kHeads) {
      float4 v[kHeads];
#pragma unroll
      for (int u = 0; u < kHeads; ++u)
        v[u] = (on && h0 + u < heads) ? load4(xr + (int64_t)(h0 + u) * hd) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < kHeads; ++u) {
        float ss = v[u].x * v[u].x + v[u].y * v[u].y + v[u].z * v[u].z + v[u].w * v[u].w;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (!on || h0 + u >= heads) continue;
        const float inv = 1.0f / sqrtf(ss / (float)hd + eps);
        const float4 w = make_float4(v[u].x * inv * g.x, v[u].y * inv * g.y, v[u].z * inv * g.z, v[u].w * inv * g.w);
        store4(yr + (int64_t)(h0 + u) * hd,
               cos_t ? make_float4(w.x * c.x - w.y * sn.x, w.y * c.y + w.x * sn.y, w.z * c.z - w.w * sn.z,
                                   w.w * c.w + w.z * sn.w)
                     : w);
      }
    }
  }
}

cudaError_t launch_qk_norm_rope(const void* x, int x_f16, int64_t M, int heads, int hd, int64_t ldx,
                                const float* gamma, float eps, const float* cos_t, const float* sin_t, int64_t ldr,
                                void* y, int y_f16, int64_t ldy, cudaStream_t s) {
  const int64_t rows = M * heads;
  const int grid = grid_for(rows * 32, 256, current_device());
  const uintptr_t ax = x_f16 ? 7 : 15, ay = y_f16 ? 7 : 15;
  const bool vec = hd % 4 == 0 && hd <= 128 && ldx % 4 == 0 && ldy % 4 == 0 &&
                   (reinterpret_cast<uintptr_t>(x) & ax) == 0 && (reinterpret_cast<uintptr_t>(y) & ay) == 0 &&
                   (!gamma || (reinterpret_cast<uintptr_t>(gamma) & 15) == 0) &&
                   (!cos_t || (ldr % 4 == 0 && (reinterpret_cast<uintptr_t>(cos_t) & 15) == 0 &&
                               (reinterpret_cast<uintptr_t>(sin_t) & 15) == 0));
  if (vec) {
    const int vgrid = grid_for(M * 32, 256, current_device());  // one warp per token
    if (x_f16 && y_f16)
      qk_norm_rope_vec4_kernel<__half, __half><<<vgrid, 256, 0, s>>>(static_cast<const __half*>(x), M, heads, hd, ldx,
                                                                   gamma, eps, cos_t, sin_t, ldr,
                                                                   static_cast<__half*>(y), ldy);
    else if (x_f16)
      qk_norm_rope_vec4_kernel<__half, float><<<vgrid, 256, 0, s>>>(static_cast<const __half*>(x), M, heads, hd, ldx,
                                                                  gamma, eps, cos_t, sin_t, ldr, static_cast<float*>(y),
                                                                  ldy);
    else if (y_f16)
      qk_norm_rope_vec4_kernel<float, __half><<<vgrid, 256, 0, s>>>(static_cast<const float*>(x), M, heads, hd, ldx,
                                                                  gamma, eps, cos_t, sin_t, ldr,
                                                                  static_cast<__half*>(y), ldy);
    else
      qk_norm_rope_vec4_kernel<float, float><<<vgrid, 256, 0, s>>>(static_cast<const float*>(x), M, heads, hd, ldx,
                                                                 gamma, eps, cos_t, sin_t, ldr, static_cast<float*>(y),
                                                                 ldy);
    note_launch();
    return cudaGetLastError();
  }
  if (x_f16) {
    if (y_f16)
      qk_norm_rope_kernel<__half, __half><<<grid, 256, 0, s>>>(static_cast<const __half*>(x), M, heads, hd, ldx,
                                                              gamma, eps, cos_t, sin_t, ldr,
                                                              static_cast<__half*>(y), ldy);
    else
      qk_norm_rope_kernel<__half, float><<<grid, 256, 0, s>>>(static_cast<const __half*>(x), M, heads, hd, ldx,
                                                             gamma, eps, cos_t, sin_t, ldr, static_cast<float*>(y),
                                                             ldy);
  } else {
    if (y_f16)
      qk_norm_rope_kernel<float, __half><<<grid, 256, 0, s>>>(static_cast<const float*>(x), M, heads, hd, ldx,
                                                             gamma, eps, cos_t, sin_t, ldr,
                                                             static_cast<__half*>(y), ldy);
    else
      qk_norm_rope_kernel<float, float><<<grid, 256, 0, s>>>(static_cast<const float*>(x), M, heads, hd, ldx, gamma,
                                                            eps, cos_t, sin_t, ldr, static_cast<float*>(y), ldy);
  }
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_convert_x(const float* x, int64_t M, int64_t K, int64_t ldx, int64_t Kp,
                             void* xh, unsigned* flags, int nflags, cudaStream_t s) {
  const int vec4 = ((reinterpret_cast<uintptr_t>(x) & 15) == 0) && (ldx % 4 == 0);
  const int64_t total = M * (Kp / 8);
  convert_x_kernel<<<grid_for(total, 256, current_device()), 256, 0, s>>>(
      x, M, K, ldx, Kp, reinterpret_cast<uint4*>(xh), vec4, flags, nflags);
  note_launch();
  return cudaGetLastError();
}

// Zeroes the GEMM's stream-K flags when there is no staging grid to do it
// (f16 activations); the GEMM follows as a programmatic dependent.
__global__ void zero_flags_kernel(unsigned* __restrict__ flags, int nflags) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  for (int i = threadIdx.x; i < nflags; i += blockDim.x) flags[i] = 0u;
}

cudaError_t launch_zero_flags(unsigned* flags, int nflags, cudaStream_t s) {
  zero_flags_kernel<<<1, 256, 0, s>>>(flags, nflags);
  note_launch();
  return cudaGetLastError();
}

}  // namespace bq4
