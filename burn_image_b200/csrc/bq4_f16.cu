// bq4_f16.cu -- packed-F16 storage: IEEE binary16 bits, two per u32 word,
// the even-index element in the low half (the VAE's weights and the F16
// profiles' tables).  Four operations, each the B200 counterpart of one
// kernel of patches/burn-cubecl-0.21.0/src/kernel/packed_f16.rs:
//
//   bq4_packed_f16_to_f32       strided widening        (:88-131)
//   bq4_packed_f16_select_rows  row gather, widened     (:296-358)
//   bq4_packed_f16_rhs_matmul   f32 lhs x f16 rhs       (:133-292)
//   bq4_packed_f16_conv2d       NCHW x OIHW, groups 1   (:421-602)
//
// Widening is bit-exact (integer arithmetic on the bit pattern, NaN payloads
// kept with the quiet bit set).  The matmul and the convolution run on the
// tensor cores as kind::tf32 through the warp-specialized GEMM
// (bq4_gemm_sm100.cu): the f16 weights are widened once into MMA-ready f32
// tiles -- exact in tf32, whose 10-bit mantissa and 8-bit exponent cover
// every binary16 value -- and the f32 activations enter with their top 10
// mantissa bits, accumulated in f32.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <new>

#include "bq4_internal.h"

namespace bq4 {
namespace {

constexpr int kMaxRank = 8;

// Grid-stride launches: at most 16 blocks per SM.
int grid_for(int64_t total, int threads, int device) {
  int64_t blocks = (total + threads - 1) / threads;
  const int64_t cap = (int64_t)device_sm_count(device) * 16;
  return (int)(blocks > cap ? cap : (blocks < 1 ? 1 : blocks));
}

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

// binary16 bits -> binary32 bits: sign, exponent rebias (15 -> 127),
// subnormals normalised, infinities kept, NaN payload kept and quieted.
__device__ __forceinline__ float widen_f16(uint32_t h) {
  const uint32_t sign = (h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1fu;
  const uint32_t m = h & 0x3ffu;
  uint32_t bits;
  if (e == 0x1fu) {
    bits = sign | 0x7f800000u | (m ? 0x00400000u | (m << 13) : 0u);
  } else if (e != 0) {
    bits = sign | ((e + 112u) << 23) | (m << 13);
  } else if (m == 0) {
    bits = sign;
  } else {
    // m * 2^-24 with the leading one of m moved to bit 10
    const uint32_t sh = (uint32_t)__clz(m) - 21u;
    bits = sign | ((113u - sh) << 23) | (((m << sh) & 0x3ffu) << 13);
  }
  return __uint_as_float(bits);
}

struct Strided {
  int64_t shape[kMaxRank];
  int64_t stride[kMaxRank];
  int rank;
};

// out (contiguous in `shape`) = widen(packed[sum coord * stride]).
__global__ void f16_to_f32_strided_kernel(const uint16_t* __restrict__ src, Strided v, int64_t total,
                                          float* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = i, off = 0;
    for (int d = v.rank - 1; d >= 0; --d) {
      const int64_t c = rem % v.shape[d];
      rem /= v.shape[d];
      off += c * v.stride[d];
    }
    out[i] = widen_f16(src[off]);
  }
}

// Contiguous source, 16-byte aligned: 8 values per thread.
__global__ void f16_to_f32_vec8_kernel(const uint4* __restrict__ src, int64_t n8, float4* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 w = src[i];
    out[2 * i] = make_float4(widen_f16(w.x & 0xffffu), widen_f16(w.x >> 16), widen_f16(w.y & 0xffffu),
                             widen_f16(w.y >> 16));
    out[2 * i + 1] = make_float4(widen_f16(w.z & 0xffffu), widen_f16(w.z >> 16), widen_f16(w.w & 0xffffu),
                                 widen_f16(w.w >> 16));
  }
}

// out[r][c] = widen(table[idx[r]][c]); an index outside [0, rows) gives a
// zero row and records BQ4_EINVAL_ARG in *err.
__global__ void f16_select_rows_kernel(const uint16_t* __restrict__ table, int64_t rows, int64_t cols,
                                       const int32_t* __restrict__ idx, int64_t n, float* __restrict__ out,
                                       int* err) {
  const int64_t total = n * cols;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i - r * cols;
    const int64_t s = idx[r];
    float v = 0.0f;
    if (s >= 0 && s < rows) {
      v = widen_f16(table[s * cols + c]);
    } else if (c == 0 && err) {
      atomicCAS(err, 0, (int)BQ4_EINVAL_ARG);
    }
    out[i] = v;
  }
}

// Same, cols % 8 == 0 and 16-byte aligned rows: 8 values per thread.
__global__ void f16_select_rows_vec8_kernel(const uint4* __restrict__ table, int64_t rows, int64_t c8,
                                            const int32_t* __restrict__ idx, int64_t n, float4* __restrict__ out,
                                            int* err) {
  const int64_t total = n * c8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / c8, c = i - r * c8;
    const int64_t s = idx[r];
    float4 lo = make_float4(0.f, 0.f, 0.f, 0.f), hi = lo;
    if (s >= 0 && s < rows) {
      const uint4 w = table[s * c8 + c];
      lo = make_float4(widen_f16(w.x & 0xffffu), widen_f16(w.x >> 16), widen_f16(w.y & 0xffffu), widen_f16(w.y >> 16));
      hi = make_float4(widen_f16(w.z & 0xffffu), widen_f16(w.z >> 16), widen_f16(w.w & 0xffffu), widen_f16(w.w >> 16));
    } else if (c == 0 && err) {
      atomicCAS(err, 0, (int)BQ4_EINVAL_ARG);
    }
    out[2 * i] = lo;
    out[2 * i + 1] = hi;
  }
}

// MMA-ready tf32 weight tiles: f32 [ntiles][nkc][128 rows][RF K] with RF =
// 16 (64-byte rows, 64-byte swizzle: 16-byte chunk j of row r stored at
// chunk j ^ ((r >> 1) & 3)) for the linear, or RF = 32 (128-byte rows,
// 128-byte swizzle: chunk j at j ^ (r & 7)) for the convolution.  One thread
// per 16-byte chunk (4 K values of one output row n).  Source element (k, n):
//   linear: packed[k * inner_stride + n * col_stride];
//   conv (taps > 0): k = tap * cp + c, packed OIHW [n][cin][taps], zero for
//   c >= cin (channel padding).
// K >= K_real and n >= N are zero.
template <int RF>
__global__ void prepare_f16_tiles_kernel(const uint16_t* __restrict__ src, int64_t K, int64_t N,
                                         int64_t inner_stride, int64_t col_stride, int taps, int cin, int cp,
                                         int64_t nkc, int64_t total, float* __restrict__ out) {
  constexpr int kJ = RF / 4;  // 16-byte chunks per row
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = i % kJ;
    const int64_t r = (i / kJ) & 127;
    const int64_t kc = (i / (kJ * 128)) % nkc;
    const int64_t tile = (i / (kJ * 128)) / nkc;
    const int64_t n = tile * 128 + r;
    float v[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int64_t k = kc * RF + j * 4 + t;
      uint32_t bits = 0;
      if (n < N && k < K) {
        if (taps > 0) {
          const int64_t tap = k / cp, c = k - tap * cp;
          if (c < cin) bits = src[(n * cin + c) * taps + tap];
        } else {
          bits = src[k * inner_stride + n * col_stride];
        }
      }
      v[t] = widen_f16(bits);
    }
    const int64_t js = RF == 16 ? (j ^ ((r >> 1) & 3)) : (j ^ (r & 7));
    *reinterpret_cast<float4*>(out + ((tile * nkc + kc) * 128 + r) * RF + js * 4) =
        make_float4(v[0], v[1], v[2], v[3]);
  }
}

// Round to the nearest tf32 value (ties away from zero), as an f32 pattern.
__device__ __forceinline__ float round_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// NCHW f32 [B][C][H][W] -> zero-padded NHWC [B][Hp][Wp][Cp] (rounded to
// tf32), input pixel (y, x) at (y + ph, x + pw).  Block (32, 8): a 32-pixel
// x 32-channel tile, read along W and written along C through shared memory.
__global__ void stage_nhwc_kernel(const float* __restrict__ in, int C, int H, int W, int Cp, int Hp, int Wp, int ph,
                                  int pw, int cblocks, float* __restrict__ out) {
  __shared__ float tile[32][33];
  const int x0 = blockIdx.x * 32;
  const int yp = blockIdx.y;
  const int b = blockIdx.z / cblocks, c0 = (blockIdx.z - b * cblocks) * 32;
  const int y = yp - ph;
  const bool row_in = y >= 0 && y < H;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = c0 + threadIdx.y + 8 * i;   // channel row of the tile
    const int xp = x0 + threadIdx.x, x = xp - pw;
    float v = 0.0f;
    if (row_in && c < C && x >= 0 && x < W) v = in[(((size_t)b * C + c) * H + y) * W + x];
    tile[threadIdx.y + 8 * i][threadIdx.x] = round_tf32(v);
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int xp = x0 + threadIdx.y + 8 * i;  // pixel of the tile
    const int c = c0 + threadIdx.x;
    if (xp < Wp && c < Cp) out[(((size_t)b * Hp + yp) * Wp + xp) * Cp + c] = tile[threadIdx.x][threadIdx.y + 8 * i];
  }
}

// Strided convolution: token rows gathered from the staged NHWC image,
// out[(b, oy, ox)][tap * Cp + c] = nhwc[b][oy * sh + ky * dh][ox * sw + kx * dw][c]
// (padded coordinates), K columns past taps * Cp zero; 16-byte copies.
__global__ void gather_rows_kernel(const float4* __restrict__ nhwc, int Hp, int Wp, int cp4, int OH, int OW, int kw,
                                   int taps, int sh, int sw, int dh, int dw, int64_t kp4, int64_t total,
                                   float4* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / kp4, k4 = i - m * kp4;
    const int64_t tap = k4 / cp4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (tap < taps) {
      const int64_t c4 = k4 - tap * cp4;
      const int64_t b = m / ((int64_t)OH * OW), r = m - b * OH * OW;
      const int oy = (int)(r / OW), ox = (int)(r - (int64_t)oy * OW);
      const int ky = (int)tap / kw, kx = (int)tap - ky * kw;
      const int64_t yp = (int64_t)oy * sh + (int64_t)ky * dh, xp = (int64_t)ox * sw + (int64_t)kx * dw;
      v = nhwc[((b * Hp + yp) * Wp + xp) * cp4 + c4];
    }
    out[i] = v;
  }
}

// Copy f32 rows [M][K] (any pitch) into [M][Kp] at pitch Kp, zero padded.
__global__ void pad_rows_kernel(const float* __restrict__ x, int64_t M, int64_t K, int64_t ldx, int64_t Kp,
                                float* __restrict__ out) {
  const int64_t total = M * Kp;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / Kp, k = i - m * Kp;
    out[i] = k < K ? x[m * ldx + k] : 0.0f;
  }
}

// ------------------------------------------------------------- attention
// softmax(scale * q k^T) v per (batch, head), unfused: S = q k^T and O = P v
// run as tf32 GEMMs (k and v read as packed-F16 weights through strided
// views), with these two passes around them.

// q rows of one head, f16 [S][D] at row pitch ldq -> f32 [S][D] (the GEMM's
// in-place token rows).
__global__ void attn_q_rows_kernel(const uint16_t* __restrict__ q, int64_t S, int D, int64_t ldq,
                                   float* __restrict__ out) {
  const int64_t total = S * D;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / D, c = i - r * D;
    out[i] = widen_f16(q[r * ldq + c]);
  }
}

// In place over rows of n scores (row pitch ld): e = exp(scale * s - max),
// and inv[r] = 1 / sum(e) for the rows of P v to be scaled afterwards
// (attn_scale_rows_kernel), so the probabilities are never normalised in
// place.  One block of 256 threads per row: a max pass, then one expf per
// score; f32 sums in a fixed order, deterministic.
__global__ void attn_softmax_kernel(float* __restrict__ s, int64_t rows, int64_t n, int64_t ld, float scale,
                                    float* __restrict__ inv) {
  __shared__ float red[8];
  __shared__ float bcast;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    float* row = s + r * ld;
    float m = -INFINITY;
    for (int64_t j = threadIdx.x; j < n; j += blockDim.x) m = fmaxf(m, row[j] * scale);
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = red[0];
      for (int w = 1; w < (int)(blockDim.x >> 5); ++w) t = fmaxf(t, red[w]);
      bcast = t;
    }
    __syncthreads();
    m = bcast;
    float sum = 0.0f;
    for (int64_t j = threadIdx.x; j < n; j += blockDim.x) {
      const float e = expf(row[j] * scale - m);
      row[j] = e;
      sum += e;
    }
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    __syncthreads();  // bcast was read by every thread
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.0f;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
      inv[r] = 1.0f / t;
    }
    __syncthreads();  // red is rewritten by the next row
  }
}

// out[r][d] *= inv[r] over rows of D values (the softmax normalisation of P v).
__global__ void attn_scale_rows_kernel(float* __restrict__ out, int64_t rows, int D, const float* __restrict__ inv) {
  const int64_t total = rows * D;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
    out[i] *= inv[i / D];
}

}  // namespace

// ------------------------------------------------------------------ host side

namespace {

struct Guard {  // restores the caller's current device
  int prev = -1;
  explicit Guard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~Guard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

bool al(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
size_t up256(size_t v) { return (v + 255) / 256 * 256; }
int64_t round_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

bool on_device(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

bq4_status need_sm100(int dev) {
  if (!device_is_sm100(dev))
    return set_error(BQ4_EUNSUPPORTED, "device %d is not sm_100 (B200); libbq4 has no kernels for it", dev);
  return BQ4_OK;
}

// Weight view of a packed-F16 operand, K x N (no allocation): tiles of
// 128 rows x rf K f32 (rf = 16 for the linear, 32 for the convolution), K
// padded to a stage (2 rf).  Conv weights: K = taps * cp, kh/kw/cin recorded.
void f16_view(int64_t K, int64_t N, bq4_weight* w, int rf = 16) {
  memset(w, 0, sizeof(*w));
  w->K = K;
  w->N = N;
  w->layout = BQ4_LAYOUT_F16;
  w->tf32 = 1;
  w->Kp = round_up(K, 2 * rf);  // a stage is two chunks
  w->nkc = w->Kp / rf;
  w->ntiles = (N + kTileN - 1) / kTileN;
  w->Np = w->ntiles * kTileN;
  // an even number of tiles: the wide kernel takes N tiles in pairs
  w->h_bytes = (size_t)((w->ntiles + 1) / 2 * 2) * w->nkc * 128 * rf * sizeof(float);
}

void conv_view(int64_t cout, int64_t cin, int kh, int kw, bq4_weight* w) {
  const int64_t cp = round_up(cin, 32);
  f16_view((int64_t)kh * kw * cp, cout, w, 32);
  w->conv_kh = kh;
  w->conv_kw = kw;
  w->conv_cin = (int32_t)cin;
  w->conv_cp = (int32_t)cp;
}

cudaError_t launch_prepare_f16(const uint16_t* src, const bq4_weight* w, int64_t inner, int64_t col,
                               cudaStream_t s) {
  const int taps = w->conv_kh ? w->conv_kh * w->conv_kw : 0;
  if (taps) {  // 128-byte rows
    const int64_t total = w->ntiles * w->nkc * 1024;
    prepare_f16_tiles_kernel<32><<<grid_for(total, 256, current_device()), 256, 0, s>>>(
        src, w->K, w->N, inner, col, taps, w->conv_cin, w->conv_cp, w->nkc, total, reinterpret_cast<float*>(w->h));
  } else {     // 64-byte rows; the tile after an odd last one is zeroed
    const int64_t total = (w->ntiles + 1) / 2 * 2 * w->nkc * 512;
    prepare_f16_tiles_kernel<16><<<grid_for(total, 256, current_device()), 256, 0, s>>>(
        src, w->K, w->N, inner, col, 0, 0, 0, w->nkc, total, reinterpret_cast<float*>(w->h));
  }
  note_launch();
  return cudaGetLastError();
}

// Allocate and fill a prepared packed-F16 weight from `count` source f16
// elements at `packed` (host or device).
bq4_status prepare_f16_weight(const uint32_t* packed, size_t count, bq4_weight* view, int64_t inner, int64_t col,
                              int32_t device, bq4_weight** out) {
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
    cudaGetLastError();
    return set_error(BQ4_EINVAL_ARG, "device %d not present", device);
  }
  bq4_status st = need_sm100(device);
  if (st) return st;
  Guard guard(device);
  view->device = device;
  const uint16_t* src = reinterpret_cast<const uint16_t*>(packed);
  void* tmp = nullptr;
  cudaError_t e = cudaSuccess;
  if (!on_device(packed)) {
    e = cudaMalloc(&tmp, count * 2);
    if (e == cudaSuccess) e = cudaMemcpy(tmp, packed, count * 2, cudaMemcpyHostToDevice);
    src = static_cast<const uint16_t*>(tmp);
  }
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&view->h), view->h_bytes);
  if (e == cudaSuccess) e = launch_prepare_f16(src, view, inner, col, nullptr);
  if (e == cudaSuccess) e = cudaStreamSynchronize(nullptr);
  if (tmp) cudaFree(tmp);
  if (e != cudaSuccess) {
    if (view->h) cudaFree(view->h);
    view->h = nullptr;
    return check_cuda(e, "packed-F16 weight preparation");
  }
  bq4_weight* w = new (std::nothrow) bq4_weight(*view);
  if (!w) {
    cudaFree(view->h);
    view->h = nullptr;
    return set_error(BQ4_ECUDA, "host allocation failed");
  }
  *out = w;
  return BQ4_OK;
}

bq4_status check_linear_geometry(int64_t K, int64_t N, int64_t inner, int64_t col) {
  if (K <= 0 || N <= 0 || K > ((int64_t)1 << 24) || N > ((int64_t)1 << 24))
    return set_error(BQ4_EINVAL_SHAPE, "K=%lld N=%lld must be in [1, 2^24]", (long long)K, (long long)N);
  if (inner < 0 || col < 0) return set_error(BQ4_EINVAL_SHAPE, "negative stride");
  return BQ4_OK;
}

// Output extent and staging of one convolution.
struct ConvShape {
  int64_t OH, OW, Hp, Wp, M;
  bool implicit;  // stride 1: shifted token rows of the padded image; else gathered rows
  size_t stage_bytes, gather_bytes;
};

bq4_status conv_shape(const bq4_weight* w, int64_t B, int64_t H, int64_t W, const bq4_conv2d_options* o,
                      ConvShape* cs) {
  if (!w || !w->tf32 || !w->conv_kh) return set_error(BQ4_EINVAL_ARG, "w is not a packed-F16 conv weight");
  if (!o) return set_error(BQ4_EINVAL_ARG, "options is NULL");
  if (o->groups != 1) return set_error(BQ4_EUNSUPPORTED, "groups=%d: only groups = 1", (int)o->groups);
  for (int i = 0; i < 2; ++i)
    if (o->stride[i] < 1 || o->dilation[i] < 1 || o->padding[i] < 0)
      return set_error(BQ4_EINVAL_ARG, "stride/dilation must be >= 1 and padding >= 0");
  if (B <= 0 || H <= 0 || W <= 0) return set_error(BQ4_EINVAL_SHAPE, "batch/height/width must be positive");
  const int64_t kh = w->conv_kh, kw = w->conv_kw;
  cs->Hp = H + 2 * (int64_t)o->padding[0];
  cs->Wp = W + 2 * (int64_t)o->padding[1];
  const int64_t eh = (int64_t)o->dilation[0] * (kh - 1) + 1, ew = (int64_t)o->dilation[1] * (kw - 1) + 1;
  if (cs->Hp < eh || cs->Wp < ew) return set_error(BQ4_EINVAL_SHAPE, "kernel larger than the padded input");
  cs->OH = (cs->Hp - eh) / o->stride[0] + 1;
  cs->OW = (cs->Wp - ew) / o->stride[1] + 1;
  cs->implicit = o->stride[0] == 1 && o->stride[1] == 1;
  cs->M = cs->implicit ? B * cs->Hp * cs->Wp : B * cs->OH * cs->OW;
  if (cs->Hp > 65535 || B * ((w->conv_cp + 31) / 32) > 65535 || cs->M > ((int64_t)1 << 30) ||
      (int64_t)o->dilation[0] * cs->Wp * kh > ((int64_t)1 << 30))
    return set_error(BQ4_EINVAL_SHAPE, "convolution too large");
  cs->stage_bytes = up256((size_t)(B * cs->Hp * cs->Wp) * (size_t)w->conv_cp * sizeof(float));
  cs->gather_bytes = cs->implicit ? 0 : up256((size_t)cs->M * (size_t)w->Kp * sizeof(float));
  return BQ4_OK;
}

bq4_status conv_workspace(const bq4_weight* w, const ConvShape& cs, int dev, GemmPlan* plan, size_t* bytes) {
  bq4_status st = plan_gemm(w, 1, cs.M, dev, plan, false, false, true);
  if (st) return st;
  *bytes = cs.stage_bytes + cs.gather_bytes + plan->workspace_bytes;
  return BQ4_OK;
}

// Stage, gather (strided) and run the implicit GEMM for a prepared conv weight.
bq4_status run_conv(const float* input, int64_t B, int64_t H, int64_t W, const bq4_weight* w, const float* bias,
                    const bq4_conv2d_options* o, float* out, uint8_t* ws, size_t ws_bytes, cudaStream_t s) {
  ConvShape cs;
  bq4_status st = conv_shape(w, B, H, W, o, &cs);
  if (st) return st;
  GemmPlan plan;
  size_t need = 0;
  st = conv_workspace(w, cs, w->device, &plan, &need);
  if (st) return st;
  if (!ws || ws_bytes < need) return set_error(BQ4_EWORKSPACE, "workspace %zu < required %zu bytes", ws_bytes, need);
  if (!al(ws, 256)) return set_error(BQ4_EALIGN, "workspace not 256-byte aligned");
  const int cp = w->conv_cp, cin = w->conv_cin;
  float* staged = reinterpret_cast<float*>(ws);
  const int cblocks = (cp + 31) / 32;
  stage_nhwc_kernel<<<dim3((unsigned)((cs.Wp + 31) / 32), (unsigned)cs.Hp, (unsigned)(B * cblocks)), dim3(32, 8), 0,
                      s>>>(input, cin, (int)H, (int)W, cp, (int)cs.Hp, (int)cs.Wp, o->padding[0], o->padding[1],
                           cblocks, staged);
  note_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return check_cuda(e, "conv staging launch");
  ConvGeom g;
  const float* x = staged;
  if (cs.implicit) {
    g.cchunks = cp / 32;
    g.taps = w->conv_kh * w->conv_kw;
    g.kw = w->conv_kw;
    g.dy = (int)(o->dilation[0] * cs.Wp);
    g.dx = o->dilation[1];
    g.hp = (int)cs.Hp;
    g.wp = (int)cs.Wp;
    g.x_cols = cp;
  } else {
    float* rows = reinterpret_cast<float*>(ws + cs.stage_bytes);
    const int64_t kp4 = w->Kp / 4, total = cs.M * kp4;
    gather_rows_kernel<<<grid_for(total, 256, w->device), 256, 0, s>>>(
        reinterpret_cast<const float4*>(staged), (int)cs.Hp, (int)cs.Wp, cp / 4, (int)cs.OH, (int)cs.OW, w->conv_kw,
        w->conv_kh * w->conv_kw, o->stride[0], o->stride[1], o->dilation[0], o->dilation[1], kp4, total,
        reinterpret_cast<float4*>(rows));
    note_launch();
    e = cudaGetLastError();
    if (e != cudaSuccess) return check_cuda(e, "conv gather launch");
    g.cchunks = (int)w->nkc;  // one "tap": the gathered rows hold every tap
    g.taps = 1;
    g.kw = 1;
    g.hp = (int)cs.OH;
    g.wp = (int)cs.OW;
    g.x_cols = w->Kp;
    x = rows;
  }
  g.oh = (int)cs.OH;
  g.ow = (int)cs.OW;
  const bq4_weight* wl[1] = {w};
  const float* b[1] = {bias};
  GemmIo io;
  io.cv = &g;
  return run_gemm(plan, wl, x, cs.M, g.x_cols, b, (int)BQ4_ACT_NONE, nullptr, out,
                  ws + cs.stage_bytes + cs.gather_bytes, s, io);
}

}  // namespace
}  // namespace bq4

using namespace bq4;

extern "C" {

bq4_status bq4_packed_f16_to_f32(const uint32_t* packed, int32_t rank, const int64_t* shape, const int64_t* strides,
                                 float* out, bq4_stream_t stream) {
  if (!packed || !out || (rank > 0 && (!shape || !strides))) return set_error(BQ4_EINVAL_ARG, "NULL pointer");
  if (rank < 0 || rank > kMaxRank) return set_error(BQ4_EINVAL_ARG, "rank %d not in [0, %d]", (int)rank, kMaxRank);
  int dev = 0;
  cudaGetDevice(&dev);
  bq4_status st = need_sm100(dev);
  if (st) return st;
  Strided v;
  memset(&v, 0, sizeof(v));
  v.rank = rank;
  int64_t total = 1, expect = 1;
  bool contiguous = true;
  for (int d = rank - 1; d >= 0; --d) {
    if (shape[d] < 0 || strides[d] < 0) return set_error(BQ4_EINVAL_SHAPE, "negative extent or stride");
    v.shape[d] = shape[d];
    v.stride[d] = strides[d];
    if (shape[d] != 1 && strides[d] != expect) contiguous = false;
    expect *= shape[d];
    total *= shape[d];
  }
  if (total == 0) return BQ4_OK;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (contiguous && total % 8 == 0 && al(packed, 16) && al(out, 16)) {
    f16_to_f32_vec8_kernel<<<grid_for(total / 8, 256, dev), 256, 0, s>>>(reinterpret_cast<const uint4*>(packed),
                                                                        total / 8, reinterpret_cast<float4*>(out));
  } else {
    f16_to_f32_strided_kernel<<<grid_for(total, 256, dev), 256, 0, s>>>(reinterpret_cast<const uint16_t*>(packed), v,
                                                                       total, out);
  }
  note_launch();
  return check_cuda(cudaGetLastError(), "packed_f16_to_f32 launch");
}

bq4_status bq4_packed_f16_select_rows(const uint32_t* table, int64_t rows, int64_t cols, const int32_t* indices,
                                      int64_t n, float* out, bq4_stream_t stream) {
  if (!table || !indices || !out) return set_error(BQ4_EINVAL_ARG, "NULL pointer");
  if (rows <= 0 || cols <= 0 || n < 0) return set_error(BQ4_EINVAL_SHAPE, "rows/cols must be positive, n >= 0");
  if (n == 0) return BQ4_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  bq4_status st = need_sm100(dev);
  if (st) return st;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int* err = device_error_word();
  if (cols % 8 == 0 && al(table, 16) && al(out, 16)) {
    const int64_t c8 = cols / 8;
    f16_select_rows_vec8_kernel<<<grid_for(n * c8, 256, dev), 256, 0, s>>>(
        reinterpret_cast<const uint4*>(table), rows, c8, indices, n, reinterpret_cast<float4*>(out), err);
  } else {
    f16_select_rows_kernel<<<grid_for(n * cols, 256, dev), 256, 0, s>>>(reinterpret_cast<const uint16_t*>(table), rows,
                                                                       cols, indices, n, out, err);
  }
  note_launch();
  return check_cuda(cudaGetLastError(), "packed_f16_select_rows launch");
}

bq4_status bq4_f16_weight_prepare(const uint32_t* packed, int64_t K, int64_t N, int64_t inner_stride,
                                  int64_t col_stride, int32_t device, bq4_weight** out) {
  if (!out) return set_error(BQ4_EINVAL_ARG, "out is NULL");
  *out = nullptr;
  if (!packed) return set_error(BQ4_EINVAL_ARG, "packed is NULL");
  bq4_status st = check_linear_geometry(K, N, inner_stride, col_stride);
  if (st) return st;
  bq4_weight view;
  f16_view(K, N, &view);
  const size_t count = (size_t)((K - 1) * inner_stride + (N - 1) * col_stride + 1);
  return prepare_f16_weight(packed, count, &view, inner_stride, col_stride, device, out);
}

bq4_status bq4_f16_conv_weight_prepare(const uint32_t* packed_oihw, int64_t out_channels, int64_t in_channels,
                                       int32_t kernel_h, int32_t kernel_w, int32_t device, bq4_weight** out) {
  if (!out) return set_error(BQ4_EINVAL_ARG, "out is NULL");
  *out = nullptr;
  if (!packed_oihw) return set_error(BQ4_EINVAL_ARG, "packed_oihw is NULL");
  if (out_channels <= 0 || in_channels <= 0 || kernel_h <= 0 || kernel_w <= 0 || out_channels > (1 << 20) ||
      in_channels > (1 << 20) || (int64_t)kernel_h * kernel_w > 1024)
    return set_error(BQ4_EINVAL_SHAPE, "conv weight [%lld, %lld, %d, %d] out of range", (long long)out_channels,
                     (long long)in_channels, (int)kernel_h, (int)kernel_w);
  bq4_weight view;
  conv_view(out_channels, in_channels, kernel_h, kernel_w, &view);
  if (view.K > ((int64_t)1 << 24)) return set_error(BQ4_EINVAL_SHAPE, "in_channels * kernel area too large");
  const size_t count = (size_t)(out_channels * in_channels * kernel_h * kernel_w);
  return prepare_f16_weight(packed_oihw, count, &view, 0, 0, device, out);
}

bq4_status bq4_packed_f16_rhs_matmul_workspace_size(int64_t M, int64_t K, int64_t N, size_t* bytes) {
  if (!bytes) return set_error(BQ4_EINVAL_ARG, "bytes is NULL");
  bq4_status st = check_linear_geometry(K, N, 0, 0);
  if (st) return st;
  int dev = 0;
  cudaGetDevice(&dev);
  bq4_weight w;
  f16_view(K, N, &w);
  GemmPlan plan;
  st = plan_gemm(&w, 1, M, dev, &plan);
  if (st) return st;
  const size_t xpad = K % 4 ? up256((size_t)M * (size_t)w.Kp * sizeof(float)) : 0;
  *bytes = up256(w.h_bytes) + xpad + plan.workspace_bytes;
  return BQ4_OK;
}

bq4_status bq4_packed_f16_rhs_matmul(const float* lhs, int64_t M, int64_t K, const uint32_t* packed_rhs,
                                     int64_t inner_stride, int64_t col_stride, int64_t N, float* out,
                                     void* workspace, size_t workspace_bytes, bq4_stream_t stream) {
  if (!lhs || !packed_rhs || !out) return set_error(BQ4_EINVAL_ARG, "NULL pointer");
  bq4_status st = check_linear_geometry(K, N, inner_stride, col_stride);
  if (st) return st;
  int dev = 0;
  cudaGetDevice(&dev);
  st = need_sm100(dev);
  if (st) return st;
  size_t need = 0;
  st = bq4_packed_f16_rhs_matmul_workspace_size(M, K, N, &need);
  if (st) return st;
  if (!workspace || workspace_bytes < need)
    return set_error(BQ4_EWORKSPACE, "workspace %zu < required %zu bytes", workspace_bytes, need);
  if (!al(workspace, 256)) return set_error(BQ4_EALIGN, "workspace not 256-byte aligned");
  if (K % 4 == 0 && !al(lhs, 16)) return set_error(BQ4_EALIGN, "lhs must be 16-byte aligned");
  if (!al(out, 4)) return set_error(BQ4_EALIGN, "out not 4-byte aligned");
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  bq4_weight w;
  f16_view(K, N, &w);
  w.device = dev;
  uint8_t* p = static_cast<uint8_t*>(workspace);
  w.h = reinterpret_cast<uint16_t*>(p);
  p += up256(w.h_bytes);
  cudaError_t e = launch_prepare_f16(reinterpret_cast<const uint16_t*>(packed_rhs), &w, inner_stride, col_stride, s);
  if (e != cudaSuccess) return check_cuda(e, "packed-F16 rhs preparation");
  const float* x = lhs;
  int64_t ldx = K;
  if (K % 4) {  // TMA rows need a 16-byte pitch: stage lhs at pitch Kp
    float* xs = reinterpret_cast<float*>(p);
    p += up256((size_t)M * (size_t)w.Kp * sizeof(float));
    pad_rows_kernel<<<grid_for(M * w.Kp, 256, dev), 256, 0, s>>>(lhs, M, K, K, w.Kp, xs);
    note_launch();
    e = cudaGetLastError();
    if (e != cudaSuccess) return check_cuda(e, "lhs staging launch");
    x = xs;
    ldx = w.Kp;
  }
  GemmPlan plan;
  st = plan_gemm(&w, 1, M, dev, &plan);
  if (st) return st;
  const bq4_weight* wl[1] = {&w};
  const float* b[1] = {nullptr};
  return run_gemm(plan, wl, x, M, ldx, b, (int)BQ4_ACT_NONE, nullptr, out, p, s);
}

bq4_status bq4_conv2d_workspace_size(const bq4_weight* w, int64_t batch, int64_t in_h, int64_t in_w,
                                     const bq4_conv2d_options* options, size_t* bytes) {
  if (!bytes) return set_error(BQ4_EINVAL_ARG, "bytes is NULL");
  ConvShape cs;
  bq4_status st = conv_shape(w, batch, in_h, in_w, options, &cs);
  if (st) return st;
  GemmPlan plan;
  return conv_workspace(w, cs, w->device, &plan, bytes);
}

bq4_status bq4_conv2d(const float* input, int64_t batch, int64_t in_h, int64_t in_w, const bq4_weight* w,
                      const float* bias, const bq4_conv2d_options* options, float* out, void* workspace,
                      size_t workspace_bytes, bq4_stream_t stream) {
  if (!input || !out) return set_error(BQ4_EINVAL_ARG, "input/out is NULL");
  if (!al(input, 4) || !al(out, 4)) return set_error(BQ4_EALIGN, "input/out not 4-byte aligned");
  if (!w || !w->h || !w->conv_kh) return set_error(BQ4_EINVAL_ARG, "w is not a prepared packed-F16 conv weight");
  Guard guard(w->device);
  return run_conv(input, batch, in_h, in_w, w, bias, options, out, static_cast<uint8_t*>(workspace), workspace_bytes,
                  reinterpret_cast<cudaStream_t>(stream));
}

bq4_status bq4_packed_f16_conv2d_workspace_size(int64_t batch, int64_t in_channels, int64_t in_h, int64_t in_w,
                                                int64_t out_channels, int32_t kernel_h, int32_t kernel_w,
                                                const bq4_conv2d_options* options, size_t* bytes) {
  if (!bytes) return set_error(BQ4_EINVAL_ARG, "bytes is NULL");
  if (out_channels <= 0 || in_channels <= 0 || kernel_h <= 0 || kernel_w <= 0 || out_channels > (1 << 20) ||
      in_channels > (1 << 20) || (int64_t)kernel_h * kernel_w > 1024)
    return set_error(BQ4_EINVAL_SHAPE, "conv weight shape out of range");
  int dev = 0;
  cudaGetDevice(&dev);
  bq4_weight w;
  conv_view(out_channels, in_channels, kernel_h, kernel_w, &w);
  w.device = dev;
  ConvShape cs;
  bq4_status st = conv_shape(&w, batch, in_h, in_w, options, &cs);
  if (st) return st;
  GemmPlan plan;
  size_t conv = 0;
  st = conv_workspace(&w, cs, dev, &plan, &conv);
  if (st) return st;
  *bytes = up256(w.h_bytes) + conv;
  return BQ4_OK;
}

bq4_status bq4_packed_f16_conv2d(const float* input, int64_t batch, int64_t in_channels, int64_t in_h, int64_t in_w,
                                 const uint32_t* packed_weight, int64_t out_channels, int32_t kernel_h,
                                 int32_t kernel_w, const float* bias, const bq4_conv2d_options* options, float* out,
                                 void* workspace, size_t workspace_bytes, bq4_stream_t stream) {
  if (!input || !packed_weight || !out) return set_error(BQ4_EINVAL_ARG, "NULL pointer");
  if (!al(input, 4) || !al(out, 4)) return set_error(BQ4_EALIGN, "input/out not 4-byte aligned");
  size_t need = 0;
  bq4_status st = bq4_packed_f16_conv2d_workspace_size(batch, in_channels, in_h, in_w, out_channels, kernel_h,
                                                       kernel_w, options, &need);
  if (st) return st;
  if (!workspace || workspace_bytes < need)
    return set_error(BQ4_EWORKSPACE, "workspace %zu < required %zu bytes", workspace_bytes, need);
  if (!al(workspace, 256)) return set_error(BQ4_EALIGN, "workspace not 256-byte aligned");
  int dev = 0;
  cudaGetDevice(&dev);
  st = need_sm100(dev);
  if (st) return st;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  bq4_weight w;
  conv_view(out_channels, in_channels, kernel_h, kernel_w, &w);
  w.device = dev;
  uint8_t* p = static_cast<uint8_t*>(workspace);
  w.h = reinterpret_cast<uint16_t*>(p);
  cudaError_t e = launch_prepare_f16(reinterpret_cast<const uint16_t*>(packed_weight), &w, 0, 0, s);
  if (e != cudaSuccess) return check_cuda(e, "packed-F16 conv weight preparation");
  const size_t wb = up256(w.h_bytes);
  return run_conv(input, batch, in_h, in_w, &w, bias, options, out, p + wb, workspace_bytes - wb, s);
}

}  // extern "C"

// ---------------------------------------------------------------- attention

namespace bq4 {
// fused attention for head_dim 128 (bq4_attn_fused.cu)
size_t attn_fused_workspace(int64_t B, int64_t Hkv, int64_t Skv);
bq4_status attn_fused_check(int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Skv);
bq4_status attn_fused(const uint16_t* q, const uint16_t* k, const uint16_t* v, int64_t B, int64_t Hq, int64_t Hkv,
                      int64_t Sq, int64_t Skv, float scale, float* out, void* workspace, cudaStream_t s);
}  // namespace bq4

namespace {

struct AttnLayout {
  size_t q32, s, kt, vt, gemm, inv, total;  // workspace parts (256-aligned offsets follow this order)
  int64_t ldS;                          // score row pitch (multiple of 4: the PV GEMM reads rows in place)
};

bq4_status attn_layout(int64_t Sq, int64_t Skv, int64_t D, int dev, AttnLayout* L, GemmPlan* ps, GemmPlan* pv) {
  if (Sq <= 0 || Skv <= 0 || D <= 0 || D % 4 || D > 1024 || Sq > (1 << 24) || Skv > (1 << 24))
    return set_error(BQ4_EINVAL_SHAPE, "Sq=%lld Skv=%lld D=%lld (D %% 4 == 0, D <= 1024)", (long long)Sq,
                     (long long)Skv, (long long)D);
  L->ldS = round_up(Skv, 4);
  bq4_weight wk, wv;
  f16_view(D, Skv, &wk);
  f16_view(Skv, D, &wv);
  bq4_status st = plan_gemm(&wk, 1, Sq, dev, ps);
  if (st) return st;
  st = plan_gemm(&wv, 1, Sq, dev, pv);
  if (st) return st;
  L->q32 = up256((size_t)Sq * D * sizeof(float));
  L->s = up256((size_t)Sq * L->ldS * sizeof(float));
  L->kt = up256(wk.h_bytes);
  L->vt = up256(wv.h_bytes);
  L->gemm = up256(ps->workspace_bytes > pv->workspace_bytes ? ps->workspace_bytes : pv->workspace_bytes);
  L->inv = up256((size_t)Sq * sizeof(float));
  L->total = L->q32 + L->s + L->kt + L->vt + L->gemm + L->inv;
  return BQ4_OK;
}

bool attn_use_fused(int64_t D) { return D == 128 && !getenv("BQ4_ATTN_UNFUSED"); }

bq4_status attn_check(int64_t B, int64_t Hq, int64_t Hkv) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || B * Hq > (1 << 20))
    return set_error(BQ4_EINVAL_SHAPE, "B=%lld Hq=%lld Hkv=%lld (Hq %% Hkv == 0)", (long long)B, (long long)Hq,
                     (long long)Hkv);
  return BQ4_OK;
}

}  // namespace

extern "C" {

bq4_status bq4_attention_workspace_size(int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Skv, int64_t D,
                                        size_t* bytes) {
  if (!bytes) return set_error(BQ4_EINVAL_ARG, "bytes is NULL");
  bq4_status st = attn_check(B, Hq, Hkv);
  if (st) return st;
  int dev = 0;
  cudaGetDevice(&dev);
  AttnLayout L;
  GemmPlan ps, pv;
  st = attn_layout(Sq, Skv, D, dev, &L, &ps, &pv);
  if (st) return st;
  if (attn_use_fused(D)) {
    st = attn_fused_check(B, Hq, Hkv, Sq, Skv);
    if (st) return st;
  }
  *bytes = attn_use_fused(D) ? attn_fused_workspace(B, Hkv, Skv) : L.total;
  return BQ4_OK;
}

bq4_status bq4_attention(const uint32_t* q, const uint32_t* k, const uint32_t* v, int64_t B, int64_t Hq, int64_t Hkv,
                         int64_t Sq, int64_t Skv, int64_t D, float scale, float* out, void* workspace,
                         size_t workspace_bytes, bq4_stream_t stream) {
  if (!q || !k || !v || !out) return set_error(BQ4_EINVAL_ARG, "NULL pointer");
  bq4_status st = attn_check(B, Hq, Hkv);
  if (st) return st;
  if (!al(out, 16)) return set_error(BQ4_EALIGN, "out must be 16-byte aligned");
  int dev = 0;
  cudaGetDevice(&dev);
  st = need_sm100(dev);
  if (st) return st;
  AttnLayout L;
  GemmPlan ps, pv;
  st = attn_layout(Sq, Skv, D, dev, &L, &ps, &pv);
  if (st) return st;
  const bool fused = attn_use_fused(D);
  if (fused) {
    st = attn_fused_check(B, Hq, Hkv, Sq, Skv);
    if (st) return st;
  }
  const size_t need = fused ? attn_fused_workspace(B, Hkv, Skv) : L.total;
  if (!workspace || workspace_bytes < need)
    return set_error(BQ4_EWORKSPACE, "workspace %zu < required %zu bytes", workspace_bytes, need);
  if (!al(workspace, 256)) return set_error(BQ4_EALIGN, "workspace not 256-byte aligned");
  if (!al(q, 16) || !al(k, 16) || !al(v, 16)) return set_error(BQ4_EALIGN, "q/k/v must be 16-byte aligned");
  const float sc = scale > 0.0f ? scale : 1.0f / std::sqrt((float)D);
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (fused)
    return attn_fused(reinterpret_cast<const uint16_t*>(q), reinterpret_cast<const uint16_t*>(k),
                      reinterpret_cast<const uint16_t*>(v), B, Hq, Hkv, Sq, Skv, sc, out, workspace, s);
  uint8_t* p = static_cast<uint8_t*>(workspace);
  float* q32 = reinterpret_cast<float*>(p);
  float* S = reinterpret_cast<float*>(p + L.q32);
  bq4_weight wk, wv;
  f16_view(D, Skv, &wk);
  f16_view(Skv, D, &wv);
  wk.device = wv.device = dev;
  wk.h = reinterpret_cast<uint16_t*>(p + L.q32 + L.s);
  wv.h = reinterpret_cast<uint16_t*>(p + L.q32 + L.s + L.kt);
  void* gws = p + L.q32 + L.s + L.kt + L.vt;
  float* inv = reinterpret_cast<float*>(p + L.q32 + L.s + L.kt + L.vt + L.gemm);
  const uint16_t* q16 = reinterpret_cast<const uint16_t*>(q);
  const uint16_t* k16 = reinterpret_cast<const uint16_t*>(k);
  const uint16_t* v16 = reinterpret_cast<const uint16_t*>(v);
  const int64_t group = Hq / Hkv;
  const bq4_weight* wl[1];
  const float* nob[1] = {nullptr};
  for (int64_t b = 0; b < B; ++b) {
    for (int64_t hk = 0; hk < Hkv; ++hk) {
      // k as the rhs [D][Skv] (element (d, j) at j * D + d), v as [Skv][D]
      const uint16_t* kb = k16 + (b * Hkv + hk) * Skv * D;
      const uint16_t* vb = v16 + (b * Hkv + hk) * Skv * D;
      cudaError_t e = launch_prepare_f16(kb, &wk, 1, D, s);
      if (e == cudaSuccess) e = launch_prepare_f16(vb, &wv, D, 1, s);
      if (e != cudaSuccess) return check_cuda(e, "attention k/v preparation");
      for (int64_t g = 0; g < group; ++g) {
        const int64_t h = hk * group + g;
        const uint16_t* qb = q16 + (b * Hq + h) * Sq * D;
        attn_q_rows_kernel<<<grid_for(Sq * D, 256, dev), 256, 0, s>>>(qb, Sq, (int)D, D, q32);
        note_launch();
        e = cudaGetLastError();
        if (e != cudaSuccess) return check_cuda(e, "attention q staging launch");
        GemmIo io;
        io.ldy = L.ldS;
        wl[0] = &wk;
        st = run_gemm(ps, wl, q32, Sq, D, nob, (int)BQ4_ACT_NONE, nullptr, S, gws, s, io);  // S = q k^T
        if (st) return st;
        const int grid = Sq < 148 * 16 ? (int)Sq : 148 * 16;
        attn_softmax_kernel<<<grid, 256, 0, s>>>(S, Sq, Skv, L.ldS, sc, inv);
        note_launch();
        e = cudaGetLastError();
        if (e != cudaSuccess) return check_cuda(e, "attention softmax launch");
        GemmIo io2;
        io2.ldy = D;
        wl[0] = &wv;
        float* ob = out + (b * Hq + h) * Sq * D;
        st = run_gemm(pv, wl, S, Sq, L.ldS, nob, (int)BQ4_ACT_NONE, nullptr, ob, gws, s, io2);  // O = e v
        if (st) return st;
        attn_scale_rows_kernel<<<grid_for(Sq * D, 256, dev), 256, 0, s>>>(ob, Sq, (int)D, inv);  // / sum(e)
        note_launch();
        e = cudaGetLastError();
        if (e != cudaSuccess) return check_cuda(e, "attention row scaling launch");
      }
    }
  }
  return BQ4_OK;
}

}  // extern "C"
