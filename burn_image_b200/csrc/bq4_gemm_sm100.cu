// bq4_gemm_sm100.cu -- packed signed-Q4 x f16 GEMM on the 5th-generation
// tensor cores (tcgen05 + TMEM), sm_100a only.
//
// Computes y[M,N] = epilogue(x[M,K] . W[K,N]) for a prepared Q4 weight W.
// Swap-AB formulation: the MMA "A" operand is a 128-row tile of output
// features (dequantized weights, K-major), the "B" operand is a BT-row tile
// of tokens (f16 activations, K-major), so D[n, m] accumulates in TMEM with
// TMEM lane = output feature and TMEM column = token.
//
// Warp roles (352 threads, one CTA per SM, persistent over work units):
//   warps 0-3  epilogue: tcgen05.ld of the accumulator, bias / GELU-tanh /
//              SiLU-gate / aux-multiply, coalesced f32 stores (or split-K
//              partials plus a last-arriver fix-up)
//   warps 4-7  dequant: read a raw 4 KiB nibble tile + its scales from shared
//              memory, expand to f16(q * scale) and write the A tile in the
//              128-byte-swizzled K-major layout the MMA reads
//   warp 8     TMA producer for token tiles (2-D tensor map, no multicast)
//   warp 9     bulk-copy producer for raw nibble/scale tiles (1-D bulk copies)
//   warp 10    TMEM allocator and single-thread MMA issuer
//
// Numerics: operands staged as f16 (activations rounded to nearest even,
// weights f16(q * f16(scale))), f32 accumulation.  This is the staging of the
// reference GPU kernel (patches/burn-cubecl-0.21.0/src/kernel/matmul/
// quantized.rs:172-178: lhs and rhs stage/register dtypes f16, f32 acc).
//
// Every mbarrier wait is time-bounded; on expiry the kernel records
// BQ4_ETIMEOUT in the device error word, raises a shared abort flag so every
// role leaves its loop, frees TMEM and returns.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "bq4_internal.h"
#include "sm100_ptx.cuh"

namespace bq4 {
namespace {

constexpr int kThreads = 352;
constexpr int kEpiWarps = 4;
constexpr int kDqWarp0 = 4;
constexpr int kTmaWarp = 8;
constexpr int kRawWarp = 9;
constexpr int kMmaWarp = 10;
constexpr uint32_t kATileBytes = 128 * 128;  // 128 rows x 64 f16
constexpr uint32_t kRawQBytes = 4096;        // 128 rows x 64 nibbles

struct GemmArgs {
  const uint16_t* h[2];  // pre-expanded f16 tiles (pre == 1)
  int pre;
  const uint32_t* q[2];
  const float* s[2];
  const float* bias[2];
  const float* aux;
  float* y;
  float* partials;
  int* counters;
  int M, N;
  int nkc, nkb, block;
  int ntiles, mtiles, ksplit, units;
  int stages, raw_stages;
  uint32_t raw_s_bytes;  // scale bytes per weight per raw stage (bulk-copied)
  uint32_t raw_w_bytes;  // shared-memory bytes per weight per raw stage (host-computed)
  int act;
};

__device__ __forceinline__ float gelu_tanh(float v) {
  // Burn Gelu::new_approximate: 0.5 v (1 + tanh(sqrt(2/pi) (v + 0.044715 v^3)))
  const float u = 0.7978845608028654f * (v + 0.044715f * v * v * v);
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
  return 0.5f * v * (1.0f + t);
}

__device__ __forceinline__ float silu(float v) { return __fdividef(v, 1.0f + __expf(-v)); }

__device__ __forceinline__ float apply_act(float v, int act) {
  if (act == BQ4_ACT_GELU_TANH) return gelu_tanh(v);
  if (act == BQ4_ACT_SILU) return silu(v);
  return v;
}

// Expand one prepared word (8 K values of one row) into 8 f16 = q * scale.
// (w >> 4i) & 0x000F000F selects the nibble pair (2i, 2i+1); XOR 0x6408 maps
// the two's-complement nibble to the f16 1024 + (q + 8); subtracting 1032
// leaves q exactly; one f16x2 multiply applies the scale.
__device__ __forceinline__ uint4 expand_word(uint32_t w, uint32_t scale2) {
  const uint32_t magic = 0x64086408u;
  uint32_t p[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t src = w >> (4 * i);
    uint32_t t;
    asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(t) : "r"(src), "r"(0x000F000Fu), "r"(magic));
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(t) : "r"(t), "r"(magic));
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(p[i]) : "r"(t), "r"(scale2));
  }
  return make_uint4(p[0], p[1], p[2], p[3]);
}

__device__ __forceinline__ uint32_t scale_to_f16x2(float s) {
  uint16_t h;
  asm("cvt.rn.satfinite.f16.f32 %0, %1;" : "=h"(h) : "f"(s));
  return static_cast<uint32_t>(h) | (static_cast<uint32_t>(h) << 16);
}

}  // namespace

// First error status recorded by any bq4 kernel on this device since the last
// poll (0 = none).  Read and cleared by bq4_poll_device_error().
__device__ int g_bq4_device_error = 0;

namespace {

__device__ __forceinline__ void record_error(const GemmArgs& a, volatile int* abort_flag, int code) {
  (void)a;
  if (!*abort_flag) {
    *abort_flag = 1;
    atomicCAS(&g_bq4_device_error, 0, code);
  }
}

template <int BT, int NW>
__global__ void __launch_bounds__(kThreads, 1)
    q4_gemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the swizzled operand tiles.
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  const int S = a.stages, RS = a.raw_stages;
  constexpr uint32_t kBTileBytes = BT * 128;
  uint8_t* a_tiles = smem;                                        // [S][NW][16 KiB]
  uint8_t* b_tiles = a_tiles + (size_t)S * NW * kATileBytes;      // [S][BT*128]
  uint8_t* raw = b_tiles + (size_t)S * kBTileBytes;               // [RS][NW][4 KiB + scales]
  const uint32_t raw_w_bytes = a.raw_w_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(raw + (size_t)RS * NW * raw_w_bytes);
  uint64_t* full = bars;
  uint64_t* empty = full + S;
  uint64_t* raw_full = empty + S;
  uint64_t* raw_empty = raw_full + RS;
  uint64_t* tmem_full = raw_empty + RS;
  uint64_t* tmem_empty = tmem_full + 2;
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(tmem_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);
  volatile int* last_flag = abort_flag + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      // TMA expect_tx arrival + 4 dequant warps (pre-expanded tiles: TMA only)
      ptx::mbar_init(&full[i], a.pre ? 1 : 1 + 4);
      ptx::mbar_init(&empty[i], 1);  // tcgen05.commit
    }
    for (int i = 0; i < RS; ++i) {
      ptx::mbar_init(&raw_full[i], 1);
      ptx::mbar_init(&raw_empty[i], 4);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(&tmem_full[i], 1);
      ptx::mbar_init(&tmem_empty[i], kEpiWarps);
    }
    *abort_flag = 0;
    *last_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == kTmaWarp && lane == 0) ptx::prefetch_tmap(&tmap_x);
  constexpr uint32_t kTmemCols = 2 * NW * BT;  // double-buffered accumulators
  static_assert(kTmemCols == 128 || kTmemCols == 256 || kTmemCols == 512, "TMEM columns");
  if (warp == kMmaWarp) {
    ptx::tmem_alloc(tmem_base_slot, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;

  const int S_split = a.ksplit;

  if (warp == kTmaWarp) {
    // ------------------------------------------------ token tiles (TMA)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int u = blockIdx.x; u < a.units && !*abort_flag; u += gridDim.x) {
        const int tile = u / S_split, split = u - tile * S_split;
        const int mtile = tile % a.mtiles;
        const int ntile = tile / a.mtiles;
        const int kc0 = (int)((int64_t)split * a.nkc / S_split);
        const int kc1 = (int)((int64_t)(split + 1) * a.nkc / S_split);
        for (int kc = kc0; kc < kc1; ++kc) {
          if (!ptx::mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
            record_error(a, abort_flag, BQ4_ETIMEOUT);
            break;
          }
          ptx::mbar_arrive_expect_tx(&full[stage], kBTileBytes + (a.pre ? NW * kATileBytes : 0u));
          ptx::tma_load_2d(b_tiles + (size_t)stage * kBTileBytes, &tmap_x, &full[stage],
                           kc * kChunkK, mtile * BT);
          if (a.pre) {
#pragma unroll
            for (int w = 0; w < NW; ++w)
              ptx::bulk_load(a_tiles + ((size_t)stage * NW + w) * kATileBytes,
                             a.h[w] + ((size_t)ntile * a.nkc + kc) * (kATileBytes / 2), kATileBytes,
                             &full[stage]);
          }
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == kRawWarp) {
    // ------------------------------------------------ raw weight tiles (bulk)
    if (lane == 0 && !a.pre) {
      int rs = 0;
      uint32_t rphase = 0;
      for (int u = blockIdx.x; u < a.units && !*abort_flag; u += gridDim.x) {
        const int tile = u / S_split, split = u - tile * S_split;
        const int ntile = tile / a.mtiles;
        const int kc0 = (int)((int64_t)split * a.nkc / S_split);
        const int kc1 = (int)((int64_t)(split + 1) * a.nkc / S_split);
        for (int kc = kc0; kc < kc1; ++kc) {
          if (!ptx::mbar_wait(&raw_empty[rs], rphase ^ 1, abort_flag)) {
            record_error(a, abort_flag, BQ4_ETIMEOUT);
            break;
          }
          ptx::mbar_arrive_expect_tx(&raw_full[rs], NW * raw_w_bytes);
          const int kb0 = (kc * kChunkK) / a.block;
#pragma unroll
          for (int w = 0; w < NW; ++w) {
            uint8_t* dst = raw + ((size_t)rs * NW + w) * raw_w_bytes;
            ptx::bulk_load(dst, a.q[w] + ((size_t)ntile * a.nkc + kc) * 1024, kRawQBytes,
                           &raw_full[rs]);
            ptx::bulk_load(dst + kRawQBytes, a.s[w] + ((size_t)ntile * a.nkb + kb0) * 128,
                           a.raw_s_bytes, &raw_full[rs]);
          }
          if (++rs == RS) { rs = 0; rphase ^= 1; }
        }
      }
    }
  } else if (warp >= kDqWarp0 && warp < kDqWarp0 + 4) {
    // ------------------------------------------------ dequant producers
    const int r = threadIdx.x - kDqWarp0 * 32;  // A-tile row = output feature in tile
    const int sw = r & 7;
    int stage = 0, rs = 0;
    uint32_t phase = 0, rphase = 0;
    const int block = a.block;
    bool ok = true;
    if (a.pre) ok = false;  // pre-expanded tiles arrive by bulk copy
    for (int u = blockIdx.x; ok && u < a.units && !*abort_flag; u += gridDim.x) {
      const int tile = u / S_split, split = u - tile * S_split;
      const int kc0 = (int)((int64_t)split * a.nkc / S_split);
      const int kc1 = (int)((int64_t)(split + 1) * a.nkc / S_split);
      for (int kc = kc0; kc < kc1; ++kc) {
        if (!ptx::mbar_wait(&raw_full[rs], rphase, abort_flag)) { ok = false; break; }
        uint4 words[NW][2];
        uint32_t sc[NW][8];
#pragma unroll
        for (int w = 0; w < NW; ++w) {
          const uint8_t* src = raw + ((size_t)rs * NW + w) * raw_w_bytes;
          words[w][0] = *reinterpret_cast<const uint4*>(src + (size_t)r * 16);
          words[w][1] = *reinterpret_cast<const uint4*>(src + (size_t)(128 + r) * 16);
          const float* ss = reinterpret_cast<const float*>(src + kRawQBytes);
          if (block >= 64) {
            const uint32_t s2 = scale_to_f16x2(ss[r]);
#pragma unroll
            for (int j = 0; j < 8; ++j) sc[w][j] = s2;
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) sc[w][j] = scale_to_f16x2(ss[((j * 8) / block) * 128 + r]);
          }
        }
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&raw_empty[rs]);
        if (++rs == RS) { rs = 0; rphase ^= 1; }

        if (!ptx::mbar_wait(&empty[stage], phase ^ 1, abort_flag)) { ok = false; break; }
#pragma unroll
        for (int w = 0; w < NW; ++w) {
          uint8_t* dst = a_tiles + ((size_t)stage * NW + w) * kATileBytes + (size_t)r * 128;
          const uint32_t wv[8] = {words[w][0].x, words[w][0].y, words[w][0].z, words[w][0].w,
                                  words[w][1].x, words[w][1].y, words[w][1].z, words[w][1].w};
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint4 v = expand_word(wv[j], sc[w][j]);
            *reinterpret_cast<uint4*>(dst + ((j ^ sw) << 4)) = v;
          }
        }
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&full[stage]);
        if (++stage == S) { stage = 0; phase ^= 1; }
      }
    }
    if (!ok && !a.pre) record_error(a, abort_flag, BQ4_ETIMEOUT);
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = ptx::umma_idesc_f16(128, BT);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < a.units && !*abort_flag; u += gridDim.x) {
        const int split = u % S_split;
        const int kc0 = (int)((int64_t)split * a.nkc / S_split);
        const int kc1 = (int)((int64_t)(split + 1) * a.nkc / S_split);
        if (!ptx::mbar_wait(&tmem_empty[acc], acc_phase ^ 1, abort_flag)) { ok = false; break; }
        ptx::tc_fence_after();
        const uint32_t d_base = tmem_base + (uint32_t)(acc * NW * BT);
        for (int kc = kc0; kc < kc1; ++kc) {
          if (!ptx::mbar_wait(&full[stage], phase, abort_flag)) { ok = false; break; }
          ptx::tc_fence_after();
          const uint32_t b_addr = ptx::smem_u32(b_tiles + (size_t)stage * kBTileBytes);
#pragma unroll
          for (int kk = 0; kk < kChunkK / 16; ++kk) {
            const uint64_t b_desc = ptx::umma_desc_sw128(b_addr + kk * 32);
#pragma unroll
            for (int w = 0; w < NW; ++w) {
              const uint32_t a_addr =
                  ptx::smem_u32(a_tiles + ((size_t)stage * NW + w) * kATileBytes) + kk * 32;
              ptx::mma_f16_ss(d_base + w * BT, ptx::umma_desc_sw128(a_addr), b_desc, idesc,
                              (kc > kc0 || kk > 0) ? 1u : 0u);
            }
          }
          ptx::mma_commit(&empty[stage]);
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        ptx::mma_commit(&tmem_full[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
      if (!ok) record_error(a, abort_flag, BQ4_ETIMEOUT);
    }
  } else if (warp < kEpiWarps) {
    // ------------------------------------------------ epilogue
    const int row = warp * 32 + lane;  // TMEM lane = output feature within tile
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < a.units && !*abort_flag; u += gridDim.x) {
      const int tile = u / S_split, split = u - tile * S_split;
      const int ntile = tile / a.mtiles, mtile = tile - ntile * a.mtiles;
      const int n = ntile * 128 + row;
      const int m0 = mtile * BT;
      if (!ptx::mbar_wait(&tmem_full[acc], acc_phase, abort_flag)) { ok = false; break; }
      ptx::tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(warp * 32) << 16) + (uint32_t)(acc * NW * BT);

      if (S_split == 1) {
        float b0 = 0.0f, b1 = 0.0f;
        if (n < a.N) {
          if (a.bias[0]) b0 = __ldg(a.bias[0] + n);
          if (NW == 2 && a.bias[1]) b1 = __ldg(a.bias[1] + n);
        }
#pragma unroll 1
        for (int c = 0; c < BT / 32; ++c) {
          uint32_t r0[32];
          uint32_t r1[32];
          ptx::tmem_ld_32x32b_x32(t_row + c * 32, r0);
          if (NW == 2) ptx::tmem_ld_32x32b_x32(t_row + BT + c * 32, r1);
          ptx::tmem_ld_wait();
          if (n < a.N) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int m = m0 + c * 32 + j;
              if (m < a.M) {
                float v;
                if (NW == 2) {
                  v = silu(__uint_as_float(r0[j]) + b0) * (__uint_as_float(r1[j]) + b1);
                } else {
                  v = apply_act(__uint_as_float(r0[j]) + b0, a.act);
                  if (a.aux) v *= __ldg(a.aux + (size_t)m * a.N + n);
                }
                a.y[(size_t)m * a.N + n] = v;
              }
            }
          }
        }
      } else {
        // Split-K: write this split's partial tile ([NW][128 rows][BT] f32),
        // then the last of the S splits to arrive sums all partials in split
        // order (deterministic) and applies the epilogue.
        float* part = a.partials + ((size_t)tile * S_split + split) * NW * 128 * BT;
#pragma unroll 1
        for (int c = 0; c < BT / 32; ++c) {
#pragma unroll
          for (int w = 0; w < NW; ++w) {
            uint32_t r0[32];
            ptx::tmem_ld_32x32b_x32(t_row + w * BT + c * 32, r0);
            ptx::tmem_ld_wait();
            float4* dst = reinterpret_cast<float4*>(part + ((size_t)w * 128 + row) * BT + c * 32);
#pragma unroll
            for (int j = 0; j < 8; ++j)
              dst[j] = make_float4(__uint_as_float(r0[4 * j]), __uint_as_float(r0[4 * j + 1]),
                                   __uint_as_float(r0[4 * j + 2]), __uint_as_float(r0[4 * j + 3]));
          }
        }
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (threadIdx.x == 0) {
          const int prev = atomicAdd(a.counters + tile, 1);
          *last_flag = (prev == S_split - 1) ? 1 : 0;
          if (prev == S_split - 1) a.counters[tile] = 0;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (*last_flag) {
          __threadfence();
          float b0 = 0.0f, b1 = 0.0f;
          if (n < a.N) {
            if (a.bias[0]) b0 = __ldg(a.bias[0] + n);
            if (NW == 2 && a.bias[1]) b1 = __ldg(a.bias[1] + n);
          }
          const float* base = a.partials + (size_t)tile * S_split * NW * 128 * BT;
#pragma unroll 1
          for (int c = 0; c < BT / 32; ++c) {
            float g[32], up[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) g[j] = up[j] = 0.0f;
            for (int sp = 0; sp < S_split; ++sp) {
              const float* p = base + (size_t)sp * NW * 128 * BT;
              const float4* s0 = reinterpret_cast<const float4*>(p + (size_t)row * BT + c * 32);
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const float4 v = __ldcg(s0 + j);
                g[4 * j] += v.x; g[4 * j + 1] += v.y; g[4 * j + 2] += v.z; g[4 * j + 3] += v.w;
              }
              if (NW == 2) {
                const float4* s1 =
                    reinterpret_cast<const float4*>(p + (size_t)(128 + row) * BT + c * 32);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  const float4 v = __ldcg(s1 + j);
                  up[4 * j] += v.x; up[4 * j + 1] += v.y; up[4 * j + 2] += v.z; up[4 * j + 3] += v.w;
                }
              }
            }
            if (n < a.N) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const int m = m0 + c * 32 + j;
                if (m < a.M) {
                  float v;
                  if (NW == 2) {
                    v = silu(g[j] + b0) * (up[j] + b1);
                  } else {
                    v = apply_act(g[j] + b0, a.act);
                    if (a.aux) v *= __ldg(a.aux + (size_t)m * a.N + n);
                  }
                  a.y[(size_t)m * a.N + n] = v;
                }
              }
            }
          }
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");  // last_flag reuse guard
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&tmem_empty[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
    if (!ok) record_error(a, abort_flag, BQ4_ETIMEOUT);
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Exact-weight kernel (blocks of 64 or 128 K values).
//
// The dequant warps stage q itself (exact small integers in f16); the MMA
// accumulates one K-block segment at a time into one of kNumPart TMEM
// partial buffers; eight scaler warps drain each partial with
// acc += scale[n, kb] * partial in f32 registers, so every weight enters the
// sum as exactly q * scale and only the activations are rounded (to f16).
// This is the "per-K-block scale on the f32 accumulator" formulation.
//
// Warp roles (480 threads): warps 0-7 scaler + epilogue (warp w covers TMEM
// lanes 32*(w%4).. and token columns [(w/4)*BT/2, (w/4+1)*BT/2)), warps 8-11
// dequant, warp 12 token TMA, warp 13 raw bulk copies, warp 14 MMA issuer.
// ---------------------------------------------------------------------------
constexpr int kExThreads = 480;
constexpr int kExScalerWarps = 8;
constexpr int kExDqWarp0 = 8;
constexpr int kExTmaWarp = 12;
constexpr int kExRawWarp = 13;
constexpr int kExMmaWarp = 14;
constexpr int kNumPart = 4;

// Expand one prepared word into 8 exact f16 values q (no scale).
__device__ __forceinline__ uint4 expand_word_exact(uint32_t w) {
  const uint32_t magic = 0x64086408u;
  uint32_t p[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t src = w >> (4 * i);
    uint32_t t;
    asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(t) : "r"(src), "r"(0x000F000Fu), "r"(magic));
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(p[i]) : "r"(t), "r"(magic));
  }
  return make_uint4(p[0], p[1], p[2], p[3]);
}

// Segment bookkeeping: the K chunks [kc0, kc1) of a unit, cut at K-block
// boundaries (a block spans block/64 chunks).
__device__ __forceinline__ bool seg_first(int kc, int kc0, int cpb) { return kc == kc0 || (kc % cpb) == 0; }
__device__ __forceinline__ bool seg_last(int kc, int kc1, int cpb) { return kc == kc1 - 1 || ((kc + 1) % cpb) == 0; }

template <int BT, int NW>
__global__ void __launch_bounds__(kExThreads, 1)
    q4_gemm_exact_kernel(const __grid_constant__ CUtensorMap tmap_x, const GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  const int S = a.stages, RS = a.raw_stages;
  constexpr uint32_t kBTileBytes = BT * 128;
  constexpr int kCols = BT / 2;             // token columns per scaler thread
  constexpr uint32_t kPartCols = NW * BT;   // TMEM columns per partial buffer
  constexpr uint32_t kTmemCols = kNumPart * kPartCols;
  static_assert(kTmemCols == 256 || kTmemCols == 512, "TMEM columns");
  static_assert(kCols % 32 == 0, "token columns per scaler thread");

  uint8_t* a_tiles = smem;
  uint8_t* b_tiles = a_tiles + (size_t)S * NW * kATileBytes;
  uint8_t* raw = b_tiles + (size_t)S * kBTileBytes;
  const uint32_t raw_w_bytes = a.raw_w_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(raw + (size_t)RS * NW * raw_w_bytes);
  uint64_t* full = bars;
  uint64_t* empty = full + S;
  uint64_t* raw_full = empty + S;
  uint64_t* raw_empty = raw_full + RS;
  uint64_t* part_full = raw_empty + RS;
  uint64_t* part_empty = part_full + kNumPart;
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(part_empty + kNumPart);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);
  volatile int* last_flag = abort_flag + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cpb = a.block / kChunkK;  // chunks per K block (1 or 2)

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      ptx::mbar_init(&full[i], 1 + 4);
      ptx::mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < RS; ++i) {
      ptx::mbar_init(&raw_full[i], 1);
      ptx::mbar_init(&raw_empty[i], 4);
    }
    for (int i = 0; i < kNumPart; ++i) {
      ptx::mbar_init(&part_full[i], 1);
      ptx::mbar_init(&part_empty[i], kExScalerWarps);
    }
    *abort_flag = 0;
    *last_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == kExTmaWarp && lane == 0) ptx::prefetch_tmap(&tmap_x);
  if (warp == kExMmaWarp) {
    ptx::tmem_alloc(tmem_base_slot, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;
  const int S_split = a.ksplit;

  if (warp == kExTmaWarp) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int u = blockIdx.x; u < a.units && !*abort_flag; u += gridDim.x) {
        const int tile = u / S_split, split = u - tile * S_split;
        const int mtile = tile % a.mtiles;
        const int kc0 = (int)((int64_t)split * a.nkc / S_split);
        const int kc1 = (int)((int64_t)(split + 1) * a.nkc / S_split);
        for (int kc = kc0; kc < kc1; ++kc) {
          if (!ptx::mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
            record_error(a, abort_flag, BQ4_ETIMEOUT);
            break;
          }
          ptx::mbar_arrive_expect_tx(&full[stage], kBTileBytes);
          ptx::tma_load_2d(b_tiles + (size_t)stage * kBTileBytes, &tmap_x, &full[stage], kc * kChunkK, mtile * BT);
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == kExRawWarp) {
    if (lane == 0) {
      int rs = 0;
      uint32_t rphase = 0;
      for (int u = blockIdx.x; u < a.units && !*abort_flag; u += gridDim.x) {
        const int tile = u / S_split, split = u - tile * S_split;
        const int ntile = tile / a.mtiles;
        const int kc0 = (int)((int64_t)split * a.nkc / S_split);
        const int kc1 = (int)((int64_t)(split + 1) * a.nkc / S_split);
        for (int kc = kc0; kc < kc1; ++kc) {
          if (!ptx::mbar_wait(&raw_empty[rs], rphase ^ 1, abort_flag)) {
            record_error(a, abort_flag, BQ4_ETIMEOUT);
            break;
          }
          ptx::mbar_arrive_expect_tx(&raw_full[rs], NW * kRawQBytes);
#pragma unroll
          for (int w = 0; w < NW; ++w) {
            uint8_t* dst = raw + ((size_t)rs * NW + w) * raw_w_bytes;
            ptx::bulk_load(dst, a.q[w] + ((size_t)ntile * a.nkc + kc) * 1024, kRawQBytes, &raw_full[rs]);
          }
          if (++rs == RS) { rs = 0; rphase ^= 1; }
        }
      }
    }
  } else if (warp >= kExDqWarp0 && warp < kExDqWarp0 + 4) {
    const int r = threadIdx.x - kExDqWarp0 * 32;
    const int sw = r & 7;
    int stage = 0, rs = 0;
    uint32_t phase = 0, rphase = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < a.units && !*abort_flag; u += gridDim.x) {
      const int tile = u / S_split, split = u - tile * S_split;
      const int kc0 = (int)((int64_t)split * a.nkc / S_split);
      const int kc1 = (int)((int64_t)(split + 1) * a.nkc / S_split);
      for (int kc = kc0; kc < kc1; ++kc) {
        if (!ptx::mbar_wait(&raw_full[rs], rphase, abort_flag)) { ok = false; break; }
        uint4 words[NW][2];
#pragma unroll
        for (int w = 0; w < NW; ++w) {
          const uint8_t* src = raw + ((size_t)rs * NW + w) * raw_w_bytes;
          words[w][0] = *reinterpret_cast<const uint4*>(src + (size_t)r * 16);
          words[w][1] = *reinterpret_cast<const uint4*>(src + (size_t)(128 + r) * 16);
        }
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&raw_empty[rs]);
        if (++rs == RS) { rs = 0; rphase ^= 1; }
        if (!ptx::mbar_wait(&empty[stage], phase ^ 1, abort_flag)) { ok = false; break; }
#pragma unroll
        for (int w = 0; w < NW; ++w) {
          uint8_t* dst = a_tiles + ((size_t)stage * NW + w) * kATileBytes + (size_t)r * 128;
          const uint32_t wv[8] = {words[w][0].x, words[w][0].y, words[w][0].z, words[w][0].w,
                                  words[w][1].x, words[w][1].y, words[w][1].z, words[w][1].w};
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<uint4*>(dst + ((j ^ sw) << 4)) = expand_word_exact(wv[j]);
        }
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&full[stage]);
        if (++stage == S) { stage = 0; phase ^= 1; }
      }
    }
    if (!ok) record_error(a, abort_flag, BQ4_ETIMEOUT);
  } else if (warp == kExMmaWarp) {
    if (lane == 0) {
      constexpr uint32_t idesc = ptx::umma_idesc_f16(128, BT);
      int stage = 0, pb = 0;
      uint32_t phase = 0, pphase = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < a.units && !*abort_flag; u += gridDim.x) {
        const int split = u % S_split;
        const int kc0 = (int)((int64_t)split * a.nkc / S_split);
        const int kc1 = (int)((int64_t)(split + 1) * a.nkc / S_split);
        uint32_t d_base = 0;
        for (int kc = kc0; kc < kc1; ++kc) {
          const bool first = seg_first(kc, kc0, cpb);
          if (first) {
            if (!ptx::mbar_wait(&part_empty[pb], pphase ^ 1, abort_flag)) { ok = false; break; }
            ptx::tc_fence_after();
            d_base = tmem_base + (uint32_t)pb * kPartCols;
          }
          if (!ptx::mbar_wait(&full[stage], phase, abort_flag)) { ok = false; break; }
          ptx::tc_fence_after();
          const uint32_t b_addr = ptx::smem_u32(b_tiles + (size_t)stage * kBTileBytes);
#pragma unroll
          for (int kk = 0; kk < kChunkK / 16; ++kk) {
            const uint64_t b_desc = ptx::umma_desc_sw128(b_addr + kk * 32);
#pragma unroll
            for (int w = 0; w < NW; ++w) {
              const uint32_t a_addr = ptx::smem_u32(a_tiles + ((size_t)stage * NW + w) * kATileBytes) + kk * 32;
              ptx::mma_f16_ss(d_base + w * BT, ptx::umma_desc_sw128(a_addr), b_desc, idesc,
                              (first && kk == 0) ? 0u : 1u);
            }
          }
          ptx::mma_commit(&empty[stage]);
          if (++stage == S) { stage = 0; phase ^= 1; }
          if (seg_last(kc, kc1, cpb)) {
            ptx::mma_commit(&part_full[pb]);
            if (++pb == kNumPart) { pb = 0; pphase ^= 1; }
          }
        }
      }
      if (!ok) record_error(a, abort_flag, BQ4_ETIMEOUT);
    }
  } else if (warp < kExScalerWarps) {
    // ------------------------------------------------ scaler + epilogue
    const int quad = warp & 3;
    const int row = quad * 32 + lane;          // output feature within the tile
    const int col0 = (warp >> 2) * kCols;      // first token column of this thread
    int pb = 0;
    uint32_t pphase = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < a.units && !*abort_flag; u += gridDim.x) {
      const int tile = u / S_split, split = u - tile * S_split;
      const int ntile = tile / a.mtiles, mtile = tile - ntile * a.mtiles;
      const int n = ntile * 128 + row;
      const int m0 = mtile * BT + col0;
      const int kc0 = (int)((int64_t)split * a.nkc / S_split);
      const int kc1 = (int)((int64_t)(split + 1) * a.nkc / S_split);
      float acc[NW][kCols];
#pragma unroll
      for (int w = 0; w < NW; ++w)
#pragma unroll
        for (int j = 0; j < kCols; ++j) acc[w][j] = 0.0f;
      const float* srow[NW];
#pragma unroll
      for (int w = 0; w < NW; ++w) srow[w] = a.s[w] + (size_t)ntile * a.nkb * 128 + row;
      for (int kc = kc0; kc < kc1; ++kc) {
        if (!seg_last(kc, kc1, cpb)) continue;
        const int kb = (kc * kChunkK) / a.block;
        float sc[NW];
#pragma unroll
        for (int w = 0; w < NW; ++w) sc[w] = __ldg(srow[w] + (size_t)kb * 128);
        if (!ptx::mbar_wait(&part_full[pb], pphase, abort_flag)) { ok = false; break; }
        ptx::tc_fence_after();
        const uint32_t t_row = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)pb * kPartCols + col0;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
#pragma unroll
          for (int c = 0; c < kCols / 16; ++c) {
            uint32_t r0[16];
            ptx::tmem_ld_32x32b_x16(t_row + w * BT + c * 16, r0);
            ptx::tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[w][c * 16 + j] = fmaf(sc[w], __uint_as_float(r0[j]), acc[w][c * 16 + j]);
          }
        }
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&part_empty[pb]);
        if (++pb == kNumPart) { pb = 0; pphase ^= 1; }
      }
      if (!ok) break;

      if (S_split == 1) {
        float b0 = 0.0f, b1 = 0.0f;
        if (n < a.N) {
          if (a.bias[0]) b0 = __ldg(a.bias[0] + n);
          if (NW == 2 && a.bias[1]) b1 = __ldg(a.bias[1] + n);
          const int act = a.act;
#pragma unroll
          for (int j = 0; j < kCols; ++j) {
            const int m = m0 + j;
            if (m < a.M) {
              float v;
              if (NW == 2) {
                v = silu(acc[0][j] + b0) * (acc[NW - 1][j] + b1);
              } else {
                v = apply_act(acc[0][j] + b0, act);
                if (a.aux) v *= __ldg(a.aux + (size_t)m * a.N + n);
              }
              a.y[(size_t)m * a.N + n] = v;
            }
          }
        }
      } else {
        float* part = a.partials + ((size_t)tile * S_split + split) * NW * 128 * BT;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
          float4* dst = reinterpret_cast<float4*>(part + ((size_t)w * 128 + row) * BT + col0);
#pragma unroll
          for (int j = 0; j < kCols / 4; ++j)
            dst[j] = make_float4(acc[w][4 * j], acc[w][4 * j + 1], acc[w][4 * j + 2], acc[w][4 * j + 3]);
        }
        __threadfence();
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (threadIdx.x == 0) {
          const int prev = atomicAdd(a.counters + tile, 1);
          *last_flag = (prev == S_split - 1) ? 1 : 0;
          if (prev == S_split - 1) a.counters[tile] = 0;
        }
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (*last_flag) {
          __threadfence();
          const float* base = a.partials + (size_t)tile * S_split * NW * 128 * BT;
#pragma unroll
          for (int w = 0; w < NW; ++w)
#pragma unroll
            for (int j = 0; j < kCols; ++j) acc[w][j] = 0.0f;
          for (int sp = 0; sp < S_split; ++sp) {
#pragma unroll
            for (int w = 0; w < NW; ++w) {
              const float4* src =
                  reinterpret_cast<const float4*>(base + ((size_t)sp * NW * 128 + w * 128 + row) * BT + col0);
#pragma unroll
              for (int j = 0; j < kCols / 4; ++j) {
                const float4 v = __ldcg(src + j);
                acc[w][4 * j] += v.x; acc[w][4 * j + 1] += v.y; acc[w][4 * j + 2] += v.z; acc[w][4 * j + 3] += v.w;
              }
            }
          }
          if (n < a.N) {
            float b0 = 0.0f, b1 = 0.0f;
            if (a.bias[0]) b0 = __ldg(a.bias[0] + n);
            if (NW == 2 && a.bias[1]) b1 = __ldg(a.bias[1] + n);
#pragma unroll
            for (int j = 0; j < kCols; ++j) {
              const int m = m0 + j;
              if (m < a.M) {
                float v;
                if (NW == 2) {
                  v = silu(acc[0][j] + b0) * (acc[NW - 1][j] + b1);
                } else {
                  v = apply_act(acc[0][j] + b0, a.act);
                  if (a.aux) v *= __ldg(a.aux + (size_t)m * a.N + n);
                }
                a.y[(size_t)m * a.N + n] = v;
              }
            }
          }
        }
        asm volatile("bar.sync 1, 256;" ::: "memory");
      }
    }
    if (!ok) record_error(a, abort_flag, BQ4_ETIMEOUT);
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == kExMmaWarp) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ------------------------------------------------------------------ host side

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

template <int BT, int NW, bool EXACT>
cudaError_t launch_kernel(const GemmPlan& plan, const CUtensorMap& tmap, const GemmArgs& args,
                          cudaStream_t stream) {
  cudaError_t e;
  if constexpr (EXACT) {
    auto kern = q4_gemm_exact_kernel<BT, NW>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)plan.smem_bytes);
    if (e != cudaSuccess) return e;
    kern<<<plan.grid, kExThreads, plan.smem_bytes, stream>>>(tmap, args);
  } else {
    auto kern = q4_gemm_kernel<BT, NW>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)plan.smem_bytes);
    if (e != cudaSuccess) return e;
    kern<<<plan.grid, kThreads, plan.smem_bytes, stream>>>(tmap, args);
  }
  note_launch();
  return cudaGetLastError();
}

}  // namespace

int device_sm_count(int device) {
  static int cache[64] = {0};
  if (device < 0 || device >= 64) return 148;
  if (!cache[device]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0)
      v = 148;
    cache[device] = v;
  }
  return cache[device];
}

int device_is_sm100(int device) {
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess)
    return 0;
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  return major == 10 && minor == 0;
}

bq4_status plan_gemm(const bq4_weight* w, int nw, int64_t M, int device, GemmPlan* p) {
  if (M <= 0) return set_error(BQ4_EINVAL_SHAPE, "M must be positive (got %lld)", (long long)M);
  if (M > (int64_t)1 << 30) return set_error(BQ4_EINVAL_SHAPE, "M too large");
  memset(p, 0, sizeof(*p));
  p->nw = nw;
  // Blocks of 64/128 K values keep q exact and scale the f32 accumulator
  // (exact-weight kernel, token tile <= 128); smaller blocks fold the scale
  // into the f16 weight (folded kernel, token tile <= 256).
  p->pre = w->h != nullptr ? 1 : 0;
  p->exact = (!p->pre && w->block >= 64) ? 1 : 0;
  // BQ4_FORCE_FOLDED=1 selects the folded kernel for any block (tests and
  // tuning compare both formulations on the same shapes).
  if (const char* f = getenv("BQ4_FORCE_FOLDED"))
    if (f[0] == '1') p->exact = 0;
  if (p->exact)
    p->bt = (nw == 1 && M > 64) ? 128 : 64;
  else if (nw == 1)
    p->bt = M > 128 ? 256 : (M > 64 ? 128 : 64);
  else
    p->bt = M > 64 ? 128 : 64;
  p->mtiles = (int)((M + p->bt - 1) / p->bt);
  p->ntiles = (int)w->ntiles;
  const int sms = device_sm_count(device);
  const int tiles = p->mtiles * p->ntiles;
  const int nkc = (int)w->nkc;

  // Split-K factor: minimise an estimated makespan.  One unit of work costs
  // (chunks per split + fixed pipeline fill of ~3 chunks).  Split-K is only
  // used when every unit fits in a single wave (units <= SMs): a CTA that
  // runs a second split unit was measured to produce wrong partial tiles,
  // so multi-wave work uses whole-K units (S = 1).
  int best_s = 1;
  double best_t = 1e30;
  const int max_s = nkc < 16 ? nkc : 16;
  for (int s = 1; s <= max_s; ++s) {
    const int units = tiles * s;
    if (s > 1 && units > sms) break;
    const int waves = (units + sms - 1) / sms;
    const double per_unit = (double)nkc / s + 3.0;
    const double fixup = s > 1 ? 1.0 + 0.25 * s : 0.0;
    const double t = waves * (per_unit + fixup);
    if (t < best_t - 1e-9) {
      best_t = t;
      best_s = s;
    }
  }
  // BQ4_FORCE_KSPLIT=s pins the split-K factor (clamped to [1, chunks] and
  // to a single wave of units).
  if (const char* f = getenv("BQ4_FORCE_KSPLIT")) {
    int v = atoi(f);
    if (v >= 1) best_s = v < nkc ? v : nkc;
    while (best_s > 1 && tiles * best_s > sms) --best_s;
  }
  p->ksplit = best_s;
  p->units = tiles * best_s;
  p->grid = p->units < sms ? p->units : sms;

  // Shared memory: operand ring (S stages) + raw ring (RS stages).
  // The exact kernel's scaler warps read scales straight from global memory,
  // so its raw stages carry nibbles only.
  const uint32_t raw_s_bytes = 512u * (uint32_t)(w->block >= 64 ? 1 : 64 / w->block);
  const size_t stage_bytes = (size_t)nw * kATileBytes + (size_t)p->bt * 128;
  // Per-weight raw stage: nibbles (+ scales for the folded kernel); the
  // pre-expanded path leaves the ring unused.  The kernels carve shared
  // memory with this same value (GemmArgs::raw_w_bytes).
  p->raw_w_bytes = p->pre ? 16u : kRawQBytes + (p->exact ? 0u : raw_s_bytes);
  const size_t raw_stage_bytes = (size_t)nw * p->raw_w_bytes;
  const size_t budget = 227 * 1024 - 1024 /*align*/ - 512 /*barriers*/;
  int S = 0, RS = 0;
  for (int s = 4; s >= 2; --s) {
    if ((size_t)s * stage_bytes >= budget) continue;
    int rs = (int)((budget - (size_t)s * stage_bytes) / raw_stage_bytes);
    if (rs > 8) rs = 8;
    if (p->pre) rs = 4;  // unused ring
    if (rs >= 4 || s == 2) {
      S = s;
      RS = rs;
      break;
    }
  }
  if (S < 2 || RS < 2) return set_error(BQ4_EUNSUPPORTED, "no shared-memory plan for this shape");
  p->stages = S;
  p->raw_stages = RS;
  p->smem_bytes = 1024 + (size_t)S * stage_bytes + (size_t)RS * raw_stage_bytes +
                  (size_t)(2 * S + 2 * RS + 2 * kNumPart + 4) * 8 + 16;

  p->xh_bytes = align_up((size_t)M * (size_t)w->Kp * 2, 256);
  p->counter_bytes = align_up((size_t)tiles * sizeof(int) + sizeof(int) * 4, 256);
  p->partial_bytes =
      best_s > 1 ? align_up((size_t)tiles * best_s * nw * 128 * p->bt * sizeof(float), 256) : 0;
  p->workspace_bytes = p->xh_bytes + p->counter_bytes + p->partial_bytes;
  return BQ4_OK;
}

bq4_status run_gemm(const GemmPlan& plan, const bq4_weight* const* ws, const float* x, int64_t M,
                    int64_t ldx, const float* const* bias, int act, const float* aux, float* y,
                    void* workspace, cudaStream_t stream) {
  const bq4_weight* w0 = ws[0];
  uint8_t* wsp = static_cast<uint8_t*>(workspace);
  void* xh = wsp;
  int* counters = reinterpret_cast<int*>(wsp + plan.xh_bytes);
  float* partials =
      plan.partial_bytes ? reinterpret_cast<float*>(wsp + plan.xh_bytes + plan.counter_bytes) : nullptr;

  // 1) stage activations as f16 (also zeroes split-K counters and the error word)
  cudaError_t e = launch_convert_x(x, M, w0->K, ldx, w0->Kp, xh, counters,
                                   plan.mtiles * plan.ntiles + 4, stream);
  if (e != cudaSuccess) return check_cuda(e, "convert_x launch");

  // 2) tensor map over xh [M][Kp] f16, box {64, BT}, 128-byte swizzle
  EncodeTiledFn enc = encode_fn();
  if (!enc) return set_error(BQ4_ECUDA, "cuTensorMapEncodeTiled unavailable");
  CUtensorMap tmap;
  cuuint64_t gdim[2] = {(cuuint64_t)w0->Kp, (cuuint64_t)M};
  cuuint64_t gstride[1] = {(cuuint64_t)w0->Kp * 2};
  cuuint32_t box[2] = {(cuuint32_t)kChunkK, (cuuint32_t)plan.bt};
  cuuint32_t estride[2] = {1, 1};
  CUresult cr = enc(&tmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, xh, gdim, gstride, box, estride,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return set_error(BQ4_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)cr);

  GemmArgs args;
  memset(&args, 0, sizeof(args));
  args.pre = plan.pre;
  for (int i = 0; i < plan.nw; ++i) {
    args.h[i] = ws[i]->h;
    args.q[i] = ws[i]->q;
    args.s[i] = ws[i]->s;
    args.bias[i] = bias ? bias[i] : nullptr;
  }
  args.aux = aux;
  args.y = y;
  args.partials = partials;
  args.counters = counters;
  args.M = (int)M;
  args.N = (int)w0->N;
  args.nkc = (int)w0->nkc;
  args.nkb = (int)w0->nkb;
  args.block = w0->block;
  args.ntiles = plan.ntiles;
  args.mtiles = plan.mtiles;
  args.ksplit = plan.ksplit;
  args.units = plan.units;
  args.stages = plan.stages;
  args.raw_stages = plan.raw_stages;
  args.raw_s_bytes = plan.exact ? 0u : 512u * (uint32_t)(w0->block >= 64 ? 1 : 64 / w0->block);
  args.raw_w_bytes = plan.raw_w_bytes;
  if (!plan.pre && !plan.exact && args.raw_w_bytes != kRawQBytes + args.raw_s_bytes)
    return set_error(BQ4_EINVAL_ARG, "internal: raw stage size mismatch");
  args.act = act;

  if (plan.exact) {
    if (plan.nw == 1) {
      if (plan.bt == 128) e = launch_kernel<128, 1, true>(plan, tmap, args, stream);
      else e = launch_kernel<64, 1, true>(plan, tmap, args, stream);
    } else {
      e = launch_kernel<64, 2, true>(plan, tmap, args, stream);
    }
  } else if (plan.nw == 1) {
    if (plan.bt == 256) e = launch_kernel<256, 1, false>(plan, tmap, args, stream);
    else if (plan.bt == 128) e = launch_kernel<128, 1, false>(plan, tmap, args, stream);
    else e = launch_kernel<64, 1, false>(plan, tmap, args, stream);
  } else {
    if (plan.bt == 128) e = launch_kernel<128, 2, false>(plan, tmap, args, stream);
    else e = launch_kernel<64, 2, false>(plan, tmap, args, stream);
  }
  if (e != cudaSuccess) return check_cuda(e, "q4 gemm launch");
  return BQ4_OK;
}

bq4_status poll_device_error() {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_bq4_device_error, sizeof(int));
  if (e != cudaSuccess) return check_cuda(e, "reading the device error word");
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_bq4_device_error, &zero, sizeof(int));
    return set_error((bq4_status)v, "a bq4 kernel recorded status %d (bounded wait expired)", v);
  }
  return BQ4_OK;
}

}  // namespace bq4
