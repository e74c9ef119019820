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

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "bq4_internal.h"
#include "sm100_ptx.cuh"

namespace bq4 {
namespace {

constexpr uint32_t kATileBytes = 128 * 128;  // 128 rows x 64 f16
constexpr uint32_t kRawQBytes = 4096;        // 128 rows x 64 nibbles

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

// Expand one prepared word into 8 exact f16 values q (no scale): the
// exact-weight formulation multiplies the f32 partial of each K block by
// the scale instead.
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

__device__ __forceinline__ void record_error_flag(volatile int* abort_flag, int code) {
  if (!*abort_flag) {
    *abort_flag = 1;
    atomicCAS(&g_bq4_device_error, 0, code);
  }
}

// ---------------------------------------------------------------------------
// Unified warp-specialized kernel (both numerics modes).
//
// The MMA issuer is a single thread, and every mbarrier wait and
// tcgen05.commit on its path costs hundreds of cycles; the pipeline is
// therefore organised so that it waits and commits once per 128-K stage
// (8 MMAs of 128 x BT x 16 per weight):
//   operand ring (S stages): per stage, A = NW x two 64-K sub-tiles of the
//     MMA-ready weight tile [128 rows][64] f16 (written by the dequant warps,
//     or bulk-copied pre-expanded tiles) and B = two 64-K token sub-tiles
//     [BT][64] f16 (TMA), all with the 128-byte swizzle; one full and one
//     empty mbarrier per stage.
//   raw ring (RS stages): the prepared nibbles of a stage (2 x 4 KiB per
//     weight, + scales in folded mode), by 1-D bulk copy.
// TMEM: NP partial accumulators of NW*BT columns.  A unit's K range is cut
// into segments (one K block of 64/128 in exact mode; the whole unit in
// folded mode); the MMA accumulates a segment into one partial buffer and
// the scaler warps fold it into f32 registers: acc += scale * partial
// (scale = 1 in folded mode).  The epilogue runs from those registers.
// Lockstep variant (exact mode, 128-blocks, 2 stages and 2 partials): a
// segment is exactly one stage and uses the partial buffer of the same
// index, so the scaler waits on the stage's `empty` barrier (its MMAs have
// retired) and announces "partial free" by arriving on the `full` barrier
// of that stage's next use; the issuer then needs no separate partial
// handshakes -- one wait and one commit per stage, as in folded mode.
//
// Warps (896 threads, 7 warpgroups, registers rebalanced with setmaxnreg):
//   WG0-3 (warps 0-15)  scaler + epilogue, 96 regs: warp w reads TMEM lanes
//                       32*(w%4).. and the token-column quarter w/4.
//   WG4-5 (warps 16-23) dequant, 48 regs: thread t handles row t%128 of
//                       64-K sub-tile t/128 (8 words) of each stage.
//   WG6   (warps 24-27) 24 token TMA, 25 weight producer, 26 MMA issuer /
//                       TMEM owner, 27 idle; 24 regs.
// ---------------------------------------------------------------------------
constexpr int kWsThreads = 896;
constexpr int kWsRegsLaunch = 72;       // 65536 / 896, rounded down to 8
constexpr int kWsRegsScaler = 96;       // 4*96 + 2*48 + 24 = 504 = 7*72
constexpr int kWsRegsDequant = 48;
constexpr int kWsRegsProducer = 24;
constexpr int kWsTmaWarp = 24, kWsWeightWarp = 25, kWsMmaWarp = 26;
constexpr int kWsDqWarp0 = 16, kWsDqWarps = 8, kWsScalerWarps = 16;
constexpr uint32_t kRawStageQBytes = 2 * kRawQBytes;  // nibbles of one 128-K stage

struct WsArgs {
  const uint32_t* q[2];
  const float* s[2];
  const uint16_t* h[2];
  const float* bias[2];
  const float* aux;
  float* y;
  float* partials;
  int* counters;
  int M, N;
  int nkc, nkb, block;
  int ntiles, mtiles, ksplit, units;
  int stages, rs;          // operand ring and raw ring depths
  int exact, pre, act;
  int lockstep;            // exact, 128-blocks, 2 stages == 2 TMEM partials (see below)
  uint32_t raw_s_bytes;    // folded: scale bytes per weight per raw stage
  uint32_t raw_w_bytes;    // raw stage bytes per weight
};

// Unit u -> (tile, split) and its chunk range [kc0, kc1); splits cut at
// stage (2-chunk) boundaries.
__device__ __forceinline__ void ws_unit(const WsArgs& a, int u, int& tile, int& split, int& kc0, int& kc1) {
  tile = u / a.ksplit;
  split = u - tile * a.ksplit;
  const int nks = a.nkc >> 1;
  kc0 = 2 * (int)((int64_t)split * nks / a.ksplit);
  kc1 = 2 * (int)((int64_t)(split + 1) * nks / a.ksplit);
}

// Segment boundaries inside [kc0, kc1): exact mode cuts at K-block edges
// (cpb chunks per block); folded mode keeps the unit whole (cpb = 0).
__device__ __forceinline__ bool ws_seg_first(int kc, int kc0, int cpb) {
  return kc == kc0 || (cpb > 0 && (kc % cpb) == 0);
}
__device__ __forceinline__ bool ws_seg_last(int kc, int kc1, int cpb) {
  return kc == kc1 - 1 || (cpb > 0 && ((kc + 1) % cpb) == 0);
}

template <int BT, int NW>
__global__ void __launch_bounds__(kWsThreads, 1)
    q4_gemm_ws_kernel(const __grid_constant__ CUtensorMap tmap_x, const WsArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  constexpr uint32_t kBSub = BT * 128;              // one 64-K token sub-tile
  constexpr uint32_t kAStage = NW * 2 * kATileBytes;
  constexpr uint32_t kStage = kAStage + 2 * kBSub;
  constexpr uint32_t kPartCols = NW * BT;
  constexpr int kNP = 512 / kPartCols;   // partial buffers in TMEM
  constexpr int kCols = BT / 4;          // token columns per scaler thread
  static_assert(kNP >= 2, "at least double buffering");
  static_assert(kCols % 16 == 0, "scaler column split");

  const int S = a.stages, RS = a.rs;
  uint8_t* ring = smem;                                     // [S][A | B]
  uint8_t* raw_ring = ring + (size_t)S * kStage;            // [RS][NW][raw_w_bytes]
  uint64_t* bars = reinterpret_cast<uint64_t*>(raw_ring + (size_t)RS * NW * a.raw_w_bytes);
  uint64_t* full = bars;
  uint64_t* empty = full + S;
  uint64_t* raw_full = empty + S;
  uint64_t* raw_empty = raw_full + RS;
  uint64_t* part_full = raw_empty + RS;
  uint64_t* part_empty = part_full + kNP;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(part_empty + kNP);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = abort_flag + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cpb = a.exact ? a.block / kChunkK : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      // TMA expect_tx (+ dequant warps) (+ scaler warps in lockstep mode)
      ptx::mbar_init(&full[i], (a.pre ? 1 : 1 + kWsDqWarps) + (a.lockstep ? kWsScalerWarps : 0));
      ptx::mbar_init(&empty[i], 1);  // tcgen05.commit
    }
    for (int i = 0; i < RS; ++i) { ptx::mbar_init(&raw_full[i], 1); ptx::mbar_init(&raw_empty[i], kWsDqWarps); }
    for (int i = 0; i < kNP; ++i) { ptx::mbar_init(&part_full[i], 1); ptx::mbar_init(&part_empty[i], kWsScalerWarps); }
    *abort_flag = 0;
    *last_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == kWsTmaWarp && lane == 0) ptx::prefetch_tmap(&tmap_x);
  if (warp == kWsMmaWarp) {
    ptx::tmem_alloc(tmem_slot, 512);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp >= kWsTmaWarp) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kWsRegsProducer));
    if (warp == kWsTmaWarp && lane == 0) {
      // ------------------------------------------------ token tiles (+ pre-expanded A)
      int s = 0;
      uint32_t ph = 0;
      for (int u = blockIdx.x; u < a.units && !*abort_flag; u += gridDim.x) {
        int tile, split, kc0, kc1;
        ws_unit(a, u, tile, split, kc0, kc1);
        const int mtile = tile % a.mtiles, ntile = tile / a.mtiles;
        for (int kc = kc0; kc < kc1; kc += 2) {
          if (!ptx::mbar_wait(&empty[s], ph ^ 1, abort_flag)) {
            record_error_flag(abort_flag, BQ4_ETIMEOUT);
            break;
          }
          uint8_t* st = ring + (size_t)s * kStage;
          ptx::mbar_arrive_expect_tx(&full[s], 2 * kBSub + (a.pre ? kAStage : 0u));
          ptx::tma_load_2d(st + kAStage, &tmap_x, &full[s], kc * kChunkK, mtile * BT);
          ptx::tma_load_2d(st + kAStage + kBSub, &tmap_x, &full[s], (kc + 1) * kChunkK, mtile * BT);
          if (a.pre) {
#pragma unroll
            for (int w = 0; w < NW; ++w)
              ptx::bulk_load(st + (size_t)w * 2 * kATileBytes,
                             a.h[w] + ((size_t)ntile * a.nkc + kc) * (kATileBytes / 2), 2 * kATileBytes, &full[s]);
          }
          if (++s == S) { s = 0; ph ^= 1; }
        }
      }
    } else if (warp == kWsWeightWarp && lane == 0 && !a.pre) {
      // ------------------------------------------------ raw weight tiles (bulk copies)
      int rs = 0;
      uint32_t rph = 0;
      for (int u = blockIdx.x; u < a.units && !*abort_flag; u += gridDim.x) {
        int tile, split, kc0, kc1;
        ws_unit(a, u, tile, split, kc0, kc1);
        const int ntile = tile / a.mtiles;
        for (int kc = kc0; kc < kc1; kc += 2) {
          if (!ptx::mbar_wait(&raw_empty[rs], rph ^ 1, abort_flag)) {
            record_error_flag(abort_flag, BQ4_ETIMEOUT);
            break;
          }
          ptx::mbar_arrive_expect_tx(&raw_full[rs], NW * (kRawStageQBytes + a.raw_s_bytes));
          const int kb0 = (kc * kChunkK) / a.block;
#pragma unroll
          for (int w = 0; w < NW; ++w) {
            uint8_t* dst = raw_ring + ((size_t)rs * NW + w) * a.raw_w_bytes;
            ptx::bulk_load(dst, a.q[w] + ((size_t)ntile * a.nkc + kc) * 1024, kRawStageQBytes, &raw_full[rs]);
            if (a.raw_s_bytes)
              ptx::bulk_load(dst + kRawStageQBytes, a.s[w] + ((size_t)ntile * a.nkb + kb0) * 128, a.raw_s_bytes,
                             &raw_full[rs]);
          }
          if (++rs == RS) { rs = 0; rph ^= 1; }
        }
      }
    } else if (warp == kWsMmaWarp && lane == 0) {
      // ------------------------------------------------ MMA issuer
      constexpr uint32_t idesc = ptx::umma_idesc_f16(128, BT);
      int s = 0, pb = 0;
      uint32_t ph = 0, pph = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < a.units && !*abort_flag; u += gridDim.x) {
        int tile, split, kc0, kc1;
        ws_unit(a, u, tile, split, kc0, kc1);
        uint32_t d_base = 0;
        for (int kc = kc0; ok && kc < kc1; kc += 2) {
          if (!ptx::mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
          ptx::tc_fence_after();
          const uint32_t st = ptx::smem_u32(ring + (size_t)s * kStage);
#pragma unroll
          for (int sub = 0; sub < 2; ++sub) {
            const int c = kc + sub;
            const bool first = ws_seg_first(c, kc0, cpb);
            if (first) {
              if (a.lockstep) {
                d_base = tmem_base + (uint32_t)s * kPartCols;  // freed via full[s]
              } else {
                if (!ptx::mbar_wait(&part_empty[pb], pph ^ 1, abort_flag)) { ok = false; break; }
                ptx::tc_fence_after();
                d_base = tmem_base + (uint32_t)pb * kPartCols;
              }
            }
            const uint32_t b_addr = st + kAStage + sub * kBSub;
#pragma unroll
            for (int kk = 0; kk < kChunkK / 16; ++kk) {
              const uint64_t b_desc = ptx::umma_desc_sw128(b_addr + kk * 32);
#pragma unroll
              for (int w = 0; w < NW; ++w)
                ptx::mma_f16_ss(d_base + w * BT,
                                ptx::umma_desc_sw128(st + (uint32_t)((w * 2 + sub) * kATileBytes) + kk * 32), b_desc,
                                idesc, (first && kk == 0) ? 0u : 1u);
            }
            if (sub == 1) ptx::mma_commit(&empty[s]);  // stage free once its MMAs retire
            if (!a.lockstep && ws_seg_last(c, kc1, cpb)) {
              ptx::mma_commit(&part_full[pb]);
              if (++pb == kNP) { pb = 0; pph ^= 1; }
            }
          }
          if (++s == S) { s = 0; ph ^= 1; }
        }
      }
      if (!ok) record_error_flag(abort_flag, BQ4_ETIMEOUT);
    }
  } else if (warp >= kWsDqWarp0) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kWsRegsDequant));
    if (!a.pre) {
      // ------------------------------------------------ dequant
      const int t = threadIdx.x - kWsDqWarp0 * 32;
      const int r = t & 127;
      const int sub = t >> 7;  // which 64-K sub-tile of the stage
      const int sw = r & 7;
      const int block = a.block;
      int rs = 0, s = 0;
      uint32_t rph = 0, ph = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < a.units && !*abort_flag; u += gridDim.x) {
        int tile, split, kc0, kc1;
        ws_unit(a, u, tile, split, kc0, kc1);
        for (int kc = kc0; kc < kc1; kc += 2) {
          if (!ptx::mbar_wait(&raw_full[rs], rph, abort_flag)) { ok = false; break; }
          uint4 wlo[NW], whi[NW];
          uint32_t sc[NW][8];
#pragma unroll
          for (int w = 0; w < NW; ++w) {
            const uint8_t* src = raw_ring + ((size_t)rs * NW + w) * a.raw_w_bytes + (size_t)sub * kRawQBytes;
            wlo[w] = *reinterpret_cast<const uint4*>(src + (size_t)r * 16);
            whi[w] = *reinterpret_cast<const uint4*>(src + (size_t)(128 + r) * 16);
            if (!a.exact) {
              const float* ss = reinterpret_cast<const float*>(raw_ring + ((size_t)rs * NW + w) * a.raw_w_bytes +
                                                               kRawStageQBytes);
              if (block >= 128) {
                const uint32_t s2 = scale_to_f16x2(ss[r]);
#pragma unroll
                for (int j = 0; j < 8; ++j) sc[w][j] = s2;
              } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) sc[w][j] = scale_to_f16x2(ss[((sub * 64 + j * 8) / block) * 128 + r]);
              }
            }
          }
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(&raw_empty[rs]);
          if (++rs == RS) { rs = 0; rph ^= 1; }
          if (!ptx::mbar_wait(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
#pragma unroll
          for (int w = 0; w < NW; ++w) {
            uint8_t* dst = ring + (size_t)s * kStage + (size_t)(w * 2 + sub) * kATileBytes + (size_t)r * 128;
            const uint32_t wv[8] = {wlo[w].x, wlo[w].y, wlo[w].z, wlo[w].w, whi[w].x, whi[w].y, whi[w].z, whi[w].w};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint4 v = a.exact ? expand_word_exact(wv[j]) : expand_word(wv[j], sc[w][j]);
              *reinterpret_cast<uint4*>(dst + ((j ^ sw) << 4)) = v;
            }
          }
          ptx::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(&full[s]);
          if (++s == S) { s = 0; ph ^= 1; }
        }
      }
      if (!ok) record_error_flag(abort_flag, BQ4_ETIMEOUT);
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kWsRegsScaler));
    // ------------------------------------------------ scaler + epilogue
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int col0 = (warp >> 2) * kCols;
    int pb = 0;
    uint32_t pph = 0;
    bool ok = true;
    if (a.lockstep && lane == 0) {
      // both partial buffers start free: the first use of each stage
      for (int i = 0; i < S; ++i) ptx::mbar_arrive(&full[i]);
    }
    for (int u = blockIdx.x; ok && u < a.units && !*abort_flag; u += gridDim.x) {
      int tile, split, kc0, kc1;
      ws_unit(a, u, tile, split, kc0, kc1);
      const int ntile = tile / a.mtiles, mtile = tile - ntile * a.mtiles;
      const int n = ntile * 128 + row;
      const int m0 = mtile * BT + col0;
      float acc[NW][kCols];
#pragma unroll
      for (int w = 0; w < NW; ++w)
#pragma unroll
        for (int j = 0; j < kCols; ++j) acc[w][j] = 0.0f;
      for (int kc = kc0; kc < kc1; ++kc) {
        if (!ws_seg_last(kc, kc1, cpb)) continue;
        float sc[NW];
#pragma unroll
        for (int w = 0; w < NW; ++w)
          sc[w] = a.exact ? __ldg(a.s[w] + ((size_t)ntile * a.nkb + (kc * kChunkK) / a.block) * 128 + row) : 1.0f;
        // lockstep: segment == stage pb (S == NP), retired when empty[pb] completes
        if (!ptx::mbar_wait(a.lockstep ? &empty[pb] : &part_full[pb], pph, abort_flag)) { ok = false; break; }
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
        if (lane == 0) ptx::mbar_arrive(a.lockstep ? &full[pb] : &part_empty[pb]);
        if (++pb == kNP) { pb = 0; pph ^= 1; }
      }
      if (!ok) break;

      const int SPL = a.ksplit;
      if (SPL > 1) {
        // Split-K: publish this split's partial, the last split sums all of
        // them in split order (deterministic) and runs the epilogue.
        float* part = a.partials + ((size_t)tile * SPL + split) * NW * 128 * BT;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
          float4* dst = reinterpret_cast<float4*>(part + ((size_t)w * 128 + row) * BT + col0);
#pragma unroll
          for (int j = 0; j < kCols / 4; ++j)
            __stcg(dst + j, make_float4(acc[w][4 * j], acc[w][4 * j + 1], acc[w][4 * j + 2], acc[w][4 * j + 3]));
        }
        __threadfence();
        asm volatile("bar.sync 1, 512;" ::: "memory");
        if (threadIdx.x == 0) {
          __threadfence();
          const int prev = atomicAdd(a.counters + tile, 1);
          *last_flag = (prev == SPL - 1) ? 1 : 0;
          if (prev == SPL - 1) a.counters[tile] = 0;
        }
        asm volatile("bar.sync 1, 512;" ::: "memory");
        const bool last = *last_flag != 0;
        asm volatile("bar.sync 1, 512;" ::: "memory");
        if (!last) continue;
        __threadfence();
        const float* base = a.partials + (size_t)tile * SPL * NW * 128 * BT;
#pragma unroll
        for (int w = 0; w < NW; ++w)
#pragma unroll
          for (int j = 0; j < kCols; ++j) acc[w][j] = 0.0f;
        for (int sp = 0; sp < SPL; ++sp) {
#pragma unroll
          for (int w = 0; w < NW; ++w) {
            const float4* src = reinterpret_cast<const float4*>(base + ((size_t)(sp * NW + w) * 128 + row) * BT + col0);
#pragma unroll
            for (int j = 0; j < kCols / 4; ++j) {
              const float4 v = __ldcg(src + j);
              acc[w][4 * j] += v.x; acc[w][4 * j + 1] += v.y; acc[w][4 * j + 2] += v.z; acc[w][4 * j + 3] += v.w;
            }
          }
        }
      }
      if (n < a.N) {
        const float b0 = a.bias[0] ? __ldg(a.bias[0] + n) : 0.0f;
        const float b1 = (NW == 2 && a.bias[1]) ? __ldg(a.bias[1] + n) : 0.0f;
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
    }
    if (!ok) record_error_flag(abort_flag, BQ4_ETIMEOUT);
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == kWsMmaWarp) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, 512);
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

// The kernel rebalances registers with setmaxnreg; the split only fits the
// pool the block was launched with when ptxas gave every thread exactly
// kWsRegsLaunch registers.  Checked once per instantiation before any launch
// (a mismatch would make setmaxnreg.inc wait forever).
template <int BT, int NW>
cudaError_t prepare_ws_kernel(size_t smem_bytes, bool* ok_regs) {
  auto kern = q4_gemm_ws_kernel<BT, NW>;
  static int checked = 0;  // 0 unknown, 1 ok, -1 bad
  if (checked == 0) {
    cudaFuncAttributes attr;
    cudaError_t e = cudaFuncGetAttributes(&attr, kern);
    if (e != cudaSuccess) return e;
    checked = (attr.numRegs == kWsRegsLaunch) ? 1 : -1;
  }
  *ok_regs = checked == 1;
  static size_t smem_set = 0;
  if (smem_set < smem_bytes) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes);
    if (e != cudaSuccess) return e;
    smem_set = smem_bytes;
  }
  return cudaSuccess;
}

template <int BT, int NW>
cudaError_t launch_ws(const GemmPlan& plan, const CUtensorMap& tmap, const WsArgs& args, cudaStream_t stream,
                      bool* ok_regs) {
  cudaError_t e = prepare_ws_kernel<BT, NW>(plan.smem_bytes, ok_regs);
  if (e != cudaSuccess || !*ok_regs) return e;
  q4_gemm_ws_kernel<BT, NW><<<plan.grid, kWsThreads, plan.smem_bytes, stream>>>(tmap, args);
  note_launch();
  return cudaGetLastError();
}

}  // namespace

namespace {
std::atomic<int> g_numerics{-1};
}

int numerics_mode() {
  int v = g_numerics.load(std::memory_order_relaxed);
  if (v < 0) {
    v = BQ4_NUMERICS_AUTO;
    if (const char* e = getenv("BQ4_NUMERICS")) {
      if (!strcmp(e, "exact")) v = BQ4_NUMERICS_EXACT;
      else if (!strcmp(e, "folded")) v = BQ4_NUMERICS_FOLDED;
    }
    int expected = -1;
    g_numerics.compare_exchange_strong(expected, v);
    v = g_numerics.load(std::memory_order_relaxed);
  }
  return v;
}

void set_numerics_mode(int mode) { g_numerics.store(mode, std::memory_order_relaxed); }

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
  // Numerics: blocks of 64/128 keep q exact in f16 and multiply the f32
  // partial of each K block by its scale (exact weights); smaller blocks
  // stage f16(q * f16(scale)) (folded); N-packed sources are pre-expanded.
  p->pre = w->h != nullptr ? 1 : 0;
  const int mode = numerics_mode();
  p->exact = (!p->pre && w->block >= 64 &&
              (mode == BQ4_NUMERICS_EXACT || (mode == BQ4_NUMERICS_AUTO && M <= kAutoExactMaxM)))
                 ? 1 : 0;
  // BQ4_FORCE_FOLDED=1 selects folded staging for any block (tests compare
  // both formulations on the same shapes).
  if (const char* f = getenv("BQ4_FORCE_FOLDED"))
    if (f[0] == '1') p->exact = 0;
  if (nw == 1)
    p->bt = M > 128 ? 256 : (M > 64 ? 128 : 64);
  else
    p->bt = M > 64 ? 128 : 64;
  // BQ4_FORCE_BT=64|128|256 pins the token tile (tuning).
  if (const char* f = getenv("BQ4_FORCE_BT")) {
    const int v = atoi(f);
    if (v == 64 || v == 128 || (v == 256 && nw == 1)) p->bt = v;
  }
  p->mtiles = (int)((M + p->bt - 1) / p->bt);
  p->ntiles = (int)w->ntiles;
  const int sms = device_sm_count(device);
  const int tiles = p->mtiles * p->ntiles;
  const int nkc = (int)w->nkc;
  const int nks = nkc / 2;  // 128-K stages

  // Split-K factor: minimise an estimated makespan (chunks per split plus a
  // pipeline fill of ~3 chunks per unit, plus the partial-tile fix-up).
  // Split-K is only used when all units fit in one wave (units <= SMs);
  // multi-wave work uses whole-K units (S = 1).
  int best_s = 1;
  double best_t = 1e30;
  const int max_s = nks < 16 ? nks : 16;
  const bool multiwave_split = getenv("BQ4_ALLOW_MULTIWAVE_SPLIT") != nullptr;
  for (int s = 1; s <= max_s; ++s) {
    const int units = tiles * s;
    if (s > 1 && units > sms && !multiwave_split) break;
    const int waves = (units + sms - 1) / sms;
    const double per_unit = (double)nkc / s + 3.0;  // chunks
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
    if (v >= 1) best_s = v < nks ? v : nks;
    while (best_s > 1 && tiles * best_s > sms && !multiwave_split) --best_s;
  }
  p->ksplit = best_s;
  p->units = tiles * best_s;
  p->grid = p->units < sms ? p->units : sms;

  // Shared memory: operand ring of 128-K stages (A + B) as deep as fits
  // (2..4 stages) next to a raw ring of 2..4 stages.
  const uint32_t raw_s_bytes = 512u * (uint32_t)(w->block >= 128 ? 1 : 128 / w->block);
  p->raw_s_bytes = p->exact || p->pre ? 0u : raw_s_bytes;
  p->raw_w_bytes = p->pre ? 16u : 2 * kRawQBytes + p->raw_s_bytes;
  const size_t stage_bytes = (size_t)nw * 2 * kATileBytes + 2 * (size_t)p->bt * 128;
  const size_t raw_stage = (size_t)nw * p->raw_w_bytes;
  const size_t budget = 227 * 1024 - 1024 /*align*/ - 512 /*barriers*/;
  int S = 0, RS = 0;
  for (int s = 4; s >= 2 && !S; --s) {
    if ((size_t)s * stage_bytes + raw_stage > budget) continue;
    int rs = (int)((budget - (size_t)s * stage_bytes) / raw_stage);
    if (rs > 4) rs = 4;
    if (p->pre) rs = 1;
    S = s;
    RS = rs;
  }
  // BQ4_FORCE_RINGS=S,RS pins the ring depths (tuning); ignored when it
  // does not fit the shared-memory budget.
  if (const char* f = getenv("BQ4_FORCE_RINGS")) {
    int fs = 0, fr = 0;
    if (sscanf(f, "%d,%d", &fs, &fr) == 2 && fs >= 2 && fr >= 1 &&
        (size_t)fs * stage_bytes + (size_t)fr * raw_stage <= budget) {
      S = fs;
      RS = p->pre ? 1 : fr;
    }
  }
  if (S < 2 || RS < 1) return set_error(BQ4_EUNSUPPORTED, "no shared-memory plan for this shape");
  p->stages = S;
  p->a_stages = S;
  p->raw_stages = RS;
  // Lockstep partial handoff: exact 128-blocks, one segment per stage, as
  // many stages as TMEM partial buffers (2).
  p->lockstep = (p->exact && w->block == 128 && S == 2 && 512 / (nw * p->bt) == 2) ? 1 : 0;
  if (getenv("BQ4_NO_LOCKSTEP")) p->lockstep = 0;
  const int np = 512 / (nw * p->bt);
  p->smem_bytes = 1024 + (size_t)S * stage_bytes + (size_t)RS * raw_stage +
                  (size_t)(2 * S + 2 * RS + 2 * np) * 8 + 16;

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

  // 1) stage activations as f16 (also zeroes the split-K tile counters)
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

  WsArgs args;
  memset(&args, 0, sizeof(args));
  for (int i = 0; i < plan.nw; ++i) {
    args.q[i] = ws[i]->q;
    args.s[i] = ws[i]->s;
    args.h[i] = ws[i]->h;
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
  args.rs = plan.raw_stages;
  args.exact = plan.exact;
  args.pre = plan.pre;
  args.lockstep = plan.lockstep;
  args.act = act;
  args.raw_s_bytes = plan.raw_s_bytes;
  args.raw_w_bytes = plan.raw_w_bytes;

  bool ok_regs = true;
  if (plan.nw == 1) {
    if (plan.bt == 256) e = launch_ws<256, 1>(plan, tmap, args, stream, &ok_regs);
    else if (plan.bt == 128) e = launch_ws<128, 1>(plan, tmap, args, stream, &ok_regs);
    else e = launch_ws<64, 1>(plan, tmap, args, stream, &ok_regs);
  } else {
    if (plan.bt == 128) e = launch_ws<128, 2>(plan, tmap, args, stream, &ok_regs);
    else e = launch_ws<64, 2>(plan, tmap, args, stream, &ok_regs);
  }
  if (e != cudaSuccess) return check_cuda(e, "q4 gemm launch");
  if (!ok_regs)
    return set_error(BQ4_EUNSUPPORTED, "q4 gemm kernel was not built with %d registers per thread",
                     kWsRegsLaunch);
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
