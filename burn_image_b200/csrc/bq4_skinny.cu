// bq4_skinny.cu -- the packed signed-Q4 linear for few tokens (decode-shaped
// and text-encoder-shaped calls), where streaming the weights from HBM, not
// the tensor core, sets the time.
//
// The tcgen05 GEMM (bq4_gemm_sm100.cu) is a persistent, warp-specialised
// kernel built for many tokens; with a handful of tokens its fixed costs
// (TMEM allocation, the activation staging launch, a split-K exchange through
// L2) dwarf the few microseconds the weight bytes take.  This kernel is one
// launch with no workspace:
//   * every warp streams its own 16 weight rows of the next D 128-K stages
//     from HBM into a private shared-memory ring with 16-byte cp.async
//     copies (the load/store path; measured on B200 it sustains the full HBM
//     rate for these per-CTA streams where small 1-D bulk copies did not),
//     waiting only on its own copy groups -- no producer warp and no
//     cross-warp barrier in the main loop;
//   * each lane unpacks its own nibbles in registers into the A fragment of
//     mma.sync.m16n8k16 (f16 x f16 -> f32): the K order inside an MMA is
//     permuted so that the 32 K values of one 16-byte row segment are exactly
//     the values that lane contributes, the same permutation is applied to
//     the activations, and no shuffle is needed;
//   * the f32 activations of the CTA's K range are read once, rounded to f16
//     (round to nearest even, as the GEMM's staging does) into swizzled
//     shared memory that every warp reads conflict-free;
//   * split-K partials meet in distributed shared memory (the CTAs of a
//     cluster), summed in a fixed order, so repeated calls give the same bits;
//   * the epilogue (bias, GELU-tanh, SiLU, aux, SiLU-gated pair, f16 output,
//     row scatter) runs once per output element.
// It is launched as a programmatic dependent of the kernel before it: the
// weight copies start before that kernel has finished, and only the reads
// of the activations (and every global write) wait for it.
//
// Numerics match the GEMM's: activations staged as f16; EXACT (block 128)
// keeps q exact in f16 and multiplies each K block's f32 partial by its
// scale; FOLDED stages f16(q * f16(scale)), the reference kernel's staging
// (patches/burn-cubecl-0.21.0/src/kernel/matmul/quantized.rs:172-178).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdlib>
#include <cstring>

#include "bq4_internal.h"
#include "sm100_ptx.cuh"

namespace bq4 {
namespace {

constexpr int kSkThreads = 256;  // 8 warps, one 16-row group of the CTA's 128-row tile each
constexpr size_t kSkCtaSmem = 110 * 1024;  // shared-memory budget: two CTAs fit on one SM
constexpr size_t kSkCtaSmem3 = 73 * 1024;  // three CTAs on one SM

struct SkArgs {
  const uint32_t* q[2];
  const float* s[2];
  const float* bias[2];
  const float* aux;
  const void* x;
  void* y;
  float* sc_y[BQ4_MAX_PEERS];  // row scatter targets (sc_rows > 0)
  int64_t ldx, ldy;
  int M, N, K;
  int nkc, nkb, nks, block;
  int kb_stage;   // scale blocks per 128-K stage (128 / block)
  int ks;         // CTAs per cluster along K (grid.y)
  int stages;     // depth D of each warp's ring
  uint32_t lane_bytes;  // ring bytes per lane per stage (weights, then scales)
  int x_f16, y_f16, xvec, yvec;
  int act;
  int sc_rows, sc_rank;
  uint32_t xs_pitch;    // bytes per token row of the staged activations
  uint32_t xs_off;      // offset of the staged activations (and, after the main loop, the partial tiles)
};

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

// The f16x2 pair (K 2i, 2i+1) of a prepared word (nibbles stored in K order
// {0,2,4,6,1,3,5,7}): (w >> 4i) & 0x000F000F, XOR 0x6408 maps the
// two's-complement nibble to f16 1024 + (q + 8), subtracting 1032 leaves q.
__device__ __forceinline__ uint32_t nib_pair(uint32_t w, int i) {
  const uint32_t magic = 0x64086408u;
  uint32_t t;
  asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(t) : "r"(w >> (4 * i)), "r"(0x000F000Fu), "r"(magic));
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(t) : "r"(t), "r"(magic));
  return t;
}

// Pair h (0 or 1) of the low byte of each half of w, unshifted: h = 0 gives
// the f16x2 q of bits [0,4), as nib_pair(w, 0); h = 1 reads bits [4,8) in
// place, which the XOR/subtract map to exactly 16 q (those bits are f16
// mantissa bits 4-7, and 1024 + 16 (n ^ 8) is exact).
__device__ __forceinline__ uint32_t nib_pair_at(uint32_t w, int h) {
  const uint32_t mask = h ? 0x00F000F0u : 0x000F000Fu;
  const uint32_t magic = h ? 0x64806480u : 0x64086408u;
  uint32_t t;
  asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(t) : "r"(w), "r"(mask), "r"(magic));
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(t) : "r"(t), "r"(magic));
  return t;
}

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

__device__ __forceinline__ uint32_t f16x2_of(float s) {
  uint16_t h;
  asm("cvt.rn.satfinite.f16.f32 %0, %1;" : "=h"(h) : "f"(s));
  return static_cast<uint32_t>(h) | (static_cast<uint32_t>(h) << 16);
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// d = A . B (accumulator input zero)
__device__ __forceinline__ void mma16816_zc(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                            uint32_t b0, uint32_t b1) {
  const float z = 0.0f;
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// Wait until at most n of this thread's copy groups are pending (n < 16).
__device__ __forceinline__ void cp_async_wait_dyn(int n) {
  switch (n) {
    case 0: cp_async_wait<0>(); break;
    case 1: cp_async_wait<1>(); break;
    case 2: cp_async_wait<2>(); break;
    case 3: cp_async_wait<3>(); break;
    case 4: cp_async_wait<4>(); break;
    case 5: cp_async_wait<5>(); break;
    case 6: cp_async_wait<6>(); break;
    case 7: cp_async_wait<7>(); break;
    case 8: cp_async_wait<8>(); break;
    case 9: cp_async_wait<9>(); break;
    case 10: cp_async_wait<10>(); break;
    case 11: cp_async_wait<11>(); break;
    case 12: cp_async_wait<12>(); break;
    case 13: cp_async_wait<13>(); break;
    case 14: cp_async_wait<14>(); break;
    default: cp_async_wait<15>(); break;
  }
}

__device__ __forceinline__ float sk_gelu_tanh(float v) {
  // Burn Gelu::new_approximate: 0.5 v (1 + tanh(sqrt(2/pi) (v + 0.044715 v^3)))
  const float u = 0.7978845608028654f * (v + 0.044715f * v * v * v);
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
  return 0.5f * v * (1.0f + t);
}

__device__ __forceinline__ float sk_silu(float v) { return __fdividef(v, 1.0f + __expf(-v)); }

// Byte offset of 16-byte chunk c (8 K values) in a staged token row: chunk
// c ^ 2 when bit 3 of c is set, so that the four K quarters a warp reads at
// once (chunks 4t + u, t = 0..3) fall in distinct banks; the row pitch is 16
// bytes past a multiple of 128, so the two token rows of one access phase
// use the other half of the banks.
__device__ __forceinline__ uint32_t xs_chunk(int c) { return (uint32_t)((c ^ (((c >> 3) & 1) << 1)) << 4); }

// One CTA: the 128-row prepared tile blockIdx.x, tokens [8 NT blockIdx.z,
// +8 NT), the K stages of split blockIdx.y (its rank in a cluster of ks CTAs
// along K).  Warp w owns rows 16 w .. 16 w + 15 of the tile: it streams
// them, stage by stage, into its own ring of D slots and consumes them.
//
// Lane (g = lane / 4, t = lane % 4) copies, per stage, the 16 bytes of rows
// g and g + 8 of its row group that hold K = 32 t .. 32 t + 31 of the stage
// (prepared chunk t / 2, half t % 2), and the scales of those rows, into its
// own ring slot, and reads back only what it copied.  MMA step (u, v)
// (u = 0..3, v = 0..1) takes K = 32 t + 8 u + 4 v + {0,1} into k-slots 2t,
// 2t + 1 and + {2,3} into 2t + 8, 2t + 9: every lane's A registers come from
// its own words, and the B fragment of token g is the same four K values of
// that token's row.
// SPL: scales per lane row per stage -- 1 (exact numerics, or blocks of 32+:
// a lane's 32 K lie in one block), 2 (blocks of 16), 4 (blocks of 8).
template <int NT, int NW, bool EXACT, int SPL, int MINB = 2>
__global__ void __launch_bounds__(kSkThreads, MINB) q4_skinny_kernel(const SkArgs a) {
  extern __shared__ __align__(128) unsigned char sk_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int tile = blockIdx.x;
  const int split = blockIdx.y;
  const int m0 = blockIdx.z * 8 * NT;
  const int S0 = (int)((int64_t)split * a.nks / a.ks), S1 = (int)((int64_t)(split + 1) * a.nks / a.ks);
  const int ns = S1 - S0;
  const int D = a.stages;
  const int row = warp * 16 + g;  // row of the tile (and row + 8)

  // ---- weight stream: this lane's slots of the warp's ring; the first D
  // stages are requested before anything else (weights are immutable, so
  // before the kernel this one depends on has finished)
  const uint32_t ring = ptx::smem_u32(sk_smem) + (uint32_t)(warp * D * 32 + lane) * a.lane_bytes;
  const uint32_t slot_stride = 32u * a.lane_bytes;
  const unsigned char* qsrc[NW];
  const float* ssrc[NW];
#pragma unroll
  for (int q = 0; q < NW; ++q) {
    qsrc[q] = reinterpret_cast<const unsigned char*>(a.q[q]) + (size_t)tile * a.nkc * 4096 + t * 2048 + row * 16;
    ssrc[q] = a.s[q] + (size_t)tile * a.nkb * 128 + row;
  }
  const int sc0 = EXACT ? 0 : (32 * t) / a.block;  // the lane's first scale block within a stage
  constexpr uint32_t kWStride = (32 + 8 * SPL + 15) & ~15u;  // one weight's bytes in a lane's slot (16-aligned)
  uint32_t fill = ring;  // the slot the next stage is copied into (the ring wraps after D slots)
  const uint32_t ring_end = ring + (uint32_t)D * slot_stride;
  auto issue = [&](int i) {  // stage S0 + i into the next slot (slot i % D)
    const int st = S0 + i;
    const uint32_t dst = fill;
    fill += slot_stride;
    if (fill == ring_end) fill = ring;
    const int kb = EXACT ? st : st * a.kb_stage + sc0;
#pragma unroll
    for (int q = 0; q < NW; ++q) {
      const uint32_t d = dst + (uint32_t)q * kWStride;
      cp_async16(d, qsrc[q] + (size_t)st * 8192);
      cp_async16(d + 16, qsrc[q] + (size_t)st * 8192 + 128);
#pragma unroll
      for (int j = 0; j < SPL; ++j) {
        cp_async4(d + 32 + 8 * j, ssrc[q] + (size_t)(kb + j) * 128);
        cp_async4(d + 36 + 8 * j, ssrc[q] + (size_t)(kb + j) * 128 + 8);
      }
    }
  };
  // (Requesting only the first two stages before the activation loads, so
  // that those loads do not queue behind the whole ring, measured slower:
  // 13.1 against 10.9 us at 1 x 2560 -> 9728.)
  for (int i = 0; i < D; ++i) {
    if (i < ns) issue(i);
    cp_async_commit();  // one group per slot, empty past the CTA's range
  }

  // ---- activations of the CTA's K range -> f16, swizzled shared memory
  ptx::griddep_launch_dependents();  // the next kernel may start its own weight stream
  ptx::griddep_wait();               // x may be the output of the kernel before this one
  // the bias of this thread's first epilogue element (see the epilogue),
  // loaded now so that its latency hides behind the main loop
  const int quads = 32, elems = 8 * NT * quads;
  const int e_first = threadIdx.x * a.ks + split;
  const int n0 = tile * 128;
  float bpre[NW][4];
#pragma unroll
  for (int q = 0; q < NW; ++q)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int nc = n0 + 4 * (e_first % quads) + c;
      bpre[q][c] = (a.bias[q] && e_first < elems && nc < a.N) ? __ldg(a.bias[q] + nc) : 0.0f;
    }
  {
    // rows past M and K values past K are zeros; each thread issues the
    // loads of kXB chunks before converting any, so their latencies overlap
    constexpr int kXB = 4;
    const int chunks = ns * 16;  // 8-K chunks per token row
    const int K0 = S0 * 128;
    const int total = 8 * NT * chunks;
    unsigned char* xs = sk_smem + a.xs_off;
    for (int base = threadIdx.x; base < total; base += kSkThreads * kXB) {
      float f[kXB][8];
      uint4 hv[kXB];
#pragma unroll
      for (int b = 0; b < kXB; ++b) {
        const int idx = base + b * kSkThreads;
        hv[b] = make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int i = 0; i < 8; ++i) f[b][i] = 0.0f;
        if (idx >= total) continue;
        const int tok = idx / chunks, c = idx - tok * chunks;
        const int m = m0 + tok, k = K0 + c * 8;
        if (m >= a.M) continue;
        if (a.x_f16) {
          const __half* xr = static_cast<const __half*>(a.x) + (size_t)m * a.ldx;
          if (k + 8 <= a.K && a.xvec) {
            hv[b] = *reinterpret_cast<const uint4*>(xr + k);
          } else {
            uint16_t e[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) e[i] = k + i < a.K ? __half_as_ushort(xr[k + i]) : (uint16_t)0;
            hv[b] = make_uint4(e[0] | (uint32_t)e[1] << 16, e[2] | (uint32_t)e[3] << 16,
                               e[4] | (uint32_t)e[5] << 16, e[6] | (uint32_t)e[7] << 16);
          }
        } else {
          const float* xr = static_cast<const float*>(a.x) + (size_t)m * a.ldx;
          if (k + 8 <= a.K && a.xvec) {
            const float4 p0 = *reinterpret_cast<const float4*>(xr + k);
            const float4 p1 = *reinterpret_cast<const float4*>(xr + k + 4);
            f[b][0] = p0.x; f[b][1] = p0.y; f[b][2] = p0.z; f[b][3] = p0.w;
            f[b][4] = p1.x; f[b][5] = p1.y; f[b][6] = p1.z; f[b][7] = p1.w;
          } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) f[b][i] = k + i < a.K ? xr[k + i] : 0.0f;
          }
        }
      }
#pragma unroll
      for (int b = 0; b < kXB; ++b) {
        const int idx = base + b * kSkThreads;
        if (idx >= total) continue;
        const int tok = idx / chunks, c = idx - tok * chunks;
        uint4 h = hv[b];
        if (!a.x_f16) {
          uint32_t p[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const __half2 v = __floats2half2_rn(f[b][2 * i], f[b][2 * i + 1]);
            p[i] = *reinterpret_cast<const uint32_t*>(&v);
          }
          h = make_uint4(p[0], p[1], p[2], p[3]);
        }
        *reinterpret_cast<uint4*>(xs + (size_t)tok * a.xs_pitch + xs_chunk(c)) = h;
      }
    }
  }
  __syncthreads();

  // ---- main loop over the CTA's stages.  The 8 MMA steps of a stage go
  // round-robin into CH independent accumulator chains, so that mma.sync
  // latency, not one dependent chain, sets the pace.  Step (u, p) takes the
  // nibble pairs p and p + 2 of the lane's word u (K = 8 u + 2 p + {0,1} and
  // 8 u + 2 p + 4 + {0,1} of its 32), and chain (2 u + p) % CH; CH is even,
  // so a chain only ever sees one p.
  //   EXACT: pairs 1 and 3 are unpacked without a shift (their nibbles sit
  //   in bits 4-7 of each f16 half, so they come out as exactly 16 q) and
  //   their chains are scaled by 1/16 (exact) when the stage's partial is
  //   summed; each chain restarts every stage (zero-accumulator MMA), and the
  //   partial, summed in chain order, is multiplied by the block's f32 scale.
  //   FOLDED: every pair is unpacked to q and multiplied by f16(scale); the
  //   chains run over all stages and are summed in chain order at the end.
  constexpr int CH = EXACT ? (NT * NW >= 4 ? 2 : 4 / (NT * NW)) : (NT * NW >= 8 ? 2 : 8 / (NT * NW));
  float acc[NW][NT][4];
#pragma unroll
  for (int i = 0; i < NW; ++i)
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[i][j][0] = acc[i][j][1] = acc[i][j][2] = acc[i][j][3] = 0.0f;
  float chain[CH][NW][NT][4];
  if constexpr (!EXACT) {
#pragma unroll
    for (int c = 0; c < CH; ++c)
#pragma unroll
      for (int i = 0; i < NW; ++i)
#pragma unroll
        for (int j = 0; j < NT; ++j) chain[c][i][j][0] = chain[c][i][j][1] = chain[c][i][j][2] = chain[c][i][j][3] = 0.0f;
  }
  // token g's row of staged activations; stage i's chunk 4 t + u sits at
  // i * 256 + xs_chunk(4 t + u) (the swizzle only moves bit 1 of the chunk
  // index within each 16-chunk stage)
  const uint32_t xs_base = ptx::smem_u32(sk_smem + a.xs_off) + (uint32_t)g * a.xs_pitch;
  uint32_t xoff[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) xoff[u] = xs_chunk(4 * t + u);
  uint32_t src = ring;  // the slot of stage i
  for (int i = 0; i < ns; ++i) {
    cp_async_wait_dyn(D - 1);  // this lane's copies of stage i have landed (one group per stage)
    uint4 w[NW][2];
    float se[NW][SPL][2];
#pragma unroll
    for (int q = 0; q < NW; ++q) {
      const uint32_t d = src + (uint32_t)q * kWStride;
      w[q][0] = lds128(d);
      w[q][1] = lds128(d + 16);
#pragma unroll
      for (int j = 0; j < SPL; ++j) {
        se[q][j][0] = __uint_as_float(lds32(d + 32 + 8 * j));
        se[q][j][1] = __uint_as_float(lds32(d + 36 + 8 * j));
      }
    }
    uint32_t sf[NW][4][2];
    if constexpr (!EXACT) {
#pragma unroll
      for (int q = 0; q < NW; ++q)
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          sf[q][u][0] = f16x2_of(se[q][u * SPL / 4][0]);
          sf[q][u][1] = f16x2_of(se[q][u * SPL / 4][1]);
        }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      // af[q][p] = {row g pair p, row g+8 pair p, row g pair p+2, row g+8 pair p+2}
      uint32_t af[NW][2][4];
#pragma unroll
      for (int q = 0; q < NW; ++q) {
        const uint32_t lo = (&w[q][0].x)[u], hi = (&w[q][1].x)[u];
        if constexpr (EXACT) {
          const uint32_t lo8 = lo >> 8, hi8 = hi >> 8;
          af[q][0][0] = nib_pair_at(lo, 0);
          af[q][0][1] = nib_pair_at(hi, 0);
          af[q][0][2] = nib_pair_at(lo8, 0);
          af[q][0][3] = nib_pair_at(hi8, 0);
          af[q][1][0] = nib_pair_at(lo, 1);  // 16 q
          af[q][1][1] = nib_pair_at(hi, 1);
          af[q][1][2] = nib_pair_at(lo8, 1);
          af[q][1][3] = nib_pair_at(hi8, 1);
        } else {
#pragma unroll
          for (int pp = 0; pp < 2; ++pp) {
            af[q][pp][0] = hmul2(nib_pair(lo, pp), sf[q][u][0]);
            af[q][pp][1] = hmul2(nib_pair(hi, pp), sf[q][u][1]);
            af[q][pp][2] = hmul2(nib_pair(lo, pp + 2), sf[q][u][0]);
            af[q][pp][3] = hmul2(nib_pair(hi, pp + 2), sf[q][u][1]);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        // token g's K values 8 u + {0..7}: word k holds K 8 u + 2 k, + 1
        const uint4 xv = lds128(xs_base + (uint32_t)(8 * j) * a.xs_pitch + (uint32_t)i * 256u + xoff[u]);
#pragma unroll
        for (int q = 0; q < NW; ++q) {
#pragma unroll
          for (int pp = 0; pp < 2; ++pp) {
            const int c = (2 * u + pp) % CH;
            const uint32_t b0 = pp ? xv.y : xv.x, b1 = pp ? xv.w : xv.z;
            if (EXACT && 2 * u + pp < CH)
              mma16816_zc(chain[c][q][j], af[q][pp][0], af[q][pp][1], af[q][pp][2], af[q][pp][3], b0, b1);
            else
              mma16816(chain[c][q][j], af[q][pp][0], af[q][pp][1], af[q][pp][2], af[q][pp][3], b0, b1);
          }
        }
      }
    }
    // the slot's data is in registers: refill it with stage i + D
    if (i + D < ns) issue(i + D);
    cp_async_commit();
    src += slot_stride;
    if (src == ring_end) src = ring;
    if constexpr (EXACT) {
#pragma unroll
      for (int q = 0; q < NW; ++q)
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          float p[4];
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            float ev = chain[0][q][j][r], od = chain[1][q][j][r];
#pragma unroll
            for (int c = 2; c < CH; c += 2) {
              ev += chain[c][q][j][r];
              od += chain[c + 1][q][j][r];
            }
            p[r] = fmaf(od, 0.0625f, ev);
          }
          acc[q][j][0] = fmaf(p[0], se[q][0][0], acc[q][j][0]);
          acc[q][j][1] = fmaf(p[1], se[q][0][0], acc[q][j][1]);
          acc[q][j][2] = fmaf(p[2], se[q][0][1], acc[q][j][2]);
          acc[q][j][3] = fmaf(p[3], se[q][0][1], acc[q][j][3]);
        }
    }
  }
  cp_async_wait<0>();  // no copy may land after this CTA's shared memory is reused or released
  if constexpr (!EXACT) {
#pragma unroll
    for (int q = 0; q < NW; ++q)
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          float v = chain[0][q][j][r];
#pragma unroll
          for (int c = 1; c < CH; ++c) v += chain[c][q][j][r];
          acc[q][j][r] = v;
        }
  }

  // ---- the warps' tiles -> [NW][8 NT tokens][128 + 4 rows] f32 (rows of
  // token t contiguous, so the epilogue reads 4 rows at once), over the
  // staged activations, which every warp has finished with
  constexpr int RP = 132;
  __syncthreads();
  float* red = reinterpret_cast<float*>(sk_smem + a.xs_off);
#pragma unroll
  for (int q = 0; q < NW; ++q)
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      float* base = red + ((size_t)q * 8 * NT + 8 * j + 2 * t) * RP + row;
      base[0] = acc[q][j][0];
      base[RP] = acc[q][j][1];
      base[8] = acc[q][j][2];
      base[RP + 8] = acc[q][j][3];
    }

  // ---- cluster sum (ranks in order) and the epilogue; rank r takes every
  // ks-th element
  if (a.ks > 1) ptx::cluster_sync();
  else __syncthreads();
  {
    for (int e = e_first; e < elems; e += kSkThreads * a.ks) {
      const int tok = e / quads, rq = e - tok * quads;
      const int m = m0 + tok;
      if (m >= a.M) continue;  // a padding token column: nothing to read or write
      float v[NW][4];
#pragma unroll
      for (int i = 0; i < NW; ++i) {
        v[i][0] = v[i][1] = v[i][2] = v[i][3] = 0.0f;
        const float* src = red + ((size_t)i * 8 * NT + tok) * RP + 4 * rq;
        for (int r = 0; r < a.ks; ++r) {
          float4 p;
          if (a.ks > 1) p = ptx::ld_shared_cluster_f4(ptx::mapa_shared(ptx::smem_u32(src), (uint32_t)r));
          else p = *reinterpret_cast<const float4*>(src);
          v[i][0] += p.x; v[i][1] += p.y; v[i][2] += p.z; v[i][3] += p.w;
        }
      }
      const int n = n0 + 4 * rq;
      float o[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int nc = n + c;
        const bool in = nc < a.N;
        float r0 = v[0][c];
        if (a.bias[0] && in) r0 += e == e_first ? bpre[0][c] : __ldg(a.bias[0] + nc);
        if constexpr (NW == 2) {
          float r1 = v[1][c];
          if (a.bias[1] && in) r1 += e == e_first ? bpre[1][c] : __ldg(a.bias[1] + nc);
          r0 = sk_silu(r0) * r1;
        } else {
          if (a.act == BQ4_ACT_GELU_TANH) r0 = sk_gelu_tanh(r0);
          else if (a.act == BQ4_ACT_SILU) r0 = sk_silu(r0);
          if (a.aux && in) r0 *= __ldg(a.aux + (size_t)m * a.N + nc);
        }
        o[c] = r0;
      }
      if (a.sc_rows) {
        const int owner = m / a.sc_rows;
        float* yr = a.sc_y[owner] + (size_t)(a.sc_rank * a.sc_rows + (m - owner * a.sc_rows)) * a.ldy;
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (n + c < a.N) yr[n + c] = o[c];
      } else if (a.y_f16) {
        __half* yr = static_cast<__half*>(a.y) + (size_t)m * a.ldy;
        if (a.yvec && n + 4 <= a.N) {
          const __half2 h0 = __floats2half2_rn(o[0], o[1]), h1 = __floats2half2_rn(o[2], o[3]);
          *reinterpret_cast<uint2*>(yr + n) =
              make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c)
            if (n + c < a.N) yr[n + c] = __float2half_rn(o[c]);
        }
      } else {
        float* yr = static_cast<float*>(a.y) + (size_t)m * a.ldy;
        if (a.yvec && n + 4 <= a.N) {
          *reinterpret_cast<float4*>(yr + n) = make_float4(o[0], o[1], o[2], o[3]);
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c)
            if (n + c < a.N) yr[n + c] = o[c];
        }
      }
    }
  }
  if (a.ks > 1) ptx::cluster_sync();  // keep this CTA's partials alive until every rank has read them
}

template <int NT, int NW, bool EXACT, int SPL, int MINB = 2>
cudaError_t launch_sk(const SkPlan& p, const SkArgs& a, cudaStream_t stream) {
  static std::atomic<int> ready[64];
  int dev = 0;
  cudaGetDevice(&dev);
  auto kern = q4_skinny_kernel<NT, NW, EXACT, SPL, MINB>;
  if (dev >= 0 && dev < 64 && !ready[dev].load(std::memory_order_acquire)) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSkMaxSmem);
    if (e != cudaSuccess) return e;
    ready[dev].store(1, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3((unsigned)p.gx, (unsigned)p.ks, (unsigned)p.gz);
  cfg.blockDim = dim3(kSkThreads, 1, 1);
  cfg.dynamicSmemBytes = p.smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[na].val.programmaticStreamSerializationAllowed = p.pdl ? 1 : 0;
  ++na;
  if (p.ks > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = (unsigned)p.ks;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
  note_launch();
  return e;
}

// Shared-memory layout of one CTA (bytes): the eight warps' rings of
// `stages` slots of 32 lanes x lane_bytes (weights, then scales; an odd
// number of 16-byte units, so the lanes of one access phase hit distinct
// banks), then the staged activation rows (8 NT tokens x kcta stages x 128 K
// in f16, 16 bytes of pitch padding) -- reused after the main loop for the
// warps' partial tiles ([NW][8 NT][132] f32).
struct SkLayout {
  uint32_t lane_bytes, xs_pitch, xs_off;
  size_t total;
};

SkLayout sk_layout(int nt, int nw, int spl, int kcta, int stages) {
  SkLayout L;
  uint32_t lb = (uint32_t)nw * ((32 + 8 * spl + 15) & ~15u);
  if (((lb >> 4) & 1) == 0) lb += 16;
  L.lane_bytes = lb;
  L.xs_pitch = (uint32_t)kcta * 256 + 16;
  L.xs_off = (uint32_t)(kSkThreads / 32) * (uint32_t)stages * 32u * lb;
  const uint32_t xs_bytes = 8u * nt * L.xs_pitch, red_bytes = (uint32_t)nw * 8 * nt * 132 * 4;
  L.total = (size_t)L.xs_off + (xs_bytes > red_bytes ? xs_bytes : red_bytes);
  return L;
}

}  // namespace

bool plan_skinny(const bq4_weight* w, int nw, int64_t M, int device, bool exact, SkPlan* p) {
  memset(p, 0, sizeof(*p));
  if (w->h || w->tf32 || !w->q || !w->s) return false;       // pre-expanded / packed-F16 weights
  if (exact && w->block != 128) return false;                // exact scale per 128-K stage only
  if (M <= 0 || M > kSkMaxM) return false;
  if (w->Kp % 128 != 0) return false;
  int sms = device_sm_count(device);
  if (sm_budget() > 0 && sm_budget() < sms) sms = sm_budget();
  // token tile: the fewest 8-token MMA columns covering M (at most 64 per CTA)
  int nt = 1;
  while (nt < 8 && 8 * nt < M) nt *= 2;
  if (nw == 2 && nt > 2) nt = 2;   // two weights' accumulators: at most 16 tokens per CTA
  if (exact && nt > 4) nt = 4;     // the exact partials: at most 32 tokens per CTA
  const int mgroups = (int)((M + 8 * nt - 1) / (8 * nt));
  const int nks = (int)(w->Kp / 128);
  const int gx = (int)w->ntiles;
  const int spl = exact || w->block >= 32 ? 1 : 128 / 4 / w->block;  // blocks of 16: 2, of 8: 4
  // K splits across a cluster (<= 8): as many as one wave of minb CTAs per
  // SM holds, each CTA keeping at least two 128-K stages.  The build for
  // three CTAs per SM (one weight, up to 16 tokens: 80 registers, a smaller
  // shared-memory budget) is taken when it allows more splits than two CTAs
  // per SM do.  Measured on B200 (graph-replayed): 76 weight tiles,
  // 1 x 2560 -> 9728: 2 splits 10.9 us, 3 splits 10.8, 5 splits at three
  // CTAs per SM 9.6; 16 x 2560 -> 9728: 15.9 / 14.3 / 13.4; 16 x 2560 ->
  // 2 x 9728 gated: 24.6 / 20.0 (two weights: two CTAs per SM); 20 tiles
  // (16 x 9728 -> 2560) keep 8 splits at two CTAs per SM (17.6 us; 21.0 at
  // three).  BQ4_SKINNY_MINB=2|3 pins the choice.
  auto splits = [&](int per_sm) {
    int k = (int)((int64_t)per_sm * sms / ((int64_t)gx * mgroups));
    if (k > 8) k = 8;
    if (k > nks / 2) k = nks / 2;
    return k < 1 ? 1 : k;
  };
  const bool can3 = nw == 1 && nt <= 2 && spl == 1;
  int minb = can3 && splits(3) > splits(2) ? 3 : 2;
  if (const char* f = getenv("BQ4_SKINNY_MINB")) {
    const int v = atoi(f);
    if (v == 2 || (v == 3 && can3)) minb = v;
  }
  int ks = 1, kcta = 1, stages = 2;
  SkLayout L;
  for (;;) {
    ks = splits(minb);
    if (const char* f = getenv("BQ4_SKINNY_KS")) {
      const int v = atoi(f);
      if (v >= 1 && v <= 8) ks = v;
    }
    if (ks > nks) ks = nks;
    kcta = (nks + ks - 1) / ks;
    // each warp's ring: as many stages as fit next to the activations (at
    // most the CTA's stage count and 15), at least 2
    const size_t budget = minb == 3 ? kSkCtaSmem3 : kSkCtaSmem;
    stages = 2;
    while (stages < kcta && stages < 15 && sk_layout(nt, nw, spl, kcta, stages + 1).total <= budget) ++stages;
    if (const char* f = getenv("BQ4_SKINNY_STAGES")) {
      const int v = atoi(f);
      if (v >= 2 && v < stages) stages = v;
    }
    L = sk_layout(nt, nw, spl, kcta, stages);
    if (minb == 3 && L.total > kSkCtaSmem3) {  // three CTAs do not fit one SM's shared memory
      minb = 2;
      continue;
    }
    break;
  }
  if (L.total > kSkMaxSmem) return false;
  p->nt = nt;
  p->nw = nw;
  p->R = 8;
  p->ks = ks;
  p->gx = gx;
  p->gz = mgroups;
  p->stages = stages;
  p->smem_bytes = L.total;
  p->exact = exact ? 1 : 0;
  p->pdl = getenv("BQ4_NO_PDL") ? 0 : 1;
  p->minb = minb;
  return true;
}

bq4_status run_skinny(const SkPlan& p, const bq4_weight* const* ws, const void* x, int x_f16, int64_t M, int64_t ldx,
                      const float* const* bias, int act, const float* aux, void* y, int y_f16, int64_t ldy,
                      const GemmIo& io, cudaStream_t stream) {
  const bq4_weight* w0 = ws[0];
  SkArgs a;
  memset(&a, 0, sizeof(a));
  for (int i = 0; i < p.nw; ++i) {
    a.q[i] = ws[i]->q;
    a.s[i] = ws[i]->s;
    a.bias[i] = bias ? bias[i] : nullptr;
  }
  a.aux = aux;
  a.x = x;
  a.y = y;
  a.ldx = ldx;
  a.ldy = ldy > 0 ? ldy : w0->N;
  a.M = (int)M;
  a.N = (int)w0->N;
  a.K = (int)w0->K;
  a.nkc = (int)w0->nkc;
  a.nkb = (int)w0->nkb;
  a.nks = (int)(w0->Kp / 128);
  a.block = w0->block;
  a.kb_stage = 128 / w0->block;
  a.ks = p.ks;
  a.stages = p.stages;
  a.x_f16 = x_f16;
  a.y_f16 = y_f16;
  a.xvec = x_f16 ? ((reinterpret_cast<uintptr_t>(x) & 15) == 0 && ldx % 8 == 0)
                 : ((reinterpret_cast<uintptr_t>(x) & 15) == 0 && ldx % 4 == 0);
  a.yvec = ((reinterpret_cast<uintptr_t>(y) & (y_f16 ? 7 : 15)) == 0 && a.ldy % 4 == 0) ? 1 : 0;
  a.act = act;
  if (io.sc_rows) {
    if (y_f16 || io.sc_nranks < 1 || io.sc_nranks > BQ4_MAX_PEERS || !io.sc_y)
      return set_error(BQ4_EINVAL_ARG, "row scatter needs f32 output and 1..%d ranks", BQ4_MAX_PEERS);
    a.sc_rows = io.sc_rows;
    a.sc_rank = io.sc_rank;
    for (int r = 0; r < io.sc_nranks; ++r) a.sc_y[r] = io.sc_y[r];
  }
  const int kcta = (a.nks + p.ks - 1) / p.ks;
  const int spl = p.exact || w0->block >= 32 ? 1 : 128 / 4 / w0->block;  // blocks of 16: 2, of 8: 4
  const SkLayout L = sk_layout(p.nt, p.nw, spl, kcta, p.stages);
  a.lane_bytes = L.lane_bytes;
  a.xs_pitch = L.xs_pitch;
  a.xs_off = L.xs_off;
  cudaError_t e = cudaSuccess;
#define BQ4_SK_CASE(NT_, NW_, EX_, SPL_)                           \
  if (p.nt == NT_ && p.nw == NW_ && p.exact == EX_ && spl == SPL_) \
    e = launch_sk<NT_, NW_, EX_, SPL_>(p, a, stream);               \
  else
#define BQ4_SK_CASE3(NT_, EX_)                                                       \
  if (p.minb == 3 && p.nt == NT_ && p.nw == 1 && p.exact == EX_ && spl == 1) \
    e = launch_sk<NT_, 1, EX_, 1, 3>(p, a, stream);                          \
  else
  BQ4_SK_CASE3(1, true) BQ4_SK_CASE3(2, true) BQ4_SK_CASE3(1, false) BQ4_SK_CASE3(2, false)
  BQ4_SK_CASE(1, 1, true, 1) BQ4_SK_CASE(2, 1, true, 1) BQ4_SK_CASE(4, 1, true, 1)
  BQ4_SK_CASE(1, 1, false, 1) BQ4_SK_CASE(2, 1, false, 1) BQ4_SK_CASE(4, 1, false, 1) BQ4_SK_CASE(8, 1, false, 1)
  BQ4_SK_CASE(1, 1, false, 2) BQ4_SK_CASE(2, 1, false, 2) BQ4_SK_CASE(4, 1, false, 2) BQ4_SK_CASE(8, 1, false, 2)
  BQ4_SK_CASE(1, 1, false, 4) BQ4_SK_CASE(2, 1, false, 4) BQ4_SK_CASE(4, 1, false, 4) BQ4_SK_CASE(8, 1, false, 4)
  BQ4_SK_CASE(1, 2, true, 1) BQ4_SK_CASE(2, 2, true, 1)
  BQ4_SK_CASE(1, 2, false, 1) BQ4_SK_CASE(2, 2, false, 1) BQ4_SK_CASE(1, 2, false, 2) BQ4_SK_CASE(2, 2, false, 2)
  BQ4_SK_CASE(1, 2, false, 4) BQ4_SK_CASE(2, 2, false, 4)
  return set_error(BQ4_EUNSUPPORTED, "no small-M kernel for %d token columns x %d weights", 8 * p.nt, p.nw);
#undef BQ4_SK_CASE
#undef BQ4_SK_CASE3
  if (e != cudaSuccess) return check_cuda(e, "small-M q4 linear launch");
  return BQ4_OK;
}

}  // namespace bq4
