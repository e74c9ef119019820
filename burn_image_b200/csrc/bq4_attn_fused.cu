// bq4_attn_fused.cu -- fused attention for head_dim 128: out = softmax(scale
// q k^T) v per (batch, query head), one CTA per 128 query rows.
//
// The scores never leave the SM.  Per 128-key block j:
//   warp 0 (TMA)      k_j [128 keys][128] f16 and v_j^T [128 d][128 keys] f16
//                     into a 2-stage ring (128-byte swizzle); q once.
//   warp 1 (MMA)      S_j = q k_j^T into TMEM buffer j % 2 (tcgen05, f16 in,
//                     f32 out), and after the softmax of block j, O += P_j v_j
//                     into the TMEM accumulator with P_j read from TMEM (the
//                     A-in-TMEM form); S_{j+2} is issued as soon as buffer
//                     j % 2 is released.
//   warps 4..19       four threads per query row (32 columns each): the row max of S_j (scaled, in
//                     log2 units), P = exp2(s - m) as f16 pairs into one of
//                     two TMEM P buffers (row i in lane i, two keys per
//                     column), the running sum, and -- only when the max jumps by more than
//                     2^8 -- O rescaled in TMEM once the previous P v is done,
//                     so the softmax of block j overlaps P_{j-1} v_{j-1}.
// At the end O / sum is written as f32.  Every wait is bounded: a timeout
// records BQ4_ETIMEOUT and every role unwinds.
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

constexpr int kAParts = 4;                       // softmax threads per query row
constexpr int kACols = 128 / kAParts;            // score / output columns per softmax thread
constexpr int kASoftWarps = 4 * kAParts;         // kAParts warps per TMEM lane quarter
constexpr int kAThreads = 128 + 32 * kASoftWarps;  // warp 0 TMA, 1 MMA, 4.. softmax
constexpr int kAKV = 2;                          // k / v ring stages
constexpr uint32_t kASub = 128 * 128;       // one [128 rows][64] f16 sub-tile (16 KB)
constexpr uint32_t kATileB = 2 * kASub;     // one [128][128] f16 operand
// q, k[kAKV], vt[kAKV]; the softmax parts' row-max slots [2][kAParts][128]
// f32; barriers.  No alignment slack: the kernel checks that its dynamic
// shared memory starts 1024-aligned (the operand tiles' swizzle needs it).
constexpr uint32_t kAXchg = 2 * kAParts * 128 * 4;
constexpr uint32_t kASmem = (1 + 2 * kAKV) * kATileB + kAXchg + 256;
// TMEM columns: S buffers at 0 and 128 (f32), O at 256 (f32), P buffers at
// 384 and 448 (128 keys as 64 columns of f16 pairs).
constexpr uint32_t kATmemO = 256, kATmemP = 384;
// A row keeps its running max until a block's max passes it by more than this
// (log2 units): P = exp2(s - m) then stays <= 2^8, which f16 holds, and O is
// rescaled -- after waiting for the previous P v -- only when the max jumps.
constexpr float kRescaleLog2 = 8.0f;

struct AttnArgs {
  float* out;     // [B*Hq][Sq][128] f32
  int Sq, Skv, Hq, Hkv, qtiles, nblk;
  float c;        // scale * log2(e)
  int* err;
};

__device__ __forceinline__ bool attn_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err) {
  if (ptx::mbar_wait(bar, parity, abort_flag)) return true;
  if (!*abort_flag) {
    *abort_flag = 1;
    if (err) atomicCAS(err, 0, (int)BQ4_ETIMEOUT);
  }
  return false;
}

// As attn_wait, polling with test_wait instead of parking the thread: for the
// MMA issuer, whose wake-up latency after a suspended try_wait (about 170
// cycles, measured) would leave the tensor core idle at every hand-off.
__device__ __forceinline__ bool attn_wait_poll(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err) {
  if (ptx::mbar_wait_spin(bar, parity, abort_flag)) return true;
  if (!*abort_flag) {
    *abort_flag = 1;
    if (err) atomicCAS(err, 0, (int)BQ4_ETIMEOUT);
  }
  return false;
}

// 2^x by the PTX instruction ex2.approx.ftz.f32 (one MUFU op; relative error
// near 2^-22, results below 2^-126 flush to 0 -- far under the smallest f16
// probability the P operand can hold).
__device__ __forceinline__ float attn_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Blackwell's three-input max and packed two-lane f32 arithmetic (PTX
// max.f32 with three sources; fma / add .f32x2 on a b64 pair, low lane first).
__device__ __forceinline__ float attn_max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ uint64_t attn_pack2(float lo, float hi) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
  return d;
}
__device__ __forceinline__ void attn_unpack2(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t attn_fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t attn_add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// 2^x for two lanes on the FMA pipe instead of the MUFU unit, which the
// exponentials of both query tiles otherwise saturate.  Cody-Waite range
// reduction x = n + f, n = round(x), f in [-1/2, 1/2]: adding 1.5 * 2^23
// rounds x to an integer held in the low mantissa bits of the sum t, and
// (t - 1.5 * 2^23) is n exactly.  2^f is a degree-3 polynomial fitted here
// by the Remez exchange for minimal relative error on [-1/2, 1/2]: 7.5e-5 in
// f32 Horner form, below the f16 rounding of the probability (2^-11).  2^n
// is applied by adding n to the exponent field: the bits of t shifted left by
// 23 are n << 23 (the rest of t's bits shift out).  x is clamped at -125 so
// that the exponent of the result stays normal (2^-125 is 0 in f16).
__device__ __forceinline__ void attn_exp2_poly2(float x0, float x1, float& p0, float& p1) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  constexpr float kC0 = 0x1.fff692p-1f, kC1 = 0x1.62f31ap-1f, kC2 = 0x1.f0de1ap-3f, kC3 = 0x1.c3f76p-5f;
  const uint64_t x = attn_pack2(fmaxf(x0, -125.0f), fmaxf(x1, -125.0f));
  const uint64_t t = attn_add2(x, attn_pack2(kRound, kRound));
  const uint64_t n = attn_add2(t, attn_pack2(-kRound, -kRound));
  const uint64_t f = attn_fma2(n, attn_pack2(-1.0f, -1.0f), x);
  uint64_t p = attn_fma2(attn_pack2(kC3, kC3), f, attn_pack2(kC2, kC2));
  p = attn_fma2(p, f, attn_pack2(kC1, kC1));
  p = attn_fma2(p, f, attn_pack2(kC0, kC0));
  float pl, ph, tl, th;
  attn_unpack2(p, pl, ph);
  attn_unpack2(t, tl, th);
  p0 = __int_as_float(__float_as_int(pl) + (__float_as_int(tl) << 23));
  p1 = __int_as_float(__float_as_int(ph) + (__float_as_int(th) << 23));
}

// Max of this thread's kN raw scores; kFull: all kN keys exist (every block
// but a ragged last one), so no key is masked.
template <int kN, bool kFull>
__device__ __forceinline__ float attn_rowmax(const uint32_t (&r)[kN], int valid) {
  if constexpr (kFull && kN % 16 == 0) {
    // eight running maxima, two new scores per three-input max
    float mp[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) mp[u] = __uint_as_float(r[u]);
#pragma unroll
    for (int i = 8; i + 16 <= kN; i += 16)
#pragma unroll
      for (int u = 0; u < 8; ++u) mp[u] = attn_max3(mp[u], __uint_as_float(r[i + u]), __uint_as_float(r[i + 8 + u]));
#pragma unroll
    for (int u = 0; u < 8; ++u) mp[u] = fmaxf(mp[u], __uint_as_float(r[kN - 8 + u]));
    return attn_max3(attn_max3(mp[0], mp[1], mp[2]), attn_max3(mp[3], mp[4], mp[5]), fmaxf(mp[6], mp[7]));
  } else {
    float mp[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) mp[u] = -INFINITY;
#pragma unroll
    for (int i = 0; i < kN; ++i)
      if (kFull || i < valid) mp[i & 7] = fmaxf(mp[i & 7], __uint_as_float(r[i]));
    return fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])), fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
  }
}

// P = 2^(s c - m) for this thread's kN keys as f16 pairs into kN / 2 TMEM
// columns of its lane from t_p (key 2 i in the low half of column i, the
// layout the A-in-TMEM MMA reads); returns the f32 sum of the probabilities.
// kPolyQ (full blocks): of every four key pairs, the first kPolyQ take the
// FMA-pipe exponential (attn_exp2_poly2), the rest ex2.approx.
template <int kN, bool kFull, int kPolyQ = 0>
__device__ __forceinline__ float attn_p_store(const uint32_t (&r)[kN], int valid, float c, float m_use,
                                              uint32_t t_p) {
  if constexpr (kFull) {
    // s c - m two keys at a time, and four packed partial sums
    const uint64_t c2 = attn_pack2(c, c), m2 = attn_pack2(-m_use, -m_use);
    uint64_t acc[4] = {0, 0, 0, 0};  // zero bits: +0.0f in both lanes
#pragma unroll
    for (int cc = 0; cc < kN / 16; ++cc) {
      uint32_t pk[8];
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        const int k0 = cc * 16 + i;
        float x0, x1, p0, p1;
        attn_unpack2(attn_fma2(attn_pack2(__uint_as_float(r[k0]), __uint_as_float(r[k0 + 1])), c2, m2), x0, x1);
        if (((i >> 1) & 3) < kPolyQ) {
          attn_exp2_poly2(x0, x1, p0, p1);
        } else {
          p0 = attn_ex2(x0);
          p1 = attn_ex2(x1);
        }
        acc[(i >> 1) & 3] = attn_add2(acc[(i >> 1) & 3], attn_pack2(p0, p1));
        const __half2 hp = __floats2half2_rn(p0, p1);
        pk[i >> 1] = *reinterpret_cast<const uint32_t*>(&hp);
      }
      ptx::tmem_st_32x32b_x8(t_p + cc * 8, pk);
    }
    float sum = 0.0f;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float lo, hi;
      attn_unpack2(acc[u], lo, hi);
      sum += lo + hi;
    }
    return sum;
  } else {
    float sp[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) sp[u] = 0.0f;
#pragma unroll
    for (int cc = 0; cc < kN / 16; ++cc) {
      uint32_t pk[8];
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        const int k0 = cc * 16 + i;
        const float p0 = (kFull || k0 < valid) ? attn_ex2(fmaf(__uint_as_float(r[k0]), c, -m_use)) : 0.0f;
        const float p1 = (kFull || k0 + 1 < valid) ? attn_ex2(fmaf(__uint_as_float(r[k0 + 1]), c, -m_use)) : 0.0f;
        sp[i >> 1] += p0 + p1;
        const __half2 hp = __floats2half2_rn(p0, p1);
        pk[i >> 1] = *reinterpret_cast<const uint32_t*>(&hp);
      }
      ptx::tmem_st_32x32b_x8(t_p + cc * 8, pk);
    }
    return ((sp[0] + sp[1]) + (sp[2] + sp[3])) + ((sp[4] + sp[5]) + (sp[6] + sp[7]));
  }
}

__global__ void __launch_bounds__(kAThreads, 1)
    attn_fused_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                      const __grid_constant__ CUtensorMap tvt, const AttnArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (ptx::smem_u32(smem_raw) & 1023) {  // uniform: every thread leaves before any barrier
    if (threadIdx.x == 0 && a.err) atomicCAS(a.err, 0, (int)BQ4_EALIGN);
    return;
  }
  uint8_t* smem = smem_raw;
  uint8_t* qs = smem;
  uint8_t* ks = qs + kATileB;          // [kAKV] stages
  uint8_t* vs = ks + kAKV * kATileB;   // [kAKV] stages
  float* xmax = reinterpret_cast<float*>(vs + kAKV * kATileB);  // [block parity][part][row]
  uint64_t* bars = reinterpret_cast<uint64_t*>(vs + kAKV * kATileB + kAXchg);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;          // [kAKV]
  uint64_t* k_empty = k_full + kAKV;    // [kAKV]
  uint64_t* v_full = k_empty + kAKV;    // [kAKV]
  uint64_t* v_empty = v_full + kAKV;    // [kAKV]
  uint64_t* s_full = v_empty + kAKV;    // [2]
  uint64_t* s_free = s_full + 2;        // [2]
  uint64_t* p_full = s_free + 2;
  uint64_t* p_free = p_full + 1;  // [2]: P_j v_j has completed (P buffer j % 2 free, O holds it)
  uint64_t* pair = p_free + 2;    // [4]: every softmax warp of a lane quarter has posted its part's max
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pair + 4);  // 24 barriers: 192 of the 256 bytes
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x / a.qtiles, qt = blockIdx.x - bh * a.qtiles;
  const int b = bh / a.Hq, h = bh - b * a.Hq;
  const int bkv = b * a.Hkv + h / (a.Hq / a.Hkv);
  const int nblk = a.nblk;

  if (threadIdx.x == 0) {
    ptx::mbar_init(q_full, 1);
    for (int i = 0; i < kAKV; ++i) {
      ptx::mbar_init(&k_full[i], 1);
      ptx::mbar_init(&k_empty[i], 1);
      ptx::mbar_init(&v_full[i], 1);
      ptx::mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(&s_full[i], 1);
      ptx::mbar_init(&s_free[i], kASoftWarps);
      ptx::mbar_init(&p_free[i], 1);
    }
    ptx::mbar_init(p_full, kASoftWarps);
    for (int i = 0; i < 4; ++i) ptx::mbar_init(&pair[i], kAParts);  // lane 0 of each part's warp
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, 512);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // S buffers at columns 0 and 128, O at 256, P buffers at 384 and 448

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      ptx::prefetch_tmap(&tq);
      ptx::prefetch_tmap(&tk);
      ptx::prefetch_tmap(&tvt);
      ptx::griddep_wait();
      const int qrow = bh * a.Sq + qt * 128;
      ptx::mbar_arrive_expect_tx(q_full, kATileB);
      ptx::tma_load_2d(qs, &tq, q_full, 0, qrow);
      ptx::tma_load_2d(qs + kASub, &tq, q_full, 64, qrow);
      for (int j = 0; j < nblk; ++j) {
        const int st = j % kAKV;
        const uint32_t ph = (j / kAKV) & 1;
        if (!attn_wait(&k_empty[st], ph ^ 1, abort_flag, a.err)) break;
        const int krow = bkv * a.Skv + j * 128;
        ptx::mbar_arrive_expect_tx(&k_full[st], kATileB);
        ptx::tma_load_2d(ks + st * kATileB, &tk, &k_full[st], 0, krow);
        ptx::tma_load_2d(ks + st * kATileB + kASub, &tk, &k_full[st], 64, krow);
        if (!attn_wait(&v_empty[st], ph ^ 1, abort_flag, a.err)) break;
        ptx::mbar_arrive_expect_tx(&v_full[st], kATileB);
        ptx::tma_load_2d(vs + st * kATileB, &tvt, &v_full[st], j * 128, bkv * 128);
        ptx::tma_load_2d(vs + st * kATileB + kASub, &tvt, &v_full[st], j * 128 + 64, bkv * 128);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      constexpr uint32_t idesc = ptx::umma_idesc_f16(128, 128);
      const uint32_t q_a = ptx::smem_u32(qs);
      bool ok = attn_wait(q_full, 0, abort_flag, a.err);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1, kst = j % kAKV;
        if (!attn_wait(&k_full[kst], (j / kAKV) & 1, abort_flag, a.err)) return false;
        if (j >= 2 && !attn_wait(&s_free[st], ((j >> 1) - 1) & 1, abort_flag, a.err)) return false;
        ptx::tc_fence_after();
        const uint32_t k_a = ptx::smem_u32(ks + kst * kATileB);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (uint32_t)(kk >> 2) * kASub + (uint32_t)(kk & 3) * 32;
          ptx::mma_f16_ss(tmem + st * 128, ptx::umma_desc_sw128(q_a + off), ptx::umma_desc_sw128(k_a + off), idesc,
                          kk > 0 ? 1u : 0u);
        }
        ptx::mma_commit(&s_full[st]);
        ptx::mma_commit(&k_empty[kst]);
        return true;
      };
      if (ok) ok = issue_s(0);
      if (ok && nblk > 1) ok = issue_s(1);
      for (int j = 0; ok && j < nblk; ++j) {
        const int st = j & 1, vst = j % kAKV;
        if (!attn_wait(p_full, j & 1, abort_flag, a.err) ||
            !attn_wait(&v_full[vst], (j / kAKV) & 1, abort_flag, a.err)) break;
        ptx::tc_fence_after();
        const uint32_t v_a = ptx::smem_u32(vs + vst * kATileB);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          // keys 16 kk .. 16 kk + 15: P columns 8 kk .. 8 kk + 7, v^T sub-tile kk / 4 at 32-byte step kk % 4
          const uint32_t off = (uint32_t)(kk >> 2) * kASub + (uint32_t)(kk & 3) * 32;
          ptx::mma_f16_ts(tmem + kATmemO, tmem + kATmemP + (uint32_t)st * 64 + (uint32_t)kk * 8,
                          ptx::umma_desc_sw128(v_a + off), idesc, (j > 0 || kk > 0) ? 1u : 0u);
        }
        ptx::mma_commit(&v_empty[vst]);
        ptx::mma_commit(&p_free[st]);
        if (j + 2 < nblk && !issue_s(j + 2)) break;
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------ softmax: kAParts threads per query row
    // Warps w, w + 4, ... share TMEM lane quarter w % 4 (rows 32 (w % 4) ..);
    // part p = (w - 4) / 4 takes score / output columns kACols p .. .  Per
    // block the parts post their max to shared memory and meet on pair[q],
    // so all use the same row max; each keeps its own partial sum.
    const int q = warp & 3, part = (warp - 4) >> 2;
    const int row = q * 32 + lane;
    const uint32_t t_quarter = tmem + ((uint32_t)(q * 32) << 16);
    const uint32_t t_lane = t_quarter + (uint32_t)(part * kACols);
    const float c = a.c;
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < nblk && ok; ++j) {
      const int st = j & 1;
      ok = __all_sync(0xffffffffu, attn_wait(&s_full[st], (j >> 1) & 1, abort_flag, a.err));
      if (!ok) break;
      ptx::tc_fence_after();
      const int valid = a.Skv - j * 128 - part * kACols;  // keys of this part (may be <= 0)
      uint32_t r[kACols];
#pragma unroll
      for (int cc = 0; cc < kACols / 16; ++cc) {
        uint32_t (&rc)[16] = *reinterpret_cast<uint32_t(*)[16]>(r + cc * 16);
        ptx::tmem_ld_32x32b_x16(t_lane + st * 128 + cc * 16, rc);
      }
      ptx::tmem_ld_wait();
      // S_j is in registers: its TMEM buffer may take S_{j+2}
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&s_free[st]);
      const bool full = valid >= kACols;  // warp-uniform: valid depends on the block and the part
      const float pm = full ? attn_rowmax<kACols, true>(r, valid) : attn_rowmax<kACols, false>(r, valid);
      xmax[(st * kAParts + part) * 128 + row] = pm;
      __syncwarp();  // the warp's slots are written before its lane 0 arrives
      if (lane == 0) ptx::mbar_arrive(&pair[q]);
      ok = __all_sync(0xffffffffu, attn_wait(&pair[q], j & 1, abort_flag, a.err));
      if (!ok) break;
      float rmax = pm;
#pragma unroll
      for (int p = 0; p < kAParts; ++p) rmax = fmaxf(rmax, xmax[(st * kAParts + p) * 128 + row]);
      const float mx = c * rmax;
      const bool jump = j == 0 || mx > m + kRescaleLog2;
      const float m_use = jump ? fmaxf(m, mx) : m;
      const float alpha = (j > 0 && jump) ? exp2f(m - m_use) : 1.0f;
      if (j >= 2) {
        // P buffer j % 2 was last read by P_{j-2} v_{j-2}
        ok = __all_sync(0xffffffffu, attn_wait(&p_free[st], ((j >> 1) - 1) & 1, abort_flag, a.err));
        if (!ok) break;
      }
      // this part's keys: kACols / 2 columns of P buffer j % 2
      const uint32_t t_p = t_quarter + kATmemP + (uint32_t)(st * 64 + part * (kACols / 2));
      const float psum = full ? attn_p_store<kACols, true>(r, valid, c, m_use, t_p)
                              : attn_p_store<kACols, false>(r, valid, c, m_use, t_p);
      if (j > 0 && __any_sync(0xffffffffu, jump)) {
        // O must hold P_{j-1} v_{j-1} before it is scaled (P_j v_j waits for p_full)
        ok = __all_sync(0xffffffffu, attn_wait(&p_free[(j - 1) & 1], ((j - 1) >> 1) & 1, abort_flag, a.err));
        if (!ok) break;
        ptx::tc_fence_after();
        uint32_t o[kACols];
#pragma unroll
        for (int cc = 0; cc < kACols / 16; ++cc) {
          uint32_t (&oc)[16] = *reinterpret_cast<uint32_t(*)[16]>(o + cc * 16);
          ptx::tmem_ld_32x32b_x16(t_lane + kATmemO + cc * 16, oc);
        }
        ptx::tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < kACols; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
#pragma unroll
        for (int cc = 0; cc < kACols / 16; ++cc) {
          const uint32_t (&oc)[16] = *reinterpret_cast<const uint32_t(*)[16]>(o + cc * 16);
          ptx::tmem_st_32x32b_x16(t_lane + kATmemO + cc * 16, oc);
        }
      }
      l = l * alpha + psum;
      m = m_use;
      ptx::tmem_st_wait();  // P (and a rescaled O) in TMEM before the MMA reads them
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(p_full);
    }
    // the last P v's commit covers every earlier MMA
    if (ok) ok = __all_sync(0xffffffffu, attn_wait(&p_free[(nblk - 1) & 1], ((nblk - 1) >> 1) & 1, abort_flag, a.err));
    if (ok) {
      // the row's sum: every part posts its own in the slot of block nblk (free:
      // block nblk - 2 used it, and every part has passed block nblk - 1)
      xmax[((nblk & 1) * kAParts + part) * 128 + row] = l;
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&pair[q]);
      ok = __all_sync(0xffffffffu, attn_wait(&pair[q], nblk & 1, abort_flag, a.err));
    }
    if (ok) {
      float lsum = 0.0f;
#pragma unroll
      for (int p = 0; p < kAParts; ++p) lsum += xmax[((nblk & 1) * kAParts + p) * 128 + row];
      const float inv = 1.0f / lsum;
      ptx::tc_fence_after();
      const int qrow = qt * 128 + row;
      float* o = a.out + ((size_t)bh * a.Sq + qrow) * 128 + part * kACols;
      uint32_t r[kACols];
#pragma unroll
      for (int cc = 0; cc < kACols / 16; ++cc) {
        uint32_t (&rc)[16] = *reinterpret_cast<uint32_t(*)[16]>(r + cc * 16);
        ptx::tmem_ld_32x32b_x16(t_lane + kATmemO + cc * 16, rc);
      }
      ptx::tmem_ld_wait();
      if (qrow < a.Sq) {
#pragma unroll
        for (int i = 0; i < kACols; i += 4)
          *reinterpret_cast<float4*>(o + i) =
              make_float4(__uint_as_float(r[i]) * inv, __uint_as_float(r[i + 1]) * inv,
                          __uint_as_float(r[i + 2]) * inv, __uint_as_float(r[i + 3]) * inv);
      }
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// Two query tiles per CTA (256 query rows), ping-ponging on the tensor core.
//
// With one tile, the tensor core waits for the softmax of every block: the
// scores of block j + 1 are ready early, but P_j v_j can only start once the
// softmax has finished block j, and the softmax's chain (TMEM load, row max,
// exponentials, P store) is about three times as long as the two MMAs of a
// block.  With two tiles A and B the MMA warp issues, per 128-key block j,
//     P_A(j) v_j,  S_A(j+1) = q_A k_{j+1}^T,  P_B(j) v_j,  S_B(j+1)
// so the tensor core runs one tile's MMAs while the other tile's softmax
// runs, and both tiles' exponentials share the MUFU unit.  Each P_t(j) v_j
// goes in two halves: keys 64..127 once the softmax has stored their
// probabilities (p_half), keys 0..63 once it has stored the rest (p_full),
// so half of the P v MMAs overlap the softmax's second exponential pass.
// (Measured on B200, one 128x128x16 tcgen05.mma takes about 108 cycles with
// both operands in shared memory and 95 with A in TMEM, against 64 of
// arithmetic: the S and P v MMAs of a tile's block take about 1600 cycles.)
//
//   warp 0        TMA: q_A, q_B once; k_j, v_j^T into a 2-stage ring.
//   warp 1        MMA issuer (one thread).
//   warps 4..7    softmax of tile A, warps 8..11 of tile B: one thread per
//                 query row (warp % 4 is the TMEM lane quarter), so the row
//                 max needs no exchange between threads.
// TMEM (512 columns): S_A 0..127, S_B 128..255 (f32), O_A 256..383, O_B
// 384..511.  P_t (f16 pairs, 64 columns) is written into columns 64..127 of
// S_t after the softmax has read them: keys 64..127 (in registers from the
// max pass) into columns 96..127, then keys 0..63 (read again from columns
// 0..63) into 64..95.
// Ordering, all from the issue order of one thread's tcgen05.mma (they
// execute in order) and from commits, which track every earlier MMA:
//   * S_t(j+1) overwrites P_t(j) only after P_t(j) v_j in issue order;
//   * s_full[t] completing for S_t(j) means P_t(j-1) v_{j-1} is done, so the
//     softmax may rescale O_t and overwrite the P_t columns right away;
//   * the MMA waits p_half[t] / p_full[t] (phase j) before the halves of
//     P_t(j) v_j; the softmax only waits s_full[t] (phase j) after arriving
//     at both for phase j-1, so no barrier runs more than one phase ahead of
//     its waiter;
//   * a rescale of O_t (a jump of the row max) is stored before p_half, so
//     no half of P_t(j) v_j adds into O_t before it is scaled.
// ---------------------------------------------------------------------------
constexpr int kPThreads = 384;
constexpr uint32_t kPSmem = 6 * kATileB + 256;  // q_A, q_B, k[2], vt[2], barriers
constexpr uint32_t kPColO = 256;
// Default share of the polynomial exponentials: none.  Measured at 24 heads x
// 4352 tokens (two tiles per CTA): 272.8 us with every exponential on
// ex2.approx, 278.8 / 286.4 / 299.3 us with one to three quarters on the FMA
// pipe -- the MUFU unit is not what limits the kernel.
constexpr int kAttnPolyQ = 0;

// Bounded wait that ignores the abort flag: for draining this CTA's own
// copies and MMAs before its shared memory and TMEM are released.
__device__ __forceinline__ void attn_drain(uint64_t* bar, uint32_t parity) {
  volatile int never = 0;
  (void)ptx::mbar_wait(bar, parity, &never);
}

__device__ __forceinline__ void attn_ld64(uint32_t taddr, uint32_t (&r)[64]) {
  ptx::tmem_ld_32x32b_x32(taddr, *reinterpret_cast<uint32_t(*)[32]>(r));
  ptx::tmem_ld_32x32b_x32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(r + 32));
  ptx::tmem_ld_wait();
}

// kPolyQ: quarters of each full block's exponentials taken on the FMA pipe.
template <int kPolyQ>
__global__ void __launch_bounds__(kPThreads, 1)
    attn_pp_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                   const __grid_constant__ CUtensorMap tvt, const AttnArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (ptx::smem_u32(smem_raw) & 1023) {  // uniform: every thread leaves before any barrier
    if (threadIdx.x == 0 && a.err) atomicCAS(a.err, 0, (int)BQ4_EALIGN);
    return;
  }
  uint8_t* qs = smem_raw;                // [2] query tiles
  uint8_t* ks = qs + 2 * kATileB;        // [kAKV]
  uint8_t* vs = ks + kAKV * kATileB;     // [kAKV]
  uint64_t* bars = reinterpret_cast<uint64_t*>(vs + kAKV * kATileB);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;           // [kAKV]
  uint64_t* k_empty = k_full + kAKV;     // [kAKV]
  uint64_t* v_full = k_empty + kAKV;     // [kAKV]
  uint64_t* v_empty = v_full + kAKV;     // [kAKV]
  uint64_t* s_full = v_empty + kAKV;     // [tile]
  uint64_t* p_half = s_full + 2;         // [tile]: P of keys 64..127 stored (lane 0 of the tile's 4 softmax warps)
  uint64_t* p_full = p_half + 2;         // [tile]: P of keys 0..63 stored
  uint64_t* o_done = p_full + 2;         // the last P_B v (and with it every MMA) has completed
  uint64_t* drain = o_done + 1;          // the MMA issuer's own end-of-work commit
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);  // 17 barriers: 136 of the 256 bytes
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x / a.qtiles, qt = blockIdx.x - bh * a.qtiles;
  const int b = bh / a.Hq, h = bh - b * a.Hq;
  const int bkv = b * a.Hkv + h / (a.Hq / a.Hkv);
  const int nblk = a.nblk;

  if (threadIdx.x == 0) {
    ptx::mbar_init(q_full, 1);
    for (int i = 0; i < kAKV; ++i) {
      ptx::mbar_init(&k_full[i], 1);
      ptx::mbar_init(&k_empty[i], 1);
      ptx::mbar_init(&v_full[i], 1);
      ptx::mbar_init(&v_empty[i], 1);
    }
    for (int t = 0; t < 2; ++t) {
      ptx::mbar_init(&s_full[t], 1);
      ptx::mbar_init(&p_half[t], 4);
      ptx::mbar_init(&p_full[t], 4);
    }
    ptx::mbar_init(o_done, 1);
    ptx::mbar_init(drain, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, 512);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      ptx::prefetch_tmap(&tq);
      ptx::prefetch_tmap(&tk);
      ptx::prefetch_tmap(&tvt);
      ptx::griddep_wait();
      const int qrow = bh * a.Sq + qt * 256;
      ptx::mbar_arrive_expect_tx(q_full, 2 * kATileB);
      for (int t = 0; t < 2; ++t) {
        ptx::tma_load_2d(qs + t * kATileB, &tq, q_full, 0, qrow + t * 128);
        ptx::tma_load_2d(qs + t * kATileB + kASub, &tq, q_full, 64, qrow + t * 128);
      }
      int k_issued = 0, v_issued = 0;  // blocks whose k / v loads were issued
      for (int j = 0; j < nblk; ++j) {
        const int st = j % kAKV;
        const uint32_t ph = (j / kAKV) & 1;
        if (!attn_wait(&k_empty[st], ph ^ 1, abort_flag, a.err)) break;
        const int krow = bkv * a.Skv + j * 128;
        ptx::mbar_arrive_expect_tx(&k_full[st], kATileB);
        ptx::tma_load_2d(ks + st * kATileB, &tk, &k_full[st], 0, krow);
        ptx::tma_load_2d(ks + st * kATileB + kASub, &tk, &k_full[st], 64, krow);
        k_issued = j + 1;
        if (!attn_wait(&v_empty[st], ph ^ 1, abort_flag, a.err)) break;
        ptx::mbar_arrive_expect_tx(&v_full[st], kATileB);
        ptx::tma_load_2d(vs + st * kATileB, &tvt, &v_full[st], j * 128, bkv * 128);
        ptx::tma_load_2d(vs + st * kATileB + kASub, &tvt, &v_full[st], j * 128 + 64, bkv * 128);
        v_issued = j + 1;
      }
      // every copy this thread started has landed before the CTA may exit
      // (on the normal path the MMAs consumed them all: these return at once)
      attn_drain(q_full, 0);
      for (int j = (k_issued > kAKV ? k_issued - kAKV : 0); j < k_issued; ++j)
        attn_drain(&k_full[j % kAKV], (j / kAKV) & 1);
      for (int j = (v_issued > kAKV ? v_issued - kAKV : 0); j < v_issued; ++j)
        attn_drain(&v_full[j % kAKV], (j / kAKV) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      constexpr uint32_t idesc = ptx::umma_idesc_f16(128, 128);
      const uint32_t q_a = ptx::smem_u32(qs);
      bool ok = attn_wait(q_full, 0, abort_flag, a.err);
      // S_t(j) = q_t k_j^T into columns 128 t; tile A is k_j's first reader, tile B its last
      auto issue_s = [&](int t, int j) -> bool {
        const int kst = j % kAKV;
        if (t == 0 && !attn_wait(&k_full[kst], (j / kAKV) & 1, abort_flag, a.err)) return false;
        ptx::tc_fence_after();
        const uint32_t k_a = ptx::smem_u32(ks + kst * kATileB), qa = q_a + (uint32_t)t * kATileB;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (uint32_t)(kk >> 2) * kASub + (uint32_t)(kk & 3) * 32;
          ptx::mma_f16_ss(tmem + (uint32_t)t * 128, ptx::umma_desc_sw128(qa + off), ptx::umma_desc_sw128(k_a + off),
                          idesc, kk > 0 ? 1u : 0u);
        }
        ptx::mma_commit(&s_full[t]);
        if (t == 1) ptx::mma_commit(&k_empty[kst]);
        return true;
      };
      // O_t (+)= P_t(j) v_j with P_t read from columns 128 t + 64 .. 127, in
      // two halves: keys 64..127 (P columns 96..127, K steps 4..7; the first
      // MMA of block 0 starts the accumulator) after p_half, keys 0..63
      // (columns 64..95) after p_full
      auto issue_pv = [&](int t, int j, int half) -> bool {
        const int vst = j % kAKV;
        if (!attn_wait_poll(half ? &p_full[t] : &p_half[t], j & 1, abort_flag, a.err)) return false;
        if (t == 0 && !half && !attn_wait(&v_full[vst], (j / kAKV) & 1, abort_flag, a.err)) return false;
        ptx::tc_fence_after();
        const uint32_t v_a = ptx::smem_u32(vs + vst * kATileB);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int kk = half ? i : 4 + i;
          const uint32_t off = (uint32_t)(kk >> 2) * kASub + (uint32_t)(kk & 3) * 32;
          ptx::mma_f16_ts(tmem + kPColO + (uint32_t)t * 128, tmem + (uint32_t)t * 128 + 64 + (uint32_t)kk * 8,
                          ptx::umma_desc_sw128(v_a + off), idesc, (j > 0 || half || i > 0) ? 1u : 0u);
        }
        if (t == 1 && half) {
          ptx::mma_commit(&v_empty[vst]);
          if (j == nblk - 1) ptx::mma_commit(o_done);
        }
        return true;
      };
      if (ok) ok = issue_s(0, 0);
      if (ok) ok = issue_s(1, 0);
      for (int j = 0; ok && j < nblk; ++j) {
        ok = issue_pv(0, j, 0) && issue_pv(0, j, 1);
        if (ok && j + 1 < nblk) ok = issue_s(0, j + 1);
        if (ok) ok = issue_pv(1, j, 0) && issue_pv(1, j, 1);
        if (ok && j + 1 < nblk) ok = issue_s(1, j + 1);
      }
      // every MMA this thread issued has completed before TMEM is released
      ptx::mma_commit(drain);
      attn_drain(drain, 0);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------ softmax: one thread per query row of tile t
    const int t = (warp - 4) >> 2, q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t t_lane = tmem + ((uint32_t)(q * 32) << 16);
    const uint32_t t_s = t_lane + (uint32_t)t * 128, t_o = t_lane + kPColO + (uint32_t)t * 128;
    const float c = a.c;
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    uint32_t r[64];
    for (int j = 0; j < nblk && ok; ++j) {
      // (a polling wait here, one lane per warp, measured slower: 252.2 vs 248.7 us)
      ok = __all_sync(0xffffffffu, attn_wait(&s_full[t], j & 1, abort_flag, a.err));
      if (!ok) break;
      ptx::tc_fence_after();
      const int valid0 = a.Skv - j * 128, valid1 = valid0 - 64;  // keys present in each 64-key half
      const bool full = valid0 >= 128;                           // warp-uniform
      attn_ld64(t_s, r);
      float pm = full ? attn_rowmax<64, true>(r, valid0) : attn_rowmax<64, false>(r, valid0);
      attn_ld64(t_s + 64, r);  // kept for the P pass
      pm = fmaxf(pm, full ? attn_rowmax<64, true>(r, valid1) : attn_rowmax<64, false>(r, valid1));
      const float mx = c * pm;
      const bool jump = j == 0 || mx > m + kRescaleLog2;
      const float m_use = jump ? fmaxf(m, mx) : m;
      const float alpha = (j > 0 && jump) ? exp2f(m - m_use) : 1.0f;
      if (j > 0 && __any_sync(0xffffffffu, jump)) {
        // O_t holds P_t(j-1) v_{j-1} (s_full's commit for S_t(j) covered it);
        // scaled 16 columns at a time, before any half of P_t(j) v_j is issued
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          uint32_t o[16];
          ptx::tmem_ld_32x32b_x16(t_o + cc * 16, o);
          ptx::tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          ptx::tmem_st_32x32b_x16(t_o + cc * 16, o);
        }
      }
      // keys 64..127 -> P columns 96..127 (S columns already read): their half of P v may start
      float psum = full ? attn_p_store<64, true, kPolyQ>(r, valid1, c, m_use, t_s + 96)
                        : attn_p_store<64, false>(r, valid1, c, m_use, t_s + 96);
      ptx::tmem_st_wait();  // P (and a rescaled O) in TMEM before the MMA reads them
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&p_half[t]);
      // keys 0..63 (read again) -> P columns 64..95
      attn_ld64(t_s, r);
      psum += full ? attn_p_store<64, true, kPolyQ>(r, valid0, c, m_use, t_s + 64)
                   : attn_p_store<64, false>(r, valid0, c, m_use, t_s + 64);
      l = l * alpha + psum;
      m = m_use;
      ptx::tmem_st_wait();
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&p_full[t]);
    }
    if (ok) ok = __all_sync(0xffffffffu, attn_wait(o_done, 0, abort_flag, a.err));
    if (ok) {
      ptx::tc_fence_after();
      const float inv = 1.0f / l;
      const int qrow = qt * 256 + t * 128 + row;
      float* o = a.out + ((size_t)bh * a.Sq + qrow) * 128;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        attn_ld64(t_o + half * 64, r);
        if (qrow < a.Sq) {
#pragma unroll
          for (int i = 0; i < 64; i += 4)
            *reinterpret_cast<float4*>(o + half * 64 + i) =
                make_float4(__uint_as_float(r[i]) * inv, __uint_as_float(r[i + 1]) * inv,
                            __uint_as_float(r[i + 2]) * inv, __uint_as_float(r[i + 3]) * inv);
        }
      }
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, 512);
  }
}

// v [B*Hkv][Skv][128] f16 -> v^T [B*Hkv][128][pitch] f16, zero for keys >= Skv
// (pitch a multiple of 128; v 16-byte aligned, rows of 256 bytes).  One CTA
// per 64 keys of one kv head: 16-byte loads of whole key rows into shared
// memory; then thread i takes the column pair d = 2 (i % 64), d + 1 and keys
// 16 (i / 64) .. + 15: it reads each key's (d, d + 1) pair as one 32-bit word
// (the lanes of a warp read 128 consecutive bytes of a key row), splits the
// pairs with byte permutes, and writes 32 bytes to each of the two v^T rows.
__global__ void __launch_bounds__(256) attn_vt_kernel(const uint16_t* __restrict__ v, int Skv, int pitch,
                                                      uint16_t* __restrict__ vt) {
  __shared__ __align__(16) uint16_t tile[64][136];  // [key][d], rows padded to 272 bytes
  const int j0 = blockIdx.x * 64, bk = blockIdx.y;
  uint4 val[4];  // all four loads in flight before the first store
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = (int)threadIdx.x + 256 * r, key = i >> 4, c = i & 15;
    val[r] = make_uint4(0, 0, 0, 0);
    if (j0 + key < Skv) val[r] = __ldg(reinterpret_cast<const uint4*>(v + ((size_t)bk * Skv + j0 + key) * 128) + c);
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = (int)threadIdx.x + 256 * r;
    *reinterpret_cast<uint4*>(&tile[i >> 4][(i & 15) * 8]) = val[r];
  }
  __syncthreads();
  const int d = 2 * (threadIdx.x & 63), k0 = 16 * (threadIdx.x >> 6);
  uint32_t lo[8], hi[8];  // keys k0 + 2 u, + 1 of column d (lo) and d + 1 (hi)
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const uint32_t a = *reinterpret_cast<const uint32_t*>(&tile[k0 + 2 * u][d]);
    const uint32_t b = *reinterpret_cast<const uint32_t*>(&tile[k0 + 2 * u + 1][d]);
    lo[u] = __byte_perm(a, b, 0x5410);
    hi[u] = __byte_perm(a, b, 0x7632);
  }
  uint4* d0 = reinterpret_cast<uint4*>(vt + ((size_t)bk * 128 + d) * pitch + j0 + k0);
  uint4* d1 = reinterpret_cast<uint4*>(vt + ((size_t)bk * 128 + d + 1) * pitch + j0 + k0);
  d0[0] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  d0[1] = make_uint4(lo[4], lo[5], lo[6], lo[7]);
  d1[0] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
  d1[1] = make_uint4(hi[4], hi[5], hi[6], hi[7]);
}

typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                             const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                             CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn attn_encode_fn() {
  static const EncodeFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeFn>(p);
    return static_cast<EncodeFn>(nullptr);
  }();
  return fn;
}

// [rows][cols] f16 at row pitch `pitch` elements, box {64, 128}, 128-byte swizzle.
bool attn_tmap(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint64_t pitch) {
  EncodeFn enc = attn_encode_fn();
  if (!enc) return false;
  cuuint64_t gdim[2] = {cols, rows};
  cuuint64_t gstride[1] = {pitch * 2};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t es[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), gdim, gstride, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// The fused kernel addresses rows of q ([B*Hq*Sq][128]) and k ([B*Hkv*Skv][128])
// by 32-bit TMA coordinates, and the v transpose puts B*Hkv on grid y.
bq4_status attn_fused_check(int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Skv) {
  constexpr int64_t kRowLimit = ((int64_t)1 << 31) - 256;
  if (B * Hq * Sq > kRowLimit || B * Hkv * Skv > kRowLimit || B * Hkv > 65535)
    return set_error(BQ4_EINVAL_SHAPE,
                     "fused attention: B*Hq*Sq=%lld and B*Hkv*Skv=%lld must be < 2^31 - 256, B*Hkv=%lld <= 65535",
                     (long long)(B * Hq * Sq), (long long)(B * Hkv * Skv), (long long)(B * Hkv));
  return BQ4_OK;
}

size_t attn_fused_workspace(int64_t B, int64_t Hkv, int64_t Skv) {
  const int64_t pitch = (Skv + 127) / 128 * 128;
  return (size_t)(B * Hkv * 128 * pitch * 2 + 255) / 256 * 256;
}

bq4_status attn_fused(const uint16_t* q, const uint16_t* k, const uint16_t* v, int64_t B, int64_t Hq, int64_t Hkv,
                      int64_t Sq, int64_t Skv, float scale, float* out, void* workspace, cudaStream_t s) {
  const int64_t pitch = (Skv + 127) / 128 * 128;
  uint16_t* vt = static_cast<uint16_t*>(workspace);
  attn_vt_kernel<<<dim3((unsigned)(pitch / 64), (unsigned)(B * Hkv)), 256, 0, s>>>(v, (int)Skv, (int)pitch, vt);
  note_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return check_cuda(e, "attention v transpose launch");
  CUtensorMap tq, tk, tvt;
  if (!attn_tmap(&tq, q, 128, (uint64_t)(B * Hq * Sq), 128) || !attn_tmap(&tk, k, 128, (uint64_t)(B * Hkv * Skv), 128) ||
      !attn_tmap(&tvt, vt, (uint64_t)pitch, (uint64_t)(B * Hkv * 128), (uint64_t)pitch))
    return set_error(BQ4_ECUDA, "cuTensorMapEncodeTiled failed for the attention operands");
  // Two query tiles per CTA whenever a head has more than one 128-row tile
  // (BQ4_ATTN_ONE_TILE=1 keeps one tile per CTA); BQ4_ATTN_POLY=0..3 sets how
  // many quarters of its exponentials take the FMA-pipe polynomial.
  const bool two = Sq > 128 && !getenv("BQ4_ATTN_ONE_TILE");
  int poly = kAttnPolyQ;
  if (const char* f = getenv("BQ4_ATTN_POLY")) {
    const int v = atoi(f);
    if (v >= 0 && v <= 3) poly = v;
  }
  auto pp = poly == 0 ? attn_pp_kernel<0> : poly == 1 ? attn_pp_kernel<1> : poly == 2 ? attn_pp_kernel<2>
                                                                                       : attn_pp_kernel<3>;
  AttnArgs a;
  a.out = out;
  a.Sq = (int)Sq;
  a.Skv = (int)Skv;
  a.Hq = (int)Hq;
  a.Hkv = (int)Hkv;
  a.qtiles = (int)(two ? (Sq + 255) / 256 : (Sq + 127) / 128);
  a.nblk = (int)((Skv + 127) / 128);
  a.c = scale * 1.4426950408889634f;  // log2(e): exp(x) = exp2(x log2 e)
  a.err = device_error_word();
  static std::atomic<int> attr_set[64];  // per-device function attributes (bit 0 one tile, 1 + poly two), set once
  int dev = 0;
  cudaGetDevice(&dev);
  const int bit = two ? 2 << poly : 1;
  if (dev < 0 || dev >= 64 || !(attr_set[dev].load(std::memory_order_relaxed) & bit)) {
    e = two ? cudaFuncSetAttribute(pp, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPSmem)
            : cudaFuncSetAttribute(attn_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kASmem);
    if (e != cudaSuccess) return check_cuda(e, "attention shared-memory attribute");
    if (dev >= 0 && dev < 64) attr_set[dev].fetch_or(bit, std::memory_order_relaxed);
  }
  if (two)
    pp<<<(unsigned)(B * Hq * a.qtiles), kPThreads, kPSmem, s>>>(tq, tk, tvt, a);
  else
    attn_fused_kernel<<<(unsigned)(B * Hq * a.qtiles), kAThreads, kASmem, s>>>(tq, tk, tvt, a);
  note_launch();
  return check_cuda(cudaGetLastError(), "fused attention launch");
}

}  // namespace bq4
