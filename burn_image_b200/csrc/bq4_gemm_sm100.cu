// bq4_gemm_sm100.cu -- packed signed-Q4 x f16 GEMM on the 5th-generation
// tensor cores (tcgen05 + TMEM), sm_100a only.
//
// Computes y[M,N] = epilogue(x[M,K] . W[K,N]) for a prepared Q4 weight W.
// Swap-AB formulation: the MMA "A" operand is a 128-row tile of output
// features (dequantized weights, K-major), the "B" operand is a BT-row tile
// of tokens (f16 activations, K-major), so D[n, m] accumulates in TMEM with
// TMEM lane = output feature and TMEM column = token.
//
// One CTA of 896 threads per SM, persistent over (M tile, N tile) units; the
// warp roles are described above q4_gemm_ws_kernel.  Split-K units of one
// tile run as one thread-block cluster: each split writes its partial tile
// to the workspace, and after one cluster barrier every CTA sums its share
// of the token columns over the splits, reading through L2.
//
// Numerics: activations staged as f16 (round to nearest even), f32
// accumulation; weights either exact (q in f16, the f32 partial of each K
// block multiplied by its scale) or folded (f16(q * f16(scale)), the staging
// of the reference GPU kernel, patches/burn-cubecl-0.21.0/src/kernel/matmul/
// quantized.rs:172-178: lhs and rhs stage dtypes f16, f32 accumulation).
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
// Lockstep variant (exact mode, 128-blocks, no more stages than partials):
// a segment is exactly one stage and uses the partial buffer of the same
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
constexpr int kMaxSplit = 8;  // split-K factor limit: the portable cluster size

struct WsArgs {
  const uint32_t* q[2];
  const float* s[2];
  const uint16_t* h[2];
  const float* bias[2];
  const float* aux;
  float* partials;         // split-K: f32 partial tiles [tiles][ksplit][NW][BT][128] (workspace)
  void* y;                 // f32 or f16 (y_f16), row pitch ldy elements
  int y_f16, ldy;
  int M, N;
  int nkc, nkb, block;
  int ntiles, mtiles, ksplit, units;
  int tile0;               // first tile of this launch (the split-K tail launch starts past the whole tiles)
  int nfast;               // 1: N tile varies fastest along the unit order
  int yvec;                // 1: y rows 16-byte aligned (float4 stores in the split epilogue)
  int stages, rs;          // operand ring and raw ring depths
  int exact, pre, act;
  int lockstep;            // exact, 128-blocks, stage s accumulates into TMEM partial s (see below)
  // Stream-K tail (whole-K units only): tiles [dp_tiles, dp_tiles + sk_tiles)
  // are dealt to the CTAs as equal ranges of sk_w 128-K stages; a tile cut
  // between CTAs c-1 and c is finished by c from the partial c-1 published.
  int dp_tiles, sk_tiles;
  int sk_w;                // grid * sk_w < 2^31 (checked by the planner)
  float* sk_part;          // [grid][NW][BT][128] f32: slot c = partial for CTA c
  unsigned* sk_flag;       // [grid]: slot c = 1 once sk_part[c] is complete (zeroed per call)
  // QK-norm + RoPE epilogue (kernels built with QK): every 128-feature N
  // tile is one head; tiles [0, qk_q) are q heads, [qk_q, qk_q + qk_k) k
  // heads, the rest pass through.  cos_t / sin_t [M][128] at row pitch
  // ld_rope (NULL: no rotation); gamma_q / gamma_k [128] (NULL: ones).
  int qk_q, qk_k, ld_rope;
  // Row scatter (kernels built with SC): row m goes to sc_y[m / sc_rows] at
  // row sc_rank * sc_rows + m % sc_rows (the owner's receive buffer, f32, pitch ldy).
  float* sc_y[BQ4_MAX_PEERS];
  int sc_rows, sc_rank;
  // Convolution (kernels built with CV): token m is position m of the
  // zero-padded NHWC image stack, [batch][cv_hp][cv_wp] positions of
  // cv_cchunks * 32 channels.  Chunk kc reads tap kc / cv_cchunks
  // (ky = tap / cv_kw, kx = tap % cv_kw) from the token rows shifted by
  // ky * cv_dy + kx * cv_dx, channels (kc % cv_cchunks) * 32..; chunks past
  // cv_taps taps read zeros.  Output NCHW f32 [batch][N][cv_oh][cv_ow];
  // positions with py >= cv_oh or px >= cv_ow are not stored.
  int cv_cchunks, cv_taps, cv_kw, cv_dy, cv_dx;
  int cv_hp, cv_wp, cv_oh, cv_ow;
  float qk_eps;
  const float* gamma_q;
  const float* gamma_k;
  const float* cos_t;
  const float* sin_t;
  uint32_t raw_s_bytes;    // folded: scale bytes per weight per raw stage
  uint32_t raw_w_bytes;    // raw stage bytes per weight
};

__device__ __forceinline__ void store_y(const WsArgs& a, int m, int n, float v) {
  if (a.y_f16)
    reinterpret_cast<__half*>(a.y)[(size_t)m * a.ldy + n] = __float2half_rn(v);
  else
    reinterpret_cast<float*>(a.y)[(size_t)m * a.ldy + n] = v;
}

// Output element (m, n); kernels built with SC (row scatter) write row m to
// its owner rank's receive buffer sc_y[m / sc_rows] at row
// sc_rank * sc_rows + m % sc_rows (f32, pitch ldy).  Without SC, store_y.
template <bool SC>
__device__ __forceinline__ void store_out(const WsArgs& a, int m, int n, float v) {
  if constexpr (SC) {
    const int owner = m / a.sc_rows;
    a.sc_y[owner][(size_t)(a.sc_rank * a.sc_rows + (m - owner * a.sc_rows)) * a.ldy + n] = v;
  } else {
    store_y(a, m, n, v);
  }
}

// Convolution: the TMA coordinates (channel column x, token row y) of chunk
// kc for the token tile starting at row m0 (see WsArgs::cv_*).  A chunk past
// the last tap (K padding) starts at row M: the whole box is out of bounds
// and reads zeros.
__device__ __forceinline__ void cv_coord(const WsArgs& a, int kc, int ck, int m0, int& x, int& y) {
  const int tap = kc / a.cv_cchunks;
  if (tap >= a.cv_taps) {
    x = 0;
    y = a.M;
    return;
  }
  const int ky = tap / a.cv_kw;
  x = (kc - tap * a.cv_cchunks) * ck;
  y = m0 + ky * a.cv_dy + (tap - ky * a.cv_kw) * a.cv_dx;
}

// Unit u -> (tile, split) and its chunk range [kc0, kc1); splits cut at
// stage (2-chunk) boundaries.  With ksplit > 1 the grid has one CTA per unit
// and the ksplit units of a tile form one cluster (split == cluster rank).
__device__ __forceinline__ void ws_unit(const WsArgs& a, int u, int& tile, int& split, int& kc0, int& kc1) {
  tile = u / a.ksplit;
  split = u - tile * a.ksplit;
  const int nks = a.nkc >> 1;
  kc0 = 2 * (int)((int64_t)split * nks / a.ksplit);
  kc1 = 2 * (int)((int64_t)(split + 1) * nks / a.ksplit);
}

// Tile -> (M tile, N tile).  Consecutive tiles run in the same wave; the
// planner makes the operand that is larger in HBM (f16 tokens vs Q4 weights)
// the one a wave shares, so it is read from DRAM about once.
__device__ __forceinline__ void ws_tile(const WsArgs& a, int tile, int& mtile, int& ntile) {
  tile += a.tile0;
  if (a.nfast) {
    mtile = tile / a.ntiles;
    ntile = tile - mtile * a.ntiles;
  } else {
    ntile = tile / a.mtiles;
    mtile = tile - ntile * a.mtiles;
  }
}

// Segment boundaries inside [kc0, kc1): exact mode cuts at K-block edges
// (cpb chunks per block); folded mode keeps the unit whole (cpb = 0).
__device__ __forceinline__ bool ws_seg_first(int kc, int kc0, int cpb) {
  return kc == kc0 || (cpb > 0 && (kc % cpb) == 0);
}
__device__ __forceinline__ bool ws_seg_last(int kc, int kc1, int cpb) {
  return kc == kc1 - 1 || (cpb > 0 && ((kc + 1) % cpb) == 0);
}

// One unit of a CTA's work: tile, 64-K chunk range, and what the scaler
// does with the result.
constexpr int kUnitFull = 0;  // whole K range (or a split-K unit): epilogue
constexpr int kUnitHead = 1;  // stream-K: first part of a tile's K range, published for CTA c+1
constexpr int kUnitTail = 2;  // stream-K: rest of the K range, finished with CTA c-1's partial
struct Unit {
  int tile, split, kc0, kc1, kind;
};

// The i-th unit of this CTA; false past the last.  Every role walks the same
// list.  kSK = false compiles only whole-tile and split-K units (kernels the
// planner never gives a stream-K tail), keeping the roles' loops lean.
// Stream-K order: the head piece of the CTA's last tile first (its
// partial is then ready long before CTA c+1 needs it), whole tiles next,
// the tail piece of its first tile last (CTA c-1 published that tile's head
// partial as its own first unit).  Ranges are at least one tile long, so a
// tile is cut at most once.
// The loop every role runs over its units.  Without stream-K it is the
// plain persistent loop u = blockIdx.x, blockIdx.x + gridDim.x, ...; with
// it, the i-th unit of cta_unit.  COND is the role's extra loop condition.
#define BQ4_FOR_UNITS(COND)                                                          \
  Unit un;                                                                           \
  for (int i = 0, u_ = (int)blockIdx.x;                                              \
       (COND) && (kSK ? cta_unit<kSK>(a, i, un) : unit_at(a, u_, un));               \
       ++i, u_ += (int)gridDim.x)

template <bool kSK>
__device__ __forceinline__ bool cta_unit(const WsArgs& a, int i, Unit& un);

// Whole-tile (or split-K) unit number u of the persistent loop.
__device__ __forceinline__ bool unit_at(const WsArgs& a, int u, Unit& un) {
  if (u >= a.units) return false;
  un.kind = kUnitFull;
  ws_unit(a, u, un.tile, un.split, un.kc0, un.kc1);
  return true;
}

template <bool kSK>
__device__ __forceinline__ bool cta_unit(const WsArgs& a, int i, Unit& un) {
  const int c = (int)blockIdx.x, P = (int)gridDim.x;
  un.split = 0;
  un.kind = kUnitFull;
  if (a.ksplit > 1) {  // one split-K unit per CTA
    if (i) return false;
    ws_unit(a, c, un.tile, un.split, un.kc0, un.kc1);
    return true;
  }
  un.kc0 = 0;
  un.kc1 = a.nkc;
  if (!kSK || a.sk_tiles == 0) {
    un.tile = c + i * P;
    return un.tile < a.units;
  }
  const int nks = a.nkc >> 1;
  const int s0 = c * a.sk_w / P, s1 = (c + 1) * a.sk_w / P;
  const int t0 = s0 / nks, t1 = (s1 - 1) / nks;
  const bool tail = (s0 % nks) != 0, head = (s1 % nks) != 0;
  const int ndp = c < a.dp_tiles ? (a.dp_tiles - 1 - c) / P + 1 : 0;
  const int f0 = tail ? t0 + 1 : t0, f1 = head ? t1 - 1 : t1;
  const int nfull = f1 >= f0 ? f1 - f0 + 1 : 0;
  int k = i;
  if (head) {
    if (k == 0) {
      un.tile = a.dp_tiles + t1;
      un.kc1 = 2 * (s1 - t1 * nks);
      un.kind = kUnitHead;
      return true;
    }
    --k;
  }
  if (k < ndp) {
    un.tile = c + k * P;
    return true;
  }
  k -= ndp;
  if (k < nfull) {
    un.tile = a.dp_tiles + f0 + k;
    return true;
  }
  k -= nfull;
  if (tail && k == 0) {
    un.tile = a.dp_tiles + t0;
    un.kc0 = 2 * (s0 - t0 * nks);
    un.kind = kUnitTail;
    return true;
  }
  return false;
}

// Stream-K head piece: publish this CTA's partial tile for CTA c+1.  Each
// scaler warp arrives on `pub_bar` after its stores; thread 0 then raises
// the flag (release at GPU scope).  Used at most once per launch (parity 0).
template <int BT, int NW, int kCols>
__device__ __forceinline__ void sk_publish(const WsArgs& a, const float (&acc)[NW][kCols], int row, int col0,
                                           uint64_t* pub_bar, volatile int* abort_flag) {
  float* part = a.sk_part + (size_t)(blockIdx.x + 1) * NW * BT * 128;
#pragma unroll
  for (int w = 0; w < NW; ++w)
#pragma unroll
    for (int j = 0; j < kCols; ++j) __stcg(part + ((size_t)w * BT + col0 + j) * 128 + row, acc[w][j]);
  __threadfence();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) ptx::mbar_arrive(pub_bar);
  if (threadIdx.x == 0) {
    if (ptx::mbar_wait(pub_bar, 0, abort_flag)) {
      __threadfence();
      asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(a.sk_flag + blockIdx.x + 1), "r"(1u) : "memory");
    } else {
      record_error_flag(abort_flag, BQ4_ETIMEOUT);
    }
  }
}

// Stream-K tail piece (always the CTA's last unit, so its operand ring is
// idle): thread 0 waits (bounded) for CTA c-1's flag, then bulk-copies the
// head partial into the ring, counted on `tail_bar`; every scaler thread
// then folds it in from shared memory first: acc = head + tail, a fixed
// order.  On a timeout thread 0 still arrives, so nobody waits twice.
template <int BT, int NW, int kCols>
__device__ __forceinline__ bool sk_absorb(const WsArgs& a, float (&acc)[NW][kCols], int row, int col0,
                                          uint8_t* ring, uint64_t* tail_bar, volatile int* abort_flag) {
  constexpr uint32_t kBytes = NW * BT * 128 * sizeof(float);
  constexpr uint32_t kChunk = kBytes < 32768u ? kBytes : 32768u;
  if (threadIdx.x == 0) {
    const unsigned* f = a.sk_flag + blockIdx.x;
    const uint64_t t0 = ptx::globaltimer();
    bool ready = false;
    while (true) {
      unsigned v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
      if (v) {
        ready = true;
        break;
      }
      if (*abort_flag || ptx::globaltimer() - t0 > ptx::kWaitTimeoutNs) {
        record_error_flag(abort_flag, BQ4_ETIMEOUT);
        break;
      }
      __nanosleep(64);
    }
    if (ready) {
      // the partial was written through the generic proxy; the copy reads it
      // through the async proxy
      asm volatile("fence.proxy.async.global;" ::: "memory");
      ptx::mbar_arrive_expect_tx(tail_bar, kBytes);
      const uint8_t* src = reinterpret_cast<const uint8_t*>(a.sk_part + (size_t)blockIdx.x * NW * BT * 128);
#pragma unroll 1
      for (uint32_t o = 0; o < kBytes; o += kChunk) ptx::bulk_load(ring + o, src + o, kChunk, tail_bar);
    } else {
      ptx::mbar_arrive(tail_bar);
    }
  }
  if (!ptx::mbar_wait(tail_bar, 0, abort_flag) || *abort_flag) return false;
  const float* part = reinterpret_cast<const float*>(ring);
#pragma unroll
  for (int w = 0; w < NW; ++w)
#pragma unroll
    for (int j = 0; j < kCols; ++j) acc[w][j] = part[(w * BT + col0 + j) * 128 + row] + acc[w][j];
  return true;
}

// QK-norm + RoPE on one q or k head tile, in place on the register
// epilogue's values (the reference applies it between the projections and
// attention: crates/burn_boogu/src/model/attention.rs:114-133, 916-928).
// Thread (quad q, lane l) of column quarter c holds feature row 32q + l of
// the head for kCols tokens.  Per token the squares are summed over the 128
// rows: for each chunk of 16 columns a reduce-scatter butterfly (masks
// 16..2, then an xor-1 add) leaves lanes 2i and 2i+1 the warp's sum of the
// chunk's column i; the four quad warps of the quarter add theirs through
// `scratch` (double-buffered by use parity, one bounded mbarrier wait per
// use); the inverse RMS goes back to every lane by shuffle.  Then
// v = v * inv * gamma[row] and the interleaved-pair rotation with the
// partner row (lane ^ 1).
template <int BT, int kCols>
__device__ __forceinline__ bool qk_epilogue(const WsArgs& a, float (&v)[kCols], int row, int mtile, int col0,
                                            bool is_q, float* scratch, uint64_t* qk_bars, uint32_t& uses,
                                            volatile int* abort_flag) {
  constexpr int kChunks = kCols / 16;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, quad = warp & 3, quarter = warp >> 2;
  float* sc = scratch + (size_t)(((uses & 1) * 4 + quarter) * 4) * kCols;  // [quad][kCols]
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    float r[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) r[i] = v[16 * c + i] * v[16 * c + i];
#pragma unroll
    for (int half = 8, mask = 16; half >= 1; half >>= 1, mask >>= 1) {
      const bool up = (lane & mask) != 0;
#pragma unroll
      for (int i = 0; i < half; ++i) {
        const float send = up ? r[i] : r[half + i];
        const float keep = up ? r[half + i] : r[i];
        r[i] = keep + __shfl_xor_sync(0xffffffffu, send, mask);
      }
    }
    r[0] += __shfl_xor_sync(0xffffffffu, r[0], 1);
    if ((lane & 1) == 0) sc[quad * kCols + 16 * c + (lane >> 1)] = r[0];
  }
  __syncwarp();
  if (lane == 0) ptx::mbar_arrive(&qk_bars[quarter]);
  if (!ptx::mbar_wait(&qk_bars[quarter], uses & 1, abort_flag)) return false;
  ++uses;
  float inv[kChunks];
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int col = 16 * c + (lane >> 1);
    const float tot = ((sc[col] + sc[kCols + col]) + sc[2 * kCols + col]) + sc[3 * kCols + col];
    inv[c] = 1.0f / sqrtf(tot * (1.0f / 128.0f) + a.qk_eps);
  }
  const float* gp = is_q ? a.gamma_q : a.gamma_k;
  const float g = gp ? __ldg(gp + row) : 1.0f;
#pragma unroll
  for (int j = 0; j < kCols; ++j) v[j] = v[j] * __shfl_sync(0xffffffffu, inv[j / 16], 2 * (j % 16)) * g;
  if (a.cos_t) {
    // 8 tokens at a time, every table load issued before any is used (one
    // L2 round trip per 8 tokens instead of per token)
    const bool odd = (row & 1) != 0;
    const int m0 = mtile * BT + col0;
#pragma unroll
    for (int c = 0; c < kCols; c += 8) {
      float cs[8], sn[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int m = m0 + c + i < a.M ? m0 + c + i : a.M - 1;
        cs[i] = __ldg(a.cos_t + (size_t)m * a.ld_rope + row);
        sn[i] = __ldg(a.sin_t + (size_t)m * a.ld_rope + row);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float partner = __shfl_xor_sync(0xffffffffu, v[c + i], 1);
        v[c + i] = odd ? v[c + i] * cs[i] + partner * sn[i] : v[c + i] * cs[i] - partner * sn[i];
      }
    }
  }
  return true;
}

// Split-K reduction across the cluster (one CTA per split, cluster rank =
// split).  After the main loop each split writes its f32 partial tile to its
// own slot of the workspace, partials[tile][split][w][col][row] (coalesced
// along the features); after one cluster barrier CTA r owns the token columns
// [c0_r, c1_r), c0_r = BT*r/splits, sums them over the splits in rank order
// (deterministic) reading through L2, and runs the epilogue.  (An exchange
// through distributed shared memory moved only ~28 GB/s per SM.)
template <int BT, int NW, int kCols>
__device__ __forceinline__ void split_publish(const WsArgs& a, int tile, int split, const float (&acc)[NW][kCols],
                                              int row, int col0) {
  float* part = a.partials + ((size_t)tile * a.ksplit + split) * NW * BT * 128;
#pragma unroll
  for (int w = 0; w < NW; ++w)
#pragma unroll
    for (int j = 0; j < kCols; ++j) __stcg(part + ((size_t)w * BT + col0 + j) * 128 + row, acc[w][j]);
  __threadfence();
}

// Owner side: warp w takes every 16th owned column from c0 + w, lane l the
// features 4l..4l+3 (bias loaded once); all splits' loads of a column are in
// flight before they are summed.
template <int BT, int NW, bool SC>
__device__ __forceinline__ void split_reduce_epilogue(const WsArgs& a) {
  const int SPL = a.ksplit;
  const int rank = (int)ptx::cluster_ctarank();
  const int tile = (int)blockIdx.x / SPL;
  int mtile, ntile;
  ws_tile(a, tile, mtile, ntile);
  const int c0 = BT * rank / SPL, c1 = BT * (rank + 1) / SPL;
  const int r4 = (int)(threadIdx.x & 31) * 4;
  const int n = ntile * 128 + r4;
  if (n >= a.N) return;
  float b[NW][4];
#pragma unroll
  for (int w = 0; w < NW; ++w)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int nn = n + i < a.N ? n + i : a.N - 1;
      b[w][i] = a.bias[w] ? __ldg(a.bias[w] + nn) : 0.0f;
    }
  const float* part = a.partials + (size_t)tile * SPL * NW * BT * 128;
  const int act = a.act;
  // bias, activation (or the gated pair) and the store of token m's four features
  auto emit = [&](int m, const float (&v)[NW][4]) {
    float o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (NW == 2) {
        o[i] = silu(v[0][i] + b[0][i]) * (v[NW - 1][i] + b[NW - 1][i]);
      } else {
        o[i] = apply_act(v[0][i] + b[0][i], act);
        if (a.aux) o[i] *= __ldg(a.aux + (size_t)m * a.N + (n + i < a.N ? n + i : a.N - 1));
      }
    }
    if (!SC && a.yvec && n + 3 < a.N) {
      if (a.y_f16) {
        const __half2 h01 = __floats2half2_rn(o[0], o[1]), h23 = __floats2half2_rn(o[2], o[3]);
        *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(a.y) + (size_t)m * a.ldy + n) =
            make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h23));
      } else {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(a.y) + (size_t)m * a.ldy + n) =
            make_float4(o[0], o[1], o[2], o[3]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (n + i < a.N) store_out<SC>(a, m, n + i, o[i]);
    }
  };
  int col = c0 + (int)(threadIdx.x >> 5);
  if constexpr (NW == 1) {
    // two of the warp's columns (col, col + 16) per round: every split's
    // loads of both are in flight before either is summed (one L2 latency
    // per two columns; the sums keep the split order)
    for (; col + 16 < c1 && mtile * BT + col + 16 < a.M; col += 32) {
      float4 t0[kMaxSplit], t1[kMaxSplit];
#pragma unroll
      for (int p = 0; p < kMaxSplit; ++p)
        if (p < SPL) {
          t0[p] = __ldcg(reinterpret_cast<const float4*>(part + ((size_t)p * BT + col) * 128 + r4));
          t1[p] = __ldcg(reinterpret_cast<const float4*>(part + ((size_t)p * BT + col + 16) * 128 + r4));
        }
      float v0[1][4] = {{0.0f, 0.0f, 0.0f, 0.0f}}, v1[1][4] = {{0.0f, 0.0f, 0.0f, 0.0f}};
#pragma unroll
      for (int p = 0; p < kMaxSplit; ++p)
        if (p < SPL) {
          v0[0][0] += t0[p].x; v0[0][1] += t0[p].y; v0[0][2] += t0[p].z; v0[0][3] += t0[p].w;
          v1[0][0] += t1[p].x; v1[0][1] += t1[p].y; v1[0][2] += t1[p].z; v1[0][3] += t1[p].w;
        }
      emit(mtile * BT + col, v0);
      emit(mtile * BT + col + 16, v1);
    }
  }
  for (; col < c1; col += 16) {
    const int m = mtile * BT + col;
    if (m >= a.M) break;
    float v[NW][4];
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      float4 t[kMaxSplit];
#pragma unroll
      for (int p = 0; p < kMaxSplit; ++p)
        if (p < SPL)
          t[p] = __ldcg(reinterpret_cast<const float4*>(part + (((size_t)p * NW + w) * BT + col) * 128 + r4));
      v[w][0] = v[w][1] = v[w][2] = v[w][3] = 0.0f;
#pragma unroll
      for (int p = 0; p < kMaxSplit; ++p)
        if (p < SPL) {
          v[w][0] += t[p].x; v[w][1] += t[p].y; v[w][2] += t[p].z; v[w][3] += t[p].w;
        }
    }
    emit(m, v);
  }
}

// TA = true: the dequantized weight tile (MMA operand A) is written to TMEM
// by the dequant warps (tcgen05.st) and read from there by the MMA, instead
// of going through shared memory.  Shared memory then holds only token
// tiles, so the ring is deeper (3 stages of BT=256 instead of 2) and more
// token bytes are in flight; TMEM holds one accumulator (columns
// [0, NW*BT)) and one 64-column A slot per stage after it.  Folded numerics,
// one weight.
// TF = true: packed-F16 weights, kind::tf32.  Both operands are f32 rows
// (pre-expanded weight tiles and f32 token tiles read by TMA straight from
// the caller's rows).  The linear uses rows of 64 bytes with the 64-byte
// swizzle: a chunk is 16 K, a stage 32 K, and a 256-token stage 48 KB, so 4
// stages are in flight where 128-byte rows fit 2.
// CV = true (implies TF): implicit-GEMM convolution.  The token rows of chunk kc
// are shifted by its kernel tap (cv_coord), and the operands are swapped:
// A = the token tile (128 tokens per MMA, BT/128 MMAs), B = the 128-channel
// weight tile, so a TMEM lane is a token and the epilogue's warps store 32
// consecutive output positions of one channel plane per instruction (NCHW).
template <int BT, int NW, bool TA, bool QK = false, bool SC = false, bool CV = false, bool TF = false>
__global__ void __launch_bounds__(kWsThreads, 1)
    q4_gemm_ws_kernel(const __grid_constant__ CUtensorMap tmap_x, const WsArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  // Operand rows: 128 bytes (64 f16, or 32 f32 for the convolution) with the
  // 128-byte swizzle; the tf32 linear uses 64-byte rows (16 f32) with the
  // 64-byte swizzle, so that a stage stays small enough for 4..8 of them to be
  // in flight.  (The convolution's row-shifted boxes measured slower that way:
  // twice the TMA row requests per byte.)
  constexpr bool kNarrow = TF && !CV;
  constexpr uint32_t kRowB = kNarrow ? 64u : 128u;
  constexpr uint32_t kATile = 128 * kRowB;          // one weight sub-tile (128 rows)
  constexpr uint32_t kBSub = BT * kRowB;            // one token sub-tile
  constexpr uint32_t kAStage = TA ? 0u : NW * 2 * kATile;
  constexpr uint32_t kStage = kAStage + 2 * kBSub;
  constexpr uint32_t kPartCols = NW * BT;
  // partial buffers in TMEM: TA keeps 256 columns for them (one 256-token
  // accumulator, or two 128-token partials for exact numerics)
  constexpr int kNP = TA ? 256 / kPartCols : 512 / kPartCols;
  constexpr uint32_t kACol0 = kNP * kPartCols;    // TA: first A-slot column
  constexpr int kCols = BT / 4;          // token columns per scaler thread
  constexpr bool kSK = !TA;              // stream-K tails are planned only for A in shared memory
  // TF with NW = 2 ("wide"): the two weights are consecutive 128-row N tiles
  // of one weight on one 256-token tile, so a CTA computes 256 x 256 outputs
  // from 2 KB of operands per K (a 128 x 256 tile needs 1.5 KB for half the
  // FLOPs).  Its accumulator pair fills TMEM: one partial buffer.
  constexpr bool kWide = TF && NW == 2;
  static_assert(TA || kNP >= 2 || kWide, "at least double buffering");
  static_assert(!TA || (NW == 1 && kACol0 == 256 && BT >= 128), "TMEM operand A: one weight, slots from column 256");
  static_assert(kCols % 16 == 0, "scaler column split");
  static_assert(!QK || (NW == 1 && BT >= 128), "QK-norm epilogue: one weight, 128- or 256-token tiles");
  static_assert(!SC || (NW == 1 && !QK), "row scatter: one weight, plain epilogue");
  static_assert(!TF || ((NW == 1 || (NW == 2 && BT == 256 && !CV)) && !TA && !QK && !SC),
                "tf32: pre-expanded weight tiles, plain epilogue");
  static_assert(!CV || (TF && BT >= 128), "convolution: tf32, 128-token MMAs");
  constexpr int kCK = TF ? (int)kRowB / 4 : kChunkK;  // K values per operand row
  constexpr int kSteps = (int)kRowB / 32;  // MMA K steps per row (32 bytes each)

  const int S = a.stages, RS = a.rs;
  uint8_t* ring = smem;                                     // [S][A | B]
  uint8_t* raw_ring = ring + (size_t)S * kStage;            // [RS][NW][raw_w_bytes]
  // QK: the epilogue's per-quarter partial sums, [2][4 quarters][4 quads][kCols] f32
  float* qk_scratch = reinterpret_cast<float*>(raw_ring + (size_t)RS * NW * a.raw_w_bytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(qk_scratch) +
                                               (QK ? (size_t)32 * kCols * sizeof(float) : 0));
  uint64_t* full = bars;
  uint64_t* empty = full + S;
  uint64_t* raw_full = empty + S;
  uint64_t* raw_empty = raw_full + RS;
  uint64_t* part_full = raw_empty + RS;
  uint64_t* part_empty = part_full + kNP;
  uint64_t* sk_bars = part_empty + kNP;  // stream-K: [0] head published, [1] head partial ready
  uint64_t* qk_bars = sk_bars + 2;       // QK: one per column quarter
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(qk_bars + (QK ? 4 : 0));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

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
    ptx::mbar_init(&sk_bars[0], kWsScalerWarps);
    ptx::mbar_init(&sk_bars[1], 1);
    if (QK)
      for (int i = 0; i < 4; ++i) ptx::mbar_init(&qk_bars[i], 4);
    *abort_flag = 0;
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
      // xh is written by the activation-staging grid launched just before
      // this one; every other operand was complete before that grid started.
      ptx::griddep_wait();
      int s = 0;
      uint32_t ph = 0;
      BQ4_FOR_UNITS(!*abort_flag) {
        const int tile = un.tile, kc0 = un.kc0, kc1 = un.kc1;
        int mtile, ntile;
        ws_tile(a, tile, mtile, ntile);
        for (int kc = kc0; kc < kc1; kc += 2) {
          if (!ptx::mbar_wait(&empty[s], ph ^ 1, abort_flag)) {
            record_error_flag(abort_flag, BQ4_ETIMEOUT);
            break;
          }
          uint8_t* st = ring + (size_t)s * kStage;
          ptx::mbar_arrive_expect_tx(&full[s], 2 * kBSub + (a.pre ? kAStage : 0u));
          int x0 = kc * kCK, y0 = mtile * BT, x1 = (kc + 1) * kCK, y1 = mtile * BT;
          if constexpr (CV) {
            cv_coord(a, kc, kCK, mtile * BT, x0, y0);
            cv_coord(a, kc + 1, kCK, mtile * BT, x1, y1);
          }
          ptx::tma_load_2d(st + kAStage, &tmap_x, &full[s], x0, y0);
          ptx::tma_load_2d(st + kAStage + kBSub, &tmap_x, &full[s], x1, y1);
          if (a.pre) {
#pragma unroll
            for (int w = 0; w < NW; ++w) {
              const int tw = kWide ? 2 * ntile + w : ntile;  // wide: N tiles 2 ntile, 2 ntile + 1
              ptx::bulk_load(st + (size_t)w * 2 * kATile, a.h[w] + ((size_t)tw * a.nkc + kc) * (kATile / 2),
                             2 * kATile, &full[s]);
            }
          }
          if (++s == S) { s = 0; ph ^= 1; }
        }
      }
    } else if (warp == kWsWeightWarp && lane == 0 && !a.pre) {
      // ------------------------------------------------ raw weight tiles (bulk copies)
      int rs = 0;
      uint32_t rph = 0;
      BQ4_FOR_UNITS(!*abort_flag) {
        const int tile = un.tile, kc0 = un.kc0, kc1 = un.kc1;
        int mtile, ntile;
        ws_tile(a, tile, mtile, ntile);
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
      constexpr uint32_t idesc = TF ? ptx::umma_idesc_tf32(128, CV ? 128 : BT) : ptx::umma_idesc_f16(128, BT);
      int s = 0, pb = 0;
      uint32_t ph = 0, pph = 0;
      bool ok = true;
      BQ4_FOR_UNITS(ok && !*abort_flag) {
        const int kc0 = un.kc0, kc1 = un.kc1;
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
            for (int kk = 0; kk < kSteps; ++kk) {
              const uint64_t b_desc =
                  kNarrow ? ptx::umma_desc_sw64(b_addr + kk * 32) : ptx::umma_desc_sw128(b_addr + kk * 32);
              if constexpr (TA) {
                ptx::mma_f16_ts(d_base, tmem_base + kACol0 + (uint32_t)s * 64 + (uint32_t)sub * 32 + kk * 8, b_desc,
                                idesc, (first && kk == 0) ? 0u : 1u);
              } else if constexpr (CV) {
                // tokens as A (128 per MMA), the weight tile as B (128 channels)
                const uint64_t w_desc = ptx::umma_desc_sw128(st + (uint32_t)(sub * kATile) + kk * 32);
#pragma unroll
                for (int h = 0; h < BT / 128; ++h)
                  ptx::mma_tf32_ss(d_base + h * 128, ptx::umma_desc_sw128(b_addr + h * 128 * kRowB + kk * 32), w_desc,
                                   idesc, (first && kk == 0) ? 0u : 1u);
              } else if constexpr (TF) {
#pragma unroll
                for (int w = 0; w < NW; ++w)
                  ptx::mma_tf32_ss(d_base + w * BT, ptx::umma_desc_sw64(st + (uint32_t)((w * 2 + sub) * kATile) + kk * 32),
                                   b_desc, idesc, (first && kk == 0) ? 0u : 1u);
              } else {
#pragma unroll
                for (int w = 0; w < NW; ++w)
                  ptx::mma_f16_ss(d_base + w * BT,
                                  ptx::umma_desc_sw128(st + (uint32_t)((w * 2 + sub) * kATileBytes) + kk * 32),
                                  b_desc, idesc, (first && kk == 0) ? 0u : 1u);
              }
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
    if (a.ksplit > 1) {  // the cluster barrier of the split reduction
      __syncwarp();
      ptx::cluster_sync();
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
      BQ4_FOR_UNITS(ok && !*abort_flag) {
        const int kc0 = un.kc0, kc1 = un.kc1;
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
          if constexpr (TA) {
            // row r = TMEM lane r (this warp's lane quarter is r / 32), the
            // sub-tile's 64 K values = 32 columns of A slot s
            ptx::tc_fence_after();
            const uint32_t wv[8] = {wlo[0].x, wlo[0].y, wlo[0].z, wlo[0].w, whi[0].x, whi[0].y, whi[0].z, whi[0].w};
            const uint32_t t_a = tmem_base + ((uint32_t)((warp & 3) * 32) << 16) + kACol0 + (uint32_t)s * 64 +
                                 (uint32_t)sub * 32;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              uint32_t v[16];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const uint4 e = a.exact ? expand_word_exact(wv[h * 4 + j]) : expand_word(wv[h * 4 + j], sc[0][h * 4 + j]);
                v[4 * j] = e.x; v[4 * j + 1] = e.y; v[4 * j + 2] = e.z; v[4 * j + 3] = e.w;
              }
              ptx::tmem_st_32x32b_x16(t_a + (uint32_t)h * 16, v);
            }
            ptx::tmem_st_wait();
            ptx::tc_fence_before();
          } else {
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
          }
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(&full[s]);
          if (++s == S) { s = 0; ph ^= 1; }
        }
      }
      if (!ok) record_error_flag(abort_flag, BQ4_ETIMEOUT);
    }
    if (a.ksplit > 1) {  // the cluster barrier of the split reduction
      __syncwarp();
      ptx::cluster_sync();
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
    bool split_synced = false;  // this warp has passed the split's cluster barrier
    uint32_t qk_uses = 0;       // QK: scratch buffer / barrier phase of this warp
    if (a.lockstep && lane == 0) {
      // both partial buffers start free: the first use of each stage
      for (int i = 0; i < S; ++i) ptx::mbar_arrive(&full[i]);
    }
    BQ4_FOR_UNITS(ok && !*abort_flag) {
      const int tile = un.tile, split = un.split, kc0 = un.kc0, kc1 = un.kc1;
      int mtile, ntile;
      ws_tile(a, tile, mtile, ntile);
      if constexpr (kWide) {
        // stream each 16-column chunk of the two accumulators from TMEM to y
        // (the pair does not fit the registers), then release the buffer
        if (!ptx::mbar_wait(&part_full[pb], pph, abort_flag)) { ok = false; break; }
        ptx::tc_fence_after();
        const uint32_t t_row = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)pb * kPartCols + col0;
        const int m0w = mtile * BT + col0;
        const int act = a.act;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
          const int nw_ = (2 * ntile + w) * 128 + row;
          const float bw = (a.bias[0] && nw_ < a.N) ? __ldg(a.bias[0] + nw_) : 0.0f;
#pragma unroll
          for (int c = 0; c < kCols / 16; ++c) {
            uint32_t r0[16];
            ptx::tmem_ld_32x32b_x16(t_row + w * BT + c * 16, r0);
            ptx::tmem_ld_wait();
            if (nw_ < a.N) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int m = m0w + c * 16 + j;
                if (m < a.M) {
                  float v = apply_act(__uint_as_float(r0[j]) + bw, act);
                  if (a.aux) v *= __ldg(a.aux + (size_t)m * a.N + nw_);
                  store_y(a, m, nw_, v);
                }
              }
            }
          }
        }
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&part_empty[pb]);
        if (++pb == kNP) { pb = 0; pph ^= 1; }
      } else {
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
          // lockstep: segment == stage pb (partial pb), retired when empty[pb] completes
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
          if (++pb == (a.lockstep ? S : kNP)) { pb = 0; pph ^= 1; }
        }
        if (!ok) break;

        if (a.ksplit > 1) {
          // Split-K (the CTA's only unit): publish this split's partial tile,
          // then the cluster barrier -- every split's tile is in the workspace.
          split_publish<BT, NW, kCols>(a, tile, split, acc, row, col0);
          __syncwarp();
          ptx::cluster_sync();
          split_synced = true;
          break;
        }
        if constexpr (kSK) {
          if (un.kind == kUnitHead) {
            sk_publish<BT, NW, kCols>(a, acc, row, col0, &sk_bars[0], abort_flag);
            continue;
          }
          if (un.kind == kUnitTail && !sk_absorb<BT, NW, kCols>(a, acc, row, col0, ring, &sk_bars[1], abort_flag)) {
            ok = false;
            break;
          }
        }
        if constexpr (CV) {
          // TMEM lane = token, columns = channels: this thread holds token
          // (col0 / 128) * 128 + row of the tile, channels col0 % 128 .. + kCols
          const int p = mtile * BT + (col0 / 128) * 128 + row;
          if (p < a.M) {
            const int img = a.cv_hp * a.cv_wp;
            const int b = p / img, r = p - b * img;
            const int py = r / a.cv_wp, px = r - py * a.cv_wp;
            if (py < a.cv_oh && px < a.cv_ow) {
              const size_t plane = (size_t)a.cv_oh * a.cv_ow;
              const int nb = ntile * 128 + (col0 & 127);
              float* o = reinterpret_cast<float*>(a.y) + ((size_t)b * a.N + nb) * plane + (size_t)py * a.cv_ow + px;
              const int act = a.act;
  #pragma unroll
              for (int j = 0; j < kCols; ++j) {
                if (nb + j < a.N) {
                  const float bj = a.bias[0] ? __ldg(a.bias[0] + nb + j) : 0.0f;
                  o[(size_t)j * plane] = apply_act(acc[0][j] + bj, act);
                }
              }
            }
          }
          continue;
        }
        if constexpr (QK) {
          const bool is_q = ntile < a.qk_q;
          if (is_q || ntile < a.qk_q + a.qk_k) {
            // a q or k head: bias, QK-norm + RoPE (every lane takes part), store
            const float b0 = (a.bias[0] && n < a.N) ? __ldg(a.bias[0] + n) : 0.0f;
  #pragma unroll
            for (int j = 0; j < kCols; ++j) acc[0][j] += b0;
            if (!qk_epilogue<BT, kCols>(a, acc[0], row, mtile, col0, is_q, qk_scratch, qk_bars, qk_uses,
                                        abort_flag)) {
              ok = false;
              break;
            }
            if (n < a.N) {
  #pragma unroll
              for (int j = 0; j < kCols; ++j)
                if (m0 + j < a.M) store_y(a, m0 + j, n, acc[0][j]);
            }
            continue;
          }
        }
        if (SC && n < a.N) {
          // row scatter: token m's partial goes to row (sc_rank sc_rows + m - owner sc_rows)
          // of its owner's receive buffer; the owner and the row address advance with m
          // (this thread's tokens are consecutive) instead of a division per element
          const float b0 = a.bias[0] ? __ldg(a.bias[0] + n) : 0.0f;
          const int act = a.act;
          int owner = m0 / a.sc_rows;
          int next = (owner + 1) * a.sc_rows;
          float* dst = a.sc_y[owner] + (size_t)(a.sc_rank * a.sc_rows + (m0 - owner * a.sc_rows)) * a.ldy + n;
  #pragma unroll
          for (int j = 0; j < kCols; ++j) {
            const int m = m0 + j;
            if (m >= a.M) break;
            if (m == next) {
              ++owner;
              next += a.sc_rows;
              dst = a.sc_y[owner] + (size_t)a.sc_rank * a.sc_rows * a.ldy + n;
            }
            float v = apply_act(acc[0][j] + b0, act);
            if (a.aux) v *= __ldg(a.aux + (size_t)m * a.N + n);
            *dst = v;
            dst += a.ldy;
          }
        } else if (n < a.N) {
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
              store_out<SC>(a, m, n, v);
            }
          }
        }
      }
    }
    if (!ok) record_error_flag(abort_flag, BQ4_ETIMEOUT);
    if (split_synced) split_reduce_epilogue<BT, NW, SC>(a);
    if (a.ksplit > 1 && !split_synced) {
      // Every role of every CTA of the cluster passes the split's cluster
      // barrier exactly once (each role branch has its own); a scaler warp
      // that left its loop early passes it here.
      __syncwarp();
      ptx::cluster_sync();
    }
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
  // a function-local static: initialised once, and no caller sees it before that ends
  static const EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFn>(p);
    return static_cast<EncodeTiledFn>(nullptr);
  }();
  return fn;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// The kernel rebalances registers with setmaxnreg; the split only fits the
// pool the block was launched with when ptxas gave every thread exactly
// kWsRegsLaunch registers.  Checked once per instantiation before any launch
// (a mismatch would make setmaxnreg.inc wait forever).
template <int BT, int NW, bool TA, bool QK = false, bool SC = false, bool CV = false, bool TF = false>
cudaError_t prepare_ws_kernel(size_t smem_bytes, bool* ok_regs) {
  auto kern = q4_gemm_ws_kernel<BT, NW, TA, QK, SC, CV, TF>;
  static std::atomic<int> checked{0};  // 0 unknown, 1 ok, -1 bad
  if (checked.load(std::memory_order_relaxed) == 0) {
    cudaFuncAttributes attr;
    cudaError_t e = cudaFuncGetAttributes(&attr, kern);
    if (e != cudaSuccess) return e;
    checked.store((attr.numRegs == kWsRegsLaunch) ? 1 : -1, std::memory_order_relaxed);
  }
  *ok_regs = checked.load(std::memory_order_relaxed) == 1;
  // the shared-memory opt-in is a per-device function attribute
  static std::atomic<size_t> smem_set[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (smem_set[dev].load(std::memory_order_relaxed) < smem_bytes) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes);
    if (e != cudaSuccess) return e;
    smem_set[dev].store(smem_bytes, std::memory_order_relaxed);
  }
  return cudaSuccess;
}

template <int BT, int NW, bool TA = false, bool QK = false, bool SC = false, bool CV = false, bool TF = false>
cudaError_t launch_ws(const GemmPlan& plan, const CUtensorMap& tmap, const WsArgs& args, cudaStream_t stream,
                      bool* ok_regs) {
  cudaError_t e = prepare_ws_kernel<BT, NW, TA, QK, SC, CV, TF>(plan.smem_bytes, ok_regs);
  if (e != cudaSuccess || !*ok_regs) return e;
  // Launched as a programmatic dependent of the activation-staging grid
  // before it (only the token loads wait for that grid, see the kernel), and
  // with split-K as clusters of the splits of one tile (grid = units).
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3((unsigned)plan.grid, 1, 1);
  cfg.blockDim = dim3(kWsThreads, 1, 1);
  cfg.dynamicSmemBytes = plan.smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (plan.pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (plan.cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = (unsigned)plan.cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  e = cudaLaunchKernelEx(&cfg, q4_gemm_ws_kernel<BT, NW, TA, QK, SC, CV, TF>, tmap, args);
  note_launch();
  return e;
}

// How many clusters of `cs` CTAs of this kernel can be resident at once on
// the current device (0 if none).  One CTA fills an SM's shared memory, so
// this depends only on the cluster size; cached per size (every GPU a
// process drives here is the same part).
template <int BT, int NW>
int cluster_capacity_t(int cs, size_t smem_bytes) {
  static std::atomic<int> cache[kMaxSplit + 1];
  if (cs < 2 || cs > kMaxSplit) return 0;
  int v = cache[cs].load(std::memory_order_relaxed);
  if (v > 0) return v - 1;
  bool ok_regs = true;
  int n = 0;
  bool known = false;
  if (prepare_ws_kernel<BT, NW, false>(smem_bytes, &ok_regs) == cudaSuccess) {
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3((unsigned)cs, 1, 1);
    cfg.blockDim = dim3(kWsThreads, 1, 1);
    cfg.dynamicSmemBytes = smem_bytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, q4_gemm_ws_kernel<BT, NW, false>, &cfg) == cudaSuccess) {
      known = true;
    } else {
      cudaGetLastError();
      n = 0;
    }
  } else {
    cudaGetLastError();
  }
  if (known) cache[cs].store(n + 1, std::memory_order_relaxed);  // failures are not cached
  return n;
}

int cluster_capacity_any(int bt, int nw, int cs, size_t smem_bytes);

int cluster_capacity(int bt, int nw, int cs, size_t smem_bytes, int device) {
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != device) cudaSetDevice(device);
  const int n = cluster_capacity_any(bt, nw, cs, smem_bytes);
  if (prev >= 0 && prev != device) cudaSetDevice(prev);
  return n;
}

int cluster_capacity_any(int bt, int nw, int cs, size_t smem_bytes) {
  if (nw == 1) {
    if (bt == 256) return cluster_capacity_t<256, 1>(cs, smem_bytes);
    if (bt == 128) return cluster_capacity_t<128, 1>(cs, smem_bytes);
    return cluster_capacity_t<64, 1>(cs, smem_bytes);
  }
  if (bt == 128) return cluster_capacity_t<128, 2>(cs, smem_bytes);
  return cluster_capacity_t<64, 2>(cs, smem_bytes);
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

namespace {
std::atomic<int> g_sm_budget{-1};
}

int sm_budget() {
  int v = g_sm_budget.load(std::memory_order_relaxed);
  if (v < 0) {
    v = 0;
    if (const char* e = getenv("BQ4_SM_BUDGET")) v = atoi(e) > 0 ? atoi(e) : 0;
    int expected = -1;
    g_sm_budget.compare_exchange_strong(expected, v);
    v = g_sm_budget.load(std::memory_order_relaxed);
  }
  return v;
}

void set_sm_budget(int sms) { g_sm_budget.store(sms > 0 ? sms : 0, std::memory_order_relaxed); }

int device_sm_count(int device) {
  static std::atomic<int> cache[64];
  if (device < 0 || device >= 64) return 148;
  int v = cache[device].load(std::memory_order_relaxed);
  if (!v) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0)
      v = 148;
    cache[device].store(v, std::memory_order_relaxed);
  }
  return v;
}

int device_is_sm100(int device) {
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess)
    return 0;
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  return major == 10 && minor == 0;
}

// Plan for one token-tile size; *cost is the estimated makespan in µs.
// Stream-K partial slots ([grid][NW][BT][128] f32) and flags ([grid]).
static size_t sk_part_bytes(int grid, int nw, int bt) {
  return align_up((size_t)grid * nw * bt * 128 * sizeof(float), 256);
}

static bq4_status plan_for_bt(const bq4_weight* w, int nw, int64_t M, int device, int bt, GemmPlan* p,
                              double* cost, bool allow_sk, bool qk, bool cv) {
  p->bt = bt;
  p->mtiles = (int)((M + p->bt - 1) / p->bt);
  p->ntiles = (int)w->ntiles;
  int sms = device_sm_count(device);
  if (sm_budget() > 0 && sm_budget() < sms) sms = sm_budget();  // leave SMs to other streams
  const int tiles = p->mtiles * p->ntiles;
  const int nks = (int)w->nkc / 2;  // 128-K stages

  // Shared memory: operand ring of 128-K stages (A + B) as deep as fits
  // (2..4 stages) next to a raw ring of 1..4 stages.
  const uint32_t raw_s_bytes = p->pre ? 0u : 512u * (uint32_t)(w->block >= 128 ? 1 : 128 / w->block);
  p->raw_s_bytes = p->exact || p->pre ? 0u : raw_s_bytes;
  p->raw_w_bytes = p->pre ? 16u : 2 * kRawQBytes + p->raw_s_bytes;
  // Operand A in TMEM (folded numerics, one weight, 256-token tiles): shared
  // memory then holds only token tiles.  BQ4_NO_TA=1 keeps A in shared memory.
  // Exact numerics need two TMEM partials, which leave room for A slots only
  // at 128-token tiles (BQ4_EXACT_TA=1 enables that combination).
  p->ta = (!p->pre && nw == 1 && !getenv("BQ4_NO_TA") &&
           ((!p->exact && p->bt == 256) || (p->exact && p->bt == 128 && getenv("BQ4_EXACT_TA")) ||
            (p->exact && p->bt == 256 && getenv("BQ4_EXACT_TA256"))))
              ? 1 : 0;
  // operand rows: 128 bytes, or 64 for the tf32 linear (whose stages are then
  // small enough for up to 8 in flight)
  const size_t row_b = (p->tf && !cv) ? 64 : 128;
  const size_t stage_bytes = (p->ta ? 0 : (size_t)nw * 2 * 128 * row_b) + 2 * (size_t)p->bt * row_b;
  const int max_stages = p->ta ? (512 - 256) / 64 : (p->tf ? 8 : 4);  // TA: one 64-column TMEM A slot per stage
  const int np = p->ta ? 256 / p->bt : 512 / (nw * p->bt);  // TMEM partial buffers of the kernel
  const size_t raw_stage = (size_t)nw * p->raw_w_bytes;
  // QK: the epilogue's partial sums, 2 x 16 warps x BT/4 columns of f32
  const size_t qk_bytes = qk ? (size_t)32 * (p->bt / 4) * sizeof(float) : 0;
  const size_t budget = 227 * 1024 - 1024 /*align*/ - 512 /*barriers*/ - qk_bytes;
  int S = 0, RS = 0;
  for (int s = max_stages; s >= 2 && !S; --s) {
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
    if (sscanf(f, "%d,%d", &fs, &fr) == 2 && fs >= 2 && fs <= max_stages && fr >= 1 &&
        (size_t)fs * stage_bytes + (size_t)fr * raw_stage <= budget) {
      S = fs;
      RS = p->pre ? 1 : fr;
    }
  }
  if (S < 2 || RS < 1) return set_error(BQ4_EUNSUPPORTED, "no shared-memory plan for this shape");
  p->stages = S;
  p->a_stages = S;
  p->raw_stages = RS;
  // Lockstep partial handoff: exact 128-blocks (one segment per stage) and
  // at most as many stages as TMEM partial buffers, so stage s always
  // accumulates into partial s.
  p->lockstep = (p->exact && w->block == 128 && S <= np) ? 1 : 0;
  if (getenv("BQ4_NO_LOCKSTEP")) p->lockstep = 0;
  p->qk = qk ? 1 : 0;
  p->smem_bytes = 1024 + (size_t)S * stage_bytes + (size_t)RS * raw_stage + qk_bytes +
                  (size_t)(2 * S + 2 * RS + 2 * np + 2 + (qk ? 4 : 0)) * 8 + 16;

  // Split-K factor: minimise the estimated makespan (µs, measured on B200):
  // waves x (128-K stages per unit x stage time + unit fill + the cluster
  // reduction, whose distributed-shared-memory traffic grows with BT).  The
  // splits of a tile form one thread-block cluster (at most 8 CTAs, the
  // portable limit), and split-K is only used when every cluster is
  // co-resident (one wave); multi-wave work uses whole-K units.
  // (a tf32 stage is 32 K at half the f16 rate: half an f16 stage's time)
  const double t_stage =
      (p->bt == 256 ? 1.1 : (p->bt == 128 ? 0.8 : 0.7)) * (nw == 2 ? 1.6 : 1.0) * (p->tf ? 0.5 : 1.0);
  const double t_red = 0.008 * p->bt * nw + 1.0;
  int best_s = 1;
  double best_t = 1e30;
  const int max_s = nks < kMaxSplit ? nks : kMaxSplit;
  for (int s = 1; s <= (qk || cv ? 1 : max_s); ++s) {  // the QK and conv epilogues need whole-K tiles
    const int units = tiles * s;
    if (s > 1 && (units > s * cluster_capacity(p->bt, nw, s, p->smem_bytes, device) || units > sms)) continue;
    const int waves = (units + sms - 1) / sms;
    const double t = waves * ((nks + s - 1) / s * t_stage + 1.0 + (s > 1 ? t_red : 0.0));
    if (t < best_t - 1e-9) {
      best_t = t;
      best_s = s;
    }
  }
  *cost = best_t + 2.0;
  // BQ4_FORCE_KSPLIT=s pins the split-K factor (clamped to [1, min(stages,
  // 8)] and to what one wave of clusters holds).
  if (const char* f = getenv("BQ4_FORCE_KSPLIT")) {
    int v = atoi(f);
    if (v >= 1) best_s = v < max_s ? v : max_s;
    if (qk || cv) best_s = 1;
    while (best_s > 1 && (tiles * best_s > best_s * cluster_capacity(p->bt, nw, best_s, p->smem_bytes, device) ||
                          tiles * best_s > sms))
      --best_s;
  }
  p->ksplit = best_s;
  p->units = tiles * best_s;
  p->cluster = best_s;
  p->grid = best_s > 1 ? p->units : (p->units < sms ? p->units : sms);

  // Stream-K tail for whole-K plans whose last wave is partial: the last
  // full wave plus the remainder (sms + rem tiles) are dealt to the CTAs as
  // equal ranges of 128-K stages, so no SM idles through the final wave.
  // Each range is at least one tile long, so a tile is cut at most once;
  // its two pieces meet through a partial slot in the workspace (about
  // t_fix µs to read back).  Measured on B200 against whole tiles it pays
  // for exact numerics and the gated pair (0.92x for 150 exact tiles, 0.82x
  // for the gated pair's 152); folded plans lose: with the weight tile in
  // TMEM the single accumulator serialises the pieces' epilogues (1.05-1.2x),
  // and 128-token folded tiles with the tail lose to 256-token whole tiles
  // (c1: 63.6 vs 55.1 µs).  Those keep whole tiles, and so does the tf32
  // linear (4096^3, 512 tiles: 256.6 vs 255.9 µs -- its operand ingest, not
  // the partial last wave, sets the time).  BQ4_NO_STREAMK=1 keeps whole
  // tiles everywhere.
  p->dp_tiles = p->sk_tiles = 0;
  p->sk_bytes = 0;
  if (best_s == 1 && allow_sk && (p->exact || nw == 2) && !p->ta && !getenv("BQ4_NO_STREAMK") && tiles > sms &&
      tiles % sms != 0 &&
      (int64_t)(2 * sms) * sms * nks < ((int64_t)1 << 31)) {
    const int full = tiles / sms, rem = tiles % sms;
    const double t_tile = nks * t_stage + 1.0;
    const double t_fix = 0.01 * p->bt * nw + 0.5;
    const double t_dp = (double)(full + 1) * t_tile;
    const double t_sk = (double)(full - 1) * t_tile + ((double)(sms + rem) * nks / sms + 1.0) * t_stage + 1.0 + t_fix;
    // the tail piece pulls its head partial into the (then idle) operand ring
    const bool fits = (size_t)nw * p->bt * 128 * sizeof(float) <= (size_t)S * stage_bytes;
    if (t_sk < t_dp && fits) {
      p->sk_tiles = sms + rem;
      p->dp_tiles = tiles - p->sk_tiles;
      p->sk_bytes = sk_part_bytes(p->grid, nw, p->bt) + align_up((size_t)p->grid * sizeof(unsigned), 256);
      best_t = t_sk;
      *cost = best_t + 2.0;
    }
  }
  // Split-K tail launch: when whole tiles leave the last wave partial (rem
  // tiles), the full waves run as one launch and the rem tiles as a second
  // one in which each tile is cut into s K ranges, a cluster of s CTAs
  // reducing through the workspace (the split-K path).  The last wave then
  // takes about 1/s of a tile plus the reduction and a launch instead of a
  // whole tile.  Not with stream-K or the QK / conv epilogues (whole-K
  // tiles), nor when the caller plans without workspace extras (allow_sk =
  // false).  Opt-in (BQ4_SPLIT_TAIL=1): measured on B200 it does not pay --
  // c1 (152 tiles, 4 in the tail, 8 splits) 50.9 vs 52.5 us, and the DiT
  // stack (qkv and up with tails) 1224 vs 1242 TFLOP/s: the cluster
  // reduction and the second launch cost about what the short wave saves.
  p->tail_tiles = p->tail_split = 0;
  if (best_s == 1 && allow_sk && p->sk_tiles == 0 && !qk && !cv && tiles > sms && tiles % sms != 0 &&
      getenv("BQ4_SPLIT_TAIL") && !getenv("BQ4_NO_TAIL")) {
    const int rem = tiles % sms;
    int s = sms / rem;
    if (s > kMaxSplit) s = kMaxSplit;
    if (s > nks) s = nks;
    const double t_tile = nks * t_stage + 1.0;
    const double t_tail = (double)((nks + s - 1) / s) * t_stage + 1.0 + t_red + 2.0;
    if (s >= 2 && t_tail < t_tile && rem <= cluster_capacity(p->bt, nw, s, p->smem_bytes, device)) {
      p->tail_tiles = rem;
      p->tail_split = s;
      p->units = tiles - rem;
      p->grid = sms;
      *cost = best_t - t_tile + t_tail + 2.0;
    }
  }
  // Unit order: the wave shares the operand that is larger in HBM -- the
  // f16 token rows (M*K*2 bytes) or the Q4 weights (nw*N*K/2 bytes).
  p->nfast = ((int64_t)M * 4 > (int64_t)nw * w->Np) ? 1 : 0;
  if (const char* f = getenv("BQ4_FORCE_NFAST")) p->nfast = f[0] == '1' ? 1 : 0;

  // Programmatic dependent launch of the GEMM after the activation staging
  // (BQ4_NO_PDL=1 launches it in plain stream order).
  p->pdl = getenv("BQ4_NO_PDL") ? 0 : 1;

  // Workspace: the stream-K slots and flags, the split-K partial tiles, then
  // the f16 copy of x (callers passing f16 activations need only the first
  // two parts).
  p->partial_bytes =
      best_s > 1 ? align_up((size_t)tiles * best_s * nw * p->bt * 128 * sizeof(float), 256) : 0;
  if (p->tail_tiles)
    p->partial_bytes = align_up((size_t)p->tail_tiles * p->tail_split * nw * p->bt * 128 * sizeof(float), 256);
  // tf32 plans read the caller's f32 rows in place (their entry points stage
  // the rows themselves when they must)
  p->xh_bytes = p->tf ? 0 : align_up((size_t)M * (size_t)w->Kp * 2, 256);
  p->workspace_bytes = p->sk_bytes + p->partial_bytes + p->xh_bytes;
  return BQ4_OK;
}


bq4_status plan_gemm(const bq4_weight* w, int nw, int64_t M, int device, GemmPlan* p, bool allow_sk, bool qk,
                     bool cv) {
  if (M <= 0) return set_error(BQ4_EINVAL_SHAPE, "M must be positive (got %lld)", (long long)M);
  if (M > (int64_t)1 << 30) return set_error(BQ4_EINVAL_SHAPE, "M too large");
  memset(p, 0, sizeof(*p));
  p->nw = nw;
  p->tf = w->tf32 ? 1 : 0;
  p->cv = cv ? 1 : 0;
  if ((p->tf || cv) && (nw != 1 || qk || (cv && !p->tf)))
    return set_error(BQ4_EINVAL_ARG, "packed-F16 plans take one packed-F16 weight and the plain or conv epilogue");
  // Numerics: blocks of 64/128 keep q exact in f16 and multiply the f32
  // partial of each K block by its scale (exact weights); smaller blocks
  // stage f16(q * f16(scale)) (folded); N-packed sources are pre-expanded.
  p->pre = (w->h != nullptr || w->tf32) ? 1 : 0;  // packed-F16 views are pre-expanded too
  const int mode = numerics_mode();
  p->exact = (!p->pre && w->block >= 64 &&
              (mode == BQ4_NUMERICS_EXACT || (mode == BQ4_NUMERICS_AUTO && M <= kAutoExactMaxM)))
                 ? 1 : 0;
  // BQ4_FORCE_FOLDED=1 selects folded staging for any block (tests compare
  // both formulations on the same shapes).
  if (const char* f = getenv("BQ4_FORCE_FOLDED"))
    if (f[0] == '1') p->exact = 0;
  // Token tile: every candidate up to 2M (the smallest always) is planned and costed;
  // BQ4_FORCE_BT=64|128|256 pins it (tuning).
  int forced = 0;
  if (const char* f = getenv("BQ4_FORCE_BT")) {
    const int v = atoi(f);
    if (v == 64 || v == 128 || (v == 256 && nw == 1)) forced = v;
  }
  // Few-token calls (up to kSkAutoMaxM rows) take the bandwidth-bound
  // small-M kernel: measured on B200 against this GEMM (graph-replayed, cold
  // L2), 1 x 2560 x 9728: 12.4 vs 31.6 us; 16 x 2560 x 9728: 17.0 vs 34.0;
  // 16 x 9728 x 2560: 16.9 vs 26.8; it loses from 64 rows (37.6 vs 34.6)
  // and at 256 (k/v: 22.6 vs 14.3).  BQ4_NO_SKINNY=1 never takes it,
  // BQ4_FORCE_SKINNY=1 takes it for every call that fits it (to 256 rows).
  SkPlan skp;
  const char* force_sk = getenv("BQ4_FORCE_SKINNY");
  const bool want_sk = (force_sk && force_sk[0] == '1') || M <= kSkAutoMaxM;
  const bool sk_ok = want_sk && !qk && !cv && !p->tf && !p->pre && !getenv("BQ4_NO_SKINNY") &&
                     plan_skinny(w, nw, M, device, p->exact != 0, &skp);
  if (sk_ok) {
    p->skinny = 1;
    p->sk = skp;
    p->bt = 8 * skp.nt;
    p->ksplit = p->cluster = skp.ks;
    p->mtiles = skp.gz;
    p->ntiles = (int)w->ntiles;
    p->units = p->grid = skp.gx * skp.ks * skp.gz;
    p->stages = skp.stages;
    p->smem_bytes = skp.smem_bytes;
    return BQ4_OK;  // no workspace
  }
  const GemmPlan base = *p;
  double best = 1e300;
  bool have = false;
  bq4_status last = BQ4_OK;
  for (int bt : {256, 128, 64}) {
    if (nw == 2 && bt == 256) continue;
    if ((qk || cv) && bt == 64) continue;  // QK: 32+ token columns per thread; conv: 128-token MMAs
    const int smallest = qk || cv ? 128 : 64;  // always a candidate, however small M is
    if (forced ? bt != forced : (bt != smallest && bt > 2 * M)) continue;
    GemmPlan cand = base;
    double cost = 0.0;
    last = plan_for_bt(w, nw, M, device, bt, &cand, &cost, allow_sk && !cv, qk, cv);
    if (last != BQ4_OK) continue;
    if (!have || cost < best - 1e-9) {
      *p = cand;
      best = cost;
      have = true;
    }
  }
  // tf32 linear with at least a wave of 256 x 256 tiles and a K loop of 16+
  // stages (512+ K): two N tiles per token tile (2/3 of the operand bytes per
  // FLOP).  Whole-K tiles, one TMEM buffer, so the epilogue of a tile holds
  // the next tile's MMAs: with a short K loop (attention scores, K = 128) the
  // tile is all epilogue and 128 x 256 tiles with two buffers are faster.
  // BQ4_NO_WIDE=1 keeps 128 x BT tiles.
  if (have && p->tf && !cv && !qk && nw == 1 && w->ntiles >= 2 && w->nkc >= 32 && !forced &&
      !getenv("BQ4_NO_WIDE")) {
    GemmPlan cand = base;
    double cost = 0.0;
    int sms = device_sm_count(device);
    if (sm_budget() > 0 && sm_budget() < sms) sms = sm_budget();
    const int pairs = (int)((w->ntiles + 1) / 2);
    const int mt = (int)((M + 255) / 256);
    if ((int64_t)mt * pairs >= sms && plan_for_bt(w, 2, M, device, 256, &cand, &cost, false, false, false) == BQ4_OK) {
      cand.nw = 1;
      cand.wide = 1;
      cand.ntiles = pairs;
      cand.ksplit = cand.cluster = 1;
      cand.units = mt * pairs;
      cand.grid = cand.units < sms ? cand.units : sms;
      cand.partial_bytes = 0;
      cand.workspace_bytes = cand.sk_bytes + cand.xh_bytes;
      *p = cand;
    }
  }
  return have ? BQ4_OK : (last != BQ4_OK ? last : set_error(BQ4_EUNSUPPORTED, "no plan for this shape"));
}

bq4_status run_gemm(const GemmPlan& plan, const bq4_weight* const* ws, const void* x, int64_t M,
                    int64_t ldx, const float* const* bias, int act, const float* aux, void* y,
                    void* workspace, cudaStream_t stream, const GemmIo& io) {
  if (plan.skinny)
    return run_skinny(plan.sk, ws, x, io.x_f16, M, ldx, bias, act, aux, y, io.y_f16, io.ldy, io, stream);
  const bq4_weight* w0 = ws[0];
  cudaError_t e = cudaSuccess;
  const void* xh = x;
  int64_t x_pitch = ldx;
  uint8_t* wsb = static_cast<uint8_t*>(workspace);
  float* sk_part = plan.sk_tiles ? reinterpret_cast<float*>(wsb) : nullptr;
  unsigned* sk_flag =
      plan.sk_tiles ? reinterpret_cast<unsigned*>(wsb + sk_part_bytes(plan.grid, plan.nw, plan.bt)) : nullptr;
  const int nflags = plan.sk_tiles ? plan.grid : 0;
  float* partials = plan.partial_bytes ? reinterpret_cast<float*>(wsb + plan.sk_bytes) : nullptr;
  if (plan.tf) {
    // tf32: the token tiles are read from the caller's f32 rows in place
    if (io.x_f16) return set_error(BQ4_EINVAL_ARG, "packed-F16 weights take f32 activations");
    if (!aligned16(x) || ldx % 4 != 0)
      return set_error(BQ4_EALIGN, "packed-F16 weights read x in place: 16-byte aligned rows, ldx %% 4 == 0");
  } else if (!io.x_f16) {
    // 1) stage activations as f16 [M][Kp] in the workspace (and zero the
    //    stream-K flags)
    void* dst = wsb + plan.sk_bytes + plan.partial_bytes;
    e = launch_convert_x(static_cast<const float*>(x), M, w0->K, ldx, w0->Kp, dst, sk_flag, nflags, stream);
    if (e != cudaSuccess) return check_cuda(e, "convert_x launch");
    xh = dst;
    x_pitch = w0->Kp;
  } else if (nflags) {
    e = launch_zero_flags(sk_flag, nflags, stream);
    if (e != cudaSuccess) return check_cuda(e, "zero_flags launch");
  }

  // 2) tensor map over the f16 tokens [M][Kp] (caller's buffer when x is
  //    already f16 with K == Kp), box {64, BT}, 128-byte swizzle
  EncodeTiledFn enc = encode_fn();
  if (!enc) return set_error(BQ4_ECUDA, "cuTensorMapEncodeTiled unavailable");
  CUtensorMap tmap;
  // tf32: f32 rows of K values (conv: x_cols staged channels), box {16, BT}
  // with the 64-byte swizzle (conv: {32, BT}, 128-byte swizzle); columns past
  // the extent read zeros
  const bool narrow = plan.tf && !plan.cv;
  const int64_t x_cols = plan.tf ? (io.cv ? io.cv->x_cols : w0->K) : w0->Kp;
  cuuint64_t gdim[2] = {(cuuint64_t)x_cols, (cuuint64_t)M};
  cuuint64_t gstride[1] = {(cuuint64_t)x_pitch * (plan.tf ? 4 : 2)};
  cuuint32_t box[2] = {(cuuint32_t)(narrow ? 16 : (plan.tf ? 32 : kChunkK)), (cuuint32_t)plan.bt};
  cuuint32_t estride[2] = {1, 1};
  CUresult cr = enc(&tmap, plan.tf ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                    const_cast<void*>(xh), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    narrow ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
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
  args.partials = partials;
  args.y = y;
  args.y_f16 = io.y_f16;
  args.ldy = (int)(io.ldy > 0 ? io.ldy : w0->N);
  args.M = (int)M;
  args.N = (int)w0->N;
  args.nkc = (int)w0->nkc;
  args.nkb = (int)w0->nkb;
  args.block = w0->block;
  args.ntiles = plan.ntiles;
  args.mtiles = plan.mtiles;
  args.ksplit = plan.ksplit;
  args.units = plan.units;
  args.nfast = plan.nfast;
  args.yvec = ((reinterpret_cast<uintptr_t>(y) & (io.y_f16 ? 7 : 15)) == 0 && args.ldy % 4 == 0) ? 1 : 0;
  args.stages = plan.stages;
  args.rs = plan.raw_stages;
  args.exact = plan.exact;
  args.pre = plan.pre;
  args.lockstep = plan.lockstep;
  args.dp_tiles = plan.dp_tiles;
  args.sk_tiles = plan.sk_tiles;
  args.sk_w = plan.sk_tiles * (int)(w0->nkc / 2);
  args.sk_part = sk_part;
  args.sk_flag = sk_flag;
  if (io.sc_rows) {
    if (io.y_f16 || io.sc_nranks < 1 || io.sc_nranks > BQ4_MAX_PEERS || !io.sc_y)
      return set_error(BQ4_EINVAL_ARG, "row scatter needs f32 output and 1..%d ranks", BQ4_MAX_PEERS);
    args.sc_rows = io.sc_rows;
    args.sc_rank = io.sc_rank;
    for (int r = 0; r < io.sc_nranks; ++r) args.sc_y[r] = io.sc_y[r];
  }
  if (plan.qk) {
    if (!io.qk) return set_error(BQ4_EINVAL_ARG, "a QK-norm plan needs its parameters");
    args.qk_q = io.qk->q_heads;
    args.qk_k = io.qk->k_heads;
    args.qk_eps = io.qk->eps;
    args.gamma_q = io.qk->gamma_q;
    args.gamma_k = io.qk->gamma_k;
    args.cos_t = io.qk->cos_t;
    args.sin_t = io.qk->sin_t;
    args.ld_rope = (int)io.qk->ld_rope;
  }
  if (plan.cv) {
    if (!io.cv) return set_error(BQ4_EINVAL_ARG, "a convolution plan needs its geometry");
    args.cv_cchunks = io.cv->cchunks;
    args.cv_taps = io.cv->taps;
    args.cv_kw = io.cv->kw;
    args.cv_dy = io.cv->dy;
    args.cv_dx = io.cv->dx;
    args.cv_hp = io.cv->hp;
    args.cv_wp = io.cv->wp;
    args.cv_oh = io.cv->oh;
    args.cv_ow = io.cv->ow;
  }
  args.act = act;
  args.raw_s_bytes = plan.raw_s_bytes;
  args.raw_w_bytes = plan.raw_w_bytes;

  // One launch of the planned kernel variant, plan `pl`, arguments `ar`.
  auto dispatch = [&](const GemmPlan& pl, WsArgs& ar) -> bq4_status {
    bool ok_regs = true;
    cudaError_t e = cudaSuccess;
    if (pl.cv) {
      if (pl.ksplit != 1 || pl.sk_tiles || pl.bt < 128) return set_error(BQ4_EUNSUPPORTED, "conv plan shape");
      if (pl.bt == 256) e = launch_ws<256, 1, false, false, false, true, true>(pl, tmap, ar, stream, &ok_regs);
      else e = launch_ws<128, 1, false, false, false, true, true>(pl, tmap, ar, stream, &ok_regs);
    } else if (pl.tf) {
      if (ar.sc_rows || pl.sk_tiles) return set_error(BQ4_EUNSUPPORTED, "tf32 plan shape");
      if (pl.wide) {
        if (pl.bt != 256 || pl.ksplit != 1) return set_error(BQ4_EUNSUPPORTED, "wide tf32 plan shape");
        ar.h[1] = ar.h[0];  // the same weight: N tiles 2t and 2t + 1
        e = launch_ws<256, 2, false, false, false, false, true>(pl, tmap, ar, stream, &ok_regs);
      } else if (pl.bt == 256) e = launch_ws<256, 1, false, false, false, false, true>(pl, tmap, ar, stream, &ok_regs);
      else if (pl.bt == 128) e = launch_ws<128, 1, false, false, false, false, true>(pl, tmap, ar, stream, &ok_regs);
      else e = launch_ws<64, 1, false, false, false, false, true>(pl, tmap, ar, stream, &ok_regs);
    } else if (ar.sc_rows) {
      if (pl.nw != 1 || pl.qk) return set_error(BQ4_EUNSUPPORTED, "row scatter: one weight, plain epilogue");
      if (pl.ta && pl.bt != 256) return set_error(BQ4_EUNSUPPORTED, "row scatter with 128-token TMEM operands");
      if (pl.ta) e = launch_ws<256, 1, true, false, true>(pl, tmap, ar, stream, &ok_regs);
      else if (pl.bt == 256) e = launch_ws<256, 1, false, false, true>(pl, tmap, ar, stream, &ok_regs);
      else if (pl.bt == 128) e = launch_ws<128, 1, false, false, true>(pl, tmap, ar, stream, &ok_regs);
      else e = launch_ws<64, 1, false, false, true>(pl, tmap, ar, stream, &ok_regs);
    } else if (pl.qk) {
      if (pl.nw != 1 || pl.ksplit != 1 || pl.bt < 128) return set_error(BQ4_EUNSUPPORTED, "QK-norm plan shape");
      if (pl.ta) e = launch_ws<256, 1, true, true>(pl, tmap, ar, stream, &ok_regs);
      else if (pl.bt == 256) e = launch_ws<256, 1, false, true>(pl, tmap, ar, stream, &ok_regs);
      else e = launch_ws<128, 1, false, true>(pl, tmap, ar, stream, &ok_regs);
    } else if (pl.nw == 1) {
      if (pl.ta && pl.bt == 256) e = launch_ws<256, 1, true>(pl, tmap, ar, stream, &ok_regs);
      else if (pl.ta) e = launch_ws<128, 1, true>(pl, tmap, ar, stream, &ok_regs);
      else if (pl.bt == 256) e = launch_ws<256, 1>(pl, tmap, ar, stream, &ok_regs);
      else if (pl.bt == 128) e = launch_ws<128, 1>(pl, tmap, ar, stream, &ok_regs);
      else e = launch_ws<64, 1>(pl, tmap, ar, stream, &ok_regs);
    } else {
      if (pl.bt == 128) e = launch_ws<128, 2>(pl, tmap, ar, stream, &ok_regs);
      else e = launch_ws<64, 2>(pl, tmap, ar, stream, &ok_regs);
    }
    if (e != cudaSuccess) return check_cuda(e, "q4 gemm launch");
    if (!ok_regs)
      return set_error(BQ4_EUNSUPPORTED, "q4 gemm kernel was not built with %d registers per thread",
                       kWsRegsLaunch);
    return BQ4_OK;
  };
  // Whole tiles, then (split-K tail plans) the tail tiles as clusters of
  // tail_split CTAs; row-scatter calls keep whole tiles throughout.
  const bool tail = plan.tail_tiles > 0 && !io.sc_rows;
  GemmPlan whole = plan;
  if (plan.tail_tiles && !tail) whole.units += plan.tail_tiles;
  args.units = whole.units;
  bq4_status st = dispatch(whole, args);
  if (st != BQ4_OK || !tail) return st;
  GemmPlan tp = plan;
  tp.ksplit = tp.cluster = plan.tail_split;
  tp.units = tp.grid = plan.tail_tiles * plan.tail_split;
  WsArgs at = args;
  at.tile0 = plan.units;
  at.ksplit = tp.ksplit;
  at.units = tp.units;
  return dispatch(tp, at);
}

int* device_error_word() {
  static std::atomic<int*> cache[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  int* p = cache[dev].load(std::memory_order_relaxed);
  if (!p) {
    void* q = nullptr;
    if (cudaGetSymbolAddress(&q, g_bq4_device_error) != cudaSuccess) return nullptr;
    p = static_cast<int*>(q);
    cache[dev].store(p, std::memory_order_relaxed);
  }
  return p;
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
