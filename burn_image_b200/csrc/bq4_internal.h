// bq4_internal.h -- definitions shared by the libbq4 translation units.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/bq4.h"

// Prepared ("re-laid-out") weight.  Device layout, chosen so that one
// (out-feature tile, K chunk) of nibbles is one contiguous 4 KiB block that a
// single 1-D bulk copy brings into shared memory, and so that 128 threads
// read it with two fully coalesced 16-byte loads each:
//
//   q: u32 [ntiles][nkc][2][128][4]   tile = 128 output rows (n), chunk = 64 K
//        half h, row r, word j hold K = 64*kc + 32*h + 8*j .. +7 of row n.
//        Inside a word the nibbles are permuted so that bits [4p,4p+3] hold
//        logical lane kPermLane[p] = {0,2,4,6,1,3,5,7}[p]: the pair
//        ((w >> 4i) & 0x000F000F) is then (lane 2i, lane 2i+1), i.e. two
//        consecutive K values land in the low/high halves of an f16x2.
//   s: f32 [ntiles][nkb][128]          scale of (row, K block), 0 in padding
//
// N is padded to Np = 128*ntiles and K to Kp = 128*(nkc/2) with zero nibbles
// and zero scales (nkc is even); nkb = Kp / block.
struct bq4_weight {
  int64_t K, N;
  int64_t Kp, Np;
  int64_t nkc, nkb, ntiles;
  int32_t block;
  int32_t layout;  // source layout (informational)
  int32_t device;
  uint32_t* q;
  float* s;
  size_t q_bytes, s_bytes;
  // Pre-expanded form (BQ4_LAYOUT_NPACKED sources): f16(q * scale) tiles,
  // [ntiles][nkc][128 rows][64 K] f16 with the 128-byte swizzle already
  // applied (16-byte chunk j of row r stored at chunk j ^ (r & 7)), so one
  // 16 KiB bulk copy lands as an MMA-ready operand tile.  q/s unused.
  uint16_t* h;
  size_t h_bytes;
  // Packed-F16 weights (tf32 = 1): h holds f32 tiles of tf32-exact widened
  // f16 values, [ntiles][nkc][128][16] in 64-byte rows with the 64-byte
  // swizzle (linear: a chunk is 16 K, Kp a multiple of 32), or
  // [ntiles][nkc][128][32] in 128-byte rows with the 128-byte swizzle
  // (convolution, conv_kh > 0: a chunk is 32 K, Kp a multiple of 64).
  // The linear's tile array holds an even number of tiles (a zero tile after
  // an odd last one), so that N tiles can be taken in pairs.
  // Convolution weights order K as (tap = ky * conv_kw + kx, channel):
  // K = taps * conv_cp, channels padded to conv_cp = a multiple of 32 with zeros.
  int32_t tf32;
  int32_t conv_kh, conv_kw, conv_cin, conv_cp;
};

namespace bq4 {

constexpr int kTileN = 128;   // output features per tile (MMA M)
constexpr int kChunkK = 64;   // K per MMA operand sub-tile (128 B of f16)
constexpr int kStageK = 128;  // K per pipeline stage (two sub-tiles); K is padded to it

// Error plumbing (thread-local message, see bq4_api.cu).
bq4_status set_error(bq4_status code, const char* fmt, ...);
bq4_status check_cuda(cudaError_t e, const char* what);
void note_launch(uint64_t n = 1);

// ------------------------------------------------------------ kernels (bq4_kernels.cu)
cudaError_t launch_prepare(const uint32_t* words, const float* scales, int64_t K, int64_t N,
                           int32_t block, int32_t layout, int64_t n0, int64_t k0,
                           int64_t src_N, int64_t src_K, const bq4_weight* w, cudaStream_t s);
cudaError_t launch_prepare_pre(const uint32_t* words, const float* scales, int64_t K, int64_t N,
                               int32_t block, int64_t n0, int64_t k0, int64_t src_N, int64_t src_K,
                               const bq4_weight* w, cudaStream_t s);
cudaError_t launch_dequant_prepared(const bq4_weight* w, float* out, int32_t out_layout,
                                    cudaStream_t s);
cudaError_t launch_dequant_raw(const uint32_t* words, const float* scales, int64_t K, int64_t N,
                               int32_t block, int32_t layout, float* out, int32_t out_layout,
                               cudaStream_t s);
// x f32 [M][ldx] -> xh f16 [M][Kp] (zero padded); also zeroes nflags
// stream-K flags (flags may be null when nflags is 0).
cudaError_t launch_convert_x(const float* x, int64_t M, int64_t K, int64_t ldx, int64_t Kp,
                             void* xh, unsigned* flags, int nflags, cudaStream_t s);
cudaError_t launch_zero_flags(unsigned* flags, int nflags, cudaStream_t s);
// Tensor-parallel exchange over peer memory (bq4_peer.cu).
cudaError_t launch_peer_signal_wait(unsigned* local, unsigned* const* peers, int nranks, int rank, unsigned epoch,
                                    int* err, cudaStream_t s);
// Bound of the peer signal/wait in ns for launches after the call (0 = the 10 s default).
void set_peer_wait_ns(uint64_t ns);
cudaError_t launch_reduce_slices(const float* recv, int P, int64_t R, int64_t H, int64_t ld, int renorm, float eps,
                                 void* out, int out_f16, int64_t ldo, cudaStream_t s);
// As launch_reduce_slices with slice s = rows [row0, row0 + R) of src_ranks[s]
// (pitch ld); with out_ranks (P pointers), row r of the result goes to
// out_ranks[q] + (row0 + r) * ldo for every q instead of out.
cudaError_t launch_reduce_slices_peer(const float* const* src_ranks, int P, int64_t row0, int64_t R, int64_t H,
                                      int64_t ld, int renorm, float eps, void* out, void* const* out_ranks,
                                      int out_f16, int64_t ldo, cudaStream_t s);
// QK-norm + RoPE over `heads` heads of hd (even, <= 256) per token; cos/sin
// NULL skips the rotation, gamma NULL means ones.
cudaError_t launch_qk_norm_rope(const void* x, int x_f16, int64_t M, int heads, int hd, int64_t ldx,
                                const float* gamma, float eps, const float* cos_t, const float* sin_t, int64_t ldr,
                                void* y, int y_f16, int64_t ldy, cudaStream_t s);

// Packed-Q4 row selection (q_select on dim 0), optionally dequantized.
cudaError_t launch_select_rows(const uint32_t* values, const float* scales, int64_t rows, int64_t cols, int block,
                               const void* ids, int ids64, int64_t n, uint32_t* out_values, float* out_scales,
                               float* out_f32, int* err, cudaStream_t s);
// Device address of the error word bq4_poll_device_error reads, on the
// current device (for kernels compiled outside the GEMM's unit).
int* device_error_word();

// Per-row RMS renormalisation (the layer-stack workload's between-block step).
cudaError_t launch_rms_renorm(const void* x, int x_f16, int64_t M, int64_t H, int64_t ldx, void* out,
                              int out_f16, int64_t ldo, float eps, cudaStream_t s);

// ------------------------------------------------------------ small-M linear (bq4_skinny.cu)
// Launch plan of the few-token kernel: 8 * nt tokens per CTA (gz token
// groups), one 128-row weight tile per CTA (gx CTAs along N; R = 8 row
// groups), ks CTAs per cluster splitting K, a ring of `stages` 128-K weight
// stages per CTA.  It needs no workspace.
constexpr int64_t kSkMaxM = 256;             // calls above this many rows always use the tcgen05 GEMM
constexpr int64_t kSkAutoMaxM = 16;          // the planner's default: the few-token kernel up to this many rows
constexpr size_t kSkMaxSmem = 200 * 1024;    // dynamic shared memory limit of one CTA
struct SkPlan {
  int nt, nw, R, ks, gx, gz, exact, pdl, stages;
  int minb;  // CTAs the kernel is compiled to fit on one SM (2, or 3 for the one-weight few-token cases)
  size_t smem_bytes;
};
// false when the weight or numerics do not fit the kernel (pre-expanded or
// packed-F16 weights, exact numerics with blocks other than 128, M above
// kSkMaxM, shared memory).
bool plan_skinny(const bq4_weight* w, int nw, int64_t M, int device, bool exact, SkPlan* p);

// ------------------------------------------------------------ GEMM (bq4_gemm_sm100.cu)
struct GemmPlan {
  int nw;          // 1 = plain, 2 = gated (gate, up)
  int exact;       // 1 = exact-weight kernel (scale on the f32 accumulator)
  int pre;         // 1 = pre-expanded f16 weight tiles (bulk-copied, no dequant)
  int lockstep;    // 1 = exact mode with stage == segment partial handoff
  int bt;          // tokens per tile (MMA N): 64, 128 or 256
  int mtiles, ntiles, ksplit, units, grid;
  int cluster;     // CTAs per cluster (= ksplit when the K range is split, else 1)
  int nfast;       // 1: N tile varies fastest along the unit order
  int pdl;         // 1: GEMM launched as a programmatic dependent of the staging grid
  int ta;          // 1: operand A (dequantized weights) staged in TMEM, not shared memory
  int qk;          // 1: QK-norm + RoPE epilogue (every 128-feature tile one head)
  int tf;          // 1: packed-F16 weight, kind::tf32 on f32 token rows (no staging pass)
  int cv;          // 1: implicit-GEMM convolution (tf32, NCHW epilogue)
  int wide;        // 1: tf32 linear on 256 x 256 tiles (two N tiles per token tile); ntiles = pairs
  // split-K tail launch: units/grid describe the whole tiles [0, units);
  // tiles [units, units + tail_tiles) follow in a second launch, each cut
  // into tail_split K ranges (clusters of tail_split CTAs)
  int tail_tiles, tail_split;
  int stages, a_stages, raw_stages;  // B ring, A ring, raw ring depths
  uint32_t raw_s_bytes;  // scale bytes per weight per raw stage (folded)
  uint32_t raw_w_bytes;  // shared-memory bytes per weight per raw stage
  size_t smem_bytes;
  int dp_tiles, sk_tiles;  // stream-K tail: tiles dealt as equal stage ranges (0 = none)
  size_t sk_bytes;         // workspace part 0: stream-K partial slots + flags (0 without)
  size_t partial_bytes;    // workspace part 1: split-K partial tiles (0 without split)
  size_t xh_bytes;         // workspace part 2: the f16 copy of x (unused with f16 x)
  size_t workspace_bytes;
  int skinny;              // 1: the few-token kernel runs the call (plan in sk; no workspace)
  SkPlan sk;
};

// allow_sk = false plans without the stream-K tail (smaller workspace);
// qk = true plans the QK-norm + RoPE epilogue (whole-K tiles of 128 or 256
// tokens, shared memory for its reduction).
bq4_status plan_gemm(const bq4_weight* w, int nw, int64_t M, int device, GemmPlan* plan, bool allow_sk = true,
                     bool qk = false, bool cv = false);

// Activation / output formats of one GEMM call: x f32 (staged to f16 in the
// workspace) or f16 (read in place; needs K == Kp), y f32 or f16 with row
// pitch ldy elements (0 = N).
// Parameters of the QK-norm + RoPE epilogue (head_dim 128).
struct QkParams {
  int q_heads = 0, k_heads = 0;
  float eps = 1e-5f;
  const float* gamma_q = nullptr;
  const float* gamma_k = nullptr;
  const float* cos_t = nullptr;
  const float* sin_t = nullptr;
  int64_t ld_rope = 128;
};

// Geometry of an implicit-GEMM convolution (kernels built with CV): see
// WsArgs::cv_* in bq4_gemm_sm100.cu.  x_cols = f32 values per token row of
// the staged activations (the row pitch too).
struct ConvGeom {
  int cchunks = 1, taps = 1, kw = 1, dy = 0, dx = 0;
  int hp = 1, wp = 1, oh = 1, ow = 1;
  int64_t x_cols = 0;
};

struct GemmIo {
  int x_f16 = 0;
  int y_f16 = 0;
  int64_t ldy = 0;
  // Row scatter (f32 y): output row m goes to sc_y[m / sc_rows] at row
  // sc_rank * sc_rows + m % sc_rows (each owner's [nranks][rows][ldy] receive buffer).
  int sc_rows = 0, sc_rank = 0, sc_nranks = 0;
  float* const* sc_y = nullptr;
  const QkParams* qk = nullptr;  // with a plan from plan_gemm(..., qk = true)
  const ConvGeom* cv = nullptr;  // with a plan from plan_gemm(..., cv = true)
};

bq4_status run_gemm(const GemmPlan& plan, const bq4_weight* const* ws, const void* x, int64_t M,
                    int64_t ldx, const float* const* bias, int act, const float* aux, void* y,
                    void* workspace, cudaStream_t stream, const GemmIo& io = GemmIo());

// The few-token kernel (bq4_skinny.cu) for a plan with skinny = 1.
bq4_status run_skinny(const SkPlan& p, const bq4_weight* const* ws, const void* x, int x_f16, int64_t M, int64_t ldx,
                      const float* const* bias, int act, const float* aux, void* y, int y_f16, int64_t ldy,
                      const GemmIo& io, cudaStream_t stream);

// Operand staging policy (bq4_numerics); AUTO keeps exact weights up to
// this many rows: the reference's own kernel test at M = 1 asks for a
// relative RMSE below 1e-4, which no f16 staging of the weights meets.
// Above it AUTO stages folded weights, the reference GPU kernel's staging,
// measured faster than exact on every M = 256 shape of the text encoder
// (q/o 19.6 vs 21.8 us, k/v 14.2 vs 15.1, gate/up 60.1 vs 69.1, down 27.8
// vs 36.7).
constexpr int64_t kAutoExactMaxM = 64;
int numerics_mode();
void set_numerics_mode(int mode);
// Resident-CTA cap for GEMM launches (0 = every SM).
int sm_budget();
void set_sm_budget(int sms);

int device_sm_count(int device);
int device_is_sm100(int device);

}  // namespace bq4
