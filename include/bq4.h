/*
 * bq4.h -- C ABI of the B200-native packed signed-Q4 linear (libbq4.so).
 *
 * Drop-in boundary for burn_image's packed-Q4 dequant-matmul.  In the
 * reference the op is Burn's `QTensorOps::q_matmul` on the CubeCL backend
 * (patches/burn-cubecl-0.21.0/src/ops/qtensor.rs:303-368), reached from
 * `linear_forward` (crates/burn_boogu/src/model/linear.rs:14-37) and
 * `qwen_linear_forward` (crates/burn_qwen3_vl/src/linear.rs:107-140).
 *
 * Format (Q4S): signed 4-bit, symmetric, one f32 scale per block of `block`
 * consecutive K values (block in {8,16,32,64,128}); 8 values per
 * little-endian u32 word, value i at bits [4i, 4i+3], two's complement.
 * Three physical layouts reach the reference op:
 *   BQ4_LAYOUT_COL (QuantStore::PackedU32(0) of a [N,K] tensor seen through a
 *       transposed view, Qwen): words [N][K/8], scales [N][K/block]
 *   BQ4_LAYOUT_ROW (QuantStore::PackedU32(1) of a [K,N] tensor, Boogu):
 *       words [K/8][N], scales [K/block][N]
 *   BQ4_LAYOUT_NPACKED (QuantStore::PackedU32(0) of a plain [K,N] tensor,
 *       blocks along N, as in crates/burn_boogu/src/artifacts.rs:10501-10584):
 *       words [K][N/8], scales [K][N/block]; needs N % 8 == 0, N % block == 0.
 *       Its scale changes along K, so it is prepared as pre-expanded f16 tiles.
 *
 * Conventions: all tensor pointers passed to compute calls are DEVICE
 * pointers on the weight's device; work is enqueued on `stream` (0 = the
 * legacy default stream) and is stream-ordered.  Calls never abort: they
 * return a status and `bq4_last_error_string()` (thread-local) says why.
 * A prepared weight is immutable and may be shared by concurrent streams.
 */
#ifndef BQ4_H
#define BQ4_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define BQ4_API __attribute__((visibility("default")))
#else
#define BQ4_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* bq4_stream_t; /* == cudaStream_t */

typedef enum {
  BQ4_OK = 0,
  BQ4_EINVAL_SHAPE = 1,   /* a dimension is zero/negative or not a multiple it must be */
  BQ4_EINVAL_BLOCK = 2,   /* block not in {8,16,32,64,128} or does not divide K */
  BQ4_EALIGN = 3,         /* pointer or stride misaligned */
  BQ4_ECUDA = 4,          /* a CUDA runtime/driver call failed */
  BQ4_ENCCL = 5,          /* reserved for collective helpers */
  BQ4_ETIMEOUT = 6,       /* a bounded device-side wait expired (kernel unwound) */
  BQ4_EINVAL_ARG = 7,     /* null pointer, bad enum, unsupported scheme */
  BQ4_EWORKSPACE = 8,     /* workspace missing or smaller than bq4_*_workspace_size */
  BQ4_ENONFINITE = 9,     /* packer: non-finite input value */
  BQ4_EUNSUPPORTED = 10   /* no kernel for this device (not sm_100) */
} bq4_status;

/* BQ4_LAYOUT_F16: reported by bq4_weight_info for weights prepared from
 * packed-F16 storage (bq4_f16_weight_prepare, bq4_f16_conv_weight_prepare);
 * not accepted by the Q4 preparation calls. */
typedef enum { BQ4_LAYOUT_COL = 0, BQ4_LAYOUT_ROW = 1, BQ4_LAYOUT_NPACKED = 2, BQ4_LAYOUT_F16 = 3 } bq4_layout;

typedef enum {
  BQ4_ACT_NONE = 0,
  BQ4_ACT_GELU_TANH = 1, /* Burn Gelu::new_approximate (crates/burn_qwen3_vl/src/vision.rs:279) */
  BQ4_ACT_SILU = 2
} bq4_act;

typedef struct bq4_weight bq4_weight; /* opaque prepared weight (device resident) */

/*
 * Operand staging of the GEMM (weights with blocks of 64/128; smaller blocks
 * and N-packed weights always use FOLDED):
 *   EXACT  -- q stays exact in f16 and each K block's f32 partial is
 *             multiplied by its scale: weights enter the sum as exactly
 *             q * scale; only activations are rounded (to f16).
 *   FOLDED -- weights staged as f16(q * f16(scale)), the staging of the
 *             reference GPU kernel (patches/burn-cubecl-0.21.0/src/kernel/
 *             matmul/quantized.rs:172-178); faster at large M.
 *   AUTO   -- EXACT for M <= 64 rows, FOLDED above (default).
 * Both are f32-accumulated; both meet the 5e-3 relative-Frobenius bound.
 * The initial value comes from the environment variable BQ4_NUMERICS
 * (auto|exact|folded), else AUTO.
 */
typedef enum { BQ4_NUMERICS_AUTO = 0, BQ4_NUMERICS_EXACT = 1, BQ4_NUMERICS_FOLDED = 2 } bq4_numerics;

/* Library version string and the message of the last failed call on this thread. */
BQ4_API const char* bq4_version(void);
BQ4_API const char* bq4_last_error_string(void);

/* ---------------------------------------------------------------- weights
 * One-time re-layout of a reference-packed weight into the device layout the
 * kernels stream (replaces the upload in `new_quantized`,
 * patches/burn-cubecl-0.21.0/src/ops/qtensor.rs:64-158, called from the loader
 * hook `q_from_data`, :167-195).  `packed_words`/`scales` may be host or
 * device pointers (detected); the result lives on `device`.  K is the
 * reduction (input) width, N the output width; K % 8 == 0, K % block == 0
 * (COL/ROW).  Allocates device memory (load time only).
 */
BQ4_API bq4_status bq4_weight_prepare(const uint32_t* packed_words, const float* scales, int64_t K,
                              int64_t N, int32_t block, bq4_layout layout, int32_t device,
                              bq4_weight** out);

/* Tensor-parallel shard of a reference-packed weight, prepared directly:
 * kind 0 = column-parallel (split N into `size` equal parts, part `rank`),
 * kind 1 = row-parallel (split K on quant-block boundaries; K/size % block == 0).
 * Same pointer rules as bq4_weight_prepare. */
BQ4_API bq4_status bq4_weight_prepare_shard(const uint32_t* packed_words, const float* scales, int64_t K,
                                    int64_t N, int32_t block, bq4_layout layout, int32_t kind,
                                    int32_t rank, int32_t size, int32_t device, bq4_weight** out);

BQ4_API bq4_status bq4_weight_free(bq4_weight* w);

/* K, N, block, source layout and device bytes held by a prepared weight. */
BQ4_API bq4_status bq4_weight_info(const bq4_weight* w, int64_t* K, int64_t* N, int32_t* block,
                           int32_t* layout, size_t* device_bytes);

/* ---------------------------------------------------------------- compute
 * Workspace: every compute call that takes `workspace` needs at least the
 * bytes reported by the matching *_workspace_size query for the same M (and
 * weights); the library never allocates on these calls.  The workspace must
 * be 256-byte aligned device memory, not shared with concurrent calls.
 */
BQ4_API bq4_status bq4_linear_workspace_size(const bq4_weight* w, int64_t M, size_t* bytes);

/*
 * The launch plan bq4_linear uses for this weight and M (diagnostics and
 * tests).  Writes min(n, 13) values to info: token tile (64/128/256; the
 * tokens per CTA, 8..64, for the few-token kernel),
 * split-K factor (1 = none), grid size, exact numerics (0/1), weight tile in
 * TMEM (0/1), operand-ring stages, stream-K tiles (0 = whole tiles only),
 * whole tiles before them, workspace bytes / 256, 1 when a packed-F16
 * weight runs on 256 x 256 tiles (two N tiles per token tile), and the
 * split-K tail: tiles of the partial last wave run in a second launch, each
 * cut into the given number of K ranges (0, 0 = none), and 1 when the
 * few-token kernel runs the call (weights streamed from HBM into registers,
 * mma.sync tensor-core steps, split-K partials summed within a thread-block
 * cluster; no workspace).  gated = 1 plans the SiLU-gated pair
 * (bq4_linear_gated) with `w` as both weights.
 */
BQ4_API bq4_status bq4_linear_plan_info(const bq4_weight* w, int64_t M, int32_t gated, int32_t* info,
                                        int32_t n);

/*
 * y[M,N] = act(x[M,K] . W + bias) (* aux)   -- the fused q_matmul + epilogue.
 * x: f32, row pitch `ldx` elements (>= K); bias: f32 [N] or NULL;
 * aux: f32 [M,N] multiplied after the activation, or NULL; y: f32 [M,N]
 * contiguous.  Operands are staged as f16 with f32 accumulation, like the
 * reference GPU kernel (patches/burn-cubecl-0.21.0/src/kernel/matmul/quantized.rs:172-178).
 */
BQ4_API bq4_status bq4_linear(const bq4_weight* w, const float* x, int64_t M, int64_t ldx,
                      const float* bias, bq4_act act, const float* aux, float* y,
                      void* workspace, size_t workspace_bytes, bq4_stream_t stream);

typedef enum { BQ4_DTYPE_F32 = 0, BQ4_DTYPE_F16 = 1 } bq4_dtype;

/* Workspace for bq4_linear_ex: the bq4_linear size for f32 x; for f16 x only the split-K
 * partial tiles and the stream-K slots (0 when the plan uses neither). */
BQ4_API bq4_status bq4_linear_ex_workspace_size(const bq4_weight* w, int64_t M, bq4_dtype x_dtype,
                                                size_t* bytes);

/*
 * bq4_linear for chains of linears whose activations stay on the device in
 * the GEMM's operand format.  The reference keeps activations f32 between
 * ops and its matmul casts them to f16 on entry (quantized.rs:172-178); here
 * a linear may instead write its output already rounded to f16 (round to
 * nearest even, the same rounding the next call's staging would apply) and a
 * linear may read f16 activations in place, skipping the staging copy.  The
 * arithmetic is unchanged, so a chain computes the same bits either way.
 *   x: f32 or f16, row pitch ldx elements.  f16 x needs K % 128 == 0, a
 *      16-byte aligned base and ldx % 8 == 0.
 *   y: f32 or f16, row pitch ldy elements (>= N; 0 means N).
 *   workspace: bq4_linear_ex_workspace_size bytes (NULL allowed when 0).
 */
BQ4_API bq4_status bq4_linear_ex(const bq4_weight* w, const void* x, bq4_dtype x_dtype, int64_t M,
                                 int64_t ldx, const float* bias, bq4_act act, const float* aux, void* y,
                                 bq4_dtype y_dtype, int64_t ldy, void* workspace, size_t workspace_bytes,
                                 bq4_stream_t stream);

BQ4_API bq4_status bq4_linear_gated_workspace_size(const bq4_weight* gate, const bq4_weight* up, int64_t M,
                                           size_t* bytes);

/*
 * y[M,N] = silu(x . Wg + bg) * (x . Wu + bu): the SwiGLU front half
 * (crates/burn_boogu/src/model/feed_forward.rs:32-36,
 * crates/burn_qwen3_vl/src/text.rs:46-52) in one kernel.  gate and up must
 * have identical K, N and block.
 */
BQ4_API bq4_status bq4_linear_gated(const bq4_weight* gate, const bq4_weight* up, const float* x,
                            int64_t M, int64_t ldx, const float* gate_bias, const float* up_bias,
                            float* y, void* workspace, size_t workspace_bytes,
                            bq4_stream_t stream);

/*
 * Bit-exact dequantization of a prepared weight: out = q * scale in f32,
 * written as the logical tensor of `out_layout` (BQ4_LAYOUT_ROW: [K][N],
 * BQ4_LAYOUT_COL: [N][K]).  Not available for weights prepared from
 * BQ4_LAYOUT_NPACKED (use bq4_dequant_raw).  Mirrors the reference `dequantize`
 * (patches/burn-cubecl-0.21.0/src/kernel/quantization/dequantize.rs:6-33).
 */
BQ4_API bq4_status bq4_dequant(const bq4_weight* w, float* out, bq4_layout out_layout, bq4_stream_t stream);

/* Same, straight from reference-packed device buffers (no preparation). */
BQ4_API bq4_status bq4_dequant_raw(const uint32_t* packed_words, const float* scales, int64_t K, int64_t N,
                           int32_t block, bq4_layout layout, float* out, bq4_layout out_layout,
                           bq4_stream_t stream);

/*
 * bq4_linear for callers that cannot allocate device memory.  No
 * counterpart in the reference: its op allocates through Burn's own
 * allocator.  Some callers of this library have no way to hand it a
 * workspace -- a runtime whose allocator owns all device memory, code that
 * must not call the (device-synchronizing) cudaMalloc, or a process that may
 * not grow its device footprint after start-up.  This entry point runs the
 * GEMM of bq4_linear with its scratch in a static device array of
 * BQ4_NOALLOC_SCRATCH_BYTES that every GPU loading the library holds until
 * exit; it allocates nothing.  When bq4_linear's workspace for the same
 * weight and M fits that size, both run the same plan and the result is
 * bit-identical to bq4_linear's.  When it does not fit because of the
 * stream-K tail (whose partial slots need workspace), this call plans whole
 * tiles instead: the tiling then differs and the result agrees with
 * bq4_linear's within the parity tolerance, not bit for bit.  Calls whose
 * scratch need still exceeds the array return BQ4_EWORKSPACE.  The first
 * call on a device looks up the array's device address, so make it before
 * any stream capture.  The address is cached for the life of the process:
 * do not call this entry point after a cudaDeviceReset (or any other
 * teardown of the device's primary context) in the same process.  All calls
 * on a device share the array: calls that overlap on the GPU race.
 */
#define BQ4_NOALLOC_SCRATCH_BYTES (32u << 20)
BQ4_API bq4_status bq4_linear_noalloc(const bq4_weight* w, const float* x, int64_t M, int64_t ldx,
                                      const float* bias, bq4_act act, const float* aux, float* y,
                                      bq4_stream_t stream);

/* ------------------------------------------------------- q_matmul mirror
 * The reference op's scheme fields (burn-std 0.21 QuantScheme) on this path.
 * q_matmul accepts exactly what the reference's packed-Q4 eligibility test
 * accepts (patches/burn-cubecl-0.21.0/src/ops/qtensor.rs:304-323): f32 lhs,
 * Symmetric, Q4S, F32 params, PackedU32(0|1), Block([b]) or Block([b,1]) with
 * b in {8,16,32,64,128}.  Everything else returns BQ4_EINVAL_ARG (the
 * reference would fall to its generic quantized matmul, which has no B200
 * counterpart here).
 */
typedef struct {
  int32_t value;       /* 0 = Q4S (only accepted value) */
  int32_t mode;        /* 0 = Symmetric */
  int32_t param;       /* 0 = F32 scales */
  int32_t store_packed_dim; /* 0 = PackedU32(0), 1 = PackedU32(1) */
  int32_t block_rank;  /* 1 = Block([b]), 2 = Block([b,1]) */
  int32_t block;       /* b */
  int32_t rhs_transposed_view; /* PackedU32(0) only: 1 = rhs is the swapped-dims view of a
                                  stored [N,K] tensor (Qwen; packed along K), 0 = stored as a
                                  plain [K,N] tensor (packed and blocked along N) */
} bq4_quant_scheme;

/*
 * Row selection from a packed Q4S matrix without widening it: QTensorOps::q_select on dim 0
 * (patches/burn-cubecl-0.21.0/src/ops/qtensor.rs:267-293; kernel
 * patches/burn-cubecl-0.21.0/src/kernel/index/select.rs:83-175), the op behind the Qwen token
 * and vision-position embedding tables.  The matrix is rows x cols logical values stored as
 * PackedU32(0) with blocks along the row: values u32 [rows][cols/8], scales f32
 * [rows][cols/block].  ids: n row indices on the device, int32 (ids_i64 = 0) or int64.
 * Output: out_values [n][cols/8], out_scales [n][cols/block] (device).  The reference does not
 * check indices; here an index outside [0, rows) selects a zero row and records BQ4_EINVAL_ARG,
 * reported by bq4_poll_device_error.
 */
BQ4_API bq4_status bq4_q_select_rows(const uint32_t* values, const float* scales, int64_t rows, int64_t cols,
                                     int32_t block, const void* ids, int32_t ids_i64, int64_t n,
                                     uint32_t* out_values, float* out_scales, bq4_stream_t stream);

/* The same selection dequantized in the same pass (what an embedding lookup does next with
 * the selected rows, dequantize.rs:6-33): out f32 [n][cols] = q * scale, bit-exact; out must be
 * 16-byte aligned. */
BQ4_API bq4_status bq4_q_select_rows_dequant(const uint32_t* values, const float* scales, int64_t rows, int64_t cols,
                                             int32_t block, const void* ids, int32_t ids_i64, int64_t n, float* out,
                                             bq4_stream_t stream);

/*
 * Stored-dtype spelling of a packed-Q4 tensor in the reference's sealed artifact inventory
 * (q4s_stored_dtype, crates/burn_boogu/src/artifacts.rs:527-537): "q4s-block{b}-f32-packed-axis0"
 * (PackedU32(0), Block([b])) or "q4s-block{b}x1-f32-packed-axis1" (PackedU32(1), Block([b,1])).
 * Returns the block and packed axis; BQ4_EINVAL_ARG for any other spelling.
 */
BQ4_API bq4_status bq4_parse_stored_dtype(const char* stored_dtype, int32_t* block, int32_t* axis);

/*
 * Loader hook: prepare a weight straight from a stored tensor's QFloat payload, the byte
 * stream the reference writes (crates/burn_qwen3_vl/src/artifacts.rs:1356-1363: every packed
 * u32 word little-endian, then every f32 scale) and whose size it checks
 * (crates/burn_qwen3_vl/src/artifacts.rs:1204-1240).  rows x cols is the stored tensor's
 * shape and stored_dtype its inventory spelling.  axis 1: the stored tensor is the [K, N]
 * weight (Boogu row layout).  axis 0: packed along cols; transposed_view = 1 when the matmul
 * uses it as the transposed view of a stored [N, K] weight (Qwen), 0 when it is a plain
 * [K, N] weight.  The payload is host or device memory; nbytes must equal
 * rows*cols/2 + rows*cols/block*4 (BQ4_EINVAL_SHAPE otherwise).
 */
BQ4_API bq4_status bq4_weight_prepare_payload(const void* payload, size_t nbytes, int64_t rows, int64_t cols,
                                              const char* stored_dtype, int32_t transposed_view, int32_t device,
                                              bq4_weight** out);

/* Workspace for bq4_q_matmul: covers an internal prepared copy of rhs. */
BQ4_API bq4_status bq4_q_matmul_workspace_size(int64_t M, int64_t K, int64_t N,
                                               const bq4_quant_scheme* scheme, size_t* bytes);

/*
 * lhs f32 [M,K] (contiguous, M = product of leading dims) times the
 * quantized rhs of logical shape [K,N] (values/scales device buffers as the
 * reference stores them) -> out f32 [M,N].  Prepares rhs into the workspace
 * on every call; production callers prepare once with bq4_weight_prepare.
 */
BQ4_API bq4_status bq4_q_matmul(const float* lhs, int64_t M, int64_t K, const uint32_t* rhs_values,
                        const float* rhs_scales, int64_t N, const bq4_quant_scheme* scheme,
                        float* out, void* workspace, size_t workspace_bytes, bq4_stream_t stream);

/* ------------------------------------------------------- host packers
 * The reference's load-time quantizers, host code.  Outputs are the
 * reference byte streams split into words and scales.
 *   column layout: crates/burn_qwen3_vl/src/artifacts.rs:1301-1366
 *     values [rows][inner], inner % 128 == 0 -> words rows*inner/8, scales rows*inner/128
 *   row layout: crates/burn_boogu/src/artifacts.rs:7296-7385
 *     values [input][output], output % 8 == 0 -> words [input/8][output],
 *     scales [input/b][output], b = largest of {128,64,32,16,8} dividing input
 */
BQ4_API bq4_status bq4_quantize_col_block128(const float* values, int64_t rows, int64_t inner,
                                     uint32_t* words, float* scales);
BQ4_API bq4_status bq4_quantize_row_up_to128(const float* values, int64_t input, int64_t output,
                                     uint32_t* words, float* scales, int32_t* block);

/* Row-layout block policy (crates/burn_boogu/src/artifacts.rs:513-525); 0 if none. */
BQ4_API int32_t bq4_row_block_for(int64_t input);

/* Reads and clears the device-side error word of the current device: BQ4_OK, or
 * BQ4_ETIMEOUT when a kernel's bounded wait expired since the last poll (the
 * kernel unwound without trapping; its output is invalid).  Synchronizes. */
BQ4_API bq4_status bq4_poll_device_error(void);

/* Process-wide operand staging for subsequent compute calls (see bq4_numerics). */
BQ4_API bq4_status bq4_set_numerics(bq4_numerics mode);

/* Caps the CTAs (one per SM) that a GEMM launch keeps resident, process-wide;
 * 0 (the default, or the environment variable BQ4_SM_BUDGET) means every SM.
 * A GEMM otherwise occupies the whole GPU until it ends; a cap leaves SMs for
 * kernels on other streams, e.g. NCCL collectives meant to overlap it.  The
 * reference has no counterpart (it runs on one device). */
BQ4_API bq4_status bq4_set_sm_budget(int32_t sms);

/* Per-token RMS renormalisation, out[m,:] = x[m,:] / sqrt(mean(x[m,:]^2) +
 * eps), f32 arithmetic, f32 or f16 in and out, rows of H values at pitches
 * ldx / ldo.  Not a step of the reference's Q4 path: it is the between-block
 * step of the DiT-shaped layer-stack workload (activations renormalised per
 * block), provided so that workload runs in one kernel per block. */
BQ4_API bq4_status bq4_rms_renorm(const void* x, bq4_dtype x_dtype, int64_t M, int64_t H, int64_t ldx, void* out,
                                  bq4_dtype out_dtype, int64_t ldo, float eps, bq4_stream_t stream);

/*
 * QK-norm + RoPE, the step between the q/k projections and attention
 * (crates/burn_boogu/src/model/attention.rs:114-133): for each of M tokens
 * and `heads` heads of head_dim values of x (row pitch ldx elements),
 *   v = x / sqrt(mean(x^2) + eps) * gamma          (Burn nn::RmsNorm, StrictF32)
 *   y[2p]   = v[2p] cos[2p] - v[2p+1] sin[2p]       (apply_rope, :916-928)
 *   y[2p+1] = v[2p+1] cos[2p+1] + v[2p] sin[2p+1]
 * with cos/sin f32 [M][head_dim] at row pitch ld_rope (both NULL: no
 * rotation) and gamma f32 [head_dim] (NULL: ones).  x and y are f32 or f16
 * at pitches ldx / ldy and may be the same buffer (same dtype and pitch).
 * head_dim is even and at most 256.  Call it once for the q section and once
 * for the k section of a projection output (their gammas differ).
 */
BQ4_API bq4_status bq4_qk_norm_rope(const void* x, bq4_dtype x_dtype, int64_t M, int64_t heads, int64_t head_dim,
                                    int64_t ldx, const float* gamma, float eps, const float* cos_t,
                                    const float* sin_t, int64_t ld_rope, void* y, bq4_dtype y_dtype, int64_t ldy,
                                    bq4_stream_t stream);

/*
 * A q/k/v projection with QK-norm + RoPE: y = x . W + bias, whose N features
 * are q_heads heads, then k_heads heads, then the remaining (v) heads, all of
 * head_dim values; the q and k heads then get bq4_qk_norm_rope with gamma_q
 * and gamma_k (the reference's separate q/k/v linears followed by
 * attention.rs:114-133).  With head_dim == 128 every 128-feature tile of the
 * GEMM is one head and the norm and rotation run in the GEMM's epilogue (no
 * second pass over y); otherwise the linear is followed by bq4_qk_norm_rope
 * in place on y.  x: f32 or f16 (as bq4_linear_ex), y: f32 or f16 at pitch
 * ldy (0 = N).  Workspace from bq4_linear_qk_norm_rope_workspace_size.
 */
BQ4_API bq4_status bq4_linear_qk_norm_rope_workspace_size(const bq4_weight* w, int64_t M, bq4_dtype x_dtype,
                                                          int64_t head_dim, size_t* bytes);
BQ4_API bq4_status bq4_linear_qk_norm_rope(const bq4_weight* w, const void* x, bq4_dtype x_dtype, int64_t M,
                                           int64_t ldx, const float* bias, int64_t q_heads, int64_t k_heads,
                                           int64_t head_dim, const float* gamma_q, const float* gamma_k, float eps,
                                           const float* cos_t, const float* sin_t, int64_t ld_rope, void* y,
                                           bq4_dtype y_dtype, int64_t ldy, void* workspace, size_t workspace_bytes,
                                           bq4_stream_t stream);

/*
 * Tensor-parallel exchange over NVLink peer memory (one process per GPU of
 * one node).  It replaces the all-reduce after a row-parallel linear
 * (o, down):
 *   1. bq4_linear_rowscatter: every rank computes its K-partial and the GEMM
 *      epilogue writes output row m straight into the receive buffer of its
 *      owner rank m / (M / nranks), at row (rank * M/nranks + m % (M/nranks)),
 *      so the exchange overlaps the GEMM;
 *   2. bq4_peer_signal_wait: a one-thread kernel publishes `epoch` to every
 *      peer's flag array and waits (bounded, 10 s) until all peers did;
 *   3. bq4_reduce_slices: each owner sums the nranks partials of its rows in
 *      rank order, optionally RMS-renormalising them, into f16/f32 rows.
 * Buffers are cudaMalloc allocations shared with CUDA IPC handles
 * (BQ4_IPC_HANDLE_BYTES bytes, exchanged by the caller, e.g. with an
 * all-gather); plain peer loads and stores between GPUs.  The reference runs
 * on one device and has no counterpart.
 */
#define BQ4_MAX_PEERS 8
#define BQ4_IPC_HANDLE_BYTES 64
/* Allocates `bytes` of zeroed device memory on `device` and writes its IPC handle. */
BQ4_API bq4_status bq4_peer_buffer_alloc(size_t bytes, int32_t device, void** ptr, void* handle);
/* Maps a peer's buffer (handle from bq4_peer_buffer_alloc in another process) on `device`. */
BQ4_API bq4_status bq4_peer_buffer_open(const void* handle, int32_t device, void** ptr);
BQ4_API bq4_status bq4_peer_buffer_close(void* ptr);
BQ4_API bq4_status bq4_peer_buffer_free(void* ptr, int32_t device);
/* flags: this rank's [nranks] u32 array; peer_flags[r]: rank r's array as
 * mapped here (peer_flags[rank] may be `flags`).  epoch grows by one per use. */
BQ4_API bq4_status bq4_peer_signal_wait(uint32_t* flags, uint32_t* const* peer_flags, int32_t nranks, int32_t rank,
                                        uint32_t epoch, bq4_stream_t stream);
/* Bound of bq4_peer_signal_wait for launches enqueued after this call, in
 * nanoseconds of the GPU's global timer, process-wide; 0 restores the 10 s
 * default.  A wait that runs out records BQ4_ETIMEOUT in the device error word
 * (bq4_poll_device_error) and its kernel returns.  No counterpart in the
 * reference, which has no cross-GPU wait. */
BQ4_API bq4_status bq4_set_peer_wait_timeout_ns(uint64_t ns);
/* out[r] = sum_s recv[s][r] (s = 0..nranks-1 in order) for rows r < rows of
 * H floats (recv pitch ld, H % 4 == 0, H <= 8192, 16-byte aligned), then
 * x / sqrt(mean(x^2) + eps) per row when renorm; out f32 or f16 at pitch ldo. */
BQ4_API bq4_status bq4_reduce_slices(const float* recv, int32_t nranks, int64_t rows, int64_t H, int64_t ld,
                                     int32_t renorm, float eps, void* out, bq4_dtype out_dtype, int64_t ldo,
                                     bq4_stream_t stream);
/* The pull form of the exchange: out[r] = sum_s src_ranks[s][(row0 + r) ld ..]
 * over s = 0..nranks-1 in order, for rows r < rows of H floats (H % 4 == 0,
 * H <= 8192, ld % 4 == 0, every src_ranks[s] 16-byte aligned), then the
 * optional renorm, as bq4_reduce_slices.  src_ranks[s] is rank s's own f32
 * partial product [M][ld] (written by a plain bq4_linear_ex into a buffer
 * shared with bq4_peer_buffer_alloc / _open), read over peer memory after a
 * bq4_peer_signal_wait; row0 = rank * rows.  No counterpart in the
 * reference, which has no multi-GPU code. */
BQ4_API bq4_status bq4_reduce_slices_peer(const float* const* src_ranks, int32_t nranks, int64_t row0, int64_t rows,
                                          int64_t H, int64_t ld, int32_t renorm, float eps, void* out,
                                          bq4_dtype out_dtype, int64_t ldo, bq4_stream_t stream);
/* bq4_reduce_slices_peer that writes the reduced rows into every rank's copy
 * of the activations instead of one local output: row r of the result goes
 * to out_ranks[q] + (row0 + r) * ldo for q = 0..nranks-1 (rank q's [M][ldo]
 * buffer, shared with bq4_peer_buffer_alloc / _open), which replaces the
 * all-gather that follows the reduction; a bq4_peer_signal_wait afterwards
 * tells every rank that its copy is complete.  No counterpart in the
 * reference, which has no multi-GPU code. */
BQ4_API bq4_status bq4_reduce_slices_peer_bcast(const float* const* src_ranks, int32_t nranks, int64_t row0,
                                                int64_t rows, int64_t H, int64_t ld, int32_t renorm, float eps,
                                                void* const* out_ranks, bq4_dtype out_dtype, int64_t ldo,
                                                bq4_stream_t stream);
/* bq4_linear_ex with f32 output scattered by row owner (see above):
 * y_ranks[r] = rank r's receive buffer [nranks][M/nranks][ldy] f32 as mapped
 * here; M % nranks == 0.  Workspace as bq4_linear_ex. */
BQ4_API bq4_status bq4_linear_rowscatter(const bq4_weight* w, const void* x, bq4_dtype x_dtype, int64_t M,
                                         int64_t ldx, const float* bias, bq4_act act, float* const* y_ranks,
                                         int32_t nranks, int32_t rank, int64_t ldy, void* workspace,
                                         size_t workspace_bytes, bq4_stream_t stream);

/* Kernel launches issued by this thread since the last reset (bench accounting). */
BQ4_API uint64_t bq4_launch_count(void);
BQ4_API void bq4_launch_count_reset(void);

/* ---------------------------------------------------------------- packed F16
 * IEEE binary16 storage bound as u32 words, two values per word, the
 * even-index value in the low half: the VAE's weights and the F16 profiles'
 * tables.  Counterparts of the four kernels of
 * patches/burn-cubecl-0.21.0/src/kernel/packed_f16.rs, which the reference
 * dispatches when a device lacks typed f16 (ops/tensor.rs:164-165, 222-223,
 * 697-698; ops/module.rs:73-74).  Widening is bit-exact to the binary16
 * value, NaN payloads kept with the quiet bit set (packed_f16.rs:48-74).
 * The matmul and convolution run on the tensor cores as kind::tf32: every
 * f16 weight is exact in tf32, the f32 activations enter with their top 10
 * mantissa bits (cut for matmul rows read in place, rounded to nearest by the
 * convolution's staging pass), and accumulation is f32; both meet the 5e-3
 * relative-Frobenius bound and reproduce the reference's small-integer cases
 * exactly.  Element strides and offsets below count f16 values.
 */

/* packed_f16_to_f32 (packed_f16.rs:88-131): out (contiguous, `rank` <= 8
 * dims of `shape`) = the widened values at sum(coord * strides) of packed. */
BQ4_API bq4_status bq4_packed_f16_to_f32(const uint32_t* packed, int32_t rank, const int64_t* shape,
                                         const int64_t* strides, float* out, bq4_stream_t stream);

/* packed_f16_select_rows (packed_f16.rs:296-358): out f32 [n][cols] = rows
 * indices[i] of the contiguous table [rows][cols].  The reference does not
 * check indices; here an index outside [0, rows) gives a zero row and records
 * BQ4_EINVAL_ARG, reported by bq4_poll_device_error. */
BQ4_API bq4_status bq4_packed_f16_select_rows(const uint32_t* table, int64_t rows, int64_t cols,
                                              const int32_t* indices, int64_t n, float* out,
                                              bq4_stream_t stream);

/* One-time preparation of a packed-F16 matmul rhs of logical shape [K, N],
 * element (k, n) at k * inner_stride + n * col_stride (the zero-copy
 * transposed view of a stored [N, K] checkpoint: inner 1, col K).  Host or
 * device source.  The result works with bq4_linear / bq4_linear_ex (f32 x
 * with 16-byte aligned rows and ldx % 4 == 0, bias and activations fused). */
BQ4_API bq4_status bq4_f16_weight_prepare(const uint32_t* packed, int64_t K, int64_t N, int64_t inner_stride,
                                          int64_t col_stride, int32_t device, bq4_weight** out);

/* packed_f16_rhs_matmul (packed_f16.rs:133-292): lhs f32 [M, K] contiguous
 * (16-byte aligned when K % 4 == 0) times the packed rhs above -> out f32
 * [M, N].  Prepares rhs into the workspace on every call. */
BQ4_API bq4_status bq4_packed_f16_rhs_matmul_workspace_size(int64_t M, int64_t K, int64_t N, size_t* bytes);
BQ4_API bq4_status bq4_packed_f16_rhs_matmul(const float* lhs, int64_t M, int64_t K, const uint32_t* packed_rhs,
                                             int64_t inner_stride, int64_t col_stride, int64_t N, float* out,
                                             void* workspace, size_t workspace_bytes, bq4_stream_t stream);

/* Burn ConvOptions<2>: [height, width] pairs; groups must be 1. */
typedef struct {
  int32_t stride[2];
  int32_t padding[2];
  int32_t dilation[2];
  int32_t groups;
} bq4_conv2d_options;

/* One-time preparation of an OIHW packed-F16 convolution weight
 * [out_channels][in_channels][kernel_h][kernel_w] (host or device). */
BQ4_API bq4_status bq4_f16_conv_weight_prepare(const uint32_t* packed_oihw, int64_t out_channels,
                                               int64_t in_channels, int32_t kernel_h, int32_t kernel_w,
                                               int32_t device, bq4_weight** out);

/* Convolution with a prepared weight: input f32 NCHW [batch][in_channels]
 * [in_h][in_w], bias f32 [out_channels] or NULL -> out f32 NCHW [batch]
 * [out_channels][out_h][out_w], out_h = (in_h + 2 pad - dil (kh - 1) - 1) /
 * stride + 1 (likewise out_w). */
BQ4_API bq4_status bq4_conv2d_workspace_size(const bq4_weight* w, int64_t batch, int64_t in_h, int64_t in_w,
                                             const bq4_conv2d_options* options, size_t* bytes);
BQ4_API bq4_status bq4_conv2d(const float* input, int64_t batch, int64_t in_h, int64_t in_w, const bq4_weight* w,
                              const float* bias, const bq4_conv2d_options* options, float* out, void* workspace,
                              size_t workspace_bytes, bq4_stream_t stream);

/* packed_f16_conv2d (packed_f16.rs:421-602): the same from the stored OIHW
 * packed weight, prepared into the workspace on every call. */
BQ4_API bq4_status bq4_packed_f16_conv2d_workspace_size(int64_t batch, int64_t in_channels, int64_t in_h,
                                                        int64_t in_w, int64_t out_channels, int32_t kernel_h,
                                                        int32_t kernel_w, const bq4_conv2d_options* options,
                                                        size_t* bytes);
BQ4_API bq4_status bq4_packed_f16_conv2d(const float* input, int64_t batch, int64_t in_channels, int64_t in_h,
                                         int64_t in_w, const uint32_t* packed_weight, int64_t out_channels,
                                         int32_t kernel_h, int32_t kernel_w, const float* bias,
                                         const bq4_conv2d_options* options, float* out, void* workspace,
                                         size_t workspace_bytes, bq4_stream_t stream);

/* ---------------------------------------------------------------- attention
 * The consumer of the q/k/v projection (crates/burn_boogu/src/model/
 * attention.rs:636-716; the reference runs it as the third-party cubek
 * FlashAttention, native_flash.rs:1006-1100, and tests it against Burn's
 * `attention`, e.g. native_flash.rs:2784-2843): out = softmax(scale q k^T) v
 * for every batch and query head, no mask.  q [B][Hq][Sq][D], k and v
 * [B][Hkv][Skv][D], binary16 (packed-F16 storage), contiguous; query head h
 * reads kv head h / (Hq / Hkv) (grouped-query attention, Hq % Hkv == 0).
 * out f32 [B][Hq][Sq][D], 16-byte aligned.  scale <= 0 means 1/sqrt(D).
 * D % 4 == 0; q, k, v 16-byte aligned.  D = 128 runs one fused kernel
 * (scores, P and O in TMEM, softmax in registers; v transposed once into
 * the workspace); it needs B*Hq*Sq and B*Hkv*Skv below 2^31 - 256 and
 * B*Hkv <= 65535, else BQ4_EINVAL_SHAPE from both calls.  Other D run unfused: per
 * head the scores q k^T and P v as tf32 GEMMs (k and v widened into the
 * weight tiles, q and the f32 scores read in place) with a row softmax
 * between them.  The environment variable BQ4_ATTN_UNFUSED=1 selects the
 * unfused path for D = 128 too. */
BQ4_API bq4_status bq4_attention_workspace_size(int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Skv,
                                                int64_t D, size_t* bytes);
BQ4_API bq4_status bq4_attention(const uint32_t* q, const uint32_t* k, const uint32_t* v, int64_t B, int64_t Hq,
                                 int64_t Hkv, int64_t Sq, int64_t Skv, int64_t D, float scale, float* out,
                                 void* workspace, size_t workspace_bytes, bq4_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* BQ4_H */
