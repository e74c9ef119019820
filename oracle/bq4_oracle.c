/*
 * bq4_oracle.c -- CPU restatement of burn_image's packed signed-Q4 linear path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * product in burn_image_b200/csrc and the timed CPU baseline of bench.py.
 * Only tests/, __graft_entry__.smoke() and bench.py (cpu_baseline leg and the
 * `--impl reference` arm) may load it.  The product path never calls it.
 *
 * The reference (mosure/burn_image) is Rust and cannot be compiled in this
 * environment, so every function below restates the reference's algorithm
 * from its source, citing file:line (paths relative to the reference root):
 *
 *   - quantize_q4s_block128_f32 (column layout, PackedU32(0))
 *       crates/burn_qwen3_vl/src/artifacts.rs:1301-1366
 *       crates/burn_boogu/src/artifacts.rs:7203-7290
 *   - quantize_row_layout_q4s_block_up_to128_f32 (row layout, PackedU32(1))
 *       crates/burn_boogu/src/artifacts.rs:7296-7385
 *       block policy crates/burn_boogu/src/artifacts.rs:513-525
 *   - unpack: nibble at bits [4i,4i+3] of a little-endian u32, sign-extended
 *       4-bit two's complement, times the f32 scale of its block.  Packers write
 *       `(q as u8) & 0x0f` (crates/burn_boogu/src/artifacts.rs:7252,7370) and
 *       tests rebuild `f32::from(q) * scale`
 *       (crates/burn_boogu/src/artifacts.rs:10428-10441).  Nibble 0x8 (-8) never
 *       occurs in reference-packed data (packers clamp to +-7); it is decoded
 *       as -8 here, the two's-complement reading (parity-unpinned for -8).
 *   - linear: y = x . W (+ bias), as linear_forward
 *       crates/burn_boogu/src/model/linear.rs:14-37 and qwen_linear_forward
 *       crates/burn_qwen3_vl/src/linear.rs:107-140, followed by the epilogues
 *       GELU-tanh (crates/burn_qwen3_vl/src/vision.rs:279,283-289) and
 *       silu(gate) * up (crates/burn_boogu/src/model/feed_forward.rs:32-36,
 *       crates/burn_qwen3_vl/src/text.rs:46-52).
 *   - QK-norm + RoPE on the q/k projections (the consumer of the qkv linear):
 *       crates/burn_boogu/src/model/attention.rs:114-133 (RMS-normalise q and
 *       k per head with norm_q / norm_k, then rotate), the StrictF32 policy
 *       crates/burn_boogu/src/model/norm.rs:86-96 (Burn nn::RmsNorm, burn-nn
 *       0.21.0: x / sqrt(mean(x^2) + eps) * gamma over the head dimension),
 *       apply_rope crates/burn_boogu/src/model/attention.rs:916-928
 *       (interleaved pairs: out[2p] = x[2p] cos - x[2p+1] sin,
 *       out[2p+1] = x[2p+1] cos + x[2p] sin), and the per-(token, dim) cos/sin
 *       tables of crates/burn_boogu/src/model/denoiser.rs:992-1032.
 *
 * Reference arithmetic lives in third-party crates that are not vendored:
 * cubek-matmul 0.2.0 / cubek-quant 0.2.0 (GPU) and burn-ndarray 0.21.0 /
 * burn-std 0.21.0 (CPU q_matmul and QuantizedBytes::into_vec_i8), pinned in
 * the reference's Cargo.lock.  The restatement follows their published
 * behaviour as used by the reference's own tests.
 *
 * Build: oracle/Makefile (gcc, -O2, -ffp-contract=off so float expressions
 * round exactly as written; OpenMP for the timed baseline).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_OK 0
#define ORC_ENONFINITE 1
#define ORC_ESHAPE 2
#define ORC_EBLOCK 3

#define ORC_LAYOUT_COL 0 /* PackedU32(0): tensor [N,K], words [N][K/8], scales [N][K/b] */
#define ORC_LAYOUT_ROW 1 /* PackedU32(1): tensor [K,N], words [K/8][N], scales [K/b][N] */

#define ORC_ACT_NONE 0
#define ORC_ACT_GELU_TANH 1
#define ORC_ACT_SILU 2

/* f32::round: half away from zero == C roundf. */
static inline int8_t q4_round_clamp(float value, float inverse) {
    float q = roundf(value * inverse);
    if (q < -7.0f) q = -7.0f;
    if (q > 7.0f) q = 7.0f;
    return (int8_t)q;
}

/* alpha == 0 -> f32::MIN_POSITIVE, else alpha / 7 (artifacts.rs:1339-1344). */
static inline float q4_scale_from_alpha(float alpha) {
    return alpha == 0.0f ? 1.17549435e-38f : alpha / 7.0f;
}

/*
 * Column layout packer: restates crates/burn_qwen3_vl/src/artifacts.rs:1301-1366.
 * `values` is row-major [rows][inner]; every contiguous 128-block of the inner
 * axis gets one scale; 8 quantized values per word, lane i at bits 4i.
 * words: rows*inner/8, scales: rows*inner/128.
 */
int orc_quantize_col_block128(const float* values, int64_t rows, int64_t inner,
                              uint32_t* words, float* scales) {
    const int64_t B = 128;
    if (rows <= 0 || inner <= 0 || inner % B != 0) return ORC_ESHAPE;
    const int64_t total = rows * inner;
    for (int64_t i = 0; i < total; ++i)
        if (!isfinite(values[i])) return ORC_ENONFINITE;
    for (int64_t blk = 0; blk < total / B; ++blk) {
        const float* v = values + blk * B;
        float alpha = 0.0f;
        for (int64_t i = 0; i < B; ++i) alpha = fmaxf(alpha, fabsf(v[i]));
        const float scale = q4_scale_from_alpha(alpha);
        scales[blk] = scale;
        const float inverse = 1.0f / scale; /* f32::recip */
        for (int64_t w = 0; w < B / 8; ++w) {
            uint32_t word = 0;
            for (int lane = 0; lane < 8; ++lane) {
                int8_t q = q4_round_clamp(v[w * 8 + lane], inverse);
                word |= ((uint32_t)((uint8_t)q & 0x0f)) << (lane * 4);
            }
            words[blk * (B / 8) + w] = word;
        }
    }
    return ORC_OK;
}

/* Block policy: largest of {128,64,32,16,8} dividing `input`
 * (crates/burn_boogu/src/artifacts.rs:7318-7326, :513-525). */
int orc_row_block_for(int64_t input) {
    static const int groups[5] = {128, 64, 32, 16, 8};
    for (int i = 0; i < 5; ++i)
        if (input > 0 && input % groups[i] == 0) return groups[i];
    return 0;
}

/*
 * Row layout packer: restates crates/burn_boogu/src/artifacts.rs:7296-7385.
 * `values` is row-major [input][output] (Burn linear layout, K x N).
 * Scale per (K-block, output column) over the column; word (kw, n) packs
 * K = 8kw..8kw+7 of column n, giving words [input/8][output] and scales
 * [input/block][output].
 */
int orc_quantize_row_up_to128(const float* values, int64_t input, int64_t output,
                              uint32_t* words, float* scales, int32_t* block_out) {
    if (input <= 0 || output <= 0 || output % 8 != 0) return ORC_ESHAPE;
    const int block = orc_row_block_for(input);
    if (block == 0) return ORC_EBLOCK;
    for (int64_t i = 0; i < input * output; ++i)
        if (!isfinite(values[i])) return ORC_ENONFINITE;
    int8_t* q = (int8_t*)malloc((size_t)(input * output));
    if (!q) return ORC_ESHAPE;
    for (int64_t kb = 0; kb < input / block; ++kb) {
        const int64_t k0 = kb * block;
        for (int64_t n = 0; n < output; ++n) {
            float alpha = 0.0f;
            for (int64_t k = k0; k < k0 + block; ++k)
                alpha = fmaxf(alpha, fabsf(values[k * output + n]));
            const float scale = q4_scale_from_alpha(alpha);
            scales[kb * output + n] = scale;
            const float inverse = 1.0f / scale;
            for (int64_t k = k0; k < k0 + block; ++k)
                q[k * output + n] = q4_round_clamp(values[k * output + n], inverse);
        }
    }
    for (int64_t kw = 0; kw < input / 8; ++kw) {
        for (int64_t n = 0; n < output; ++n) {
            uint32_t word = 0;
            for (int lane = 0; lane < 8; ++lane)
                word |= ((uint32_t)((uint8_t)q[(kw * 8 + lane) * output + n] & 0x0f)) << (lane * 4);
            words[kw * output + n] = word;
        }
    }
    free(q);
    *block_out = block;
    return ORC_OK;
}

/* Sign-extend the 4-bit two's-complement nibble `lane` of `word`. */
static inline int32_t q4_nibble(uint32_t word, int lane) {
    int32_t v = (int32_t)((word >> (4 * lane)) & 0xF);
    return v >= 8 ? v - 16 : v;
}

static int check_geometry(int64_t K, int64_t N, int32_t block, int32_t layout) {
    if (!(block == 8 || block == 16 || block == 32 || block == 64 || block == 128)) return ORC_EBLOCK;
    if (K <= 0 || N <= 0 || K % 8 != 0 || K % block != 0) return ORC_ESHAPE;
    if (layout != ORC_LAYOUT_COL && layout != ORC_LAYOUT_ROW) return ORC_ESHAPE;
    return ORC_OK;
}

/*
 * Unpack to the logical weight W [K][N] (y = x . W): w = q * scale in f32.
 * Column layout (tensor [N,K], PackedU32(0)): word (n, kw), scale (n, k/b).
 * Row layout (tensor [K,N], PackedU32(1)): word (kw, n), scale (k/b, n).
 */
int orc_unpack(const uint32_t* words, const float* scales, int64_t K, int64_t N,
               int32_t block, int32_t layout, float* w_kn) {
    int rc = check_geometry(K, N, block, layout);
    if (rc) return rc;
    const int64_t KW = K / 8, KB = K / block;
    for (int64_t k = 0; k < K; ++k) {
        const int64_t kw = k / 8, lane = k % 8, kb = k / block;
        for (int64_t n = 0; n < N; ++n) {
            uint32_t word;
            float scale;
            if (layout == ORC_LAYOUT_COL) {
                word = words[n * KW + kw];
                scale = scales[n * KB + kb];
            } else {
                word = words[kw * N + n];
                scale = scales[kb * N + n];
            }
            w_kn[k * N + n] = (float)q4_nibble(word, (int)lane) * scale;
        }
    }
    return ORC_OK;
}

/* Row selection of a packed Q4S matrix [rows][cols], PackedU32(0) with
 * blocks along the row: words [rows][cols/8], scales [rows][cols/block].
 * Restates the reference's q_select kernel
 * (patches/burn-cubecl-0.21.0/src/kernel/index/select.rs:83-108: output word
 * and scale (r, c) are the source's (indices[r], c)).  out_f32 (optional)
 * receives the selected rows dequantized as in orc_unpack.  An index outside
 * [0, rows) yields a zero row and ORC_ESHAPE (the reference reads out of
 * bounds). */
int orc_select_rows(const uint32_t* words, const float* scales, int64_t rows, int64_t cols, int32_t block,
                    const int64_t* ids, int64_t n, uint32_t* out_words, float* out_scales, float* out_f32) {
    if (!(block == 8 || block == 16 || block == 32 || block == 64 || block == 128)) return ORC_EBLOCK;
    if (rows <= 0 || cols <= 0 || n < 0 || cols % block != 0) return ORC_ESHAPE;
    const int64_t wpr = cols / 8, spr = cols / block;
    int rc = ORC_OK;
    for (int64_t r = 0; r < n; ++r) {
        const int64_t id = ids[r];
        const int ok = id >= 0 && id < rows;
        if (!ok) rc = ORC_ESHAPE;
        for (int64_t w = 0; w < wpr; ++w) {
            const uint32_t word = ok ? words[id * wpr + w] : 0u;
            if (out_words) out_words[r * wpr + w] = word;
            if (out_f32) {
                const float sc = ok ? scales[id * spr + (w * 8) / block] : 0.0f;
                for (int lane = 0; lane < 8; ++lane)
                    out_f32[r * cols + w * 8 + lane] = (float)q4_nibble(word, lane) * sc;
            }
        }
        if (out_scales)
            for (int64_t c = 0; c < spr; ++c) out_scales[r * spr + c] = ok ? scales[id * spr + c] : 0.0f;
    }
    return rc;
}

static inline double act_f64(double v, int32_t act) {
    if (act == ORC_ACT_GELU_TANH) {
        /* Burn Gelu::new_approximate: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))) */
        const double c = sqrt(2.0 / 3.14159265358979323846);
        return 0.5 * v * (1.0 + tanh(c * (v + 0.044715 * v * v * v)));
    }
    if (act == ORC_ACT_SILU) return v / (1.0 + exp(-v));
    return v;
}

/*
 * The checker: f64-accumulated y[m][n] = act(sum_k x[m][k] W[k][n] + bias[n])
 * (times aux[m][n] when aux is given), W the unpacked logical weight.
 */
void orc_linear_f64(const float* x, int64_t M, int64_t K, int64_t ldx, const float* w_kn,
                    int64_t N, const float* bias, int32_t act, const float* aux, float* y) {
    double* acc = (double*)malloc(sizeof(double) * (size_t)N);
    for (int64_t m = 0; m < M; ++m) {
        for (int64_t n = 0; n < N; ++n) acc[n] = 0.0;
        for (int64_t k = 0; k < K; ++k) {
            const double xv = (double)x[m * ldx + k];
            const float* wr = w_kn + k * N;
            for (int64_t n = 0; n < N; ++n) acc[n] += xv * (double)wr[n];
        }
        for (int64_t n = 0; n < N; ++n) {
            double v = acc[n] + (bias ? (double)bias[n] : 0.0);
            v = act_f64(v, act);
            if (aux) v *= (double)aux[m * N + n];
            y[m * N + n] = (float)v;
        }
    }
    free(acc);
}

/* y = silu(x Wg + bg) * (x Wu + bu), f64 accumulate. */
void orc_linear_gated_f64(const float* x, int64_t M, int64_t K, int64_t ldx, const float* wg_kn,
                          const float* wu_kn, int64_t N, const float* bg, const float* bu,
                          float* y) {
    double* g = (double*)malloc(sizeof(double) * (size_t)N);
    double* u = (double*)malloc(sizeof(double) * (size_t)N);
    for (int64_t m = 0; m < M; ++m) {
        for (int64_t n = 0; n < N; ++n) g[n] = u[n] = 0.0;
        for (int64_t k = 0; k < K; ++k) {
            const double xv = (double)x[m * ldx + k];
            for (int64_t n = 0; n < N; ++n) {
                g[n] += xv * (double)wg_kn[k * N + n];
                u[n] += xv * (double)wu_kn[k * N + n];
            }
        }
        for (int64_t n = 0; n < N; ++n) {
            double gv = g[n] + (bg ? (double)bg[n] : 0.0);
            double uv = u[n] + (bu ? (double)bu[n] : 0.0);
            y[m * N + n] = (float)(act_f64(gv, ORC_ACT_SILU) * uv);
        }
    }
    free(g);
    free(u);
}

/*
 * QK-norm + RoPE checker, f64: for every token m and head h of
 * x[m][h*hd + d] (row pitch ldx), v = x / sqrt(mean_d(x^2) + eps) * gamma[d]
 * (gamma NULL: 1), then, when cos_t/sin_t are given ([m][d], row pitch ldr),
 * the interleaved-pair rotation.  y has row pitch ldy.  hd must be even.
 */
void orc_qk_norm_rope_f64(const float* x, int64_t M, int64_t heads, int64_t hd, int64_t ldx,
                          const float* gamma, double eps, const float* cos_t, const float* sin_t,
                          int64_t ldr, float* y, int64_t ldy) {
    double* v = (double*)malloc(sizeof(double) * (size_t)hd);
    for (int64_t m = 0; m < M; ++m) {
        for (int64_t h = 0; h < heads; ++h) {
            const float* xr = x + m * ldx + h * hd;
            double ss = 0.0;
            for (int64_t d = 0; d < hd; ++d) ss += (double)xr[d] * (double)xr[d];
            const double rms = sqrt(ss / (double)hd + eps);
            for (int64_t d = 0; d < hd; ++d) v[d] = (double)xr[d] / rms * (gamma ? (double)gamma[d] : 1.0);
            float* yr = y + m * ldy + h * hd;
            for (int64_t d = 0; d < hd; d += 2) {
                if (cos_t && sin_t) {
                    const double c0 = cos_t[m * ldr + d], s0 = sin_t[m * ldr + d];
                    const double c1 = cos_t[m * ldr + d + 1], s1 = sin_t[m * ldr + d + 1];
                    yr[d] = (float)(v[d] * c0 - v[d + 1] * s0);
                    yr[d + 1] = (float)(v[d + 1] * c1 + v[d] * s1);
                } else {
                    yr[d] = (float)v[d];
                    yr[d + 1] = (float)v[d + 1];
                }
            }
        }
    }
    free(v);
}

/* ------------------------------------------------------------------------
 * Timed CPU baseline: dequantize once to f32, then a blocked SGEMM with the
 * epilogue fused, OpenMP over all requested threads.  This is the shape of
 * Burn NdArray's q_matmul (dequantize, then the matrixmultiply sgemm); it is
 * a restatement, not the reference binary.
 * ---------------------------------------------------------------------- */

#define NR 16  /* columns per packed panel */
#define MR 6   /* rows per micro-tile */
#define KC 256 /* k-blocking */

static inline float act_f32(float v, int32_t act) {
    if (act == ORC_ACT_GELU_TANH) {
        const float c = 0.7978845608028654f;
        return 0.5f * v * (1.0f + tanhf(c * (v + 0.044715f * v * v * v)));
    }
    if (act == ORC_ACT_SILU) return v / (1.0f + expf(-v));
    return v;
}

/* Dequantize into column panels: panel p holds columns [16p,16p+16) as
 * [K][16] (zero-padded past N). */
static void dequant_panels(const uint32_t* words, const float* scales, int64_t K, int64_t N,
                           int32_t block, int32_t layout, float* panels) {
    const int64_t P = (N + NR - 1) / NR, KW = K / 8, KB = K / block;
#pragma omp parallel for schedule(static)
    for (int64_t p = 0; p < P; ++p) {
        float* dst = panels + p * K * NR;
        for (int64_t k = 0; k < K; ++k) {
            for (int j = 0; j < NR; ++j) {
                const int64_t n = p * NR + j;
                float v = 0.0f;
                if (n < N) {
                    uint32_t word;
                    float s;
                    if (layout == ORC_LAYOUT_COL) {
                        word = words[n * KW + k / 8];
                        s = scales[n * KB + k / block];
                    } else {
                        word = words[(k / 8) * N + n];
                        s = scales[(k / block) * N + n];
                    }
                    v = (float)q4_nibble(word, (int)(k % 8)) * s;
                }
                dst[k * NR + j] = v;
            }
        }
    }
}

#if defined(__x86_64__)
#include <immintrin.h>
__attribute__((target("avx2,fma"))) static void micro_avx2(const float* x, int64_t ldx,
                                                           const float* panel, int64_t k0,
                                                           int64_t kc, int rows, float acc[MR][NR]) {
    __m256 c[MR][2];
    for (int r = 0; r < MR; ++r) {
        c[r][0] = _mm256_loadu_ps(acc[r]);
        c[r][1] = _mm256_loadu_ps(acc[r] + 8);
    }
    for (int64_t k = k0; k < k0 + kc; ++k) {
        const __m256 b0 = _mm256_loadu_ps(panel + k * NR);
        const __m256 b1 = _mm256_loadu_ps(panel + k * NR + 8);
        for (int r = 0; r < MR; ++r) {
            if (r >= rows) break;
            const __m256 a = _mm256_broadcast_ss(x + r * ldx + k);
            c[r][0] = _mm256_fmadd_ps(a, b0, c[r][0]);
            c[r][1] = _mm256_fmadd_ps(a, b1, c[r][1]);
        }
    }
    for (int r = 0; r < MR; ++r) {
        _mm256_storeu_ps(acc[r], c[r][0]);
        _mm256_storeu_ps(acc[r] + 8, c[r][1]);
    }
}
#endif

static void micro_scalar(const float* x, int64_t ldx, const float* panel, int64_t k0, int64_t kc,
                         int rows, float acc[MR][NR]) {
    for (int64_t k = k0; k < k0 + kc; ++k)
        for (int r = 0; r < rows; ++r) {
            const float a = x[r * ldx + k];
            for (int j = 0; j < NR; ++j) acc[r][j] += a * panel[k * NR + j];
        }
}

static int g_have_avx2 = -1;

int orc_cpu_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/*
 * Timed baseline entry: y = act(x . deq(W) + bias) (* aux), f32 throughout.
 * `threads` <= 0 uses every available thread.  Returns ORC_OK or an error.
 */
int orc_cpu_linear(const uint32_t* words, const float* scales, int64_t K, int64_t N,
                   int32_t block, int32_t layout, const float* x, int64_t M, int64_t ldx,
                   const float* bias, int32_t act, const float* aux, float* y, int32_t threads) {
    int rc = check_geometry(K, N, block, layout);
    if (rc) return rc;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
#if defined(__x86_64__)
    if (g_have_avx2 < 0) {
        __builtin_cpu_init();
        g_have_avx2 = __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
    }
#else
    g_have_avx2 = 0;
#endif
    const int64_t P = (N + NR - 1) / NR;
    float* panels = (float*)aligned_alloc(64, sizeof(float) * (size_t)(P * K * NR) + 64);
    if (!panels) return ORC_ESHAPE;
    dequant_panels(words, scales, K, N, block, layout, panels);
    const int64_t MB = (M + MR - 1) / MR;
#pragma omp parallel for collapse(2) schedule(dynamic, 4)
    for (int64_t p = 0; p < P; ++p) {
        for (int64_t mb = 0; mb < MB; ++mb) {
            const int64_t m0 = mb * MR;
            const int rows = (int)((M - m0) < MR ? (M - m0) : MR);
            float acc[MR][NR];
            memset(acc, 0, sizeof(acc));
            const float* panel = panels + p * K * NR;
            for (int64_t k0 = 0; k0 < K; k0 += KC) {
                const int64_t kc = (K - k0) < KC ? (K - k0) : KC;
#if defined(__x86_64__)
                if (g_have_avx2)
                    micro_avx2(x + m0 * ldx, ldx, panel, k0, kc, rows, acc);
                else
#endif
                    micro_scalar(x + m0 * ldx, ldx, panel, k0, kc, rows, acc);
            }
            for (int r = 0; r < rows; ++r) {
                for (int j = 0; j < NR; ++j) {
                    const int64_t n = p * NR + j;
                    if (n >= N) break;
                    float v = acc[r][j] + (bias ? bias[n] : 0.0f);
                    v = act_f32(v, act);
                    if (aux) v *= aux[(m0 + r) * N + n];
                    y[(m0 + r) * N + n] = v;
                }
            }
        }
    }
    free(panels);
    return ORC_OK;
}

/* ========================================================================
 * Packed-F16 storage (the VAE's weights; next to the Q4 path in the same
 * patched backend): patches/burn-cubecl-0.21.0/src/kernel/packed_f16.rs.
 * IEEE binary16 bits, two per u32 word, the even-index value in the low half
 * (load_packed_f16, :77-86).
 * ====================================================================== */

/*
 * Widening, restated from widen_f16_bits_to_f32 (packed_f16.rs:48-74) and its
 * test twin reference_f16_bits_to_f32_bits (crates/burn_boogu/src/model/
 * packed_f16.rs:554-568): sign moved to bit 31; zero exponent with zero
 * mantissa -> signed zero; subnormal m -> normalised (exponent 113 - shift,
 * shift = leading zeros of m within its 10 bits + 1); exponent 31 -> infinity,
 * or NaN with the quiet bit set and the payload shifted up; otherwise the
 * exponent rebiased by 112 and the mantissa shifted up 13 bits.
 */
static uint32_t f16_bits_to_f32_bits(uint32_t bits) {
    const uint32_t sign = (bits & 0x8000u) << 16;
    const uint32_t exponent = (bits >> 10) & 0x1fu;
    const uint32_t mantissa = bits & 0x03ffu;
    if (exponent == 0) {
        if (mantissa == 0) return sign;
        uint32_t shift = 1; /* leading zeros of the 10-bit field, plus one */
        while (!((mantissa << shift) & 0x400u)) ++shift;
        return sign | ((113u - shift) << 23) | (((mantissa << shift) & 0x03ffu) << 13);
    }
    if (exponent == 0x1fu) {
        if (mantissa == 0) return sign | 0x7f800000u;
        return sign | 0x7fc00000u | (mantissa << 13);
    }
    return sign | ((exponent + 112u) << 23) | (mantissa << 13);
}

static inline float f16_value(uint16_t bits) {
    const uint32_t b = f16_bits_to_f32_bits(bits);
    float f;
    memcpy(&f, &b, sizeof(f));
    return f;
}

void orc_f16_widen_bits(const uint16_t* h, int64_t n, uint32_t* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = f16_bits_to_f32_bits(h[i]);
}

/*
 * packed_f16_rhs_matmul (packed_f16.rs:133-292), checker in f64:
 * out[m][n] = sum_k lhs[m][k] * widen(rhs[k * inner + n * col]).
 */
void orc_f16_matmul_f64(const float* lhs, int64_t M, int64_t K, const uint16_t* rhs, int64_t inner, int64_t col,
                        int64_t N, const float* bias, double* out) {
    double* w = (double*)malloc(sizeof(double) * (size_t)(K * N));
    for (int64_t k = 0; k < K; ++k)
        for (int64_t n = 0; n < N; ++n) w[k * N + n] = (double)f16_value(rhs[k * inner + n * col]);
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; ++m) {
        double* o = out + m * N;
        for (int64_t n = 0; n < N; ++n) o[n] = bias ? (double)bias[n] : 0.0;
        for (int64_t k = 0; k < K; ++k) {
            const double a = (double)lhs[m * K + k];
            const double* wr = w + k * N;
            for (int64_t n = 0; n < N; ++n) o[n] += a * wr[n];
        }
    }
    free(w);
}

/*
 * packed_f16_conv2d (packed_f16.rs:375-602), checker in f64: NCHW input
 * [B][C][H][W], OIHW weight [O][C][kh][kw], groups 1,
 * out[b][o][oy][ox] = bias[o] + sum_{c,ky,kx} in[b][c][iy][ix] * widen(w[o][c][ky][kx]),
 * iy = oy*sh + ky*dh - ph, ix = ox*sw + kx*dw - pw, zero outside the input
 * (packed_conv2d_input_value, :375-419); OH = (H + 2ph - dh(kh-1) - 1)/sh + 1.
 */
void orc_f16_conv2d_f64(const float* in, int64_t B, int64_t C, int64_t H, int64_t W, const uint16_t* wt, int64_t O,
                        int64_t kh, int64_t kw, const float* bias, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                        int64_t dh, int64_t dw, double* out) {
    const int64_t OH = (H + 2 * ph - dh * (kh - 1) - 1) / sh + 1;
    const int64_t OW = (W + 2 * pw - dw * (kw - 1) - 1) / sw + 1;
    const int64_t inner = C * kh * kw;
    double* w = (double*)malloc(sizeof(double) * (size_t)(O * inner));
    for (int64_t i = 0; i < O * inner; ++i) w[i] = (double)f16_value(wt[i]);
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t b = 0; b < B; ++b)
        for (int64_t o = 0; o < O; ++o) {
            for (int64_t oy = 0; oy < OH; ++oy)
                for (int64_t ox = 0; ox < OW; ++ox) {
                    double acc = bias ? (double)bias[o] : 0.0;
                    for (int64_t c = 0; c < C; ++c)
                        for (int64_t ky = 0; ky < kh; ++ky) {
                            const int64_t iy = oy * sh + ky * dh - ph;
                            if (iy < 0 || iy >= H) continue;
                            for (int64_t kx = 0; kx < kw; ++kx) {
                                const int64_t ix = ox * sw + kx * dw - pw;
                                if (ix < 0 || ix >= W) continue;
                                acc += (double)in[((b * C + c) * H + iy) * W + ix] *
                                       w[((o * C + c) * kh + ky) * kw + kx];
                            }
                        }
                    out[((b * O + o) * OH + oy) * OW + ox] = acc;
                }
        }
    free(w);
}

/*
 * Timed CPU arms for the packed-F16 rows (f32 throughout, OpenMP): the rhs
 * widened once into column panels, then the blocked SGEMM above; the
 * convolution as im2col rows per output row block, then the same SGEMM.
 */
static void f16_panels(const uint16_t* rhs, int64_t K, int64_t N, int64_t inner, int64_t col, float* panels) {
    const int64_t P = (N + NR - 1) / NR;
#pragma omp parallel for schedule(static)
    for (int64_t p = 0; p < P; ++p) {
        float* dst = panels + p * K * NR;
        for (int64_t k = 0; k < K; ++k)
            for (int j = 0; j < NR; ++j) {
                const int64_t n = p * NR + j;
                dst[k * NR + j] = n < N ? f16_value(rhs[k * inner + n * col]) : 0.0f;
            }
    }
}

static void sgemm_panels(const float* x, int64_t M, int64_t K, int64_t ldx, const float* panels, int64_t N,
                         float* y, int64_t ldy_n, int64_t ldy_m) {
    const int64_t P = (N + NR - 1) / NR, MB = (M + MR - 1) / MR;
#pragma omp parallel for collapse(2) schedule(dynamic, 4)
    for (int64_t p = 0; p < P; ++p)
        for (int64_t mb = 0; mb < MB; ++mb) {
            const int64_t m0 = mb * MR;
            const int rows = (int)((M - m0) < MR ? (M - m0) : MR);
            float acc[MR][NR];
            memset(acc, 0, sizeof(acc));
            const float* panel = panels + p * K * NR;
            for (int64_t k0 = 0; k0 < K; k0 += KC) {
                const int64_t kc = (K - k0) < KC ? (K - k0) : KC;
#if defined(__x86_64__)
                if (g_have_avx2)
                    micro_avx2(x + m0 * ldx, ldx, panel, k0, kc, rows, acc);
                else
#endif
                    micro_scalar(x + m0 * ldx, ldx, panel, k0, kc, rows, acc);
            }
            for (int r = 0; r < rows; ++r)
                for (int j = 0; j < NR; ++j) {
                    const int64_t n = p * NR + j;
                    if (n < N) y[(m0 + r) * ldy_m + n * ldy_n] = acc[r][j];
                }
        }
}

static void detect_avx2(void) {
#if defined(__x86_64__)
    if (g_have_avx2 < 0) {
        __builtin_cpu_init();
        g_have_avx2 = __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
    }
#else
    g_have_avx2 = 0;
#endif
}

int orc_cpu_f16_matmul(const float* lhs, int64_t M, int64_t K, const uint16_t* rhs, int64_t inner, int64_t col,
                       int64_t N, float* out, int32_t threads) {
    if (M <= 0 || K <= 0 || N <= 0) return ORC_ESHAPE;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
    detect_avx2();
    const int64_t P = (N + NR - 1) / NR;
    float* panels = (float*)aligned_alloc(64, sizeof(float) * (size_t)(P * K * NR) + 64);
    if (!panels) return ORC_ESHAPE;
    f16_panels(rhs, K, N, inner, col, panels);
    sgemm_panels(lhs, M, K, K, panels, N, out, 1, N);
    free(panels);
    return ORC_OK;
}

/* out NCHW f32; the rows of one image's output plane block are gathered
 * (im2col, [rows][C*kh*kw]) and multiplied by the OIHW weight panels. */
int orc_cpu_f16_conv2d(const float* in, int64_t B, int64_t C, int64_t H, int64_t W, const uint16_t* wt, int64_t O,
                       int64_t kh, int64_t kw, const float* bias, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                       int64_t dh, int64_t dw, float* out, int32_t threads) {
    const int64_t OH = (H + 2 * ph - dh * (kh - 1) - 1) / sh + 1;
    const int64_t OW = (W + 2 * pw - dw * (kw - 1) - 1) / sw + 1;
    if (B <= 0 || C <= 0 || O <= 0 || OH <= 0 || OW <= 0) return ORC_ESHAPE;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
    detect_avx2();
    const int64_t inner = C * kh * kw, P = (O + NR - 1) / NR;
    /* OIHW is [O][inner]: element (k, o) at o * inner + k */
    float* panels = (float*)aligned_alloc(64, sizeof(float) * (size_t)(P * inner * NR) + 64);
    const int64_t RB = 4096; /* output positions per im2col block */
    float* cols = (float*)aligned_alloc(64, sizeof(float) * (size_t)(RB * inner) + 64);
    if (!panels || !cols) {
        free(panels);
        free(cols);
        return ORC_ESHAPE;
    }
    f16_panels(wt, inner, O, 1, inner, panels);
    const int64_t plane = OH * OW;
    for (int64_t b = 0; b < B; ++b)
        for (int64_t r0 = 0; r0 < plane; r0 += RB) {
            const int64_t rows = plane - r0 < RB ? plane - r0 : RB;
#pragma omp parallel for schedule(static)
            for (int64_t r = 0; r < rows; ++r) {
                const int64_t oy = (r0 + r) / OW, ox = (r0 + r) % OW;
                float* dst = cols + r * inner;
                for (int64_t c = 0; c < C; ++c)
                    for (int64_t ky = 0; ky < kh; ++ky)
                        for (int64_t kx = 0; kx < kw; ++kx) {
                            const int64_t iy = oy * sh + ky * dh - ph, ix = ox * sw + kx * dw - pw;
                            *dst++ = (iy >= 0 && iy < H && ix >= 0 && ix < W) ? in[((b * C + c) * H + iy) * W + ix]
                                                                               : 0.0f;
                        }
            }
            /* y[(b, o, r0 + r)] : row r of this block, column o -> plane stride */
            sgemm_panels(cols, rows, inner, inner, panels, O, out + b * O * plane + r0, plane, 1);
        }
    if (bias)
        for (int64_t b = 0; b < B; ++b)
            for (int64_t o = 0; o < O; ++o)
                for (int64_t i = 0; i < plane; ++i) out[(b * O + o) * plane + i] += bias[o];
    free(panels);
    free(cols);
    return ORC_OK;
}

/*
 * Attention checker, f64: out[b][h][i] = sum_j p_j v[b][h/g][j],
 * p = softmax_j(scale * q[b][h][i] . k[b][h/g][j]) with g = Hq / Hkv (grouped
 * query heads share a kv head).  This is Burn's `attention` with default
 * options (no mask, scale 1/sqrt(D)), the composition the reference's
 * attention tests compare against (crates/burn_boogu/src/model/
 * native_flash.rs:2784-2843, with the kv heads repeated per group).
 * q [B][Hq][Sq][D], k and v [B][Hkv][Skv][D], out [B][Hq][Sq][D].
 */
void orc_attention_f64(const float* q, const float* k, const float* v, int64_t B, int64_t Hq, int64_t Hkv,
                       int64_t Sq, int64_t Skv, int64_t D, double scale, double* out) {
    const int64_t g = Hq / Hkv;
#pragma omp parallel
    {
        double* p = (double*)malloc(sizeof(double) * (size_t)Skv);
#pragma omp for collapse(3) schedule(static)
        for (int64_t b = 0; b < B; ++b)
            for (int64_t h = 0; h < Hq; ++h)
                for (int64_t i = 0; i < Sq; ++i) {
                    const float* qi = q + ((b * Hq + h) * Sq + i) * D;
                    const float* kb = k + (b * Hkv + h / g) * Skv * D;
                    const float* vb = v + (b * Hkv + h / g) * Skv * D;
                    double m = -INFINITY;
                    for (int64_t j = 0; j < Skv; ++j) {
                        double t = 0.0;
                        for (int64_t d = 0; d < D; ++d) t += (double)qi[d] * (double)kb[j * D + d];
                        p[j] = t * scale;
                        if (p[j] > m) m = p[j];
                    }
                    double sum = 0.0;
                    for (int64_t j = 0; j < Skv; ++j) {
                        p[j] = exp(p[j] - m);
                        sum += p[j];
                    }
                    double* o = out + ((b * Hq + h) * Sq + i) * D;
                    for (int64_t d = 0; d < D; ++d) o[d] = 0.0;
                    for (int64_t j = 0; j < Skv; ++j) {
                        const double w = p[j] / sum;
                        for (int64_t d = 0; d < D; ++d) o[d] += w * (double)vb[j * D + d];
                    }
                }
        free(p);
    }
}
