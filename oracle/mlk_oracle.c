/*
 * CPU restatement (plain C, f64) of the reference's buffer executor for the
 * kernels on the B200 path: the parity oracle.
 *
 * TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline leg load this library, and only as the checker or
 * the timed CPU baseline; the shipped path (mlk2_b200/libmlkb200.so) never
 * links or calls it.
 *
 * Pinned: tests/test_oracle.py checks every function here against the
 * reference itself (oracle/_ref/libmlkref.so, built from the reference
 * sources by oracle/ref.mk) and against the committed golden vectors in
 * tests/golden/, which that compiled reference produced.
 *
 * Each function cites the reference code it restates (paths relative to the
 * reference repository).
 */
#include "mlk_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define MAX_TEMPS 64 /* kMaxTempSlots, runtime/src/execution/kernel_buffers.cpp:35 */

/* MathOp numbering, compiler/include/mlk/ir/math_op.h:18-36. */
enum {
    OP_ADD = 0, OP_SUB, OP_MUL, OP_DIV, OP_NEG, OP_POW, OP_EXP, OP_LOG,
    OP_SIN, OP_COS, OP_TAN, OP_TANH, OP_SQRT, OP_RSQRT, OP_ERF, OP_GELU
};
/* KernelOperand::Kind, compiler/include/mlk/support/kernel_ir.h:59-67. */
enum { K_CONST = 0, K_ELEM_A, K_ELEM_B, K_SCALAR, K_TEMP };

/* ExprEvaluator::apply, kernel_buffers.cpp:130-159; poly7 selects the
 * "poly7" Sin family (resolveFamily, :42-51: Sin only). */
static double poly7_sin(double x);
static double apply_op(int op, double a, double b, int poly7) {
    switch (op) {
        case OP_ADD: return a + b;
        case OP_SUB: return a - b;
        case OP_MUL: return a * b;
        case OP_DIV: return b != 0.0 ? a / b : 0.0;
        case OP_NEG: return -a;
        case OP_POW: return (a == 2.0 && b == 2.0) ? a * a : pow(a, b);
        case OP_EXP: return exp(a);
        case OP_LOG: return a > 0.0 ? log(a) : 0.0;
        case OP_SIN: return poly7 ? poly7_sin(a) : sin(a);
        case OP_COS: return cos(a);
        case OP_TAN: return tan(a);
        case OP_TANH: return tanh(a);
        case OP_SQRT: return a >= 0.0 ? sqrt(a) : 0.0;
        case OP_RSQRT: return a > 0.0 ? 1.0 / sqrt(a) : 0.0;
        case OP_ERF: return erf(a);
        case OP_GELU:
            return 0.5 * a *
                   (1.0 + tanh(0.7978845608028654 * (a + 0.044715 * a * a * a)));
        default: return 0.0;
    }
}

/* families::polySin, the "poly7" sine family
 * (compiler/include/mlk/support/math_families.h:22-90): Cody-Waite quadrant
 * reduction with pi/2 = hi + lo (:24-26, :69-76), then the degree-13 sine or
 * degree-12 cosine residual polynomial (:30-65) picked by the quadrant
 * (:81-90). Plain IEEE f64, no contraction (the oracle builds with
 * -ffp-contract=off), in the reference's evaluation order. */
static double poly7_sin_reduced(double x) {
    const double r2 = x * x;
    double p = 1.58962301576546568060e-10;
    p = p * r2 + -2.50507477628578072866e-8;
    p = p * r2 + 2.75573136213857245213e-6;
    p = p * r2 + -1.98412698295895385996e-4;
    p = p * r2 + 8.33333333332211858878e-3;
    p = p * r2 + -1.66666666666666307295e-1;
    return x + x * r2 * p;
}

static double poly7_cos_reduced(double x) {
    const double r2 = x * x;
    double p = -1.13585365213876817300e-11;
    p = p * r2 + 2.08757530072652689750e-9;
    p = p * r2 + -2.75573142103085808917e-7;
    p = p * r2 + 2.48015872890001867312e-5;
    p = p * r2 + -1.38888888888783992457e-3;
    p = p * r2 + 4.16666666666666435770e-2;
    return 1.0 - r2 * 0.5 + r2 * r2 * p;
}

static double poly7_sin(double x) {
    const double n = floor(x / 1.57079632679489661923 + 0.5);
    const double r = (x - n * 1.5707963267948965580e+00) - n * 6.1232339957367660359e-17;
    /* For x NaN or infinite, fmod(n, 4) is NaN: the reference converts it to
     * int, which x86-64 yields as INT_MIN, and its switch takes the default
     * branch (-cos of a NaN residual). Take that branch without the
     * undefined conversion, so even the NaN's sign matches. */
    const double f = fmod(n, 4.0);
    int q = isnan(f) ? 3 : (int)f;
    if (q < 0) q += 4;
    switch (q) {
        case 0: return poly7_sin_reduced(r);
        case 1: return poly7_cos_reduced(r);
        case 2: return -poly7_sin_reduced(r);
        default: return -poly7_cos_reduced(r);
    }
}

/* Unary classification, kernel_buffers.cpp:164-171. */
static int is_unary(int op) {
    return op == OP_NEG || op == OP_EXP || op == OP_LOG || op == OP_SIN ||
           op == OP_COS || op == OP_TAN || op == OP_TANH || op == OP_SQRT ||
           op == OP_RSQRT || op == OP_ERF || op == OP_GELU;
}

/* ExprEvaluator::evalOne, kernel_buffers.cpp:106-128 (1-D kinds only). */
static double eval_operand(int kind, int64_t index, double value,
                           const double* a, const double* b, int64_t i,
                           const double* scalars, int64_t n_scalars,
                           const double* temps) {
    switch (kind) {
        case K_CONST: return value;
        case K_ELEM_A: return a[i];
        case K_ELEM_B: return b != NULL ? b[i] : 0.0;
        case K_SCALAR:
            return (index >= 0 && index < n_scalars) ? scalars[index] : 0.0;
        case K_TEMP:
            return (index >= 0 && index < MAX_TEMPS) ? temps[index] : 0.0;
        default: return 0.0;
    }
}

/* ExprEvaluator::run, kernel_buffers.cpp:161-178, driven per element by
 * runElementwiseRange (:342-402) over each top-level Loop (:921-953). */
int mlko_chain(int32_t n_roots, const int32_t* root_len, const mlkb_expr* exprs,
               int32_t poly7, const double* a, const double* b, double* const* outs,
               int64_t n, const double* scalars, int64_t n_scalars) {
    int32_t off = 0;
    for (int32_t r = 0; r < n_roots; ++r) {
        const mlkb_expr* ex = exprs + off;
        const int32_t len = root_len[r];
        double* out = outs[r];
        double temps[MAX_TEMPS];
        if (len <= 0) return 8;
        for (int64_t i = 0; i < n; ++i) {
            int32_t k;
            memset(temps, 0, sizeof(temps));
            for (k = 0; k < len && k < MAX_TEMPS; ++k) {
                const double va = eval_operand(ex[k].a_kind, ex[k].a_index,
                                               ex[k].a_value, a, b, i, scalars,
                                               n_scalars, temps);
                const double vb =
                    is_unary(ex[k].op)
                        ? 0.0
                        : eval_operand(ex[k].b_kind, ex[k].b_index, ex[k].b_value,
                                       a, b, i, scalars, n_scalars, temps);
                temps[k] = apply_op(ex[k].op, va, vb, poly7);
            }
            out[i] = (len - 1 < MAX_TEMPS) ? temps[len - 1] : 0.0;
        }
        off += len;
    }
    return 0;
}

/* execSoftmaxCall, kernel_buffers.cpp:290-340: four ascending passes per
 * row (max select, exp into the output row, sum, guarded divide). */
int mlko_softmax(const double* a, double* y, int64_t rows, int64_t cols) {
    if (rows <= 0 || cols <= 0) return 8;
    for (int64_t i = 0; i < rows; ++i) {
        const double* row = a + i * cols;
        double* yrow = y + i * cols;
        double r = -INFINITY, s = 0.0;
        int64_t p;
        for (p = 0; p < cols; ++p) r = (row[p] > r) ? row[p] : r;
        for (p = 0; p < cols; ++p) yrow[p] = exp(row[p] - r);
        for (p = 0; p < cols; ++p) s += yrow[p];
        for (p = 0; p < cols; ++p) yrow[p] = s != 0.0 ? yrow[p] / s : 0.0;
    }
    return 0;
}

/* execReduceSumCall, kernel_buffers.cpp:237-277: ascending-k row sums. */
int mlko_reducesum(const double* a, double* y, int64_t rows, int64_t cols) {
    if (rows <= 0 || cols <= 0) return 8;
    for (int64_t i = 0; i < rows; ++i) {
        double acc = 0.0;
        for (int64_t p = 0; p < cols; ++p) acc += a[i * cols + p];
        y[i] = acc;
    }
    return 0;
}

/* gemmRowBlock, kernel_buffers.cpp:406-432, with the default tiles
 * 64/64/32 (compiler/include/mlk/core/constants.h:84-86): C += A*B,
 * i-p-j order inside (tileM, tileN, tileK) blocks, zero-a terms skipped.
 * rows [row_begin, row_end) only, so callers can sample row blocks. */
int mlko_matmul_rows(const double* a, const double* b, double* c, int64_t n,
                     int64_t k, int64_t row_begin, int64_t row_end) {
    const int64_t tm = 64, tn = 64, tk = 32;
    for (int64_t ii = row_begin; ii < row_end; ii += tm) {
        const int64_t ie = ii + tm < row_end ? ii + tm : row_end;
        for (int64_t jj = 0; jj < n; jj += tn) {
            const int64_t je = jj + tn < n ? jj + tn : n;
            for (int64_t kk = 0; kk < k; kk += tk) {
                const int64_t ke = kk + tk < k ? kk + tk : k;
                for (int64_t i = ii; i < ie; ++i) {
                    const double* arow = a + i * k;
                    double* crow = c + i * n;
                    for (int64_t p = kk; p < ke; ++p) {
                        const double aik = arow[p];
                        const double* brow;
                        if (aik == 0.0) continue;
                        brow = b + p * n;
                        for (int64_t j = jj; j < je; ++j) crow[j] += aik * brow[j];
                    }
                }
            }
        }
    }
    return 0;
}

int mlko_matmul(const double* a, const double* b, double* c, int64_t m,
                int64_t n, int64_t k) {
    if (m <= 0 || n <= 0 || k <= 0) return 8;
    return mlko_matmul_rows(a, b, c, n, k, 0, m);
}

/* ---- deterministic synthetic inputs (not reference code) ----------------
 * Counter-based SplitMix64: word(seed, stream, i) = mix(seed + stream*2^40 +
 * (i+1)*golden). The device generator (mlk2_b200/csrc/fill.cu) uses the
 * same word, so uniform streams agree bit for bit. */
static uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t mlko_word(uint64_t seed, uint32_t stream_id, uint64_t i) {
    return mix64(seed + ((uint64_t)stream_id << 40) + (i + 1) * 0x9E3779B97F4A7C15ull);
}

void mlko_fill_uniform_f32(float* out, int64_t n, uint64_t seed,
                           uint32_t stream_id, double lo, double hi,
                           int64_t first) {
    for (int64_t i = 0; i < n; ++i) {
        const uint64_t k = mlko_word(seed, stream_id, (uint64_t)(first + i)) >> 40;
        out[i] = (float)(lo + (hi - lo) * ((double)k * 0x1p-24));
    }
}
