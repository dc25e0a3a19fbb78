/*
 * TEST INFRASTRUCTURE ONLY.  This CPU restatement of the reference's int8
 * quantized-linear path is the checker for the CUDA library in
 * kansaiml_b200/csrc.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / reference legs may load it; the product path never does.
 *
 * Parity is pinned: tests/test_oracle_golden.py checks every function here
 * against golden vectors produced by the reference's own Python
 * (python/kansai/quantize.py) running over the reference's own C++ core,
 * compiled from source (oracle/Makefile, target `ref`).
 *
 * Semantics restated (reference file:line in each comment):
 *   - absmax and scale: quantize.py:66-68.  Every fp32 element is widened to
 *     a double (Tensor.tolist), max|v| is taken in double, the scale is the
 *     double max_abs / 127.0, or 1.0 when max_abs == 0.
 *   - codes: quantize.py:69.  q = clamp(round(v / scale), -127, 127), where
 *     v / scale is the correctly rounded double quotient and round() is
 *     round-half-to-even (nearbyint under the default FE_TONEAREST mode).
 *     Python raises on NaN (ValueError) and Inf (OverflowError) inputs; here
 *     those return KZO_ERR_NONFINITE.
 *   - dequantize: quantize.py:76-77 then Tensor::from_flat (Tensor.cpp:94-100):
 *     the double product q * scale narrowed to fp32.
 *   - fp32 matmul: backend/cpu/src/Ops.cpp:328-337, the non-Accelerate i-k-j
 *     loop: out starts at +0.0f and accumulates av*bv in k order, each product
 *     and each sum rounded to fp32 separately (this file is compiled with
 *     -ffp-contract=off so no fused multiply-add can creep in).
 *   - bias add: Ops.cpp:34-38.  relu: Ops.cpp:197-199.  gelu: Ops.cpp:250-256.
 *
 * Extensions with no reference implementation (the W8A8 path), defined here
 * by applying the same rounding rules to each new granularity:
 *   - per-column weight scales (one per output feature = one per column of
 *     the reference's [in, out] weight, nn.py:74-81) with codes stored
 *     K-major [N, K];
 *   - per-row activation scales;
 *   - int8 x int8 -> int32 GEMM (exact integer arithmetic);
 *   - epilogue y = ((float)acc * row_scale) * col_scale (+ bias) (+ act), every
 *     step an fp32 operation rounded to nearest, scales narrowed from double
 *     to float once.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define KZO_OK 0
#define KZO_ERR_NONFINITE 2

static int is_finite_f(float v) { return isfinite(v); }

/* quantize.py:66-68 */
int kzo_absmax_f32(const float* x, int64_t n, double* out_absmax) {
    double m = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        if (!is_finite_f(x[i])) return KZO_ERR_NONFINITE;
        double a = fabs((double)x[i]);
        if (a > m) m = a;
    }
    *out_absmax = m;
    return KZO_OK;
}

double kzo_scale_from_absmax(double max_abs) { return max_abs > 0.0 ? max_abs / 127.0 : 1.0; }

/* quantize.py:69, one element */
static inline int8_t quant_one(float v, double scale) {
    double t = nearbyint((double)v / scale);
    if (t > 127.0) t = 127.0;
    if (t < -127.0) t = -127.0;
    return (int8_t)t;
}

int kzo_quantize_tensor_f32(const float* x, int64_t n, int8_t* q, double* out_scale) {
    double m;
    int st = kzo_absmax_f32(x, n, &m);
    if (st) return st;
    double s = kzo_scale_from_absmax(m);
    for (int64_t i = 0; i < n; ++i) q[i] = quant_one(x[i], s);
    *out_scale = s;
    return KZO_OK;
}

/* Per-tensor quantize with an externally supplied absmax (the multi-rank
 * case, where absmax is the max over every rank's shard). */
void kzo_quantize_with_absmax_f32(const float* x, int64_t n, double max_abs, int8_t* q, double* out_scale) {
    double s = kzo_scale_from_absmax(max_abs);
    for (int64_t i = 0; i < n; ++i) q[i] = quant_one(x[i], s);
    *out_scale = s;
}

/* Per-output-channel: w is the reference's row-major [K, N] weight; channel n
 * is column n.  Codes are written K-major: qT[n * K + k]. */
int kzo_quantize_cols_f32(const float* w, int64_t K, int64_t N, int8_t* qT, double* scales) {
    for (int64_t n = 0; n < N; ++n) {
        double m = 0.0;
        for (int64_t k = 0; k < K; ++k) {
            float v = w[k * N + n];
            if (!is_finite_f(v)) return KZO_ERR_NONFINITE;
            double a = fabs((double)v);
            if (a > m) m = a;
        }
        double s = kzo_scale_from_absmax(m);
        scales[n] = s;
        for (int64_t k = 0; k < K; ++k) qT[n * K + k] = quant_one(w[k * N + n], s);
    }
    return KZO_OK;
}

/* Per-row: x is row-major [M, K]; row m gets its own scale. */
int kzo_quantize_rows_f32(const float* x, int64_t M, int64_t K, int8_t* q, double* scales) {
    for (int64_t m = 0; m < M; ++m) {
        double s;
        int st = kzo_quantize_tensor_f32(x + m * K, K, q + m * K, &s);
        if (st) return st;
        scales[m] = s;
    }
    return KZO_OK;
}

/* quantize.py:76-77 + Tensor.cpp:94-100 */
void kzo_dequantize_i8(const int8_t* q, int64_t n, double scale, float* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = (float)((double)q[i] * scale);
}

/* ---------------------------------------------------------------- threads */

typedef void (*row_fn)(void* ctx, int64_t r0, int64_t r1);
struct row_job { row_fn fn; void* ctx; int64_t r0, r1; };

static void* row_trampoline(void* p) {
    struct row_job* j = (struct row_job*)p;
    j->fn(j->ctx, j->r0, j->r1);
    return NULL;
}

static void parallel_rows(row_fn fn, void* ctx, int64_t rows, int threads) {
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if (threads > rows) threads = (int)(rows > 0 ? rows : 1);
    if (threads == 1) { fn(ctx, 0, rows); return; }
    pthread_t tid[256];
    struct row_job jobs[256];
    int64_t per = (rows + threads - 1) / threads;
    int started = 0;
    for (int t = 0; t < threads; ++t) {
        int64_t r0 = (int64_t)t * per, r1 = r0 + per;
        if (r0 >= rows) break;
        if (r1 > rows) r1 = rows;
        jobs[t].fn = fn; jobs[t].ctx = ctx; jobs[t].r0 = r0; jobs[t].r1 = r1;
        if (pthread_create(&tid[t], NULL, row_trampoline, &jobs[t]) != 0) {
            fn(ctx, r0, r1);
            jobs[t].fn = NULL;
        }
        started = t + 1;
    }
    for (int t = 0; t < started; ++t)
        if (jobs[t].fn) pthread_join(tid[t], NULL);
}

/* ----------------------------------------------------- fp32 matmul (W8A32) */

struct mm_ctx { const float* a; const float* b; float* out; int64_t K, N; };

/* Ops.cpp:328-337: rows [r0, r1) of out = a @ b, i-k-j order. */
static void mm_rows(void* p, int64_t r0, int64_t r1) {
    struct mm_ctx* c = (struct mm_ctx*)p;
    for (int64_t i = r0; i < r1; ++i) {
        float* orow = c->out + i * c->N;
        for (int64_t j = 0; j < c->N; ++j) orow[j] = 0.0f;
        for (int64_t k = 0; k < c->K; ++k) {
            float av = c->a[i * c->K + k];
            const float* brow = c->b + k * c->N;
            for (int64_t j = 0; j < c->N; ++j) orow[j] += av * brow[j];
        }
    }
}

void kzo_matmul_f32(const float* a, const float* b, float* out, int64_t M, int64_t K, int64_t N, int threads) {
    struct mm_ctx c = {a, b, out, K, N};
    parallel_rows(mm_rows, &c, M, threads);
}

/* Ops.cpp:34-38 (in place) */
void kzo_add_bias_f32(float* x, const float* bias, int64_t M, int64_t N) {
    for (int64_t i = 0; i < M; ++i)
        for (int64_t j = 0; j < N; ++j) x[i * N + j] = x[i * N + j] + bias[j];
}

/* Ops.cpp:197-199 */
static inline float relu_f(float v) { return v > 0.0f ? v : 0.0f; }

/* Ops.cpp:246-256 */
static inline float gelu_f(float v) {
    const float inv_sqrt2 = 0.7071067811865476f;
    float cdf = 0.5f * (1.0f + erff(v * inv_sqrt2));
    return v * cdf;
}

void kzo_act_f32(float* x, int64_t n, int act) {
    if (act == 1) for (int64_t i = 0; i < n; ++i) x[i] = relu_f(x[i]);
    else if (act == 2) for (int64_t i = 0; i < n; ++i) x[i] = gelu_f(x[i]);
}

/* qlinear (quantize.py:115-122) with reference semantics, followed by an
 * optional activation (act: 0 none, 1 relu, 2 gelu):
 *   out = act(x @ dequantize(q, scale) + bias), q row-major [K, N]. */
void kzo_qlinear_w8a32(const float* x, int64_t M, int64_t K, const int8_t* q, double scale,
                       const float* bias, int64_t N, int act, float* out, int threads) {
    float* w = (float*)malloc((size_t)(K * N) * sizeof(float));
    kzo_dequantize_i8(q, K * N, scale, w);
    kzo_matmul_f32(x, w, out, M, K, N, threads);
    free(w);
    if (bias) kzo_add_bias_f32(out, bias, M, N);
    kzo_act_f32(out, M * N, act);
}

/* --------------------------------------------------- int8 GEMM (W8A8) */

struct gi_ctx { const int8_t* a; const int8_t* b; int32_t* out; int64_t N, K; };

static void gi_rows(void* p, int64_t r0, int64_t r1) {
    struct gi_ctx* c = (struct gi_ctx*)p;
    int64_t K = c->K;
    for (int64_t m = r0; m < r1; ++m) {
        const int8_t* ar = c->a + m * K;
        for (int64_t n = 0; n < c->N; ++n) {
            const int8_t* br = c->b + n * K;
            int32_t acc = 0;
            for (int64_t k = 0; k < K; ++k) acc += (int32_t)ar[k] * (int32_t)br[k];
            c->out[m * c->N + n] = acc;
        }
    }
}

/* acc[m, n] = sum_k a[m, k] * b[n, k]; a is [M, K], b is [N, K], both K-major. */
void kzo_gemm_i8_i32(const int8_t* a, const int8_t* b, int32_t* out, int64_t M, int64_t N, int64_t K, int threads) {
    struct gi_ctx c = {a, b, out, N, K};
    parallel_rows(gi_rows, &c, M, threads);
}

/* y = act(((float)acc * rs) * cs + bias); rs = row_scale[m * rs_stride],
 * cs = col_scale[n * cs_stride]; bias may be NULL. */
void kzo_epilogue_f32(const int32_t* acc, int64_t M, int64_t N, const float* row_scale, int64_t rs_stride,
                      const float* col_scale, int64_t cs_stride, const float* bias, int act, float* out) {
    for (int64_t m = 0; m < M; ++m) {
        float rs = row_scale[m * rs_stride];
        for (int64_t n = 0; n < N; ++n) {
            float y = (float)acc[m * N + n];
            y = y * rs;
            y = y * col_scale[n * cs_stride];
            if (bias) y = y + bias[n];
            if (act == 1) y = relu_f(y);
            else if (act == 2) y = gelu_f(y);
            out[m * N + n] = y;
        }
    }
}

/* ------------------------------------------------------------- LayerNorm */

/* LayerNorm over the last axis of x[M, D] (optionally of x + res, with the
 * sum written to sum_out), in the reference's operation order:
 *   nn.py:323-331        mean(dim), sub, mul, mean(dim), add(eps), sqrt, div,
 *                        mul(weight), add(bias), each a separate fp32 op;
 *   Tensor.cpp:864-880   mean(dim) = sum(dim, keepdim) * fl32(1.0f / D);
 *   Tensor.cpp:831-841 -> Ops.cpp:157-190  sum(dim): reduce_to_shape zeroes the
 *                        output and adds the row's elements in index order;
 *   Ops.cpp:205-207      sqrt per element (sqrtf);
 *   Tensor.cpp:677-679   div(other) = mul(other.reciprocal()), reciprocal
 *                        1.0f / v per element (Ops.cpp:213-215);
 *   eps is fl32(eps), as from_flat([eps], [1]) narrows it.
 * gamma / beta may be NULL (ones / zeros). */
void kzo_layernorm_f32(const float* x, const float* res, int64_t M, int64_t D, const float* gamma,
                       const float* beta, float eps, float* sum_out, float* y) {
    const float inv_d = 1.0f / (float)D;
    float* row = (float*)malloc((size_t)D * sizeof(float));
    float* cen = (float*)malloc((size_t)D * sizeof(float));
    for (int64_t m = 0; m < M; ++m) {
        const float* xr = x + m * D;
        for (int64_t j = 0; j < D; ++j) row[j] = res ? xr[j] + res[m * D + j] : xr[j];
        if (res && sum_out)
            for (int64_t j = 0; j < D; ++j) sum_out[m * D + j] = row[j];
        float s = 0.0f;
        for (int64_t j = 0; j < D; ++j) s += row[j];
        const float mean = s * inv_d;
        for (int64_t j = 0; j < D; ++j) cen[j] = row[j] - mean;
        float q = 0.0f;
        for (int64_t j = 0; j < D; ++j) {
            const float sq = cen[j] * cen[j];
            q += sq;
        }
        const float var = q * inv_d;
        const float den = sqrtf(var + eps);
        const float rden = 1.0f / den;
        for (int64_t j = 0; j < D; ++j) {
            float o = cen[j] * rden;
            o = o * (gamma ? gamma[j] : 1.0f);
            o = o + (beta ? beta[j] : 0.0f);
            y[m * D + j] = o;
        }
    }
    free(row);
    free(cen);
}

/* Scaled dot-product attention as the reference composes it in
 * MultiHeadAttention.forward (python/kansai/nn.py:410-427) from its Tensor
 * ops, one (batch, head) at a time:
 *   scores = q.matmul(k^T)      Ops.cpp:328-337: +0.0f, then += q*k, t ascending
 *   .mul(scale)                 fp32 multiply
 *   .add(mask)                  optional, broadcast by the strides
 *   .softmax(3)                 Tensor.cpp:906-913: max over the row (Ops.cpp:
 *                               275-292), sub, exp, sum (reduce_to_shape,
 *                               Ops.cpp:177-190: +0.0f, += e, j ascending),
 *                               div = mul by 1.0f/sum (Tensor.cpp:677-679)
 *   weights.matmul(v)           +0.0f, += w*v, j ascending
 * exp_mode 0: the correctly rounded fp32 exp (exp in double, narrowed), the
 * one the CUDA kernel computes; 1: the host libm's expf, the one the reference
 * calls (std::exp on a float).  causal: keys j > i masked, as causal_mask()'s
 * -1e9 entries do (given here as the flag; the reference adds the mask, and
 * every such key's exp is exactly 0).  Layouts as kz_attention_f32's. */
void kzo_attention_f32(const float* q, const float* k, const float* v, int64_t B, int64_t H, int64_t Sq,
                       int64_t Sk, int64_t dk, int64_t q_rs, int64_t k_rs, int64_t v_rs, const float* mask,
                       int64_t m_bs, int64_t m_hs, int64_t m_rs, int causal, float scale, float* out,
                       int64_t o_rs, int exp_mode) {
    float* s = (float*)malloc((size_t)(Sk > 0 ? Sk : 1) * sizeof(float));
    for (int64_t b = 0; b < B; ++b)
        for (int64_t h = 0; h < H; ++h)
            for (int64_t i = 0; i < Sq; ++i) {
                const float* qi = q + (b * Sq + i) * q_rs + h * dk;
                for (int64_t j = 0; j < Sk; ++j) {
                    const float* kj = k + (b * Sk + j) * k_rs + h * dk;
                    float acc = 0.0f;
                    for (int64_t t = 0; t < dk; ++t) {
                        const float p = qi[t] * kj[t];
                        acc = acc + p;
                    }
                    float sc = acc * scale;
                    if (causal)
                        sc = sc + (j > i ? -1e9f : 0.0f);
                    else if (mask)
                        sc = sc + mask[b * m_bs + h * m_hs + i * m_rs + j];
                    s[j] = sc;
                }
                float m = s[0];
                for (int64_t j = 1; j < Sk; ++j)
                    if (s[j] > m) m = s[j];
                float den = 0.0f;
                for (int64_t j = 0; j < Sk; ++j) {
                    const float x = s[j] - m;
                    s[j] = exp_mode ? expf(x) : (float)exp((double)x);
                    den = den + s[j];
                }
                const float r = 1.0f / den;
                for (int64_t j = 0; j < Sk; ++j) s[j] = s[j] * r;
                float* oi = out + (b * Sq + i) * o_rs + h * dk;
                for (int64_t t = 0; t < dk; ++t) {
                    float acc = 0.0f;
                    for (int64_t j = 0; j < Sk; ++j) {
                        const float p = s[j] * v[(b * Sk + j) * v_rs + h * dk + t];
                        acc = acc + p;
                    }
                    oi[t] = acc;
                }
            }
    free(s);
}

/* The host libm's expf, elementwise: what the reference's exp_fwd
 * (Ops.cpp:221-223, std::exp on a float) computes. */
void kzo_expf_f32(const float* x, int64_t n, float* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = expf(x[i]);
}
