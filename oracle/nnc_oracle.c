/*
 * nnc_oracle.c — CPU restatement of nnc-py's operator semantics.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker for the CUDA
 * operator library: only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg may load it. Nothing in the product path (libnnc_cuda.so,
 * the nnc_cuda package, generated model code) links or calls it.
 *
 * Each function restates the algorithm of the reference implementation
 * (nnc-py runtime/x86/ops.c, cited per function): same accumulation types,
 * same loop/summation order where it affects rounding, same broadcast and
 * window rules, same quirks. It exports the reference's symbol names so the
 * parity tests drive it exactly like the CUDA library. It is pinned against
 * the reference itself (oracle/_ref/libref_ops.so built from the reference
 * sources) and against golden vectors in tests/golden/.
 *
 * Build: make -C oracle   (gcc -O2 -ffp-contract=off, no FMA contraction).
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "nnc_ops.h"

static int64_t count_of(const Tensor* t) {
    int64_t n = 1;
    for (int d = 0; d < t->ndim; ++d) n *= t->shape[d];
    return n;
}

/* Splits t around `axis` (negative counts from the end) into
 * [outer, t->shape[axis], inner]. */
static int around_axis(const Tensor* t, int axis, int64_t* outer, int64_t* mid, int64_t* inner) {
    int a = axis < 0 ? axis + t->ndim : axis;
    *outer = 1;
    *inner = 1;
    for (int d = 0; d < a; ++d) *outer *= t->shape[d];
    for (int d = a + 1; d < t->ndim; ++d) *inner *= t->shape[d];
    *mid = t->shape[a];
    return a;
}

/* ---------------------------------------------------------------------------
 * Binary element-wise with the reference's modular suffix broadcast
 * (ops.c:82-224, :3233-3346). The first min(n, na, nb) outputs combine
 * a[i] and b[i]; when exactly one operand has n elements the rest of the
 * output indexes the other operand modulo its length.
 * ------------------------------------------------------------------------- */
typedef float (*binary_fn)(float, float);

static float f_add(float x, float y) { return x + y; }
static float f_sub(float x, float y) { return x - y; }
static float f_mul(float x, float y) { return x * y; }
static float f_div(float x, float y) { return x / y; }
static float f_add_relu(float x, float y) {
    float s = x + y;
    return s > 0.0f ? s : 0.0f;
}
static float f_add_sigmoid(float x, float y) {
    float s = x + y;
    return 1.0f / (1.0f + expf(-s));
}

static void broadcast_apply(Tensor* a, Tensor* b, Tensor* out, binary_fn f) {
    const int64_t n = count_of(out), na = count_of(a), nb = count_of(b);
    const float* x = (const float*)a->data;
    const float* y = (const float*)b->data;
    float* z = (float*)out->data;
    int64_t head = n;
    if (na < head) head = na;
    if (nb < head) head = nb;
    for (int64_t i = 0; i < head; ++i) z[i] = f(x[i], y[i]);
    if (nb == n && na < n) {
        for (int64_t i = head; i < n; ++i) z[i] = f(x[i % na], y[i]);
    } else if (na == n && nb < n) {
        for (int64_t i = head; i < n; ++i) z[i] = f(x[i], y[i % nb]);
    }
}

void nnc_add(Tensor* a, Tensor* b, Tensor* out) { broadcast_apply(a, b, out, f_add); }
void nnc_sub(Tensor* a, Tensor* b, Tensor* out) { broadcast_apply(a, b, out, f_sub); }
void nnc_mul(Tensor* a, Tensor* b, Tensor* out) { broadcast_apply(a, b, out, f_mul); }
void nnc_div(Tensor* a, Tensor* b, Tensor* out) { broadcast_apply(a, b, out, f_div); }
void nnc_add_relu(Tensor* a, Tensor* b, Tensor* out) { broadcast_apply(a, b, out, f_add_relu); }
void nnc_add_sigmoid(Tensor* a, Tensor* b, Tensor* out) { broadcast_apply(a, b, out, f_add_sigmoid); }

/* ---------------------------------------------------------------------------
 * Unary element-wise over numel(output) (ops.c:230-258, :2253-2262,
 * :2434-2515), with libm expf/tanhf/sqrtf/logf as in the reference.
 * fmaxf/fminf are spelled out because their signed-zero result depends on
 * argument order, which gcc may swap: the compiled reference returns the
 * non-NaN operand for a NaN and the SECOND argument for equal operands, with
 * relu's fmaxf(0.0f, x) emitted as a call on (x, 0) — so relu(-0) = +0.
 * ------------------------------------------------------------------------- */
static float max_second_on_tie(float x, float y) {
    if (isnan(x)) return y;
    if (isnan(y)) return x;
    return x > y ? x : y;
}
static float min_second_on_tie(float x, float y) {
    if (isnan(x)) return y;
    if (isnan(y)) return x;
    return x < y ? x : y;
}

typedef float (*unary_fn)(float, float, float);

static float u_relu(float v, float lo, float hi) { (void)lo; (void)hi; return v > 0.0f ? v : 0.0f; }
static float u_sigmoid(float v, float lo, float hi) { (void)lo; (void)hi; return 1.0f / (1.0f + expf(-v)); }
static float u_tanh(float v, float lo, float hi) { (void)lo; (void)hi; return tanhf(v); }
static float u_clip(float v, float lo, float hi) { return min_second_on_tie(max_second_on_tie(v, lo), hi); }
static float u_sqrt(float v, float lo, float hi) { (void)lo; (void)hi; return v >= 0.0f ? sqrtf(v) : NAN; }
static float u_pow2(float v, float lo, float hi) { (void)lo; (void)hi; return v * v; }
static float u_exp(float v, float lo, float hi) { (void)lo; (void)hi; return expf(v); }
static float u_log(float v, float lo, float hi) { (void)lo; (void)hi; return v > 0.0f ? logf(v) : NAN; }
static float u_abs(float v, float lo, float hi) { (void)lo; (void)hi; return fabsf(v); }
static float u_neg(float v, float lo, float hi) { (void)lo; (void)hi; return -v; }

static void map_unary(Tensor* in, Tensor* out, unary_fn f, float lo, float hi) {
    const int64_t n = count_of(out);
    const float* x = (const float*)in->data;
    float* z = (float*)out->data;
    for (int64_t i = 0; i < n; ++i) z[i] = f(x[i], lo, hi);
}

void nnc_relu(Tensor* in, Tensor* out) { map_unary(in, out, u_relu, 0, 0); }
void nnc_sigmoid(Tensor* in, Tensor* out) { map_unary(in, out, u_sigmoid, 0, 0); }
void nnc_tanh(Tensor* in, Tensor* out) { map_unary(in, out, u_tanh, 0, 0); }
void nnc_clip(Tensor* in, Tensor* out, float lo, float hi) { map_unary(in, out, u_clip, lo, hi); }
void nnc_sqrt(Tensor* in, Tensor* out) { map_unary(in, out, u_sqrt, 0, 0); }
void nnc_pow(Tensor* in, Tensor* out) { map_unary(in, out, u_pow2, 0, 0); }
void nnc_exp(Tensor* in, Tensor* out) { map_unary(in, out, u_exp, 0, 0); }
void nnc_log(Tensor* in, Tensor* out) { map_unary(in, out, u_log, 0, 0); }
void nnc_abs(Tensor* in, Tensor* out) { map_unary(in, out, u_abs, 0, 0); }
void nnc_neg(Tensor* in, Tensor* out) { map_unary(in, out, u_neg, 0, 0); }

/* ---------------------------------------------------------------------------
 * Softmax (ops.c:260-310): per [outer, :, inner] column — running max with
 * '>', sequential fp32 sum of expf(x - max), then expf(x - max) / sum.
 * ------------------------------------------------------------------------- */
void nnc_softmax(Tensor* in, Tensor* out, int axis) {
    int64_t outer, dim, inner;
    around_axis(in, axis, &outer, &dim, &inner);
    const float* x = (const float*)in->data;
    float* z = (float*)out->data;
    for (int64_t o = 0; o < outer; ++o) {
        for (int64_t j = 0; j < inner; ++j) {
            const int64_t base = o * dim * inner + j;
            float m = -INFINITY;
            for (int64_t s = 0; s < dim; ++s)
                if (x[base + s * inner] > m) m = x[base + s * inner];
            float total = 0.0f;
            for (int64_t s = 0; s < dim; ++s) total += expf(x[base + s * inner] - m);
            for (int64_t s = 0; s < dim; ++s) z[base + s * inner] = expf(x[base + s * inner] - m) / total;
        }
    }
}

/* ---------------------------------------------------------------------------
 * LayerNorm (ops.c:2095-2171): each [norm, inner] slab — sequential fp32
 * mean and variance, std = sqrtf(var + eps), y = g[i] * ((x - mean) / std)
 * + b[i] with g/b indexed by the axis coordinate (NULL: 1 / 0).
 * ------------------------------------------------------------------------- */
void nnc_layernorm(Tensor* in, Tensor* scale, Tensor* bias, Tensor* out, int axis, float eps) {
    int64_t outer, norm, inner;
    around_axis(in, axis, &outer, &norm, &inner);
    const float* x = (const float*)in->data;
    const float* g = scale ? (const float*)scale->data : NULL;
    const float* bb = bias ? (const float*)bias->data : NULL;
    float* z = (float*)out->data;
    const int64_t len = norm * inner;
    for (int64_t o = 0; o < outer; ++o) {
        const float* row = x + o * len;
        float* dst = z + o * len;
        float mean = 0.0f;
        for (int64_t i = 0; i < len; ++i) mean += row[i];
        mean /= (float)len;
        float var = 0.0f;
        for (int64_t i = 0; i < len; ++i) {
            float d = row[i] - mean;
            var += d * d;
        }
        var /= (float)len;
        const float sd = sqrtf(var + eps);
        for (int64_t i = 0; i < norm; ++i) {
            const float gi = g ? g[i] : 1.0f;
            const float bi = bb ? bb[i] : 0.0f;
            for (int64_t j = 0; j < inner; ++j) {
                float t = (row[i * inner + j] - mean) / sd;
                dst[i * inner + j] = gi * t + bi;
            }
        }
    }
}

/* ---------------------------------------------------------------------------
 * ReduceSum / ReduceMean over one axis (ops.c:1892-1989): Kahan-compensated
 * fp32 sum per output, mean = sum / (float)dim; keepdims does not change the
 * output's linear layout.
 * ------------------------------------------------------------------------- */
static void reduce_axis(Tensor* in, Tensor* out, int axis, int mean) {
    int64_t outer, dim, inner;
    around_axis(in, axis, &outer, &dim, &inner);
    const float* x = (const float*)in->data;
    float* z = (float*)out->data;
    for (int64_t o = 0; o < outer; ++o) {
        for (int64_t j = 0; j < inner; ++j) {
            float acc = 0.0f, lost = 0.0f;
            for (int64_t r = 0; r < dim; ++r) {
                float y = x[(o * dim + r) * inner + j] - lost;
                float t = acc + y;
                lost = (t - acc) - y;
                acc = t;
            }
            z[o * inner + j] = mean ? acc / (float)dim : acc;
        }
    }
}

void nnc_reducemean(Tensor* in, Tensor* out, int axis, int keepdims) { (void)keepdims; reduce_axis(in, out, axis, 1); }
void nnc_reducesum(Tensor* in, Tensor* out, int axis, int keepdims) { (void)keepdims; reduce_axis(in, out, axis, 0); }

/* ---------------------------------------------------------------------------
 * Pooling (ops.c:316-461): window start o*stride - pad, clamped to the input;
 * output extent from output->shape. Max: first value, then strictly greater;
 * empty window -3.402823e38f. Avg: sequential fp32 sum / in-bounds count.
 * ------------------------------------------------------------------------- */
static void pool2d(Tensor* in, Tensor* out, int kh, int kw, int sh, int sw, int ph, int pw, int is_max) {
    if (!in || !out || !in->data || !out->data || in->ndim != 4 || out->ndim != 4) return;
    const int N = (int)in->shape[0], C = (int)in->shape[1], H = (int)in->shape[2], W = (int)in->shape[3];
    const int OH = (int)out->shape[2], OW = (int)out->shape[3];
    const float* x = (const float*)in->data;
    float* z = (float*)out->data;
    for (int64_t nc = 0; nc < (int64_t)N * C; ++nc) {
        const float* plane = x + nc * H * W;
        for (int oh = 0; oh < OH; ++oh) {
            for (int ow = 0; ow < OW; ++ow) {
                int h0 = oh * sh - ph, w0 = ow * sw - pw;
                int h1 = h0 + kh, w1 = w0 + kw;
                if (h0 < 0) h0 = 0;
                if (w0 < 0) w0 = 0;
                if (h1 > H) h1 = H;
                if (w1 > W) w1 = W;
                float acc = is_max ? -3.402823e38f : 0.0f;
                int seen = 0;
                for (int h = h0; h < h1; ++h) {
                    for (int w = w0; w < w1; ++w) {
                        const float v = plane[h * W + w];
                        if (is_max) {
                            if (!seen || v > acc) acc = v;
                        } else {
                            acc += v;
                        }
                        ++seen;
                    }
                }
                if (!is_max) acc = seen > 0 ? acc / seen : 0.0f;
                z[(nc * OH + oh) * OW + ow] = acc;
            }
        }
    }
}

void nnc_maxpool2d(Tensor* in, Tensor* out, int kh, int kw, int sh, int sw, int ph, int pw) { pool2d(in, out, kh, kw, sh, sw, ph, pw, 1); }
void nnc_avgpool2d(Tensor* in, Tensor* out, int kh, int kw, int sh, int sw, int ph, int pw) { pool2d(in, out, kh, kw, sh, sw, ph, pw, 0); }

/* ---------------------------------------------------------------------------
 * Convolution (ops.c:720-1050 and its specialisations :1052-1447): for each
 * output, fp64 sum starting at the bias, over (c_in, kh, kw) with
 * out-of-range taps skipped, one rounding to fp32, then the activation.
 * ------------------------------------------------------------------------- */
enum { ACT_NONE = 0, ACT_RELU = 1, ACT_SIGMOID = 2 };

static float activate(float v, int act) {
    if (act == ACT_RELU) return v > 0.0f ? v : 0.0f;
    if (act == ACT_SIGMOID) return 1.0f / (1.0f + expf(-v));
    return v;
}

static void conv2d(Tensor* in, Tensor* wt, Tensor* bias, Tensor* out, int kh, int kw, int sh, int sw,
                   int ph, int pw, int act) {
    if (!in || !wt || !out || !in->data || !wt->data || !out->data) return;
    const int N = (int)in->shape[0], C = (int)in->shape[1], H = (int)in->shape[2], W = (int)in->shape[3];
    const int CO = (int)wt->shape[0], OH = (int)out->shape[2], OW = (int)out->shape[3];
    const float* x = (const float*)in->data;
    const float* w = (const float*)wt->data;
    const float* b = bias ? (const float*)bias->data : NULL;
    float* z = (float*)out->data;
    for (int n = 0; n < N; ++n) {
        for (int co = 0; co < CO; ++co) {
            for (int oh = 0; oh < OH; ++oh) {
                for (int ow = 0; ow < OW; ++ow) {
                    double acc = b ? (double)b[co] : 0.0;
                    for (int ci = 0; ci < C; ++ci) {
                        const float* xp = x + ((int64_t)n * C + ci) * H * W;
                        const float* wp = w + ((int64_t)co * C + ci) * kh * kw;
                        for (int i = 0; i < kh; ++i) {
                            const int h = oh * sh - ph + i;
                            if (h < 0 || h >= H) continue;
                            for (int j = 0; j < kw; ++j) {
                                const int ww = ow * sw - pw + j;
                                if (ww < 0 || ww >= W) continue;
                                acc += (double)xp[h * W + ww] * (double)wp[i * kw + j];
                            }
                        }
                    }
                    z[(((int64_t)n * CO + co) * OH + oh) * OW + ow] = activate((float)acc, act);
                }
            }
        }
    }
}

void nnc_conv(Tensor* i, Tensor* w, Tensor* b, Tensor* o, int kh, int kw, int sh, int sw, int ph, int pw) { conv2d(i, w, b, o, kh, kw, sh, sw, ph, pw, ACT_NONE); }
void nnc_conv_relu(Tensor* i, Tensor* w, Tensor* b, Tensor* o, int kh, int kw, int sh, int sw, int ph, int pw) { conv2d(i, w, b, o, kh, kw, sh, sw, ph, pw, ACT_RELU); }
void nnc_conv_sigmoid(Tensor* i, Tensor* w, Tensor* b, Tensor* o, int kh, int kw, int sh, int sw, int ph, int pw) { conv2d(i, w, b, o, kh, kw, sh, sw, ph, pw, ACT_SIGMOID); }
void nnc_conv1x1(Tensor* i, Tensor* w, Tensor* b, Tensor* o, int sh, int sw, int ph, int pw) { conv2d(i, w, b, o, 1, 1, sh, sw, ph, pw, ACT_NONE); }
void nnc_conv_relu1x1(Tensor* i, Tensor* w, Tensor* b, Tensor* o, int sh, int sw, int ph, int pw) { conv2d(i, w, b, o, 1, 1, sh, sw, ph, pw, ACT_RELU); }
void nnc_conv3x3_s1(Tensor* i, Tensor* w, Tensor* b, Tensor* o) { conv2d(i, w, b, o, 3, 3, 1, 1, 1, 1, ACT_NONE); }
void nnc_conv_relu3x3_s1(Tensor* i, Tensor* w, Tensor* b, Tensor* o) { conv2d(i, w, b, o, 3, 3, 1, 1, 1, 1, ACT_RELU); }
void nnc_conv7x7_s2(Tensor* i, Tensor* w, Tensor* b, Tensor* o) { conv2d(i, w, b, o, 7, 7, 2, 2, 3, 3, ACT_NONE); }
void nnc_conv_relu7x7_s2(Tensor* i, Tensor* w, Tensor* b, Tensor* o) { conv2d(i, w, b, o, 7, 7, 2, 2, 3, 3, ACT_RELU); }

/* The fused residual group is the reference composition nnc_conv followed
 * by nnc_add_relu (ops.c:1449, :3233). */
void nnc_conv_add_relu(Tensor* i, Tensor* w, Tensor* b, Tensor* r, Tensor* o, int kh, int kw, int sh,
                       int sw, int ph, int pw) {
    conv2d(i, w, b, o, kh, kw, sh, sw, ph, pw, ACT_NONE);
    nnc_add_relu(o, r, o);
}
/* The cuda target's fused Conv -> Relu -> MaxPool group: the reference
 * composition nnc_conv_relu (ops.c:3122-3194) into an NCHW temporary of
 * conv_h x conv_w, then nnc_maxpool2d (ops.c:316-391). */
void nnc_conv_relu_maxpool(Tensor* i, Tensor* w, Tensor* b, Tensor* o, int kh, int kw, int sh, int sw,
                           int ph, int pw, int conv_h, int conv_w, int pkh, int pkw, int psh, int psw,
                           int pph, int ppw) {
    int64_t shape[4] = {i->shape[0], w->shape[0], conv_h, conv_w};
    const int64_t n = shape[0] * shape[1] * shape[2] * shape[3];
    float* buf = (float*)malloc((size_t)(n > 0 ? n : 1) * sizeof(float));
    if (!buf) return;
    Tensor t = {buf, NNC_DTYPE_FLOAT32, shape, 4, n * (int64_t)sizeof(float)};
    nnc_conv_relu(i, w, b, &t, kh, kw, sh, sw, ph, pw);
    nnc_maxpool2d(&t, o, pkh, pkw, psh, psw, pph, ppw);
    free(buf);
}
void nnc_conv_add_relu1x1(Tensor* i, Tensor* w, Tensor* b, Tensor* r, Tensor* o, int sh, int sw, int ph, int pw) {
    nnc_conv_add_relu(i, w, b, r, o, 1, 1, sh, sw, ph, pw);
}
void nnc_conv_add_relu3x3_s1(Tensor* i, Tensor* w, Tensor* b, Tensor* r, Tensor* o) {
    nnc_conv_add_relu(i, w, b, r, o, 3, 3, 1, 1, 1, 1);
}

/* ---------------------------------------------------------------------------
 * Gemm (ops.c:1732-1841) and Gemm-NT (ops.c:1843-1886): fp64 dot product,
 * times alpha, plus beta * c ([N] when 1-D, else [M, N]), one rounding.
 * ------------------------------------------------------------------------- */
static void gemm_core(const float* A, const float* B, const Tensor* c, float* D, int M, int N, int K,
                      int ta, int tb, float alpha, float beta, int relu) {
    const float* C = c ? (const float*)c->data : NULL;
    for (int i = 0; i < M; ++i) {
        for (int j = 0; j < N; ++j) {
            double acc = 0.0;
            for (int k = 0; k < K; ++k) {
                const float av = ta ? A[(int64_t)k * M + i] : A[(int64_t)i * K + k];
                const float bv = tb ? B[(int64_t)j * K + k] : B[(int64_t)k * N + j];
                acc += (double)av * (double)bv;
            }
            acc *= (double)alpha;
            if (C) acc += (double)beta * (double)(c->ndim == 1 ? C[j] : C[(int64_t)i * N + j]);
            float v = (float)acc;
            if (relu) v = v > 0.0f ? v : 0.0f;
            D[(int64_t)i * N + j] = v;
        }
    }
}

static void gemm_dispatch(Tensor* a, Tensor* b, Tensor* c, Tensor* out, float alpha, float beta, int ta,
                          int tb, int relu) {
    int M, N, K;
    if (a->ndim == 2 && b->ndim == 2) {
        M = (int)(ta ? a->shape[1] : a->shape[0]);
        K = (int)(ta ? a->shape[0] : a->shape[1]);
        N = (int)(tb ? b->shape[0] : b->shape[1]);
    } else if (a->ndim == 1 && b->ndim == 2) {
        M = 1; K = (int)a->shape[0]; N = (int)b->shape[1]; ta = 0;
    } else if (a->ndim == 2 && b->ndim == 1) {
        M = (int)a->shape[0]; K = (int)a->shape[1]; N = 1; tb = 0;
    } else {
        /* The reference's flattened fallback leaves ta/tb as passed. */
        M = 1; K = (int)count_of(a); N = (int)count_of(b);
    }
    gemm_core((const float*)a->data, (const float*)b->data, c, (float*)out->data, M, N, K, ta, tb, alpha, beta, relu);
}

void nnc_gemm(Tensor* a, Tensor* b, Tensor* c, Tensor* o, float alpha, float beta, int ta, int tb) { gemm_dispatch(a, b, c, o, alpha, beta, ta, tb, 0); }
void nnc_gemm_relu(Tensor* a, Tensor* b, Tensor* c, Tensor* o, float alpha, float beta, int ta, int tb) { gemm_dispatch(a, b, c, o, alpha, beta, ta, tb, 1); }

static void gemm_nt_dispatch(Tensor* a, Tensor* b, Tensor* c, Tensor* out, float alpha, float beta, int relu) {
    int M, N, K;
    if (a->ndim == 2 && b->ndim == 2) {
        M = (int)a->shape[0]; K = (int)a->shape[1]; N = (int)b->shape[0];
    } else if (a->ndim == 1 && b->ndim == 2) {
        M = 1; K = (int)a->shape[0]; N = (int)b->shape[0];
    } else {
        M = 1; K = (int)count_of(a); N = b->ndim == 2 ? (int)b->shape[0] : (int)count_of(b);
    }
    gemm_core((const float*)a->data, (const float*)b->data, c, (float*)out->data, M, N, K, 0, 1, alpha, beta, relu);
}

void nnc_gemm_nt(Tensor* a, Tensor* b, Tensor* c, Tensor* o, float alpha, float beta) { gemm_nt_dispatch(a, b, c, o, alpha, beta, 0); }
void nnc_gemm_nt_relu(Tensor* a, Tensor* b, Tensor* c, Tensor* o, float alpha, float beta) { gemm_nt_dispatch(a, b, c, o, alpha, beta, 1); }

/* ---------------------------------------------------------------------------
 * MatMul (ops.c:1607-1730): Kahan-compensated fp32 dot products. For the
 * batched case the reference offsets batch i of `a` by i * (numel(a) /
 * (rows * cols)) elements — the matrix count, not the matrix size — and the
 * same for `b` unless b has fewer dims than the output (offset 0); output
 * batches are dense. That rule is restated here unchanged.
 * ------------------------------------------------------------------------- */
static float kahan_dot(const float* a, int64_t sa, const float* b, int64_t sb, int K) {
    float acc = 0.0f, lost = 0.0f;
    for (int k = 0; k < K; ++k) {
        float y = a[k * sa] * b[k * sb] - lost;
        float t = acc + y;
        lost = (t - acc) - y;
        acc = t;
    }
    return acc;
}

static void matmul_any(Tensor* a, Tensor* b, const Tensor* bias, Tensor* out, int relu) {
    const float* A = (const float*)a->data;
    const float* B = (const float*)b->data;
    const float* bs = bias ? (const float*)bias->data : NULL;
    float* D = (float*)out->data;
    int64_t batches = 1, a_off = 0, b_off = 0;
    int M, N, K;
    if (a->ndim == 2 && b->ndim == 2) {
        M = (int)a->shape[0]; K = (int)a->shape[1]; N = (int)b->shape[1];
    } else if (a->ndim == 1 && b->ndim == 2) {
        M = 1; K = (int)a->shape[0]; N = (int)b->shape[1];
    } else if (a->ndim == 2 && b->ndim == 1) {
        M = (int)a->shape[0]; K = (int)a->shape[1]; N = 1;
    } else if (a->ndim >= 2 && b->ndim >= 2) {
        const int od = out->ndim;
        for (int d = 0; d < od - 2; ++d) batches *= out->shape[d];
        M = (int)out->shape[od - 2];
        N = (int)out->shape[od - 1];
        K = (int)a->shape[a->ndim - 1];
        a_off = count_of(a) / (a->shape[a->ndim - 2] * a->shape[a->ndim - 1]);
        b_off = b->ndim < od ? 0 : count_of(b) / (b->shape[b->ndim - 2] * b->shape[b->ndim - 1]);
    } else {
        return;
    }
    for (int64_t bi = 0; bi < batches; ++bi) {
        const float* Ab = A + bi * a_off;
        const float* Bb = B + bi * b_off;
        float* Db = D + bi * (int64_t)M * N;
        for (int i = 0; i < M; ++i) {
            for (int j = 0; j < N; ++j) {
                float v = kahan_dot(Ab + (int64_t)i * K, 1, Bb + j, N, K);
                if (bs) v += bs[j];
                if (relu) v = v > 0.0f ? v : 0.0f;
                Db[(int64_t)i * N + j] = v;
            }
        }
    }
}

void nnc_matmul(Tensor* a, Tensor* b, Tensor* out) { matmul_any(a, b, NULL, out, 0); }
/* The symbol nnc-py's CEmitter emits for FUSED_MATMUL_RELU
 * (codegen/c_emitter.py:1143-1171), absent from the reference's ops.c:
 * restated as relu(matmul(a, b) + bias). */
void nnc_matmul_relu(Tensor* a, Tensor* b, Tensor* bias, Tensor* out) { matmul_any(a, b, bias, out, 1); }
/* MatMul -> Add(bias[N]) of the reference (ops.c:1607-1730, then the
 * modular broadcast add of ops.c:90-118 with the bias as the short operand). */
void nnc_matmul_bias(Tensor* a, Tensor* b, Tensor* bias, Tensor* out) { matmul_any(a, b, bias, out, 0); }
/* MatMul -> scale -> Softmax over the last axis (ops.c:1607-1730, ops.c:260-310):
 * the product rounded to fp32, times alpha (one rounding; exact for the
 * power-of-two alpha the codegen fuses, equal to the reference's division by
 * 1 / alpha), then the reference's softmax. */
void nnc_matmul_scale_softmax(Tensor* a, Tensor* b, Tensor* out, float alpha) {
    matmul_any(a, b, NULL, out, 0);
    float* D = (float*)out->data;
    const int64_t n = count_of(out);
    for (int64_t i = 0; i < n; ++i) D[i] = D[i] * alpha;
    nnc_softmax(out, out, -1);
}

/* Add -> LayerNormalization, the cuda target's O3 residual join: the
 * reference's add (ops.c:82-118) into a temporary, then its layernorm
 * (ops.c:2095-2171). */
void nnc_add_layernorm(Tensor* a, Tensor* b, Tensor* scale, Tensor* bias, Tensor* out, int axis,
                       float eps) {
    const int64_t n = count_of(a);
    float* sum = (float*)malloc((size_t)(n > 0 ? n : 1) * sizeof(float));
    Tensor t = *a;
    t.data = sum;
    nnc_add(a, b, &t);
    nnc_layernorm(&t, scale, bias, out, axis, eps);
    free(sum);
}

/* GlobalAveragePool -> Flatten -> Gemm(transB = 1), the cuda target's O3
 * head group: the reference's avgpool with kernel = stride = H x W
 * (ops.c:393-461), its flatten (a copy, ops.c:1521) and gemm_nt
 * (ops.c:1843-1886), composed. */
void nnc_gap_gemm_nt(Tensor* in, Tensor* b, Tensor* c, Tensor* out, float alpha, float beta) {
    const int64_t N = in->shape[0], C = in->shape[1];
    const int H = (int)in->shape[2], W = (int)in->shape[3];
    float* pooled = (float*)malloc((size_t)(N * C > 0 ? N * C : 1) * sizeof(float));
    int64_t s4[4] = {N, C, 1, 1}, s2[2] = {N, C};
    Tensor p4 = {pooled, NNC_DTYPE_FLOAT32, s4, 4, N * C * 4};
    Tensor p2 = {pooled, NNC_DTYPE_FLOAT32, s2, 2, N * C * 4};
    nnc_avgpool2d(in, &p4, H, W, H, W, 0, 0);
    nnc_gemm_nt(&p2, b, c, out, alpha, beta);
    free(pooled);
}

/* ---------------------------------------------------------------------------
 * Data movement (ops.c:1510-1601, :1995-2086, :2173-2251).
 * ------------------------------------------------------------------------- */
static void copy_prefix(Tensor* in, Tensor* out) {
    const int64_t n = count_of(out);
    memmove(out->data, in->data, (size_t)n * sizeof(float));
}
void nnc_reshape(Tensor* in, Tensor* out, int64_t* shape, int ndim) { (void)shape; (void)ndim; copy_prefix(in, out); }
void nnc_flatten(Tensor* in, Tensor* out, int axis) { (void)axis; copy_prefix(in, out); }
void nnc_squeeze(Tensor* in, Tensor* out, int axis) { (void)axis; copy_prefix(in, out); }
void nnc_unsqueeze(Tensor* in, Tensor* out, int axis) { (void)axis; copy_prefix(in, out); }
void nnc_identity(Tensor* in, Tensor* out) {
    int64_t n = count_of(out), m = count_of(in);
    memmove(out->data, in->data, (size_t)(n < m ? n : m) * sizeof(float));
}

void nnc_transpose(Tensor* in, Tensor* out, int64_t* perm, int ndim) {
    int64_t p[8], in_stride[8], dims[8];
    for (int d = 0; d < ndim; ++d) p[d] = perm ? perm[d] : ndim - 1 - d;
    in_stride[ndim - 1] = 1;
    for (int d = ndim - 2; d >= 0; --d) in_stride[d] = in_stride[d + 1] * in->shape[d + 1];
    for (int d = 0; d < ndim; ++d) dims[d] = out->shape[d];
    const float* x = (const float*)in->data;
    float* z = (float*)out->data;
    const int64_t n = count_of(out);
    for (int64_t o = 0; o < n; ++o) {
        int64_t rem = o, src = 0;
        for (int d = ndim - 1; d >= 0; --d) {
            src += (rem % dims[d]) * in_stride[p[d]];
            rem /= dims[d];
        }
        z[o] = x[src];
    }
}

/* Reshape -> Transpose / Transpose -> Reshape of the cuda target's O3
 * groups: the reference's reshape (a copy, ops.c:1510), transpose
 * (ops.c:1531-1581) and reshape composed, through views of the same bytes. */
void nnc_transpose_shaped(Tensor* in, Tensor* out, int64_t* in_shape, int64_t* perm, int ndim) {
    int64_t ish[8], osh[8];
    for (int d = 0; d < ndim; ++d) ish[d] = in_shape ? in_shape[d] : in->shape[d];
    for (int d = 0; d < ndim; ++d) osh[d] = ish[perm ? perm[d] : ndim - 1 - d];
    Tensor vin = *in, vout = *out;
    vin.shape = ish;
    vin.ndim = ndim;
    vout.shape = osh;
    vout.ndim = ndim;
    nnc_transpose(&vin, &vout, perm, ndim);
}

void nnc_concat(Tensor** inputs, Tensor* out, int num, int axis) {
    int64_t outer, odim, inner;
    const int a = around_axis(out, axis, &outer, &odim, &inner);
    const size_t es = out->dtype == NNC_DTYPE_INT64 ? 8 : 4;
    int64_t offset = 0;
    for (int k = 0; k < num; ++k) {
        const int64_t d = inputs[k]->shape[a];
        for (int64_t o = 0; o < outer; ++o)
            memcpy((char*)out->data + (size_t)((o * odim + offset) * inner) * es,
                   (const char*)inputs[k]->data + (size_t)(o * d * inner) * es, (size_t)(d * inner) * es);
        offset += d;
    }
}

void nnc_split(Tensor* in, Tensor** outputs, int num, int axis) {
    int64_t outer, dim, inner;
    around_axis(in, axis, &outer, &dim, &inner);
    const int64_t part = dim / num; /* equal parts only */
    const size_t es = in->dtype == NNC_DTYPE_INT64 ? 8 : 4;
    for (int k = 0; k < num; ++k)
        for (int64_t o = 0; o < outer; ++o)
            memcpy((char*)outputs[k]->data + (size_t)(o * part * inner) * es,
                   (const char*)in->data + (size_t)((o * dim + k * part) * inner) * es, (size_t)(part * inner) * es);
}

/* ---------------------------------------------------------------------------
 * The rest of the operator library (ops.c:2088-3116).
 * ------------------------------------------------------------------------- */

/* ops.c:2517-2599: numel(input) elements; integer targets truncate (C casts,
 * the x86 conversion); float16 and unknown targets copy 4-byte elements. */
void nnc_cast(Tensor* in, Tensor* out, int to) {
    const int64_t n = count_of(in);
    const int from_bool = in->dtype == NNC_DTYPE_BOOL;
    const float* f = (const float*)in->data;
    const uint8_t* u = (const uint8_t*)in->data;
    if (to == NNC_DTYPE_FLOAT32) {
        if (!from_bool) { memcpy(out->data, in->data, (size_t)n * 4); return; }
        for (int64_t i = 0; i < n; ++i) ((float*)out->data)[i] = (float)u[i];
    } else if (to == NNC_DTYPE_INT32) {
        for (int64_t i = 0; i < n; ++i) ((int32_t*)out->data)[i] = from_bool ? (int32_t)u[i] : (int32_t)f[i];
    } else if (to == NNC_DTYPE_INT64) {
        for (int64_t i = 0; i < n; ++i) ((int64_t*)out->data)[i] = from_bool ? (int64_t)u[i] : (int64_t)f[i];
    } else if (to == NNC_DTYPE_BOOL) {
        if (from_bool) { memcpy(out->data, in->data, (size_t)n); return; }
        for (int64_t i = 0; i < n; ++i) ((uint8_t*)out->data)[i] = f[i] != 0.0f;
    } else {
        memcpy(out->data, in->data, (size_t)n * 4);
    }
}

/* ops.c:2342-2432: index by index over min(n, a_n, b_n), then the modular
 * broadcast of the shorter operand when the other spans the output. */
static void compare_apply(Tensor* a, Tensor* b, Tensor* out, int is_and) {
    const int64_t n = count_of(out), an = count_of(a), bn = count_of(b);
    const float* x = (const float*)a->data;
    const float* y = (const float*)b->data;
    float* z = (float*)out->data;
    int64_t m = n < an ? n : an;
    if (bn < m) m = bn;
    const int64_t end = (an == n || bn == n) ? n : m;
    for (int64_t i = 0; i < end; ++i) {
        const float p = x[i < an ? i : i % an], q = y[i < bn ? i : i % bn];
        const int r = is_and ? (p != 0.0f && q != 0.0f) : (p == q);
        z[i] = r ? 1.0f : 0.0f;
    }
}
void nnc_equal(Tensor* a, Tensor* b, Tensor* out) { compare_apply(a, b, out, 0); }
void nnc_and(Tensor* a, Tensor* b, Tensor* out) { compare_apply(a, b, out, 1); }

/* ops.c:2655-2703. */
void nnc_greater(Tensor* a, Tensor* b, Tensor* out) {
    const int64_t n = count_of(out), an = count_of(a), bn = count_of(b);
    for (int64_t i = 0; i < n; ++i)
        ((uint8_t*)out->data)[i] = ((const float*)a->data)[i % an] > ((const float*)b->data)[i % bn];
}
void nnc_or(Tensor* a, Tensor* b, Tensor* out) {
    const int64_t n = count_of(out);
    for (int64_t i = 0; i < n; ++i)
        ((uint8_t*)out->data)[i] = ((const uint8_t*)a->data)[i] || ((const uint8_t*)b->data)[i];
}
void nnc_not(Tensor* in, Tensor* out) {
    const int64_t n = count_of(out);
    for (int64_t i = 0; i < n; ++i) ((uint8_t*)out->data)[i] = !((const uint8_t*)in->data)[i];
}

/* ops.c:2601-2653. */
void nnc_shape(Tensor* in, Tensor* out, int64_t* shape_data, int ndim) {
    for (int d = 0; d < ndim; ++d) ((int64_t*)out->data)[d] = shape_data ? shape_data[d] : in->shape[d];
}
void nnc_constantofshape(Tensor* out, float value, int ndim) {
    (void)ndim;
    const int64_t n = count_of(out);
    for (int64_t i = 0; i < n; ++i) ((float*)out->data)[i] = value;
}
void nnc_expand(Tensor* in, Tensor* out, int64_t* shape, int ndim) {
    (void)shape; (void)ndim;
    const int64_t n = count_of(out), m = count_of(in);
    for (int64_t i = 0; i < n; ++i) ((float*)out->data)[i] = ((const float*)in->data)[i % m];
}

/* ops.c:2264-2336: the output coordinates (over the output's extents), the
 * first input-rank of them taken modulo the input's extents. */
void nnc_tile(Tensor* in, Tensor* out, int64_t* repeats, int ndim) {
    (void)ndim;
    const int64_t n = count_of(out);
    const float* x = (const float*)in->data;
    float* z = (float*)out->data;
    if (!repeats) { memcpy(z, x, (size_t)n * 4); return; }
    int64_t stride[8];
    stride[in->ndim - 1] = 1;
    for (int d = in->ndim - 2; d >= 0; --d) stride[d] = stride[d + 1] * in->shape[d + 1];
    for (int64_t o = 0; o < n; ++o) {
        int64_t c[8], rem = o, src = 0;
        for (int d = out->ndim - 1; d >= 0; --d) { c[d] = rem % out->shape[d]; rem /= out->shape[d]; }
        for (int d = 0; d < in->ndim; ++d) src += (c[d] % in->shape[d]) * stride[d];
        z[o] = x[src];
    }
}

/* ops.c:2705-2910: the reference's cascade of gather cases. */
static int64_t wrap_clamp(int64_t g, int64_t extent) {
    if (g < 0) g += extent;
    if (g < 0) g = 0;
    if (g >= extent) g = extent - 1;
    return g;
}
void nnc_gather(Tensor* data, Tensor* indices, Tensor* out, int axis, int data_dtype) {
    const int rank = data->ndim, irank = indices->ndim, orank = out->ndim;
    const int64_t* idx = (const int64_t*)indices->data;
    const float* df = (const float*)data->data;
    const int64_t* dl = (const int64_t*)data->data;
    float* of = (float*)out->data;
    int64_t* ol = (int64_t*)out->data;
    const int64_t on = count_of(out);
    if (axis < 0) axis += rank;
    if (axis < 0) axis = 0;
    if (axis >= rank) axis = rank - 1;
    if (irank == 0 || (irank == 1 && indices->shape[0] == 1)) {
        const int64_t g = wrap_clamp(idx[0], data->shape[axis]);
        if (data_dtype == 1) {
            if (rank == 1) { ol[0] = dl[g]; return; }
            int64_t copy = 1;
            for (int d = axis + 1; d < rank; ++d) copy *= data->shape[d];
            for (int64_t i = 0; i < copy; ++i) ol[i] = dl[g * copy + i];
            return;
        }
        if (rank == 1) { for (int64_t i = 0; i < on; ++i) of[i] = df[g]; return; }
        if (rank == 2 && orank == 2) {
            const int64_t d1 = data->shape[1];
            for (int64_t i = 0; i < out->shape[0]; ++i)
                for (int64_t j = 0; j < out->shape[1]; ++j)
                    of[i * out->shape[1] + j] = axis == 0 ? df[g * d1 + j] : df[i * d1 + g];
            return;
        }
        if (rank == 3) {
            const int64_t d0 = data->shape[0], d1 = data->shape[1], d2 = data->shape[2];
            if (axis == 0 && (orank == 2 || orank == 3)) {
                const int64_t n0 = orank == 2 ? 1 : out->shape[0];
                const int64_t n1 = orank == 2 ? d1 : out->shape[1], n2 = orank == 2 ? d2 : out->shape[2];
                for (int64_t i = 0; i < n0; ++i)
                    for (int64_t j = 0; j < n1; ++j)
                        for (int64_t k = 0; k < n2; ++k) of[(i * n1 + j) * n2 + k] = df[(g * d1 + j) * d2 + k];
                return;
            }
            if (axis == 1) {
                for (int64_t i = 0; i < d0; ++i)
                    for (int64_t k = 0; k < d2; ++k) of[i * d2 + k] = df[(i * d1 + g) * d2 + k];
                return;
            }
            if (axis == 2) {
                for (int64_t i = 0; i < d0; ++i)
                    for (int64_t j = 0; j < d1; ++j) of[i * d1 + j] = df[(i * d1 + j) * d2 + g];
                return;
            }
        }
    }
    if (irank == 1) {
        const int64_t num = indices->shape[0];
        if (data_dtype == 1 && rank == 1) {
            for (int64_t k = 0; k < num; ++k) ol[k] = dl[wrap_clamp(idx[k], data->shape[0])];
            return;
        }
        if (rank == 2) {
            const int64_t d1 = data->shape[1];
            for (int64_t k = 0; k < num; ++k) {
                const int64_t g = wrap_clamp(idx[k], data->shape[axis]);
                if (axis == 0) {
                    for (int64_t j = 0; j < d1; ++j) of[k * d1 + j] = df[g * d1 + j];
                } else {
                    for (int64_t i = 0; i < data->shape[0]; ++i) of[i * num + k] = df[i * d1 + g];
                }
            }
            return;
        }
    }
    const int64_t dn = count_of(data);
    for (int64_t i = 0; i < on; ++i) {
        if (data_dtype == 1) ol[i] = dl[i % dn];
        else of[i] = df[i % dn];
    }
}

/* ops.c:2088-2093: an empty TODO in the reference. */
void nnc_batchnorm(Tensor* input, Tensor* scale, Tensor* bias, Tensor* mean, Tensor* var,
                   Tensor* output, float epsilon, int momentum) {
    (void)input; (void)scale; (void)bias; (void)mean; (void)var; (void)output; (void)epsilon; (void)momentum;
}

/* ops.c:2928-3116: gate order I, O, F, C; each gate a sequential fp32 sum of
 * W x, then R h, then the sum of its two biases; one state carried through
 * every (step, batch item); Y indexed by the forward step. */
void nnc_lstm(Tensor* X, Tensor* W, Tensor* R, Tensor* B, Tensor* Y, Tensor* Y_h, Tensor* Y_c,
              int direction, int hidden) {
    const int64_t T = X->shape[0], Bn = X->shape[1], I = X->shape[2], H = hidden;
    const int dirs = direction == 2 ? 2 : 1;
    float* h = calloc((size_t)H, sizeof(float));
    float* c = calloc((size_t)H, sizeof(float));
    float* hn = calloc((size_t)H, sizeof(float));
    float* cn = calloc((size_t)H, sizeof(float));
    for (int dir = 0; dir < dirs; ++dir) {
        memset(h, 0, (size_t)H * sizeof(float));
        memset(c, 0, (size_t)H * sizeof(float));
        const float* w = (const float*)W->data + (int64_t)dir * 4 * H * I;
        const float* r = (const float*)R->data + (int64_t)dir * 4 * H * H;
        const float* bb = B ? (const float*)B->data + (int64_t)dir * 8 * H : NULL;
        for (int64_t t = 0; t < T; ++t) {
            const int64_t tt = dir == 1 ? T - 1 - t : t;
            for (int64_t b = 0; b < Bn; ++b) {
                const float* x = (const float*)X->data + (tt * Bn + b) * I;
                for (int64_t row = 0; row < H; ++row) {
                    float g[4];
                    for (int q = 0; q < 4; ++q) {
                        float s = 0.0f;
                        for (int64_t j = 0; j < I; ++j) s += w[(q * H + row) * I + j] * x[j];
                        for (int64_t j = 0; j < H; ++j) s += r[(q * H + row) * H + j] * h[j];
                        if (bb) s += bb[q * H + row] + bb[(4 + q) * H + row];
                        g[q] = s;
                    }
                    const float ig = 1.0f / (1.0f + expf(-g[0])), og = 1.0f / (1.0f + expf(-g[1]));
                    const float fg = 1.0f / (1.0f + expf(-g[2])), gg = tanhf(g[3]);
                    cn[row] = fg * c[row] + ig * gg;
                    hn[row] = og * tanhf(cn[row]);
                }
                memcpy(h, hn, (size_t)H * sizeof(float));
                memcpy(c, cn, (size_t)H * sizeof(float));
                memcpy((float*)Y->data + ((t * dirs + dir) * Bn + b) * H, h, (size_t)H * sizeof(float));
            }
        }
        for (int64_t b = 0; b < Bn; ++b) {
            memcpy((float*)Y_h->data + (dir * Bn + b) * H, h, (size_t)H * sizeof(float));
            memcpy((float*)Y_c->data + (dir * Bn + b) * H, c, (size_t)H * sizeof(float));
        }
    }
    free(h); free(c); free(hn); free(cn);
}
