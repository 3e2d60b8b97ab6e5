/*
 * ref_cpu.c -- CPU oracle for the jax4j FP32 hot path (test infrastructure).
 *
 * A plain-C restatement of the reference's pure-Java host implementation.
 * Used only as the checker by tests/, __graft_entry__.smoke() and the CPU
 * baseline leg of bench.py; never linked into or called by the product.
 * Build with -O2 -ffp-contract=off -fno-fast-math (see oracle/build.py):
 * Java evaluates float expressions without fused multiply-add.
 *
 * Citations are file:line in marmanis/jax4j, relative to
 * src/main/java/com/marmanis/jax4j/.
 */
#include "ref_cpu.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ */
/* Random.java:39-150 (SplitMix64 streams)                             */
/* ------------------------------------------------------------------ */
#define GOLDEN_GAMMA 0x9E3779B97F4A7C15ULL
#define SPLIT_TAG 0xD1B54A32D192ED03ULL
#define SAMPLE_TAG 0x2545F4914F6CDD1DULL

/* api/Random.java:44-48 */
uint64_t orc_mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

/* api/Random.java:56-58 */
static uint64_t stream_value(uint64_t state, uint64_t tag, uint64_t index) {
    return orc_mix64(state ^ tag ^ (GOLDEN_GAMMA * (index + 1)));
}

/* api/Random.java:61-65: top 24 bits / 2^24, an exact float division */
static float raw_uniform01(uint64_t state, uint64_t i) {
    uint64_t bits = stream_value(state, SAMPLE_TAG, i);
    int32_t top24 = (int32_t)(bits >> 40);
    return (float)top24 / (float)(1 << 24);
}

/* api/Random.java:70-76 */
void orc_split(uint64_t state, int num, uint64_t *out) {
    for (int i = 0; i < num; i++)
        out[i] = orc_mix64(state ^ SPLIT_TAG ^ (GOLDEN_GAMMA * (uint64_t)(i + 1)));
}

/* api/Random.java:86-93: lo + u * (hi - lo), each step rounded to float */
/* Random.permutation (api/Random.java:130-140): Fisher-Yates from the top. */
void orc_permutation(uint64_t state, int64_t n, int32_t *out) {
    for (int64_t i = 0; i < n; i++) out[i] = (int32_t)i;
    for (int64_t i = n - 1; i > 0; i--) {
        float u = raw_uniform01(state, (uint64_t)i);
        float prod = u * (float)(i + 1);
        int64_t j = (int64_t)(int32_t)prod;
        if (j > i) j = i;
        int32_t t = out[i];
        out[i] = out[j];
        out[j] = t;
    }
}

void orc_uniform(uint64_t state, int64_t n, float lo, float hi, float *out) {
    float span = hi - lo;
    for (int64_t i = 0; i < n; i++) {
        float u = raw_uniform01(state, (uint64_t)i);
        float scaled = u * span;
        out[i] = lo + scaled;
    }
}

/* api/Random.java:104-113: Box-Muller in double, narrowed to float */
void orc_normal(uint64_t state, int64_t n, float *out) {
    const double two_pi = 2.0 * 3.141592653589793;
    for (int64_t i = 0; i < n; i++) {
        float u1 = raw_uniform01(state, 2ULL * (uint64_t)i);
        if (!(u1 >= 1e-7f)) u1 = 1e-7f; /* Math.max(u1, 1e-7f); u1 is never NaN */
        float u2 = raw_uniform01(state, 2ULL * (uint64_t)i + 1ULL);
        out[i] = (float)(sqrt(-2.0 * log((double)u1)) * cos(two_pi * (double)u2));
    }
}

/* api/Random.java:147-150 */
void orc_glorot_uniform(uint64_t state, int64_t n, int fan_in, int fan_out, float *out) {
    float limit = (float)sqrt(6.0 / (double)(fan_in + fan_out));
    orc_uniform(state, n, -limit, limit, out);
}

/* ------------------------------------------------------------------ */
/* Shape.java:37-101                                                   */
/* ------------------------------------------------------------------ */
static int64_t shape_size(const int64_t *d, int r) {
    int64_t s = 1;
    for (int i = 0; i < r; i++) s *= d[i];
    return s;
}

static int shape_equal(const int64_t *a, int ar, const int64_t *b, int br) {
    if (ar != br) return 0;
    for (int i = 0; i < ar; i++)
        if (a[i] != b[i]) return 0;
    return 1;
}

/* core/Shape.java:83-101 */
int64_t orc_broadcast_index(const int64_t *dims, int rank, const int64_t *out_dims, int out_rank,
                            int64_t flat) {
    if (shape_equal(dims, rank, out_dims, out_rank)) return flat;
    int64_t coords[16];
    int64_t rem = flat;
    for (int i = out_rank - 1; i >= 0; i--) {
        coords[i] = rem % out_dims[i];
        rem /= out_dims[i];
    }
    int offset = out_rank - rank;
    int64_t f = 0;
    for (int i = 0; i < rank; i++) {
        int64_t dim = dims[i];
        int64_t c = dim == 1 ? 0 : coords[i + offset];
        f = f * dim + c;
    }
    return f;
}

/* ------------------------------------------------------------------ */
/* java.lang.Math.max/min(double,double): NaN wins, max(-0,+0) = +0     */
/* ------------------------------------------------------------------ */
static double java_max(double a, double b) {
    if (a != a) return a;
    if (a == 0.0 && b == 0.0 && signbit(a)) return b;
    return (a >= b) ? a : b;
}

static double java_min(double a, double b) {
    if (a != a) return a;
    if (a == 0.0 && b == 0.0 && signbit(b)) return b;
    return (a <= b) ? a : b;
}

static double binary_op(int prim, double a, double b) {
    switch (prim) {
    case ORC_ADD: return a + b;
    case ORC_SUB: return a - b;
    case ORC_MUL: return a * b;
    case ORC_DIV: return a / b;
    case ORC_MAX: return java_max(a, b);
    case ORC_MIN: return java_min(a, b);
    default: return NAN;
    }
}

/* core/ConcreteNDArray.java:274-292: op in double, narrowed to float */
int orc_binary_f32(int prim, const float *a, const int64_t *ad, int ar, const float *b,
                   const int64_t *bd, int br, float *out, const int64_t *od, int orank) {
    if (prim != ORC_ADD && prim != ORC_SUB && prim != ORC_MUL && prim != ORC_DIV &&
        prim != ORC_MAX && prim != ORC_MIN)
        return -1;
    int64_t n = shape_size(od, orank);
    for (int64_t i = 0; i < n; i++) {
        float v1 = a[orc_broadcast_index(ad, ar, od, orank, i)];
        float v2 = b[orc_broadcast_index(bd, br, od, orank, i)];
        out[i] = (float)binary_op(prim, (double)v1, (double)v2);
    }
    return 0;
}

static int compare_d(int prim, double a, double b) {
    switch (prim) {
    case ORC_GT: return a > b;
    case ORC_GE: return a >= b;
    case ORC_LT: return a < b;
    case ORC_LE: return a <= b;
    case ORC_EQ: return a == b;
    case ORC_NE: return a != b;
    default: return 0;
    }
}

static int compare_l(int prim, int64_t a, int64_t b) {
    switch (prim) {
    case ORC_GT: return a > b;
    case ORC_GE: return a >= b;
    case ORC_LT: return a < b;
    case ORC_LE: return a <= b;
    case ORC_EQ: return a == b;
    case ORC_NE: return a != b;
    default: return 0;
    }
}

/* core/ConcreteNDArray.java:343-396: F32/F64/I32 compare as double, I64 as long */
int orc_compare(int prim, int dtype, const void *a, const int64_t *ad, int ar, const void *b,
                const int64_t *bd, int br, uint8_t *out, const int64_t *od, int orank) {
    if (prim < ORC_GT || prim > ORC_NE) return -1;
    int64_t n = shape_size(od, orank);
    for (int64_t i = 0; i < n; i++) {
        int64_t ia = orc_broadcast_index(ad, ar, od, orank, i);
        int64_t ib = orc_broadcast_index(bd, br, od, orank, i);
        int r;
        switch (dtype) {
        case ORC_F32: r = compare_d(prim, ((const float *)a)[ia], ((const float *)b)[ib]); break;
        case ORC_F64: r = compare_d(prim, ((const double *)a)[ia], ((const double *)b)[ib]); break;
        case ORC_I32: r = compare_d(prim, ((const int32_t *)a)[ia], ((const int32_t *)b)[ib]); break;
        case ORC_I64: r = compare_l(prim, ((const int64_t *)a)[ia], ((const int64_t *)b)[ib]); break;
        default: return -1; /* BOOL is not comparable (ConcreteNDArray.java:393-394) */
        }
        out[i] = (uint8_t)r;
    }
    return 0;
}

/* core/ConcreteNDArray.java:648-664: (float) Math.f((double) x) */
int orc_unary_f32(int prim, const float *in, int64_t n, float *out) {
    for (int64_t i = 0; i < n; i++) {
        double x = (double)in[i];
        double r;
        switch (prim) {
        case ORC_EXP: r = exp(x); break;
        case ORC_LOG: r = log(x); break;
        case ORC_SIN: r = sin(x); break;
        case ORC_COS: r = cos(x); break;
        case ORC_TANH: r = tanh(x); break;
        case ORC_RELU: r = java_max(0.0, x); break;
        case ORC_SIGMOID: r = 1.0 / (1.0 + exp(-x)); break;
        default: return -1;
        }
        out[i] = (float)r;
    }
    return 0;
}

/* JLS 5.1.3 narrowing of a floating value to int/long: NaN -> 0,
 * out-of-range values saturate, otherwise truncation toward zero. */
static int32_t java_d2i(double v) {
    if (v != v) return 0;
    if (v >= 2147483647.0) return INT32_MAX;
    if (v <= -2147483648.0) return INT32_MIN;
    return (int32_t)v;
}

static int64_t java_d2l(double v) {
    if (v != v) return 0;
    if (v >= 9223372036854775807.0) return INT64_MAX;
    if (v <= -9223372036854775808.0) return INT64_MIN;
    return (int64_t)v;
}

/* core/ConcreteNDArray.java:666-730 */
int orc_cast(int src, int dst, const void *in, int64_t n, void *out) {
    for (int64_t i = 0; i < n; i++) {
        double dv = 0;
        int64_t lv = 0;
        int is_long = 0, truth = 0;
        switch (src) {
        case ORC_F32: dv = ((const float *)in)[i]; truth = ((const float *)in)[i] != 0.0f; break;
        case ORC_F64: dv = ((const double *)in)[i]; truth = ((const double *)in)[i] != 0.0; break;
        case ORC_I32: lv = ((const int32_t *)in)[i]; is_long = 1; truth = lv != 0; break;
        case ORC_I64: lv = ((const int64_t *)in)[i]; is_long = 1; truth = lv != 0; break;
        case ORC_BOOL: lv = ((const uint8_t *)in)[i] ? 1 : 0; is_long = 1; truth = lv != 0; break;
        default: return -1;
        }
        switch (dst) {
        case ORC_F32:
            if (src == ORC_F32) ((float *)out)[i] = ((const float *)in)[i];
            else if (is_long) ((float *)out)[i] = (float)lv; /* round to nearest */
            else ((float *)out)[i] = (float)dv;
            break;
        case ORC_F64:
            ((double *)out)[i] = is_long ? (double)lv : dv;
            break;
        case ORC_I32:
            if (is_long) ((int32_t *)out)[i] = (int32_t)(uint32_t)(uint64_t)lv; /* narrows */
            else ((int32_t *)out)[i] = java_d2i(dv);
            break;
        case ORC_I64:
            ((int64_t *)out)[i] = is_long ? lv : java_d2l(dv);
            break;
        case ORC_BOOL:
            ((uint8_t *)out)[i] = (uint8_t)truth;
            break;
        default: return -1;
        }
    }
    return 0;
}

/* backend/HostBackend.java:117-124: sequential float sum from 0f; mean divides by (float) n */
void orc_reduce_all_f32(int prim, const float *in, int64_t n, float *out) {
    float sum = 0.0f;
    for (int64_t i = 0; i < n; i++) sum += in[i];
    if (prim == ORC_MEAN) sum = sum / (float)n;
    out[0] = sum;
}

/* core/ConcreteNDArray.java:536-547 */
void orc_reduce_axis_f32(int prim, const float *in, int64_t outer, int64_t axis, int64_t inner,
                         float *out) {
    for (int64_t o = 0; o < outer; o++) {
        for (int64_t r = 0; r < inner; r++) {
            float total = 0.0f;
            for (int64_t a = 0; a < axis; a++) total += in[o * axis * inner + a * inner + r];
            out[o * inner + r] = prim == ORC_MEAN_AXIS ? total / (float)axis : total;
        }
    }
}

/* core/ConcreteNDArray.java:602-617: first strict extremum wins */
void orc_argreduce_f32(int prim, const float *in, int64_t outer, int64_t axis, int64_t inner,
                       int32_t *out) {
    int is_max = prim == ORC_ARGMAX;
    for (int64_t o = 0; o < outer; o++) {
        for (int64_t r = 0; r < inner; r++) {
            int32_t best_idx = 0;
            float best = in[o * axis * inner + r];
            for (int64_t a = 1; a < axis; a++) {
                float v = in[o * axis * inner + a * inner + r];
                if (is_max ? v > best : v < best) {
                    best = v;
                    best_idx = (int32_t)a;
                }
            }
            out[o * inner + r] = best_idx;
        }
    }
}

/* ------------------------------------------------------------------ */
/* dot: core/ConcreteNDArray.java:452-459, backend/HostBackend.java:56-66 */
/* For every (i, j) the k-sum is the same sequential float sum from 0f.  */
/* The loops run i-k-j so the j lanes vectorise; each c[i][j] still sees  */
/* its products in k order, so the result is bit-identical to i-j-k.     */
/* ------------------------------------------------------------------ */
typedef struct {
    const float *a, *b;
    float *c;
    int64_t K, N, r0, r1;
} dot_job;

static void *dot_rows(void *arg) {
    dot_job *j = (dot_job *)arg;
    for (int64_t i = j->r0; i < j->r1; i++) {
        float *crow = j->c + i * j->N;
        for (int64_t n = 0; n < j->N; n++) crow[n] = 0.0f;
        const float *arow = j->a + i * j->K;
        for (int64_t k = 0; k < j->K; k++) {
            float av = arow[k];
            const float *brow = j->b + k * j->N;
            for (int64_t n = 0; n < j->N; n++) {
                float p = av * brow[n];
                crow[n] = crow[n] + p;
            }
        }
    }
    return NULL;
}

void orc_dot_f32(const float *a, const float *b, float *c, int64_t M, int64_t K, int64_t N,
                 int64_t row_begin, int64_t row_end, int threads) {
    (void)M;
    if (threads < 1) threads = 1;
    int64_t rows = row_end - row_begin;
    if (rows <= 0) return;
    if (threads > rows) threads = (int)rows;
    pthread_t tid[256];
    dot_job jobs[256];
    if (threads > 256) threads = 256;
    int64_t per = (rows + threads - 1) / threads;
    int started = 0;
    for (int t = 0; t < threads; t++) {
        int64_t r0 = row_begin + t * per;
        int64_t r1 = r0 + per > row_end ? row_end : r0 + per;
        if (r0 >= r1) break;
        jobs[t].a = a; jobs[t].b = b; jobs[t].c = c;
        jobs[t].K = K; jobs[t].N = N; jobs[t].r0 = r0; jobs[t].r1 = r1;
        if (threads == 1) {
            dot_rows(&jobs[t]);
        } else {
            pthread_create(&tid[t], NULL, dot_rows, &jobs[t]);
            started++;
        }
    }
    for (int t = 0; t < started; t++) pthread_join(tid[t], NULL);
}

/* ------------------------------------------------------------------ */
/* Grad.java host helpers                                              */
/* ------------------------------------------------------------------ */

/* api/Grad.java:562-581 (FLOAT32 branch of broadcastLike) */
void orc_broadcast_like_f32(const float *g, const int64_t *gd, int gr, float *out,
                            const int64_t *td, int tr) {
    int64_t gs = shape_size(gd, gr), ts = shape_size(td, tr);
    if (gs == ts) { /* equal shapes or a pure reshape */
        memcpy(out, g, (size_t)gs * sizeof(float));
        return;
    }
    if (gs < ts) {
        for (int64_t i = 0; i < ts; i++) out[i] = g[orc_broadcast_index(gd, gr, td, tr, i)];
    } else {
        for (int64_t i = 0; i < ts; i++) out[i] = 0.0f;
        for (int64_t i = 0; i < gs; i++) out[orc_broadcast_index(td, tr, gd, gr, i)] += g[i];
    }
}

/* api/Grad.java:593-597 */
void orc_relu_grad_f32(const float *g, const float *x, int64_t n, float *out) {
    for (int64_t i = 0; i < n; i++) out[i] = x[i] > 0 ? g[i] : 0.0f;
}

/* api/Grad.java:630-640 */
void orc_axis_broadcast_like_f32(const float *g, const int64_t *dims, int rank, int axis,
                                 float *out) {
    int64_t axis_size = dims[axis], outer = 1, inner = 1;
    for (int i = 0; i < axis; i++) outer *= dims[i];
    for (int i = axis + 1; i < rank; i++) inner *= dims[i];
    for (int64_t o = 0; o < outer; o++)
        for (int64_t r = 0; r < inner; r++) {
            float v = g[o * inner + r];
            for (int64_t a = 0; a < axis_size; a++) out[o * axis_size * inner + a * inner + r] = v;
        }
}

/* api/Grad.java:656-663 */
void orc_transpose_f32(const float *in, int64_t rows, int64_t cols, float *out) {
    for (int64_t i = 0; i < rows; i++)
        for (int64_t j = 0; j < cols; j++) out[j * rows + i] = in[i * cols + j];
}

/* api/Grad.java:517-527: a wins ties; gA/gB are full output-shaped arrays
 * (the caller applies broadcastLike to each, Grad.java:528-529) */
void orc_maxmin_grad_f32(int is_max, const float *g, const int64_t *od, int orank, const float *a,
                         const int64_t *ad, int ar, const float *b, const int64_t *bd, int br,
                         float *ga_full, float *gb_full) {
    int64_t n = shape_size(od, orank);
    for (int64_t i = 0; i < n; i++) {
        float va = a[orc_broadcast_index(ad, ar, od, orank, i)];
        float vb = b[orc_broadcast_index(bd, br, od, orank, i)];
        int a_wins = is_max ? va >= vb : va <= vb;
        ga_full[i] = a_wins ? g[i] : 0.0f;
        gb_full[i] = a_wins ? 0.0f : g[i];
    }
}

/* api/SharedCollective.java:44-54: every shard sums slots d = 0..D-1 from 0f */
void orc_psum_f32(const float *const *slots, int num_devices, int64_t n, float *out) {
    for (int64_t i = 0; i < n; i++) out[i] = 0.0f;
    for (int d = 0; d < num_devices; d++)
        for (int64_t i = 0; i < n; i++) out[i] += slots[d][i];
}

/* ------------------------------------------------------------------ */
/* MLP cross-entropy loss and its gradTree, in the order the Grad       */
/* interpreter executes the traced equations of                          */
/* examples/MNISTFromScratch.java:103-125 (predict + loss):              */
/*   h = a.dot(w); z = h.add(b); a' = act(z)   (hidden layers)           */
/*   e = exp(z_L); s = e.sum(-1, true); p = e.div(s); lp = p.log()        */
/*   m = lp.mul(t); r = m.sum(-1); mu = r.mean(); L = mu.mul([-1])        */
/* Backward follows Grad.computeVJPs (Grad.java:341-472) rule by rule.    */
/* ------------------------------------------------------------------ */
typedef struct {
    int L;
    int64_t B, C;
    float **h;  /* pre-bias dot outputs (not needed after bias add) */
    float **z;  /* z[l] = h[l] + b[l] */
    float **a;  /* a[0] = x, a[l+1] = act(z[l]) */
    float *e, *s, *p, *lp, *m, *r;
    float mu, loss;
} mlp_fwd;

static float *fbuf(int64_t n) { return (float *)malloc((size_t)(n > 0 ? n : 1) * sizeof(float)); }

/* z = h + b with b of shape [cols] broadcast over rows (ConcreteNDArray.java:286-290) */
static void add_row_bias(const float *h, const float *b, int64_t rows, int64_t cols, float *z) {
    for (int64_t i = 0; i < rows; i++)
        for (int64_t j = 0; j < cols; j++)
            z[i * cols + j] = (float)((double)h[i * cols + j] + (double)b[j]);
}

static void mlp_forward(mlp_fwd *f, int L, const int64_t *dims, int act, const float *const *w,
                        const float *const *b, const float *x, const float *t, int64_t B,
                        int threads) {
    f->L = L;
    f->B = B;
    f->C = dims[L];
    f->h = (float **)calloc((size_t)L, sizeof(float *));
    f->z = (float **)calloc((size_t)L, sizeof(float *));
    f->a = (float **)calloc((size_t)L + 1, sizeof(float *));
    f->a[0] = (float *)x;
    for (int l = 0; l < L; l++) {
        int64_t din = dims[l], dout = dims[l + 1];
        f->h[l] = fbuf(B * dout);
        orc_dot_f32(f->a[l], w[l], f->h[l], B, din, dout, 0, B, threads);
        f->z[l] = fbuf(B * dout);
        add_row_bias(f->h[l], b[l], B, dout, f->z[l]);
        free(f->h[l]);
        f->h[l] = NULL;
        if (l < L - 1) {
            f->a[l + 1] = fbuf(B * dout);
            orc_unary_f32(act == 0 ? ORC_TANH : ORC_RELU, f->z[l], B * dout, f->a[l + 1]);
        }
    }
    int64_t C = f->C, n = B * C;
    f->e = fbuf(n);
    orc_unary_f32(ORC_EXP, f->z[L - 1], n, f->e);
    f->s = fbuf(B);
    orc_reduce_axis_f32(ORC_SUM_AXIS, f->e, B, C, 1, f->s);
    f->p = fbuf(n);
    for (int64_t i = 0; i < B; i++)
        for (int64_t j = 0; j < C; j++) f->p[i * C + j] = f->e[i * C + j] / f->s[i];
    f->lp = fbuf(n);
    orc_unary_f32(ORC_LOG, f->p, n, f->lp);
    f->m = fbuf(n);
    for (int64_t i = 0; i < n; i++) f->m[i] = f->lp[i] * t[i];
    f->r = fbuf(B);
    orc_reduce_axis_f32(ORC_SUM_AXIS, f->m, B, C, 1, f->r);
    orc_reduce_all_f32(ORC_MEAN, f->r, B, &f->mu);
    f->loss = f->mu * -1.0f;
}

static void mlp_free(mlp_fwd *f) {
    for (int l = 0; l < f->L; l++) {
        free(f->z[l]);
        if (l + 1 < f->L) free(f->a[l + 1]);
    }
    free(f->h); free(f->z); free(f->a);
    free(f->e); free(f->s); free(f->p); free(f->lp); free(f->m); free(f->r);
}

int orc_mlp_loss_f32(int num_layers, const int64_t *dims, int act, const float *const *w,
                     const float *const *b, const float *x, const float *onehot, int64_t batch,
                     float *loss, int threads) {
    mlp_fwd f;
    mlp_forward(&f, num_layers, dims, act, w, b, x, onehot, batch, threads);
    *loss = f.loss;
    mlp_free(&f);
    return 0;
}

int orc_mlp_loss_grad_f32(int num_layers, const int64_t *dims, int act, const float *const *w,
                          const float *const *b, const float *x, const float *onehot,
                          int64_t batch, float *loss, float *const *gw, float *const *gb,
                          float *gx, const uint8_t *const *relu_masks, int threads) {
    int L = num_layers;
    int64_t B = batch;
    mlp_fwd f;
    mlp_forward(&f, L, dims, act, w, b, x, onehot, B, threads);
    *loss = f.loss;
    int64_t C = f.C, n = B * C;

    /* L = mu * [-1]: MUL VJP (Grad.java:345) with seed ones([1]) */
    float g_mu = 1.0f * -1.0f;
    /* MEAN VJP (Grad.java:354-358): g / (float) n, broadcast to [B] */
    float g_r_val = g_mu / (float)B;
    /* SUM_AXIS VJP (Grad.java:360-363): broadcast over the class axis;
     * MUL VJP (Grad.java:345): g_lp = g_m * t; LOG VJP (Grad.java:371): g_p = g_lp / p */
    float *g_p = fbuf(n);
    for (int64_t i = 0; i < n; i++) {
        float g_lp = g_r_val * onehot[i];
        g_p[i] = g_lp / f.p[i];
    }
    /* DIV VJP (Grad.java:346-353) for p = e / s */
    float *g_e = fbuf(n);
    float *g_s = fbuf(B);
    for (int64_t i = 0; i < B; i++) g_s[i] = 0.0f;
    for (int64_t i = 0; i < B; i++)
        for (int64_t j = 0; j < C; j++) {
            int64_t k = i * C + j;
            float s = f.s[i];
            g_e[k] = g_p[k] / s;
            float gb_ = g_p[k] * f.e[k];
            gb_ = gb_ / s;
            gb_ = gb_ / s;
            gb_ = gb_ * -1.0f;
            g_s[i] += gb_; /* broadcastLike sum-down, flat order (Grad.java:577-579) */
        }
    /* SUM_AXIS(e, keepDims) VJP merged into g_e by add (Grad.java:157, 180) */
    for (int64_t i = 0; i < B; i++)
        for (int64_t j = 0; j < C; j++) g_e[i * C + j] = g_e[i * C + j] + g_s[i];
    /* EXP VJP (Grad.java:370): g * exp(z) with exp recomputed */
    float *g_z = fbuf(n);
    {
        float *ez = fbuf(n);
        orc_unary_f32(ORC_EXP, f.z[L - 1], n, ez);
        for (int64_t i = 0; i < n; i++) g_z[i] = g_e[i] * ez[i];
        free(ez);
    }
    free(g_p); free(g_e); free(g_s);

    for (int l = L - 1; l >= 0; l--) {
        int64_t din = dims[l], dout = dims[l + 1];
        /* ADD VJP with bias broadcast: column sum-down in flat order (Grad.java:343, 577-579) */
        for (int64_t j = 0; j < dout; j++) gb[l][j] = 0.0f;
        for (int64_t i = 0; i < B; i++)
            for (int64_t j = 0; j < dout; j++) gb[l][j] += g_z[i * dout + j];
        /* DOT VJP (Grad.java:385-390): dW = transpose(a) . g, dA = g . transpose(W) */
        float *aT = fbuf(din * B);
        orc_transpose_f32(f.a[l], B, din, aT);
        orc_dot_f32(aT, g_z, gw[l], din, B, dout, 0, din, threads);
        free(aT);
        if (l == 0 && !gx) break; /* x is a constant here: its cotangent is never read */
        float *wT = fbuf(dout * din);
        orc_transpose_f32(w[l], din, dout, wT);
        float *g_a = l == 0 ? gx : fbuf(B * din);
        orc_dot_f32(g_z, wT, g_a, B, dout, din, 0, B, threads);
        free(wT);
        if (l == 0) break;
        free(g_z);
        g_z = fbuf(B * din);
        const float *zin = f.z[l - 1];
        if (act == 0) {
            /* TANH VJP (Grad.java:374-378): g * (1 - t*t), t recomputed */
            for (int64_t i = 0; i < B * din; i++) {
                float t = (float)tanh((double)zin[i]);
                float tt = t * t;
                float one_m = 1.0f - tt;
                g_z[i] = g_a[i] * one_m;
            }
        } else if (relu_masks && relu_masks[l - 1]) {
            /* relu'(z) from a caller-supplied sign pattern of z (see header) */
            const uint8_t *mk = relu_masks[l - 1];
            for (int64_t i = 0; i < B * din; i++) g_z[i] = mk[i] ? g_a[i] : 0.0f;
        } else {
            orc_relu_grad_f32(g_a, zin, B * din, g_z); /* Grad.java:585-598 */
        }
        free(g_a);
    }
    free(g_z);
    mlp_free(&f);
    return 0;
}

/* ------------------------------------------------------------------ */
/* Elementwise sweep: z = where(x.gt(0), tanh(x)*sigmoid(y),             */
/* relu(y).clip(-1, 1)); z.sum(-1, true); z.argmax(-1).                  */
/* where = c*x + (1-c)*y with c = BOOL->FLOAT32 (api/Numpy.java:39-44);   */
/* clip = max(lo).min(hi) (core/NDArray.java:82).                         */
/* ------------------------------------------------------------------ */
void orc_sweep_f32(const float *x, const float *y, int64_t rows, int64_t cols, float *z,
                   float *row_sum, int32_t *row_argmax) {
    for (int64_t i = 0; i < rows; i++) {
        float total = 0.0f;
        int32_t best_idx = 0;
        float best = 0.0f;
        for (int64_t j = 0; j < cols; j++) {
            int64_t k = i * cols + j;
            float xv = x[k], yv = y[k];
            float c = ((double)xv > 0.0) ? 1.0f : 0.0f;
            float t = (float)tanh((double)xv);
            float s = (float)(1.0 / (1.0 + exp(-(double)yv)));
            float ts = t * s;
            float r = (float)java_max(0.0, (double)yv);
            float cl = (float)java_max((double)r, -1.0);
            cl = (float)java_min((double)cl, 1.0);
            float inv = 1.0f - c;
            float zv = c * ts + inv * cl;
            if (z) z[k] = zv;
            total += zv;
            if (j == 0 || zv > best) { /* ConcreteNDArray.java:606-613 */
                best = zv;
                best_idx = (int32_t)j;
            }
        }
        row_sum[i] = total;
        row_argmax[i] = best_idx;
    }
}

#define ORC_PI 3.14159265358979323846 /* the double nearest pi, Java's Math.PI */

/* ---- Fft (api/Fft.java) ------------------------------------------------------------
 * The reference's iterative radix-2 Cooley-Tukey, restated: a bit-reversal
 * permutation, then stages of butterflies whose twiddle advances by the
 * rotation w <- w * w_step, w_step = (cos, sin)(sign * 2 pi / len)
 * (Fft.java:292-331 in FP64).  The FP32 form (Fft.java:333-371) keeps the
 * twiddle and each butterfly's product in double and rounds every result to
 * float; the inverse then multiplies by the float 1/n.  3-D transforms run
 * the line transform along axis 2, then 1, then 0 (Fft.java:571-612), a
 * line at a time. */
static void fft_line_f64(double *re, double *im, int64_t n, int inverse) {
    for (int64_t i = 1, j = 0; i < n; i++) {
        int64_t bit = n >> 1;
        for (; (j & bit) != 0; bit >>= 1) j ^= bit;
        j ^= bit;
        if (i < j) {
            double t = re[i]; re[i] = re[j]; re[j] = t;
            t = im[i]; im[i] = im[j]; im[j] = t;
        }
    }
    const double sign = inverse ? 1.0 : -1.0;
    for (int64_t len = 2; len <= n; len <<= 1) {
        const double theta = sign * 2.0 * ORC_PI / (double)len;
        const double sr = cos(theta), si = sin(theta);
        const int64_t half = len >> 1;
        for (int64_t i = 0; i < n; i += len) {
            double wr = 1.0, wi = 0.0;
            for (int64_t k = 0; k < half; k++) {
                const int64_t a = i + k, b = a + half;
                const double tr = wr * re[b] - wi * im[b];
                const double ti = wr * im[b] + wi * re[b];
                re[b] = re[a] - tr;
                im[b] = im[a] - ti;
                re[a] += tr;
                im[a] += ti;
                const double nr = wr * sr - wi * si, ni = wr * si + wi * sr;
                wr = nr;
                wi = ni;
            }
        }
    }
    if (inverse) {
        const double inv = 1.0 / (double)n;
        for (int64_t i = 0; i < n; i++) { re[i] *= inv; im[i] *= inv; }
    }
}

static void fft_line_f32(float *re, float *im, int64_t n, int inverse) {
    for (int64_t i = 1, j = 0; i < n; i++) {
        int64_t bit = n >> 1;
        for (; (j & bit) != 0; bit >>= 1) j ^= bit;
        j ^= bit;
        if (i < j) {
            float t = re[i]; re[i] = re[j]; re[j] = t;
            t = im[i]; im[i] = im[j]; im[j] = t;
        }
    }
    const double sign = inverse ? 1.0 : -1.0;
    for (int64_t len = 2; len <= n; len <<= 1) {
        const double theta = sign * 2.0 * ORC_PI / (double)len;
        const double sr = cos(theta), si = sin(theta);
        const int64_t half = len >> 1;
        for (int64_t i = 0; i < n; i += len) {
            double wr = 1.0, wi = 0.0;
            for (int64_t k = 0; k < half; k++) {
                const int64_t a = i + k, b = a + half;
                const double tr = wr * (double)re[b] - wi * (double)im[b];
                const double ti = wr * (double)im[b] + wi * (double)re[b];
                re[b] = (float)((double)re[a] - tr);
                im[b] = (float)((double)im[a] - ti);
                re[a] = (float)((double)re[a] + tr);
                im[a] = (float)((double)im[a] + ti);
                const double nr = wr * sr - wi * si, ni = wr * si + wi * sr;
                wr = nr;
                wi = ni;
            }
        }
    }
    if (inverse) {
        const float inv = 1.0f / (float)n;
        for (int64_t i = 0; i < n; i++) { re[i] *= inv; im[i] *= inv; }
    }
}

/* One axis of a [n0, n1, n2] grid: gather each line, transform, scatter. */
static void fft_axis(int dtype, void *re, void *im, const int64_t *d, int axis, int inverse) {
    const int64_t n = d[axis];
    const int64_t stride = axis == 0 ? d[1] * d[2] : axis == 1 ? d[2] : 1;
    const int64_t lines = d[0] * d[1] * d[2] / n;
    const size_t es = dtype == ORC_F64 ? sizeof(double) : sizeof(float);
    char *tr = malloc(es * (size_t)n), *ti = malloc(es * (size_t)n);
    for (int64_t l = 0; l < lines; l++) {
        /* line l: the base index with the transformed axis at 0 */
        int64_t base;
        if (axis == 0) base = l;                                       /* (j, k) -> j * n2 + k */
        else if (axis == 1) base = (l / d[2]) * d[1] * d[2] + l % d[2]; /* (i, k) */
        else base = l * d[2];                                          /* (i, j) */
        for (int64_t t = 0; t < n; t++) {
            memcpy(tr + es * t, (char *)re + es * (base + t * stride), es);
            memcpy(ti + es * t, (char *)im + es * (base + t * stride), es);
        }
        if (dtype == ORC_F64) fft_line_f64((double *)tr, (double *)ti, n, inverse);
        else fft_line_f32((float *)tr, (float *)ti, n, inverse);
        for (int64_t t = 0; t < n; t++) {
            memcpy((char *)re + es * (base + t * stride), tr + es * t, es);
            memcpy((char *)im + es * (base + t * stride), ti + es * t, es);
        }
    }
    free(tr);
    free(ti);
}

static void dims3(int rank, const int64_t *dims, int64_t *d) {
    if (rank == 1) { d[0] = 1; d[1] = 1; d[2] = dims[0]; }
    else { d[0] = dims[0]; d[1] = dims[1]; d[2] = dims[2]; }
}

void orc_fft(int dtype, int rank, const int64_t *dims, void *re, void *im, int inverse) {
    int64_t d[3];
    dims3(rank, dims, d);
    for (int axis = 2; axis >= 0; axis--)
        if (rank == 3 || axis == 2) fft_axis(dtype, re, im, d, axis, inverse);
}

/* rfft / rfft3 (Fft.java:93-127, 423-492): each row of the last axis as the
 * complex transform of (x, 0) cut to n/2 + 1 bins, then axes 1 and 0 of the
 * half spectrum. */
void orc_rfft(int dtype, int rank, const int64_t *dims, const void *x, void *ore, void *oim) {
    int64_t d[3];
    dims3(rank, dims, d);
    const int64_t n = d[2], h = n / 2 + 1, rows = d[0] * d[1];
    const size_t es = dtype == ORC_F64 ? sizeof(double) : sizeof(float);
    char *tr = calloc((size_t)n, es), *ti = calloc((size_t)n, es);
    for (int64_t r = 0; r < rows; r++) {
        memcpy(tr, (const char *)x + es * r * n, es * (size_t)n);
        memset(ti, 0, es * (size_t)n);
        if (dtype == ORC_F64) fft_line_f64((double *)tr, (double *)ti, n, 0);
        else fft_line_f32((float *)tr, (float *)ti, n, 0);
        memcpy((char *)ore + es * r * h, tr, es * (size_t)h);
        memcpy((char *)oim + es * r * h, ti, es * (size_t)h);
    }
    free(tr);
    free(ti);
    if (rank == 3) {
        const int64_t dh[3] = {d[0], d[1], h};
        fft_axis(dtype, ore, oim, dh, 1, 0);
        fft_axis(dtype, ore, oim, dh, 0, 0);
    }
}

/* irfft / irfft3 (Fft.java:130-186, 494-568): inverse transforms of axes 0
 * and 1 of the half spectrum, then per row the Hermitian mirror
 * X[n-k] = conj(X[k]) (k = 1 .. h-2), the inverse transform and its real part. */
void orc_irfft(int dtype, int rank, const int64_t *dims, const void *re, const void *im, void *out) {
    int64_t d[3];
    dims3(rank, dims, d);
    const int64_t n = d[2], h = n / 2 + 1, rows = d[0] * d[1];
    const size_t es = dtype == ORC_F64 ? sizeof(double) : sizeof(float);
    char *wr = malloc(es * (size_t)(rows * h)), *wi = malloc(es * (size_t)(rows * h));
    memcpy(wr, re, es * (size_t)(rows * h));
    memcpy(wi, im, es * (size_t)(rows * h));
    if (rank == 3) {
        const int64_t dh[3] = {d[0], d[1], h};
        fft_axis(dtype, wr, wi, dh, 0, 1);
        fft_axis(dtype, wr, wi, dh, 1, 1);
    }
    char *tr = calloc((size_t)n, es), *ti = calloc((size_t)n, es);
    for (int64_t r = 0; r < rows; r++) {
        memset(tr, 0, es * (size_t)n);
        memset(ti, 0, es * (size_t)n);
        memcpy(tr, wr + es * r * h, es * (size_t)h);
        memcpy(ti, wi + es * r * h, es * (size_t)h);
        if (dtype == ORC_F64) {
            double *a = (double *)tr, *b = (double *)ti;
            for (int64_t k = 1; k < h - 1; k++) { a[n - k] = a[k]; b[n - k] = -b[k]; }
            fft_line_f64(a, b, n, 1);
        } else {
            float *a = (float *)tr, *b = (float *)ti;
            for (int64_t k = 1; k < h - 1; k++) { a[n - k] = a[k]; b[n - k] = -b[k]; }
            fft_line_f32(a, b, n, 1);
        }
        memcpy((char *)out + es * r * n, tr, es * (size_t)n);
    }
    free(tr);
    free(ti);
    free(wr);
    free(wi);
}

/* dctI (Fft.java:200-227, 373-398): the real part of the FP64 transform of
 * [x0 .. x_{n-1}, x_{n-2} .. x1], rounded to the input dtype. */
void orc_dct1(int dtype, int64_t n, const void *x, void *out) {
    if (n == 1) {
        memcpy(out, x, dtype == ORC_F64 ? sizeof(double) : sizeof(float));
        return;
    }
    const int64_t m = 2 * (n - 1);
    double *re = calloc((size_t)m, sizeof(double)), *im = calloc((size_t)m, sizeof(double));
    for (int64_t k = 0; k < m; k++) {
        const int64_t src = k < n ? k : m - k;
        re[k] = dtype == ORC_F64 ? ((const double *)x)[src] : (double)((const float *)x)[src];
    }
    fft_line_f64(re, im, m, 0);
    for (int64_t k = 0; k < n; k++) {
        if (dtype == ORC_F64) ((double *)out)[k] = re[k];
        else ((float *)out)[k] = (float)re[k];
    }
    free(re);
    free(im);
}

/* ------------------------------------------------------------------ */
/* api/Linalg.java: LU with partial pivoting, its solves and Hager's   */
/* condition estimate, in FP64 on row-major arrays.                    */
/* ------------------------------------------------------------------ */

/* Linalg.luFactorInPlace (Linalg.java:1021-1085).  a (n x n, row-major) is
 * overwritten by the packed Doolittle factors; piv[i] = the row of the
 * original matrix that row i of the factors comes from; norms[0] =
 * max |a_ij|, norms[1] = max_i sum_j |a_ij| of the input.  Returns 0, or
 * ORC_LU_ZERO_PIVOT / ORC_LU_SUBMATRIX with *fail_k = the elimination step
 * and *fail_piv = the pivot magnitude there (the reference's exceptions). */
int orc_lu_factor(double *a, int64_t n, int submatrix_check, int64_t *piv, double *norms, int64_t *fail_k,
                  double *fail_piv) {
    double amax = 0.0, rmax = 0.0;
    for (int64_t i = 0; i < n * n; i++) {
        const double v = fabs(a[i]);
        if (v > amax) amax = v;
    }
    for (int64_t i = 0; i < n; i++) {
        double row = 0.0;
        for (int64_t j = 0; j < n; j++) row += fabs(a[i * n + j]);
        if (row > rmax) rmax = row;
    }
    norms[0] = amax;
    norms[1] = rmax;
    const double tol = submatrix_check ? 1e-14 * amax : 0.0;
    for (int64_t i = 0; i < n; i++) piv[i] = i;
    for (int64_t k = 0; k < n; k++) {
        int64_t best = k;
        double best_abs = fabs(a[k * n + k]);
        for (int64_t i = k + 1; i < n; i++)
            if (fabs(a[i * n + k]) > best_abs) {
                best_abs = fabs(a[i * n + k]);
                best = i;
            }
        if (best_abs == 0.0 || best_abs <= tol) {
            *fail_k = k;
            *fail_piv = best_abs;
            return best_abs == 0.0 ? ORC_LU_ZERO_PIVOT : ORC_LU_SUBMATRIX;
        }
        if (best != k) {
            for (int64_t j = 0; j < n; j++) {
                const double t = a[k * n + j];
                a[k * n + j] = a[best * n + j];
                a[best * n + j] = t;
            }
            const int64_t t = piv[k];
            piv[k] = piv[best];
            piv[best] = t;
        }
        const double inv = 1.0 / a[k * n + k];
        for (int64_t i = k + 1; i < n; i++) {
            const double l = a[i * n + k] * inv;
            a[i * n + k] = l;
            if (l == 0.0) continue;
            for (int64_t j = k + 1; j < n; j++) a[i * n + j] -= l * a[k * n + j];
        }
    }
    return 0;
}

/* LU.substitute (Linalg.java:178-197): x = A^-1 b. */
void orc_lu_solve(const double *lu, const int64_t *piv, int64_t n, const double *b, double *x) {
    double *y = malloc(sizeof(double) * (size_t)n);
    for (int64_t i = 0; i < n; i++) {
        double acc = b[piv[i]];
        for (int64_t j = 0; j < i; j++) acc -= lu[i * n + j] * y[j];
        y[i] = acc;
    }
    for (int64_t i = n - 1; i >= 0; i--) {
        double acc = y[i];
        for (int64_t j = i + 1; j < n; j++) acc -= lu[i * n + j] * x[j];
        x[i] = acc / lu[i * n + i];
    }
    free(y);
}

/* LU.solveTranspose (Linalg.java:206-232): x = A^-T b = P^-1 L^-T U^-T b. */
void orc_lu_solve_t(const double *lu, const int64_t *piv, int64_t n, const double *b, double *x) {
    double *y = malloc(sizeof(double) * (size_t)n), *w = malloc(sizeof(double) * (size_t)n);
    for (int64_t i = 0; i < n; i++) {
        double acc = b[i];
        for (int64_t j = 0; j < i; j++) acc -= lu[j * n + i] * y[j];
        y[i] = acc / lu[i * n + i];
    }
    for (int64_t i = n - 1; i >= 0; i--) {
        double acc = y[i];
        for (int64_t j = i + 1; j < n; j++) acc -= lu[j * n + i] * w[j];
        w[i] = acc;
    }
    for (int64_t i = 0; i < n; i++) x[piv[i]] = w[i];
    free(y);
    free(w);
}

/* Linalg.reciprocalConditionNumber + hagerNormInvInf (Linalg.java:1102-1153). */
double orc_lu_rcond(const double *lu, const int64_t *piv, int64_t n, double inf_norm) {
    if (inf_norm == 0.0) return 0.0;
    double *x = malloc(sizeof(double) * (size_t)n), *y = malloc(sizeof(double) * (size_t)n);
    double *xi = malloc(sizeof(double) * (size_t)n), *z = malloc(sizeof(double) * (size_t)n);
    for (int64_t i = 0; i < n; i++) x[i] = 1.0 / (double)n;
    double estimate = 0.0;
    for (int iter = 0; iter < 5; iter++) {
        orc_lu_solve_t(lu, piv, n, x, y);
        double y1 = 0.0;
        for (int64_t i = 0; i < n; i++) y1 += fabs(y[i]);
        if (iter > 0 && y1 <= estimate) break;
        estimate = y1;
        for (int64_t i = 0; i < n; i++) xi[i] = y[i] >= 0.0 ? 1.0 : -1.0;
        orc_lu_solve(lu, piv, n, xi, z);
        int64_t jstar = 0;
        double zmax = fabs(z[0]), ztx = 0.0;
        for (int64_t i = 1; i < n; i++)
            if (fabs(z[i]) > zmax) {
                zmax = fabs(z[i]);
                jstar = i;
            }
        for (int64_t i = 0; i < n; i++) ztx += z[i] * x[i];
        if (zmax <= fabs(ztx)) break;
        for (int64_t i = 0; i < n; i++) x[i] = 0.0;
        x[jstar] = 1.0;
    }
    free(x);
    free(y);
    free(xi);
    free(z);
    return estimate == 0.0 ? INFINITY : 1.0 / (inf_norm * estimate);
}

/* java.lang.Math.max(double, double): NaN if either argument is NaN. */
static double jmax(double a, double b) {
    if (a != a) return a;
    if (b != b) return b;
    return a >= b ? a : b;
}

#define RM(M, ld, i, j) (M)[(int64_t)(i) * (ld) + (j)]

/* Linalg.reduceToHessenberg (Linalg.java:815-847): Householder similarity
 * transforms zero column k below the subdiagonal, k = 0..n-3. */
static void hessenberg(double *H, int64_t n) {
    double *u = calloc((size_t)n + 1, sizeof(double));
    for (int64_t k = 0; k + 2 < n; k++) {
        double scale = 0.0;
        for (int64_t i = k + 1; i < n; i++) scale = jmax(scale, fabs(RM(H, n, i, k)));
        if (scale == 0.0) continue;
        double h = 0.0;
        for (int64_t i = k + 1; i < n; i++) {
            u[i] = RM(H, n, i, k) / scale;
            h += u[i] * u[i];
        }
        const double f = u[k + 1];
        const double g = f >= 0 ? -sqrt(h) : sqrt(h);
        h -= f * g;
        u[k + 1] = f - g;
        for (int64_t j = k; j < n; j++) { /* from the left, rows k+1.. */
            double acc = 0.0;
            for (int64_t i = k + 1; i < n; i++) acc += u[i] * RM(H, n, i, j);
            acc /= h;
            for (int64_t i = k + 1; i < n; i++) RM(H, n, i, j) -= acc * u[i];
        }
        for (int64_t i = 0; i < n; i++) { /* from the right, columns k+1.. */
            double acc = 0.0;
            for (int64_t j = k + 1; j < n; j++) acc += u[j] * RM(H, n, i, j);
            acc /= h;
            for (int64_t j = k + 1; j < n; j++) RM(H, n, i, j) -= acc * u[j];
        }
        RM(H, n, k + 1, k) = scale * g;
        for (int64_t i = k + 2; i < n; i++) RM(H, n, i, k) = 0.0;
    }
    free(u);
}

/* Linalg.francisQR (Linalg.java:856-1005): the implicit double-shift QR
 * iteration with deflation on an upper-Hessenberg matrix (EISPACK hqr's
 * steps), eigenvalues in the order they deflate.  Returns 1 if an
 * eigenvalue needs more than 300 n iterations (the reference throws). */
static int francis_qr(double *H, int64_t nn, double *wr, double *wi) {
    const double eps = ldexp(1.0, -52);
    int64_t n = nn - 1, iter = 0;
    double exshift = 0.0, p = 0, q = 0, r = 0, s = 0, z = 0, w, x, y;
    double norm = 0.0;
    for (int64_t i = 0; i < nn; i++)
        for (int64_t j = i > 0 ? i - 1 : 0; j < nn; j++) norm += fabs(RM(H, nn, i, j));
    while (n >= 0) {
        int64_t l = n;
        for (; l > 0; l--) { /* a negligible subdiagonal entry splits the matrix */
            s = fabs(RM(H, nn, l - 1, l - 1)) + fabs(RM(H, nn, l, l));
            if (s == 0.0) s = norm;
            if (fabs(RM(H, nn, l, l - 1)) < eps * s) break;
        }
        if (l == n) { /* a 1 x 1 block: one real eigenvalue */
            RM(H, nn, n, n) += exshift;
            wr[n] = RM(H, nn, n, n);
            wi[n] = 0.0;
            n--;
            iter = 0;
            continue;
        }
        if (l == n - 1) { /* a 2 x 2 block: a real pair or a conjugate pair */
            w = RM(H, nn, n, n - 1) * RM(H, nn, n - 1, n);
            p = (RM(H, nn, n - 1, n - 1) - RM(H, nn, n, n)) / 2.0;
            q = p * p + w;
            z = sqrt(fabs(q));
            RM(H, nn, n, n) += exshift;
            RM(H, nn, n - 1, n - 1) += exshift;
            x = RM(H, nn, n, n);
            if (q >= 0) {
                z = p >= 0 ? p + z : p - z;
                wr[n - 1] = x + z;
                wr[n] = z != 0.0 ? x - w / z : wr[n - 1];
                wi[n - 1] = wi[n] = 0.0;
            } else {
                wr[n - 1] = wr[n] = x + p;
                wi[n - 1] = z;
                wi[n] = -z;
            }
            n -= 2;
            iter = 0;
            continue;
        }
        /* the shift: the trailing 2 x 2 block, or the exceptional one at
         * iterations 10 and 20 */
        x = RM(H, nn, n, n);
        y = RM(H, nn, n - 1, n - 1);
        w = RM(H, nn, n, n - 1) * RM(H, nn, n - 1, n);
        if (iter == 10 || iter == 20) {
            exshift += x;
            for (int64_t i = 0; i <= n; i++) RM(H, nn, i, i) -= x;
            s = fabs(RM(H, nn, n, n - 1)) + fabs(RM(H, nn, n - 1, n - 2));
            x = y = 0.75 * s;
            w = -0.4375 * s * s;
        }
        if (++iter > 300 * nn) return 1;
        /* where two consecutive subdiagonal entries are small enough to start the sweep */
        int64_t m = n - 2;
        for (;; m--) {
            z = RM(H, nn, m, m);
            r = x - z;
            s = y - z;
            p = (r * s - w) / RM(H, nn, m + 1, m) + RM(H, nn, m, m + 1);
            q = RM(H, nn, m + 1, m + 1) - z - r - s;
            r = RM(H, nn, m + 2, m + 1);
            s = fabs(p) + fabs(q) + fabs(r);
            p /= s;
            q /= s;
            r /= s;
            if (m == l) break;
            if (fabs(RM(H, nn, m, m - 1)) * (fabs(q) + fabs(r)) <
                eps * fabs(p) * (fabs(RM(H, nn, m - 1, m - 1)) + fabs(z) + fabs(RM(H, nn, m + 1, m + 1))))
                break;
        }
        for (int64_t i = m + 2; i <= n; i++) {
            RM(H, nn, i, i - 2) = 0.0;
            if (i > m + 2) RM(H, nn, i, i - 3) = 0.0;
        }
        for (int64_t k = m; k <= n - 1; k++) { /* the double-shift bulge chase */
            const int notlast = k != n - 1;
            if (k != m) {
                p = RM(H, nn, k, k - 1);
                q = RM(H, nn, k + 1, k - 1);
                r = notlast ? RM(H, nn, k + 2, k - 1) : 0.0;
                x = fabs(p) + fabs(q) + fabs(r);
                if (x == 0.0) continue;
                p /= x;
                q /= x;
                r /= x;
            }
            s = sqrt(p * p + q * q + r * r);
            if (p < 0) s = -s;
            if (s == 0.0) continue;
            if (k != m) RM(H, nn, k, k - 1) = -s * x;
            else if (l != m) RM(H, nn, k, k - 1) = -RM(H, nn, k, k - 1);
            p += s;
            x = p / s;
            y = q / s;
            z = r / s;
            q /= p;
            r /= p;
            for (int64_t j = k; j < nn; j++) { /* rows k..k+2 */
                p = RM(H, nn, k, j) + q * RM(H, nn, k + 1, j);
                if (notlast) {
                    p += r * RM(H, nn, k + 2, j);
                    RM(H, nn, k + 2, j) -= p * z;
                }
                RM(H, nn, k, j) -= p * x;
                RM(H, nn, k + 1, j) -= p * y;
            }
            const int64_t imax = n < k + 3 ? n : k + 3;
            for (int64_t i = 0; i <= imax; i++) { /* columns k..k+2 */
                p = x * RM(H, nn, i, k) + y * RM(H, nn, i, k + 1);
                if (notlast) {
                    p += z * RM(H, nn, i, k + 2);
                    RM(H, nn, i, k + 2) -= p * r;
                }
                RM(H, nn, i, k) -= p;
                RM(H, nn, i, k + 1) -= p * q;
            }
        }
    }
    return 0;
}

/* Linalg.eig(A) (Linalg.java:768-800): FP64 for both dtypes; 0 or 1 (no convergence). */
int orc_eig(int dtype, int64_t n, const void *a, void *wr, void *wi) {
    double *H = malloc(sizeof(double) * (size_t)(n * n + 1));
    double *r = malloc(sizeof(double) * (size_t)(n + 1)), *im = malloc(sizeof(double) * (size_t)(n + 1));
    for (int64_t i = 0; i < n * n; i++)
        H[i] = dtype == ORC_F64 ? ((const double *)a)[i] : (double)((const float *)a)[i];
    hessenberg(H, n);
    const int rc = francis_qr(H, n, r, im);
    for (int64_t i = 0; i < n; i++) {
        if (dtype == ORC_F64) {
            ((double *)wr)[i] = r[i];
            ((double *)wi)[i] = im[i];
        } else {
            ((float *)wr)[i] = (float)r[i];
            ((float *)wi)[i] = (float)im[i];
        }
    }
    free(H);
    free(r);
    free(im);
    return rc;
}

/* Linalg.golubKahanBidiagonalize (Linalg.java:485-583): Householder
 * reflections from both sides bring A (m x n, m >= n) to upper-bidiagonal
 * form (diagonal s, superdiagonal e), and U (m x n), V (n x n) accumulate
 * them.  The published Golub-Reinsch / LINPACK dsvdc first phase. */
static void bidiagonalize(double *A, double *U, double *V, double *s, double *e, int64_t m, int64_t n) {
    const int64_t nct = m - 1 < n ? m - 1 : n;
    const int64_t nrt0 = n - 2 < m ? n - 2 : m, nrt = nrt0 > 0 ? nrt0 : 0;
    double *work = malloc(sizeof(double) * (size_t)(m + 1));
    for (int64_t k = 0; k < (nct > nrt ? nct : nrt); k++) {
        if (k < nct) { /* the column reflector below the diagonal */
            double nrm = 0.0;
            for (int64_t i = k; i < m; i++) nrm = hypot(nrm, RM(A, n, i, k));
            if (nrm != 0.0) {
                if (RM(A, n, k, k) < 0.0) nrm = -nrm;
                for (int64_t i = k; i < m; i++) RM(A, n, i, k) /= nrm;
                RM(A, n, k, k) += 1.0;
            }
            s[k] = -nrm;
        }
        for (int64_t j = k + 1; j < n; j++) {
            if (k < nct && s[k] != 0.0) {
                double t = 0.0;
                for (int64_t i = k; i < m; i++) t += RM(A, n, i, k) * RM(A, n, i, j);
                t = -t / RM(A, n, k, k);
                for (int64_t i = k; i < m; i++) RM(A, n, i, j) += t * RM(A, n, i, k);
            }
            e[j] = RM(A, n, k, j);
        }
        if (k < nrt) { /* the row reflector right of the superdiagonal */
            double nrm = 0.0;
            for (int64_t i = k + 1; i < n; i++) nrm = hypot(nrm, e[i]);
            if (nrm != 0.0) {
                if (e[k + 1] < 0.0) nrm = -nrm;
                for (int64_t i = k + 1; i < n; i++) e[i] /= nrm;
                e[k + 1] += 1.0;
            }
            e[k] = -nrm;
            if (k + 1 < m && e[k] != 0.0) {
                for (int64_t i = 0; i < m; i++) work[i] = 0.0;
                for (int64_t j = k + 1; j < n; j++)
                    for (int64_t i = k + 1; i < m; i++) work[i] += e[j] * RM(A, n, i, j);
                for (int64_t j = k + 1; j < n; j++) {
                    const double t = -e[j] / e[k + 1];
                    for (int64_t i = k + 1; i < m; i++) RM(A, n, i, j) += t * work[i];
                }
            }
            for (int64_t i = k + 1; i < n; i++) RM(V, n, i, k) = e[i];
        }
    }
    const int64_t p = n < m + 1 ? n : m + 1;
    if (nct < n) s[nct] = RM(A, n, nct, nct);
    if (m < p) s[p - 1] = 0.0;
    if (nrt + 1 < p) e[nrt] = RM(A, n, nrt, p - 1);
    e[p - 1] = 0.0;
    for (int64_t j = nct; j < n; j++) { /* U: the left reflectors applied to the identity */
        for (int64_t i = 0; i < m; i++) RM(U, n, i, j) = 0.0;
        RM(U, n, j, j) = 1.0;
    }
    for (int64_t k = nct - 1; k >= 0; k--) {
        if (s[k] != 0.0) {
            for (int64_t j = k + 1; j < n; j++) {
                double t = 0.0;
                for (int64_t i = k; i < m; i++) t += RM(A, n, i, k) * RM(U, n, i, j);
                t = -t / RM(A, n, k, k);
                for (int64_t i = k; i < m; i++) RM(U, n, i, j) += t * RM(A, n, i, k);
            }
            for (int64_t i = k; i < m; i++) RM(U, n, i, k) = -RM(A, n, i, k);
            RM(U, n, k, k) = 1.0 + RM(U, n, k, k);
            for (int64_t i = 0; i < k - 1; i++) RM(U, n, i, k) = 0.0;
        } else {
            for (int64_t i = 0; i < m; i++) RM(U, n, i, k) = 0.0;
            RM(U, n, k, k) = 1.0;
        }
    }
    for (int64_t k = n - 1; k >= 0; k--) { /* V: the right reflectors */
        if (k < nrt && e[k] != 0.0) {
            for (int64_t j = k + 1; j < n; j++) {
                double t = 0.0;
                for (int64_t i = k + 1; i < n; i++) t += RM(V, n, i, k) * RM(V, n, i, j);
                t = -t / RM(V, n, k + 1, k);
                for (int64_t i = k + 1; i < n; i++) RM(V, n, i, j) += t * RM(V, n, i, k);
            }
        }
        for (int64_t i = 0; i < n; i++) RM(V, n, i, k) = 0.0;
        RM(V, n, k, k) = 1.0;
    }
    free(work);
}

/* Rotate columns (j, k) of M (rows x ld): (Mj, Mk) <- (c Mj + s Mk, -s Mj + c Mk). */
static void rotate_cols(double *M, int64_t rows, int64_t ld, int64_t j, int64_t k, double c, double s) {
    for (int64_t i = 0; i < rows; i++) {
        const double x = c * RM(M, ld, i, j) + s * RM(M, ld, i, k);
        RM(M, ld, i, k) = -s * RM(M, ld, i, j) + c * RM(M, ld, i, k);
        RM(M, ld, i, j) = x;
    }
}

static void swap_cols(double *M, int64_t rows, int64_t ld, int64_t j, int64_t k) {
    for (int64_t i = 0; i < rows; i++) {
        const double t = RM(M, ld, i, j);
        RM(M, ld, i, j) = RM(M, ld, i, k);
        RM(M, ld, i, k) = t;
    }
}

/* Linalg.golubReinschDiagonalize (Linalg.java:591-749): implicit-shift QR
 * sweeps on the bidiagonal, the four cases of the published algorithm
 * (negligible s[p-1]; a split at a negligible s[k]; a QR step; a converged
 * value, made non-negative and moved into descending order).  Returns 1
 * after more than 500 QR steps on one value (the reference throws). */
static int golub_reinsch(double *U, double *V, double *s, double *e, int64_t m, int64_t n) {
    int64_t p = n < m + 1 ? n : m + 1;
    const double eps = ldexp(1.0, -52), tiny = ldexp(1.0, -966);
    int iter = 0;
    while (p > 0) {
        int64_t k, kase;
        for (k = p - 2; k >= 0; k--) {
            const double thresh = tiny + eps * (fabs(s[k]) + fabs(s[k + 1]));
            if (fabs(e[k]) <= thresh || e[k] != e[k]) {
                e[k] = 0.0;
                break;
            }
        }
        if (k == p - 2) {
            kase = 4;
        } else {
            int64_t ks;
            for (ks = p - 1; ks > k; ks--) {
                const double t = (ks != p ? fabs(e[ks]) : 0.0) + (ks != k + 1 ? fabs(e[ks - 1]) : 0.0);
                if (fabs(s[ks]) <= tiny + eps * t) {
                    s[ks] = 0.0;
                    break;
                }
            }
            if (ks == k) kase = 3;
            else if (ks == p - 1) kase = 1;
            else {
                kase = 2;
                k = ks;
            }
        }
        k++;
        if (kase == 1) { /* deflate the negligible s[p-1] */
            double f = e[p - 2];
            e[p - 2] = 0.0;
            for (int64_t j = p - 2; j >= k; j--) {
                const double t = hypot(s[j], f), cs = s[j] / t, sn = f / t;
                s[j] = t;
                if (j != k) {
                    f = -sn * e[j - 1];
                    e[j - 1] = cs * e[j - 1];
                }
                rotate_cols(V, n, n, j, p - 1, cs, sn);
            }
        } else if (kase == 2) { /* split at the negligible s[k-1] */
            double f = e[k - 1];
            e[k - 1] = 0.0;
            for (int64_t j = k; j < p; j++) {
                const double t = hypot(s[j], f), cs = s[j] / t, sn = f / t;
                s[j] = t;
                f = -sn * e[j];
                e[j] = cs * e[j];
                rotate_cols(U, m, n, j, k - 1, cs, sn);
            }
        } else if (kase == 3) { /* one implicit-shift QR step on [k, p-1] */
            const double scale = jmax(jmax(jmax(jmax(fabs(s[p - 1]), fabs(s[p - 2])), fabs(e[p - 2])), fabs(s[k])),
                                      fabs(e[k]));
            const double sp = s[p - 1] / scale, spm1 = s[p - 2] / scale, epm1 = e[p - 2] / scale;
            const double sk = s[k] / scale, ek = e[k] / scale;
            const double b = ((spm1 + sp) * (spm1 - sp) + epm1 * epm1) / 2.0;
            const double c = (sp * epm1) * (sp * epm1);
            double shift = 0.0;
            if (b != 0.0 || c != 0.0) {
                shift = sqrt(b * b + c);
                if (b < 0.0) shift = -shift;
                shift = c / (b + shift);
            }
            double f = (sk + sp) * (sk - sp) + shift, g = sk * ek;
            for (int64_t j = k; j < p - 1; j++) {
                double t = hypot(f, g), cs = f / t, sn = g / t;
                if (j != k) e[j - 1] = t;
                f = cs * s[j] + sn * e[j];
                e[j] = cs * e[j] - sn * s[j];
                g = sn * s[j + 1];
                s[j + 1] = cs * s[j + 1];
                rotate_cols(V, n, n, j, j + 1, cs, sn);
                t = hypot(f, g);
                cs = f / t;
                sn = g / t;
                s[j] = t;
                f = cs * e[j] + sn * s[j + 1];
                s[j + 1] = -sn * e[j] + cs * s[j + 1];
                g = sn * e[j + 1];
                e[j + 1] = cs * e[j + 1];
                if (j < m - 1) rotate_cols(U, m, n, j, j + 1, cs, sn);
            }
            e[p - 2] = f;
            iter++;
        } else { /* s[k] converged */
            if (s[k] <= 0.0) {
                s[k] = -s[k];
                for (int64_t i = 0; i < n; i++) RM(V, n, i, k) = -RM(V, n, i, k);
            }
            for (; k < p - 1 && !(s[k] >= s[k + 1]); k++) {
                const double t = s[k];
                s[k] = s[k + 1];
                s[k + 1] = t;
                if (k < n - 1) swap_cols(V, n, n, k, k + 1);
                if (k < m - 1) swap_cols(U, m, n, k, k + 1);
            }
            iter = 0;
            p--;
        }
        if (iter > 500) return 1;
    }
    return 0;
}

/* Linalg.svd (Linalg.java:411-460): thin SVD of an m x n matrix (m >= n),
 * FP64 outputs u [m, n], s [n] (descending, non-negative), vt [n, n].
 * Returns 0, or 1 if the QR sweeps did not converge. */
int orc_svd(int dtype, int64_t m, int64_t n, const void *a, double *u, double *s, double *vt) {
    double *A = malloc(sizeof(double) * (size_t)(m * n + 1));
    double *V = calloc((size_t)(n * n + 1), sizeof(double)), *e = calloc((size_t)n + 1, sizeof(double));
    for (int64_t i = 0; i < m * n; i++)
        A[i] = dtype == ORC_F64 ? ((const double *)a)[i] : (double)((const float *)a)[i];
    for (int64_t i = 0; i < m * n; i++) u[i] = 0.0;
    for (int64_t i = 0; i < n; i++) s[i] = 0.0;
    bidiagonalize(A, u, V, s, e, m, n);
    const int rc = golub_reinsch(u, V, s, e, m, n);
    for (int64_t k = 0; k < n; k++) /* non-negative values, the sign moved into U */
        if (s[k] < 0.0) {
            s[k] = -s[k];
            for (int64_t i = 0; i < m; i++) RM(u, n, i, k) = -RM(u, n, i, k);
        }
    for (int64_t k = 0; k + 1 < n; k++) { /* descending order */
        int64_t best = k;
        for (int64_t j = k + 1; j < n; j++)
            if (s[j] > s[best]) best = j;
        if (best != k) {
            const double t = s[k];
            s[k] = s[best];
            s[best] = t;
            swap_cols(u, m, n, k, best);
            swap_cols(V, n, n, k, best);
        }
    }
    for (int64_t i = 0; i < n; i++)
        for (int64_t j = 0; j < n; j++) RM(vt, n, i, j) = RM(V, n, j, i);
    free(A);
    free(V);
    free(e);
    return rc;
}
