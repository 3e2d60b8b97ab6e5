/*
 * ref_cpu.h -- CPU oracle for the jax4j FP32 hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the host
 * (pure Java) implementation of marmanis/jax4j, used as the checker for the
 * CUDA library.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg may load it; nothing in the product links or calls it.
 *
 * The reference itself cannot run here (it needs JDK 25 plus the TornadoVM
 * jars), so every function restates a specific Java method, cited by
 * file:line relative to the reference project root, with its loop order and
 * rounding kept:
 *   - float elementwise ops are evaluated in double and narrowed to float
 *     (ConcreteNDArray.java:283), which equals correctly rounded FP32;
 *   - every accumulation (sum, mean, dot, broadcast sum-down, psum) is a
 *     sequential float loop in the reference's index order;
 *   - Math.max/min keep Java's NaN and signed-zero rules;
 *   - casts follow the JLS narrowing rules (NaN -> 0, saturation).
 * The build uses -ffp-contract=off so no multiply-add is fused, as in Java.
 *
 * Parity of the restatement itself is pinned by the known-answer tests of
 * the reference's JUnit suite (transcribed with file:line citations in
 * tests/golden/kats.json).
 */
#ifndef J4C_ORACLE_REF_CPU_H
#define J4C_ORACLE_REF_CPU_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Primitive ordinals (ir/Primitive.java:6-42) and DType ordinals
 * (core/DType.java:7-11); the CUDA library uses the same numbering. */
enum {
    ORC_ADD = 0, ORC_SUB = 1, ORC_MUL = 2, ORC_DIV = 3, ORC_DOT = 4,
    ORC_EXP = 5, ORC_LOG = 6, ORC_SIN = 7, ORC_COS = 8,
    ORC_SUM = 9, ORC_MEAN = 10, ORC_SUM_AXIS = 11, ORC_MEAN_AXIS = 12,
    ORC_TANH = 13, ORC_RELU = 14, ORC_SIGMOID = 15,
    ORC_GT = 19, ORC_GE = 20, ORC_LT = 21, ORC_LE = 22, ORC_EQ = 23, ORC_NE = 24,
    ORC_MAX = 25, ORC_MIN = 26, ORC_ARGMAX = 27, ORC_ARGMIN = 28
};
enum { ORC_F32 = 0, ORC_F64 = 1, ORC_I32 = 2, ORC_I64 = 3, ORC_BOOL = 4 };

/* ---- Random.java ---- */
uint64_t orc_mix64(uint64_t z);
void orc_split(uint64_t state, int num, uint64_t *out);
void orc_uniform(uint64_t state, int64_t n, float lo, float hi, float *out);
void orc_permutation(uint64_t state, int64_t n, int32_t *out);
void orc_normal(uint64_t state, int64_t n, float *out);
void orc_glorot_uniform(uint64_t state, int64_t n, int fan_in, int fan_out, float *out);

/* ---- Shape.java ---- */
int64_t orc_broadcast_index(const int64_t *dims, int rank,
                            const int64_t *out_dims, int out_rank, int64_t flat);

/* ---- ConcreteNDArray.java ---- */
int orc_binary_f32(int prim, const float *a, const int64_t *ad, int ar,
                   const float *b, const int64_t *bd, int br,
                   float *out, const int64_t *od, int orank);
int orc_compare(int prim, int dtype, const void *a, const int64_t *ad, int ar,
                const void *b, const int64_t *bd, int br,
                uint8_t *out, const int64_t *od, int orank);
int orc_unary_f32(int prim, const float *in, int64_t n, float *out);
int orc_cast(int src, int dst, const void *in, int64_t n, void *out);
void orc_reduce_all_f32(int prim, const float *in, int64_t n, float *out);
void orc_reduce_axis_f32(int prim, const float *in, int64_t outer, int64_t axis,
                         int64_t inner, float *out);
void orc_argreduce_f32(int prim, const float *in, int64_t outer, int64_t axis,
                       int64_t inner, int32_t *out);
/* row_begin/row_end restrict the computed rows of C (the rows are
 * independent, so a row range is the exact restriction of the full loop);
 * threads > 1 splits the rows across pthreads like the reference's
 * row-parallel CPU-N benchmark (BackendBenchmark.java:281-291). */
void orc_dot_f32(const float *a, const float *b, float *c, int64_t M, int64_t K,
                 int64_t N, int64_t row_begin, int64_t row_end, int threads);

/* ---- Grad.java host helpers ---- */
void orc_broadcast_like_f32(const float *g, const int64_t *gd, int gr,
                            float *out, const int64_t *td, int tr);
void orc_relu_grad_f32(const float *g, const float *x, int64_t n, float *out);
void orc_axis_broadcast_like_f32(const float *g, const int64_t *dims, int rank,
                                 int axis, float *out);
void orc_transpose_f32(const float *in, int64_t rows, int64_t cols, float *out);
void orc_maxmin_grad_f32(int is_max, const float *g, const int64_t *od, int orank,
                         const float *a, const int64_t *ad, int ar,
                         const float *b, const int64_t *bd, int br,
                         float *ga_full, float *gb_full);

/* ---- SharedCollective.java ---- */
void orc_psum_f32(const float *const *slots, int num_devices, int64_t n, float *out);

/* ---- MLP loss/grad as the reference's Grad interpreter evaluates it ----
 * layers: L weight matrices w[l] of [dims[l], dims[l+1]] and biases b[l];
 * act: 0 = tanh (MNISTFromScratch.java:103-115), 1 = relu.
 * Writes the loss (scalar) and the gradient of every w/b leaf, and, when gx
 * is not NULL, the gradient with respect to x (the DOT VJP's first output).
 * relu_masks (optional, relu only): one [batch, dims[l+1]] byte array per
 * hidden layer giving the sign pattern z > 0 to use in relu's VJP.  relu' is
 * discontinuous at 0, so an element whose pre-activation is within rounding
 * of 0 can take the other branch under a different (equally valid) summation
 * order; a checker passes the device's pattern after verifying every
 * disagreement is such a near-tie. */
int orc_mlp_loss_grad_f32(int num_layers, const int64_t *dims, int act,
                          const float *const *w, const float *const *b,
                          const float *x, const float *onehot, int64_t batch,
                          float *loss, float *const *gw, float *const *gb, float *gx,
                          const uint8_t *const *relu_masks, int threads);
/* Loss-only forward (same equation order). */
int orc_mlp_loss_f32(int num_layers, const int64_t *dims, int act,
                     const float *const *w, const float *const *b,
                     const float *x, const float *onehot, int64_t batch,
                     float *loss, int threads);

/* ---- Elementwise sweep (where/tanh/sigmoid/relu/clip + sum(-1,keep) + argmax(-1)) ---- */
void orc_sweep_f32(const float *x, const float *y, int64_t rows, int64_t cols,
                   float *z, float *row_sum, int32_t *row_argmax);

/* Fft (api/Fft.java): rank 1 or 3, power-of-two extents; in place for orc_fft. */
void orc_fft(int dtype, int rank, const int64_t *dims, void *re, void *im, int inverse);
void orc_rfft(int dtype, int rank, const int64_t *dims, const void *x, void *out_re, void *out_im);
void orc_irfft(int dtype, int rank, const int64_t *dims, const void *re, const void *im, void *out);
void orc_dct1(int dtype, int64_t n, const void *x, void *out);

/* Linalg (api/Linalg.java): FP64, row-major. */
#define ORC_LU_ZERO_PIVOT 1
#define ORC_LU_SUBMATRIX 2
int orc_lu_factor(double *a, int64_t n, int submatrix_check, int64_t *piv, double *norms, int64_t *fail_k,
                  double *fail_piv);
void orc_lu_solve(const double *lu, const int64_t *piv, int64_t n, const double *b, double *x);
void orc_lu_solve_t(const double *lu, const int64_t *piv, int64_t n, const double *b, double *x);
double orc_lu_rcond(const double *lu, const int64_t *piv, int64_t n, double inf_norm);
/* eigenvalues in deflation order (input dtype); thin SVD (FP64).  0, or 1 if the iteration did not converge. */
int orc_eig(int dtype, int64_t n, const void *a, void *wr, void *wi);
int orc_svd(int dtype, int64_t m, int64_t n, const void *a, double *u, double *s, double *vt);

#ifdef __cplusplus
}
#endif
#endif
