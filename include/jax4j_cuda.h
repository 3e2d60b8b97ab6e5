/*
 * jax4j_cuda.h -- C ABI of libjax4j_cuda.so, the B200 (sm_100a) execution
 * backend for jax4j.
 *
 * This header is the drop-in boundary.  Each entry point replaces one method
 * of the reference's operator SPI (backend/ExecutionBackend.java), of its
 * host array core (core/ConcreteNDArray.java), of the Grad interpreter's host
 * helpers (api/Grad.java) or of its in-process collective
 * (api/SharedCollective.java); the comment above each declaration cites the
 * reference method it replaces (paths relative to
 * src/main/java/com/marmanis/jax4j/).
 *
 * Conventions
 *  - Plain pointers and sizes only.  Device pointers live on the calling
 *    thread's current CUDA device (j4c_set_device); host pointers are
 *    ordinary (preferably pinned) memory.
 *  - Every function returns an int status: J4C_OK (0) or a J4C_E_* code.  The
 *    calling thread's last error message is available from j4c_last_error().
 *    No exception crosses the ABI and there is no host fallback: a request
 *    the device path cannot serve fails with J4C_E_UNSUPPORTED.
 *  - Work is enqueued on the given stream (a cudaStream_t; NULL = the legacy
 *    default stream) and is asynchronous unless stated otherwise.
 *  - Inputs are never modified; outputs are caller-allocated and must not
 *    alias inputs unless stated.  The caller owns every buffer.
 *  - prim is the ordinal of ir/Primitive.java and dtype the ordinal of
 *    core/DType.java, so a Java caller passes Enum.ordinal() unchanged.
 *  - Shapes are row-major int64 dimension arrays (dims, rank); rank 0 means
 *    one element.  Broadcasting follows core/Shape.java:37-49 (align right,
 *    size-1 dimensions stretch).
 *  - Thread safety: calls from different host threads on different streams
 *    (one pmap shard per thread) are safe.
 */
#ifndef JAX4J_CUDA_H
#define JAX4J_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define J4C_ABI_VERSION 2

#if defined(__GNUC__)
#define J4C_API __attribute__((visibility("default")))
#else
#define J4C_API
#endif

/* status codes */
#define J4C_OK 0
#define J4C_E_INVALID 1     /* bad argument: shape, dtype, op, size, pointer */
#define J4C_E_UNSUPPORTED 2 /* valid request the device path does not implement */
#define J4C_E_CUDA 3        /* CUDA runtime/driver error */
#define J4C_E_OOM 4         /* device allocation failed */
#define J4C_E_NCCL 5        /* NCCL error */
#define J4C_E_TIMEOUT 6     /* a collective or a device-side wait exceeded its limit */
#define J4C_E_DEVICE 7      /* a kernel reported an error through its status word */

/* ir/Primitive.java:6-42 ordinals used by this ABI */
#define J4C_ADD 0
#define J4C_SUB 1
#define J4C_MUL 2
#define J4C_DIV 3
#define J4C_DOT 4
#define J4C_EXP 5
#define J4C_LOG 6
#define J4C_SIN 7
#define J4C_COS 8
#define J4C_SUM 9
#define J4C_MEAN 10
#define J4C_SUM_AXIS 11
#define J4C_MEAN_AXIS 12
#define J4C_TANH 13
#define J4C_RELU 14
#define J4C_SIGMOID 15
#define J4C_GT 19
#define J4C_GE 20
#define J4C_LT 21
#define J4C_LE 22
#define J4C_EQ 23
#define J4C_NE 24
#define J4C_MAX 25
#define J4C_MIN 26
#define J4C_ARGMAX 27
#define J4C_ARGMIN 28
#define J4C_PSUM 30
#define J4C_ALL_GATHER 31
#define J4C_CAST 32

/* core/DType.java:7-11 ordinals; BOOL is one byte holding 0 or 1 */
#define J4C_FLOAT32 0
#define J4C_FLOAT64 1
#define J4C_INT32 2
#define J4C_INT64 3
#define J4C_BOOL 4

typedef void *j4c_stream;           /* cudaStream_t */
typedef struct j4c_comm_s *j4c_comm; /* one rank of a collective group */

/* ------------------------------------------------------------------ */
/* Runtime, devices, errors                                            */
/* ------------------------------------------------------------------ */

J4C_API int j4c_abi_version(void);
/* Number of kernels this library has launched in the process (all devices). */
J4C_API int j4c_kernel_launches(uint64_t *out);
/* Message of the last failed call on this thread ("" if none). */
J4C_API const char *j4c_last_error(void);
/* Replaces Device.getDevices (core/Device.java:53-77): CUDA device count. */
J4C_API int j4c_device_count(int *out);
/* Binds the calling thread to a CUDA ordinal (pmap shard i -> GPU i). */
J4C_API int j4c_set_device(int device);
J4C_API int j4c_get_device(int *out);
/* Enables peer access from `device` to `peer` (both directions when possible). */
J4C_API int j4c_enable_peer_access(int device, int peer);
/* Blocks until all work on the stream is done; returns any asynchronous
 * kernel error, including device-side status words (J4C_E_DEVICE). */
J4C_API int j4c_stream_synchronize(j4c_stream stream);
J4C_API int j4c_stream_create(j4c_stream *out);
J4C_API int j4c_stream_destroy(j4c_stream stream);
/* Reads and clears the library's device status word on the current device:
 * non-zero after a kernel gave up a bounded wait or rejected its input. */
J4C_API int j4c_device_status(int *out_code);
/* No counterpart in the reference (its collectives and kernels wait without
 * limit).  Sets, for kernels launched afterwards in this process, how long
 * a pipeline wait of the persistent GEMM may see no progress before the
 * kernel gives up: it records device status 0x7C05, stops its pipeline,
 * waits (always up to 2 s) for its own copies and tensor-core work in flight,
 * releases its tensor memory and returns, leaving C unspecified.  ns > 0;
 * the previous limit goes to *previous (may be NULL).  Default 2 s; below
 * 1 ms the waits poll without suspending (a limit for testing this path). */
J4C_API int j4c_set_wait_limit_ns(uint64_t ns, uint64_t *previous);

/* ------------------------------------------------------------------ */
/* Storage: replaces ConcreteNDArray's host Storage records             */
/* (core/ConcreteNDArray.java:47-87) and TornadoVM's per-call copies      */
/* (backend/TornadoVMBackend.java:33-44) with resident device buffers.    */
/* ------------------------------------------------------------------ */

/* Stream-ordered allocation from the device's memory pool. */
J4C_API int j4c_malloc(size_t bytes, void **out, j4c_stream stream);
J4C_API int j4c_free(void *ptr, j4c_stream stream);
J4C_API int j4c_memcpy_h2d(void *dst, const void *src, size_t bytes, j4c_stream stream);
J4C_API int j4c_memcpy_d2h(void *dst, const void *src, size_t bytes, j4c_stream stream);
J4C_API int j4c_memcpy_d2d(void *dst, const void *src, size_t bytes, j4c_stream stream);
/* Fills n elements of dtype with value (Grad.java:847-903 ones/zeros/minusOne). */
J4C_API int j4c_fill(int dtype, void *out, int64_t n, double value, j4c_stream stream);

/* ------------------------------------------------------------------ */
/* Elementwise                                                          */
/* ------------------------------------------------------------------ */

/* ExecutionBackend.binary (backend/ExecutionBackend.java:13) generalised to
 * ConcreteNDArray.elementwise's broadcasting (core/ConcreteNDArray.java:219-316):
 * prim in {ADD, SUB, MUL, DIV, MAX, MIN}; dtype FLOAT32 or FLOAT64; both
 * operands share dtype.  out has the broadcast shape.  Results equal the
 * reference's `(float) op((double) a, (double) b)`: correctly rounded
 * IEEE arithmetic, Java Math.max/min NaN and signed-zero rules. */
J4C_API int j4c_binary(int prim, int dtype, const void *a, const int64_t *a_dims, int a_rank,
               const void *b, const int64_t *b_dims, int b_rank, void *out, j4c_stream stream);

/* ConcreteNDArray.compareElementwise (core/ConcreteNDArray.java:328-404):
 * prim in {GT, GE, LT, LE, EQ, NE}; dtype FLOAT32, FLOAT64, INT32 or INT64
 * (BOOL operands are rejected, as in the reference); out is BOOL (uint8 0/1)
 * with the broadcast shape.  Bit-exact. */
J4C_API int j4c_compare(int prim, int dtype, const void *a, const int64_t *a_dims, int a_rank,
                const void *b, const int64_t *b_dims, int b_rank, uint8_t *out,
                j4c_stream stream);

/* ExecutionBackend.unary (backend/ExecutionBackend.java:16) /
 * ConcreteNDArray.unary (core/ConcreteNDArray.java:627-664): prim in {EXP,
 * LOG, SIN, COS, TANH, RELU, SIGMOID}; dtype FLOAT32 or FLOAT64.  out may
 * alias in. */
J4C_API int j4c_unary(int prim, int dtype, const void *in, int64_t n, void *out, j4c_stream stream);

/* ConcreteNDArray.astype (core/ConcreteNDArray.java:666-730): any pair of
 * the five dtypes with Java's conversion rules (float->int truncates, NaN->0,
 * saturates; long->int wraps; x->BOOL is "!= 0"; BOOL->x is 1/0).  Bit-exact. */
J4C_API int j4c_cast(int src_dtype, int dst_dtype, const void *in, int64_t n, void *out,
             j4c_stream stream);

/* ------------------------------------------------------------------ */
/* Reductions                                                           */
/* ------------------------------------------------------------------ */

/* ExecutionBackend.reduce (backend/ExecutionBackend.java:22) /
 * HostBackend.reduce (backend/HostBackend.java:117-124): prim SUM or MEAN
 * over n elements into out[0]; dtype FLOAT32 or FLOAT64.  Deterministic
 * (fixed tree order); mean divides the sum by (T) n. */
J4C_API int j4c_reduce_all(int prim, int dtype, const void *in, int64_t n, void *out,
                   j4c_stream stream);

/* ConcreteNDArray.reduceAxis (core/ConcreteNDArray.java:510-548): the input
 * is viewed as [outer, axis_len, inner]; out is [outer, inner].  prim
 * SUM_AXIS or MEAN_AXIS.  Deterministic. */
J4C_API int j4c_reduce_axis(int prim, int dtype, const void *in, int64_t outer, int64_t axis_len,
                    int64_t inner, void *out, j4c_stream stream);

/* No counterpart in the reference.  The same per-axis sum/mean as
 * j4c_reduce_axis (same kernels, same bits), for callers that cannot allocate
 * device memory: a host runtime that hands all of the GPU's memory to its own
 * arena at start-up and lets native code take no more, or code that must not
 * block, since cudaFree synchronises the device and a pool allocation may
 * stall while the pool grows.  Its only scratch -- the partial sums when the
 * axis is split across CTAs -- lives in a static device array of
 * J4C_REDUCE_NOALLOC_SCRATCH_BYTES that every GPU loading the library holds
 * until the process exits; a reduction needing more is rejected with
 * J4C_E_INVALID (use j4c_reduce_axis).  The first call on each device looks
 * the array's address up (cudaGetSymbolAddress).  Under CUDA's lazy module
 * loading (the default on current drivers) that lookup may be what loads the
 * library's device image onto the device, and the driver then reserves the
 * image's memory, this array included: make the first call at start-up,
 * before the host hands the device's memory to its arena and before any
 * stream capture on that device.  All calls share the one array: calls
 * whose work overlaps on the GPU (other streams, other threads) race on it;
 * nothing needs clearing between calls. */
#define J4C_REDUCE_NOALLOC_SCRATCH_BYTES (256 * 1024)
J4C_API int j4c_reduce_axis_noalloc(int prim, int dtype, const void *in, int64_t outer,
                                    int64_t axis_len, int64_t inner, void *out, j4c_stream stream);

/* ConcreteNDArray.argReduceAxis (core/ConcreteNDArray.java:571-618): prim
 * ARGMAX or ARGMIN over [outer, axis_len, inner] -> int32 [outer, inner];
 * the first strict extremum wins, as the reference's sequential scan.
 * Bit-exact. */
J4C_API int j4c_argreduce(int prim, int dtype, const void *in, int64_t outer, int64_t axis_len,
                  int64_t inner, int32_t *out, j4c_stream stream);

/* ------------------------------------------------------------------ */
/* Grad.java host helpers as device ops                                 */
/* ------------------------------------------------------------------ */

/* Grad.broadcastLike (api/Grad.java:539-582): reconciles g with the
 * target shape -- equal size: copy (reshape); smaller g: broadcast it out;
 * larger g: sum the broadcast contributions back down (deterministic).
 * Also serves Grad.axisBroadcastLike (api/Grad.java:608-641) with g viewed as
 * [outer, 1, inner] and the target as [outer, axis, inner]. */
J4C_API int j4c_broadcast_like(int dtype, const void *g, const int64_t *g_dims, int g_rank, void *out,
                       const int64_t *t_dims, int t_rank, j4c_stream stream);

/* Grad.reluGrad (api/Grad.java:585-598): out = x > 0 ? g : 0. */
J4C_API int j4c_relu_grad(int dtype, const void *g, const void *x, int64_t n, void *out,
                  j4c_stream stream);

/* Grad.maxMinGrad (api/Grad.java:500-530): routes g to the operand that won
 * (ties go to a).  ga_full and gb_full have g's (broadcast) shape; apply
 * j4c_broadcast_like to reduce them to the operand shapes. */
J4C_API int j4c_maxmin_grad(int is_max, int dtype, const void *g, const int64_t *g_dims, int g_rank,
                    const void *a, const int64_t *a_dims, int a_rank, const void *b,
                    const int64_t *b_dims, int b_rank, void *ga_full, void *gb_full,
                    j4c_stream stream);

/* Grad.transpose (api/Grad.java:643-664): out[cols, rows] = in[rows, cols]. */
J4C_API int j4c_transpose(int dtype, const void *in, int64_t rows, int64_t cols, void *out,
                  j4c_stream stream);

/* Numpy.take (api/Numpy.java:54-76, primitive GATHER): out[p, :] =
 * table[idx[p], :] for a [rows, dim] table and n INT32/INT64 indices (out is
 * [n, dim]); an index outside [0, rows) yields a zero row (callers validate
 * indices first, as the reference's array copy would throw).  Its VJP
 * (Grad.gatherBackward, api/Grad.java:474-493): gtable (zeroed by the
 * caller, [rows, dim]) += g rows scattered to their indices; repeated indices
 * accumulate (atomic adds, so their order is unspecified). */
J4C_API int j4c_gather_rows(int dtype, const void *table, int64_t rows, int64_t dim, int idx_dtype,
                            const void *idx, int64_t n, void *out, j4c_stream stream);
J4C_API int j4c_scatter_add_rows(int dtype, const void *g, int64_t rows, int64_t dim, int idx_dtype,
                                 const void *idx, int64_t n, void *gtable, j4c_stream stream);

/* ------------------------------------------------------------------ */
/* dot                                                                  */
/* ------------------------------------------------------------------ */

/* ExecutionBackend.matmul (backend/ExecutionBackend.java:19) /
 * ConcreteNDArray.dot (core/ConcreteNDArray.java:406-461), with layout flags
 * so the DOT VJP (api/Grad.java:385-390) needs no materialised transpose:
 *   C[M,N] = op(A)[M,K] . op(B)[K,N]
 *   op(A) = A stored [M,K] (trans_a = 0) or A stored [K,M] (trans_a = 1)
 *   op(B) = B stored [K,N] (trans_b = 0) or B stored [N,K] (trans_b = 1)
 * FLOAT32 runs on the 5th-generation tensor cores (tcgen05, TMA-fed) with a
 * three-product split (a = hi + lo; a.b ~ hi.hi + hi.lo + lo.hi, in FP16 with
 * per-line power-of-two scales or in TF32; see j4c_dot_split_kind) so the
 * result has FP32 accuracy, and operands holding a NaN or an infinity get the
 * reference's sequential FP32 sum exactly; FLOAT64 runs a CUDA-core kernel.  Scratch for the split
 * operands comes from the library's stream-ordered pool. */
J4C_API int j4c_dot(int dtype, const void *a, const void *b, void *c, int64_t M, int64_t K, int64_t N,
            int trans_a, int trans_b, j4c_stream stream);
/* Same, with caller-provided scratch of at least j4c_dot_workspace_size bytes. */
J4C_API int j4c_dot_ws(int dtype, const void *a, const void *b, void *c, int64_t M, int64_t K,
               int64_t N, int trans_a, int trans_b, void *workspace, size_t workspace_bytes,
               j4c_stream stream);
J4C_API size_t j4c_dot_workspace_size(int dtype, int64_t M, int64_t K, int64_t N);

/* The FLOAT32 dot in two steps, so a tensor that takes part in several
 * products (a layer's input, weight and output gradient each appear in two
 * of the forward/VJP dots) is split once per use.  A split of x stored
 * [rows, cols] is two caller-allocated device arrays, hi and lo, of
 * j4c_split_floats(rows, cols) floats each (16-byte aligned; for the
 * transposed split j4c_split_floats(cols, rows)); j4c_dot_split then
 * computes C = op(A) . op(B) as j4c_dot does, from the splits of A and B
 * (trans flags as for j4c_dot).  Which split an operand takes follows from
 * how the GEMM reads it:
 *   op(A) = A, A stored [M, K]     (trans_a = 0): j4c_split_f32(A)
 *   op(A) = A^T, A stored [K, M]   (trans_a = 1): j4c_split_f32_cols(A), or
 *                                  j4c_split_f32_transposed(A) with trans_a = 0
 *   op(B) = B, B stored [K, N]     (trans_b = 0): j4c_split_f32_cols(B), or
 *                                  j4c_split_f32_transposed(B) with trans_b = 1
 *   op(B) = B^T, B stored [N, K]   (trans_b = 1): j4c_split_f32(B)
 * i.e. a split read K-major (K along its rows) has one line per row, one read
 * MN-major one line per column.  A GEMM given a split of the wrong kind
 * computes nothing and records device status 0x7C06 (j4c_device_status).
 * The split of an unchanged tensor may be reused by any number of products;
 * the tensor itself must stay allocated and unchanged while its splits are
 * used (a product whose operand holds a NaN or an infinity reads it).
 * The format is the library's (j4c_dot_split_kind), fixed for the process:
 *   1, 3xFP16 (default): each line (a row or a column of the data) is scaled
 *      by the power of two 2^e that brings its largest finite |x| into
 *      [2^14, 2^15) (e in [-113, 127]), hi = fp16(x 2^e) and lo =
 *      fp16(x 2^e - hi) as 2-byte halves in rows of j4c_split_pitch(cols)
 *      elements (padding zero); the hi array then holds a 32-byte header and
 *      the line maxima the epilogue scales by;
 *   0, 3xTF32 (environment J4C_GEMM_SPLIT=tf32): the same line scales (they
 *      keep FP32 subnormals, which TF32 products flush, exact), hi =
 *      tf32(x 2^e), lo = tf32(x 2^e - hi) as floats in rows of
 *      j4c_split_pitch(cols) elements, then the header and line maxima.
 * Special values: a split records whether x holds a NaN or an infinity (it
 * stores them as zero); a product either of whose operands does is computed
 * on the CUDA cores as the reference's sequential FP32 sum of x's own values
 * (core/ConcreteNDArray.java:452-459), bit for bit, NaN/Inf rules included. */
J4C_API int j4c_dot_split_kind(void);
/* Elements per row of a split's data with `cols` columns (halves under
 * 3xFP16, floats under 3xTF32); -1 for a negative extent. */
J4C_API int64_t j4c_split_pitch(int64_t cols);
/* Floats to allocate for each of hi and lo of a split whose data is
 * [rows, cols]; -1 for a negative extent. */
J4C_API int64_t j4c_split_floats(int64_t rows, int64_t cols);
/* The stored-layout split with one line per row (read K-major). */
J4C_API int j4c_split_f32(const float *x, int64_t rows, int64_t cols, float *hi, float *lo, j4c_stream stream);
/* The stored-layout split with one line per column (read MN-major). */
J4C_API int j4c_split_f32_cols(const float *x, int64_t rows, int64_t cols, float *hi, float *lo,
                               j4c_stream stream);
/* The split of x^T (data [cols, rows], its rows -- x's columns -- as lines;
 * read K-major).  A product whose A and B are both stored with K as the
 * leading (slow) dimension, such as the weight gradient x^T . dy, runs
 * fastest with one of them given in this form (and its trans flag flipped). */
J4C_API int j4c_split_f32_transposed(const float *x, int64_t rows, int64_t cols, float *hi, float *lo,
                                     j4c_stream stream);
/* Both j4c_split_f32 (hi/lo) and j4c_split_f32_transposed (hi_t/lo_t) in
 * one pass over x (an output gradient that is the left operand of g . W^T
 * and the right one of x^T . g). */
J4C_API int j4c_split_f32_both(const float *x, int64_t rows, int64_t cols, float *hi, float *lo, float *hi_t,
                               float *lo_t, j4c_stream stream);
/* Any of the splits above in one pass -- hi/lo (row lines), hi_c/lo_c
 * (column lines) or hi_t/lo_t (transposed), each pair optional, hi_c and
 * hi_t not both -- with x's line maxima computed already: lines (device, may
 * be NULL) holds rows + cols + 1 words, the bits of the largest finite |x| of
 * each row and then of each column, then a word nonzero when x holds a NaN
 * or an infinity, as j4c_split_lines or j4c_dot_split_ep_max's out_lines
 * leave them; it replaces the split's own max pass. */
J4C_API int j4c_split_f32_ex(const float *x, int64_t rows, int64_t cols, float *hi, float *lo, float *hi_c,
                             float *lo_c, float *hi_t, float *lo_t, const uint32_t *lines, j4c_stream stream);
/* lines [rows + cols + 1] (device): the line maxima of x (rows, then
 * columns) and its NaN/Inf flag in one pass, for several later
 * j4c_split_f32_ex calls. */
J4C_API int j4c_split_lines(const float *x, int64_t rows, int64_t cols, uint32_t *lines, j4c_stream stream);
/* The SGD update of a [rows, cols] FLOAT32 weight, out = w - ((g * scale) * lr)
 * elementwise (the reference's update, w.sub(g.mul(scale).mul(lr)), bit for
 * bit), with out's line words in lines (rows + cols + 1 words: row maxima,
 * column maxima, NaN/Inf flag, as j4c_split_lines leaves them; zeroed by the
 * call) so that out's next splits need no max pass.  out must not alias w or g. */
J4C_API int j4c_sgd_update_lines(const float *w, const float *g, int64_t rows, int64_t cols, float scale, float lr,
                                 float *out, uint32_t *lines, j4c_stream stream);
J4C_API int j4c_dot_split(const float *a_hi, const float *a_lo, const float *b_hi, const float *b_lo, float *c,
                          int64_t M, int64_t K, int64_t N, int trans_a, int trans_b, j4c_stream stream);
/* j4c_dot_split with elementwise work fused into the store of C [M, N] (each
 * pointer may be NULL; none may alias C):
 *   C = op(A).op(B) + bias        bias [N], broadcast over rows -- the bias
 *                                 add of a dense layer (ConcreteNDArray.add)
 *   C = mask > 0 ? C : 0          mask [M, N] -- relu' (api/Grad.java:585-598)
 *                                 applied to an input gradient
 *   act = max(0, C)               act [M, N] -- the layer's relu output
 * c may be NULL when act is given (only the relu output is stored).
 * Each value is rounded exactly as the separate add / relu / relu' kernels
 * round it, so results equal the unfused sequence bit for bit. */
/* Strided-batched j4c_dot_split (vmap's batched dot, api/Vmap.java:269-297):
 * for b < batch, C[b] = op(A[b]) . op(B[b]) with C [batch, M, N].  An operand
 * flagged batched holds `batch` split matrices back to back (the split of its
 * [batch * rows, cols] storage, of the kind its use needs as above); an
 * unbatched one is shared by every b.  One persistent launch covers every
 * (b, tile).  trans_a && !trans_b is rejected (pass one operand's transposed
 * split instead, as for j4c_dot_split). */
J4C_API int j4c_dot_split_batched(const float *a_hi, const float *a_lo, const float *b_hi, const float *b_lo,
                                  float *c, int64_t batch, int64_t M, int64_t K, int64_t N, int trans_a,
                                  int trans_b, int a_batched, int b_batched, j4c_stream stream);
J4C_API int j4c_dot_split_ep(const float *a_hi, const float *a_lo, const float *b_hi, const float *b_lo,
                             float *c, int64_t M, int64_t K, int64_t N, int trans_a, int trans_b,
                             const float *bias, const float *mask, float *act, j4c_stream stream);
/* j4c_dot_split_ep that also leaves in out_lines (M + N + 1 device uint32
 * words) the line maxima of what it writes to act (or to c when act is
 * NULL): the bits of the largest finite |value| of each of the M rows, then
 * of each of the N columns, then a word nonzero when a written value is a
 * NaN or an infinity -- what a later j4c_split_f32_ex of that output takes
 * instead of scanning it again. */
J4C_API int j4c_dot_split_ep_max(const float *a_hi, const float *a_lo, const float *b_hi, const float *b_lo,
                                 float *c, int64_t M, int64_t K, int64_t N, int trans_a, int trans_b,
                                 const float *bias, const float *mask, float *act, uint32_t *out_lines,
                                 j4c_stream stream);
/* j4c_dot_split_ep_max with relu bits (Grad.reluGrad, api/Grad.java:585-598,
 * fed by bits instead of a float array): act_bits (may be NULL; needs act)
 * receives one bit per element of act, set where act > 0 -- bit c & 31 of
 * word c / 32 of each of the M rows of ceil(N / 32) uint32 words -- and
 * mask_bits (may be NULL; not with mask) masks C by such bits (C = bit ?
 * C : 0, as mask > 0 does).  1/32 of the bytes of the float mask.  Bits need
 * the form that stores C untransposed: trans_b = 1 (for A . B, pass B's
 * transposed split) or trans_a = 1; with trans_a = trans_b = 0 they are
 * rejected (J4C_E_INVALID). */
J4C_API int j4c_dot_split_ep_bits(const float *a_hi, const float *a_lo, const float *b_hi, const float *b_lo,
                                  float *c, int64_t M, int64_t K, int64_t N, int trans_a, int trans_b,
                                  const float *bias, const float *mask, const uint32_t *mask_bits, float *act,
                                  uint32_t *act_bits, uint32_t *out_lines, j4c_stream stream);

/* ------------------------------------------------------------------ */
/* Discrete Fourier transforms: replace api/Fft.java's radix-2 host     */
/* transforms (Fft.java:292-371) and its per-call TornadoVM cuFFT path  */
/* (Fft.java:760-1100).  A complex signal is two arrays (real, imag)    */
/* as in the reference; rank 1 (a vector) or 3 (an N0 x N1 x N2 grid);  */
/* every extent a power of two (J4C_E_INVALID otherwise); FLOAT32 or    */
/* FLOAT64, outputs of the input's dtype, caller-allocated.             */
/* ------------------------------------------------------------------ */
/* Fft.fft / ifft / fft3 / ifft3 (Fft.java:64-80, 405-418): every axis;
 * the inverse scales by 1/N. */
J4C_API int j4c_fft(int dtype, int rank, const int64_t *dims, const void *re, const void *im, void *out_re,
                    void *out_im, int inverse, j4c_stream stream);
/* Fft.rfft / rfft3 (Fft.java:93-127, 423-492): real x with extents `dims`
 * -> the half spectrum [.., dims[rank-1]/2 + 1] (real and imaginary parts). */
J4C_API int j4c_rfft(int dtype, int rank, const int64_t *dims, const void *x, void *out_re, void *out_im,
                     j4c_stream stream);
/* Fft.irfft / irfft3 (Fft.java:130-186, 494-568): half spectrum
 * [.., dims[rank-1]/2 + 1] -> real signal with extents `dims`
 * (dims[rank-1] >= 2); the imaginary parts of the DC and Nyquist bins are
 * ignored, as the reference's Hermitian mirror ignores them. */
J4C_API int j4c_irfft(int dtype, int rank, const int64_t *dims, const void *re, const void *im, void *out,
                      j4c_stream stream);
/* Fft.dctI (Fft.java:200-227): unnormalised DCT-I of n values, n = 1 or
 * n - 1 a power of two, computed in FP64 for both dtypes. */
J4C_API int j4c_dct1(int dtype, int64_t n, const void *x, void *out, j4c_stream stream);

/* ------------------------------------------------------------------ */
/* Dense linear algebra: replace api/Linalg.java's host LU, solves,     */
/* Hager condition estimate, Francis-QR eigenvalues and Golub-Kahan-    */
/* Reinsch SVD.  Matrices are row-major FLOAT32 or FLOAT64 on the       */
/* device; everything is computed in FP64 as in the reference.          */
/* ------------------------------------------------------------------ */
/* The factorisation of Linalg.luFactorInPlace (Linalg.java:1021-1085):
 * P A = L U of the n x n matrix a, into caller-allocated device arrays lu
 * (n*n FP64, column-major, L's unit diagonal implied) and ipiv (n int64,
 * 1-based row swaps in elimination order).  Host outputs: pivots[k] =
 * |U_kk| for k = 0..n-1 (elimination order, so the first k that fails a
 * singularity check is the step at which the reference throws), norms[0] =
 * max |a_ij| and norms[1] = max_i sum_j |a_ij| of a.  Synchronous.  A zero
 * pivot is not an error here: the caller applies the check. */
J4C_API int j4c_lu_factor(int dtype, int64_t n, const void *a, double *lu, int64_t *ipiv, double *pivots,
                          double *norms, j4c_stream stream);
/* LU.solve / LU.solveTranspose (Linalg.java:141-233): A X = B
 * (transpose = 0) or A^T X = B (transpose = 1) against a factorisation;
 * b and x are row-major [n, nrhs] of `dtype` (a vector when nrhs = 1). */
J4C_API int j4c_lu_solve(int64_t n, int64_t nrhs, const double *lu, const int64_t *ipiv, int transpose, int dtype,
                         const void *b, void *x, j4c_stream stream);
/* Linalg.reciprocalConditionNumber (Linalg.java:1102-1153): Hager's
 * estimate of 1 / (||A||_inf ||A^-1||_inf), inf_norm = norms[1] of the
 * factorisation; at most 5 iterations of two solves each.  *rcond (host)
 * is 0 when inf_norm is 0 and +inf when the estimate of ||A^-1|| is 0.
 * Synchronous. */
J4C_API int j4c_lu_rcond(int64_t n, const double *lu, const int64_t *ipiv, double inf_norm, double *rcond,
                         j4c_stream stream);
/* Linalg.eig(A) (Linalg.java:768-800): the n eigenvalues of a real square
 * matrix, real and imaginary parts in the input's dtype; complex ones in
 * adjacent conjugate pairs.  The order may differ from the reference's
 * Francis-QR deflation order.  Synchronous. */
J4C_API int j4c_eig(int dtype, int64_t n, const void *a, void *wr, void *wi, j4c_stream stream);
/* Linalg.svd (Linalg.java:411-460): thin SVD of an m x n matrix, m >= n:
 * u [m, n], sigma [n] (descending, non-negative) and vt [n, n], row-major
 * FP64 for both input dtypes, as the reference returns.  Synchronous. */
J4C_API int j4c_svd(int dtype, int64_t m, int64_t n, const void *a, double *u, double *sigma, double *vt,
                    j4c_stream stream);

/* ------------------------------------------------------------------ */
/* Fused elementwise programs: replace TornadoJitCompiler.compile       */
/* (backend/TornadoJitCompiler.java:82-246), which runs one kernel per   */
/* Jaxpr equation, with one generated kernel per chain.                  */
/* ------------------------------------------------------------------ */

/* A program works on a [rows, cols] view of the chain's shape (cols = the
 * last dimension).  Each input is read with one of four broadcast patterns. */
#define J4C_BCAST_FULL 0   /* [rows, cols] */
#define J4C_BCAST_ROW 1    /* [cols]: one value per column, shared by all rows */
#define J4C_BCAST_COL 2    /* [rows, 1]: one value per row */
#define J4C_BCAST_SCALAR 3 /* a single value */

/* Instruction opcodes beyond the primitive ordinals. */
#define J4C_OP_INPUT (-1)     /* the value of input slot `a` */
#define J4C_OP_CONST (-2)     /* the constant `value` */
#define J4C_OP_RELU_GRAD (-3) /* Grad.reluGrad (api/Grad.java:593-597): b > 0 ? a : 0 */

typedef struct {
    int32_t op;    /* primitive ordinal (ADD..MIN, EXP..SIGMOID, GT..NE, CAST) or J4C_OP_* */
    int32_t dtype; /* dtype of the result (FLOAT32, FLOAT64, INT32 or BOOL) */
    int32_t a, b;  /* operand instruction indices (-1 unused); for INPUT, a = input slot */
    double value;  /* for CONST */
} j4c_insn;

typedef struct {
    int32_t n_insns;
    const j4c_insn *insns; /* in dependency order */
    int32_t n_inputs;      /* <= 16 */
    const int32_t *input_dtype;
    const int32_t *input_bcast;
    int32_t n_outputs;         /* <= 16; each written as a [rows, cols] array */
    const int32_t *output_insn;
    int32_t n_tails;           /* <= 8; one value per row */
    const int32_t *tail_op;    /* SUM_AXIS, MEAN_AXIS (-> insn dtype), ARGMAX, ARGMIN (-> INT32) */
    const int32_t *tail_insn;
} j4c_program;

/* Generates, compiles (NVRTC, sm_100a) and caches the program's kernels on
 * the current device; *handle stays valid for the process lifetime.  Calls
 * with an identical program return the same handle. */
J4C_API int j4c_fused_compile(const j4c_program *prog, void **handle);
/* Runs a compiled program: inputs/outputs/tails are arrays of device
 * pointers in slot order.  Elementwise results equal the unfused kernels'
 * bit for bit; tails are deterministic tree reductions of each row. */
/* Diagnostics: the CUDA C++ source j4c_fused_compile would generate for
 * `prog` (NUL-terminated, truncated to cap bytes; *len = full size + 1), and
 * when `compile` is nonzero its NVRTC compilation for sm_100a, which needs no
 * GPU.  Returns J4C_E_INVALID for a malformed program and J4C_E_CUDA with the
 * compiler log in j4c_last_error() when compilation fails. */
J4C_API int j4c_fused_source(const j4c_program *prog, int compile, char *buf, size_t cap, size_t *len);

J4C_API int j4c_fused_launch(void *handle, int64_t rows, int64_t cols, const void *const *inputs,
                             void *const *outputs, void *const *tails, j4c_stream stream);

/* ------------------------------------------------------------------ */
/* Random (api/Random.java:39-150): SplitMix64 streams, bit-exact       */
/* ------------------------------------------------------------------ */

/* Random.uniform (api/Random.java:86-93): out[i] = lo + u(offset+i)*(hi-lo)
 * in float.  offset lets each shard generate its slice of one global array. */
/* Random.permutation (api/Random.java:130-140): a permutation of 0..n-1 as
 * INT32, the reference's Fisher-Yates over the key's uniform stream
 * (bit-identical; the swaps run sequentially on one GPU thread). */
J4C_API int j4c_random_permutation(uint64_t key, int64_t n, int32_t *out, j4c_stream stream);
J4C_API int j4c_random_uniform(uint64_t key, int64_t offset, int64_t n, float lo, float hi, float *out,
                       j4c_stream stream);
/* Random.normal (api/Random.java:104-113): Box-Muller in double. */
J4C_API int j4c_random_normal(uint64_t key, int64_t offset, int64_t n, float *out, j4c_stream stream);

/* ------------------------------------------------------------------ */
/* Collectives: replace SharedCollective (api/SharedCollective.java)    */
/* ------------------------------------------------------------------ */

/* Number of bytes of a collective group id (the NCCL unique id). */
#define J4C_COMM_ID_BYTES 128
/* Creates a group id on rank 0; the caller distributes it to every rank. */
J4C_API int j4c_comm_unique_id(void *out, size_t len);
/* Joins rank `rank` of an nranks group on CUDA device `device`
 * (one process per GPU).  Initialisation and every collective are bounded
 * by timeout_ms: on expiry the communicator is aborted and the call returns
 * J4C_E_TIMEOUT instead of hanging (the reference's barrier waits forever,
 * api/SharedCollective.java:78-85). */
J4C_API int j4c_comm_init_rank(const void *id, size_t len, int nranks, int rank, int device,
                       int64_t timeout_ms, j4c_comm *out);
/* One process driving ndev GPUs (the reference's thread-per-shard pmap,
 * api/Pmap.java:135-166): out[i] is the rank bound to devices[i]. */
J4C_API int j4c_comm_init_all(const int *devices, int ndev, int64_t timeout_ms, j4c_comm *out);
J4C_API int j4c_comm_rank(j4c_comm comm, int *rank, int *nranks);
J4C_API int j4c_comm_destroy(j4c_comm comm);
J4C_API int j4c_comm_abort(j4c_comm comm);
/* SharedCollective.psum (api/SharedCollective.java:44-54): all-reduce sum of
 * n elements (FLOAT32/FLOAT64) enqueued on `stream`; in and out may alias.
 * Asynchronous like every other op: j4c_comm_wait bounds the wait for it. */
J4C_API int j4c_psum(j4c_comm comm, int dtype, const void *in, void *out, int64_t n, j4c_stream stream);
/* SharedCollective.allGather (api/SharedCollective.java:61-76): out is
 * [nranks, n] in rank order. */
J4C_API int j4c_all_gather(j4c_comm comm, int dtype, const void *in, void *out, int64_t n,
                   j4c_stream stream);
/* Reduce-scatter: in [nranks * n] on every rank; out [n] on rank r = the sum
 * over ranks of their slice r (the transpose of all-gather, used by the
 * optional reduce-scatter ALL_GATHER VJP; the reference's VJP,
 * api/Grad.java:437-441, takes the local slice without communication). */
J4C_API int j4c_reduce_scatter(j4c_comm comm, int dtype, const void *in, void *out, int64_t n,
                               j4c_stream stream);
/* Waits until the work enqueued on `stream` is done, bounded by the
 * communicator's timeout; on expiry aborts the communicator and returns
 * J4C_E_TIMEOUT (replaces the unbounded CyclicBarrier.await,
 * api/SharedCollective.java:78-85). */
J4C_API int j4c_comm_wait(j4c_comm comm, j4c_stream stream);
/* In-process psum over shards that share one device (several pmap shards on
 * one GPU, or peer-mapped slots): out[i] = 0 + slot0[i] + slot1[i] + ... in
 * slot order, bit-identical to the reference's summation order
 * (api/SharedCollective.java:47-51).  slots is a HOST array of nslots device
 * pointers; out may alias any slot. */
J4C_API int j4c_psum_slots(int dtype, const void *const *slots, int nslots, void *out, int64_t n,
                   j4c_stream stream);

/* ---- gradient all-reduce fused with the SGD update (one process per GPU) ----
 * Replaces, for a data-parallel step, Lax.psum of every gradient
 * (api/SharedCollective.java:44-54) followed by the elementwise update
 * w - g * scale * lr on each parameter.  Buffers a peer must read live in
 * peer buffers: device memory allocated with j4c_peer_alloc, whose handle
 * (J4C_PEER_HANDLE_BYTES) the caller sends to every other rank, which maps it
 * with j4c_peer_open (CUDA IPC; the ranks' GPUs must reach one another over
 * NVLink).  j4c_peer_close unmaps a peer's buffer, j4c_peer_free releases
 * one's own.  Peer buffers start zeroed. */
#define J4C_PEER_HANDLE_BYTES 64
J4C_API int j4c_peer_alloc(size_t bytes, void **ptr, void *handle, size_t handle_len);
J4C_API int j4c_peer_open(const void *handle, size_t handle_len, void **ptr);
J4C_API int j4c_peer_close(void *ptr);
J4C_API int j4c_peer_free(void *ptr);
/* Bytes of the flag block each rank keeps in a peer buffer (16-byte
 * aligned, zeroed at allocation, one per group of ranks; a group's calls
 * are issued in the same order on every rank, on one stream per rank). */
J4C_API size_t j4c_psum_sgd_flag_bytes(void);
/* One bucket of n floats (a multiple of 4, at least 4 per rank): grads[p],
 * upd[p] and flags[p] are rank p's packed gradients, exchange buffer (n
 * floats) and flag block, as mapped in this process (this rank's own
 * pointers at index rank); all are HOST arrays of nranks device pointers,
 * nranks <= 8.  This rank's parameters of the bucket are nsegs <= 16
 * segments (params[i], seg_len[i] floats each, multiples of 4, 16-byte
 * aligned) in bucket order.  stage is local scratch of n + 4 * nranks
 * floats.  out (n floats) receives
 *     w - ((sum over ranks p = 0..nranks-1, in order, of grads[p]) * scale) * lr
 * for every element, the same bits on every rank: rank r reduces and updates
 * the r-th slice (the peers' gradients of it copied over NVLink by the copy
 * engines into stage), and gathers the other slices from the peers'
 * exchange buffers the same way; no rank writes another rank's memory but
 * its flag words.  Every cross-rank wait is bounded (j4c_set_wait_limit_ns):
 * on expiry the waiting kernel records device status 0x7C05 and returns;
 * the group is then unusable. */
J4C_API int j4c_psum_sgd(const float *const *grads, const float *const *upd, uint32_t *const *flags, int nranks,
                         int rank, int64_t n, int nsegs, const int64_t *seg_len, const float *const *params,
                         float scale, float lr, float *stage, float *out, j4c_stream stream);

#ifdef __cplusplus
}
#endif
#endif /* JAX4J_CUDA_H */
