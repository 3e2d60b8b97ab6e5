// linalg.cu -- api/Linalg.java's dense real linear algebra on the device.
//
// The reference factors, solves and decomposes on the host in FP64, for
// FLOAT32 input too (Linalg.java:313-333, 1021-1085, 411-460, 768-800).
// Here the matrices stay resident and cuSOLVER's 64-bit API does the
// O(n^3) work in FP64 on column-major copies:
//
//   j4c_lu_factor  P A = L U with partial pivoting (Xgetrf: the pivot of a
//                  column is its first entry of largest magnitude, the
//                  reference's rule), and for the reference's singularity
//                  checks the pivot magnitudes |U_kk| in elimination order,
//                  max_ij |a_ij| and the row-sum norm max_i sum_j |a_ij|
//   j4c_lu_solve   A X = B or A^T X = B against a factorisation (Xgetrs);
//                  X in B's dtype (LU.solve / solveTranspose,
//                  Linalg.java:141-233)
//   j4c_lu_rcond   1 / (||A||_inf ||A^-1||_inf) by Hager's estimate, the
//                  iteration of Linalg.java:1102-1153 with both solves and
//                  the O(n) reductions on the device and one 32-byte read
//                  back per iteration for its stopping rules
//   j4c_eig        eigenvalues of a real square matrix (Xgeev; the
//                  reference reduces to Hessenberg form and runs Francis
//                  QR, Linalg.java:768-800), real and imaginary parts in
//                  the input's dtype
//   j4c_svd        thin SVD of an m x n matrix, m >= n (Xgesvd; the
//                  reference runs Golub-Kahan-Reinsch, Linalg.java:411-460):
//                  U [m, n], sigma [n] descending and non-negative,
//                  Vt [n, n], all FP64 as in the reference
//
// Row-major operands are moved to and from cuSOLVER's column-major layout
// by a shared-memory tiled transpose that also converts the element type.
// The factorisation, rcond, eig and svd entry points synchronise the
// stream: their results (pivots, info, the estimate) are read on the host,
// where singular or failed factorisations become errors as the reference
// throws.
#include <cusolverDn.h>

#include <mutex>
#include <vector>

#include "common.cuh"

namespace j4c {
namespace la {

static int solver_error(cusolverStatus_t st, const char *what) {
    return set_error(st == CUSOLVER_STATUS_ALLOC_FAILED ? J4C_E_OOM : J4C_E_CUDA, "%s: cuSOLVER status %d", what,
                     (int)st);
}

#define J4C_SOLVER(expr)                                                         \
    do {                                                                         \
        cusolverStatus_t _st = (expr);                                           \
        if (_st != CUSOLVER_STATUS_SUCCESS) return ::j4c::la::solver_error(_st, #expr); \
    } while (0)

// One handle and one params object per device, used under its lock.
struct Solver {
    cusolverDnHandle_t handle = nullptr;
    cusolverDnParams_t params = nullptr;
    std::mutex mu;
};

static int get_solver(Solver **out) {
    static std::mutex mu;
    static std::vector<Solver *> solvers;
    int dev = 0;
    J4C_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    if ((int)solvers.size() <= dev) solvers.resize(dev + 1, nullptr);
    if (!solvers[dev]) {
        Solver *s = new Solver();
        J4C_SOLVER(cusolverDnCreate(&s->handle));
        J4C_SOLVER(cusolverDnCreateParams(&s->params));
        solvers[dev] = s;
    }
    *out = solvers[dev];
    return J4C_OK;
}

// Stream-ordered scratch released on every exit path.
struct Scratch {
    std::vector<void *> blocks;
    cudaStream_t s;
    explicit Scratch(cudaStream_t st) : s(st) {}
    ~Scratch() {
        for (void *p : blocks) scratch_free(p, s);
    }
    int get(size_t bytes, void **p) {
        int rc = scratch_alloc(bytes ? bytes : 16, p, s);
        if (!rc) blocks.push_back(*p);
        return rc;
    }
};

// ---- layout / type conversion ----------------------------------------------
constexpr int kTile = 32, kTileRows = 8;

// out[c * rows + r] = (Tout) in[r * cols + c]: a row-major [rows, cols]
// array to its transpose, i.e. to column-major [rows, cols] (and back, with
// rows and cols exchanged).  32 x 32 tiles through shared memory, so both
// the loads and the stores are coalesced.
template <typename Tin, typename Tout>
__global__ void transpose_cast_kernel(const Tin *__restrict__ in, int64_t rows, int64_t cols, Tout *__restrict__ out) {
    __shared__ Tout tile[kTile][kTile + 1];
    const int64_t c0 = (int64_t)blockIdx.x * kTile, r0 = (int64_t)blockIdx.y * kTile;
    for (int dy = threadIdx.y; dy < kTile; dy += kTileRows) {
        const int64_t r = r0 + dy, c = c0 + threadIdx.x;
        if (r < rows && c < cols) tile[dy][threadIdx.x] = (Tout)in[r * cols + c];
    }
    __syncthreads();
    for (int dy = threadIdx.y; dy < kTile; dy += kTileRows) {
        const int64_t c = c0 + dy, r = r0 + threadIdx.x;
        if (c < cols && r < rows) out[c * rows + r] = tile[threadIdx.x][dy];
    }
}

template <typename Tin, typename Tout>
__global__ void cast_kernel(const Tin *__restrict__ in, int64_t n, Tout *__restrict__ out) {
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < n; k += (int64_t)gridDim.x * blockDim.x)
        out[k] = (Tout)in[k];
}

template <typename Tin, typename Tout>
static int transpose_cast(const void *in, int64_t rows, int64_t cols, void *out, cudaStream_t s) {
    if (rows == 1 || cols == 1) {
        cast_kernel<Tin, Tout><<<grid_for(rows * cols, 256), 256, 0, s>>>((const Tin *)in, rows * cols, (Tout *)out);
        J4C_LAUNCH_CHECK("cast_kernel");
        return J4C_OK;
    }
    const int64_t gx = ceil_div(cols, kTile), gy = ceil_div(rows, kTile);
    J4C_REQUIRE(gy <= 65535 && gx <= 0x7fffffff, "linalg: a %lld x %lld matrix is too large", (long long)rows,
                (long long)cols);
    transpose_cast_kernel<Tin, Tout><<<dim3((unsigned)gx, (unsigned)gy), dim3(kTile, kTileRows), 0, s>>>(
        (const Tin *)in, rows, cols, (Tout *)out);
    J4C_LAUNCH_CHECK("transpose_cast_kernel");
    return J4C_OK;
}

// Row-major [rows, cols] of dtype -> column-major FP64.
static int to_colmajor(int dtype, const void *a, int64_t rows, int64_t cols, double *out, cudaStream_t s) {
    return dtype == J4C_FLOAT64 ? transpose_cast<double, double>(a, rows, cols, out, s)
                                : transpose_cast<float, double>(a, rows, cols, out, s);
}

// Column-major FP64 [rows, cols] -> row-major dtype.
static int from_colmajor(int dtype, const double *a, int64_t rows, int64_t cols, void *out, cudaStream_t s) {
    return dtype == J4C_FLOAT64 ? transpose_cast<double, double>(a, cols, rows, out, s)
                                : transpose_cast<double, float>(a, cols, rows, out, s);
}

// ---- reductions ---------------------------------------------------------------
// Non-negative doubles order like their bit patterns as signed 64-bit
// integers, so an integer atomicMax is a max over them.
__device__ __forceinline__ void atomic_max_nonneg(double *p, double v) {
    atomicMax(reinterpret_cast<long long *>(p), __double_as_longlong(v));
}

// norms[0] = max_ij |a_ij|, norms[1] = max_i sum_j |a_ij| of a row-major
// [n, n] matrix (norms zeroed beforehand).  One warp per row.  As in the
// reference's `if (v > max)` scans, a NaN entry or row sum never becomes
// the maximum (Linalg.java:1026-1040).
template <typename T>
__global__ void norms_kernel(const T *__restrict__ a, int64_t n, double *__restrict__ norms) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t r = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; r < n; r += warps) {
        double sum = 0.0, mx = 0.0;
        for (int64_t c = lane; c < n; c += 32) {
            const double v = fabs((double)a[r * n + c]);
            sum += v;
            if (v > mx) mx = v;
        }
        for (int o = 16; o > 0; o >>= 1) {
            sum += __shfl_xor_sync(0xffffffffu, sum, o);
            const double m2 = __shfl_xor_sync(0xffffffffu, mx, o);
            if (m2 > mx) mx = m2;
        }
        if (lane == 0) {
            if (mx > 0.0) atomic_max_nonneg(&norms[0], mx);
            if (sum > 0.0) atomic_max_nonneg(&norms[1], sum);
        }
    }
}

// piv[k] = |U_kk| of a column-major n x n factorisation.
__global__ void pivots_kernel(const double *__restrict__ lu, int64_t n, double *__restrict__ piv) {
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < n; k += (int64_t)gridDim.x * blockDim.x)
        piv[k] = fabs(lu[k * n + k]);
}

// complex W [n] -> (re, im)
template <typename T>
__global__ void split_complex_kernel(const double2 *__restrict__ w, int64_t n, T *__restrict__ re, T *__restrict__ im) {
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < n; k += (int64_t)gridDim.x * blockDim.x) {
        re[k] = (T)w[k].x;
        im[k] = (T)w[k].y;
    }
}

// ---- Hager's iteration ----------------------------------------------------------
constexpr int kHagerThreads = 1024;

// x = 1/n everywhere (j < 0) or the unit vector e_j.
__global__ void hager_start_kernel(double *__restrict__ x, int64_t n, int64_t j) {
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < n; k += (int64_t)gridDim.x * blockDim.x)
        x[k] = j < 0 ? 1.0 / (double)n : (k == j ? 1.0 : 0.0);
}

// stats[0] = ||y||_1; xi = sign(y) with sign(0) = +1 (Linalg.java:1133-1139).
__global__ void __launch_bounds__(kHagerThreads) hager_norm_sign_kernel(const double *__restrict__ y, int64_t n,
                                                                        double *__restrict__ xi,
                                                                        double *__restrict__ stats) {
    __shared__ double part[kHagerThreads / 32];
    double sum = 0.0;
    for (int64_t k = threadIdx.x; k < n; k += blockDim.x) {
        const double v = y[k];
        sum += fabs(v);
        xi[k] = v >= 0.0 ? 1.0 : -1.0;
    }
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sum;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += part[w];
        stats[0] = t;
    }
}

// stats[1] = max_i |z_i|, stats[2] = its first index, stats[3] = z . x
// (Linalg.java:1141-1148).
__global__ void __launch_bounds__(kHagerThreads) hager_z_kernel(const double *__restrict__ z,
                                                                const double *__restrict__ x, int64_t n,
                                                                double *__restrict__ stats) {
    __shared__ double s_max[kHagerThreads / 32], s_dot[kHagerThreads / 32];
    __shared__ long long s_arg[kHagerThreads / 32];
    double mx = -1.0, dot = 0.0;
    long long arg = 0;
    for (int64_t k = threadIdx.x; k < n; k += blockDim.x) {
        const double a = fabs(z[k]);
        if (a > mx) {  // a thread's indices rise, so its first maximum is kept
            mx = a;
            arg = k;
        }
        dot += z[k] * x[k];
    }
    for (int o = 16; o > 0; o >>= 1) {
        const double m2 = __shfl_xor_sync(0xffffffffu, mx, o);
        const long long a2 = __shfl_xor_sync(0xffffffffu, arg, o);
        if (m2 > mx || (m2 == mx && a2 < arg)) {
            mx = m2;
            arg = a2;
        }
        dot += __shfl_xor_sync(0xffffffffu, dot, o);
    }
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        s_max[w] = mx;
        s_arg[w] = arg;
        s_dot[w] = dot;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        double bm = s_max[0], bd = s_dot[0];
        long long ba = s_arg[0];
        for (int i = 1; i < (int)(blockDim.x >> 5); i++) {
            if (s_max[i] > bm || (s_max[i] == bm && s_arg[i] < ba)) {
                bm = s_max[i];
                ba = s_arg[i];
            }
            bd += s_dot[i];
        }
        stats[1] = bm;
        stats[2] = (double)ba;
        stats[3] = bd;
    }
}

static int check_dtype(int dtype, const char *who) {
    J4C_REQUIRE(dtype == J4C_FLOAT32 || dtype == J4C_FLOAT64, "%s: dtype %s (FLOAT32 or FLOAT64 required)", who,
                dtype_name(dtype));
    return J4C_OK;
}

}  // namespace la
}  // namespace j4c

using namespace j4c;

extern "C" {

int j4c_lu_factor(int dtype, int64_t n, const void *a, double *lu, int64_t *ipiv, double *pivots, double *norms,
                  j4c_stream stream) {
    int rc = la::check_dtype(dtype, "j4c_lu_factor");
    if (rc) return rc;
    J4C_REQUIRE(n >= 1 && a && lu && ipiv && pivots && norms, "j4c_lu_factor: bad arguments (n %lld)", (long long)n);
    cudaStream_t s = as_stream(stream);
    la::Solver *sv = nullptr;
    if ((rc = la::get_solver(&sv))) return rc;
    la::Scratch sc(s);
    void *d_norms = nullptr, *d_piv = nullptr, *d_info = nullptr, *work = nullptr;
    if ((rc = sc.get(2 * sizeof(double), &d_norms)) || (rc = sc.get(sizeof(double) * (size_t)n, &d_piv)) ||
        (rc = sc.get(sizeof(int), &d_info)))
        return rc;
    J4C_CUDA(cudaMemsetAsync(d_norms, 0, 2 * sizeof(double), s));
    const unsigned nb = grid_for(n * 32, 256);
    if (dtype == J4C_FLOAT64) la::norms_kernel<double><<<nb, 256, 0, s>>>((const double *)a, n, (double *)d_norms);
    else la::norms_kernel<float><<<nb, 256, 0, s>>>((const float *)a, n, (double *)d_norms);
    J4C_LAUNCH_CHECK("norms_kernel");
    if ((rc = la::to_colmajor(dtype, a, n, n, lu, s))) return rc;
    {
        std::lock_guard<std::mutex> lock(sv->mu);
        J4C_SOLVER(cusolverDnSetStream(sv->handle, s));
        size_t dev_bytes = 0, host_bytes = 0;
        J4C_SOLVER(cusolverDnXgetrf_bufferSize(sv->handle, sv->params, n, n, CUDA_R_64F, lu, n, CUDA_R_64F,
                                               &dev_bytes, &host_bytes));
        if ((rc = sc.get(dev_bytes, &work))) return rc;
        std::vector<char> host_work(host_bytes ? host_bytes : 1);
        J4C_SOLVER(cusolverDnXgetrf(sv->handle, sv->params, n, n, CUDA_R_64F, lu, n, ipiv, CUDA_R_64F, work,
                                    dev_bytes, host_work.data(), host_bytes, (int *)d_info));
        la::pivots_kernel<<<grid_for(n, 256), 256, 0, s>>>(lu, n, (double *)d_piv);
        J4C_LAUNCH_CHECK("pivots_kernel");
        J4C_CUDA(cudaMemcpyAsync(norms, d_norms, 2 * sizeof(double), cudaMemcpyDeviceToHost, s));
        J4C_CUDA(cudaMemcpyAsync(pivots, d_piv, sizeof(double) * (size_t)n, cudaMemcpyDeviceToHost, s));
        J4C_CUDA(cudaStreamSynchronize(s));
    }
    return J4C_OK;
}

int j4c_lu_solve(int64_t n, int64_t nrhs, const double *lu, const int64_t *ipiv, int transpose, int dtype,
                 const void *b, void *x, j4c_stream stream) {
    int rc = la::check_dtype(dtype, "j4c_lu_solve");
    if (rc) return rc;
    J4C_REQUIRE(n >= 1 && nrhs >= 1 && lu && ipiv && b && x, "j4c_lu_solve: bad arguments (n %lld, nrhs %lld)",
                (long long)n, (long long)nrhs);
    cudaStream_t s = as_stream(stream);
    la::Solver *sv = nullptr;
    if ((rc = la::get_solver(&sv))) return rc;
    la::Scratch sc(s);
    void *rhs = nullptr, *d_info = nullptr;
    if ((rc = sc.get(sizeof(double) * (size_t)(n * nrhs), &rhs)) || (rc = sc.get(sizeof(int), &d_info))) return rc;
    if ((rc = la::to_colmajor(dtype, b, n, nrhs, (double *)rhs, s))) return rc;
    {
        std::lock_guard<std::mutex> lock(sv->mu);
        J4C_SOLVER(cusolverDnSetStream(sv->handle, s));
        J4C_SOLVER(cusolverDnXgetrs(sv->handle, sv->params, transpose ? CUBLAS_OP_T : CUBLAS_OP_N, n, nrhs,
                                    CUDA_R_64F, lu, n, ipiv, CUDA_R_64F, rhs, n, (int *)d_info));
    }
    return la::from_colmajor(dtype, (const double *)rhs, n, nrhs, x, s);
}

int j4c_lu_rcond(int64_t n, const double *lu, const int64_t *ipiv, double inf_norm, double *rcond,
                 j4c_stream stream) {
    J4C_REQUIRE(n >= 1 && lu && ipiv && rcond, "j4c_lu_rcond: bad arguments (n %lld)", (long long)n);
    if (inf_norm == 0.0) {  // Linalg.java:1103
        *rcond = 0.0;
        return J4C_OK;
    }
    cudaStream_t s = as_stream(stream);
    la::Solver *sv = nullptr;
    int rc = la::get_solver(&sv);
    if (rc) return rc;
    la::Scratch sc(s);
    void *x = nullptr, *y = nullptr, *z = nullptr, *d_stats = nullptr, *d_info = nullptr;
    const size_t vec = sizeof(double) * (size_t)n;
    if ((rc = sc.get(vec, &x)) || (rc = sc.get(vec, &y)) || (rc = sc.get(vec, &z)) ||
        (rc = sc.get(4 * sizeof(double), &d_stats)) || (rc = sc.get(sizeof(int), &d_info)))
        return rc;
    la::hager_start_kernel<<<grid_for(n, 256), 256, 0, s>>>((double *)x, n, -1);
    J4C_LAUNCH_CHECK("hager_start_kernel");
    double estimate = 0.0, stats[4];
    std::lock_guard<std::mutex> lock(sv->mu);
    J4C_SOLVER(cusolverDnSetStream(sv->handle, s));
    for (int iter = 0; iter < 5; iter++) {
        // y = A^-T x (B x for B = A^-T); xi = sign(y); z = A^-1 xi (B^T xi)
        J4C_CUDA(cudaMemcpyAsync(y, x, vec, cudaMemcpyDeviceToDevice, s));
        J4C_SOLVER(cusolverDnXgetrs(sv->handle, sv->params, CUBLAS_OP_T, n, 1, CUDA_R_64F, lu, n, ipiv, CUDA_R_64F, y,
                                    n, (int *)d_info));
        la::hager_norm_sign_kernel<<<1, la::kHagerThreads, 0, s>>>((const double *)y, n, (double *)z,
                                                                    (double *)d_stats);
        J4C_LAUNCH_CHECK("hager_norm_sign_kernel");
        J4C_SOLVER(cusolverDnXgetrs(sv->handle, sv->params, CUBLAS_OP_N, n, 1, CUDA_R_64F, lu, n, ipiv, CUDA_R_64F, z,
                                    n, (int *)d_info));
        la::hager_z_kernel<<<1, la::kHagerThreads, 0, s>>>((const double *)z, (const double *)x, n,
                                                            (double *)d_stats);
        J4C_LAUNCH_CHECK("hager_z_kernel");
        J4C_CUDA(cudaMemcpyAsync(stats, d_stats, sizeof(stats), cudaMemcpyDeviceToHost, s));
        J4C_CUDA(cudaStreamSynchronize(s));
        if (iter > 0 && stats[0] <= estimate) break;
        estimate = stats[0];
        if (stats[1] <= fabs(stats[3])) break;  // Hager's stopping rule
        la::hager_start_kernel<<<grid_for(n, 256), 256, 0, s>>>((double *)x, n, (int64_t)stats[2]);
        J4C_LAUNCH_CHECK("hager_start_kernel");
    }
    *rcond = estimate == 0.0 ? INFINITY : 1.0 / (inf_norm * estimate);  // Linalg.java:1104-1106
    J4C_CUDA(cudaStreamSynchronize(s));
    return J4C_OK;
}

int j4c_eig(int dtype, int64_t n, const void *a, void *wr, void *wi, j4c_stream stream) {
    int rc = la::check_dtype(dtype, "j4c_eig");
    if (rc) return rc;
    J4C_REQUIRE(n >= 1 && a && wr && wi, "j4c_eig: bad arguments (n %lld)", (long long)n);
    cudaStream_t s = as_stream(stream);
    la::Solver *sv = nullptr;
    if ((rc = la::get_solver(&sv))) return rc;
    la::Scratch sc(s);
    void *m = nullptr, *w = nullptr, *d_info = nullptr, *work = nullptr;
    if ((rc = sc.get(sizeof(double) * (size_t)(n * n), &m)) || (rc = sc.get(2 * sizeof(double) * (size_t)n, &w)) ||
        (rc = sc.get(sizeof(int), &d_info)))
        return rc;
    if ((rc = la::to_colmajor(dtype, a, n, n, (double *)m, s))) return rc;
    int info = 0;
    {
        std::lock_guard<std::mutex> lock(sv->mu);
        J4C_SOLVER(cusolverDnSetStream(sv->handle, s));
        size_t dev_bytes = 0, host_bytes = 0;
        J4C_SOLVER(cusolverDnXgeev_bufferSize(sv->handle, sv->params, CUSOLVER_EIG_MODE_NOVECTOR,
                                              CUSOLVER_EIG_MODE_NOVECTOR, n, CUDA_R_64F, m, n, CUDA_C_64F, w,
                                              CUDA_R_64F, nullptr, 1, CUDA_R_64F, nullptr, 1, CUDA_R_64F, &dev_bytes,
                                              &host_bytes));
        if ((rc = sc.get(dev_bytes, &work))) return rc;
        std::vector<char> host_work(host_bytes ? host_bytes : 1);
        J4C_SOLVER(cusolverDnXgeev(sv->handle, sv->params, CUSOLVER_EIG_MODE_NOVECTOR, CUSOLVER_EIG_MODE_NOVECTOR, n,
                                   CUDA_R_64F, m, n, CUDA_C_64F, w, CUDA_R_64F, nullptr, 1, CUDA_R_64F, nullptr, 1,
                                   CUDA_R_64F, work, dev_bytes, host_work.data(), host_bytes, (int *)d_info));
        J4C_CUDA(cudaMemcpyAsync(&info, d_info, sizeof(int), cudaMemcpyDeviceToHost, s));
        J4C_CUDA(cudaStreamSynchronize(s));  // the host workspace must outlive the call
    }
    J4C_REQUIRE(info == 0, "eig: the QR iteration did not converge (info %d)", info);
    if (dtype == J4C_FLOAT64)
        la::split_complex_kernel<double>
            <<<grid_for(n, 256), 256, 0, s>>>((const double2 *)w, n, (double *)wr, (double *)wi);
    else
        la::split_complex_kernel<float><<<grid_for(n, 256), 256, 0, s>>>((const double2 *)w, n, (float *)wr, (float *)wi);
    J4C_LAUNCH_CHECK("split_complex_kernel");
    return J4C_OK;
}

int j4c_svd(int dtype, int64_t m, int64_t n, const void *a, double *u, double *sigma, double *vt,
            j4c_stream stream) {
    int rc = la::check_dtype(dtype, "j4c_svd");
    if (rc) return rc;
    J4C_REQUIRE(n >= 1 && m >= n && a && u && sigma && vt, "j4c_svd: bad arguments (m %lld, n %lld; m >= n >= 1)",
                (long long)m, (long long)n);
    cudaStream_t s = as_stream(stream);
    la::Solver *sv = nullptr;
    if ((rc = la::get_solver(&sv))) return rc;
    la::Scratch sc(s);
    void *am = nullptr, *d_u = nullptr, *d_vt = nullptr, *d_info = nullptr, *work = nullptr;
    if ((rc = sc.get(sizeof(double) * (size_t)(m * n), &am)) || (rc = sc.get(sizeof(double) * (size_t)(m * n), &d_u)) ||
        (rc = sc.get(sizeof(double) * (size_t)(n * n), &d_vt)) || (rc = sc.get(sizeof(int), &d_info)))
        return rc;
    if ((rc = la::to_colmajor(dtype, a, m, n, (double *)am, s))) return rc;
    int info = 0;
    {
        std::lock_guard<std::mutex> lock(sv->mu);
        J4C_SOLVER(cusolverDnSetStream(sv->handle, s));
        size_t dev_bytes = 0, host_bytes = 0;
        J4C_SOLVER(cusolverDnXgesvd_bufferSize(sv->handle, sv->params, 'S', 'A', m, n, CUDA_R_64F, am, m, CUDA_R_64F,
                                               sigma, CUDA_R_64F, d_u, m, CUDA_R_64F, d_vt, n, CUDA_R_64F, &dev_bytes,
                                               &host_bytes));
        if ((rc = sc.get(dev_bytes, &work))) return rc;
        std::vector<char> host_work(host_bytes ? host_bytes : 1);
        J4C_SOLVER(cusolverDnXgesvd(sv->handle, sv->params, 'S', 'A', m, n, CUDA_R_64F, am, m, CUDA_R_64F, sigma,
                                    CUDA_R_64F, d_u, m, CUDA_R_64F, d_vt, n, CUDA_R_64F, work, dev_bytes,
                                    host_work.data(), host_bytes, (int *)d_info));
        J4C_CUDA(cudaMemcpyAsync(&info, d_info, sizeof(int), cudaMemcpyDeviceToHost, s));
        J4C_CUDA(cudaStreamSynchronize(s));
    }
    J4C_REQUIRE(info == 0, "svd: the bidiagonal QR iteration did not converge (info %d)", info);
    if ((rc = la::from_colmajor(J4C_FLOAT64, (const double *)d_u, m, n, u, s)) ||
        (rc = la::from_colmajor(J4C_FLOAT64, (const double *)d_vt, n, n, vt, s)))
        return rc;
    return J4C_OK;
}

}  // extern "C"
