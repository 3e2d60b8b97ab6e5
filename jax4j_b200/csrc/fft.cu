// fft.cu -- discrete Fourier transforms of api/Fft.java on the device.
//
// The reference keeps a complex signal as two arrays (real, imaginary) and
// transforms it with an iterative radix-2 Cooley-Tukey on the host
// (Fft.java:292-371), or with cuFFT behind TornadoVM with copies every call
// (Fft.java:760-1100).  Here the arrays stay resident: a pack kernel
// interleaves (re, im) into cuFFT's complex layout, cuFFT transforms it
// (FP32: C2C / R2C / C2R, FP64: Z2Z / D2Z / Z2D), and an unpack kernel
// splits the result and applies the inverse's 1/N.  Plans are made once per
// (device, kind, dtype, extents) and reused.
//
//   fft / ifft     every axis of a 1-D vector or a 3-D grid (Fft.java:64-80, 405-418)
//   rfft           the non-redundant half along the last axis (Fft.java:93-127, 423-492):
//                  cuFFT's R2C is the reference's complex transform of (x, 0) cut to N/2+1
//   irfft          Fft.java:130-186, 494-568: the inverse over the leading axes as complex
//                  transforms, then along the last axis the real part of the inverse of the
//                  Hermitian mirror -- exactly cuFFT's C2R, which like the mirror ignores the
//                  imaginary parts of the DC and Nyquist bins
//   dct1           Fft.java:200-227, 373-398: the real part of the FFT of
//                  [x0..x_{n-1}, x_{n-2}..x1], in FP64 for both dtypes as the reference
//
// Extents must be powers of two (the reference's constraint; cuFFT itself
// would take any size).  Axes of extent 1 are dropped from a plan.
#include <cufft.h>

#include <map>
#include <memory>
#include <mutex>
#include <tuple>
#include <vector>

#include "common.cuh"

namespace j4c {
namespace fft {

static int cufft_error(cufftResult r, const char *what) {
    return set_error(r == CUFFT_ALLOC_FAILED ? J4C_E_OOM : J4C_E_CUDA, "%s: cuFFT error %d", what, (int)r);
}

#define J4C_CUFFT(expr)                                                  \
    do {                                                                 \
        cufftResult _r = (expr);                                         \
        if (_r != CUFFT_SUCCESS) return cufft_error(_r, #expr);          \
    } while (0)

enum Kind { kC2C = 0, kR2C = 1, kC2R = 2, kLeading = 3 };

// kC2C / kR2C / kC2R: `batch` transforms over `dims` (kR2C / kC2R: dims are
// the real extents), one after another in memory.  kLeading: complex
// transforms over dims[0..rank-2] of an array whose last axis (dims[rank-1]
// entries, the half spectrum) is the batch -- irfft's leading axes.
struct Plan {
    cufftHandle handle = 0;
    std::mutex mu;  // a plan runs on one stream at a time
};

using Key = std::tuple<int, int, int, long long, std::vector<long long>>;

static int get_plan(int kind, int dtype, const std::vector<long long> &dims, long long batch, Plan **out) {
    static std::mutex mu;
    static std::map<Key, std::unique_ptr<Plan>> plans;
    int dev = 0;
    J4C_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    const Key key{dev, kind, dtype, batch, dims};
    auto it = plans.find(key);
    if (it != plans.end()) {
        *out = it->second.get();
        return J4C_OK;
    }
    const bool f64 = dtype == J4C_FLOAT64;
    auto plan = std::make_unique<Plan>();
    J4C_CUFFT(cufftCreate(&plan->handle));
    size_t work = 0;
    std::vector<long long> n = dims;
    const int rank = (int)n.size();
    cufftResult r;
    if (kind == kLeading) {
        // transforms over the leading axes; element (i.., k) at ((i..) * h + k)
        const long long h = n.back();
        std::vector<long long> lead(n.begin(), n.end() - 1);
        r = cufftMakePlanMany64(plan->handle, rank - 1, lead.data(), lead.data(), h, 1, lead.data(), h, 1,
                                f64 ? CUFFT_Z2Z : CUFFT_C2C, h, &work);
    } else {
        const cufftType t = kind == kC2C ? (f64 ? CUFFT_Z2Z : CUFFT_C2C)
                            : kind == kR2C ? (f64 ? CUFFT_D2Z : CUFFT_R2C)
                                           : (f64 ? CUFFT_Z2D : CUFFT_C2R);
        r = cufftMakePlanMany64(plan->handle, rank, n.data(), nullptr, 1, 0, nullptr, 1, 0, t, batch, &work);
    }
    if (r != CUFFT_SUCCESS) {
        cufftDestroy(plan->handle);
        return cufft_error(r, "cufftMakePlanMany64");
    }
    *out = plan.get();
    plans.emplace(key, std::move(plan));
    return J4C_OK;
}

template <typename T> struct Cx;
template <> struct Cx<float> { using type = cufftComplex; };
template <> struct Cx<double> { using type = cufftDoubleComplex; };

template <typename T>
__global__ void pack_kernel(const T *__restrict__ re, const T *__restrict__ im, int64_t n,
                            typename Cx<T>::type *__restrict__ out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        out[i].x = re[i];
        out[i].y = im ? im[i] : T(0);
    }
}

// re/im = in * scale (scale 1 leaves the values untouched)
template <typename T>
__global__ void unpack_kernel(const typename Cx<T>::type *__restrict__ in, int64_t n, T scale, int scaled,
                              T *__restrict__ re, T *__restrict__ im) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        re[i] = scaled ? in[i].x * scale : in[i].x;
        im[i] = scaled ? in[i].y * scale : in[i].y;
    }
}

template <typename T>
__global__ void scale_kernel(T *__restrict__ x, int64_t n, T scale) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        x[i] = x[i] * scale;
}

// w = [x0, x1, .., x_{n-1}, x_{n-2}, .., x1] in FP64 (m = 2 (n - 1) entries)
template <typename T>
__global__ void mirror_kernel(const T *__restrict__ x, int64_t n, double *__restrict__ w) {
    const int64_t m = 2 * (n - 1);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < m; i += (int64_t)gridDim.x * blockDim.x)
        w[i] = (double)x[i < n ? i : m - i];
}

template <typename T>
__global__ void real_part_kernel(const cufftDoubleComplex *__restrict__ in, int64_t n, T *__restrict__ out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = (T)in[i].x;
}

template <typename T>
__global__ void copy_kernel(const T *__restrict__ in, int64_t n, T *__restrict__ out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = in[i];
}

static int exec_c2c(Plan *p, bool f64, void *in, void *out, int dir, cudaStream_t s) {
    std::lock_guard<std::mutex> lock(p->mu);
    J4C_CUFFT(cufftSetStream(p->handle, s));
    if (f64) J4C_CUFFT(cufftExecZ2Z(p->handle, (cufftDoubleComplex *)in, (cufftDoubleComplex *)out, dir));
    else J4C_CUFFT(cufftExecC2C(p->handle, (cufftComplex *)in, (cufftComplex *)out, dir));
    count_launch();
    return J4C_OK;
}

static int exec_r2c(Plan *p, bool f64, void *in, void *out, cudaStream_t s) {
    std::lock_guard<std::mutex> lock(p->mu);
    J4C_CUFFT(cufftSetStream(p->handle, s));
    if (f64) J4C_CUFFT(cufftExecD2Z(p->handle, (cufftDoubleReal *)in, (cufftDoubleComplex *)out));
    else J4C_CUFFT(cufftExecR2C(p->handle, (cufftReal *)in, (cufftComplex *)out));
    count_launch();
    return J4C_OK;
}

static int exec_c2r(Plan *p, bool f64, void *in, void *out, cudaStream_t s) {
    std::lock_guard<std::mutex> lock(p->mu);
    J4C_CUFFT(cufftSetStream(p->handle, s));
    if (f64) J4C_CUFFT(cufftExecZ2D(p->handle, (cufftDoubleComplex *)in, (cufftDoubleReal *)out));
    else J4C_CUFFT(cufftExecC2R(p->handle, (cufftComplex *)in, (cufftReal *)out));
    count_launch();
    return J4C_OK;
}

static bool pow2(int64_t n) { return n >= 1 && (n & (n - 1)) == 0; }

static std::vector<long long> non_unit(const int64_t *dims, int rank) {
    std::vector<long long> v;
    for (int i = 0; i < rank; i++)
        if (dims[i] != 1) v.push_back(dims[i]);
    return v;
}

static int64_t count(const int64_t *dims, int rank) {
    int64_t n = 1;
    for (int i = 0; i < rank; i++) n *= dims[i];
    return n;
}

// Complex transform over every axis; inverse scales by 1/N.
template <typename T>
static int fft_t(int rank, const int64_t *dims, const T *re, const T *im, T *ore, T *oim, bool inverse,
                 cudaStream_t s) {
    using C = typename Cx<T>::type;
    const int64_t n = count(dims, rank);
    const std::vector<long long> axes = non_unit(dims, rank);
    if (axes.empty()) {  // every extent 1: the transform is the identity
        copy_kernel<T><<<grid_for(n, 256), 256, 0, s>>>(re, n, ore);
        J4C_LAUNCH_CHECK("copy_kernel");
        copy_kernel<T><<<grid_for(n, 256), 256, 0, s>>>(im, n, oim);
        J4C_LAUNCH_CHECK("copy_kernel");
        return J4C_OK;
    }
    Plan *p = nullptr;
    int rc = get_plan(kC2C, sizeof(T) == 8 ? J4C_FLOAT64 : J4C_FLOAT32, axes, 1, &p);
    if (rc) return rc;
    void *buf = nullptr;
    if ((rc = scratch_alloc(sizeof(C) * (size_t)n, &buf, s))) return rc;
    pack_kernel<T><<<grid_for(n, 256), 256, 0, s>>>(re, im, n, (C *)buf);
    J4C_LAUNCH_CHECK("pack_kernel");
    if (!(rc = exec_c2c(p, sizeof(T) == 8, buf, buf, inverse ? CUFFT_INVERSE : CUFFT_FORWARD, s))) {
        unpack_kernel<T><<<grid_for(n, 256), 256, 0, s>>>((const C *)buf, n, T(1) / (T)n, inverse ? 1 : 0, ore,
                                                          oim);
        J4C_LAUNCH_CHECK("unpack_kernel");
    }
    scratch_free(buf, s);
    return rc;
}

// Real-input transform: out [.., dims[rank-1]/2 + 1] complex.
template <typename T>
static int rfft_t(int rank, const int64_t *dims, const T *x, T *ore, T *oim, cudaStream_t s) {
    using C = typename Cx<T>::type;
    const int64_t last = dims[rank - 1], h = last / 2 + 1, rows = count(dims, rank - 1);
    const int64_t nout = rows * h;
    if (last == 1) {  // the last axis is trivial: a complex transform of (x, 0) over the others
        void *zero = nullptr;
        int rc = scratch_alloc(sizeof(T) * (size_t)nout, &zero, s);
        if (rc) return rc;
        J4C_CUDA(cudaMemsetAsync(zero, 0, sizeof(T) * (size_t)nout, s));
        rc = fft_t<T>(rank, dims, x, (const T *)zero, ore, oim, false, s);
        scratch_free(zero, s);
        return rc;
    }
    std::vector<long long> axes = non_unit(dims, rank - 1);
    axes.push_back(last);
    Plan *p = nullptr;
    int rc = get_plan(kR2C, sizeof(T) == 8 ? J4C_FLOAT64 : J4C_FLOAT32, axes, 1, &p);
    if (rc) return rc;
    void *buf = nullptr;
    if ((rc = scratch_alloc(sizeof(C) * (size_t)nout, &buf, s))) return rc;
    if (!(rc = exec_r2c(p, sizeof(T) == 8, const_cast<T *>(x), buf, s))) {
        unpack_kernel<T><<<grid_for(nout, 256), 256, 0, s>>>((const C *)buf, nout, T(1), 0, ore, oim);
        J4C_LAUNCH_CHECK("unpack_kernel");
    }
    scratch_free(buf, s);
    return rc;
}

// Inverse real transform: (re, im) [.., h] -> out [.., dims[rank-1]], h = dims[rank-1]/2 + 1.
template <typename T>
static int irfft_t(int rank, const int64_t *dims, const T *re, const T *im, T *out, cudaStream_t s) {
    using C = typename Cx<T>::type;
    const int64_t last = dims[rank - 1], h = last / 2 + 1, rows = count(dims, rank - 1);
    const int64_t nin = rows * h, nout = rows * last;
    const bool f64 = sizeof(T) == 8;
    const int dt = f64 ? J4C_FLOAT64 : J4C_FLOAT32;
    void *buf = nullptr;
    int rc = scratch_alloc(sizeof(C) * (size_t)nin, &buf, s);
    if (rc) return rc;
    pack_kernel<T><<<grid_for(nin, 256), 256, 0, s>>>(re, im, nin, (C *)buf);
    J4C_LAUNCH_CHECK("pack_kernel");
    // 1. inverse complex transforms over the leading axes, each half-spectrum column alone
    std::vector<long long> lead = non_unit(dims, rank - 1);
    if (!lead.empty()) {
        lead.push_back(h);
        Plan *p = nullptr;
        if ((rc = get_plan(kLeading, dt, lead, h, &p)) || (rc = exec_c2c(p, f64, buf, buf, CUFFT_INVERSE, s))) {
            scratch_free(buf, s);
            return rc;
        }
    }
    // 2. along the last axis, per row: the real inverse of the half spectrum
    Plan *p = nullptr;
    if (!(rc = get_plan(kC2R, dt, std::vector<long long>{(long long)last}, rows, &p)) &&
        !(rc = exec_c2r(p, f64, buf, out, s))) {
        const int64_t n = nout;
        scale_kernel<T><<<grid_for(n, 256), 256, 0, s>>>(out, n, T(1) / (T)n);
        J4C_LAUNCH_CHECK("scale_kernel");
    }
    scratch_free(buf, s);
    return rc;
}

// DCT-I of n = 2^k + 1 values through a length-2(n-1) FP64 real transform.
template <typename T>
static int dct1_t(int64_t n, const T *x, T *out, cudaStream_t s) {
    if (n == 1) {
        copy_kernel<T><<<1, 32, 0, s>>>(x, 1, out);
        J4C_LAUNCH_CHECK("copy_kernel");
        return J4C_OK;
    }
    const int64_t m = 2 * (n - 1);
    void *w = nullptr, *spec = nullptr;
    int rc = scratch_alloc(sizeof(double) * (size_t)m, &w, s);
    if (rc) return rc;
    if ((rc = scratch_alloc(sizeof(cufftDoubleComplex) * (size_t)n, &spec, s))) {
        scratch_free(w, s);
        return rc;
    }
    mirror_kernel<T><<<grid_for(m, 256), 256, 0, s>>>(x, n, (double *)w);
    J4C_LAUNCH_CHECK("mirror_kernel");
    Plan *p = nullptr;
    if (!(rc = get_plan(kR2C, J4C_FLOAT64, std::vector<long long>{(long long)m}, 1, &p)) &&
        !(rc = exec_r2c(p, true, w, spec, s))) {
        real_part_kernel<T><<<grid_for(n, 256), 256, 0, s>>>((const cufftDoubleComplex *)spec, n, out);
        J4C_LAUNCH_CHECK("real_part_kernel");
    }
    scratch_free(spec, s);
    scratch_free(w, s);
    return rc;
}

static int check_dims(const char *who, int rank, const int64_t *dims) {
    J4C_REQUIRE(rank == 1 || rank == 3, "%s: rank %d (1-D vectors or 3-D grids)", who, rank);
    J4C_REQUIRE(dims, "%s: NULL dims", who);
    for (int i = 0; i < rank; i++)
        J4C_REQUIRE(pow2(dims[i]) && dims[i] < (1ll << 31), "%s: extent %lld is not a power of two", who,
                    (long long)dims[i]);
    return J4C_OK;
}

}  // namespace fft
}  // namespace j4c

using namespace j4c;

extern "C" {

int j4c_fft(int dtype, int rank, const int64_t *dims, const void *re, const void *im, void *out_re, void *out_im,
            int inverse, j4c_stream stream) {
    int rc = fft::check_dims("j4c_fft", rank, dims);
    if (rc) return rc;
    J4C_REQUIRE(dtype == J4C_FLOAT32 || dtype == J4C_FLOAT64, "j4c_fft: dtype %s", dtype_name(dtype));
    J4C_REQUIRE(re && im && out_re && out_im, "j4c_fft: NULL pointer");
    cudaStream_t s = as_stream(stream);
    if (dtype == J4C_FLOAT64)
        return fft::fft_t<double>(rank, dims, (const double *)re, (const double *)im, (double *)out_re,
                                  (double *)out_im, inverse != 0, s);
    return fft::fft_t<float>(rank, dims, (const float *)re, (const float *)im, (float *)out_re, (float *)out_im,
                             inverse != 0, s);
}

int j4c_rfft(int dtype, int rank, const int64_t *dims, const void *x, void *out_re, void *out_im,
             j4c_stream stream) {
    int rc = fft::check_dims("j4c_rfft", rank, dims);
    if (rc) return rc;
    J4C_REQUIRE(dtype == J4C_FLOAT32 || dtype == J4C_FLOAT64, "j4c_rfft: dtype %s", dtype_name(dtype));
    J4C_REQUIRE(x && out_re && out_im, "j4c_rfft: NULL pointer");
    cudaStream_t s = as_stream(stream);
    if (dtype == J4C_FLOAT64)
        return fft::rfft_t<double>(rank, dims, (const double *)x, (double *)out_re, (double *)out_im, s);
    return fft::rfft_t<float>(rank, dims, (const float *)x, (float *)out_re, (float *)out_im, s);
}

int j4c_irfft(int dtype, int rank, const int64_t *dims, const void *re, const void *im, void *out,
              j4c_stream stream) {
    int rc = fft::check_dims("j4c_irfft", rank, dims);
    if (rc) return rc;
    J4C_REQUIRE(dims[rank - 1] >= 2, "j4c_irfft: the last extent must be at least 2");
    J4C_REQUIRE(dtype == J4C_FLOAT32 || dtype == J4C_FLOAT64, "j4c_irfft: dtype %s", dtype_name(dtype));
    J4C_REQUIRE(re && im && out, "j4c_irfft: NULL pointer");
    cudaStream_t s = as_stream(stream);
    if (dtype == J4C_FLOAT64)
        return fft::irfft_t<double>(rank, dims, (const double *)re, (const double *)im, (double *)out, s);
    return fft::irfft_t<float>(rank, dims, (const float *)re, (const float *)im, (float *)out, s);
}

int j4c_dct1(int dtype, int64_t n, const void *x, void *out, j4c_stream stream) {
    J4C_REQUIRE(n == 1 || (n >= 2 && fft::pow2(n - 1) && n - 1 < (1ll << 30)),
                "j4c_dct1: n - 1 = %lld is not a power of two", (long long)(n - 1));
    J4C_REQUIRE(dtype == J4C_FLOAT32 || dtype == J4C_FLOAT64, "j4c_dct1: dtype %s", dtype_name(dtype));
    J4C_REQUIRE(x && out, "j4c_dct1: NULL pointer");
    cudaStream_t s = as_stream(stream);
    if (dtype == J4C_FLOAT64) return fft::dct1_t<double>(n, (const double *)x, (double *)out, s);
    return fft::dct1_t<float>(n, (const float *)x, (float *)out, s);
}

}  // extern "C"
