// dot.cu -- the j4c_dot entry points (ConcreteNDArray.dot,
// core/ConcreteNDArray.java:406-461; ExecutionBackend.matmul,
// backend/ExecutionBackend.java:19).  Chooses the kernel for a shape/dtype.
#include <algorithm>
#include <cstdlib>

#include "common.cuh"

namespace j4c {
int simt_gemm(int dtype, const void *a, const void *b, void *c, int64_t M, int64_t K, int64_t N,
              int trans_a, int trans_b, cudaStream_t s);
int dmma_gemm(const double *a, const double *b, double *c, int64_t M, int64_t K, int64_t N, int trans_a,
              int trans_b, cudaStream_t s);
int tc_gemm_workspace(int64_t M, int64_t K, int64_t N, size_t *bytes);
int64_t tc_split_floats(int64_t rows, int64_t cols);
int64_t tc_split_pitch(int64_t cols);
int tc_split_kind();
int tc_gemm_f32(const float *a, const float *b, float *c, int64_t M, int64_t K, int64_t N,
                int trans_a, int trans_b, void *ws, size_t ws_bytes, cudaStream_t s);
bool tc_gemm_supported(int64_t M, int64_t K, int64_t N);
int tc_split_any(const float *x, int64_t rows, int64_t cols, float *hr, float *lr, float *hc, float *lc, float *ht,
                 float *lt, const uint32_t *lines_in, cudaStream_t s);
int tc_split_lines(const float *x, int64_t rows, int64_t cols, uint32_t *lines, cudaStream_t s);
int tc_sgd_update_lines(const float *w, const float *g, int64_t rows, int64_t cols, float scale, float lr, float *out,
                        uint32_t *lines, cudaStream_t s);
int tc_gemm_presplit(const float *ah, const float *al, const float *bh, const float *bl, float *c, int64_t M,
                     int64_t K, int64_t N, int trans_a, int trans_b, const float *bias, const float *mask,
                     float *act, int64_t batch, int a_batched, int b_batched, cudaStream_t s,
                     uint32_t *out_lines = nullptr, const uint32_t *mask_bits = nullptr,
                     uint32_t *act_bits = nullptr);
}  // namespace j4c

using namespace j4c;

extern "C" {

size_t j4c_dot_workspace_size(int dtype, int64_t M, int64_t K, int64_t N) {
    if (dtype != J4C_FLOAT32 || !tc_gemm_supported(M, K, N)) return 0;
    size_t bytes = 0;
    tc_gemm_workspace(M, K, N, &bytes);
    return bytes;
}

int j4c_dot_ws(int dtype, const void *a, const void *b, void *c, int64_t M, int64_t K, int64_t N,
               int trans_a, int trans_b, void *workspace, size_t workspace_bytes,
               j4c_stream stream) {
    J4C_REQUIRE(M >= 0 && K >= 0 && N >= 0, "j4c_dot: negative dimension");
    J4C_REQUIRE(dtype == J4C_FLOAT32 || dtype == J4C_FLOAT64,
                "dot requires FLOAT32 or FLOAT64 operands, got %s", dtype_name(dtype));
    cudaStream_t s = as_stream(stream);
    if (M == 0 || N == 0) return J4C_OK;
    J4C_REQUIRE(a && b && c, "j4c_dot: NULL pointer");
    if (K == 0) return j4c_fill(dtype, c, M * N, 0.0, stream);
    if (dtype == J4C_FLOAT32 && tc_gemm_supported(M, K, N)) {
        size_t need = 0;
        tc_gemm_workspace(M, K, N, &need);
        J4C_REQUIRE(workspace_bytes >= need && (need == 0 || workspace),
                    "j4c_dot_ws: workspace of %zu bytes is smaller than the %zu required",
                    workspace_bytes, need);
        return tc_gemm_f32((const float *)a, (const float *)b, (float *)c, M, K, N, trans_a,
                           trans_b, workspace, workspace_bytes, s);
    }
    // FLOAT64 on the FP64 tensor path (DMMA) unless J4C_DOT64=simt asks for
    // the CUDA-core kernel (kept for comparison)
    static const bool simt64 = [] {
        const char *v = getenv("J4C_DOT64");
        return v && v[0] == 's';
    }();
    if (dtype == J4C_FLOAT64 && !simt64)
        return dmma_gemm((const double *)a, (const double *)b, (double *)c, M, K, N, trans_a, trans_b, s);
    return simt_gemm(dtype, a, b, c, M, K, N, trans_a, trans_b, s);
}

int j4c_dot(int dtype, const void *a, const void *b, void *c, int64_t M, int64_t K, int64_t N,
            int trans_a, int trans_b, j4c_stream stream) {
    size_t need = j4c_dot_workspace_size(dtype, M, K, N);
    void *ws = nullptr;
    cudaStream_t s = as_stream(stream);
    if (need) {
        int rc = scratch_alloc(need, &ws, s);
        if (rc) return rc;
    }
    int rc = j4c_dot_ws(dtype, a, b, c, M, K, N, trans_a, trans_b, ws, need, stream);
    if (ws) scratch_free(ws, s);
    return rc;
}

int64_t j4c_split_pitch(int64_t cols) { return cols < 0 ? -1 : tc_split_pitch(cols); }

int64_t j4c_split_floats(int64_t rows, int64_t cols) {
    return rows < 0 || cols < 0 ? -1 : tc_split_floats(std::max<int64_t>(rows, 1), std::max<int64_t>(cols, 1));
}

int j4c_dot_split_kind(void) { return tc_split_kind(); }

static int split_entry(const char *name, const float *x, int64_t rows, int64_t cols, float *hr, float *lr,
                       float *hc, float *lc, float *ht, float *lt, const uint32_t *lines_in, j4c_stream stream) {
    J4C_REQUIRE(rows >= 0 && cols >= 0, "%s: negative extent", name);
    if (rows == 0 || cols == 0) return J4C_OK;
    J4C_REQUIRE(x && (hr || hc || ht) && !hr == !lr && !hc == !lc && !ht == !lt, "%s: NULL pointer", name);
    return tc_split_any(x, rows, cols, hr, lr, hc, lc, ht, lt, lines_in, as_stream(stream));
}

int j4c_split_f32(const float *x, int64_t rows, int64_t cols, float *hi, float *lo, j4c_stream stream) {
    return split_entry("j4c_split_f32", x, rows, cols, hi, lo, nullptr, nullptr, nullptr, nullptr, nullptr, stream);
}

int j4c_split_f32_cols(const float *x, int64_t rows, int64_t cols, float *hi, float *lo, j4c_stream stream) {
    return split_entry("j4c_split_f32_cols", x, rows, cols, nullptr, nullptr, hi, lo, nullptr, nullptr, nullptr,
                       stream);
}

int j4c_split_f32_both(const float *x, int64_t rows, int64_t cols, float *hi, float *lo, float *hi_t,
                       float *lo_t, j4c_stream stream) {
    J4C_REQUIRE(!rows || !cols || (hi && lo && hi_t && lo_t), "j4c_split_f32_both: NULL pointer");
    return split_entry("j4c_split_f32_both", x, rows, cols, hi, lo, nullptr, nullptr, hi_t, lo_t, nullptr, stream);
}

int j4c_split_f32_transposed(const float *x, int64_t rows, int64_t cols, float *hi, float *lo,
                             j4c_stream stream) {
    return split_entry("j4c_split_f32_transposed", x, rows, cols, nullptr, nullptr, nullptr, nullptr, hi, lo,
                       nullptr, stream);
}

int j4c_split_f32_ex(const float *x, int64_t rows, int64_t cols, float *hi, float *lo, float *hi_c, float *lo_c,
                     float *hi_t, float *lo_t, const uint32_t *lines, j4c_stream stream) {
    return split_entry("j4c_split_f32_ex", x, rows, cols, hi, lo, hi_c, lo_c, hi_t, lo_t, lines, stream);
}

int j4c_split_lines(const float *x, int64_t rows, int64_t cols, uint32_t *lines, j4c_stream stream) {
    J4C_REQUIRE(rows >= 0 && cols >= 0, "j4c_split_lines: negative extent");
    J4C_REQUIRE(lines && (x || rows == 0 || cols == 0), "j4c_split_lines: NULL pointer");
    return tc_split_lines(x, rows, cols, lines, as_stream(stream));
}

int j4c_sgd_update_lines(const float *w, const float *g, int64_t rows, int64_t cols, float scale, float lr,
                         float *out, uint32_t *lines, j4c_stream stream) {
    if (rows == 0 || cols == 0) return J4C_OK;
    return tc_sgd_update_lines(w, g, rows, cols, scale, lr, out, lines, as_stream(stream));
}

int j4c_dot_split_ep_bits(const float *a_hi, const float *a_lo, const float *b_hi, const float *b_lo, float *c,
                          int64_t M, int64_t K, int64_t N, int trans_a, int trans_b, const float *bias,
                          const float *mask, const uint32_t *mask_bits, float *act, uint32_t *act_bits,
                          uint32_t *out_lines, j4c_stream stream) {
    J4C_REQUIRE(M >= 0 && K >= 0 && N >= 0, "j4c_dot_split: negative dimension");
    J4C_REQUIRE(!(mask && mask_bits), "j4c_dot_split_ep_bits: the mask as floats or as bits, not both");
    cudaStream_t s = as_stream(stream);
    if (M == 0 || N == 0) {
        if (out_lines) J4C_CUDA(cudaMemsetAsync(out_lines, 0, (size_t)(M + N + 1) * sizeof(uint32_t), s));
        return J4C_OK;
    }
    J4C_REQUIRE(c || act, "j4c_dot_split: NULL output");
    J4C_REQUIRE(K > 0 || (!bias && !mask && !mask_bits && !act), "j4c_dot_split_ep: K = 0 with an epilogue");
    if (K == 0) {
        if (out_lines) J4C_CUDA(cudaMemsetAsync(out_lines, 0, (size_t)(M + N + 1) * sizeof(uint32_t), s));
        return j4c_fill(J4C_FLOAT32, c, M * N, 0.0, stream);
    }
    J4C_REQUIRE(a_hi && a_lo && b_hi && b_lo, "j4c_dot_split: NULL operand");
    if (!tc_gemm_supported(M, K, N))
        return set_error(J4C_E_UNSUPPORTED, "j4c_dot_split: shape %lld x %lld x %lld is too large", (long long)M,
                         (long long)K, (long long)N);
    return tc_gemm_presplit(a_hi, a_lo, b_hi, b_lo, c, M, K, N, trans_a, trans_b, bias, mask, act, 1, 0, 0, s,
                            out_lines, mask_bits, act_bits);
}

int j4c_dot_split_ep_max(const float *a_hi, const float *a_lo, const float *b_hi, const float *b_lo, float *c,
                         int64_t M, int64_t K, int64_t N, int trans_a, int trans_b, const float *bias,
                         const float *mask, float *act, uint32_t *out_lines, j4c_stream stream) {
    return j4c_dot_split_ep_bits(a_hi, a_lo, b_hi, b_lo, c, M, K, N, trans_a, trans_b, bias, mask, nullptr, act,
                                 nullptr, out_lines, stream);
}

int j4c_dot_split_ep(const float *a_hi, const float *a_lo, const float *b_hi, const float *b_lo, float *c,
                     int64_t M, int64_t K, int64_t N, int trans_a, int trans_b, const float *bias,
                     const float *mask, float *act, j4c_stream stream) {
    return j4c_dot_split_ep_max(a_hi, a_lo, b_hi, b_lo, c, M, K, N, trans_a, trans_b, bias, mask, act, nullptr,
                                stream);
}

int j4c_dot_split_batched(const float *a_hi, const float *a_lo, const float *b_hi, const float *b_lo, float *c,
                          int64_t batch, int64_t M, int64_t K, int64_t N, int trans_a, int trans_b,
                          int a_batched, int b_batched, j4c_stream stream) {
    J4C_REQUIRE(batch >= 0 && M >= 0 && K >= 0 && N >= 0, "j4c_dot_split_batched: negative dimension");
    if (batch == 0 || M == 0 || N == 0) return J4C_OK;
    J4C_REQUIRE(c, "j4c_dot_split_batched: NULL output");
    if (K == 0) return j4c_fill(J4C_FLOAT32, c, batch * M * N, 0.0, stream);
    J4C_REQUIRE(a_hi && a_lo && b_hi && b_lo, "j4c_dot_split_batched: NULL operand");
    J4C_REQUIRE(batch < (1ll << 31), "j4c_dot_split_batched: batch too large");
    if (!tc_gemm_supported(M, K, N))
        return set_error(J4C_E_UNSUPPORTED, "j4c_dot_split_batched: shape %lld x %lld x %lld is too large",
                         (long long)M, (long long)K, (long long)N);
    J4C_REQUIRE(!(trans_a && !trans_b),
                "j4c_dot_split_batched: A^T . B takes one operand's transposed split (flip its flag)");
    return tc_gemm_presplit(a_hi, a_lo, b_hi, b_lo, c, M, K, N, trans_a, trans_b, nullptr, nullptr, nullptr,
                            batch, a_batched, b_batched, as_stream(stream));
}

int j4c_dot_split(const float *a_hi, const float *a_lo, const float *b_hi, const float *b_lo, float *c,
                  int64_t M, int64_t K, int64_t N, int trans_a, int trans_b, j4c_stream stream) {
    return j4c_dot_split_ep(a_hi, a_lo, b_hi, b_lo, c, M, K, N, trans_a, trans_b, nullptr, nullptr, nullptr,
                            stream);
}

}  // extern "C"
