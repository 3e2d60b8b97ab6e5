// fused.cu -- generated kernels for fused elementwise chains with row-reduction
// tails (j4c_fused_compile / j4c_fused_launch).
//
// The reference's "JIT" (backend/TornadoJitCompiler.java:82-246) compiles a
// Jaxpr into one TornadoVM task per equation, so a chain of k elementwise
// ops streams its arrays through memory k times.  Here the host side groups a
// chain into a small SSA program; this file turns the program into CUDA C++,
// compiles it once per device with NVRTC for sm_100a, and launches it: every
// input is read once, only the values needed later are written, and
// reductions over the last axis (sum/mean/argmax/argmin) are computed in the
// same pass.  Elementwise arithmetic uses the same rounding rules as the
// unfused kernels (explicit round-to-nearest ops, no FMA contraction, Java's
// max/min and cast rules), so fused and unfused elementwise results agree bit
// for bit.
#include <nvrtc.h>

#include <algorithm>
#include <cinttypes>
#include <cstddef>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <sstream>
#include <string>
#include <vector>

#include "common.cuh"
#include "jmath.cuh"

namespace j4c {
namespace fused {

constexpr int kMaxIn = 16, kMaxOut = 16, kMaxTail = 8;

// The ABI structs' layout is what foreign callers (ctypes, Java FFM) mirror.
static_assert(sizeof(j4c_insn) == 24 && offsetof(j4c_insn, value) == 16, "j4c_insn layout");
static_assert(offsetof(j4c_program, insns) == 8 && offsetof(j4c_program, input_bcast) == 32 &&
                  offsetof(j4c_program, tail_insn) == 72 && sizeof(j4c_program) == 80,
              "j4c_program layout");

struct Args {
    const void *in[kMaxIn];
    void *out[kMaxOut];
    void *tail[kMaxTail];
};

struct Entry {
    cudaLibrary_t library = nullptr;
    cudaKernel_t flat[2] = {}, rows_warp[2] = {}, rows_block[2] = {};  // [0]: 1 element, [1]: 4 per thread
    bool needs_rows = false;  // tails or row/column-broadcast inputs
    bool wide_sum = false;    // an 8-byte SUM/MEAN tail: summed element by element, as the row reduction does
    int n_in = 0, n_out = 0, n_tail = 0;
    int in_size[kMaxIn] = {}, in_bcast[kMaxIn] = {}, out_size[kMaxOut] = {};
};

static const char *kPreamble = R"(
typedef long long i64;
#define J_INF __longlong_as_double(0x7ff0000000000000LL)
struct Args { const void *in[16]; void *out[16]; void *tail[8]; };
__device__ __forceinline__ float j_add(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float j_sub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float j_mul(float a, float b) { return __fmul_rn(a, b); }
// A zero dividend over a non-zero, non-NaN divisor: the signed zero IEEE
// division defines, answered directly (as the eager kernels do).
__device__ __forceinline__ float j_div(float a, float b) {
    if (a == 0.0f && b == b && b != 0.0f)
        return __int_as_float((__float_as_int(a) ^ __float_as_int(b)) & (int)0x80000000);
    return __fdiv_rn(a, b);
}
__device__ __forceinline__ double j_add(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double j_sub(double a, double b) { return __dsub_rn(a, b); }
__device__ __forceinline__ double j_mul(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ double j_div(double a, double b) { return __ddiv_rn(a, b); }
__device__ __forceinline__ bool j_neg(float a) { return __float_as_int(a) < 0; }
__device__ __forceinline__ bool j_neg(double a) { return __double_as_longlong(a) < 0; }
template <class T> __device__ __forceinline__ T j_max(T a, T b) {
    if (a != a) return a;
    if (a == T(0) && b == T(0) && j_neg(a)) return b;
    return (a >= b) ? a : b;
}
template <class T> __device__ __forceinline__ T j_min(T a, T b) {
    if (a != a) return a;
    if (a == T(0) && b == T(0) && j_neg(b)) return b;
    return (a <= b) ? a : b;
}
// float Math.max / Math.min in four instructions: equal operands (this
// includes +0 / -0) combine their bit patterns, which gives +0 for max and
// -0 for min; otherwise max.NaN / min.NaN return the larger / smaller value
// or NaN when either operand is NaN (as the canonical NaN).
template <> __device__ __forceinline__ float j_max<float>(float a, float b) {
    float m;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(m) : "f"(a), "f"(b));
    return a == b ? __int_as_float(__float_as_int(a) & __float_as_int(b)) : m;
}
template <> __device__ __forceinline__ float j_min<float>(float a, float b) {
    float m;
    asm("min.NaN.f32 %0, %1, %2;" : "=f"(m) : "f"(a), "f"(b));
    return a == b ? __int_as_float(__float_as_int(a) | __float_as_int(b)) : m;
}
// Per-thread asynchronous copies into shared memory (cp.async, 16 bytes):
// a thread stages its own future vectors and reads back only what it
// staged, so the wait_group on its own copies is the only ordering needed.
__device__ __forceinline__ void j_cp16(void *smem, const void *g) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(g) : "memory");
}
__device__ __forceinline__ void j_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void j_cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ float j_max_nz(float a, float b) {
    float m;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(m) : "f"(a), "f"(b));
    return m;
}
__device__ __forceinline__ float j_min_nz(float a, float b) {
    float m;
    asm("min.NaN.f32 %0, %1, %2;" : "=f"(m) : "f"(a), "f"(b));
    return m;
}
__device__ __forceinline__ float j_where(unsigned char c, float x, float y) {
    const float s = c ? x : y, t = c ? y : x;
    return __fadd_rn(s, __fmul_rn(0.0f, t));
}
template <class T> __device__ __forceinline__ T j_relu(T x) { return (T(0) >= x) ? T(0) : x; }
__device__ __forceinline__ int j_d2i(double v) {
    if (v != v) return 0;
    if (v >= 2147483647.0) return 2147483647;
    if (v <= -2147483648.0) return (-2147483647 - 1);
    return (int)v;
}
__device__ __forceinline__ i64 j_d2l(double v) {
    if (v != v) return 0;
    if (v >= 9223372036854775807.0) return 9223372036854775807LL;
    if (v <= -9223372036854775808.0) return (-9223372036854775807LL - 1);
    return (i64)v;
}
template <class T> __device__ __forceinline__ T j_warp_sum(T v) {
    for (int o = 16; o > 0; o >>= 1) v = j_add(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
// (best, bi): a lane's first strict extremum, bi < 0 when the lane saw
// none.  Combines lanes: any candidate beats none, then the larger
// (smaller) value, then the smaller index.
template <class T, bool MAX> __device__ __forceinline__ void j_warp_arg(T &best, int &bi) {
    for (int o = 16; o > 0; o >>= 1) {
        T v = __shfl_xor_sync(0xffffffffu, best, o);
        int i = __shfl_xor_sync(0xffffffffu, bi, o);
        if (i >= 0 && (bi < 0 || (MAX ? v > best : v < best) || (v == best && i < bi))) { best = v; bi = i; }
    }
}
)";

static const char *ctype(int dt) {
    switch (dt) {
    case J4C_FLOAT32: return "float";
    case J4C_FLOAT64: return "double";
    case J4C_INT32: return "int";
    case J4C_INT64: return "i64";
    case J4C_BOOL: return "unsigned char";
    default: return nullptr;
    }
}

static bool is_float(int dt) { return dt == J4C_FLOAT32 || dt == J4C_FLOAT64; }

static std::string const_literal(int dt, double v) {
    char buf[96];
    if (dt == J4C_FLOAT32) {
        float f = (float)v;
        uint32_t u;
        memcpy(&u, &f, 4);
        snprintf(buf, sizeof(buf), "__int_as_float(0x%08x)", u);
    } else if (dt == J4C_FLOAT64) {
        uint64_t u;
        memcpy(&u, &v, 8);
        snprintf(buf, sizeof(buf), "__longlong_as_double(0x%016" PRIx64 "LL)", u);
    } else if (dt == J4C_INT32) {
        snprintf(buf, sizeof(buf), "(int)%lld", (long long)v);
    } else if (dt == J4C_INT64) {
        snprintf(buf, sizeof(buf), "(i64)%lldLL", (long long)v);
    } else {
        snprintf(buf, sizeof(buf), "(unsigned char)%d", v != 0.0 ? 1 : 0);
    }
    return buf;
}

// Validates the program; returns an error code or J4C_OK.
static int validate(const j4c_program *p) {
    J4C_REQUIRE(p && p->insns && p->n_insns > 0, "fused program: no instructions");
    J4C_REQUIRE(p->n_inputs >= 0 && p->n_inputs <= kMaxIn, "fused program: at most %d inputs", kMaxIn);
    J4C_REQUIRE(p->n_outputs >= 0 && p->n_outputs <= kMaxOut, "fused program: at most %d outputs", kMaxOut);
    J4C_REQUIRE(p->n_tails >= 0 && p->n_tails <= kMaxTail, "fused program: at most %d tails", kMaxTail);
    J4C_REQUIRE(p->n_outputs + p->n_tails > 0, "fused program: nothing to write");
    for (int i = 0; i < p->n_inputs; i++) {
        J4C_REQUIRE(ctype(p->input_dtype[i]) && p->input_bcast[i] >= 0 && p->input_bcast[i] <= 3,
                    "fused program: bad input %d", i);
    }
    for (int i = 0; i < p->n_insns; i++) {
        const j4c_insn &q = p->insns[i];
        J4C_REQUIRE(ctype(q.dtype), "fused program: insn %d has bad dtype %d", i, q.dtype);
        auto opnd = [&](int k) { return k >= 0 && k < i; };
        switch (q.op) {
        case J4C_OP_INPUT:
            J4C_REQUIRE(q.a >= 0 && q.a < p->n_inputs && p->input_dtype[q.a] == q.dtype,
                        "fused program: insn %d reads a bad input", i);
            break;
        case J4C_OP_CONST: break;
        case J4C_OP_RELU_GRAD:
            J4C_REQUIRE(opnd(q.a) && opnd(q.b) && is_float(q.dtype) && p->insns[q.a].dtype == q.dtype &&
                            p->insns[q.b].dtype == q.dtype,
                        "fused program: bad relu_grad at %d", i);
            break;
        case J4C_ADD: case J4C_SUB: case J4C_MUL: case J4C_DIV: case J4C_MAX: case J4C_MIN:
            J4C_REQUIRE(opnd(q.a) && opnd(q.b) && is_float(q.dtype) && p->insns[q.a].dtype == q.dtype &&
                            p->insns[q.b].dtype == q.dtype,
                        "fused program: bad binary op at %d", i);
            break;
        case J4C_EXP: case J4C_LOG: case J4C_SIN: case J4C_COS: case J4C_TANH: case J4C_RELU:
        case J4C_SIGMOID:
            J4C_REQUIRE(opnd(q.a) && is_float(q.dtype) && p->insns[q.a].dtype == q.dtype,
                        "fused program: bad unary op at %d", i);
            break;
        case J4C_GT: case J4C_GE: case J4C_LT: case J4C_LE: case J4C_EQ: case J4C_NE:
            J4C_REQUIRE(opnd(q.a) && opnd(q.b) && q.dtype == J4C_BOOL &&
                            p->insns[q.a].dtype == p->insns[q.b].dtype && p->insns[q.a].dtype != J4C_BOOL,
                        "fused program: bad comparison at %d", i);
            break;
        case J4C_CAST: J4C_REQUIRE(opnd(q.a), "fused program: bad cast at %d", i); break;
        default: return set_error(J4C_E_INVALID, "fused program: unsupported op %d at %d", q.op, i);
        }
    }
    for (int k = 0; k < p->n_outputs; k++)
        J4C_REQUIRE(p->output_insn[k] >= 0 && p->output_insn[k] < p->n_insns, "fused program: bad output");
    for (int k = 0; k < p->n_tails; k++) {
        int t = p->tail_insn[k], op = p->tail_op[k];
        J4C_REQUIRE(t >= 0 && t < p->n_insns && is_float(p->insns[t].dtype), "fused program: bad tail");
        J4C_REQUIRE(op == J4C_SUM_AXIS || op == J4C_MEAN_AXIS || op == J4C_ARGMAX || op == J4C_ARGMIN,
                    "fused program: bad tail op %d", op);
    }
    return J4C_OK;
}

// Numpy.where's blend (api/Numpy.java:39-44): ADD(MUL(c, x), MUL(SUB(1, c), y))
// with c a BOOL cast to FLOAT32, so c is exactly 0 or 1.  With c = 1 the
// blend is x + (+0 * y), with c = 0 it is (+0 * x) + y; as IEEE addition
// commutes (signed zeros and NaN included) both are s + (+0 * t) with
// s = the selected operand and t = the other -- two selects, one multiply
// and one add instead of the cast, three multiplies/adds and a subtract,
// bit for bit the arithmetic blend (NaN and Inf in the unselected operand
// still make the result NaN).  Returns the BOOL insn and x, y.
static bool where_blend(const j4c_program *p, int i, int *cond, int *x, int *y) {
    const j4c_insn &q = p->insns[i];
    if (q.op != J4C_ADD || q.dtype != J4C_FLOAT32) return false;
    auto mul_of = [&](int k, int want, int *other) {
        const j4c_insn &m = p->insns[k];
        if (m.op != J4C_MUL || m.dtype != J4C_FLOAT32) return -1;
        const j4c_insn &a = p->insns[m.a], &b = p->insns[m.b];
        auto is_c = [&](const j4c_insn &c, int idx) {
            return want < 0 ? (c.op == J4C_CAST && p->insns[c.a].dtype == J4C_BOOL) : idx == want;
        };
        if (is_c(a, m.a)) { *other = m.b; return m.a; }
        if (is_c(b, m.b)) { *other = m.a; return m.b; }
        return -1;
    };
    for (int order = 0; order < 2; order++) {
        const int t1 = order ? q.b : q.a, t2 = order ? q.a : q.b;
        int xv, yv;
        const int c = mul_of(t1, -1, &xv);
        if (c < 0) continue;
        // the other term multiplies SUB(CONST 1, c)
        for (int k = 0; k < i; k++) {
            const j4c_insn &sb = p->insns[k];
            if (sb.op != J4C_SUB || sb.dtype != J4C_FLOAT32 || sb.b != c) continue;
            const j4c_insn &one = p->insns[sb.a];
            if (one.op != J4C_OP_CONST || one.value != 1.0) continue;
            if (mul_of(t2, k, &yv) == k) {
                *cond = p->insns[c].a;
                *x = xv;
                *y = yv;
                return true;
            }
        }
    }
    return false;
}

// A float MAX / MIN with a constant operand other than +-0: Java's Math.max /
// Math.min differ from max.NaN / min.NaN only on a +0 / -0 pair, which a
// non-zero constant rules out, so the single instruction is exact.
static bool nonzero_const(const j4c_program *p, int k) {
    const j4c_insn &c = p->insns[k];
    return c.op == J4C_OP_CONST && c.dtype == J4C_FLOAT32 && (float)c.value != 0.0f;
}

// Code for one element.  The element's inputs are read from `ld<k>` (a
// register array filled before the lane loop) and its outputs go to
// `st<k>`; lane `l` is the element's position inside the thread's group of V.
static std::string gen_element(const j4c_program *p) {
    std::ostringstream o;
    for (int i = 0; i < p->n_insns; i++) {
        const j4c_insn &q = p->insns[i];
        const char *T = ctype(q.dtype);
        o << "        const " << T << " v" << i << " = ";
        int wc, wx, wy;
        if (where_blend(p, i, &wc, &wx, &wy)) {
            o << "j_where(v" << wc << ", v" << wx << ", v" << wy << ");\n";
            continue;
        }
        if ((q.op == J4C_MAX || q.op == J4C_MIN) && q.dtype == J4C_FLOAT32 &&
            (nonzero_const(p, q.a) || nonzero_const(p, q.b))) {
            o << (q.op == J4C_MAX ? "j_max_nz(v" : "j_min_nz(v") << q.a << ", v" << q.b << ");\n";
            continue;
        }
        switch (q.op) {
        case J4C_OP_INPUT: o << "ld" << q.a << "[l];\n"; continue;
        case J4C_OP_CONST: o << const_literal(q.dtype, q.value) << ";\n"; continue;
        case J4C_OP_RELU_GRAD: o << "(v" << q.b << " > (" << T << ")0) ? v" << q.a << " : (" << T << ")0;\n"; continue;
        case J4C_ADD: o << "j_add(v" << q.a << ", v" << q.b << ");\n"; continue;
        case J4C_SUB: o << "j_sub(v" << q.a << ", v" << q.b << ");\n"; continue;
        case J4C_MUL: o << "j_mul(v" << q.a << ", v" << q.b << ");\n"; continue;
        case J4C_DIV: o << "j_div(v" << q.a << ", v" << q.b << ");\n"; continue;
        case J4C_MAX: o << "j_max(v" << q.a << ", v" << q.b << ");\n"; continue;
        case J4C_MIN: o << "j_min(v" << q.a << ", v" << q.b << ");\n"; continue;
        case J4C_GT: o << "(unsigned char)(v" << q.a << " > v" << q.b << ");\n"; continue;
        case J4C_GE: o << "(unsigned char)(v" << q.a << " >= v" << q.b << ");\n"; continue;
        case J4C_LT: o << "(unsigned char)(v" << q.a << " < v" << q.b << ");\n"; continue;
        case J4C_LE: o << "(unsigned char)(v" << q.a << " <= v" << q.b << ");\n"; continue;
        case J4C_EQ: o << "(unsigned char)(v" << q.a << " == v" << q.b << ");\n"; continue;
        case J4C_NE: o << "(unsigned char)(v" << q.a << " != v" << q.b << ");\n"; continue;
        default: break;
        }
        const bool f = q.dtype == J4C_FLOAT32;
        std::string x = "v" + std::to_string(q.a);
        switch (q.op) {
        case J4C_EXP: o << (f ? "expf(" : "exp(") << x << ");\n"; break;
        case J4C_LOG: o << (f ? "logf(" : "log(") << x << ");\n"; break;
        case J4C_SIN: o << (f ? "sinf(" : "sin(") << x << ");\n"; break;
        case J4C_COS: o << (f ? "cosf(" : "cos(") << x << ");\n"; break;
        case J4C_TANH: o << (f ? "j_tanh(" : "tanh(") << x << ");\n"; break;
        case J4C_RELU: o << "j_relu(" << x << ");\n"; break;
        case J4C_SIGMOID:  // 1 / (1 + e^-x): jmath.cuh's j_sigmoid for FP32, as the eager kernel
            if (f) o << "j_sigmoid(" << x << ");\n";
            else o << "__drcp_rn(__dadd_rn(1.0, exp(-" << x << ")));\n";
            break;
        case J4C_CAST: {
            int src = p->insns[q.a].dtype, dst = q.dtype;
            if (dst == J4C_BOOL) o << "(unsigned char)(" << x << " != 0);\n";
            else if (src == J4C_BOOL) o << "(" << x << " ? (" << T << ")1 : (" << T << ")0);\n";
            else if (dst == J4C_INT32 && is_float(src)) o << "j_d2i((double)" << x << ");\n";
            else if (dst == J4C_INT32) o << "(int)(unsigned int)(unsigned long long)(i64)" << x << ";\n";
            else if (dst == J4C_INT64 && is_float(src)) o << "j_d2l((double)" << x << ");\n";
            else o << "(" << T << ")" << x << ";\n";
            break;
        }
        default: o << "0;\n"; break;
        }
    }
    for (int k = 0; k < p->n_outputs; k++) o << "        st" << k << "[l] = v" << p->output_insn[k] << ";\n";
    return o.str();
}

static int dsize(int dt) { return dt == J4C_FLOAT64 || dt == J4C_INT64 ? 8 : dt == J4C_BOOL ? 1 : 4; }

// Row kernels with 4 elements per thread stage their full-size FP32 inputs
// through shared memory S iterations ahead (cp.async): the loads in flight
// no longer depend on how many registers the chain leaves for them (a
// thread's S - 1 future vectors per input wait in shared memory, not in
// registers), which is what keeps HBM busy while the chain computes.
// Returns the staged slot of input i, or -1.
static int staged_slot(const j4c_program *p, int i) {
    if (p->input_bcast[i] != J4C_BCAST_FULL || p->input_dtype[i] != J4C_FLOAT32) return -1;
    int k = 0;
    for (int q = 0; q < i; q++)
        if (p->input_bcast[q] == J4C_BCAST_FULL && p->input_dtype[q] == J4C_FLOAT32) k++;
    return k;
}
static int n_staged(const j4c_program *p) {
    int n = 0;
    for (int i = 0; i < p->n_inputs; i++) n += staged_slot(p, i) >= 0;
    return n;
}
// Stages in flight: S * NS * 256 threads * 16 bytes stays <= 32 KB.
static int stage_depth(const j4c_program *p) {
    const int n = n_staged(p);
    return n == 0 ? 0 : n <= 2 ? 4 : n <= 4 ? 2 : 0;
}

// Loads the V consecutive elements starting at element `base` (row/flat
// position) into ld<k>, and declares st<k>.  4-byte types move as one
// 128-bit access when V == 4; the launcher only picks V == 4 when every
// such pointer is 16-byte aligned and the extent is a multiple of 4.
static std::string gen_loads(const j4c_program *p, bool flat, int V, bool staged = false) {
    std::ostringstream o;
    for (int i = 0; i < p->n_inputs; i++) {
        const char *T = ctype(p->input_dtype[i]);
        const int b = p->input_bcast[i];
        o << "      " << T << " ld" << i << "[" << V << "];\n";
        if (staged && staged_slot(p, i) >= 0) {
            o << "      { const float4 t = s_stage[sc][" << staged_slot(p, i) << "][threadIdx.x]; ld" << i
              << "[0] = t.x; ld" << i << "[1] = t.y; ld" << i << "[2] = t.z; ld" << i << "[3] = t.w; }\n";
            continue;
        }
        std::string ptr = std::string("((const ") + T + " *)a.in[" + std::to_string(i) + "])";
        if (b == J4C_BCAST_SCALAR || b == J4C_BCAST_COL) {
            const char *at = b == J4C_BCAST_SCALAR ? "0" : "r";
            o << "      { const " << T << " t = " << ptr << "[" << at << "];";
            for (int l = 0; l < V; l++) o << " ld" << i << "[" << l << "] = t;";
            o << " }\n";
            continue;
        }
        std::string idx = flat ? "e" : (b == J4C_BCAST_ROW ? "j" : "(r * C + j)");
        if (V == 4 && dsize(p->input_dtype[i]) == 4) {
            const char *T4 = p->input_dtype[i] == J4C_FLOAT32 ? "float4" : "int4";
            o << "      { const " << T4 << " t = *(const " << T4 << " *)(" << ptr << " + " << idx << ");"
              << " ld" << i << "[0] = t.x; ld" << i << "[1] = t.y; ld" << i << "[2] = t.z; ld" << i
              << "[3] = t.w; }\n";
        } else {
            for (int l = 0; l < V; l++)
                o << "      ld" << i << "[" << l << "] = " << ptr << "[" << idx << " + " << l << "];\n";
        }
    }
    for (int k = 0; k < p->n_outputs; k++)
        o << "      " << ctype(p->insns[p->output_insn[k]].dtype) << " st" << k << "[" << V << "];\n";
    return o.str();
}

static std::string gen_stores(const j4c_program *p, bool flat, int V) {
    std::ostringstream o;
    std::string idx = flat ? "e" : "(r * C + j)";
    for (int k = 0; k < p->n_outputs; k++) {
        const int dt = p->insns[p->output_insn[k]].dtype;
        const char *T = ctype(dt);
        std::string ptr = std::string("((") + T + " *)a.out[" + std::to_string(k) + "])";
        if (V == 4 && dsize(dt) == 4) {
            const char *T4 = dt == J4C_FLOAT32 ? "float4" : "int4";
            o << "      *(" << T4 << " *)(" << ptr << " + " << idx << ") = make_" << T4 << "(st" << k << "[0], st"
              << k << "[1], st" << k << "[2], st" << k << "[3]);\n";
        } else {
            for (int l = 0; l < V; l++)
                o << "      " << ptr << "[" << idx << " + " << l << "] = st" << k << "[" << l << "];\n";
        }
    }
    return o.str();
}

static std::string gen_source(const j4c_program *p, bool *needs_rows) {
    bool rows = p->n_tails > 0;
    for (int i = 0; i < p->n_inputs; i++)
        if (p->input_bcast[i] == J4C_BCAST_ROW || p->input_bcast[i] == J4C_BCAST_COL) rows = true;
    *needs_rows = rows;
    const std::string element = gen_element(p);
    std::ostringstream o;
    o << kPreamble << J4C_MATH_SRC << "\n";
    if (!rows) {
        for (int V : {1, 4}) {
            const int S = V == 4 ? stage_depth(p) : 0;
            o << "extern \"C\" __global__ void __launch_bounds__(256) k_flat" << (V == 4 ? "4" : "")
              << "(i64 N, Args a) {\n";
            if (S > 0) {
                // the grid-stride sequence of a thread, staged S - 1 vectors ahead
                auto issue = [&](const char *eexpr, const char *slot) {
                    std::ostringstream c;
                    for (int i = 0; i < p->n_inputs; i++) {
                        const int k = staged_slot(p, i);
                        if (k < 0) continue;
                        c << "j_cp16(&s_stage[" << slot << "][" << k << "][threadIdx.x], (const float *)a.in[" << i
                          << "] + " << eexpr << "); ";
                    }
                    return c.str();
                };
                o << "    __shared__ float4 s_stage[" << S << "][" << n_staged(p) << "][256];\n"
                  << "    const i64 G4 = (i64)gridDim.x * blockDim.x * 4;\n"
                  << "    const i64 e0 = (blockIdx.x * (i64)blockDim.x + threadIdx.x) * 4;\n"
                  << "    #pragma unroll\n    for (int s = 0; s < " << S - 1 << "; s++) {\n"
                  << "      const i64 ee = e0 + (i64)s * G4;\n"
                  << "      if (ee < N) { " << issue("ee", "s") << "}\n"
                  << "      j_cp_commit();\n    }\n"
                  << "    int it = 0;\n"
                  << "    for (i64 e = e0; e < N; e += G4, it++) {\n"
                  << "      { const i64 en = e + " << S - 1 << " * G4; const int sn = (it + " << S - 1 << ") & "
                  << S - 1 << ";\n"
                  << "        if (en < N) { " << issue("en", "sn") << "}\n"
                  << "        j_cp_commit(); }\n"
                  << "      j_cp_wait<" << S - 1 << ">();\n"
                  << "      const int sc = it & " << S - 1 << ";\n"
                  << gen_loads(p, true, V, true);
            } else {
                o << "    for (i64 e = (blockIdx.x * (i64)blockDim.x + threadIdx.x) * " << V << "; e < N;\n"
                  << "         e += (i64)gridDim.x * blockDim.x * " << V << ") {\n"
                  << gen_loads(p, true, V);
            }
            o << "      #pragma unroll\n      for (int l = 0; l < " << V << "; l++) {\n"
              << element << "      }\n"
              << gen_stores(p, true, V) << "    }\n}\n";
        }
        return o.str();
    }
    // Row kernels: TPR threads per row (32: a warp per row, 256: a CTA per
    // row), each thread taking V consecutive elements per iteration.
    for (int V : {1, 4})
    for (int tpr : {32, 256}) {
        std::string name = std::string(tpr == 32 ? "k_rows_warp" : "k_rows_block") + (V == 4 ? "4" : "");
        o << "extern \"C\" __global__ void __launch_bounds__(256) " << name << "(i64 R, i64 C, Args a) {\n";
        if (tpr == 256) o << "    __shared__ double s_d[8]; __shared__ float s_f[8]; __shared__ int s_i[8];\n";
        if (V == 4 && stage_depth(p) > 0)
            o << "    __shared__ float4 s_stage[" << stage_depth(p) << "][" << n_staged(p) << "][256];\n";
        o << "    const int sub = threadIdx.x % " << tpr << ";\n"
          << "    const int rows_per_cta = 256 / " << tpr << ";\n"
          << "    for (i64 r0 = (i64)blockIdx.x * rows_per_cta; r0 < R; r0 += (i64)gridDim.x * rows_per_cta) {\n"
          << "      const i64 r = r0 + threadIdx.x / " << tpr << ";\n";
        for (int k = 0; k < p->n_tails; k++) {
            const char *T = ctype(p->insns[p->tail_insn[k]].dtype);
            int op = p->tail_op[k];
            if (op == J4C_SUM_AXIS || op == J4C_MEAN_AXIS) {
                o << "      " << T << " acc" << k << " = (" << T << ")0;\n";
            } else {
                bool mx = op == J4C_ARGMAX;
                o << "      " << T << " best" << k << " = (" << T << ")(" << (mx ? "-" : "") << "J_INF);\n"
                  << "      int bi" << k << " = -1; int nan" << k << " = 0;\n";
            }
        }
        const int S = V == 4 ? stage_depth(p) : 0;
        o << "      if (r < R) {\n";
        if (S > 0) {
            // each thread's vector j lands in slot (iteration % S); the copy
            // for iteration it + S - 1 is issued before iteration it waits
            auto issue = [&](const char *jexpr, const char *slot) {
                std::ostringstream c;
                for (int i = 0; i < p->n_inputs; i++) {
                    const int k = staged_slot(p, i);
                    if (k < 0) continue;
                    c << "j_cp16(&s_stage[" << slot << "][" << k << "][threadIdx.x], (const float *)a.in[" << i
                      << "] + r * C + " << jexpr << "); ";
                }
                return c.str();
            };
            o << "      #pragma unroll\n      for (int s = 0; s < " << S - 1 << "; s++) {\n"
              << "        const i64 jj = (i64)sub * 4 + (i64)s * " << tpr * 4 << ";\n"
              << "        if (jj < C) { " << issue("jj", "s") << "}\n"
              << "        j_cp_commit();\n      }\n"
              << "      int it = 0;\n"
              << "      for (i64 j = (i64)sub * 4; j < C; j += " << tpr * 4 << ", it++) {\n"
              << "      { const i64 jn = j + " << (S - 1) * tpr * 4 << "; const int sn = (it + " << S - 1 << ") & "
              << S - 1 << ";\n"
              << "        if (jn < C) { " << issue("jn", "sn") << "}\n"
              << "        j_cp_commit(); }\n"
              << "      j_cp_wait<" << S - 1 << ">();\n"
              << "      const int sc = it & " << S - 1 << ";\n"
              << gen_loads(p, false, V, true);
        } else {
            o << "      for (i64 j = (i64)sub * " << V << "; j < C; j += " << tpr * V << ") {\n"
              << gen_loads(p, false, V);
        }
        // a lane's sum takes its V consecutive elements as ((x0 + x1) + (x2 + x3)),
        // the order of the row reduction kernel, so fused and eager sums agree
        for (int k = 0; k < p->n_tails; k++)
            if (V == 4 && (p->tail_op[k] == J4C_SUM_AXIS || p->tail_op[k] == J4C_MEAN_AXIS))
                o << "      " << ctype(p->insns[p->tail_insn[k]].dtype) << " tv" << k << "[4];\n";
        o << "      #pragma unroll\n      for (int l = 0; l < " << V << "; l++) {\n" << element;
        for (int k = 0; k < p->n_tails; k++) {
            int op = p->tail_op[k], t = p->tail_insn[k];
            if (op == J4C_SUM_AXIS || op == J4C_MEAN_AXIS) {
                if (V == 4) o << "        tv" << k << "[l] = v" << t << ";\n";
                else o << "        acc" << k << " = j_add(acc" << k << ", v" << t << ");\n";
            } else {
                bool mx = op == J4C_ARGMAX;
                // The reference keeps the first strict extremum, starting from
                // element 0: a NaN there wins, later NaNs never compare
                // greater.  A lane sees its elements in increasing order, so a
                // strict comparison keeps its first extremum; a row of only
                // -inf (+inf for argmin) or NaN leaves no candidate and gives 0.
                o << "        if (l == 0 && j == 0 && v" << t << " != v" << t << ") nan" << k << " = 1;\n"
                  << "        if (v" << t << (mx ? " > " : " < ") << "best" << k << ") { best" << k << " = v" << t
                  << "; bi" << k << " = (int)(j + l); }\n";
            }
        }
        o << "      }\n";
        if (V == 4)
            for (int k = 0; k < p->n_tails; k++)
                if (p->tail_op[k] == J4C_SUM_AXIS || p->tail_op[k] == J4C_MEAN_AXIS)
                    o << "      acc" << k << " = j_add(acc" << k << ", j_add(j_add(tv" << k << "[0], tv" << k
                      << "[1]), j_add(tv" << k << "[2], tv" << k << "[3])));\n";
        o << gen_stores(p, false, V) << "      }\n      }\n";
        // reductions
        for (int k = 0; k < p->n_tails; k++) {
            int op = p->tail_op[k];
            const char *T = ctype(p->insns[p->tail_insn[k]].dtype);
            const bool dbl = p->insns[p->tail_insn[k]].dtype == J4C_FLOAT64;
            const char *S = dbl ? "s_d" : "s_f";
            if (op == J4C_SUM_AXIS || op == J4C_MEAN_AXIS) {
                o << "      acc" << k << " = j_warp_sum(acc" << k << ");\n";
                if (tpr == 256) {
                    o << "      if ((threadIdx.x & 31) == 0) " << S << "[threadIdx.x >> 5] = acc" << k << ";\n"
                      << "      __syncthreads();\n"
                      << "      if (threadIdx.x < 32) { " << T << " t = threadIdx.x < 8 ? " << S
                      << "[threadIdx.x] : (" << T << ")0; acc" << k << " = j_warp_sum(t); }\n"
                      << "      __syncthreads();\n";
                }
                o << "      if (sub == 0 && r < R) ((" << T << " *)a.tail[" << k << "])[r] = "
                  << (op == J4C_MEAN_AXIS ? "j_div(acc" + std::to_string(k) + ", (" + T + ")C)"
                                          : "acc" + std::to_string(k))
                  << ";\n";
            } else {
                const char *mx = op == J4C_ARGMAX ? "true" : "false";
                o << "      j_warp_arg<" << T << ", " << mx << ">(best" << k << ", bi" << k << ");\n";
                if (tpr == 256) {
                    o << "      if ((threadIdx.x & 31) == 0) { " << S << "[threadIdx.x >> 5] = best" << k
                      << "; s_i[threadIdx.x >> 5] = bi" << k << "; }\n"
                      << "      __syncthreads();\n"
                      << "      if (threadIdx.x < 32) { best" << k << " = threadIdx.x < 8 ? " << S
                      << "[threadIdx.x] : (" << T << ")(" << (op == J4C_ARGMAX ? "-" : "") << "J_INF); bi" << k
                      << " = threadIdx.x < 8 ? s_i[threadIdx.x] : -1; j_warp_arg<" << T << ", " << mx
                      << ">(best" << k << ", bi" << k << "); }\n"
                      << "      __syncthreads();\n";
                }
                o << "      if (sub == 0 && r < R) ((int *)a.tail[" << k << "])[r] = (nan" << k << " || bi" << k
                  << " < 0) ? 0 : bi" << k << ";\n";
            }
        }
        o << "    }\n}\n";
    }
    return o.str();
}

static std::mutex g_mu;
static std::map<std::string, std::unique_ptr<Entry>> g_cache;  // key: device + source

static int nvrtc_cubin(const std::string &src, std::vector<char> *cubin) {
    nvrtcProgram prog;
    nvrtcResult nr = nvrtcCreateProgram(&prog, src.c_str(), "j4c_fused.cu", 0, nullptr, nullptr);
    if (nr != NVRTC_SUCCESS) return set_error(J4C_E_CUDA, "nvrtcCreateProgram: %s", nvrtcGetErrorString(nr));
    // Same contraction setting as the library's own nvcc build, so the CUDA
    // math functions (expf, tanhf, ...) compile to the same code; the chain's
    // own arithmetic uses explicit round-to-nearest ops that never contract.
    const char *opts[] = {"--gpu-architecture=sm_100a", "-std=c++17", "--fmad=true"};
    nr = nvrtcCompileProgram(prog, 3, opts);
    if (nr != NVRTC_SUCCESS) {
        size_t n = 0;
        nvrtcGetProgramLogSize(prog, &n);
        std::string log(n, '\0');
        nvrtcGetProgramLog(prog, &log[0]);
        nvrtcDestroyProgram(&prog);
        return set_error(J4C_E_CUDA, "fused kernel compilation failed: %s", log.c_str());
    }
    size_t n = 0;
    nvrtcGetCUBINSize(prog, &n);
    cubin->resize(n);
    nvrtcGetCUBIN(prog, cubin->data());
    nvrtcDestroyProgram(&prog);
    return J4C_OK;
}

static int compile(const std::string &src, Entry *e) {
    std::vector<char> cubin;
    int rc = nvrtc_cubin(src, &cubin);
    if (rc) return rc;
    J4C_CUDA(cudaLibraryLoadData(&e->library, cubin.data(), nullptr, nullptr, 0, nullptr, nullptr, 0));
    if (e->needs_rows) {
        J4C_CUDA(cudaLibraryGetKernel(&e->rows_warp[0], e->library, "k_rows_warp"));
        J4C_CUDA(cudaLibraryGetKernel(&e->rows_block[0], e->library, "k_rows_block"));
        J4C_CUDA(cudaLibraryGetKernel(&e->rows_warp[1], e->library, "k_rows_warp4"));
        J4C_CUDA(cudaLibraryGetKernel(&e->rows_block[1], e->library, "k_rows_block4"));
    } else {
        J4C_CUDA(cudaLibraryGetKernel(&e->flat[0], e->library, "k_flat"));
        J4C_CUDA(cudaLibraryGetKernel(&e->flat[1], e->library, "k_flat4"));
    }
    return J4C_OK;
}

}  // namespace fused
}  // namespace j4c

using namespace j4c;
using namespace j4c::fused;

extern "C" {

int j4c_fused_compile(const j4c_program *prog, void **handle) {
    J4C_REQUIRE(handle, "j4c_fused_compile: handle is NULL");
    int rc = validate(prog);
    if (rc) return rc;
    int dev = 0;
    J4C_CUDA(cudaGetDevice(&dev));
    J4C_CUDA(cudaSetDevice(dev));  // makes the device's primary context current for the driver API
    bool needs_rows = false;
    std::string src = gen_source(prog, &needs_rows);
    std::string key = std::to_string(dev) + "\n" + src;
    std::lock_guard<std::mutex> lock(g_mu);
    auto it = g_cache.find(key);
    if (it != g_cache.end()) {
        *handle = it->second.get();
        return J4C_OK;
    }
    auto e = std::make_unique<Entry>();
    e->needs_rows = needs_rows;
    for (int k = 0; k < prog->n_tails; k++)
        if ((prog->tail_op[k] == J4C_SUM_AXIS || prog->tail_op[k] == J4C_MEAN_AXIS) &&
            dsize(prog->insns[prog->tail_insn[k]].dtype) == 8)
            e->wide_sum = true;
    e->n_in = prog->n_inputs;
    e->n_out = prog->n_outputs;
    e->n_tail = prog->n_tails;
    for (int i = 0; i < prog->n_inputs; i++) {
        e->in_size[i] = dsize(prog->input_dtype[i]);
        e->in_bcast[i] = prog->input_bcast[i];
    }
    for (int k = 0; k < prog->n_outputs; k++) e->out_size[k] = dsize(prog->insns[prog->output_insn[k]].dtype);
    rc = compile(src, e.get());
    if (rc) return rc;
    *handle = e.get();
    g_cache.emplace(key, std::move(e));
    return J4C_OK;
}

int j4c_fused_source(const j4c_program *prog, int compile, char *buf, size_t cap, size_t *len) {
    int rc = validate(prog);
    if (rc) return rc;
    bool needs_rows = false;
    std::string src = gen_source(prog, &needs_rows);
    if (len) *len = src.size() + 1;
    if (buf && cap) {
        size_t n = std::min(cap - 1, src.size());
        memcpy(buf, src.data(), n);
        buf[n] = '\0';
    }
    if (compile) {
        std::vector<char> cubin;
        return nvrtc_cubin(src, &cubin);
    }
    return J4C_OK;
}

int j4c_fused_launch(void *handle, int64_t rows, int64_t cols, const void *const *inputs,
                     void *const *outputs, void *const *tails, j4c_stream stream) {
    J4C_REQUIRE(handle, "j4c_fused_launch: NULL handle");
    J4C_REQUIRE(rows >= 0 && cols >= 0, "j4c_fused_launch: negative extent");
    const Entry *e = static_cast<const Entry *>(handle);
    if (rows == 0 || cols == 0) return J4C_OK;
    Args a;
    memset(&a, 0, sizeof(a));
    for (int i = 0; i < e->n_in; i++) a.in[i] = inputs[i];
    for (int i = 0; i < e->n_out; i++) a.out[i] = outputs[i];
    for (int i = 0; i < e->n_tail; i++) a.tail[i] = tails[i];
    // 4 elements per thread when the extent allows it and every 128-bit
    // access is aligned (4-byte types; wider and narrower types are read
    // element by element inside the 4-wide loop).
    const int64_t extent = e->needs_rows ? cols : rows * cols;
    bool v4 = extent % 4 == 0 && !(e->needs_rows && e->wide_sum);
    for (int i = 0; i < e->n_in && v4; i++)
        if (e->in_size[i] == 4 && (e->in_bcast[i] == J4C_BCAST_FULL || e->in_bcast[i] == J4C_BCAST_ROW) &&
            reinterpret_cast<uintptr_t>(a.in[i]) % 16 != 0)
            v4 = false;
    for (int k = 0; k < e->n_out && v4; k++)
        if (e->out_size[k] == 4 && reinterpret_cast<uintptr_t>(a.out[k]) % 16 != 0) v4 = false;
    const int V = v4 ? 4 : 1;
    cudaStream_t s = as_stream(stream);
    cudaError_t r;
    if (!e->needs_rows) {
        int64_t N = rows * cols;
        void *params[] = {&N, &a};
        r = cudaLaunchKernel((const void *)e->flat[v4], dim3(grid_for(ceil_div(N, (int64_t)V), 256)), dim3(256),
                             params, 0, s);
    } else if (cols >= 2048) {  // a CTA per row from 2048 columns, as the row reduction kernel
        void *params[] = {&rows, &cols, &a};
        unsigned g = (unsigned)std::min<int64_t>(rows, (int64_t)sm_count() * 8);
        r = cudaLaunchKernel((const void *)e->rows_block[v4], dim3(g), dim3(256), params, 0, s);
    } else {
        void *params[] = {&rows, &cols, &a};
        unsigned g = (unsigned)std::min<int64_t>(ceil_div(rows, (int64_t)8), (int64_t)sm_count() * 8);
        r = cudaLaunchKernel((const void *)e->rows_warp[v4], dim3(g), dim3(256), params, 0, s);
    }
    count_launch();
    if (r != cudaSuccess) return cuda_status(r, "cudaLaunchKernel(fused)");
    return J4C_OK;
}

}  // extern "C"
