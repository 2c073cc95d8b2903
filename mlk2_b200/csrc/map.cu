// Fused elementwise maps (reference runtime/src/execution/kernel_buffers.cpp:
// ExprEvaluator :106-178, runElementwiseRange :342-402, 1-D Loop dispatch
// :921-1000).
//
// Two families:
//   * specialised streaming kernels for the chains the BASELINE configs use,
//     y = sin(x^2 + 3x) and its calculus-pass derivative
//     dy = cos(x^2 + 3x) * (2x + 3), over f32 HBM arrays. The arithmetic is
//     the reference's f64 chain: u = fl64(x*x + 3x) exactly as the reference
//     forms it (x*x and 3x are exact in f64 for f32 x, so one FMA reproduces
//     the Add's single rounding), sin/cos of u in f64, one final rounding to
//     f32. HBM-bound: 8 B (map) or 12 B (map + derivative) per element.
//   * a generic chain interpreter for any chain of scalar-realisable ops
//     (register-slot form for chains with at most 8 temps alive at once and
//     16-byte aligned buffers, a local-array form otherwise),
//     f32 or f64 buffers, with the reference's guarded semantics
//     (Div by 0 -> 0, Log of <= 0 -> 0, Sqrt of < 0 -> 0, Rsqrt of <= 0 -> 0,
//     Pow(2,2) -> a*a). Add/Sub/Mul/Div use round-to-nearest intrinsics so
//     no FMA contraction changes a rounding: arithmetic-only chains are
//     bit-exact with the reference.
#include <cuda_fp16.h>

#include <atomic>
#include <vector>

#include "common.cuh"

namespace mlkb {
namespace {

constexpr int kMapThreads = 256;

// Near-minimax polynomials on |r| <= pi/4 (fitted for this library by
// weighted least squares on Chebyshev nodes): sin r = r + r^3 S(r^2) with
// relative error < 3.9e-9, cos r = 1 + r^2 C(r^2) with relative error
// < 3.9e-8. An f32 result needs relative error below half an f32 ulp
// (2^-25 = 3e-8 at worst, 6e-8 typically) for its rounding to land within one
// ulp of the correctly rounded value; these stay there. (Degree 9/8 forms
// round ~99.97 % of outputs exactly but cost ~5 % of this HBM-bound kernel's
// time under the power cap, where the f64 pipe sets the clock.)
// cos(0) = 1 and sin(r) = r for tiny r hold exactly.
__device__ __forceinline__ double sin_r(double r, double z) {
    double p = fma(z, -0.0001951397821210659, 0.008332151315419242);
    p = fma(z, p, -0.16666654462992936);
    return fma(r * z, p, r);
}

__device__ __forceinline__ double cos_r(double z) {
    double p = fma(z, -0.0013590647071255219, 0.04165568770925181);
    p = fma(z, p, -0.49999883312661797);
    return fma(z, p, 1.0);
}

// u = fl64(x*x + 3x), exactly the reference chain's value: x*x and 3x are
// exact in f64 for an f32 x, so one FMA reproduces the Add's single rounding.
__device__ __forceinline__ double u_of(float x) {
    const double xd = static_cast<double>(x);
    return fma(3.0, xd, xd * xd);
}

// |x| < 1000 for all four lanes keeps |u| < 2^20, the range of the two-term
// reduction. A NaN lane is ignored by the max and takes the fast path, whose
// arithmetic carries the NaN through to both outputs; inf fails the test.
__device__ __forceinline__ bool fast_range(float4 v) {
    const float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    return m < 1000.0f;
}

// Sign bit 31 set when bit 1 of q is: the quadrant's sign flip, applied to the
// rounded f32 (round-to-nearest is symmetric, so this equals rounding -v).
__device__ __forceinline__ float flip_if(float v, int q) {
    return __uint_as_float(__float_as_uint(v) ^ ((static_cast<uint32_t>(q) << 30) & 0x80000000u));
}

// sin alone reduces by pi instead of pi/2: sin(u) = (-1)^k sin(r) with
// r = u - k*pi in [-pi/2, pi/2] (two-term pi, the first FMA term exact as
// above), and one odd polynomial r + r^3 S(r^2) of degree 9 on that range
// (near-minimax, relative error < 6.2e-9) serves every k: no quadrant select.
__device__ __forceinline__ double sin_half_period(double u, int& k) {
    const double kInvPi = 0.3183098861837907;        // fl64(1/pi)
    const double kPiHi = 3.141592653589793;          // fl64(pi)
    const double kPiLo = 1.2246467991473532e-16;     // fl64(pi - kPiHi)
    const double kMagic = 6755399441055744.0;        // 1.5 * 2^52
    const double t = fma(u, kInvPi, kMagic);
    const double kd = t - kMagic;
    k = __double2loint(t);
    const double r = fma(-kd, kPiLo, fma(-kd, kPiHi, u));
    const double z = r * r;
    double p = fma(z, 2.6054811598334154e-06, -0.00019809474742454904);
    p = fma(z, p, 0.008333064608556094);
    p = fma(z, p, -0.1666665949166532);
    return fma(r * z, p, r);
}

// Per op: kUnroll float4 vectors per thread per step (plus a prefetched
// step) and at most kBlocksPerSm blocks per SM in the grid. The two-output
// map streams 12 B per element and wants more bytes in flight and many short
// blocks the hardware can balance across SMs (measured on a 2^28 run: 4 and
// 64 take it from 0.58 to 0.49 ms at full clock); the single-output map is
// compute-heavier per byte and runs best with 2 and 8.
struct SinOp {
    static constexpr int kOuts = 1;
    static constexpr int kUnroll = 2;
    static constexpr int kBlocksPerSm = 8;
    __device__ __forceinline__ static void fast(float x, float& y0, float&) {
        int k;
        const double v = sin_half_period(u_of(x), k);
        // (-1)^k: bit 0 of k into the sign bit of the rounded result
        y0 = __uint_as_float(__float_as_uint(static_cast<float>(v)) ^
                             (static_cast<uint32_t>(k) << 31));
    }
    __device__ __noinline__ static float2 slow(float x) {
        return make_float2(static_cast<float>(dev::sin_f64(u_of(x))), 0.0f);
    }
};

struct SinDsinOp {
    static constexpr int kOuts = 2;
    static constexpr int kUnroll = 4;
    static constexpr int kBlocksPerSm = 64;
    __device__ __forceinline__ static void fast(float x, float& y0, float& y1) {
        int q;
        const double r = dev::reduce_pio2(u_of(x), q);
        const double z = r * r;
        const double sr = sin_r(r, z), cr = cos_r(z);
        // quadrant q: (sin u, cos u) = (sr, cr), (cr, -sr), (-sr, -cr), (-cr, sr)
        const bool odd = (q & 1) != 0;
        const double a = odd ? cr : sr;
        const double b = odd ? sr : cr;
        const double g = fma(2.0, static_cast<double>(x), 3.0);  // fl64(2x + 3), as the reference
        y0 = flip_if(static_cast<float>(a), q);
        y1 = flip_if(static_cast<float>(b * g), q + 1);
    }
    __device__ __noinline__ static float2 slow(float x) {
        double s, c;
        dev::sincos_f64(u_of(x), s, c);
        return make_float2(static_cast<float>(s),
                           static_cast<float>(c * fma(2.0, static_cast<double>(x), 3.0)));
    }
};

template <class Op>
__device__ __forceinline__ void eval4(float4 v, float4& o0, float4& o1) {
    if (fast_range(v)) {
        Op::fast(v.x, o0.x, o1.x);
        Op::fast(v.y, o0.y, o1.y);
        Op::fast(v.z, o0.z, o1.z);
        Op::fast(v.w, o0.w, o1.w);
    } else {  // NaN, inf or |x| >= 1000 somewhere in the vector
        const float2 a = Op::slow(v.x), b = Op::slow(v.y), c = Op::slow(v.z), d = Op::slow(v.w);
        o0 = make_float4(a.x, b.x, c.x, d.x);
        o1 = make_float4(a.y, b.y, c.y, d.y);
    }
}

// Vector body: each CTA strides over blocks of kMapThreads*Op::kUnroll
// float4; each thread keeps the next block's loads in flight while it
// computes the current one. 16-byte aligned pointers only.
template <class Op>
__global__ void __launch_bounds__(kMapThreads)
map_vec_kernel(const float4* __restrict__ x, float4* __restrict__ y0,
               float4* __restrict__ y1, int64_t nvec) {
    // Launched with programmatic stream serialization: wait until the
    // preceding grid in the stream has finished and its writes are visible,
    // then let the next grid's blocks be scheduled as ours retire (it waits
    // the same way), so back-to-back maps overlap launch and tail.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    constexpr int64_t kBlock = static_cast<int64_t>(kMapThreads) * Op::kUnroll;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kBlock;
    int64_t base = static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    float4 cur[Op::kUnroll];
#pragma unroll
    for (int u = 0; u < Op::kUnroll; ++u) {
        const int64_t i = base + u * kMapThreads;
        if (i < nvec) cur[u] = __ldcs(x + i);
    }
    for (; base < nvec; base += stride) {
        float4 nxt[Op::kUnroll];
        const int64_t nb = base + stride;
#pragma unroll
        for (int u = 0; u < Op::kUnroll; ++u) {
            const int64_t i = nb + u * kMapThreads;
            if (i < nvec) nxt[u] = __ldcs(x + i);
        }
#pragma unroll
        for (int u = 0; u < Op::kUnroll; ++u) {
            const int64_t i = base + u * kMapThreads;
            if (i < nvec) {
                float4 o0, o1;
                eval4<Op>(cur[u], o0, o1);
                __stcs(y0 + i, o0);
                if (Op::kOuts > 1) __stcs(y1 + i, o1);
            }
            cur[u] = nxt[u];
        }
    }
}

// Scalar body for the ragged tail or unaligned pointers.
template <class Op>
__global__ void map_scalar_kernel(const float* __restrict__ x, float* __restrict__ y0,
                                  float* __restrict__ y1, int64_t begin, int64_t n) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = begin + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
         i < n; i += stride) {
        const float2 o = Op::slow(x[i]);
        y0[i] = o.x;
        if (Op::kOuts > 1) y1[i] = o.y;
    }
}

int gridFor(int64_t work, int per_block, int blocks_per_sm = 8) {
    const int64_t blocks = (work + per_block - 1) / per_block;
    const int64_t cap = static_cast<int64_t>(smCount()) * blocks_per_sm;
    return static_cast<int>(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

template <class Op>
int launchMap(const float* x, float* y0, float* y1, int64_t n, void* stream) {
    if (n < 0) return setError(MLKB_ERR_INVALID, "map: negative element count");
    if (n == 0) return okStatus();
    if (x == nullptr || y0 == nullptr || (Op::kOuts > 1 && y1 == nullptr)) {
        return setError(MLKB_ERR_INVALID, "map: null buffer");
    }
    cudaStream_t s = asStream(stream);
    const bool vec = aligned16(x) && aligned16(y0) && (Op::kOuts < 2 || aligned16(y1));
    int64_t done = 0;
    if (vec && n >= 4) {
        const int64_t nvec = n / 4;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(gridFor(nvec, kMapThreads * Op::kUnroll, Op::kBlocksPerSm));
        cfg.blockDim = dim3(kMapThreads);
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        const cudaError_t le = cudaLaunchKernelEx(
            &cfg, map_vec_kernel<Op>, reinterpret_cast<const float4*>(x),
            reinterpret_cast<float4*>(y0), reinterpret_cast<float4*>(y1), nvec);
        if (le != cudaSuccess) return setCudaError(MLKB_ERR_LAUNCH, le, "map kernel launch");
        done = nvec * 4;
    }
    if (done < n) {
        map_scalar_kernel<Op><<<gridFor(n - done, 256), 256, 0, s>>>(x, y0, y1, done, n);
    }
    return checkLaunch("map kernel launch");
}

// ---- generic chain interpreter ---------------------------------------------

// MathOp / KernelOperand::Kind numbering (include/mlkb200.h).
enum : uint8_t {
    kAdd = 0, kSub, kMul, kDiv, kNeg, kPow, kExp, kLog, kSin, kCos, kTan,
    kTanh, kSqrt, kRsqrt, kErf, kGelu
};
enum : uint8_t { kConst = 0, kElemA, kElemB, kScalar, kTemp };

constexpr int kMaxExprs = 64;

struct DevExpr {
    uint8_t op, akind, bkind, unary;
    int16_t aidx, bidx;
    double aval, bval;
};

// Passed by value as a __grid_constant__ kernel parameter (about 1.6 KB), so
// a launch needs no device allocation. ScalarParam operands are resolved on
// the host into constants before launch (the reference reads scalars[idx],
// or 0 past the table's end, kernel_buffers.cpp:114-117), so the table may
// be any size.
struct ChainParams {
    int32_t n_exprs;
    int32_t poly7;
    DevExpr e[kMaxExprs];
};

// The reference's "poly7" sine family, families::polySin
// (compiler/include/mlk/support/math_families.h:22-90): Cody-Waite reduction
// by pi/2 = hi + lo, then a degree-13 odd sine or degree-12 even cosine
// residual polynomial on [-pi/4, pi/4] picked by the quadrant. The reference
// evaluates it in plain IEEE f64 without contraction; every step here is the
// same correctly rounded operation in the same order (__d*_rn, no FMA), so
// the result is bit-identical. The coefficients are the reference's own
// published constants (math_families.h:30-35, :49-54).
__device__ __forceinline__ double poly7_sin_reduced(double x) {
    const double r2 = __dmul_rn(x, x);
    double p = 1.58962301576546568060e-10;
    p = __dadd_rn(__dmul_rn(p, r2), -2.50507477628578072866e-8);
    p = __dadd_rn(__dmul_rn(p, r2), 2.75573136213857245213e-6);
    p = __dadd_rn(__dmul_rn(p, r2), -1.98412698295895385996e-4);
    p = __dadd_rn(__dmul_rn(p, r2), 8.33333333332211858878e-3);
    p = __dadd_rn(__dmul_rn(p, r2), -1.66666666666666307295e-1);
    return __dadd_rn(x, __dmul_rn(__dmul_rn(x, r2), p));  // x + x*r2*p, left to right
}

__device__ __forceinline__ double poly7_cos_reduced(double x) {
    const double r2 = __dmul_rn(x, x);
    double p = -1.13585365213876817300e-11;
    p = __dadd_rn(__dmul_rn(p, r2), 2.08757530072652689750e-9);
    p = __dadd_rn(__dmul_rn(p, r2), -2.75573142103085808917e-7);
    p = __dadd_rn(__dmul_rn(p, r2), 2.48015872890001867312e-5);
    p = __dadd_rn(__dmul_rn(p, r2), -1.38888888888783992457e-3);
    p = __dadd_rn(__dmul_rn(p, r2), 4.16666666666666435770e-2);
    // 1 - r2*0.5 + r2*r2*p, left to right
    return __dadd_rn(__dsub_rn(1.0, __dmul_rn(r2, 0.5)), __dmul_rn(__dmul_rn(r2, r2), p));
}

__device__ __forceinline__ double poly7_sin(double x) {
    const double kPio2Hi = 1.5707963267948965580e+00;  // also the reference's kPiHalf
    const double kPio2Lo = 6.1232339957367660359e-17;
    const double n = floor(__dadd_rn(__ddiv_rn(x, kPio2Hi), 0.5));
    const double r = __dsub_rn(__dsub_rn(x, __dmul_rn(n, kPio2Hi)), __dmul_rn(n, kPio2Lo));
    // For x NaN or infinite, fmod(n, 4) is NaN and r is NaN. The reference
    // converts that NaN to int (INT_MIN on its x86-64 host) and its switch
    // takes the default branch, -cos(r): the same branch here keeps even the
    // NaN's sign bit-identical.
    const double f = fmod(n, 4.0);
    int q = (f == f) ? static_cast<int>(f) : 3;
    if (q < 0) q += 4;
    switch (q) {
        case 0: return poly7_sin_reduced(r);
        case 1: return poly7_cos_reduced(r);
        case 2: return -poly7_sin_reduced(r);
        default: return -poly7_cos_reduced(r);
    }
}

// kF64Out: the chain result is stored in f64, so sin/cos use CUDA's double
// routines (about 1 ULP of f64); f32 outputs use the fast reduction +
// polynomial path above, whose error is far below f32 resolution. With
// `poly7` Sin is the reference's poly7 family in either case (Cos and the
// other ops keep the libm family, as resolveFamily does,
// kernel_buffers.cpp:42-51).
template <bool kF64Out>
__device__ __forceinline__ double apply(uint8_t op, double a, double b, bool poly7) {
    switch (op) {
        case kAdd: return __dadd_rn(a, b);
        case kSub: return __dsub_rn(a, b);
        case kMul: return __dmul_rn(a, b);
        case kDiv: return b != 0.0 ? __ddiv_rn(a, b) : 0.0;
        case kNeg: return -a;
        case kPow: return (a == 2.0 && b == 2.0) ? __dmul_rn(a, a) : ::pow(a, b);
        case kExp: return ::exp(a);
        case kLog: return a > 0.0 ? ::log(a) : 0.0;
        case kSin: return poly7 ? poly7_sin(a) : kF64Out ? ::sin(a) : dev::sin_f64(a);
        case kCos: {
            if (kF64Out) return ::cos(a);
            double s, c;
            dev::sincos_f64(a, s, c);
            return c;
        }
        case kTan: return ::tan(a);
        case kTanh: return ::tanh(a);
        case kSqrt: return a >= 0.0 ? __dsqrt_rn(a) : 0.0;
        case kRsqrt: return a > 0.0 ? __ddiv_rn(1.0, __dsqrt_rn(a)) : 0.0;
        case kErf: return ::erf(a);
        case kGelu: {
            // 0.5*a*(1 + tanh(c*(a + 0.044715*a*a*a))), left-to-right as in C++.
            const double a3 = __dmul_rn(__dmul_rn(__dmul_rn(0.044715, a), a), a);
            const double in = __dmul_rn(0.7978845608028654, __dadd_rn(a, a3));
            return __dmul_rn(__dmul_rn(0.5, a), __dadd_rn(1.0, ::tanh(in)));
        }
        default: return 0.0;
    }
}

template <typename T>
__global__ void chain_kernel(const __grid_constant__ ChainParams p,
                             const T* __restrict__ a, const T* __restrict__ b,
                             T* __restrict__ out, int64_t n) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += stride) {
        double t[kMaxExprs];
        const double va = a != nullptr ? static_cast<double>(a[i]) : 0.0;
        const double vb = b != nullptr ? static_cast<double>(b[i]) : 0.0;
        for (int k = 0; k < p.n_exprs; ++k) {
            const DevExpr& e = p.e[k];
            double x[2];
#pragma unroll
            for (int s = 0; s < 2; ++s) {
                const uint8_t kind = s == 0 ? e.akind : e.bkind;
                const int idx = s == 0 ? e.aidx : e.bidx;
                const double val = s == 0 ? e.aval : e.bval;
                double v = 0.0;
                if (kind == kConst) v = val;
                else if (kind == kElemA) v = va;
                else if (kind == kElemB) v = vb;
                else if (kind == kTemp) v = t[idx];  // 0 <= idx < k (host-checked)
                x[s] = v;
            }
            t[k] = apply<sizeof(T) == 8>(e.op, x[0], e.unary ? 0.0 : x[1], p.poly7 != 0);
        }
        out[i] = static_cast<T>(t[p.n_exprs - 1]);
    }
}

// ---- register-slot chain interpreter ---------------------------------------------
// The interpreter above keeps every temp of an element in a 64-entry
// per-thread array indexed at run time, so it lives in local memory, and it
// streams one element per thread: ~10 % of HBM bandwidth on short chains.
// This one keeps the temps in R registers (R = 4 or 8): on the host each
// expression's result is given a slot by liveness (an SSA result's slot is
// free again after its last reader), so a chain needs as many slots as it
// has temps alive at once, and every operand names a constant, ElemA, ElemB
// or a slot. Slot reads and writes are switches on a warp-uniform value whose
// cases index the register array statically. Each thread evaluates 4
// elements at a time, and its inputs arrive through a kChainStages-deep
// cp.async pipeline into shared memory (each thread copies and reads only its
// own elements, so no block barrier is needed), so the loads stay in flight
// whatever the register count.
constexpr int kChainThreads = 256;
constexpr int kChainElems = 4;                       // elements per thread per tile
constexpr int kChainTile = kChainThreads * kChainElems;
constexpr int kChainStages = 4;

// Operand sources: 0 constant, 1 ElemA, 2 ElemB, 3 + s register slot s.
struct SlotExpr {
    uint8_t op, asrc, bsrc, dst;
    int32_t pad;
    double aval, bval;
};

struct SlotChain {
    int32_t n_exprs;
    int32_t poly7;
    int32_t out_slot;
    int32_t uses_b;
    SlotExpr e[kMaxExprs];
};

template <int R>
__device__ __forceinline__ void fetch4(uint8_t src, double val, const double (&va)[4],
                                       const double (&vb)[4], const double (&t)[R][4],
                                       double (&x)[4]) {
#define MLKB_SLOT_CASE(j)                                           \
    case 3 + j:                                                     \
        if constexpr (j < R) {                                      \
            _Pragma("unroll") for (int q = 0; q < 4; ++q) x[q] = t[j][q]; \
        }                                                           \
        break;
    switch (src) {
        case 0:
#pragma unroll
            for (int q = 0; q < 4; ++q) x[q] = val;
            break;
        case 1:
#pragma unroll
            for (int q = 0; q < 4; ++q) x[q] = va[q];
            break;
        case 2:
#pragma unroll
            for (int q = 0; q < 4; ++q) x[q] = vb[q];
            break;
        MLKB_SLOT_CASE(0) MLKB_SLOT_CASE(1) MLKB_SLOT_CASE(2) MLKB_SLOT_CASE(3)
        MLKB_SLOT_CASE(4) MLKB_SLOT_CASE(5) MLKB_SLOT_CASE(6) MLKB_SLOT_CASE(7)
        default: break;
    }
#undef MLKB_SLOT_CASE
}

template <int R>
__device__ __forceinline__ void put4(uint8_t dst, double (&t)[R][4], const double (&r)[4]) {
#define MLKB_SLOT_PUT(j)                                            \
    case j:                                                         \
        if constexpr (j < R) {                                      \
            _Pragma("unroll") for (int q = 0; q < 4; ++q) t[j][q] = r[q]; \
        }                                                           \
        break;
    switch (dst) {
        MLKB_SLOT_PUT(0) MLKB_SLOT_PUT(1) MLKB_SLOT_PUT(2) MLKB_SLOT_PUT(3)
        MLKB_SLOT_PUT(4) MLKB_SLOT_PUT(5) MLKB_SLOT_PUT(6) MLKB_SLOT_PUT(7)
        default: break;
    }
#undef MLKB_SLOT_PUT
}

// The operation of one expression over 4 elements; one switch per expression,
// the same per-element arithmetic as apply<> (the reference's guards and
// rounding; poly7 for Sin when asked).
// The elementary functions, out of line: inlined four times into the
// interpreter loop they would hold its registers (and occupancy) hostage.
template <bool kF64Out>
__device__ __noinline__ double apply_call(uint8_t op, double a, double b, int poly7) {
    return apply<kF64Out>(op, a, b, poly7 != 0);
}

template <bool kF64Out>
__device__ __forceinline__ void apply4(uint8_t op, const double (&x)[4], const double (&y)[4],
                                       double (&r)[4], bool poly7) {
#define MLKB_EACH(expr) _Pragma("unroll") for (int q = 0; q < 4; ++q) { const double a = x[q]; const double b = y[q]; (void)b; r[q] = (expr); } break;
    switch (op) {
        case kAdd: MLKB_EACH(__dadd_rn(a, b))
        case kSub: MLKB_EACH(__dsub_rn(a, b))
        case kMul: MLKB_EACH(__dmul_rn(a, b))
        case kDiv: MLKB_EACH(b != 0.0 ? __ddiv_rn(a, b) : 0.0)
        case kNeg: MLKB_EACH(-a)
        default: MLKB_EACH((apply_call<kF64Out>(op, a, b, poly7 ? 1 : 0)))
    }
#undef MLKB_EACH
}

template <typename T>
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
                 "l"(src), "r"(bytes)
                 : "memory");
}

template <typename T, int R>
__global__ void __launch_bounds__(kChainThreads)
chain_tile_kernel(const __grid_constant__ SlotChain p, const T* __restrict__ a,
                  const T* __restrict__ b, T* __restrict__ out, int64_t n) {
    extern __shared__ __align__(16) uint8_t chain_smem[];
    // [stage][input][kChainTile] elements of T
    T* const tiles_smem = reinterpret_cast<T*>(chain_smem);
    const int inputs = p.uses_b ? 2 : 1;
    const int64_t tiles = (n + kChainTile - 1) / kChainTile;
    const int tid = static_cast<int>(threadIdx.x);
    constexpr int kChunks = kChainElems * static_cast<int>(sizeof(T)) / 16;  // 16 B copies per input
    constexpr int kPerChunk = 16 / static_cast<int>(sizeof(T));
    auto slot_ptr = [&](int stage, int input) {
        return tiles_smem + (static_cast<size_t>(stage) * inputs + input) * kChainTile +
               static_cast<size_t>(tid) * kChainElems;
    };
    // Copies this thread's elements of `tile` (zero past n) into `stage`.
    auto issue = [&](int64_t tile, int stage) {
        if (tile < tiles) {
            const int64_t base = tile * kChainTile + static_cast<int64_t>(tid) * kChainElems;
#pragma unroll
            for (int c = 0; c < kChunks; ++c) {
                const int64_t e0 = base + c * kPerChunk;
                const int64_t left = n - e0;
                const uint32_t bytes =
                    left <= 0 ? 0u
                              : static_cast<uint32_t>((left < kPerChunk ? left : kPerChunk) *
                                                      static_cast<int64_t>(sizeof(T)));
                const int64_t src = bytes != 0 ? e0 : 0;  // no byte is read when bytes == 0
                cp_async16<T>(slot_ptr(stage, 0) + c * kPerChunk, a + src, bytes);
                if (p.uses_b) cp_async16<T>(slot_ptr(stage, 1) + c * kPerChunk, b + src, bytes);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    const int64_t g = gridDim.x;
    int64_t tile = blockIdx.x;
#pragma unroll
    for (int st = 0; st < kChainStages - 1; ++st) issue(tile + st * g, st);
    for (int it = 0; tile < tiles; ++it, tile += g) {
        const int stage = it % kChainStages;
        asm volatile("cp.async.wait_group %0;" ::"n"(kChainStages - 2) : "memory");
        double va[4], vb[4];
        const T* sa = slot_ptr(stage, 0);
#pragma unroll
        for (int q = 0; q < 4; ++q) va[q] = static_cast<double>(sa[q]);
        if (p.uses_b) {
            const T* sb = slot_ptr(stage, 1);
#pragma unroll
            for (int q = 0; q < 4; ++q) vb[q] = static_cast<double>(sb[q]);
        } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) vb[q] = 0.0;
        }
        // the stage read above is free: refill it with the tile S-1 ahead
        issue(tile + (kChainStages - 1) * g, (it + kChainStages - 1) % kChainStages);
        double t[R][4];  // every slot is written before it is read (allocateSlots)
        for (int k = 0; k < p.n_exprs; ++k) {
            const SlotExpr& e = p.e[k];
            double x[4], y[4], r[4];
            fetch4<R>(e.asrc, e.aval, va, vb, t, x);
            fetch4<R>(e.bsrc, e.bval, va, vb, t, y);
            apply4<sizeof(T) == 8>(e.op, x, y, r, p.poly7 != 0);
            put4<R>(e.dst, t, r);
        }
        double res[4];
        fetch4<R>(static_cast<uint8_t>(3 + p.out_slot), 0.0, va, vb, t, res);
        const int64_t base = tile * kChainTile + static_cast<int64_t>(tid) * kChainElems;
        if (base + kChainElems <= n) {
            if constexpr (sizeof(T) == 4) {
                *reinterpret_cast<float4*>(out + base) =
                    make_float4(static_cast<float>(res[0]), static_cast<float>(res[1]),
                                static_cast<float>(res[2]), static_cast<float>(res[3]));
            } else {
                reinterpret_cast<double2*>(out + base)[0] = make_double2(res[0], res[1]);
                reinterpret_cast<double2*>(out + base)[1] = make_double2(res[2], res[3]);
            }
        } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                if (base + q < n) out[base + q] = static_cast<T>(res[q]);
            }
        }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
}

template <typename T, int R>
int launchChainTile(const SlotChain& sc, const void* a, const void* b, void* out, int64_t n,
                    cudaStream_t s) {
    const size_t smem = static_cast<size_t>(kChainStages) * (sc.uses_b ? 2 : 1) * kChainTile *
                        sizeof(T);
    static std::atomic<int> blocksPerSm[64];
    int dev = 0;
    cudaGetDevice(&dev);
    int per = dev >= 0 && dev < 64 ? blocksPerSm[dev].load() : 0;
    if (per == 0) {
        cudaError_t e = cudaFuncSetAttribute(chain_tile_kernel<T, R>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kChainStages * 2 * kChainTile *
                                                              sizeof(T)));
        if (e != cudaSuccess) return setCudaError(MLKB_ERR_LAUNCH, e, "chain smem attribute");
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, chain_tile_kernel<T, R>,
                                                          kChainThreads, smem);
        if (e != cudaSuccess || per <= 0) per = 1;
        if (dev >= 0 && dev < 64) blocksPerSm[dev] = per;
    }
    const int64_t tiles = (n + kChainTile - 1) / kChainTile;
    const int64_t cap = static_cast<int64_t>(smCount()) * per;
    const int grid = static_cast<int>(tiles < cap ? tiles : cap);
    chain_tile_kernel<T, R><<<grid, kChainThreads, smem, s>>>(
        sc, static_cast<const T*>(a), static_cast<const T*>(b), static_cast<T*>(out), n);
    return checkLaunch("chain kernel launch");
}

// Slots for a chain by liveness: returns the slot count, or -1 when the
// chain needs more than `limit` (or has an operand of another kind).
int allocateSlots(const DevExpr* ex, int n, int limit, SlotChain& sc) {
    std::vector<int> last(static_cast<size_t>(n), -1);
    for (int k = 0; k < n; ++k) {
        for (int side = 0; side < 2; ++side) {
            if (side == 1 && ex[k].unary) break;
            if ((side == 0 ? ex[k].akind : ex[k].bkind) == kTemp) {
                last[static_cast<size_t>(side == 0 ? ex[k].aidx : ex[k].bidx)] = k;
            }
        }
    }
    last[static_cast<size_t>(n - 1)] = n;  // the chain's result
    std::vector<int> slotOf(static_cast<size_t>(n), -1);
    std::vector<int> freeSlots;
    int used = 0;
    for (int k = 0; k < n; ++k) {
        SlotExpr& e = sc.e[k];
        e.op = ex[k].op;
        for (int side = 0; side < 2; ++side) {
            uint8_t kind = side == 0 ? ex[k].akind : ex[k].bkind;
            double val = side == 0 ? ex[k].aval : ex[k].bval;
            const int idx = side == 0 ? ex[k].aidx : ex[k].bidx;
            uint8_t src = 0;
            if (side == 1 && ex[k].unary) {
                src = 0;
                val = 0.0;
            } else if (kind == kConst) {
                src = 0;
            } else if (kind == kElemA) {
                src = 1;
            } else if (kind == kElemB) {
                src = 2;
            } else if (kind == kTemp) {
                src = static_cast<uint8_t>(3 + slotOf[static_cast<size_t>(idx)]);
            } else {
                return -1;
            }
            (side == 0 ? e.asrc : e.bsrc) = src;
            (side == 0 ? e.aval : e.bval) = val;
        }
        // Operands read for the last time here free their slots before this
        // result takes one (operands are read before the result is written).
        for (int side = 0; side < 2; ++side) {
            if (side == 1 && ex[k].unary) break;
            if ((side == 0 ? ex[k].akind : ex[k].bkind) != kTemp) continue;
            const int idx = side == 0 ? ex[k].aidx : ex[k].bidx;
            if (last[static_cast<size_t>(idx)] == k && slotOf[static_cast<size_t>(idx)] >= 0) {
                freeSlots.push_back(slotOf[static_cast<size_t>(idx)]);
                slotOf[static_cast<size_t>(idx)] = -2;  // released (both operands may name it)
            }
        }
        int slot;
        if (!freeSlots.empty()) {
            slot = freeSlots.back();
            freeSlots.pop_back();
        } else {
            slot = used++;
        }
        if (used > limit) return -1;
        slotOf[static_cast<size_t>(k)] = slot;
        e.dst = static_cast<uint8_t>(slot);
        if (last[static_cast<size_t>(k)] < 0) {  // never read: free at once
            freeSlots.push_back(slot);
            slotOf[static_cast<size_t>(k)] = -2;
        }
    }
    sc.n_exprs = n;
    sc.out_slot = slotOf[static_cast<size_t>(n - 1)] >= 0 ? slotOf[static_cast<size_t>(n - 1)]
                                                          : sc.e[n - 1].dst;
    return used;
}

}  // namespace

bool isUnaryOp(int op) {
    return op == kNeg || op == kExp || op == kLog || op == kSin || op == kCos ||
           op == kTan || op == kTanh || op == kSqrt || op == kRsqrt || op == kErf ||
           op == kGelu;
}

// Validates a host chain; returns MLKB_OK or an error status.
int checkChain(const mlkb_expr* exprs, int32_t n_exprs, bool has_b) {
    if (exprs == nullptr || n_exprs <= 0 || n_exprs > kMaxExprs) {
        return setError(MLKB_ERR_UNSUPPORTED, "chain: 1..64 expressions required");
    }
    for (int k = 0; k < n_exprs; ++k) {
        const mlkb_expr& e = exprs[k];
        if (e.op < kAdd || e.op > kGelu) {
            return setError(MLKB_ERR_UNSUPPORTED, "chain: op is not scalar-realisable");
        }
        for (int s = 0; s < 2; ++s) {
            if (s == 1 && isUnaryOp(e.op)) break;
            const int kind = s == 0 ? e.a_kind : e.b_kind;
            const int64_t idx = s == 0 ? e.a_index : e.b_index;
            if (kind < kConst || kind > kTemp) {
                return setError(MLKB_ERR_UNSUPPORTED, "chain: operand kind not 1-D");
            }
            if (kind == kElemB && !has_b) {
                return setError(MLKB_ERR_INVALID, "chain: ElemB read but no B buffer");
            }
            // Temps are SSA results of EARLIER expressions; the reference reads
            // a stale slot for anything else, which no lowering produces.
            if (kind == kTemp && (idx < 0 || idx >= k)) {
                return setError(MLKB_ERR_UNSUPPORTED, "chain: temp operand is not an earlier expression");
            }
        }
    }
    return okStatus();
}

}  // namespace mlkb

extern "C" int mlkb_map_sin_f32(const float* x, float* y, int64_t n, void* stream) {
    return mlkb::launchMap<mlkb::SinOp>(x, y, nullptr, n, stream);
}

extern "C" int mlkb_map_sin_dsin_f32(const float* x, float* y, float* dy, int64_t n,
                                     void* stream) {
    return mlkb::launchMap<mlkb::SinDsinOp>(x, y, dy, n, stream);
}

extern "C" int mlkb_map_chain(const mlkb_expr* exprs, int32_t n_exprs, int32_t poly7_sin,
                              const void* a, const void* b, void* out, int32_t elem_dtype,
                              int64_t n, const double* scalars, int64_t n_scalars,
                              void* stream) {
    using namespace mlkb;
    if (n < 0) return setError(MLKB_ERR_INVALID, "chain: negative element count");
    if (n == 0) return okStatus();
    if (out == nullptr) return setError(MLKB_ERR_INVALID, "chain: null output");
    if (int st = checkChain(exprs, n_exprs, b != nullptr)) return st;
    if (elem_dtype != MLKB_F32 && elem_dtype != MLKB_F64) {
        return setError(MLKB_ERR_INVALID, "chain: element dtype must be f32 or f64");
    }
    if (n_scalars < 0 || (n_scalars > 0 && scalars == nullptr)) {
        return setError(MLKB_ERR_INVALID, "chain: bad scalar table");
    }
    ChainParams p{};
    p.n_exprs = n_exprs;
    p.poly7 = poly7_sin != 0 ? 1 : 0;
    for (int k = 0; k < n_exprs; ++k) {
        const mlkb_expr& x = exprs[k];
        DevExpr& e = p.e[k];
        e.op = static_cast<uint8_t>(x.op);
        e.unary = isUnaryOp(x.op) ? 1 : 0;
        for (int side = 0; side < 2; ++side) {
            int kind = side == 0 ? x.a_kind : x.b_kind;
            const int64_t idx = side == 0 ? x.a_index : x.b_index;
            double val = side == 0 ? x.a_value : x.b_value;
            if (kind == kScalar) {  // a ScalarParam is a constant for the whole launch
                val = (idx >= 0 && idx < n_scalars) ? scalars[idx] : 0.0;
                kind = kConst;
            }
            (side == 0 ? e.akind : e.bkind) = static_cast<uint8_t>(kind);
            (side == 0 ? e.aidx : e.bidx) = static_cast<int16_t>(kind == kTemp ? idx : 0);
            (side == 0 ? e.aval : e.bval) = val;
        }
    }
    cudaStream_t s = asStream(stream);
    // The register-slot interpreter when the chain fits 8 slots and every
    // buffer is 16-byte aligned (cp.async and vector stores); else the
    // local-array interpreter below.
    const bool aligned = aligned16(a) && aligned16(out) && (b == nullptr || aligned16(b));
    if (aligned && a != nullptr) {
        SlotChain sc{};
        sc.poly7 = p.poly7;
        const int used = allocateSlots(p.e, n_exprs, 8, sc);
        if (used > 0) {
            bool uses_b = false;
            for (int k = 0; k < n_exprs; ++k) {
                uses_b = uses_b || sc.e[k].asrc == 2 || sc.e[k].bsrc == 2;
            }
            if (uses_b && b == nullptr) return setError(MLKB_ERR_INVALID, "chain: ElemB read but no B buffer");
            sc.uses_b = uses_b ? 1 : 0;
            if (elem_dtype == MLKB_F32) {
                return used <= 4 ? launchChainTile<float, 4>(sc, a, b, out, n, s)
                                 : launchChainTile<float, 8>(sc, a, b, out, n, s);
            }
            return used <= 4 ? launchChainTile<double, 4>(sc, a, b, out, n, s)
                             : launchChainTile<double, 8>(sc, a, b, out, n, s);
        }
    }
    const int grid = gridFor(n, 256);
    if (elem_dtype == MLKB_F32) {
        chain_kernel<float><<<grid, 256, 0, s>>>(p,
                                                 static_cast<const float*>(a),
                                                 static_cast<const float*>(b),
                                                 static_cast<float*>(out), n);
    } else {
        chain_kernel<double><<<grid, 256, 0, s>>>(p,
                                                  static_cast<const double*>(a),
                                                  static_cast<const double*>(b),
                                                  static_cast<double*>(out), n);
    }
    return checkLaunch("chain kernel launch");
}
