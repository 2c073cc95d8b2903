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
//   * mlkb_map_chain for any chain of scalar-realisable ops: a kernel
//     compiled at run time for the chain (chain_jit.cpp) when NVRTC is
//     available, else the chain interpreter here (register-slot form for
//     chains with at most 8 temps alive at once and 16-byte aligned buffers,
//     a local-array form otherwise); both use chain_math.cuh's apply<>,
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

// |x| < 1000 keeps |u| < 2^20, the range of the two-term reduction. A NaN
// takes the fast path, whose arithmetic carries the NaN through to both
// outputs; inf and |x| >= 1000 take the slow one. The choice is made per
// element, so an element's result never depends on its neighbours or on the
// buffers' alignment (a shard boundary or an unaligned buffer gives the same
// bits as the vector path).
__device__ __forceinline__ bool fast_elem(float x) { return !(fabsf(x) >= 1000.0f); }

__device__ __forceinline__ bool fast_range(float4 v) {
    return fast_elem(v.x) && fast_elem(v.y) && fast_elem(v.z) && fast_elem(v.w);
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

// One element, the path fast_elem picks for it.
template <class Op>
__device__ __forceinline__ void eval1(float x, float& o0, float& o1) {
    if (fast_elem(x)) {
        Op::fast(x, o0, o1);
    } else {
        const float2 r = Op::slow(x);
        o0 = r.x;
        o1 = r.y;
    }
}

template <class Op>
__device__ __forceinline__ void eval4(float4 v, float4& o0, float4& o1) {
    if (fast_range(v)) {
        Op::fast(v.x, o0.x, o1.x);
        Op::fast(v.y, o0.y, o1.y);
        Op::fast(v.z, o0.z, o1.z);
        Op::fast(v.w, o0.w, o1.w);
    } else {  // inf or |x| >= 1000 somewhere in the vector: each lane on its own
        eval1<Op>(v.x, o0.x, o1.x);
        eval1<Op>(v.y, o0.y, o1.y);
        eval1<Op>(v.z, o0.z, o1.z);
        eval1<Op>(v.w, o0.w, o1.w);
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

// Scalar body for the ragged tail or unaligned pointers (per element the same
// arithmetic as the vector body).
template <class Op>
__global__ void map_scalar_kernel(const float* __restrict__ x, float* __restrict__ y0,
                                  float* __restrict__ y1, int64_t begin, int64_t n) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = begin + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
         i < n; i += stride) {
        float o0, o1 = 0.0f;
        eval1<Op>(x[i], o0, o1);
        y0[i] = o0;
        if (Op::kOuts > 1) y1[i] = o1;
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

using namespace chain;  // op and operand numbering, poly7, apply<> (chain_math.cuh)

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
// `code` is the expression's fused form (below) or -1.
struct SlotExpr {
    uint8_t op, asrc, bsrc, dst;
    int32_t code;
    double aval, bval;
};

// Fused forms, for the 4-slot instance: an Add, Sub or Mul (op 0..2) whose
// operand sources (0..6) and destination slot (0..3) are folded into one
// case label, ((op·7 + asrc)·7 + bsrc)·4 + dst, so the whole expression —
// both operand reads, the arithmetic over 4 elements and the slot write — is
// one jump-table dispatch with static register operands, instead of one
// switch per operand, per operation and per write.
constexpr int kFusedSrcs = 7;
constexpr int kFusedSlots = 4;
constexpr int kFusedOps = 3;

__host__ __device__ constexpr int fusedCode(int op, int asrc, int bsrc, int dst) {
    return ((op * kFusedSrcs + asrc) * kFusedSrcs + bsrc) * kFusedSlots + dst;
}

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

template <int S, int R>
__device__ __forceinline__ double fusedSrc(const double (&t)[R][4], const double (&va)[4],
                                           const double (&vb)[4], double c, int q) {
    if constexpr (S == 0) return c;
    else if constexpr (S == 1) return va[q];
    else if constexpr (S == 2) return vb[q];
    else return t[S - 3][q];
}

template <int O, int A, int B, int D, int R>
__device__ __forceinline__ void fusedStep(double (&t)[R][4], const double (&va)[4],
                                          const double (&vb)[4], double av, double bv) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const double x = fusedSrc<A, R>(t, va, vb, av, q);
        const double y = fusedSrc<B, R>(t, va, vb, bv, q);
        t[D][q] = O == kAdd ? __dadd_rn(x, y) : O == kSub ? __dsub_rn(x, y) : __dmul_rn(x, y);
    }
}

// One expression of the 4-slot instance: its fused case when it has one,
// else the operand / operation / write switches.
template <bool kF64Out>
__device__ __forceinline__ void fusedOrGeneric(const SlotExpr& e, double (&t)[4][4],
                                               const double (&va)[4], const double (&vb)[4],
                                               bool poly7) {
#define MLKB_FC(o, a, b, d)                                       \
    case fusedCode(o, a, b, d):                                   \
        fusedStep<o, a, b, d, 4>(t, va, vb, e.aval, e.bval);      \
        break;
#define MLKB_FC_D(o, a, b) MLKB_FC(o, a, b, 0) MLKB_FC(o, a, b, 1) MLKB_FC(o, a, b, 2) MLKB_FC(o, a, b, 3)
#define MLKB_FC_B(o, a)                                                                    \
    MLKB_FC_D(o, a, 0) MLKB_FC_D(o, a, 1) MLKB_FC_D(o, a, 2) MLKB_FC_D(o, a, 3)             \
    MLKB_FC_D(o, a, 4) MLKB_FC_D(o, a, 5) MLKB_FC_D(o, a, 6)
#define MLKB_FC_A(o)                                                                       \
    MLKB_FC_B(o, 0) MLKB_FC_B(o, 1) MLKB_FC_B(o, 2) MLKB_FC_B(o, 3) MLKB_FC_B(o, 4)         \
    MLKB_FC_B(o, 5) MLKB_FC_B(o, 6)
    switch (e.code) {
        MLKB_FC_A(0) MLKB_FC_A(1) MLKB_FC_A(2)
        default: {
            double x[4], y[4], r[4];
            fetch4<4>(e.asrc, e.aval, va, vb, t, x);
            fetch4<4>(e.bsrc, e.bval, va, vb, t, y);
            apply4<kF64Out>(e.op, x, y, r, poly7);
            put4<4>(e.dst, t, r);
        }
    }
#undef MLKB_FC_A
#undef MLKB_FC_B
#undef MLKB_FC_D
#undef MLKB_FC
}
static_assert(kAdd == 0 && kSub == 1 && kMul == 2, "fused op numbering");

template <typename T>
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
                 "l"(src), "r"(bytes)
                 : "memory");
}

template <typename T, int R>
__global__ void __launch_bounds__(kChainThreads, 2)
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
            if constexpr (R == kFusedSlots) {
                fusedOrGeneric<sizeof(T) == 8>(e, t, va, vb, p.poly7 != 0);
            } else {
                double x[4], y[4], r[4];
                fetch4<R>(e.asrc, e.aval, va, vb, t, x);
                fetch4<R>(e.bsrc, e.bval, va, vb, t, y);
                apply4<sizeof(T) == 8>(e.op, x, y, r, p.poly7 != 0);
                put4<R>(e.dst, t, r);
            }
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
    for (int k = 0; k < n; ++k) {
        SlotExpr& e = sc.e[k];
        const bool fusable = used <= kFusedSlots && e.op < kFusedOps && e.asrc < kFusedSrcs &&
                             e.bsrc < kFusedSrcs && e.dst < kFusedSlots;
        e.code = fusable ? fusedCode(e.op, e.asrc, e.bsrc, e.dst) : -1;
    }
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

namespace {

// The device form of a host chain; a ScalarParam operand becomes the
// constant scalars[idx] (0 past the table's end), as the reference reads it
// (kernel_buffers.cpp:114-117).
void fillChainParams(const mlkb_expr* exprs, int32_t n_exprs, int32_t poly7_sin,
                     const double* scalars, int64_t n_scalars, ChainParams& p) {
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
}

void toJit(const ChainParams& p, JitExpr* je) {
    for (int k = 0; k < p.n_exprs; ++k) {
        const DevExpr& e = p.e[k];
        je[k] = JitExpr{e.op, e.akind, e.bkind, e.unary, e.aidx, e.bidx, e.aval, e.bval};
    }
}

}  // namespace
}  // namespace mlkb

namespace mlkb {
int toJitChain(const mlkb_expr* exprs, int32_t n_exprs, bool has_b, const double* scalars,
               int64_t n_scalars, JitExpr* out) {
    if (int st = checkChain(exprs, n_exprs, has_b)) return st;
    if (n_scalars < 0 || (n_scalars > 0 && scalars == nullptr)) {
        return setError(MLKB_ERR_INVALID, "chain: bad scalar table");
    }
    ChainParams p{};
    fillChainParams(exprs, n_exprs, 0, scalars, n_scalars, p);
    toJit(p, out);
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
    fillChainParams(exprs, n_exprs, poly7_sin, scalars, n_scalars, p);
    cudaStream_t s = asStream(stream);
    // A compiled straight-line kernel for the chain when run-time
    // compilation is available (chain_jit.cpp), else an interpreter.
    {
        JitExpr je[kMaxExprs];
        toJit(p, je);
        const int st = launchChainJit(je, n_exprs, p.poly7 != 0, a, b, out, elem_dtype, n, s);
        if (st != kJitUnavailable) return st;
    }
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

extern "C" int mlkb_chain_build(const mlkb_expr* exprs, int32_t n_exprs, int32_t poly7_sin,
                                int32_t elem_dtype, int32_t has_b) {
    using namespace mlkb;
    if (int st = checkChain(exprs, n_exprs, has_b != 0)) return st;
    if (elem_dtype != MLKB_F32 && elem_dtype != MLKB_F64) {
        return setError(MLKB_ERR_INVALID, "chain: element dtype must be f32 or f64");
    }
    ChainParams p{};
    fillChainParams(exprs, n_exprs, poly7_sin, nullptr, 0, p);
    JitExpr je[kMaxExprs];
    toJit(p, je);
    const char* why = nullptr;
    if (buildChainJit(je, n_exprs, p.poly7 != 0, elem_dtype, &why) == kJitUnavailable) {
        return setError(MLKB_ERR_UNSUPPORTED, why != nullptr ? why : "chain compilation unavailable");
    }
    return okStatus();
}
