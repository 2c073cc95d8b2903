// Device math shared by the chain interpreter (map.cu), the softmax kernels
// (softmax.cu) and the chain kernels compiled at run time (chain_jit.cpp),
// which embeds this file's text and compiles it with NVRTC: it includes no
// header and uses only builtin types, so both compilers see the same code
// and the compiled chains round exactly as the interpreter does.
#pragma once

namespace mlkb::dev {

// f64 argument reduction by pi/2 for |u| < 2^20 (Cody-Waite, two-term
// constant, FMA). r1 = u - k*P1 is exact (both terms are multiples of 2^-52
// or finer and |r1| < 1 fits in 53 bits); the second term carries pi/2 - P1.
// Returns k mod 4 in q.
__device__ __forceinline__ double reduce_pio2(double u, int& q) {
    const double kTwoOverPi = 0.6366197723675814;   // fl64(2/pi)
    const double kP1 = 1.5707963267948966;            // fl64(pi/2)
    const double kP2 = 6.123233995736766e-17;           // fl64(pi/2 - kP1)
    const double kMagic = 6755399441055744.0;            // 1.5 * 2^52
    const double t = fma(u, kTwoOverPi, kMagic);
    const double kd = t - kMagic;
    q = __double2loint(t);
    const double r1 = fma(-kd, kP1, u);
    return fma(-kd, kP2, r1);
}

// sin and cos of the reduced argument |r| <= pi/4 (+ a rounding margin),
// Taylor series through r^17 (sin) and r^16 (cos), Horner form in f64:
// truncation below 1e-19 / 3e-18, so both are accurate to about an f64 ulp,
// as the host libm the reference calls is. (A value that later cancels
// against a nearby constant in a chain must be as accurate as the
// reference's, or the cancellation magnifies the difference.)
__device__ __forceinline__ double sin_poly(double r, double z) {
    double p = 2.8114572543455206e-15;     // 1/17!
    p = fma(z, p, -7.647163731819816e-13);   // -1/15!
    p = fma(z, p, 1.6059043836821613e-10);   // 1/13!
    p = fma(z, p, -2.505210838544172e-08);   // -1/11!
    p = fma(z, p, 2.7557319223985893e-06);   // 1/9!
    p = fma(z, p, -1.984126984126984e-04);   // -1/7!
    p = fma(z, p, 8.333333333333333e-03);    // 1/5!
    p = fma(z, p, -1.6666666666666666e-01);  // -1/3!
    return fma(r * z, p, r);
}

__device__ __forceinline__ double cos_poly(double z) {
    double p = 4.779477332387385e-14;      // 1/16!
    p = fma(z, p, -1.1470745597729725e-11);  // -1/14!
    p = fma(z, p, 2.08767569878681e-09);     // 1/12!
    p = fma(z, p, -2.755731922398589e-07);   // -1/10!
    p = fma(z, p, 2.48015873015873e-05);     // 1/8!
    p = fma(z, p, -1.388888888888889e-03);   // -1/6!
    p = fma(z, p, 4.1666666666666664e-02);   // 1/4!
    p = fma(z, p, -0.5);
    return fma(z, p, 1.0);
}

// sin(u), cos(u) in f64 for any u: the reduction above for |u| < 2^20,
// CUDA's own sincos otherwise (and for NaN / inf).
__device__ __forceinline__ void sincos_f64(double u, double& s, double& c) {
    if (fabs(u) < 1048576.0) {
        int q;
        const double r = reduce_pio2(u, q);
        const double z = r * r;
        const double sr = sin_poly(r, z);
        const double cr = cos_poly(z);
        // quadrant q: (sin, cos) = (sr, cr), (cr, -sr), (-sr, -cr), (-cr, sr)
        const double a = (q & 1) ? cr : sr;
        const double b = (q & 1) ? sr : cr;
        s = (q & 2) ? -a : a;
        c = ((q + 1) & 2) ? -b : b;
    } else {
        ::sincos(u, &s, &c);
    }
}

// sin(r) for |r| <= pi/2 (+ a rounding margin): the Taylor series through
// r^21 (truncation below 2e-18), Horner form in f64.
__device__ __forceinline__ double sin_half(double r) {
    const double z = r * r;
    double p = 1.9572941063391263e-20;       // 1/21!
    p = fma(z, p, -8.22063524662433e-18);    // -1/19!
    p = fma(z, p, 2.8114572543455206e-15);   // 1/17!
    p = fma(z, p, -7.647163731819816e-13);   // -1/15!
    p = fma(z, p, 1.6059043836821613e-10);   // 1/13!
    p = fma(z, p, -2.505210838544172e-08);   // -1/11!
    p = fma(z, p, 2.7557319223985893e-06);   // 1/9!
    p = fma(z, p, -1.984126984126984e-04);   // -1/7!
    p = fma(z, p, 8.333333333333333e-03);    // 1/5!
    p = fma(z, p, -1.6666666666666666e-01);  // -1/3!
    return fma(r * z, p, r);
}

// sin(u) alone, for |u| < 2^20: u = k*pi + r with |r| <= pi/2 and
// sin(u) = (-1)^k sin(r). One odd series and a sign, no quadrant select: the
// reduced argument is small exactly where sin(u) is, so the result keeps
// its relative accuracy near the zeros. The first reduction step is exact
// (for k != 0, |u| >= pi/2: u and k*fl(pi) are multiples of 2^-52 and their
// difference is below 2); the second carries pi - fl(pi).
__device__ __forceinline__ double sin_f64(double u) {
    if (fabs(u) < 1048576.0) {
        const double kInvPi = 0.3183098861837907;      // fl64(1/pi)
        const double kPiHi = 3.141592653589793;        // fl64(pi)
        const double kPiLo = 1.2246467991473532e-16;   // fl64(pi - kPiHi)
        const double kMagic = 6755399441055744.0;      // 1.5 * 2^52
        const double t = fma(u, kInvPi, kMagic);
        const double kd = t - kMagic;
        const int k = __double2loint(t);
        const double v = sin_half(fma(-kd, kPiLo, fma(-kd, kPiHi, u)));
        return (k & 1) ? -v : v;
    }
    return ::sin(u);
}

// cos(u) alone, for |u| < 2^20: u = (k + 1/2)*pi + r with |r| <= pi/2 (+ a
// margin) and cos(u) = (-1)^(k+1) sin(r); r = u - m*pi/2 with m = 2k + 1,
// in two steps as above (the first exact). Near the zeros of cos, r is small
// and the result keeps its relative accuracy.
__device__ __forceinline__ double cos_f64(double u) {
    if (fabs(u) < 1048576.0) {
        const double kInvPi = 0.3183098861837907;      // fl64(1/pi)
        const double kP1 = 1.5707963267948966;         // fl64(pi/2)
        const double kP2 = 6.123233995736766e-17;      // fl64(pi/2 - kP1)
        const double kMagic = 6755399441055744.0;      // 1.5 * 2^52
        const double t = fma(u, kInvPi, -0.5) + kMagic;  // rint(u/pi - 1/2), by rounding
        const double kd = t - kMagic;
        const int k = __double2loint(t);
        const double m = fma(2.0, kd, 1.0);              // exact
        const double v = sin_half(fma(-m, kP2, fma(-m, kP1, u)));
        return (k & 1) ? v : -v;
    }
    double s, c;
    ::sincos(u, &s, &c);
    return c;
}

// exp(d) in f64 for d <= 0 (softmax exponents). Values below -120 return 0:
// they lie under half the smallest f32 subnormal times any row sum >= 1, and
// add nothing to an f64 sum >= 1. NaN propagates; -inf gives 0.
// Method: k = rint(d/ln2) by the 1.5*2^52 shifter, r = d - k*ln2 with a
// two-term ln2 (the first product is exact under FMA), Taylor series of e^r
// through r^8 on |r| <= ln2/2 (truncation < 3e-10 relative), scale by 2^k.
__device__ __forceinline__ double exp_neg_f64(double d) {
    if (!(d >= -120.0)) return (d != d) ? d : 0.0;
    const double kLog2e = 1.4426950408889634;
    const double kLn2Hi = 0.6931471805599453;    // fl64(ln 2)
    const double kLn2Lo = 2.3190468138462996e-17;  // fl64(ln 2 - kLn2Hi)
    const double kMagic = 6755399441055744.0;
    const double t = fma(d, kLog2e, kMagic);
    const double kd = t - kMagic;
    const int k = __double2loint(t);
    double r = fma(-kd, kLn2Hi, d);
    r = fma(-kd, kLn2Lo, r);
    double p = 2.48015873015873e-05;     // 1/8!
    p = fma(r, p, 1.984126984126984e-04);   // 1/7!
    p = fma(r, p, 1.388888888888889e-03);   // 1/6!
    p = fma(r, p, 8.333333333333333e-03);   // 1/5!
    p = fma(r, p, 4.1666666666666664e-02);   // 1/4!
    p = fma(r, p, 1.6666666666666666e-01);   // 1/3!
    p = fma(r, p, 0.5);
    p = fma(r, p, 1.0);
    p = fma(r, p, 1.0);
    // 2^k for -175 <= k <= 1 is a normal double: build its bit pattern.
    const double scale = __hiloint2double((k + 1023) << 20, 0);
    return p * scale;
}

}  // namespace mlkb::dev

namespace mlkb::chain {

// MathOp / KernelOperand::Kind numbering (include/mlkb200.h).
enum : unsigned char {
    kAdd = 0, kSub, kMul, kDiv, kNeg, kPow, kExp, kLog, kSin, kCos, kTan,
    kTanh, kSqrt, kRsqrt, kErf, kGelu
};
enum : unsigned char { kConst = 0, kElemA, kElemB, kScalar, kTemp };

// The reference's "poly7" sine family, families::polySin
// (compiler/include/mlk/support/math_families.h:22-90): Cody-Waite reduction
// by pi/2 = hi + lo, then a degree-13 odd sine or degree-12 even cosine
// residual polynomial on [-pi/4, pi/4] picked by the quadrant. The reference
// evaluates it in plain IEEE f64 without contraction; every step here is the
// same correctly rounded operation in the same order (__d*_rn, no FMA), so
// the result is bit-identical. The coefficients are the reference's own
// published constants (math_families.h:30-35, :49-54).
// The sine (cosine = false) or cosine residual polynomial of the poly7
// family for the reduced argument x, as one chain of the same correctly
// rounded steps with per-element coefficient selects, so lanes of a warp in
// different quadrants run one path: sine x + (x*r2)*p, cosine
// (1 - r2*0.5) + (r2*r2)*p, each p a 6-coefficient Horner chain in r2.
__device__ __forceinline__ double poly7_residual(double x, bool cosine) {
    const double r2 = __dmul_rn(x, x);
    double p = cosine ? -1.13585365213876817300e-11 : 1.58962301576546568060e-10;
    p = __dadd_rn(__dmul_rn(p, r2), cosine ? 2.08757530072652689750e-9 : -2.50507477628578072866e-8);
    p = __dadd_rn(__dmul_rn(p, r2), cosine ? -2.75573142103085808917e-7 : 2.75573136213857245213e-6);
    p = __dadd_rn(__dmul_rn(p, r2), cosine ? 2.48015872890001867312e-5 : -1.98412698295895385996e-4);
    p = __dadd_rn(__dmul_rn(p, r2), cosine ? -1.38888888888783992457e-3 : 8.33333333332211858878e-3);
    p = __dadd_rn(__dmul_rn(p, r2), cosine ? 4.16666666666666435770e-2 : -1.66666666666666307295e-1);
    const double head = cosine ? __dsub_rn(1.0, __dmul_rn(r2, 0.5)) : x;
    const double scale = cosine ? __dmul_rn(r2, r2) : __dmul_rn(x, r2);
    return __dadd_rn(head, __dmul_rn(scale, p));
}

__device__ __forceinline__ double poly7_sin(double x) {
    const double kPio2Hi = 1.5707963267948965580e+00;  // also the reference's kPiHalf
    const double kPio2Lo = 6.1232339957367660359e-17;
    const double n = floor(__dadd_rn(__ddiv_rn(x, kPio2Hi), 0.5));
    const double r = __dsub_rn(__dsub_rn(x, __dmul_rn(n, kPio2Hi)), __dmul_rn(n, kPio2Lo));
    // The reference takes fmod(n, 4) of the integer-valued n; every step of
    // n - 4*trunc(n/4) is exact, so it is the same remainder (a zero may
    // differ in sign, which does not change the quadrant). For x NaN or
    // infinite it is NaN and r is NaN: the reference converts that NaN to
    // int (INT_MIN on its x86-64 host) and its switch takes the default
    // branch, -cos(r); the same branch here keeps even the NaN's sign
    // bit-identical.
    const double f = n - 4.0 * trunc(n * 0.25);
    int q = (f == f) ? static_cast<int>(f) : 3;
    if (q < 0) q += 4;
    const double v = poly7_residual(r, (q & 1) != 0);  // quadrants 1, 3: cosine
    return q >= 2 ? -v : v;
}

// kF64Out: the chain result is stored in f64, so sin/cos use CUDA's double
// routines (about 1 ULP of f64); f32 outputs use the fast reduction +
// polynomial path above, whose error is far below f32 resolution. With
// `poly7` Sin is the reference's poly7 family in either case (Cos and the
// other ops keep the libm family, as resolveFamily does,
// kernel_buffers.cpp:42-51).
template <bool kF64Out>
__device__ __forceinline__ double apply(unsigned op, double a, double b, bool poly7) {
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
        case kCos: return kF64Out ? ::cos(a) : dev::cos_f64(a);
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

}  // namespace mlkb::chain
