// Shared device/host helpers for libmlkb200 (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

#include "../../include/mlkb200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libmlkb200 is built for sm_100a only"
#endif

namespace mlkb {

// Records `msg` as this thread's last error and returns `code`.
int setError(int code, const char* msg);
int setCudaError(int code, cudaError_t e, const char* what);
int okStatus();

inline cudaStream_t asStream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Number of SMs of the current device (cached per device).
int smCount();

// The current device's status word (device memory, allocated once per
// device): kernels whose bounded waits give up store MLKB_ERR_TIMEOUT there;
// mlkb_take_device_error() reads and clears it. nullptr if allocation failed.
int* deviceStatusPtr();

// Scaled-scores softmax Y[b] = softmax_rows(scale * Q[b] K[b]^T), Q [batch, m,
// d] f16; K given as [batch, s, d] (kt false) or as Kt [batch, d, s] (kt
// true); Y [batch, m, s] f32 (qk_softmax.cu).
int launchQkSoftmax(const void* q, const void* k, float* y, int64_t batch, int64_t m, int64_t s,
                    int64_t d, double scale, bool kt, cudaStream_t st);

// Launch-check helper: maps a launch error to MLKB_ERR_LAUNCH.
inline int checkLaunch(const char* what) {
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? okStatus() : setCudaError(MLKB_ERR_LAUNCH, e, what);
}

inline bool aligned16(const void* p) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

}  // namespace mlkb

// ---- device math helpers ----------------------------------------------------
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
// Taylor series through r^11 (sin) and r^12 (cos), Horner form in f64.
// Truncation error < 1e-11 relative, far below f32 resolution.
__device__ __forceinline__ double sin_poly(double r, double z) {
    double p = -2.505210838544172e-08;   // -1/11!
    p = fma(z, p, 2.7557319223985893e-06);  // 1/9!
    p = fma(z, p, -1.984126984126984e-04); // -1/7!
    p = fma(z, p, 8.333333333333333e-03);  // 1/5!
    p = fma(z, p, -1.6666666666666666e-01); // -1/3!
    return fma(r * z, p, r);
}

__device__ __forceinline__ double cos_poly(double z) {
    double p = 2.08767569878681e-09;     // 1/12!
    p = fma(z, p, -2.755731922398589e-07);  // -1/10!
    p = fma(z, p, 2.48015873015873e-05);   // 1/8!
    p = fma(z, p, -1.388888888888889e-03);  // -1/6!
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

__device__ __forceinline__ double sin_f64(double u) {
    if (fabs(u) < 1048576.0) {
        int q;
        const double r = reduce_pio2(u, q);
        const double z = r * r;
        const double v = (q & 1) ? cos_poly(z) : sin_poly(r, z);
        return (q & 2) ? -v : v;
    }
    return ::sin(u);
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
