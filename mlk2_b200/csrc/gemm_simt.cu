// SIMT GEMMs: f32 (FMA, no TF32) and f64 (the reference's exact order).
//
// Reference: gemmRowBlock, runtime/src/execution/kernel_buffers.cpp:406-432
// (C += A*B, row-major, i-p-j order with zero-a terms skipped).
//   * f64: one thread per C element runs p = 0..K-1 ascending with separate
//     multiply and add roundings and the a == 0 skip, over shared-memory
//     tiles, so results are bit-exact with the reference.
//   * f32: 64x64 register-blocked tiles (4x4 outputs per thread), f32 FMA
//     accumulation: the config-4' (1024^3 f32) path, vectorised and
//     double-buffered when the shape allows. Within the stated relative-error
//     bound, not bit-exact.
#include "common.cuh"

namespace mlkb {
namespace {

constexpr int kT64 = 16;

__global__ void gemm_f64_kernel(const double* __restrict__ a, const double* __restrict__ b,
                                double* __restrict__ c, int64_t m, int64_t n, int64_t k,
                                int accumulate) {
    __shared__ double as[kT64][kT64];
    __shared__ double bs[kT64][kT64 + 1];
    const int64_t row = static_cast<int64_t>(blockIdx.y) * kT64 + threadIdx.y;
    const int64_t col = static_cast<int64_t>(blockIdx.x) * kT64 + threadIdx.x;
    double acc = (accumulate && row < m && col < n) ? c[row * n + col] : 0.0;
    for (int64_t p0 = 0; p0 < k; p0 += kT64) {
        const int64_t pa = p0 + threadIdx.x, pb = p0 + threadIdx.y;
        as[threadIdx.y][threadIdx.x] = (row < m && pa < k) ? a[row * k + pa] : 0.0;
        bs[threadIdx.y][threadIdx.x] = (pb < k && col < n) ? b[pb * n + col] : 0.0;
        __syncthreads();
        const int lim = (k - p0) < kT64 ? static_cast<int>(k - p0) : kT64;
        for (int p = 0; p < lim; ++p) {
            const double aik = as[threadIdx.y][p];
            if (aik != 0.0) acc = __dadd_rn(acc, __dmul_rn(aik, bs[p][threadIdx.x]));
        }
        __syncthreads();
    }
    if (row < m && col < n) c[row * n + col] = acc;
}

constexpr int kBM = 64, kBN = 64, kBK = 16;

__global__ void __launch_bounds__(256)
gemm_f32_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ c,
                int64_t m, int64_t n, int64_t k, int accumulate) {
    __shared__ float as[kBK][kBM + 4];
    __shared__ float bs[kBK][kBN + 4];
    const int tid = threadIdx.x;
    const int tr = tid / 16, tc = tid % 16;  // 16x16 threads, 4x4 outputs each
    const int64_t row0 = static_cast<int64_t>(blockIdx.y) * kBM;
    const int64_t col0 = static_cast<int64_t>(blockIdx.x) * kBN;
    float acc[4][4] = {};
    for (int64_t p0 = 0; p0 < k; p0 += kBK) {
        // A tile [64 x 16] -> as[p][i]; B tile [16 x 64] -> bs[p][j]
        for (int e = tid; e < kBM * kBK; e += 256) {
            const int i = e / kBK, p = e % kBK;
            const int64_t gr = row0 + i, gp = p0 + p;
            as[p][i] = (gr < m && gp < k) ? a[gr * k + gp] : 0.0f;
        }
        for (int e = tid; e < kBK * kBN; e += 256) {
            const int p = e / kBN, j = e % kBN;
            const int64_t gp = p0 + p, gc = col0 + j;
            bs[p][j] = (gp < k && gc < n) ? b[gp * n + gc] : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int p = 0; p < kBK; ++p) {
            float av[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) av[i] = as[p][tr * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) bv[j] = bs[p][tc * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t r = row0 + tr * 4 + i;
        if (r >= m) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t cc = col0 + tc * 4 + j;
            if (cc >= n) continue;
            const float v = accumulate ? c[r * n + cc] + acc[i][j] : acc[i][j];
            c[r * n + cc] = v;
        }
    }
}

// Vectorised f32 path (k % 4 == 0, n % 4 == 0, 16-byte aligned A and B):
// 64x64 tiles, 256 threads x 4x4 outputs, K in steps of 16 through a
// double-buffered shared-memory tile fed by 128-bit global loads staged in
// registers (the next step's loads are in flight while this step computes),
// one barrier per step, and packed f32x2 FMAs. Each output is the same
// sequence of single-rounding FMAs over ascending k as the scalar kernel.
__global__ void __launch_bounds__(256)
gemm_f32_vec_kernel(const float* __restrict__ a, const float* __restrict__ b,
                    float* __restrict__ c, int64_t m, int64_t n, int64_t k, int accumulate) {
    __shared__ __align__(16) float as[2][kBK][kBM + 4];
    __shared__ __align__(16) float bs[2][kBK][kBN + 4];
    const int tid = threadIdx.x;
    const int tr = tid / 16, tc = tid % 16;
    const int64_t row0 = static_cast<int64_t>(blockIdx.y) * kBM;
    const int64_t col0 = static_cast<int64_t>(blockIdx.x) * kBN;
    // global -> register mapping: A row ai, k offset ak; B k row bp, col bj
    const int ai = tid >> 2, ak = (tid & 3) * 4;
    const int bp = tid >> 4, bj = (tid & 15) * 4;
    const int64_t arow = row0 + ai, bcol = col0 + bj;
    auto load = [&](int64_t p0, float4& ra, float4& rb) {
        const int64_t ka = p0 + ak, kb = p0 + bp;
        ra = (arow < m && ka < k) ? *reinterpret_cast<const float4*>(a + arow * k + ka)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
        rb = (kb < k && bcol < n) ? *reinterpret_cast<const float4*>(b + kb * n + bcol)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
    };
    auto store = [&](int buf, const float4& ra, const float4& rb) {
        as[buf][ak + 0][ai] = ra.x;
        as[buf][ak + 1][ai] = ra.y;
        as[buf][ak + 2][ai] = ra.z;
        as[buf][ak + 3][ai] = ra.w;
        *reinterpret_cast<float4*>(&bs[buf][bp][bj]) = rb;
    };
    float2 acc[4][2];
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = make_float2(0.f, 0.f);
    const int steps = static_cast<int>((k + kBK - 1) / kBK);
    float4 ra, rb;
    load(0, ra, rb);
    store(0, ra, rb);
    __syncthreads();
    for (int t = 0; t < steps; ++t) {
        const int cur = t & 1;
        if (t + 1 < steps) load(static_cast<int64_t>(t + 1) * kBK, ra, rb);
#pragma unroll
        for (int p = 0; p < kBK; ++p) {
            const float4 av = *reinterpret_cast<const float4*>(&as[cur][p][tr * 4]);
            const float4 bv = *reinterpret_cast<const float4*>(&bs[cur][p][tc * 4]);
            const float2 b01 = make_float2(bv.x, bv.y), b23 = make_float2(bv.z, bv.w);
            const float ai4[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 aa = make_float2(ai4[i], ai4[i]);
                acc[i][0] = __ffma2_rn(aa, b01, acc[i][0]);
                acc[i][1] = __ffma2_rn(aa, b23, acc[i][1]);
            }
        }
        if (t + 1 < steps) store(cur ^ 1, ra, rb);
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t r = row0 + tr * 4 + i;
        const int64_t cc = col0 + tc * 4;
        if (r >= m || cc >= n) continue;  // n % 4 == 0: the 4 columns are in or out together
        float4 v = make_float4(acc[i][0].x, acc[i][0].y, acc[i][1].x, acc[i][1].y);
        float4* dst = reinterpret_cast<float4*>(c + r * n + cc);
        if (accumulate) {
            const float4 o = *dst;
            v.x = o.x + v.x;
            v.y = o.y + v.y;
            v.z = o.z + v.z;
            v.w = o.w + v.w;
        }
        *dst = v;
    }
}

int checkGemm(const void* a, const void* b, const void* c, int64_t m, int64_t n, int64_t k) {
    if (a == nullptr || b == nullptr || c == nullptr) {
        return setError(MLKB_ERR_INVALID, "gemm: null buffer");
    }
    if (m <= 0 || n <= 0 || k <= 0) return setError(MLKB_ERR_INVALID, "gemm: shape must be positive");
    if ((m + 63) / 64 > 65535) return setError(MLKB_ERR_INVALID, "gemm: M too large for the grid");
    return okStatus();
}

}  // namespace
}  // namespace mlkb

extern "C" int mlkb_gemm_f64(const double* a, const double* b, double* c, int64_t m, int64_t n,
                             int64_t k, int32_t accumulate, void* stream) {
    using namespace mlkb;
    if (int st = checkGemm(a, b, c, m, n, k)) return st;
    if ((m + kT64 - 1) / kT64 > 65535) return setError(MLKB_ERR_INVALID, "gemm f64: M too large");
    const dim3 grid(static_cast<unsigned>((n + kT64 - 1) / kT64),
                    static_cast<unsigned>((m + kT64 - 1) / kT64));
    gemm_f64_kernel<<<grid, dim3(kT64, kT64), 0, asStream(stream)>>>(a, b, c, m, n, k,
                                                                    accumulate ? 1 : 0);
    return checkLaunch("gemm f64 launch");
}

extern "C" int mlkb_gemm_f32(const float* a, const float* b, float* c, int64_t m, int64_t n,
                             int64_t k, int32_t accumulate, void* stream) {
    using namespace mlkb;
    if (int st = checkGemm(a, b, c, m, n, k)) return st;
    const dim3 grid(static_cast<unsigned>((n + kBN - 1) / kBN),
                    static_cast<unsigned>((m + kBM - 1) / kBM));
    if (k % 4 == 0 && n % 4 == 0 && aligned16(a) && aligned16(b) && aligned16(c)) {
        gemm_f32_vec_kernel<<<grid, 256, 0, asStream(stream)>>>(a, b, c, m, n, k,
                                                                accumulate ? 1 : 0);
    } else {
        gemm_f32_kernel<<<grid, 256, 0, asStream(stream)>>>(a, b, c, m, n, k, accumulate ? 1 : 0);
    }
    return checkLaunch("gemm f32 launch");
}
