// SIMT GEMMs: f32 (FMA, no TF32) and f64 (the reference's exact order).
//
// Reference: gemmRowBlock, runtime/src/execution/kernel_buffers.cpp:406-432
// (C += A*B, row-major, i-p-j order with zero-a terms skipped).
//   * f64: one thread per C element runs p = 0..K-1 ascending with separate
//     multiply and add roundings and the a == 0 skip, over shared-memory
//     tiles, so results are bit-exact with the reference.
//   * f32: 64x64 register-blocked tiles (4x4 outputs per thread), f32 FMA
//     accumulation: the config-4' (1024^3 f32) path. Within the stated
//     relative-error bound, not bit-exact.
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
    gemm_f32_kernel<<<grid, 256, 0, asStream(stream)>>>(a, b, c, m, n, k, accumulate ? 1 : 0);
    return checkLaunch("gemm f32 launch");
}
