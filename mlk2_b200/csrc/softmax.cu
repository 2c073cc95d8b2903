// Row softmax and row sums (reference runtime/src/execution/kernel_buffers.cpp:
// execSoftmaxCall :290-340, execReduceSumCall :237-277).
//
// Reference semantics kept exactly:
//   r = -inf; r = (x > r) ? x : r      NaN never wins the max select
//   e = exp(x - r); s = sum e          NaN anywhere poisons the whole row
//   y = (s != 0) ? e / s : 0
//
// f32 path (the BASELINE config, HBM-bound, 8 B per element): one CTA per
// row, the row held in registers after ONE coalesced float4 read; the max in
// f32 (exact), x - r and exp in f64, the sum in f64, and y = e * (1/s)
// rounded once to f32. Rows that do not fit the register tile (or are not
// float4-aligned) take a three-pass streaming kernel with the same
// arithmetic.
#include "common.cuh"

namespace mlkb {
namespace {

constexpr int kRowThreads = 256;
constexpr int kRowWarps = kRowThreads / 32;

__device__ __forceinline__ float warpMax(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float w = __shfl_xor_sync(0xffffffffu, v, o);
        v = (w > v) ? w : v;
    }
    return v;
}

__device__ __forceinline__ double warpSum(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Block-wide max / sum over kRowThreads threads; every thread gets the result.
__device__ __forceinline__ float blockMax(float v, float* sm) {
    v = warpMax(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) sm[w] = v;
    __syncthreads();
    float r = sm[0];
#pragma unroll
    for (int i = 1; i < kRowWarps; ++i) r = (sm[i] > r) ? sm[i] : r;
    __syncthreads();
    return r;
}

__device__ __forceinline__ double blockSum(double v, double* sm) {
    v = warpSum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) sm[w] = v;
    __syncthreads();
    double r = 0.0;
#pragma unroll
    for (int i = 0; i < kRowWarps; ++i) r += sm[i];
    __syncthreads();
    return r;
}

// Register-resident row softmax: thread t owns float4 vectors t + 256*j,
// j < NV, of its row (cols <= 1024*NV, cols % 4 == 0, 16-byte aligned rows).
template <int NV>
__global__ void __launch_bounds__(kRowThreads)
softmax_rows_reg(const float* __restrict__ x, float* __restrict__ y, int64_t rows,
                 int64_t cols) {
    __shared__ float smax[kRowWarps];
    __shared__ double ssum[kRowWarps];
    const int64_t nvec = cols >> 2;
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const float4* xr = reinterpret_cast<const float4*>(x + row * cols);
        float4* yr = reinterpret_cast<float4*>(y + row * cols);
        float4 v[NV];
        float m = -INFINITY;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int64_t c = threadIdx.x + static_cast<int64_t>(j) * kRowThreads;
            if (c < nvec) {
                v[j] = __ldcs(xr + c);
                m = (v[j].x > m) ? v[j].x : m;
                m = (v[j].y > m) ? v[j].y : m;
                m = (v[j].z > m) ? v[j].z : m;
                m = (v[j].w > m) ? v[j].w : m;
            }
        }
        m = blockMax(m, smax);
        const double md = static_cast<double>(m);
        double e[NV][4];
        double s = 0.0;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int64_t c = threadIdx.x + static_cast<int64_t>(j) * kRowThreads;
            if (c < nvec) {
                e[j][0] = dev::exp_neg_f64(static_cast<double>(v[j].x) - md);
                e[j][1] = dev::exp_neg_f64(static_cast<double>(v[j].y) - md);
                e[j][2] = dev::exp_neg_f64(static_cast<double>(v[j].z) - md);
                e[j][3] = dev::exp_neg_f64(static_cast<double>(v[j].w) - md);
                s += (e[j][0] + e[j][1]) + (e[j][2] + e[j][3]);
            }
        }
        s = blockSum(s, ssum);
        const bool nz = (s != 0.0);
        const double inv = nz ? 1.0 / s : 0.0;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int64_t c = threadIdx.x + static_cast<int64_t>(j) * kRowThreads;
            if (c < nvec) {
                float4 o;
                o.x = nz ? static_cast<float>(e[j][0] * inv) : 0.0f;
                o.y = nz ? static_cast<float>(e[j][1] * inv) : 0.0f;
                o.z = nz ? static_cast<float>(e[j][2] * inv) : 0.0f;
                o.w = nz ? static_cast<float>(e[j][3] * inv) : 0.0f;
                __stcs(yr + c, o);
            }
        }
    }
}

// Exponential used by the streaming kernel: the f32 path uses the same
// f64 routine as the register kernel; the f64 path (reference-facing f64 ABI)
// calls CUDA's double exp and divides exactly like the reference.
template <typename T>
struct SoftmaxMath;

template <>
struct SoftmaxMath<float> {
    __device__ static double ex(double d) { return dev::exp_neg_f64(d); }
    __device__ static float out(double e, double s) {
        return s != 0.0 ? static_cast<float>(e * (1.0 / s)) : 0.0f;
    }
};

template <>
struct SoftmaxMath<double> {
    __device__ static double ex(double d) { return ::exp(d); }
    __device__ static double out(double e, double s) { return s != 0.0 ? e / s : 0.0; }
};

// Three-pass streaming row softmax, any cols and alignment: max, sum, write.
template <typename T>
__global__ void __launch_bounds__(kRowThreads)
softmax_rows_stream(const T* __restrict__ x, T* __restrict__ y, int64_t rows,
                    int64_t cols) {
    __shared__ float smax[kRowWarps];
    __shared__ double ssum[kRowWarps];
    __shared__ double smaxd[kRowWarps];
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const T* xr = x + row * cols;
        T* yr = y + row * cols;
        double m = -INFINITY;
        for (int64_t c = threadIdx.x; c < cols; c += kRowThreads) {
            const double v = static_cast<double>(xr[c]);
            m = (v > m) ? v : m;
        }
        // block max in f64 (exact for both element types)
        {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const double w = __shfl_xor_sync(0xffffffffu, m, o);
                m = (w > m) ? w : m;
            }
            if ((threadIdx.x & 31) == 0) smaxd[threadIdx.x >> 5] = m;
            __syncthreads();
            m = smaxd[0];
#pragma unroll
            for (int i = 1; i < kRowWarps; ++i) m = (smaxd[i] > m) ? smaxd[i] : m;
            __syncthreads();
        }
        double s = 0.0;
        for (int64_t c = threadIdx.x; c < cols; c += kRowThreads) {
            s += SoftmaxMath<T>::ex(static_cast<double>(xr[c]) - m);
        }
        s = blockSum(s, ssum);
        for (int64_t c = threadIdx.x; c < cols; c += kRowThreads) {
            yr[c] = SoftmaxMath<T>::out(SoftmaxMath<T>::ex(static_cast<double>(xr[c]) - m), s);
        }
    }
    (void)smax;
}

// Row sums in ascending k, one thread per row, f64 accumulation: the
// reference's exact order, so f64 results are bit-exact.
template <typename T>
__global__ void reducesum_rows(const T* __restrict__ x, T* __restrict__ y, int64_t rows,
                               int64_t cols) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; r < rows;
         r += stride) {
        const T* xr = x + r * cols;
        double acc = 0.0;
        for (int64_t k = 0; k < cols; ++k) acc = __dadd_rn(acc, static_cast<double>(xr[k]));
        y[r] = static_cast<T>(acc);
    }
}

int rowGrid(int64_t rows, int per_sm) {
    const int64_t cap = static_cast<int64_t>(smCount()) * per_sm;
    return static_cast<int>(rows < cap ? rows : cap);
}

int checkRows(const void* x, const void* y, int64_t rows, int64_t cols) {
    if (x == nullptr || y == nullptr) return setError(MLKB_ERR_INVALID, "rows: null buffer");
    if (rows <= 0 || cols <= 0) {
        return setError(MLKB_ERR_INVALID, "rows: shape must be positive (reference :313)");
    }
    return okStatus();
}

}  // namespace
}  // namespace mlkb

extern "C" int mlkb_softmax_f32(const float* x, float* y, int64_t rows, int64_t cols,
                                void* stream) {
    using namespace mlkb;
    if (int st = checkRows(x, y, rows, cols)) return st;
    cudaStream_t s = asStream(stream);
    const bool vec = (cols % 4 == 0) && aligned16(x) && aligned16(y);
    if (vec && cols <= 1024) {
        softmax_rows_reg<1><<<rowGrid(rows, 8), kRowThreads, 0, s>>>(x, y, rows, cols);
    } else if (vec && cols <= 2048) {
        softmax_rows_reg<2><<<rowGrid(rows, 8), kRowThreads, 0, s>>>(x, y, rows, cols);
    } else if (vec && cols <= 4096) {
        softmax_rows_reg<4><<<rowGrid(rows, 8), kRowThreads, 0, s>>>(x, y, rows, cols);
    } else if (vec && cols <= 8192) {
        softmax_rows_reg<8><<<rowGrid(rows, 4), kRowThreads, 0, s>>>(x, y, rows, cols);
    } else {
        softmax_rows_stream<float><<<rowGrid(rows, 8), kRowThreads, 0, s>>>(x, y, rows, cols);
    }
    return checkLaunch("softmax launch");
}

extern "C" int mlkb_softmax_f64(const double* x, double* y, int64_t rows, int64_t cols,
                                void* stream) {
    using namespace mlkb;
    if (int st = checkRows(x, y, rows, cols)) return st;
    softmax_rows_stream<double><<<rowGrid(rows, 8), kRowThreads, 0, asStream(stream)>>>(
        x, y, rows, cols);
    return checkLaunch("softmax f64 launch");
}

extern "C" int mlkb_reducesum_f32(const float* x, float* y, int64_t rows, int64_t cols,
                                  void* stream) {
    using namespace mlkb;
    if (int st = checkRows(x, y, rows, cols)) return st;
    const int64_t blocks = (rows + 127) / 128;
    reducesum_rows<float><<<static_cast<int>(blocks < 65535 ? blocks : 65535), 128, 0,
                            asStream(stream)>>>(x, y, rows, cols);
    return checkLaunch("reducesum launch");
}

extern "C" int mlkb_reducesum_f64(const double* x, double* y, int64_t rows, int64_t cols,
                                  void* stream) {
    using namespace mlkb;
    if (int st = checkRows(x, y, rows, cols)) return st;
    const int64_t blocks = (rows + 127) / 128;
    reducesum_rows<double><<<static_cast<int>(blocks < 65535 ? blocks : 65535), 128, 0,
                             asStream(stream)>>>(x, y, rows, cols);
    return checkLaunch("reducesum f64 launch");
}
