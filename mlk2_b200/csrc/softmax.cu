// Row softmax and row sums (reference runtime/src/execution/kernel_buffers.cpp:
// execSoftmaxCall :290-340, execReduceSumCall :237-277).
//
// Reference semantics kept exactly:
//   r = -inf; r = (x > r) ? x : r      NaN never wins the max select
//   e = exp(x - r); s = sum e          NaN anywhere poisons the whole row
//   y = (s != 0) ? e / s : 0
//
// f32 path (the BASELINE config, HBM-bound, 8 B per element): a 256-thread
// CTA works one row at a time (rows blockIdx.x + i*gridDim.x), the row
// brought into shared memory by one TMA bulk copy two rows ahead and then
// held in registers; the max in f32 (exact), x - r and exp in f64, the sum
// in f64, and y = e * (1/s) rounded once to f32: read once, write once.
// Rows that do not fit the register tile (or are not float4-aligned) take a
// three-pass streaming kernel with the same arithmetic.
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "tc_common.cuh"

namespace mlkb {
namespace {

constexpr int kRowThreads = 256;
constexpr int kRowWarps = kRowThreads / 32;
static_assert(kRowThreads == 256, "the exp table is filled one entry per thread");

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

// Block-wide sum over kRowThreads threads; every thread gets the result.
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

// exp(d) in f64 for d <= 0: k = rint(256 d / ln2), r = d - k ln2/256 (one
// FMA with fl64(ln2/256): |k| <= 44320 keeps the constant's error below 1e-14
// relative), |r| <= ln2/512, so 1 + r + r^2/2 has relative error < 4.2e-10
// (under 0.01 f32 ulp); then 2^(k/256) = 2^(k>>8) * T[k&255] with the power
// of two added to T's exponent field. d < -700 (and -inf) is clamped to -700,
// which still builds a normal scale (2^-1010): every term below -120 is under
// half the smallest f32 subnormal relative to any row sum >= 1, so it adds
// nothing to the sum and stores 0, as exp(d) would. NaN passes the clamp and
// propagates. tab[j] = 2^(j/256).
__device__ __forceinline__ double exp_neg_tab(double d, const double* tab) {
    // Branch-free: every lane evaluates the formula (the table index k & 255 is
    // always in range).
    d = (d < -700.0) ? -700.0 : d;
    const double kMagic = 6755399441055744.0;  // 1.5 * 2^52
    const double t = fma(d, 369.3299304675746, kMagic);
    const double kd = t - kMagic;
    const int k = __double2loint(t);
    const double r = fma(-kd, 0.0027076061740622863, d);
    double p = fma(r, 0.5, 1.0);
    p = fma(p, r, 1.0);
    const double tj = tab[k & 255];
    const double scale = __hiloint2double(__double2hiint(tj) + ((k >> 8) << 20),
                                          __double2loint(tj));
    return p * scale;
}

// max of three, NaN-ignoring like the reference's (x > r) ? x : r scan.
__device__ __forceinline__ float max3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

__device__ __forceinline__ void bulk_load(void* smem_dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(tc::smem_u32(smem_dst)), "l"(src), "r"(bytes), "r"(tc::smem_u32(bar))
        : "memory");
}

constexpr uint64_t kRowWaitLimitNs = 2000000000ull;

// Row softmax: each CTA owns rows blockIdx.x + i*gridDim.x (6 CTAs resident
// per SM at 4096 columns, a grid of four such waves).
// A TMA bulk copy brings row i+2 into a shared-memory double buffer while row
// i is computed, so HBM reads stay in flight across the block reductions.
// Two block barriers per row: one for the max (it also carries the vote on
// the bounded wait), one for the sum.
// Thread t owns float4 vectors t + 256*j (j < NV) of its row; exponentials
// are kept in registers between the sum and the write (read once, write
// once). cols % 4 == 0, cols <= 1024*NV, 16-byte aligned rows.
template <int NV, bool kFull>
__global__ void __launch_bounds__(kRowThreads)
softmax_rows_tma(const float* __restrict__ x, float* __restrict__ y, int64_t rows,
                 int64_t cols, int* __restrict__ status) {
    extern __shared__ __align__(128) uint8_t dyn[];
    __shared__ uint64_t full[2];
    __shared__ double tab[256];
    __shared__ float smax[kRowWarps];
    __shared__ double ssum[kRowWarps];
    const uint32_t row_bytes = static_cast<uint32_t>(cols) * 4u;
    const uint32_t buf_bytes = (row_bytes + 127u) & ~127u;
    const int nvec = static_cast<int>(cols >> 2);
    const int tid = threadIdx.x;
    if (tid == 0) {
        tc::mbar_init(&full[0], 1);
        tc::mbar_init(&full[1], 1);
        tc::fence_barrier_init();
    }
    tab[tid] = exp2(static_cast<double>(tid) * (1.0 / 256.0));  // kRowThreads == 256
    __syncthreads();
    // Programmatic dependent launch: the set-up above overlaps the tail of
    // the preceding grid in the stream; wait for it to finish (its writes
    // visible) before touching global memory, and let the next grid's CTAs
    // be scheduled as ours retire. Both are no-ops for a plain launch.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (tid == 0) {
        for (int b = 0; b < 2; ++b) {
            const int64_t r = blockIdx.x + static_cast<int64_t>(b) * gridDim.x;
            if (r < rows) {
                tc::mbar_arrive_expect_tx(&full[b], row_bytes);
                bulk_load(dyn + b * buf_bytes, x + r * cols, row_bytes, &full[b]);
            }
        }
    }
    const int warp = tid >> 5, lane = tid & 31;
    int it = 0;
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x, ++it) {
        const int b = it & 1;
        int never = 0;
        const bool ok = tc::mbar_wait(&full[b], (it >> 1) & 1, &never, kRowWaitLimitNs);
        const float4* xr = reinterpret_cast<const float4*>(dyn + b * buf_bytes);
        float4 v[NV];
        float m = -INFINITY;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int c = tid + j * kRowThreads;
            if (kFull || c < nvec) {
                v[j] = xr[c];
                m = max3(m, v[j].x, v[j].y);
                m = max3(m, v[j].z, v[j].w);
            }
        }
        m = warpMax(m);
        if (lane == 0) smax[warp] = m;
        // Barrier A (one of two per row): publishes the warp maxima, votes on
        // the wait outcome, and marks buffer b as read by every thread. The
        // previous row's sums were read before any thread got here, and this
        // row's maxima are read before barrier B, so one slot array each is
        // enough.
        if (__syncthreads_or(!ok)) {
            if (tid == 0 && status != nullptr) atomicExch(status, MLKB_ERR_TIMEOUT);
            break;
        }
        m = smax[0];
#pragma unroll
        for (int i = 1; i < kRowWarps; ++i) m = (smax[i] > m) ? smax[i] : m;
        if (tid == 0) {
            const int64_t nxt = row + 2 * static_cast<int64_t>(gridDim.x);
            if (nxt < rows) {
                tc::fence_proxy_async();
                tc::mbar_arrive_expect_tx(&full[b], row_bytes);
                bulk_load(dyn + b * buf_bytes, x + nxt * cols, row_bytes, &full[b]);
            }
        }
        const double md = static_cast<double>(m);
        double e[NV][4];
        double s = 0.0;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int c = tid + j * kRowThreads;
            if (kFull || c < nvec) {
                e[j][0] = exp_neg_tab(static_cast<double>(v[j].x) - md, tab);
                e[j][1] = exp_neg_tab(static_cast<double>(v[j].y) - md, tab);
                e[j][2] = exp_neg_tab(static_cast<double>(v[j].z) - md, tab);
                e[j][3] = exp_neg_tab(static_cast<double>(v[j].w) - md, tab);
                s += (e[j][0] + e[j][1]) + (e[j][2] + e[j][3]);
            }
        }
        s = warpSum(s);
        if (lane == 0) ssum[warp] = s;
        __syncthreads();  // barrier B: the warp sums
        s = 0.0;
#pragma unroll
        for (int i = 0; i < kRowWarps; ++i) s += ssum[i];
        // s == 0 only if every e is 0, so e * 0 gives the reference's 0.
        const double inv = (s != 0.0) ? 1.0 / s : 0.0;
        float4* yr = reinterpret_cast<float4*>(y + row * cols);
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int c = tid + j * kRowThreads;
            if (kFull || c < nvec) {
                float4 o;
                o.x = static_cast<float>(e[j][0] * inv);
                o.y = static_cast<float>(e[j][1] * inv);
                o.z = static_cast<float>(e[j][2] * inv);
                o.w = static_cast<float>(e[j][3] * inv);
                __stcs(yr + c, o);
            }
        }
    }
    // Drain: a prefetch that was issued is complete before the CTA exits.
    if (tid == 0) {
        for (int j = it; j < it + 2; ++j) {
            const int64_t r = blockIdx.x + static_cast<int64_t>(j) * gridDim.x;
            if (r < rows) {
                int never = 0;
                (void)tc::mbar_wait(&full[j & 1], (j >> 1) & 1, &never, kRowWaitLimitNs);
            }
        }
    }
}

// Exponential and final scaling of the streaming kernel (f32 rows that the
// register kernel does not take): the same f64 routine as the register
// kernel. The f64 rows have their own kernel below.
template <typename T>
struct SoftmaxMath;

template <>
struct SoftmaxMath<float> {
    __device__ static double ex(double d) { return dev::exp_neg_f64(d); }
    __device__ static float out(double e, double s) {
        return s != 0.0 ? static_cast<float>(e * (1.0 / s)) : 0.0f;
    }
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

// f64 row softmax in the reference's own order (execSoftmaxCall,
// kernel_buffers.cpp:317-339): the row max (exact in any order; a NaN never
// wins the select, and the sign of a zero maximum does not change x - r),
// e = exp(x - r) written into the output row, the sum of the row's e in
// ASCENDING k by one thread, then y = e / s (0 when s == 0); in place (x ==
// y) too, as each element is read before it is written. Only the
// exponential (CUDA's against the reference host's libm) can differ, so the
// result stays within a few f64 ULP whatever the row length; a tree sum
// drifts by up to ~cols * 2^-53. This is the reference-ABI path, not a
// throughput kernel: the ascending sum is one dependent chain per row.
constexpr int kRefRowThreads = 128;

__global__ void __launch_bounds__(kRefRowThreads)
softmax_rows_f64_ref(const double* __restrict__ x, double* __restrict__ y, int64_t rows,
                     int64_t cols) {
    __shared__ double smax[kRefRowThreads / 32];
    __shared__ double ssum;
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const double* xr = x + row * cols;
        double* yr = y + row * cols;
        double m = -INFINITY;
        for (int64_t c = threadIdx.x; c < cols; c += kRefRowThreads) {
            const double v = xr[c];
            m = (v > m) ? v : m;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const double w = __shfl_xor_sync(0xffffffffu, m, o);
            m = (w > m) ? w : m;
        }
        if ((threadIdx.x & 31) == 0) smax[threadIdx.x >> 5] = m;
        __syncthreads();
        m = smax[0];
#pragma unroll
        for (int i = 1; i < kRefRowThreads / 32; ++i) m = (smax[i] > m) ? smax[i] : m;
        for (int64_t c = threadIdx.x; c < cols; c += kRefRowThreads) {
            yr[c] = ::exp(__dsub_rn(xr[c], m));
        }
        __syncthreads();  // the row's e are in y, visible to the whole block
        if (threadIdx.x == 0) {
            double acc = 0.0;
            for (int64_t c = 0; c < cols; ++c) acc = __dadd_rn(acc, yr[c]);
            ssum = acc;
        }
        __syncthreads();
        const double sum = ssum;
        for (int64_t c = threadIdx.x; c < cols; c += kRefRowThreads) {
            yr[c] = sum != 0.0 ? __ddiv_rn(yr[c], sum) : 0.0;
        }
        __syncthreads();  // smax / ssum are reused by the next row
    }
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

namespace mlkb {
namespace {

template <int NV, bool kFull>
int launchRowsTma(const float* x, float* y, int64_t rows, int64_t cols, cudaStream_t s) {
    const uint32_t buf = ((static_cast<uint32_t>(cols) * 4u + 127u) & ~127u);
    const size_t smem = 2 * static_cast<size_t>(buf);
    static std::atomic<bool> attr[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(softmax_rows_tma<NV, kFull>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   64 * 1024);
        if (e != cudaSuccess) return setCudaError(MLKB_ERR_LAUNCH, e, "softmax smem attribute");
        attr[dev] = true;
    }
    // Resident CTAs per SM are 8 / 6 / 3 (shared memory); the grid holds four
    // times that, so each CTA streams ~18 rows at 65536 x 4096 and the
    // hardware rebalances the short CTAs across SMs (6 % faster than one
    // resident wave of persistent CTAs).
    const int per_sm = 4 * (NV <= 2 ? 8 : NV <= 4 ? 6 : 3);
    // Launched with programmatic stream serialization (the kernel waits for
    // its predecessor itself): back-to-back launches overlap launch and tail.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(rowGrid(rows, per_sm));
    cfg.blockDim = dim3(kRowThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    const cudaError_t le = cudaLaunchKernelEx(&cfg, softmax_rows_tma<NV, kFull>, x, y, rows, cols,
                                              deviceStatusPtr());
    if (le != cudaSuccess) return setCudaError(MLKB_ERR_LAUNCH, le, "softmax launch");
    return checkLaunch("softmax launch");
}

template <int NV>
int launchRows(const float* x, float* y, int64_t rows, int64_t cols, cudaStream_t s) {
    return cols == NV * 4 * kRowThreads ? launchRowsTma<NV, true>(x, y, rows, cols, s)
                                        : launchRowsTma<NV, false>(x, y, rows, cols, s);
}

}  // namespace
}  // namespace mlkb

extern "C" int mlkb_softmax_f32(const float* x, float* y, int64_t rows, int64_t cols,
                                void* stream) {
    using namespace mlkb;
    if (int st = checkRows(x, y, rows, cols)) return st;
    cudaStream_t s = asStream(stream);
    const bool vec = (cols % 4 == 0) && aligned16(x) && aligned16(y);
    if (vec && cols <= 1024) return launchRows<1>(x, y, rows, cols, s);
    if (vec && cols <= 2048) return launchRows<2>(x, y, rows, cols, s);
    if (vec && cols <= 4096) return launchRows<4>(x, y, rows, cols, s);
    if (vec && cols <= 8192) return launchRows<8>(x, y, rows, cols, s);
    softmax_rows_stream<float><<<rowGrid(rows, 8), kRowThreads, 0, s>>>(x, y, rows, cols);
    return checkLaunch("softmax launch");
}

extern "C" int mlkb_softmax_f64(const double* x, double* y, int64_t rows, int64_t cols,
                                void* stream) {
    using namespace mlkb;
    if (int st = checkRows(x, y, rows, cols)) return st;
    softmax_rows_f64_ref<<<rowGrid(rows, 16), kRefRowThreads, 0, asStream(stream)>>>(
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

// ---- allocation-free entry ---------------------------------------------------------
// mlkb_softmax_f32 and the other entries whose kernels have bounded waits keep
// their status word in device memory the library obtains with cudaMalloc on
// the first call on each device. This entry runs the same TMA row kernel with
// that scratch in a fixed array of this file instead, so it never allocates.
namespace mlkb {
namespace {

// The scratch of mlkb_softmax_f32_noalloc: 256 bytes, of which the kernel
// uses the first word (the status its bounded waits report through, whatever
// the shape). Every device that loads the library holds one copy until the
// process exits. In host code this name is only a stand-in for the symbol:
// kernels get the device address from cudaGetSymbolAddress below.
constexpr size_t kNoAllocScratchBytes = 256;
constexpr size_t kNoAllocStatusBytes = sizeof(int);
static_assert(kNoAllocStatusBytes <= kNoAllocScratchBytes, "status word fits the scratch");
static __device__ __align__(256) int g_softmax_noalloc_scratch[kNoAllocScratchBytes / sizeof(int)];

// Device address of the scratch on the current device, looked up once per
// device (with that device current) and kept.
int noAllocScratch(int** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return setCudaError(MLKB_ERR_NO_DEVICE, e, "softmax_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= 64) return setError(MLKB_ERR_INVALID, "softmax_noalloc: device index past 63");
    static std::mutex mu;
    static int* addr[64] = {nullptr};
    std::lock_guard<std::mutex> lock(mu);
    if (addr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_softmax_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            return setCudaError(MLKB_ERR_LAUNCH, e, "softmax_noalloc: cudaGetSymbolAddress");
        }
        addr[dev] = static_cast<int*>(p);
    }
    *out = addr[dev];
    return okStatus();
}

template <int NV, bool kFull>
int launchRowsNoAlloc(const float* x, float* y, int64_t rows, int64_t cols, int* status,
                      cudaStream_t s) {
    const uint32_t buf = ((static_cast<uint32_t>(cols) * 4u + 127u) & ~127u);
    const size_t smem = 2 * static_cast<size_t>(buf);
    static std::atomic<bool> attr[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(softmax_rows_tma<NV, kFull>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   64 * 1024);
        if (e != cudaSuccess) return setCudaError(MLKB_ERR_LAUNCH, e, "softmax_noalloc smem attribute");
        attr[dev] = true;
    }
    const int per_sm = 4 * (NV <= 2 ? 8 : NV <= 4 ? 6 : 3);
    softmax_rows_tma<NV, kFull><<<rowGrid(rows, per_sm), kRowThreads, smem, s>>>(x, y, rows,
                                                                                 cols, status);
    return checkLaunch("softmax_noalloc launch");
}

template <int NV>
int launchRowsNoAlloc(const float* x, float* y, int64_t rows, int64_t cols, int* status,
                      cudaStream_t s) {
    return cols == NV * 4 * kRowThreads ? launchRowsNoAlloc<NV, true>(x, y, rows, cols, status, s)
                                        : launchRowsNoAlloc<NV, false>(x, y, rows, cols, status, s);
}

}  // namespace
}  // namespace mlkb

extern "C" int mlkb_softmax_f32_noalloc(const float* x, float* y, int64_t rows, int64_t cols,
                                        int32_t wait, void* stream) {
    using namespace mlkb;
    if (int st = checkRows(x, y, rows, cols)) return st;
    if (cols > 8192 || cols % 4 != 0 || !aligned16(x) || !aligned16(y)) {
        return setError(MLKB_ERR_INVALID,
                        "softmax_noalloc: rows of at most 8192 columns, a multiple of 4, with "
                        "16-byte aligned buffers (other shapes: mlkb_softmax_f32)");
    }
    int* status = nullptr;
    if (int st = noAllocScratch(&status)) return st;
    cudaStream_t s = asStream(stream);
    // The status word must start at zero on every call.
    cudaError_t e = cudaMemsetAsync(status, 0, kNoAllocStatusBytes, s);
    if (e != cudaSuccess) return setCudaError(MLKB_ERR_LAUNCH, e, "softmax_noalloc: clear status");
    int rc = cols <= 1024   ? launchRowsNoAlloc<1>(x, y, rows, cols, status, s)
             : cols <= 2048 ? launchRowsNoAlloc<2>(x, y, rows, cols, status, s)
             : cols <= 4096 ? launchRowsNoAlloc<4>(x, y, rows, cols, status, s)
                            : launchRowsNoAlloc<8>(x, y, rows, cols, status, s);
    if (rc != MLKB_OK || wait == 0) return rc;
    int word = 0;
    e = cudaMemcpyAsync(&word, status, sizeof(word), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return setCudaError(MLKB_ERR_LAUNCH, e, "softmax_noalloc: status read");
    return word == 0 ? okStatus() : setError(word, "softmax_noalloc: a bounded device wait gave up");
}
