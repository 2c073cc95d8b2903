// Deterministic synthetic inputs generated on the device.
//
// word(seed, stream, i) = SplitMix64 finaliser of seed + stream*2^40 +
// (i+1)*0x9E3779B97F4A7C15. Uniform values take the top 24 bits k:
// lo + (hi-lo)*k*2^-24, exact in f32 for the power-of-two ranges the
// configs use, and bit-identical to the host generator in oracle/. Normal
// values use Box-Muller on two 53-bit uniforms from words 2i and 2i+1.
#include <cuda_fp16.h>

#include "common.cuh"

namespace mlkb {
namespace {

__device__ __forceinline__ uint64_t word(uint64_t seed, uint32_t stream_id, uint64_t i) {
    uint64_t z = seed + (static_cast<uint64_t>(stream_id) << 40) + (i + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ double sample(uint64_t seed, uint32_t sid, int64_t i, int dist,
                                         double lo, double hi) {
    if (dist == 0) {
        const uint64_t k = word(seed, sid, static_cast<uint64_t>(i)) >> 40;
        return lo + (hi - lo) * (static_cast<double>(k) * 0x1p-24);
    }
    const uint64_t w1 = word(seed, sid, 2 * static_cast<uint64_t>(i));
    const uint64_t w2 = word(seed, sid, 2 * static_cast<uint64_t>(i) + 1);
    const double u1 = (static_cast<double>(w1 >> 11) + 0.5) * 0x1p-53;
    const double u2 = static_cast<double>(w2 >> 11) * 0x1p-53;
    const double r = sqrt(-2.0 * log(u1));
    return lo + hi * r * cospi(2.0 * u2);
}

template <typename T>
__global__ void fill_kernel(T* out, int64_t n, uint64_t seed, uint32_t sid, int dist, double lo,
                            double hi) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += stride) {
        const double v = sample(seed, sid, i, dist, lo, hi);
        if constexpr (sizeof(T) == 2) {
            out[i] = __double2half(v);
        } else {
            out[i] = static_cast<T>(v);
        }
    }
}

template <typename T>
int launchFill(T* out, int64_t n, uint64_t seed, uint32_t sid, int32_t dist, double lo,
               double hi, void* stream) {
    if (out == nullptr || n < 0 || (dist != 0 && dist != 1)) {
        return setError(MLKB_ERR_INVALID, "fill: bad argument");
    }
    if (n == 0) return okStatus();
    const int64_t blocks = (n + 255) / 256;
    const int64_t cap = static_cast<int64_t>(smCount()) * 16;
    fill_kernel<T><<<static_cast<int>(blocks < cap ? blocks : cap), 256, 0, asStream(stream)>>>(
        out, n, seed, sid, dist, lo, hi);
    return checkLaunch("fill launch");
}

}  // namespace
}  // namespace mlkb

extern "C" int mlkb_fill_f32(float* out, int64_t n, uint64_t seed, uint32_t stream_id,
                             int32_t dist, double lo, double hi, void* stream) {
    return mlkb::launchFill<float>(out, n, seed, stream_id, dist, lo, hi, stream);
}

extern "C" int mlkb_fill_f16(void* out, int64_t n, uint64_t seed, uint32_t stream_id,
                             int32_t dist, double lo, double hi, void* stream) {
    return mlkb::launchFill<__half>(static_cast<__half*>(out), n, seed, stream_id, dist, lo, hi,
                                    stream);
}
