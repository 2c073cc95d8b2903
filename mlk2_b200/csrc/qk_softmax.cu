// Batched scaled-scores softmax: Y[b] = softmax_rows(scale * Q[b] * K[b]^T).
//
// The reference has no fused operator: its composition is Call(MatMul) ->
// scale map -> Call(Softmax) (runtime/src/execution/kernel_buffers.cpp:
// 1001-1085, :342-402, :290-340), evaluated in f64 with K^T materialised.
// Here Q and K are f16 [batch, s, d] row-major, so K is already the
// K-major operand the tcgen05 MMA wants: no transpose is materialised.
//
// Current form: the tcgen05 GEMM writes scale * Q K^T straight into Y
// (scale applied in the TMEM epilogue), then the row-softmax kernel
// normalises Y in place (each row is read into registers before it is
// overwritten, so in place is safe). Y is the only memory touched besides Q
// and K.
#include "common.cuh"

namespace mlkb {
int launchGemmTc(const void* a, const void* b, float* c, int64_t batch, int64_t m, int64_t n,
                 int64_t k, bool b_kmajor, int accumulate, float scale, cudaStream_t s);
}  // namespace mlkb

extern "C" int mlkb_qk_softmax_f16(const void* q, const void* k, float* y, int64_t batch,
                                   int64_t s, int64_t d, double scale, void* stream) {
    using namespace mlkb;
    if (q == nullptr || k == nullptr || y == nullptr) {
        return setError(MLKB_ERR_INVALID, "qk_softmax: null buffer");
    }
    if (batch <= 0 || s <= 0 || d <= 0) {
        return setError(MLKB_ERR_INVALID, "qk_softmax: shape must be positive");
    }
    if (d % 8 != 0 || s % 8 != 0 || !aligned16(q) || !aligned16(k) || !aligned16(y) ||
        batch * s > (int64_t(1) << 30)) {
        return setError(MLKB_ERR_INVALID,
                        "qk_softmax: d and s must be multiples of 8 with 16-byte aligned buffers");
    }
    cudaStream_t st = asStream(stream);
    if (int rc = launchGemmTc(q, k, y, batch, s, s, d, true, 0, static_cast<float>(scale), st)) {
        return rc;
    }
    return mlkb_softmax_f32(y, y, batch * s, s, stream);
}
