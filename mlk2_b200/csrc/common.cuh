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

// One chain expression for the run-time compiled chain kernels
// (chain_jit.cpp): op and operand kinds as in mlkb_expr, ScalarParam
// operands already resolved to constants (kind kConst), temps as indices of
// earlier expressions.
struct JitExpr {
    int op, akind, bkind, unary, aidx, bidx;
    double aval, bval;
};
// Returned by the two calls below when the chain was not compiled (NVRTC
// absent, compilation switched off, or it failed): the caller interprets it.
constexpr int kJitUnavailable = -100;
// Runs the chain over n elements of a (and b) into out (dtype MLKB_F32 or
// MLKB_F64) as a compiled straight-line kernel, compiling it on first use.
int launchChainJit(const JitExpr* e, int n_exprs, bool poly7, const void* a, const void* b,
                   void* out, int dtype, int64_t n, cudaStream_t s);
// The same for a GROUP of at most kMaxJitOuts chains that read the same a
// (and b) over the same n elements: one kernel loads the inputs once and
// stores chain j's result to outs[j]. poly7[j] selects chain j's Sin family.
constexpr int kMaxJitOuts = 8;
int launchChainsJit(const JitExpr* const* chains, const int* n_exprs, const bool* poly7,
                    int n_chains, const void* a, const void* b, void* const* outs, int dtype,
                    int64_t n, cudaStream_t s);
// A host chain in the compiled form: checked as mlkb_map_chain checks it
// (MLKB_OK or an error status), ScalarParams resolved against the table.
int toJitChain(const mlkb_expr* exprs, int32_t n_exprs, bool has_b, const double* scalars,
               int64_t n_scalars, JitExpr* out);
// Compiles (and caches) the chain's kernel without launching it; *why gets
// the reason when it returns kJitUnavailable.
int buildChainJit(const JitExpr* e, int n_exprs, bool poly7, int dtype, const char** why);

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


#include "chain_math.cuh"
