// Host-side Kernel IR module: parsed from the reference's `mlk-kernel` JSON
// wire format (reference compiler/src/support/kernel_ir.cpp:97-254, the
// types of compiler/include/mlk/support/kernel_ir.h:22-217) and classified
// into one of the kernel families this library runs.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "../../include/mlkb200.h"

namespace mlkb {

// KernelOp numbering and names (reference kernel_ir.h:22-34, kernel_ir.cpp:6-21).
enum class KOp : int { Loop = 0, Compute, Load, Store, Alloc, Copy, Barrier, Trace, Guard, Call };

// Math ops beyond the scalar chain set (reference math_op.h).
constexpr int kMathMatMul = 16;
constexpr int kMathReduceSum = 21;
constexpr int kMathSoftmax = 24;

struct KBuffer {
    std::string name;
    int dtype = MLKB_F32;  // from the "dtype" field; f64 when absent
    bool input = false, output = false, temp = false;
    int64_t elements = -1;
    std::vector<int64_t> dims;
};

struct KNode {
    KOp op = KOp::Loop;
    int math = -1;  // Compute: MathOp of the node (legacy single-op form); Call: -1 unless given
    std::string family;
    int64_t begin = 0, end = -1, step = 1;
    int64_t a = -1, b = -1, out = -1;
    bool multiDimFeature = false;  // affine bounds/stores/guards, accumulate, end_buf
    std::vector<mlkb_expr> exprs;
    std::vector<uint32_t> children;
};

// One 1-D root: for i in [begin, end): buffers[out][i] = chain(A[i], B[i]).
struct MapRoot {
    std::vector<mlkb_expr> chain;
    int a = -1, b = -1, out = -1;
    bool poly7 = false;
    int64_t begin = 0, end = -1;  // end == -1: the caller's element count
};

struct Module {
    std::vector<KBuffer> buffers;
    std::vector<KNode> nodes;
    std::vector<std::pair<std::string, int64_t>> schedule;

    int kind = 0;          // MLKB_KIND_*
    bool multiDim = false; // the reference isMultiDimModule rule
    std::vector<int> bindable;  // buffer ids in table order (inputs, outputs)

    std::vector<MapRoot> roots;              // MLKB_KIND_MAP; QK: the scale map
    int callA = -1, callB = -1, callOut = -1;  // Call kinds
    int64_t m = 0, k = 0, n = 0;             // Call shapes (A=[m,k], B=[k,n])
    // MLKB_KIND_QK_SOFTMAX: S = Q*Kt (Call(MatMul), Q = callA [m,k], Kt =
    // callB [k,n]), Sc = S * scale (the map, roots[0]), Y = softmax(Sc)
    // (callOut). With S and Sc temps the module is the fused kernel; with
    // both as outputs the three steps run as the reference runs them.
    double scale = 1.0;
    int qkS = -1, qkSc = -1;
    bool qkFused = false;
};

// Parses `json` into `out` and classifies it. Returns an MLKB status; the
// message is recorded with setError on failure.
int parseModule(const char* json, Module& out);

// True when every Store of the module's Loop roots reads only 1-D operands
// (the fused-map family); exposed for tests through the module kind.
bool isUnaryOp(int op);
int checkChain(const mlkb_expr* exprs, int32_t n_exprs, bool has_b);

}  // namespace mlkb
