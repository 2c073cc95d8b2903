// C-ABI driver over the REFERENCE's own CPU KernelModule executor.
//
// TEST INFRASTRUCTURE ONLY. Linked against the reference library sources
// compiled by oracle/ref.mk into oracle/_ref/libmlkref.so. It builds the
// KernelModules the B200 path is checked on -- with the reference's own
// types -- and runs them through the reference's executeKernelOnBuffers
// (reference runtime/src/execution/kernel_buffers.cpp:839-1106). Only tests,
// __graft_entry__.smoke() and bench.py's CPU-baseline leg load it.
//
// Module shapes mirror the reference's own constructions:
//   - fused 1-D chain: Loop{Compute(exprs); Store} with a dynamic bound, the
//     form lower.to_kernel_ir emits (compiler/src/passes/lower/
//     lower.to_kernel_ir.cpp:369-425);
//   - multi-root chains: one Loop/Compute/Store per output, each storing to
//     its own buffer (the executor pairs each Loop with its Store,
//     kernel_buffers.cpp:921-953);
//   - Call(MatMul / Softmax / ReduceSum) over rank-2 buffers, the
//     construction of tools/mlk-poly/poly_bench.cpp:123-160.
// It also
//   - reads any 1-D `mlk-kernel` JSON module back into the reference's
//     KernelModule (the reference only writes the format, with
//     KernelModule::toJson, compiler/src/support/kernel_ir.cpp:97-254), so
//     the reference executor runs exactly the document the B200 path runs;
//   - produces modules with the reference's OWN compiler: a GraphBuilder
//     graph through PipelineRunner at Tier 1
//     (compiler/src/pipeline/pipeline_runner.cpp:33-53), the way mlkc does
//     (tools/mlkc/mlkc.cpp:117-150).
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "mlk/core/constants.h"
#include "mlk/runtime/execution.h"
#include "mlk/support/json.h"
#include "mlk/support/kernel_ir.h"

#include "../include/mlkb200.h"
#include "ref_modules.h"

namespace {

using mlkb_oracle::g_err;
using mlkb_oracle::loadModule;
using mlkb_oracle::pipelineModule;

int fail(const mlk::Error& e) {
    g_err = e.message;
    return 100 + static_cast<int>(e.code);
}

mlk::KernelOperand operand(int32_t kind, int64_t index, double value) {
    mlk::KernelOperand o;
    o.kind = static_cast<mlk::KernelOperand::Kind>(kind);
    o.index = index;
    o.constValue = value;
    return o;
}

// Appends one Loop{Compute; Store} root to `km` (table order is up to the
// caller: buffers are added before the roots).
void addRoot(mlk::KernelModule& km, mlk::SymbolTable& symbols,
             const mlkb_expr* exprs, int n_exprs, uint32_t bufA,
             uint32_t bufB, uint32_t bufOut, bool poly7, int rootIdx) {
    mlk::KernelNode loop;
    loop.op = mlk::KernelOp::Loop;
    loop.var = symbols.intern("i" + std::to_string(rootIdx));
    loop.begin = 0;
    loop.end = mlk::constants::kKernelLoopDynamicBound;
    loop.parallel = true;
    mlk::KernelNode compute;
    compute.op = mlk::KernelOp::Compute;
    compute.math = static_cast<mlk::MathOp>(exprs[n_exprs - 1].op);
    compute.bufferA = bufA;
    compute.bufferB = bufB;
    if (poly7) compute.family = symbols.intern("poly7");
    for (int k = 0; k < n_exprs; ++k) {
        mlk::KernelExpr e;
        e.op = static_cast<mlk::MathOp>(exprs[k].op);
        e.a = operand(exprs[k].a_kind, exprs[k].a_index, exprs[k].a_value);
        e.b = operand(exprs[k].b_kind, exprs[k].b_index, exprs[k].b_value);
        compute.exprs.push_back(e);
    }
    mlk::KernelNode store;
    store.op = mlk::KernelOp::Store;
    store.bufferOut = bufOut;
    const uint32_t loopId = km.addNode(loop);
    const uint32_t cId = km.addNode(compute);
    const uint32_t sId = km.addNode(store);
    km.nodes[loopId].children.push_back(cId);
    km.nodes[loopId].children.push_back(sId);
}

// Multi-root chain module: n_inputs (1 or 2) input buffers, n_roots outputs.
mlk::KernelModule buildChainModule(mlk::SymbolTable& symbols, int n_roots,
                                   const int32_t* root_len,
                                   const mlkb_expr* exprs, int n_inputs,
                                   bool poly7, int64_t threads) {
    mlk::KernelModule km;
    km.name = symbols.intern("fused_map");
    mlk::KernelBuffer a;
    a.name = symbols.intern("x");
    a.dtype = mlk::Dtype::F32;
    a.isInput = true;
    const uint32_t bufA = km.addBuffer(a);
    uint32_t bufB = mlk::constants::kInvalidId;
    if (n_inputs > 1) {
        mlk::KernelBuffer b;
        b.name = symbols.intern("w");
        b.dtype = mlk::Dtype::F32;
        b.isInput = true;
        bufB = km.addBuffer(b);
    }
    std::vector<uint32_t> outs;
    for (int r = 0; r < n_roots; ++r) {
        mlk::KernelBuffer o;
        o.name = symbols.intern("y" + std::to_string(r));
        o.dtype = mlk::Dtype::F32;
        o.isOutput = true;
        outs.push_back(km.addBuffer(o));
    }
    int off = 0;
    for (int r = 0; r < n_roots; ++r) {
        addRoot(km, symbols, exprs + off, root_len[r], bufA, bufB, outs[r],
                poly7, r);
        off += root_len[r];
    }
    if (threads > 0) *km.scheduleParams.findOrInsert(symbols.intern("threads"), nullptr) = threads;
    return km;
}

mlk::KernelModule buildCallModule(mlk::SymbolTable& symbols, mlk::MathOp op,
                                  int64_t m, int64_t k, int64_t n,
                                  int64_t threads) {
    mlk::KernelModule km;
    km.name = symbols.intern("call");
    mlk::KernelBuffer a;
    a.name = symbols.intern("A");
    a.dtype = mlk::Dtype::F32;
    a.dims = mlk::SmallVector<int64_t, 4>{m, k};
    a.isInput = true;
    const uint32_t bufA = km.addBuffer(a);
    uint32_t bufB = mlk::constants::kInvalidId;
    if (op == mlk::MathOp::MatMul) {
        mlk::KernelBuffer b;
        b.name = symbols.intern("B");
        b.dtype = mlk::Dtype::F32;
        b.dims = mlk::SmallVector<int64_t, 4>{k, n};
        b.isInput = true;
        bufB = km.addBuffer(b);
    }
    mlk::KernelBuffer out;
    out.isOutput = true;
    out.dtype = mlk::Dtype::F32;
    if (op == mlk::MathOp::MatMul) {
        out.name = symbols.intern("C");
        out.dims = mlk::SmallVector<int64_t, 4>{m, n};
    } else if (op == mlk::MathOp::Softmax) {
        out.name = symbols.intern("Y");
        out.dims = mlk::SmallVector<int64_t, 4>{m, k};
    } else {
        out.name = symbols.intern("Y");
        out.dims = mlk::SmallVector<int64_t, 4>{m};
    }
    const uint32_t bufOut = km.addBuffer(out);
    mlk::KernelNode call;
    call.op = mlk::KernelOp::Call;
    call.math = op;
    call.bufferA = bufA;
    call.bufferB = bufB;
    call.bufferOut = bufOut;
    (void)km.addNode(call);
    if (threads > 0) *km.scheduleParams.findOrInsert(symbols.intern("threads"), nullptr) = threads;
    return km;
}

int copyJson(const mlk::KernelModule& km, mlk::SymbolTable& symbols,
             char* buf, int64_t cap) {
    const std::string s = mlk::json::serialize(km.toJson(symbols));
    if (static_cast<int64_t>(s.size()) + 1 > cap) return -static_cast<int>(s.size() + 1);
    std::memcpy(buf, s.c_str(), s.size() + 1);
    return 0;
}

}  // namespace

extern "C" {

const char* mlkref_last_error(void) { return g_err.c_str(); }

// Multi-root fused chain over f64 buffers: outs[r][i] = chain_r(a[i], b[i]).
// threads <= 0 keeps the executor's default (<= kKernelExecMaxThreads).
int mlkref_chain(int32_t n_roots, const int32_t* root_len,
                 const mlkb_expr* exprs, int32_t poly7, const double* a,
                 const double* b, double* const* outs, int64_t n,
                 const double* scalars, int64_t n_scalars, int64_t threads) {
    mlk::SymbolTable symbols;
    mlk::KernelModule km = buildChainModule(symbols, n_roots, root_len, exprs,
                                            b != nullptr ? 2 : 1, poly7 != 0,
                                            threads);
    mlk::KernelBufferBindings io;
    io.inputs.push_back(const_cast<double*>(a));
    if (b != nullptr) io.inputs.push_back(const_cast<double*>(b));
    for (int r = 0; r < n_roots; ++r) io.outputs.push_back(outs[r]);
    for (int64_t s = 0; s < n_scalars; ++s) io.scalars.push_back(scalars[s]);
    io.elements = n;
    auto r = mlk::executeKernelOnBuffers(km, symbols, io, nullptr);
    return r.has_value() ? 0 : fail(r.error());
}

static int runCall(mlk::MathOp op, const double* a, const double* b,
                   double* y, int64_t m, int64_t k, int64_t n,
                   int64_t threads) {
    mlk::SymbolTable symbols;
    mlk::KernelModule km = buildCallModule(symbols, op, m, k, n, threads);
    mlk::KernelBufferBindings io;
    io.inputs.push_back(const_cast<double*>(a));
    if (b != nullptr) io.inputs.push_back(const_cast<double*>(b));
    io.outputs.push_back(y);
    io.elements = m * (op == mlk::MathOp::MatMul ? n : k);
    auto r = mlk::executeKernelOnBuffers(km, symbols, io, nullptr);
    return r.has_value() ? 0 : fail(r.error());
}

int mlkref_softmax(const double* a, double* y, int64_t rows, int64_t cols) {
    return runCall(mlk::MathOp::Softmax, a, nullptr, y, rows, cols, 0, 0);
}

int mlkref_reducesum(const double* a, double* y, int64_t rows, int64_t cols) {
    return runCall(mlk::MathOp::ReduceSum, a, nullptr, y, rows, cols, 0, 0);
}

// C += A*B (the reference accumulates into C).
int mlkref_matmul(const double* a, const double* b, double* c, int64_t m,
                  int64_t n, int64_t k, int64_t threads) {
    return runCall(mlk::MathOp::MatMul, a, b, c, m, k, n, threads);
}

// toJson of the module the driver would build, for wire-format tests of the
// B200 shim's module parser. kind: MLKB_KIND_MAP uses (n_roots, root_len,
// exprs, n_inputs); the Call kinds use (m, k, n).
int mlkref_module_json(int32_t kind, int32_t n_roots, const int32_t* root_len,
                       const mlkb_expr* exprs, int32_t n_inputs, int32_t poly7,
                       int64_t m, int64_t k, int64_t n, char* buf,
                       int64_t cap) {
    mlk::SymbolTable symbols;
    if (kind == MLKB_KIND_MAP) {
        return copyJson(buildChainModule(symbols, n_roots, root_len, exprs,
                                         n_inputs, poly7 != 0, 0),
                        symbols, buf, cap);
    }
    const mlk::MathOp op = kind == MLKB_KIND_SOFTMAX ? mlk::MathOp::Softmax
                           : kind == MLKB_KIND_MATMUL ? mlk::MathOp::MatMul
                                                      : mlk::MathOp::ReduceSum;
    return copyJson(buildCallModule(symbols, op, m, k, n, 0), symbols, buf, cap);
}

// Runs an `mlk-kernel` JSON module through executeKernelOnBuffers over f64
// buffers given in table order (inputs, then outputs; temps are the
// executor's own). n is KernelBufferBindings::elements.
int mlkref_run_json(const char* json, double* const* bufs, int32_t n_bufs, int64_t n,
                    const double* scalars, int64_t n_scalars, int64_t threads) {
    mlk::SymbolTable symbols;
    mlk::KernelModule km;
    if (json == nullptr || !loadModule(json, symbols, km)) return 200;
    if (threads > 0) *km.scheduleParams.findOrInsert(symbols.intern("threads"), nullptr) = threads;
    mlk::KernelBufferBindings io;
    int32_t k = 0;
    for (const mlk::KernelBuffer& b : km.buffers) {
        if (!b.isInput && !b.isOutput) continue;
        if (k >= n_bufs) {
            g_err = "fewer buffers than the module binds";
            return 201;
        }
        (b.isInput ? io.inputs : io.outputs).push_back(bufs[k++]);
    }
    if (k != n_bufs) {
        g_err = "more buffers than the module binds";
        return 201;
    }
    for (int64_t i = 0; i < n_scalars; ++i) io.scalars.push_back(scalars[i]);
    io.elements = n;
    auto r = mlk::executeKernelOnBuffers(km, symbols, io, nullptr);
    return r.has_value() ? 0 : fail(r.error());
}

// toJson of a module the reference's own pipeline compiles (pipelineModule
// above); *patched counts the constants whose unset type was restored.
int mlkref_pipeline_json(int32_t which, int64_t n, int32_t f32, char* buf, int64_t cap,
                         int32_t* patched) {
    mlk::SymbolTable symbols;
    mlk::KernelModule km;
    int p = 0;
    if (!pipelineModule(which, n, f32 != 0, symbols, km, &p)) return 202;
    if (patched != nullptr) *patched = p;
    return copyJson(km, symbols, buf, cap);
}

}  // extern "C"
