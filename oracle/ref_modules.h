// Reference-side helpers shared by the oracle's drivers (ref_driver.cpp,
// ref_loader_check.cpp). TEST INFRASTRUCTURE ONLY: compiled against the
// reference's headers and library by oracle/ref.mk; never part of the
// shipped path.
#pragma once

#include <cstdint>
#include <string>

#include "mlk/core/constants.h"
#include "mlk/core/diagnostics.h"
#include "mlk/ir/graph_builder.h"
#include "mlk/pass/pass_registry.h"
#include "mlk/pass/register_all.h"
#include "mlk/pipeline/pipeline_runner.h"
#include "mlk/runtime/telemetry.h"
#include "mlk/support/json.h"
#include "mlk/support/kernel_ir.h"
#include "mlk/type/domain_profile.h"

namespace mlkb_oracle {

inline thread_local std::string g_err;

// ---- `mlk-kernel` JSON -> KernelModule ------------------------------------------
// The inverse of KernelModule::toJson for the fields 1-D modules carry
// (buffers; Loop / Compute / Store / Call nodes with begin, end, step, a, b,
// out, family, exprs, children; schedule). toJson does not write a Call's
// math (kernel_ir.cpp:130-135), so it is inferred from the operands the
// executor validates, as the B200 path's own parser does: a B operand means
// MatMul, otherwise a rank-2 output Softmax and a rank-1 output ReduceSum.
inline bool loadModule(const std::string& text, mlk::SymbolTable& sy, mlk::KernelModule& km) {
    auto doc = mlk::json::parse(text);
    if (!doc.has_value() || !doc->isObject()) {
        g_err = "module JSON does not parse";
        return false;
    }
    const mlk::json::Value* bufs = doc->find("buffers");
    const mlk::json::Value* nodes = doc->find("nodes");
    if (bufs == nullptr || !bufs->isArray() || nodes == nullptr || !nodes->isArray()) {
        g_err = "module JSON lacks buffers / nodes";
        return false;
    }
    auto str = [](const mlk::json::Value& o, const char* k) -> std::string {
        const mlk::json::Value* v = o.find(k);
        return (v != nullptr && v->isString()) ? v->asString() : std::string();
    };
    auto num = [](const mlk::json::Value& o, const char* k, int64_t d) -> int64_t {
        const mlk::json::Value* v = o.find(k);
        return (v != nullptr && v->isNumber()) ? v->asInt() : d;
    };
    auto flag = [](const mlk::json::Value& o, const char* k) {
        const mlk::json::Value* v = o.find(k);
        return v != nullptr && v->isBool() && v->asBool();
    };
    if (const std::string nm = str(*doc, "name"); !nm.empty()) km.name = sy.intern(nm);
    for (const mlk::json::Value& b : bufs->asArray()) {
        mlk::KernelBuffer kb;
        kb.name = sy.intern(str(b, "name"));
        const std::string dt = str(b, "dtype");
        for (uint8_t i = 0; i <= static_cast<uint8_t>(mlk::Dtype::C128); ++i) {
            if (dt == mlk::dtypeName(static_cast<mlk::Dtype>(i))) kb.dtype = static_cast<mlk::Dtype>(i);
        }
        kb.isInput = flag(b, "input");
        kb.isOutput = flag(b, "output");
        kb.isTemp = flag(b, "temp");
        kb.elements = num(b, "elements", mlk::constants::kKernelLoopDynamicBound);
        if (const mlk::json::Value* d = b.find("dims"); d != nullptr && d->isArray()) {
            for (const mlk::json::Value& x : d->asArray()) kb.dims.push_back(x.asInt());
        }
        (void)km.addBuffer(kb);
    }
    for (const mlk::json::Value& n : nodes->asArray()) {
        mlk::KernelNode kn;
        const std::string op = str(n, "op");
        bool found = false;
        for (int i = 0; i < static_cast<int>(mlk::KernelOp::kCount); ++i) {
            if (op == mlk::kernelOpName(static_cast<mlk::KernelOp>(i))) {
                kn.op = static_cast<mlk::KernelOp>(i);
                found = true;
            }
        }
        if (!found) {
            g_err = "unknown node op " + op;
            return false;
        }
        if (n.find("math") != nullptr) (void)mlk::opByName(str(n, "math").c_str(), kn.math);
        if (const std::string f = str(n, "family"); !f.empty()) kn.family = sy.intern(f);
        if (const std::string v = str(n, "var"); !v.empty()) kn.var = sy.intern(v);
        kn.begin = num(n, "begin", 0);
        kn.end = num(n, "end", mlk::constants::kKernelLoopDynamicBound);
        kn.step = num(n, "step", 1);
        kn.parallel = flag(n, "parallel");
        auto id = [&](const char* k) {
            const int64_t v = num(n, k, -1);
            return v < 0 ? mlk::constants::kInvalidId : static_cast<uint32_t>(v);
        };
        kn.bufferA = id("a");
        kn.bufferB = id("b");
        kn.bufferOut = id("out");
        if (const mlk::json::Value* xs = n.find("exprs"); xs != nullptr && xs->isArray()) {
            for (const mlk::json::Value& x : xs->asArray()) {
                mlk::KernelExpr e;
                (void)mlk::opByName(str(x, "op").c_str(), e.op);
                for (int side = 0; side < 2; ++side) {
                    const mlk::json::Value* o = x.find(side == 0 ? "a" : "b");
                    mlk::KernelOperand& kop = side == 0 ? e.a : e.b;
                    if (o == nullptr) continue;
                    static const char* kKinds[] = {"const", "elem_a", "elem_b", "scalar_param",
                                                   "temp"};
                    const std::string k = str(*o, "kind");
                    for (int i = 0; i < 5; ++i) {
                        if (k == kKinds[i]) kop.kind = static_cast<mlk::KernelOperand::Kind>(i);
                    }
                    kop.index = num(*o, "index", 0);
                    if (const mlk::json::Value* v = o->find("value"); v != nullptr && v->isNumber()) {
                        kop.constValue = v->asDouble();
                    }
                }
                kn.exprs.push_back(e);
            }
        }
        if (const mlk::json::Value* cs = n.find("children"); cs != nullptr && cs->isArray()) {
            for (const mlk::json::Value& c : cs->asArray()) {
                kn.children.push_back(static_cast<uint32_t>(c.asInt()));
            }
        }
        if (kn.op == mlk::KernelOp::Call && n.find("math") == nullptr) {
            if (kn.bufferB != mlk::constants::kInvalidId) {
                kn.math = mlk::MathOp::MatMul;
            } else if (kn.bufferOut < km.buffers.size() && km.buffers[kn.bufferOut].dims.size() == 2) {
                kn.math = mlk::MathOp::Softmax;
            } else {
                kn.math = mlk::MathOp::ReduceSum;
            }
        }
        (void)km.addNode(kn);
    }
    if (const mlk::json::Value* sc = doc->find("schedule"); sc != nullptr && sc->isObject()) {
        for (const mlk::json::Member& kv : sc->asObject()) {
            if (kv.value != nullptr && kv.value->isNumber()) {
                *km.scheduleParams.findOrInsert(sy.intern(kv.key), nullptr) = kv.value->asInt();
            }
        }
    }
    return true;
}

// ---- modules from the reference's own compiler ------------------------------
// Graphs of `x`, a tensor [n] of f32 or f64 (the constant 3 carries the same
// tensor type: the Tier-1 type inference rejects a scalar constant against a
// tensor operand):
//   which 0: sin(x*x + 3x)               the graph of examples/scalar/sin_graph.mlk
//   which 1: Derivative(sin(x*x + 3x), x) first lowered by the reference's
//            calculus.derivative_symbolic and calculus.derivative_simplify
//            (the Tier-2/3 calculus steps, pipeline_runner.cpp:71-72; Tier 1
//            lists neither, so Tier 1 alone would leave the Derivative op in
//            the chain)
//   which 2: the scalar form of which 0 (x a scalar f64 placeholder), which
//            lowers to a one-element kernel reading x as ScalarParam 0.
// Then the Tier-1 pipeline to a KernelModule, as mlkc runs it. One
// workaround for a reference defect is applied and reported: after the
// calculus steps, math.canonicalize folds the product rule's 3*1 into a
// constant whose type is left unset, which the following type inference
// rejects ("operands require implicit coercion"); such constants are given
// x's type before the pipeline runs.
inline bool pipelineModule(int which, int64_t n, bool f32, mlk::SymbolTable& symbols,
                    mlk::KernelModule& kernel, int* patched) {
    mlk::passes::registerAllPasses(symbols);
    mlk::DiagnosticEngine diag;
    mlk::MathDomainProfile profile;
    profile.name = symbols.intern("mlkb-oracle");
    profile.capabilities.set(mlk::Capability::HasNumericValues);
    profile.capabilities.set(mlk::Capability::HasFloatingPoint);
    profile.capabilities.set(mlk::Capability::HasTensorDomain);
    profile.capabilities.set(mlk::Capability::HasCalculus);
    profile.capabilities.set(mlk::Capability::HasDerivatives);
    profile.capabilities.set(mlk::Capability::HasAlgebraicRewriting);
    profile.capabilities.set(mlk::Capability::HasKernelFusion);
    profile.capabilities.set(mlk::Capability::HasCPUBackend);
    profile.lawCommutativeMul = mlk::TriState::True;
    profile.lawAssociativeAdd = mlk::TriState::Unknown;
    mlk::AccuracyContract contract;
    mlk::GraphBuilder b(symbols);
    const mlk::Dtype dt = f32 ? mlk::Dtype::F32 : mlk::Dtype::F64;
    const mlk::MathType ty = which == 2
                                 ? mlk::MathType::scalar(mlk::Domain::Float, mlk::Dtype::F64)
                                 : mlk::MathType::tensorValue(dt, {n});
    const mlk::ValueId x = b.placeholder("x", ty);
    const mlk::ValueId three = b.constant(3.0, ty);
    auto xx = b.op(mlk::MathOp::Mul, {x, x});
    auto tx = b.op(mlk::MathOp::Mul, {three, x});
    if (!xx || !tx) return false;
    auto u = b.op(mlk::MathOp::Add, {*xx, *tx});
    if (!u) return false;
    auto s = b.op(mlk::MathOp::Sin, {*u});
    if (!s) return false;
    mlk::PassContext ctx;
    ctx.domainProfile = &profile;
    ctx.accuracy = &contract;
    ctx.diag = &diag;
    ctx.symbols = &symbols;
    *patched = 0;
    if (which == 1) {
        auto d = b.op(mlk::MathOp::Derivative, {*s, x});
        if (!d) return false;
        b.output(*d);
        ctx.tier = mlk::Tier::Tier2;
        for (const char* nm : {"calculus.derivative_symbolic", "calculus.derivative_simplify"}) {
            mlk::Pass* pass = mlk::PassRegistry::instance().byName(symbols, symbols.intern(nm));
            if (pass == nullptr) {
                g_err = std::string("pass not registered: ") + nm;
                return false;
            }
            auto r = pass->run(ctx, b.graph());
            if (!r.has_value()) {
                g_err = r.error().message;
                return false;
            }
        }
        for (uint32_t v = 0; v < b.graph().numValues(); ++v) {
            mlk::Value& val = b.graph().value(v);
            if (val.kind == mlk::ValueKind::Constant && val.type.domain == mlk::Domain::Unknown) {
                val.type = ty;
                ++*patched;
            }
        }
    } else {
        b.output(*s);
    }
    mlk::TelemetrySink telemetry;
    mlk::PipelineRunner runner(symbols, &telemetry);
    ctx.telemetry = &telemetry;
    ctx.tier = mlk::Tier::Tier1;
    ctx.kernelOut = &kernel;
    auto r = runner.run(mlk::Tier::Tier1, ctx, b.graph(), &kernel);
    if (!r.has_value()) {
        g_err = r.error().message;
        return false;
    }
    return true;
}

}  // namespace mlkb_oracle
