// Drop-in check: drives the B200 shim through the REFERENCE's own artifact
// loader, exactly as its fastkernel search and mlk-poly bench do.
//
// TEST INFRASTRUCTURE ONLY (run by tests/test_dropin_gpu.py on a GPU box).
//
// For each module it
//   1. builds the KernelModule with the reference's types,
//   2. binds it in the shim with mlk_bind_module(toJson(module)),
//   3. loads the shim with mlk::loadKernelLibrary (reference
//      backends/cpu/src/backend_driver.cpp:607-630) and calls
//      LoadedKernel::run (:821-1050) over host f64 buffers,
//   4. runs the same module through mlk::executeKernelOnBuffers
//      (runtime/src/execution/kernel_buffers.cpp:839) and prints the largest
//      f64 ULP distance between the two, one JSON line per case.
// Exit status: 0 when every case ran (the calling test checks the distances).
#include <dlfcn.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "mlk/backend/backend_driver.h"
#include "mlk/runtime/execution.h"
#include "mlk/support/json.h"
#include "mlk/support/kernel_ir.h"
#include "ref_modules.h"

namespace {

using BindFn = int (*)(const char*);
using StatusFn = int (*)();

double ulp64(double a, double b) {
    if (std::isnan(a) && std::isnan(b)) return 0.0;
    if (std::isnan(a) || std::isnan(b)) return INFINITY;
    if (a == b) return 0.0;
    auto ord = [](double d) {
        int64_t v;
        std::memcpy(&v, &d, 8);
        return v >= 0 ? v : static_cast<int64_t>(0x8000000000000000LL) - v;
    };
    const int64_t x = ord(a), y = ord(b);
    return static_cast<double>(x > y ? x - y : y - x);
}

mlk::KernelOperand opnd(mlk::KernelOperand::Kind k, double v = 0.0,
                        int64_t idx = 0) {
    mlk::KernelOperand o;
    o.kind = k;
    o.constValue = v;
    o.index = idx;
    return o;
}

mlk::KernelExpr ex(mlk::MathOp op, mlk::KernelOperand a,
                   mlk::KernelOperand b = {}) {
    mlk::KernelExpr e;
    e.op = op;
    e.a = a;
    e.b = b;
    return e;
}

using K = mlk::KernelOperand::Kind;

// u = x*x + 3x as the reference lowering emits it (Mul, Mul, Add).
void pushU(mlk::KernelNode& c) {
    c.exprs.push_back(ex(mlk::MathOp::Mul, opnd(K::ElemA), opnd(K::ElemA)));
    c.exprs.push_back(ex(mlk::MathOp::Mul, opnd(K::Const, 3.0), opnd(K::ElemA)));
    c.exprs.push_back(ex(mlk::MathOp::Add, opnd(K::Temp, 0, 0), opnd(K::Temp, 0, 1)));
}

void addRoot(mlk::KernelModule& km, mlk::SymbolTable& sy, uint32_t in,
             uint32_t out, bool deriv, bool poly7 = false) {
    mlk::KernelNode loop;
    loop.op = mlk::KernelOp::Loop;
    loop.var = sy.intern(deriv ? "j" : "i");
    mlk::KernelNode c;
    c.op = mlk::KernelOp::Compute;
    c.bufferA = in;
    pushU(c);
    if (!deriv) {
        c.exprs.push_back(ex(mlk::MathOp::Sin, opnd(K::Temp, 0, 2)));
    } else {
        c.exprs.push_back(ex(mlk::MathOp::Cos, opnd(K::Temp, 0, 2)));
        c.exprs.push_back(ex(mlk::MathOp::Mul, opnd(K::Const, 2.0), opnd(K::ElemA)));
        c.exprs.push_back(ex(mlk::MathOp::Add, opnd(K::Temp, 0, 4), opnd(K::Const, 3.0)));
        c.exprs.push_back(ex(mlk::MathOp::Mul, opnd(K::Temp, 0, 3), opnd(K::Temp, 0, 5)));
    }
    c.math = c.exprs[c.exprs.size() - 1].op;
    if (poly7) c.family = sy.intern("poly7");
    mlk::KernelNode st;
    st.op = mlk::KernelOp::Store;
    st.bufferOut = out;
    const uint32_t l = km.addNode(loop);
    const uint32_t ci = km.addNode(c);
    const uint32_t si = km.addNode(st);
    km.nodes[l].children.push_back(ci);
    km.nodes[l].children.push_back(si);
}

mlk::KernelBuffer buf(mlk::SymbolTable& sy, const char* name, bool in,
                      std::vector<int64_t> dims) {
    mlk::KernelBuffer b;
    b.name = sy.intern(name);
    b.isInput = in;
    b.isOutput = !in;
    for (int64_t d : dims) b.dims.push_back(d);
    return b;
}

struct Case {
    std::string name;
    mlk::KernelModule km;
    std::vector<std::vector<double>> ins;
    std::vector<size_t> outSizes;
    int64_t elements;
    std::vector<double> scalars = {};
};

int runCase(Case& c, mlk::SymbolTable& sy, const std::string& shim,
            BindFn bind, StatusFn status) {
    const std::string js = mlk::json::serialize(c.km.toJson(sy));
    const int b = bind(js.c_str());
    std::vector<std::vector<double>> ref, got;
    for (size_t s : c.outSizes) {
        ref.emplace_back(s, 0.0);
        got.emplace_back(s, 0.0);
    }
    auto bindIo = [&](std::vector<std::vector<double>>& outs) {
        mlk::KernelBufferBindings io;
        for (auto& v : c.ins) io.inputs.push_back(v.data());
        for (auto& v : outs) io.outputs.push_back(v.data());
        io.elements = c.elements;
        for (double v : c.scalars) io.scalars.push_back(v);
        return io;
    };
    auto rr = mlk::executeKernelOnBuffers(c.km, sy, bindIo(ref), nullptr);
    auto loaded = mlk::loadKernelLibrary(c.km, sy, shim);
    if (b != 0 || !rr.has_value() || !loaded.has_value()) {
        std::printf("{\"case\":\"%s\",\"ok\":false,\"stage\":\"%s\"}\n",
                    c.name.c_str(), b != 0 ? "bind" : !rr.has_value() ? "ref" : "load");
        return 1;
    }
    auto rg = loaded->run(c.km, sy, bindIo(got));
    const int st = status();
    double worst = 0.0;
    for (size_t o = 0; o < ref.size(); ++o) {
        for (size_t i = 0; i < ref[o].size(); ++i) {
            const double d = ulp64(ref[o][i], got[o][i]);
            if (d > worst) worst = d;
        }
    }
    std::printf("{\"case\":\"%s\",\"ok\":%s,\"status\":%d,\"multi_dim\":%s,"
                "\"max_ulp_f64\":%.17g}\n",
                c.name.c_str(), rg.has_value() ? "true" : "false", st,
                loaded->isMultiDim() ? "true" : "false", worst);
    return rg.has_value() ? 0 : 1;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 2) {
        std::fprintf(stderr, "usage: %s <libmlkb200.so>\n", argv[0]);
        return 2;
    }
    const std::string shim = argv[1];
    void* h = ::dlopen(shim.c_str(), RTLD_NOW | RTLD_LOCAL);
    if (h == nullptr) {
        std::fprintf(stderr, "dlopen: %s\n", ::dlerror());
        return 2;
    }
    auto bind = reinterpret_cast<BindFn>(::dlsym(h, "mlk_bind_module"));
    auto status = reinterpret_cast<StatusFn>(::dlsym(h, "mlk_last_status"));
    if (bind == nullptr || status == nullptr) return 2;

    mlk::SymbolTable sy;
    std::vector<Case> cases;
    const int64_t n = 1 << 16;
    std::vector<double> x(n);
    for (int64_t i = 0; i < n; ++i) x[i] = -4.0 + 8.0 * (double)i / (double)n;
    {  // config-1 shape: y = sin(x^2 + 3x)
        Case c{"map_sin", {}, {x}, {(size_t)n}, n};
        const uint32_t in = c.km.addBuffer(buf(sy, "x", true, {}));
        const uint32_t out = c.km.addBuffer(buf(sy, "y", false, {}));
        addRoot(c.km, sy, in, out, false);
        cases.push_back(std::move(c));
    }
    {  // config-2 shape: two roots, y and dy/dx
        Case c{"map_sin_dsin", {}, {x}, {(size_t)n, (size_t)n}, n};
        const uint32_t in = c.km.addBuffer(buf(sy, "x", true, {}));
        const uint32_t y = c.km.addBuffer(buf(sy, "y", false, {}));
        const uint32_t dy = c.km.addBuffer(buf(sy, "dy", false, {}));
        addRoot(c.km, sy, in, y, false);
        addRoot(c.km, sy, in, dy, true);
        cases.push_back(std::move(c));
    }
    {  // Call(Softmax) with the reference test's inputs and a NaN row
        const int64_t m = 12, k = 8;
        std::vector<double> a(m * k);
        for (int64_t i = 0; i < m * k; ++i) a[i] = ((i * 13) % 19) * 0.25 - 2.0;
        a[9 * k + 2] = std::nan("");
        Case c{"softmax", {}, {a}, {(size_t)(m * k)}, m * k};
        const uint32_t ia = c.km.addBuffer(buf(sy, "A", true, {m, k}));
        const uint32_t iy = c.km.addBuffer(buf(sy, "Y", false, {m, k}));
        mlk::KernelNode call;
        call.op = mlk::KernelOp::Call;
        call.math = mlk::MathOp::Softmax;
        call.bufferA = ia;
        call.bufferOut = iy;
        (void)c.km.addNode(call);
        cases.push_back(std::move(c));
    }
    {  // Call(MatMul): the cuda_driver_honest_skip operands (bit-exact bar)
        const int64_t m = 16, kk = 14, nn = 12;
        std::vector<double> a(m * kk), b(kk * nn);
        for (int64_t i = 0; i < m * kk; ++i) a[i] = (i % 7) * 0.25;
        for (int64_t i = 0; i < kk * nn; ++i) b[i] = (i % 5) * 0.5;
        Case c{"matmul", {}, {a, b}, {(size_t)(m * nn)}, m * nn};
        const uint32_t ia = c.km.addBuffer(buf(sy, "A", true, {m, kk}));
        const uint32_t ib = c.km.addBuffer(buf(sy, "B", true, {kk, nn}));
        const uint32_t ic = c.km.addBuffer(buf(sy, "C", false, {m, nn}));
        mlk::KernelNode call;
        call.op = mlk::KernelOp::Call;
        call.math = mlk::MathOp::MatMul;
        call.bufferA = ia;
        call.bufferB = ib;
        call.bufferOut = ic;
        (void)c.km.addNode(call);
        cases.push_back(std::move(c));
    }
    {  // config-1 chain with the poly7 sine family (bit-exact bar)
        Case c{"map_poly7", {}, {x}, {(size_t)n}, n};
        const uint32_t in = c.km.addBuffer(buf(sy, "x", true, {}));
        const uint32_t out = c.km.addBuffer(buf(sy, "y", false, {}));
        addRoot(c.km, sy, in, out, false, true);
        cases.push_back(std::move(c));
    }
    {  // the scaled-scores composite as the reference runs it: S += Q*Kt,
       // Sc = S * 1/sqrt(d), Y = softmax(Sc), every intermediate an output
        const int64_t s_ = 128, d = 64;
        std::vector<double> q(s_ * d), kt(d * s_);
        for (int64_t i = 0; i < s_ * d; ++i) q[i] = ((i * 37) % 23) * 0.125 - 1.375;
        for (int64_t i = 0; i < d * s_; ++i) kt[i] = ((i * 11) % 17) * 0.0625 - 0.5;
        Case c{"qk_composite", {}, {q, kt}, {(size_t)(s_ * s_), (size_t)(s_ * s_), (size_t)(s_ * s_)},
               s_ * s_};
        const uint32_t iq = c.km.addBuffer(buf(sy, "Q", true, {s_, d}));
        const uint32_t ik = c.km.addBuffer(buf(sy, "Kt", true, {d, s_}));
        const uint32_t is = c.km.addBuffer(buf(sy, "S", false, {s_, s_}));
        const uint32_t isc = c.km.addBuffer(buf(sy, "Sc", false, {s_, s_}));
        const uint32_t iy = c.km.addBuffer(buf(sy, "Y", false, {s_, s_}));
        mlk::KernelNode mm;
        mm.op = mlk::KernelOp::Call;
        mm.math = mlk::MathOp::MatMul;
        mm.bufferA = iq;
        mm.bufferB = ik;
        mm.bufferOut = is;
        (void)c.km.addNode(mm);
        mlk::KernelNode loop;
        loop.op = mlk::KernelOp::Loop;
        loop.var = sy.intern("i");
        mlk::KernelNode comp;
        comp.op = mlk::KernelOp::Compute;
        comp.bufferA = is;
        comp.exprs.push_back(ex(mlk::MathOp::Mul, opnd(K::ElemA), opnd(K::Const, 0.125)));
        comp.math = mlk::MathOp::Mul;
        mlk::KernelNode st;
        st.op = mlk::KernelOp::Store;
        st.bufferOut = isc;
        const uint32_t l = c.km.addNode(loop);
        const uint32_t ci = c.km.addNode(comp);
        const uint32_t si = c.km.addNode(st);
        c.km.nodes[l].children.push_back(ci);
        c.km.nodes[l].children.push_back(si);
        mlk::KernelNode sm;
        sm.op = mlk::KernelOp::Call;
        sm.math = mlk::MathOp::Softmax;
        sm.bufferA = isc;
        sm.bufferOut = iy;
        (void)c.km.addNode(sm);
        cases.push_back(std::move(c));
    }
    // Modules the reference's own Tier-1 pipeline compiles (ref_modules.h):
    // sin(x^2+3x) over x[n], its derivative through the calculus passes, and
    // the scalar form (x a ScalarParam). Each gets its own symbol table.
    static mlk::SymbolTable psy[3];
    for (int which = 0; which < 3; ++which) {
        static const char* kNames[3] = {"pipeline_sin", "pipeline_dsin", "pipeline_scalar"};
        const int64_t pn = which == 2 ? 1 : n;
        Case c{kNames[which], {}, {}, {(size_t)pn}, pn};
        int patched = 0;
        if (!mlkb_oracle::pipelineModule(which, pn, false, psy[which], c.km, &patched)) {
            std::printf("{\"case\":\"%s\",\"ok\":false,\"stage\":\"pipeline\",\"error\":\"%s\"}\n",
                        kNames[which], mlkb_oracle::g_err.c_str());
            return 1;
        }
        if (which == 2) {
            c.scalars = {2.0};
        } else {
            c.ins = {x};
        }
        cases.push_back(std::move(c));
    }
    int bad = 0;
    for (size_t i = 0; i < cases.size(); ++i) {
        Case& c = cases[i];
        const bool pipe = c.name.rfind("pipeline_", 0) == 0;
        mlk::SymbolTable& table = pipe ? psy[c.name == "pipeline_sin" ? 0 : c.name == "pipeline_dsin" ? 1 : 2] : sy;
        bad += runCase(c, table, shim, bind, status);
    }
    return bad == 0 ? 0 : 1;
}
