// Integration check of libmlkb200 with a PATCHED copy of the reference
// (oracle/ref_patches/*.patch, built by oracle/ref_patched.mk).
//
// TEST INFRASTRUCTURE ONLY (tests/test_ref_integration.py; the fastkernel
// mode also runs on a GPU box). One JSON line per result.
//
//   ref_integration_check lowering
//       the reference's own compiler on a graph with TWO outputs,
//       y = sin(x^2+3x) and dy = Derivative(y, x) over x[4096]: its calculus
//       passes, then Tier 1 with the patched lowering (each output's Store
//       targets its own buffer); prints the module's mlk-kernel JSON.
//   ref_integration_check arch
//       the patched arch validation through buildGpuKernelArtifact (emit +
//       nvcc, no launch) for sm_100a, sm_90a and two malformed names.
//   ref_integration_check fastkernel <libmlkb200.so>
//       runFastKernelSearch (fastkernel/src/fast_kernel.cpp) with the walker
//       and a NativeCuda candidate on the prebuilt library, over a GEMM graph
//       (bit-exact policy) and the config-1 map graph (declared ULP bound).
#include <cstdio>
#include <cstdlib>
#include <string>

#include "mlk/backend/backend_driver.h"
#include "mlk/fastkernel/fast_kernel.h"
#include "ref_modules.h"

namespace {

std::string quoted(const std::string& s) {
    std::string o = "\"";
    for (char c : s) {
        if (c == '"' || c == '\\') o += '\\';
        if (c == '\n') {
            o += "\\n";
            continue;
        }
        o += c;
    }
    return o + "\"";
}

mlk::MathDomainProfile profileFor(mlk::SymbolTable& symbols) {
    mlk::MathDomainProfile profile;
    profile.name = symbols.intern("mlkb-integration");
    profile.capabilities.set(mlk::Capability::HasNumericValues);
    profile.capabilities.set(mlk::Capability::HasFloatingPoint);
    profile.capabilities.set(mlk::Capability::HasTensorDomain);
    profile.capabilities.set(mlk::Capability::HasKernelFusion);
    profile.capabilities.set(mlk::Capability::HasAlgebraicRewriting);
    profile.capabilities.set(mlk::Capability::HasDerivatives);
    profile.capabilities.set(mlk::Capability::HasCalculus);
    profile.capabilities.set(mlk::Capability::HasApproximation);
    return profile;
}

int lowering() {
    mlk::SymbolTable symbols;
    mlk::passes::registerAllPasses(symbols);
    mlk::MathDomainProfile profile = profileFor(symbols);
    mlk::DiagnosticEngine diag;
    mlk::AccuracyContract contract;
    mlk::GraphBuilder b(symbols);
    const mlk::MathType ty = mlk::MathType::tensorValue(mlk::Dtype::F32, {4096});
    const mlk::ValueId x = b.placeholder("x", ty);
    const mlk::ValueId three = b.constant(3.0, ty);
    auto u = b.op(mlk::MathOp::Add, {*b.op(mlk::MathOp::Mul, {x, x}),
                                     *b.op(mlk::MathOp::Mul, {three, x})});
    auto y = b.op(mlk::MathOp::Sin, {*u});
    auto dy = b.op(mlk::MathOp::Derivative, {*y, x});
    if (!y || !dy) return 1;
    b.output(*y);
    b.output(*dy);
    mlk::PassContext ctx;
    ctx.domainProfile = &profile;
    ctx.accuracy = &contract;
    ctx.diag = &diag;
    ctx.symbols = &symbols;
    ctx.tier = mlk::Tier::Tier2;
    for (const char* nm : {"calculus.derivative_symbolic", "calculus.derivative_simplify"}) {
        auto r = mlk::PassRegistry::instance().byName(symbols, symbols.intern(nm))->run(ctx, b.graph());
        if (!r.has_value()) {
            std::printf("{\"ok\":false,\"stage\":%s,\"error\":%s}\n", quoted(nm).c_str(),
                        quoted(r.error().message).c_str());
            return 1;
        }
    }
    // The one reference defect the unpatched pipeline also needs worked
    // around (oracle/ref_modules.h): a folded constant left untyped.
    for (uint32_t v = 0; v < b.graph().numValues(); ++v) {
        mlk::Value& val = b.graph().value(v);
        if (val.kind == mlk::ValueKind::Constant && val.type.domain == mlk::Domain::Unknown) {
            val.type = ty;
        }
    }
    mlk::TelemetrySink telemetry;
    mlk::KernelModule kernel;
    mlk::PipelineRunner runner(symbols, &telemetry);
    ctx.telemetry = &telemetry;
    ctx.tier = mlk::Tier::Tier1;
    ctx.kernelOut = &kernel;
    auto r = runner.run(mlk::Tier::Tier1, ctx, b.graph(), &kernel);
    if (!r.has_value()) {
        std::printf("{\"ok\":false,\"stage\":\"tier1\",\"error\":%s}\n",
                    quoted(r.error().message).c_str());
        return 1;
    }
    std::printf("%s\n", mlk::json::serialize(kernel.toJson(symbols)).c_str());
    return 0;
}

int arch() {
    mlk::SymbolTable symbols;
    mlk::KernelModule km;
    mlk::KernelBuffer in, out;
    in.name = symbols.intern("x");
    in.isInput = true;
    out.name = symbols.intern("y");
    out.isOutput = true;
    (void)km.addBuffer(in);
    (void)km.addBuffer(out);
    mlk::KernelNode loop, comp, st;
    loop.op = mlk::KernelOp::Loop;
    loop.var = symbols.intern("i");
    comp.op = mlk::KernelOp::Compute;
    comp.math = mlk::MathOp::Neg;
    comp.bufferA = 0;
    st.op = mlk::KernelOp::Store;
    st.bufferOut = 1;
    const uint32_t l = km.addNode(loop);
    const uint32_t c = km.addNode(comp);
    const uint32_t s = km.addNode(st);
    km.nodes[l].children = {c, s};
    for (const char* a : {"sm_100a", "sm_90a", "sm_100x", "sm_a"}) {
        mlk::GpuBackendDriverConfig cfg;
        cfg.arch = a;
        cfg.workdirBase = "oracle/_ref/patched/work";
        auto built = mlk::buildGpuKernelArtifact(km, symbols, cfg);
        std::printf("{\"arch\":%s,\"built\":%s,\"code\":%d,\"error\":%s}\n", quoted(a).c_str(),
                    built.has_value() ? "true" : "false",
                    built.has_value() ? 0 : static_cast<int>(built.error().code),
                    quoted(built.has_value() ? "" : built.error().message.substr(0, 160)).c_str());
    }
    return 0;
}

int fastkernel(const std::string& lib) {
    using namespace mlk::fastkernel;
    struct Job {
        const char* name;
        uint32_t maxUlp;
    };
    for (const Job job : {Job{"gemm_64x48x56", 0}, Job{"map_sin_4096", 16}}) {
        mlk::SymbolTable symbols;
        mlk::passes::registerAllPasses(symbols);
        mlk::MathDomainProfile profile = profileFor(symbols);
        mlk::GraphBuilder b(symbols);
        if (job.maxUlp == 0) {
            const mlk::ValueId pa = b.placeholder("A", mlk::MathType::tensorValue(mlk::Dtype::F64, {64, 48}));
            const mlk::ValueId pb = b.placeholder("B", mlk::MathType::tensorValue(mlk::Dtype::F64, {48, 56}));
            b.output(*b.op(mlk::MathOp::MatMul, {pa, pb}));
        } else {
            const mlk::MathType ty = mlk::MathType::tensorValue(mlk::Dtype::F64, {4096});
            const mlk::ValueId x = b.placeholder("x", ty);
            const mlk::ValueId three = b.constant(3.0, ty);
            auto u = b.op(mlk::MathOp::Add, {*b.op(mlk::MathOp::Mul, {x, x}),
                                             *b.op(mlk::MathOp::Mul, {three, x})});
            b.output(*b.op(mlk::MathOp::Sin, {*u}));
        }
        mlk::MathGraph graph = b.graph();
        FastKernelSearchConfig cfg;
        cfg.tileSizes = {0};
        cfg.execPaths = {ExecPath::Walker, ExecPath::NativeCuda};
        cfg.threadCounts = {0};
        cfg.warmupReps = 1;
        cfg.benchReps = 3;
        cfg.budget.mode = BudgetMode::SameComptime;
        cfg.budget.baselineComptimeSec = 600.0;
        cfg.measureEnvironment = false;
        cfg.env.bandwidthBytesPerSec = 2.5e10;
        cfg.env.throughputOpsPerSec = 2.5e9;
        cfg.env.hardwareThreads = 2;
        cfg.env.descriptor = "mlkb-integration-env";
        cfg.gpu.arch = "sm_100a";
        cfg.gpu.prebuiltLibrary = lib;
        cfg.cudaMaxUlp = job.maxUlp;
        auto report = runFastKernelSearch(graph, symbols, profile, cfg);
        if (!report.has_value()) {
            std::printf("{\"graph\":%s,\"ok\":false,\"error\":%s}\n", quoted(job.name).c_str(),
                        quoted(report.error().message).c_str());
            continue;
        }
        for (const VariantOutcome& o : report->candidates) {
            std::printf("{\"graph\":%s,\"exec\":%s,\"admissible\":%s,\"identity\":%s,"
                        "\"policy\":%s,\"max_abs_diff\":%.17g,\"max_ulp\":%.17g,"
                        "\"reject\":%s,\"detail\":%s,\"runtime_sec\":%.9g,\"library\":%s}\n",
                        quoted(job.name).c_str(), quoted(execPathName(o.config.exec)).c_str(),
                        o.admissible ? "true" : "false",
                        o.cert.identityCertified ? "true" : "false",
                        quoted(o.cert.identityPolicy).c_str(), o.cert.identityMaxAbsDiff,
                        o.cert.identityMaxUlp, quoted(rejectReasonName(o.reject)).c_str(),
                        quoted(o.rejectDetail.substr(0, 200)).c_str(),
                        o.cert.runtimeUpperBoundSec, quoted(o.cert.libraryPath).c_str());
        }
    }
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    const std::string mode = argc > 1 ? argv[1] : "";
    if (mode == "lowering") return lowering();
    if (mode == "arch") return arch();
    if (mode == "fastkernel" && argc > 2) return fastkernel(argv[2]);
    std::fprintf(stderr, "usage: %s lowering | arch | fastkernel <libmlkb200.so>\n", argv[0]);
    return 2;
}
