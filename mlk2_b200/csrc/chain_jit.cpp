// Chains compiled at run time into straight-line streaming kernels.
//
// The reference turns a Kernel IR module into CUDA source
// (backends/cpu/src/cuda_emitter.cpp:1558 emitCudaSource), writes it and
// builds it with an out-of-process nvcc (backends/cpu/src/backend_driver.cpp:
// 348-360, stages 3-4 at :720-733). This
// library keeps its drop-in promise — no nvcc, no files — and still avoids an
// interpreter's per-expression dispatch on the generic chain path: the first
// launch of a chain STRUCTURE (ops, operand kinds, temp indices, poly7,
// element type, second input) generates a kernel whose body is the chain
// written out as SSA statements, compiles it in-process with NVRTC for
// sm_100a straight to a cubin, loads it with cudaLibraryLoadData and caches
// it. Constant and ScalarParam operands are kernel parameters, not literals,
// so one compiled kernel serves every value of them (a scalar table that
// changes per call does not recompile). The statements call the same
// `mlkb::chain::apply<>` the interpreter uses (chain_math.cuh, embedded
// below and compiled by both compilers with the same contraction setting),
// so the compiled and the interpreted chain round identically.
//
// NVRTC is loaded with dlopen (MLKB_NVRTC_LIB, else libnvrtc.so.12): a host
// without it runs every chain on the interpreter; nothing here is needed for
// correctness. MLKB_CHAIN_JIT=0 in the environment, or mlkb_chain_compile(0,
// ...), selects the interpreter. MLKB_CACHE_DIR keeps compiled chains on disk
// for later processes (off unless set).
#include <dlfcn.h>
#include <nvrtc.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"

namespace mlkb {
namespace {

const char kChainMathSrc[] =
#include "chain_math_src.inc"
    ;

constexpr int kJitThreads = 256;
constexpr int kJitUnroll = 1;  // 16-byte vectors per thread per step (1, 2 and 4 measured)

// ---- NVRTC, loaded on first use ------------------------------------------------
struct NvrtcApi {
    bool ok = false;
    std::string why;
    nvrtcResult (*create)(nvrtcProgram*, const char*, const char*, int, const char* const*,
                          const char* const*) = nullptr;
    nvrtcResult (*compile)(nvrtcProgram, int, const char* const*) = nullptr;
    nvrtcResult (*cubinSize)(nvrtcProgram, size_t*) = nullptr;
    nvrtcResult (*cubin)(nvrtcProgram, char*) = nullptr;
    nvrtcResult (*logSize)(nvrtcProgram, size_t*) = nullptr;
    nvrtcResult (*log)(nvrtcProgram, char*) = nullptr;
    nvrtcResult (*destroy)(nvrtcProgram*) = nullptr;
    nvrtcResult (*version)(int*, int*) = nullptr;
};

const NvrtcApi& nvrtc() {
    static const NvrtcApi api = [] {
        NvrtcApi a;
        const char* env = std::getenv("MLKB_NVRTC_LIB");
        void* h = nullptr;
        if (env != nullptr && env[0] != '\0') {
            h = ::dlopen(env, RTLD_NOW | RTLD_LOCAL);
        } else {
            h = ::dlopen("libnvrtc.so.12", RTLD_NOW | RTLD_LOCAL);
            if (h == nullptr) h = ::dlopen("libnvrtc.so", RTLD_NOW | RTLD_LOCAL);
        }
        if (h == nullptr) {
            const char* e = ::dlerror();
            a.why = std::string("NVRTC not loadable: ") + (e != nullptr ? e : "?");
            return a;
        }
        auto sym = [&](const char* name) { return ::dlsym(h, name); };
        a.create = reinterpret_cast<decltype(a.create)>(sym("nvrtcCreateProgram"));
        a.compile = reinterpret_cast<decltype(a.compile)>(sym("nvrtcCompileProgram"));
        a.cubinSize = reinterpret_cast<decltype(a.cubinSize)>(sym("nvrtcGetCUBINSize"));
        a.cubin = reinterpret_cast<decltype(a.cubin)>(sym("nvrtcGetCUBIN"));
        a.logSize = reinterpret_cast<decltype(a.logSize)>(sym("nvrtcGetProgramLogSize"));
        a.log = reinterpret_cast<decltype(a.log)>(sym("nvrtcGetProgramLog"));
        a.destroy = reinterpret_cast<decltype(a.destroy)>(sym("nvrtcDestroyProgram"));
        a.version = reinterpret_cast<decltype(a.version)>(sym("nvrtcVersion"));
        a.ok = a.create && a.compile && a.cubinSize && a.cubin && a.logSize && a.log && a.destroy &&
               a.version;
        if (!a.ok) a.why = "NVRTC library lacks an entry point";
        return a;
    }();
    return api;
}

std::atomic<int> g_mode{-1};              // -1: not yet read from the environment
std::atomic<int64_t> g_compiled{0}, g_launched{0};

int jitMode() {
    int m = g_mode.load();
    if (m < 0) {
        const char* env = std::getenv("MLKB_CHAIN_JIT");
        m = (env != nullptr && env[0] == '0') ? 0 : 1;
        int expect = -1;
        g_mode.compare_exchange_strong(expect, m);
        m = g_mode.load();
    }
    return m;
}

// ---- source generation -----------------------------------------------------------
// One kernel evaluates a GROUP of chains (the roots of a map module that read
// the same inputs over the same range; a lone chain is a group of one): the
// inputs are loaded once and every chain's result is stored to its own
// output. The loop: a grid-stride loop over 16-byte vectors (kJitUnroll of
// them in flight per thread, streaming loads and stores) when every buffer is
// 16-byte aligned, then an element loop for the tail or for unaligned
// buffers. Launched with programmatic stream serialization, like the other
// map kernels: it waits for the preceding grid before touching memory and
// lets the next grid's blocks be scheduled as its own retire.
const char kPreludeSrc[] = R"MLKB(
template <typename V> struct MlkbVec;
template <> struct MlkbVec<float> { typedef float4 V; enum { kN = 4 }; };
template <> struct MlkbVec<double> { typedef double2 V; enum { kN = 2 }; };
struct MlkbOuts { MlkbT* p[8]; };
template <int R> __device__ double mlkb_eval(double A, double B, const MlkbConsts& c);
template <int R>
__device__ __forceinline__ float4 mlkb_eval_vec(float4 x, float4 y, const MlkbConsts& c) {
    return make_float4(static_cast<float>(mlkb_eval<R>(x.x, y.x, c)),
                       static_cast<float>(mlkb_eval<R>(x.y, y.y, c)),
                       static_cast<float>(mlkb_eval<R>(x.z, y.z, c)),
                       static_cast<float>(mlkb_eval<R>(x.w, y.w, c)));
}
template <int R>
__device__ __forceinline__ double2 mlkb_eval_vec(double2 x, double2 y, const MlkbConsts& c) {
    return make_double2(mlkb_eval<R>(x.x, y.x, c), mlkb_eval<R>(x.y, y.y, c));
}
)MLKB";

const char kKernelHead[] = R"MLKB(
extern "C" __global__ void __launch_bounds__(256)
mlkb_chain_kernel(const MlkbT* __restrict__ a, const MlkbT* __restrict__ b,
                  const __grid_constant__ MlkbOuts o, long long n, int vec,
                  const __grid_constant__ MlkbConsts c) {
    typedef typename MlkbVec<MlkbT>::V V;
    const int kN = MlkbVec<MlkbT>::kN;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const long long nth = static_cast<long long>(gridDim.x) * blockDim.x;
    const long long tid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    long long done = 0;
    if (vec) {
        const long long nv = n / kN;
        const V* av = reinterpret_cast<const V*>(a);
        const V* bv = reinterpret_cast<const V*>(b);
        for (long long base = tid; base < nv; base += nth * MLKB_UNROLL) {
            V x[MLKB_UNROLL] = {}, y[MLKB_UNROLL] = {};
#pragma unroll
            for (int u = 0; u < MLKB_UNROLL; ++u) {
                const long long i = base + u * nth;
                if (i < nv) {
                    if (MLKB_USES_A) x[u] = __ldcs(av + i);
                    if (MLKB_USES_B) y[u] = __ldcs(bv + i);
                }
            }
#pragma unroll
            for (int u = 0; u < MLKB_UNROLL; ++u) {
                const long long i = base + u * nth;
                if (i < nv) {
)MLKB";

const char kKernelMid[] = R"MLKB(
                }
            }
        }
        done = nv * kN;
    }
    for (long long i = done + tid; i < n; i += nth) {
        const double va = MLKB_USES_A ? static_cast<double>(a[i]) : 0.0;
        const double vb = MLKB_USES_B ? static_cast<double>(b[i]) : 0.0;
)MLKB";

const char kKernelTail[] = R"MLKB(
    }
}
)MLKB";

// A group's generated source. The text determines the compiled kernel, so it
// is also the cache key; constants are numbered in operand order over all
// chains and read from the kernel's parameter block.
struct Generated {
    std::string src;
    std::vector<double> consts;
    bool usesA = false, usesB = false;
};

Generated generate(const JitExpr* const* chains, const int* ns, const bool* poly7, int nChains,
                   bool f64) {
    Generated g;
    std::string evals;
    char buf[256];
    auto operand = [&](int kind, int idx, double val) -> std::string {
        switch (kind) {
            case chain::kElemA: g.usesA = true; return "A";
            case chain::kElemB: g.usesB = true; return "B";
            case chain::kTemp:
                std::snprintf(buf, sizeof buf, "t%d", idx);
                return buf;
            default:
                std::snprintf(buf, sizeof buf, "c.v[%zu]", g.consts.size());
                g.consts.push_back(val);
                return buf;
        }
    };
    for (int j = 0; j < nChains; ++j) {
        const JitExpr* e = chains[j];
        std::snprintf(buf, sizeof buf,
                      "template <> __device__ __forceinline__ double mlkb_eval<%d>("
                      "double A, double B, const MlkbConsts& c) {\n"
                      "    (void)A; (void)B; (void)c;\n", j);
        evals += buf;
        for (int k = 0; k < ns[j]; ++k) {
            const std::string x = operand(e[k].akind, e[k].aidx, e[k].aval);
            const std::string y =
                e[k].unary ? std::string("0.0") : operand(e[k].bkind, e[k].bidx, e[k].bval);
            std::snprintf(buf, sizeof buf, "    const double t%d = mlkb::chain::apply<%s>(%uu, ",
                          k, f64 ? "true" : "false", static_cast<unsigned>(e[k].op));
            evals += buf;
            evals += x + ", " + y + (poly7[j] ? ", true);\n" : ", false);\n");
        }
        std::snprintf(buf, sizeof buf, "    return t%d;\n}\n", ns[j] - 1);
        evals += buf;
    }
    const size_t nc = g.consts.empty() ? 1 : g.consts.size();
    std::snprintf(buf, sizeof buf,
                  "#include \"mlkb_chain_math.cuh\"\n"
                  "typedef %s MlkbT;\n"
                  "#define MLKB_UNROLL %d\n#define MLKB_USES_A %d\n#define MLKB_USES_B %d\n"
                  "struct MlkbConsts { double v[%zu]; };\n",
                  f64 ? "double" : "float", kJitUnroll, g.usesA ? 1 : 0, g.usesB ? 1 : 0, nc);
    g.src = buf;
    g.src += kPreludeSrc;
    g.src += evals;
    g.src += kKernelHead;
    for (int j = 0; j < nChains; ++j) {  // vector stores, one per chain
        std::snprintf(buf, sizeof buf,
                      "                    __stcs(reinterpret_cast<V*>(o.p[%d]) + i, "
                      "mlkb_eval_vec<%d>(x[u], y[u], c));\n", j, j);
        g.src += buf;
    }
    g.src += kKernelMid;
    for (int j = 0; j < nChains; ++j) {  // element stores
        std::snprintf(buf, sizeof buf,
                      "        o.p[%d][i] = static_cast<MlkbT>(mlkb_eval<%d>(va, vb, c));\n", j, j);
        g.src += buf;
    }
    g.src += kKernelTail;
    return g;
}

// ---- compile, load, cache ---------------------------------------------------------
struct Compiled {
    std::vector<char> cubin;
    std::string error;            // non-empty: compilation failed (the log's head)
    cudaLibrary_t lib = nullptr;  // loaded on first launch
    cudaKernel_t kernel = nullptr;
    int blocksPerSm[64] = {};
};

std::mutex g_cacheMu;
std::unordered_map<std::string, std::unique_ptr<Compiled>> g_cache;

// A group's structure as a compact byte string (everything generate() turns
// into source text except the constants' values), so a repeated launch finds
// its kernel without generating the source again.
struct Known {
    Compiled* c;
    bool usesA, usesB;
};
std::unordered_map<std::string, Known> g_known;  // guarded by g_cacheMu

std::string structKey(const JitExpr* const* chains, const int* ns, const bool* poly7, int nChains,
                      bool f64) {
    std::string k;
    k.reserve(16 + 8 * 64);
    k.push_back(static_cast<char>(f64 ? 1 : 0));
    k.push_back(static_cast<char>(nChains));
    for (int j = 0; j < nChains; ++j) {
        k.push_back(static_cast<char>(poly7[j] ? 1 : 0));
        k.push_back(static_cast<char>(ns[j]));
        for (int e = 0; e < ns[j]; ++e) {
            const JitExpr& x = chains[j][e];
            const bool tempA = x.akind == chain::kTemp, tempB = x.bkind == chain::kTemp;
            k.push_back(static_cast<char>(x.op));
            k.push_back(static_cast<char>(x.unary));
            k.push_back(static_cast<char>(x.akind));
            k.push_back(static_cast<char>(tempA ? x.aidx : 0));
            k.push_back(static_cast<char>(x.unary ? 0 : x.bkind));
            k.push_back(static_cast<char>(!x.unary && tempB ? x.bidx : 0));
        }
    }
    return k;
}

// The constants of a group in generate()'s numbering: operand order, chain
// by chain (every operand that is not ElemA, ElemB or a temp; a unary op's
// second operand is not an operand).
void constsOf(const JitExpr* const* chains, const int* ns, int nChains, std::vector<double>& v) {
    auto take = [&](int kind, double val) {
        if (kind != chain::kElemA && kind != chain::kElemB && kind != chain::kTemp) v.push_back(val);
    };
    for (int j = 0; j < nChains; ++j) {
        for (int e = 0; e < ns[j]; ++e) {
            const JitExpr& x = chains[j][e];
            take(x.akind, x.aval);
            if (!x.unary) take(x.bkind, x.bval);
        }
    }
}

// ---- optional cache of compiled chains on disk ------------------------------------
// With MLKB_CACHE_DIR set, every compiled cubin is also written there and
// later processes load it instead of compiling. A file holds a magic word,
// the length of the generated source, the source itself and the cubin; it
// is used only when its source equals the one wanted, so a hash collision
// cannot load a wrong kernel. The file name hashes the source with the NVRTC
// version and the target, so a new compiler or header never reuses an old
// file. Files are written to a temporary name and renamed into place.
constexpr char kCacheMagic[8] = {'M', 'L', 'K', 'B', 'C', 'U', 'B', '1'};

std::string cachePath(const std::string& src) {
    const char* dir = std::getenv("MLKB_CACHE_DIR");
    if (dir == nullptr || dir[0] == '\0') return std::string();
    int major = 0, minor = 0;
    nvrtc().version(&major, &minor);
    const std::string key = src + "|sm_100a|nvrtc" + std::to_string(major) + "." +
                            std::to_string(minor);
    uint64_t h = 1469598103934665603ull;  // FNV-1a, 64 bit
    for (unsigned char ch : key) {
        h ^= ch;
        h *= 1099511628211ull;
    }
    char name[64];
    std::snprintf(name, sizeof name, "/mlkb-chain-%016llx.cubin",
                  static_cast<unsigned long long>(h));
    return std::string(dir) + name;
}

bool loadCached(const std::string& path, const std::string& src, std::vector<char>& cubin) {
    FILE* f = std::fopen(path.c_str(), "rb");
    if (f == nullptr) return false;
    char magic[8];
    uint64_t len = 0;
    bool ok = std::fread(magic, 1, 8, f) == 8 && std::memcmp(magic, kCacheMagic, 8) == 0 &&
              std::fread(&len, sizeof len, 1, f) == 1 && len == src.size();
    if (ok) {
        std::string stored(len, '\0');
        ok = std::fread(&stored[0], 1, len, f) == len && stored == src;
    }
    if (ok) {
        std::vector<char> bin;
        char buf[65536];
        size_t got;
        while ((got = std::fread(buf, 1, sizeof buf, f)) > 0) bin.insert(bin.end(), buf, buf + got);
        ok = !bin.empty();
        if (ok) cubin.swap(bin);
    }
    std::fclose(f);
    return ok;
}

void storeCached(const std::string& path, const std::string& src, const std::vector<char>& cubin) {
    const std::string dir = path.substr(0, path.rfind('/'));
    ::mkdir(dir.c_str(), 0755);  // one level; an existing directory is fine
    const std::string tmp = path + ".tmp." + std::to_string(::getpid());
    FILE* f = std::fopen(tmp.c_str(), "wb");
    if (f == nullptr) return;
    const uint64_t len = src.size();
    const bool ok = std::fwrite(kCacheMagic, 1, 8, f) == 8 &&
                    std::fwrite(&len, sizeof len, 1, f) == 1 &&
                    std::fwrite(src.data(), 1, src.size(), f) == src.size() &&
                    std::fwrite(cubin.data(), 1, cubin.size(), f) == cubin.size();
    if (std::fclose(f) == 0 && ok) {
        std::rename(tmp.c_str(), path.c_str());
    } else {
        std::remove(tmp.c_str());
    }
}

void compileInto(const std::string& src, Compiled& c) {
    const NvrtcApi& api = nvrtc();
    const std::string cached = cachePath(src);
    if (!cached.empty() && loadCached(cached, src, c.cubin)) return;
    nvrtcProgram prog = nullptr;
    const char* hdrs[1] = {kChainMathSrc};
    const char* names[1] = {"mlkb_chain_math.cuh"};
    if (api.create(&prog, src.c_str(), "mlkb_chain.cu", 1, hdrs, names) != NVRTC_SUCCESS) {
        c.error = "nvrtcCreateProgram failed";
        return;
    }
    const char* opts[] = {"--gpu-architecture=sm_100a", "--std=c++17", "--fmad=true"};
    const nvrtcResult r = api.compile(prog, 3, opts);
    if (r != NVRTC_SUCCESS) {
        size_t ls = 0;
        api.logSize(prog, &ls);
        std::string log(ls, '\0');
        if (ls > 0) api.log(prog, &log[0]);
        c.error = "chain compile failed: " + log.substr(0, 400);
    } else {
        size_t cs = 0;
        api.cubinSize(prog, &cs);
        c.cubin.resize(cs);
        if (cs == 0 || api.cubin(prog, c.cubin.data()) != NVRTC_SUCCESS) {
            c.error = "chain compile produced no cubin";
        } else {
            ++g_compiled;
            if (!cached.empty()) storeCached(cached, src, c.cubin);
        }
    }
    api.destroy(&prog);
}

// The cache entry for `src`, compiled if new (under the cache lock: a
// compile takes a fraction of a second, and two threads wanting the same new
// chain should not both build it).
Compiled* entryFor(const std::string& src) {
    std::lock_guard<std::mutex> lk(g_cacheMu);
    auto it = g_cache.find(src);
    if (it != g_cache.end()) return it->second.get();
    auto c = std::make_unique<Compiled>();
    compileInto(src, *c);
    Compiled* p = c.get();
    g_cache.emplace(src, std::move(c));
    return p;
}

}  // namespace

int launchChainsJit(const JitExpr* const* chains, const int* n_exprs, const bool* poly7,
                    int n_chains, const void* a, const void* b, void* const* outs, int dtype,
                    int64_t n, cudaStream_t s) {
    if (jitMode() == 0 || !nvrtc().ok || n_chains < 1 || n_chains > kMaxJitOuts) {
        return kJitUnavailable;
    }
    const bool f64 = dtype == MLKB_F64;
    const std::string key = structKey(chains, n_exprs, poly7, n_chains, f64);
    Known known{nullptr, false, false};
    {
        std::lock_guard<std::mutex> lk(g_cacheMu);
        auto it = g_known.find(key);
        if (it != g_known.end()) known = it->second;
    }
    if (known.c == nullptr) {  // first launch of this structure: generate, compile
        Generated g = generate(chains, n_exprs, poly7, n_chains, f64);
        known = Known{entryFor(g.src), g.usesA, g.usesB};
        std::lock_guard<std::mutex> lk(g_cacheMu);
        g_known.emplace(key, known);
    }
    Compiled* c = known.c;
    if ((known.usesA && a == nullptr) || (known.usesB && b == nullptr)) return kJitUnavailable;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
    int per = 0;
    {
        std::lock_guard<std::mutex> lk(g_cacheMu);  // c->error, c->lib and the occupancy cache
        if (!c->error.empty()) return kJitUnavailable;
        if (c->lib == nullptr) {
            // A cubin the driver will not load (a damaged cache file, say) is
            // not an error for the caller: the entry is marked unusable and
            // the chain runs on the interpreter.
            cudaError_t le = cudaLibraryLoadData(&c->lib, c->cubin.data(), nullptr, nullptr, 0,
                                                 nullptr, nullptr, 0);
            if (le == cudaSuccess) le = cudaLibraryGetKernel(&c->kernel, c->lib, "mlkb_chain_kernel");
            if (le != cudaSuccess) {
                cudaGetLastError();
                c->lib = nullptr;
                c->error = std::string("compiled chain not loadable: ") + cudaGetErrorString(le);
                return kJitUnavailable;
            }
        }
        per = dev >= 0 && dev < 64 ? c->blocksPerSm[dev] : 0;
        if (per == 0) {
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                    &per, reinterpret_cast<const void*>(c->kernel), kJitThreads, 0) !=
                    cudaSuccess ||
                per <= 0) {
                per = 1;
            }
            if (dev >= 0 && dev < 64) c->blocksPerSm[dev] = per;
        }
    }
    struct {
        void* p[8];
    } o = {};
    bool vec = aligned16(a) && aligned16(b);
    for (int j = 0; j < n_chains; ++j) {
        o.p[j] = outs[j];
        vec = vec && aligned16(outs[j]);
    }
    // threads wanted: one per kJitUnroll vectors (16 B each), or one per element
    const int64_t units = vec ? (n / (f64 ? 2 : 4) + kJitUnroll - 1) / kJitUnroll : n;
    const int64_t need = (units + kJitThreads - 1) / kJitThreads;
    const int64_t cap = static_cast<int64_t>(smCount()) * per;
    const int grid = static_cast<int>(need < cap ? (need > 0 ? need : 1) : cap);

    std::vector<double> consts;
    constsOf(chains, n_exprs, n_chains, consts);
    if (consts.empty()) consts.push_back(0.0);
    long long nn = n;
    int vflag = vec ? 1 : 0;
    void* args[6] = {const_cast<void**>(&a), const_cast<void**>(&b), &o, &nn, &vflag,
                     consts.data()};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kJitThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t le =
        cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(c->kernel), args);
    if (le != cudaSuccess) return setCudaError(MLKB_ERR_LAUNCH, le, "compiled chain launch");
    ++g_launched;
    return okStatus();
}

int launchChainJit(const JitExpr* e, int n_exprs, bool poly7, const void* a, const void* b,
                   void* out, int dtype, int64_t n, cudaStream_t s) {
    const JitExpr* chains[1] = {e};
    const int ns[1] = {n_exprs};
    const bool p7[1] = {poly7};
    void* outs[1] = {out};
    return launchChainsJit(chains, ns, p7, 1, a, b, outs, dtype, n, s);
}

int buildChainJit(const JitExpr* e, int n_exprs, bool poly7, int dtype, const char** why) {
    if (!nvrtc().ok) {
        if (why) *why = nvrtc().why.c_str();
        return kJitUnavailable;
    }
    const JitExpr* chains[1] = {e};
    const int ns[1] = {n_exprs};
    const bool p7[1] = {poly7};
    Generated g = generate(chains, ns, p7, 1, dtype == MLKB_F64);
    const Compiled* c = entryFor(g.src);  // entries live as long as the process
    std::lock_guard<std::mutex> lk(g_cacheMu);
    if (!c->error.empty()) {
        if (why) *why = c->error.c_str();  // set once, never changed afterwards
        return kJitUnavailable;
    }
    return MLKB_OK;
}

}  // namespace mlkb

extern "C" int32_t mlkb_chain_compile(int32_t mode, int64_t* compiled, int64_t* launched) {
    using namespace mlkb;
    jitMode();
    if (mode == 0 || mode == 1) g_mode.store(mode);
    if (compiled != nullptr) *compiled = g_compiled.load();
    if (launched != nullptr) *launched = g_launched.load();
    return g_mode.load() != 0 && nvrtc().ok ? 1 : 0;
}
