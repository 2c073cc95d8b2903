// `mlk-kernel` JSON parsing and module classification.
//
// The wire format is what KernelModule::toJson writes (reference
// compiler/src/support/kernel_ir.cpp:97-254). Classification mirrors the
// reference executor's dispatch (runtime/src/execution/kernel_buffers.cpp):
//   * any multi-dim feature (accumulate/max stores, affine bounds, stores or
//     guards, buffer-dim bounds, ElemIdx operands; :883-901 and the artifact
//     ABI rule isMultiDimModule, backends/cpu/src/cpp_emitter.cpp:667-687)
//     marks the module multi-dim. Poly-scheduled nests are not this path:
//     such modules are reported MLKB_ERR_UNSUPPORTED;
//   * top-level Loop nodes pair their Compute with the first Store among
//     their children (:921-953): one MapRoot each;
//   * a single top-level Call is MatMul / Softmax / ReduceSum (:1001-1085).
//     toJson does not serialise a Call's `math` (kernel_ir.cpp:130-135), so
//     when the field is absent the op is inferred from the operands the
//     executor validates: a B operand means MatMul (:1014-1037); otherwise a
//     rank-2 output means Softmax (:301-304) and a rank-1 output ReduceSum
//     (:248-251).
//   * three top-level nodes Call(MatMul) -> Loop{x * const} -> Call(Softmax)
//     chained through their buffers are the scaled-scores softmax composite.
#include <cctype>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>

#include "common.cuh"
#include "module.h"

namespace mlkb {
namespace {

// ---- minimal JSON DOM -------------------------------------------------------
struct JVal {
    enum T { Null, Bool, Num, Str, Arr, Obj } t = Null;
    bool b = false;
    double num = 0.0;
    bool isInt = false;
    int64_t i = 0;
    std::string s;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;

    const JVal* get(const char* key) const {
        if (t != Obj) return nullptr;
        for (const auto& kv : obj) {
            if (kv.first == key) return &kv.second;
        }
        return nullptr;
    }
};

struct Parser {
    const char* p;
    const char* end;
    bool ok = true;

    void ws() {
        while (p < end && std::isspace(static_cast<unsigned char>(*p))) ++p;
    }
    bool lit(const char* w) {
        const size_t n = std::strlen(w);
        if (static_cast<size_t>(end - p) >= n && std::strncmp(p, w, n) == 0) {
            p += n;
            return true;
        }
        return false;
    }
    std::string str() {
        std::string out;
        if (p >= end || *p != '"') {
            ok = false;
            return out;
        }
        ++p;
        while (p < end && *p != '"') {
            if (*p == '\\' && p + 1 < end) {
                ++p;
                switch (*p) {
                    case 'n': out += '\n'; break;
                    case 't': out += '\t'; break;
                    case 'r': out += '\r'; break;
                    case 'b': out += '\b'; break;
                    case 'f': out += '\f'; break;
                    case 'u': {
                        if (end - p < 5) { ok = false; return out; }
                        const long cp = std::strtol(std::string(p + 1, p + 5).c_str(), nullptr, 16);
                        out += cp < 0x80 ? static_cast<char>(cp) : '?';
                        p += 4;
                        break;
                    }
                    default: out += *p; break;
                }
                ++p;
            } else {
                out += *p++;
            }
        }
        if (p >= end) {
            ok = false;
            return out;
        }
        ++p;
        return out;
    }
    JVal val(int depth) {
        JVal v;
        if (depth > 64) {
            ok = false;
            return v;
        }
        ws();
        if (p >= end) {
            ok = false;
            return v;
        }
        if (*p == '{') {
            ++p;
            v.t = JVal::Obj;
            ws();
            if (p < end && *p == '}') {
                ++p;
                return v;
            }
            while (ok) {
                ws();
                std::string k = str();
                ws();
                if (p >= end || *p != ':') {
                    ok = false;
                    break;
                }
                ++p;
                v.obj.emplace_back(std::move(k), val(depth + 1));
                ws();
                if (p < end && *p == ',') {
                    ++p;
                    continue;
                }
                if (p < end && *p == '}') {
                    ++p;
                    break;
                }
                ok = false;
            }
        } else if (*p == '[') {
            ++p;
            v.t = JVal::Arr;
            ws();
            if (p < end && *p == ']') {
                ++p;
                return v;
            }
            while (ok) {
                v.arr.push_back(val(depth + 1));
                ws();
                if (p < end && *p == ',') {
                    ++p;
                    continue;
                }
                if (p < end && *p == ']') {
                    ++p;
                    break;
                }
                ok = false;
            }
        } else if (*p == '"') {
            v.t = JVal::Str;
            v.s = str();
        } else if (lit("true")) {
            v.t = JVal::Bool;
            v.b = true;
        } else if (lit("false")) {
            v.t = JVal::Bool;
        } else if (lit("null")) {
            v.t = JVal::Null;
        } else {
            const char* s0 = p;
            bool frac = false;
            while (p < end && (std::isdigit(static_cast<unsigned char>(*p)) || *p == '-' ||
                               *p == '+' || *p == '.' || *p == 'e' || *p == 'E')) {
                frac = frac || *p == '.' || *p == 'e' || *p == 'E';
                ++p;
            }
            if (p == s0) {
                ok = false;
                return v;
            }
            const std::string tok(s0, p);
            v.t = JVal::Num;
            v.num = std::strtod(tok.c_str(), nullptr);
            if (!frac) {
                v.isInt = true;
                v.i = std::strtoll(tok.c_str(), nullptr, 10);
            } else {
                v.i = static_cast<int64_t>(v.num);
            }
        }
        return v;
    }
};

int64_t getInt(const JVal& o, const char* k, int64_t dflt) {
    const JVal* v = o.get(k);
    return (v != nullptr && v->t == JVal::Num) ? v->i : dflt;
}
bool getBool(const JVal& o, const char* k) {
    const JVal* v = o.get(k);
    return v != nullptr && v->t == JVal::Bool && v->b;
}
std::string getStr(const JVal& o, const char* k) {
    const JVal* v = o.get(k);
    return (v != nullptr && v->t == JVal::Str) ? v->s : std::string();
}

int mathByName(const std::string& s) {
    static const char* kNames[] = {"add", "sub", "mul", "div", "neg", "pow", "exp", "log",
                                   "sin", "cos", "tan", "tanh", "sqrt", "rsqrt", "erf", "gelu",
                                   "matmul", "dot", "transpose", "reshape", "broadcast",
                                   "reduce_sum", "reduce_max", "reduce_mean", "softmax"};
    for (int i = 0; i < static_cast<int>(sizeof(kNames) / sizeof(kNames[0])); ++i) {
        if (s == kNames[i]) return i;
    }
    return -1;
}

int kopByName(const std::string& s) {
    static const char* kNames[] = {"loop", "compute", "load", "store", "alloc",
                                   "copy", "barrier", "trace", "guard", "call"};
    for (int i = 0; i < 10; ++i) {
        if (s == kNames[i]) return i;
    }
    return -1;
}

int dtypeByName(const std::string& s) {
    if (s == "f16") return MLKB_F16;
    if (s == "f32") return MLKB_F32;
    if (s == "f64") return MLKB_F64;
    return 0;  // other element types: not this path
}

int operandKind(const std::string& s) {
    if (s == "const") return 0;
    if (s == "elem_a") return 1;
    if (s == "elem_b") return 2;
    if (s == "scalar_param") return 3;
    if (s == "temp") return 4;
    if (s == "elem_idx") return 5;
    return -1;
}

int classify(Module& m) {
    // isMultiDimModule (cpp_emitter.cpp:667-687).
    for (const KNode& n : m.nodes) m.multiDim = m.multiDim || n.multiDimFeature;
    for (int b = 0; b < static_cast<int>(m.buffers.size()); ++b) {
        if (m.buffers[b].input || m.buffers[b].output) m.bindable.push_back(b);
    }
    if (m.multiDim) {
        return setError(MLKB_ERR_UNSUPPORTED,
                        "module: multi-dim (poly-scheduled) nests are not on the B200 path");
    }
    std::vector<uint8_t> isChild(m.nodes.size(), 0);
    for (const KNode& n : m.nodes) {
        for (uint32_t c : n.children) {
            if (c >= m.nodes.size()) return setError(MLKB_ERR_INVALID, "module: child out of range");
            isChild[c] = 1;
        }
    }
    std::vector<int> tops;
    for (int i = 0; i < static_cast<int>(m.nodes.size()); ++i) {
        const KOp op = m.nodes[i].op;
        // Standalone non-Loop/Call ops are ignored by the executor (:1086-1099).
        if (!isChild[i] && (op == KOp::Loop || op == KOp::Call)) tops.push_back(i);
    }
    if (tops.empty()) return setError(MLKB_ERR_UNSUPPORTED, "module: no Loop or Call root");
    const int nb = static_cast<int>(m.buffers.size());
    auto validBuf = [&](int64_t id) { return id >= 0 && id < nb; };

    bool allLoops = true;
    for (int t : tops) allLoops = allLoops && m.nodes[t].op == KOp::Loop;
    if (allLoops) {
        for (int t : tops) {
            const KNode& loop = m.nodes[t];
            const KNode* store = nullptr;
            for (uint32_t c : loop.children) {
                if (m.nodes[c].op == KOp::Store) {
                    store = &m.nodes[c];
                    break;
                }
            }
            for (uint32_t c : loop.children) {
                const KNode& comp = m.nodes[c];
                if (comp.op != KOp::Compute) continue;
                MapRoot r;
                r.begin = loop.begin;
                r.end = loop.end;
                r.poly7 = comp.family == "poly7";
                r.a = static_cast<int>(comp.a);
                r.b = static_cast<int>(comp.b);
                r.out = static_cast<int>(store != nullptr ? store->out : comp.out);
                if (comp.exprs.empty()) {
                    // Legacy single-op Compute: math over ElemA (+ElemB) (:390-401).
                    mlkb_expr e{};
                    e.op = comp.math;
                    e.a_kind = 1;
                    e.b_kind = 2;
                    r.chain.push_back(e);
                } else {
                    r.chain = comp.exprs;
                }
                bool readsA = false, readsB = false;
                for (const mlkb_expr& e : r.chain) {
                    readsA = readsA || e.a_kind == 1 || (!isUnaryOp(e.op) && e.b_kind == 1);
                    readsB = readsB || e.a_kind == 2 || (!isUnaryOp(e.op) && e.b_kind == 2);
                }
                if (!readsA) r.a = -1;
                if (!readsB) r.b = -1;
                if (!validBuf(r.out) || (readsA && !validBuf(r.a)) || (readsB && !validBuf(r.b))) {
                    return setError(MLKB_ERR_INVALID, "module: map root buffer out of range");
                }
                if (int st = checkChain(r.chain.data(), static_cast<int32_t>(r.chain.size()),
                                        readsB)) {
                    return st;
                }
                m.roots.push_back(std::move(r));
            }
        }
        if (m.roots.empty()) return setError(MLKB_ERR_UNSUPPORTED, "module: loops without compute");
        m.kind = MLKB_KIND_MAP;
        return okStatus();
    }

    auto callMath = [&](const KNode& c) -> int {
        if (c.math >= 0) return c.math;
        if (c.b >= 0) return kMathMatMul;
        if (validBuf(c.out) && m.buffers[c.out].dims.size() == 2) return kMathSoftmax;
        return kMathReduceSum;
    };

    if (tops.size() == 1 && m.nodes[tops[0]].op == KOp::Call) {
        const KNode& c = m.nodes[tops[0]];
        const int math = callMath(c);
        if (!validBuf(c.a) || !validBuf(c.out) || (math == kMathMatMul && !validBuf(c.b))) {
            return setError(MLKB_ERR_INVALID, "call: buffer id out of range");
        }
        const KBuffer& ba = m.buffers[c.a];
        const KBuffer& bo = m.buffers[c.out];
        m.callA = static_cast<int>(c.a);
        m.callB = static_cast<int>(c.b);
        m.callOut = static_cast<int>(c.out);
        if (math == kMathMatMul) {
            const KBuffer& bb = m.buffers[c.b];
            if (ba.dims.size() != 2 || bb.dims.size() != 2 || bo.dims.size() != 2) {
                return setError(MLKB_ERR_INVALID, "matmul requires rank-2 buffer dims");
            }
            m.m = ba.dims[0];
            m.k = ba.dims[1];
            m.n = bb.dims[1];
            if (bb.dims[0] != m.k || bo.dims[0] != m.m || bo.dims[1] != m.n || m.m <= 0 ||
                m.k <= 0 || m.n <= 0) {
                return setError(MLKB_ERR_INVALID, "matmul operand shapes incompatible");
            }
            m.kind = MLKB_KIND_MATMUL;
        } else if (math == kMathSoftmax) {
            if (ba.dims.size() != 2 || bo.dims.size() != 2) {
                return setError(MLKB_ERR_INVALID, "softmax requires rank-2 operand and output");
            }
            m.m = ba.dims[0];
            m.k = ba.dims[1];
            if (bo.dims[0] != m.m || bo.dims[1] != m.k || m.k <= 0 || m.m <= 0) {
                return setError(MLKB_ERR_INVALID, "softmax operand shapes incompatible");
            }
            m.kind = MLKB_KIND_SOFTMAX;
        } else if (math == kMathReduceSum) {
            if (ba.dims.size() != 2 || bo.dims.size() != 1) {
                return setError(MLKB_ERR_INVALID, "reducesum requires rank-2 input over rank-1 output");
            }
            m.m = ba.dims[0];
            m.k = ba.dims[1];
            if (bo.dims[0] != m.m || m.k <= 0 || m.m <= 0) {
                return setError(MLKB_ERR_INVALID, "reducesum operand shapes incompatible");
            }
            m.kind = MLKB_KIND_REDUCESUM;
        } else {
            return setError(MLKB_ERR_UNSUPPORTED, "call: no executor for call target");
        }
        return okStatus();
    }

    // Call(MatMul) -> Loop{ElemA * const} -> Call(Softmax) composite: the
    // executor runs the three top-level nodes in order (:921-1085), so
    // S (+)= Q*Kt, Sc[i] = S[i] * scale over the loop range, Y = softmax(Sc).
    if (tops.size() == 3 && m.nodes[tops[0]].op == KOp::Call &&
        m.nodes[tops[1]].op == KOp::Loop && m.nodes[tops[2]].op == KOp::Call) {
        const KNode& mm = m.nodes[tops[0]];
        const KNode& sm = m.nodes[tops[2]];
        const KNode& loop = m.nodes[tops[1]];
        const KNode* comp = nullptr;
        const KNode* store = nullptr;
        for (uint32_t c : loop.children) {
            if (m.nodes[c].op == KOp::Compute && comp == nullptr) comp = &m.nodes[c];
            if (m.nodes[c].op == KOp::Store && store == nullptr) store = &m.nodes[c];
        }
        if (callMath(mm) == kMathMatMul && callMath(sm) == kMathSoftmax && comp != nullptr &&
            store != nullptr && comp->exprs.size() == 1 && comp->exprs[0].op == 2 &&
            validBuf(mm.a) && validBuf(mm.b) && validBuf(mm.out) && validBuf(sm.out) &&
            validBuf(store->out) && comp->a == mm.out && store->out == sm.a) {
            const mlkb_expr& e = comp->exprs[0];
            const bool aConst = e.a_kind == 0 && e.b_kind == 1;
            const bool bConst = e.b_kind == 0 && e.a_kind == 1;
            const KBuffer& bq = m.buffers[mm.a];
            const KBuffer& bk = m.buffers[mm.b];
            const KBuffer& bs = m.buffers[mm.out];
            const KBuffer& bsc = m.buffers[store->out];
            const KBuffer& by = m.buffers[sm.out];
            if ((aConst || bConst) && bq.dims.size() == 2 && bk.dims.size() == 2) {
                const int64_t rows = bq.dims[0], d = bq.dims[1], keys = bk.dims[1];
                auto is2 = [&](const KBuffer& b) {
                    return b.dims.size() == 2 && b.dims[0] == rows && b.dims[1] == keys;
                };
                // The shape checks execGemm and execSoftmaxCall make (:1014-1037, :294-316).
                if (bk.dims[0] != d || rows <= 0 || d <= 0 || keys <= 0 || !is2(bs) || !is2(by) ||
                    (!bsc.dims.empty() && !is2(bsc))) {
                    return setError(MLKB_ERR_INVALID, "qk composite: operand shapes incompatible");
                }
                if (mm.a == mm.out || mm.b == mm.out || store->out == sm.out || mm.out == sm.out ||
                    !(bq.input && bk.input) || !by.output) {
                    return setError(MLKB_ERR_UNSUPPORTED,
                                    "qk composite: Q and Kt must be inputs and Y an output, "
                                    "all distinct");
                }
                // The scores S and scaled scores Sc are either both temps
                // (only Y observable: the fused kernel) or both outputs.
                const bool sTemp = bs.temp && !bs.output, scTemp = bsc.temp && !bsc.output;
                if (sTemp != scTemp || (!sTemp && !(bs.output && bsc.output))) {
                    return setError(MLKB_ERR_UNSUPPORTED,
                                    "qk composite: S and Sc must be both temps or both outputs");
                }
                if (loop.begin < 0 || (loop.end >= 0 && loop.end > rows * keys)) {
                    return setError(MLKB_ERR_INVALID, "qk composite: scale map range exceeds S");
                }
                MapRoot r;
                r.begin = loop.begin;
                r.end = loop.end;
                r.a = static_cast<int>(mm.out);
                r.out = static_cast<int>(store->out);
                r.chain = comp->exprs;
                m.roots.clear();
                m.roots.push_back(std::move(r));
                m.scale = aConst ? e.a_value : e.b_value;
                m.callA = static_cast<int>(mm.a);
                m.callB = static_cast<int>(mm.b);
                m.qkS = static_cast<int>(mm.out);
                m.qkSc = static_cast<int>(store->out);
                m.qkFused = sTemp;
                m.callOut = static_cast<int>(sm.out);
                m.m = rows;
                m.k = d;
                m.n = keys;
                m.kind = MLKB_KIND_QK_SOFTMAX;
                return okStatus();
            }
        }
    }
    return setError(MLKB_ERR_UNSUPPORTED, "module: node forest not recognised by the B200 path");
}

}  // namespace

int parseModule(const char* json, Module& out) {
    if (json == nullptr) return setError(MLKB_ERR_INVALID, "module: null JSON");
    Parser ps{json, json + std::strlen(json)};
    JVal doc = ps.val(0);
    if (!ps.ok || doc.t != JVal::Obj) return setError(MLKB_ERR_INVALID, "module: malformed JSON");
    if (getStr(doc, "format") != "mlk-kernel") {
        return setError(MLKB_ERR_INVALID, "module: format is not mlk-kernel");
    }
    const JVal* bufs = doc.get("buffers");
    const JVal* nodes = doc.get("nodes");
    if (bufs == nullptr || bufs->t != JVal::Arr || nodes == nullptr || nodes->t != JVal::Arr) {
        return setError(MLKB_ERR_INVALID, "module: buffers/nodes arrays missing");
    }
    Module m;
    for (const JVal& b : bufs->arr) {
        KBuffer kb;
        kb.name = getStr(b, "name");
        const std::string dt = getStr(b, "dtype");
        kb.dtype = dt.empty() ? MLKB_F64 : dtypeByName(dt);
        kb.input = getBool(b, "input");
        kb.output = getBool(b, "output");
        kb.temp = getBool(b, "temp");
        kb.elements = getInt(b, "elements", -1);
        if (const JVal* d = b.get("dims"); d != nullptr && d->t == JVal::Arr) {
            for (const JVal& x : d->arr) kb.dims.push_back(x.i);
        }
        // Every later size computation starts from these shapes: each extent
        // in [0, 2^31) and at most 2^40 elements, so byte counts cannot overflow.
        constexpr int64_t kMaxElements = int64_t(1) << 40;
        int64_t count = 1;
        for (const int64_t d : kb.dims) {
            if (d < 0 || d > INT32_MAX || (d != 0 && count > kMaxElements / d)) {
                return setError(MLKB_ERR_INVALID, "module: buffer shape out of range");
            }
            count *= d;
        }
        if (kb.elements > kMaxElements) {
            return setError(MLKB_ERR_INVALID, "module: buffer element count out of range");
        }
        m.buffers.push_back(std::move(kb));
    }
    for (const JVal& n : nodes->arr) {
        KNode kn;
        const int op = kopByName(getStr(n, "op"));
        if (op < 0) return setError(MLKB_ERR_INVALID, "module: unknown node op");
        kn.op = static_cast<KOp>(op);
        kn.math = n.get("math") != nullptr ? mathByName(getStr(n, "math")) : -1;
        kn.family = getStr(n, "family");
        kn.begin = getInt(n, "begin", 0);
        kn.end = getInt(n, "end", -1);
        kn.step = getInt(n, "step", 1);
        kn.a = getInt(n, "a", -1);
        kn.b = getInt(n, "b", -1);
        kn.out = getInt(n, "out", -1);
        kn.multiDimFeature = n.get("end_buf") != nullptr || n.get("begin_coeffs") != nullptr ||
                             n.get("end_coeffs") != nullptr ||
                             n.get("out_index_coeffs") != nullptr ||
                             n.get("accumulate") != nullptr || n.get("guard_coeffs") != nullptr;
        if (const JVal* xs = n.get("exprs"); xs != nullptr && xs->t == JVal::Arr) {
            for (const JVal& x : xs->arr) {
                mlkb_expr e{};
                e.op = mathByName(getStr(x, "op"));
                for (int s = 0; s < 2; ++s) {
                    const JVal* o = x.get(s == 0 ? "a" : "b");
                    int kind = 0;
                    int64_t idx = 0;
                    double val = 0.0;
                    if (o != nullptr && o->t == JVal::Obj) {
                        kind = operandKind(getStr(*o, "kind"));
                        idx = getInt(*o, "index", 0);
                        if (const JVal* v = o->get("value"); v != nullptr && v->t == JVal::Num) {
                            val = v->num;
                        }
                        if (kind == 5) kn.multiDimFeature = true;  // ElemIdx
                    }
                    if (s == 0) {
                        e.a_kind = kind;
                        e.a_index = idx;
                        e.a_value = val;
                    } else {
                        e.b_kind = kind;
                        e.b_index = idx;
                        e.b_value = val;
                    }
                }
                kn.exprs.push_back(e);
            }
        }
        if (const JVal* cs = n.get("children"); cs != nullptr && cs->t == JVal::Arr) {
            for (const JVal& c : cs->arr) kn.children.push_back(static_cast<uint32_t>(c.i));
        }
        m.nodes.push_back(std::move(kn));
    }
    if (const JVal* sc = doc.get("schedule"); sc != nullptr && sc->t == JVal::Obj) {
        for (const auto& kv : sc->obj) m.schedule.emplace_back(kv.first, kv.second.i);
    }
    if (int st = classify(m)) return st;
    out = std::move(m);
    return okStatus();
}

}  // namespace mlkb
