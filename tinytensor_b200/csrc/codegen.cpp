// CUDA source generation for fused elementwise regions (compiled by NVRTC for
// sm_100a).  Each region becomes one kernel in which every thread handles `unroll`
// vectors of `vec` consecutive innermost elements: float4 (128-bit) coalesced loads
// for unit-stride operands, one scalar load per vector for operands broadcast along
// the innermost dim (stride 0, kept in registers), strided scalar loads otherwise.
//
// Arithmetic follows the reference's eager ops (src/core/operators.cpp:180-232):
// one IEEE rounding per add/sub/mul/div (the program is compiled with --fmad=false,
// so no a*b+c contraction), relu as x > 0 ? x : 0, the two-branch stable sigmoid.
#include <algorithm>
#include <cstring>
#include <iomanip>
#include <sstream>

#include "schedule.hpp"

namespace ttb {

namespace {

std::string flit(float v) {
    uint32_t u;
    std::memcpy(&u, &v, 4);
    std::ostringstream ss;
    ss << "__int_as_float(0x" << std::hex << std::setw(8) << std::setfill('0') << u << "u)";
    return ss.str();
}

struct Dim {
    int64_t size;
    std::vector<int64_t> st;  // per access: ext accesses then stores
};

}  // namespace

static void emit_region(std::ostringstream& ss, const Plan& p, Region& r) {
    const Graph& g = p.g;
    const size_t next = r.ext.size();
    const size_t nsto = r.store_ref.size();
    // Dims with per-access strides; stores are contiguous.
    Shape shape = r.shape.empty() ? Shape{1} : r.shape;
    std::vector<Dim> dims;
    {
        std::vector<int64_t> rm(shape.size());
        int64_t acc = 1;
        for (size_t i = shape.size(); i-- > 0;) {
            rm[i] = acc;
            acc *= shape[i];
        }
        for (size_t d = 0; d < shape.size(); ++d) {
            if (shape[d] == 1 && shape.size() > 1) continue;
            Dim dm;
            dm.size = shape[d];
            for (size_t e = 0; e < next; ++e)
                dm.st.push_back(r.ext_access[e].imm || r.shape.empty() ? 0 : r.ext_access[e].strides[d]);
            for (size_t s = 0; s < nsto; ++s) dm.st.push_back(rm[d]);
            dims.push_back(dm);
        }
        if (dims.empty()) {
            Dim dm;
            dm.size = 1;
            dm.st.assign(next + nsto, 0);
            dims.push_back(dm);
        }
        // collapse adjacent dims that are contiguous for every access
        for (size_t k = dims.size(); k-- > 1;) {
            bool ok = true;
            for (size_t a = 0; a < next + nsto; ++a)
                ok &= dims[k - 1].st[a] == dims[k].st[a] * dims[k].size;
            if (ok) {
                for (size_t a = 0; a < next + nsto; ++a) dims[k - 1].st[a] = dims[k].st[a];
                dims[k - 1].size *= dims[k].size;
                dims.erase(dims.begin() + static_cast<long>(k));
            }
        }
    }
    const int64_t n = numel(shape);
    const Dim& inner = dims.back();
    int vec = 4;
    if (inner.size % 4 != 0) vec = 1;
    for (size_t e = 0; e < next && vec == 4; ++e) {
        if (r.ext_access[e].imm) continue;
        int64_t si = inner.st[e];
        if (si != 0 && si != 1) vec = 1;
        if (si == 1) {
            if (r.ext_access[e].offset % 4) vec = 1;
            for (size_t d = 0; d + 1 < dims.size(); ++d)
                if (dims[d].st[e] % 4) vec = 1;
        }
    }
    r.vec = vec;
    const int64_t nvec = n / vec;
    r.unroll = nvec >= 4 * 256 * 148 ? 4 : (nvec >= 256 * 148 ? 2 : 1);
    const int64_t per_block = 256LL * r.unroll;
    r.grid = n == 0 ? 0 : (nvec + per_block - 1) / per_block;
    int64_t maxoff = n;
    for (size_t e = 0; e < next; ++e) {
        if (r.ext_access[e].imm) continue;
        int64_t o = r.ext_access[e].offset;
        for (const Dim& d : dims) o += (d.size - 1) * d.st[e];
        maxoff = std::max(maxoff, o + 1);
    }
    const char* it = (maxoff < (1LL << 31) - 1024 && nvec * vec < (1LL << 31) - 1024) ? "int" : "long long";

    ss << "// region " << r.kernel << ": " << (r.is_copy ? "copy" : "fused") << " over " << shape_str(r.shape)
       << ", " << dims.size() << " collapsed dim(s), vec " << vec << ", unroll " << r.unroll << "\n";
    ss << "extern \"C\" __global__ void __launch_bounds__(256) " << r.kernel << "(";
    for (size_t e = 0; e < next; ++e) ss << (e ? ", " : "") << "const float* __restrict__ x" << e;
    for (size_t s = 0; s < nsto; ++s) ss << (next + s ? ", " : "") << "float* __restrict__ y" << s;
    ss << ") {\n";
    ss << "  typedef " << it << " I;\n";
    ss << "  const I NV = " << nvec << ";\n";
    ss << "  const I b0 = (I)blockIdx.x * " << per_block << " + (I)threadIdx.x;\n";
    ss << "#pragma unroll\n  for (int u = 0; u < " << r.unroll << "; ++u) {\n";
    ss << "    const I v = b0 + (I)u * 256;\n    if (v >= NV) break;\n";
    ss << "    const I e = v * " << vec << ";\n";
    // coordinates
    ss << "    I t = e;\n";
    for (size_t d = dims.size(); d-- > 0;) {
        if (d == 0) ss << "    const I c0 = t;\n";
        else ss << "    const I c" << d << " = t % " << dims[d].size << "; t /= " << dims[d].size << ";\n";
    }
    // loads
    for (size_t e = 0; e < next; ++e) {
        const Access& a = r.ext_access[e];
        if (a.imm) {
            ss << "    const float a" << e << " = " << flit(a.value) << ";\n";
            continue;
        }
        std::ostringstream off;
        off << a.offset;
        for (size_t d = 0; d < dims.size(); ++d)
            if (dims[d].st[e] != 0) off << " + c" << d << " * (I)" << dims[d].st[e];
        int64_t si = inner.st[e];
        if (vec == 4 && si == 1) {
            ss << "    float a" << e << "[4]; { const float4 q = __ldg(reinterpret_cast<const float4*>(x" << e << " + ("
               << off.str() << "))); a" << e << "[0] = q.x; a" << e << "[1] = q.y; a" << e << "[2] = q.z; a" << e
               << "[3] = q.w; }\n";
        } else if (vec == 4 && si == 0) {
            ss << "    const float a" << e << " = __ldg(x" << e << " + (" << off.str() << "));\n";
        } else if (vec == 4) {
            ss << "    float a" << e << "[4];\n";
            ss << "#pragma unroll\n    for (int l = 0; l < 4; ++l) a" << e << "[l] = __ldg(x" << e << " + (" << off.str()
               << " + (I)l * " << si << "));\n";
        } else {
            ss << "    const float a" << e << " = __ldg(x" << e << " + (" << off.str() << "));\n";
        }
    }
    // compute
    auto ref = [&](int node) -> std::string {
        auto itx = std::find(r.ext.begin(), r.ext.end(), node);
        if (itx != r.ext.end()) {
            size_t e = static_cast<size_t>(itx - r.ext.begin());
            const Access& a = r.ext_access[e];
            bool lane = vec == 4 && !a.imm && inner.st[e] != 0;
            return "a" + std::to_string(e) + (lane ? "[l]" : "");
        }
        return "v" + std::to_string(node);
    };
    for (size_t s = 0; s < nsto; ++s) ss << "    float o" << s << "[" << vec << "];\n";
    ss << "#pragma unroll\n    for (int l = 0; l < " << vec << "; ++l) {\n";
    for (int i : r.nodes) {
        const Node& nd = g.nodes[static_cast<size_t>(i)];
        std::string x = ref(nd.in[0]);
        std::string y = nd.in.size() > 1 ? ref(nd.in[1]) : "";
        ss << "      const float v" << i << " = ";
        switch (nd.op) {
            case TT_OP_ADD: ss << x << " + " << y; break;
            case TT_OP_SUB: ss << x << " - " << y; break;
            case TT_OP_MUL: ss << x << " * " << y; break;
            case TT_OP_DIV: ss << x << " / " << y; break;
            case TT_OP_RELU: ss << "(" << x << " > 0.0f) ? " << x << " : 0.0f"; break;
            case TT_OP_STEP: ss << "(" << x << " > 0.0f) ? 1.0f : 0.0f"; break;
            case TT_OP_NEG: ss << "-" << x; break;
            case TT_OP_EXP: ss << "tt_exp(" << x << ")"; break;
            case TT_OP_TANH: ss << "tt_tanh(" << x << ")"; break;
            case TT_OP_SIGMOID:
                ss << "tt_sigmoid(" << x << ")";
                break;
            default: fail(TT_ERR_COMPILE, "internal: non-elementwise op in region");
        }
        ss << ";\n";
    }
    for (size_t s = 0; s < nsto; ++s) {
        std::string val = r.is_copy ? ref(r.ext[0]) : "v" + std::to_string(r.stores[s]);
        ss << "      o" << s << "[l] = " << val << ";\n";
    }
    ss << "    }\n";
    for (size_t s = 0; s < nsto; ++s) {
        if (vec == 4)
            ss << "    *reinterpret_cast<float4*>(y" << s << " + e) = make_float4(o" << s << "[0], o" << s << "[1], o" << s
               << "[2], o" << s << "[3]);\n";
        else
            ss << "    y" << s << "[e] = o" << s << "[0];\n";
    }
    ss << "  }\n}\n\n";
}

std::string generate_source(Plan& p) {
    std::ostringstream ss;
    ss << "// Generated by the TinyTensor B200 backend (sm_100a, NVRTC, --fmad=false)\n";
    ss << "// Program IR:\n";
    {
        std::istringstream ir(ir_text(p.g));
        std::string line;
        while (std::getline(ir, line)) ss << "//   " << line << "\n";
    }
    ss << "\n// exp and tanh: CUDA's float expf / tanhf (within 2 ulp, like the reference's float\n"
          "// libm calls std::exp / std::tanh, which are not correctly rounded either).\n";
    ss << "__device__ __forceinline__ float tt_exp(float x) { return expf(x); }\n";
    ss << "__device__ __forceinline__ float tt_tanh(float x) { return tanhf(x); }\n";
    ss << "// Two-branch stable sigmoid in float, src/core/operators.cpp:211-232.\n";
    ss << "__device__ __forceinline__ float tt_sigmoid(float x) {\n"
          "  if (x >= 0.0f) return 1.0f / (1.0f + tt_exp(-x));\n"
          "  const float ex = tt_exp(x);\n"
          "  return ex / (1.0f + ex);\n"
          "}\n\n";
    for (Launch& L : p.launches)
        if (L.type == LT_REGION) emit_region(ss, p, p.regions[static_cast<size_t>(L.region)]);
    return ss.str();
}

}  // namespace ttb
