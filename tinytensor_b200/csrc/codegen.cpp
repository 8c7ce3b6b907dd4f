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

// The expression of one region node, operands x (and y).
std::string node_expr(const Node& nd, const std::string& x, const std::string& y) {
    std::ostringstream ss;
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
        case TT_OP_SIGMOID: ss << "tt_sigmoid(" << x << ")"; break;
        default: fail(TT_ERR_COMPILE, "internal: non-elementwise op in region");
    }
    return ss.str();
}

int64_t round4c(int64_t x) { return (x + 3) / 4 * 4; }

// Ext index of the role (1 = A, 2 = B) operand of the small-K matmul node `mm`.
size_t mm_operand(const Region& r, int mm, int role) {
    for (size_t e = 0; e < r.ext.size(); ++e)
        if (r.ext_access[e].mm == mm && r.ext_access[e].role == role) return e;
    fail(TT_ERR_COMPILE, "internal: small-K matmul operand missing");
    return 0;
}

}  // namespace

// A region that also writes hi/lo operand copies of its stored [R][C] matrix X (for
// tensor-core GEMMs that read X without a pre-pass of their own).  A CTA computes one
// 32-row x 128-column tile: each warp takes rows w, w+8, w+16, w+24 with a float4 of
// columns per lane, issuing the four rows' loads before any arithmetic (so they are in
// flight together), then stores fp32 values and row-layout copies (coalesced) and parks
// the tile in shared memory; then each lane reads 4-column float4 chunks of its row
// (lane = row) and writes the transposed copies, one 128-B run per column and warp.
// The tile pitch of 132 floats keeps both the float4 stores and the float4 column-chunk
// reads at the minimum four shared-memory wavefronts.  Tiles are numbered rows first,
// so the CTAs resident together write neighbouring runs of each transposed row; one
// CTA per tile (the hardware balances the SMs).
#ifndef TT_TILED_MM_CTAS
#define TT_TILED_MM_CTAS 5
#endif
static void emit_region_tiled(std::ostringstream& ss, const Plan& p, Region& r) {
    const Graph& g = p.g;
    const size_t next = r.ext.size(), nsto = r.store_ref.size();
    const int64_t R = r.copy_R, C = r.copy_C, Cp = round4c(C), Rp = round4c(R);
    const int64_t tiles_r = (R + 31) / 32, tiles = tiles_r * ((C + 127) / 128);
    r.vec = 4;
    r.unroll = 1;
    r.grid = tiles;
    int64_t maxoff = std::max(R * Cp, C * Rp);
    for (size_t e = 0; e < next; ++e) {
        const Access& a = r.ext_access[e];
        if (!a.imm)
            maxoff = std::max(maxoff, a.offset + (R - 1) * a.strides[0] + (C - 1) * a.strides[1] +
                                          (a.kcount > 0 ? (a.kcount - 1) * a.kstride : 0) + 1);
    }
    const char* it = maxoff < (1LL << 31) - 1024 ? "int" : "long long";
    const size_t cs = static_cast<size_t>(r.copy_store);
    ss << "// region " << r.kernel << ": fused over " << shape_str(r.shape) << ", tiled, hi/lo copies of store " << cs
       << (r.copy_rows ? " [R][C]" : "") << (r.copy_t ? " [C][R]" : "") << (r.drop_f32 ? ", its fp32 not stored" : "")
       << "\n";
    // A region that forms a small-K product holds the four rows' products and loads in
    // registers; its launch bound asks for TT_TILED_MM_CTAS resident CTAs per SM.  Measured
    // on the MLP's dZ2 region at [32768, 4096] (one box, two runs each): 4 CTAs 0.57-0.58 ms
    // (64 registers), 5 CTAs 0.53-0.54 ms (48 registers and a few bytes of spill), 6 CTAs
    // 0.56 ms (40 registers, more spill).
    bool has_mm = false;
    for (int i : r.nodes) has_mm |= g.nodes[static_cast<size_t>(i)].inline_mm;
    ss << "extern \"C\" __global__ void __launch_bounds__(256";
    if (has_mm) ss << ", " << TT_TILED_MM_CTAS;
    ss << ") " << r.kernel << "(";
    for (size_t e = 0; e < next; ++e) ss << (e ? ", " : "") << "const float* __restrict__ x" << e;
    for (size_t k = 0; k < nsto; ++k) ss << (next + k ? ", " : "") << "float* __restrict__ y" << k;
    ss << ", float* __restrict__ ch, float* __restrict__ cl, float* __restrict__ th, float* __restrict__ tl) {\n";
    ss << "  typedef " << it << " I;\n";
    if (r.copy_t) ss << "  __shared__ __align__(16) float tile[32][132];\n";
    ss << "  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;\n";
    ss << "  const I t = blockIdx.x;\n";
    ss << "  const I r0 = (t % " << tiles_r << ") * 32, c0 = (t / " << tiles_r << ") * 128;\n";
    ss << "  const I c = c0 + 4 * lane;\n";
    // loads of the four rows: a<e>[i][l] (0 outside X); scalar per row when broadcast along columns
    for (size_t e = 0; e < next; ++e) {
        const Access& a = r.ext_access[e];
        if (a.role != 0) continue;  // small-K matmul operands are read where the product is formed
        if (a.imm) {
            ss << "  const float a" << e << " = " << flit(a.value) << ";\n";
            continue;
        }
        ss << (a.strides[1] == 0 ? "  float a" + std::to_string(e) + "[4];\n"
                                 : "  float a" + std::to_string(e) + "[4][4];\n");
    }
    ss << "#pragma unroll\n  for (int i = 0; i < 4; ++i) {\n";
    ss << "    const I rr = r0 + w + 8 * i;\n";
    ss << "    const bool rin = rr < (I)" << R << ", full = rin && c + 3 < (I)" << C << ";\n";
    for (size_t e = 0; e < next; ++e) {
        const Access& a = r.ext_access[e];
        if (a.imm || a.role != 0) continue;
        const int64_t sr = a.strides[0], sc = a.strides[1];
        std::ostringstream base;
        base << a.offset << " + rr * (I)" << sr;
        if (sc == 0) {
            ss << "    a" << e << "[i] = rin ? __ldg(x" << e << " + (" << base.str() << ")) : 0.0f;\n";
        } else if (sc == 1 && sr % 4 == 0 && a.offset % 4 == 0 && C % 4 == 0) {
            ss << "    { float4 q = make_float4(0.0f, 0.0f, 0.0f, 0.0f);\n";
            ss << "      if (full) q = __ldg(reinterpret_cast<const float4*>(x" << e << " + (" << base.str() << " + c)));\n";
            ss << "      a" << e << "[i][0] = q.x; a" << e << "[i][1] = q.y; a" << e << "[i][2] = q.z; a" << e
               << "[i][3] = q.w; }\n";
        } else {
            ss << "#pragma unroll\n    for (int l = 0; l < 4; ++l) a" << e << "[i][l] = (rin && c + l < (I)" << C
               << ") ? __ldg(x" << e << " + (" << base.str() << " + (c + l) * (I)" << sc << ")) : 0.0f;\n";
        }
    }
    ss << "  }\n";
    auto ref = [&](int node) -> std::string {
        for (size_t e = 0; e < next; ++e) {
            if (r.ext[e] != node || r.ext_access[e].role != 0) continue;
            const Access& a = r.ext_access[e];
            if (a.imm) return "a" + std::to_string(e);
            return "a" + std::to_string(e) + (a.strides[1] != 0 ? "[i][l]" : "[i]");
        }
        return "v" + std::to_string(node);
    };
    // small-K matmul operands: the tile's 32 rows of A and 128 columns of B staged in shared
    // memory once per CTA (read in the order that is contiguous in global memory)
    bool staged = false;
    for (int i : r.nodes) {
        if (!g.nodes[static_cast<size_t>(i)].inline_mm) continue;
        const size_t ea = mm_operand(r, i, 1), eb = mm_operand(r, i, 2);
        const Access& a = r.ext_access[ea];
        const Access& b = r.ext_access[eb];
        const int64_t K = a.kcount;
        ss << "  __shared__ float sa" << i << "[32][" << K << "];\n";
        // pitch 132: the staging stores (consecutive k in consecutive lanes) spread over 8 bank
        // groups, and each row stays 16-B aligned for the float4 column reads
        ss << "  __shared__ __align__(16) float sb" << i << "[" << K << "][132];\n";
        ss << "  for (int e = threadIdx.x; e < " << 32 * K << "; e += 256) {\n";
        if (a.kstride == 1) ss << "    const int q = e / " << K << ", k = e % " << K << ";\n";
        else ss << "    const int k = e / 32, q = e % 32;\n";
        ss << "    sa" << i << "[q][k] = r0 + q < (I)" << R << " ? __ldg(x" << ea << " + (" << a.offset << " + (r0 + q) * (I)"
           << a.strides[0] << " + (I)k * " << a.kstride << ")) : 0.0f;\n  }\n";
        ss << "  for (int e = threadIdx.x; e < " << 128 * K << "; e += 256) {\n";
        if (b.kstride == 1) ss << "    const int q = e / " << K << ", k = e % " << K << ";\n";
        else ss << "    const int k = e / 128, q = e % 128;\n";
        ss << "    sb" << i << "[k][q] = c0 + q < (I)" << C << " ? __ldg(x" << eb << " + (" << b.offset << " + (c0 + q) * (I)"
           << b.strides[1] << " + (I)k * " << b.kstride << ")) : 0.0f;\n  }\n";
        staged = true;
    }
    if (staged) ss << "  __syncthreads();\n";
    // the four rows' products for the lane's four columns, k outermost: one float4 of B per
    // k serves the four rows (B is not held for every k), and each element is still one
    // sequential fmaf chain over k
    for (int i : r.nodes) {
        if (!g.nodes[static_cast<size_t>(i)].inline_mm) continue;
        const int64_t K = r.ext_access[mm_operand(r, i, 1)].kcount;
        ss << "  float pm" << i << "[4][4];\n";
        ss << "#pragma unroll\n  for (int i = 0; i < 4; ++i)\n#pragma unroll\n    for (int l = 0; l < 4; ++l) pm" << i
           << "[i][l] = 0.0f;\n";
        ss << "#pragma unroll\n  for (int k = 0; k < " << K << "; ++k) {\n";
        ss << "    const float4 bv = *reinterpret_cast<const float4*>(&sb" << i << "[k][4 * lane]);\n";
        ss << "#pragma unroll\n    for (int i = 0; i < 4; ++i) {\n";
        ss << "      const float av = sa" << i << "[w + 8 * i][k];\n";
        ss << "      pm" << i << "[i][0] = fmaf(av, bv.x, pm" << i << "[i][0]); pm" << i << "[i][1] = fmaf(av, bv.y, pm" << i
           << "[i][1]);\n";
        ss << "      pm" << i << "[i][2] = fmaf(av, bv.z, pm" << i << "[i][2]); pm" << i << "[i][3] = fmaf(av, bv.w, pm" << i
           << "[i][3]);\n    }\n  }\n";
    }
    ss << "#pragma unroll\n  for (int i = 0; i < 4; ++i) {\n";
    ss << "    const I rr = r0 + w + 8 * i;\n";
    ss << "    const bool rin = rr < (I)" << R << ", full = rin && c + 3 < (I)" << C << ";\n";
    for (size_t k = 0; k < nsto; ++k) ss << "    float o" << k << "[4];\n";
    ss << "#pragma unroll\n    for (int l = 0; l < 4; ++l) {\n";
    for (int i : r.nodes) {
        const Node& nd = g.nodes[static_cast<size_t>(i)];
        if (nd.inline_mm) {  // formed above: one sequential fmaf chain over k per element
            ss << "      const float v" << i << " = pm" << i << "[i][l];\n";
            continue;
        }
        ss << "      const float v" << i << " = "
           << node_expr(nd, ref(nd.in[0]), nd.in.size() > 1 ? ref(nd.in[1]) : "") << ";\n";
    }
    for (size_t k = 0; k < nsto; ++k) ss << "      o" << k << "[l] = v" << r.stores[k] << ";\n";
    ss << "    }\n";
    // fp32 stores of [R][C] matrices (row stride C)
    for (size_t k = 0; k < nsto; ++k) {
        if (k == cs && r.drop_f32) continue;
        if (C % 4 == 0)
            ss << "    if (full) *reinterpret_cast<float4*>(y" << k << " + rr * (I)" << C << " + c) = make_float4(o" << k
               << "[0], o" << k << "[1], o" << k << "[2], o" << k << "[3]);\n    else";
        ss << "    if (rin) { for (int l = 0; l < 4; ++l) if (c + l < (I)" << C << ") y" << k << "[rr * (I)" << C
           << " + c + l] = o" << k << "[l]; }\n";
    }
    if (r.copy_rows) {  // copies in X's layout, row pitch round4(C)
        ss << "    if (rin) {\n      float4 h, q;\n";
        ss << "      tt_split(o" << cs << "[0], h.x, q.x); tt_split(o" << cs << "[1], h.y, q.y);\n";
        ss << "      tt_split(o" << cs << "[2], h.z, q.z); tt_split(o" << cs << "[3], h.w, q.w);\n";
        ss << "      if (c + 3 < (I)" << C << ") { *reinterpret_cast<float4*>(ch + rr * (I)" << Cp
           << " + c) = h; *reinterpret_cast<float4*>(cl + rr * (I)" << Cp << " + c) = q; }\n";
        ss << "      else { const float hv[4] = {h.x, h.y, h.z, h.w}, lv[4] = {q.x, q.y, q.z, q.w};\n";
        ss << "        for (int l = 0; l < 4; ++l) if (c + l < (I)" << C << ") { ch[rr * (I)" << Cp
           << " + c + l] = hv[l]; cl[rr * (I)" << Cp << " + c + l] = lv[l]; } }\n";
        ss << "    }\n";
    }
    if (r.copy_t)
        ss << "    *reinterpret_cast<float4*>(&tile[w + 8 * i][4 * lane]) = make_float4(o" << cs << "[0], o" << cs
           << "[1], o" << cs << "[2], o" << cs << "[3]);\n";
    ss << "  }\n";
    if (r.copy_t) {  // transposed copies [C][round4(R)]: lane = row, one 128-B run per column
        ss << "  __syncthreads();\n";
        ss << "  const I rr = r0 + lane;\n";
        ss << "#pragma unroll\n  for (int j = 0; j < 4; ++j) {\n";
        ss << "    const float4 q = *reinterpret_cast<const float4*>(&tile[lane][w * 16 + 4 * j]);\n";
        ss << "    const float qv[4] = {q.x, q.y, q.z, q.w};\n";
        ss << "#pragma unroll\n    for (int u = 0; u < 4; ++u) {\n";
        ss << "      const I cc = c0 + w * 16 + 4 * j + u;\n";
        ss << "      if (cc < (I)" << C << " && rr < (I)" << R << ") {\n";
        ss << "        float h, l;\n        tt_split(qv[u], h, l);\n";
        ss << "        th[cc * (I)" << Rp << " + rr] = h;\n        tl[cc * (I)" << Rp << " + rr] = l;\n      }\n";
        ss << "    }\n  }\n";
    }
    ss << "}\n\n";
}

static void emit_region(std::ostringstream& ss, const Plan& p, Region& r) {
    if (r.copy_store >= 0) {
        emit_region_tiled(ss, p, r);
        return;
    }
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
        if (r.ext_access[e].imm || r.ext_access[e].role != 0) continue;
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
        if (r.ext_access[e].kcount > 0) o += (r.ext_access[e].kcount - 1) * r.ext_access[e].kstride;
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
    // loads (small-K matmul operands are read where the product is formed)
    std::vector<std::string> offs(next);
    for (size_t e = 0; e < next; ++e) {
        const Access& a = r.ext_access[e];
        if (a.imm) continue;
        std::ostringstream off;
        off << a.offset;
        for (size_t d = 0; d < dims.size(); ++d)
            if (dims[d].st[e] != 0) off << " + c" << d << " * (I)" << dims[d].st[e];
        offs[e] = off.str();
    }
    for (size_t e = 0; e < next; ++e) {
        const Access& a = r.ext_access[e];
        if (a.role != 0) continue;
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
        for (size_t e = 0; e < next; ++e) {
            if (r.ext[e] != node || r.ext_access[e].role != 0) continue;
            const Access& a = r.ext_access[e];
            bool lane = vec == 4 && !a.imm && inner.st[e] != 0;
            return "a" + std::to_string(e) + (lane ? "[l]" : "");
        }
        return "v" + std::to_string(node);
    };
    // small-K matmul: A's K values of this element's row (shared by the vector's lanes)
    for (int i : r.nodes) {
        if (!g.nodes[static_cast<size_t>(i)].inline_mm) continue;
        const size_t ea = mm_operand(r, i, 1);
        const Access& a = r.ext_access[ea];
        ss << "    float am" << i << "[" << a.kcount << "];\n";
        ss << "#pragma unroll\n    for (int k = 0; k < " << a.kcount << "; ++k) am" << i << "[k] = __ldg(x" << ea << " + ("
           << offs[ea] << " + (I)k * " << a.kstride << "));\n";
    }
    for (size_t s = 0; s < nsto; ++s) ss << "    float o" << s << "[" << vec << "];\n";
    ss << "#pragma unroll\n    for (int l = 0; l < " << vec << "; ++l) {\n";
    for (int i : r.nodes) {
        const Node& nd = g.nodes[static_cast<size_t>(i)];
        if (nd.inline_mm) {  // one sequential fmaf chain over k, as the small-K GEMM kernel computes it
            const size_t eb = mm_operand(r, i, 2);
            const Access& b = r.ext_access[eb];
            ss << "      float v" << i << " = 0.0f;\n";
            ss << "#pragma unroll\n      for (int k = 0; k < " << b.kcount << "; ++k) v" << i << " = fmaf(am" << i
               << "[k], __ldg(x" << eb << " + (" << offs[eb] << " + (I)l * " << inner.st[eb] << " + (I)k * "
               << b.kstride << ")), v" << i << ");\n";
            continue;
        }
        std::string x = ref(nd.in[0]);
        std::string y = nd.in.size() > 1 ? ref(nd.in[1]) : "";
        ss << "      const float v" << i << " = " << node_expr(nd, x, y) << ";\n";
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
          "}\n";
    ss << "// hi/lo operand split of the 3xTF32 GEMM (the pre-pass's split_tf32, bit for bit): hi = x\n"
          "// with its low 13 mantissa bits cleared, lo = the same of x - hi (exact), or the sign\n"
          "// marker hi * 2^-24 when that is zero and x is not; +-inf -> (x, x); NaN -> the\n"
          "// canonical quiet NaN twice.  A nonzero lo keeps inf * finite products infinite.\n";
    ss << "__device__ __forceinline__ void tt_split(float x, float& hi, float& lo) {\n"
          "  const unsigned u = __float_as_uint(x);\n"
          "  if ((u & 0x7F800000u) != 0x7F800000u) {\n"
          "    hi = __uint_as_float(u & 0xFFFFE000u);\n"
          "    const float r = __uint_as_float(__float_as_uint(__fsub_rn(x, hi)) & 0xFFFFE000u);\n"
          "    lo = (r == 0.0f && x != 0.0f) ? __uint_as_float(__float_as_uint(__fmul_rn(hi, 0x1p-24f)) & 0xFFFFE000u)"
          " : r;\n"
          "  } else {\n"
          "    hi = (u & 0x7FFFFFFFu) > 0x7F800000u ? __uint_as_float(0x7FC00000u) : x;\n"
          "    lo = hi;\n"
          "  }\n"
          "}\n\n";
    for (Launch& L : p.launches)
        if (L.type == LT_REGION) emit_region(ss, p, p.regions[static_cast<size_t>(L.region)]);
    return ss.str();
}

}  // namespace ttb
