// Scheduling of a TinyTensor graph for the GPU:
//  1. group elementwise nodes of equal shape into fused regions (one generated
//     kernel each; a node joins a producer's region unless that would create a
//     cycle through another launch);
//  2. fold views (transpose / reshape / expand) into the strides their consumers
//     read with, so no transpose is materialised for reductions, GEMMs or regions;
//  3. order the launches (regions, reductions, GEMMs) topologically;
//  4. plan memory: the reference MemoryPlanner's lifetimes and greedy first-fit slot
//     reuse (src/optimizer/memory_planner.cpp:21-89), applied to launch steps and
//     mapped onto ONE device arena (slot offsets = 256-B aligned prefix sums).
#include <algorithm>
#include <cstring>
#include <functional>
#include <map>
#include <queue>
#include <set>
#include <sstream>

#include "schedule.hpp"

namespace ttb {

namespace {

std::vector<int64_t> rowmajor(const Shape& s) {
    std::vector<int64_t> st(s.size());
    int64_t acc = 1;
    for (size_t i = s.size(); i-- > 0;) {
        st[i] = acc;
        acc *= s[i];
    }
    return st;
}

bool is_contiguous(const Storage& s, const Shape& shape) {
    auto rm = rowmajor(shape);
    for (size_t i = 0; i < shape.size(); ++i)
        if (shape[i] != 1 && s.strides[i] != rm[i]) return false;
    return true;
}

int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }
int64_t round4i(int64_t x) { return (x + 3) / 4 * 4; }

// Access of `src` (shape `from`) broadcast to the iteration shape `to`.
Access broadcast_access(const Storage& s, int node, const Shape& from, const Shape& to) {
    Access a;
    if (s.kind == SK_IMM) {
        a.imm = true;
        a.value = s.imm;
        return a;
    }
    a.node = s.root;
    a.offset = s.offset;
    a.strides.assign(to.size(), 0);
    size_t r = to.size(), rf = from.size();
    for (size_t i = 0; i < rf; ++i) {
        size_t j = r - rf + i;
        a.strides[j] = (from[i] == 1 && to[j] != 1) ? 0 : s.strides[i];
    }
    (void)node;
    return a;
}

// GEMM epilogues.  (a) The ReLU derivative mask step(x) equals step(relu(x)) bit for
// bit (relu maps NaN and -0 to +0, and step maps +0, -0 and NaN alike to 0), so a mask
// reads the ReLU's output when the graph has one; the matmul before the ReLU then has
// no other reader.  (b) A matmul whose only reader is a ReLU or tanh (the matmul not a
// graph output) applies the activation in its own epilogue and stores the activated
// value; the activation node becomes a view of the matmul's storage (or, when it is a
// graph output, the matmul writes that output).  This removes one HBM pass over the
// activation (read + write) per folded node.
void fold_gemm_epilogues(Graph& g, const std::vector<int>& out_pos) {
    const size_t n = g.nodes.size();
    std::vector<int> relu_of(n, -1);
    for (size_t i = 0; i < n; ++i)
        if (g.nodes[i].op == TT_OP_RELU) {
            const size_t x = static_cast<size_t>(g.nodes[i].in[0]);
            if (relu_of[x] < 0) relu_of[x] = static_cast<int>(i);
        }
    for (size_t i = 0; i < n; ++i) {
        Node& s = g.nodes[i];
        if (s.op != TT_OP_STEP) continue;
        const int r = relu_of[static_cast<size_t>(s.in[0])];
        if (r >= 0 && r < static_cast<int>(i)) s.in[0] = r;  // keeps the node order topological
    }
    std::vector<int> readers(n, 0), reader(n, -1);
    for (size_t i = 0; i < n; ++i)
        for (int q : g.nodes[i].in) {
            ++readers[static_cast<size_t>(q)];
            reader[static_cast<size_t>(q)] = static_cast<int>(i);
        }
    for (size_t m = 0; m < n; ++m) {
        Node& mm = g.nodes[m];
        if (mm.op != TT_OP_MATMUL || out_pos[m] >= 0 || readers[m] != 1) continue;
        Node& a = g.nodes[static_cast<size_t>(reader[m])];
        if ((a.op != TT_OP_RELU && a.op != TT_OP_TANH) || a.shape != mm.shape) continue;
        mm.epilogue = a.op == TT_OP_RELU ? EP_RELU : EP_TANH;
        a.fused_into = static_cast<int>(m);
    }
}

// Small-K matmuls evaluated inside their readers' fused region.  A 2-D matmul with
// K <= 16 (a product bound by writing C) whose readers are all elementwise nodes of its
// shape is computed where those readers run: each element is a K-term fmaf chain over a
// row of A and a column of B read from their buffers, so the product is never stored and
// read back.  The operands must be addressable buffers: not a value of the product's own
// shape computed in a region (it could live in registers of the same region), not a
// scalar constant, not another inlined product.
void mark_inline_matmuls(Graph& g, const std::vector<int>& out_pos) {
    const size_t n = g.nodes.size();
    std::vector<std::vector<int>> readers(n);
    for (size_t i = 0; i < n; ++i)
        for (int q : g.nodes[i].in) readers[static_cast<size_t>(q)].push_back(static_cast<int>(i));
    auto base_of = [&](int q) {
        while (is_view(g.nodes[static_cast<size_t>(q)].op)) q = g.nodes[static_cast<size_t>(q)].in[0];
        return q;
    };
    for (size_t m = 0; m < n; ++m) {
        Node& mm = g.nodes[m];
        if (mm.op != TT_OP_MATMUL || mm.epilogue != 0 || out_pos[m] >= 0 || mm.shape.size() != 2) continue;
        const Shape& sa = g.nodes[static_cast<size_t>(mm.in[0])].shape;
        const Shape& sb = g.nodes[static_cast<size_t>(mm.in[1])].shape;
        if (sa.size() != 2 || sb.size() != 2 || mm.shape[0] < 2 || mm.shape[1] < 2) continue;
        if (sa[1] < 1 || sa[1] > 16 || readers[m].empty()) continue;
        bool ok = true;
        for (int u : readers[m]) {
            const Node& un = g.nodes[static_cast<size_t>(u)];
            ok &= is_elementwise(un.op) && un.fused_into < 0 && un.shape == mm.shape;
        }
        for (int k = 0; k < 2 && ok; ++k) {
            const Node& b = g.nodes[static_cast<size_t>(base_of(mm.in[static_cast<size_t>(k)]))];
            if (is_elementwise(b.op) && b.shape == mm.shape) ok = false;
            if (b.op == TT_OP_CONSTANT && b.cdata.size() <= 1) ok = false;
            if (b.op == TT_OP_MATMUL && b.inline_mm) ok = false;
        }
        mm.inline_mm = ok;
    }
}

}  // namespace

int64_t split_copies_bytes(int64_t R, int64_t C, bool rows, bool t) {
    return (rows ? 2 * align256(R * round4i(C) * 4) : 0) + (t ? 2 * align256(C * round4i(R) * 4) : 0);
}

int64_t split_copies_offset(int64_t R, int64_t C, bool rows, int layout, int lo) {
    const int64_t rcap = rows ? align256(R * round4i(C) * 4) : 0;
    if (layout == 0) return lo ? rcap : 0;
    return 2 * rcap + (lo ? align256(C * round4i(R) * 4) : 0);
}

Plan schedule(const Graph& gin, const ScheduleOptions& opt) {
    Plan p;
    p.g = gin;
    Graph& g = p.g;
    const size_t N0 = g.nodes.size();

    std::vector<int> out_pos(N0, -1);
    for (size_t k = 0; k < g.outputs.size(); ++k) out_pos[static_cast<size_t>(g.outputs[k])] = static_cast<int>(k);
    if (opt.gemm_epilogue) fold_gemm_epilogues(g, out_pos);
    if (opt.gemm_epilogue && opt.fuse) mark_inline_matmuls(g, out_pos);
    std::vector<std::vector<int>> users(N0);
    for (size_t i = 0; i < N0; ++i)
        for (int q : g.nodes[i].in) users[static_cast<size_t>(q)].push_back(static_cast<int>(i));

    // ---- 1. grouping ----
    p.region_of.assign(N0, -1);
    std::vector<std::vector<int>> deps(N0);  // sorted ids of regions each node depends on
    for (size_t i = 0; i < N0; ++i) {
        const Node& n = g.nodes[i];
        std::vector<int> d;
        for (int q : n.in) {
            const auto& dq = deps[static_cast<size_t>(q)];
            d.insert(d.end(), dq.begin(), dq.end());
        }
        if (n.dtype != TT_FLOAT32) fail(TT_ERR_COMPILE, "The CUDA backend computes in float32 only (node %" +
                                                            std::to_string(n.id) + " is float64)");
        if ((is_elementwise(n.op) && n.fused_into < 0) || n.inline_mm) {
            int R = -1;
            if (opt.fuse) {
                for (int q : n.in) {
                    int rq = p.region_of[static_cast<size_t>(q)];
                    if (rq < 0 || g.nodes[static_cast<size_t>(q)].shape != n.shape) continue;
                    bool safe = true;
                    for (int q2 : n.in) {
                        if (p.region_of[static_cast<size_t>(q2)] == rq) continue;
                        const auto& d2 = deps[static_cast<size_t>(q2)];
                        if (std::find(d2.begin(), d2.end(), rq) != d2.end()) safe = false;
                    }
                    if (safe) {
                        R = rq;
                        break;
                    }
                }
            }
            if (R < 0) {
                R = static_cast<int>(p.regions.size());
                Region reg;
                reg.shape = n.shape;
                p.regions.push_back(reg);
            }
            p.region_of[i] = R;
            p.regions[static_cast<size_t>(R)].nodes.push_back(static_cast<int>(i));
            d.push_back(R);
        }
        std::sort(d.begin(), d.end());
        d.erase(std::unique(d.begin(), d.end()), d.end());
        deps[i] = std::move(d);
    }

    // ---- 1b. merge a producer region into its consumer region of the same shape when
    // no other launch lies on a path between them (contracting the edge keeps the
    // launch graph acyclic).  E.g. relu(a*b+c)*0.5 - exp(-a) becomes one kernel.
    if (opt.fuse && p.regions.size() > 1) {
        const int nr = static_cast<int>(p.regions.size());
        std::vector<int> unit_of(N0, -1);
        int nu = nr;
        for (size_t i = 0; i < N0; ++i) {
            const Node& n = g.nodes[i];
            if (p.region_of[i] >= 0) unit_of[i] = p.region_of[i];
            else if (n.op == TT_OP_MATMUL || is_reduce(n.op)) unit_of[i] = nu++;
            else if (is_view(n.op) || n.fused_into >= 0) unit_of[i] = unit_of[static_cast<size_t>(n.in[0])];
        }
        std::vector<int> alias(static_cast<size_t>(nu));
        for (int u = 0; u < nu; ++u) alias[static_cast<size_t>(u)] = u;
        std::function<int(int)> find = [&](int u) {
            while (alias[static_cast<size_t>(u)] != u) u = alias[static_cast<size_t>(u)];
            return u;
        };
        for (bool changed = true; changed;) {
            changed = false;
            std::vector<std::set<int>> succ(static_cast<size_t>(nu));
            for (size_t i = 0; i < N0; ++i) {
                if (unit_of[i] < 0 || is_view(g.nodes[i].op) || g.nodes[i].fused_into >= 0) continue;
                int ui = find(unit_of[i]);
                for (int q : g.nodes[i].in) {
                    int uq = unit_of[static_cast<size_t>(q)];
                    if (uq < 0) continue;
                    uq = find(uq);
                    if (uq != ui) succ[static_cast<size_t>(uq)].insert(ui);
                }
            }
            auto indirect = [&](int from, int to) {  // path from->...->to avoiding the direct edge
                std::vector<char> seen(static_cast<size_t>(nu), 0);
                std::vector<int> stack;
                for (int s : succ[static_cast<size_t>(from)])
                    if (s != to) stack.push_back(s);
                while (!stack.empty()) {
                    int u = stack.back();
                    stack.pop_back();
                    if (u == to) return true;
                    if (seen[static_cast<size_t>(u)]) continue;
                    seen[static_cast<size_t>(u)] = 1;
                    for (int s : succ[static_cast<size_t>(u)]) stack.push_back(s);
                }
                return false;
            };
            for (int r1 = 0; r1 < nr && !changed; ++r1) {
                if (find(r1) != r1) continue;
                for (int r2 : succ[static_cast<size_t>(r1)]) {
                    if (r2 >= nr) continue;  // not a region
                    if (p.regions[static_cast<size_t>(r1)].shape != p.regions[static_cast<size_t>(r2)].shape) continue;
                    if (indirect(r1, r2)) continue;
                    alias[static_cast<size_t>(r1)] = r2;
                    changed = true;
                    break;
                }
            }
        }
        // Compact: renumber surviving regions, node lists in topological (index) order.
        std::vector<int> new_id(static_cast<size_t>(nr), -1);
        std::vector<Region> merged;
        for (int r = 0; r < nr; ++r)
            if (find(r) == r) {
                new_id[static_cast<size_t>(r)] = static_cast<int>(merged.size());
                Region reg;
                reg.shape = p.regions[static_cast<size_t>(r)].shape;
                merged.push_back(reg);
            }
        for (size_t i = 0; i < N0; ++i)
            if (p.region_of[i] >= 0) {
                int r = new_id[static_cast<size_t>(find(p.region_of[i]))];
                p.region_of[i] = r;
                merged[static_cast<size_t>(r)].nodes.push_back(static_cast<int>(i));
            }
        p.regions = std::move(merged);
    }

    // ---- 2. storage ----
    std::vector<bool> stored(N0, false);
    for (size_t i = 0; i < N0; ++i) {
        if ((!is_elementwise(g.nodes[i].op) && !g.nodes[i].inline_mm) || g.nodes[i].fused_into >= 0) continue;
        bool s = out_pos[i] >= 0;
        for (int u : users[i]) s |= p.region_of[static_cast<size_t>(u)] != p.region_of[i];
        stored[i] = s;
    }
    p.st.assign(N0, Storage{});
    std::vector<int> copy_of;  // materialised reshapes: region index per node (-1)
    auto make_root = [&](size_t i) {
        Storage s;
        s.kind = SK_BUF;
        s.root = static_cast<int>(i);
        s.strides = rowmajor(g.nodes[i].shape);
        return s;
    };
    auto add_copy_region = [&](int src, const Storage& src_st, const Shape& src_shape, int dst) {
        Region r;
        r.shape = src_shape;
        r.is_copy = true;
        r.ext.push_back(src);
        r.ext_access.push_back(broadcast_access(src_st, src, src_shape, src_shape));
        r.stores.push_back(dst);
        p.regions.push_back(r);
        return static_cast<int>(p.regions.size()) - 1;
    };
    for (size_t i = 0; i < N0; ++i) {
        const Node& n = g.nodes[i];
        if (n.fused_into >= 0) {  // computed by the matmul's epilogue: a view of its storage
            p.st[i] = p.st[static_cast<size_t>(n.fused_into)];
            continue;
        }
        if (n.inline_mm) {  // computed in its region like an elementwise node
            if (stored[i]) p.st[i] = make_root(i);
            else p.st[i].kind = SK_REG;
            continue;
        }
        switch (n.op) {
            case TT_OP_INPUT:
                p.st[i] = make_root(i);
                break;
            case TT_OP_CONSTANT:
                if (n.cdata.size() == 1) {
                    p.st[i].kind = SK_IMM;
                    p.st[i].imm = n.cdata[0];
                } else {
                    p.st[i] = make_root(i);
                }
                break;
            case TT_OP_MATMUL:
            case TT_OP_REDUCE_SUM:
            case TT_OP_REDUCE_MEAN:
            case TT_OP_REDUCE_MAX:
                p.st[i] = make_root(i);
                break;
            case TT_OP_TRANSPOSE: case TT_OP_RESHAPE: case TT_OP_EXPAND: {
                const Storage& b = p.st[static_cast<size_t>(n.in[0])];
                const Shape& bs = g.nodes[static_cast<size_t>(n.in[0])].shape;
                if (b.kind == SK_IMM) {
                    p.st[i] = b;
                    break;
                }
                if (b.kind != SK_BUF) fail(TT_ERR_COMPILE, "internal: view of an unstored value");
                Storage s = b;
                if (n.op == TT_OP_TRANSPOSE) {
                    std::swap(s.strides[static_cast<size_t>(n.dim0)], s.strides[static_cast<size_t>(n.dim1)]);
                } else if (n.op == TT_OP_EXPAND) {
                    Access a = broadcast_access(b, n.in[0], bs, n.shape);
                    s.strides = a.strides;
                } else {  // reshape
                    bool same = n.shape == bs;
                    if (same && out_pos[i] < 0) {
                        // identity reshape: plain view
                    } else if (is_contiguous(b, bs) && !same) {
                        s.strides = rowmajor(n.shape);
                    } else {
                        s = make_root(i);
                        add_copy_region(n.in[0], b, bs, static_cast<int>(i));
                    }
                }
                p.st[i] = s;
                break;
            }
            default:
                if (is_elementwise(n.op)) {
                    if (stored[i]) p.st[i] = make_root(i);
                    else p.st[i].kind = SK_REG;
                } else {
                    fail(TT_ERR_COMPILE, std::string("Unsupported op in CUDA backend: ") + op_name(n.op));
                }
        }
    }

    // ---- region externals / stores ----
    for (size_t R = 0; R < p.regions.size(); ++R) {
        Region& r = p.regions[R];
        if (r.is_copy) continue;
        for (int i : r.nodes) {
            const Node& nd = g.nodes[static_cast<size_t>(i)];
            if (nd.inline_mm) {  // operands: A varies with the row, B with the column, both along K
                for (int k = 0; k < 2; ++k) {
                    const int q = nd.in[static_cast<size_t>(k)];
                    const Storage& sq = p.st[static_cast<size_t>(q)];
                    if (sq.kind != SK_BUF) fail(TT_ERR_COMPILE, "internal: small-K matmul operand is not a buffer");
                    Access a;
                    a.node = sq.root;
                    a.offset = sq.offset;
                    a.role = k + 1;
                    a.mm = i;
                    a.strides = k == 0 ? std::vector<int64_t>{sq.strides[0], 0} : std::vector<int64_t>{0, sq.strides[1]};
                    a.kstride = k == 0 ? sq.strides[1] : sq.strides[0];
                    a.kcount = g.nodes[static_cast<size_t>(q)].shape[k == 0 ? 1 : 0];
                    r.ext.push_back(q);
                    r.ext_access.push_back(a);
                }
                if (stored[static_cast<size_t>(i)]) r.stores.push_back(i);
                continue;
            }
            for (int q : nd.in) {
                if (p.region_of[static_cast<size_t>(q)] == static_cast<int>(R)) continue;
                bool have = false;
                for (size_t e = 0; e < r.ext.size(); ++e) have |= r.ext[e] == q && r.ext_access[e].role == 0;
                if (have) continue;
                const Storage& sq = p.st[static_cast<size_t>(q)];
                if (sq.kind == SK_REG) fail(TT_ERR_COMPILE, "internal: region reads an unstored value");
                r.ext.push_back(q);
                r.ext_access.push_back(broadcast_access(sq, q, g.nodes[static_cast<size_t>(q)].shape, r.shape));
            }
            if (stored[static_cast<size_t>(i)]) r.stores.push_back(i);
        }
    }
    p.fused_regions = 0;
    for (const Region& r : p.regions)
        if (!r.is_copy && r.nodes.size() > 1) ++p.fused_regions;

    // ---- GEMM / reduction operands that need a dense copy ----
    auto materialise = [&](int src) -> int {
        Node m;
        m.op = TT_OP_RESHAPE;
        m.dtype = g.nodes[static_cast<size_t>(src)].dtype;
        m.in = {src};
        m.shape = g.nodes[static_cast<size_t>(src)].shape;
        m.id = g.next_id;
        int idx = g.add(m);
        p.st.push_back(make_root(static_cast<size_t>(idx)));
        p.region_of.push_back(-1);
        add_copy_region(src, p.st[static_cast<size_t>(src)], g.nodes[static_cast<size_t>(src)].shape, idx);
        return idx;
    };
    auto gemm_ok = [&](int q, bool is_a) {
        const Storage& s = p.st[static_cast<size_t>(q)];
        if (s.kind != SK_BUF) return false;
        const Shape& sh = g.nodes[static_cast<size_t>(q)].shape;
        size_t r = sh.size();
        int64_t s0 = s.strides[r - 2], s1 = s.strides[r - 1];
        (void)is_a;
        bool inner_unit = (s1 == 1 || sh[r - 1] == 1) || (s0 == 1 || sh[r - 2] == 1);
        if (!inner_unit) return false;
        // batch dims must collapse to one stride
        if (r > 3) {
            for (size_t d = 0; d + 1 < r - 2; ++d)
                if (sh[d + 1] != 1 && s.strides[d] != s.strides[d + 1] * sh[d + 1] && sh[d] != 1) return false;
        }
        return true;
    };
    // The GEMM kernels take one batch stride per operand.  Aligned to the output's batch
    // dims, the operand's batch offsets must be linear in the flattened batch index
    // (offset = b * unit, unit 0 when the operand is broadcast over the whole batch);
    // a partial broadcast such as [2,1,.,.] x [5,.,.] -> [2,5,.,.] is not.
    auto batch_linear = [&](int q, const Shape& out) -> bool {
        const Storage& s = p.st[static_cast<size_t>(q)];
        const Shape& sh = g.nodes[static_cast<size_t>(q)].shape;
        const size_t r = sh.size(), rc = out.size();
        if (rc <= 2) return true;
        const size_t nb = rc - 2, own = r - 2;
        int64_t inner = 1, unit = 0;
        bool have = false;
        for (size_t d = nb; d-- > 0;) {
            if (out[d] != 1) {
                int64_t st = 0;
                if (d + own >= nb) {
                    const size_t od = d + own - nb;
                    if (sh[od] != 1) st = s.strides[od];
                }
                if (st % inner != 0) return false;
                if (have && st / inner != unit) return false;
                unit = st / inner;
                have = true;
            }
            inner *= out[d];
        }
        return true;
    };
    // Dense copy of `src` broadcast to the output's batch dims: [out batch..., rows, cols].
    auto materialise_batch = [&](int src, const Shape& out) -> int {
        const Shape& sh = g.nodes[static_cast<size_t>(src)].shape;
        Shape full(out.begin(), out.end() - 2);
        full.push_back(sh[sh.size() - 2]);
        full.push_back(sh[sh.size() - 1]);
        Node m;
        m.op = TT_OP_EXPAND;
        m.dtype = g.nodes[static_cast<size_t>(src)].dtype;
        m.in = {src};
        m.shape = full;
        m.id = g.next_id;
        int idx = g.add(m);
        p.st.push_back(make_root(static_cast<size_t>(idx)));
        p.region_of.push_back(-1);
        Region r;
        r.shape = full;
        r.is_copy = true;
        r.ext.push_back(src);
        r.ext_access.push_back(broadcast_access(p.st[static_cast<size_t>(src)], src, sh, full));
        r.stores.push_back(idx);
        p.regions.push_back(r);
        return idx;
    };
    std::vector<int> launch_nodes;  // reduce / matmul nodes, original order
    g.nodes.reserve(N0 * 3 + 8);      // materialise() appends nodes: no reference is held across it
    for (size_t i = 0; i < N0; ++i) {
        const int op = g.nodes[i].op;
        if (op == TT_OP_MATMUL && !g.nodes[i].inline_mm) {
            for (size_t k = 0; k < 2; ++k) {
                const int src = g.nodes[i].in[k];
                if (!batch_linear(src, g.nodes[i].shape)) {
                    const Shape out = g.nodes[i].shape;
                    g.nodes[i].in[k] = materialise_batch(src, out);
                } else if (!gemm_ok(src, k == 0)) {
                    const int m = materialise(src);
                    g.nodes[i].in[k] = m;
                }
            }
            launch_nodes.push_back(static_cast<int>(i));
        } else if (is_reduce(op)) {
            const int src = g.nodes[i].in[0];
            if (p.st[static_cast<size_t>(src)].kind != SK_BUF) {
                const int m = materialise(src);
                g.nodes[i].in[0] = m;
            }
            launch_nodes.push_back(static_cast<int>(i));
        }
    }

    // ---- graph outputs ----
    const size_t N = g.nodes.size();
    p.root_ref.assign(N, BufRef{});
    for (size_t k = 0; k < g.inputs.size(); ++k) {
        BufRef r;
        r.kind = BK_INPUT;
        r.index = static_cast<int>(k);
        p.root_ref[static_cast<size_t>(g.inputs[k])] = r;
    }
    std::vector<int> out_copy_region(g.outputs.size(), -1);
    for (size_t k = 0; k < g.outputs.size(); ++k) {
        int n = g.outputs[k];
        const Node& nd = g.nodes[static_cast<size_t>(n)];
        const Storage& s = p.st[static_cast<size_t>(n)];
        const bool folded = nd.fused_into >= 0 && s.kind == SK_BUF && s.root == nd.fused_into;  // GEMM epilogue
        bool own = (s.kind == SK_BUF && s.root == n && nd.op != TT_OP_INPUT && nd.op != TT_OP_CONSTANT) || folded;
        if (own) {
            BufRef r;
            r.kind = BK_OUTPUT;
            r.index = static_cast<int>(k);
            p.root_ref[static_cast<size_t>(s.root)] = r;
        } else {
            Region r;
            r.shape = nd.shape;
            r.is_copy = true;
            r.ext.push_back(n);
            r.ext_access.push_back(broadcast_access(s, n, nd.shape, nd.shape));
            BufRef br;
            br.kind = BK_OUTPUT;
            br.index = static_cast<int>(k);
            r.store_ref.push_back(br);
            p.regions.push_back(r);
            out_copy_region[k] = static_cast<int>(p.regions.size()) - 1;
        }
    }

    // ---- 3. launch units and their order ----
    struct Unit {
        int type, idx, key;
        std::vector<int> reads, writes;  // root nodes
    };
    std::vector<Unit> units;
    for (size_t R = 0; R < p.regions.size(); ++R) {
        Region& r = p.regions[R];
        Unit u{LT_REGION, static_cast<int>(R), 0, {}, {}};
        int key = 1 << 30;
        for (int i : r.nodes) key = std::min(key, i);
        for (size_t e = 0; e < r.ext.size(); ++e) {
            if (!r.ext_access[e].imm) u.reads.push_back(r.ext_access[e].node);
            key = std::min(key, r.ext[e] + 1);
        }
        for (int s : r.stores) {
            u.writes.push_back(s);
            key = std::min(key, s);
        }
        if (r.nodes.empty() && r.stores.empty()) key = static_cast<int>(N) + static_cast<int>(R);  // output copies last
        u.key = key;
        units.push_back(u);
    }
    for (int i : launch_nodes) {
        const Node& n = g.nodes[static_cast<size_t>(i)];
        Unit u{n.op == TT_OP_MATMUL ? LT_GEMM : LT_REDUCE, i, i, {}, {i}};
        for (int q : n.in) u.reads.push_back(p.st[static_cast<size_t>(q)].root);
        units.push_back(u);
    }
    std::map<int, int> producer;  // root -> unit
    for (size_t u = 0; u < units.size(); ++u)
        for (int w : units[u].writes) producer[w] = static_cast<int>(u);
    std::vector<std::vector<int>> succ(units.size());
    std::vector<int> indeg(units.size(), 0);
    for (size_t u = 0; u < units.size(); ++u) {
        std::set<int> pre;
        for (int r : units[u].reads) {
            auto it = producer.find(r);
            if (it != producer.end() && it->second != static_cast<int>(u)) pre.insert(it->second);
        }
        for (int v : pre) {
            succ[static_cast<size_t>(v)].push_back(static_cast<int>(u));
            indeg[u]++;
        }
    }
    // Among ready launches, those that finish a graph output go first (then graph
    // order): a caller waiting on an output (e.g. a gradient to all-reduce while the
    // backward pass continues) can start as early as the dependencies allow.
    for (Unit& u : units) {
        bool writes_output = false;
        for (int w : u.writes)
            if (p.root_ref[static_cast<size_t>(w)].kind == BK_OUTPUT) writes_output = true;
        if (u.type == LT_REGION && !p.regions[static_cast<size_t>(u.idx)].store_ref.empty()) {
            for (const BufRef& b : p.regions[static_cast<size_t>(u.idx)].store_ref)
                if (b.kind == BK_OUTPUT) writes_output = true;
        }
        if (writes_output && u.key < static_cast<int>(N)) u.key -= static_cast<int>(N) + 1;
    }
    using QE = std::pair<int, int>;
    std::priority_queue<QE, std::vector<QE>, std::greater<QE>> ready;
    for (size_t u = 0; u < units.size(); ++u)
        if (indeg[u] == 0) ready.push({units[u].key, static_cast<int>(u)});
    std::vector<int> order;
    while (!ready.empty()) {
        int u = ready.top().second;
        ready.pop();
        order.push_back(u);
        for (int v : succ[static_cast<size_t>(u)])
            if (--indeg[static_cast<size_t>(v)] == 0) ready.push({units[static_cast<size_t>(v)].key, v});
    }
    if (order.size() != units.size()) fail(TT_ERR_COMPILE, "internal: cyclic launch schedule");

    // ---- launches ----
    for (int u : order) {
        const Unit& un = units[static_cast<size_t>(u)];
        Launch L;
        L.type = un.type;
        if (un.type == LT_REGION) {
            L.region = un.idx;
            Region& r = p.regions[static_cast<size_t>(un.idx)];
            r.kernel = "ttk_region_" + std::to_string(un.idx);
            std::ostringstream lb;
            if (r.is_copy) lb << "copy" << shape_str(r.shape);
            else {
                lb << "fused[";
                for (size_t k = 0; k < r.nodes.size(); ++k)
                    lb << (k ? "," : "") << op_name(g.nodes[static_cast<size_t>(r.nodes[k])].op);
                lb << "]" << shape_str(r.shape);
            }
            L.label = lb.str();
        } else if (un.type == LT_REDUCE) {
            const Node& n = g.nodes[static_cast<size_t>(un.idx)];
            const Node& a = g.nodes[static_cast<size_t>(n.in[0])];
            const Storage& s = p.st[static_cast<size_t>(n.in[0])];
            L.in_node = s.root;
            L.out_node = un.idx;
            ReduceDesc& d = L.rd;
            d.op = n.op == TT_OP_REDUCE_SUM ? RO_SUM : n.op == TT_OP_REDUCE_MEAN ? RO_MEAN : RO_MAX;
            d.in_offset = s.offset;
            auto ax = normalized_axes(n, static_cast<int64_t>(a.shape.size()));
            std::vector<int64_t> ks, kst, rs, rst;
            for (size_t dd = 0; dd < a.shape.size(); ++dd) {
                if (a.shape[dd] == 1) continue;
                bool red = std::binary_search(ax.begin(), ax.end(), static_cast<int64_t>(dd));
                (red ? rs : ks).push_back(a.shape[dd]);
                (red ? rst : kst).push_back(s.strides[dd]);
            }
            auto collapse = [](std::vector<int64_t>& sz, std::vector<int64_t>& st) {
                for (size_t k = sz.size(); k-- > 1;) {
                    if (st[k - 1] == st[k] * sz[k]) {
                        sz[k - 1] *= sz[k];
                        st[k - 1] = st[k];
                        sz.erase(sz.begin() + static_cast<long>(k));
                        st.erase(st.begin() + static_cast<long>(k));
                    }
                }
            };
            collapse(ks, kst);
            collapse(rs, rst);
            int64_t count = 1;
            for (int64_t v : rs) count *= v;
            int64_t outn = 1;
            for (int64_t v : ks) outn *= v;
            d.mean_scale = static_cast<float>(1.0 / static_cast<double>(count > 0 ? count : 1));
            if (numel(a.shape) == 0) count = 0;
            if (rs.size() <= 1 && ks.size() <= 1 && (rs.empty() || rst[0] == 1)) {
                d.kind = RK_ROW;
                d.outer = outn;
                d.R = rs.empty() ? 1 : rs[0];
                d.s_red = 1;
                d.s_outer = ks.empty() ? 0 : kst[0];
            } else if (rs.size() == 1 && ks.size() == 1 && kst[0] == 1) {
                d.kind = RK_COL;
                d.outer = ks[0];
                d.R = rs[0];
                d.s_red = rst[0];
                d.s_outer = 1;
            } else {
                d.kind = RK_GENERIC;
                d.nk = static_cast<int>(ks.size());
                d.nr = static_cast<int>(rs.size());
                for (int k = 0; k < d.nk; ++k) {
                    d.ksize[k] = ks[static_cast<size_t>(k)];
                    d.kstride[k] = kst[static_cast<size_t>(k)];
                }
                for (int k = 0; k < d.nr; ++k) {
                    d.rsize[k] = rs[static_cast<size_t>(k)];
                    d.rstride[k] = rst[static_cast<size_t>(k)];
                }
                d.outer = outn;
                d.R = count;
            }
            if (numel(a.shape) == 0) {  // empty input: sum -> 0 (operators.cpp:428-430)
                d.kind = RK_ROW;
                d.outer = outn;
                d.R = 0;
            }
            L.scratch_bytes = reduce_prepare(d);
            std::ostringstream lb;
            lb << op_name(n.op) << (d.kind == RK_ROW ? "/row" : d.kind == RK_COL ? "/col" : "/generic")
               << shape_str(a.shape);
            L.label = lb.str();
        } else {
            const Node& n = g.nodes[static_cast<size_t>(un.idx)];
            const Node& A = g.nodes[static_cast<size_t>(n.in[0])];
            const Node& B = g.nodes[static_cast<size_t>(n.in[1])];
            const Storage& sa = p.st[static_cast<size_t>(n.in[0])];
            const Storage& sb = p.st[static_cast<size_t>(n.in[1])];
            L.in_node = sa.root;
            L.in_node2 = sb.root;
            L.out_node = un.idx;
            GemmDesc& d = L.gd;
            size_t ra = A.shape.size(), rb = B.shape.size(), rc = n.shape.size();
            d.M = n.shape[rc - 2];
            d.N = n.shape[rc - 1];
            d.K = A.shape[ra - 1];
            d.batch = 1;
            for (size_t k = 0; k + 2 < rc; ++k) d.batch *= n.shape[k];
            d.a_sm = sa.strides[ra - 2];
            d.a_sk = sa.strides[ra - 1];
            d.b_sk = sb.strides[rb - 2];
            d.b_sn = sb.strides[rb - 1];
            d.a_off = sa.offset;
            d.b_off = sb.offset;
            // batch stride of an operand: its innermost batch dim (broadcast -> 0)
            auto bstride = [&](const Storage& s, const Shape& sh, size_t r) -> int64_t {
                if (r <= 2 || d.batch == 1) return 0;
                size_t lead = rc - 2, own = r - 2;
                int64_t st = 0;
                for (size_t k = 0; k < own; ++k)
                    if (sh[k] != 1) st = s.strides[k];
                (void)lead;
                if (own < lead) {
                    // operand has fewer batch dims: broadcast over the extra leading ones
                    int64_t own_count = 1;
                    for (size_t k = 0; k < own; ++k) own_count *= sh[k];
                    if (own_count != 1 && own_count != d.batch)
                        fail(TT_ERR_COMPILE, "batched matmul with partial batch broadcast is not supported");
                    if (own_count == 1) return 0;
                }
                int64_t own_count = 1;
                for (size_t k = 0; k < own; ++k) own_count *= sh[k];
                if (own_count == 1) return 0;
                if (own_count != d.batch)
                    fail(TT_ERR_COMPILE, "batched matmul with partial batch broadcast is not supported");
                return st;
            };
            d.a_sb = bstride(sa, A.shape, ra);
            d.b_sb = bstride(sb, B.shape, rb);
            d.c_sb = d.M * d.N;
            d.epilogue = n.epilogue;
            if (d.M == 1) d.a_sm = d.a_sk == 1 ? d.K : 1;
            plan_gemm(d);
            L.scratch_bytes = gemm_scratch_bytes(d);
            std::ostringstream lb;
            lb << "gemm/" << gemm_algo_name(d.algo) << "[" << d.M << "x" << d.N << "x" << d.K;
            if (d.batch > 1) lb << " b" << d.batch;
            if (d.ksplit > 1) lb << " splitk" << d.ksplit;
            if (d.tail_split > 0) lb << " tail" << d.tail_tiles << "x" << d.tail_split;
            lb << (d.a_sk == 1 ? " A:K" : " A:M") << (d.b_sn == 1 ? " B:N" : " B:K");
            if (d.epilogue != EP_NONE) lb << (d.epilogue == EP_RELU ? " +relu" : " +tanh");
            lb << "]";
            L.label = lb.str();
        }
        p.launches.push_back(L);
    }

    // ---- hi/lo operand copies written by the producing region ----
    // A tensor-core GEMM operand that is a whole 2-D matrix stored by an elementwise
    // region, read as it is along K (A = X, or B = X^T) or across K (A = X^T, or B = X),
    // is not split by a pre-pass of its own: the region writes the hi/lo copies in the
    // layout(s) its GEMM readers use, from the values it has in registers (a tiled
    // kernel; the transposed copies go out through shared memory in 128-B runs).  When
    // nothing else reads the matrix, its fp32 value is not stored at all.  This replaces
    // a re-read of the matrix (and its fp32 write) per reading GEMM.
    std::vector<char> dropped(g.nodes.size(), 0);
    if (opt.gemm_epilogue) {
        std::map<int, std::pair<int, int>> store_of;  // node -> (region launch, store index)
        for (size_t s = 0; s < p.launches.size(); ++s) {
            const Launch& L = p.launches[s];
            if (L.type != LT_REGION) continue;
            const Region& r = p.regions[static_cast<size_t>(L.region)];
            if (r.is_copy || r.stores.empty()) continue;
            for (size_t j = 0; j < r.stores.size(); ++j) {
                const Shape& sh = g.nodes[static_cast<size_t>(r.stores[j])].shape;
                if (sh.size() == 2 && sh[0] > 1 && sh[1] > 1 && sh == r.shape)
                    store_of[r.stores[j]] = {static_cast<int>(s), static_cast<int>(j)};
            }
        }
        for (size_t c = 0; c < p.launches.size(); ++c) {
            Launch& L = p.launches[c];
            if (L.type != LT_GEMM || L.gd.algo != 2 || L.gd.batch != 1) continue;
            GemmDesc& d = L.gd;
            for (int k = 0; k < 2; ++k) {
                const int node = k == 0 ? L.in_node : L.in_node2;
                auto it = store_of.find(node);
                if (it == store_of.end() || it->second.first >= static_cast<int>(c)) continue;
                Launch& P = p.launches[static_cast<size_t>(it->second.first)];
                Region& pr = p.regions[static_cast<size_t>(P.region)];
                if (pr.copy_store >= 0 && pr.copy_store != it->second.second) continue;  // one copied store per region
                const Shape& sh = g.nodes[static_cast<size_t>(node)].shape;
                const int64_t pm = sh[0], pn = sh[1];  // X: [pm][pn], row stride pn
                int layout = -1;
                if (k == 0 && d.a_off == 0) {  // A[m][k]; its K-major copy is [M][round4(K)]
                    if (d.a_sk == 1 && d.a_sm == pn && d.M == pm && d.K == pn) layout = 0;       // A = X
                    else if (d.a_sm == 1 && d.a_sk == pn && d.M == pn && d.K == pm) layout = 1;  // A = X^T
                } else if (k == 1 && d.b_off == 0) {  // B[k][n]; its K-major copy is [N][round4(K)]
                    if (d.b_sk == 1 && d.b_sn == pn && d.N == pm && d.K == pn) layout = 0;       // B = X^T
                    else if (d.b_sn == 1 && d.b_sk == pn && d.N == pn && d.K == pm) layout = 1;  // B = X
                }
                if (layout < 0) continue;
                pr.copy_store = it->second.second;
                pr.copy_R = pm;
                pr.copy_C = pn;
                if (layout == 0) pr.copy_rows = true;
                else pr.copy_t = true;
                if (k == 0) {
                    d.a_presplit = 1;
                    L.a_split_src = it->second.first;
                    L.a_split_layout = layout;
                } else {
                    d.b_presplit = 1;
                    L.b_split_src = it->second.first;
                    L.b_split_layout = layout;
                }
                std::ostringstream lb;
                lb << " (" << (k == 0 ? "A" : "B") << " hi/lo from [" << it->second.first << "])";
                L.label += lb.str();
            }
            L.scratch_bytes = gemm_scratch_bytes(d);
        }
        // a copied matrix whose only readers take the copies is not stored in fp32
        for (Launch& L : p.launches) {
            if (L.type != LT_REGION) continue;
            Region& r = p.regions[static_cast<size_t>(L.region)];
            if (r.copy_store < 0) continue;
            const int q = r.stores[static_cast<size_t>(r.copy_store)];
            bool other = out_pos.size() > static_cast<size_t>(q) && out_pos[static_cast<size_t>(q)] >= 0;
            for (const Launch& U : p.launches) {
                if (U.type == LT_REGION) {
                    for (const Access& a : p.regions[static_cast<size_t>(U.region)].ext_access)
                        other |= !a.imm && a.node == q;
                } else if (U.type == LT_REDUCE) {
                    other |= U.in_node == q;
                } else {
                    other |= (U.in_node == q && !U.gd.a_presplit) || (U.in_node2 == q && !U.gd.b_presplit);
                }
            }
            r.drop_f32 = !other;
            if (r.drop_f32) dropped[static_cast<size_t>(q)] = 1;
            L.label += r.copy_rows && r.copy_t ? " (writes hi/lo of X and X^T" : r.copy_rows ? " (writes hi/lo of X"
                                                                                             : " (writes hi/lo of X^T";
            L.label += r.drop_f32 ? ", not X)" : ")";
        }
    }

    // ---- concurrent GEMM pairs ----
    // Two adjacent tensor-core GEMM launches, the second neither reading the first's
    // output nor writing what the first reads, each of at most four waves of CTAs, run
    // side by side on two streams: the CTAs of one fill the part-empty last wave of the
    // other.  Measured on B200 for the MLP gradient program: 2 % faster with 4096-row
    // shards (two 512-CTA GEMMs), equal at 8192 rows, 7 % slower at 32768 rows (two big
    // GEMMs interleaved thrash each other's L2 working set) -- hence the size limit.  For
    // the memory plan a pair is one step, so none of their buffers or scratch share a slot.
    const size_t nl = p.launches.size();
    std::vector<int> plan_step(nl + 1, 0);
    {
        int stp = 0;
        for (size_t s = 0; s < nl; ++s) {
            plan_step[s] = stp;
            const int64_t wave4 = 4 * 148;
            if (opt.concurrent_gemms && s + 1 < nl && p.launches[s].type == LT_GEMM &&
                p.launches[s + 1].type == LT_GEMM && gemm_tc_ctas(p.launches[s].gd) > 0 &&
                gemm_tc_ctas(p.launches[s].gd) <= wave4 && gemm_tc_ctas(p.launches[s + 1].gd) > 0 &&
                gemm_tc_ctas(p.launches[s + 1].gd) <= wave4) {
                const Launch& a = p.launches[s];
                const Launch& b = p.launches[s + 1];
                const bool dep = b.in_node == a.out_node || b.in_node2 == a.out_node || a.in_node == b.out_node ||
                                 a.in_node2 == b.out_node || a.out_node == b.out_node;
                if (!dep) {
                    p.launches[s].concurrent_next = true;
                    plan_step[s + 1] = stp;
                    ++s;
                }
            }
            ++stp;
        }
        plan_step[nl] = stp;
    }

    // ---- 4. memory plan ----
    // Roots needing arena slots: computed roots not bound to an output buffer.
    std::vector<int> step_of_unit(units.size());
    for (size_t s = 0; s < order.size(); ++s) step_of_unit[static_cast<size_t>(order[s])] = plan_step[s];
    struct Life {
        int root;  // node, or -1 - launch index for scratch
        int first, last;
        int64_t bytes;
        int slot = -1;
    };
    std::vector<Life> lives;
    std::map<int, size_t> life_of;
    for (size_t u = 0; u < units.size(); ++u)
        for (int w : units[u].writes) {
            if (p.root_ref[static_cast<size_t>(w)].kind == BK_OUTPUT) continue;
            if (dropped[static_cast<size_t>(w)]) continue;  // fp32 value never stored (copies only)
            Life l{w, step_of_unit[u], step_of_unit[u],
                   numel(g.nodes[static_cast<size_t>(w)].shape) * static_cast<int64_t>(sizeof(float))};
            life_of[w] = lives.size();
            lives.push_back(l);
        }
    for (size_t u = 0; u < units.size(); ++u)
        for (int r : units[u].reads) {
            auto it = life_of.find(r);
            if (it != life_of.end()) lives[it->second].last = std::max(lives[it->second].last, step_of_unit[u]);
        }
    for (size_t s = 0; s < p.launches.size(); ++s)
        if (p.launches[s].scratch_bytes > 0)
            lives.push_back(Life{-1 - static_cast<int>(s), plan_step[s], plan_step[s], p.launches[s].scratch_bytes});
    // a region's hi/lo operand copies: from the region to its last GEMM reader
    const int nlaunch = static_cast<int>(p.launches.size());
    for (size_t s = 0; s < p.launches.size(); ++s) {
        const Launch& L = p.launches[s];
        if (L.type != LT_REGION || p.regions[static_cast<size_t>(L.region)].copy_store < 0) continue;
        const Region& r = p.regions[static_cast<size_t>(L.region)];
        int last = plan_step[s];
        for (size_t c = 0; c < p.launches.size(); ++c) {
            const Launch& C = p.launches[c];
            if (C.a_split_src == static_cast<int>(s) || C.b_split_src == static_cast<int>(s))
                last = std::max(last, plan_step[c]);
        }
        lives.push_back(Life{-1 - nlaunch - static_cast<int>(s), plan_step[s], last,
                             split_copies_bytes(r.copy_R, r.copy_C, r.copy_rows, r.copy_t)});
    }
    p.num_intermediates = lives.size();
    for (const Life& l : lives) p.total_alloc_bytes += l.bytes;
    for (size_t s = 0; s <= p.launches.size(); ++s) {
        int64_t live = 0;
        for (const Life& l : lives)
            if (l.first <= static_cast<int>(s) && static_cast<int>(s) <= l.last) live += l.bytes;
        p.theoretical_peak_bytes = std::max(p.theoretical_peak_bytes, live);
    }
    std::stable_sort(lives.begin(), lives.end(), [](const Life& a, const Life& b) { return a.first < b.first; });
    for (Life& l : lives) {
        bool found = false;
        for (size_t k = 0; k < p.slots.size(); ++k) {
            Slot& sl = p.slots[k];
            if (sl.last_step < l.first) {
                sl.last_step = l.last;
                sl.capacity = std::max(sl.capacity, align256(l.bytes));
                l.slot = static_cast<int>(k);
                found = true;
                ++p.reused_buffers;
                break;
            }
        }
        if (!found) {
            Slot sl;
            sl.capacity = align256(l.bytes);
            sl.last_step = l.last;
            p.slots.push_back(sl);
            l.slot = static_cast<int>(p.slots.size()) - 1;
        }
    }
    // Arena: [constants][slots][input staging][output staging][status word]
    int64_t off = 0;
    for (size_t i = 0; i < N; ++i) {
        const Node& n = g.nodes[i];
        if (n.op == TT_OP_CONSTANT && n.cdata.size() > 1) {
            BufRef r;
            r.kind = BK_ARENA;
            r.offset = off;
            p.root_ref[i] = r;
            p.constants.push_back({off, static_cast<int>(i)});
            off += align256(static_cast<int64_t>(n.cdata.size() * sizeof(float)));
        }
    }
    p.const_bytes = off;
    for (Slot& sl : p.slots) {
        sl.offset = off;
        off += sl.capacity;
    }
    p.slot_bytes = off - p.const_bytes;
    p.peak_planned_bytes = p.slot_bytes;
    for (const Life& l : lives) {
        BufRef r;
        r.kind = BK_ARENA;
        r.offset = p.slots[static_cast<size_t>(l.slot)].offset;
        if (l.root >= 0) p.root_ref[static_cast<size_t>(l.root)] = r;
        else if (-1 - l.root < nlaunch) p.launches[static_cast<size_t>(-1 - l.root)].scratch_ref = r;
        else p.launches[static_cast<size_t>(-1 - nlaunch - l.root)].split_ref = r;
    }
    p.stage_in_offset = off;
    for (int k : g.inputs) {
        p.stage_in.push_back(off);
        off += align256(numel(g.nodes[static_cast<size_t>(k)].shape) * static_cast<int64_t>(sizeof(float)));
    }
    p.stage_out_offset = off;
    for (int k : g.outputs) {
        p.stage_out.push_back(off);
        off += align256(numel(g.nodes[static_cast<size_t>(k)].shape) * static_cast<int64_t>(sizeof(float)));
    }
    p.status_offset = off;
    off += 256;
    p.arena_bytes = off;

    // ---- bind launch buffers ----
    for (Launch& L : p.launches) {
        if (L.type == LT_REGION) {
            Region& r = p.regions[static_cast<size_t>(L.region)];
            if (r.store_ref.empty())
                for (int s : r.stores) r.store_ref.push_back(p.root_ref[static_cast<size_t>(s)]);
        } else {
            L.in_ref = p.root_ref[static_cast<size_t>(L.in_node)];
            if (L.in_node2 >= 0) L.in_ref2 = p.root_ref[static_cast<size_t>(L.in_node2)];
            L.out_ref = p.root_ref[static_cast<size_t>(L.out_node)];
        }
    }
    (void)out_copy_region;
    // launch after which each graph output is complete (its last writer)
    // last launch that reads each graph input's buffer (a caller may overwrite the input,
    // e.g. a parameter update, once that launch is done)
    p.input_last_step.assign(g.inputs.size(), -1);
    {
        std::map<int, size_t> input_of;
        for (size_t k = 0; k < g.inputs.size(); ++k) input_of[g.inputs[k]] = k;
        for (size_t s = 0; s < p.launches.size(); ++s) {
            const Launch& L = p.launches[s];
            auto mark = [&](int root) {
                auto it = input_of.find(root);
                if (it != input_of.end()) p.input_last_step[it->second] = static_cast<int>(s);
            };
            if (L.type == LT_REGION) {
                for (const Access& a : p.regions[static_cast<size_t>(L.region)].ext_access)
                    if (!a.imm) mark(a.node);
            } else {
                mark(L.in_node);
                if (L.in_node2 >= 0) mark(L.in_node2);
            }
        }
    }
    p.output_step.assign(g.outputs.size(), -1);
    for (size_t s = 0; s < p.launches.size(); ++s) {
        const Launch& L = p.launches[s];
        auto mark = [&](const BufRef& b) {
            if (b.kind == BK_OUTPUT) p.output_step[static_cast<size_t>(b.index)] = static_cast<int>(s);
        };
        if (L.type == LT_REGION) {
            for (const BufRef& b : p.regions[static_cast<size_t>(L.region)].store_ref) mark(b);
        } else {
            mark(L.out_ref);
        }
    }
    return p;
}

static const char* kind_name(int k) {
    switch (k) {
        case BK_ARENA: return "arena";
        case BK_INPUT: return "input";
        case BK_OUTPUT: return "output";
        default: return "-";
    }
}

std::string plan_text(const Plan& p) {
    std::ostringstream ss;
    ss << "Device Arena: " << p.arena_bytes << " bytes (constants " << p.const_bytes << ", slots " << p.slot_bytes
       << " in " << p.slots.size() << " slots, staging " << (p.status_offset - p.stage_in_offset) << ")\n";
    for (size_t k = 0; k < p.slots.size(); ++k)
        ss << "  slot " << k << " @ " << p.slots[k].offset << " capacity " << p.slots[k].capacity << "\n";
    ss << "Kernel Launches (" << p.launches.size() << "):\n";
    for (size_t s = 0; s < p.launches.size(); ++s) {
        const Launch& L = p.launches[s];
        ss << "  [" << s << "] " << L.label;
        if (L.type == LT_REGION) {
            const Region& r = p.regions[static_cast<size_t>(L.region)];
            ss << " kernel=" << r.kernel << " vec=" << r.vec << " grid=" << r.grid << " ->";
            for (const BufRef& b : r.store_ref) ss << " " << kind_name(b.kind) << ":" << (b.kind == BK_ARENA ? b.offset : b.index);
            if (r.copy_store >= 0)
                ss << " copies=" << split_copies_bytes(r.copy_R, r.copy_C, r.copy_rows, r.copy_t) << "@"
                   << L.split_ref.offset;
        } else {
            ss << " ->" << " " << kind_name(L.out_ref.kind) << ":"
               << (L.out_ref.kind == BK_ARENA ? L.out_ref.offset : L.out_ref.index);
            if (L.scratch_bytes) ss << " scratch=" << L.scratch_bytes << "@" << L.scratch_ref.offset;
        }
        if (L.concurrent_next) ss << "  || runs beside [" << s + 1 << "] on the second stream";
        ss << "\n";
    }
    return ss.str();
}

}  // namespace ttb
