// Graph import, shape rules, verification, canonical IR text and the
// graph-level clean-ups (fused-node expansion, DCE, CSE) of the B200 backend.
//
// Shape rules follow the reference Graph builders (src/graph/graph.cpp:51-200) and
// IRVerifier (src/ir/verifier.cpp:7-202); the IR text follows IRPrinter
// (src/ir/printer.cpp:6-62) so that cache keys and diagnostics read the same.
#include <algorithm>
#include <cstring>
#include <map>
#include <set>
#include <sstream>
#include <unordered_map>

#include "ttb.hpp"

namespace ttb {

void fail(int status, const std::string& msg) { throw Error(status, msg); }

int Graph::add(Node n) {
    if (n.id < next_id) n.id = next_id;
    next_id = n.id + 1;
    nodes.push_back(std::move(n));
    return static_cast<int>(nodes.size()) - 1;
}

int64_t numel(const Shape& s) {
    int64_t n = 1;
    for (int64_t d : s) n *= d;
    return n;
}

std::string shape_str(const Shape& s) {
    std::ostringstream ss;
    ss << "[";
    for (size_t i = 0; i < s.size(); ++i) ss << (i ? ", " : "") << s[i];
    ss << "]";
    return ss.str();
}

// Tensor::broadcast_shapes (src/core/tensor.cpp:189-215): right-aligned, 1 stretches.
Shape broadcast_shapes(const Shape& a, const Shape& b) {
    size_t r = std::max(a.size(), b.size());
    Shape out(r);
    for (size_t i = 0; i < r; ++i) {
        int64_t da = (i + a.size() >= r) ? a[i + a.size() - r] : 1;
        int64_t db = (i + b.size() >= r) ? b[i + b.size() - r] : 1;
        if (da != db && da != 1 && db != 1)
            fail(TT_ERR_BROADCAST, "Shapes " + shape_str(a) + " and " + shape_str(b) + " are not broadcastable");
        out[i] = (da == 1) ? db : da;
    }
    return out;
}

std::vector<int64_t> normalized_axes(const Node& n, int64_t rank) {
    std::set<int64_t> s;
    if (n.axes.empty()) {
        for (int64_t i = 0; i < rank; ++i) s.insert(i);
    } else {
        for (int64_t ax : n.axes) {
            int64_t a = ax < 0 ? ax + rank : ax;
            if (a < 0 || a >= rank)
                fail(TT_ERR_DIMENSION, "Reduction axis " + std::to_string(ax) + " out of bounds for rank " +
                                           std::to_string(rank));
            s.insert(a);
        }
    }
    return {s.begin(), s.end()};
}

const char* op_name(int op) {
    switch (op) {
        case TT_OP_INPUT: return "input";
        case TT_OP_CONSTANT: return "constant";
        case TT_OP_ADD: return "add";
        case TT_OP_SUB: return "sub";
        case TT_OP_MUL: return "mul";
        case TT_OP_DIV: return "div";
        case TT_OP_RELU: return "relu";
        case TT_OP_SIGMOID: return "sigmoid";
        case TT_OP_MATMUL: return "matmul";
        case TT_OP_TRANSPOSE: return "transpose";
        case TT_OP_REDUCE_SUM: return "reduce_sum";
        case TT_OP_REDUCE_MEAN: return "reduce_mean";
        case TT_OP_OUTPUT: return "output";
        case TT_OP_FUSED_ELEMENTWISE: return "fused_elementwise";
        case TT_OP_EXP: return "exp";
        case TT_OP_NEG: return "neg";
        case TT_OP_TANH: return "tanh";
        case TT_OP_REDUCE_MAX: return "reduce_max";
        case TT_OP_STEP: return "step";
        case TT_OP_RESHAPE: return "reshape";
        case TT_OP_EXPAND: return "expand";
        default: return "unknown";
    }
}

bool is_elementwise(int op) {
    switch (op) {
        case TT_OP_ADD: case TT_OP_SUB: case TT_OP_MUL: case TT_OP_DIV:
        case TT_OP_RELU: case TT_OP_SIGMOID: case TT_OP_EXP: case TT_OP_NEG:
        case TT_OP_TANH: case TT_OP_STEP:
            return true;
        default:
            return false;
    }
}
bool is_view(int op) { return op == TT_OP_TRANSPOSE || op == TT_OP_RESHAPE || op == TT_OP_EXPAND; }
bool is_reduce(int op) { return op == TT_OP_REDUCE_SUM || op == TT_OP_REDUCE_MEAN || op == TT_OP_REDUCE_MAX; }

static int arity(int op) {
    switch (op) {
        case TT_OP_INPUT: case TT_OP_CONSTANT: return 0;
        case TT_OP_ADD: case TT_OP_SUB: case TT_OP_MUL: case TT_OP_DIV: case TT_OP_MATMUL: return 2;
        case TT_OP_FUSED_ELEMENTWISE: return -1;
        default: return 1;
    }
}

// Output shape of a node from its inputs (graph.cpp:51-200 builders).
void infer_shape(Graph& g, Node& n) {
    auto in = [&](int i) -> const Node& { return g.nodes[static_cast<size_t>(n.in[static_cast<size_t>(i)])]; };
    switch (n.op) {
        case TT_OP_INPUT:
        case TT_OP_CONSTANT:
        case TT_OP_RESHAPE:
        case TT_OP_EXPAND:
        case TT_OP_FUSED_ELEMENTWISE:
            return;  // shape given
        case TT_OP_ADD: case TT_OP_SUB: case TT_OP_MUL: case TT_OP_DIV:
            if (in(0).dtype != in(1).dtype) fail(TT_ERR_TYPE, std::string("DType mismatch in ") + op_name(n.op));
            n.shape = broadcast_shapes(in(0).shape, in(1).shape);
            n.dtype = in(0).dtype;
            return;
        case TT_OP_RELU: case TT_OP_SIGMOID: case TT_OP_EXP: case TT_OP_NEG: case TT_OP_TANH: case TT_OP_STEP:
            n.shape = in(0).shape;
            n.dtype = in(0).dtype;
            return;
        case TT_OP_MATMUL: {
            const Shape& a = in(0).shape;
            const Shape& b = in(1).shape;
            if (in(0).dtype != in(1).dtype) fail(TT_ERR_TYPE, "DType mismatch in matmul");
            if (a.size() < 2 || b.size() < 2) fail(TT_ERR_DIMENSION, "Unsupported ranks for matmul");
            int64_t ka = a[a.size() - 1], kb = b[b.size() - 2];
            if (ka != kb)
                fail(TT_ERR_SHAPE, "Matmul inner dimensions mismatch: " + std::to_string(ka) + " vs " +
                                       std::to_string(kb));
            Shape out;
            if (a.size() > 2 || b.size() > 2)
                out = broadcast_shapes(Shape(a.begin(), a.end() - 2), Shape(b.begin(), b.end() - 2));
            out.push_back(a[a.size() - 2]);
            out.push_back(b[b.size() - 1]);
            n.shape = out;
            n.dtype = in(0).dtype;
            return;
        }
        case TT_OP_TRANSPOSE: {
            int64_t r = static_cast<int64_t>(in(0).shape.size());
            int64_t d0 = n.dim0 < 0 ? n.dim0 + r : n.dim0;
            int64_t d1 = n.dim1 < 0 ? n.dim1 + r : n.dim1;
            if (d0 < 0 || d0 >= r || d1 < 0 || d1 >= r)
                fail(TT_ERR_DIMENSION, "Invalid transpose axes for rank " + std::to_string(r));
            n.dim0 = d0;
            n.dim1 = d1;
            n.shape = in(0).shape;
            std::swap(n.shape[static_cast<size_t>(d0)], n.shape[static_cast<size_t>(d1)]);
            n.dtype = in(0).dtype;
            return;
        }
        case TT_OP_REDUCE_SUM: case TT_OP_REDUCE_MEAN: case TT_OP_REDUCE_MAX: {
            const Shape& a = in(0).shape;
            auto ax = normalized_axes(n, static_cast<int64_t>(a.size()));
            Shape out;
            for (size_t i = 0; i < a.size(); ++i) {
                bool red = std::binary_search(ax.begin(), ax.end(), static_cast<int64_t>(i));
                if (red) {
                    if (n.keepdims) out.push_back(1);
                } else {
                    out.push_back(a[i]);
                }
            }
            n.shape = out;
            n.dtype = in(0).dtype;
            return;
        }
        default:
            fail(TT_ERR_IR, std::string("Unknown op code ") + std::to_string(n.op));
    }
}

Graph import_graph(const tt_graph* cg) {
    if (!cg) fail(TT_ERR_INVALID, "null graph");
    if (cg->num_nodes < 0 || (cg->num_nodes > 0 && !cg->nodes)) fail(TT_ERR_INVALID, "bad node array");
    Graph g;
    for (int32_t i = 0; i < cg->num_nodes; ++i) {
        const tt_node& c = cg->nodes[i];
        Node n;
        n.op = c.op;
        n.dtype = c.dtype;
        if (c.dtype != TT_FLOAT32 && c.dtype != TT_FLOAT64) fail(TT_ERR_TYPE, "Unknown dtype");
        if (c.rank < 0 || c.rank > TT_MAX_RANK) fail(TT_ERR_DIMENSION, "rank out of range");
        if (c.num_inputs < 0 || c.num_inputs > TT_MAX_NODE_INPUTS) fail(TT_ERR_IR, "bad input count");
        int ar = arity(c.op);
        if (ar >= 0 && ar != c.num_inputs)
            fail(TT_ERR_IR, std::string("Node %") + std::to_string(c.id) + " (" + op_name(c.op) + ") requires exactly " +
                                std::to_string(ar) + " inputs");
        for (int32_t k = 0; k < c.num_inputs; ++k) {
            if (c.inputs[k] < 0 || c.inputs[k] >= i)
                fail(TT_ERR_IR, "Topological ordering violation: node %" + std::to_string(c.id) +
                                    " uses an operand defined later or not at all");
            n.in.push_back(c.inputs[k]);
        }
        n.shape.assign(c.shape, c.shape + c.rank);
        n.id = c.id;
        n.dim0 = c.dim0;
        n.dim1 = c.dim1;
        if (c.num_axes < 0 || c.num_axes > TT_MAX_RANK) fail(TT_ERR_DIMENSION, "bad axis count");
        n.axes.assign(c.axes, c.axes + c.num_axes);
        n.keepdims = c.keepdims != 0;
        if (c.name) n.name = c.name;
        if (c.expr) n.expr = c.expr;
        if (c.op == TT_OP_INPUT) {
            for (int64_t d : n.shape)
                if (d < 0) fail(TT_ERR_IR, "Input node %" + std::to_string(c.id) + " has negative dimension");
        }
        if (c.op == TT_OP_CONSTANT) {
            int64_t ne = numel(n.shape);
            if (ne > 0 && !c.data) fail(TT_ERR_IR, "Constant node without data");
            n.cdata.resize(static_cast<size_t>(ne));
            if (c.dtype == TT_FLOAT32) {
                if (ne) std::memcpy(n.cdata.data(), c.data, static_cast<size_t>(ne) * sizeof(float));
            } else {
                const double* d = static_cast<const double*>(c.data);
                for (int64_t k = 0; k < ne; ++k) n.cdata[static_cast<size_t>(k)] = static_cast<float>(d[k]);
            }
        }
        Shape given = n.shape;
        infer_shape(g, n);
        if (c.op != TT_OP_INPUT && c.op != TT_OP_CONSTANT && c.op != TT_OP_RESHAPE && c.op != TT_OP_EXPAND &&
            c.op != TT_OP_FUSED_ELEMENTWISE && n.shape != given)
            fail(TT_ERR_IR, std::string("Shape mismatch in ") + op_name(c.op) + " %" + std::to_string(c.id) +
                                ": expected " + shape_str(n.shape) + " but got " + shape_str(given));
        g.nodes.push_back(std::move(n));
        g.next_id = std::max(g.next_id, c.id + 1);
    }
    for (int32_t i = 0; i < cg->num_inputs; ++i) {
        int32_t k = cg->inputs[i];
        if (k < 0 || k >= cg->num_nodes || g.nodes[static_cast<size_t>(k)].op != TT_OP_INPUT)
            fail(TT_ERR_IR, "graph input list names a node that is not an Input");
        g.inputs.push_back(k);
    }
    for (int32_t i = 0; i < cg->num_outputs; ++i) {
        int32_t k = cg->outputs[i];
        if (k < 0 || k >= cg->num_nodes) fail(TT_ERR_IR, "Graph output does not exist in graph");
        if (std::find(g.outputs.begin(), g.outputs.end(), k) == g.outputs.end()) g.outputs.push_back(k);
    }
    return g;
}

// IRVerifier::verify rules (src/ir/verifier.cpp:7-202) on an imported graph.
void verify(const Graph& g) {
    for (size_t i = 0; i < g.nodes.size(); ++i) {
        const Node& n = g.nodes[i];
        for (int k : n.in)
            if (k < 0 || static_cast<size_t>(k) >= i)
                fail(TT_ERR_IR, "Topological ordering violation at node %" + std::to_string(n.id));
        for (int k : n.in)
            if (g.nodes[static_cast<size_t>(k)].dtype != n.dtype)
                fail(TT_ERR_IR, std::string("Type mismatch in ") + op_name(n.op) + " %" + std::to_string(n.id));
        switch (n.op) {
            case TT_OP_CONSTANT:
                if (static_cast<int64_t>(n.cdata.size()) != numel(n.shape))
                    fail(TT_ERR_IR, "Constant node %" + std::to_string(n.id) + " shape mismatch with underlying tensor");
                break;
            case TT_OP_RESHAPE:
                if (numel(n.shape) != numel(g.nodes[static_cast<size_t>(n.in[0])].shape))
                    fail(TT_ERR_SHAPE, "reshape changes the element count");
                break;
            case TT_OP_EXPAND: {
                Shape b = broadcast_shapes(g.nodes[static_cast<size_t>(n.in[0])].shape, n.shape);
                if (b != n.shape) fail(TT_ERR_SHAPE, "expand target is not a broadcast of the operand");
                break;
            }
            case TT_OP_FUSED_ELEMENTWISE:
                if (n.in.empty()) fail(TT_ERR_IR, "Fused elementwise op requires at least 1 input");
                break;
            default:
                break;
        }
    }
    for (int o : g.outputs)
        if (o < 0 || static_cast<size_t>(o) >= g.nodes.size())
            fail(TT_ERR_IR, "Graph output does not exist in graph");
}

static const char* dtype_name(int dt) { return dt == TT_FLOAT64 ? "float64" : "float32"; }

// IRPrinter::to_string (src/ir/printer.cpp:6-62).  Nodes are kept in creation
// order, which is the order the reference DFS topological sort yields for graphs
// whose operands always precede their users.
std::string ir_text(const Graph& g) {
    std::ostringstream ss;
    for (const Node& n : g.nodes) {
        ss << "%" << n.id << " = " << op_name(n.op);
        if (n.op == TT_OP_INPUT || n.op == TT_OP_CONSTANT) {
            ss << "<" << dtype_name(n.dtype) << ">" << shape_str(n.shape);
            if (n.op == TT_OP_INPUT && !n.name.empty()) ss << " ; name=\"" << n.name << "\"";
        } else {
            ss << " ";
            for (size_t i = 0; i < n.in.size(); ++i)
                ss << "%" << g.nodes[static_cast<size_t>(n.in[i])].id << (i + 1 < n.in.size() ? ", " : "");
            if (n.op == TT_OP_TRANSPOSE) {
                ss << " dims=[" << n.dim0 << ", " << n.dim1 << "]";
            } else if (is_reduce(n.op)) {
                ss << " axes=[";
                for (size_t i = 0; i < n.axes.size(); ++i) ss << n.axes[i] << (i + 1 < n.axes.size() ? ", " : "");
                ss << "] keepdims=" << (n.keepdims ? "true" : "false");
            } else if (n.op == TT_OP_FUSED_ELEMENTWISE) {
                ss << " expr=\"" << n.expr << "\"";
            } else if (n.op == TT_OP_RESHAPE || n.op == TT_OP_EXPAND) {
                ss << " shape=" << shape_str(n.shape);
            }
        }
        ss << "\n";
    }
    if (!g.outputs.empty()) {
        ss << "return ";
        for (size_t i = 0; i < g.outputs.size(); ++i)
            ss << "%" << g.nodes[static_cast<size_t>(g.outputs[i])].id << (i + 1 < g.outputs.size() ? ", " : "");
        ss << "\n";
    }
    return ss.str();
}

// Rebuilds a graph keeping the nodes for which keep[i] is true, remapping inputs.
static Graph rebuild(const Graph& g, const std::vector<int>& remap_in, const std::vector<bool>& keep) {
    Graph out;
    out.next_id = g.next_id;
    std::vector<int> idx(g.nodes.size(), -1);
    for (size_t i = 0; i < g.nodes.size(); ++i) {
        if (!keep[i]) continue;
        Node n = g.nodes[i];
        for (int& k : n.in) k = idx[static_cast<size_t>(remap_in[static_cast<size_t>(k)])];
        idx[i] = static_cast<int>(out.nodes.size());
        out.nodes.push_back(std::move(n));
    }
    for (int k : g.inputs) {
        int r = idx[static_cast<size_t>(k)];
        if (r >= 0) out.inputs.push_back(r);
    }
    for (int k : g.outputs) {
        int r = idx[static_cast<size_t>(remap_in[static_cast<size_t>(k)])];
        if (std::find(out.outputs.begin(), out.outputs.end(), r) == out.outputs.end()) out.outputs.push_back(r);
    }
    return out;
}

// The reference FusedElementwise node carries expr "relu(<op>(@0, @1))"
// (src/optimizer/fusion.cpp:45-52), but its codegen always emits relu(a + b)
// (src/codegen/cpp_backend.cpp:345-387).  Here the expression is parsed and
// expanded into primitive nodes so the recorded semantics are the ones computed.
Graph expand_fused(const Graph& g) {
    bool any = false;
    for (const Node& n : g.nodes) any |= n.op == TT_OP_FUSED_ELEMENTWISE;
    if (!any) return g;
    Graph out;
    out.next_id = g.next_id;
    std::vector<int> idx(g.nodes.size(), -1);
    auto parse_op = [](const std::string& s) {
        static const std::map<std::string, int> ops = {{"add", TT_OP_ADD}, {"sub", TT_OP_SUB}, {"mul", TT_OP_MUL},
                                                       {"div", TT_OP_DIV}, {"relu", TT_OP_RELU},
                                                       {"sigmoid", TT_OP_SIGMOID}, {"exp", TT_OP_EXP},
                                                       {"neg", TT_OP_NEG}, {"tanh", TT_OP_TANH}};
        auto it = ops.find(s);
        if (it == ops.end()) fail(TT_ERR_COMPILE, "Unsupported op in fused expression: " + s);
        return it->second;
    };
    for (size_t i = 0; i < g.nodes.size(); ++i) {
        const Node& n = g.nodes[i];
        if (n.op != TT_OP_FUSED_ELEMENTWISE) {
            Node c = n;
            for (int& k : c.in) k = idx[static_cast<size_t>(k)];
            idx[i] = static_cast<int>(out.nodes.size());
            out.nodes.push_back(std::move(c));
            continue;
        }
        // Parse outer(inner(@0[, @1])) — nested calls separated by '('.
        std::string e = n.expr;
        e.erase(std::remove(e.begin(), e.end(), ' '), e.end());
        size_t p1 = e.find('(');
        size_t p2 = e.find('(', p1 + 1);
        if (p1 == std::string::npos || p2 == std::string::npos)
            fail(TT_ERR_COMPILE, "Cannot parse fused expression: " + n.expr);
        int outer = parse_op(e.substr(0, p1));
        int inner = parse_op(e.substr(p1 + 1, p2 - p1 - 1));
        std::vector<int> args;
        for (int k : n.in) args.push_back(idx[static_cast<size_t>(k)]);
        Node a;
        a.op = inner;
        a.dtype = n.dtype;
        bool inner_binary = inner == TT_OP_ADD || inner == TT_OP_SUB || inner == TT_OP_MUL || inner == TT_OP_DIV;
        if (inner_binary && args.size() != 2) fail(TT_ERR_IR, "Fused binary expression needs 2 inputs");
        a.in = inner_binary ? args : std::vector<int>{args[0]};
        a.id = out.next_id++;
        infer_shape(out, a);
        int ai = static_cast<int>(out.nodes.size());
        out.nodes.push_back(a);
        Node b;
        b.op = outer;
        b.dtype = n.dtype;
        b.in = {ai};
        b.id = n.id;
        infer_shape(out, b);
        if (b.shape != n.shape) fail(TT_ERR_IR, "Fused expression shape mismatch");
        idx[i] = static_cast<int>(out.nodes.size());
        out.nodes.push_back(b);
    }
    for (int k : g.inputs) out.inputs.push_back(idx[static_cast<size_t>(k)]);
    for (int k : g.outputs) out.outputs.push_back(idx[static_cast<size_t>(k)]);
    return out;
}

// Dead code elimination: keeps graph inputs (their positions are the ABI) and
// everything that reaches an output.
Graph dce(const Graph& g, size_t* removed) {
    std::vector<bool> live(g.nodes.size(), false);
    for (int o : g.outputs) live[static_cast<size_t>(o)] = true;
    for (size_t i = g.nodes.size(); i-- > 0;)
        if (live[i])
            for (int k : g.nodes[i].in) live[static_cast<size_t>(k)] = true;
    for (int k : g.inputs) live[static_cast<size_t>(k)] = true;
    std::vector<int> ident(g.nodes.size());
    for (size_t i = 0; i < ident.size(); ++i) ident[i] = static_cast<int>(i);
    size_t cnt = 0;
    for (bool b : live) cnt += !b;
    if (removed) *removed = cnt;
    return rebuild(g, ident, live);
}

// Common subexpression elimination keyed like src/optimizer/cse.cpp:9-40
// (op, operand ids, shape, dtype, attributes); constants merge only on equal bits.
Graph cse(const Graph& g, size_t* removed) {
    std::map<std::string, int> seen;
    std::vector<int> remap(g.nodes.size());
    std::vector<bool> keep(g.nodes.size(), true);
    size_t cnt = 0;
    for (size_t i = 0; i < g.nodes.size(); ++i) {
        const Node& n = g.nodes[i];
        remap[i] = static_cast<int>(i);
        if (n.op == TT_OP_INPUT) continue;
        if (n.op == TT_OP_CONSTANT && n.cdata.size() > 64) continue;
        std::ostringstream key;
        key << n.op << "|" << n.dtype << "|" << shape_str(n.shape) << "|";
        for (int k : n.in) key << remap[static_cast<size_t>(k)] << ",";
        key << "|" << n.dim0 << "," << n.dim1 << "|" << n.keepdims << "|";
        for (int64_t a : n.axes) key << a << ",";
        key << "|" << n.expr << "|";
        if (n.op == TT_OP_CONSTANT) {
            for (float f : n.cdata) {
                uint32_t u;
                std::memcpy(&u, &f, 4);
                key << u << ",";
            }
        }
        auto it = seen.find(key.str());
        if (it != seen.end()) {
            remap[i] = it->second;
            keep[i] = false;
            ++cnt;
        } else {
            seen.emplace(key.str(), static_cast<int>(i));
        }
    }
    if (removed) *removed = cnt;
    // Inputs of kept nodes must be remapped before rebuild sees them.
    Graph tmp = g;
    for (size_t i = 0; i < tmp.nodes.size(); ++i)
        for (int& k : tmp.nodes[i].in) k = remap[static_cast<size_t>(k)];
    for (int& o : tmp.outputs) o = remap[static_cast<size_t>(o)];
    std::vector<int> ident(g.nodes.size());
    for (size_t i = 0; i < ident.size(); ++i) ident[i] = static_cast<int>(i);
    return rebuild(tmp, ident, keep);
}

}  // namespace ttb
