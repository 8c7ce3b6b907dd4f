// Symbolic reverse-mode autodiff: emits the backward pass as graph nodes so the
// gradient computation is scheduled, fused, memory-planned and run on the GPU like
// any forward graph.
//
// The vector-Jacobian products and their evaluation order restate the reference's
// eager Autodiff::compute_gradients (src/autodiff/gradient.cpp:52-332): nodes are
// visited in reverse topological order, contributions are accumulated with add in
// that order, and unbroadcast (gradient.cpp:10-50) sums leading axes, then
// singleton axes, then reshapes.  Ops the reference lacks (exp, neg, tanh, step,
// reshape, expand) get their standard derivatives.
#include <algorithm>
#include <cmath>
#include <unordered_map>

#include "ttb.hpp"

namespace ttb {

namespace {

struct Builder {
    Graph& g;

    int mk(int op, std::vector<int> in) {
        Node n;
        n.op = op;
        n.dtype = g.nodes[static_cast<size_t>(in[0])].dtype;
        n.in = std::move(in);
        n.id = g.next_id;
        infer_shape(g, n);
        return g.add(std::move(n));
    }
    int scalar(float v, int dtype) {
        Node n;
        n.op = TT_OP_CONSTANT;
        n.dtype = dtype;
        n.cdata = {v};
        n.id = g.next_id;
        return g.add(std::move(n));
    }
    int view(int op, int a, const Shape s) {
        const Node& an = g.nodes[static_cast<size_t>(a)];
        if (an.shape == s) return a;
        Node n;
        n.op = op;
        n.dtype = an.dtype;
        n.in = {a};
        n.shape = s;
        n.id = g.next_id;
        return g.add(std::move(n));
    }
    int transpose(int a, int64_t d0, int64_t d1) {
        Node n;
        n.op = TT_OP_TRANSPOSE;
        n.dtype = g.nodes[static_cast<size_t>(a)].dtype;
        n.in = {a};
        n.dim0 = d0;
        n.dim1 = d1;
        n.id = g.next_id;
        infer_shape(g, n);
        return g.add(std::move(n));
    }
    int reduce_sum(int a, std::vector<int64_t> axes, bool keepdims) {
        Node n;
        n.op = TT_OP_REDUCE_SUM;
        n.dtype = g.nodes[static_cast<size_t>(a)].dtype;
        n.in = {a};
        n.axes = std::move(axes);
        n.keepdims = keepdims;
        n.id = g.next_id;
        infer_shape(g, n);
        return g.add(std::move(n));
    }
    Shape shape(int a) const { return g.nodes[static_cast<size_t>(a)].shape; }  // by value: g.nodes grows
    int dtype(int a) const { return g.nodes[static_cast<size_t>(a)].dtype; }

    // Autodiff::unbroadcast (gradient.cpp:10-50).
    int unbroadcast(int grad, const Shape target) {
        if (shape(grad) == target) return grad;
        if (target.empty()) return reduce_sum(grad, {}, false);
        int cur = grad;
        size_t gr = shape(grad).size(), tr = target.size();
        if (gr > tr) {
            std::vector<int64_t> lead;
            for (size_t i = 0; i < gr - tr; ++i) lead.push_back(static_cast<int64_t>(i));
            cur = reduce_sum(cur, lead, false);
        }
        std::vector<int64_t> single;
        for (size_t i = 0; i < tr; ++i)
            if (target[i] == 1 && shape(cur)[i] > 1) single.push_back(static_cast<int64_t>(i));
        if (!single.empty()) cur = reduce_sum(cur, single, true);
        if (shape(cur) != target) cur = view(TT_OP_RESHAPE, cur, target);
        return cur;
    }

    // Reduced axes replaced by 1, so the gradient broadcasts back (gradient.cpp:262-324).
    Shape kept_shape(const Node& red, const Shape& in_shape) {
        auto ax = normalized_axes(red, static_cast<int64_t>(in_shape.size()));
        Shape s;
        for (size_t i = 0; i < in_shape.size(); ++i)
            s.push_back(std::binary_search(ax.begin(), ax.end(), static_cast<int64_t>(i)) ? 1 : in_shape[i]);
        return s;
    }
};

}  // namespace

void append_gradients(Graph& g, int loss, const std::vector<int>& wrt) {
    if (loss < 0 || static_cast<size_t>(loss) >= g.nodes.size()) fail(TT_ERR_INVALID, "loss node out of range");
    const size_t nfwd = static_cast<size_t>(loss) + 1;  // nodes after the loss cannot reach it
    Builder b{g};
    std::unordered_map<int, int> grads;
    auto accumulate = [&](int target, int contrib) {
        auto it = grads.find(target);
        if (it == grads.end())
            grads[target] = contrib;
        else
            it->second = b.mk(TT_OP_ADD, {it->second, contrib});
    };

    // Seed dL/dL = ones(loss.shape) (gradient.cpp:131).
    {
        int one = b.scalar(1.0f, b.dtype(loss));
        grads[loss] = b.view(TT_OP_EXPAND, one, b.shape(loss));
    }

    for (size_t ii = nfwd; ii-- > 0;) {
        int i = static_cast<int>(ii);
        auto git = grads.find(i);
        if (git == grads.end()) continue;
        const int gidx = git->second;
        const Node n = g.nodes[ii];  // copy: g.nodes grows below
        const int dt = n.dtype;
        switch (n.op) {
            case TT_OP_INPUT:
            case TT_OP_CONSTANT:
            case TT_OP_STEP:
                break;
            case TT_OP_ADD:
                accumulate(n.in[0], b.unbroadcast(gidx, b.shape(n.in[0])));
                accumulate(n.in[1], b.unbroadcast(gidx, b.shape(n.in[1])));
                break;
            case TT_OP_SUB: {
                accumulate(n.in[0], b.unbroadcast(gidx, b.shape(n.in[0])));
                int neg = b.mk(TT_OP_MUL, {gidx, b.scalar(-1.0f, dt)});
                accumulate(n.in[1], b.unbroadcast(neg, b.shape(n.in[1])));
                break;
            }
            case TT_OP_MUL: {
                int ga = b.mk(TT_OP_MUL, {gidx, n.in[1]});
                int gb = b.mk(TT_OP_MUL, {gidx, n.in[0]});
                accumulate(n.in[0], b.unbroadcast(ga, b.shape(n.in[0])));
                accumulate(n.in[1], b.unbroadcast(gb, b.shape(n.in[1])));
                break;
            }
            case TT_OP_DIV: {
                int ga = b.mk(TT_OP_DIV, {gidx, n.in[1]});
                accumulate(n.in[0], b.unbroadcast(ga, b.shape(n.in[0])));
                int bsq = b.mk(TT_OP_MUL, {n.in[1], n.in[1]});
                int negg = b.mk(TT_OP_MUL, {gidx, b.scalar(-1.0f, dt)});
                int negga = b.mk(TT_OP_MUL, {negg, n.in[0]});
                int gb = b.mk(TT_OP_DIV, {negga, bsq});
                accumulate(n.in[1], b.unbroadcast(gb, b.shape(n.in[1])));
                break;
            }
            case TT_OP_RELU: {
                int mask = b.mk(TT_OP_STEP, {n.in[0]});
                accumulate(n.in[0], b.mk(TT_OP_MUL, {gidx, mask}));
                break;
            }
            case TT_OP_SIGMOID: {
                int oms = b.mk(TT_OP_SUB, {b.view(TT_OP_EXPAND, b.scalar(1.0f, dt), n.shape), i});
                int ds = b.mk(TT_OP_MUL, {i, oms});
                accumulate(n.in[0], b.mk(TT_OP_MUL, {gidx, ds}));
                break;
            }
            case TT_OP_EXP:
                accumulate(n.in[0], b.mk(TT_OP_MUL, {gidx, i}));
                break;
            case TT_OP_NEG:
                accumulate(n.in[0], b.mk(TT_OP_NEG, {gidx}));
                break;
            case TT_OP_TANH: {
                int tt = b.mk(TT_OP_MUL, {i, i});
                int om = b.mk(TT_OP_SUB, {b.view(TT_OP_EXPAND, b.scalar(1.0f, dt), n.shape), tt});
                accumulate(n.in[0], b.mk(TT_OP_MUL, {gidx, om}));
                break;
            }
            case TT_OP_MATMUL: {
                int bt = b.transpose(n.in[1], -2, -1);
                int at = b.transpose(n.in[0], -2, -1);
                int ga = b.mk(TT_OP_MATMUL, {gidx, bt});
                int gb = b.mk(TT_OP_MATMUL, {at, gidx});
                accumulate(n.in[0], b.unbroadcast(ga, b.shape(n.in[0])));
                accumulate(n.in[1], b.unbroadcast(gb, b.shape(n.in[1])));
                break;
            }
            case TT_OP_TRANSPOSE:
                accumulate(n.in[0], b.transpose(gidx, n.dim0, n.dim1));
                break;
            case TT_OP_RESHAPE:
                accumulate(n.in[0], b.view(TT_OP_RESHAPE, gidx, b.shape(n.in[0])));
                break;
            case TT_OP_EXPAND:
                accumulate(n.in[0], b.unbroadcast(gidx, b.shape(n.in[0])));
                break;
            case TT_OP_REDUCE_SUM: {
                const Shape ash = b.shape(n.in[0]);
                int gs = n.keepdims ? gidx : b.view(TT_OP_RESHAPE, gidx, b.kept_shape(n, ash));
                accumulate(n.in[0], b.view(TT_OP_EXPAND, gs, ash));
                break;
            }
            case TT_OP_REDUCE_MEAN: {
                const Shape ash = b.shape(n.in[0]);
                int64_t gn = numel(b.shape(gidx));
                int64_t nred = numel(ash) / (gn > 0 ? gn : 1);
                if (nred <= 0) nred = 1;
                float factor = static_cast<float>(1.0 / static_cast<double>(nred));
                int scaled = b.mk(TT_OP_MUL, {gidx, b.scalar(factor, dt)});
                int gs = n.keepdims ? scaled : b.view(TT_OP_RESHAPE, scaled, b.kept_shape(n, ash));
                accumulate(n.in[0], b.view(TT_OP_EXPAND, gs, ash));
                break;
            }
            case TT_OP_REDUCE_MAX:
                fail(TT_ERR_COMPILE, "reduce_max has no gradient in this backend");
            default:
                fail(TT_ERR_COMPILE, std::string("Unsupported op in backward pass: ") + op_name(n.op));
        }
    }

    for (int w : wrt) {
        if (w < 0 || static_cast<size_t>(w) >= nfwd) fail(TT_ERR_INVALID, "gradient target out of range");
        auto it = grads.find(w);
        int out;
        if (it != grads.end()) {
            out = it->second;
        } else {
            out = b.view(TT_OP_EXPAND, b.scalar(0.0f, b.dtype(w)), b.shape(w));
        }
        // A gradient that is just a view of the seed or another value is still a
        // separate output buffer; the scheduler materialises views that are outputs.
        if (std::find(g.outputs.begin(), g.outputs.end(), out) != g.outputs.end() || out == w)
            out = b.view(TT_OP_RESHAPE, out, Shape{-1});  // placeholder fixed below
        g.outputs.push_back(out);
    }
    // Replace placeholders (reshape to [-1]) by a reshape to the node's own shape, which
    // the scheduler treats as a copy when the node is an output.
    for (int& o : g.outputs) {
        Node& n = g.nodes[static_cast<size_t>(o)];
        if (n.op == TT_OP_RESHAPE && n.shape.size() == 1 && n.shape[0] == -1)
            n.shape = g.nodes[static_cast<size_t>(n.in[0])].shape;
    }
}

}  // namespace ttb
