"""Generates tests/golden/*.npz from the reference TinyTensor itself.

Run here, where the reference sources exist (the GPU machine only reads the .npz):
    make -C oracle ref && python tests/golden/make_golden.py

For every case of tests/golden/cases.py this records the seeded inputs and the
outputs of the reference's Interpreter with optimize=False (the path whose
reductions accumulate in double and which has no fusion miscompile), computed by
oracle/_ref/libttref.so (the reference's own sources, compiled by oracle/Makefile).
Gradient cases record Autodiff::compute_gradients.  Cases with ops the reference
lacks (exp, tanh, neg) run through reference-op identities; reduce_max has no
reference form and its golden values come from numpy.max, an independent
implementation.  The reference IR text (IRPrinter::to_string) is stored too.
"""

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))
sys.path.insert(0, HERE)

from cases import CASES, build  # noqa: E402

from oracle.oracle import REDUCE_MAX, Reference  # noqa: E402


def _numpy_reduce_max(graph, feed, outs):
    vals = {n.index: feed[n] for n in graph.inputs}
    res = []
    for n in graph.nodes:
        if n.index in vals:
            continue
        x = vals[n.inputs[0].index]
        if n.op == 9:
            vals[n.index] = np.swapaxes(x, n.dim0, n.dim1)
        elif n.op == REDUCE_MAX:
            ax = tuple(a % x.ndim for a in n.axes) if n.axes else None
            vals[n.index] = np.max(x, axis=ax, keepdims=n.keepdims).astype(np.float32)
    for o in outs:
        res.append(np.asarray(vals[o.index], dtype=np.float32))
    return res


def main():
    ref = Reference()
    for name in CASES:
        c = build(name)
        g, feed = c["graph"], c["feed"]
        data = {}
        for i, n in enumerate(g.inputs):
            data[f"in{i}"] = np.asarray(feed[n], dtype=np.float32)
        if c["kind"] == "forward":
            if name == "reduce_max":
                outs = _numpy_reduce_max(g, feed, c["outputs"])
            else:
                for o in c["outputs"]:
                    g.mark_output(o)
                outs = ref.run(g, feed, mode="interpreted", optimize=False)
                if c["ref_ok"]:
                    data["ir"] = np.array(ref.ir(g))
        else:
            outs = ref.gradients(g, c["loss"], feed, c["wrt"])
        for i, o in enumerate(outs):
            data[f"out{i}"] = o
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **data)
        print(f"{name}: {len(outs)} outputs")


if __name__ == "__main__":
    main()
