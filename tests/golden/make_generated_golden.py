"""Generated-model fixtures from the reference's own graph interpreter.

Run in a container where the reference checkout is available; the fixtures
(tests/golden/generated_*.npz) are committed, so the tests never need the
reference:

  python tests/golden/make_generated_golden.py /path/to/ponni-reference

For each network below the script builds the reference generator's canonical
graph directly (its IR classes, src/generator/kokkos_nn/ir.py: Graph, Node,
TensorValue, ConstantTensor; the ONNX importer is not needed) with the fused
node kinds the generator's passes produce -- DenseBiasActivation, Dense,
DenseResidualActivation and LayerNormalization -- and evaluates it with the
reference's verification interpreter (kokkos_nn.interpreter.run_graph,
src/generator/kokkos_nn/interpreter.py:430) on seeded inputs, in float64 and
in float32.  Each fixture holds the node list (JSON), the parameters
(W [out, in], bias, LayerNorm scale / bias), the inputs [features, batch] and
both outputs.
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, input width, nodes): node = (op, name, out width, activation, residual)
NETWORKS = [
    ("dense_silu", 10, [("DenseBiasActivation", "fc1", 32, "Silu", None),
                        ("DenseBiasActivation", "fc2", 32, "Silu", None),
                        ("Dense", "fc3", 6, None, None)]),
    ("layernorm", 12, [("Dense", "fc1", 48, None, None),
                       ("LayerNormalization", "ln1", 48, None, None),
                       ("DenseBiasActivation", "fc2", 48, "Gelu", None),
                       ("Dense", "fc3", 5, None, None)]),
    ("residual", 8, [("DenseBiasActivation", "fc1", 24, "Relu", None),
                     ("DenseResidualActivation", "fc2", 24, "Tanh", "fc1"),
                     ("DenseResidualActivation", "fc3", 24, "Silu", "fc2"),
                     ("LayerNormalization", "ln1", 24, None, None),
                     ("Dense", "fc4", 3, None, None)]),
    ("residual_input", 16, [("DenseResidualActivation", "fc1", 16, "Relu", "input"),
                            ("LayerNormalization", "ln1", 16, None, None),
                            ("Dense", "fc2", 4, None, None)]),
]
BATCH = 300


def build_graph(kn, nin, nodes, params, np_dtype):
    from kokkos_nn.ir import ConstantTensor, DType, Graph, Node, Symbol, TensorValue

    dt = DType.FLOAT64 if np_dtype == np.float64 else DType.FLOAT32
    batch = Symbol("batch")
    tensors, graph_nodes, constants = {}, [], {}

    def tensor(name, shape, const=None):
        tid = len(tensors)
        tensors[tid] = TensorValue(tid, name, shape, dt, is_constant=const is not None, constant_name=const)
        return tid

    def constant(name):
        v = params[name].astype(np_dtype)
        constants[name] = ConstantTensor(name, tuple(v.shape), dt, v, learned=True)
        return tensor(name, tuple(v.shape), name)

    x = tensor("input", (batch, nin))
    tensors[x].is_input = True
    ids = {"input": x}
    cur = x
    for op, name, nout, act, residual in nodes:
        if op == "LayerNormalization":
            inputs = [cur, constant(f"{name}.scale"), constant(f"{name}.bias")]
            attrs = {"epsilon": 1e-5}
        else:
            inputs = [cur]
            attrs = {"weight": constant(f"{name}.weight"), "bias": constant(f"{name}.bias")}
            if act is not None:
                attrs["activation"] = act
            if residual is not None:
                attrs["residual"] = ids[residual]
        out = tensor(name, (batch, nout))
        graph_nodes.append(Node(len(graph_nodes), op, inputs, [out], attrs, source_name=name))
        ids[name] = out
        cur = out
    tensors[cur].is_output = True
    g = Graph(inputs=[x], outputs=[cur], tensors=tensors, nodes=graph_nodes, constants=constants,
              metadata={"fixture": kn})
    g.rebuild_links()
    return g


def make_params(rng, nin, nodes):
    params, width = {}, nin
    for op, name, nout, _, _ in nodes:
        if op == "LayerNormalization":
            params[f"{name}.scale"] = rng.normal(1.0, 0.2, nout)
            params[f"{name}.bias"] = rng.normal(0.0, 0.2, nout)
        else:
            params[f"{name}.weight"] = rng.normal(0.0, 1.0 / np.sqrt(width), (nout, width))
            params[f"{name}.bias"] = rng.normal(0.0, 0.1, nout)
        width = nout
    return params


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("PONNI_REFERENCE", "")
    if not ref or not os.path.isdir(ref):
        raise SystemExit("usage: make_generated_golden.py <reference checkout>")
    sys.path.insert(0, os.path.join(ref, "src", "generator"))
    from kokkos_nn.interpreter import run_graph

    for i, (kn, nin, nodes) in enumerate(NETWORKS):
        rng = np.random.default_rng(4321 + i)
        params = make_params(rng, nin, nodes)
        x = rng.normal(0.0, 1.0, (nin, BATCH))
        # parameters and inputs are first rounded to float32, so that both
        # evaluations see the same values
        params = {k: v.astype(np.float32).astype(np.float64) for k, v in params.items()}
        x = x.astype(np.float32).astype(np.float64)
        y64 = run_graph(build_graph(kn, nin, nodes, params, np.float64), x)
        y32 = run_graph(build_graph(kn, nin, nodes, params, np.float32), x.astype(np.float32))
        spec = [{"op": op, "name": name, "nout": nout, "activation": act, "residual": res}
                for op, name, nout, act, res in nodes]
        np.savez_compressed(os.path.join(HERE, f"generated_{kn}.npz"), spec=np.array(json.dumps(spec)),
                            x=x, y64=y64, y32=y32.astype(np.float32),
                            **{f"param:{k}": v for k, v in params.items()})
        print(f"generated_{kn}.npz: {nin} -> {y64.shape[0]}, {len(nodes)} nodes, batch {BATCH}")


if __name__ == "__main__":
    main()
