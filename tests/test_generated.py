"""Generated-model arithmetic (ARITH_GENERATED) and the GeneratedModel
mirror of the reference's generated struct (emitter.py:693-735, :967-1010,
:1724-1955): dense sums start at the bias, 16-bit products are fused
multiply-adds, weights are [out, in]."""
import os

import numpy as np
import pytest

import ponni_b200 as pb
from oracle import oracle
from tests import kat_models as K


def dense_chain(rng, dims=(6, 9, 7, 3), acts=("silu", "relu", None)):
    out = []
    for i in range(len(dims) - 1):
        w = rng.normal(0, 1 / np.sqrt(dims[i]), (dims[i + 1], dims[i]))
        b = rng.normal(0, 0.2, dims[i + 1]) if i != 1 else None  # one layer without bias
        out.append(pb.Dense(f"fc{i}", w, b, acts[i]))
    return out


def numpy_generated(dense, x, dtype):
    """Direct restatement of the emitted loops: sum = b(i); sum += W(i,j) * x(j)."""
    if dtype == pb.F16:
        cur = x.astype(np.float16)
        for d in dense:
            w = d.weight.astype(np.float16)
            nxt = np.empty((w.shape[0], cur.shape[1]), np.float16)
            for i in range(w.shape[0]):
                s = (d.bias.astype(np.float16)[i] if d.bias is not None else np.float16(0)) * np.ones(cur.shape[1], np.float16)
                for j in range(w.shape[1]):  # one rounding per fused multiply-add
                    s = (w[i, j].astype(np.float64) * cur[j].astype(np.float64) + s.astype(np.float64)).astype(np.float16)
                nxt[i] = s
            cur = act_np(d.activation, nxt.astype(np.float32)).astype(np.float16)
        return cur
    cur = x.astype(np.float64)
    for d in dense:
        s = d.weight @ cur + (d.bias[:, None] if d.bias is not None else 0.0)
        cur = act_np(d.activation, s)
    return cur


def act_np(a, v):
    if a is None:
        return v
    if a == "relu":
        return np.maximum(v, 0)
    if a == "silu":
        return v / (1 + np.exp(-v))
    raise ValueError(a)


def test_oracle_generated_fp64_closed_form():
    rng = np.random.default_rng(1)
    dense = dense_chain(rng)
    x = rng.normal(0, 1, (6, 50))
    layers = pb.GeneratedModel(dense, np.float64)._layer_list(dense)
    y = oracle.forward(layers, pb.F64, x, generated=True)
    assert np.max(np.abs(y - numpy_generated(dense, x, pb.F64))) <= 1e-12


def test_oracle_generated_half_fused():
    rng = np.random.default_rng(2)
    dense = dense_chain(rng)
    x = rng.normal(0, 1, (6, 40))
    layers = pb.GeneratedModel(dense)._layer_list(dense)
    y = pb.from_dtype_bytes(oracle.forward(layers, pb.F16, pb.to_dtype_bytes(x, pb.F16), generated=True), pb.F16)
    ref = numpy_generated(dense, x, pb.F16).astype(np.float32)
    assert np.max(np.abs(y - ref)) <= 2e-3 * np.max(np.abs(ref))  # transcendental rounding may differ by a unit


def test_generated_parameters_round_trip():
    rng = np.random.default_rng(3)
    g = pb.GeneratedModel(dense_chain(rng))
    n = g.get_num_parameters()
    assert n == 6 * 9 + 9 + 9 * 7 + 7 * 3 + 3
    v = g.get_parameters()
    g.set_parameters(v[::-1].copy())
    assert np.array_equal(g.get_parameters(), v[::-1])
    with pytest.raises(pb.PonniError):
        g.set_parameters(v[:-1])
    bad = v.copy()
    bad[0] = np.nan
    with pytest.raises(pb.PonniError):
        g.set_parameters(bad)


def test_generated_trainable_order():
    """Generated order (W[out, in], then bias) -> Inference tuple order
    (Matvec W[in][out], then Bias): the permutation device updates use."""
    rng = np.random.default_rng(4)
    g = pb.GeneratedModel(dense_chain(rng))
    perm = g._trainable_order()
    want = np.concatenate([L.parameters().reshape(-1) for L in g._layer_list(g.dense)
                           if L.get_num_trainable_parameters()])
    assert np.array_equal(g.get_parameters().astype(np.float64)[perm], want.astype(np.float32).astype(np.float64))
    assert np.array_equal(np.sort(perm), np.arange(g.get_num_parameters()))


def test_generated_half_mirror_rounds_through_scalar():
    """The fp16 mirror is fp16(float(Scalar value)) (emitter.py:1742-1743)."""
    g = pb.GeneratedModel([pb.Dense("a", np.zeros((1, 1)))], np.float64)
    v = np.array([1.0 + 2.0 ** -11 + 2.0 ** -40])  # a tie for fp16 only after rounding to float
    assert g._mirror_values(v)[0] == np.float32(v[0])


def test_generated_load_named_weights():
    """Named tensors of a .ponni file (the reference-generated pytorch_resnet
    fixture) load by name, shape-checked."""
    path = os.path.join(K.GOLDEN, "pytorch_resnet.ponni")
    for i in range(1, 6):
        t = K.read_tensor(path, f"fc{i}.weight").astype(np.float64)
        g = pb.GeneratedModel([pb.Dense(f"fc{i}", np.zeros(t.shape))])
        g.load_weights(path)
        assert np.array_equal(g.dense[0].weight, t)
    g = pb.GeneratedModel([pb.Dense("fc1", np.zeros((3, 3)))])
    with pytest.raises(pb.PonniError):
        g.load_weights(path)  # wrong shape


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [pb.F32, pb.F64, pb.F16, pb.BF16])
def test_gpu_generated_arithmetic(dtype):
    import torch
    from tests.test_gpu_parity import check, from_torch, to_torch
    rng = np.random.default_rng(4)
    dense = dense_chain(rng, dims=(12, 40, 33, 5))
    layers = pb.GeneratedModel(dense)._layer_list(dense)
    m = pb.Inference(layers, dtype=dtype, arithmetic=pb._abi.ARITH_GENERATED)
    assert m.kernel() == pb._abi.KERNEL_TILE
    x = pb.to_dtype_bytes(rng.normal(0, 1, (12, 3001)), dtype)
    y = from_torch(m.forward_batch_parallel(to_torch(x, dtype).cuda()), dtype)
    torch.cuda.synchronize()
    check(y, oracle.forward(layers, dtype, x, generated=True), dtype, layers, x)


@pytest.mark.gpu
def test_gpu_generated_model_api():
    rng = np.random.default_rng(5)
    dense = dense_chain(rng, dims=(12, 40, 33, 5))
    g = pb.GeneratedModel(dense)
    x = rng.normal(0, 1, (12, 2000)).astype(np.float32)
    layers = g._layer_list(dense)
    y = g.infer_batch(x)
    ref = oracle.forward(layers, pb.F32, x, generated=True)
    assert K.normwise_err(y, ref) <= 1e-5
    yh = g.infer_batch_half2(x)
    refh = pb.from_dtype_bytes(oracle.forward(layers, pb.F16, pb.to_dtype_bytes(x, pb.F16), generated=True), pb.F16)
    assert yh.dtype == np.float32 and K.normwise_err(yh, refh) <= 2e-3
    assert np.allclose(g.infer_one(x[:, 7]), y[:, 7], rtol=1e-6, atol=1e-7)


# ---- pinned to the reference's own graph interpreter -------------------------
# tests/golden/generated_*.npz come from tests/golden/make_generated_golden.py:
# canonical graphs of the reference generator's IR (DenseBiasActivation, Dense,
# DenseResidualActivation, LayerNormalization) evaluated by the reference's
# kokkos_nn.interpreter.run_graph in float64 and float32.

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
FIXTURES = ["dense_silu", "layernorm", "residual", "residual_input"]


def load_fixture(name):
    import json
    z = np.load(os.path.join(GOLDEN, f"generated_{name}.npz"))
    spec = json.loads(str(z["spec"]))
    p = {k[len("param:"):]: z[k] for k in z.files if k.startswith("param:")}
    nodes = []
    for n in spec:
        if n["op"] == "LayerNormalization":
            nodes.append(pb.GeneratedLayerNorm(n["name"], p[n["name"] + ".scale"], p[n["name"] + ".bias"], 1e-5))
        else:
            act = n["activation"].lower() if n["activation"] else None
            nodes.append(pb.Dense(n["name"], p[n["name"] + ".weight"], p[n["name"] + ".bias"], act,
                                  residual=n["residual"]))
    return nodes, z["x"], z["y64"], z["y32"]


@pytest.mark.parametrize("name", FIXTURES)
def test_oracle_generated_matches_reference_interpreter(name):
    """The oracle's generated arithmetic (Welford LayerNorm, bias-first sums,
    residual before the activation) reproduces the reference interpreter."""
    nodes, x, y64, y32 = load_fixture(name)
    layers = pb.GeneratedModel(nodes, np.float64)._layer_list(nodes)
    o64 = oracle.forward(layers, pb.F64, x, generated=True)
    assert K.normwise_err(o64, y64) <= 1e-12
    o32 = oracle.forward(layers, pb.F32, x.astype(np.float32), generated=True)
    assert K.normwise_err(o32, y64) <= 1e-5
    assert K.normwise_err(o32, y32) <= 1e-5


def test_generated_model_structure_checks():
    rng = np.random.default_rng(9)
    a = pb.Dense("a", rng.normal(0, 1, (8, 4)), np.zeros(8), "relu")
    with pytest.raises(ValueError):  # residual of another width
        pb.GeneratedModel([a, pb.Dense("b", rng.normal(0, 1, (8, 8)), None, None, residual="input")])
    with pytest.raises(ValueError):  # residual that is not earlier
        pb.GeneratedModel([a, pb.Dense("b", rng.normal(0, 1, (8, 8)), None, None, residual="c")])
    g = pb.GeneratedModel([a, pb.GeneratedLayerNorm("ln", np.ones(8), np.zeros(8)),
                           pb.Dense("b", rng.normal(0, 1, (8, 8)), np.zeros(8), "tanh", residual="a")])
    assert g.get_num_parameters() == 8 * 4 + 8 + 16 + 64 + 8
    kinds = [type(l).__name__ for l in g._layer_list(g.dense)]
    assert kinds == ["Matvec", "Bias", "Relu", "Save_State", "LayerNorm", "Matvec", "Bias", "Binop_Add", "Tanh"]


@pytest.mark.gpu
@pytest.mark.parametrize("name", FIXTURES)
def test_generated_model_gpu_matches_reference_interpreter(name):
    """GeneratedModel.infer_batch (float and double) and infer_batch_half2 on
    the GPU against the reference interpreter's outputs and the oracle's
    generated arithmetic."""
    nodes, x, y64, y32 = load_fixture(name)
    g64 = pb.GeneratedModel([_copy(n) for n in nodes], np.float64)
    layers = g64._layer_list(g64.dense)
    assert K.normwise_err(g64.infer_batch(x), oracle.forward(layers, pb.F64, x, generated=True)) <= 1e-12
    assert K.normwise_err(g64.infer_batch(x), y64) <= 1e-12
    g32 = pb.GeneratedModel([_copy(n) for n in nodes], np.float32)
    y = g32.infer_batch(x.astype(np.float32))
    assert K.normwise_err(y, oracle.forward(layers, pb.F32, x.astype(np.float32), generated=True)) <= 1e-5
    assert K.normwise_err(y, y64) <= 1e-5
    yh = g32.infer_batch_half2(x.astype(np.float32))
    half_layers = g32._layer_list(g32.dense, g32._mirror_values)
    oh = pb.from_dtype_bytes(oracle.forward(half_layers, pb.F16, pb.to_dtype_bytes(x, pb.F16), generated=True), pb.F16)
    assert K.normwise_err(yh, oh) <= 2e-3
    assert K.normwise_err(yh, y64) <= 3e-2  # fp16 storage and fp16 accumulation


def _copy(n):
    import copy
    return copy.deepcopy(n)
