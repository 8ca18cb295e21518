"""Parameter updates of planned models on the GPU (device images rewritten in
place, no re-plan).

Every update path must leave the model bit-identical to a model planned from
scratch with the same parameters: the outputs of one forward are compared
bit for bit, on every kernel (tile, narrow, specialised narrow, resident and
streamed tensor-core, generated arithmetic).  The device check
(parameters_synchronized / parameters_are_finite, reference
src/generator/kokkos_nn/emitter.py:1868-1895) must report no disagreement
after each update.
"""
import numpy as np
import pytest

import ponni_b200 as pb
from ponni_b200 import configs
from tests.test_gpu_parity import all_kinds_model, to_torch

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

A = pb._abi
BATCH = 777


def _cfg_layers(name):
    return configs.ALL[name](batch=8).layers


def _mixed_trainable(rng):
    # a frozen layer in the middle: its values stay as planned
    return [pb.Matvec(rng.normal(0, 0.3, (20, 48))), pb.Bias(rng.normal(0, 0.1, 48)), pb.Relu(48),
            pb.Matvec(rng.normal(0, 0.2, (48, 48)), trainable=False), pb.Bias(rng.normal(0, 0.1, 48)),
            pb.Tanh(48), pb.Matvec(rng.normal(0, 0.2, (48, 7)))]


# name -> (layers factory, dtype, arithmetic, expected kernel, env)
CASES = {
    "tile_all_kinds_f32": (lambda r: all_kinds_model(r), pb.F32, None, A.KERNEL_TILE, {}),
    "tile_all_kinds_f64": (lambda r: all_kinds_model(r), pb.F64, None, A.KERNEL_TILE, {}),
    "tile_all_kinds_bf16": (lambda r: all_kinds_model(r), pb.BF16, None, A.KERNEL_TILE, {}),
    "tile_generated_f16": (lambda r: _cfg_layers("cfg3"), pb.F16, A.ARITH_GENERATED, A.KERNEL_TILE, {}),
    "narrow_specialised": (lambda r: _cfg_layers("cfg1"), pb.F32, None, A.KERNEL_NARROW_JIT, {}),
    "narrow_generic": (lambda r: _cfg_layers("cfg1"), pb.F32, None, A.KERNEL_NARROW,
                       {"PONNI_B200_NARROW_JIT": "0"}),
    "tensor_f32_split": (lambda r: _cfg_layers("cfg2"), pb.F32, None, A.KERNEL_TENSOR, {}),
    "tensor_f32_frozen_layer": (_mixed_trainable, pb.F32, None, A.KERNEL_TENSOR, {}),
    "tensor_resid_cfg4": (lambda r: _cfg_layers("cfg4"), pb.F32, None, A.KERNEL_TENSOR_RESID, {}),
    "tensor_f16": (lambda r: _cfg_layers("cfg3"), pb.F16, A.ARITH_TENSOR, A.KERNEL_TENSOR, {}),
    "tensor_streamed_bf16": (lambda r: _cfg_layers("cfg5"), pb.BF16, A.ARITH_TENSOR, A.KERNEL_TENSOR_STREAM, {}),
    "tensor_streamed_f16": (lambda r: _cfg_layers("cfg3"), pb.F16, A.ARITH_TENSOR, A.KERNEL_TENSOR_STREAM,
                            {"PONNI_B200_TC_STREAM": "1"}),
}


def _setup(name, monkeypatch):
    make_layers, dtype, arith, kernel, env = CASES[name]
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    rng = np.random.default_rng(5)
    layers = make_layers(rng)
    nin = layers[0].num_inputs
    x = to_torch(pb.to_dtype_bytes(rng.normal(0, 1, (nin, BATCH)), dtype), dtype).cuda()
    return layers, dtype, arith, kernel, x, rng


def _model(layers, dtype, arith):
    return pb.Inference(layers, dtype=dtype, arithmetic=arith)


def _fwd(m, x):
    y = m.forward_batch_parallel(x).clone()
    torch.cuda.synchronize()
    return y


def _fresh(layers, dtype, arith, values, x, monkeypatch):
    """A model planned from scratch with `values` (the slow path)."""
    monkeypatch.setenv("PONNI_B200_PARAM_SCATTER", "0")
    m = _model(layers, dtype, arith)
    m.set_trainable_parameters(values)
    y = _fwd(m, x)
    monkeypatch.delenv("PONNI_B200_PARAM_SCATTER")
    return y


def _bits_equal(a, b):
    if a.dtype == torch.bfloat16 or a.dtype == torch.float16:
        return torch.equal(a.view(torch.int16), b.view(torch.int16))
    if a.dtype == torch.float32:
        return torch.equal(a.view(torch.int32), b.view(torch.int32))
    return torch.equal(a.view(torch.int64), b.view(torch.int64))


def _canonical(values64, dtype):
    """The model dtype's value of each update value (fp64 kept, others via fp32)."""
    v = np.asarray(values64, dtype=np.float64)
    if dtype != pb.F64:
        v = v.astype(np.float32).astype(np.float64)
    return pb.from_dtype_bytes(pb.to_dtype_bytes(v, dtype), dtype)


@pytest.mark.parametrize("name", sorted(CASES))
def test_host_update_matches_fresh_plan(name, monkeypatch):
    layers, dtype, arith, kernel, x, rng = _setup(name, monkeypatch)
    m = _model(layers, dtype, arith)
    assert m.kernel() == kernel
    _fwd(m, x)
    n = m.get_num_trainable_parameters()
    for it in range(2):  # two updates back to back: the pinned staging buffer is reused
        vals = rng.normal(0, 0.25, n)
        m.set_trainable_parameters(vals)
        y = _fwd(m, x)
        assert m.kernel() == kernel
        assert _bits_equal(y, _fresh(layers, dtype, arith, vals, x, monkeypatch)), f"update {it}"
        assert m.check_parameters() == (0, 0)
        np.testing.assert_array_equal(m.get_trainable_parameters(),
                                      pb.from_dtype_bytes(pb.to_dtype_bytes(vals, dtype), dtype))


SRC_TYPES = [torch.float32, torch.float64, torch.float16, torch.bfloat16]


@pytest.mark.parametrize("src", SRC_TYPES, ids=lambda t: str(t).replace("torch.", ""))
@pytest.mark.parametrize("name", sorted(CASES))
def test_device_update_matches_fresh_plan(name, src, monkeypatch):
    layers, dtype, arith, kernel, x, rng = _setup(name, monkeypatch)
    m = _model(layers, dtype, arith)
    _fwd(m, x)
    n = m.get_num_trainable_parameters()
    vals = torch.from_numpy(rng.normal(0, 0.25, n)).to(src).cuda()
    m.set_trainable_parameters_device(vals)
    y = _fwd(m, x)
    want = _canonical(vals.double().cpu().numpy(), dtype)
    assert m.check_parameters() == (0, 0)
    dev = m.get_trainable_parameters_device(torch.float64).cpu().numpy()
    np.testing.assert_array_equal(dev, want)
    assert _bits_equal(y, _fresh(layers, dtype, arith, want, x, monkeypatch))
    # the host copy is read back on demand
    np.testing.assert_array_equal(m.get_trainable_parameters(), want)


@pytest.mark.parametrize("name", ["tensor_f32_split", "narrow_specialised", "tile_all_kinds_f32",
                                  "tensor_streamed_bf16"])
def test_device_update_on_a_side_stream(name, monkeypatch):
    layers, dtype, arith, kernel, x, rng = _setup(name, monkeypatch)
    m = _model(layers, dtype, arith)
    _fwd(m, x)
    n = m.get_num_trainable_parameters()
    s = torch.cuda.Stream()
    outs, sets = [], []
    with torch.cuda.stream(s):
        for _ in range(3):  # update, forward, update, forward ... all queued on s
            v = torch.randn(n, dtype=torch.float64, device="cuda") * 0.25
            sets.append(v)
            m.set_trainable_parameters_device(v)
            outs.append(m.forward_batch_parallel(x).clone())
    s.synchronize()
    for v, y in zip(sets, outs):
        want = _canonical(v.cpu().numpy(), dtype)
        assert _bits_equal(y, _fresh(layers, dtype, arith, want, x, monkeypatch))


@pytest.mark.parametrize("name", ["tensor_f32_split", "tile_all_kinds_f64", "tensor_f16"])
def test_nonfinite_values_are_counted(name, monkeypatch):
    layers, dtype, arith, kernel, x, rng = _setup(name, monkeypatch)
    m = _model(layers, dtype, arith)
    m.kernel()
    n = m.get_num_trainable_parameters()
    v = torch.from_numpy(rng.normal(0, 0.25, n)).cuda()
    v[[0, n // 2, n - 1]] = torch.tensor([float("nan"), float("inf"), -float("inf")], dtype=v.dtype, device="cuda")
    m.set_trainable_parameters_device(v)
    mism, nonfinite = m.check_parameters()
    assert (mism, nonfinite) == (0, 3)
    assert not m.parameters_are_finite() and m.parameters_synchronized()
    m.set_trainable_parameters(np.zeros(n))
    assert m.parameters_are_finite()


def test_load_weights_into_planned_model(tmp_path, monkeypatch):
    layers, dtype, arith, kernel, x, rng = _setup("tensor_f32_split", monkeypatch)
    src = _model(layers, dtype, arith)
    vals = rng.normal(0, 0.25, src.get_num_trainable_parameters())
    src.set_trainable_parameters(vals)
    ok, err = src.save_weights(tmp_path / "w.ponni")
    assert ok, err
    m = _model(layers, dtype, arith)
    _fwd(m, x)
    ok, err = m.load_weights(tmp_path / "w.ponni")
    assert ok, err
    assert _bits_equal(_fwd(m, x), _fresh(layers, dtype, arith, _canonical(vals, dtype), x, monkeypatch))
    assert m.check_parameters() == (0, 0)


def test_arithmetic_change_after_device_update_keeps_values(monkeypatch):
    """A re-plan after a device update starts from the device values."""
    layers, dtype, arith, kernel, x, rng = _setup("tensor_f16", monkeypatch)
    m = _model(layers, dtype, A.ARITH_TENSOR)
    _fwd(m, x)
    v = torch.from_numpy(rng.normal(0, 0.25, m.get_num_trainable_parameters())).cuda()
    m.set_trainable_parameters_device(v)
    m.set_arithmetic(A.ARITH_REFERENCE)
    y = _fwd(m, x)
    assert m.kernel() == A.KERNEL_TILE
    want = _canonical(v.cpu().numpy(), dtype)
    assert _bits_equal(y, _fresh(layers, dtype, A.ARITH_REFERENCE, want, x, monkeypatch))


def _dense(rng, dims):
    out = []
    for i in range(len(dims) - 1):
        out.append(pb.Dense(f"l{i}", rng.normal(0, 1 / np.sqrt(dims[i]), (dims[i + 1], dims[i])),
                            rng.normal(0, 0.1, dims[i + 1]), "relu" if i + 2 < len(dims) else None))
    return out


@pytest.mark.parametrize("scalar", [np.float32, np.float64])
def test_generated_model_device_parameters(scalar):
    rng = np.random.default_rng(9)
    dims = [12, 40, 40, 3]
    g = pb.GeneratedModel(_dense(rng, dims), scalar=scalar)
    x = rng.normal(0, 1, (12, 300))
    g.infer_batch(x.astype(scalar))
    g.infer_batch_half2(x.astype(np.float32))  # creates the fp16 mirror
    p = torch.from_numpy(rng.normal(0, 0.2, g.get_num_parameters())).cuda()
    g.set_parameters_device(p)
    assert g.parameters_synchronized() and g.parameters_are_finite()
    y = g.infer_batch(x.astype(scalar))
    yh = g.infer_batch_half2(x.astype(np.float32))
    np.testing.assert_array_equal(g.get_parameters(), p.cpu().numpy().astype(scalar))
    np.testing.assert_array_equal(g.get_parameters_device().cpu().numpy(), p.cpu().numpy().astype(scalar))
    # a model built from the same values on the host
    ref = pb.GeneratedModel(_dense(rng, dims), scalar=scalar)
    ref.set_parameters(p.cpu().numpy())
    np.testing.assert_array_equal(y, ref.infer_batch(x.astype(scalar)))
    np.testing.assert_array_equal(yh, ref.infer_batch_half2(x.astype(np.float32)))
    # host update of a model with both mirrors planned
    q = rng.normal(0, 0.2, g.get_num_parameters())
    g.set_parameters(q)
    ref.set_parameters(q)
    assert g.parameters_synchronized()
    np.testing.assert_array_equal(g.infer_batch_half2(x.astype(np.float32)),
                                  ref.infer_batch_half2(x.astype(np.float32)))
