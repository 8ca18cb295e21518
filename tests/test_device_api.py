"""In-kernel device API (include/ponni_b200_device.cuh): an application
kernel evaluates the model one sample per thread through
forward_batch_parallel_in_kernel (tests/cuda/device_api_kernel.cu).  Results
are checked against the CPU oracle with the parity gates of the fused
kernels, and for fp32 / fp64 against the tile kernel, which runs the same
operations in the same order."""
import ctypes
import os

import numpy as np
import pytest

import ponni_b200 as pb
from ponni_b200 import configs
from tests import kat_models as K
from tests.test_gpu_parity import check, from_torch, to_torch

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

LIB = os.path.join(os.path.dirname(os.path.abspath(__file__)), "cuda", "libpb_device_api_test.so")


@pytest.fixture(scope="module")
def embedded():
    pb._abi.lib()  # the library the test kernel links against
    lib = ctypes.CDLL(LIB)
    f = lib.pb_test_embedded_forward
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64]
    return f


def run_embedded(fn, layers, dtype, x_raw, arithmetic=None):
    m = pb.Inference(layers, dtype=dtype, arithmetic=arithmetic)
    x = to_torch(x_raw, dtype).cuda()
    y = torch.empty((m.get_num_outputs(), x.shape[1]), dtype=x.dtype, device="cuda")
    rc = fn(m._m, x.data_ptr(), x.stride(0), y.data_ptr(), y.stride(0), x.shape[1])
    assert rc == 0, rc
    return from_torch(y, dtype)


def tile_forward(layers, dtype, x_raw, monkeypatch):
    monkeypatch.setenv("PONNI_B200_FORCE_TILE", "1")
    m = pb.Inference(layers, dtype=dtype, arithmetic=pb._abi.ARITH_REFERENCE)
    assert m.kernel() == pb._abi.KERNEL_TILE
    y = m.forward_batch_parallel(to_torch(x_raw, dtype).cuda())
    torch.cuda.synchronize()
    return from_torch(y, dtype)


NETS = {
    "readme": K.readme_mlp,
    "four_block": K.four_block,
    "softmax_mixed": K.softmax_mixed,
    "projection_add": K.projection_add_model,
    "pytorch_resnet": lambda: K.pytorch_resnet()[0],
    "cfg2": lambda: configs.cfg2(batch=1).layers,
    "cfg4": lambda: configs.cfg4(batch=1).layers,
}


@pytest.mark.parametrize("dtype", [pb.F32, pb.F64, pb.F16, pb.BF16])
@pytest.mark.parametrize("net", list(NETS))
def test_embedded_matches_oracle(net, dtype, embedded, oracle_lib, monkeypatch):
    layers = NETS[net]()
    rng = np.random.default_rng(17)
    nin = pb.Inference(layers, dtype=dtype).get_num_inputs()
    x = pb.to_dtype_bytes(rng.normal(0, 1, (nin, 1537)), dtype)
    y = run_embedded(embedded, layers, dtype, x)
    ref = oracle_lib.forward(layers, dtype, x)
    if net == "softmax_mixed":
        # one output is tanh(1 - 1) = 0 exactly: a relative norm would divide
        # rounding noise by zero, so this network is checked absolutely
        tol = {pb.F32: 1e-6, pb.F64: 1e-14, pb.F16: 4e-3, pb.BF16: 3e-2}[dtype]
        assert np.max(np.abs(K.as_float(y, dtype) - K.as_float(ref, dtype))) <= tol
    elif net == "cfg4" and dtype in (pb.F16, pb.BF16):
        # four LayerNorm/GELU residual blocks in per-operation 16-bit
        # arithmetic: a transcendental rounded one unit differently on the two
        # sides is amplified by the normalisations; gate at 8 units of the type
        tol = 8 * {pb.F16: 2.0 ** -11, pb.BF16: 2.0 ** -8}[dtype]
        assert K.normwise_err(K.as_float(y, dtype), K.as_float(ref, dtype)) <= tol
    else:
        check(y, ref, dtype, layers, x)
    if dtype in (pb.F32, pb.F64):
        t = tile_forward(layers, dtype, x, monkeypatch)
        assert K.normwise_err(y, t) <= (1e-6 if dtype == pb.F32 else 1e-14)


@pytest.mark.parametrize("dtype", [pb.F32, pb.F64, pb.F16])
@pytest.mark.parametrize("name", ["layernorm", "residual"])
def test_embedded_generated_arithmetic(name, dtype, embedded, oracle_lib):
    """A generated model (Welford LayerNorm, residual before the activation,
    bias-first sums) through the device API, against the oracle's generated
    arithmetic and the reference interpreter's fixture."""
    from tests.test_generated import load_fixture
    nodes, x, y64, _ = load_fixture(name)
    g = pb.GeneratedModel(nodes, np.float64 if dtype == pb.F64 else np.float32)
    layers = g._layer_list(g.dense, g._mirror_values if dtype == pb.F16 else (lambda a: a))
    xr = pb.to_dtype_bytes(x, dtype)
    y = K.as_float(run_embedded(embedded, layers, dtype, xr, pb._abi.ARITH_GENERATED), dtype)
    ref = K.as_float(oracle_lib.forward(layers, dtype, xr, generated=True), dtype)
    tol = {pb.F32: 1e-5, pb.F64: 1e-12, pb.F16: 2e-3}[dtype]
    assert K.normwise_err(y, ref) <= tol
    assert K.normwise_err(y, y64) <= {pb.F32: 1e-5, pb.F64: 1e-12, pb.F16: 3e-2}[dtype]


def test_embedded_golden_fixture(embedded):
    """The reference's pytorch_resnet fixture through the device API (abs 1e-5)."""
    layers, x, expected = K.pytorch_resnet()
    y = run_embedded(embedded, layers, pb.F32, np.ascontiguousarray(x.astype(np.float32)))
    assert np.max(np.abs(y - expected)) <= 1e-5


def device_params_ptr(m):
    prog, params = ctypes.c_void_p(), ctypes.c_void_p()
    maxw, nbuf = ctypes.c_int(), ctypes.c_int()
    assert pb._abi.lib().ponni_b200_model_device_program(m._m, ctypes.byref(prog), ctypes.byref(params),
                                                         ctypes.byref(maxw), ctypes.byref(nbuf)) == 0
    return params.value


def test_device_parameter_update_is_seen_by_application_kernels(embedded):
    """The device view points at the packed parameters, which parameter
    updates rewrite in place: the view's pointers stay valid and an
    application kernel sees the new values."""
    layers = configs.cfg2(batch=1).layers
    rng = np.random.default_rng(21)
    x_raw = rng.normal(0, 1, (30, 513)).astype(np.float32)
    m = pb.Inference(layers, dtype=pb.F32)
    x = to_torch(x_raw, pb.F32).cuda()
    y = torch.empty((m.get_num_outputs(), x.shape[1]), dtype=x.dtype, device="cuda")
    assert embedded(m._m, x.data_ptr(), x.stride(0), y.data_ptr(), y.stride(0), x.shape[1]) == 0
    v = rng.normal(0, 0.2, m.get_num_trainable_parameters())
    before = device_params_ptr(m)
    m.set_trainable_parameters_device(torch.from_numpy(v).cuda())
    torch.cuda.synchronize()
    assert device_params_ptr(m) == before
    assert embedded(m._m, x.data_ptr(), x.stride(0), y.data_ptr(), y.stride(0), x.shape[1]) == 0
    fresh = pb.Inference(layers, dtype=pb.F32)
    fresh.set_trainable_parameters(v)
    y2 = torch.empty_like(y)
    assert embedded(fresh._m, x.data_ptr(), x.stride(0), y2.data_ptr(), y2.stride(0), x.shape[1]) == 0
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int32), y2.view(torch.int32))
