"""The allocation-free host-buffer forward (ponni_b200_forward_host_static).

It exists for callers that cannot allocate device memory during inference
(an application that owns all GPU memory through its own pool, a solver with
a fixed memory budget, code that must not trigger the synchronising
cudaMalloc).  It stages through a static device array instead of cudaMalloc'd
buffers.  This file is collected last so that a stop-at-first-failure run has
already run every other test; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

import ponni_b200 as pb
from ponni_b200 import configs
from tests import kat_models as K

pytestmark = pytest.mark.gpu


def _static_forward(model, x, nout):
    out = np.empty((nout, x.shape[1]), dtype=x.dtype)
    st = pb._abi.lib().ponni_b200_forward_host_static(model._m, x.ctypes.data, x.shape[1], out.ctypes.data,
                                                      out.shape[1], x.shape[1])
    return st, out


def test_static_forward_matches_forward_host_twice():
    cfg = configs.cfg2(batch=100_003)
    model = pb.Inference(cfg.layers, dtype=cfg.dtype)
    model.kernel()  # prepares the model (uploads parameters) before the allocation-free calls
    for call, seed in enumerate((11, 12)):  # two calls in a row, different inputs
        x = np.ascontiguousarray(configs.host_inputs(cfg, cfg.batch, seed=seed))
        ref = model.forward_batch_parallel(x)  # ponni_b200_forward_host (cudaMalloc'd staging)
        st, y = _static_forward(model, x, cfg.layers[-1].num_outputs)
        assert st == 0, pb._abi.lib().ponni_b200_last_error(model._m).decode()
        assert K.normwise_err(y, ref) <= 1e-5, f"call {call}"


def test_static_forward_16bit_model():
    cfg = configs.cfg3(batch=4099)
    model = pb.Inference(cfg.layers, dtype=cfg.dtype)
    model.kernel()
    x = np.ascontiguousarray(configs.host_inputs(cfg, cfg.batch))
    ref = model.forward_batch_parallel(x)
    for _ in range(2):
        st, y = _static_forward(model, x, cfg.layers[-1].num_outputs)
        assert st == 0
        assert K.normwise_err(K.as_float(y, cfg.dtype), K.as_float(ref, cfg.dtype)) <= 2e-3


def test_static_forward_rejects_oversize_and_unprepared():
    cfg = configs.cfg2(batch=10)
    model = pb.Inference(cfg.layers, dtype=cfg.dtype)
    x = np.zeros((30, 10), np.float32)
    st, _ = _static_forward(model, x, 10)  # not prepared yet
    assert st != 0 and "not prepared" in pb._abi.lib().ponni_b200_last_error(model._m).decode()
    model.kernel()
    big = 64 * 1024 * 1024 // (40 * 4) + 1  # one column more than the 64 MiB staging holds
    xb = np.zeros((30, big), np.float32)
    st, _ = _static_forward(model, xb, 10)
    msg = pb._abi.lib().ponni_b200_last_error(model._m).decode()
    assert st == 1  # PONNI_B200_ERR_INVALID_ARGUMENT
    assert "static staging buffer" in msg


def test_static_forward_allocates_nothing(oracle_lib):
    """A freshly prepared model's first allocation-free calls leave the
    device's free memory unchanged (no staging buffer is created; the static
    array itself is loaded with the library's module before the check)."""
    torch = pytest.importorskip("torch")
    cfg = configs.cfg2(batch=100_003)
    warm = pb.Inference(cfg.layers, dtype=cfg.dtype)
    warm.kernel()
    x = np.ascontiguousarray(configs.host_inputs(cfg, cfg.batch))
    assert _static_forward(warm, x, 10)[0] == 0  # loads the module holding the static array
    model = pb.Inference(cfg.layers, dtype=cfg.dtype)
    model.kernel()  # prepares (allocates parameters) before the measurement
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(0)[0]
    for _ in range(2):
        st, y = _static_forward(model, x, 10)
        assert st == 0, pb._abi.lib().ponni_b200_last_error(model._m).decode()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(0)[0] == free0
    ref = oracle_lib.forward(cfg.layers, cfg.dtype, x)
    check_y = K.normwise_err(y, ref)
    assert check_y <= 1e-5


def test_static_forward_at_the_size_limit(oracle_lib):
    """A batch within a few bytes of the 64 MiB staging limit: the output is
    staged right after the input (no alignment padding fits), with the
    unpadded row stride; the result still matches the oracle, twice."""
    cfg = configs.cfg1(batch=64 * 1024 * 1024 // 12)  # 2 inputs + 1 output, fp32: 12 bytes per column
    model = pb.Inference(cfg.layers, dtype=cfg.dtype)
    model.kernel()
    x = np.ascontiguousarray(configs.host_inputs(cfg, cfg.batch))
    ref = oracle_lib.forward(cfg.layers, cfg.dtype, x)
    for _ in range(2):
        st, y = _static_forward(model, x, 1)
        assert st == 0, pb._abi.lib().ponni_b200_last_error(model._m).decode()
        assert K.normwise_err(y, ref) <= 1e-5
