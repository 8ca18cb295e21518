"""The CPU oracle pinned against the reference's own known answers and fixtures."""
import numpy as np
import pytest

import ponni_b200 as pb
from tests import kat_models as K


def f32(a):
    return np.asarray(a, dtype=np.float32)


def test_ones_network(oracle_lib):
    y = oracle_lib.forward(K.ones_network(), pb.F32, f32([[1.0], [2.0]]))
    assert np.allclose(y, 4.0, atol=1e-6)


def test_four_block_closed_form(oracle_lib):
    x = K.four_block_input()
    assert np.allclose(oracle_lib.forward(K.four_block(), pb.F32, x), K.four_block_expected(x), atol=1e-4)


def test_softmax_barrier_mid_chain(oracle_lib):
    y = oracle_lib.forward(K.softmax_mixed(), pb.F32, np.full((2, 2), 0.5, np.float32))
    assert np.allclose(y[0], np.tanh(1.0), atol=1e-5) and np.allclose(y[1], 0.0, atol=1e-5)


@pytest.mark.parametrize("idx", range(15))
def test_activation_kats(idx, oracle_lib):
    layer, expected, tol = K.activation_kats()[idx]
    y = oracle_lib.forward([layer], pb.F32, f32([[-1.0], [0.0], [2.0]]))
    assert np.allclose(y[:, 0], expected, atol=tol), (layer.label, y[:, 0], expected)


def test_layernorm_minmax_projection_kats(oracle_lib):
    y = oracle_lib.forward([pb.LayerNorm(np.ones(4), np.zeros(4))], pb.F32, f32([[1.0], [2.0], [3.0], [4.0]]))
    assert abs(float(np.mean(y))) < 1e-4
    y = oracle_lib.forward([pb.MinMaxNorm(3, -1.0, 1.0)], pb.F32, f32([[2.0], [5.0], [8.0]]))
    assert abs(y[0, 0] + 1.0) < 1e-5 and abs(y[2, 0] - 1.0) < 1e-5
    y = oracle_lib.forward(K.projection_add_model(), pb.F32, f32([[4.0], [5.0]]))
    assert np.allclose(y[:, 0], [5.1, 7.2, 7.8], atol=1e-5)


def test_readme_and_perf_benchmark(oracle_lib):
    y = oracle_lib.forward(K.readme_mlp(), pb.F32, np.ones((2, 1000), np.float32))
    assert np.allclose(y, 0.7, atol=1e-6)
    y = oracle_lib.forward(K.perf_benchmark(), pb.F32, np.full((8, 4096), 0.1, np.float32))
    assert abs(float(np.mean(y.astype(np.float64))) - 15.4) <= 1e-3


def test_pytorch_resnet_fixture(oracle_lib):
    layers, xin, xout = K.pytorch_resnet()
    y = oracle_lib.forward(layers, pb.F32, np.ascontiguousarray(xin))
    assert y.shape == xout.shape
    assert np.max(np.abs(y - xout)) <= 1e-5


def test_half_rounding_kats(oracle_lib):
    # TwoHalf rounding KATs (unit/core/test_core_unit.cpp:1019-1070): exact
    # small integers, round-to-nearest-even ties, overflow to inf.
    L = oracle_lib.lib()
    assert L.ponni_oracle_round_f16(6.0) == 6.0 and L.ponni_oracle_round_f16(-13.0) == -13.0
    assert L.ponni_oracle_round_f16(2049.0) == 2048.0  # tie -> even
    assert L.ponni_oracle_round_f16(2051.0) == 2052.0
    assert np.isinf(L.ponni_oracle_round_f16(70000.0))
    assert L.ponni_oracle_round_f16(1e-8) == 0.0
    vals = np.random.default_rng(0).normal(0, 100, 2000).astype(np.float32)
    for v in vals[:200]:
        assert L.ponni_oracle_round_f16(float(v)) == float(np.float16(v))
        assert L.ponni_oracle_round_bf16(float(v)) == float(pb.bf16_to_f32(pb.bf16_bits(np.float32(v)))[0])
    sub = np.float32(3.3e-6)  # half subnormal range
    assert L.ponni_oracle_round_f16(float(sub)) == float(np.float16(sub))


def test_half_model_is_per_op_rounded(oracle_lib):
    # The template half model accumulates in half: with 2048 + 1 + 1 the
    # per-operation rounding loses both ones (reference Matvec with real = half_t).
    layers = [pb.Matvec(np.ones((3, 1)))]
    x = np.array([[2048.0], [1.0], [1.0]], dtype=np.float16)
    assert float(oracle_lib.forward(layers, pb.F16, x)[0, 0]) == 2048.0
    assert float(oracle_lib.forward(layers, pb.F32, x.astype(np.float32))[0, 0]) == 2050.0


def test_double_model(oracle_lib):
    layers, xin, xout = K.pytorch_resnet()
    y = oracle_lib.forward(layers, pb.F64, np.ascontiguousarray(xin, dtype=np.float64))
    assert np.max(np.abs(y - xout)) <= 1e-5
