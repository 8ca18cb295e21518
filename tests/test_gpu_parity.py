"""GPU parity: libponni_b200 (through the C ABI) against the CPU oracle.

Tolerances: fp32 -- normwise error per output feature <= 1e-5 against the
oracle, and elementwise and rms accuracy against float64 no worse than the
reference's (kat_models.fp_parity); fp64 -- normwise <= 1e-12; fp16/bf16
with the reference's arithmetic -- normwise <= 2e-3 against the oracle's
per-operation-rounded half/bfloat16 arithmetic (measured: bit-identical).
"""
import numpy as np
import pytest

import ponni_b200 as pb
from ponni_b200 import configs
from tests import kat_models as K

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = {pb.F32: 1e-5, pb.F64: 1e-12}


def to_torch(x_raw, dtype):
    if dtype == pb.BF16:
        return torch.from_numpy(np.ascontiguousarray(x_raw).view(np.int16)).view(torch.bfloat16)
    return torch.from_numpy(np.ascontiguousarray(x_raw))


def from_torch(y, dtype):
    if dtype == pb.BF16:
        return y.view(torch.int16).cpu().numpy().view(np.uint16)
    return y.cpu().numpy()


def run_device(layers, dtype, x_raw, arithmetic=None):
    m = pb.Inference(layers, dtype=dtype, arithmetic=arithmetic)
    y = m.forward_batch_parallel(to_torch(x_raw, dtype).cuda())
    torch.cuda.synchronize()
    return from_torch(y, dtype)


def check(y_raw, ref_raw, dtype, layers=None, x_raw=None):
    y, ref = K.as_float(y_raw, dtype), K.as_float(ref_raw, dtype)
    assert np.all(np.isfinite(y))
    if dtype == pb.F64:
        nw = K.normwise_err(y, ref)
        assert nw <= TOL[dtype], f"normwise error {nw:.3e}"
    elif dtype == pb.F32:
        from oracle import oracle
        exact = oracle.forward(layers, pb.F64, K.as_float(x_raw, dtype))
        nw, ratio, el_ratio = K.fp_parity(y, ref, exact, TOL[dtype])
        assert nw <= TOL[dtype], f"normwise error {nw:.3e}"
        assert ratio <= 1.0, f"rms accuracy ratio {ratio:.3f}"
        assert el_ratio <= 1.0, f"elementwise accuracy ratio {el_ratio:.3f}"
    else:
        e = K.normwise_err(y, ref)
        assert e <= 2e-3, f"normwise error {e:.3e}"


@pytest.mark.parametrize("name", ["cfg1", "cfg2", "cfg3", "cfg4", "cfg5"])
@pytest.mark.parametrize("batch", [1, 3, 129, 4099])
def test_configs_vs_oracle(name, batch, oracle_lib):
    cfg = configs.ALL[name](batch=batch)
    x = configs.host_inputs(cfg, batch)
    y = run_device(cfg.layers, cfg.dtype, x)
    ref = oracle_lib.forward(cfg.layers, cfg.dtype, x)
    check(y, ref, cfg.dtype, cfg.layers, x)


def all_kinds_model(rng, n=12):
    return [pb.Matvec(rng.normal(0, 0.4, (6, n))), pb.Bias(rng.normal(0, 0.1, n)), pb.Elu(n, 0.7),
            pb.Save_State(n, 0), pb.Selu(n), pb.Softplus(n, 1.5), pb.Matvec(rng.normal(0, 0.3, (n, n))),
            pb.Gelu(n), pb.Gelu(n, True), pb.Mish(n), pb.LayerNorm(rng.normal(1, 0.1, n), rng.normal(0, 0.1, n)),
            pb.HardSigmoid(n), pb.HardSwish(n), pb.Binop_Add(n, 0), pb.Save_State(n, 1),
            pb.Sigmoid(n), pb.Tanh(n), pb.Silu(n), pb.MinMaxNorm(n, -1.0, 2.0),
            pb.Binop_Concatenate(n, 2 * n, True, 1), pb.Relu(2 * n), pb.LeakyRelu(2 * n, 0.05),
            pb.Save_State(2 * n, 2), pb.Softmax(2 * n),
            pb.Binop_Projection_Add(rng.normal(0, 0.2, (2 * n, 2 * n)), rng.normal(0, 0.1, 2 * n), True, 2),
            pb.LogSoftmax(2 * n), pb.Matvec(rng.normal(0, 0.3, (2 * n, 5))), pb.Bias(rng.normal(0, 0.1, 5))]


@pytest.mark.parametrize("dtype", [pb.F32, pb.F64, pb.F16, pb.BF16])
def test_all_layer_kinds(dtype, oracle_lib):
    rng = np.random.default_rng(7)
    layers = all_kinds_model(rng)
    batch = 1000
    x = pb.to_dtype_bytes(rng.normal(0, 1, (6, batch)), dtype)
    y = run_device(layers, dtype, x)
    check(y, oracle_lib.forward(layers, dtype, x), dtype, layers, x)


def test_concatenate_before_and_barrier_first(oracle_lib):
    rng = np.random.default_rng(3)
    layers = [pb.Save_State(4, 0), pb.LayerNorm(4), pb.Binop_Concatenate(4, 8, False, 0), pb.Tanh(8),
              pb.Matvec(rng.normal(0, 0.5, (8, 3)))]
    x = rng.normal(0, 1, (4, 777)).astype(np.float32)
    check(run_device(layers, pb.F32, x), oracle_lib.forward(layers, pb.F32, x), pb.F32, layers, x)


def test_kats_on_gpu():
    y = run_device(K.ones_network(), pb.F32, np.array([[1.0], [2.0]], np.float32))
    assert np.allclose(y, 4.0)
    x = K.four_block_input()
    assert np.allclose(run_device(K.four_block(), pb.F32, x), K.four_block_expected(x), atol=1e-4)
    y = run_device(K.softmax_mixed(), pb.F32, np.full((2, 2), 0.5, np.float32))
    assert np.allclose(y[0], np.tanh(1.0), atol=1e-5) and np.allclose(y[1], 0.0, atol=1e-5)
    y = run_device(K.readme_mlp(), pb.F32, np.ones((2, 100000), np.float32))
    assert np.allclose(y, 0.7, atol=1e-6)
    y = run_device(K.perf_benchmark(), pb.F32, np.full((8, 1 << 16), 0.1, np.float32))
    assert abs(float(np.mean(y.astype(np.float64))) - 15.4) <= 1e-3
    y = run_device(K.projection_add_model(), pb.F32, np.array([[4.0], [5.0]], np.float32))
    assert np.allclose(y[:, 0], [5.1, 7.2, 7.8], atol=1e-5)
    for layer, expected, tol in K.activation_kats():
        y = run_device([layer], pb.F32, np.array([[-1.0], [0.0], [2.0]], np.float32))
        assert np.allclose(y[:, 0], expected, atol=tol), layer.label
    layers, xin, xout = K.pytorch_resnet()
    y = run_device(layers, pb.F32, np.ascontiguousarray(xin))
    assert np.max(np.abs(y - xout)) <= 1e-5


@pytest.mark.parametrize("offset", [0, 1, 3])
def test_strided_and_misaligned_views(offset, oracle_lib):
    cfg = configs.cfg2(batch=1000)
    x = configs.host_inputs(cfg, 1000)
    ref = oracle_lib.forward(cfg.layers, cfg.dtype, x)
    m = pb.Inference(cfg.layers, dtype=cfg.dtype)
    big = torch.zeros((30, 1000 + 17), dtype=torch.float32, device="cuda")
    big[:, offset:offset + 1000] = torch.from_numpy(x).cuda()
    out_big = torch.full((10, 1000 + 9), float("nan"), device="cuda")
    out = out_big[:, offset:offset + 1000]
    m.forward_batch_parallel(big[:, offset:offset + 1000], out)
    torch.cuda.synchronize()
    check(out.cpu().numpy(), ref, cfg.dtype, cfg.layers, x)
    assert torch.isnan(out_big[:, :offset]).all() and torch.isnan(out_big[:, offset + 1000:]).all()


@pytest.mark.parametrize("name", ["cfg1", "cfg2", "cfg3"])
def test_host_pipeline(name, oracle_lib):
    cfg = configs.ALL[name](batch=300_001)
    x = configs.host_inputs(cfg, cfg.batch)
    m = pb.Inference(cfg.layers, dtype=cfg.dtype)
    y = m.forward_batch_parallel(x)
    check(y, oracle_lib.forward(cfg.layers, cfg.dtype, x), cfg.dtype, cfg.layers, x)


def test_capacity_semantics():
    # unit/core/test_core_unit.cpp:241-256
    m = pb.create_inference_model(*K.ones_network())
    assert m.internal_state_capacity() == 0
    m.forward_batch_parallel(torch.ones((2, 1), device="cuda"))
    assert m.internal_state_capacity() == 1
    m.forward_batch_parallel(torch.ones((2, 4), device="cuda"))
    assert m.internal_state_capacity() == 4
    m.forward_batch_parallel(torch.ones((2, 1), device="cuda"))
    assert m.internal_state_capacity() == 4
    m.reallocate_internal_state(2)
    assert m.internal_state_capacity() == 2
    assert m.scratch_bytes() == 0


def test_save_load_roundtrip_gpu(tmp_path):
    m = pb.create_inference_model(*K.ones_network())
    ok, err = m.save_weights(str(tmp_path / "w.ponni"))
    assert ok, err
    x = torch.tensor([[1.0], [2.0]], device="cuda")
    assert torch.allclose(m.forward_batch_parallel(x), torch.full((2, 1), 4.0, device="cuda"))
    m.set_trainable_parameters(np.zeros(m.get_num_trainable_parameters()))
    assert torch.allclose(m.forward_batch_parallel(x), torch.zeros(2, 1, device="cuda"))
    ok, err = m.load_weights(str(tmp_path / "w.ponni"))
    assert ok, err
    assert torch.allclose(m.forward_batch_parallel(x), torch.full((2, 1), 4.0, device="cuda"))


def test_errors_leave_context_usable():
    m = pb.create_inference_model(*K.ones_network())
    with pytest.raises(pb.PonniError):
        m.forward_batch_parallel(torch.ones((3, 4), device="cuda"))
    with pytest.raises(pb.PonniError):
        m.forward_batch_parallel(torch.ones((2, 0), device="cuda"))
    assert torch.allclose(m.forward_batch_parallel(torch.tensor([[1.0], [2.0]], device="cuda")),
                          torch.full((2, 1), 4.0, device="cuda"))


@pytest.mark.parametrize("name", ["cfg2", "cfg3", "cfg4", "cfg5"])
def test_full_size_shard_consistency(name):
    """At each config's full size: column slices computed alone equal the
    same columns of the full-batch result bit for bit (samples are
    independent), and a strided sample of about 4096 columns of the full
    result passes the config's parity gate against the oracle."""
    from oracle import oracle
    from tests.test_gpu_tensor import check_acc32

    cfg = configs.ALL[name]()
    arith = pb._abi.ARITH_TENSOR if cfg.arith == "tensor" else None
    m = pb.Inference(cfg.layers, dtype=cfg.dtype, arithmetic=arith)
    tdt = m.torch_dtype()
    nin = cfg.layers[0].num_inputs
    x = torch.empty((nin, cfg.batch), device="cuda", dtype=tdt)
    pb.fill_synthetic(x, configs.INPUT_SEED, dist=cfg.input_dist, lo=cfg.lo, hi=cfg.hi)
    y = m.forward_batch_parallel(x)
    m.synchronize()
    for c0, n in [(0, 4096), (12345, 777), (cfg.batch - 1000, 1000)]:
        part = torch.empty((nin, n), device="cuda", dtype=tdt)
        pb.fill_synthetic(part, configs.INPUT_SEED, col0=c0, dist=cfg.input_dist, lo=cfg.lo, hi=cfg.hi)
        assert torch.equal(part, x[:, c0:c0 + n])
        assert torch.equal(m.forward_batch_parallel(part), y[:, c0:c0 + n])
    step = cfg.batch // 4096 + 1
    cols = torch.arange(0, cfg.batch, step, device="cuda")
    xs = from_torch(x[:, cols].contiguous(), cfg.dtype)
    ys = from_torch(y[:, cols].contiguous(), cfg.dtype)
    assert np.all(np.isfinite(K.as_float(ys, cfg.dtype)))
    del x, y
    torch.cuda.empty_cache()
    if arith == pb._abi.ARITH_TENSOR and cfg.dtype != pb.F32:
        check_acc32(ys, cfg.layers, cfg.dtype, xs, oracle)
    else:
        check(ys, oracle.forward(cfg.layers, cfg.dtype, xs), cfg.dtype, cfg.layers, xs)


@pytest.mark.parametrize("jit", [True, False])
@pytest.mark.parametrize("dtype", [pb.F32, pb.F64, pb.F16, pb.BF16])
@pytest.mark.parametrize("maxw", [3, 8, 13, 32])
def test_narrow_kernel(dtype, maxw, jit, oracle_lib, monkeypatch):
    """Narrow chains on the model-specialised (NVRTC) kernel and on the
    generic narrow kernel (PONNI_B200_NARROW_JIT=0)."""
    if not jit:
        monkeypatch.setenv("PONNI_B200_NARROW_JIT", "0")
    want = pb._abi.KERNEL_NARROW_JIT if jit else pb._abi.KERNEL_NARROW
    rng = np.random.default_rng(maxw)
    dims = [min(maxw, 5), maxw, max(2, maxw // 2), 3]
    layers = []
    for i in range(3):
        layers += [pb.Matvec(rng.normal(0, 1 / np.sqrt(dims[i]), (dims[i], dims[i + 1]))),
                   pb.Bias(rng.normal(0, 0.1, dims[i + 1]))]
        if i < 2:
            layers.append([pb.Relu, pb.Silu, pb.Tanh][i % 3](dims[i + 1]))
    ref_arith = pb._abi.ARITH_REFERENCE  # (fp32 chains wider than 16 go to tensor cores under AUTO)
    # second network: a leading pointwise run (its own step), LeakyReLU on the
    # register path, a Bias-free dense layer, GELU + Sigmoid on the staged path
    layers2 = [pb.Tanh(dims[0]), pb.LeakyRelu(dims[0], 0.05),
               pb.Matvec(rng.normal(0, 1 / np.sqrt(dims[0]), (dims[0], dims[1]))), pb.LeakyRelu(dims[1], 0.2),
               pb.Matvec(rng.normal(0, 1 / np.sqrt(dims[1]), (dims[1], dims[3]))),
               pb.Bias(rng.normal(0, 0.1, dims[3])), pb.Gelu(dims[3]), pb.Sigmoid(dims[3])]
    for net in (layers, layers2):
        m = pb.Inference(net, dtype=dtype, arithmetic=ref_arith)
        assert m.kernel() == want
        for batch in (1, 7, 1001, 4099):
            x = pb.to_dtype_bytes(rng.normal(0, 1, (dims[0], batch)), dtype)
            check(run_device(net, dtype, x, ref_arith), oracle_lib.forward(net, dtype, x), dtype, net, x)


def test_tile_kernel_on_narrow_models(monkeypatch):
    # the tile kernel still serves narrow chains when forced (and every
    # program with barriers); rerun the known answers on it
    monkeypatch.setenv("PONNI_B200_FORCE_TILE", "1")
    m = pb.Inference(K.readme_mlp())
    assert m.kernel() == pb._abi.KERNEL_TILE
    test_kats_on_gpu()


@pytest.mark.parametrize("dtype", [pb.F32, pb.F64, pb.F16, pb.BF16])
def test_narrow_jit_matches_generic(dtype, monkeypatch):
    """The model-specialised narrow kernel performs the same operations in the
    same order as the generic narrow kernel: results agree bit for bit."""
    rng = np.random.default_rng(7)
    net = [pb.Matvec(rng.normal(0, 0.5, (6, 8))), pb.Bias(rng.normal(0, 0.1, 8)), pb.Silu(8),
           pb.Matvec(rng.normal(0, 0.5, (8, 5))), pb.Bias(rng.normal(0, 0.1, 5)), pb.LeakyRelu(5, 0.1),
           pb.Matvec(rng.normal(0, 0.5, (5, 2))), pb.Bias(rng.normal(0, 0.1, 2)), pb.Tanh(2)]
    x = pb.to_dtype_bytes(rng.normal(0, 1, (6, 70001)), dtype)
    ref = pb._abi.ARITH_REFERENCE
    y_jit = run_device(net, dtype, x, ref)
    assert pb.Inference(net, dtype=dtype, arithmetic=ref).kernel() == pb._abi.KERNEL_NARROW_JIT
    monkeypatch.setenv("PONNI_B200_NARROW_JIT", "0")
    assert pb.Inference(net, dtype=dtype, arithmetic=ref).kernel() == pb._abi.KERNEL_NARROW
    y_gen = run_device(net, dtype, x, ref)
    assert np.array_equal(np.asarray(y_jit).view(np.uint8), np.asarray(y_gen).view(np.uint8))


def test_narrow_jit_weights_change_reuses_kernel(oracle_lib):
    """Two models of one structure share the compiled kernel; each runs with
    its own weights (they travel as a kernel parameter)."""
    rng = np.random.default_rng(11)
    for seed in (1, 2):
        r = np.random.default_rng(seed)
        net = [pb.Matvec(r.normal(0, 1, (2, 3))), pb.Bias(r.normal(0, 1, 3)), pb.Relu(3),
               pb.Matvec(r.normal(0, 1, (3, 1))), pb.Bias(r.normal(0, 1, 1))]
        assert pb.Inference(net).kernel() == pb._abi.KERNEL_NARROW_JIT
        x = pb.to_dtype_bytes(rng.normal(0, 1, (2, 5000)), pb.F32)
        check(run_device(net, pb.F32, x), oracle_lib.forward(net, pb.F32, x), pb.F32, net, x)


def test_caller_device_is_restored(oracle_lib):
    """Every entry point runs on the model's device and leaves the caller's
    current device as it found it (one-process multi-GPU applications)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    torch.cuda.set_device(0)
    for cfg in (configs.cfg4(batch=300), configs.cfg1(batch=300)):
        m = pb.Inference(cfg.layers, dtype=cfg.dtype, device=1)
        assert m.kernel() > 0
        assert torch.cuda.current_device() == 0
        x = configs.host_inputs(cfg, cfg.batch)
        y = m.forward_batch_parallel(torch.from_numpy(x).to("cuda:1"))
        m.synchronize()
        assert torch.cuda.current_device() == 0
        yh = m.forward_batch_parallel(x)  # host buffers
        assert torch.cuda.current_device() == 0
        m.set_trainable_parameters(m.get_trainable_parameters())
        assert torch.cuda.current_device() == 0
        ref = oracle_lib.forward(cfg.layers, cfg.dtype, x)
        check(y.cpu().numpy(), ref, cfg.dtype, cfg.layers, x)
        check(yh, ref, cfg.dtype, cfg.layers, x)
        del m
        assert torch.cuda.current_device() == 0


@pytest.mark.parametrize("name", ["cfg1", "cfg2", "cfg3", "cfg4", "cfg5"])
@pytest.mark.parametrize("dtype", [pb.F32, pb.F16, pb.BF16])
def test_configs_vs_reference_itself(name, dtype):
    """Each config on the GPU against the reference's own code (its template
    headers compiled against the host Kokkos shim, oracle/_ref): fp32 through
    the default kernels with the fp32 gate; 16-bit with the reference's
    arithmetic (tile / narrow kernels) bit for bit (the 16-bit path evaluates
    its float transcendentals correctly rounded, as the host C library)."""
    from oracle import ref
    if not ref.available():
        pytest.skip("oracle/_ref not built")
    cfg = configs.ALL[name](batch=3001)
    x = pb.to_dtype_bytes(K.as_float(configs.host_inputs(cfg, cfg.batch), cfg.dtype), dtype)
    arith = None if dtype == pb.F32 else pb._abi.ARITH_REFERENCE
    y = run_device(cfg.layers, dtype, x, arith)
    r = ref.forward(cfg.layers, dtype, x)
    if dtype == pb.F32:
        check(y, r, dtype, cfg.layers, x)
    else:
        assert np.array_equal(y.view(np.uint16), r.view(np.uint16))
