"""The oracle pinned to the reference's own code.

oracle/_ref/ holds the reference's unmodified template headers compiled
against the from-scratch host Kokkos shim (oracle/kokkos_shim/), built by
oracle/Makefile where the reference checkout exists:
  * the reference's own test programs (unit/core/test_core_unit.cpp,
    unit/core/test_template_coverage.cpp, unit/pytorch_resnet and
    unit/projection_skip with the fixtures their generator scripts wrote)
    must pass under the shim, which validates the shim with the reference's
    known answers;
  * libponni_ref.so runs the reference's Inference::forward_batch_parallel on
    the benchmark networks and on a network with every layer kind; the C
    port (oracle/ponni_oracle.c, the checker of every GPU parity test) must
    agree with it bit for bit in fp32, fp64, fp16 and bf16.
Skipped where oracle/_ref was not built.
"""
import os
import subprocess

import numpy as np
import pytest

import ponni_b200 as pb
from ponni_b200 import configs
from oracle import oracle, ref
from tests import kat_models as K

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref")
GOLDEN = os.path.join(ROOT, "tests", "golden")

needs_ref = pytest.mark.skipif(not ref.available(), reason="oracle/_ref not built (no reference checkout)")


@pytest.mark.parametrize("prog,args", [("test_core_unit", []), ("test_template_coverage", []),
                                       ("test_pytorch_resnet", ["pytorch_resnet.ponni"]),
                                       ("test_projection_skip", ["projection_skip.ponni"])])
def test_reference_unit_programs_pass_under_the_shim(prog, args, tmp_path):
    exe = os.path.join(REF, prog)
    if not os.path.exists(exe):
        pytest.skip(f"{prog} not built (no reference checkout)")
    p = subprocess.run([exe] + [os.path.join(GOLDEN, a) for a in args], cwd=tmp_path, capture_output=True,
                       text=True, timeout=600)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-2000:]


def _all_kinds(rng, sixteen):
    from tests.test_gpu_parity import all_kinds_model
    layers = all_kinds_model(rng)
    if sixteen:  # the reference's ELU / SELU do not compile for 16-bit `real`
        layers = [l for l in layers if type(l).__name__ not in ("Elu", "Selu")]
    return layers


@needs_ref
@pytest.mark.parametrize("dtype", [pb.F32, pb.F64, pb.F16, pb.BF16])
@pytest.mark.parametrize("name", ["cfg1", "cfg2", "cfg3", "cfg4", "cfg5", "all_kinds", "ones"])
@pytest.mark.parametrize("batch", [1, 3, 257])
def test_port_equals_reference_bit_for_bit(name, dtype, batch):
    rng = np.random.default_rng(batch)
    if name == "all_kinds":
        layers = _all_kinds(rng, dtype in (pb.F16, pb.BF16))
        x = pb.to_dtype_bytes(rng.normal(0, 1, (6, batch)), dtype)
    elif name == "ones":
        layers = K.ones_network()
        x = pb.to_dtype_bytes(rng.normal(0, 1, (2, batch)), dtype)
    else:
        cfg = configs.ALL[name](batch=batch)
        layers = cfg.layers
        x = pb.to_dtype_bytes(K.as_float(configs.host_inputs(cfg, batch), cfg.dtype), dtype)
    assert ref.network_of(layers) is not None
    r = ref.forward(layers, dtype, x)
    o = oracle.forward(layers, dtype, x)
    assert np.array_equal(r.view(np.uint8), o.view(np.uint8)), f"{name} {dtype}: port and reference differ"


@needs_ref
def test_reference_known_answers():
    # unit/core/test_core_unit.cpp:200-238: the ones network gives 4, 4
    y = ref.forward(K.ones_network(), pb.F32, np.array([[1.0], [2.0]], np.float32))
    assert np.allclose(y.ravel(), [4.0, 4.0])
