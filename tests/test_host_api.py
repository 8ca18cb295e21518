"""Host-side logic of libponni_b200 (no GPU needed): exported symbols,
validation, planning queries, fingerprints and the .ponni weight contract."""
import os
import re
import struct

import numpy as np
import pytest

import ponni_b200 as pb
from ponni_b200 import _abi
from tests import kat_models as K

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    text = open(os.path.join(ROOT, "include", "ponni_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ponni_b200_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _abi.lib()
    names = header_functions()
    assert len(names) >= 30
    for n in names:
        assert hasattr(lib, n), n
        assert n in _abi.SIGNATURES, n
    assert lib.ponni_b200_abi_version() == 1


def fnv1a64(data: bytes) -> str:
    h = 14695981039346656037
    for b in data:
        h ^= b
        h = (h * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return f"fnv1a64:{h:016x}"


def test_schema_fingerprint_matches_reference_text():
    # src/ponni_Inference.h:270-288: "ponni-template-model-v1\n" then
    # "I\tlabel\tnin\tnout\tntrain\n" per layer.
    m = pb.create_inference_model(*K.four_block())
    text = "ponni-template-model-v1\n" + "".join(
        f"{i}\t{L.label}\t{L.num_inputs}\t{L.num_outputs}\t{L.get_num_trainable_parameters()}\n"
        for i, L in enumerate(m.layers))
    assert m.weight_schema_fingerprint() == fnv1a64(text.encode())
    frozen = pb.create_inference_model(pb.Matvec(np.ones((2, 2)), trainable=False), pb.Bias(np.ones(2)))
    assert frozen.get_num_trainable_parameters() == 2
    assert "Matvec\t2\t2\t0\n" in "0\tMatvec\t2\t2\t0\n"


def test_summary_and_counts():
    m = pb.create_inference_model(*K.ones_network())
    s = m.summary()
    assert s.startswith("Inference model has 3 layers -- with 6 total trainable parameters.")
    assert "LeakyReLU" in s
    assert m.get_num_trainable_parameters() == 6


@pytest.mark.parametrize("layers,msg", [
    ([pb.Matvec(np.ones((2, 3))), pb.Bias(np.ones(4))], "num outputs != next layer's num inputs"),
    ([pb.Matvec(np.ones((2, 3))), pb.Binop_Add(3, 0)], "Binop_Add: Saved layer"),
    ([pb.Save_State(3, 0), pb.Binop_Concatenate(3, 5, True, 0)], "Binop_Concatenate: this layer's num outputs"),
    ([pb.LayerNorm(3, epsilon=0.0)], "epsilon must be > 0"),
    ([pb.Relu(0)], "ReLU num_inputs must be > 0"),
    ([pb.Save_State(2, 0), pb.Binop_Projection_Add(np.ones((3, 2)), np.ones(2))], "saved layer size incompatible"),
])
def test_validation_errors(layers, msg):
    m = pb.create_inference_model(*layers)
    with pytest.raises(pb.PonniError) as e:
        m.validate()
    assert e.value.status == 2 and msg in e.value.message


def test_planned_temporary_sizes():
    # unit/core/test_core_unit.cpp:320-323: widths 5,3,7 -> tmp1 7, tmp2 3
    m = pb.create_inference_model(*K.four_block())
    assert m.get_planned_temporary_size(0) == 7 and m.get_planned_temporary_size(1) == 3
    # :364-368: softmax barrier -> tmp1 3, no tmp2
    m = pb.create_inference_model(*K.softmax_mixed())
    assert m.get_planned_temporary_size(0) == 3 and m.get_planned_temporary_size(1) == 0
    # a single fused block needs no temporary
    m = pb.create_inference_model(*K.ones_network())
    assert m.get_planned_temporary_size(0) == 0 and m.get_planned_temporary_size(1) == 0
    layers, _, _ = K.pytorch_resnet()
    m = pb.create_inference_model(*layers)
    assert m.get_num_saved_states() == 1 and m.get_saved_state_size(0) == 5


def test_capacity_bookkeeping_without_gpu():
    m = pb.create_inference_model(*K.ones_network())
    assert m.internal_state_capacity() == 0
    m.reallocate_internal_state(5)
    assert m.internal_state_capacity() == 5
    m.reallocate_internal_state(0)
    assert m.internal_state_capacity() == 0
    with pytest.raises(pb.PonniError):
        m.reallocate_internal_state(-1)
    assert m.scratch_bytes() == 0


def test_parameters_round_trip_all_dtypes():
    for dt in (pb.F32, pb.F64, pb.F16, pb.BF16):
        m = pb.Inference(K.four_block(), dtype=dt)
        n = m.get_num_trainable_parameters()
        v = np.linspace(-2, 2, n)
        m.set_trainable_parameters(v)
        got = m.get_trainable_parameters()
        want = pb.from_dtype_bytes(pb.to_dtype_bytes(v, dt), dt)
        assert np.array_equal(got, want)


def read_file(path):
    b = open(path, "rb").read()
    hs = struct.unpack("<Q", b[:8])[0]
    return b, hs


def test_save_load_round_trip_and_format(tmp_path):
    m = pb.create_inference_model(*K.four_block())
    p = str(tmp_path / "w.ponni")
    ok, err = m.save_weights(p)
    assert ok, err
    b, hs = read_file(p)
    assert hs % 8 == 0
    import json
    hdr = json.loads(b[8:8 + hs])
    meta = hdr["__metadata__"]
    n = m.get_num_trainable_parameters()
    assert hdr["parameters"] == {"dtype": "F32", "shape": [n], "data_offsets": [0, 4 * n]}
    assert meta["ponni.profile_version"] == "1" and meta["ponni.target"] == "template"
    assert meta["ponni.model_fingerprint"] == m.weight_schema_fingerprint()
    assert meta["ponni.payload_checksum_fnv1a64"] == fnv1a64(b[8 + hs:])
    assert meta["ponni.schema_fingerprint"] == fnv1a64(f"ponni-tensor-schema-v1\nparameters\tF32\t{n}\n".encode())
    vals = m.get_trainable_parameters()
    m.set_trainable_parameters(np.zeros(n))
    ok, err = m.load_weights(p)
    assert ok, err
    assert np.array_equal(m.get_trainable_parameters(), vals)
    # double models store F64
    md = pb.create_inference_model_double_precision(*K.four_block())
    ok, _ = md.save_weights(str(tmp_path / "d.ponni"))
    b, hs = read_file(str(tmp_path / "d.ponni"))
    assert b'"dtype":"F64"' in b[8:8 + hs]
    ok, err = m.load_weights(str(tmp_path / "d.ponni"))
    assert not ok and "dtype mismatch" in err


def corrupt(src, dst, fn):
    b = bytearray(open(src, "rb").read())
    fn(b)
    open(dst, "wb").write(bytes(b))


@pytest.mark.parametrize("case,msg", [
    ("truncate", "Safetensors"),
    ("flip_payload", "checksum mismatch"),
    ("dup_key", "duplicate object key"),
    ("bad_header_size", "invalid Safetensors header size"),
    ("trailing", "unindexed trailing bytes"),
])
def test_corrupt_files_rejected(tmp_path, case, msg):
    m = pb.create_inference_model(*K.ones_network())
    p = str(tmp_path / "w.ponni")
    m.save_weights(p)
    q = str(tmp_path / "bad.ponni")
    b, hs = read_file(p)

    def edit(x):
        if case == "truncate":
            del x[len(x) - 3:]
        elif case == "flip_payload":
            x[-1] ^= 0x40
        elif case == "dup_key":
            hdr = bytes(x[8:8 + hs]).decode()
            hdr2 = hdr.replace('{"__metadata__":{', '{"__metadata__":{"ponni.target":"x",', 1)
            hdr2 += " " * ((8 - len(hdr2) % 8) % 8)
            x[:] = struct.pack("<Q", len(hdr2)) + hdr2.encode() + bytes(x[8 + hs:])
        elif case == "bad_header_size":
            x[0:8] = struct.pack("<Q", 1 << 40)
        elif case == "trailing":
            x.extend(b"\0\0\0\0")
    corrupt(p, q, edit)
    ok, err = m.load_weights(q)
    assert not ok and msg in err, err


def test_wrong_model_fingerprint(tmp_path):
    a = pb.create_inference_model(*K.ones_network())
    b = pb.create_inference_model(pb.Matvec(np.ones((2, 2))), pb.Bias(np.ones(2)), pb.Relu(2))
    p = str(tmp_path / "w.ponni")
    a.save_weights(p)
    ok, err = b.load_weights(p)
    assert not ok and "model fingerprint does not match" in err


def test_reference_written_fixture_is_readable():
    # pytorch_resnet.ponni is written by the reference's own Python writer.
    layers, xin, xout = K.pytorch_resnet()
    assert xin.shape == (12, 1) and xout.shape == (4, 1)
    assert layers[0].num_inputs == 12 and layers[-1].num_outputs == 4
    with pytest.raises(pb.PonniError):
        K.read_tensor(os.path.join(K.GOLDEN, "pytorch_resnet.ponni"), "no.such.tensor")


def test_forward_fails_loudly_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    m = pb.create_inference_model(*K.ones_network())
    with pytest.raises(pb.PonniError):
        m.forward_batch_parallel(np.ones((2, 3), np.float32))
