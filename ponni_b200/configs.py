"""The benchmark networks (the five configurations the B200 build is measured on).

Weights are made on the host from a seeded numpy generator (seed 1234); the
reference's Kokkos initializers (src/initializers/ponni_initializer.h) are not
reproduced.  The distributions:
  cfg1  README 2->3->1 MLP, W/b ~ U(-1, 1), fp32, inputs N(0,1), batch 1,000,000
  cfg2  column-physics emulator 30->64->64->64->10, ReLU, He-normal W, zero b, fp32, batch 2^24
  cfg3  cfg2 in half precision, inputs U(-2, 2), batch 2^26
  cfg4  residual MLP 16->128, 4 x [Save_State, LayerNorm(128), Dense128, GELU, Dense128, Binop_Add],
        ->8, Glorot-uniform W, zero b, fp32, batch 2^25
  cfg5  wide chain 64->256x5->32, SiLU, Glorot-normal W, b ~ N(0, 0.01), bfloat16, batch 2^27
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import _abi
from . import layers as L

WEIGHT_SEED = 1234
INPUT_SEED = 5678


@dataclass
class Config:
    name: str
    layers: list
    dtype: int
    batch: int
    input_dist: str = "normal"  # "normal" N(0,1) or "uniform" U(lo, hi)
    lo: float = -1.0
    hi: float = 1.0
    flops_per_sample: int = 0
    bytes_per_sample: int = 0
    bound: str = "hbm"
    description: str = ""
    arith: str = "auto"  # cfg3/cfg5 are specified with fp32 accumulation: "tensor"


def _dense_flops(layers) -> int:
    return sum(2 * l.num_inputs * l.num_outputs for l in layers if isinstance(l, L.Matvec))


def _elem(dtype: int) -> int:
    return {_abi.F32: 4, _abi.F64: 8, _abi.F16: 2, _abi.BF16: 2}[dtype]


def _finish(cfg: Config) -> Config:
    cfg.flops_per_sample = _dense_flops(cfg.layers)
    cfg.bytes_per_sample = (cfg.layers[0].num_inputs + cfg.layers[-1].num_outputs) * _elem(cfg.dtype)
    return cfg


def cfg1(batch: int = 1_000_000) -> Config:
    rng = np.random.default_rng(WEIGHT_SEED)
    layers = [L.Matvec(rng.uniform(-1, 1, (2, 3))), L.Bias(rng.uniform(-1, 1, 3)), L.Relu(3),
              L.Matvec(rng.uniform(-1, 1, (3, 1))), L.Bias(rng.uniform(-1, 1, 1))]
    return _finish(Config("cfg1_mlp_2_3_1_fp32", layers, _abi.F32, batch, bound="hbm",
                          description="README MLP 2->3->1 fp32"))


def _emulator_layers(rng):
    dims = [30, 64, 64, 64, 10]
    layers = []
    for i in range(4):
        nin, nout = dims[i], dims[i + 1]
        layers.append(L.Matvec(rng.normal(0.0, np.sqrt(2.0 / nin), (nin, nout))))
        layers.append(L.Bias(np.zeros(nout)))
        if i < 3:
            layers.append(L.Relu(nout))
    return layers


def cfg2(batch: int = 1 << 24) -> Config:
    rng = np.random.default_rng(WEIGHT_SEED)
    return _finish(Config("cfg2_emulator_30_64x3_10_fp32", _emulator_layers(rng), _abi.F32, batch,
                          bound="tensor", description="Column-physics emulator MLP fp32"))


def cfg3(batch: int = 1 << 26) -> Config:
    rng = np.random.default_rng(WEIGHT_SEED)
    return _finish(Config("cfg3_emulator_30_64x3_10_fp16", _emulator_layers(rng), _abi.F16, batch,
                          input_dist="uniform", lo=-2.0, hi=2.0, bound="tensor", arith="tensor",
                          description="Column-physics emulator MLP fp16, fp32 accumulate"))


def cfg4(batch: int = 1 << 25) -> Config:
    rng = np.random.default_rng(WEIGHT_SEED)

    def glorot_u(nin, nout):
        lim = np.sqrt(6.0 / (nin + nout))
        return rng.uniform(-lim, lim, (nin, nout))

    layers = [L.Matvec(glorot_u(16, 128)), L.Bias(np.zeros(128))]
    for _ in range(4):
        layers += [L.Save_State(128, 0), L.LayerNorm(128), L.Matvec(glorot_u(128, 128)), L.Bias(np.zeros(128)),
                   L.Gelu(128), L.Matvec(glorot_u(128, 128)), L.Bias(np.zeros(128)), L.Binop_Add(128, 0)]
    layers += [L.Matvec(glorot_u(128, 8)), L.Bias(np.zeros(8))]
    return _finish(Config("cfg4_resmlp_16_128_ln_gelu_8_fp32", layers, _abi.F32, batch, bound="tensor",
                          description="Residual MLP with LayerNorm/GELU fp32"))


def cfg5(batch: int = 1 << 27) -> Config:
    rng = np.random.default_rng(WEIGHT_SEED)
    dims = [64, 256, 256, 256, 256, 256, 32]
    layers = []
    for i in range(6):
        nin, nout = dims[i], dims[i + 1]
        layers.append(L.Matvec(rng.normal(0.0, np.sqrt(2.0 / (nin + nout)), (nin, nout))))
        layers.append(L.Bias(rng.normal(0.0, 0.01, nout)))
        if i < 5:
            layers.append(L.Silu(nout))
    return _finish(Config("cfg5_wide_64_256x5_32_bf16", layers, _abi.BF16, batch, bound="tensor", arith="tensor",
                          description="Wide dense chain bf16, fp32 accumulate"))


ALL = {"cfg1": cfg1, "cfg2": cfg2, "cfg3": cfg3, "cfg4": cfg4, "cfg5": cfg5}


def host_inputs(cfg: Config, batch: int, col0: int = 0, seed: int = INPUT_SEED) -> np.ndarray:
    """Seeded host inputs [nin, batch] in the model dtype's storage (bf16 as uint16 bits)."""
    from .inference import to_dtype_bytes

    rng = np.random.default_rng([seed, col0])
    nin = cfg.layers[0].num_inputs
    if cfg.input_dist == "normal":
        x = rng.normal(0.0, 1.0, (nin, batch))
    else:
        x = rng.uniform(cfg.lo, cfg.hi, (nin, batch))
    return to_dtype_bytes(x, cfg.dtype)
