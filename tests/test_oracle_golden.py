"""The CPU oracle reproduces the reference's own outputs (golden vectors) exactly.

The golden vectors come from the reference itself (tests/golden/make_golden.py):
its torch path, and its Triton kernels run by the Triton interpreter, whose row
reductions use ``np.sum`` — so the oracle is evaluated with ``sumsq_numpy`` here.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import w8a8_oracle as O
from lynnreal_omni_b200 import workloads

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN / "w8a8_small.npz")


def f32(bits):
    return O.from_bf16_bits(bits)


def assert_bits(actual_f32, expected_bits):
    got = O.bf16_bits(actual_f32)
    np.testing.assert_array_equal(got, np.asarray(expected_bits, np.uint16))


@pytest.mark.parametrize("name", ["lin_a", "lin_b", "lin_c"])
def test_int8_linear_forward(g, name):
    x = f32(g[f"{name}.x"])
    bias = f32(g[f"{name}.bias"]) if f"{name}.bias" in g.files else None
    y = O.int8_linear_forward(x, g[f"{name}.w"], g[f"{name}.ws"], bias)
    assert_bits(y, g[f"{name}.y"])


def test_weight_quantisation(g):
    w = f32(g["wq.w"])
    q, s = O.quantize_weight(w)
    np.testing.assert_array_equal(q, g["wq.q"])
    np.testing.assert_array_equal(s, g["wq.s"])


@pytest.mark.parametrize("name", ["mm_a", "mm_b", "mm_c", "mm_d"])
def test_torch_matmul_kat(g, name):
    bias = f32(g[f"{name}.bias"]) if f"{name}.bias" in g.files else None
    y = O.int8_matmul(g[f"{name}.a"], g[f"{name}.b_nk"].T, g[f"{name}.rs"], g[f"{name}.cs"], bias)
    assert_bits(y, g[f"{name}.y"])


@pytest.mark.parametrize("name", ["pro_a", "pro_b", "pro_c"])
def test_prologue_kernels(g, name):
    x = f32(g[f"{name}.x"])
    y = f32(g[f"{name}.y"])
    b, s, d = x.shape
    x2, y2 = x.reshape(-1, d), y.reshape(-1, d)
    w = f32(g[f"{name}.w"])
    table = f32(g[f"{name}.table"])
    idx = g[f"{name}.idx"]
    eps = float(g[f"{name}.eps"][0])
    for slot, key in ((2, "gated2"), (5, "gated5")):
        assert_bits(O.gated_residual(x2, y2, table, idx, slot, sequence=s),
                    g[f"{name}.{key}"].reshape(-1, d))
    rms = O.rms_adaln(x2, w, eps, table, idx, 0, 1, sequence=s, reduce=O.sumsq_numpy)
    assert_bits(rms, g[f"{name}.rms01"].reshape(-1, d))
    for slots, key in (((0, 1), "01"), ((3, 4), "34")):
        q, sc = O.rms_adaln_quant_int8(x2, w, eps, table, idx, *slots, sequence=s, reduce=O.sumsq_numpy)
        np.testing.assert_array_equal(q, g[f"{name}.q{key}"])
        np.testing.assert_array_equal(sc, g[f"{name}.s{key}"])
    r, q, sc = O.residual_rms_quant(x2, y2, w, eps, table, idx, sequence=s, reduce=O.sumsq_numpy)
    assert_bits(r, g[f"{name}.rr"].reshape(-1, d))
    np.testing.assert_array_equal(q, g[f"{name}.rq"])
    np.testing.assert_array_equal(sc, g[f"{name}.rs"])


@pytest.mark.parametrize("name", ["qr_a", "qr_b", "qr_c", "qr_d"])
def test_quantize_rows(g, name):
    q, s = O.quantize_rows(f32(g[f"{name}.x"]))
    np.testing.assert_array_equal(q, g[f"{name}.q"])
    np.testing.assert_array_equal(s, g[f"{name}.s"])


def test_quantize_zero_rows(g):
    q, s = O.quantize_rows(np.zeros((2, 64), np.float32))
    np.testing.assert_array_equal(q, g["qr_zero.q"])
    np.testing.assert_array_equal(s, g["qr_zero.s"])


@pytest.mark.parametrize("name", ["sw_a", "sw_b", "sw_c"])
def test_swiglu(g, name):
    p = f32(g[f"{name}.p"])
    y = O.swiglu(p)
    # the interpreter's sigmoid uses np.exp like the oracle: exact
    assert_bits(y, g[f"{name}.y"])
    q, s = O.swiglu_quant_int8(p)
    np.testing.assert_array_equal(q, g[f"{name}.q"])
    np.testing.assert_array_equal(s, g[f"{name}.s"])


def test_int8_epilogue(g):
    bias = f32(g["epi.bias"])
    assert_bits(O.int8_epilogue(g["epi.acc"], g["epi.rs"], g["epi.cs"], bias), g["epi.y"])
    assert_bits(O.int8_epilogue(g["epi.acc"], g["epi.rs"], g["epi.cs"], None), g["epi.y_nobias"])


def test_tree_sum_is_a_sum():
    rng = np.random.default_rng(1)
    for width in (1, 192, 2048, 5376, 6144, 24576):
        v = rng.standard_normal((3, width)).astype(np.float32)
        exact = np.sum(v.astype(np.float64) ** 2, axis=1)
        np.testing.assert_allclose(O.sumsq_tree(v), exact, rtol=2e-6)


def test_qk_sums_are_sums():
    rng = np.random.default_rng(3)
    for width in (8, 64, 96, 128, 256):
        v = O.bf16_round(rng.standard_normal((5, width)).astype(np.float32))
        exact = np.sum(v.astype(np.float64) ** 2, axis=1)
        for rot in (width, width // 2):
            np.testing.assert_allclose(O.sumsq_qk(v, rot), exact, rtol=2e-6)


def test_bf16_rounding_matches_torch():
    rng = np.random.default_rng(2)
    v = (rng.standard_normal(100000) * np.exp(rng.uniform(-20, 20, 100000))).astype(np.float32)
    v[:4] = [0.0, -0.0, 1.00390625, 1.01171875]  # ties: 1 + 2^-8 rounds down, 1 + 3*2^-8 up
    expect = torch.from_numpy(v).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(O.bf16_bits(v), expect)


@pytest.mark.slow
def test_config0_fingerprint():
    """Full-size config 0 (M=1024, K=N=6144): the oracle's bf16 output hashes to
    the reference's own Int8Linear output."""
    import hashlib
    fp = json.loads((GOLDEN / "fingerprints.json").read_text())["config0"]
    x, pl = workloads.config0(seed=fp["seed"])
    y = O.int8_linear_forward(O.to_numpy_f32(x), pl.weight.numpy(), pl.scale.numpy(),
                              O.to_numpy_f32(pl.bias))
    assert hashlib.sha256(O.bf16_bits(y).tobytes()).hexdigest() == fp["sha256"]


def test_quantize_transformer_report_shape():
    report = json.loads((GOLDEN / "quantize_transformer.json").read_text())
    assert report["quantized_blocks"] == [1, 2]
    assert report["quantized_linears"] == 8


@pytest.mark.parametrize("name", ["qk_full", "qk_part", "qk_ord", "qk_96"])
def test_qk_norm_rope_golden(g, name):
    """The reference's Q/K RMSNorm+RoPE kernels (model/kernels.py:188-257,
    331-402), run by the interpreter, equal the oracle in the interpreter's
    sum order."""
    b, s, h, d, rot, ordered = (int(v) for v in g[f"{name}.dims"])
    qkv = f32(g[f"{name}.qkv"]).reshape(b, s, 3 * h * d)
    q = qkv[..., :h * d].reshape(-1, d)
    k = qkv[..., h * d:2 * h * d].reshape(-1, d)
    tokens = (np.arange(b * s * h) // h) % s
    for x, w, key in ((q, "wq", "qo"), (k, "wk", "ko")):
        ref = O.qk_norm_rope(x, f32(g[f"{name}.{w}"]), 1e-6, g[f"{name}.cos"], g[f"{name}.sin"], rot, tokens,
                             reduce=lambda v: O.sumsq_qk_reference(v, rot, bool(ordered)))
        assert_bits(ref, g[f"{name}.{key}"].reshape(-1, d))
