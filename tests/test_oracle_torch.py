"""The multi-threaded torch-CPU port equals the numpy oracle bit for bit."""
from __future__ import annotations

import numpy as np
import torch

from oracle import w8a8_oracle as O
from oracle import w8a8_torch as T
from lynnreal_omni_b200 import block, workloads


def bits32(t: torch.Tensor) -> np.ndarray:
    return O.bf16_bits(t.numpy())


def test_quantize_and_matmul_equal():
    x, pl = workloads.config0(seed=4, m=37, k=512, n=264)
    q, s = T.quantize_rows(x)
    rq, rs = O.quantize_rows(O.to_numpy_f32(x))
    np.testing.assert_array_equal(q.numpy(), rq)
    np.testing.assert_array_equal(s.numpy(), rs)
    y = T.int8_matmul(q, pl.weight.t(), s, pl.scale, pl.bias)
    ry = O.int8_matmul(rq, pl.weight.numpy().T, rs, pl.scale.numpy(), O.to_numpy_f32(pl.bias))
    np.testing.assert_array_equal(bits32(y), O.bf16_bits(ry))


def test_rms_and_residual_equal():
    p = workloads.config1(seed=2, m=19, d=6144)
    x = p.x.view(19, 6144)
    for slots in ((0, 1), (3, 4)):
        a = T.rms_adaln(x, p.norm_weight, p.eps, p.table, p.indices, *slots)
        b = O.rms_adaln(O.to_numpy_f32(x), O.to_numpy_f32(p.norm_weight), p.eps, O.to_numpy_f32(p.table),
                        p.indices.numpy(), *slots)
        np.testing.assert_array_equal(bits32(a), O.bf16_bits(b))
    a = T.gated_residual(x, p.y.view(19, 6144), p.table, p.indices, 2)
    b = O.gated_residual(O.to_numpy_f32(x), O.to_numpy_f32(p.y.view(19, 6144)), O.to_numpy_f32(p.table),
                         p.indices.numpy(), 2)
    np.testing.assert_array_equal(bits32(a), O.bf16_bits(b))


def test_small_block_runs():
    w = block.make_weights(seed=1, hidden=256, ffn=512, text_dim=128)
    x, table, idx, ctx = block.make_inputs(24, seed=2, hidden=256, text_tokens=16, text_dim=128)
    h, kv = T.flash_block(x.view(24, 256), table, idx, ctx, w)
    assert h.shape == (24, 256) and kv.shape == (16, 512)
    assert torch.isfinite(h).all()
