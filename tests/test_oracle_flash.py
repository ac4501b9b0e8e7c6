"""The token-compression oracle reproduces the reference's own outputs exactly.

Golden vectors: tests/golden/make_golden_flash.py (the reference's
``spatial_layout`` and ``configure_flash`` hooks run on the CPU).
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from flash_stub import CASES, StubTransformer
from oracle import flash_oracle as F
from oracle import w8a8_oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN / "flash_small.npz")


def bf(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


@pytest.mark.parametrize("name", ["grid", "odd", "groups", "orphan", "float"])
def test_spatial_layout(g, name):
    keep, inverse = F.spatial_layout(g[f"layout.{name}.positions"], g[f"layout.{name}.tags"])
    np.testing.assert_array_equal(keep, g[f"layout.{name}.keep"])
    np.testing.assert_array_equal(inverse, g[f"layout.{name}.inverse"])


def test_spatial_layout_rejects_what_the_reference_rejects():
    with pytest.raises(ValueError, match="single shared packed layout"):
        F.spatial_layout(np.zeros((4, 2)), np.zeros(4))
    with pytest.raises(ValueError, match="video tokens"):
        F.spatial_layout(np.zeros((4, 3)), np.ones(4))


def test_nearest_anchor_ties_take_the_first_anchor():
    pos = np.array([[0, 1, 1], [0, 0, 0], [0, 0, 2], [0, 2, 0], [0, 2, 2]], np.float32)
    assert F.nearest_anchor(pos, np.array([0]), np.array([4, 3, 2, 1]))[0] == 0
    assert F.nearest_anchor(pos, np.array([0]), np.array([1, 2, 3, 4]))[0] == 0


@pytest.mark.parametrize("name", list(CASES))
def test_hooked_forward(g, name):
    """StubTransformer with the reference's hook sequence (prefix blocks, one
    gather, compressed blocks on gathered indices/rotary/mask, restore, suffix
    blocks), every gather and the restore done by the oracle."""
    layout, _, _, layers, prefix, suffix, gain, with_mask = CASES[name]
    keep, inverse = F.spatial_layout(g[f"layout.{layout}.positions"], g[f"layout.{layout}.tags"])
    hidden = bf(g[f"{name}.hidden"])
    temb = bf(g[f"{name}.temb"])
    cos, sin = torch.from_numpy(g[f"{name}.cos"]), torch.from_numpy(g[f"{name}.sin"])
    idx = torch.from_numpy(g[f"{name}.indices"])
    mask = torch.from_numpy(g[f"{name}.mask"]) if with_mask else None
    blocks = StubTransformer(layers).transformer_blocks
    with torch.no_grad():
        for b in blocks[:prefix]:
            hidden = b(hidden, temb, idx, (cos, sin), mask)
        full = hidden
        take = lambda t, axis: torch.from_numpy(F.gather_rows(t.numpy(), keep, axis))  # noqa: E731
        hidden = bf(F.gather_rows(full.view(torch.int16).numpy(), keep, 1).view(np.uint16))
        start = hidden
        c_args = (take(idx, 0), (take(cos, -2), take(sin, -2)), None if mask is None else take(mask, -1))
        for b in blocks[prefix:layers - suffix]:
            hidden = b(hidden, temb, c_args[0], c_args[1], c_args[2])
        restored = F.restore(O.to_numpy_f32(full), O.to_numpy_f32(hidden), O.to_numpy_f32(start), inverse, gain)
        hidden = O.to_torch_bf16(restored)
        for b in blocks[layers - suffix:]:
            hidden = b(hidden, temb, idx, (cos, sin), mask)
    np.testing.assert_array_equal(hidden.view(torch.int16).numpy().view(np.uint16), g[f"{name}.out"])
