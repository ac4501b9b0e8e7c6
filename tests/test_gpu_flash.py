"""GPU tests of Flash token compression (lynnreal_omni_b200.flash).

Bars (all bit-exact):
  * spatial_layout on the device == the reference's keep/inverse (golden);
  * index_select / restore == the oracle, for every row width the gather
    kernel distinguishes and for ragged hidden sizes; at the full config-4
    size, sampled rows against the oracle;
  * a StubTransformer with this package's configure_flash hooks == the same
    model with the reference's hooks (golden), on every golden case.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from flash_stub import CASES, StubTransformer
from oracle import flash_oracle as F
from oracle import w8a8_oracle as O
from lynnreal_omni_b200 import _lib, flash

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
DEV = "cuda"


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN / "flash_small.npz")


def bf(bits, device=DEV):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(device)


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("name", ["grid", "odd", "groups", "orphan", "float"])
def test_spatial_layout_matches_reference(g, name):
    pos = torch.from_numpy(g[f"layout.{name}.positions"]).to(DEV)
    tags = torch.from_numpy(g[f"layout.{name}.tags"]).to(DEV)
    keep, inverse = flash.spatial_layout(pos, tags)
    np.testing.assert_array_equal(keep.cpu().numpy(), g[f"layout.{name}.keep"])
    np.testing.assert_array_equal(inverse.cpu().numpy(), g[f"layout.{name}.inverse"])


def test_spatial_layout_video_grid_full_size():
    """A 21 x 48 x 64 video grid (64512 rows, the config-4 latent): kept rows
    and every dropped row's anchor against the oracle."""
    t, h, w = torch.meshgrid(torch.arange(21), torch.arange(48), torch.arange(64), indexing="ij")
    pos = torch.stack([t, h, w], -1).reshape(-1, 3)
    tags = torch.zeros(pos.shape[0], dtype=torch.int64)
    keep, inverse = flash.spatial_layout(pos.to(DEV), tags.to(DEV))
    assert keep.numel() == 21 * 25 * 33
    rk, rinv = F.spatial_layout(pos.numpy(), tags.numpy())
    np.testing.assert_array_equal(keep.cpu().numpy(), rk)
    np.testing.assert_array_equal(inverse.cpu().numpy(), rinv)


@pytest.mark.parametrize("shape,dtype,dim", [
    ((2, 37, 40), torch.bfloat16, 1),     # 80-byte rows: 16-byte vectors, warp per row
    ((3, 50, 36), torch.bfloat16, 1),     # 72-byte rows: 8-byte vectors
    ((1, 300, 6144), torch.bfloat16, 1),  # hidden rows of the real width
    ((153, 16), torch.float32, -2),       # rotary rows
    ((153,), torch.int64, 0),             # adaLN indices
    ((2, 153), torch.float32, -1),        # mask columns, 4-byte rows
    ((2, 1, 153), torch.bool, -1),        # 1-byte rows
    ((5, 7, 3), torch.float16, 1),        # 6-byte rows: 2-byte vectors
])
def test_index_select_matches_oracle(shape, dtype, dim):
    gen = torch.Generator().manual_seed(len(shape) * 100 + shape[-1])
    src = torch.randn(shape, generator=gen)
    src = (src > 0) if dtype == torch.bool else (src * 1000).to(dtype)
    rows = shape[dim]
    index = torch.randint(0, rows, (rows // 2 + 3,), generator=gen)
    got = flash.index_select(src.to(DEV), dim, index.to(DEV))
    expect = F.gather_rows(src.numpy() if dtype != torch.bfloat16 else src.view(torch.int16).numpy(),
                           index.numpy(), dim)
    out = got.cpu()
    np.testing.assert_array_equal(out.view(torch.int16).numpy() if dtype == torch.bfloat16 else out.numpy(), expect)


def test_index_select_out_of_range_sets_status_and_zeros():
    _lib.device_status(clear=True)
    src = torch.ones(4, 64, device=DEV, dtype=torch.bfloat16)
    got = flash.index_select(src, 0, torch.tensor([1, 7, -1, 2], device=DEV))
    assert _lib.device_status(clear=True) & 4
    np.testing.assert_array_equal(got.float().cpu().numpy()[[1, 2]], 0.0)
    np.testing.assert_array_equal(got.float().cpu().numpy()[[0, 3]], 1.0)


@pytest.mark.parametrize("b,s,k,d,gain", [(2, 300, 77, 6144, 1.0), (1, 129, 40, 64, 0.75), (2, 61, 17, 36, 1.5),
                                          (1, 50, 13, 40, 1.0)])
def test_restore_matches_oracle(b, s, k, d, gain):
    gen = torch.Generator().manual_seed(s + d)
    full, comp, inp = (torch.randn(shape, generator=gen).to(torch.bfloat16) for shape in ((b, s, d), (b, k, d), (b, k, d)))
    inverse = torch.randint(0, k, (s,), generator=gen)
    got = flash.restore(full.to(DEV), comp.to(DEV), inp.to(DEV), inverse.to(DEV), gain)
    expect = F.restore(O.to_numpy_f32(full), O.to_numpy_f32(comp), O.to_numpy_f32(inp), inverse.numpy(), gain)
    np.testing.assert_array_equal(bits(got), O.bf16_bits(expect))


def test_restore_full_size_sampled_rows():
    """[1, 64512, 6144] from 17325 compressed rows; 256 sampled rows against the oracle."""
    b, s, k, d = 1, 64512, 17325, 6144
    gen = torch.Generator(device=DEV).manual_seed(3)
    full = torch.randn(b, s, d, device=DEV, generator=gen).to(torch.bfloat16)
    comp = torch.randn(b, k, d, device=DEV, generator=gen).to(torch.bfloat16)
    inp = torch.randn(b, k, d, device=DEV, generator=gen).to(torch.bfloat16)
    inverse = torch.randint(0, k, (s,), device=DEV, generator=gen)
    got = flash.restore(full, comp, inp, inverse, 1.0)
    rows = torch.randint(0, s, (256,), device=DEV, generator=gen)
    inv = inverse[rows]
    expect = F.restore(O.to_numpy_f32(full[:, rows].cpu()), O.to_numpy_f32(comp[:, inv].cpu()),
                       O.to_numpy_f32(inp[:, inv].cpu()), np.arange(256), 1.0)
    np.testing.assert_array_equal(bits(got[:, rows]), O.bf16_bits(expect))
    assert _lib.device_status(clear=True) == 0


def _case_kwargs(g, name):
    layout = CASES[name][0]
    kwargs = {
        "hidden_states": bf(g[f"{name}.hidden"]),
        "timestep": bf(g[f"{name}.temb"]),
        "position_ids": torch.from_numpy(g[f"layout.{layout}.positions"]).to(DEV),
        "token_tags": torch.from_numpy(g[f"layout.{layout}.tags"]).to(DEV),
        "rotary_emb": (torch.from_numpy(g[f"{name}.cos"]).to(DEV), torch.from_numpy(g[f"{name}.sin"]).to(DEV)),
        "adaln_indices": torch.from_numpy(g[f"{name}.indices"]).to(DEV),
        "attention_mask": torch.from_numpy(g[f"{name}.mask"]).to(DEV) if f"{name}.mask" in g.files else None,
    }
    return kwargs


@pytest.mark.parametrize("name", list(CASES))
def test_configure_flash_matches_reference_hooks(g, name):
    from flash_stub import flash_config
    _, _, _, layers, prefix, suffix, gain, _ = CASES[name]
    model = StubTransformer(layers).eval()
    flash.configure_flash(model, flash_config(layers, prefix, suffix, gain))
    kwargs = _case_kwargs(g, name)
    with torch.no_grad():
        first = model(**kwargs)
        second = model(**kwargs)  # cached layout, state cleared in between
    np.testing.assert_array_equal(bits(first), g[f"{name}.out"])
    np.testing.assert_array_equal(bits(second), g[f"{name}.out"])
    assert _lib.device_status(clear=True) == 0


def test_configure_flash_contract():
    from flash_stub import flash_config
    model = StubTransformer(4).eval()
    with pytest.raises(ValueError, match="prefix and suffix"):
        flash.configure_flash(model, flash_config(4, 0, 1, 1.0))
    flash.configure_flash(model, flash_config(4, 1, 1, 1.0))
    with pytest.raises(ValueError, match="already configured"):
        flash.configure_flash(model, flash_config(4, 1, 1, 1.0))
    x = torch.zeros(1, 3, 8, device=DEV, dtype=torch.bfloat16)
    pos = torch.tensor([[0, 0, 0], [0, 0, 1], [0, 1, 0]], device=DEV)
    with pytest.raises(ValueError, match="frozen inference"):
        model(x, x[:, 0], pos, torch.zeros(3, dtype=torch.int64, device=DEV),
              (torch.zeros(3, 4, device=DEV), torch.zeros(3, 4, device=DEV)), torch.zeros(3, dtype=torch.int64,
                                                                                        device=DEV))


def test_compressed_stack_equals_the_hook_schedule():
    """stack.FlashStackW8A8 with token compression (blocks [1, 3) of 4, two
    denoiser steps) equals the same blocks run with the reference hooks'
    schedule written in torch ops: gather the kept rows before block 1,
    restore full + ((out - in) * gain)[inverse] before block 3."""
    from lynnreal_omni_b200 import stack as S
    frames, height, width, hidden = 2, 6, 10, 256
    model = S.FlashStackW8A8(4, DEV, seed=5, hidden=hidden, ffn=512, text_dim=128, steps=2)
    comp = S.Compression(frames, height, width, DEV, start=1, end=3, gain=0.75)
    m = frames * height * width
    g = torch.Generator(device=DEV).manual_seed(9)
    x = torch.randn(1, m, hidden, device=DEV, generator=g).to(torch.bfloat16)
    ctx = torch.randn(16, 128, device=DEV, generator=g).to(torch.bfloat16)
    idx = torch.zeros(m, dtype=torch.int64, device=DEV)
    got = model.forward(x, idx, ctx, compression=comp)
    h = x
    for tables in model.tables:
        for i, (blk, table) in enumerate(zip(model.blocks, tables)):
            if i == 1:
                full, h = h, h.index_select(1, comp.keep)
                start = h
            if i == 3:
                h = full + ((h - start) * 0.75).index_select(1, comp.inverse)
            ids = idx.index_select(0, comp.keep) if 1 <= i < 3 else idx
            h, _ = blk(h, table, ids, ctx)
    assert torch.equal(got, h)
    assert comp.kept_rows() == frames * 4 * 6  # rows {0,2,4,5} x columns {0,2,4,6,8,9}
    assert _lib.device_status(clear=True) == 0
