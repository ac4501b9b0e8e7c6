"""A stand-in transformer for the Flash token-compression hooks (model/flash.py:36-94).

The hooks rewrite a block's five positional arguments (hidden, temb, adaLN
indices, rotary (cos, sin), attention mask) and restore the residual before
the first suffix block. ``StubBlock`` reads every one of them with
element-wise bf16 arithmetic only — each torch op rounds its fp32 result to
bf16 once, identically on the CPU and on the GPU — so the output of
``StubTransformer`` depends on the hooks' gathers and restore exactly, and a
CPU run of the reference's hooks can serve as the golden for a GPU run of
this package's hooks.

Layouts: ``layouts()`` builds packed (time, row, column) positions and token
tags (0 video, 1 text, 2 audio) covering the cases ``spatial_layout``
distinguishes: even and odd grids, offset and multi-grid coordinate
alphabets, interleaved non-video rows, a dropped row with no same-time
anchor, and non-integer time coordinates.
"""
from __future__ import annotations

import torch
from torch import nn


class StubBlock(nn.Module):
    def __init__(self, number: int):
        super().__init__()
        self.number = number

    def forward(self, hidden, temb, indices, rotary, mask):
        cos, sin = rotary
        row = (cos[:, :1] + sin[:, 1:2]).to(torch.bfloat16)  # [S, 1]
        shift = indices.to(torch.bfloat16)[:, None] * 0.25  # [S, 1]
        out = hidden * (1.0 - 0.0625 * self.number) + row * temb[:, None, :] + shift
        if mask is not None:
            out = out + mask[..., None].to(out.dtype)
        return out


class StubTransformer(nn.Module):
    def __init__(self, layers: int):
        super().__init__()
        self.transformer_blocks = nn.ModuleList(StubBlock(i) for i in range(layers))

    def forward(self, hidden_states, timestep, position_ids, token_tags, rotary_emb, adaln_indices,
                attention_mask=None):
        for block in self.transformer_blocks:
            hidden_states = block(hidden_states, timestep, adaln_indices, rotary_emb, attention_mask)
        return hidden_states


def flash_config(layers: int, prefix: int, suffix: int, gain: float) -> dict:
    return {"num_layers": layers,
            "token_compression": {"reduction": "select", "spatial_stride": 2, "preserve_text_tokens": True,
                                  "preserve_audio_tokens": True, "full_prefix_blocks": prefix,
                                  "full_suffix_blocks": suffix, "residual_gain": gain}}


def _grid(t_values, rows, cols):
    return [(t, h, w) for t in t_values for h in rows for w in cols]


def layouts() -> dict:
    """name -> (positions int64/float32 [S, 3], tags int64 [S])."""
    out = {}

    def pack(parts):
        pos, tag = [], []
        for kind, coords in parts:
            pos += coords
            tag += [kind] * len(coords)
        return pos, tag

    # even grid (last row/column appended to the stride-2 selection), text first, audio last
    p, t = pack([(1, [(0, 0, 0)] * 5), (0, _grid(range(3), range(6), range(8))), (2, [(k, 0, 0) for k in range(4)])])
    out["grid"] = (torch.tensor(p, dtype=torch.int64), torch.tensor(t, dtype=torch.int64))
    # odd grid with offset coordinates, text after the video
    p, t = pack([(0, _grid(range(2), range(3, 10), range(5))), (1, [(0, 0, 0)] * 3)])
    out["odd"] = (torch.tensor(p, dtype=torch.int64), torch.tensor(t, dtype=torch.int64))
    # a reference-image grid beside the video grid (union alphabets), audio between frames
    parts = [(0, _grid([-1], range(0, 8, 2), range(0, 8, 2)))]
    for frame in range(3):
        parts += [(0, _grid([frame], range(6), range(7))), (2, [(frame, 0, 0)] * 2)]
    p, t = pack(parts)
    out["groups"] = (torch.tensor(p, dtype=torch.int64), torch.tensor(t, dtype=torch.int64))
    # a frame whose only video row is dropped: no same-time anchor
    p, t = pack([(0, _grid(range(2), range(5), range(6))), (0, [(9, 1, 3)]), (1, [(0, 0, 0)] * 2)])
    out["orphan"] = (torch.tensor(p, dtype=torch.int64), torch.tensor(t, dtype=torch.int64))
    # float positions with non-integer times
    p, t = pack([(1, [(0.0, 0.0, 0.0)] * 2), (0, _grid([0.0, 0.5, 1.25], range(4), range(9)))])
    out["float"] = (torch.tensor(p, dtype=torch.float32), torch.tensor(t, dtype=torch.int64))
    return out


# name -> (layout, batch, hidden, layers, prefix, suffix, gain, with_mask)
CASES = {
    "grid_b1": ("grid", 1, 64, 5, 1, 2, 1.0, False),
    "grid_b2_gain": ("grid", 2, 64, 5, 2, 1, 0.75, True),
    "odd_ragged": ("odd", 1, 36, 4, 1, 1, 1.0, True),
    "groups": ("groups", 2, 40, 6, 2, 2, 1.0, False),
    "orphan_gain": ("orphan", 1, 24, 4, 1, 2, 1.5, False),
    "float": ("float", 1, 64, 4, 1, 1, 1.0, True),
}


def case_inputs(name: str, seed: int = 0):
    """Seeded CPU inputs of one case: (positions, tags, kwargs of StubTransformer.forward, config)."""
    layout, batch, hidden, layers, prefix, suffix, gain, with_mask = CASES[name]
    positions, tags = layouts()[layout]
    s = tags.numel()
    g = torch.Generator().manual_seed(seed + 1000 * len(name))
    kwargs = {
        "hidden_states": torch.randn(batch, s, hidden, generator=g).to(torch.bfloat16),
        "timestep": torch.randn(batch, hidden, generator=g).to(torch.bfloat16),
        "position_ids": positions,
        "token_tags": tags,
        "rotary_emb": (torch.randn(s, 16, generator=g), torch.randn(s, 16, generator=g)),
        "adaln_indices": torch.randint(0, 3, (s,), generator=g),
        "attention_mask": torch.randn(batch, s, generator=g) if with_mask else None,
    }
    return kwargs, flash_config(layers, prefix, suffix, gain), layers
