"""Golden vectors of Flash token compression, made by the reference itself.

Usage (needs the reference source tree, which the GPU box does not have):

    python tests/golden/make_golden_flash.py <reference-root>

Runs on the CPU: the reference's ``spatial_layout`` (model/flash.py:6-33) on
every layout of ``tests/flash_stub.py``, and its ``configure_flash`` hooks
(model/flash.py:36-94) installed on ``StubTransformer`` for every case there.
Writes flash_small.npz: per case the inputs, the reference's keep/inverse,
and the hooked transformer's output (bf16 bits).
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))

from flash_stub import CASES, StubTransformer, case_inputs, layouts  # noqa: E402


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main(reference_root: str) -> None:
    sys.path.insert(0, reference_root)
    from model import flash as ref_flash

    out = {}
    for name, (positions, tags) in layouts().items():
        keep, inverse = ref_flash.spatial_layout(positions, tags)
        out[f"layout.{name}.positions"] = positions.numpy()
        out[f"layout.{name}.tags"] = tags.numpy()
        out[f"layout.{name}.keep"] = keep.numpy()
        out[f"layout.{name}.inverse"] = inverse.numpy()
    for name in CASES:
        kwargs, config, layers = case_inputs(name)
        model = StubTransformer(layers).eval()
        ref_flash.configure_flash(model, config)
        with torch.no_grad():
            y = model(**kwargs)
        out[f"{name}.hidden"] = bits(kwargs["hidden_states"])
        out[f"{name}.temb"] = bits(kwargs["timestep"])
        out[f"{name}.cos"], out[f"{name}.sin"] = (v.numpy() for v in kwargs["rotary_emb"])
        out[f"{name}.indices"] = kwargs["adaln_indices"].numpy()
        if kwargs["attention_mask"] is not None:
            out[f"{name}.mask"] = kwargs["attention_mask"].numpy()
        out[f"{name}.out"] = bits(y)
    np.savez_compressed(HERE / "flash_small.npz", **out)
    print("wrote", HERE / "flash_small.npz", len(out), "arrays")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    main(sys.argv[1])
