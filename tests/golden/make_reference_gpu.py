"""Record the reference's compiled Triton kernels' outputs on a B200.

Usage (on a GPU box, with the reference installed into baseline/_ref by
``pip install --no-index --no-build-isolation --no-deps --target baseline/_ref
<copy of the reference>``):

    python tests/golden/make_reference_gpu.py [out.json]

Inputs are regenerated from seeds on the CPU (``reference_gpu_inputs`` below,
also imported by the test), so only SHA-256 digests of the outputs are stored:
``tests/golden/reference_gpu.json``. The digests pin what the reference
computes on the GPU (div.full / rsqrt.approx arithmetic, its compiled tl.sum
order), which its Triton interpreter and its torch path do not reproduce.
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path
from types import SimpleNamespace

import torch

ROOT = Path(__file__).resolve().parents[2]
CASES = [  # (name, rows, width, seed)
    ("rms_6144", 96, 6144, 11),
    ("rms_5376", 80, 5376, 12),
    ("rms_4096", 64, 4096, 13),
    ("quant_24576", 48, 24576, 14),
    ("swiglu_14336", 48, 14336, 15),
    ("swiglu_2688", 40, 2688, 16),
]


def reference_gpu_inputs(rows: int, width: int, seed: int, device):
    """Seeded CPU inputs of one case (bf16), moved to `device`."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(1, rows, width, generator=g).to(torch.bfloat16)
    y = torch.randn(1, rows, width, generator=g).to(torch.bfloat16)
    weight = (1 + 0.05 * torch.randn(width, generator=g)).to(torch.bfloat16)
    table = (0.1 * torch.randn(3, 6 * width, generator=g)).to(torch.bfloat16)
    idx = torch.randint(0, 3, (rows,), generator=g)
    proj = (2 * torch.randn(rows, 2 * width, generator=g)).to(torch.bfloat16)
    to = lambda t: t.to(device)  # noqa: E731
    return SimpleNamespace(x=to(x), y=to(y), norm=SimpleNamespace(weight=to(weight), eps=1e-6), table=to(table),
                           idx=to(idx), proj=to(proj))


def digest(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().contiguous().cpu().view(torch.uint8).numpy().tobytes()).hexdigest()


def outputs(mod, kind: str, inp):
    """The outputs of one case through `mod` (the reference's or this package's kernels module)."""
    rows, width = inp.x.shape[1], inp.x.shape[2]
    if kind == "rms":
        out = {}
        out["quantize_rows"] = mod.quantize_rows(inp.x.view(rows, width))
        for slots in ((0, 1), (3, 4)):
            out[f"rms_adaln_quant_{slots[0]}{slots[1]}"] = mod._rms_adaln_quant_int8(inp.x, inp.norm, inp.table,
                                                                                    inp.idx, *slots)
            out[f"rms_adaln_{slots[0]}{slots[1]}"] = (mod._rms_adaln(inp.x, inp.norm, inp.table, inp.idx, *slots),)
        out["residual_rms_quant"] = mod.residual_rms_quant(inp.x, inp.y, inp.norm, inp.table, inp.idx)
        out["gated_residual"] = (mod._gated_residual(inp.x, inp.y, inp.table, inp.idx, 5),)
        return out
    if kind == "quant":
        return {"quantize_rows": mod.quantize_rows(inp.x.view(rows, width))}
    return {"swiglu": (mod._swiglu(inp.proj),), "swiglu_quant": mod._swiglu_quant_int8(inp.proj)}


def main(out_path: str) -> None:
    sys.path.insert(0, str(ROOT / "baseline" / "_ref"))
    import lynnreal.model.kernels as rk
    record = {"gpu": torch.cuda.get_device_name(0), "cases": {}}
    for name, rows, width, seed in CASES:
        inp = reference_gpu_inputs(rows, width, seed, "cuda")
        res = outputs(rk, name.split("_")[0], inp)
        record["cases"][name] = {"rows": rows, "width": width, "seed": seed,
                                 "sha256": {k: [digest(t) for t in v] for k, v in res.items()}}
    Path(out_path).write_text(json.dumps(record, indent=1) + "\n")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(ROOT / "tests" / "golden" / "reference_gpu.json"))
