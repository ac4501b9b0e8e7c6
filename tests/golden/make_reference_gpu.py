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
QK_CASES = [  # (name, tokens, heads, head_dim, rotary_dim, seed)
    ("qk_128_full", 64, 8, 128, 128, 21),
    ("qk_128_partial", 64, 8, 128, 64, 22),
    ("qk_96_full", 48, 4, 96, 96, 23),
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


def qk_inputs(tokens: int, heads: int, head_dim: int, rotary_dim: int, seed: int, device):
    """Seeded CPU inputs of one Q/K case: Q and K as strided views of a fused
    QKV output, norm modules and the rotary tables."""
    g = torch.Generator().manual_seed(seed)
    qkv = torch.randn(1, tokens, 3 * heads * head_dim, generator=g).to(torch.bfloat16).to(device)
    q, k, _ = [t.unflatten(-1, (heads, -1)) for t in qkv.chunk(3, dim=-1)]
    norms = [SimpleNamespace(weight=(1 + 0.05 * torch.randn(head_dim, generator=g)).to(torch.bfloat16).to(device),
                             eps=1e-6) for _ in range(2)]
    phase = torch.randn(tokens, rotary_dim, generator=g)
    return SimpleNamespace(q=q, k=k, norm_q=norms[0], norm_k=norms[1], cos=phase.cos().to(device),
                           sin=phase.sin().to(device))


def reference_qk(rk, inp):
    """The reference's Q/K kernels launched as its FusedAttention does
    (model/fusion.py:29-54; on B200 without the ordered reduction)."""
    import triton
    q, k = inp.q, inp.k
    _, s, h, d = q.shape
    rot = inp.cos.shape[-1]
    q_out = torch.empty_like(q, memory_format=torch.contiguous_format)
    k_out = torch.empty_like(k, memory_format=torch.contiguous_format)
    common = (q, k, inp.norm_q.weight, inp.norm_k.weight, inp.cos, inp.sin, q_out, k_out, s, h, q.stride(1),
              q.stride(2), k.stride(1), k.stride(2), d)
    grid = (q.numel() // d,)
    if rot == d:
        rk._qk_norm_full_rope_paired_kernel[grid](*common, float(inp.norm_q.eps), triton.next_power_of_2(d // 2),
                                                 num_warps=4, enable_fp_fusion=False)
    else:
        rk._qk_norm_rope_kernel[grid](*common, rot, float(inp.norm_q.eps), triton.next_power_of_2(d),
                                      num_warps=4, enable_fp_fusion=False)
    return q_out, k_out


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
    record["qk"] = {}
    for name, tokens, heads, head_dim, rot, seed in QK_CASES:
        out = reference_qk(rk, qk_inputs(tokens, heads, head_dim, rot, seed, "cuda"))
        record["qk"][name] = {"tokens": tokens, "heads": heads, "head_dim": head_dim, "rotary_dim": rot,
                              "seed": seed, "sha256": [digest(t) for t in out]}
    Path(out_path).write_text(json.dumps(record, indent=1) + "\n")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(ROOT / "tests" / "golden" / "reference_gpu.json"))
