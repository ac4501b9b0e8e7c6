"""Generate the golden vectors of the W8A8 projection path from the reference itself.

Usage (needs the reference source tree, which the GPU box does not have):

    python tests/golden/make_golden.py <reference-root>

What runs, all on the CPU:
  * the reference's torch path: ``Int8Linear`` (model/int8.py), ``_torch_matmul``
    (model/int8_gemm.py:84-92) and ``quantize_transformer`` (model/int8.py:71-104);
  * the reference's Triton kernels (model/kernels.py) under the Triton
    interpreter (TRITON_INTERPRET=1), with two substitutions that give the
    interpreter the GPU's semantics:
      - the interpreter cannot run the libdevice ``nearbyint`` used by the
        quantising kernels, so the module global ``nearbyint`` is replaced by
        ``(x + 1.5*2**23) - 1.5*2**23``, which is round-half-to-even for
        |x| < 2**22 in float32 — the same function on the clamped range
        [-127, 127] it is applied to;
      - the interpreter truncates float32 -> bf16 casts, while compiled Triton
        rounds them to nearest even; its conversion is replaced by RNE;
      - the interpreter adds/multiplies bf16 operands as their raw uint16 bit
        patterns; bf16 arithmetic is replaced by float32 arithmetic rounded to
        bf16, as compiled Triton computes it.
    The interpreter reduces with ``np.sum`` over the kernel's power-of-two
    block (zero padded), which the oracle's ``sumsq_numpy`` reproduces.

Outputs (committed): w8a8_small.npz (inputs and outputs of every small case),
fingerprints.json (SHA-256 of full-size outputs whose inputs are regenerated
from seeds by lynnreal_omni_b200.workloads), quantize_transformer.json.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
from pathlib import Path
from types import SimpleNamespace

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402
import triton  # noqa: E402
import triton.language as tl  # noqa: E402,F401  (the interpreter needs it in this module's globals)
from torch import nn  # noqa: E402


from triton.runtime import interpreter as _interp  # noqa: E402


@triton.jit
def _rne(x):
    return (x + 12582912.0) - 12582912.0


_convert_float = _interp._convert_float


def _convert_float_rne(data, src, dst, rounding_mode):
    """float32 -> bf16 with round-to-nearest-even.

    On the GPU, Triton lowers ``.to(tl.bfloat16)`` and the implicit cast of a
    float32 value stored through a bf16 pointer to a round-to-nearest-even
    conversion; the interpreter's own cast truncates. Every other conversion
    keeps the interpreter's implementation.
    """
    if src == tl.float32 and dst == tl.bfloat16:
        u = np.frombuffer(np.ascontiguousarray(data).tobytes(), np.uint32).astype(np.uint64)
        r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
        return r.reshape(np.shape(data))
    return _convert_float(data, src, dst, rounding_mode)


_interp._convert_float = _convert_float_rne


def _bf16_arith(op):
    """bf16 (+, -, *, /) as compiled Triton does it: operate in float32 and
    round the result to bf16 (nearest even). The interpreter keeps bf16 values
    as uint16 bit patterns and would otherwise combine the raw integers."""
    def apply(self, lhs, rhs):
        if lhs.dtype.scalar != tl.bfloat16:
            return self.binary_op(lhs, rhs, op)
        a = (lhs.data.astype(np.uint32) << 16).view(np.float32)
        b = (rhs.data.astype(np.uint32) << 16).view(np.float32)
        r = op(a, b).astype(np.float32)
        return _interp.TensorHandle(_convert_float_rne(r, tl.float32, tl.bfloat16, None), tl.bfloat16)
    return apply


for _name, _op in (("create_fadd", np.add), ("create_fsub", np.subtract),
                   ("create_fmul", np.multiply), ("create_fdiv", np.divide)):
    setattr(_interp.InterpreterBuilder, _name, _bf16_arith(_op))


HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
from lynnreal_omni_b200 import workloads  # noqa: E402


def bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> uint16 bit pattern."""
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(bits(t).tobytes()).hexdigest()


def main(reference_root: str) -> None:
    sys.path.insert(0, reference_root)
    from model import int8 as ref_int8
    from model import int8_gemm as ref_gemm
    from model import kernels as ref_k

    ref_k.nearbyint = _rne
    out: dict[str, np.ndarray] = {}
    g = torch.Generator().manual_seed(20260)

    # ---- Int8Linear torch path (model/int8.py:26-68) ---------------------------
    for name, (m, k, n, with_bias) in {"lin_a": (67, 512, 384, True), "lin_b": (1, 256, 136, False),
                                       "lin_c": (9, 6144, 32, True)}.items():
        x = workloads.activations(m, k, g)
        pl = workloads.packed_linear(n, k, g, bias=with_bias)
        layer = ref_int8.Int8Linear.from_packed(pl.weight, pl.scale, pl.bias, gemm="torch")
        y = layer(x.view(1, m, k))
        out[f"{name}.x"] = bits(x)
        out[f"{name}.w"] = pl.weight.numpy()
        out[f"{name}.ws"] = pl.scale.numpy()
        if with_bias:
            out[f"{name}.bias"] = bits(pl.bias)
        out[f"{name}.y"] = bits(y.reshape(m, n))

    # ---- Int8Linear(source) weight quantisation (model/int8.py:7-20) ----------
    src = nn.Linear(96, 40, bias=True)
    with torch.no_grad():
        src.weight.copy_(torch.randn(40, 96, generator=g))
        src.bias.copy_(torch.randn(40, generator=g) * 0.1)
    layer = ref_int8.Int8Linear(src.to(torch.bfloat16), gemm="torch")
    out["wq.w"] = bits(src.weight)
    out["wq.q"] = layer.weight_int8.t().contiguous().numpy()
    out["wq.s"] = layer.weight_scale.t().contiguous().numpy()

    # ---- _torch_matmul, the reference's integer KAT (script/precompile.py:55-62)
    for name, (m, k, n, with_bias) in {"mm_a": (1, 64, 48, False), "mm_b": (7, 96, 40, True),
                                       "mm_c": (33, 256, 264, False), "mm_d": (130, 256, 136, True)}.items():
        a, b, rs, cs, bb = workloads.gemm_operands(m, k, n, seed=1000 + m, bias=with_bias)
        y = ref_gemm._torch_matmul(a, b, rs, cs, bb)
        out[f"{name}.a"] = a.numpy()
        out[f"{name}.b_nk"] = b.t().contiguous().numpy()
        out[f"{name}.rs"] = rs.numpy()
        out[f"{name}.cs"] = cs.numpy()
        if with_bias:
            out[f"{name}.bias"] = bits(bb)
        out[f"{name}.y"] = bits(y)

    # ---- Triton kernels under the interpreter (model/kernels.py) --------------
    def prologue_case(name, b, s, d, table_rows, eps, unit_weight=False):
        x = torch.randn(b, s, d, generator=g).to(torch.bfloat16)
        y = torch.randn(b, s, d, generator=g).to(torch.bfloat16)
        w = torch.ones(d, dtype=torch.bfloat16) if unit_weight else \
            (1 + 0.05 * torch.randn(d, generator=g)).to(torch.bfloat16)
        table = (0.3 * torch.randn(table_rows, 6 * d, generator=g)).to(torch.bfloat16)
        idx = torch.arange(s) % table_rows
        norm = SimpleNamespace(weight=w, eps=eps)
        out[f"{name}.x"] = bits(x)
        out[f"{name}.y"] = bits(y)
        out[f"{name}.w"] = bits(w)
        out[f"{name}.table"] = bits(table)
        out[f"{name}.idx"] = idx.numpy()
        out[f"{name}.eps"] = np.array([eps], np.float64)
        out[f"{name}.gated2"] = bits(ref_k._gated_residual(x, y, table, idx, 2))
        out[f"{name}.gated5"] = bits(ref_k._gated_residual(x, y, table, idx, 5))
        out[f"{name}.rms01"] = bits(ref_k._rms_adaln(x, norm, table, idx, 0, 1))
        q, sc = ref_k._rms_adaln_quant_int8(x, norm, table, idx, 0, 1)
        out[f"{name}.q01"], out[f"{name}.s01"] = q.numpy(), sc.numpy()
        q, sc = ref_k._rms_adaln_quant_int8(x, norm, table, idx, 3, 4)
        out[f"{name}.q34"], out[f"{name}.s34"] = q.numpy(), sc.numpy()
        r, q, sc = ref_k.residual_rms_quant(x, y, norm, table, idx)
        out[f"{name}.rr"], out[f"{name}.rq"], out[f"{name}.rs"] = bits(r), q.numpy(), sc.numpy()

    prologue_case("pro_a", 1, 37, 192, 3, 1e-6)
    prologue_case("pro_b", 2, 4, 5376, 2, 1e-5, unit_weight=True)
    prologue_case("pro_c", 1, 4, 6144, 1, 1e-6)

    for name, (rows, width) in {"qr_a": (37, 192), "qr_b": (5, 6144), "qr_c": (2, 24576),
                                "qr_d": (4, 200)}.items():
        x = workloads.activations(rows, width, g)
        q, sc = ref_k.quantize_rows(x)
        out[f"{name}.x"], out[f"{name}.q"], out[f"{name}.s"] = bits(x), q.numpy(), sc.numpy()
    zero = torch.zeros(2, 64, dtype=torch.bfloat16)
    q, sc = ref_k.quantize_rows(zero)
    out["qr_zero.q"], out["qr_zero.s"] = q.numpy(), sc.numpy()

    for name, (rows, inner) in {"sw_a": (9, 96), "sw_b": (3, 2048), "sw_c": (2, 14336)}.items():
        p = (2.0 * torch.randn(rows, 2 * inner, generator=g)).to(torch.bfloat16)
        out[f"{name}.p"] = bits(p)
        out[f"{name}.y"] = bits(ref_k._swiglu(p))
        q, sc = ref_k._swiglu_quant_int8(p)
        out[f"{name}.q"], out[f"{name}.s"] = q.numpy(), sc.numpy()

    acc = torch.randint(-2 ** 24, 2 ** 24, (13, 40), generator=g, dtype=torch.int32)
    rs = torch.rand(13, 1, generator=g) / 127
    cs = torch.rand(1, 40, generator=g) / 127
    bias = (0.02 * torch.randn(40, generator=g)).to(torch.bfloat16)
    out["epi.acc"], out["epi.rs"], out["epi.cs"] = acc.numpy(), rs.numpy(), cs.numpy()
    out["epi.bias"] = bits(bias)
    out["epi.y"] = bits(ref_k.int8_epilogue(acc, rs, cs, bias))
    out["epi.y_nobias"] = bits(ref_k.int8_epilogue(acc, rs, cs, None))

    # ---- Q/K RMSNorm + RoPE (model/kernels.py:188-257, 331-402), called the way
    # FusedAttention calls them (model/fusion.py:29-54): strided views into a
    # fused QKV output, fp32 cos/sin tables [S, rotary_dim]
    for name, (b, s, h, d, rot, ordered) in {"qk_full": (1, 5, 3, 128, 128, False),
                                             "qk_part": (2, 4, 2, 128, 64, False),
                                             "qk_ord": (1, 3, 2, 128, 32, True),
                                             "qk_96": (1, 6, 2, 96, 48, False)}.items():
        qkv = torch.randn(b, s, 3 * h * d, generator=g).to(torch.bfloat16)
        q, kk, _ = [t.unflatten(-1, (h, -1)) for t in qkv.chunk(3, dim=-1)]
        wq = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
        wk = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
        phase = torch.randn(s, rot, generator=g)
        cos, sin = phase.cos(), phase.sin()
        qo = torch.empty_like(q, memory_format=torch.contiguous_format)
        ko = torch.empty_like(kk, memory_format=torch.contiguous_format)
        common = (q, kk, wq, wk, cos, sin, qo, ko, s, h, q.stride(1), q.stride(2), kk.stride(1), kk.stride(2), d)
        grid = (q.numel() // d,)
        if rot == d:
            ref_k._qk_norm_full_rope_paired_kernel[grid](*common, 1e-6, triton.next_power_of_2(d // 2),
                                                         num_warps=4, enable_fp_fusion=False)
        else:
            ref_k._qk_norm_rope_kernel[grid](*common, rot, 1e-6, triton.next_power_of_2(d),
                                             ordered_reduction=ordered, num_warps=1 if ordered else 4,
                                             enable_fp_fusion=False)
        out[f"{name}.qkv"] = bits(qkv)
        out[f"{name}.wq"], out[f"{name}.wk"] = bits(wq), bits(wk)
        out[f"{name}.cos"], out[f"{name}.sin"] = cos.numpy(), sin.numpy()
        out[f"{name}.dims"] = np.array([b, s, h, d, rot, int(ordered)], np.int64)
        out[f"{name}.qo"], out[f"{name}.ko"] = bits(qo), bits(ko)

    np.savez_compressed(HERE / "w8a8_small.npz", **out)

    # ---- full-size fingerprints (inputs regenerated from seeds) --------------
    fp = {}
    x, pl = workloads.config0(seed=0)
    layer = ref_int8.Int8Linear.from_packed(pl.weight, pl.scale, pl.bias, gemm="torch")
    fp["config0"] = {"seed": 0, "m": 1024, "k": 6144, "n": 6144, "sha256": sha(layer(x))}
    for m, n, k in ((32, 21504, 5376), (32, 5376, 7168), (32, 28672, 5376), (32, 5376, 14336),
                    (300, 6144, 6144)):
        a, b, rs, cs, _ = workloads.gemm_operands(m, k, n, seed=219)
        fp[f"kat_{m}_{n}_{k}"] = {"seed": 219, "m": m, "n": n, "k": k,
                                  "sha256": sha(ref_gemm._torch_matmul(a, b, rs, cs, None))}
    (HERE / "fingerprints.json").write_text(json.dumps(fp, indent=1) + "\n")

    # ---- quantize_transformer on a stub transformer (model/int8.py:71-104) ----
    class Attn(nn.Module):
        def __init__(self, d):
            super().__init__()
            self.to_q, self.to_k, self.to_v = nn.Linear(d, d), nn.Linear(d, d), nn.Linear(d, d, bias=False)
            self.to_out = nn.ModuleList([nn.Linear(d, d), nn.Dropout(0.0)])

    class Proj(nn.Module):
        def __init__(self, d, f):
            super().__init__()
            self.proj = nn.Linear(d, f)

    class Block(nn.Module):
        def __init__(self, d, f):
            super().__init__()
            self.attn = Attn(d)
            self.ff = SimpleNamespace(net=nn.ModuleList([Proj(d, f), nn.Dropout(0.0), nn.Linear(f, d)]))

    torch.manual_seed(5)
    model = SimpleNamespace(transformer_blocks=[Block(32, 64) for _ in range(4)])
    report = ref_int8.quantize_transformer(model, protected_edges=1, gemm="torch")
    (HERE / "quantize_transformer.json").write_text(json.dumps(report, indent=1) + "\n")
    print("wrote", sorted(p.name for p in HERE.iterdir() if p.suffix in (".npz", ".json")))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    main(sys.argv[1])
