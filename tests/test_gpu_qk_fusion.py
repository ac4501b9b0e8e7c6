"""GPU tests of the Q/K RMSNorm+RoPE kernel and of the fused-block caller.

Q/K bar: bit-exact against the oracle evaluated in the kernels' documented
sum order (8-element chunks per lane + xor butterfly); against the reference's own
kernels (golden vectors; their sums run in another order) at most 1 bf16 ulp
on at most 0.5 % of the elements.

Caller bar: ``fusion.fused_block`` on a block with the reference block's
interface (adaln_proj, norm1/norm2, attn.to_qkv/to_out/norm_q/norm_k, ff.net)
produces exactly the output of the same kernels called one by one in the
reference's order (model/fusion.py:61-98).
"""
from __future__ import annotations

from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest
import torch
import torch.nn.functional as F
from torch import nn

from oracle import w8a8_oracle as O
from lynnreal_omni_b200 import _lib, fusion, kernels as K, workloads
from lynnreal_omni_b200.attention import attention_bshd
from lynnreal_omni_b200.int8 import Int8Linear

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
DEV = "cuda"


def bf_dev(bits_or_f32):
    a = np.asarray(bits_or_f32)
    if a.dtype != np.uint16:
        a = O.bf16_bits(a)
    return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).to(DEV)


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def ulp_census(got, ref):
    key = lambda v: np.where(v & 0x8000, -(v & 0x7FFF), v.astype(np.int32))  # noqa: E731
    d = np.abs(key(got.astype(np.int32)) - key(ref.astype(np.int32)))
    return d.max(), (d > 0).mean()


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN / "w8a8_small.npz")


@pytest.mark.parametrize("name", ["qk_full", "qk_part", "qk_ord", "qk_96"])
def test_qk_norm_rope_vs_oracle_and_reference(g, name):
    b, s, h, d, rot, ordered = (int(v) for v in g[f"{name}.dims"])
    qkv = bf_dev(g[f"{name}.qkv"]).view(b, s, 3 * h * d)
    q, k, _ = [t.unflatten(-1, (h, -1)) for t in qkv.chunk(3, dim=-1)]
    nq = SimpleNamespace(weight=bf_dev(g[f"{name}.wq"]), eps=1e-6)
    nk = SimpleNamespace(weight=bf_dev(g[f"{name}.wk"]), eps=1e-6)
    cos = torch.from_numpy(g[f"{name}.cos"]).to(DEV)
    sin = torch.from_numpy(g[f"{name}.sin"]).to(DEV)
    qo, ko = K.qk_norm_rope(q, k, nq, nk, (cos, sin))
    tokens = (np.arange(b * s * h) // h) % s
    qkv_np = O.from_bf16_bits(g[f"{name}.qkv"]).reshape(b, s, 3 * h * d)
    for out, x, w, key in ((qo, qkv_np[..., :h * d], "wq", "qo"), (ko, qkv_np[..., h * d:2 * h * d], "wk", "ko")):
        ref = O.qk_norm_rope(x.reshape(-1, d), O.from_bf16_bits(g[f"{name}.{w}"]), 1e-6, g[f"{name}.cos"],
                             g[f"{name}.sin"], rot, tokens)
        np.testing.assert_array_equal(bits(out).reshape(-1, d), O.bf16_bits(ref))
        mx, frac = ulp_census(bits(out).reshape(-1), g[f"{name}.{key}"].reshape(-1))
        assert mx <= 1 and frac <= 0.005, (mx, frac)


@pytest.mark.parametrize("b,s,h,d,rot", [(1, 9, 4, 64, 64), (2, 3, 3, 256, 128), (1, 17, 48, 128, 128),
                                         (1, 5, 2, 128, 0)])
def test_qk_norm_rope_shapes(b, s, h, d, rot):
    gen = torch.Generator().manual_seed(b * 100 + s + h + d)
    qkv = torch.randn(b, s, 3 * h * d, generator=gen).to(torch.bfloat16)
    wq = (1 + 0.1 * torch.randn(d, generator=gen)).to(torch.bfloat16)
    wk = (1 + 0.1 * torch.randn(d, generator=gen)).to(torch.bfloat16)
    phase = torch.randn(s, rot, generator=gen)
    q, k, _ = [t.unflatten(-1, (h, -1)) for t in qkv.to(DEV).chunk(3, dim=-1)]
    qo, ko = K.qk_norm_rope(q, k, SimpleNamespace(weight=wq.to(DEV), eps=1e-6),
                            SimpleNamespace(weight=wk.to(DEV), eps=1e-6),
                            (phase.cos().to(DEV), phase.sin().to(DEV)))
    tokens = (np.arange(b * s * h) // h) % s
    x = O.to_numpy_f32(qkv)
    for out, part, w in ((qo, 0, wq), (ko, 1, wk)):
        rows = x[..., part * h * d:(part + 1) * h * d].reshape(-1, d)
        ref = O.qk_norm_rope(rows, O.to_numpy_f32(w), 1e-6, phase.cos().numpy(), phase.sin().numpy(), rot, tokens)
        np.testing.assert_array_equal(bits(out).reshape(-1, d), O.bf16_bits(ref))


@pytest.mark.parametrize("d,rot", [(128, 128), (64, 32), (256, 0)])
def test_qk_general_layout_equals_fast_layout(d, rot):
    """Head rows with padding between heads take the general kernel; its sum
    order is the fast kernel's, so the bits agree."""
    b, s, h = 2, 7, 5
    gen = torch.Generator().manual_seed(d + rot)
    qkv = torch.randn(b, s, 3 * h * d, generator=gen).to(torch.bfloat16).to(DEV)
    q, k, _ = [t.unflatten(-1, (h, -1)) for t in qkv.chunk(3, dim=-1)]
    padded = torch.zeros(2, b, s, h, d + 8, dtype=torch.bfloat16, device=DEV)
    padded[0, ..., :d], padded[1, ..., :d] = q, k
    norm = SimpleNamespace(weight=(1 + 0.1 * torch.randn(d, generator=gen)).to(torch.bfloat16).to(DEV), eps=1e-6)
    phase = torch.randn(s, rot, generator=gen).to(DEV)
    rope = (phase.cos(), phase.sin())
    fast = K.qk_norm_rope(q, k, norm, norm, rope)
    general = K.qk_norm_rope(padded[0, ..., :d], padded[1, ..., :d], norm, norm, rope)
    for a, c in zip(fast, general):
        assert torch.equal(a, c)


def test_qk_norm_rope_rejects_odd_rotary():
    q = torch.zeros(1, 2, 1, 8, dtype=torch.bfloat16, device=DEV)
    n = SimpleNamespace(weight=torch.ones(8, dtype=torch.bfloat16, device=DEV), eps=1e-6)
    with pytest.raises(ValueError):
        K.qk_norm_rope(q, q, n, n, (torch.ones(2, 3, device=DEV), torch.zeros(2, 3, device=DEV)))


# ------------------------------------------------------------- fused block
class _Norm(nn.Module):
    def __init__(self, d, gen, eps=1e-6):
        super().__init__()
        self.weight = nn.Parameter((1 + 0.05 * torch.randn(d, generator=gen)).to(torch.bfloat16),
                                   requires_grad=False)
        self.eps = eps


class _Attn(nn.Module):
    def __init__(self, hidden, heads, gen):
        super().__init__()
        self.heads = heads
        hd = hidden // heads
        mk = lambda n, k: Int8Linear.from_packed(*_packed(n, k, gen))  # noqa: E731
        self.to_qkv = mk(3 * hidden, hidden)
        self.to_out = nn.ModuleList([mk(hidden, hidden), nn.Dropout(0.0)])
        self.norm_q, self.norm_k = _Norm(hd, gen), _Norm(hd, gen)
        self.fused_projections = True
        self.processor = None

    def set_processor(self, processor):
        self.processor = processor

    def forward(self, hidden_states, rotary_emb=None, attention_mask=None):
        return self.processor(self, hidden_states, rotary_emb, attention_mask)


class _Up(nn.Module):
    def __init__(self, proj):
        super().__init__()
        self.proj = proj


class _FF(nn.Module):
    def __init__(self, hidden, inner, gen):
        super().__init__()
        self.net = nn.ModuleList([_Up(Int8Linear.from_packed(*_packed(2 * inner, hidden, gen))), nn.Dropout(0.0),
                                  Int8Linear.from_packed(*_packed(hidden, inner, gen))])


class _Block(nn.Module):
    """The interface of the reference's H3 block that fused_block uses."""

    def __init__(self, hidden, heads, inner, gen):
        super().__init__()
        lin = nn.Linear(hidden, 6 * hidden).to(torch.bfloat16)
        with torch.no_grad():
            lin.weight.copy_((0.02 * torch.randn(6 * hidden, hidden, generator=gen)).to(torch.bfloat16))
            lin.bias.copy_((0.02 * torch.randn(6 * hidden, generator=gen)).to(torch.bfloat16))
        self.adaln_linear = lin
        self.adaln_proj = SimpleNamespace(linear=lin, hidden_size=hidden)
        self.norm1, self.norm2 = _Norm(hidden, gen), _Norm(hidden, gen)
        self.attn = _Attn(hidden, heads, gen)
        self.ff = _FF(hidden, inner, gen)


def _packed(n, k, gen):
    p = workloads.packed_linear(n, k, gen)
    return p.weight, p.scale, p.bias


def manual_block(block, x, temb, idx, rot, hidden, heads):
    """The fused block's kernels called one by one in the reference's order
    (model/fusion.py:61-98)."""
    lin = block.adaln_proj.linear
    table = lin(F.silu(temb).to(lin.weight.dtype)).view(-1, 6 * hidden)
    q8, sc = K._rms_adaln_quant_int8(x, block.norm1, table, idx, 0, 1)
    qkv = block.attn.to_qkv.forward_quantized(q8, sc, x.shape[:-1])
    q, k, v = [t.unflatten(-1, (heads, -1)) for t in qkv.chunk(3, dim=-1)]
    qo, ko = K.qk_norm_rope(q, k, block.attn.norm_q, block.attn.norm_k, rot)
    att = attention_bshd(qo, ko, v)
    ao = block.attn.to_out[0](att.flatten(2, 3).type_as(qo))
    h, q8, sc = K.residual_rms_quant(x, ao, block.norm2, table, idx)
    proj = block.ff.net[0].proj.forward_quantized(q8, sc, h.shape[:-1])
    q8, sc = K._swiglu_quant_int8(proj)
    out = block.ff.net[2].forward_quantized(q8, sc, proj.shape[:-1])
    return K._gated_residual(h, out, table, idx, 5)


def test_fused_block_runs_the_reference_sequence():
    gen = torch.Generator().manual_seed(61)
    hidden, heads, inner, s = 512, 4, 768, 300
    block = _Block(hidden, heads, inner, gen).to(DEV)
    report = fusion.enable_fusion(SimpleNamespace(transformer_blocks=[block]), fused_quant=True)
    assert report["residual_ffn_norm_fused"] and report["activation_quantization_fused"]
    x = torch.randn(1, s, hidden, generator=gen).to(torch.bfloat16).to(DEV)
    temb = torch.randn(1, hidden, generator=gen).to(torch.bfloat16).to(DEV)
    idx = torch.zeros(s, dtype=torch.int64, device=DEV)
    phase = torch.randn(s, hidden // heads, generator=gen).to(DEV)
    rot = (phase.cos(), phase.sin())
    got = block.forward(x, temb, idx, rot)

    expect = manual_block(block, x, temb, idx, rot, hidden, heads)
    assert torch.equal(got, expect)
    assert _lib.device_status(clear=True) == 0


def test_flash_block_module_through_enable_fusion():
    """lynnreal_omni_b200.flash_block.FlashH3Block (released Flash block layout,
    reduced widths here) runs through enable_fusion and equals the manual
    kernel sequence."""
    from lynnreal_omni_b200 import flash_block as FB
    hidden, heads = 512, 4
    block = FB.FlashH3Block(seed=3, device=DEV, hidden=hidden, heads=heads, ffn_inner=640).eval()
    fusion.enable_fusion(SimpleNamespace(transformer_blocks=[block]), fused_quant=True)
    x, temb, idx, rot = FB.make_inputs(257, seed=4, device=DEV, hidden=hidden)
    with torch.no_grad():
        got = block.forward(x, temb, idx, rot)
        expect = manual_block(block, x, temb, idx, rot, hidden, heads)
    assert torch.equal(got, expect)
    assert torch.isfinite(got.float()).all()
    assert _lib.device_status(clear=True) == 0


# ------------------------------------------------------- bf16 block routes
def _bf16_linear(n_in, n_out, gen):
    lin = nn.Linear(n_in, n_out).to(torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_((torch.randn(n_out, n_in, generator=gen) / n_in ** 0.5).to(torch.bfloat16))
        lin.bias.copy_((0.02 * torch.randn(n_out, generator=gen)).to(torch.bfloat16))
    return lin


def _native_norm(d, gen):
    norm = nn.RMSNorm(d, eps=1e-6).to(torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_((1 + 0.05 * torch.randn(d, generator=gen)).to(torch.bfloat16))
    return norm


class _Bf16Attn(_Attn):
    """Unquantised projections (no ``forward_quantized``): the bf16 route."""

    def __init__(self, hidden, heads, gen):
        nn.Module.__init__(self)
        self.heads = heads
        self.to_qkv = _bf16_linear(hidden, 3 * hidden, gen)
        self.to_out = nn.ModuleList([_bf16_linear(hidden, hidden, gen), nn.Dropout(0.0)])
        self.norm_q, self.norm_k = _Norm(hidden // heads, gen), _Norm(hidden // heads, gen)
        self.fused_projections = True
        self.processor = None


class _NativeAttn(nn.Module):
    """Stands in for a native attention module: (x, rotary, mask) -> x W^T + b."""

    def __init__(self, hidden, gen):
        super().__init__()
        self.proj = _bf16_linear(hidden, hidden, gen)

    def forward(self, hidden_states, rotary_emb=None, attention_mask=None):
        return self.proj(hidden_states)


class _Bf16Block(_Block):
    def __init__(self, hidden, heads, inner, gen, native_modules):
        super().__init__(hidden, heads, inner, gen)
        if native_modules:
            self.norm1, self.norm2 = _native_norm(hidden, gen), _native_norm(hidden, gen)
            self.attn = _NativeAttn(hidden, gen)
        else:
            self.attn = _Bf16Attn(hidden, heads, gen)
        self.ff.net = nn.ModuleList([_Up(_bf16_linear(hidden, 2 * inner, gen)), nn.Dropout(0.0),
                                     _bf16_linear(inner, hidden, gen)])


def _block_inputs(gen, s, hidden, heads, rows=1):
    x = torch.randn(1, s, hidden, generator=gen).to(torch.bfloat16).to(DEV)
    temb = torch.randn(rows, hidden, generator=gen).to(torch.bfloat16).to(DEV)
    idx = torch.randint(0, rows, (s,), generator=gen).to(DEV)
    phase = torch.randn(s, hidden // heads, generator=gen).to(DEV)
    return x, temb, idx, (phase.cos(), phase.sin())


def test_fused_block_bf16_route():
    """enable_fusion without quantisation: the bf16 route of
    model/fusion.py:81-98 (RMSNorm+adaLN kernel, bf16 projections, gated
    residual, SwiGLU), equal to the kernels called one by one."""
    gen = torch.Generator().manual_seed(71)
    hidden, heads, inner, s = 512, 4, 768, 260
    block = _Bf16Block(hidden, heads, inner, gen, native_modules=False).to(DEV)
    fusion.enable_fusion(SimpleNamespace(transformer_blocks=[block]))
    x, temb, idx, rot = _block_inputs(gen, s, hidden, heads, rows=3)
    with torch.no_grad():
        got = block.forward(x, temb, idx, rot)
        lin = block.adaln_proj.linear
        table = lin(F.silu(temb).to(lin.weight.dtype)).view(-1, 6 * hidden)
        qkv = block.attn.to_qkv(K._rms_adaln(x, block.norm1, table, idx, 0, 1))
        q, k, v = [t.unflatten(-1, (heads, -1)) for t in qkv.chunk(3, dim=-1)]
        qo, ko = K.qk_norm_rope(q, k, block.attn.norm_q, block.attn.norm_k, rot)
        ao = block.attn.to_out[0](attention_bshd(qo, ko, v).flatten(2, 3).type_as(qo))
        h = K._gated_residual(x, ao, table, idx, 2)
        proj = block.ff.net[0].proj(K._rms_adaln(h, block.norm2, table, idx, 3, 4))
        expect = K._gated_residual(h, block.ff.net[2](K._swiglu(proj)), table, idx, 5)
    assert torch.equal(got, expect)
    assert _lib.device_status(clear=True) == 0


def test_elementwise_block_matches_reference_composition():
    """enable_elementwise_fusion: native norms and attention, gated residuals
    and SwiGLU on the kernels; equal to model/elementwise_fusion.py:7-19
    written out with table.chunk(6)."""
    from lynnreal_omni_b200 import elementwise_fusion
    gen = torch.Generator().manual_seed(72)
    hidden, heads, inner, s = 512, 4, 768, 301
    block = _Bf16Block(hidden, heads, inner, gen, native_modules=True).to(DEV).eval()
    elementwise_fusion.enable_elementwise_fusion(SimpleNamespace(transformer_blocks=[block], training=False))
    x, temb, idx, rot = _block_inputs(gen, s, hidden, heads, rows=2)
    with torch.no_grad():
        got = block.forward(x, temb, idx, rot)
        lin = block.adaln_proj.linear
        table = lin(F.silu(temb).to(lin.weight.dtype)).view(-1, 6 * hidden)
        shift, scale, _, ff_shift, ff_scale, _ = table.chunk(6, dim=-1)
        n = block.norm1(x) * (1 + scale.index_select(0, idx)) + shift.index_select(0, idx)
        h = K._gated_residual(x, block.attn(n, rot, None), table, idx, 2)
        n = block.norm2(h) * (1 + ff_scale.index_select(0, idx)) + ff_shift.index_select(0, idx)
        update = block.ff.net[2](K._swiglu(block.ff.net[0].proj(n)))
        expect = K._gated_residual(h, update, table, idx, 5)
    assert torch.equal(got, expect)
    assert torch.isfinite(got.float()).all()
    assert _lib.device_status(clear=True) == 0
