"""GPU tests of the tcgen05 attention kernel (lynnreal_omni_b200.attention).

Reference: plain PyTorch fp32 attention of the same bf16 inputs (scores,
softmax and the weighted sum in fp32). Tolerance: the kernel rounds the
probabilities to bf16 for the second product and the output to bf16, so
|out - ref| <= 0.02 + 0.02 |ref| per element and relative L2 error <= 1e-2;
and it may not be worse than torch's own bf16 SDPA by more than 2x (+1e-3).
"""
from __future__ import annotations

import math

import pytest
import torch

from lynnreal_omni_b200 import _lib
from lynnreal_omni_b200.attention import attention_bshd

pytestmark = pytest.mark.gpu
DEV = "cuda"


def reference(q, k, v, scale):
    qf, kf, vf = (t.float().transpose(1, 2) for t in (q, k, v))  # [B, H, S, D]
    p = torch.softmax((qf @ kf.transpose(-1, -2)) * scale, dim=-1)
    return (p @ vf).transpose(1, 2)


def check_close(got, ref, q, k, v, scale):
    err = (got.float() - ref).abs()
    assert torch.all(err <= 0.02 + 0.02 * ref.abs()), float(err.max())
    rel = float(torch.linalg.vector_norm(got.float() - ref) / torch.linalg.vector_norm(ref))
    assert rel <= 1e-2, rel
    sdpa = torch.nn.functional.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                                            scale=scale).transpose(1, 2)
    rel_sdpa = float(torch.linalg.vector_norm(sdpa.float() - ref) / torch.linalg.vector_norm(ref))
    assert rel <= 2 * rel_sdpa + 1e-3, (rel, rel_sdpa)


@pytest.mark.parametrize("b,sq,skv,h,spread", [
    (1, 128, 128, 1, 1.0),     # one tile
    (2, 300, 300, 3, 1.0),     # ragged query and key tiles
    (1, 1000, 1000, 2, 1.0),
    (1, 200, 77, 4, 1.0),      # cross attention, one partial key tile
    (1, 96, 50, 2, 1.0),       # fewer than 64 keys: the second key half of every row is empty
    (1, 130, 64, 1, 4.0),      # exactly one key half
    (1, 257, 65, 2, 8.0),      # the second key half holds one key
    (1, 4096, 4096, 2, 1.0),   # long rows: 32 key tiles
    (2, 513, 640, 2, 4.0),     # peaked scores: the running max moves often
])
def test_attention_matches_fp32(b, sq, skv, h, spread):
    g = torch.Generator(device=DEV).manual_seed(sq * 7 + skv + h)
    q = (spread * torch.randn(b, sq, h, 128, device=DEV, generator=g)).to(torch.bfloat16)
    k = (spread * torch.randn(b, skv, h, 128, device=DEV, generator=g)).to(torch.bfloat16)
    v = torch.randn(b, skv, h, 128, device=DEV, generator=g).to(torch.bfloat16)
    scale = 1.0 / math.sqrt(128)
    got = attention_bshd(q, k, v)
    check_close(got, reference(q, k, v, scale), q, k, v, scale)
    assert _lib.device_status(clear=True) == 0


def test_attention_on_fused_qkv_views():
    """Q/K/V as strided views of one [B, S, 3*H*D] projection output."""
    b, s, h = 2, 333, 4
    g = torch.Generator(device=DEV).manual_seed(5)
    qkv = torch.randn(b, s, 3 * h * 128, device=DEV, generator=g).to(torch.bfloat16)
    q, k, v = [t.unflatten(-1, (h, -1)) for t in qkv.chunk(3, dim=-1)]
    got = attention_bshd(q, k, v)
    scale = 1.0 / math.sqrt(128)
    check_close(got, reference(q, k, v, scale), q, k, v, scale)


def test_attention_on_misaligned_views():
    """Views whose rows are not 16-byte aligned are copied, not refused."""
    b, s, h = 1, 130, 2
    g = torch.Generator(device=DEV).manual_seed(11)
    base = torch.randn(b, s, h * 128 + 4, device=DEV, generator=g).to(torch.bfloat16)
    q = base[..., 4:].unflatten(-1, (h, 128))  # token stride 260: rows 8-byte aligned only
    k = torch.randn(b, s, h, 128, device=DEV, generator=g).to(torch.bfloat16)
    v = torch.randn(b, s, h, 128, device=DEV, generator=g).to(torch.bfloat16)
    scale = 1.0 / math.sqrt(128)
    check_close(attention_bshd(q, k, v), reference(q, k, v, scale), q, k, v, scale)


def test_attention_rejects_unsupported():
    x = torch.zeros(1, 8, 2, 64, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        attention_bshd(x, x, x)
    y = torch.zeros(1, 8, 2, 128, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        attention_bshd(y, y, y, attn_mask=torch.ones(1, 1, 8, 8, device=DEV, dtype=torch.bool))
