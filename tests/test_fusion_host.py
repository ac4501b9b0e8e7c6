"""CPU tests of the fused-block installer and the adaLN-table cache
(lynnreal_omni_b200.fusion, elementwise_fusion), following the contract of
model/fusion.py:101-162 and model/elementwise_fusion.py:22-30: which report
keys and values come back, which configurations are refused, and when an
adaLN table is computed, reused and evicted. No kernel runs here."""
from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch
import torch.nn.functional as F
from torch import nn

from lynnreal_omni_b200 import elementwise_fusion, fusion


class _CountingLinear(nn.Linear):
    def __init__(self, hidden):
        super().__init__(hidden, 6 * hidden)
        self.calls = 0

    def forward(self, x):
        self.calls += 1
        return super().forward(x)


class _Attn(nn.Module):
    def __init__(self):
        super().__init__()
        self.processor = None

    def set_processor(self, processor):
        self.processor = processor


class _Block(nn.Module):
    def __init__(self, hidden):
        super().__init__()
        self.adaln_linear = _CountingLinear(hidden)
        self.adaln_proj = SimpleNamespace(linear=self.adaln_linear, hidden_size=hidden)
        self.attn = _Attn()


class _Transformer(nn.Module):
    """forward(hidden_states, timestep=...) resolves every block's adaLN table."""

    def __init__(self, hidden=8, depth=2):
        super().__init__()
        self.transformer_blocks = nn.ModuleList([_Block(hidden) for _ in range(depth)])

    def forward(self, hidden_states, timestep=None):
        temb = timestep.float().view(-1, 1).expand(-1, hidden_states.shape[-1])
        return [fusion.resolve_adaln_table(block, temb) for block in self.transformer_blocks]


def _fused(model):
    fusion.enable_fusion(model)
    return fusion.cache_time_modulation(model)


def test_enable_fusion_report():
    model = _Transformer(depth=3)
    report = fusion.enable_fusion(model)
    assert report == dict(rmsnorm_adaln=True, qk_norm_rope=True, swiglu=True,
                          qk_output_allocation="contiguous_without_copy", residual_block=1024, gated_residual=True,
                          activation_quantization_fused=False, residual_ffn_norm_fused=False,
                          qk_ordered_reduction=False, int8_epilogue_fused=False, blocks=3, token_dropping=False)
    for block in model.transformer_blocks:
        assert isinstance(block.attn.processor, fusion.FusedAttention)
        assert block.forward.__func__ is fusion.guarded_block
    quant = fusion.enable_fusion(_Transformer(), fused_quant=True)
    assert quant["activation_quantization_fused"] and quant["residual_ffn_norm_fused"]
    assert quant["int8_epilogue_fused"] and quant["qk_ordered_reduction"]


def test_enable_fusion_keeps_the_first_native_entry_points():
    model = _Transformer(depth=1)
    block = model.transformer_blocks[0]
    native = block.forward
    fusion.enable_fusion(model)
    fusion.enable_fusion(model, fused_quant=True)
    assert block._lynnreal_native_forward == native
    assert block._lynnreal_native_processor is None
    assert block._lynnreal_fused_quant and block._lynnreal_residual_quant


@pytest.mark.parametrize("name", ["h3_attention_token_stride", "h3_ffn_token_stride", "h3_depth_span"])
def test_enable_fusion_refuses_strided_blocks(name):
    model = _Transformer(depth=2)
    setattr(model.transformer_blocks[1], name, 2)
    with pytest.raises(ValueError, match="dense attention and FFN"):
        fusion.enable_fusion(model)


def test_time_modulation_requires_fused_blocks():
    with pytest.raises(ValueError, match="requires fused blocks"):
        fusion.cache_time_modulation(_Transformer())


def test_time_modulation_report_and_frozen_inference():
    model = _Transformer().eval()
    report = _fused(model)
    assert report == {"kind": "exact AdaLN tables", "key": "complete input noise-time tensor",
                      "maximum_entries_per_block": 16, "requires_immutable_weights": True}
    x = torch.zeros(1, 4, 8)
    with pytest.raises(ValueError, match="frozen inference"):
        model(x, timestep=torch.tensor([3.0]))  # gradients enabled
    model.train()
    with torch.no_grad(), pytest.raises(ValueError, match="frozen inference"):
        model(x, timestep=torch.tensor([3.0]))


def test_time_modulation_caches_per_timestep_tensor():
    model = _Transformer().eval()
    _fused(model)
    x = torch.zeros(1, 4, 8)
    calls = lambda: [b.adaln_linear.calls for b in model.transformer_blocks]  # noqa: E731
    with torch.no_grad():
        first = model(x, timestep=torch.tensor([3.0]))
        assert calls() == [1, 1]
        again = model(x, timestep=torch.tensor([3.0]))
        assert calls() == [1, 1]
        assert all(a is b for a, b in zip(first, again))
        model(x, timestep=torch.tensor([3.0, 3.0]))  # another shape: another key
        model(x, timestep=torch.tensor([3.0], dtype=torch.float64))  # another dtype: another key
        assert calls() == [3, 3]
        # the cached table is the computed one
        block = model.transformer_blocks[0]
        temb = torch.full((1, 8), 3.0)
        expect = block.adaln_linear(F.silu(temb)).view(-1, 48)
        assert torch.equal(first[0], expect)


def test_time_modulation_evicts_oldest_first():
    model = _Transformer(depth=1).eval()
    _fused(model)
    block = model.transformer_blocks[0]
    x = torch.zeros(1, 4, 8)
    with torch.no_grad():
        for t in range(fusion.CACHE_ENTRIES):
            model(x, timestep=torch.tensor([float(t)]))
        assert len(block._lynnreal_adaln_cache) == fusion.CACHE_ENTRIES
        model(x, timestep=torch.tensor([100.0]))  # evicts timestep 0
        assert len(block._lynnreal_adaln_cache) == fusion.CACHE_ENTRIES
        n = block.adaln_linear.calls
        model(x, timestep=torch.tensor([1.0]))  # still cached
        assert block.adaln_linear.calls == n
        model(x, timestep=torch.tensor([0.0]))  # recomputed
        assert block.adaln_linear.calls == n + 1


def test_adaln_table_passed_in_wins():
    block = _Block(8)
    given = torch.ones(2, 48)
    assert fusion.resolve_adaln_table(block, torch.zeros(1, 8), given) is given
    assert block.adaln_linear.calls == 0


def test_elementwise_fusion_contract():
    model = _Transformer(depth=2).eval()
    report = elementwise_fusion.enable_elementwise_fusion(model)
    assert report == {"kind": "elementwise", "swiglu": True, "gated_residual": True, "normalization": "native",
                      "attention_processor": "native", "blocks": 2, "activation_quantization_fused": False}
    assert all(b.forward.__func__ is elementwise_fusion.block_forward for b in model.transformer_blocks)
    with pytest.raises(ValueError, match="evaluation-mode BF16"):
        elementwise_fusion.enable_elementwise_fusion(model, fused_quant=True)
    with pytest.raises(ValueError, match="evaluation-mode BF16"):
        elementwise_fusion.enable_elementwise_fusion(_Transformer().train())
