"""W8A8 projections of the DiT blocks on the sm_100a kernels.

The interface is the one of model/int8.py:6-104, kept so the reference's block
code and its packed checkpoints load unchanged: ``Int8Linear`` with the buffers
``weight_int8`` (the [K, N] transpose view of a row-major int8 [N, K] matrix),
``weight_scale`` (fp32 [1, N]), ``bias`` (bf16 [N] or None) and
``_dtype_token`` (an empty bf16 tensor that ``weight`` returns), the attributes
``in_features``, ``out_features``, ``gemm`` and ``fused_ops``, ``from_packed``,
``forward`` and ``forward_quantized``; and ``quantize_transformer`` with its
report dict.

What runs: every projection is the tcgen05 INT8 GEMM of liblr_w8a8.so with the
dequantising epilogue fused (``int8_gemm.int8_matmul``). The reference's
``gemm`` argument chose between two GPU backends, Triton and cuBLASLt
(``torch._int_mm`` followed by a torch or a fused epilogue). Both produce the
same int32 accumulators and the same epilogue rounding, and the sm_100a kernel
reproduces that output bit for bit, so here ``gemm`` only names the backend in
reports. ``fused_ops`` keeps its meaning for the activation quantiser: on, the
fused kernel's arithmetic (the device's mode; by default that of the
reference's compiled Triton kernel); off, the arithmetic of the reference's
unfused PyTorch ops on a CUDA device. The same CUDA kernel runs both.
"""
from __future__ import annotations

import torch
from torch import nn

from .int8_gemm import int8_matmul
from .kernels import quantize_rows

# Backend names accepted by ``gemm`` and what ``quantize_transformer`` reports
# for each: (gemm, tile_selection). "torch" and "triton" keep the reference's
# report values (model/int8.py:99-104) so consumers of the report see the same
# dict; "b200" names this build's kernel.
_REPORTED_BACKEND = {
    "torch": ("torch._int_mm", None),
    "triton": ("Triton INT8 with fused BF16 epilogue", "device-specific autotune with persistent cache"),
    "b200": ("sm_100a tcgen05 INT8 with fused BF16 epilogue", "fixed 256x256 CTA-pair tile, persistent"),
}


def _require_backend(gemm: str) -> None:
    if gemm not in _REPORTED_BACKEND:
        raise ValueError("unsupported INT8 GEMM backend")


def _rowwise_int8(matrix: torch.Tensor):
    """Symmetric int8 codes per row (model/int8.py:10-11): scale = max(absmax,
    1e-8) / 127 in fp32 and codes = round-half-even(value / scale) within
    [-127, 127]. Load-time only; returns (int8 [rows, cols], fp32 [rows, 1])."""
    values = matrix.detach().float()
    scale = torch.clamp(values.abs().amax(dim=1, keepdim=True), min=1e-8) / 127
    codes = torch.clamp(torch.round(values / scale), min=-127, max=127)
    return codes.to(torch.int8), scale


class Int8Linear(nn.Module):
    """Per-token dynamic int8 activations x per-output-channel int8 weights,
    exact int32 accumulation, bf16 output."""

    def __init__(self, source, gemm="torch"):
        super().__init__()
        codes, scale = _rowwise_int8(source.weight)
        bias = None if source.bias is None else source.bias.detach().to(torch.bfloat16)
        self._adopt(codes.contiguous(), scale, bias, source.weight.new_empty(0), gemm)

    @classmethod
    def from_packed(cls, weight, scale, bias=None, gemm="triton"):
        """A layer over already-quantised rows, used as stored (no float round
        trip): weight int8 [out, in], scale [out, 1], bias [out] or None."""
        if weight.dtype != torch.int8 or scale.shape != (weight.shape[0], 1):
            raise ValueError("expected INT8 [out,in] weights and [out,1] scales")
        layer = cls.__new__(cls)
        nn.Module.__init__(layer)
        token = torch.empty(0, device=weight.device, dtype=torch.bfloat16)
        layer._adopt(weight, scale, bias, token, gemm)
        return layer

    def _adopt(self, rows_nk: torch.Tensor, scale_n1: torch.Tensor, bias, dtype_token: torch.Tensor,
               gemm: str) -> None:
        """Install a packed projection: int8 rows [N, K], fp32 scales [N, 1]."""
        _require_backend(gemm)
        self.out_features, self.in_features = rows_nk.shape
        self.register_buffer("weight_int8", rows_nk.t())
        self.register_buffer("weight_scale", scale_n1.t().contiguous())
        self.register_buffer("bias", bias)
        self.register_buffer("_dtype_token", dtype_token, persistent=False)
        self.gemm = gemm
        self.fused_ops = False

    @property
    def weight(self):
        return self._dtype_token

    def forward_quantized(self, quantized, scale, output_shape):
        """Project quantised rows (int8 [..., in], fp32 [rows, 1]) -> bf16 [*output_shape, out]."""
        rows = quantized.reshape(-1, self.in_features).contiguous()
        projected = int8_matmul(rows, self.weight_int8, scale, self.weight_scale, self.bias)
        return projected.view(*output_shape, self.out_features)

    def forward(self, value):
        rows = value.reshape(-1, self.in_features)
        codes, scale = quantize_rows(rows, arithmetic=None if self.fused_ops else "torch_cuda")
        return self.forward_quantized(codes, scale, value.shape[:-1])


def _concatenated(parts) -> nn.Linear:
    """One nn.Linear whose output rows are those of ``parts`` in order; when any
    part has a bias, the others contribute zeros (model/int8.py:80-88)."""
    if not all(isinstance(part, nn.Linear) for part in parts):
        raise ValueError("quantization requires an unconverted transformer")
    ref = parts[0].weight
    with_bias = any(part.bias is not None for part in parts)
    joined = nn.Linear(parts[0].in_features, sum(part.out_features for part in parts), bias=with_bias,
                       device=ref.device, dtype=ref.dtype)
    joined.weight.copy_(torch.cat([part.weight for part in parts]))
    if with_bias:
        joined.bias.copy_(torch.cat([part.bias if part.bias is not None else ref.new_zeros(part.out_features)
                                     for part in parts]))
    return joined


@torch.no_grad()
def quantize_transformer(transformer, protected_edges=1, gemm="torch"):
    """Post-training W8A8 of a standard DiT (model/int8.py:71-104): every block
    gets a fused ``to_qkv``; the blocks between the ``protected_edges`` first
    and last ones have QKV, the attention output and both FFN projections
    replaced by ``Int8Linear``. Returns the reference's report dict."""
    _require_backend(gemm)
    blocks = transformer.transformer_blocks
    if protected_edges < 0 or 2 * protected_edges >= len(blocks):
        raise ValueError("invalid number of protected edge blocks")
    inner = range(protected_edges, len(blocks) - protected_edges)
    for index, block in enumerate(blocks):
        attn = block.attn
        qkv = _concatenated([attn.to_q, attn.to_k, attn.to_v])
        attn.to_q = attn.to_k = attn.to_v = None
        attn.fused_projections = True
        if index not in inner:
            attn.to_qkv = qkv
            continue
        attn.to_qkv = Int8Linear(qkv, gemm)
        attn.to_out[0] = Int8Linear(attn.to_out[0], gemm)
        ffn = block.ff.net
        ffn[0].proj = Int8Linear(ffn[0].proj, gemm)
        ffn[2] = Int8Linear(ffn[2], gemm)
    reported_gemm, tile_selection = _REPORTED_BACKEND[gemm]
    converted = list(inner)
    return {"format": "W8A8", "gemm": reported_gemm, "accumulator": "INT32", "tile_selection": tile_selection,
            "activation_scale": "per-token", "weight_scale": "per-output-channel", "rounding": "nearest-even",
            "protected_edge_blocks": protected_edges, "quantized_blocks": converted,
            "quantized_linears": 4 * len(converted), "qkv_fused": True,
            "adaln_and_refiner_and_io_quantized": False}
