"""Flash token compression on the sm_100a kernels.

Replaces model/flash.py: ``spatial_layout`` (:6-33) and ``configure_flash``
(:36-94), same arguments, return values, hooks and error messages. The
middle blocks of a Flash transformer run on a stride-2 spatial subset of the
packed video rows; before the first full-resolution suffix block, the change
those blocks made is added back onto the full sequence, a dropped row taking
its nearest same-time kept row's update.

What runs where:
  * the row gathers of the ``compress`` hook (hidden rows, adaLN indices,
    rotary rows, attention-mask columns) are ``lr_gather_rows``;
  * the ``restore`` hook is one ``lr_flash_restore`` pass instead of the
    reference's four tensor ops (subtract, scale, index_select, add) and
    their two full-size temporaries;
  * ``spatial_layout`` runs once per packed layout (cached by the hooks): the
    coordinate alphabets and row lists use torch's device sort/unique/nonzero,
    and the dropped-row -> anchor search, the only part whose cost grows with
    rows x anchors, is ``lr_flash_nearest_anchor``.
The ``compress`` hook gathers the (unchanged) indices, rotary tables and mask
once per forward instead of once per compressed block; the values are the
same tensors' rows either way.
"""
from __future__ import annotations

import inspect
import math

import torch

from . import _lib
from ._lib import check, ptr, stream_of

__all__ = ["index_select", "restore", "spatial_layout", "configure_flash"]


def _require_cuda(name: str, *tensors: torch.Tensor) -> None:
    for t in tensors:
        if not t.is_cuda:
            raise ValueError(f"{name}: expected CUDA tensors")


def index_select(value: torch.Tensor, dim: int, index: torch.Tensor) -> torch.Tensor:
    """``value.index_select(dim, index)`` as one ``lr_gather_rows`` launch
    (any dtype; the output is a new contiguous tensor)."""
    _require_cuda("index_select", value, index)
    dim = dim % value.ndim if value.ndim else 0
    value = value.contiguous()
    index = index.reshape(-1)
    if index.dtype != torch.int64:
        index = index.to(torch.int64)
    index = index.contiguous()
    shape = list(value.shape)
    rows, n = shape[dim], index.numel()
    outer = math.prod(shape[:dim])
    row_bytes = math.prod(shape[dim + 1:]) * value.element_size()
    shape[dim] = n
    out = torch.empty(shape, device=value.device, dtype=value.dtype)
    if out.numel():
        if rows == 0:
            raise IndexError("index_select(): index out of range in an empty dimension")
        check(_lib.load().lr_gather_rows(ptr(value), outer, rows * row_bytes, rows, row_bytes, ptr(index), n,
                                         ptr(out), n * row_bytes, stream_of(value)), "index_select")
    return out


def restore(full: torch.Tensor, compressed: torch.Tensor, compressed_input: torch.Tensor,
            inverse: torch.Tensor, gain: float = 1.0) -> torch.Tensor:
    """``full + ((compressed - compressed_input) * gain).index_select(1, inverse)``
    in one pass (model/flash.py:81-84); bf16 [B, S, D] from [B, K, D] pairs."""
    _require_cuda("restore", full, compressed, compressed_input, inverse)
    for t in (full, compressed, compressed_input):
        if t.dtype != torch.bfloat16:
            raise ValueError(f"restore: expected bfloat16 tensors, got {t.dtype}")
    if compressed.shape != compressed_input.shape:
        raise ValueError("restore: compressed output and input shapes differ")
    b, s, d = full.shape
    if compressed.shape[0] != b or compressed.shape[2] != d or inverse.numel() != s:
        raise ValueError("restore: shapes do not describe one compressed sequence")
    full, compressed, compressed_input = full.contiguous(), compressed.contiguous(), compressed_input.contiguous()
    inverse = inverse.reshape(-1).to(torch.int64).contiguous()
    out = torch.empty_like(full)
    check(_lib.load().lr_flash_restore(ptr(full), ptr(compressed), ptr(compressed_input), ptr(inverse), b, s,
                                       compressed.shape[1], d, float(gain), ptr(out), stream_of(full)), "restore")
    return out


def _retained(column: torch.Tensor, stride: int) -> torch.Tensor:
    """For video rows' coordinates on one axis: whether each survives stride
    selection over the sorted alphabet (every stride-th value, and the last)."""
    alphabet = torch.unique(column, sorted=True)
    rank = torch.searchsorted(alphabet, column)
    return (rank % stride == 0) | (rank == alphabet.numel() - 1)


def spatial_layout(positions: torch.Tensor, tags: torch.Tensor, stride: int = 2):
    """(keep, inverse) of a packed layout (model/flash.py:6-33).

    positions [S, 3] (time, row, column), tags [S] (0 = video). ``keep``: the
    rows the compressed blocks see, in order (all non-video rows, and video
    rows whose row and column coordinates both survive stride selection).
    ``inverse[t]``: the compressed row whose update row t receives: its own
    for kept rows, else its nearest same-time kept video row's."""
    if positions.ndim != 2 or tags.ndim != 1 or positions.shape != (tags.numel(), 3):
        raise ValueError("Flash requires a single shared packed layout")
    _require_cuda("spatial_layout", positions, tags)
    video = tags == 0
    video_rows = video.nonzero().flatten()
    if not video_rows.numel():
        raise ValueError("Flash requires video tokens")
    coords = index_select(positions, 0, video_rows)
    kept_video = _retained(coords[:, 1], stride) & _retained(coords[:, 2], stride)
    mask = ~video
    mask[video_rows] = kept_video
    keep = mask.nonzero().flatten()
    inverse = torch.empty(tags.numel(), device=tags.device, dtype=torch.int64)
    inverse[keep] = torch.arange(keep.numel(), device=tags.device)
    dropped = video_rows[~kept_video]
    anchors = video_rows[kept_video]
    if dropped.numel():
        if not anchors.numel():
            raise RuntimeError("Flash layout drops video rows but keeps no anchor")
        pos32 = positions.to(torch.float32).contiguous()
        check(_lib.load().lr_flash_nearest_anchor(ptr(pos32), pos32.shape[0], ptr(dropped), dropped.numel(),
                                                  ptr(anchors), anchors.numel(), ptr(inverse),
                                                  stream_of(positions)), "spatial_layout")
    return keep, inverse


def configure_flash(transformer, config):
    """Install the Flash inference hooks (model/flash.py:36-94); weights and
    the transformer's own code stay as they are."""
    blocks = transformer.transformer_blocks
    compression = config["token_compression"]
    if len(blocks) != config["num_layers"]:
        raise ValueError("Flash depth and exported weights disagree")
    supported = (compression["reduction"] == "select" and compression["spatial_stride"] == 2
                 and compression["preserve_text_tokens"] and compression["preserve_audio_tokens"]
                 and not compression.get("full_refresh_blocks")
                 and compression.get("text_stride", 1) == 1 and compression.get("audio_stride", 1) == 1)
    if not supported:
        raise ValueError("unsupported Flash token layout")
    start = compression["full_prefix_blocks"]
    end = len(blocks) - compression["full_suffix_blocks"]
    if not 0 < start < end < len(blocks):
        raise ValueError("Flash requires nonempty full-resolution prefix and suffix")
    if hasattr(transformer, "_lynnreal_flash_hooks"):
        raise ValueError("Flash is already configured")
    transformer.h3_token_compression = None
    gain = float(compression.get("residual_gain", 1.0))
    signature = inspect.signature(transformer.forward)
    state = {}
    layout = {}

    def begin(module, args, kwargs):
        if module.training or torch.is_grad_enabled():
            raise ValueError("Flash hooks require frozen inference")
        if state:
            raise RuntimeError("Flash transformer does not support concurrent forwards")
        bound = signature.bind(*args, **kwargs).arguments
        positions, tags = bound["position_ids"], bound["token_tags"]
        same = (layout and layout["positions"].shape == positions.shape and layout["tags"].shape == tags.shape
                and torch.equal(positions, layout["positions"]) and torch.equal(tags, layout["tags"]))
        if not same:
            keep, inverse = spatial_layout(positions, tags)
            layout.update(positions=positions.clone(), tags=tags.clone(), keep=keep, inverse=inverse)
        state["keep"], state["inverse"] = layout["keep"], layout["inverse"]
        state["gathered"] = {}

    def gathered(value, dim):
        # the same tensor (identity, storage and version) gathers to the same rows
        key = (id(value), value.data_ptr(), value._version, dim)
        hit = state["gathered"].get(key)
        if hit is None:
            hit = state["gathered"][key] = (value, index_select(value, dim, state["keep"]))
        return hit[1]

    def compress(module, args):
        hidden, temb, indices, rotary, mask = args
        if "full" not in state:
            state["full"] = hidden
            hidden = index_select(hidden, 1, state["keep"])
            state["input"] = hidden
        return (hidden, temb, gathered(indices, 0), tuple(gathered(v, -2) for v in rotary),
                None if mask is None else gathered(mask, -1))

    def restore_hook(module, args):
        hidden = restore(state.pop("full"), args[0], state.pop("input"), state["inverse"], gain)
        return (hidden, *args[1:])

    def finish(*_):
        state.clear()

    handles = [transformer.register_forward_pre_hook(begin, with_kwargs=True)]
    handles += [block.register_forward_pre_hook(compress) for block in blocks[start:end]]
    handles += [blocks[end].register_forward_pre_hook(restore_hook),
                transformer.register_forward_hook(finish, always_call=True)]
    transformer._lynnreal_flash_hooks = handles
