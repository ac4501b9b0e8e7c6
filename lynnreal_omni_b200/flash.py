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
    column = column.contiguous()
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


def _compression_span(config, depth: int) -> tuple[int, int, float]:
    """Validate the checkpoint's token-compression settings (the only layout
    the released hooks support) and return (first compressed block, first
    restored block, residual gain)."""
    c = config["token_compression"]
    if depth != config["num_layers"]:
        raise ValueError("Flash depth and exported weights disagree")
    fixed = {"reduction": "select", "spatial_stride": 2}
    if (any(c[name] != value for name, value in fixed.items())
            or not (c["preserve_text_tokens"] and c["preserve_audio_tokens"])
            or c.get("full_refresh_blocks") or c.get("text_stride", 1) != 1 or c.get("audio_stride", 1) != 1):
        raise ValueError("unsupported Flash token layout")
    first, restored = c["full_prefix_blocks"], depth - c["full_suffix_blocks"]
    if not 0 < first < restored < depth:
        raise ValueError("Flash requires nonempty full-resolution prefix and suffix")
    return first, restored, float(c.get("residual_gain", 1.0))


class _FlashHooks:
    """Hook state of one configured transformer. ``on_forward`` (pre-hook of
    the transformer) resolves the packed layout of this forward (cached while
    positions and tags stay the same); ``on_compressed_block`` (pre-hook of
    each compressed block) swaps in the kept rows — the hidden stream once,
    the adaLN indices, rotary rows and mask once per forward; ``on_restore``
    (pre-hook of the first suffix block) adds the compressed blocks' change
    back onto the full sequence; ``on_done`` (forward hook, always called)
    resets the per-forward state."""

    def __init__(self, signature, gain: float):
        self.signature = signature
        self.gain = gain
        self.layout = None        # (positions, tags, keep, inverse) of the last layout seen
        self.active = False
        self.full = None          # hidden stream entering the first compressed block
        self.entry = None         # its compressed rows (the first compressed block's input)
        self.selected = {}        # per-forward gathers of the unchanged block arguments

    def on_forward(self, module, args, kwargs):
        if module.training or torch.is_grad_enabled():
            raise ValueError("Flash hooks require frozen inference")
        if self.active:
            raise RuntimeError("Flash transformer does not support concurrent forwards")
        bound = self.signature.bind(*args, **kwargs).arguments
        positions, tags = bound["position_ids"], bound["token_tags"]
        known = self.layout
        if not (known is not None and known[0].shape == positions.shape and known[1].shape == tags.shape
                and torch.equal(positions, known[0]) and torch.equal(tags, known[1])):
            self.layout = (positions.clone(), tags.clone(), *spatial_layout(positions, tags))
        self.active = True

    def _select(self, value, dim):
        # the same tensor (identity, storage and version) gathers to the same rows
        key = (id(value), value.data_ptr(), value._version, dim)
        if key not in self.selected:
            self.selected[key] = (value, index_select(value, dim, self.layout[2]))
        return self.selected[key][1]

    def on_compressed_block(self, module, args):
        hidden, temb, indices, rotary, mask = args
        if self.full is None:
            self.full = hidden
            hidden = self.entry = index_select(hidden, 1, self.layout[2])
        return (hidden, temb, self._select(indices, 0), tuple(self._select(v, -2) for v in rotary),
                None if mask is None else self._select(mask, -1))

    def on_restore(self, module, args):
        hidden = restore(self.full, args[0], self.entry, self.layout[3], self.gain)
        self.full = self.entry = None
        return (hidden, *args[1:])

    def on_done(self, *_):
        self.active = False
        self.full = self.entry = None
        self.selected = {}


def configure_flash(transformer, config):
    """Install the Flash inference hooks (model/flash.py:36-94); weights and
    the transformer's own code stay as they are."""
    blocks = transformer.transformer_blocks
    first, restored, gain = _compression_span(config, len(blocks))
    if hasattr(transformer, "_lynnreal_flash_hooks"):
        raise ValueError("Flash is already configured")
    transformer.h3_token_compression = None
    hooks = _FlashHooks(inspect.signature(transformer.forward), gain)
    handles = [transformer.register_forward_pre_hook(hooks.on_forward, with_kwargs=True)]
    handles += [block.register_forward_pre_hook(hooks.on_compressed_block) for block in blocks[first:restored]]
    handles.append(blocks[restored].register_forward_pre_hook(hooks.on_restore))
    handles.append(transformer.register_forward_hook(hooks.on_done, always_call=True))
    transformer._lynnreal_flash_hooks = handles
