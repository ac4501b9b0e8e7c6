"""Run one kernel of the W8A8 path on synthetic inputs (for profilers and timing).

    python -m lynnreal_omni_b200.profile_case gemm --m 2048 --k 6144 --n 24576 --epi gelu
    python -m lynnreal_omni_b200.profile_case rms --m 12240 --d 6144
    python -m lynnreal_omni_b200.profile_case quant --m 12240 --d 24576
    python -m lynnreal_omni_b200.profile_case gated --m 12240 --d 6144
    python -m lynnreal_omni_b200.profile_case qk --m 12240 --d 6144
    python -m lynnreal_omni_b200.profile_case compress --d 6144   (21 x 48 x 64 video grid)
    python -m lynnreal_omni_b200.profile_case restore --d 6144
    python -m lynnreal_omni_b200.profile_case restore_torch --d 6144   (the reference's tensor ops)
    python -m lynnreal_omni_b200.profile_case layout
    python -m lynnreal_omni_b200.profile_case attn --m 12240 --d 6144   (48 heads x 128)
    python -m lynnreal_omni_b200.profile_case attn_sdpa --m 12240 --d 6144   (torch SDPA, same inputs)

Each case launches its kernel ``--iters`` times on cuda:0 and prints the mean
CUDA-event time per launch and the algorithmic rate (TOP/s or GB/s).
"""
from __future__ import annotations

import argparse
import json
from types import SimpleNamespace

import torch


def _time(fn, iters: int, warmup: int, graph: bool = False):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if graph:
        # capture `iters` calls once and time one replay: device time without
        # the host-side cost of issuing each call
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(iters):
                fn()
        g.replay()
        torch.cuda.synchronize()
        run = g.replay
        reps = 1
    else:
        run = fn
        reps = iters
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        run()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("case", choices=["gemm", "rms", "quant", "gated", "residual_rms", "qk", "compress", "restore",
                                    "restore_torch", "layout", "attn", "attn_sdpa"])
    p.add_argument("--m", type=int, default=12240)
    p.add_argument("--k", type=int, default=6144)
    p.add_argument("--n", type=int, default=24576)
    p.add_argument("--d", type=int, default=6144)
    p.add_argument("--epi", choices=["none", "gelu", "gated"], default="none")
    p.add_argument("--iters", type=int, default=3)
    p.add_argument("--warmup", type=int, default=1)
    p.add_argument("--graph", action="store_true", help="time a CUDA-graph replay of the launches")
    a = p.parse_args(argv)

    from . import kernels as K
    from .int8_gemm import int8_matmul, int8_matmul_gated_residual, int8_matmul_gelu
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    out = {"case": a.case, "graph": a.graph}
    if a.case == "gemm":
        A = torch.randint(-127, 128, (a.m, a.k), device=dev, dtype=torch.int8, generator=g)
        B = torch.randint(-127, 128, (a.n, a.k), device=dev, dtype=torch.int8, generator=g).t()
        rs = torch.rand(a.m, 1, device=dev, generator=g) / 127
        cs = torch.rand(1, a.n, device=dev, generator=g) / 127
        bias = (0.02 * torch.randn(a.n, device=dev, generator=g)).to(torch.bfloat16)
        if a.epi == "gelu":
            fn = lambda: int8_matmul_gelu(A, B, rs, cs, bias)  # noqa: E731
        elif a.epi == "gated":
            res = torch.randn(1, a.m, a.n, device=dev, generator=g).to(torch.bfloat16)
            table = (0.1 * torch.randn(1, 6 * a.n, device=dev, generator=g)).to(torch.bfloat16)
            idx = torch.zeros(a.m, dtype=torch.int64, device=dev)
            fn = lambda: int8_matmul_gated_residual(A, B, rs, cs, bias, res, table, idx, 5)  # noqa: E731
        else:
            fn = lambda: int8_matmul(A, B, rs, cs, bias)  # noqa: E731
        ms = _time(fn, a.iters, a.warmup, a.graph)
        out.update(m=a.m, k=a.k, n=a.n, epi=a.epi, ms=ms, tops=2.0 * a.m * a.n * a.k / (ms / 1e3) / 1e12,
                   algorithmic_bytes=a.m * a.k + a.n * a.k + 2 * a.m * a.n + 4 * a.m + 6 * a.n)
    elif a.case == "qk":
        heads, hd = a.d // 128, 128
        qkv = torch.randn(1, a.m, 3 * a.d, device=dev, generator=g).to(torch.bfloat16)
        q, k, _ = [t.unflatten(-1, (heads, -1)) for t in qkv.chunk(3, dim=-1)]
        nq = SimpleNamespace(weight=torch.ones(hd, device=dev, dtype=torch.bfloat16), eps=1e-6)
        phase = torch.randn(a.m, hd, device=dev, generator=g)
        rot = (phase.cos(), phase.sin())
        ms = _time(lambda: K.qk_norm_rope(q, k, nq, nq, rot), a.iters, a.warmup, a.graph)
        nbytes = 8 * a.m * a.d + 8 * a.m * hd + 4 * hd
        out.update(m=a.m, d=a.d, heads=heads, ms=ms, algorithmic_bytes=nbytes, gbs=nbytes / (ms / 1e3) / 1e9)
    elif a.case in ("attn", "attn_sdpa"):
        from .attention import attention_bshd
        heads = a.d // 128
        qkv = torch.randn(1, a.m, 3 * a.d, device=dev, generator=g).to(torch.bfloat16)
        q, k, v = [t.unflatten(-1, (heads, -1)) for t in qkv.chunk(3, dim=-1)]
        if a.case == "attn":
            fn = lambda: attention_bshd(q, k, v)  # noqa: E731
        else:
            qt, kt, vt = (t.transpose(1, 2) for t in (q, k, v))
            fn = lambda: torch.nn.functional.scaled_dot_product_attention(qt, kt, vt)  # noqa: E731
        ms = _time(fn, a.iters, a.warmup, a.graph)
        flops = 4.0 * heads * a.m * a.m * 128
        out.update(m=a.m, heads=heads, ms=ms, tflops=flops / (ms / 1e3) / 1e12)
    elif a.case in ("compress", "restore", "restore_torch", "layout"):
        from . import flash
        t, h, w = torch.meshgrid(torch.arange(21), torch.arange(48), torch.arange(64), indexing="ij")
        pos = torch.stack([t, h, w], -1).reshape(-1, 3).to(dev)
        tags = torch.zeros(pos.shape[0], dtype=torch.int64, device=dev)
        keep, inverse = flash.spatial_layout(pos, tags)
        s, kept = pos.shape[0], keep.numel()
        if a.case == "layout":
            ms = _time(lambda: flash.spatial_layout(pos, tags), a.iters, a.warmup, False)
            out.update(rows=s, kept=kept, ms=ms)
        else:
            full = torch.randn(1, s, a.d, device=dev, generator=g).to(torch.bfloat16)
            if a.case == "compress":
                fn = lambda: flash.index_select(full, 1, keep)  # noqa: E731
                nbytes = 4 * kept * a.d + 8 * kept
            else:
                comp = torch.randn(1, kept, a.d, device=dev, generator=g).to(torch.bfloat16)
                inp = torch.randn(1, kept, a.d, device=dev, generator=g).to(torch.bfloat16)
                if a.case == "restore":
                    fn = lambda: flash.restore(full, comp, inp, inverse, 1.0)  # noqa: E731
                else:
                    fn = lambda: full + ((comp - inp) * 1.0).index_select(1, inverse)  # noqa: E731
                nbytes = 4 * s * a.d + 4 * kept * a.d + 8 * s
            ms = _time(fn, a.iters, a.warmup, a.graph)
            out.update(rows=s, kept=kept, d=a.d, ms=ms, algorithmic_bytes=nbytes, gbs=nbytes / (ms / 1e3) / 1e9)
    else:
        x = torch.randn(1, a.m, a.d, device=dev, generator=g).to(torch.bfloat16)
        y = torch.randn(1, a.m, a.d, device=dev, generator=g).to(torch.bfloat16)
        table = (0.1 * torch.randn(1, 6 * a.d, device=dev, generator=g)).to(torch.bfloat16)
        idx = torch.zeros(a.m, dtype=torch.int64, device=dev)
        norm = SimpleNamespace(weight=(1 + 0.05 * torch.randn(a.d, device=dev, generator=g)).to(torch.bfloat16),
                               eps=1e-6)
        if a.case == "rms":
            fn, per_elem = (lambda: K._rms_adaln_quant_int8(x, norm, table, idx, 0, 1)), 3
        elif a.case == "quant":
            fn, per_elem = (lambda: K.quantize_rows(x.view(a.m, a.d))), 3
        elif a.case == "gated":
            fn, per_elem = (lambda: K._gated_residual(x, y, table, idx, 2)), 6
        else:
            fn, per_elem = (lambda: K.residual_rms_quant(x, y, norm, table, idx)), 7
        ms = _time(fn, a.iters, a.warmup, a.graph)
        nbytes = per_elem * a.m * a.d + 4 * a.m
        out.update(m=a.m, d=a.d, ms=ms, algorithmic_bytes=nbytes, gbs=nbytes / (ms / 1e3) / 1e9)
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
