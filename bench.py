#!/usr/bin/env python
"""Benchmark of the B200 W8A8 projection path: DiT-block tokens/s on 1..8 GPUs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

For N > 1 launch one process per GPU with torch.distributed.run. A step is one
forward of the W8A8 path of one Flash-like DiT block (config 2: M=12240 tokens,
D=6144, QKV 18432, FFN 24576 GELU-tanh, cross-attention Q/O with text K/V from a
512x4096 context) over one 12240-token latent whose token rows are split into
contiguous blocks, one per GPU (1530 rows each at N=8), with the int8 weights
replicated; every step ends with one NCCL all_gather_into_tensor of the bf16
block output, inside the timed region (strong scaling: the path is independent
per token row, the gather is its only exchange). The timed region holds exactly
K steps between a barrier and a device synchronize; the step time is the
maximum over ranks of CUDA-event time.

``--impl reference`` times the reference's own PyTorch CPU implementation of
the same block (the torch port under oracle/) on the host cores, rank 0 only,
all 12240 rows every step.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "W8A8 DiT-block tokens/s at 1/2/4/8 B200; INT8 GEMM TOPS vs tensor peak"
NOMINAL_INT8_TOPS = 4500.0
FALLBACK_BF16_BURST_TFLOPS = 1590.0


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--tokens", type=int, default=12240,
                   help="block: token rows of the latent, sharded over the GPUs; flash: token rows per GPU")
    p.add_argument("--gather", choices=["peer", "nccl"], default="peer",
                   help="block workload at N > 1: 'peer' writes the FFN-down GEMM's output rows straight into every "
                        "rank's gathered tensor over NVLink (the epilogue is the all-gather); 'nccl' runs "
                        "all_gather_into_tensor after the block")
    p.add_argument("--eager", action="store_true",
                   help="block workload: time the steps as eager launches instead of one CUDA-graph replay of the "
                        "K steps (every launch and the gather barrier of each step captured)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--workload", choices=["block", "stack", "sweep", "flash", "reference_kernels", "kernel"],
                   default="block",
                   help="block: config 2 per GPU (weak scaling); stack: config 4, 42 blocks x 3 denoiser "
                        "steps on 64512 tokens sharded over the GPUs with a final all-gather; sweep: "
                        "config 3 GEMM shapes, row-sharded, TOP/s per shape beside cuBLASLt; flash: one "
                        "block at the released Flash shapes through the fused-block caller, attention included; "
                        "reference_kernels: each kernel beside the reference's compiled GPU kernel (installed in "
                        "baseline/_ref) on the same inputs, device time and output identity; kernel: one kernel "
                        "(--case) on synthetic inputs, for profilers and timing")
    p.add_argument("--case", default="rms",
                   choices=["gemm", "rms", "quant", "gated", "residual_rms", "qk", "compress", "restore",
                            "restore_torch", "layout", "attn", "attn_sdpa"], help="kernel workload: which kernel")
    p.add_argument("--m", type=int, default=12240, help="kernel workload: rows / tokens")
    p.add_argument("--k", type=int, default=6144, help="kernel workload: GEMM depth")
    p.add_argument("--n", type=int, default=24576, help="kernel workload: GEMM width")
    p.add_argument("--d", type=int, default=6144, help="kernel workload: hidden size")
    p.add_argument("--epi", choices=["none", "gelu", "gated"], default="none", help="kernel workload: GEMM epilogue")
    p.add_argument("--graph", action="store_true", help="kernel workload: time a CUDA-graph replay of the launches")
    p.add_argument("--layers", type=int, default=42)
    p.add_argument("--stack-tokens", type=int, default=64512)
    p.add_argument("--compress", action="store_true",
                   help="stack: Flash token compression in blocks 2-27 of a 21x48x64 video grid (the released "
                        "schedule), shards of whole frames")
    return p.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def bind_local_numa(local_rank: int) -> dict:
    """Run this rank on the CPUs local to its GPU's PCIe root (sysfs), so its
    pinned host buffers are first touched next to the GPU. Best effort: the
    result records the NUMA node, the CPUs bound and, when nothing was bound,
    why (a node of -1 means the platform reports no NUMA locality)."""
    info = {"node": None, "cpus": None, "reason": None}
    try:
        props = torch.cuda.get_device_properties(local_rank)
        dev = f"{props.pci_domain_id:04x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        base = Path("/sys/bus/pci/devices") / dev
        info["pci"] = dev
        node = int((base / "numa_node").read_text().strip())
        info["node"] = node
        cpus = set()
        for part in (base / "local_cpulist").read_text().strip().split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        allowed = os.sched_getaffinity(0)
        local = cpus & allowed
        if not local:
            info["reason"] = "no CPU of local_cpulist is in this process's affinity"
            return info
        if local == allowed:
            info["reason"] = "every allowed CPU is already local to the GPU (nothing to bind)"
            info["cpus"] = len(local)
            return info
        os.sched_setaffinity(0, local)
        info["cpus"] = len(local)
        return info
    except (OSError, ValueError, AttributeError) as error:
        info["reason"] = f"sysfs topology not readable: {type(error).__name__}: {error}"
        return info


def workload_config(args, world):
    """The workload of the config-2 line; identical in both arms at every N."""
    from lynnreal_omni_b200 import workloads as W
    from lynnreal_omni_b200.parallel import shard_bounds
    sizes = sorted({e - s for s, e in (shard_bounds(args.tokens, world, r) for r in range(world))})
    return {
        "workload": "config2: one Flash-like DiT block, W8A8 projection path, token rows sharded over the GPUs",
        "model": "Flash-like DiT block (D=6144, 48x128 heads, FFN 24576 GELU-tanh)",
        "global_tokens": args.tokens,
        "tokens_per_gpu": sizes[0] if len(sizes) == 1 else sizes,
        "global_batch": 1,
        "seq_len": args.tokens,
        "projections": {"qkv": [W.HIDDEN, 3 * W.HIDDEN], "o": [W.HIDDEN, W.HIDDEN],
                        "cross_q": [W.HIDDEN, W.HIDDEN], "cross_kv": [W.TEXT_DIM, 2 * W.HIDDEN],
                        "cross_o": [W.HIDDEN, W.HIDDEN], "up": [W.HIDDEN, W.FFN], "down": [W.FFN, W.HIDDEN]},
        "text_context": [W.TEXT_TOKENS, W.TEXT_DIM],
        "attention": "cores stubbed (self-attn returns V, cross-attn returns Q): out of scope",
        "parallelism": (f"{world} GPU(s): contiguous token-row shards, int8 weights replicated, "
                        "the bf16 block output all-gathered to every GPU each step"
                        if world > 1 else "1 GPU: all token rows, no collective"),
        "l2": "no flush: per-step working set (0.58 GB int8 weights + activations) >> 126 MB L2",
    }


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        return json.loads(path.read_text())
    except (OSError, ValueError):
        return {}


def profile_traffic(kernel_tag: str):
    """Per-launch DRAM bytes of the dominant kernel from a committed ncu summary
    (a line 'traffic_bytes_per_launch: N' in profiles/<kernel_tag>*.md), or None."""
    for path in sorted((ROOT / "profiles").glob(f"{kernel_tag}*.md")):
        for line in path.read_text().splitlines():
            if line.strip().startswith("traffic_bytes_per_launch:"):
                try:
                    return int(float(line.split(":", 1)[1].strip().split()[0]))
                except ValueError:
                    return None
    return None


def clock_sampler(device: torch.device, local_rank: int):
    """NVML sampler in its own process; nvidia-smi if NVML is unavailable."""
    try:
        import pynvml
        pynvml.nvmlInit()
        from lynnreal_omni_b200.clocks import ClockSampler as NvmlSampler
        return NvmlSampler(str(torch.cuda.get_device_properties(device).uuid))
    except Exception:
        return SmiSampler(local_rank)


class SmiSampler:
    """nvidia-smi clocks/throttle sampling during the timed region (rank 0)."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, local_rank: int):
        visible = os.environ.get("CUDA_VISIBLE_DEVICES")
        self.index = visible.split(",")[local_rank] if visible else str(local_rank)
        self.file = tempfile.NamedTemporaryFile(prefix="clocks", suffix=".csv", delete=False)
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.index, f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.close()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}

        def num(v):
            try:
                return float(v)
            except ValueError:
                return None
        power = [num(r[3]) for r in rows if num(r[3]) is not None]
        hi = max(power) if power else 0.0
        loaded = [r for r in rows if num(r[3]) is not None and num(r[3]) >= 0.5 * hi] or rows
        sm = [num(r[1]) for r in loaded if num(r[1]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in loaded for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": num(rows[0][2]),
                "reasons": reasons, "samples": len(rows), "samples_under_load": len(loaded),
                "power_w_max": hi}


def _cpu_times(fn, warmup: int, repeats: int):
    for _ in range(warmup):
        fn()
    ts = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return ts


def cpu_block_rate(weights_cpu, tokens: int, repeats: int = 3, extrapolation_rows: int = 512):
    """Tokens/s of the reference's PyTorch CPU path (oracle/w8a8_torch.py) on
    this host for the whole block of ``tokens`` rows: one warm-up, median of
    ``repeats`` timed runs. Beside it, the earlier bounded-sample estimate
    (``extrapolation_rows`` rows timed, extrapolated linearly) for comparison."""
    from oracle import w8a8_torch as T
    from lynnreal_omni_b200 import block
    torch.set_num_threads(os.cpu_count() or 1)
    x, table, idx, ctx = block.make_inputs(tokens, seed=7)
    x2 = x.view(tokens, -1)
    full = statistics.median(_cpu_times(lambda: T.flash_block(x2, table, idx, ctx, weights_cpu), 1, repeats))

    xs = x2[:extrapolation_rows].contiguous()
    ids = idx[:extrapolation_rows].contiguous()
    t_sample = statistics.median(_cpu_times(lambda: T.flash_block(xs, table, ids, ctx, weights_cpu), 1, repeats))

    def fixed():
        q, s = T.quantize_rows(ctx)
        T.int8_matmul(q, weights_cpu.cross_kv.weight.t(), s, weights_cpu.cross_kv.scale, weights_cpu.cross_kv.bias)
    t_fixed = statistics.median(_cpu_times(fixed, 1, repeats))
    t_extrapolated = t_fixed + max(t_sample - t_fixed, 1e-9) * tokens / extrapolation_rows
    return tokens / full, {"t_block_s": full, "cores": torch.get_num_threads(), "repeats": repeats,
                           "extrapolated_from_sample": {"rows": extrapolation_rows,
                                                        "tokens_per_s": tokens / t_extrapolated,
                                                        "t_block_s": t_extrapolated}}


def run_reference(args, world):
    """Rank 0: the reference's PyTorch CPU path on all host threads; every step
    is the whole config-2 block (all token rows, unsharded) on the CPU."""
    from oracle import w8a8_torch as T
    from lynnreal_omni_b200 import block
    torch.set_num_threads(os.cpu_count() or 1)
    weights = block.make_weights(seed=0)
    x, table, idx, ctx = block.make_inputs(args.tokens, seed=7)
    x2 = x.view(args.tokens, -1)
    ts = _cpu_times(lambda: T.flash_block(x2, table, idx, ctx, weights), args.warmup, args.steps)
    t_step = statistics.mean(ts)
    value = args.tokens / t_step
    cores = torch.get_num_threads()
    sample = (f"every step is the whole block: all {args.tokens} token rows, text K/V projection included "
              f"(mean of {args.steps} steps after {args.warmup} warm-up)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_step * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": workload_config(args, world),
        "execution": "rank 0 only, host CPU, all threads, unsharded (the reference has no GPU or multi-process "
                     "path for this block)",
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample,
                         "implementation": "reference PyTorch path (Int8Linear torch path + torch restatement "
                                           "of the Triton kernels), oracle/w8a8_torch.py"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def int8_ceiling_cublaslt(m: int, k: int, n: int, dev, reps: int = 10) -> float:
    """Measured int8 tensor ceiling on this GPU: cuBLASLt ``torch._int_mm`` at
    the dominant kernel's shape (int32 output, no epilogue), TOP/s over
    ``reps`` back-to-back launches after warm-up, CUDA events."""
    g = torch.Generator(device=dev).manual_seed(5)
    mp = max(32, -(-m // 8) * 8)
    a = torch.randint(-127, 128, (mp, k), generator=g, device=dev, dtype=torch.int8)
    b = torch.randint(-127, 128, (n, k), generator=g, device=dev, dtype=torch.int8).t()
    for _ in range(3):
        torch._int_mm(a, b)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(reps):
        torch._int_mm(a, b)
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / reps
    del a, b
    return 2.0 * m * n * k / (ms / 1e3) / 1e12


def run_ours(args, rank, world, local):
    """Config 2: one block over ``args.tokens`` token rows, sharded into
    contiguous row blocks over the ranks; every step ends with the NCCL
    all-gather of the bf16 block output, inside the timed region."""
    import torch.distributed as dist
    from lynnreal_omni_b200 import block, _lib
    from lynnreal_omni_b200 import workloads as W
    from lynnreal_omni_b200.parallel import RowGather, shard_bounds

    if not torch.cuda.is_available():
        raise RuntimeError("bench.py needs a CUDA GPU")
    torch.cuda.set_device(local)
    numa = bind_local_numa(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    _lib.load()

    total, d = args.tokens, W.HIDDEN
    start_row, stop_row = shard_bounds(total, world, rank)
    m = stop_row - start_row
    weights = block.make_weights(seed=0, device=dev)  # replicated: same seed on every rank
    blk = block.FlashBlockW8A8(weights)
    x_full, table, idx_full, ctx = block.make_inputs(total, seed=100, device=dev)  # same latent on every rank
    x = x_full[:, start_row:stop_row].contiguous()
    idx = idx_full[start_row:stop_row].contiguous()
    from lynnreal_omni_b200.parallel import PeerRows
    peer = PeerRows(total, d, dev) if world > 1 and args.gather == "peer" else None
    gather = RowGather(total) if world > 1 and peer is None else None
    out_buf = torch.empty(total, d, dtype=torch.bfloat16, device=dev) if gather else None
    torch.cuda.synchronize()
    counter = [0]

    def barrier():
        if world > 1:
            dist.barrier()

    def step(xin, ffn_ev=None, ag_ev=None, out=None):
        if peer is not None:
            # the FFN-down epilogue writes this rank's rows into every rank's
            # buffer `slot`; the barrier after it makes all rows visible
            slot = counter[0] & 1
            counter[0] += 1
            blk(xin, table, idx, ctx, ffn_events=ffn_ev, rows_to=peer.destinations(slot))
            if ag_ev is not None:
                ag_ev[0].record()
            peer.barrier()
            if ag_ev is not None:
                ag_ev[1].record()
            return peer.local[slot]
        h, _ = blk(xin, table, idx, ctx, ffn_events=ffn_ev)
        if gather is None:
            return h.view(m, d)
        if ag_ev is not None:
            ag_ev[0].record()
        res = gather(h.view(m, d), out)
        if ag_ev is not None:
            ag_ev[1].record()
        return res

    for _ in range(args.warmup):
        step(x, out=out_buf)
    torch.cuda.synchronize()

    ev = lambda: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))  # noqa: E731
    # events inside a captured graph are record nodes of their own (external)
    ev_x = lambda: (torch.cuda.Event(enable_timing=True, external=True),  # noqa: E731
                    torch.cuda.Event(enable_timing=True, external=True))
    graph, graph_note = None, None
    if not args.eager:
        # The K timed steps as one CUDA graph: the same launches (and, at N > 1,
        # the same stream-ordered NCCL barrier per step) replayed without the
        # host issuing them one by one. Every rank agrees on the outcome of the
        # capture before any rank replays; a failed capture times eager launches.
        ffn = [ev_x() for _ in range(args.steps)]
        ag = [ev_x() for _ in range(args.steps)]
        barrier()
        torch.cuda.synchronize()
        err = None
        try:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for i in range(args.steps):
                    out = step(x, ffn[i], ag[i], out_buf)
        except Exception as exc:  # noqa: BLE001 - reported in the JSON line
            graph, err = None, f"{type(exc).__name__}: {exc}"[:200]
        torch.cuda.synchronize()
        if world > 1:
            okg = torch.tensor([0 if graph is None else 1], device=dev)
            dist.all_reduce(okg, op=dist.ReduceOp.MIN)
            if okg.item() == 0:
                graph = None
                err = err or "capture failed on another rank"
        if graph is not None:
            graph.replay()  # one untimed replay
            torch.cuda.synchronize()
            graph_note = {"timed": "one CUDA-graph replay of the K steps",
                          "launches_per_step": block.LAUNCHES_PER_FORWARD}
        else:
            graph_note = {"timed": "eager launches", "capture_error": err}
            ffn = [ev() for _ in range(args.steps)]
            ag = [ev() for _ in range(args.steps)]
    else:
        graph_note = {"timed": "eager launches (--eager)"}
        ffn = [ev() for _ in range(args.steps)]
        ag = [ev() for _ in range(args.steps)]

    sampler = clock_sampler(dev, local) if rank == 0 else None
    if sampler:
        sampler.start()
    start, end = ev()
    barrier()
    torch.cuda.synchronize()
    start.record()
    if graph is not None:
        graph.replay()
    else:
        for i in range(args.steps):
            out = step(x, ffn[i], ag[i], out_buf)
    end.record()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop() if sampler else None
    elapsed_ms = start.elapsed_time(end)
    ffn_ms = statistics.mean(a.elapsed_time(b) for a, b in ffn)
    ag_ms = statistics.mean(a.elapsed_time(b) for a, b in ag) if world > 1 else 0.0
    t = torch.tensor([elapsed_ms, ffn_ms, ag_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms, ffn_ms, ag_ms = t.tolist()
    status = _lib.device_status(clear=True)

    # the gathered rows equal the unsharded block (rows are independent)
    gathered_ok = None
    if world > 1:
        ok = torch.tensor([1], device=dev)
        if rank == 0:
            ok[0] = int(torch.equal(out, blk(x_full, table, idx_full, ctx)[0].view(total, d)))
        dist.broadcast(ok, 0)
        gathered_ok = bool(ok.item())
        torch.cuda.synchronize()

    # weak-scaling replica figure (each rank the whole latent, no collective): an extra key
    replica = None
    if world > 1:
        reps = max(3, min(args.steps, 10))
        for _ in range(2):
            blk(x_full, table, idx_full, ctx)
        r0, r1 = ev()
        barrier()
        torch.cuda.synchronize()
        r0.record()
        for _ in range(reps):
            blk(x_full, table, idx_full, ctx)
        r1.record()
        torch.cuda.synchronize()
        barrier()
        tr = torch.tensor([r0.elapsed_time(r1)], device=dev, dtype=torch.float64)
        dist.all_reduce(tr, op=dist.ReduceOp.MAX)
        replica = {"tokens_per_s": world * total * reps / (tr.item() / 1e3), "steps": reps,
                   "what": f"each of the {world} ranks runs all {total} rows, no collective (weak scaling)"}

    # end to end through the public API: every step copies this rank's latent
    # shard and the text context from pinned host memory, runs the block,
    # all-gathers the output and reads this rank's row range of the gathered
    # output back to pinned host memory (the ranks together read the whole
    # output once); HostPipeline overlaps step i's compute with the copies of
    # steps i+1 / i-1.
    e2e = None
    if not args.no_e2e:
        from lynnreal_omni_b200.pipeline import HostPipeline
        x_h = [x.cpu().pin_memory() for _ in range(2)]
        ctx_h = ctx.cpu().pin_memory()
        out_h = [torch.empty(m, d, dtype=torch.bfloat16).pin_memory() for _ in range(2)]

        def api(xd, cd):
            if peer is not None:  # this rank's rows of the gathered output, copied out of the reused buffer
                return step(xd)[start_row:stop_row].clone()
            h, _ = blk(xd, table, idx, cd)
            if gather is None:
                return h.view(m, d)
            return gather(h.view(m, d))[start_row:stop_row]  # fresh buffer per step: read while the next runs
        pipe = HostPipeline(api, dev, [x_h[0], ctx_h])
        ins = [[x_h[i & 1], ctx_h] for i in range(args.steps)]
        outs = [out_h[i & 1] for i in range(args.steps)]
        pipe.run(ins[:2], outs[:2])
        torch.cuda.synchronize()
        barrier()
        s2, e2 = ev()
        s2.record()
        pipe.run(ins, outs)
        e2.record()
        torch.cuda.synchronize()
        barrier()
        ok = torch.equal(out_h[(args.steps - 1) & 1], out[start_row:stop_row].cpu() if world > 1 else out.cpu())
        te = torch.tensor([s2.elapsed_time(e2)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_ms = te.item()
        e2e = {"value": total * args.steps / (e2e_ms / 1e3), "unit": "tokens/s",
               "h2d_bytes_per_step": x_h[0].numel() * 2 + ctx_h.numel() * 2,
               "d2h_bytes_per_step": out_h[0].numel() * 2,
               "bytes_per_step_are": "per rank (this rank's shard in, its row range of the gathered output out)",
               "h2d_bytes_per_step_all_ranks": total * d * 2 + world * ctx_h.numel() * 2,
               "d2h_bytes_per_step_all_ranks": total * d * 2,
               "ms_per_step": e2e_ms / args.steps,
               "result_matches_device_path": ok,
               "api": "HostPipeline over FlashBlockW8A8.forward (Int8Linear / kernels / int8_gemm over "
                      "liblr_w8a8.so) + parallel.RowGather; pinned host input and output every step, copies "
                      "overlapped with compute"}

    ceiling = None
    if rank == 0:
        ceiling = int8_ceiling_cublaslt(m, W.HIDDEN, W.FFN, dev)
    # a graph holding NCCL calls is released before the process group goes
    torch.cuda.synchronize()
    graph = None
    if peer is not None:
        torch.cuda.synchronize()
        barrier()
        peer.close()
        barrier()
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return

    # The dominant kernel runs in a timed region of ~0.1 s at full SM clock (see
    # "clocks"), so its denominator is the burst figure: twice the measured
    # burst bf16 rate (the B200 dense int8 rate is twice bf16 per clock).
    peaks = measured_peaks()
    bf16_burst = peaks.get("bf16_tflops")
    peak = 2.0 * (bf16_burst if bf16_burst else FALLBACK_BF16_BURST_TFLOPS)
    up_ops = 2.0 * m * W.FFN * W.HIDDEN
    achieved = up_ops / (ffn_ms / 1e3) / 1e12
    roofline = {
        "kernel": "ffn_up int8 GEMM + GELU-tanh epilogue (CTA-pair gemm_tc2_kernel<kGelu>), "
                  f"M={m} K={W.HIDDEN} N={W.FFN}",
        "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TOP/s (int8)",
        "frac": achieved / peak,
        "peak_source": ("of measured: 2 x bf16_tflops burst in MEASURED_PEAKS.json (B200 dense int8 = 2 x bf16 "
                        "per clock)" if bf16_burst else "of fallback: 2 x 1590 TFLOP/s bf16 burst"),
        "peak_int8_cublaslt_measured": ceiling,
        "frac_of_cublaslt_measured": achieved / ceiling if ceiling else None,
        "cublaslt_note": "torch._int_mm (cuBLASLt, int32 out, no epilogue) at the same shape on this GPU, this run",
        "peak_int8_at_sm_clock": 148 * 16384 * (clocks["sm_mhz"] if clocks and clocks.get("sm_mhz") else 1965.0)
        * 1e6 / 1e12,
        "frac_of_nominal_4500": achieved / NOMINAL_INT8_TOPS,
        "algorithmic_ops_per_launch": up_ops,
        "launch_ms": ffn_ms,
        "traffic": profile_traffic("gemm_ffn_up_m12240") if m == 12240 else None,
    }
    block_ops = 2.0 * total * W.HIDDEN * (3 * W.HIDDEN + 3 * W.HIDDEN + 2 * W.FFN) \
        + 2.0 * world * W.TEXT_TOKENS * W.TEXT_DIM * 2 * W.HIDDEN
    step_ms = elapsed_ms / args.steps
    line = {
        "metric": METRIC,
        "value": total * args.steps / (elapsed_ms / 1e3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": step_ms,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int8",
        "data": "synthetic (seeded; random-init int8 weights)",
        "config": workload_config(args, world),
        "block_tops": block_ops / (step_ms / 1e3) / 1e12,
        "allgather": None if world == 1 else {
            "mode": ("peer: the FFN-down GEMM epilogue stores its rows into every rank's gathered tensor over "
                     "NVLink (lr_int8_gemm_rows_to), then one stream-ordered NCCL barrier"
                     if peer is not None else "nccl: all_gather_into_tensor after the block"),
            "ms_per_step": ag_ms, "share_of_step": ag_ms / step_ms,
            "bytes_received_per_rank": (total - m) * d * 2,
            "algbw_GBps": total * d * 2 / (ag_ms / 1e3) / 1e9 if peer is None else None,
            "busbw_GBps": (world - 1) / world * total * d * 2 / (ag_ms / 1e3) / 1e9 if peer is None else None,
            "gathered_matches_unsharded": gathered_ok,
            "timing": ("CUDA events around the barrier after the fused GEMM (the transfer itself is inside the GEMM)"
                       if peer is not None else
                       "CUDA events around all_gather_into_tensor on the compute stream") +
                      ", mean over steps, max over ranks"},
        "replica": replica,
        "roofline": roofline,
        "clocks": clocks,
        "gpu_launches": block.LAUNCHES_PER_FORWARD * args.steps,
        "device_status": status,
        "step_graph": graph_note,
        "e2e": e2e,
    }
    if world == 1 and not args.no_cpu_baseline:
        wcpu = block.BlockWeights(**{k: (v.to("cpu") if hasattr(v, "to") else v)
                                     for k, v in weights.__dict__.items()})
        rate, info = cpu_block_rate(wcpu, total)
        line["cpu_baseline"] = {
            "value": rate, "unit": "tokens/s", "cores": info["cores"], "kind": "port",
            "sample": (f"the whole block: all {total} token rows, median of {info['repeats']} runs after one "
                       "warm-up"),
            "t_block_s": info["t_block_s"],
            "extrapolated_from_sample": info["extrapolated_from_sample"],
        }
    if isinstance(line.get("e2e"), dict):
        line["e2e"]["host_numa"] = numa
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_stack(args, rank, world, local):
    """Config 4: 42-block stack, 3 denoiser steps, 64512 tokens sharded by rows
    over the GPUs, one NCCL all-gather of the bf16 output at the end of a step.
    A step is one full stack forward (every denoiser step through every block)."""
    import torch.distributed as dist
    from lynnreal_omni_b200 import _lib, stack as S
    from lynnreal_omni_b200 import workloads as W
    from lynnreal_omni_b200.parallel import shard_bounds

    torch.cuda.set_device(local)
    numa = bind_local_numa(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    _lib.load()
    total = args.stack_tokens
    comp = None
    bounds = None
    if args.compress:
        from lynnreal_omni_b200.parallel import frame_bounds
        grid_h, grid_w = 48, 64
        if total % (grid_h * grid_w):
            raise SystemExit("--compress needs --stack-tokens a multiple of 48 x 64")
        frames = total // (grid_h * grid_w)
        bounds = [frame_bounds(frames, grid_h * grid_w, world, r) for r in range(world)]
        start_row, stop_row = bounds[rank]
        comp = S.Compression((stop_row - start_row) // (grid_h * grid_w), grid_h, grid_w, dev,
                             end=min(28, args.layers - 1), first_frame=start_row // (grid_h * grid_w))
    else:
        start_row, stop_row = shard_bounds(total, world, rank)
    m = stop_row - start_row
    model = S.FlashStackW8A8(args.layers, dev, seed=0)
    g = W.generator(100 + rank, dev)
    x_local = torch.randn(1, m, W.HIDDEN, generator=g, device=dev).to(torch.bfloat16)
    ctx = torch.randn(W.TEXT_TOKENS, W.TEXT_DIM, generator=g, device=dev).to(torch.bfloat16)
    idx = torch.zeros(m, dtype=torch.int64, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def step(ev=None, xin=None):
        return model.sharded_forward(x_local if xin is None else xin, total, world, rank, idx, ctx, ffn_events=ev,
                                     compression=comp, bounds=bounds)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    sampler = clock_sampler(dev, local) if rank == 0 else None
    if sampler:
        sampler.start()
    ffn = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    t0.record()
    for i in range(args.steps):
        out = step(ffn[i])
    t1.record()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop() if sampler else None
    t = torch.tensor([t0.elapsed_time(t1), statistics.mean(a.elapsed_time(b) for a, b in ffn)], device=dev,
                     dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms, ffn_ms = t.tolist()
    status = _lib.device_status(clear=True)

    # end to end: the latent rows from pinned host memory in, the gathered output back
    x_h = x_local.cpu().pin_memory()
    out_h = torch.empty((total, W.HIDDEN), dtype=torch.bfloat16).pin_memory()
    x_d = torch.empty_like(x_local)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        x_d.copy_(x_h, non_blocking=True)
        res = step(xin=x_d)
        out_h.copy_(res.view(total, W.HIDDEN) if world > 1 else res.view(-1, W.HIDDEN), non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    barrier()
    te = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    passes = S.DENOISER_STEPS * args.layers
    if rank == 0:
        peaks = measured_peaks()
        peak = 2.0 * (peaks.get("bf16_tflops") or FALLBACK_BF16_BURST_TFLOPS)
        up_ops = 2.0 * m * W.FFN * W.HIDDEN
        achieved = up_ops / (ffn_ms / 1e3) / 1e12
        if comp is not None:
            kept = comp.kept_rows()
            glob_kept = kept * world  # frames are alike: every full frame keeps the same rows
            token_passes = S.DENOISER_STEPS * (total * (args.layers - (comp.end - comp.start)) +
                                               glob_kept * (comp.end - comp.start))
        else:
            token_passes = total * passes
        line = {
            "metric": METRIC if comp is None else "Flash stack latent tokens/s (token compression in blocks 2-27)",
            "value": (total * passes if comp is None else total * S.DENOISER_STEPS) * args.steps / (elapsed_ms / 1e3),
            "unit": ("tokens/s (block-token passes: tokens x blocks x denoiser steps)" if comp is None
                     else "latent tokens/s (tokens x denoiser steps)"),
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic (seeded; random-init int8 weights)",
            "config": {"workload": "config4: 42-block Flash-like stack, 3 denoiser steps, tokens sharded by rows, "
                                   "final NCCL all-gather of the bf16 output",
                       "model": f"{args.layers} x Flash-like DiT block (D=6144, FFN 24576 GELU-tanh)",
                       "global_tokens": total, "tokens_per_gpu": m, "layers": args.layers,
                       "denoiser_steps": S.DENOISER_STEPS, "global_batch": 1, "seq_len": total,
                       "parallelism": f"dp{world} over token rows, weights replicated, all-gather at the end",
                       "l2": "no flush: 24.4 GB of weights streamed per denoiser step"},
            "latent_tokens_per_s": total * S.DENOISER_STEPS * args.steps / (elapsed_ms / 1e3),
            "block_token_passes_per_s": token_passes * args.steps / (elapsed_ms / 1e3),
            "compression": None if comp is None else {
                "grid": [total // 3072, 48, 64], "kept_rows_per_rank": comp.kept_rows(),
                "compressed_blocks": [comp.start, comp.end], "shards": "whole frames"},
            "roofline": {"kernel": f"ffn_up int8 GEMM + GELU (CTA-pair gemm_tc2_kernel<kGelu>), M={m} K={W.HIDDEN} N={W.FFN}",
                         "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TOP/s (int8)",
                         "frac": achieved / peak, "frac_of_nominal_4500": achieved / NOMINAL_INT8_TOPS,
                         "launch_ms": ffn_ms, "traffic": None},
            "clocks": clocks,
            "gpu_launches": (model.launches_per_forward() + (2 * S.DENOISER_STEPS if comp is not None else 0)) * args.steps,
            "device_status": status,
            "e2e": {"value": (total * passes if comp is None else total * S.DENOISER_STEPS) * args.steps
                              / (te.item() / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": x_h.numel() * 2, "d2h_bytes_per_step": out_h.numel() * 2,
                    "ms_per_step": te.item() / args.steps},
        }
        if isinstance(line.get("e2e"), dict):
            line["e2e"]["host_numa"] = numa
        print(json.dumps(line), flush=True)
    del out
    if world > 1:
        dist.destroy_process_group()


def run_sweep(args, rank, world, local):
    """Config 3: INT8 GEMM sweep M x (K, N), each shape's rows sharded over the
    ranks. Per shape: our GEMM (bf16 dequant epilogue) and cuBLASLt torch._int_mm
    (int32 out, no epilogue) on the same operands, each timed as a CUDA-graph
    replay of `steps` launches (device time, no host issue cost), max over ranks."""
    import torch.distributed as dist
    from lynnreal_omni_b200 import _lib, workloads as W
    from lynnreal_omni_b200.int8_gemm import int8_matmul
    from lynnreal_omni_b200.parallel import shard_bounds

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    _lib.load()

    def graph_ms(fn, reps):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(reps):
                fn()
        g.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        g.replay()
        t1.record()
        torch.cuda.synchronize()
        t = torch.tensor([t0.elapsed_time(t1) / reps], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        del g
        return t.item()

    peaks = measured_peaks()
    peak = 2.0 * (peaks.get("bf16_tflops") or FALLBACK_BF16_BURST_TFLOPS)
    rows = []
    for m_total in W.SWEEP_M:
        start, stop = shard_bounds(m_total, world, rank)
        m = stop - start
        for k, n in W.SWEEP_KN:
            gen = W.generator(1000 + m_total + k + n + rank, dev)
            a = torch.randint(-127, 128, (m, k), generator=gen, device=dev, dtype=torch.int8)
            b = torch.randint(-127, 128, (n, k), generator=gen, device=dev, dtype=torch.int8).t()
            rs = torch.rand(m, 1, generator=gen, device=dev) / 127
            cs = torch.rand(1, n, generator=gen, device=dev) / 127
            reps = max(3, min(args.steps, int(2e12 // max(1, 2 * m * n * k)) + 3))
            ours = graph_ms(lambda: int8_matmul(a, b, rs, cs), reps)
            a_pad = a if m >= 32 and m % 8 == 0 else torch.nn.functional.pad(a, (0, 0, 0, max(32, -(-m // 8) * 8) - m))
            cublas = graph_ms(lambda: torch._int_mm(a_pad, b), reps)
            ops = 2.0 * m_total * n * k
            rows.append({"m": m_total, "k": k, "n": n, "m_per_gpu": m, "ms": ours,
                         "tops": ops / (ours / 1e3) / 1e12, "frac_of_peak": ops / (ours / 1e3) / 1e12 / peak,
                         "cublaslt_int_mm_ms": cublas, "cublaslt_tops": ops / (cublas / 1e3) / 1e12,
                         "split_k": _lib.load().lr_int8_gemm_workspace_bytes(m, n, k) > 0})
            del a, b, rs, cs, a_pad
            torch.cuda.empty_cache()
    if rank == 0:
        total_ops = sum(2.0 * r["m"] * r["n"] * r["k"] for r in rows)
        total_ms = sum(r["ms"] for r in rows)
        line = {"metric": METRIC, "workload": "config3 GEMM sweep",
                "value": total_ops / (total_ms / 1e3) / 1e12, "unit": "TOP/s (int8, all shapes)",
                "n_gpus": world, "steps": args.steps, "higher_is_better": True, "scaling": "strong",
                "dtype": "int8", "data": "synthetic (seeded)", "peak": peak,
                "peak_source": "of measured: 2 x bf16_tflops burst (MEASURED_PEAKS.json)",
                "timing": "CUDA-graph replay per shape, device time, max over ranks",
                "shapes": rows}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_flash(args, rank, world, local):
    """One Flash DiT block at the released shapes (hidden 5376, 56 x 128 heads,
    SwiGLU 14336) per GPU, run through fusion.enable_fusion / fused_block:
    adaLN prologue, QKV GEMM, Q/K RMSNorm+RoPE, tcgen05 attention, O GEMM,
    residual+FFN prologue, SwiGLU FFN and gated residual, all on this package's
    kernels. Weak scaling: each rank runs its own latent."""
    import torch.distributed as dist
    import torch.nn.functional as F
    from types import SimpleNamespace
    from lynnreal_omni_b200 import _lib, fusion
    from lynnreal_omni_b200 import flash_block as FB
    from lynnreal_omni_b200.attention import attention_bshd

    torch.cuda.set_device(local)
    numa = bind_local_numa(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    _lib.load()
    m = args.tokens
    block = FB.FlashH3Block(seed=0, device=dev).eval()
    att_events = []

    def timed_attention(q, k, v, mask=None):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        out = attention_bshd(q, k, v, mask)
        b.record()
        att_events.append((a, b))
        return out

    fusion.enable_fusion(SimpleNamespace(transformer_blocks=[block]), fused_quant=True, attention_fn=timed_attention)
    x, temb, idx, rope = FB.make_inputs(m, seed=1 + rank, device=dev)
    with torch.no_grad():
        lin = block.adaln_proj.linear
        table = lin(F.silu(temb).to(lin.weight.dtype)).view(-1, 6 * FB.HIDDEN)

    def barrier():
        if world > 1:
            dist.barrier()

    def step(inp):
        with torch.no_grad():
            return block.forward(inp, temb, idx, rope, adaln_table=table)

    for _ in range(args.warmup):
        step(x)
    torch.cuda.synchronize()
    att_events.clear()
    sampler = clock_sampler(dev, local) if rank == 0 else None
    if sampler:
        sampler.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    t0.record()
    for _ in range(args.steps):
        out = step(x)
    t1.record()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop() if sampler else None
    att_ms = statistics.mean(a.elapsed_time(b) for a, b in att_events)
    t = torch.tensor([t0.elapsed_time(t1), att_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms, att_ms = t.tolist()
    status = _lib.device_status(clear=True)

    # end to end: latent in from pinned host memory, block output back, every step
    x_h = x.cpu().pin_memory()
    out_h = torch.empty(x.shape, dtype=torch.bfloat16).pin_memory()
    x_d = torch.empty_like(x)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        x_d.copy_(x_h, non_blocking=True)
        out_h.copy_(step(x_d), non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    barrier()
    te = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    if rank == 0:
        peaks = measured_peaks()
        bf16_peak = peaks.get("bf16_tflops") or FALLBACK_BF16_BURST_TFLOPS
        gemm_ops, att_flops = FB.ops_per_token(m)
        att_achieved = att_flops * m / (att_ms / 1e3) / 1e12
        line = {
            "metric": "Flash DiT-block tokens/s (released shapes, attention included)",
            "value": m * world * args.steps / (elapsed_ms / 1e3), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8 projections, bf16 attention",
            "data": "synthetic (seeded; random-init int8 weights)",
            "config": {"workload": "flash: one Flash DiT block at the released shapes through fusion.fused_block",
                       "model": "hidden 5376, 56 x 128 heads (QKV 5376->21504, O 7168->5376), SwiGLU 5376->2x14336->5376",
                       "tokens_per_gpu": m, "global_batch": world, "seq_len": m,
                       "parallelism": f"dp{world} (own latent per GPU, no collective)",
                       "adaln_table": "precomputed once (time-modulation cache)",
                       "l2": "no flush: per-step working set (0.38 GB int8 weights + ~1.5 GB activations) >> 126 MB L2"},
            "block_int8_tops": gemm_ops * m / ((elapsed_ms - att_ms * args.steps) / args.steps / 1e3) / 1e12,
            "roofline": {"kernel": f"tcgen05 attention (attention_kernel), {m} tokens x 56 heads x 128",
                         "bound": "tensor", "achieved": att_achieved, "peak": bf16_peak, "unit": "TFLOP/s (bf16)",
                         "frac": att_achieved / bf16_peak,
                         "peak_source": "of measured: bf16_tflops burst in MEASURED_PEAKS.json",
                         "launch_ms": att_ms, "share_of_step": att_ms / (elapsed_ms / args.steps), "traffic": None},
            "clocks": clocks,
            "gpu_launches": 11 * args.steps,
            "device_status": status,
            "e2e": {"value": m * world * args.steps / (te.item() / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": x_h.numel() * 2, "d2h_bytes_per_step": out_h.numel() * 2,
                    "ms_per_step": te.item() / args.steps},
        }
        if isinstance(line.get("e2e"), dict):
            line["e2e"]["host_numa"] = numa
        print(json.dumps(line), flush=True)
    del out
    if world > 1:
        dist.destroy_process_group()


def run_reference_kernels(args, rank, world, local):
    """The path's kernels beside the reference's own compiled GPU kernels on
    one B200 (the reference installed into baseline/_ref): per op, the device
    time of each (CUDA-graph replay of `steps` calls, warm) and whether the
    outputs are identical. The reference's INT8 GEMM kernel does not compile
    under this image's Triton, so its int8_matmul runs its PyTorch path
    (cuBLASLt integer GEMM + torch epilogue), which is what it executes here."""
    if rank != 0:
        return
    import warnings
    from types import SimpleNamespace
    ref_root = Path(__file__).resolve().parent / "baseline" / "_ref"
    if not (ref_root / "lynnreal" / "model" / "kernels.py").exists():
        print(json.dumps({"workload": "reference_kernels", "unavailable": "reference not installed in baseline/_ref"}))
        return
    sys.path.insert(0, str(ref_root))
    import triton
    import lynnreal.model.int8_gemm as rg
    import lynnreal.model.kernels as rk
    from lynnreal_omni_b200 import _lib, kernels as K
    from lynnreal_omni_b200.int8_gemm import int8_matmul
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    _lib.load()
    _lib.set_arithmetic("reference_gpu")
    g = torch.Generator(device=dev).manual_seed(0)
    m, d, inner = args.tokens, 6144, 14336

    def device_us(fn, reps):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(reps):
                fn()
        graph.replay()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        graph.replay()
        t1.record()
        torch.cuda.synchronize()
        del graph
        return t0.elapsed_time(t1) / reps * 1e3

    x = torch.randn(1, m, d, device=dev, generator=g).bfloat16()
    y = torch.randn(1, m, d, device=dev, generator=g).bfloat16()
    norm = SimpleNamespace(weight=(1 + 0.05 * torch.randn(d, device=dev, generator=g)).bfloat16(), eps=1e-6)
    table = (0.1 * torch.randn(1, 6 * d, device=dev, generator=g)).bfloat16()
    idx = torch.zeros(m, dtype=torch.int64, device=dev)
    xw = torch.randn(m, 4 * d, device=dev, generator=g).bfloat16()
    proj = torch.randn(m, 2 * inner, device=dev, generator=g).bfloat16()
    heads = 48
    qkv = torch.randn(1, m, 3 * heads * 128, device=dev, generator=g).bfloat16()
    q, k, _ = [t.unflatten(-1, (heads, -1)) for t in qkv.chunk(3, dim=-1)]
    phase = torch.randn(m, 128, device=dev, generator=g)
    cos, sin = phase.cos(), phase.sin()

    def ref_qk():
        q_out = torch.empty_like(q, memory_format=torch.contiguous_format)
        k_out = torch.empty_like(k, memory_format=torch.contiguous_format)
        rk._qk_norm_full_rope_paired_kernel[(q.numel() // 128,)](
            q, k, norm.weight[:128], norm.weight[128:256], cos, sin, q_out, k_out, m, heads, q.stride(1),
            q.stride(2), k.stride(1), k.stride(2), 128, 1e-6, 64, num_warps=4, enable_fp_fusion=False)
        return q_out, k_out

    nq = SimpleNamespace(weight=norm.weight[:128], eps=1e-6)
    nk = SimpleNamespace(weight=norm.weight[128:256], eps=1e-6)
    ops = [
        ("quantize_rows", [m, d], lambda: K.quantize_rows(x.view(m, d)), lambda: rk.quantize_rows(x.view(m, d))),
        ("quantize_rows", [m, 4 * d], lambda: K.quantize_rows(xw), lambda: rk.quantize_rows(xw)),
        ("_rms_adaln_quant_int8", [m, d], lambda: K._rms_adaln_quant_int8(x, norm, table, idx, 0, 1),
         lambda: rk._rms_adaln_quant_int8(x, norm, table, idx, 0, 1)),
        ("_rms_adaln", [m, d], lambda: K._rms_adaln(x, norm, table, idx, 3, 4),
         lambda: rk._rms_adaln(x, norm, table, idx, 3, 4)),
        ("residual_rms_quant", [m, d], lambda: K.residual_rms_quant(x, y, norm, table, idx),
         lambda: rk.residual_rms_quant(x, y, norm, table, idx)),
        ("_gated_residual", [m, d], lambda: K._gated_residual(x, y, table, idx, 2),
         lambda: rk._gated_residual(x, y, table, idx, 2)),
        ("_swiglu", [m, 2 * inner], lambda: K._swiglu(proj), lambda: rk._swiglu(proj)),
        ("_swiglu_quant_int8", [m, 2 * inner], lambda: K._swiglu_quant_int8(proj), lambda: rk._swiglu_quant_int8(proj)),
        ("qk_norm_rope (full rotary)", [m, heads, 128], lambda: K.qk_norm_rope(q, k, nq, nk, (cos, sin)), ref_qk),
    ]
    for kk, nn in ((d, d), (d, 4 * d), (4 * d, d)):
        a = torch.randint(-127, 128, (m, kk), generator=g, device=dev, dtype=torch.int8)
        b = torch.randint(-127, 128, (nn, kk), generator=g, device=dev, dtype=torch.int8).t()
        rs = torch.rand(m, 1, generator=g, device=dev) / 127
        cs = torch.rand(1, nn, generator=g, device=dev) / 127
        bias = (0.02 * torch.randn(nn, generator=g, device=dev)).bfloat16()
        ops.append(("int8_matmul", [m, kk, nn], (lambda a=a, b=b, rs=rs, cs=cs, bias=bias: int8_matmul(a, b, rs, cs, bias)),
                    (lambda a=a, b=b, rs=rs, cs=cs, bias=bias: rg.int8_matmul(a, b, rs, cs, bias))))
    rows = []
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")  # the reference reports its GEMM falling back to its torch path
        for name, shape, ours, theirs in ops:
            a_out, b_out = ours(), theirs()
            a_out = a_out if isinstance(a_out, tuple) else (a_out,)
            b_out = b_out if isinstance(b_out, tuple) else (b_out,)
            identical = all(torch.equal(u, v) for u, v in zip(a_out, b_out))
            reps = max(3, args.steps)
            t_ours, t_ref = device_us(ours, reps), device_us(theirs, reps)
            rows.append({"op": name, "shape": shape, "ours_us": round(t_ours, 1), "reference_us": round(t_ref, 1),
                         "speedup": round(t_ref / t_ours, 2), "identical": identical})
    print(json.dumps({"workload": "reference_kernels", "gpu": torch.cuda.get_device_name(dev),
                      "arithmetic": _lib.arithmetic(), "timing": "CUDA-graph replay, device time per call",
                      "reference": f"baseline/_ref, Triton {triton.__version__}", "ops": rows}))


def _case_time(fn, iters: int, warmup: int, graph: bool = False):
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


def run_kernel_case(args):
    """One kernel of the path on synthetic inputs, for profilers and timing:
    ``--case`` gemm (``--epi`` none/gelu/gated), rms (K4), quant (K1), gated
    (K5), residual_rms (K8), qk (Q/K RMSNorm + RoPE), compress / restore /
    restore_torch / layout (token compression on a 21 x 48 x 64 grid), attn /
    attn_sdpa (48 heads x 128 at ``--m`` tokens). Launches the kernel
    ``--steps`` times on cuda:0 after ``--warmup`` calls (``--graph``: as one
    CUDA-graph replay) and prints the mean CUDA-event time per launch and the
    algorithmic rate."""
    from types import SimpleNamespace
    from lynnreal_omni_b200 import _lib
    _lib.load()
    a = args
    from lynnreal_omni_b200 import kernels as K
    from lynnreal_omni_b200.int8_gemm import int8_matmul, int8_matmul_gated_residual, int8_matmul_gelu
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
        ms = _case_time(fn, a.steps, a.warmup, a.graph)
        out.update(m=a.m, k=a.k, n=a.n, epi=a.epi, ms=ms, tops=2.0 * a.m * a.n * a.k / (ms / 1e3) / 1e12,
                   algorithmic_bytes=a.m * a.k + a.n * a.k + 2 * a.m * a.n + 4 * a.m + 6 * a.n)
    elif a.case == "qk":
        heads, hd = a.d // 128, 128
        qkv = torch.randn(1, a.m, 3 * a.d, device=dev, generator=g).to(torch.bfloat16)
        q, k, _ = [t.unflatten(-1, (heads, -1)) for t in qkv.chunk(3, dim=-1)]
        nq = SimpleNamespace(weight=torch.ones(hd, device=dev, dtype=torch.bfloat16), eps=1e-6)
        phase = torch.randn(a.m, hd, device=dev, generator=g)
        rot = (phase.cos(), phase.sin())
        ms = _case_time(lambda: K.qk_norm_rope(q, k, nq, nq, rot), a.steps, a.warmup, a.graph)
        nbytes = 8 * a.m * a.d + 8 * a.m * hd + 4 * hd
        out.update(m=a.m, d=a.d, heads=heads, ms=ms, algorithmic_bytes=nbytes, gbs=nbytes / (ms / 1e3) / 1e9)
    elif a.case in ("attn", "attn_sdpa"):
        from lynnreal_omni_b200.attention import attention_bshd
        heads = a.d // 128
        qkv = torch.randn(1, a.m, 3 * a.d, device=dev, generator=g).to(torch.bfloat16)
        q, k, v = [t.unflatten(-1, (heads, -1)) for t in qkv.chunk(3, dim=-1)]
        if a.case == "attn":
            fn = lambda: attention_bshd(q, k, v)  # noqa: E731
        else:
            qt, kt, vt = (t.transpose(1, 2) for t in (q, k, v))
            fn = lambda: torch.nn.functional.scaled_dot_product_attention(qt, kt, vt)  # noqa: E731
        ms = _case_time(fn, a.steps, a.warmup, a.graph)
        flops = 4.0 * heads * a.m * a.m * 128
        out.update(m=a.m, heads=heads, ms=ms, tflops=flops / (ms / 1e3) / 1e12)
    elif a.case in ("compress", "restore", "restore_torch", "layout"):
        from lynnreal_omni_b200 import flash
        t, h, w = torch.meshgrid(torch.arange(21), torch.arange(48), torch.arange(64), indexing="ij")
        pos = torch.stack([t, h, w], -1).reshape(-1, 3).to(dev)
        tags = torch.zeros(pos.shape[0], dtype=torch.int64, device=dev)
        keep, inverse = flash.spatial_layout(pos, tags)
        s, kept = pos.shape[0], keep.numel()
        if a.case == "layout":
            ms = _case_time(lambda: flash.spatial_layout(pos, tags), a.steps, a.warmup, False)
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
            ms = _case_time(fn, a.steps, a.warmup, a.graph)
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
        ms = _case_time(fn, a.steps, a.warmup, a.graph)
        nbytes = per_elem * a.m * a.d + 4 * a.m
        out.update(m=a.m, d=a.d, ms=ms, algorithmic_bytes=nbytes, gbs=nbytes / (ms / 1e3) / 1e9)
    print(json.dumps(out), flush=True)


def main():
    args = parse_args()
    rank, world, local = dist_env()
    if args.impl == "reference":
        if rank == 0:
            run_reference(args, world)
        return
    if args.workload == "stack":
        run_stack(args, rank, world, local)
    elif args.workload == "sweep":
        run_sweep(args, rank, world, local)
    elif args.workload == "flash":
        run_flash(args, rank, world, local)
    elif args.workload == "reference_kernels":
        run_reference_kernels(args, rank, world, local)
    elif args.workload == "kernel":
        run_kernel_case(args)
    else:
        run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
