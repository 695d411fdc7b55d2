#!/usr/bin/env python
"""Benchmark of the B200 attention engine on tensorsmith's attention path.

Workload ("c5"): long-context causal prefill + cached
decode, bf16, B=32, H=32, D=128, T=32768 prefill then 128 decode steps, inputs
~ N(0,1) from a seed, (batch, head) pairs sharded over the N GPUs of one node
with no reduction and every output gathered to rank 0 over NCCL.  Total work
is fixed as N grows (strong scaling).

One step = prefill forward of the whole batch (tcgen05 kernel) + gather of O,
then 128 x (KV append + split-K decode + gather of the token's output).

Metric: prefill TFLOP/s & % bf16 peak; decode tokens/s & HBM
GB/s.  ``value`` is whole-job prefill TFLOP/s (causal algorithmic FLOPs
4*D*pairs / max-over-ranks device time); decode figures ride along under
``decode``.  ``e2e`` repeats the step through the public API with pinned host
inputs (H2D of Q/K/V and every decode token, D2H of O and decode outputs).

``--impl reference`` times the reference algorithm (the NumPy port under
oracle/, the reference being Python that cannot travel) on the host cores on a
bounded sample of the same workload, and prints the same metric.
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

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT), str(ROOT / "custom-ml-library_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "prefill TFLOP/s & % bf16 peak; decode tokens/s & HBM GB/s; at 1/2/4/8 GPUs"
WORKLOADS = {
    "c5": dict(batch=32, heads=32, head_dim=128, prefill=32768, decode_steps=128),
    # reduced shape of the same kernels, for profiler captures only
    "small": dict(batch=4, heads=32, head_dim=128, prefill=4096, decode_steps=4),
    # the C5 prefill shape on 8 (b,h) pairs (forward + backward, 268 MB of inputs): profiler captures
    "c5slice": dict(batch=1, heads=8, head_dim=128, prefill=32768, scale_inputs=False),
    # causal attention forward + backward, fp32 (the exact CUDA-core kernels)
    "c1": dict(batch=2, heads=4, head_dim=64, prefill=256),
    # causal prefill bf16 forward + backward
    "c3": dict(batch=8, heads=16, head_dim=128, prefill=4096, scale_inputs=True),
    # 4-layer decoder LM training step (fp16 autocast, fp32 params), B=16, T=256
    "c2": dict(batch=16, seq=256, vocab=8192, dim=256, heads=4, layers=4, hidden=1024),
    # fp16 KV-cache decode, ragged lengths U[1024, 8192], 256 steps with append
    "c4": dict(batch=64, heads=32, head_dim=128, min_len=1024, max_len=8192, decode_steps=256),
    # config 3 with the int8 KV cache (KVCache(quantized=True)): quantising append + fused-dequant decode
    "c4q": dict(batch=64, heads=32, head_dim=128, min_len=1024, max_len=8192, decode_steps=256),
    # config 3 with grouped-query attention (4 query heads per KV head): the grouped decode kernel
    "c4gqa": dict(batch=64, heads=32, kv_heads=8, head_dim=128, min_len=1024, max_len=8192, decode_steps=256),
    # reduced c4q (0.55 GB int8 cache, still larger than L2), for profiler captures only
    "c4q_small": dict(batch=8, heads=32, head_dim=128, min_len=1024, max_len=8192, decode_steps=16),
}
# Query rows per prefill chunk when N > 1 (each chunk's output gather overlaps the next chunk).
PREFILL_CHUNK_ROWS = 4096
# CTAs the overlapped prefill gathers may use (NCCL config max_ctas of their own process group):
# NCCL's blocks take whole SMs from the compute-bound forward while they run.  Measured on 2 B200s
# (prefill ms = forward + gather tail): NCCL's default 164.2 + 0.6, a cap of 2 152.4 + 25.4, 4
# 153.2 + 10.6, 8 155.1 + 4.1, 16 157.7 + 2.1; one gather after an unchunked forward 151.0 + 6.2.
PREFILL_GATHER_CTAS = 8
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of the scored kernel, from the ncu
# captures summarised under profiles/, per unit of work so a launch of any size scales by its units.
PROFILED_TRAFFIC = {
    # tc_fwd_pair_kernel<128,bf16> at T=32768, 8 (b,h) pairs: (202.6 + 49.2) MB / 8 pairs
    "c5": dict(bytes_per_unit=31.48e6, unit="(b,h) pair at T=32768",
               source="profiles/tc_fwd_pair_kernel_c5slice.md"),
    # tc_bwd_kernel<128,bf16> at the C3 shape: 809.6 MB read + 494.3 MB written per launch
    "c3": dict(bytes_per_unit=1303.9e6, unit="C3 backward launch", source="profiles/tc_bwd_kernel_c3.md"),
    # split-K decode: DRAM bytes / algorithmic K+V bytes = (268.6 + 4.1) / 268.5
    "c4": dict(bytes_per_unit=1.0156, unit="algorithmic K+V byte", source="profiles/decode_split_kernel_small.md"),
    # grouped decode on the tcgen05 kernel: (1363.9 + 4.6) / 1345.5 (algorithmic K+V bytes of that step)
    "c4gqa": dict(bytes_per_unit=1.0171, unit="algorithmic K+V byte",
                  source="profiles/tc_fwd_kernel_gqa_decode_c4gqa.md"),
}


def profiled_traffic(key: str, units: float):
    """Per-launch DRAM traffic scaled from a committed ncu capture, or None."""
    entry = PROFILED_TRAFFIC.get(key)
    if entry is None:
        return None
    return {"bytes": entry["bytes_per_unit"] * units, "per": entry["unit"], "units": units,
            "source": entry["source"] + " (ncu capture, scaled by the units of this launch)"}
CLOCK_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["engine", "reference"], default="engine")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="c5")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU-baseline sample budget")
    ap.add_argument("--dropout", type=float, default=0.0,
                    help="c3: attention dropout probability in the timed forward and backward")
    ap.add_argument("--clock-log", default=None,
                    help="file for the nvidia-smi clock samples of the timed region (default: a temp file)")
    return ap.parse_args()


def causal_flops(pairs: int, tq: int, tk: int, offset: int, d: int) -> float:
    """Forward FLOPs 4*D*sum_i min(Tk, i+1+offset) over all (b,h) pairs."""
    import numpy as np

    i = np.arange(tq, dtype=np.int64)
    return 4.0 * d * pairs * float(np.minimum(tk, i + 1 + offset).sum())


def load_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return data, "measured"
    return FALLBACK_PEAKS, "fallback"


# --------------------------------------------------------------------------
# parity of the timed outputs: an fp64 restatement of attention on sampled
# rows, run on the host after the timed region (not the oracle package)
# --------------------------------------------------------------------------
def ref_rows(q_rows, k, v, limits, scale):
    """fp64 attention of query rows q_rows [R, D] against k [L, D] / v [L, C]; row r sees keys
    [0, limits[r]).  Returns (out [R, C], lse [R])."""
    import torch

    s = (q_rows.double() @ k.double().T) * scale
    keys = torch.arange(k.shape[0])
    s = s.masked_fill(keys[None, :] >= torch.as_tensor(limits)[:, None], float("-inf"))
    m = s.max(dim=1, keepdim=True).values
    e = torch.exp(s - m)
    l = e.sum(dim=1, keepdim=True)
    return (e @ v.double()) / l, (m + torch.log(l))[:, 0]


def ref_slice_backward(q, k, v, do, scale, keep=None, drop_p=0.0):
    """fp64 causal attention of one (b, h) slice and its VJP: (o, lse, dq, dk, dv).  With a
    keep mask [T, T] the probabilities are scaled by keep / (1 - drop_p) before P.V and dP by
    the same factor, as the reference's dense dropout (nn/attention.py:140-144, 212-216)."""
    import torch

    q, k, v, do = (x.double() for x in (q, k, v, do))
    t = q.shape[0]
    s = (q @ k.T) * scale
    s = s.masked_fill(torch.ones(t, t, dtype=torch.bool).triu(1), float("-inf"))
    lse = torch.logsumexp(s, dim=1)
    p = torch.exp(s - lse[:, None])
    f = None if keep is None else keep.double() / (1.0 - drop_p)
    pd = p if f is None else p * f
    o = pd @ v
    dv = pd.T @ do
    dp = do @ v.T
    if f is not None:
        dp = dp * f
    ds = p * (dp - (do * o).sum(dim=1, keepdim=True)) * scale
    return o, lse, ds @ k, ds.T @ q, dv


def max_abs(got, ref) -> float:
    return float((got.double().cpu() - ref.double().cpu()).abs().max())


# --------------------------------------------------------------------------
# clocks sampled during the timed region
# --------------------------------------------------------------------------
class ClockSampler:
    def __init__(self, gpu_index: int, path=None):
        self.proc = None
        if path is None:
            fd, path = tempfile.mkstemp(prefix=f"ts_clocks_gpu{gpu_index}_", suffix=".csv")
            os.close(fd)
        self.path = Path(path)
        try:
            self.path.parent.mkdir(parents=True, exist_ok=True)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={CLOCK_FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(gpu_index), "-lms", "200"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons = [], 0.0, set()
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                clock, cmax = float(parts[1]), float(parts[2])
            except ValueError:
                continue
            sm.append(clock)
            mx = max(mx, cmax)
            names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        loaded = [c for c in sm if c > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------------
# reference arm / CPU baseline: the NumPy port of the reference algorithm
# --------------------------------------------------------------------------
def cpu_prefill_sample(cfg, rows: int, budget_s: float, seed: int = 0):
    """Streaming-forward of the last ``rows`` queries of one (b,h) slice.

    Returns (algorithmic FLOPs per rep, seconds per rep, reps)."""
    import numpy as np

    import oracle

    t, d = cfg["prefill"], cfg["head_dim"]
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((1, 1, rows, d), dtype=np.float32)
    k = rng.standard_normal((1, 1, t, d), dtype=np.float32)
    v = rng.standard_normal((1, 1, t, d), dtype=np.float32)
    flops = causal_flops(1, rows, t, t - rows, d)
    times = []
    start = time.perf_counter()
    while not times or (time.perf_counter() - start < budget_s and len(times) < 50):
        t0 = time.perf_counter()
        oracle.attention_forward(q, k, v, is_causal=True, causal_offset=t - rows,
                                 algorithm="streaming", block_size=2048)
        times.append(time.perf_counter() - t0)
    return flops, statistics.median(times), len(times)


def cpu_decode_sample(cfg, pairs: int, reps: int = 3, seed: int = 1):
    """One decode step for ``pairs`` (b,h) pairs against an fp16 cache of length T."""
    import numpy as np

    import oracle

    t, d = cfg["prefill"], cfg["head_dim"]
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((1, pairs, t, d)).astype(np.float16)
    v = rng.standard_normal((1, pairs, t, d)).astype(np.float16)
    q = rng.standard_normal((1, pairs, 1, d)).astype(np.float16)
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        oracle.attention_forward(q, k, v, is_causal=True, causal_offset=t - 1, algorithm="dense")
        times.append(time.perf_counter() - t0)
    per_pair = statistics.median(times) / pairs
    bytes_per_pair = 2.0 * t * d * 2
    return per_pair, bytes_per_pair


def cpu_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_baseline(cfg, budget_s: float):
    rows = 512
    flops, sec, reps = cpu_prefill_sample(cfg, rows, budget_s)
    per_pair, bpp = cpu_decode_sample(cfg, 2)
    b, h = cfg["batch"], cfg["heads"]
    return {
        "value": flops / sec / 1e12,
        "unit": "TFLOP/s",
        "cores": cpu_cores(),
        "kind": "port",
        "sample": (f"oracle streaming forward (NumPy fp32, block 2048) of the last {rows} query rows of one "
                   f"(b,h) slice vs T={cfg['prefill']} keys, median of {reps} reps; decode: 2 (b,h) pairs "
                   f"x 1 token vs fp16 cache T={cfg['prefill']}"),
        "decode_tokens_per_s": b / (per_pair * b * h),
        "decode_gbs": bpp / per_pair / 1e9,
    }


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return
    cfg = WORKLOADS[args.workload]
    if "prefill" not in cfg:
        print(json.dumps({"impl": "reference", "workload": args.workload,
                          "unavailable": "the reference arm times the prefill+decode workloads (c5, small, c3); "
                                         "the decode-only configs report the oracle port as cpu_baseline"}))
        return
    budget = max(2.0, min(args.cpu_seconds, 8.0))
    values, decode = [], []
    for step in range(args.warmup + args.steps):
        base = cpu_baseline(cfg, budget if step >= args.warmup else 1.0)
        if step >= args.warmup:
            values.append(base["value"])
            decode.append(base["decode_tokens_per_s"])
    value = statistics.median(values)
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{args.workload}: causal prefill B={cfg['batch']} H={cfg['heads']} "
                               f"D={cfg['head_dim']} T={cfg['prefill']} + {cfg['decode_steps']} decode steps",
                   "sample": "bounded CPU sample, see cpu_baseline"},
        "impl": "reference",
        "decode": {"tokens_per_s": statistics.median(decode)},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cpu_cores(), "kind": "port",
                         "sample": base["sample"]},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
# engine arm
# --------------------------------------------------------------------------
def parity_c5(q, kc, vc, prefill_rows, qd, od, T, S, D, seed=7):
    """Sampled check of the timed step's outputs on this rank: the first and last (b,h) pair,
    the last 128 prefill rows plus 128 random ones, and decode steps 0 and S-1."""
    import torch

    gen = torch.Generator().manual_seed(seed)
    n = q.shape[1]
    rows = torch.cat([torch.arange(T - 128, T), torch.randperm(T - 128, generator=gen)[:128].sort().values])
    scale = D ** -0.5
    err_o = err_d = 0.0
    for pr in sorted({0, n - 1}):
        kh, vh = kc[0, pr, : T + S].cpu(), vc[0, pr, : T + S].cpu()
        ref, _ = ref_rows(q[0, pr].cpu()[rows], kh[:T], vh[:T], rows + 1, scale)
        err_o = max(err_o, max_abs(prefill_rows(pr)[rows], ref))
        for st in sorted({0, S - 1}):
            ref_d, _ = ref_rows(qd[st, 0, pr].cpu(), kh, vh, [T + st + 1], scale)
            err_d = max(err_d, max_abs(od[st, 0, pr].cpu(), ref_d))
    return {"max_abs_prefill_out": err_o, "max_abs_decode_out": err_d, "tolerance_max_abs": 2e-2,
            "pass": max(err_o, err_d) <= 2e-2,
            "rows": f"(b,h) pairs {sorted({0, n - 1})} of rank 0: last 128 + 128 random prefill rows, "
                    f"decode steps {sorted({0, S - 1})}; fp64 reference on the host"}


def run_engine(args, rank: int, world: int, local_rank: int):
    import numpy as np
    import torch
    import torch.distributed as dist

    from tensorsmith_b200 import engine
    from tensorsmith_b200.distributed import RootWindow, ShardPlan, gather_to_root

    cfg = WORKLOADS[args.workload]
    B, H, D, T, S = cfg["batch"], cfg["heads"], cfg["head_dim"], cfg["prefill"], cfg["decode_steps"]
    cap = T + S
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    plan = ShardPlan(B, H, world, rank)
    n = plan.size  # pairs on this rank, laid out as [1, n, T, D]
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    bf = torch.bfloat16

    def randn(*shape):
        return torch.randn(*shape, generator=gen, device=dev, dtype=torch.float32).to(bf)

    q = randn(1, n, T, D)
    kc = torch.zeros(1, n, cap, D, dtype=bf, device=dev)
    vc = torch.zeros_like(kc)
    kc[:, :, :T].copy_(randn(1, n, T, D))
    vc[:, :, :T].copy_(randn(1, n, T, D))
    o = torch.empty(1, n, T, D, dtype=bf, device=dev) if world == 1 else None
    qd = randn(S, 1, n, 1, D)
    kd = randn(S, 1, n, 1, D)
    vd = randn(S, 1, n, 1, D)
    od = torch.empty(S, 1, n, 1, D, dtype=bf, device=dev)
    od_full = torch.empty(S, world, n, 1, D, dtype=bf, device=dev) if rank == 0 and world > 1 else None
    ws = torch.empty(max(16, engine.decode_workspace_bytes(qd[0], kc[:, :, : T + 1], vc[:, :, : T + 1],
                                                             is_causal=True, causal_offset=T)),
                     dtype=torch.uint8, device=dev)
    torch.cuda.synchronize()

    splits = engine.decode_workspace_bytes(qd[0], kc[:, :, :cap], vc[:, :, :cap], is_causal=True,
                                           causal_offset=cap - 1) > 0
    # With N > 1 the prefill runs in query-row chunks, longest first, and each
    # chunk's output is gathered asynchronously (on the process group's stream)
    # while the next chunk computes; the step waits for the gathers before the
    # decode loop.  The CTAs of one chunk have similar causal lengths, so the
    # chunks add little tail (splitting by blocks of pairs instead costs a full
    # causal tail per block).  Rank 0 receives chunk c of every rank in
    # o_full_parts[c] ([world, pairs, rows_c, D]).  One GPU runs one launch.
    # Each decode token's gather is queued the same way and waited for at the
    # end of the step, so it overlaps the next token's append and decode.
    rows_per_chunk = T if world == 1 else min(T, PREFILL_CHUNK_ROWS)
    chunks = [(r0, min(T, r0 + rows_per_chunk)) for r0 in range(0, T, rows_per_chunk)][::-1]
    o_parts = ([torch.empty(1, n, r1 - r0, D, dtype=bf, device=dev) for r0, r1 in chunks] if world > 1 else None)
    # Prefill outputs reach rank 0 by copy-engine writes into one buffer of rank
    # 0 (CUDA IPC over NVLink; no SMs taken from the forward that runs
    # meanwhile); chunk c of rank r lands at [c][r] of it.  Where a rank cannot
    # map rank 0's buffer, every rank keeps the NCCL gathers.
    window = None
    chunk_elems = [world * n * (r1 - r0) * D for r0, r1 in chunks]
    chunk_base = [sum(chunk_elems[:c]) for c in range(len(chunks))]
    if world > 1:
        window = RootWindow((sum(chunk_elems),), bf, dev)
        if not window.ok:
            window.close()
            window = None
    if window is not None:
        o_full_parts = ([window.buffer[chunk_base[c]: chunk_base[c] + chunk_elems[c]].view(world, n, r1 - r0, D)
                         for c, (r0, r1) in enumerate(chunks)] if rank == 0 else None)
    else:
        o_full_parts = ([torch.empty(world, n, r1 - r0, D, dtype=bf, device=dev) for r0, r1 in chunks]
                        if rank == 0 and world > 1 else None)
    copy_stream = torch.cuda.Stream(device=dev) if window is not None else None
    chunk_done = [torch.cuda.Event() for _ in chunks]
    # Chunks alternate between two streams: they are independent, so each
    # chunk's CTAs fill the SMs that the previous chunk's last wave leaves idle.
    chunk_streams = [torch.cuda.Stream(device=dev) for _ in range(2)] if world > 1 else None
    launches_per_step = len(chunks) + S * (2 + (1 if splits else 0))

    def prefill_rows(pr):
        """Prefill output rows of local pair ``pr`` on the host, [T, D]."""
        if o_parts is None:
            return o[0, pr].cpu()
        return torch.cat([o_parts[c][0, pr].cpu() for c in sorted(range(len(chunks)), key=lambda c: chunks[c][0])])

    def gather(src, dst):
        if world > 1:
            gather_to_root(src, plan, out=dst)

    def gather_async(src, full, group=None):
        # full: [world, ...] on rank 0; rank r's shard lands in full[r:r+1]
        targets = None if full is None else [full[r : r + 1] for r in range(world)]
        return gather_to_root(src, plan, out=targets, async_op=True, group=group)

    prefill_group = None
    if world > 1:
        opts = dist.ProcessGroupNCCL.Options()
        opts.config.max_ctas = PREFILL_GATHER_CTAS
        prefill_group = dist.new_group(list(range(world)), pg_options=opts)

    def step(ev):
        ev[0].record()
        works = []
        if world == 1:
            engine.forward(q, kc[:, :, :T], vc[:, :, :T], is_causal=True, need_lse=False, out=o)
        else:
            main = torch.cuda.current_stream()
            for cs in chunk_streams:
                cs.wait_stream(main)
            for c, (r0, r1) in enumerate(chunks):
                with torch.cuda.stream(chunk_streams[c % 2]):
                    engine.forward(q[:, :, r0:r1], kc[:, :, :r1], vc[:, :, :r1], is_causal=True, causal_offset=r0,
                                   need_lse=False, out=o_parts[c])
                    if window is not None:
                        chunk_done[c].record()
                        copy_stream.wait_event(chunk_done[c])
                        window.put(o_parts[c], 2 * (chunk_base[c] + rank * n * (r1 - r0) * D), copy_stream)
                    else:
                        works.append(gather_async(o_parts[c], None if o_full_parts is None else o_full_parts[c],
                                                  prefill_group))
            for cs in chunk_streams:
                main.wait_stream(cs)
        ev[1].record()
        if window is not None:
            torch.cuda.current_stream().wait_stream(copy_stream)
            window.done(dev)
        for work in works:
            work.wait()
        ev[2].record()
        works = []
        for s in range(S):
            engine.kv_append(kd[s], vd[s], kc, vc, position=T + s)
            engine.decode(qd[s], kc[:, :, : T + s + 1], vc[:, :, : T + s + 1], is_causal=True,
                          causal_offset=T + s, out=od[s], workspace=ws)
            if world > 1:
                works.append(gather_async(od[s], None if od_full is None else od_full[s]))
        for work in works:
            work.wait()
        ev[3].record()

    def new_events():
        return [torch.cuda.Event(enable_timing=True) for _ in range(4)]

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step(new_events())
    barrier()
    engine.check_device_status(dev)
    sampler = ClockSampler(local_rank, args.clock_log) if rank == 0 else None
    barrier()
    evs = [new_events() for _ in range(args.steps)]
    t_start = torch.cuda.Event(enable_timing=True)
    t_stop = torch.cuda.Event(enable_timing=True)
    t_start.record()
    for ev in evs:
        step(ev)
    t_stop.record()
    barrier()
    clocks = sampler.stop() if sampler else None
    engine.check_device_status(dev)
    prefill_transport = "copy engine (CUDA IPC)" if window is not None else "NCCL"
    if window is not None:
        # Every rank's last chunk as rank 0 received it must equal the rank's own output.
        sums = [None] * world
        dist.all_gather_object(sums, [float(o_parts[c].double().sum()) for c in range(len(chunks))])
        if rank == 0:
            for c in range(len(chunks)):
                assert torch.equal(o_full_parts[c][0], o_parts[c][0]), "copy-engine gather: rank 0's shard differs"
                for r in range(1, world):
                    got = float(o_full_parts[c][r].double().sum())
                    assert abs(got - sums[r][c]) <= 1e-9 * max(1.0, abs(sums[r][c])), \
                        f"copy-engine gather: chunk {c} of rank {r} differs ({got} vs {sums[r][c]})"
        window.close()

    kern_ms = [e[0].elapsed_time(e[1]) for e in evs]
    prefill_ms = [e[0].elapsed_time(e[2]) for e in evs]
    decode_ms = [e[2].elapsed_time(e[3]) for e in evs]
    total_ms = t_start.elapsed_time(t_stop)
    local = torch.tensor([statistics.mean(kern_ms), statistics.mean(prefill_ms),
                          statistics.mean(decode_ms), total_ms / args.steps], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(local, op=dist.ReduceOp.MAX)
    kern, pre, dec, step_ms = local.tolist()

    flops = causal_flops(B * H, T, T, 0, D)
    flops_rank = causal_flops(n, T, T, 0, D)
    value = flops / (pre / 1e3) / 1e12
    lens = np.arange(T + 1, T + S + 1)
    kv_bytes = float(2 * B * H * D * 2 * lens.sum())  # K and V bf16 reads over all decode steps
    dec_tokens = B * S / (dec / 1e3)
    peaks, peak_src = load_peaks()

    # --- e2e through the public API with pinned host buffers ----------------
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, cfg, plan, rank, world, local_rank, q, kc, vc, qd, kd, vd, ws, barrier, gather)

    result = None
    if rank == 0:
        achieved = flops_rank / (kern / 1e3) / 1e12
        peak = peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops"))
        result = {
            "metric": METRIC,
            "value": value,
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": step_ms,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": {
                "workload": (f"{args.workload}: causal prefill bf16 B={B} H={H} D={D} T={T}, then {S} decode "
                             f"steps (KV append + split-K decode), (b,h) pairs sharded over {world} GPU(s), "
                             + ("one prefill launch, outputs stay on the GPU" if world == 1 else
                                "outputs gathered to rank 0 (the prefill runs in "
                                f"{len(chunks)} query-row chunks, longest first, alternating over two streams, "
                                "each chunk's output sent to rank 0 while later chunks compute, by "
                                f"{prefill_transport}; decode gathers over NCCL, queued and waited for at the end "
                                "of the step)")),
                "global_batch": B, "seq_len": T, "parallelism": f"bxh-shard{world}",
                "l2": "inputs larger than L2 (Q/K/V/cache >= 8 GB per step)",
            },
            "prefill": {"tflops": value, "frac_of_measured_bf16_sustained": value / world / peak,
                        "frac_of_nominal_2250": value / world / 2250.0, "ms": pre,
                        "kernel_ms": kern, "gather_ms": pre - kern},
            "decode": {"tokens_per_s": dec_tokens, "hbm_gbs": kv_bytes / (dec / 1e3) / 1e9,
                       "hbm_gbs_per_gpu": kv_bytes / world / (dec / 1e3) / 1e9,
                       "frac_of_measured_hbm": kv_bytes / world / (dec / 1e3) / 1e9 / peaks["hbm_gbs"],
                       "ms_per_token_step": dec / S},
            "roofline": {"bound": "tensor", "kernel": "tc_fwd_pair_kernel<128,bf16>", "achieved": achieved,
                         "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                         "peak_source": f"{peak_src} bf16_tflops_sustained",
                         "traffic": profiled_traffic("c5", n) if T == 32768 else None,
                         "algorithmic": f"4*D*causal_pairs = {flops_rank:.4g} FLOP per launch on rank 0; "
                                        f"bytes Q+K+V read, O written = {4 * n * T * D * 2:.4g}"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
        }
        if e2e is not None:
            result["e2e"] = e2e
        result["parity"] = parity_c5(q, kc, vc, prefill_rows, qd, od, T, S, D)
        if world == 1 and not args.no_cpu_baseline:
            result["cpu_baseline"] = cpu_baseline(cfg, args.cpu_seconds)
    return result


def run_e2e(args, cfg, plan, rank, world, local_rank, q, kc, vc, qd, kd, vd, ws, barrier, gather):
    """The same step through the public API with inputs in pinned host memory."""
    import torch

    from tensorsmith_b200 import engine

    B, H, D, T, S = cfg["batch"], cfg["heads"], cfg["head_dim"], cfg["prefill"], cfg["decode_steps"]
    dev = q.device
    n = plan.size
    try:
        hq = torch.empty_like(q, device="cpu").pin_memory()
        hk = torch.empty(1, n, T, D, dtype=q.dtype).pin_memory()
        hv = torch.empty_like(hk).pin_memory()
        ho = torch.empty((world if rank == 0 else 1) * n * T * D, dtype=q.dtype).pin_memory()
        hqd = torch.empty_like(qd, device="cpu").pin_memory()
        hkd = torch.empty_like(kd, device="cpu").pin_memory()
        hvd = torch.empty_like(vd, device="cpu").pin_memory()
        hod = torch.empty((S, world if rank == 0 else 1, n, 1, D), dtype=q.dtype).pin_memory()
    except RuntimeError as error:
        return {"value": None, "unit": "TFLOP/s", "note": f"pinned host allocation failed: {error}"}
    hq.copy_(q.cpu())
    hk.copy_(kc[:, :, :T].cpu())
    hv.copy_(vc[:, :, :T].cpu())
    hqd.copy_(qd.cpu())
    hkd.copy_(kd.cpu())
    hvd.copy_(vd.cpu())
    dq = torch.empty_like(q)
    do = torch.empty_like(q)
    o_full = torch.empty(world, n, T, D, dtype=q.dtype, device=dev) if rank == 0 and world > 1 else None
    # Decode inputs in two sets, by step parity, so a step's copy-in never
    # overwrites what the previous step's last chunks still read.
    dqd_sets = [torch.empty_like(qd) for _ in range(2)]
    dkd_sets = [torch.empty_like(kd) for _ in range(2)]
    dvd_sets = [torch.empty_like(vd) for _ in range(2)]
    dod = torch.empty_like(qd)
    od_full = torch.empty(S, world, n, 1, D, dtype=q.dtype, device=dev) if rank == 0 and world > 1 else None

    # (b,h) pairs are independent through prefill and decode, so the step runs chunk by chunk of
    # pairs: chunk c's inputs land on a copy stream while earlier chunks compute, then chunk c's
    # prefill and its S decode steps run, and its prefill output goes back to the host on a
    # second copy stream while later chunks compute.  Consecutive steps overlap the same way: a
    # step's chunk c is copied in as soon as the previous step finished with chunk c (its prefill
    # output copied out, its decode steps done), so the copy-in of one step runs under the compute
    # of the previous one and the PCIe transfers, not the pipeline fill, bound the step.  The
    # decode inputs (small) land first, in the set of the step's parity; the decode outputs go
    # back at the end.  With N > 1 every rank's outputs are gathered to rank 0 after the last
    # chunk and copied back from there.  Every step's copies are inside the timed region.
    n_chunks = max(1, min(8, n))
    bounds = [round(i * n / n_chunks) for i in range(n_chunks + 1)]
    compute = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    od_all = torch.empty((world * S,) + tuple(qd.shape[1:]), dtype=q.dtype, device=dev) if rank == 0 and world > 1 else None
    ho_v = ho.view(1, n, T, D) if world == 1 else None
    chunk_free = [None] * n_chunks  # event: the previous step is done with chunk c
    parity = [0]

    def step():
        par = parity[0]
        parity[0] ^= 1
        dqd, dkd, dvd = dqd_sets[par], dkd_sets[par], dvd_sets[par]
        landed = []
        with torch.cuda.stream(s_in):
            dqd.copy_(hqd, non_blocking=True)
            dkd.copy_(hkd, non_blocking=True)
            dvd.copy_(hvd, non_blocking=True)
            for c in range(n_chunks):
                c0, c1 = bounds[c], bounds[c + 1]
                if chunk_free[c] is not None:
                    s_in.wait_event(chunk_free[c])
                dq[:, c0:c1].copy_(hq[:, c0:c1], non_blocking=True)
                kc[:, c0:c1, :T].copy_(hk[:, c0:c1], non_blocking=True)
                vc[:, c0:c1, :T].copy_(hv[:, c0:c1], non_blocking=True)
                landed.append(s_in.record_event())
        for c in range(n_chunks):
            c0, c1 = bounds[c], bounds[c + 1]
            # landed[c] follows chunk_free[c] on the copy-in stream, so the previous
            # step's copy-out of do[chunk c] has completed too.
            compute.wait_event(landed[c])
            engine.forward(dq[:, c0:c1], kc[:, c0:c1, :T], vc[:, c0:c1, :T], is_causal=True, need_lse=False,
                           out=do[:, c0:c1])
            if ho_v is not None:
                s_out.wait_event(compute.record_event())
                with torch.cuda.stream(s_out):
                    ho_v[:, c0:c1].copy_(do[:, c0:c1], non_blocking=True)
            for s in range(S):
                engine.kv_append(dkd[s][:, c0:c1], dvd[s][:, c0:c1], kc[:, c0:c1], vc[:, c0:c1], position=T + s)
                engine.decode(dqd[s][:, c0:c1], kc[:, c0:c1, : T + s + 1], vc[:, c0:c1, : T + s + 1], is_causal=True,
                              causal_offset=T + s, out=dod[s][:, c0:c1], workspace=ws)
            # Chunk c is free for the next step once its decode steps ran and its
            # prefill output left (the copy-out stream is in order).
            s_out.wait_event(compute.record_event())
            chunk_free[c] = s_out.record_event()
        if world > 1:
            gather(do, o_full)
            gather(dod, od_all)
        if rank == 0:
            s_out.wait_event(compute.record_event())
            with torch.cuda.stream(s_out):
                if world > 1:
                    ho.view(-1).copy_(o_full.view(-1), non_blocking=True)
                hod.view(-1).copy_((od_all if od_all is not None else dod).view(-1), non_blocking=True)
        compute.wait_event(s_out.record_event())

    steps = max(1, args.steps)
    step()
    barrier()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    evs[0].record()
    for i in range(steps):
        step()
        evs[i + 1].record()
    barrier()
    import torch.distributed as dist

    per_step = [evs[i].elapsed_time(evs[i + 1]) for i in range(steps)]
    stats = torch.tensor([evs[0].elapsed_time(evs[-1]) / steps, min(per_step), max(per_step)], device=dev,
                         dtype=torch.float64)
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    ms, ms_min, ms_max = stats.tolist()
    flops = causal_flops(B * H, T, T, 0, D)
    esz = q.element_size()
    h2d = (3 * n * T * D + 3 * S * n * D) * esz
    d2h = (world * n * T * D + S * world * n * D) * esz if rank == 0 else 0
    return {"value": flops / (ms / 1e3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms,
            "ms_per_step_min": ms_min, "ms_per_step_max": ms_max,
            "value_min": flops / (ms_max / 1e3) / 1e12, "value_max": flops / (ms_min / 1e3) / 1e12,
            "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h, "steps": steps,
            "path": "tensorsmith_b200.engine (C ABI) with pinned host inputs/outputs; the step runs in "
                    f"{n_chunks} chunks of (b,h) pairs: a chunk's inputs are copied in on a copy stream while "
                    "earlier chunks (of this step or, for a step's first chunks, of the previous step) compute, "
                    "and its prefill output is copied back while later chunks run"}


def _timed(args, step, n_events):
    """Warm up, then time ``args.steps`` calls of ``step(events)`` with CUDA events."""
    import torch

    from tensorsmith_b200 import engine

    for _ in range(args.warmup):
        step([torch.cuda.Event(enable_timing=True) for _ in range(n_events)])
    torch.cuda.synchronize()
    engine.check_device_status()
    sampler = ClockSampler(torch.cuda.current_device(), args.clock_log)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(n_events)] for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for ev in evs:
        step(ev)
    t1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    engine.check_device_status()
    return evs, t0.elapsed_time(t1) / args.steps, clocks


def run_c3(args):
    """Causal prefill bf16 forward + backward: B=8 H=16 T=4096 D=128 (Q/K/V scaled
    by 1/sqrt(D)), or the C5 prefill shape on 8 (b,h) pairs (``c5slice``, unscaled N(0,1) inputs)."""
    import numpy as np
    import torch

    from tensorsmith_b200 import engine

    cfg = WORKLOADS[args.workload]
    B, H, T, D = cfg["batch"], cfg["heads"], cfg["prefill"], cfg["head_dim"]
    in_scale = D ** -0.5 if cfg.get("scale_inputs") else 1.0
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(2)
    q, k, v = ((torch.randn(B, H, T, D, generator=gen, device=dev) * in_scale).to(torch.bfloat16) for _ in range(3))
    do = torch.randn(B, H, T, D, generator=gen, device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    lse = torch.empty(B, H, T, dtype=torch.float32, device=dev)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)

    if args.dropout > 0 and T > 8192:
        raise SystemExit("--dropout: the parity check holds the slice's mask in full, so T <= 8192 (c3)")
    drop = (args.dropout, 1234, 0) if args.dropout > 0 else None

    def step(ev):
        ev[0].record()
        engine.forward(q, k, v, is_causal=True, out=out, lse=lse, dropout=drop)
        ev[1].record()
        engine.backward(q, k, v, out, lse, do, is_causal=True, dq=dq, dk=dk, dv=dv, dropout=drop)
        ev[2].record()

    evs, step_ms, clocks = _timed(args, step, 3)
    fwd = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    bwd = statistics.mean(e[1].elapsed_time(e[2]) for e in evs)
    pairs_flops = causal_flops(B * H, T, T, 0, D) / 4.0  # D * P
    peaks, src = load_peaks()
    value = 14.0 * pairs_flops / ((fwd + bwd) / 1e3) / 1e12
    bwd_tf = 10.0 * pairs_flops / (bwd / 1e3) / 1e12
    fwd_tf = 4.0 * pairs_flops / (fwd / 1e3) / 1e12
    # parity of the last timed step, fp64 on the host: one (b,h) slice in full (forward and
    # gradients), or at T = 32768 the forward on 256 sampled rows of it
    bs, hs = B - 1, H - 1
    if T <= 8192:
        keep = None
        if drop is not None:  # the kernels' own mask, materialised for this slice only
            keep = engine.dropout_mask(B, H, T, T, drop, dev)[bs, hs].cpu()
        ro, rl, rdq, rdk, rdv = ref_slice_backward(q[bs, hs].cpu(), k[bs, hs].cpu(), v[bs, hs].cpu(),
                                                   do[bs, hs].cpu(), D ** -0.5, keep, args.dropout)
        errs = {"out": max_abs(out[bs, hs], ro), "lse": max_abs(lse[bs, hs], rl), "dq": max_abs(dq[bs, hs], rdq),
                "dk": max_abs(dk[bs, hs], rdk), "dv": max_abs(dv[bs, hs], rdv)}
        peaks_ref = {"dq": float(rdq.abs().max()), "dk": float(rdk.abs().max()), "dv": float(rdv.abs().max())}
        rows_note = f"(b,h) = ({bs},{hs}) in full"
    else:
        rows = torch.cat([torch.arange(T - 128, T), torch.randperm(T - 128, generator=torch.Generator().manual_seed(7))[:128].sort().values])
        ro, rl = ref_rows(q[bs, hs].cpu()[rows], k[bs, hs].cpu(), v[bs, hs].cpu(), rows + 1, D ** -0.5)
        errs = {"out": max_abs(out[bs, hs].cpu()[rows], ro), "lse": max_abs(lse[bs, hs].cpu()[rows], rl)}
        peaks_ref = {}
        rows_note = f"(b,h) = ({bs},{hs}): forward on the last 128 + 128 random rows"
    parity = {"max_abs": errs, "max_abs_ref_grad": peaks_ref, "tolerance_max_abs": 2e-2,
              "pass": max(errs["out"], errs["lse"]) <= 2e-2
              and all(errs[g] <= 2e-2 * max(1.0, peaks_ref[g]) for g in peaks_ref),
              "rows": rows_note + "; fp64 reference on the host; gradients held to 2e-2 * max(1, max|ref|)"}
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"{args.workload}: causal attention bf16 B={B} H={H} T={T} D={D}, forward + "
                               "backward, Q/K/V ~ N(0,1)" + ("/sqrt(128)" if in_scale != 1.0 else "")
                               + ", dO ~ N(0,1)"
                               + (f", attention dropout p={args.dropout} (in-kernel Philox mask)" if drop else ""),
                   "l2": f"inputs larger than L2 ({5 * B * H * T * D * 2 / 1e9:.2f} GB per step)"},
        "parity": parity,
        "forward": {"tflops": fwd_tf, "ms": fwd, "frac_of_measured_bf16": fwd_tf / peaks["bf16_tflops"]},
        "backward": {"tflops": bwd_tf, "ms": bwd, "frac_of_measured_bf16": bwd_tf / peaks["bf16_tflops"],
                     "launches": "row-statistics preprocess + dQ accumulator memset + tc_bwd_kernel + dQ convert"},
        "roofline": {"bound": "tensor", "kernel": "backward call (tc_bwd_kernel dominant)", "achieved": bwd_tf,
                     "peak": peaks["bf16_tflops"], "unit": "TFLOP/s", "frac": bwd_tf / peaks["bf16_tflops"],
                     "peak_source": f"{src} bf16_tflops (burst; the call runs ~ms)",
                     "traffic": profiled_traffic("c3", 1) if args.workload == "c3" else None,
                     "algorithmic": f"10*D*causal_pairs = {10 * pairs_flops:.4g} FLOP per backward call"},
        "gpu_launches": 4 * args.steps,  # tc_fwd_pair_kernel, bwd_stats_kernel, tc_bwd_kernel, dq_convert_kernel
        "clocks": clocks,
    }
    if not args.no_cpu_baseline and args.workload == "c3":
        line["cpu_baseline"] = cpu_c3_baseline(cfg, args.cpu_seconds)
    return line


def run_c2(args):
    """decoder-only LM (4 layers, d_model 256, 4 heads of 64, FFN 1024, vocab 8192)
    forward + backward under fp16 autocast with fp32 parameters, B=16, T=256, synthetic tokens.
    The attention path (RoPE, attention forward and backward) runs on the engine; projections, norms,
    the MLP and the loss are torch ops.  ``value`` is training tokens/s of the whole step; the
    ``attention`` object times the engine's attention forward + backward at the step's shapes."""
    import numpy as np
    import torch

    from tensorsmith_b200 import engine, nn

    cfg = WORKLOADS["c2"]
    B, T, V, E, H, L = cfg["batch"], cfg["seq"], cfg["vocab"], cfg["dim"], cfg["heads"], cfg["layers"]
    D = E // H
    np.random.seed(11)
    model = nn.TransformerLM(nn.TransformerConfig(V, dim=E, num_heads=H, num_layers=L, hidden_dim=cfg["hidden"],
                                                  max_seq_len=T), device="cuda").train()
    params = model.parameters()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(12)
    tokens = torch.randint(0, V, (B, T + 1), generator=gen, device="cuda")

    def step(ev):
        ev[0].record()
        for prm in params:
            prm.grad = None
        with torch.autocast("cuda", dtype=torch.float16):
            loss = model.loss(tokens[:, :-1], tokens[:, 1:])
        loss.backward()
        ev[1].record()

    evs, step_ms, clocks = _timed(args, step, 2)
    ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    # the engine's attention alone at the step's shapes (fp16 q/k/v as autocast hands them over)
    q, k, v, g = (torch.randn(B, H, T, D, generator=gen, device="cuda").half() for _ in range(4))
    out, lse = engine.forward(q, k, v, is_causal=True)

    def attn(ev):
        ev[0].record()
        for _ in range(L):
            o, l = engine.forward(q, k, v, is_causal=True, out=out, lse=lse)
        ev[1].record()
        for _ in range(L):
            engine.backward(q, k, v, out, lse, g, is_causal=True)
        ev[2].record()

    aevs, _, _ = _timed(args, attn, 3)
    a_fwd = statistics.mean(e[0].elapsed_time(e[1]) for e in aevs)
    a_bwd = statistics.mean(e[1].elapsed_time(e[2]) for e in aevs)
    dp = causal_flops(B * H, T, T, 0, D) / 4.0 * L  # D * causal pairs over the layers
    # parity of one attention call at this shape (sampled (b,h) slice in full, fp64 on the host)
    dq, dk, dv = engine.backward(q, k, v, out, lse, g, is_causal=True)
    ro, rl, rdq, rdk, rdv = ref_slice_backward(q[-1, -1].cpu(), k[-1, -1].cpu(), v[-1, -1].cpu(), g[-1, -1].cpu(),
                                               D ** -0.5)
    errs = {"out": max_abs(out[-1, -1], ro), "dq": max_abs(dq[-1, -1], rdq), "dk": max_abs(dk[-1, -1], rdk),
            "dv": max_abs(dv[-1, -1], rdv)}
    peaks, src = load_peaks()
    line = {
        "metric": METRIC, "value": B * T / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": f"c2: decoder LM {L} layers, d_model {E}, {H} heads x {D}, FFN {cfg['hidden']}, "
                               f"vocab {V}, B={B} T={T}, fp16 autocast with fp32 parameters, forward + loss + "
                               "backward (tokens uniform from a seed, weights random-init)",
                   "l2": "activations fit L2; the step is launch- and GEMM-bound at this size"},
        "attention": {"fwd_ms": a_fwd, "bwd_ms": a_bwd, "fwd_tflops": 4 * dp / (a_fwd / 1e3) / 1e12,
                      "bwd_tflops": 10 * dp / (a_bwd / 1e3) / 1e12,
                      "share_of_step": (a_fwd + a_bwd) / ms,
                      "kernels": "tcgen05 forward / backward at D=64 (fp16)"},
        "parity": {"max_abs": errs, "tolerance_max_abs": 2e-2,
                   "pass": errs["out"] <= 2e-2 and all(errs[x] <= 2e-2 * max(1.0, float(r.abs().max()))
                                                       for x, r in (("dq", rdq), ("dk", rdk), ("dv", rdv))),
                   "rows": "one attention call at the step's shape, (b,h) = last slice in full"},
        "roofline": {"bound": "tensor", "kernel": "attention forward + backward at the C2 shape",
                     "achieved": 14 * dp / ((a_fwd + a_bwd) / 1e3) / 1e12, "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": 14 * dp / ((a_fwd + a_bwd) / 1e3) / 1e12 / peaks["bf16_tflops"],
                     "peak_source": f"{src} bf16_tflops (dense fp16 = bf16 rate)", "traffic": None,
                     "algorithmic": f"14*D*causal_pairs over {L} layers = {14 * dp:.4g} FLOP per step"},
        "gpu_launches": None,
        "clocks": clocks,
    }
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_c2_attention_baseline(B, H, T, D, L, args.cpu_seconds)
    return line


def cpu_c2_attention_baseline(B, H, T, D, L, budget_s):
    """The oracle's attention forward + backward (NumPy, fp32 compute of fp16 inputs) at the C2 shape on
    one (b,h) slice, scaled to the step's B*H slices and L layers."""
    import numpy as np

    import oracle

    rng = np.random.default_rng(13)
    q, k, v, g = (rng.standard_normal((1, 1, T, D)).astype(np.float16).astype(np.float32) for _ in range(4))
    times, start = [], time.perf_counter()
    while not times or (time.perf_counter() - start < budget_s and len(times) < 50):
        t0 = time.perf_counter()
        o, l = oracle.attention_forward(q, k, v, is_causal=True, algorithm="dense")
        oracle.attention_backward(q, k, v, o, l, g, is_causal=True)
        times.append(time.perf_counter() - t0)
    per = statistics.median(times) * B * H * L
    return {"value": B * T / per, "unit": "tokens/s (attention only)", "cores": cpu_cores(), "kind": "port",
            "sample": f"oracle fwd+bwd of one (b,h) slice T={T} D={D}, median of {len(times)} reps, scaled x{B * H * L}"}


def run_c1(args):
    """Causal attention forward + backward in fp32, B=2 H=4 T=256 D=64, Q/K/V/dO ~ N(0,1) from seed 0
    (the case tensorsmith runs on its NumPy CPU backend today): the exact fp32
    CUDA-core kernels, checked in full against fp64."""
    import torch

    from tensorsmith_b200 import engine

    cfg = WORKLOADS[args.workload]
    B, H, T, D = cfg["batch"], cfg["heads"], cfg["prefill"], cfg["head_dim"]
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    q, k, v, do = (torch.randn(B, H, T, D, generator=gen, device=dev) for _ in range(4))
    out = torch.empty_like(q)
    lse = torch.empty(B, H, T, dtype=torch.float32, device=dev)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    path = engine.fwd_path(q, k, v, is_causal=True)

    def step(ev):
        ev[0].record()
        engine.forward(q, k, v, is_causal=True, out=out, lse=lse)
        ev[1].record()
        engine.backward(q, k, v, out, lse, do, is_causal=True, dq=dq, dk=dk, dv=dv)
        ev[2].record()

    evs, eager_ms, clocks = _timed(args, step, 3)
    fwd = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    bwd = statistics.mean(e[1].elapsed_time(e[2]) for e in evs)
    pairs_flops = causal_flops(B * H, T, T, 0, D) / 4.0  # D * P
    # The step is also captured once in a CUDA graph and replayed (the same kernels
    # and buffers without the host in the loop); `value` is the replayed step.  At
    # this size the replay takes as long as the eager calls: the kernels bound it.
    graph_note = "the forward and backward calls captured once in a CUDA graph, replayed per step"
    try:
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(3):
                step([torch.cuda.Event(enable_timing=True) for _ in range(3)])
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            engine.forward(q, k, v, is_causal=True, out=out, lse=lse)
            engine.backward(q, k, v, out, lse, do, is_causal=True, dq=dq, dk=dk, dv=dv)
        for _ in range(max(3, args.warmup)):
            graph.replay()
        torch.cuda.synchronize()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        for _ in range(args.steps):
            graph.replay()
        g1.record()
        torch.cuda.synchronize()
        engine.check_device_status()
        step_ms = g0.elapsed_time(g1) / args.steps
    except Exception as error:  # capture refused: keep the eager timing
        step_ms = eager_ms
        graph_note = f"CUDA graph unavailable ({error!r}); eager calls timed"
    value = 14.0 * pairs_flops / (step_ms / 1e3) / 1e12
    # parity of the last timed step: every (b,h) slice in full against fp64 on the host
    errs = {"out": 0.0, "lse": 0.0, "dq": 0.0, "dk": 0.0, "dv": 0.0}
    peaks_ref = {"out": 0.0, "lse": 0.0, "dq": 0.0, "dk": 0.0, "dv": 0.0}
    for bb in range(B):
        for hh in range(H):
            ref = ref_slice_backward(q[bb, hh].cpu(), k[bb, hh].cpu(), v[bb, hh].cpu(), do[bb, hh].cpu(), D ** -0.5)
            for name, got, r in zip(("out", "lse", "dq", "dk", "dv"),
                                    (out[bb, hh], lse[bb, hh], dq[bb, hh], dk[bb, hh], dv[bb, hh]), ref):
                errs[name] = max(errs[name], max_abs(got, r))
                peaks_ref[name] = max(peaks_ref[name], float(r.abs().max()))
    rel = {name: errs[name] / max(1.0, peaks_ref[name]) for name in errs}
    # nominal fp32 FMA rate of the CUDA cores: 148 SMs x 128 lanes x 2 FLOP x the maximum SM clock
    fp32_peak = 148 * 128 * 2 * 1.965e9 / 1e12
    return {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"c1: causal attention fp32 B={B} H={H} T={T} D={D}, forward + backward, "
                               "Q/K/V/dO ~ N(0,1) from seed 0 (BASELINE config 0); " + graph_note,
                   "l2": "inputs fit in L2 (1 MB)"},
        "eager": {"ms_per_step": eager_ms, "tflops": 14.0 * pairs_flops / (eager_ms / 1e3) / 1e12,
                  "note": "the same calls from Python every step"},
        "parity": {"max_abs": errs, "max_rel": rel, "tolerance_rel": 1e-4, "pass": max(rel.values()) <= 1e-4,
                   "rows": "every (b,h) slice in full; fp64 reference on the host; errors relative to "
                           "max(1, max|ref|)"},
        "forward": {"tflops": 4.0 * pairs_flops / (fwd / 1e3) / 1e12, "ms": fwd, "path": path},
        "backward": {"tflops": 10.0 * pairs_flops / (bwd / 1e3) / 1e12, "ms": bwd},
        "roofline": {"bound": "fma", "kernel": "simt_fwd_kernel + simt_bwd_{delta,dq,dkdv} (exact fp32)",
                     "achieved": value, "peak": fp32_peak, "unit": "TFLOP/s", "frac": value / fp32_peak,
                     "peak_source": "nominal fp32 CUDA-core FMA rate at the maximum SM clock (no measured figure)",
                     "traffic": None,
                     "algorithmic": f"14*D*causal_pairs = {14 * pairs_flops:.4g} FLOP per step"},
        "gpu_launches": 4 * args.steps,  # simt_fwd_kernel, simt_bwd_delta, simt_bwd_dq, simt_bwd_dkdv
        "clocks": clocks,
        **({} if args.no_cpu_baseline else {"cpu_baseline": cpu_c1_baseline(cfg, args.cpu_seconds)}),
    }


def cpu_c1_baseline(cfg, budget_s):
    """The oracle (tensorsmith's NumPy algorithm) on the whole C1 problem: dense forward and VJP in fp32."""
    import numpy as np

    import oracle

    B, H, T, D = cfg["batch"], cfg["heads"], cfg["prefill"], cfg["head_dim"]
    rng = np.random.default_rng(0)
    q, k, v, g = (rng.standard_normal((B, H, T, D)).astype(np.float32) for _ in range(4))
    flops = 14.0 * causal_flops(B * H, T, T, 0, D) / 4.0
    times, start = [], time.perf_counter()
    while not times or (time.perf_counter() - start < budget_s and len(times) < 50):
        t0 = time.perf_counter()
        o, l = oracle.attention_forward(q, k, v, is_causal=True, algorithm="dense")
        oracle.attention_backward(q, k, v, o, l, g, is_causal=True)
        times.append(time.perf_counter() - t0)
    return {"value": flops / statistics.median(times) / 1e12, "unit": "TFLOP/s", "cores": cpu_cores(),
            "kind": "port", "sample": f"the whole C1 problem (B={B} H={H} T={T} D={D}), oracle dense forward + "
                                      f"VJP in NumPy fp32, median of {len(times)} reps"}


def cpu_c3_baseline(cfg, budget_s):
    """Oracle streaming forward + blockwise backward on one (b,h) slice, rows sub-sampled."""
    import numpy as np

    import oracle

    T, D = cfg["prefill"], cfg["head_dim"]
    rows = 512
    rng = np.random.default_rng(3)
    q = (rng.standard_normal((1, 1, rows, D)) / D ** 0.5).astype(np.float32)
    k = (rng.standard_normal((1, 1, T, D)) / D ** 0.5).astype(np.float32)
    v = (rng.standard_normal((1, 1, T, D)) / D ** 0.5).astype(np.float32)
    g = rng.standard_normal((1, 1, rows, D)).astype(np.float32)
    flops = 14.0 * causal_flops(1, rows, T, T - rows, D) / 4.0
    times, start = [], time.perf_counter()
    while not times or (time.perf_counter() - start < budget_s and len(times) < 20):
        t0 = time.perf_counter()
        o, l = oracle.attention_forward(q, k, v, is_causal=True, causal_offset=T - rows, algorithm="streaming",
                                        block_size=1024)
        oracle.attention_backward(q, k, v, o, l, g, is_causal=True, causal_offset=T - rows, block_size=1024)
        times.append(time.perf_counter() - t0)
    return {"value": flops / statistics.median(times) / 1e12, "unit": "TFLOP/s", "cores": cpu_cores(),
            "kind": "port", "sample": f"oracle fwd+bwd (NumPy fp32, block 1024) of the last {rows} query rows of "
                                      f"one (b,h) slice vs T={T} keys, median of {len(times)} reps"}


def run_c4(args, quantized=False):
    """fp16 KV-cache decode, B=64 H=32 D=128, ragged lengths, 256 steps with append;
    ``quantized``: the same steps over an int8 cache (quantising append + fused-dequant decode)."""
    import numpy as np
    import torch

    from tensorsmith_b200 import engine

    cfg = WORKLOADS[args.workload]
    B, H, D, S = cfg["batch"], cfg["heads"], cfg["head_dim"], cfg["decode_steps"]
    Hkv = cfg.get("kv_heads", H)
    cap = cfg["max_len"] + S
    dev = torch.device("cuda", 0)
    lens0 = np.random.default_rng(4).integers(cfg["min_len"], cfg["max_len"] + 1, B)
    gen = torch.Generator(device=dev)
    gen.manual_seed(4)
    kc = torch.randn(B, Hkv, cap, D, generator=gen, device=dev).to(torch.float16)
    vc = torch.randn(B, Hkv, cap, D, generator=gen, device=dev).to(torch.float16)
    qn = torch.randn(S, B, H, 1, D, generator=gen, device=dev).to(torch.float16)
    kn, vn = (torch.randn(S, B, Hkv, 1, D, generator=gen, device=dev).to(torch.float16) for _ in range(2))
    out = torch.empty(S, B, H, 1, D, dtype=torch.float16, device=dev)
    start_lens = torch.tensor(lens0, dtype=torch.int32, device=dev)
    lens = [torch.empty_like(start_lens), torch.empty_like(start_lens)]
    if quantized:
        # Quantise the synthetic fp16 prefix once (the same kernel a prefill append runs).
        k8 = torch.empty(B, Hkv, cap, D, dtype=torch.int8, device=dev)
        v8 = torch.empty_like(k8)
        ks = torch.ones(B, Hkv, cap, dtype=torch.float32, device=dev)
        vs = torch.ones_like(ks)
        engine.kv_append_int8(kc, vc, k8, v8, ks, vs, compute_dtype=torch.float16, position=0)
        del kc, vc
        kc, vc = k8, v8
        need = engine.decode_int8_workspace_bytes(qn[0], kc, vc, is_causal=True, kv_lens=start_lens)
    else:
        need = engine.decode_workspace_bytes(qn[0], kc, vc, is_causal=True, kv_lens=start_lens)
    ws = torch.empty(max(16, need), dtype=torch.uint8, device=dev)
    splits = ws.numel() > 16

    def step(ev):
        lens[0].copy_(start_lens)
        ev[0].record()
        for s in range(S):
            cur, nxt = lens[s & 1], lens[(s + 1) & 1]
            if quantized:
                engine.kv_append_int8(kn[s], vn[s], kc, vc, ks, vs, compute_dtype=torch.float16, positions=cur,
                                      positions_out=nxt)
                engine.decode_int8(qn[s], kc, vc, ks, vs, is_causal=True, kv_lens=nxt, out=out[s], workspace=ws)
            else:
                engine.kv_append(kn[s], vn[s], kc, vc, positions=cur, positions_out=nxt)
                engine.decode(qn[s], kc, vc, is_causal=True, kv_lens=nxt, out=out[s], workspace=ws)
        ev[1].record()

    evs, step_ms, clocks = _timed(args, step, 2)
    dec = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    # parity of the last decode step of the last timed step (4 sampled (b, h) rows, fp64 on the host)
    prng = np.random.default_rng(5)
    sample = [(B - 1, H - 1)] + [(int(prng.integers(B)), int(prng.integers(H))) for _ in range(3)]
    err = 0.0
    for b, h in sample:
        hk, n = h // (H // Hkv), int(lens0[b]) + S
        if quantized:
            kh = kc[b, hk, :n].cpu().double() * ks[b, hk, :n].cpu().double()[:, None]
            vh = vc[b, hk, :n].cpu().double() * vs[b, hk, :n].cpu().double()[:, None]
        else:
            kh, vh = kc[b, hk, :n].cpu(), vc[b, hk, :n].cpu()
        ref, _ = ref_rows(qn[S - 1, b, h].cpu(), kh, vh, [n], D ** -0.5)
        err = max(err, max_abs(out[S - 1, b, h], ref))
    parity = {"max_abs_out": err, "tolerance_max_abs": 2e-2, "pass": err <= 2e-2,
              "rows": f"last decode step, (b,h) = {sample}, dequantised cache" if quantized
              else f"last decode step, (b,h) = {sample}"}
    row_bytes = D + 4 if quantized else 2 * D  # int8 row + fp32 scale, or fp16 row
    kv_bytes = float(sum(2 * Hkv * row_bytes * (lens0 + s + 1).sum() for s in range(S)))
    peaks, src = load_peaks()
    gbs = kv_bytes / (dec / 1e3) / 1e9
    tokens = B * S / (dec / 1e3)
    line = {
        "metric": METRIC, "value": tokens, "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": (f"{args.workload}: fp16 decode over an int8 KV cache (fp32 scale per token/head) "
                                if quantized else f"{args.workload}: fp16 KV-cache decode ")
                               + f"B={B} H={H} KV heads={Hkv} D={D}, lengths U[{cfg['min_len']},"
                               f"{cfg['max_len']}] per row, {S} decode steps each appending one token",
                   "l2": f"cache {2 * B * Hkv * cap * (D + 4) / 1e9 if quantized else 4 * B * Hkv * cap * D / 1e9:.1f} GB, "
                         "larger than L2"},
        "parity": parity,
        "decode": {"tokens_per_s": tokens, "hbm_gbs": gbs, "ms_per_token_step": dec / S,
                   "frac_of_measured_hbm": gbs / peaks["hbm_gbs"], "frac_of_nominal_8000": gbs / 8000.0},
        "roofline": {"bound": "hbm",
                     "kernel": ("decode step (kv_append_int8 + decode_int8 + combine)" if quantized
                                else "decode step (kv_append + tc_fwd_kernel over query-head rows)" if Hkv != H
                                else "decode step (kv_append + decode_split + combine)"),
                     "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": gbs / peaks["hbm_gbs"],
                     "peak_source": f"{src} hbm_gbs",
                     "traffic": (None if quantized else
                                 profiled_traffic("c4gqa" if Hkv != H else "c4", kv_bytes / S)),
                     "algorithmic": ("sum_b 2*Hkv*L_b*(D+4) bytes (int8 K+V rows and fp32 scales read) per step"
                                     if quantized else "sum_b 2*Hkv*L_b*D*2 bytes (K+V fp16 read once per KV head) per step")},
        "gpu_launches": S * (2 + (1 if splits else 0)) * args.steps,
        "clocks": clocks,
    }
    if not args.no_cpu_baseline:
        cfg5 = dict(prefill=cfg["max_len"], head_dim=D)
        per_pair, bpp = cpu_decode_sample(cfg5, 2)
        mean_len = float(lens0.mean())
        per_pair *= mean_len / cfg["max_len"]
        # The reference broadcasts each KV head to its query heads (nn/attention.py:93-100),
        # so its decode cost scales with the query heads.
        line["cpu_baseline"] = {"value": B / (per_pair * B * H), "unit": "tokens/s", "cores": cpu_cores(),
                                "kind": "port", "sample": "oracle dense decode of 2 (b,h) pairs vs an fp16 cache "
                                f"of {cfg['max_len']} keys, scaled to the mean length {mean_len:.0f}"}
    return line


def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if world != args.gpus and "RANK" in os.environ:
        args.gpus = world
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    import torch
    import torch.distributed as dist

    if world > 1:
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        from tensorsmith_b200 import _lib

        build = {"lib": str(_lib.LIB_PATH.relative_to(ROOT)), "source_digest": _lib.library_digest()}
        if args.workload in ("c1", "c2", "c3", "c5slice", "c4", "c4q", "c4q_small", "c4gqa"):
            if world > 1:
                raise SystemExit("the c1 / c2 / c3 / c4 parity configs run on one GPU; c5 is the multi-GPU workload")
            result = (run_c1(args) if args.workload == "c1" else run_c2(args) if args.workload == "c2"
                      else run_c3(args) if args.workload in ("c3", "c5slice")
                      else run_c4(args, quantized=args.workload.startswith("c4q")))
        else:
            result = run_engine(args, rank, world, local_rank)
        if rank == 0 and result is not None:
            result["build"] = build
            print(json.dumps(result), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
