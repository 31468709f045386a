"""Benchmark of the PASA attention forward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config wan14b-720p] [--impl reference]

A step is one PASA forward (block statistics -> selection -> attention) over
the configured workload.  With N > 1 (launched by torchrun, one rank per
GPU) the heads are split into contiguous ranges, each rank runs its own heads
with no collective on the data path, and the whole-job throughput is the
total work over the slowest rank's time (strong scaling: the call's total work
is fixed).  Inputs are seeded synthetic tensors generated on the device; at
the Wan2.1-14B shape q, k, v are 2.3 GB, far larger than the 126 MB L2, so
no explicit flush is needed between steps.

Printed (rank 0, one JSON line): the metric of BASELINE.json (effective
TFLOP/s on the exact-block FLOPs, plus ms per call), the end-to-end number
through the public API with host buffers, the roofline of the attention
kernel, the CPU baseline (the numpy restatement of the reference on the host
cores, a bounded sample) and the SM clocks sampled during the timed region.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "PASA attn effective TFLOP/s (exact-block FLOPs) at Wan2.1-14B 720p shape"
UNIT = "TFLOP/s"
PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

# DRAM bytes (read + write) per launch of the attention kernel from one ncu
# capture of 4 of the 40 heads (237.4 MB read + 61.3 MB written), scaled by
# 10 (work and bytes are per head).  Keyed by (workload, kernel).
ATTN_TRAFFIC_BYTES = {("wan14b-720p", "tcgen05"): 2.994e9}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="wan14b-720p")
    ap.add_argument("--impl", default="pasa_b200", choices=["pasa_b200", "reference"])
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end leg (profiling runs)")
    ap.add_argument("--e2e-chunk", type=int, default=1, help="heads per chunk of the end-to-end host pipeline")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--kernel", default="auto", choices=["auto", "tcgen05", "simt"])
    ap.add_argument("--heads", type=int, default=0, help="run only this many heads (small profiling cases)")
    ap.add_argument("--place", action="store_true",
                    help="time the HunyuanVideo token placement (forward on q, k, v and inverse on o) at the "
                         "hunyuan-720p shape")
    ap.add_argument("--classify", action="store_true",
                    help="time the head classification (pasa_sample_mse) at the hunyuan-720p shape")
    ap.add_argument("--dit", action="store_true",
                    help="time the full Wan2.1-14B DiT denoising step (PASA in every layer, Ulysses over ranks)")
    ap.add_argument("--dit-layers", type=int, default=40, help="blocks in the DiT step (40 = the full model)")
    ap.add_argument("--dit-density", type=float, default=0.1)
    ap.add_argument("--dit-frames", type=int, default=0, help="latent frames (0 = 21, the 81-frame video)")
    ap.add_argument("--dit-exchange", default="peer", choices=["peer", "nccl"],
                    help="Ulysses exchange with N > 1: kernels storing into peer memory (fused), or NCCL all-to-all")
    ap.add_argument("--dit-torch", action="store_true",
                    help="DiT step with torch elementwise ops instead of the row kernels (comparison)")
    return ap.parse_args()


def load_peaks():
    if PEAKS_FILE.exists():
        p = json.loads(PEAKS_FILE.read_text())
        return p, "measured"
    return FALLBACK_PEAKS, "fallback"


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices):
        self.gpus = set(gpu_indices)
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = [r for r in self.rows if r[0].isdigit() and int(r[0]) in self.gpus]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows),
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


# ---------------------------------------------------------------------------
# CPU baseline and reference arm: the oracle (numpy restatement of the
# reference's PASA forward) on one full head, over all host cores
# ---------------------------------------------------------------------------
def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _shm_put(arr, keep):
    from multiprocessing import shared_memory

    import numpy as np

    arr = np.ascontiguousarray(arr)
    shm = shared_memory.SharedMemory(create=True, size=max(1, arr.nbytes))
    np.ndarray(arr.shape, arr.dtype, buffer=shm.buf)[...] = arr
    keep.append(shm)
    return (shm.name, arr.shape, arr.dtype.str)


_ATTACHED = {}


def _shm_get(desc):
    from multiprocessing import shared_memory

    import numpy as np

    name, shape, dt = desc
    if name not in _ATTACHED:
        _ATTACHED[name] = shared_memory.SharedMemory(name=name)
    return np.ndarray(shape, np.dtype(dt), buffer=_ATTACHED[name].buf)


def _shm_release():
    for shm in _ATTACHED.values():
        shm.close()
    _ATTACHED.clear()


def _ref_warm(_):
    from oracle import pasa_oracle  # noqa: F401

    return os.getpid()


def _ref_stats(task):
    """Block statistics and group means of whole groups [g0, g1) (oracle)."""
    from oracle import pasa_oracle as O

    qd, kd, vd, T, g0, g1, dt = task
    t0, t1 = g0 * 2048, min(T, g1 * 2048)
    q, k, v = (_shm_get(d)[None, t0:t1] for d in (qd, kd, vd))
    qc, kc, vc, hc, hn = O.chunk_reduce(q, k, v, 64, dt)
    hg = O.group_mean(hc, 32, dt)
    _shm_release()
    return g0, qc[0], kc[0], vc[0], hn[0], hg[0]


def _ref_select(task):
    from oracle import pasa_oracle as O

    qcd, kcd, hnd, i0, i1, scale, NS, dt = task
    qc, kc, hn = _shm_get(qcd), _shm_get(kcd), _shm_get(hnd)
    idx, _ = O.select_blocks(qc[None, i0:i1], kc[None], hn[None], scale, NS, dt)
    _shm_release()
    return i0, idx[0]


def _ref_attn(task):
    import numpy as np

    from oracle import pasa_oracle as O

    qd, kd, vd, kcd, vcd, hgd, idxd, scale, T, qb, dt = task
    arrs = [_shm_get(d)[None] for d in (qd, kd, vd, kcd, vcd, hgd, idxd)]
    o = O.attention(*arrs, scale, T, dtype=dt, qblocks=np.asarray(qb))
    _shm_release()
    return float(np.abs(o).sum())


class OracleHead:
    """One head of the PASA forward on the oracle, split over a pool of
    single-threaded worker processes (spawned, so it is safe next to CUDA):
    block statistics by group ranges, selection by query-block ranges,
    attention by query-block ranges.  Each piece computes what the whole-head
    oracle computes for its blocks."""

    def __init__(self, workers=None):
        import multiprocessing as mp

        self.workers = workers or len(os.sched_getaffinity(0))
        for var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
            os.environ[var] = "1"  # one thread per worker process
        self.pool = mp.get_context("spawn").Pool(self.workers)
        self.pool.map(_ref_warm, range(self.workers))  # worker start-up and imports stay out of the timing

    def close(self):
        self.pool.close()
        self.pool.join()

    def run(self, q, k, v, w):
        """q, k, v: one head as float32 [T, D] arrays holding the workload's
        values.  Returns (seconds, checksum)."""
        import numpy as np

        dt = "bf16" if w.dtype_name == "bf16" else "fp32"
        keep = []
        try:
            # zero rows past T up to whole blocks, so the workers' block views
            # of q, k, v need no copy (the oracle masks by T itself)
            pad = w.NT * 64 - w.T
            qd, kd, vd = (_shm_put(np.concatenate([x, np.zeros((pad, x.shape[1]), np.float32)]) if pad else x, keep)
                          for x in (q, k, v))
            t0 = time.perf_counter()
            NG = w.NG
            n = self.workers
            ranges = np.array_split(np.arange(NG), min(NG, 4 * n))
            res = self.pool.map(_ref_stats, [(qd, kd, vd, w.T, int(r[0]), int(r[-1]) + 1, dt)
                                             for r in ranges if len(r)])
            res.sort(key=lambda x: x[0])
            qc, kc, vc, hn, hg = (np.concatenate([x[i] for x in res]) for i in range(1, 6))
            qcd, kcd, vcd, hnd, hgd = (_shm_put(x, keep) for x in (qc, kc, vc, hn, hg))
            rows = np.array_split(np.arange(w.NT), min(w.NT, 4 * n))
            sel = self.pool.map(_ref_select, [(qcd, kcd, hnd, int(r[0]), int(r[-1]) + 1, w.D ** -0.5, w.NS, dt)
                                              for r in rows if len(r)])
            sel.sort(key=lambda x: x[0])
            idx = np.concatenate([x[1] for x in sel]).astype(np.int32)
            idxd = _shm_put(idx, keep)
            qbs = np.array_split(np.arange(w.NT), min(w.NT, 4 * n))
            sums = self.pool.map(_ref_attn, [(qd, kd, vd, kcd, vcd, hgd, idxd, w.D ** -0.5, w.T, r.tolist(), dt)
                                             for r in qbs if len(r)])
            return time.perf_counter() - t0, float(sum(sums))
        finally:
            for shm in keep:
                shm.close()
                shm.unlink()


def _head_arrays(w, head, seed=0):
    import torch

    from pasa_b200 import synth

    torch.set_num_threads(os.cpu_count() or 1)
    q, k, v = synth.head_qkv(w, head, "cpu", seed)
    return tuple(t.float().numpy() for t in (q, k, v))


def cpu_baseline(w, seed=0, oracle=None):
    """The oracle on head 0 of the workload (all blocks: statistics,
    selection and attention) over all host cores; extrapolated x heads."""
    own = oracle is None
    oracle = oracle or OracleHead()
    try:
        secs, _ = oracle.run(*_head_arrays(w, 0, seed), w)
    finally:
        if own:
            oracle.close()
    value = w.exact_flops(1) / secs / 1e12
    sample = (f"oracle (numpy restatement) on head 0 of {w.name}, all {w.NT} blocks: statistics, selection and "
              f"attention, {secs:.2f} s on {oracle.workers} single-threaded worker processes; the call has "
              f"{w.heads} such heads ({secs * w.heads:.0f} s extrapolated)")
    return {"value": value, "unit": UNIT, "cores": oracle.workers, "kind": "port", "sample": sample,
            "cpu_model": cpu_model(), "s_per_head": secs}


# ---------------------------------------------------------------------------
def init_dist():
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        # host buffers of this rank on its GPU's NUMA node (end-to-end copies)
        from pasa_b200 import dist as pdist

        os.environ["PASA_NUMA_NODE"] = str(pdist.pin_to_gpu_numa(local))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def max_over_ranks(x: float, world: int) -> float:
    from pasa_b200 import dist as pdist

    return pdist.max_over_ranks(x) if world > 1 else x


def barrier(world):
    from pasa_b200 import dist as pdist

    if world > 1:
        pdist.barrier()


def run_reference(args):
    """The reference arm: the reference's CPU implementation of the path (the
    oracle port; the reference's own PASA op is Python + Triton and needs a
    GPU or the Triton interpreter) on the host cores.  One step is one full
    head of the configured workload (heads in turn), so ms_per_step is the
    measured time of one head; the call has w.heads of them."""
    from pasa_b200 import synth

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    w = synth.WORKLOADS[args.config]
    oracle = OracleHead()
    secs = []
    try:
        for i in range(args.warmup + args.steps):
            s, _ = oracle.run(*_head_arrays(w, i % w.heads), w)
            if i >= args.warmup:
                secs.append(s)
    finally:
        oracle.close()
    sec = statistics.median(secs)
    value = w.exact_flops(1) / sec / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16" if w.dtype_name == "bf16" else "f32",
        "data": "synthetic (seeded, generated on the host)",
        "config": {"workload": w.name, "heads": w.heads, "seq_len": w.T, "head_dim": w.D, "density": w.density,
                   "block": 64, "group": 32, "top_k": w.NS,
                   "step": f"one full head (all {w.NT} blocks), heads taken in turn; the call is {w.heads} heads",
                   "ms_per_call_extrapolated": sec * 1e3 * w.heads},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": oracle.workers, "kind": "port",
                         "cpu_model": cpu_model(),
                         "sample": f"median of {args.steps} steps of one full head each on {oracle.workers} "
                                   f"single-threaded worker processes (oracle port of the reference)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_dit(args):
    """One denoising step of the Wan2.1-14B DiT at 720p (81 frames -> 21 x 45 x
    80 = 75600 tokens): patch embedding, 40 blocks with PASA self-attention,
    output head.  With N ranks every rank holds 75600/N tokens and the self-
    attention reshards sequence <-> heads with NCCL all-to-alls (Ulysses)."""
    import dataclasses

    import torch
    import torch.distributed as dist

    from pasa_b200 import dit, ops

    world, rank, local = init_dist()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg = dataclasses.replace(dit.WAN14B_720P, layers=args.dit_layers, density=args.dit_density)
    if args.dit_frames:
        cfg = dataclasses.replace(cfg, frames=args.dit_frames)
    if cfg.heads % world:
        raise SystemExit(f"{cfg.heads} heads do not split over {world} ranks")
    group = dist.group.WORLD if world > 1 else None
    t0, t1 = dit.local_slice(cfg, rank, world)
    stream = torch.cuda.current_stream(dev)

    # identical weights and inputs on every rank (same seeds); latents and text on the host
    blocks = [dit.init_block(cfg, 1000 + i, dev) for i in range(cfg.layers)]
    embed = dit.init_embed(cfg, 999, dev)
    g = torch.Generator().manual_seed(0)
    lat = torch.randn((1, cfg.in_channels, cfg.frames, 2 * cfg.height, 2 * cfg.width), generator=g)
    text_h = torch.randn((1, cfg.text_len, cfg.text_dim), generator=g).to(torch.bfloat16).pin_memory()
    lat_h = dit.patchify(lat)[:, t0:t1].to(torch.bfloat16).contiguous().pin_memory()
    out_h = torch.empty((1, t1 - t0, cfg.in_channels * 4), dtype=torch.bfloat16).pin_memory()
    cos, sin = dit.rope_table(cfg, dev)
    rope = (cos[t0:t1].contiguous(), sin[t0:t1].contiguous())
    timestep = torch.tensor([900], device=dev)
    lat_d, text_d = lat_h.to(dev), text_h.to(dev)

    attn_events, a2a_events = [], []

    def timed(fn, events):
        def run(*a, **kw):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            r = fn(*a, **kw)
            e1.record(stream)
            events.append((e0, e1))
            return r
        return run

    # time the Ulysses all-to-alls (resharding copies included)
    dit.seq_to_head = timed(dit.seq_to_head, a2a_events)
    dit.head_to_tokens = timed(dit.head_to_tokens, a2a_events)

    def core(q, k, v):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        o = ops.pisa_pg_attention(q, k, v, density=cfg.density, out_layout="bthd")
        e1.record(stream)
        attn_events.append((e0, e1))
        return o

    fused = not args.dit_torch
    exchange = None
    if world > 1 and fused and args.dit_exchange == "peer":
        from pasa_b200.exchange import UlyssesPeerExchange

        exchange = UlyssesPeerExchange(group, dev, cfg.heads, cfg.head_dim, t1 - t0)
        # time the two fused exchanges like the all-to-alls (kernel + its barrier)
        exchange.attention = timed(exchange.attention, attn_events)
        exchange.scatter_qkv = timed(exchange.scatter_qkv, a2a_events)

    def step(ex=exchange):
        return dit.step(lat_d, timestep, text_d, rope, embed, blocks, cfg, core, group, fused=fused, exchange=ex)

    def e2e_step():
        # the public call with host buffers: latents and text in, predicted patches out
        lat_g = lat_h.to(dev, non_blocking=True)
        text_g = text_h.to(dev, non_blocking=True)
        out = dit.step(lat_g, timestep, text_g, rope, embed, blocks, cfg, core, group, fused=fused,
                       exchange=exchange)
        out_h.copy_(out, non_blocking=True)

    with torch.no_grad():
        if exchange is not None:
            # the fused exchange moves the same values as the all-to-alls:
            # the step's output must be bit-identical to the NCCL path's
            same = torch.equal(step(), step(ex=None))
            flags = torch.tensor([0 if same else 1], device=dev)
            dist.all_reduce(flags)
            if int(flags.item()):
                raise SystemExit("peer-memory exchange differs from the NCCL all-to-all path")
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        attn_events.clear()
        a2a_events.clear()
        gpu_ids = [int(x) for x in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if x.strip().isdigit()]
        sampler = ClockSampler([gpu_ids[local] if local < len(gpu_ids) else local])
        with sampler:
            time.sleep(0.3)
            barrier(world)
            torch.cuda.synchronize()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
            for _ in range(args.steps):
                out = step()
            end.record(stream)
            torch.cuda.synchronize()
            barrier(world)
        assert torch.isfinite(out).all()
        ms_step = max_over_ranks(start.elapsed_time(end) / args.steps, world)
        attn_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in attn_events) / args.steps, world)
        a2a_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in a2a_events) / args.steps, world)
        attn_events.clear()
        e2e_ms = None
        if not args.no_e2e:
            e2e_step()
            torch.cuda.synchronize()
            barrier(world)
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            for _ in range(args.steps):
                e2e_step()
            s1.record(stream)
            torch.cuda.synchronize()
            barrier(world)
            e2e_ms = max_over_ranks(s0.elapsed_time(s1) / args.steps, world)
            assert torch.isfinite(out_h.float()).all()

    clocks = sampler.summary()
    nbytes = lambda t: t.numel() * t.element_size()
    tokens = cfg.tokens
    C, Fd, Lt = cfg.hidden, cfg.ffn, cfg.text_len
    # GEMM FLOPs of one step (all ranks): per block 4 self-attention and 2
    # cross-attention C x C projections over the video tokens, 2 over the text,
    # the FFN pair, and the cross-attention scores/values
    gemm = cfg.layers * (2 * tokens * C * C * 6 + 2 * Lt * C * C * 2 + 2 * 2 * tokens * C * Fd
                         + 4 * tokens * Lt * C)
    if rank == 0:
        line = {
            "metric": "Wan2.1-14B DiT denoising step, PASA in every layer (ms per step)",
            "value": ms_step, "unit": "ms", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_step, "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded N(0,1) latents and text embeddings, random-init weights)",
            "config": {"workload": "wan14b-720p-dit-step" + (f"-{cfg.frames}f" if args.dit_frames else ""),
                       "layers": cfg.layers, "hidden": C, "heads": cfg.heads,
                       "ffn": Fd, "tokens": tokens, "text_len": Lt, "density": cfg.density,
                       "parallelism": f"ulysses{world}" if world > 1 else "none",
                       "elementwise": "row kernels (pasa_dit_row_norm, pasa_dit_qkv_rope)" if fused else "torch ops",
                       "exchange": (None if world == 1 else
                                    "fused peer-memory scatter (qkv_rope_scatter + forward_scatter, NCCL barrier)"
                                    if exchange is not None else "NCCL all-to-all"),
                       "l2": "activations 0.77 GB per tensor > 126 MB L2; no flush"},
            "kernels_ms": {"pasa_attention_per_step": attn_ms, "attention_share": attn_ms / ms_step,
                           ("ulysses_qkv_scatter_per_step" if exchange is not None else
                            "ulysses_all_to_all_per_step"): a2a_ms if world > 1 else 0.0},
            "gemm_tflop_per_step": gemm / 1e12,
            "e2e": None if e2e_ms is None else {
                "value": e2e_ms, "unit": "ms", "h2d_bytes_per_step": (nbytes(lat_h) + nbytes(text_h)) * world,
                "d2h_bytes_per_step": nbytes(out_h) * world,
                "note": "dit.step from pinned host latents/text to pinned host output, per rank, summed over ranks"},
            "clocks": clocks,
            # per block: prep, select, attention, plus with the row kernels 3 norms
            # and 3 producers (q/k/v, cross q, cross k); one more norm per step
            "gpu_launches": ((9 * cfg.layers + 1) if fused else 3 * cfg.layers) * args.steps,
        }
        print(json.dumps(line), flush=True)
    if exchange is not None:
        exchange.close()
    if world > 1:
        dist.destroy_process_group()


def run_place(args):
    """The token placement of the HunyuanVideo processors (placement.py) at
    the hunyuan-720p shape: frame-major -> token-major on q, k and v, and the
    inverse on the attention output, for half of the 24 heads temporal.  A
    pure copy: the roofline is HBM bandwidth, 2 x the bytes moved."""
    import torch

    from pasa_b200 import ops, synth

    if args.impl == "reference":
        print(json.dumps({"impl": "reference", "unavailable": "the reference's placement kernels are Triton GPU "
                          "kernels (placement.py), which cannot run here; its CPU form is the torch reordering the "
                          "oracle restates"}), flush=True)
        return
    dev = torch.device("cuda", 0)
    w = synth.WORKLOADS["hunyuan-720p"]
    H, T, D = args.heads or w.heads, w.T, w.D
    ctx, F, S = w.text_tokens, w.frames, w.frame_tokens
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    q, k, v = (torch.randn((1, H, T, D), generator=g, device=dev).to(torch.bfloat16) for _ in range(3))
    qo, ko, vo, back = (torch.empty_like(q) for _ in range(4))
    best = (torch.arange(H, device=dev) % 2).reshape(1, H)  # every other head temporal

    def step():
        ops.hunyuan_sparse_head_placement(q, k, v, qo, ko, vo, best, ctx, F, S)
        ops.hunyuan_hidden_states_placement(vo, back, best, ctx, F, S)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    assert torch.equal(back, v), "inverse placement does not restore the input"
    stream = torch.cuda.current_stream(dev)
    sampler = ClockSampler([0])
    with sampler:
        time.sleep(0.2)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    nbytes = 4 * q.numel() * q.element_size() * 2  # 4 tensors, read + write
    peaks, kind = load_peaks()
    gbs = nbytes / (ms * 1e-3) / 1e9
    print(json.dumps({
        "metric": "HunyuanVideo token placement, GB/s moved (forward on q, k, v + inverse on o)",
        "value": gbs, "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1))",
        "config": {"workload": "hunyuan-720p placement", "heads": H, "seq_len": T, "head_dim": D,
                   "context_length": ctx, "num_frame": F, "frame_size": S, "temporal_heads": H // 2,
                   "l2": "4 x 0.73 GB tensors > 126 MB L2; no flush"},
        "roofline": {"kernel": "place_kernel", "bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": gbs / peaks["hbm_gbs"], "traffic": None,
                     "peak_source": f"{kind} hbm_gbs"},
        "clocks": sampler.summary(), "gpu_launches": 4 * args.steps,
    }), flush=True)


def run_classify(args):
    """Head classification (pasa_sample_mse) at the hunyuan-720p shape: 32
    sampled rows against all 119056 keys of each of the 24 heads, three
    masks.  HBM-bound: K is read twice and V once per head."""
    import torch

    from pasa_b200 import classify, synth

    if args.impl == "reference":
        print(json.dumps({"impl": "reference", "unavailable": "the reference builds its emulated masks as dense "
                          "T x T tensors with a Python double loop (14 GB at this shape) before sample_mse"}),
              flush=True)
        return
    dev = torch.device("cuda", 0)
    w = synth.WORKLOADS["hunyuan-720p"]
    H, T, D = args.heads or w.heads, w.T, w.D
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    q, k, v = (torch.randn((1, H, T, D), generator=g, device=dev).to(torch.bfloat16) for _ in range(3))
    rows = torch.randint(0, 10000, (32,), generator=torch.Generator().manual_seed(1))

    def step():
        return classify.sample_mse(q, k, v, model="hunyuan", context_length=w.text_tokens, num_frame=w.frames,
                                   frame_size=w.frame_tokens, rows=rows)

    for _ in range(args.warmup):
        out = step()
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    stream = torch.cuda.current_stream(dev)
    sampler = ClockSampler([0])
    with sampler:
        time.sleep(0.2)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    nbytes = 3 * H * T * D * 2  # K twice, V once
    peaks, kind = load_peaks()
    gbs = nbytes / (ms * 1e-3) / 1e9
    print(json.dumps({
        "metric": "Head classification (sampled-row MSE of the spatial/temporal masks), ms per call",
        "value": ms, "unit": "ms", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1))",
        "config": {"workload": "hunyuan-720p sample_mse", "heads": H, "seq_len": T, "head_dim": D,
                   "sampled_rows": 32, "context_length": w.text_tokens, "num_frame": w.frames,
                   "frame_size": w.frame_tokens},
        "roofline": {"kernel": "mse_stats_kernel + mse_pv_kernel", "bound": "hbm", "achieved": gbs,
                     "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": gbs / peaks["hbm_gbs"], "traffic": None,
                     "peak_source": f"{kind} hbm_gbs", "algorithmic_bytes": nbytes},
        "clocks": sampler.summary(), "gpu_launches": 4 * args.steps,
    }), flush=True)


def main():
    args = parse()
    if args.place:
        run_place(args)
        return
    if args.classify:
        run_classify(args)
        return
    if args.dit:
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the reference's DiT step needs diffusers and "
                              "model checkpoints, neither present"}), flush=True)
            return
        run_dit(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    import torch

    from pasa_b200 import _lib, ops, synth

    world, rank, local = init_dist()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    w = synth.WORKLOADS[args.config]
    if args.heads:
        import dataclasses

        w = dataclasses.replace(w, heads=args.heads)
    # heads split over the ranks when the world size divides them; otherwise
    # (12 heads over 8 GPUs, say) ranges of query blocks, each rank preparing
    # the heads its range touches (pasa_forward_range)
    block_mode = world > 1 and w.heads % world != 0
    if block_mode:
        blk_b, blk_e = synth.shard_blocks(w.heads, w.NT, rank, world)
        heads = range(blk_b // w.NT, -(-blk_e // w.NT))
        blk_b, blk_e = blk_b - heads.start * w.NT, blk_e - heads.start * w.NT  # within the rank's heads
        units = (blk_e - blk_b) / w.NT  # heads' worth of query blocks
    else:
        heads = synth.shard_heads(w.heads, rank, world)
        units = len(heads)
    nh = len(heads)
    kernel = {"auto": _lib.ATTN_AUTO, "tcgen05": _lib.ATTN_TCGEN05, "simt": _lib.ATTN_SIMT}[args.kernel]

    q, k, v = synth.make_inputs(w, heads, dev)
    B, H, T, D = q.shape
    scale = D ** -0.5
    NT, NG, NS = _lib.derive(T, w.density)
    dcode = ops._dtype_code(q)
    st = ops.Stages(B, H, T, D, NT, NG, NS, q.dtype, dev)
    o = torch.empty_like(v)
    stream = torch.cuda.current_stream(dev)

    def step(ev=None):
        if block_mode:  # one call: prep and selection of the touched heads, attention on the range
            if ev: ev[0].record(stream)
            if ev: ev[1].record(stream)
            if ev: ev[2].record(stream)
            ops.pisa_pg_attention_range(q, k, v, blk_b, blk_e, density=w.density, out=o)
            if ev: ev[3].record(stream)
            return
        if ev: ev[0].record(stream)
        ops.prep(q, k, v, st)
        if ev: ev[1].record(stream)
        ops.select(st, D, dcode, scale, True, None)
        if ev: ev[2].record(stream)
        ops.attn(q, k, v, st, scale, o, kernel)
        if ev: ev[3].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ops.check_device_errors(st)

    events = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    gpu_ids = [int(x) for x in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if x.strip().isdigit()]
    phys = gpu_ids[local] if local < len(gpu_ids) else local
    sampler = ClockSampler([phys])
    with sampler:
        time.sleep(0.3)
        barrier(world)
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for i in range(args.steps):
            step(events[i])
        end.record(stream)
        torch.cuda.synchronize()
        barrier(world)
    ops.check_device_errors(st)
    total_ms = start.elapsed_time(end)
    t_prep = [e[0].elapsed_time(e[1]) for e in events]
    t_sel = [e[1].elapsed_time(e[2]) for e in events]
    t_attn = [e[2].elapsed_time(e[3]) for e in events]
    ms_step = max_over_ranks(total_ms / args.steps, world)
    attn_ms = max_over_ranks(statistics.mean(t_attn), world)
    prep_ms = max_over_ranks(statistics.mean(t_prep), world)
    sel_ms = max_over_ranks(statistics.mean(t_sel), world)
    clocks = sampler.summary()

    F = w.exact_flops()
    Fc = w.corr_flops()
    value = F / (ms_step * 1e-3) / 1e12

    # ---- end to end: public API, host buffers, copies inside the timed region
    e2e = None
    if not args.no_e2e:
        qh, kh, vh = (t.cpu().pin_memory() for t in (q, k, v))
        oh = torch.empty(o.shape, dtype=o.dtype).pin_memory()
        rows = slice(blk_b * 64, min(blk_e * 64, H * T)) if block_mode else None

        def e2e_step():
            if block_mode:
                # the touched heads in, the rank's rows out (no chunk pipeline)
                for hd, dd in ((qh, q), (kh, k), (vh, v)):
                    dd.copy_(hd, non_blocking=True)
                ops.pisa_pg_attention_range(q, k, v, blk_b, blk_e, density=w.density, out=o)
                oh.view(H * T, D)[rows].copy_(o.view(H * T, D)[rows], non_blocking=True)
                return
            # host buffers in, host buffer out: the copies of head chunk i+1 (in)
            # and i-1 (out) overlap the GPU work on chunk i (pasa_forward_host)
            ops.pisa_pg_attention_host(qh, kh, vh, density=w.density, heads_per_chunk=args.e2e_chunk, out=oh,
                                       device=dev, kernel=kernel)

        for _ in range(max(1, args.warmup)):
            e2e_step()
        torch.cuda.synchronize()
        barrier(world)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        s1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        e2e_ms = max_over_ranks(s0.elapsed_time(s1) / args.steps, world)
        # every step's result is read back: check it once (cheap) after timing
        assert torch.isfinite(oh.float()).all()
        nbytes = lambda t: t.numel() * t.element_size()
        h2d = max_over_ranks(nbytes(q) + nbytes(k) + nbytes(v), world) * world
        d2h = (rows.stop - rows.start) * D * o.element_size() if block_mode else nbytes(o)
        e2e = {"value": F / (e2e_ms * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": max_over_ranks(d2h, world) * world,
               "heads_per_chunk": None if block_mode else args.e2e_chunk,
               "h2d_gbs_per_rank": (nbytes(q) + nbytes(k) + nbytes(v)) / (e2e_ms * 1e-3) / 1e9,
               "numa_node": int(os.environ.get("PASA_NUMA_NODE", "-1")),
               "note": ("per rank (the largest), times the ranks; " if world > 1 else "")
               + ("pinned host q/k/v of the rank's heads in, the rank's rows of o out, pisa_pg_attention_range"
                  if block_mode else "pisa_pg_attention_host: pinned host q/k/v in, pinned host o out, copies "
                  "pipelined over head chunks")}

    peaks, peak_kind = load_peaks()
    # the attention kernel runs inside a call of ~25 ms, so the burst figure
    # is its denominator; the sustained one is reported beside it
    peak_tf = peaks.get("bf16_tflops") or peaks.get("bf16_tflops_sustained")
    peak_sus = peaks.get("bf16_tflops_sustained") or peak_tf
    F_rank = w.exact_flops(units)
    achieved = F_rank / (attn_ms * 1e-3) / 1e12
    resolved = kernel if kernel != _lib.ATTN_AUTO else (
        _lib.ATTN_TCGEN05 if q.dtype == torch.bfloat16 else _lib.ATTN_SIMT)  # as pasa_attn resolves AUTO
    traffic = ATTN_TRAFFIC_BYTES.get((w.name, "tcgen05" if resolved == _lib.ATTN_TCGEN05 else "simt"))
    if traffic is not None:
        full = synth.WORKLOADS[args.config].heads
        traffic = traffic * units / full  # this rank's launch covers `units` of the workload's heads
    # MMA work the tensor-core kernel executes on this call's selections: a CTA
    # serves query blocks 2p and 2p+1 and takes ceil(|S_2p ∪ S_2p+1| / 2)
    # steps of two key blocks (score and P.V MMAs, M=128, N=K=128), then one
    # step per 32-block group (scores N=32, P_g.vc_g K=32, U.H_g K=D)
    exec_flop = None
    if resolved == _lib.ATTN_TCGEN05 and not block_mode:
        m = st.sel_mask.view(torch.int32)
        a, b = m[:, 0::2], m[:, 1::2]
        if b.shape[1] < a.shape[1]:
            b = torch.cat([b, torch.zeros_like(a[:, :1])], 1)
        union = torch.bitwise_or(a, b)
        bits = sum(((union >> i) & 1).sum(-1) for i in range(32))          # [BH, pairs]
        steps1 = int(((bits + 1) // 2).sum())
        tiles = int(a.shape[0] * a.shape[1])
        exec_flop = steps1 * 4 * 128 * 128 * D + tiles * NG * (4 * 128 * 32 * D + 2 * 128 * D * D)
    roofline = {
        "kernel": f"attn_tc_kernel<{D}>" if resolved == _lib.ATTN_TCGEN05 else f"attn_simt_kernel<{D}>",
        "bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
        "frac": achieved / peak_tf, "traffic": traffic,
        "peak_source": f"{peak_kind} bf16_tflops (burst: the kernel runs inside a ~25 ms call)",
        "peak_sustained": peak_sus, "frac_sustained": achieved / peak_sus,
        "achieved_basis": ("exact-block FLOPs per launch / mean CUDA-event launch time" if not block_mode else
                           "exact-block FLOPs of the rank's blocks / whole pasa_forward_range call (prep and "
                           "selection included)"),
        "achieved_incl_correction": (w.exact_flops(units) + w.corr_flops(units)) / (attn_ms * 1e-3) / 1e12,
    }
    if exec_flop is not None:
        # the MMAs the kernel runs (union of two query blocks' selections per
        # tile, plus the correction): how busy the tensor core is kept
        roofline["executed_tflop"] = exec_flop / 1e12
        roofline["achieved_executed"] = exec_flop / (attn_ms * 1e-3) / 1e12
        roofline["frac_executed"] = roofline["achieved_executed"] / peak_tf
        roofline["frac_executed_sustained"] = roofline["achieved_executed"] / peak_sus

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(w)
        cpu.pop("s_per_head", None)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16" if w.dtype == torch.bfloat16 else "f32",
            "data": "synthetic (seeded N(0,1), AR(1) keys across frames; generated on the device)",
            "config": {"workload": w.name, "heads": w.heads, "seq_len": T, "head_dim": D, "density": w.density,
                       "block": 64, "group": 32, "top_k": NS,
                       "parallelism": (f"query-block ranges/{world} (heads do not divide)" if block_mode
                                       else f"heads/{world}"),
                       "l2": "inputs 2.3 GB per call > 126 MB L2; no flush" if w.name == "wan14b-720p" else
                       "see workload size"},
            "kernels_ms": ({"forward_range": attn_ms} if block_mode else
                           {"prep": prep_ms, "select": sel_ms, "attn": attn_ms}),
            "exact_tflop": F / 1e12, "corr_tflop": Fc / 1e12,
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks,
            "gpu_launches": 3 * args.steps,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
