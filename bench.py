"""Benchmark: fused 2D-RoPE SDPA forward+backward TFLOP/s on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config vit_b|vit_s|vit_l|vit_h]
                    [--impl ours|reference]

One step = one forward and one backward pass of the fused RoPE attention over
the whole configured batch (ViT-B/16 by default: B=256, H=12, N=197, D=64,
bf16), inputs resident in HBM. FLOPs per step = 14 B H N^2 D (forward 4,
backward 10). Multi-GPU: every rank runs the same per-GPU workload on its own
(batch x heads) shard with no collective on the data path ("weak" scaling);
the step time is the max over ranks of CUDA-event time.

``--impl reference`` times the reference's own algorithm on the host CPU: the
PyTorch-SDPA + Python-2D-RoPE restatement in ``oracle/`` (the reference ships
no CPU kernel and its Triton kernels are GPU-only), on a bounded sample.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "fused RoPE-SDPA fwd+bwd TFLOP/s per B200 and box at 1/2/4/8 GPUs (ViT-B/16 shape)"

# name -> (B, H, H_img, has_cls, D, input scale, description)
CONFIGS = {
    "vit_s": (512, 6, 14, True, 64, 1.0, "ViT-S/16-224 attention layer"),
    "vit_b": (256, 12, 14, True, 64, 1.0, "ViT-B/16-224 attention layer"),
    "vit_l": (128, 16, 24, False, 64, 1.0, "ViT-L/16-384 attention layer, no CLS"),
    "vit_h": (64, 16, 37, True, 80, 2.0, "ViT-H/14-518 attention layer"),
}


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
                "source": "fallback"}


def load_traffic(config_name):
    """Per-launch DRAM traffic of the dominant kernel from the committed ncu summary, or None."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(config_name)
    except Exception:
        return None


class ClockSampler:
    """Samples SM clocks and throttle reasons of the given GPUs during the timed region.

    One ``nvidia-smi --query-gpu ... -lms 200`` process streams samples for all
    listed GPUs (a read-only query; nothing is changed on the GPU). Only one
    rank runs it, so an N-rank job does not fork N samplers.
    """

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices):
        self.gpus = list(gpu_indices)
        self.samples = []
        self._proc = None
        self._thr = None

    def _reader(self):
        for line in self._proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.samples.append(parts)

    def start(self):
        try:
            self._proc = subprocess.Popen(
                ["nvidia-smi", "-i", ",".join(str(g) for g in self.gpus),
                 f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self._proc = None
            return
        self._thr = threading.Thread(target=self._reader, daemon=True)
        self._thr.start()

    def stop(self):
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except Exception:
                self._proc.kill()
        if self._thr:
            self._thr.join(timeout=5)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"],
                    "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [v for v in (num(s[1]) for s in self.samples) if v is not None]
        mx = [v for v in (num(s[2]) for s in self.samples) if v is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for s in self.samples:
            for n, v in zip(names, s[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(self.samples), "gpus": self.gpus}


def shape_of(name):
    B, H, side, has_cls, D, amp, desc = CONFIGS[name]
    N = side * side + (1 if has_cls else 0)
    return B, H, side, has_cls, N, D, amp, desc


def flops_fwd(B, H, N, D):
    return 4.0 * B * H * N * N * D


def flops_bwd(B, H, N, D):
    return 10.0 * B * H * N * N * D


def bytes_fwd(B, H, N, D, elt=2):
    return 4.0 * B * H * N * D * elt + 4.0 * B * H * N   # Q,K,V in, O out, LSE out


def bytes_bwd(B, H, N, D, elt=2):
    return 8.0 * B * H * N * D * elt + 4.0 * B * H * N   # Q,K,V,O,dO in, dQ,dK,dV out, LSE in


REF_DIR = os.path.join(ROOT, "baseline", "_ref")
REF_FILE = os.path.join(REF_DIR, "fa_rope_full .py")


# Autotune configurations of the reference that Triton failed to compile (see below).
REF_COMPILER_FAILURES = []


def _score_compiler_failures_as_slow():
    """Let Triton's autotuner skip reference configs its compiler cannot build.

    On this image (Triton 3.6, sm_100) some of the reference's autotune configs
    of ``_attn_bwd_dk_dv_rope`` (fa_rope_full .py:359-373) make Triton's
    software pipeliner fail an internal assertion ("PassManager::run failed"),
    intermittently. Triton's autotuner already scores configs that fail with
    OutOfResources or a PTXAS error as infinitely slow; this extends the same
    treatment to this compiler failure, so the autotuner picks the fastest of
    the configs that build. The reference's source and its kernels are used
    unchanged; the failures are recorded in REF_COMPILER_FAILURES.
    """
    from triton.runtime import autotuner
    if getattr(autotuner.Autotuner, "_frsa_scores_failures", False):
        return
    orig = autotuner.Autotuner._bench

    def _bench(self, *args, config, **meta):
        try:
            return orig(self, *args, config=config, **meta)
        except RuntimeError as e:
            if "PassManager::run failed" not in str(e):
                raise
            REF_COMPILER_FAILURES.append(f"{self.base_fn.__name__}: {config}")
            return [float("inf"), float("inf"), float("inf")]

    autotuner.Autotuner._bench = _bench
    autotuner.Autotuner._frsa_scores_failures = True


def load_reference_triton():
    """Import the reference's own module (its Triton kernels) from ``baseline/_ref``.

    ``baseline/_ref`` is an untracked copy of the reference's single source
    file (fa_rope_full .py); it is never part of this repository's product.
    Triton's autotune results are cached under ``baseline/_ref/triton_cache``
    (``TRITON_CACHE_AUTOTUNING``), so a run after the first one compiles only
    the configurations the reference's own autotuner chose on this hardware.
    Returns ``(module, None)`` or ``(None, reason)``.
    """
    if not os.path.exists(REF_FILE):
        return None, f"reference source absent ({os.path.relpath(REF_FILE, ROOT)} not installed)"
    os.environ.setdefault("TRITON_CACHE_DIR", os.path.join(REF_DIR, "triton_cache"))
    os.environ.setdefault("TRITON_CACHE_AUTOTUNING", "1")
    _score_compiler_failures_as_slow()
    import importlib.util
    try:
        spec = importlib.util.spec_from_file_location("fa_rope_full_reference", REF_FILE)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    except Exception as e:  # noqa: BLE001 - reported, not hidden
        return None, f"reference import failed: {type(e).__name__}: {str(e)[:200]}"
    return mod, None


def reference_triton_run(name, q, k, v, do, steps, warmup):
    """Time the reference's Triton kernels through its public autograd class.

    ``TritonAttention.apply(Q, K, V, cos_sin, H_img, has_cls)`` (fa_rope_full
    .py:1011-1138) on the same device tensors as this repository's arm; the
    forward and the autograd backward are timed separately with CUDA events
    on the current stream after ``warmup`` untimed steps (the first of which
    runs the reference's autotuner, or loads its cached choice).
    """
    B, H, side, has_cls, N, D, amp, _ = shape_of(name)
    ref, why = load_reference_triton()
    if ref is None:
        return {"unavailable": why}
    dev = q.device
    qr, kr, vr = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
    try:
        cs = ref.CosSinTable(100.0, side, D, device=dev)
        t0 = time.time()
        o = ref.TritonAttention.apply(qr, kr, vr, cs, side, has_cls)
        o.backward(do)
        torch.cuda.synchronize(dev)
        first_s = time.time() - t0
    except Exception as e:  # noqa: BLE001 - e.g. D=80: tl.arange needs a power of two
        msg = " ".join(str(e).split())[:240]
        return {"unavailable": f"reference Triton kernel failed at {name} (D={D}): "
                               f"{type(e).__name__}: {msg}"}
    for _ in range(max(3, warmup)):
        o = ref.TritonAttention.apply(qr, kr, vr, cs, side, has_cls)
        o.backward(do)
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    for i in range(steps):
        qr.grad = kr.grad = vr.grad = None
        ev[i][0].record(stream)
        o = ref.TritonAttention.apply(qr, kr, vr, cs, side, has_cls)
        ev[i][1].record(stream)
        o.backward(do)
        ev[i][2].record(stream)
    torch.cuda.synchronize(dev)
    fwd_ms = sum(e[0].elapsed_time(e[1]) for e in ev) / steps
    bwd_ms = sum(e[1].elapsed_time(e[2]) for e in ev) / steps
    fl = flops_fwd(B, H, N, D) + flops_bwd(B, H, N, D)
    return {"fwd_ms": round(fwd_ms, 4), "bwd_ms": round(bwd_ms, 4),
            "ms_per_step": round(fwd_ms + bwd_ms, 4),
            "tflops": round(fl / ((fwd_ms + bwd_ms) * 1e-3) / 1e12, 1),
            "first_call_s": round(first_s, 1), "steps": steps,
            "autotune_configs_failed_to_compile": len(REF_COMPILER_FAILURES),
            "api": "reference TritonAttention.apply + autograd backward (baseline/_ref)"}


def init_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("gloo")
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_rows(vals, world, device):
    """All ranks' lists of floats, in rank order (every rank receives all of them)."""
    mine = torch.tensor(vals, dtype=torch.float64, device=device)
    if world == 1:
        return [mine.tolist()]
    allr = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(allr, mine)
    return [x.tolist() for x in allr]


def barrier(world):
    if world > 1:
        dist.barrier()


def cpu_reference_run(name, steps, warmup, budget_s=60.0, threads=None):
    """Time the reference algorithm (PyTorch SDPA + Python 2D RoPE, fp32) on host cores.

    Each step runs fwd+bwd on a batch sample of the configured workload, sized
    so the whole run stays within ``budget_s``. Returns
    ``(tflops, sample_desc, cores, ms_per_step)``.
    """
    from oracle import attn_fwd_bwd_torch, rope_tables_np
    B, H, side, has_cls, N, D, amp, _ = shape_of(name)
    cores = threads or len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    cos, sin = rope_tables_np(side, D, 100.0)

    def run(bs):
        g = torch.Generator().manual_seed(0)
        q, k, v, do = (torch.randn(bs, H, N, D, generator=g) for _ in range(4))
        t0 = time.perf_counter()
        attn_fwd_bwd_torch(q * amp, k * amp, v * amp, do, cos, sin, has_cls)
        return time.perf_counter() - t0

    run(1)
    t1 = run(1)
    total_steps = max(1, steps + warmup)
    bs = int(max(1, min(B, budget_s / total_steps / max(t1, 1e-6))))
    for _ in range(warmup):
        run(bs)
    times = [run(bs) for _ in range(max(1, steps))]
    t = sum(times) / len(times)
    fl = flops_fwd(bs, H, N, D) + flops_bwd(bs, H, N, D)
    sample = (f"{bs} of {B} batch items x {H} heads (N={N}, D={D}) per step, fp32, "
              f"torch CPU SDPA+RoPE restatement, {cores} threads")
    return fl / t / 1e12, sample, cores, t * 1e3


def make_inputs(name, B, dev, seed):
    """Seeded N(0,1) q/k/v/dO of the config's shape (q/k/v times its amplitude), bf16."""
    _, H, _, _, N, D, amp, _ = shape_of(name)
    g = torch.Generator(device=dev).manual_seed(seed)
    q, k, v, do = (torch.randn(B, H, N, D, generator=g, device=dev, dtype=torch.float32)
                   for _ in range(4))
    q, k, v = (t * amp for t in (q, k, v))
    return [t.to(torch.bfloat16) for t in (q, k, v, do)]


def time_ours(name, q, k, v, do, steps, warmup, world=1, sampler=None):
    """Device-timed fwd + bwd steps of this repository's kernels through the C ABI.

    Returns total elapsed ms (CUDA events around all steps), mean fwd/bwd ms
    per step (events around each call) and the host time spent enqueueing.
    """
    from triton_fused_rope_flash_attn_b200 import (CosSinTable, _lib, fused_rope_attention_bwd,
                                                   fused_rope_attention_fwd)
    _, _, side, has_cls, _, D, _, _ = shape_of(name)
    dev = q.device
    cs = CosSinTable(100.0, side, D, device=dev)
    cosp, sinp = cs.tables()
    for _ in range(max(3, warmup)):
        o, lse = fused_rope_attention_fwd(q, k, v, cosp, sinp, has_cls)
        fused_rope_attention_bwd(q, k, v, o, lse, do, cosp, sinp, has_cls)
    torch.cuda.synchronize(dev)
    assert _lib.load().frsa_query_status() == 0, "device status error after warm-up"
    stream = torch.cuda.current_stream(dev)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    if sampler is not None:
        sampler.start()
        time.sleep(0.5)
    barrier(world)
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_host = time.perf_counter()
    start.record(stream)
    for i in range(steps):
        ev[i][0].record(stream)
        o, lse = fused_rope_attention_fwd(q, k, v, cosp, sinp, has_cls)
        ev[i][1].record(stream)
        fused_rope_attention_bwd(q, k, v, o, lse, do, cosp, sinp, has_cls)
        ev[i][2].record(stream)
    end.record(stream)
    host_ms = (time.perf_counter() - t_host) * 1e3
    torch.cuda.synchronize(dev)
    barrier(world)
    if sampler is not None:
        sampler.stop()
    status = _lib.load().frsa_query_status()
    assert status == 0, f"device status {status}"
    return {"elapsed_ms": start.elapsed_time(end),
            "fwd_ms": sum(e[0].elapsed_time(e[1]) for e in ev) / steps,
            "bwd_ms": sum(e[1].elapsed_time(e[2]) for e in ev) / steps,
            "host_enqueue_ms_per_step": host_ms / steps, "cs": cs}


def roofline_of(B, H, N, D, ms, flops, nbytes, peaks):
    """Bound (HBM or tensor, by arithmetic intensity against the measured ridge) and the
    achieved fraction of it for `flops` FLOPs / `nbytes` algorithmic bytes in `ms`."""
    ridge = peaks["bf16_tflops"] * 1e12 / (peaks["hbm_gbs"] * 1e9)
    if flops / nbytes < ridge:
        ach = nbytes / (ms * 1e-3) / 1e9
        return {"bound": "hbm", "achieved": round(ach, 1), "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": round(ach / peaks["hbm_gbs"], 4)}
    ach = flops / (ms * 1e-3) / 1e12
    return {"bound": "tensor", "achieved": round(ach, 1), "peak": peaks["bf16_tflops"],
            "unit": "TFLOP/s", "frac": round(ach / peaks["bf16_tflops"], 4)}


def launches_per_step(N, D):
    # fwd + bwd; the general backward adds its row pre-pass and the dQ
    # finalize pass (the counter clear is a cudaMemsetAsync, not a kernel of
    # this library).
    return 2 if (N <= 256 and D <= 64) else 4


def gpu_arm(args, world, rank, local):
    from triton_fused_rope_flash_attn_b200 import sdpa_triton_fa_rope
    from triton_fused_rope_flash_attn_b200.build import build_library

    build_library()
    dev = torch.device("cuda", local)
    B, H, side, has_cls, N, D, amp, desc = shape_of(args.config)
    if args.batch:
        B = args.batch
    q, k, v, do = make_inputs(args.config, B, dev, 1234 + rank)
    sampler = ClockSampler(range(world)) if local == 0 else None
    K = args.steps
    t = time_ours(args.config, q, k, v, do, K, args.warmup, world, sampler)
    cs = t.pop("cs")
    fwd_ms, bwd_ms = t["fwd_ms"], t["bwd_ms"]

    # Per-rank figures, gathered to rank 0 (the step time is the max over ranks).
    allr = gather_rows([t["elapsed_ms"], fwd_ms, bwd_ms, t["host_enqueue_ms_per_step"]], world,
                       dev)
    per_rank = [{"rank": i, "ms_per_step": round(float(x[0]) / K, 4),
                 "fwd_ms": round(float(x[1]), 4), "bwd_ms": round(float(x[2]), 4),
                 "host_enqueue_ms_per_step": round(float(x[3]), 4)} for i, x in enumerate(allr)]
    elapsed_max = max(float(x[0]) for x in allr)
    ms_per_step = elapsed_max / K
    step_flops = flops_fwd(B, H, N, D) + flops_bwd(B, H, N, D)
    value = step_flops * world / (ms_per_step * 1e-3) / 1e12

    # End to end through the public API: pinned host inputs copied in and the
    # loss copied out inside the timed region, autograd backward included.
    hq, hk, hv, hdo = (x.cpu().pin_memory() for x in (q, k, v, do))
    loss_h = torch.empty((), dtype=torch.float32).pin_memory()
    E = max(3, min(args.e2e_steps, K))
    stream = torch.cuda.current_stream(dev)

    def e2e_step():
        qd, kd, vd = (x.to(dev, non_blocking=True).requires_grad_(True) for x in (hq, hk, hv))
        dod = hdo.to(dev, non_blocking=True)
        out = sdpa_triton_fa_rope(qd, kd, vd, cs, has_cls=has_cls, H_img=side)
        out.backward(dod)
        loss_h.copy_(out.detach().float().sum(), non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(dev)
    barrier(world)
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record(stream)
    for _ in range(E):
        e2e_step()
    e2.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(s2.elapsed_time(e2) / E, world, dev)
    e2e_value = step_flops * world / (e2e_ms * 1e-3) / 1e12
    h2d = sum(x.numel() * x.element_size() for x in (hq, hk, hv, hdo))

    peaks = load_peaks()
    fb, bb = flops_bwd(B, H, N, D), bytes_bwd(B, H, N, D)
    psrc = "of measured (MEASURED_PEAKS.json)" if peaks["source"] == "measured" else "of fallback"
    roof = roofline_of(B, H, N, D, bwd_ms, fb, bb, peaks)
    small = N <= 256 and D <= 64
    traffic = load_traffic(args.config) if not args.batch else None
    roof.update({"traffic": traffic, "kernel": "bwd_small_kernel" if small else "bwd_kernel",
                 "peak_source": psrc, "algorithmic_bytes_per_launch": bb,
                 "algorithmic_flops_per_launch": fb,
                 "tensor_frac": round(fb / (bwd_ms * 1e-3) / 1e12 / peaks["bf16_tflops"], 4)})
    mb = B * H * N * D * 2 / 1e6
    return {
        "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": K, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) q/k/v/dO on device)",
        "config": {"workload": f"{args.config}: {desc} fwd+bwd, B={B} H={H} N={N} D={D} "
                               f"has_cls={has_cls} bf16, RoPE base 100, per GPU",
                   "B_per_gpu": B, "H": H, "N": N, "D": D, "has_cls": has_cls,
                   "global_batch": B * world, "seq_len": N,
                   "parallelism": f"dp{world} (B x H shards, no collective)",
                   "l2": f"inputs 4 x {mb:.0f} MB per rank exceed the 126 MB L2; no flush"},
        "kernels": {"fwd_ms": round(fwd_ms, 4), "bwd_ms": round(bwd_ms, 4),
                    "fwd_tflops": round(flops_fwd(B, H, N, D) / (fwd_ms * 1e-3) / 1e12, 1),
                    "bwd_tflops": round(fb / (bwd_ms * 1e-3) / 1e12, 1),
                    "fwd_gbs": round(bytes_fwd(B, H, N, D) / (fwd_ms * 1e-3) / 1e9, 1),
                    "bwd_gbs": round(bb / (bwd_ms * 1e-3) / 1e9, 1)},
        "roofline": roof,
        "e2e": {"value": round(e2e_value, 2), "unit": "TFLOP/s", "ms_per_step": round(e2e_ms, 3),
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
                "api": "sdpa_triton_fa_rope + autograd backward, pinned host inputs"},
        "gpu_launches": launches_per_step(N, D) * K,
        "per_rank": per_rank,
        "clocks": sampler.summary() if sampler is not None else None,
    }, (q, k, v, do)


def other_config(name, steps, warmup, with_reference):
    """Kernel timing of another BASELINE config on this GPU (N=1 runs only), with the
    reference's Triton kernels on the same inputs when they compile for it."""
    B, H, side, has_cls, N, D, amp, desc = shape_of(name)
    dev = torch.device("cuda", torch.cuda.current_device())
    q, k, v, do = make_inputs(name, B, dev, 4321)
    t = time_ours(name, q, k, v, do, steps, warmup)
    t.pop("cs")
    peaks = load_peaks()
    ff, fb = flops_fwd(B, H, N, D), flops_bwd(B, H, N, D)
    ms = t["fwd_ms"] + t["bwd_ms"]
    out = {"workload": f"{desc} fwd+bwd, B={B} H={H} N={N} D={D} has_cls={has_cls} bf16"
                       + (f", q/k/v x{amp}" if amp != 1.0 else ""),
           "fwd_ms": round(t["fwd_ms"], 4), "bwd_ms": round(t["bwd_ms"], 4),
           "ms_per_step": round(ms, 4), "tflops": round((ff + fb) / (ms * 1e-3) / 1e12, 1),
           "fwd_tflops": round(ff / (t["fwd_ms"] * 1e-3) / 1e12, 1),
           "bwd_tflops": round(fb / (t["bwd_ms"] * 1e-3) / 1e12, 1),
           "tensor_frac": round((ff + fb) / (ms * 1e-3) / 1e12 / peaks["bf16_tflops"], 4),
           "roofline_bwd": roofline_of(B, H, N, D, t["bwd_ms"], fb, bytes_bwd(B, H, N, D), peaks),
           "roofline_fwd": roofline_of(B, H, N, D, t["fwd_ms"], ff, bytes_fwd(B, H, N, D), peaks),
           "steps": steps}
    if with_reference:
        r = reference_triton_run(name, q, k, v, do, steps, warmup)
        if "ms_per_step" in r:
            r["ours_over_reference"] = round(r["ms_per_step"] / ms, 3)
        out["reference_triton"] = r
    return out


def reference_arm(args, world, rank):
    if rank == 0:
        tf, sample, cores, ms = cpu_reference_run(args.config, args.steps, args.warmup)
        B, H, side, has_cls, N, D, amp, desc = shape_of(args.config)
        line = {"metric": METRIC, "value": round(tf, 4), "unit": "TFLOP/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f32", "data": "synthetic (seeded N(0,1))", "impl": "reference",
                "config": {"workload": f"{args.config}: {desc} fwd+bwd, B={B} H={H} N={N} "
                                       f"D={D} has_cls={has_cls}",
                           "B_per_gpu": B, "H": H, "N": N, "D": D, "has_cls": has_cls,
                           "global_batch": B * world, "seq_len": N,
                           "parallelism": f"dp{world} (B x H shards, no collective)"},
                "cpu_baseline": {"value": round(tf, 4), "unit": "TFLOP/s", "cores": cores,
                                 "kind": "port", "sample": sample},
                "e2e": {"value": round(tf, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--config", default="vit_b", choices=sorted(CONFIGS))
    ap.add_argument("--batch", type=int, default=0, help="override B (profiling small cases)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reference-triton", action="store_true",
                    help="skip timing the reference's Triton kernels beside this arm (N=1)")
    ap.add_argument("--no-other-configs", action="store_true",
                    help="skip the other BASELINE configs (N=1 runs add them to the line)")
    args = ap.parse_args()
    world, rank, local = init_dist()

    if args.impl == "reference":
        reference_arm(args, world, rank)
        if world > 1:
            dist.destroy_process_group()
        return

    line, tensors = gpu_arm(args, world, rank, local)
    if rank == 0 and world == 1:
        if not args.no_cpu_baseline:
            tf, sample, cores, _ = cpu_reference_run(args.config, 3, 1, budget_s=20.0)
            line["cpu_baseline"] = {"value": round(tf, 4), "unit": "TFLOP/s", "cores": cores,
                                    "kind": "port", "sample": sample}
        if not args.no_reference_triton:
            r = reference_triton_run(args.config, *tensors, steps=min(args.steps, 50),
                                     warmup=args.warmup)
            if "ms_per_step" in r:
                r["ours_over_reference"] = round(
                    r["ms_per_step"] / (line["kernels"]["fwd_ms"] + line["kernels"]["bwd_ms"]), 3)
            line["reference_triton"] = r
        del tensors
        if not args.no_other_configs and not args.batch:
            line["configs"] = {name: other_config(name, min(args.steps, 20), 3,
                                                  not args.no_reference_triton)
                               for name in sorted(CONFIGS) if name != args.config}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
