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
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []
        self._stop = threading.Event()
        self._thr = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(
                    ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.QUERY}",
                     "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                line = out.stdout.strip().splitlines()
                if line:
                    self.samples.append([x.strip() for x in line[0].split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def start(self):
        self._thr = threading.Thread(target=self._run, daemon=True)
        self._thr.start()

    def stop(self):
        self._stop.set()
        if self._thr:
            self._thr.join(timeout=10)

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
                "samples": len(self.samples)}


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


def gpu_arm(args, world, rank, local):
    from triton_fused_rope_flash_attn_b200 import (CosSinTable, fused_rope_attention_bwd,
                                                   fused_rope_attention_fwd, sdpa_triton_fa_rope)
    from triton_fused_rope_flash_attn_b200 import _lib
    from triton_fused_rope_flash_attn_b200.build import build_library

    build_library()
    dev = torch.device("cuda", local)
    B, H, side, has_cls, N, D, amp, desc = shape_of(args.config)
    if args.batch:
        B = args.batch
    dtype = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    q, k, v, do = (torch.randn(B, H, N, D, generator=g, device=dev, dtype=torch.float32)
                   for _ in range(4))
    q, k, v = (t * amp for t in (q, k, v))
    q, k, v, do = (t.to(dtype) for t in (q, k, v, do))
    cs = CosSinTable(100.0, side, D, device=dev)
    cosp, sinp = cs.tables()

    for _ in range(max(3, args.warmup)):
        o, lse = fused_rope_attention_fwd(q, k, v, cosp, sinp, has_cls)
        fused_rope_attention_bwd(q, k, v, o, lse, do, cosp, sinp, has_cls)
    torch.cuda.synchronize(dev)
    assert _lib.load().frsa_query_status() == 0, "device status error after warm-up"

    stream = torch.cuda.current_stream(dev)
    K = args.steps
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(K)]
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(K):
        ev[i][0].record(stream)
        o, lse = fused_rope_attention_fwd(q, k, v, cosp, sinp, has_cls)
        ev[i][1].record(stream)
        fused_rope_attention_bwd(q, k, v, o, lse, do, cosp, sinp, has_cls)
        ev[i][2].record(stream)
    end.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    sampler.stop()
    elapsed_ms = start.elapsed_time(end)
    fwd_ms = sum(e[0].elapsed_time(e[1]) for e in ev) / K
    bwd_ms = sum(e[1].elapsed_time(e[2]) for e in ev) / K
    status = _lib.load().frsa_query_status()
    assert status == 0, f"device status {status}"

    elapsed_max = max_over_ranks(elapsed_ms, world, dev)
    ms_per_step = elapsed_max / K
    step_flops = flops_fwd(B, H, N, D) + flops_bwd(B, H, N, D)
    value = step_flops * world / (ms_per_step * 1e-3) / 1e12

    # End to end through the public API: pinned host inputs copied in and the
    # loss copied out inside the timed region, autograd backward included.
    hq, hk, hv, hdo = (t.cpu().pin_memory() for t in (q, k, v, do))
    loss_h = torch.empty((), dtype=torch.float32).pin_memory()
    E = max(3, min(args.e2e_steps, K))

    def e2e_step():
        qd, kd, vd = (t.to(dev, non_blocking=True).requires_grad_(True) for t in (hq, hk, hv))
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
    h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv, hdo))

    peaks = load_peaks()
    ridge = peaks["bf16_tflops"] * 1e12 / (peaks["hbm_gbs"] * 1e9)
    fb, bb = flops_bwd(B, H, N, D), bytes_bwd(B, H, N, D)
    psrc = "of measured (MEASURED_PEAKS.json)" if peaks["source"] == "measured" else "of fallback"
    if fb / bb < ridge:
        ach = bb / (bwd_ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": round(ach, 1), "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": round(ach / peaks["hbm_gbs"], 4)}
    else:
        ach = fb / (bwd_ms * 1e-3) / 1e12
        roof = {"bound": "tensor", "achieved": round(ach, 1), "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": round(ach / peaks["bf16_tflops"], 4)}
    small = N <= 256 and D <= 64
    traffic = load_traffic(args.config) if not args.batch else None
    roof.update({"traffic": traffic, "kernel": "bwd_small_kernel" if small else "bwd_kernel",
                 "peak_source": psrc, "algorithmic_bytes_per_launch": bb,
                 "algorithmic_flops_per_launch": fb,
                 "tensor_frac": round(fb / (bwd_ms * 1e-3) / 1e12 / peaks["bf16_tflops"], 4)})
    # fwd + bwd; the general backward adds its Delta pass and dQ finalize.
    launches_per_step = 2 if (N <= 256 and D <= 64) else 4
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
        "gpu_launches": launches_per_step * K,
        "clocks": sampler.summary(),
    }


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
    args = ap.parse_args()
    world, rank, local = init_dist()

    if args.impl == "reference":
        if rank == 0:
            tf, sample, cores, ms = cpu_reference_run(args.config, args.steps, args.warmup)
            B, H, side, has_cls, N, D, amp, desc = shape_of(args.config)
            line = {"metric": METRIC, "value": round(tf, 4), "unit": "TFLOP/s", "n_gpus": world,
                    "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
                    "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                    "dtype": "f32", "data": "synthetic (seeded N(0,1))", "impl": "reference",
                    "config": {"workload": f"{args.config}: {desc} fwd+bwd, B={B} H={H} N={N} "
                                           f"D={D} has_cls={has_cls}", "seq_len": N},
                    "cpu_baseline": {"value": round(tf, 4), "unit": "TFLOP/s", "cores": cores,
                                     "kind": "port", "sample": sample},
                    "e2e": {"value": round(tf, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                            "d2h_bytes_per_step": 0}}
            print(json.dumps(line), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return

    line = gpu_arm(args, world, rank, local)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tf, sample, cores, _ = cpu_reference_run(args.config, 3, 1, budget_s=20.0)
        line["cpu_baseline"] = {"value": round(tf, 4), "unit": "TFLOP/s", "cores": cores,
                                "kind": "port", "sample": sample}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
