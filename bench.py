#!/usr/bin/env python
"""Benchmark of the JoLT / FlashJoLT compress + decompress path on B200.

One step = compress every layer's K and V of a model-shaped KV cache, then
decompress every layer, with the inputs resident in HBM.  The default cache
is the Llama-3-8B-shaped batch 8 x 32k bf16 cache (64 cells of 512 MiB:
32 GiB per step, far larger than L2, so no flush is needed) compressed with
FlashJoLT 4x.  The headline ``value`` is whole-cache compress tokens/s
(batch * T tokens per step); decompress GB/s sits beside it.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  torchrun --nproc-per-node N bench.py --gpus N ...   (one rank per GPU)

With N ranks the cache's (layer, K|V) cells are split across the ranks
(rank r holds layers [r L / N, (r + 1) L / N)): strong scaling of one cache.
The allocation is agreed once over NCCL (``JointAllocator.optimize_distributed``
all-gathers the per-cell tables) and nothing else crosses GPUs; times are the
maximum over ranks.  At N = 1 the line also carries the single-B200 config
(Llama-3-8B, one 8k sequence) under ``single_gpu_config``.

``--impl reference`` times the reference kvcompress itself (its torch CPU
path, installed under ``baseline/_ref``) on the host cores, one layer of the
workload per step.
"""

from __future__ import annotations

import argparse
import gc
import dataclasses
import json
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "compress tokens/s + decompress GB/s (Llama-3-8B KV shape) at 1/2/4/8 B200, %roofline"
DEFAULT_WORKLOAD = "llama3-8b-kv-b8-t32768-bf16"
SINGLE_GPU_WORKLOAD = "llama3-8b-kv-b1-t8192-bf16"
STREAM_WORKLOAD = "qwen2-7b-kv-b4-t131072-bf16"
QCAP_WORKLOAD = "llama3-8b-kv-b8-t4096-bf16-qcap"
FP32_WORKLOAD = "tinyllama-1.1b-kv-t2048-fp32"
BREAKDOWN_STEPS = 3  # traced steps for the per-stage times, before the timed region
FALLBACK_HBM_GBS = 6650.0
REFERENCE_DIR = os.path.join(ROOT, "baseline", "_ref")
REFERENCE_BUDGET_S = 100.0  # CPU seconds the reference arm's timed steps may take


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD)
    ap.add_argument("--single-gpu-workload", default=SINGLE_GPU_WORKLOAD,
                    help="the single-B200 config measured beside the headline at N = 1 ('' to skip)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-chunk", type=int, default=4, help="layers per compress_many call in the e2e line")
    ap.add_argument("--e2e-host-layers", type=int, default=8,
                    help="distinct layers held in pinned host memory for the e2e line (reused cyclically)")
    ap.add_argument("--stream-block", type=int, default=256, help="tokens per block of the decode-stream line (0: no such line)")
    ap.add_argument("--qcap-workload", default=QCAP_WORKLOAD,
                    help="the q-capped sketch config measured at N = 1 ('' to skip)")
    ap.add_argument("--fp32-workload", default=FP32_WORKLOAD,
                    help="the fp32, head-dim 64 config measured at N = 1 ('' to skip)")
    ap.add_argument("--stream-workload", default=STREAM_WORKLOAD,
                    help="the decode-stream config measured at N = 1, with the int4 / fp8 baselines ('' to skip)")
    ap.add_argument("--layers", type=int, default=0,
                    help="override the workload's layer count (profiling a smaller case)")
    return ap.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9 or not f[0].isdigit() or int(f[0]) != self.gpu:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def physical_gpu(local: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        try:
            return int(vis.split(",")[local])
        except (ValueError, IndexError):
            return local
    return local


def my_layers(n_layers: int, world: int, rank: int) -> list[int]:
    """The contiguous block of layers (both K and V cells) rank ``rank`` compresses."""
    return list(range(rank * n_layers // world, (rank + 1) * n_layers // world))


def _cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


# ----------------------------------------------------------------- CPU legs


def _import_reference():
    """The reference kvcompress package installed under ``baseline/_ref``, or None."""
    if not os.path.isdir(os.path.join(REFERENCE_DIR, "kvcompress")):
        return None
    if REFERENCE_DIR not in sys.path:
        sys.path.insert(0, REFERENCE_DIR)
    try:
        import kvcompress  # noqa: F401
        from kvcompress import build_compressor
    except Exception:
        return None
    return build_compressor


def reference_cpu(w, *, steps: int = 1, budget_s: float | None = None, batch: int | None = None):
    """The reference's own CPU path (``build_compressor(method).compress`` /
    ``.decompress``, torch on all host cores) on one layer of the workload per
    step; compress tokens/s extrapolated to every layer.

    ``batch`` < the workload's batch times a slice of the layer (its first
    ``batch`` sequences, every head and token) and scales the time by the
    rows, for a bounded sample of a large cache; the reference's cost grows a
    little faster than its rows, so the slice overstates its speed."""
    build = _import_reference()
    if build is None:
        return None
    threads0 = torch.get_num_threads()
    torch.set_num_threads(os.cpu_count() or 1)
    try:
        return _reference_cpu_run(build, w, steps=steps, budget_s=budget_s, batch=batch)
    finally:
        # the GPU lines measured after this one run with the process's own setting
        torch.set_num_threads(threads0)


def _reference_cpu_run(build, w, *, steps, budget_s, batch):
    from kvcompress_b200.synthetic import make_kv_layer

    full_m = w.cell_shape[0]
    if batch is not None and batch < w.batch:
        w = dataclasses.replace(w, batch=int(batch))
    scale = full_m / w.cell_shape[0]
    m, t, d = w.cell_shape
    comp = build(w.method, compression_ratio=w.compression_ratio, bits=tuple(w.bits))
    # warm the library paths on a small input (first-call costs are not the workload's)
    sk, sv = make_kv_layer(w, 0, tokens=256, batch=1)
    comp.compress(sk.reshape(-1, 256, d), sv.reshape(-1, 256, d))
    c_times, d_times = [], []
    alloc = None
    spent = 0.0
    # one layer, generated once: every layer costs the same
    k, v = make_kv_layer(w, 0)
    k, v = k.reshape(m, t, d), v.reshape(m, t, d)
    for _ in range(max(1, steps)):
        t0 = time.perf_counter()
        kp, vp = comp.compress(k, v)
        t1 = time.perf_counter()
        comp.decompress(kp, vp)
        t2 = time.perf_counter()
        c_times.append(t1 - t0)
        d_times.append(t2 - t1)
        alloc = [int(kp.metadata["r_token"]), int(kp.metadata["r_feature"]), int(kp.metadata["bits"])]
        spent += t2 - t0
        if budget_s is not None and spent + (t2 - t0) > budget_s:
            break
    per_c, per_d = statistics.median(c_times) * scale, statistics.median(d_times) * scale
    el = torch.tensor([], dtype=w.dtype).element_size()
    dec_bytes_layer = 2 * (m * t * d * (alloc[2] / 8.0) + m * t * d * el) * scale
    what = ("one layer (K+V)" if scale == 1 else
            f"a slice of one layer (K+V), {w.batch} of {int(round(w.batch * scale))} sequences, time x{scale:g},")
    return {
        "value": w.batch * scale * w.tokens / (per_c * w.layers), "unit": "tokens/s",
        "cores": int(torch.get_num_threads()), "kind": "reference",
        "sample": (f"{what} of {w.layers} per step, median of {len(c_times)}, extrapolated x{w.layers}; "
                   f"kvcompress {w.method} compress + decompress on CPU torch from baseline/_ref"),
        "decompress_gbs": dec_bytes_layer / per_d / 1e9, "cpu_model": _cpu_model(),
        "compress_s_per_layer": per_c, "decompress_s_per_layer": per_d, "steps_timed": len(c_times),
        "allocation": alloc,
    }


def port_cpu(w, steps: int = 1):
    """The numpy restatement of the reference algorithm (``oracle/``) on host
    cores, one layer; a second CPU figure beside the reference's own."""
    import numpy as np
    from threadpoolctl import threadpool_info

    import oracle
    from kvcompress_b200.compressor.jl import gaussian_projection
    from kvcompress_b200.synthetic import make_kv_layer

    m, t, d = w.cell_shape
    dt = {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}[w.dtype]
    proj = gaussian_projection(d, d, seed=0).matrix.numpy()
    alloc = oracle.allocate([w.cell_shape, w.cell_shape], w.compression_ratio,
                            bits_grid=tuple(w.bits))["allocations"][0]
    cap = oracle.flashjolt_cap(t, w.compression_ratio) if w.method == "flashjolt" else None
    mode = "randomised" if w.method == "flashjolt" else "exact"

    def omega_fn(n, k):
        torch.manual_seed(0)
        return torch.randn(n, k).numpy()

    k_, v_ = make_kv_layer(w, 0)
    layer = (k_.reshape(m, t, d).float().numpy(), v_.reshape(m, t, d).float().numpy())
    times = []
    for _ in range(max(1, steps)):
        tc = 0.0
        for x in layer:
            t0 = time.perf_counter()
            oracle.jolt_compress_cell(x, dt, alloc, proj=proj, svd_mode=mode, cap=cap, omega_fn=omega_fn)
            tc += time.perf_counter() - t0
        times.append(tc)
    per_c = statistics.median(times)
    threads = sum(p.get("num_threads", 0) for p in threadpool_info() if p.get("user_api") == "blas") or 1
    return {"value": w.batch * w.tokens / (per_c * w.layers), "unit": "tokens/s", "cores": int(threads),
            "kind": "port", "sample": f"one layer (K+V) of {w.layers}, median of {len(times)}, extrapolated "
                                      f"x{w.layers}; numpy restatement (oracle/)"}


def run_reference(args, w):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    cb = reference_cpu(w, steps=max(1, args.steps), budget_s=REFERENCE_BUDGET_S)
    if cb is None:
        # the reference package is not installed: its numpy restatement stands in
        pc = port_cpu(w, steps=1)
        cb = dict(pc, decompress_gbs=None, compress_s_per_layer=w.batch * w.tokens / pc["value"] / w.layers,
                  allocation=None)
    line = {
        "impl": "reference", "metric": METRIC, "value": cb["value"], "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * cb["compress_s_per_layer"] * w.layers,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": workload_config(w, args.gpus, cb["allocation"]),
        "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "decompress": {"value": cb["decompress_gbs"], "unit": "GB/s"},
        "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(w, n, alloc):
    return {
        "workload": w.name, "layers": w.layers, "batch": w.batch, "n_kv_heads": w.n_kv,
        "head_dim": w.head_dim, "seq_len": w.tokens, "kv_dtype": str(w.dtype).replace("torch.", ""),
        "method": w.method, "compression_ratio": w.compression_ratio, "bits": list(w.bits),
        "allocation": alloc,
        "parallelism": f"cells sharded over {n} rank(s): contiguous blocks of {w.layers // max(n, 1)} layers "
                       f"(K and V) per rank",
        "l2": "inputs larger than L2 (no flush)",
    }


# ----------------------------------------------------------------- GPU legs

PROFILE_SUMMARY = os.path.join(ROOT, "profiles", "tc_encode_llama3-8b-b8-t32768-1layer.md")


def ncu_traffic(stage: str, cells: int, rows_per_cell: int):
    """DRAM bytes (read + write) of one launch of ``stage`` from the committed
    ncu summary (bytes per row of a captured launch), scaled by the rows the
    launch processes; None when the summary has no figure for the stage."""
    try:
        with open(PROFILE_SUMMARY) as f:
            for line in f:
                parts = line.split()
                if len(parts) == 3 and parts[0] == "traffic_per_row_bytes" and parts[1] == stage:
                    return float(parts[2]) * cells * rows_per_cell
    except OSError:
        pass
    return None


def _by_stage(log):
    out = {}
    for name, e0, e1, _n_launch, nbytes in log:
        s = out.setdefault(name, [0.0, 0, 0])
        s[0] += e0.elapsed_time(e1)
        s[1] += 1
        s[2] += nbytes
    return out


def measure(comp, pairs, w, *, steps: int, warmup: int, world: int, dev, peak: float):
    """Device-timed compress_many + decompress_many steps over this rank's
    layers; times are the maximum over ranks."""
    import torch.distributed as dist

    from kvcompress_b200 import ops

    def step():
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record()
        payloads = comp.compress_many(pairs)
        ev[1].record()
        outs = comp.decompress_many(payloads)
        ev[2].record()
        return ev, payloads, outs

    # garbage from the lines measured before (payload dicts, traces, the CPU
    # legs' objects) is collected here, not inside this line's timed steps
    gc.collect()
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    # the stage breakdown comes from a few traced steps before the timed region:
    # an event pair around every stage costs the stream time (about 0.14 ms a
    # compress for all ten stages), so the timed steps record only the
    # dominant stage (for the roofline) and the decode
    ops.trace_start()
    for _ in range(BREAKDOWN_STEPS):
        step()
    torch.cuda.synchronize()
    breakdown = _by_stage(ops.trace_stop())
    dominant = max(breakdown.items(), key=lambda kv: kv[1][0])[0]
    stage_bytes = sum(v[2] for k, v in breakdown.items() if k not in ("decompress",)) / BREAKDOWN_STEPS
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ops.trace_start(stages={dominant, "decompress"})
    launches0 = ops.launch_count()  # the library counts its own kernel launches
    t_all0 = torch.cuda.Event(enable_timing=True)
    t_all1 = torch.cuda.Event(enable_timing=True)
    t_all0.record()
    evs = []
    payloads = outs = None
    for _ in range(steps):
        # release the previous step's payloads first, as the warm-up does, so
        # the caching allocator reuses its blocks instead of calling cudaMalloc
        payloads = outs = None
        ev, payloads, outs = step()
        evs.append(ev)
    t_all1.record()
    launches = ops.launch_count() - launches0
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    stage = _by_stage(ops.trace_stop())
    total_ms = t_all0.elapsed_time(t_all1) / steps
    comp_ms = sum(e[0].elapsed_time(e[1]) for e in evs) / steps
    dec_ms = sum(e[1].elapsed_time(e[2]) for e in evs) / steps
    pay_bytes = sum(p.bytes_compressed for pair in payloads for p in pair)
    out_bytes = sum(o.numel() * o.element_size() for pair in outs for o in pair)
    dms, dcalls, dbytes = stage[dominant]
    dec_stage = stage.get("decompress", [dec_ms * steps, steps, (pay_bytes + out_bytes) * steps])
    vals = torch.tensor([total_ms, comp_ms, dec_ms, dms / dcalls, dec_stage[0] / dec_stage[1]], dtype=torch.float64,
                        device=dev)
    sums = torch.tensor([pay_bytes + out_bytes, stage_bytes, dbytes / dcalls, dec_stage[2] / dec_stage[1],
                         float(launches)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
        dist.all_reduce(sums, op=dist.ReduceOp.SUM)
    total_ms, comp_ms, dec_ms, dom_ms, dec_kernel_ms = vals.tolist()
    dec_bytes_all, stage_bytes_all, dom_bytes_all, dec_kernel_bytes_all, launches_all = sums.tolist()
    # per-rank roofline of the dominant kernel (algorithmic bytes of this rank's
    # launch over the slowest rank's launch time)
    dom_achieved = dom_bytes_all / world / (dom_ms / 1000.0) / 1e9
    dec_kernel_gbs = dec_kernel_bytes_all / world / (dec_kernel_ms / 1000.0) / 1e9
    stagewise_gbs = stage_bytes_all / (comp_ms / 1000.0) / 1e9
    return {
        "payloads": payloads, "outs": outs, "total_ms": total_ms, "comp_ms": comp_ms, "dec_ms": dec_ms,
        "dec_gbs": dec_bytes_all / (dec_ms / 1000.0) / 1e9, "dec_kernel_gbs": dec_kernel_gbs,
        "launches": int(launches_all), "dominant": dominant, "dom_ms": dom_ms, "dom_bytes": dom_bytes_all / world,
        "dom_achieved": dom_achieved, "breakdown": {k: v[0] / BREAKDOWN_STEPS for k, v in sorted(breakdown.items())},
        "stagewise": {"bytes_per_step": stage_bytes_all, "achieved_gbs": stagewise_gbs,
                      "frac": stagewise_gbs / (world * peak),
                      "what": "algorithmic HBM bytes of every compress stage (4 reads of x, codes, x_proj) over "
                              "the compress time, against N x the measured copy peak"},
    }


def run_ours(args, w):
    import torch.distributed as dist

    from kvcompress_b200 import build_compressor
    from kvcompress_b200.compressor.allocator import Cell
    from kvcompress_b200.synthetic import WORKLOADS, make_kv_layer

    world, rank, local = dist_env()
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    peak, peak_kind = peaks()

    m, t, d = w.cell_shape
    layers = my_layers(w.layers, world, rank)
    comp = build_compressor(w.method, compression_ratio=w.compression_ratio, bits=w.bits)
    # this rank's share of the one cache: its layers' K and V, on the device
    pairs = []
    for li in layers:
        k, v = make_kv_layer(w, li, device=dev)
        pairs.append((k.reshape(m, t, d), v.reshape(m, t, d)))
    local_alloc = comp.allocator.optimize([Cell(shape=(m, t, d)), Cell(shape=(m, t, d))])
    alloc = list(local_alloc.allocations[0].tuple)
    if world > 1:
        # the allocation agreed over all ranks' cells (one all-gather of the
        # per-cell tables) equals the per-layer allocation every rank uses
        cells = [Cell(shape=(m, t, d), kind=kind) for _ in layers for kind in ("key", "value")]
        glob, mine = comp.allocator.optimize_distributed(cells)
        assert len(glob.allocations) == 2 * w.layers
        assert [a.tuple for a in glob.allocations] == [tuple(alloc)] * (2 * w.layers)

    # nvidia-smi starts before the warm-up: its start-up stalls the GPU
    # driver for up to a second and must not land in the timed region
    clocks = ClockSampler(physical_gpu(local))
    clocks.start()
    time.sleep(1.5)
    r = measure(comp, pairs, w, steps=args.steps, warmup=args.warmup, world=world, dev=dev, peak=peak)
    clk = clocks.stop()

    tokens = w.batch * w.tokens
    dname = r["dominant"]
    rows_per_cell = m * t
    line = {
        "metric": METRIC,
        "value": tokens / (r["comp_ms"] / 1000.0),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": r["total_ms"],
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16" if w.dtype == torch.bfloat16 else str(w.dtype).replace("torch.", ""),
        "data": "synthetic",
        "config": workload_config(w, world, alloc),
        "compress_ms_per_step": r["comp_ms"],
        "compress_stagewise": r["stagewise"],
        "decompress": {"value": r["dec_gbs"], "unit": "GB/s", "ms_per_step": r["dec_ms"],
                       "kernel_gbs": r["dec_kernel_gbs"], "kernel_frac_of_hbm": r["dec_kernel_gbs"] / peak},
        "gpu_launches": r["launches"],
        "clocks": clk,
        "roofline": {"bound": "hbm", "kernel": dname, "achieved": r["dom_achieved"], "peak": peak, "unit": "GB/s",
                     "frac": r["dom_achieved"] / peak, "peak_source": peak_kind,
                     "traffic": ncu_traffic(dname, 2 * len(layers), rows_per_cell),
                     "traffic_unit": "bytes per launch", "algorithmic_bytes": r["dom_bytes"],
                     "launch_ms": r["dom_ms"]},
        "stages_ms_per_step": r["breakdown"],
        "stages_from": f"{BREAKDOWN_STEPS} traced steps before the timed region (an event pair around every stage)",
    }
    payloads = r["payloads"]
    if args.stream_block > 0:
        line["decode_stream"] = decode_stream(payloads, world, dev, block=args.stream_block)
    del r
    if not args.no_e2e:
        line["e2e"] = e2e(comp, pairs, w, dev, world, steps=min(args.steps, 3), chunk=args.e2e_chunk,
                          host_layers=args.e2e_host_layers)
    del payloads
    # the GPU-only lines first, then the single-B200 config with its CPU legs
    if world == 1 and args.qcap_workload:
        pairs = None
        torch.cuda.empty_cache()
        line["qcap_config"] = single_gpu(WORKLOADS[args.qcap_workload], args, dev, peak, cpu=False)
    if world == 1 and args.fp32_workload:
        pairs = None
        torch.cuda.empty_cache()
        line["fp32_config"] = single_gpu(WORKLOADS[args.fp32_workload], args, dev, peak, cpu=False)
    if world == 1 and args.single_gpu_workload and args.single_gpu_workload != w.name:
        pairs = None
        torch.cuda.empty_cache()
        line["single_gpu_config"] = single_gpu(WORKLOADS[args.single_gpu_workload], args, dev, peak,
                                               cpu=not args.no_cpu_baseline)
    if world == 1 and args.stream_workload and args.stream_block > 0:
        pairs = None
        torch.cuda.empty_cache()
        line["decode_stream_config"] = stream_config(WORKLOADS[args.stream_workload], dev, peak, args.stream_block)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # a bounded sample: one sequence's slice of a layer when the layer is large
        cb = reference_cpu(w, steps=1, batch=1 if w.batch > 1 else None)
        if cb is not None:
            line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
            line["cpu_baseline"]["decompress_gbs"] = cb["decompress_gbs"]
        else:
            line["cpu_baseline"] = port_cpu(w, steps=1)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def single_gpu(w, args, dev, peak, cpu: bool):
    """The single-B200 config (one Llama-3-8B 8k sequence, every layer on this
    GPU): compress / decompress times, its dominant kernel's roofline and the
    CPU figures (reference and numpy restatement) on the same layer shape."""
    from kvcompress_b200 import build_compressor
    from kvcompress_b200.synthetic import make_kv_layer

    m, t, d = w.cell_shape
    comp = build_compressor(w.method, compression_ratio=w.compression_ratio, bits=w.bits)
    pairs = []
    for li in range(w.layers):
        k, v = make_kv_layer(w, li, device=dev)
        pairs.append((k.reshape(m, t, d), v.reshape(m, t, d)))
    r = measure(comp, pairs, w, steps=max(args.steps, 10), warmup=args.warmup, world=1, dev=dev, peak=peak)
    out = {
        "workload": w.name, "config": workload_config(w, 1, list(r["payloads"][0][0].metadata[k]
                                                                   for k in ("r_token", "r_feature", "bits"))),
        "value": w.batch * w.tokens / (r["comp_ms"] / 1000.0), "unit": "tokens/s",
        "compress_ms_per_step": r["comp_ms"], "ms_per_step": r["total_ms"],
        "compress_stagewise": r["stagewise"],
        "decompress": {"value": r["dec_gbs"], "unit": "GB/s", "ms_per_step": r["dec_ms"],
                       "kernel_gbs": r["dec_kernel_gbs"], "kernel_frac_of_hbm": r["dec_kernel_gbs"] / peak},
        "roofline": {"kernel": r["dominant"], "achieved": r["dom_achieved"], "peak": peak,
                     "frac": r["dom_achieved"] / peak, "unit": "GB/s", "launch_ms": r["dom_ms"],
                     "algorithmic_bytes": r["dom_bytes"],
                     "traffic": ncu_traffic(r["dominant"], 2 * w.layers, m * t)},
        "stages_ms_per_step": r["breakdown"], "gpu_launches": r["launches"],
    }
    del r
    if cpu:
        cb = reference_cpu(w, steps=3)
        if cb is not None:
            out["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
        out["cpu_port"] = port_cpu(w, steps=1)
    return out


def _timed(fn, reps: int = 3):
    """Device time (ms) of fn() on the current stream: one untimed call, then
    the mean of ``reps``."""
    out = fn()
    torch.cuda.synchronize()
    del out
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        out = fn()
        del out
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def stream_config(w, dev, peak, block: int):
    """The decode-time config: the cache compressed once with FlashJoLT, then
    reconstructed in ``block``-token blocks through DecodeStream (eager and as
    one CUDA graph), next to a whole-cache decode and the int4 per-channel and
    fp8 quantise-only baselines (quantization_only.py:125-198, identity.py:
    68-89) compressing and decoding the same tensors."""
    from kvcompress_b200 import build_compressor
    from kvcompress_b200.synthetic import make_kv_layer

    m, t, d = w.cell_shape
    comp = build_compressor(w.method, compression_ratio=w.compression_ratio, bits=w.bits)
    pairs = []
    for li in range(w.layers):
        k, v = make_kv_layer(w, li, device=dev)
        pairs.append((k.reshape(m, t, d), v.reshape(m, t, d)))
    in_bytes = sum(x.numel() * x.element_size() for pair in pairs for x in pair)
    comp_ms = _timed(lambda: comp.compress_many(pairs), reps=2)
    payloads = comp.compress_many(pairs)
    pay_bytes = sum(p.bytes_compressed for pair in payloads for p in pair)
    out = {"workload": w.name, "config": workload_config(w, 1, [payloads[0][0].metadata[k]
                                                               for k in ("r_token", "r_feature", "bits")]),
           "cache_bytes": in_bytes, "compress_ms": comp_ms,
           "compress_tokens_per_s": w.batch * w.tokens / (comp_ms / 1000.0)}
    out["stream"] = decode_stream(payloads, 1, dev, block=block, passes=2)
    out["stream"]["graph"]["frac_of_hbm"] = out["stream"]["graph"]["value"] / peak
    dec_ms = _timed(lambda: comp.decompress_many(payloads), reps=2)
    out["full_decode"] = {"ms": dec_ms, "value": (pay_bytes + in_bytes) / (dec_ms / 1000.0) / 1e9, "unit": "GB/s",
                          "frac_of_hbm": (pay_bytes + in_bytes) / (dec_ms / 1000.0) / 1e9 / peak}
    del payloads
    base = {}
    for name in ("int4", "fp8"):
        bc = build_compressor(name)
        c_ms = _timed(lambda: [bc.compress(k_, v_) for k_, v_ in pairs], reps=2)
        pays = [bc.compress(k_, v_) for k_, v_ in pairs]
        pb = sum(p.bytes_compressed for pair in pays for p in pair)
        d_ms = _timed(lambda: [bc.decompress(kp, vp) for kp, vp in pays], reps=2)
        base[name] = {"compress_ms": c_ms, "compress_gbs": (in_bytes + pb) / (c_ms / 1000.0) / 1e9,
                      "decompress_ms": d_ms, "decompress_gbs": (in_bytes + pb) / (d_ms / 1000.0) / 1e9,
                      "decompress_frac_of_hbm": (in_bytes + pb) / (d_ms / 1000.0) / 1e9 / peak,
                      "ratio_vs_16bit": in_bytes / pb,
                      "per_block_us": 1000.0 * d_ms / ((t + block - 1) // block)}
        del pays
    out["baselines"] = base
    out["what"] = ("FlashJoLT payloads decoded block by block (DecodeStream; graph = one CUDA graph over every block) "
                   "and whole; int4 per-channel / fp8 baselines compress and decode every layer's K and V "
                   "(per_block_us: their whole decode divided by the blocks of the stream)")
    return out


def decode_stream(payloads, world, dev, block: int = 256, passes: int = 3):
    """Every layer's K and V decoded in consecutive blocks of ``block``
    tokens through ``DecodeStream`` (plan made once, one launch per block and group):
    the per-block cost a blockwise consumer pays, device-timed."""
    import torch.distributed as dist

    from kvcompress_b200 import DecodeStream

    stream = DecodeStream(payloads)
    tokens = stream.tokens
    n_blocks = (tokens + block - 1) // block
    for t0, t1, _ in stream.blocks(block):  # warm-up pass
        pass
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(passes):
        for t0, t1, _ in stream.blocks(block):
            pass
    e1.record()
    torch.cuda.synchronize()
    # the same blocks recorded once as a CUDA graph and replayed
    cap = stream.capture(block)
    cap.replay()
    torch.cuda.synchronize()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record()
    for _ in range(passes):
        cap.replay()
    g1.record()
    torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1) / passes, g0.elapsed_time(g1) / passes], dtype=torch.float64,
                      device=dev)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms, gms = (float(v) for v in ms.tolist())
    del cap
    nbytes = torch.tensor([sum(p.shape[0] * p.shape[1] * p.shape[2] * 2 for pair in payloads for p in pair)
                           + sum(p.data["residual_packed"].numel() for pair in payloads for p in pair)],
                          dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(nbytes)
    nbytes = float(nbytes.item())
    return {"block_tokens": block, "blocks_per_pass": n_blocks, "planned": stream.planned,
            "ms_per_pass": ms, "us_per_block": 1000.0 * ms / n_blocks,
            "value": nbytes / (ms / 1000.0) / 1e9, "unit": "GB/s",
            "graph": {"ms_per_pass": gms, "us_per_block": 1000.0 * gms / n_blocks,
                      "value": nbytes / (gms / 1000.0) / 1e9, "unit": "GB/s"},
            "what": "every layer's K and V of this rank, tokens [t0, t0 + block) per launch pair, through "
                    "DecodeStream; graph: the same blocks as one CUDA graph (DecodeStream.capture)"}


def e2e(comp, pairs, w, dev, world, steps: int = 2, chunk: int = 4, host_layers: int = 8):
    """Compress from pinned host buffers through the public batched API
    (``compress_many`` over ``chunk`` layers at a time); the H2D copies of the
    inputs and the D2H copies of every payload tensor are inside the timed
    region.

    Pinned host memory holds ``host_layers`` distinct layers of this rank
    (all of them when fewer), and layer i of a step is uploaded from host
    slot i mod host_layers: every step moves the bytes of every layer (the
    compress cost does not depend on the values).  Copies overlap the
    compression the way an offload loop would run it: the H2D of chunk i + 1
    (copy stream) is queued before chunk i is compressed (current stream),
    and chunk i's payloads go back on a third stream into one pinned chunk
    buffer while chunk i + 1 compresses.  Two device input slots per chunk."""
    import torch.distributed as dist

    n_layers = len(pairs)
    nh = max(1, min(host_layers, n_layers))
    host = [(pairs[i][0].cpu().pin_memory(), pairs[i][1].cpu().pin_memory()) for i in range(nh)]
    layer_bytes = host[0][0].numel() * host[0][0].element_size() * 2
    h2d = layer_bytes * n_layers
    chunks = [list(range(i, min(i + chunk, n_layers))) for i in range(0, n_layers, chunk)]
    slots = [[(torch.empty_like(pairs[0][0]), torch.empty_like(pairs[0][1])) for _ in range(chunk)] for _ in range(2)]
    pinned_out: list[torch.Tensor] = []  # one chunk's payload tensors (reused by every chunk)
    comp_stream = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    n = len(chunks)

    def once():
        moved = 0
        loaded = [torch.cuda.Event() for _ in range(n)]
        used = [torch.cuda.Event() for _ in range(n)]

        def upload(i):
            if i >= 2:
                up.wait_event(used[i - 2])  # the slot's previous chunk has been compressed
            with torch.cuda.stream(up):
                for j, li in enumerate(chunks[i]):
                    kd, vd = slots[i % 2][j]
                    kd.copy_(host[li % nh][0], non_blocking=True)
                    vd.copy_(host[li % nh][1], non_blocking=True)
                loaded[i].record(up)

        up.wait_stream(comp_stream)  # the previous step is done with both slots
        upload(0)
        for i in range(n):
            if i + 1 < n:
                upload(i + 1)
            comp_stream.wait_event(loaded[i])
            pays = comp.compress_many(slots[i % 2][:len(chunks[i])])
            used[i].record(comp_stream)
            down.wait_event(used[i])
            with torch.cuda.stream(down):
                # every device tensor of the chunk's payloads, copied once per
                # allocation they are views of
                bases = {}
                for pair in pays:
                    for p in pair:
                        for t_ in p.data.values():
                            if t_.is_cuda:
                                b = t_._base if t_._base is not None else t_
                                bases.setdefault(b.data_ptr(), b)
                for slot, b in enumerate(bases.values()):
                    if slot == len(pinned_out):
                        pinned_out.append(torch.empty(b.numel() * b.element_size(), dtype=torch.uint8,
                                                      pin_memory=True))
                    dst = pinned_out[slot]
                    if dst.numel() < b.numel() * b.element_size():
                        dst = pinned_out[slot] = torch.empty(b.numel() * b.element_size(), dtype=torch.uint8,
                                                             pin_memory=True)
                    dst[:b.numel() * b.element_size()].view(b.dtype).view(b.shape).copy_(b, non_blocking=True)
                    b.record_stream(down)
                    moved += b.numel() * b.element_size()
        comp_stream.wait_stream(down)
        comp_stream.wait_stream(up)
        return moved

    once()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    d2h = 0
    for _ in range(steps):
        d2h = once()
    e1.record()
    torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device=dev)
    tot = torch.tensor([float(h2d), float(d2h)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        dist.all_reduce(tot)
    ms = float(ms.item())
    h2d_all, d2h_all = (int(v) for v in tot.tolist())
    return {"value": w.batch * w.tokens / (ms / 1000.0), "unit": "tokens/s",
            "h2d_bytes_per_step": h2d_all, "d2h_bytes_per_step": d2h_all, "ms_per_step": ms,
            "h2d_gbs": h2d_all / (ms / 1000.0) / 1e9,
            "api": (("FlashJoLTCompressor" if w.method == "flashjolt" else "JoLTCompressor")
                    + f".compress_many over {chunk} layers at a time; H2D / compress / D2H overlapped on three "
                      f"streams; pinned host memory holds {nh} distinct layers per rank, reused cyclically")}


def main():
    args = parse_args()
    from kvcompress_b200.synthetic import WORKLOADS

    w = WORKLOADS[args.workload]
    if args.layers:
        w = dataclasses.replace(w, layers=args.layers)
    if args.impl == "reference":
        run_reference(args, w)
    else:
        run_ours(args, w)


if __name__ == "__main__":
    main()
