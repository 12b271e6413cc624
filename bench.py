#!/usr/bin/env python
"""Benchmark of the JoLT / FlashJoLT compress + decompress path on B200.

One step = compress every layer's K and V of a model-shaped KV cache, then
decompress every layer, with the inputs resident in HBM (1 GiB per step for
the default Llama-3-8B / 8k workload: larger than L2, so no flush is
needed).  The headline ``value`` is whole-job compress tokens/s
(batch * T tokens per rank per step); decompress GB/s sits beside it.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  torchrun --nproc-per-node N bench.py --gpus N ...   (one rank per GPU)

With N ranks every rank compresses its own cache (different seeds: data
parallel replicas, weak scaling); the allocation is agreed once over NCCL
(``JointAllocator.optimize_distributed``) and nothing else crosses GPUs.
``--impl reference`` times the CPU restatement of the reference algorithm
(``oracle/``) on the host cores instead, on a one-layer sample.
"""

from __future__ import annotations

import argparse
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
BREAKDOWN_STEPS = 3  # traced steps for the per-stage times, before the timed region
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", default="llama3-8b-kv-b1-t8192-bf16")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-chunk", type=int, default=4, help="layers per compress_many call in the e2e line")
    ap.add_argument("--stream-block", type=int, default=256, help="tokens per block of the decode-stream line (0: no such line)")
    ap.add_argument("--cpu-sample-layers", type=int, default=1)
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


def cpu_baseline(w, sample_layers: int = 1, steps: int = 1, warmup: int = 0):
    """Time the CPU restatement of the reference path (oracle) on host cores."""
    import numpy as np
    from threadpoolctl import threadpool_info

    import oracle
    from kvcompress_b200.compressor.jl import gaussian_projection
    from kvcompress_b200.synthetic import make_kv_layer

    torch.set_num_threads(os.cpu_count() or 1)
    m, t, d = w.cell_shape
    dt = {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}[w.dtype]
    proj = gaussian_projection(d, d, seed=0).matrix.numpy()
    shapes = [w.cell_shape, w.cell_shape]
    alloc = oracle.allocate(shapes, w.compression_ratio, bits_grid=tuple(w.bits))["allocations"][0]
    cap = oracle.flashjolt_cap(t, w.compression_ratio) if w.method == "flashjolt" else None
    mode = "randomised" if w.method == "flashjolt" else "exact"

    def omega_fn(n, k):
        torch.manual_seed(0)
        return torch.randn(n, k).numpy()

    layers = []
    for li in range(sample_layers):
        k_, v_ = make_kv_layer(w, li)
        layers.append((k_.reshape(m, t, d).float().numpy(), v_.reshape(m, t, d).float().numpy()))
    c_times, d_times = [], []
    for it in range(warmup + steps):
        tc = td = 0.0
        for kx, vx in layers:
            for x in (kx, vx):
                t0 = time.perf_counter()
                out = oracle.jolt_compress_cell(x, dt, alloc, proj=proj, svd_mode=mode, cap=cap,
                                                omega_fn=omega_fn)
                t1 = time.perf_counter()
                oracle.jolt_decompress_cell(out["core"].astype(np.float16), out["u_token"].astype(np.float16),
                                            out["u_feature"].astype(np.float16), out["packed"], out["scale"],
                                            out["zero_point"], out["bits"], proj, dt, (m, t, d))
                t2 = time.perf_counter()
                tc += t1 - t0
                td += t2 - t1
        if it >= warmup:
            c_times.append(tc)
            d_times.append(td)
    tc = statistics.median(c_times)
    td = statistics.median(d_times)
    per_layer_c = tc / sample_layers
    per_layer_d = td / sample_layers
    tokens = w.batch * w.tokens
    threads = sum(p.get("num_threads", 0) for p in threadpool_info() if p.get("user_api") == "blas") or 1
    dec_bytes_layer = 2 * (m * t * d * (alloc[2] / 8.0) + m * t * d * torch.tensor([], dtype=w.dtype).element_size())
    return {
        "value": tokens / (per_layer_c * w.layers),
        "unit": "tokens/s",
        "cores": int(threads),
        "kind": "port",
        "sample": f"{sample_layers} of {w.layers} layers (K+V), median of {steps}, extrapolated x{w.layers}",
        "decompress_gbs": dec_bytes_layer / per_layer_d / 1e9,
        "cpu_model": _cpu_model(),
        "compress_s_per_layer": per_layer_c,
        "decompress_s_per_layer": per_layer_d,
    }


def _cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def run_reference(args, w):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    cb = cpu_baseline(w, sample_layers=args.cpu_sample_layers, steps=max(1, args.steps),
                      warmup=max(0, min(args.warmup, 1)))
    line = {
        "impl": "reference", "metric": METRIC, "value": cb["value"], "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * cb["compress_s_per_layer"] * w.layers,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": workload_config(w, args.gpus, None),
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
        "allocation": alloc, "parallelism": f"replicas x{n} (data parallel)",
        "l2": "inputs larger than L2 (no flush)",
    }


PROFILE_SUMMARY = os.path.join(os.path.dirname(os.path.abspath(__file__)), "profiles",
                               "tc_kernels_llama3-8b-8layers.md")


def ncu_traffic(stage: str, cells: int):
    """DRAM bytes (read + write) of one launch of ``stage`` from the committed
    ncu summary (a 16-cell capture), scaled by the cells processed; None when
    the summary has no figure for the stage."""
    try:
        with open(PROFILE_SUMMARY) as f:
            for line in f:
                parts = line.split()
                if len(parts) == 3 and parts[0] == "traffic_per_cell_bytes" and parts[1] == stage:
                    return float(parts[2]) * cells
    except OSError:
        pass
    return None


def run_ours(args, w):
    import torch.distributed as dist

    from kvcompress_b200 import build_compressor, ops
    from kvcompress_b200.compressor.allocator import Cell
    from kvcompress_b200.synthetic import make_kv_layer

    world, rank, local = dist_env()
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    m, t, d = w.cell_shape
    comp = build_compressor(w.method, compression_ratio=w.compression_ratio, bits=w.bits)
    # cache on the device: every layer's K and V, one replica per rank
    pairs = []
    for li in range(w.layers):
        k, v = make_kv_layer(w, li, seed=rank, device=dev)
        pairs.append((k.reshape(m, t, d), v.reshape(m, t, d)))
    local_alloc = comp.allocator.optimize([Cell(shape=(m, t, d)), Cell(shape=(m, t, d))])
    alloc = list(local_alloc.allocations[0].tuple)
    if world > 1:
        glob, _ = comp.allocator.optimize_distributed([Cell(shape=(m, t, d), kind=k) for k in ("key", "value")])
        assert [a.tuple for a in glob.allocations] == [tuple(alloc)] * (2 * world)

    def step():
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record()
        payloads = comp.compress_many(pairs)
        ev[1].record()
        outs = comp.decompress_many(payloads)
        ev[2].record()
        return ev, payloads, outs

    # nvidia-smi starts before the warm-up: its start-up stalls the GPU
    # driver for up to a second and must not land in the timed region
    clocks = ClockSampler(physical_gpu(local))
    clocks.start()
    time.sleep(1.5)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    def by_stage(log):
        out = {}
        for name, e0, e1, _n_launch, nbytes in log:
            s = out.setdefault(name, [0.0, 0, 0])
            s[0] += e0.elapsed_time(e1)
            s[1] += 1
            s[2] += nbytes
        return out

    # the stage breakdown comes from a few traced steps before the timed region:
    # an event pair around every stage costs the stream time (about 0.14 ms a
    # compress for all ten stages), so the timed steps record only the
    # dominant stage (for the roofline) and the decode
    ops.trace_start()
    for _ in range(BREAKDOWN_STEPS):
        step()
    torch.cuda.synchronize()
    breakdown = by_stage(ops.trace_stop())
    dominant_name = max(breakdown.items(), key=lambda kv: kv[1][0])[0]
    if world > 1:
        dist.barrier()
    ops.trace_start(stages={dominant_name, "decompress"})
    launches0 = ops.launch_count()  # the library counts its own kernel launches
    t_all0 = torch.cuda.Event(enable_timing=True)
    t_all1 = torch.cuda.Event(enable_timing=True)
    t_all0.record()
    evs = []
    payloads = outs = None
    for _ in range(args.steps):
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
    log = ops.trace_stop()
    clk = clocks.stop()

    if os.environ.get("KVC_BENCH_VERBOSE"):
        for i, e in enumerate(evs):
            print(f"step {i}: compress {e[0].elapsed_time(e[1]):.3f} ms, decompress {e[1].elapsed_time(e[2]):.3f} ms",
                  file=sys.stderr)
    total_ms = t_all0.elapsed_time(t_all1) / args.steps
    comp_ms = sum(e[0].elapsed_time(e[1]) for e in evs) / args.steps
    dec_ms = sum(e[1].elapsed_time(e[2]) for e in evs) / args.steps
    # payload + output bytes of one decompress pass
    pay_bytes = sum(p.bytes_compressed for pair in payloads for p in pair)
    out_bytes = sum(o.numel() * o.element_size() for pair in outs for o in pair)
    stage = by_stage(log)
    times = torch.tensor([total_ms, comp_ms, dec_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    total_ms, comp_ms, dec_ms = times.tolist()

    peak, peak_kind = peaks()
    dname = dominant_name
    dms, dcalls, dbytes = stage[dname]
    achieved = dbytes / (dms / 1000.0) / 1e9
    dec_stage = stage.get("decompress", [dec_ms * args.steps, args.steps, (pay_bytes + out_bytes) * args.steps])
    dec_gbs_kernel = dec_stage[2] / (dec_stage[0] / 1000.0) / 1e9

    tokens = w.batch * w.tokens
    line = {
        "metric": METRIC,
        "value": world * tokens / (comp_ms / 1000.0),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": total_ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16" if w.dtype == torch.bfloat16 else str(w.dtype).replace("torch.", ""),
        "data": "synthetic",
        "config": workload_config(w, world, alloc),
        "compress_ms_per_step": comp_ms,
        "decompress": {"value": world * (pay_bytes + out_bytes) / (dec_ms / 1000.0) / 1e9, "unit": "GB/s",
                       "ms_per_step": dec_ms, "kernel_gbs": dec_gbs_kernel,
                       "kernel_frac_of_hbm": dec_gbs_kernel / peak},
        "gpu_launches": launches,
        "clocks": clk,
        "roofline": {"bound": "hbm", "kernel": dname, "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_source": peak_kind,
                     "traffic": ncu_traffic(dname, 2 * w.layers), "traffic_unit": "bytes per launch",
                     "algorithmic_bytes": dbytes / dcalls, "launch_ms": dms / dcalls},
        "stages_ms_per_step": {k: v[0] / BREAKDOWN_STEPS for k, v in sorted(breakdown.items())},
        "stages_from": f"{BREAKDOWN_STEPS} traced steps before the timed region (an event pair around every stage)",
    }
    if args.stream_block > 0:
        line["decode_stream"] = decode_stream(payloads, world, dev, block=args.stream_block)
    if not args.no_e2e:
        line["e2e"] = e2e(comp, pairs, w, dev, world, steps=min(args.steps, 3), chunk=args.e2e_chunk)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = cpu_baseline(w, sample_layers=args.cpu_sample_layers)
        line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


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
    out_bytes = sum(p.shape[0] * p.shape[1] * p.shape[2] * 2 for pair in payloads for p in pair)
    code_bytes = sum(p.data["residual_packed"].numel() for pair in payloads for p in pair)
    return {"block_tokens": block, "blocks_per_pass": n_blocks, "planned": stream.planned,
            "ms_per_pass": ms, "us_per_block": 1000.0 * ms / n_blocks,
            "value": world * (out_bytes + code_bytes) / (ms / 1000.0) / 1e9, "unit": "GB/s",
            "graph": {"ms_per_pass": gms, "us_per_block": 1000.0 * gms / n_blocks,
                      "value": world * (out_bytes + code_bytes) / (gms / 1000.0) / 1e9, "unit": "GB/s"},
            "what": "all layers' K and V, tokens [t0, t0 + block) per launch pair, through DecodeStream; "
                    "graph: the same blocks as one CUDA graph (DecodeStream.capture)"}


def e2e(comp, pairs, w, dev, world, steps: int = 2, chunk: int = 4):
    """Compress from pinned host buffers through the public batched API
    (``compress_many`` over ``chunk`` layers at a time); the H2D copies of the
    inputs and the D2H copies of every payload tensor are inside the timed
    region.

    Copies overlap the compression the way an offload loop would run it: the
    H2D of chunk i + 1 (copy stream) is queued before chunk i is compressed
    (current stream), and chunk i's payloads go back on a third stream while
    chunk i + 1 compresses.  Two device input slots per chunk."""
    import torch.distributed as dist

    host = [(k.cpu().pin_memory(), v.cpu().pin_memory()) for k, v in pairs]
    h2d = sum(k.numel() * k.element_size() * 2 for k, _ in host)
    chunks = [list(range(i, min(i + chunk, len(host)))) for i in range(0, len(host), chunk)]
    slots = [[(torch.empty_like(pairs[0][0]), torch.empty_like(pairs[0][1])) for _ in range(chunk)] for _ in range(2)]
    pinned_out: list[torch.Tensor] = []
    comp_stream = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    n = len(chunks)

    def once():
        slot = 0
        loaded = [torch.cuda.Event() for _ in range(n)]
        used = [torch.cuda.Event() for _ in range(n)]

        def upload(i):
            if i >= 2:
                up.wait_event(used[i - 2])  # the slot's previous chunk has been compressed
            with torch.cuda.stream(up):
                for j, li in enumerate(chunks[i]):
                    kd, vd = slots[i % 2][j]
                    kd.copy_(host[li][0], non_blocking=True)
                    vd.copy_(host[li][1], non_blocking=True)
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
                for b in bases.values():
                    if slot == len(pinned_out):
                        pinned_out.append(torch.empty(b.shape, dtype=b.dtype, pin_memory=True))
                    pinned_out[slot].copy_(b, non_blocking=True)
                    b.record_stream(down)
                    slot += 1
        comp_stream.wait_stream(down)
        comp_stream.wait_stream(up)
        return pinned_out[:slot]

    once()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    d2h = 0
    for _ in range(steps):
        outs = once()
        d2h = sum(o.numel() * o.element_size() for o in outs)
    e1.record()
    torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    return {"value": world * w.batch * w.tokens / (ms / 1000.0), "unit": "tokens/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": ms,
            "h2d_gbs": h2d / (ms / 1000.0) / 1e9,
            "api": (("FlashJoLTCompressor" if w.method == "flashjolt" else "JoLTCompressor")
                    + f".compress_many over {chunk} layers at a time; H2D / compress / D2H overlapped on three streams")}


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
