#!/usr/bin/env python
"""Benchmark of the fused decomposed-rel-pos attention on B200 ("config 4").

One step = one pass of SAM ViT-H's encoder attention over a batch of synthetic inputs resident in HBM:
32 layers in encoder order (src/sam1/encoder.rs:23 VIT_H: global attention at layers 7, 15, 23, 31, 14x14
windowed attention elsewhere), 32 images per GPU, bf16, 16 heads, head_dim 80:
    global layer   : bh = 32*16      = 512   heads of 64x64 = 4096 tokens
    windowed layer : bh = 32*25*16   = 12800 windows-heads of 14x14 = 196 tokens (64x64 grid padded to 70x70)
Algorithmic FLOPs: 4*N^2*hd per head (QK^T + PV); 481.3 GFLOP per image, 15.40 TFLOP per step per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N   (one rank per GPU)

Multi-GPU: the image batch is sharded (32 images per rank, weak scaling); there is no collective in the
data path. NCCL is used after the timed region to take the max of the per-rank device times and to
gather per-rank output checksums.

--impl reference times the reference's CPU implementation of the path (the C restatement under
oracle/, the reference itself being Rust that cannot be built here) on the host cores of rank 0, on a
bounded sample of the same workload (whole images, all 32 layers).
"""
import argparse
import ctypes
import importlib
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "fused rel-pos attn TFLOP/s (SAM ViT-H encoder attention, 32 layers) & images/s"
UNIT = "TFLOP/s"
HEADS, HD, DEPTH = 16, 80, 32
GLOBAL_LAYERS = (7, 15, 23, 31)
WINDOWS = 25  # 64x64 tokens padded to 70x70 -> 5x5 windows of 14x14


def layer_geoms(images):
    """[(kind, h, w, bh)] for the 32 layers of one step."""
    out = []
    for layer in range(DEPTH):
        if layer in GLOBAL_LAYERS:
            out.append(("global", 64, 64, images * HEADS))
        else:
            out.append(("window", 14, 14, images * WINDOWS * HEADS))
    return out


def layer_flops(h, w, bh, hd=HD):
    n = h * w
    return 4.0 * n * n * hd * bh


def layer_bytes(h, w, bh, hd=HD, es=2):
    """Algorithmic HBM bytes of one launch: q, kt, v read once, out written once, plus the table."""
    n = h * w
    return es * (4.0 * bh * n * hd + (2 * h - 1 + 2 * w - 1) * hd)


def shard_images(global_images, rank, world):
    """Contiguous shard [start, start+count) of the image batch owned by `rank`."""
    base, extra = divmod(global_images, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def max_over_ranks(value, dist, device):
    import torch
    if dist is None:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_floats(values, dist, device):
    """All-gather a short list of floats from every rank -> list per rank."""
    import torch
    if dist is None:
        return [list(values)]
    t = torch.tensor(values, dtype=torch.float64, device=device)
    parts = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, t)
    return [p.cpu().tolist() for p in parts]


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), \
            "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


def load_traffic():
    """Per-launch DRAM bytes of the kernels from the committed ncu summary (None if absent)."""
    path = os.path.join(ROOT, "profiles", "dram_traffic.txt")
    out = {}
    try:
        for line in open(path):
            parts = line.split()
            if len(parts) >= 2 and not line.startswith("#"):
                out[parts[0]] = float(parts[1])
    except OSError:
        pass
    return out


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]
        return False

    def summary(self):
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in getattr(self, "lines", []):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() in ("active", "1"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": smax, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------------------------------------
# CPU reference arm / CPU baseline
# --------------------------------------------------------------------------------------------

def cpu_sample(images=1, seed=7):
    """Time the reference's CPU path (oracle restatement) on `images` whole images of the workload.
    Returns (tflops, seconds, sample description, threads, kind-of-path)."""
    import numpy as np
    from oracle import oracle
    mode = "bf16" if oracle.cpu_has_bf16() else "exact"
    # all host threads this process may use (torchrun sets OMP_NUM_THREADS=1 for its workers)
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    rng = np.random.default_rng(seed)
    sets = {}
    for kind, h, w, bh in {g[:3] + (g[3],) for g in layer_geoms(images)}:
        n = h * w
        sets[kind] = (rng.standard_normal((bh, n, HD), dtype=np.float32),
                      rng.standard_normal((bh, HD, n), dtype=np.float32),
                      rng.standard_normal((bh, n, HD), dtype=np.float32),
                      (rng.standard_normal((4 * h - 2, HD), dtype=np.float32) * 0.5).astype(np.float32), h, w)
    flops = 0.0
    t0 = time.perf_counter()
    for kind, h, w, bh in layer_geoms(images):
        q, kt, v, t, _, _ = sets[kind]
        oracle.attention_relpos(q, kt, v, t, h, w, HD ** -0.5, threads=threads, mode=mode)
        flops += layer_flops(h, w, bh)
    dt = time.perf_counter() - t0
    desc = (f"{images} image(s) x 32 layers of the config-4 workload ({mode} CPU path of src/kernels.rs:131-225"
            f"{' + src/cpu_gemm.rs' if mode == 'bf16' else ''}), {threads} threads")
    return flops / dt / 1e12, dt, desc, threads, mode


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    for _ in range(args.warmup):
        cpu_sample(images=1)
    vals, secs = [], []
    desc, threads, mode = "", 0, "exact"
    for _ in range(args.steps):
        v, s, desc, threads, mode = cpu_sample(images=1)
        vals.append(v)
        secs.append(s)
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * statistics.median(secs),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 GEMMs, f32 softmax" if mode == "bf16" else "f32",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.5) rel-pos tables)",
        "config": {"workload": "config 4 sample: SAM ViT-H attention, 1 image per step, 32 layers", "images_per_step": 1},
        "images_per_s": 1.0 / statistics.median(secs),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": desc},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------------------------------
# GPU arm
# --------------------------------------------------------------------------------------------

def run_ours(args):
    import torch
    samrs = importlib.import_module("sam-rs_b200")
    lib = samrs._abi.lib()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as tdist
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
        dist = tdist

    images = args.images
    geoms = layer_geoms(images)
    gen = torch.Generator(device=device).manual_seed(1000 + rank)
    stream = torch.cuda.current_stream(device)
    sptr = stream.cuda_stream

    def rnd(*shape, std=1.0):
        return (torch.randn(*shape, device=device, generator=gen) * std).to(torch.bfloat16)

    sets = {}
    for kind, h, w, bh in {(g[0], g[1], g[2], g[3]) for g in geoms}:
        n = h * w
        sets[kind] = dict(q=rnd(bh, n, HD), kt=rnd(bh, HD, n), v=rnd(bh, n, HD),
                          out=torch.empty(bh, n, HD, device=device, dtype=torch.bfloat16))
    tables = [rnd(4 * h - 2, HD, std=0.5) for (_, h, w, _) in geoms]
    scale = HD ** -0.5

    def launch(li):
        kind, h, w, bh = geoms[li]
        s = sets[kind]
        rc = lib.samrs_relpos_attn_fwd(s["q"].data_ptr(), s["kt"].data_ptr(), s["v"].data_ptr(),
                                       tables[li].data_ptr(), s["out"].data_ptr(), bh, h, w, HD, scale, 2, sptr)
        if rc != 0:
            raise RuntimeError(lib.samrs_last_error().decode())

    for _ in range(args.warmup):
        for li in range(DEPTH):
            launch(li)
    torch.cuda.synchronize()
    if samrs.device_status() != 0:
        raise RuntimeError("device status word set during warm-up")

    K = args.steps
    ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(DEPTH)]
          for _ in range(K)]
    step_start = torch.cuda.Event(enable_timing=True)
    step_end = torch.cuda.Event(enable_timing=True)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        step_start.record(stream)
        for k in range(K):
            for li in range(DEPTH):
                ev[k][li][0].record(stream)
                launch(li)
                ev[k][li][1].record(stream)
        step_end.record(stream)
        torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    local_ms = step_start.elapsed_time(step_end)
    max_ms = max_over_ranks(local_ms, dist, device)
    per_kind = {"global": [], "window": []}
    for k in range(K):
        for li in range(DEPTH):
            per_kind[geoms[li][0]].append(ev[k][li][0].elapsed_time(ev[k][li][1]))
    status = samrs.device_status()

    flops_step = sum(layer_flops(h, w, bh) for (_, h, w, bh) in geoms)
    total_flops = flops_step * K * world
    value = total_flops / (max_ms / 1e3) / 1e12
    ms_per_step = max_ms / K
    images_per_s = images * world * K / (max_ms / 1e3)

    # checksums of the last outputs, gathered to rank 0 (after timing)
    csum = [float(sets["global"]["out"].float().sum().item()), float(sets["window"]["out"].float().sum().item())]
    all_csum = gather_floats(csum + [local_ms, float(status)], dist, device)

    hbm, tf_burst, tf_sust, peak_src = load_peaks()
    traffic = load_traffic()

    def roof(kind):
        _, h, w, bh = next(g for g in geoms if g[0] == kind)
        avg_ms = statistics.mean(per_kind[kind])
        if kind == "global":
            ach = layer_flops(h, w, bh) / (avg_ms / 1e3) / 1e12
            peak = tf_burst
            r = {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TFLOP/s", "frac": ach / peak,
                 "peak_source": f"{peak_src} bf16 burst (MEASURED_PEAKS.json)" if peak_src == "measured" else "fallback"}
        else:
            ach = layer_bytes(h, w, bh) / (avg_ms / 1e3) / 1e9
            peak = hbm
            r = {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                 "peak_source": f"{peak_src} HBM copy (MEASURED_PEAKS.json)" if peak_src == "measured" else "fallback"}
        r["traffic"] = traffic.get(kind)
        r["kernel"] = f"relpos_attn ({kind}, h={h} w={w} bh={bh} hd={HD})" + (
            "; time of the single-pass kernel and its fixup launch together" if kind == "global" else "")
        r["avg_launch_ms"] = avg_ms
        r["launches"] = len(per_kind[kind])
        r["time_share"] = sum(per_kind[kind]) / sum(sum(v) for v in per_kind.values())
        return r

    roofs = {k: roof(k) for k in ("global", "window")}
    dominant = max(roofs, key=lambda k: roofs[k]["time_share"])

    neighbours = run_neighbours(samrs, lib, images, device, sptr, hbm) if not args.no_neighbours else None

    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, samrs, lib, geoms, sets, tables, device, stream, dist, world)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        v, s, desc, threads, _ = cpu_sample(images=1)
        cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "sample": desc}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K, "warmup": args.warmup,
            "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded N(0,1) activations, N(0,0.5) rel-pos tables)",
            "config": {"workload": "config 4: SAM ViT-H encoder attention (rel-pos), bf16, 32 layers "
                                   "(global 7,15,23,31 / windowed 14x14), head_dim 80, 16 heads",
                       "images_per_gpu": images, "global_batch": images * world, "parallelism": f"dp{world}",
                       "l2": "no flush; every launch's inputs (>= 1 GB) exceed the 126 MB L2"},
            "images_per_s": images_per_s,
            "tflops_by_layer": {k: layer_flops(*next(g for g in geoms if g[0] == k)[1:]) /
                                (statistics.mean(per_kind[k]) / 1e3) / 1e12 for k in per_kind},
            "roofline": roofs[dominant],
            "roofline_other": roofs["window" if dominant == "global" else "global"],
            # a bf16 global layer is two launches: the single-pass kernel and the fixup of the CTAs it marked
            "gpu_launches": K * sum(2 if g[0] == "global" else 1 for g in geoms),
            "clocks": clk.summary(),
            "device_status": [int(c[-1]) for c in all_csum],
            "rank_ms": [c[-2] for c in all_csum],
            "checksums": [c[:2] for c in all_csum],
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if e2e is not None:
            line["e2e"] = e2e
        if neighbours is not None:
            line["neighbours"] = neighbours
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_neighbours(samrs, lib, images, device, sptr, hbm, reps=10):
    """The path's neighbours on the token grid at the bench workload (not part of the metric): the qkv
    split fused with the window partition and the head merge fused with the unpartition, for the windowed
    (ws 14, pad 64 -> 70) and the global (one 64x64 window) layers. Algorithmic bytes: the real tokens'
    y (3C) read and q, kt, v (pads included) written; the real tokens' attention rows read and written."""
    import torch
    nh, c, es = 16, 16 * HD, 2
    out = {}
    y = (torch.randn(images * 4096, 3 * c, device=device) * 0.5).to(torch.bfloat16)
    bias = (torch.randn(3 * c, device=device) * 0.1).to(torch.bfloat16)
    for name, ws in (("window", 14), ("global", 0)):
        n, nwin = (196, 25) if ws else (4096, 1)
        bh = images * nwin * nh
        packed = torch.empty(3 * bh * n * HD, device=device, dtype=torch.bfloat16)
        attn = torch.empty(bh, n, HD, device=device, dtype=torch.bfloat16)
        merged = torch.empty(images * 4096, c, device=device, dtype=torch.bfloat16)
        calls = {
            "qkv_split_window": (lambda: lib.samrs_qkv_split_window_fwd(
                y.data_ptr(), bias.data_ptr(), packed.data_ptr(), images, 64, 64, ws, nh, HD, 2, sptr),
                images * 4096 * 3 * c * es + 3 * bh * n * HD * es),
            "window_merge": (lambda: lib.samrs_window_merge_fwd(
                attn.data_ptr(), merged.data_ptr(), images, 64, 64, ws, nh, HD, 2, sptr),
                2 * images * 4096 * c * es),
        }
        for kname, (fn, nbytes) in calls.items():
            for _ in range(3):
                if fn() != 0:
                    raise RuntimeError(lib.samrs_last_error().decode())
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            a.record()
            for _ in range(reps):
                fn()
            b.record()
            torch.cuda.synchronize()
            ms = a.elapsed_time(b) / reps
            gbs = nbytes / (ms / 1e3) / 1e9
            out[f"{kname} ({name})"] = {"ms": ms, "GB/s": gbs, "frac_of_hbm": gbs / hbm, "bytes": nbytes}
        del packed, attn, merged
    if samrs.device_status() != 0:
        raise RuntimeError("device status word set by the neighbour kernels")
    return out


def run_e2e(args, samrs, lib, geoms, sets, tables, device, stream, dist, world):
    """Same workload through the C ABI with host (pinned) buffers: every layer copies its q, kt, v
    host->device, runs the op, and copies its output device->host, all inside the timed region.
    Serving-style pipelining: two device buffer sets per layer kind and three streams (upload, compute,
    download) ordered by events, so layer l+1's upload, layer l's kernel and layer l-1's download overlap
    (PCIe is full duplex)."""
    import torch
    host = {}
    dev = {}
    for kind, s in sets.items():
        host[kind] = {k: torch.empty(s[k].shape, dtype=s[k].dtype, pin_memory=True) for k in ("q", "kt", "v", "out")}
        for k in ("q", "kt", "v"):
            host[kind][k].copy_(s[k])
        dev[kind] = [s, {k: torch.empty_like(s[k]) for k in ("q", "kt", "v", "out")}]
    torch.cuda.synchronize()
    s_up, s_down = torch.cuda.Stream(device), torch.cuda.Stream(device)
    sptr = stream.cuda_stream
    scale = HD ** -0.5
    # per (kind, buffer): the compute that last read the inputs / wrote the output, the download of it
    comp_done = {k: [None, None] for k in sets}
    down_done = {k: [None, None] for k in sets}
    h2d = d2h = 0

    def step():
        nonlocal h2d, d2h
        h2d = d2h = 0
        use = {k: 0 for k in sets}
        for li, (kind, h, w, bh) in enumerate(geoms):
            bi = use[kind] & 1
            use[kind] += 1
            d, hb = dev[kind][bi], host[kind]
            up = torch.cuda.Event()
            with torch.cuda.stream(s_up):
                if comp_done[kind][bi] is not None:
                    s_up.wait_event(comp_done[kind][bi])  # the kernel that read this buffer set is done
                for k in ("q", "kt", "v"):
                    d[k].copy_(hb[k], non_blocking=True)
                    h2d += hb[k].numel() * hb[k].element_size()
                up.record(s_up)
            stream.wait_event(up)
            if down_done[kind][bi] is not None:
                stream.wait_event(down_done[kind][bi])  # the previous output in this set is on the host
            rc = lib.samrs_relpos_attn_fwd(d["q"].data_ptr(), d["kt"].data_ptr(), d["v"].data_ptr(),
                                           tables[li].data_ptr(), d["out"].data_ptr(), bh, h, w, HD, scale, 2, sptr)
            if rc != 0:
                raise RuntimeError(lib.samrs_last_error().decode())
            cd = torch.cuda.Event()
            cd.record(stream)
            comp_done[kind][bi] = cd
            dd = torch.cuda.Event()
            with torch.cuda.stream(s_down):
                s_down.wait_event(cd)
                hb["out"].copy_(d["out"], non_blocking=True)
                d2h += hb["out"].numel() * hb["out"].element_size()
                dd.record(s_down)
            down_done[kind][bi] = dd

    def join():
        # the compute stream waits for the other two, so one event on it closes the step
        for st in (s_up, s_down):
            e = torch.cuda.Event()
            e.record(st)
            stream.wait_event(e)

    step()
    join()
    torch.cuda.synchronize()
    k = max(1, min(args.steps, args.e2e_steps))
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(stream)
    s_up.wait_event(a)
    s_down.wait_event(a)
    for _ in range(k):
        step()
    join()
    b.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(a.elapsed_time(b), dist, device)
    flops = sum(layer_flops(h, w, bh) for (_, h, w, bh) in geoms) * k * world
    return {"value": flops / (ms / 1e3) / 1e12, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "steps": k, "ms_per_step": ms / k,
            "path": "C ABI samrs_relpos_attn_fwd, pinned host buffers, upload/compute/download streams"}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--images", type=int, default=32, help="images per GPU (config 4: 32)")
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-neighbours", action="store_true", help="skip timing the qkv split / head merge kernels")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
