#!/usr/bin/env python
"""Benchmark of the fused decomposed-rel-pos attention on B200 (4 and 5).

One step = one pass of a SAM ViT encoder's attention over a batch of synthetic inputs resident in HBM, all
layers in encoder order (src/sam1/encoder.rs:19-23), bf16:
    config 4 (default, the metric's configuration): ViT-H, 32 images per GPU, 16 heads, head_dim 80, 32 layers,
        global attention at layers 7, 15, 23, 31 and 14x14 windowed attention elsewhere:
        global layer   : bh = 32*16      = 512   heads of 64x64 = 4096 tokens
        windowed layer : bh = 32*25*16   = 12800 windows-heads of 14x14 = 196 tokens (64x64 padded to 70x70)
        481.3 GFLOP per image, 15.40 TFLOP per step per GPU (4*N^2*hd per head: QK^T + PV)
    config 3: ViT-L, 16 images per GPU, 16 heads, head_dim 64, 24 layers, global at 5, 11, 17, 23
    config 5: config 4 swept over 8, 16, 32, 64 and 128 images per GPU
    config 2: the whole ViT-B encoder block stack (LayerNorm, the qkv / proj / MLP GEMMs with their fused
        epilogues, the attention), f16, 8 images per GPU, 12 blocks
    config 1: the ViT-B op in f32, one image: the windowed and the global layer, each through the f32
        tensor-core kernel (3xTF32) and through the CUDA-core kernel
The default run prints the config-4 line and carries configs 1, 2, 3 and 5 (shorter timings) in its "configs"
object, and the block's GEMMs at the ViT-H shapes in "gemms"; --config 1 / 2 / 3 / 5 print their own line
(--config 1: one step = the windowed and the global f32 layer of one image, K steps per layer kind).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 1|2|3|4|5]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N   (one rank per GPU)

Multi-GPU: the image batch is sharded (the per-GPU image count is fixed, weak scaling); there is no collective
in the data path. NCCL is used after the timed region to take the max of the per-rank device times and to
gather per-rank output checksums.

--library-context times the two attention kernels against torch SDPA on its cuDNN backend (no bias) on the
config-4 layer shapes, with clocks and power per phase, and prints one line of its own.

--impl reference --reference-path cuda times the reference's own CUDA path on the GPU instead (its
kernels/sam.cu relpos_softmax between cuBLAS bmm's, compiled into oracle/_ref), on the same workload.

--impl reference times the reference's CPU implementation of the path (the C restatement under
oracle/, the reference itself being Rust that cannot be built here) on the host cores of rank 0, on a
bounded sample of the same workload (whole images, all layers).
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
WINDOWS = 25  # 64x64 tokens padded to 70x70 -> 5x5 windows of 14x14
KINDS = ("global", "window")  # fixed order: inputs are drawn from the generator in this order


class Workload:
    """One ViT's attention stack (src/sam1/encoder.rs:19-23: VIT_L, VIT_H)."""

    def __init__(self, name, heads, hd, depth, global_layers, images):
        self.name, self.heads, self.hd, self.depth = name, heads, hd, depth
        self.global_layers, self.images = tuple(global_layers), images

    def describe(self):
        return (f"{self.name} encoder attention (rel-pos), bf16, {self.depth} layers (global "
                f"{','.join(map(str, self.global_layers))} / windowed 14x14), head_dim {self.hd}, {self.heads} heads")


VIT_H = dict(name="SAM ViT-H", heads=16, hd=80, depth=32, global_layers=(7, 15, 23, 31))
VIT_L = dict(name="SAM ViT-L", heads=16, hd=64, depth=24, global_layers=(5, 11, 17, 23))
CONFIGS = {3: Workload(images=16, **VIT_L), 4: Workload(images=32, **VIT_H)}
# config 2: the whole ViT-B block stack (src/sam1/encoder.rs:19-23 VIT_B, Block::forward :115-129), f16
VIT_B_STACK = dict(images=8, c=768, heads=12, depth=12, global_layers=(2, 5, 8, 11), window=14)
SWEEP_IMAGES = (8, 16, 32, 64, 128)  # config 5: config 4 at these images per GPU
HD = VIT_H["hd"]


def layer_geoms(images, wl=None):
    """[(kind, h, w, bh)] for the layers of one step, in encoder order."""
    wl = wl or CONFIGS[4]
    out = []
    for layer in range(wl.depth):
        if layer in wl.global_layers:
            out.append(("global", 64, 64, images * wl.heads))
        else:
            out.append(("window", 14, 14, images * WINDOWS * wl.heads))
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
    """SM clock, power and clock-event (throttle) reasons of one GPU, sampled every 10 ms through NVML from a
    background thread while the timed region runs (nvidia-smi every 200 ms where NVML is unavailable). The GPU
    is the CUDA device `gpu_index`, matched to its NVML handle by PCI bus id. Reads only; changes nothing."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits, in the order of the names summary() reports
    REASON_BITS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
                   ("sw_power_cap", 0x4))

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.thread = None
        self.lines = []

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        if torch.cuda.is_available():
            pr = torch.cuda.get_device_properties(self.gpu)
            for bus in (f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0",
                        f"{pr.pci_domain_id:04X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"):
                try:
                    return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
                except pynvml.NVMLError:
                    pass
        return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.gpu)

    def __enter__(self):
        import threading
        self.lines = []
        try:
            nv, h = self._nvml_handle()
            smax = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            stop = threading.Event()

            def run():
                while not stop.is_set():
                    try:
                        sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                        watts = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                        bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    except nv.NVMLError:
                        break
                    flags = ["Active" if bits & bit else "Not Active" for _, bit in self.REASON_BITS]
                    self.lines.append(",".join([str(self.gpu), str(sm), str(smax), f"{watts:.1f}", hex(bits)] + flags))
                    stop.wait(0.01)

            self._stop = stop
            self.thread = threading.Thread(target=run, daemon=True)
            self.thread.start()
            return self
        except Exception:
            self.thread = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.thread is not None:
            self._stop.set()
            self.thread.join(timeout=5)
            return False
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
        sm, smax, reasons, watts = [], None, set(), []
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
            try:
                watts.append(float(f[3]))
            except ValueError:
                pass
            for name, val in zip(names, f[5:9]):
                if val.lower() in ("active", "1"):
                    reasons.add(name)
        how = "nvml every 10 ms" if self.thread is not None else "nvidia-smi every 200 ms"
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": smax, "reasons": [], "samples": 0, "sampler": how}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": len(sm),
                "power_w": statistics.median(watts) if watts else None, "sampler": how}


# --------------------------------------------------------------------------------------------
# CPU reference arm / CPU baseline
# --------------------------------------------------------------------------------------------

def cpu_sample(images=1, seed=7, wl=None):
    """Time the reference's CPU path (oracle restatement) on `images` whole images of the workload.
    Returns (tflops, seconds, sample description, threads, kind-of-path)."""
    import numpy as np
    from oracle import oracle
    wl = wl or CONFIGS[4]
    mode = "bf16" if oracle.cpu_has_bf16() else "exact"
    # all host threads this process may use (torchrun sets OMP_NUM_THREADS=1 for its workers)
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    rng = np.random.default_rng(seed)
    geoms = layer_geoms(images, wl)
    sets = {}
    for kind in KINDS:
        _, h, w, bh = next(g for g in geoms if g[0] == kind)
        n = h * w
        sets[kind] = (rng.standard_normal((bh, n, wl.hd), dtype=np.float32),
                      rng.standard_normal((bh, wl.hd, n), dtype=np.float32),
                      rng.standard_normal((bh, n, wl.hd), dtype=np.float32),
                      (rng.standard_normal((4 * h - 2, wl.hd), dtype=np.float32) * 0.5).astype(np.float32), h, w)
    flops = 0.0
    t0 = time.perf_counter()
    for kind, h, w, bh in geoms:
        q, kt, v, t, _, _ = sets[kind]
        oracle.attention_relpos(q, kt, v, t, h, w, wl.hd ** -0.5, threads=threads, mode=mode)
        flops += layer_flops(h, w, bh, wl.hd)
    dt = time.perf_counter() - t0
    desc = (f"{images} image(s) x {wl.depth} layers of the {wl.name} workload ({mode} CPU path of "
            f"src/kernels.rs:131-225{' + src/cpu_gemm.rs' if mode == 'bf16' else ''}), {threads} threads")
    return flops / dt / 1e12, dt, desc, threads, mode


def config1_cpu_sample(seed=7):
    """The reference's f32 CPU path (the oracle's exact restatement of src/kernels.rs:131-225) on BASELINE
    config 1: the windowed layer (300 heads of 14x14) and the global layer (12 heads of 64x64), hd 64."""
    import numpy as np
    from oracle import oracle
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    rng = np.random.default_rng(seed)
    flops, dt = 0.0, 0.0
    for h, bh in ((14, 300), (64, 12)):
        n, hd = h * h, 64
        q = rng.standard_normal((bh, n, hd), dtype=np.float32)
        kt = rng.standard_normal((bh, hd, n), dtype=np.float32)
        v = rng.standard_normal((bh, n, hd), dtype=np.float32)
        t = (rng.standard_normal((4 * h - 2, hd), dtype=np.float32) * 0.5).astype(np.float32)
        t0 = time.perf_counter()
        oracle.attention_relpos(q, kt, v, t, h, h, hd ** -0.5, threads=threads, mode="exact")
        dt += time.perf_counter() - t0
        flops += layer_flops(h, h, bh, hd)
    desc = (f"config 1 (windowed 300 heads + global 12 heads, hd 64, one image) through the f32 CPU path of "
            f"src/kernels.rs:131-225, {threads} threads")
    return flops / dt / 1e12, dt, desc, threads


def run_reference_cuda(args):
    """The reference's own CUDA path on this GPU: bmm(relpos_softmax(bmm(q, kt)), v) per layer
    (src/sam1/encoder.rs:81). Its kernels/sam.cu is compiled into oracle/_ref by oracle/build_ref_cuda.py and
    launched as the reference launches it; the bmm's are cuBLAS in the I/O dtype with f32 accumulation, as
    candle's are. Same workload, inputs resident in HBM, CUDA events around K steps."""
    import torch
    from oracle.ref_cuda import RefCuda, RefCudaError
    wl = CONFIGS[3 if args.config == 3 else 4]
    images = args.images or wl.images
    try:
        ref = RefCuda()
    except (RefCudaError, OSError) as e:
        print(json.dumps({"impl": "reference", "reference_path": "cuda", "unavailable": str(e)}), flush=True)
        return 0
    device = torch.device("cuda", 0)
    g = torch.Generator(device=device).manual_seed(1234)
    sets = {}
    for kind in KINDS:
        _, h, w, bh = next(x for x in layer_geoms(images, wl) if x[0] == kind)
        n = h * w
        sets[kind] = (h, w, torch.randn(bh, n, wl.hd, device=device, generator=g).bfloat16(),
                      torch.randn(bh, wl.hd, n, device=device, generator=g).bfloat16(),
                      torch.randn(bh, n, wl.hd, device=device, generator=g).bfloat16(),
                      (torch.randn(4 * h - 2, wl.hd, device=device, generator=g) * 0.5).bfloat16())
    geoms = layer_geoms(images, wl)
    scale = wl.hd ** -0.5

    def step():
        for kind, *_ in geoms:
            h, w, q, kt, v, t = sets[kind]
            ref.attention(q, kt, v, t, h, w, scale)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        a.record()
        for _ in range(args.steps):
            step()
        b.record()
        b.synchronize()
    ms = a.elapsed_time(b) / args.steps
    flops = sum(layer_flops(h, w, bh, wl.hd) for _, h, w, bh in geoms)
    value = flops / (ms / 1e3) / 1e12
    line = {
        "impl": "reference", "reference_path": "cuda", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.5) rel-pos tables)",
        "config": {"workload": f"config {3 if args.config == 3 else 4}: " + wl.describe(), "images_per_gpu": images,
                   "path": "the reference's CUDA path: cuBLAS bmm (I/O dtype, f32 accumulation), its "
                           "relpos_softmax kernel (kernels/sam.cu, built with its own nvcc flags), cuBLAS bmm; "
                           "inputs resident in HBM"},
        "images_per_s": images / (ms / 1e3),
        "clocks": clk.summary(),
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    if args.reference_path == "cuda":
        return run_reference_cuda(args)
    if args.config == 1:
        for _ in range(args.warmup):
            config1_cpu_sample()
        vals, secs = [], []
        desc, threads = "", 0
        for _ in range(args.steps):
            v, s, desc, threads = config1_cpu_sample()
            vals.append(v)
            secs.append(s)
        value = statistics.median(vals)
        line = {
            "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * statistics.median(secs),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.5) rel-pos tables)",
            "config": {"workload": "config 1: ViT-B attention op, f32, 1 image (windowed 300 heads 14x14 + global "
                                   "12 heads 64x64, hd 64)"},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": desc},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return 0
    wl = CONFIGS[3 if args.config == 3 else 4]
    for _ in range(args.warmup):
        cpu_sample(images=1, wl=wl)
    vals, secs = [], []
    desc, threads, mode = "", 0, "exact"
    for _ in range(args.steps):
        v, s, desc, threads, mode = cpu_sample(images=1, wl=wl)
        vals.append(v)
        secs.append(s)
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * statistics.median(secs),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 GEMMs, f32 softmax" if mode == "bf16" else "f32",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.5) rel-pos tables)",
        "config": {"workload": f"config {3 if args.config == 3 else 4} sample: {wl.name} attention, 1 image per step, "
                               f"{wl.depth} layers", "images_per_step": 1},
        "images_per_s": 1.0 / statistics.median(secs),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": desc},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------------------------------
# GPU arm
# --------------------------------------------------------------------------------------------

def bind_to_gpu_numa_node(local_rank):
    """Pin this process to the CPUs of its GPU's NUMA node, so that the pinned host buffers of the e2e leg
    are first-touched there. Returns the node (None if the host reports none)."""
    try:
        import pynvml
        pynvml.nvmlInit()
        handle = pynvml.nvmlDeviceGetHandleByIndex(local_rank)
        bus = pynvml.nvmlDeviceGetPciInfo(handle).busId
        bus = bus.decode() if isinstance(bus, bytes) else bus
        bus = bus.lower()[-12:]  # domain:bus:device.function as sysfs spells it
        with open(f"/sys/bus/pci/devices/{bus}/numa_node") as f:
            node = int(f.read().strip())
        if node < 0:
            return None
        with open(f"/sys/devices/system/node/node{node}/cpulist") as f:
            cpus = set()
            for part in f.read().strip().split(","):
                a, _, b = part.partition("-")
                cpus.update(range(int(a), int(b or a) + 1))
        cpus &= os.sched_getaffinity(0) or cpus
        if cpus:
            os.sched_setaffinity(0, cpus)
        return node
    except Exception:
        return None


def relpos_attention_fp32(torch, q, kt, v, table, h, w, scale):
    """Plain PyTorch fp32 reference of the op on the device (the math of the reference's tensor definition,
    src/kernels.rs:20-42): softmax(scale q kt + q.Th[i-kh+h-1] + q.Tw[j-kw+w-1]) v with the N x N scores
    materialised. q, v [b, n, hd]; kt [b, hd, n]; table [(2h-1)+(2w-1), hd]; all fp32."""
    b, n, hd = q.shape
    dev = q.device
    th, tw = table[: 2 * h - 1], table[2 * h - 1:]
    ih = torch.arange(h, device=dev)
    iw = torch.arange(w, device=dev)
    rel_h = th[ih[:, None] - ih[None, :] + h - 1]  # [i, kh, hd]
    rel_w = tw[iw[:, None] - iw[None, :] + w - 1]  # [j, kw, hd]
    qg = q.view(b, h, w, hd)
    rh = torch.einsum("bijd,ikd->bijk", qg, rel_h)  # [b, i, j, kh]
    rw = torch.einsum("bijd,jkd->bijk", qg, rel_w)  # [b, i, j, kw]
    tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        s = torch.bmm(q, kt) * scale
        s = s.view(b, h, w, h, w) + rh[:, :, :, :, None] + rw[:, :, :, None, :]
        return torch.bmm(torch.softmax(s.view(b, n, n), dim=-1), v)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = tf32


class Step:
    """The layers of one step of a workload, with inputs resident on the device (drawn in a fixed order from a
    per-rank generator, so a rank's inputs and outputs do not depend on the world size)."""

    def __init__(self, torch, lib, wl, images, device, rank, sptr, table_std=0.5):
        self.lib, self.wl, self.images, self.sptr = lib, wl, images, sptr
        self.geoms = layer_geoms(images, wl)
        gen = torch.Generator(device=device).manual_seed(1000 + rank)

        def rnd(*shape, std=1.0):
            return (torch.randn(*shape, device=device, generator=gen) * std).to(torch.bfloat16)

        hd = wl.hd
        self.sets = {}
        for kind in KINDS:
            _, h, w, bh = next(g for g in self.geoms if g[0] == kind)
            n = h * w
            self.sets[kind] = dict(q=rnd(bh, n, hd), kt=rnd(bh, hd, n), v=rnd(bh, n, hd),
                                   out=torch.empty(bh, n, hd, device=device, dtype=torch.bfloat16))
        self.tables = [rnd(4 * h - 2, hd, std=table_std) for (_, h, w, _) in self.geoms]
        self.scale = hd ** -0.5
        self.flops = sum(layer_flops(h, w, bh, hd) for (_, h, w, bh) in self.geoms)

    def launch(self, li, sets=None, stream_ptr=None):
        kind, h, w, bh = self.geoms[li]
        s = (sets or self.sets)[kind]
        rc = self.lib.samrs_relpos_attn_fwd(s["q"].data_ptr(), s["kt"].data_ptr(), s["v"].data_ptr(),
                                            self.tables[li].data_ptr(), s["out"].data_ptr(), bh, h, w, self.wl.hd,
                                            self.scale, 2, stream_ptr or self.sptr)
        if rc != 0:
            raise RuntimeError(self.lib.samrs_last_error().decode())

    def run(self):
        for li in range(len(self.geoms)):
            self.launch(li)

    def checksums(self):
        return [float(self.sets[k]["out"].float().sum().item()) for k in KINDS]

    def sampled_parity(self, torch, heads=(2, 8)):
        """Plain max|got-ref|/max|ref| of heads sampled evenly over the batch (2 global, 8 windowed) of each
        kind's last output (its last layer's table) against relpos_attention_fp32 on the same bf16 inputs."""
        errs = []
        for kind, nh in zip(KINDS, heads):
            li = max(i for i, g in enumerate(self.geoms) if g[0] == kind)
            _, h, w, bh = self.geoms[li]
            st = self.sets[kind]
            idx = torch.linspace(0, bh - 1, nh, device=st["q"].device).round().long().unique()
            ref = relpos_attention_fp32(torch, st["q"][idx].float(), st["kt"][idx].float(), st["v"][idx].float(),
                                        self.tables[li].float(), h, w, self.scale)
            errs.append(float((st["out"][idx].float() - ref).abs().max() / ref.abs().max()))
        return errs


def time_workload(torch, samrs, step, stream, dist, device, steps, warmup, per_launch=False, clocks=None):
    """W untimed warm-up steps, then K steps timed with CUDA events on the launch stream between barriers;
    returns (local ms, max-over-ranks ms, {kind: [per-launch ms]})."""
    for _ in range(warmup):
        step.run()
    torch.cuda.synchronize()
    if samrs.device_status() != 0:
        raise RuntimeError("device status word set during warm-up")
    depth = len(step.geoms)
    ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(depth)]
          for _ in range(steps)] if per_launch else None
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    if clocks is not None:
        clocks.__enter__()
    a.record(stream)
    for k in range(steps):
        for li in range(depth):
            if per_launch:
                ev[k][li][0].record(stream)
            step.launch(li)
            if per_launch:
                ev[k][li][1].record(stream)
    b.record(stream)
    torch.cuda.synchronize()
    if clocks is not None:
        clocks.__exit__(None, None, None)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    local_ms = a.elapsed_time(b)
    per_kind = {k: [] for k in KINDS}
    if per_launch:
        for k in range(steps):
            for li in range(depth):
                per_kind[step.geoms[li][0]].append(ev[k][li][0].elapsed_time(ev[k][li][1]))
    return local_ms, max_over_ranks(local_ms, dist, device), per_kind


def summary_line(step, world, steps, max_ms):
    return {"value": step.flops * steps * world / (max_ms / 1e3) / 1e12, "unit": UNIT,
            "images_per_s": step.images * world * steps / (max_ms / 1e3), "ms_per_step": max_ms / steps,
            "images_per_gpu": step.images, "steps": steps}


def run_ours(args):
    import torch
    samrs = importlib.import_module("sam-rs_b200")
    lib = samrs._abi.lib()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    numa = bind_to_gpu_numa_node(local)
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as tdist
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
        dist = tdist
    stream = torch.cuda.current_stream(device)
    sptr = stream.cuda_stream
    hbm, tf_burst, tf_sust, peak_src = load_peaks()

    if args.config == 1:
        c1 = run_config1(torch, samrs, device, reps=args.steps, warmup=args.warmup)
        e2e1 = config1_e2e(torch, samrs, device, steps=args.steps, warmup=args.warmup)
        if rank == 0:
            ms = c1["layer_ms_tc"]
            flops = layer_flops(14, 14, 300, 64) + layer_flops(64, 64, 12, 64)
            line = {"metric": METRIC, "value": flops / (ms / 1e3) / 1e12, "unit": UNIT, "n_gpus": world,
                    "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                    "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                    "data": "synthetic (seeded N(0,1) activations, N(0,0.5) rel-pos tables)",
                    "config": {"workload": c1["workload"], "parallelism": f"dp{world}"},
                    "layers": c1, "gpu_launches": 6 * args.steps, "e2e": e2e1}
            if world == 1 and not args.no_cpu:
                v, _, desc, threads = config1_cpu_sample()
                line["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "sample": desc}
            print(json.dumps(line), flush=True)
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return 0

    if args.config == 2:
        c2 = run_config2(torch, samrs, device, rank, dist, world, args.steps, args.warmup, stream)
        if rank == 0:
            line = {"metric": METRIC, "value": c2["tflops"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
                    "warmup": args.warmup, "ms_per_step": c2["ms_per_step"], "higher_is_better": True,
                    "scaling": "weak", "vs_baseline": None, "dtype": "f16",
                    "data": "synthetic (seeded N(0,1) tokens, N(0,0.02) weights, N(0,0.5) rel-pos tables)",
                    "config": {"workload": c2["workload"], "images_per_gpu": c2["images_per_gpu"],
                               "parallelism": f"dp{world}"},
                    "images_per_s": c2["images_per_s"], "flops_per_step": c2["flops_per_step"],
                    "gpu_launches": c2["gpu_launches_per_step"] * args.steps}
            print(json.dumps(line), flush=True)
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return 0

    if args.config == 5:
        sweep = run_sweep(torch, samrs, lib, device, rank, sptr, stream, dist, world, args.steps, args.warmup)
        if rank == 0:
            best = max(sweep, key=lambda r: r["value"])
            line = {"metric": METRIC, "value": best["value"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
                    "warmup": args.warmup, "ms_per_step": best["ms_per_step"], "higher_is_better": True,
                    "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                    "data": "synthetic (seeded N(0,1) activations, N(0,0.5) rel-pos tables)",
                    "config": {"workload": "config 5: config 4 (" + CONFIGS[4].describe() + ") at 8-128 images per "
                                           "GPU; value = the best point of the sweep", "parallelism": f"dp{world}"},
                    "sweep": sweep, "gpu_launches": sum(36 * r["steps"] for r in sweep)}
            print(json.dumps(line), flush=True)
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return 0

    wl = CONFIGS[args.config]
    images = args.images or wl.images
    step = Step(torch, lib, wl, images, device, rank, sptr)
    K = args.steps
    clk = ClockSampler(local)
    samrs.recompute_count(clear=True)
    local_ms, max_ms, per_kind = time_workload(torch, samrs, step, stream, dist, device, K, args.warmup,
                                               per_launch=True, clocks=clk)
    recomputed = samrs.recompute_count(clear=True)
    status = samrs.device_status()
    summ = summary_line(step, world, K, max_ms)

    # checksums of the last outputs, sampled parity, per-rank time and status, gathered to rank 0 (after timing)
    all_csum = gather_floats(step.checksums() + step.sampled_parity(torch) + [local_ms, float(status)], dist, device)
    traffic = load_traffic() if args.config == 4 else {}

    def roof(kind):
        _, h, w, bh = next(g for g in step.geoms if g[0] == kind)
        avg_ms = statistics.mean(per_kind[kind])
        if kind == "global":
            # the kernel runs inside a long step (tens of ms, steps back to back) under the 1000 W cap, so its
            # denominator is the sustained bf16 figure; the burst fraction is reported beside it
            ach = layer_flops(h, w, bh, wl.hd) / (avg_ms / 1e3) / 1e12
            peak = tf_sust
            r = {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TFLOP/s", "frac": ach / peak,
                 "peak_source": (f"{peak_src} bf16 sustained (MEASURED_PEAKS.json): timed inside a long step, "
                                 "power-capped" if peak_src == "measured" else "fallback sustained"),
                 "frac_of_burst": ach / tf_burst, "burst_peak": tf_burst}
        else:
            ach = layer_bytes(h, w, bh, wl.hd) / (avg_ms / 1e3) / 1e9
            peak = hbm
            r = {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                 "peak_source": f"{peak_src} HBM copy (MEASURED_PEAKS.json)" if peak_src == "measured" else "fallback"}
        r["traffic"] = traffic.get(kind)
        r["kernel"] = f"relpos_attn ({kind}, h={h} w={w} bh={bh} hd={wl.hd})" + (
            "; time of the single-pass kernel and its fixup launch together" if kind == "global" else "")
        r["avg_launch_ms"] = avg_ms
        r["launches"] = len(per_kind[kind])
        r["time_share"] = sum(per_kind[kind]) / sum(sum(v) for v in per_kind.values())
        return r

    roofs = {k: roof(k) for k in KINDS}
    dominant = max(roofs, key=lambda k: roofs[k]["time_share"])
    n_global = sum(1 for g in step.geoms if g[0] == "global")
    global_ctas = (K + args.warmup) * n_global * step.geoms[wl.global_layers[0]][3] * 16  # warm-up steps count too

    extra = {}
    if args.config == 4 and not args.no_configs:
        extra["3"] = run_config3(torch, samrs, lib, device, rank, sptr, stream, dist, world, min(K, 5), args.warmup)
        extra["5"] = run_sweep(torch, samrs, lib, device, rank, sptr, stream, dist, world, min(K, 5), args.warmup)
        extra["recompute_by_table_std"], extra["global_policy_by_table_std"] = recompute_rates(
            torch, samrs, lib, device, sptr)
        extra["2"] = run_config2(torch, samrs, device, rank, dist, world, min(K, 5), args.warmup, stream)
        extra["1"] = run_config1(torch, samrs, device)

    neighbours = run_neighbours(samrs, lib, images, device, sptr, hbm, wl) \
        if not args.no_neighbours and args.config == 4 else None
    gemms = run_gemms(samrs, lib, device, sptr, tf_burst) if not args.no_neighbours and args.config == 4 else None

    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, samrs, step, device, stream, dist, world, max_ms / K)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        v, s, desc, threads, _ = cpu_sample(images=1, wl=wl)
        cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "sample": desc}

    if rank == 0:
        line = {
            "metric": METRIC, "value": summ["value"], "unit": UNIT, "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": summ["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.5) rel-pos tables)",
            "config": {"workload": f"config {args.config}: " + wl.describe(),
                       "images_per_gpu": images, "global_batch": images * world, "parallelism": f"dp{world}",
                       "l2": "no flush; every launch's inputs (>= 0.3 GB) exceed the 126 MB L2"},
            "images_per_s": summ["images_per_s"],
            "tflops_by_layer": {k: layer_flops(*next(g for g in step.geoms if g[0] == k)[1:], wl.hd) /
                                (statistics.mean(per_kind[k]) / 1e3) / 1e12 for k in KINDS},
            "roofline": roofs[dominant],
            "roofline_other": roofs["window" if dominant == "global" else "global"],
            # a bf16 global layer is two launches: the single-pass kernel and the fixup of the CTAs it marked
            "gpu_launches": K * sum(2 if g[0] == "global" else 1 for g in step.geoms),
            "recomputed_global_ctas": {"ctas": recomputed, "of": global_ctas,
                                       "fraction": recomputed / global_ctas if global_ctas else 0.0},
            "clocks": clk.summary(),
            "device_status": [int(c[-1]) for c in all_csum],
            "rank_ms": [c[-2] for c in all_csum],
            "checksums": [c[:2] for c in all_csum],
            "parity_vs_torch_fp32": {
                "what": "plain max|got-ref|/max|ref| per rank of sampled heads (2 global, 8 windowed) of the last "
                        "outputs against a PyTorch fp32 reference on the same bf16 inputs (bar 3e-3 + half a bf16 ulp)",
                "by_rank": [{"global": c[2], "window": c[3]} for c in all_csum]},
            "numa_node": numa,
        }
        if extra:
            line["configs"] = extra
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if e2e is not None:
            line["e2e"] = e2e
        if neighbours is not None:
            line["neighbours"] = neighbours
        if gemms is not None:
            line["gemms"] = gemms
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def config2_flops(images, c=768, heads=12, depth=12, global_layers=(2, 5, 8, 11)):
    """Algorithmic FLOPs of one ViT-B stack step on the real tokens: the four projections (qkv 3C, proj C,
    lin1 4C, lin2 4C: 2 * T * C * 12 C per block) and the attention (4 N^2 hd per head)."""
    t, hd = images * 4096, c // heads
    gemm = 2.0 * t * c * 12 * c * depth
    att = sum(layer_flops(64, 64, images * heads, hd) if i in global_layers else
              layer_flops(14, 14, images * WINDOWS * heads, hd) for i in range(depth))
    return gemm, att


def run_config2(torch, samrs, device, rank, dist, world, steps, warmup, stream):
    """the ViT-B encoder block stack (12 blocks, global at 2, 5, 8, 11), f16, 8 images per
    GPU, random-init weights ~ N(0, 0.02), tokens ~ N(0, 1), every op on this library's kernels (LayerNorm,
    the fused qkv GEMM, the attention, the head merge, the proj / lin1 / lin2 GEMMs with their epilogues)."""
    cfg = VIT_B_STACK
    c, nh, images = cfg["c"], cfg["heads"], cfg["images"]
    hd = c // nh
    gen = torch.Generator(device=device).manual_seed(2000 + rank)

    def rnd(*shape, std=0.02):
        return (torch.randn(*shape, device=device, generator=gen) * std).half()

    blocks = []
    for i in range(cfg["depth"]):
        win = 0 if i in cfg["global_layers"] else cfg["window"]
        size = win if win else 64
        p = dict(qkv_w=rnd(3 * c, c), qkv_b=rnd(3 * c), proj_w=rnd(c, c), proj_b=rnd(c), lin1_w=rnd(4 * c, c),
                 lin1_b=rnd(4 * c), lin2_w=rnd(c, 4 * c), lin2_b=rnd(c), norm1_w=1 + rnd(c, std=0.1),
                 norm1_b=rnd(c), norm2_w=1 + rnd(c, std=0.1), norm2_b=rnd(c), rel_pos_h=rnd(2 * size - 1, hd, std=0.5),
                 rel_pos_w=rnd(2 * size - 1, hd, std=0.5))
        blocks.append(samrs.Block(p, nh, win))
    x0 = rnd(images, 64, 64, c, std=1.0)

    def step():
        y = x0
        for blk in blocks:
            y = blk.forward(y)
        return y

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if samrs.device_status() != 0:
        raise RuntimeError("device status word set during the config-2 warm-up")
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        y = step()
    b.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(a.elapsed_time(b), dist, device)
    gemm, att = config2_flops(images)
    launches = sum(8 if i in cfg["global_layers"] else 9 for i in range(cfg["depth"]))
    out = {"workload": "config 2: SAM ViT-B encoder block stack, f16, 12 blocks (global 2,5,8,11 / windowed 14x14), "
                       "C 768, 12 heads, random-init weights N(0, 0.02)",
           "images_per_gpu": images, "steps": steps, "ms_per_step": ms / steps,
           "images_per_s": images * world * steps / (ms / 1e3),
           "tflops": (gemm + att) * world * steps / (ms / 1e3) / 1e12,
           "flops_per_step": {"gemm": gemm, "attention": att}, "gpu_launches_per_step": launches,
           "checksum_rank0": float(y.float().sum().item()) if rank == 0 else None}
    del blocks, x0, y
    torch.cuda.empty_cache()
    return out


def run_gemms(samrs, lib, device, sptr, tf_peak, images=32, reps=5):
    """The tensor-core GEMMs with their fused epilogues at the ViT-H block's shapes (config 4, 32 images:
    T = 131072 tokens, C = 1280), against torch (cuBLAS) plus the separate epilogue on the same inputs."""
    import torch
    import torch.nn.functional as F
    t, c, nh, hd = images * 4096, 1280, 16, 80
    g = torch.Generator(device=device).manual_seed(9)

    def rnd(*shape, std=1.0):
        return (torch.randn(*shape, device=device, generator=g) * std).to(torch.bfloat16)

    def timed(fn):
        for _ in range(2):
            fn()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps

    out = {}
    x = rnd(t, c)
    res = rnd(t, c)
    cases = {"qkv (window layout)": (3 * c, c), "proj + bias_residual": (c, c), "lin1 + bias_gelu": (4 * c, c),
             "lin2 + bias_residual": (c, 4 * c)}
    for name, (n, k) in cases.items():
        a = x if k == c else rnd(t, k)
        w, bias = rnd(n, k, std=0.02), rnd(n, std=0.02)
        flops = 2.0 * t * n * k
        if name.startswith("qkv"):
            ours = lambda: samrs.qkv_linear_window(a, w, bias, images, 64, 64, 14, nh, hd)
            ref = lambda: samrs.qkv_split_window(a @ w.T, bias, images, 64, 64, 14, nh, hd)
            ref_name = "torch matmul (cuBLAS) + qkv_split_window kernel"
        elif "gelu" in name:
            ours = lambda: samrs.linear(a, w, bias, epilogue="bias_gelu")
            ref = lambda: F.gelu(F.linear(a, w, bias))
            ref_name = "torch F.linear (cuBLAS, bias in the epilogue) + F.gelu"
        else:
            ours = lambda: samrs.linear(a, w, bias, res=res, epilogue="bias_residual")
            ref = lambda: torch.addmm(bias, a, w.T).add_(res)
            ref_name = "torch addmm (cuBLAS) + add"
        ms, ms_ref = timed(ours), timed(ref)
        out[name] = {"shape": [t, n, k], "ms": ms, "tflops": flops / (ms / 1e3) / 1e12,
                     "frac_of_bf16_peak": flops / (ms / 1e3) / 1e12 / tf_peak, "torch_ms": ms_ref,
                     "torch_tflops": flops / (ms_ref / 1e3) / 1e12, "torch_path": ref_name}
    if samrs.device_status() != 0:
        raise RuntimeError("device status word set by the GEMMs")
    return out


def run_config3(torch, samrs, lib, device, rank, sptr, stream, dist, world, steps, warmup):
    """BASELINE config 3 (ViT-L, 16 images per GPU, hd 64, 24 layers), timed like the headline."""
    step = Step(torch, lib, CONFIGS[3], CONFIGS[3].images, device, rank, sptr)
    _, max_ms, per_kind = time_workload(torch, samrs, step, stream, dist, device, steps, warmup, per_launch=True)
    out = summary_line(step, world, steps, max_ms)
    out["workload"] = "config 3: " + CONFIGS[3].describe()
    for kind in KINDS:
        _, h, w, bh = next(g for g in step.geoms if g[0] == kind)
        ms = statistics.mean(per_kind[kind])
        out[f"{kind}_ms"] = ms
        out[f"{kind}_tflops"] = layer_flops(h, w, bh, 64) / (ms / 1e3) / 1e12
        out[f"{kind}_gbs"] = layer_bytes(h, w, bh, 64) / (ms / 1e3) / 1e9
    out["checksums_rank0"] = step.checksums() if rank == 0 else None
    del step
    torch.cuda.empty_cache()
    return out


def run_config1(torch, samrs, device, reps=20, warmup=3):
    """the ViT-B op in f32, one image (windowed: 25 windows x 12 heads of 14x14, hd 64;
    global: 12 heads of 64x64, hd 64; tables N(0, 0.5)). Each layer through the f32 tensor-core kernel (3xTF32
    tcgen05, the library's default for f32) and through the CUDA-core kernel, L2 flushed before every timed
    launch (the inputs fit in L2). Also the f32 kernel at the config-4 layer shapes (32 ViT-H images)."""
    g = torch.Generator(device=device).manual_seed(101)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)

    def timed(fn):
        for _ in range(warmup):
            fn()
        total = 0.0
        for _ in range(reps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            b.synchronize()
            total += a.elapsed_time(b)
        return total / reps

    out = {"workload": "config 1: ViT-B attention op, f32, 1 image (windowed 300 heads 14x14 + global 12 heads 64x64, "
                       "hd 64); L2 flushed before each timed launch"}
    for kind, h, bh, hd, impls in (("window", 14, 300, 64, ("tc", "simt")), ("global", 64, 12, 64, ("tc", "simt")),
                                   ("window_vith32", 14, 12800, 80, ("tc",)), ("global_vith32", 64, 512, 80, ("tc",))):
        n = h * h
        q = torch.randn(bh, n, hd, device=device, generator=g)
        kt = torch.randn(bh, hd, n, device=device, generator=g)
        v = torch.randn(bh, n, hd, device=device, generator=g)
        t = torch.randn(4 * h - 2, hd, device=device, generator=g) * 0.5
        o = torch.empty_like(q)
        for impl in impls:
            ms = timed(lambda: samrs.attention_relpos(q, kt, v, t, h, h, hd ** -0.5, impl=impl, out=o))
            out[f"{kind}_{impl}_ms"] = ms
            out[f"{kind}_{impl}_tflops"] = layer_flops(h, h, bh, hd) / (ms / 1e3) / 1e12
        del q, kt, v, o
    if samrs.device_status() != 0:
        raise RuntimeError("device status word set by the f32 layers")
    out["layer_ms_tc"] = out["window_tc_ms"] + out["global_tc_ms"]
    out["layer_ms_simt"] = out["window_simt_ms"] + out["global_simt_ms"]
    del flush
    torch.cuda.empty_cache()
    return out


def config1_e2e(torch, samrs, device, steps, warmup):
    """Config 1 end to end through the library's public call: each step copies both layers' q, kt, v from
    pinned host memory, runs the two f32 layers, and copies both outputs back (one stream, CUDA events)."""
    g = torch.Generator().manual_seed(5)
    layers = []
    h2d = d2h = 0
    for h, bh in ((14, 300), (64, 12)):
        n, hd = h * h, 64
        host = [torch.randn(*shape, generator=g).pin_memory() for shape in ((bh, n, hd), (bh, hd, n), (bh, n, hd))]
        dev = [torch.empty_like(x, device=device) for x in host]
        t = (torch.randn(4 * h - 2, hd, generator=g) * 0.5).to(device)
        out, out_host = torch.empty_like(dev[0]), torch.empty_like(host[0]).pin_memory()
        layers.append((h, hd, host, dev, t, out, out_host))
        h2d += sum(x.numel() * 4 for x in host)
        d2h += out_host.numel() * 4

    def step():
        for h, hd, host, dev, t, out, out_host in layers:
            for d, x in zip(dev, host):
                d.copy_(x, non_blocking=True)
            samrs.attention_relpos(dev[0], dev[1], dev[2], t, h, h, hd ** -0.5, out=out)
            out_host.copy_(out, non_blocking=True)

    for _ in range(warmup):
        step()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record()
    for _ in range(steps):
        step()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    flops = layer_flops(14, 14, 300, 64) + layer_flops(64, 64, 12, 64)
    return {"value": flops / (ms / 1e3) / 1e12, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": ms, "path": "samrs.attention_relpos (C ABI), pinned host buffers, one stream"}


def run_sweep(torch, samrs, lib, device, rank, sptr, stream, dist, world, steps, warmup):
    """config 4 at 8, 16, 32, 64 and 128 images per GPU."""
    rows = []
    for images in SWEEP_IMAGES:
        step = Step(torch, lib, CONFIGS[4], images, device, rank, sptr)
        _, max_ms, _ = time_workload(torch, samrs, step, stream, dist, device, steps, warmup)
        rows.append(summary_line(step, world, steps, max_ms))
        del step
        torch.cuda.empty_cache()
    return rows


def recompute_rates(torch, samrs, lib, device, sptr, images=8, reps=5):
    """Share of bf16 global-layer CTAs the exact second pass recomputes, by rel-pos table std (activations
    N(0,1)), and one case with activations N(0,2) as well; the library's per-layer choice after that first
    (measured) call, and the time of the first call (speculative pass + fixup) against the mean of the next
    `reps` calls (the exact kernel alone where the choice switched). The choices are forgotten afterwards."""
    out, policy = {}, {}
    gen = torch.Generator(device=device).manual_seed(77)
    bh, n, hd = images * 16, 4096, HD
    for label, a_std, t_std in (("t0.5", 1.0, 0.5), ("t1", 1.0, 1.0), ("t2", 1.0, 2.0), ("t2_a2", 2.0, 2.0)):
        q = (torch.randn(bh, n, hd, device=device, generator=gen) * a_std).bfloat16()
        kt = (torch.randn(bh, hd, n, device=device, generator=gen) * a_std).bfloat16()
        v = torch.randn(bh, n, hd, device=device, generator=gen).bfloat16()
        t = (torch.randn(254, hd, device=device, generator=gen) * t_std).bfloat16()
        o = torch.empty_like(q)

        def call():
            rc = lib.samrs_relpos_attn_fwd(q.data_ptr(), kt.data_ptr(), v.data_ptr(), t.data_ptr(), o.data_ptr(), bh,
                                           64, 64, hd, hd ** -0.5, 2, sptr)
            if rc != 0:
                raise RuntimeError(lib.samrs_last_error().decode())

        samrs.global_policy(t, reset=True)
        samrs.recompute_count(clear=True)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        call()
        b.record()
        out[label] = samrs.recompute_count(clear=True) / (bh * 16)
        share, exact = samrs.global_policy(t)
        first_ms = a.elapsed_time(b)
        a.record()
        for _ in range(reps):
            call()
        b.record()
        b.synchronize()
        policy[label] = {"measured_share": share, "switched_to_exact": exact, "first_call_ms": first_ms,
                         "next_calls_ms": a.elapsed_time(b) / reps}
        samrs.recompute_count(clear=True)
    samrs.global_policy(t, reset=True)
    return out, policy


def run_neighbours(samrs, lib, images, device, sptr, hbm, wl, reps=10):
    """The path's neighbours on the token grid at the bench workload (not part of the metric): the qkv
    split fused with the window partition and the head merge fused with the unpartition, for the windowed
    (ws 14, pad 64 -> 70) and the global (one 64x64 window) layers. Algorithmic bytes: the real tokens'
    y (3C) read and q, kt, v (pads included) written; the real tokens' attention rows read and written."""
    import torch
    nh, hd, es = wl.heads, wl.hd, 2
    c = nh * hd
    out = {}
    gen = torch.Generator(device=device).manual_seed(5)
    y = (torch.randn(images * 4096, 3 * c, device=device, generator=gen) * 0.5).to(torch.bfloat16)
    bias = (torch.randn(3 * c, device=device, generator=gen) * 0.1).to(torch.bfloat16)
    for name, ws in (("window", 14), ("global", 0)):
        n, nwin = (196, 25) if ws else (4096, 1)
        bh = images * nwin * nh
        packed = torch.empty(3 * bh * n * hd, device=device, dtype=torch.bfloat16)
        attn = torch.empty(bh, n, hd, device=device, dtype=torch.bfloat16)
        merged = torch.empty(images * 4096, c, device=device, dtype=torch.bfloat16)
        calls = {
            "qkv_split_window": (lambda: lib.samrs_qkv_split_window_fwd(
                y.data_ptr(), bias.data_ptr(), packed.data_ptr(), images, 64, 64, ws, nh, hd, 2, sptr),
                images * 4096 * 3 * c * es + 3 * bh * n * hd * es),
            "window_merge": (lambda: lib.samrs_window_merge_fwd(
                attn.data_ptr(), merged.data_ptr(), images, 64, 64, ws, nh, hd, 2, sptr),
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


def copy_bandwidth(torch, device, dist, nbytes=1 << 30, reps=4, ratio=1):
    """Measured pinned host <-> device copy bandwidth of this rank (GB/s), with every rank copying at the same
    time (the host side is shared): one cudaMemcpyAsync per buffer, H2D and D2H each alone, then both at once
    on two streams with `ratio` bytes up per byte down, as the e2e step moves them ("both": the aggregate)."""
    host = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    host2 = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    dev = torch.empty(nbytes, dtype=torch.uint8, device=device)
    dev2 = torch.empty(nbytes, dtype=torch.uint8, device=device)
    s1, s2 = torch.cuda.Stream(device), torch.cuda.Stream(device)
    res = {}
    for name in ("h2d", "d2h", "both"):
        dev.copy_(host, non_blocking=True)
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        up = reps * (ratio if name == "both" else 1)
        for i in range(max(up, reps)):
            if name in ("h2d", "both") and i < up:
                with torch.cuda.stream(s1):
                    dev.copy_(host, non_blocking=True)
            if name in ("d2h", "both") and i < reps:
                with torch.cuda.stream(s2):
                    host2.copy_(dev2, non_blocking=True)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        moved = {"h2d": reps, "d2h": reps, "both": up + reps}[name]
        res[name] = nbytes * moved / dt / 1e9
    del host, host2, dev, dev2
    return res


def run_e2e(args, samrs, step, device, stream, dist, world, device_ms_per_step):
    """Same workload through the C ABI with host (pinned) buffers: every layer copies its q, kt, v
    host->device, runs the op, and copies its output device->host, all inside the timed region.
    Serving-style pipelining: two device buffer sets per layer kind and three streams (upload, compute,
    download) ordered by events, so layer l+1's upload, layer l's kernel and layer l-1's download overlap
    (PCIe is full duplex). The roofline of this leg is the host link: the measured pinned-copy bandwidth
    of the box at this world size."""
    import torch
    sets = step.sets
    host = {}
    dev = {}
    for kind in KINDS:
        s = sets[kind]
        host[kind] = {k: torch.empty(s[k].shape, dtype=s[k].dtype, pin_memory=True) for k in ("q", "kt", "v", "out")}
        for k in ("q", "kt", "v"):
            host[kind][k].copy_(s[k])
        dev[kind] = [s, {k: torch.empty_like(s[k]) for k in ("q", "kt", "v", "out")}]
    torch.cuda.synchronize()
    s_up, s_down = torch.cuda.Stream(device), torch.cuda.Stream(device)
    sptr = stream.cuda_stream
    # per (kind, buffer): the compute that last read the inputs / wrote the output, the download of it
    comp_done = {k: [None, None] for k in KINDS}
    down_done = {k: [None, None] for k in KINDS}
    h2d = d2h = 0

    def one_step():
        nonlocal h2d, d2h
        h2d = d2h = 0
        use = {k: 0 for k in KINDS}
        for li, (kind, h, w, bh) in enumerate(step.geoms):
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
            step.launch(li, sets={kind: d}, stream_ptr=sptr)
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

    one_step()
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
        one_step()
    join()
    b.record(stream)
    torch.cuda.synchronize()
    local_ms = a.elapsed_time(b)
    ms = max_over_ranks(local_ms, dist, device)
    del host, dev
    torch.cuda.empty_cache()
    bw = copy_bandwidth(torch, device, dist, ratio=max(1, round(h2d / max(d2h, 1))))
    bw_min = {kname: max_over_ranks(-v, dist, device) * -1 for kname, v in bw.items()}  # slowest rank
    step_s = local_ms / k / 1e3
    # the host-link bound of one step: uploads and downloads overlap (full duplex), and neither beats the
    # measured copy rates; the device compute is the third term
    bound_s = max(h2d / (bw_min["h2d"] * 1e9), d2h / (bw_min["d2h"] * 1e9), (h2d + d2h) / (bw_min["both"] * 1e9),
                  device_ms_per_step / 1e3)
    return {"value": step.flops * k * world / (ms / 1e3) / 1e12, "unit": UNIT, "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "steps": k, "ms_per_step": ms / k,
            "h2d_gbs": h2d / step_s / 1e9, "d2h_gbs": d2h / step_s / 1e9,
            "copy_gbs_measured": bw_min,
            "roofline": {"bound": "host link (pinned cudaMemcpyAsync, all ranks at once)", "bound_ms_per_step":
                         bound_s * 1e3, "frac": bound_s / (ms / k / 1e3)},
            "path": "C ABI samrs_relpos_attn_fwd, pinned host buffers, upload/compute/download streams"}


def run_library_context(args):
    """Context for the attention kernels' rooflines: the fused rel-pos kernels against the library's plain
    attention (torch SDPA on its cuDNN backend, no bias at all: less work than the fused op) on the same
    shapes, one GPU. Each is run back to back for `--context-seconds` in alternating phases (ours, library,
    ours, library) with the clocks sampled during each phase, so that the two are compared at the clocks the
    power cap leaves each of them. Prints one JSON line ("impl": "library-context")."""
    import torch
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    samrs = importlib.import_module("sam-rs_b200")
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    peaks = load_peaks()
    g = torch.Generator(device=device).manual_seed(11)
    images, heads, hd = 32, VIT_H["heads"], VIT_H["hd"]

    def phase(fn, secs):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        times = []
        with ClockSampler(0) as clk:
            t0 = time.time()
            while time.time() - t0 < secs:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                for _ in range(5):
                    fn()
                b.record()
                b.synchronize()
                times.append(a.elapsed_time(b) / 5)
        c = clk.summary()
        ms = statistics.median(times)
        return {"ms": ms, "min_ms": min(times), "launches": 5 * len(times), "sm_mhz": c["sm_mhz"],
                "power_w": c["power_w"], "reasons": c["reasons"],
                "mcycles_per_launch": ms * c["sm_mhz"] / 1e3 if c["sm_mhz"] else None}

    out = {"impl": "library-context", "n_gpus": 1, "dtype": "bf16", "data": "synthetic (seeded N(0,1), tables N(0,0.5))",
           "library": f"torch {torch.__version__} scaled_dot_product_attention, cuDNN backend "
                      f"{torch.backends.cudnn.version()}, no bias",
           "peaks": {"hbm_gbs": peaks[0], "bf16_burst_tflops": peaks[1], "bf16_sustained_tflops": peaks[2],
                     "source": peaks[3]}, "layers": {}}
    for kind, side, bh in (("global", 64, images * heads), ("window", 14, images * 25 * heads)):
        n = side * side
        q = torch.randn(bh, n, hd, device=device, generator=g).bfloat16()
        kt = torch.randn(bh, hd, n, device=device, generator=g).bfloat16()
        v = torch.randn(bh, n, hd, device=device, generator=g).bfloat16()
        t = (torch.randn(4 * side - 2, hd, device=device, generator=g) * 0.5).bfloat16()
        b = bh // heads
        q4, v4 = q.view(b, heads, n, hd), v.view(b, heads, n, hd)
        k4 = kt.view(b, heads, hd, n).transpose(2, 3).contiguous()

        def ours():
            samrs.attention_relpos(q, kt, v, t, side, side, hd ** -0.5, impl="tc")

        def library():
            with sdpa_kernel([SDPBackend.CUDNN_ATTENTION]):
                F.scaled_dot_product_attention(q4, k4, v4)

        flops, nbytes = layer_flops(side, side, bh, hd), layer_bytes(side, side, bh, hd)
        res = {"bh": bh, "tokens": n, "hd": hd, "gflop": flops / 1e9, "algorithmic_mb": nbytes / 1e6}
        for rnd in range(2):
            for name, fn in (("fused_relpos", ours), ("cudnn_sdpa_no_bias", library)):
                try:
                    r = phase(fn, args.context_seconds)
                except RuntimeError as e:
                    r = {"unavailable": str(e).splitlines()[0][:160]}
                if "ms" in r:
                    r["tflops"] = flops / r["ms"] / 1e9
                    r["gbs"] = nbytes / r["ms"] / 1e6
                res.setdefault(name, []).append(r)
        out["layers"][kind] = res
        del q, kt, v, q4, k4, v4
        torch.cuda.empty_cache()
    print(json.dumps(out), flush=True)
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, choices=[1, 2, 3, 4, 5], default=4)
    ap.add_argument("--images", type=int, default=0, help="images per GPU (default: the config's, 32 for config 4)")
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip configs 3 and 5 in the default config-4 run")
    ap.add_argument("--no-neighbours", action="store_true", help="skip timing the qkv split / head merge kernels")
    ap.add_argument("--reference-path", choices=["cpu", "cuda"], default="cpu",
                    help="with --impl reference: the reference's CPU path (default; the oracle's restatement) or "
                         "its own CUDA kernels (oracle/_ref, built from its kernels/sam.cu) on this GPU")
    ap.add_argument("--library-context", action="store_true",
                    help="time the attention kernels against torch SDPA (cuDNN, no bias) on the same shapes")
    ap.add_argument("--context-seconds", type=float, default=6.0)
    args = ap.parse_args(argv)
    if args.library_context:
        return run_library_context(args)
    if args.warmup < 3:
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
