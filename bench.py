#!/usr/bin/env python3
"""Benchmark of the NOVA F(6,3) Winograd conv forward on B200.

Workload: the ResNet-50 3x3 stride-1 layer sweep
C = K = 64 @ 56x56, 128 @ 28x28, 256 @ 14x14, 512 @ 7x7, FP16 N(0,1) inputs,
FP32 Kaiming-normal weights, synthetic seeded data.  One step = one forward of
each of the four layers at batch --batch (default 128, the sweep's largest) per
GPU.  Metric: effective TFLOP/s = direct-conv FLOPs (2*B*K*C*H_out*W_out*9) /
time.  Multi-GPU: one process per GPU, each runs the same per-GPU batch (batch
partitioning, no collective on the data path) -> weak scaling.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl nova|reference]

Prints one JSON line on rank 0.  --impl reference times the reference's CPU
implementation of this path (the NOVA transform math, restated in
oracle/nova_oracle.py because the reference's HIP code cannot run here) on the
host cores, on a bounded sample of the same workload.
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (os.path.join(ROOT, "nova-wino-amd_b200"), os.path.join(ROOT, "oracle")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

LAYERS = [  # (name, C = K, H = W)
    ("conv2_x", 64, 56),
    ("conv3_x", 128, 28),
    ("conv4_x", 256, 14),
    ("conv5_x", 512, 7),
]
# SD 1.5 UNet 3x3 stride-1 shapes at a 64x64 latent (configs 4 and 5 use these
# channel counts): per-layer timing only, the UNet model itself is not built.
UNET_LAYERS = [
    ("sd_320_64", 320, 64),
    ("sd_640_32", 640, 32),
    ("sd_1280_16", 1280, 16),
    ("sd_1280_8", 1280, 8),
]
# SDXL UNet 3x3 stride-1 shapes at a 128x128 latent (config 5).
SDXL_LAYERS = [
    ("sdxl_320_128", 320, 128),
    ("sdxl_640_64", 640, 64),
    ("sdxl_1280_32", 1280, 32),
]
METRIC = "F(6,3) conv eff. TFLOP/s (direct-conv FLOPs / time), ResNet-50 3x3 s1 layer sweep"
UNIT = "TFLOP/s"
L2_BYTES = 126 * 1024 * 1024
PARITY_TOL = 1e-2      # rel L2 against the oracle (tests/test_gpu_parity.py)
ACCURACY_FACTOR = 1.1  # error vs FP64 direct conv <= 1.1x the oracle's


def direct_flops(B, C, K, H):
    return 2.0 * B * K * C * H * H * 9


def live_tiles(H):
    return -(-H // 6)


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


# ---------------------------------------------------------------------------
# CPU side: the oracle restatement of the reference's NOVA math.
# ---------------------------------------------------------------------------

def cpu_nova_sample(batch, seconds_budget=12.0):
    """Times the NOVA FP32 math (reference precision) on the host on a bounded
    sample: each sweep layer at `batch`, filter transform precomputed (the GPU
    path caches it too).  Returns (TFLOP/s, threads, sample text, extra)."""
    import numpy as np
    import nova_oracle as o
    cases = []
    for name, C, H in LAYERS:
        x, w = o.synthetic_case(batch, C, C, H, H, seed=1234 + C)
        U = o.filter_transform(w, "ref")
        cases.append((name, C, H, x, U))

    def one_pass():
        for name, C, H, x, U in cases:
            nh = nw = live_tiles(H)
            V = o.input_transform(x, nh, nw, 1, "ref")
            M = o.gemm(U, V, "ref")
            o.output_transform(M, batch, nh, nw, H, H, "ref")

    one_pass()  # warm-up
    reps, t0 = 0, time.perf_counter()
    while True:
        one_pass()
        reps += 1
        el = time.perf_counter() - t0
        if el > seconds_budget or reps >= 20:
            break
    flops = reps * sum(direct_flops(batch, C, C, H) for _, C, H in LAYERS)
    threads = len(os.sched_getaffinity(0))
    sample = f"{reps} pass(es) of the 4 sweep layers at batch {batch}"
    extra = {}
    try:  # F.conv2d FP32 on the same sample, for context
        import torch
        import torch.nn.functional as F
        torch.set_num_threads(threads)
        xs = [torch.from_numpy(c[3].astype(np.float32)) for c in cases]
        ws = [torch.randn(C, C, 3, 3) for _, C, _ in LAYERS]
        for xx, ww in zip(xs, ws):
            F.conv2d(xx, ww, padding=1)
        t1 = time.perf_counter()
        for xx, ww in zip(xs, ws):
            F.conv2d(xx, ww, padding=1)
        dt = time.perf_counter() - t1
        extra["torch_conv2d_fp32_tflops"] = sum(direct_flops(batch, C, C, H)
                                                for _, C, H in LAYERS) / dt / 1e12
    except Exception as e:  # pragma: no cover
        extra["torch_conv2d_fp32_error"] = str(e)
    return flops / el / 1e12, threads, sample, extra


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cpu_batch = args.cpu_batch
    for _ in range(max(1, args.warmup)):
        cpu_nova_sample(cpu_batch, seconds_budget=2.0)
    vals, sample, threads = [], "", 1
    for _ in range(args.steps):
        v, threads, sample, _ = cpu_nova_sample(cpu_batch, seconds_budget=4.0)
        vals.append(v)
    value = statistics.median(vals)
    # The GPU arm's workload: every sweep layer at --batch per GPU.  Each step
    # times a per-image sample of it (cpu_batch images of each layer); the
    # metric is a throughput, so ms_per_step is that of the whole batch.
    flops_step = sum(direct_flops(args.batch, C, C, H) for _, C, H in LAYERS)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": flops_step / (value * 1e12) * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) FP16 inputs, Kaiming-normal FP32 weights)",
        "config": {"workload": "resnet50_3x3_sweep", "layers": [l[0] for l in LAYERS],
                   "batch_per_gpu": args.batch, "parallelism": f"dp{world} (batch-partitioned)",
                   "l2": "n/a (host)"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{sample}, i.e. {cpu_batch} of the {args.batch} images of "
                                   "each layer per step", "cpu_model": cpu_model()},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference is HIP/rocBLAS for MI300X and cannot run here; its NOVA math is "
                "timed as the numpy restatement (oracle/nova_oracle.py) on the host cores",
    }
    emit(line)


# ---------------------------------------------------------------------------
# GPU side.
# ---------------------------------------------------------------------------

class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id):
        self.gpu_id = gpu_id
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu_id), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["sampler unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) == 7:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        smax = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[3 + i] == "Active"})
        pw = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": reasons,
                "samples": len(rows),
                "power_w_median": statistics.median(pw) if pw else None}


def setup_dist():
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    return world, rank, local, dist


def barrier(dist):
    import torch
    if dist is not None:
        dist.barrier()
    if torch.cuda.is_available():
        torch.cuda.synchronize()


def max_over_ranks(dist, value):
    """Max of a per-rank time over all ranks (NCCL tensors on the GPU, gloo on CPU)."""
    import torch
    if dist is None:
        return value
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def build_layers(batch, device, shapes=None):
    import numpy as np
    import torch
    from nova_winograd import NovaWinogradConv2d
    layers = []
    for name, C, H in (shapes or LAYERS):
        rng = np.random.default_rng(1234 + C)
        x = torch.from_numpy(rng.standard_normal((batch, C, H, H), dtype=np.float32)).to(
            device=device, dtype=torch.float16)
        w = torch.from_numpy(rng.standard_normal((C, C, 3, 3), dtype=np.float32)
                             * np.float32(np.sqrt(2.0 / (9 * C))))
        conv = NovaWinogradConv2d(C, C, kernel_size=3, padding=1).to(device)
        with torch.no_grad():
            conv.weight.copy_(w)
        layers.append((name, C, H, conv, x))
    return layers


def make_flush(device):
    import torch
    wr = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=device)
    rd = torch.ones(2 * L2_BYTES // 4, dtype=torch.float32, device=device)

    def flush():
        # Write a buffer twice the L2 size, then read another one: the read
        # evicts the dirty lines the write left, so their write-back does not
        # land on the next timed kernel.
        wr.fill_(1.0)
        rd.sum()
    return flush


def time_kernel(fn, reps, flush):
    """Mean device time (ms) of fn() with an L2 flush before each launch (one
    untimed call first).  CUDA event timestamps on this platform advance in
    steps of about 2.05 us, so a median of single launches is quantised to that
    step; the mean over launches whose start falls at random phases of the step
    is not."""
    import torch
    fn()
    evs = []
    for _ in range(reps):
        flush()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        evs.append((s, e))
    torch.cuda.synchronize()
    return statistics.mean(s.elapsed_time(e) for s, e in evs)


def stage_profile(layers, batch, flush, reps=20, nhwc=False):
    """Per-stage device times through the stage C-ABI entries (one launch each,
    whole batch), with the algorithmic bytes / FLOPs of each launch.  nhwc:
    the channels-last stage entries on the channels-last copies of the inputs
    (the same bytes: x and y hold the same elements in either layout)."""
    import torch
    from nova_winograd import ops
    lib = ops.get_lib()
    out = []
    for name, C, H, conv, x in layers:
        if nhwc:
            x = x.contiguous(memory_format=torch.channels_last)
        nt = live_tiles(H)
        BP = batch * nt * nt
        V = torch.empty(64, BP, C, dtype=torch.float16, device=x.device)
        M = torch.empty(64, BP, C, dtype=torch.float16, device=x.device)
        y = torch.empty(batch, C, H, H, dtype=torch.float16, device=x.device)
        conv(x)  # make sure the handle holds the weights
        h = conv._handle
        s = ops.stream_ptr()

        it_fn = lib.nova_input_transform_nhwc_v2 if nhwc else lib.nova_input_transform_v2
        ot_fn = lib.nova_output_transform_nhwc_v2 if nhwc else lib.nova_output_transform_v2
        if nhwc:
            y = y.contiguous(memory_format=torch.channels_last)

        def it():
            ops.check(it_fn(ops.ptr(x), ops.ptr(V), batch, C, H, H, 1, nt, nt, BP, s),
                      "input_transform")

        def gm():
            ops.check(lib.nova_batched_gemm_v2(h, ops.ptr(V), ops.ptr(M), BP, s), "gemm")

        def ot():
            ops.check(ot_fn(ops.ptr(M), ops.ptr(y), batch, C, H, H, nt, nt, BP, s),
                      "output_transform")

        x_b = y_b = batch * C * H * H * 2
        v_b = m_b = 64 * BP * C * 2
        u_b = 64 * C * C * 2
        gflop = 2.0 * 64 * C * C * BP
        sfx = "_nhwc" if nhwc else ""
        for kname, fn, nbytes, flops in (
                ("input_transform_kernel" + sfx, it, x_b + v_b, 0.0),
                ("gemm_tc_kernel", gm, v_b + u_b + m_b, gflop),
                ("output_transform_kernel" + sfx, ot, m_b + y_b, 0.0)):
            ms = time_kernel(fn, reps, flush)
            out.append({"layer": name, "kernel": kname, "ms": ms, "bytes": nbytes,
                        "flops": flops, "gbs": nbytes / ms / 1e6,
                        "tflops": flops / ms / 1e9 if flops else None})
    return out


def vendor_layer_times(layers, flush, reps=20, channels_last=False):
    """Whole-layer device time of our forward and of torch's FP16 conv2d (cuDNN)
    on the same layer, L2 flushed before each launch (context, like the
    reference's MIOpen comparison in benchmarks/bench_layers.py).  With
    channels_last, also both on the channels-last copy of the input (our NHWC
    kernels; cuDNN's channels-last kernels), with the NHWC outputs of sampled
    images checked against the oracle."""
    import torch
    import torch.nn.functional as F
    res = {}
    torch.backends.cudnn.benchmark = True
    for name, C, H, conv, x in layers:
        w16 = conv.weight.detach().half()
        with torch.no_grad():
            for _ in range(3):  # cuDNN algorithm selection happens here
                F.conv2d(x, w16, padding=1)
        with torch.no_grad():
            ours = time_kernel(lambda: conv(x), reps, flush)
            cudnn = time_kernel(lambda: F.conv2d(x, w16, padding=1), reps, flush)
        fl = direct_flops(x.shape[0], C, C, H)
        res[name] = {"nova_us": round(ours * 1e3, 1), "cudnn_fp16_us": round(cudnn * 1e3, 1),
                     "nova_eff_tflops": round(fl / ours / 1e9, 1),
                     "cudnn_eff_tflops": round(fl / cudnn / 1e9, 1)}
        if channels_last:
            xl = x.contiguous(memory_format=torch.channels_last)
            wl = w16.contiguous(memory_format=torch.channels_last)
            with torch.no_grad():
                for _ in range(3):
                    F.conv2d(xl, wl, padding=1)
                yl = conv(xl)
                ours_cl = time_kernel(lambda: conv(xl), reps, flush)
                cudnn_cl = time_kernel(lambda: F.conv2d(xl, wl, padding=1), reps, flush)
            torch.cuda.synchronize()
            par = sample_parity(name, x, conv.weight, yl.contiguous())
            res[name].update({
                "nova_nhwc_us": round(ours_cl * 1e3, 1),
                "cudnn_fp16_channels_last_us": round(cudnn_cl * 1e3, 1),
                "nova_nhwc_eff_tflops": round(fl / ours_cl / 1e9, 1),
                "cudnn_channels_last_eff_tflops": round(fl / cudnn_cl / 1e9, 1),
                "nhwc_output_channels_last": bool(yl.is_contiguous(
                    memory_format=torch.channels_last)),
                "nhwc_parity": {k: par[k] for k in ("images", "rel_l2_vs_oracle", "ok")}})
            del xl, yl
    return res


# DRAM bytes (read, write) per launch at batch 128, from one ncu capture of the
# stage entries (bench.py --profile-stages, one launch per kernel and layer).
# ncu flushes the caches before each kernel and counts no write-back of lines
# still dirty in L2 when the kernel ends, so the writes of V and M that stay in
# the 126 MB L2 are missing here; the totals therefore sit below the algorithmic
# bytes rather than above them (no kernel re-reads its input).
NCU_DRAM_BYTES_B128 = {
    "conv2_x": {"input_transform_kernel": (51412736, 43130112),
                "gemm_tc_kernel": (105418496, 55179776),
                "output_transform_kernel": (104874752, 16134656)},
    "conv3_x": {"input_transform_kernel": (25713664, 752640),
                "gemm_tc_kernel": (54562816, 3790848),
                "output_transform_kernel": (52446464, 66560)},
    "conv4_x": {"input_transform_kernel": (12875520, 0),
                "gemm_tc_kernel": (46173952, 204544),
                "output_transform_kernel": (37768448, 0)},
    "conv5_x": {"input_transform_kernel": (6443264, 0),
                "gemm_tc_kernel": (67145216, 401664),
                "output_transform_kernel": (33572352, 0)},
}


def ncu_traffic(kernel, batch):
    """Mean DRAM bytes per launch of `kernel` over the sweep layers (ncu), scaled
    from batch 128 by the tiles processed; None when no capture applies."""
    vals = [sum(v[kernel]) for v in NCU_DRAM_BYTES_B128.values() if kernel in v]
    if not vals:
        return None
    return sum(vals) / len(vals) * batch / 128.0


def roofline_from_stages(stages, peaks, batch=128):
    by_kernel = {}
    for s in stages:
        d = by_kernel.setdefault(s["kernel"], {"ms": 0.0, "bytes": 0.0, "flops": 0.0, "n": 0})
        d["ms"] += s["ms"]
        d["bytes"] += s["bytes"]
        d["flops"] += s["flops"]
        d["n"] += 1
    top = max(by_kernel, key=lambda k: by_kernel[k]["ms"])
    d = by_kernel[top]
    t_hbm = d["bytes"] / (peaks["hbm_gbs"] * 1e9)
    t_tc = d["flops"] / (peaks["bf16_tflops"] * 1e12)
    if t_tc > t_hbm:
        achieved = d["flops"] / (d["ms"] / 1e3) / 1e12
        rl = {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
              "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"]}
    else:
        achieved = d["bytes"] / (d["ms"] / 1e3) / 1e9
        rl = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
              "frac": achieved / peaks["hbm_gbs"]}
    tot = sum(x["ms"] for x in by_kernel.values())
    rl.update({"kernel": top, "launches_per_step": d["n"], "avg_launch_ms": d["ms"] / d["n"],
               "traffic": ncu_traffic(top, batch), "traffic_unit": "bytes per launch (ncu)",
               "algorithmic_bytes_per_launch": d["bytes"] / d["n"],
               "peak_source": peaks["source"],
               "shares": {k: v["ms"] / tot for k, v in by_kernel.items()}})
    return rl


def b1_latency(device, reps=200, nhwc=True):
    """Per-layer batch-1 latency (us): back-to-back module calls (host overhead
    included) and the same call replayed from a CUDA graph (device only); the
    same for the channels-last input (the NHWC kernels) under "nhwc"."""
    import torch
    res = {}
    for name, C, H, conv, x in build_layers(1, device):
        res[name] = _b1_one(conv, x, C, H, reps)
        if nhwc:
            res[name]["nhwc"] = _b1_one(conv, x.contiguous(memory_format=torch.channels_last), C,
                                        H, reps)
    return res


def _b1_one(conv, x, C, H, reps):
    """Eager and graph-replayed batch-1 latency of one layer (see b1_latency)."""
    import torch
    for _ in range(20):
        conv(x)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        conv(x)
    e.record()
    torch.cuda.synchronize()
    us_eager = s.elapsed_time(e) / reps * 1e3
    g = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        conv(x)
        st.synchronize()
        with torch.cuda.graph(g, stream=st):
            for _ in range(10):
                conv(x)
    torch.cuda.synchronize()
    g.replay()
    torch.cuda.synchronize()
    s.record()
    for _ in range(reps // 10):
        g.replay()
    e.record()
    torch.cuda.synchronize()
    us_graph = s.elapsed_time(e) / reps * 1e3
    return {"us_eager": round(us_eager, 2), "us_graph": round(us_graph, 2),
            "eff_tflops_graph": round(direct_flops(1, C, C, H) / us_graph / 1e6, 2)}


class _TorchCuda:
    """The CUDA primitives the pipelined end-to-end loop uses (a CPU test
    substitutes fakes)."""

    def __init__(self):
        import torch
        self.torch = torch

    def stream(self):
        return self.torch.cuda.Stream()

    def current(self):
        return self.torch.cuda.current_stream()

    def event(self, timing=False):
        return self.torch.cuda.Event(enable_timing=timing)

    def use(self, stream):
        return self.torch.cuda.stream(stream)

    def synchronize(self):
        self.torch.cuda.synchronize()


def e2e_pipelined(hx, dx, hy, forwards, steps, cu, before_timing=None):
    """End to end with the copies overlapped: every step copies each layer's
    pinned host input to the device, runs the layer, and copies its output back
    to pinned host memory.  Host-to-device copies run on one stream and
    device-to-host copies on another, so layer i + 1's input crosses PCIe while
    layer i computes and layer i - 1's output returns.  A device input buffer
    is refilled only after the forward that read it.  Each output is held by
    reference until the next step's forward of the same layer, and that forward
    first waits (on the compute stream) for the output's copy out: only then is
    the old output released, so the allocator can hand its memory to later
    compute-stream work only after the copy has read it.  Returns the elapsed ms
    of the ``steps`` steps (CUDA events on the compute stream, which waits for
    the last copy out)."""
    comp = cu.current()
    s_in, s_out = cu.stream(), cu.stream()
    consumed = [None] * len(hx)
    copied = [None] * len(hx)
    held = [None] * len(hx)
    start, end = cu.event(True), cu.event(True)
    if before_timing is not None:
        before_timing()
    start.record(comp)
    s_in.wait_event(start)
    for _ in range(steps):
        for i, fwd in enumerate(forwards):
            with cu.use(s_in):
                if consumed[i] is not None:
                    s_in.wait_event(consumed[i])
                dx[i].copy_(hx[i], non_blocking=True)
                landed = cu.event()
                landed.record(s_in)
            comp.wait_event(landed)
            if copied[i] is not None:
                comp.wait_event(copied[i])
                held[i] = None  # its copy out is ordered before all later compute work
            y = fwd(dx[i])
            held[i] = y
            done = cu.event()
            done.record(comp)
            consumed[i] = done
            with cu.use(s_out):
                s_out.wait_event(done)
                hy[i].copy_(y, non_blocking=True)
                out_ev = cu.event()
                out_ev.record(s_out)
                copied[i] = out_ev
    last = cu.event()
    last.record(s_out)
    comp.wait_event(last)
    end.record(comp)
    cu.synchronize()
    return start.elapsed_time(end)


def choose_e2e(serial_ms, pipe_ms, pipe_ok, note=None):
    """Which end-to-end figure the line reports: the faster of the serial run
    and the overlapped run, the overlapped one only when its outputs were
    verified.  Returns (ms, mode, note)."""
    serial_mode = "serial (one stream)"
    pipe_mode = "copies overlapped (H2D / compute / D2H streams)"
    if not pipe_ok:
        return serial_ms, serial_mode, note or "overlapped run not verified; serial figure reported"
    if pipe_ms <= serial_ms:
        return pipe_ms, pipe_mode, note
    return serial_ms, serial_mode, note or "overlapped run was slower; serial figure reported"


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def sample_indices(batch):
    """Images whose outputs the parity check compares: the first two and the
    last two of the batch."""
    return sorted({0, min(1, batch - 1), max(0, batch - 2), batch - 1})


def sample_parity(name, x, w, y):
    """rel L2 of sampled output images against the CPU oracle's reference
    precision NOVA math, and both errors against an FP64 direct convolution.
    Runs outside every timed region (the oracle is the checker only)."""
    import numpy as np
    import nova_oracle as o
    idx = sample_indices(x.shape[0])
    xs = x[idx].cpu().numpy()
    ws = w.detach().float().cpu().numpy()
    ys = y[idx].cpu().numpy()
    y_o = o.nova_forward(xs, ws, 1, "ref")
    d = o.direct_conv_fp64(xs, ws, 1)
    par, err, err_o = o.rel_l2(ys, y_o), o.rel_l2(ys, d), o.rel_l2(y_o, d)
    finite = bool(np.isfinite(ys.astype(np.float32)).all())
    return {"images": idx, "rel_l2_vs_oracle": round(par, 6), "rel_err_vs_fp64": round(err, 6),
            "oracle_rel_err_vs_fp64": round(err_o, 6),
            "ok": bool(finite and par <= PARITY_TOL and err <= ACCURACY_FACTOR * err_o)}


def graph_of(fn):
    """fn() captured once into a CUDA graph on a side stream."""
    import torch
    g = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        fn()
        st.synchronize()
        with torch.cuda.graph(g, stream=st):
            fn()
    torch.cuda.current_stream().wait_stream(st)
    torch.cuda.synchronize()
    return g


def back_to_back_us(fn, reps=100, warmup=20):
    """Mean time of `reps` back-to-back calls between two events, L2 warm: the
    reference's own per-layer method (benchmarks/bench_layers.py:18-30)."""
    import torch
    for _ in range(warmup):
        fn()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / reps * 1e3


def config2_grid(device, flush, batches=(1, 8, 32, 128), reps=20):
    """BASELINE config 2's grid: every sweep layer at each batch, with torch's FP16 conv2d (cuDNN) on the same layer and the
    sampled-image parity of the timed outputs.  Per point: `us` = device time
    of one forward replayed from a CUDA graph with L2 flushed before it (mean);
    `us_b2b` = the reference's method, back-to-back eager module calls with L2
    warm (host submission included where it is the longer)."""
    import torch
    import torch.nn.functional as F
    torch.backends.cudnn.benchmark = True
    grid = {}
    for B in batches:
        for name, C, H, conv, x in build_layers(B, device):
            w16 = conv.weight.detach().half()
            with torch.no_grad():
                for _ in range(3):
                    F.conv2d(x, w16, padding=1)
                g_ours = graph_of(lambda: conv(x))
                g_cud = graph_of(lambda: F.conv2d(x, w16, padding=1))
                ours = time_kernel(g_ours.replay, reps, flush)
                cud = time_kernel(g_cud.replay, reps, flush)
                ours_b2b = back_to_back_us(lambda: conv(x))
                cud_b2b = back_to_back_us(lambda: F.conv2d(x, w16, padding=1))
                y = conv(x)
                # The same point channels-last: our NHWC kernels and cuDNN's
                # channels-last convolution, graph-replayed after an L2 flush.
                xl = x.contiguous(memory_format=torch.channels_last)
                wl = w16.contiguous(memory_format=torch.channels_last)
                for _ in range(3):
                    F.conv2d(xl, wl, padding=1)
                g_ours_l = graph_of(lambda: conv(xl))
                g_cud_l = graph_of(lambda: F.conv2d(xl, wl, padding=1))
                ours_l = time_kernel(g_ours_l.replay, reps, flush)
                cud_l = time_kernel(g_cud_l.replay, reps, flush)
                yl = conv(xl)
            fl = direct_flops(B, C, C, H)
            grid.setdefault(name, {})[str(B)] = {
                "us": round(ours * 1e3, 2), "eff_tflops": round(fl / ours / 1e9, 1),
                "cudnn_fp16_us": round(cud * 1e3, 2),
                "us_b2b": round(ours_b2b, 2), "cudnn_fp16_us_b2b": round(cud_b2b, 2),
                "parity": sample_parity(name, x, conv.weight, y),
                "nhwc_us": round(ours_l * 1e3, 2), "nhwc_eff_tflops": round(fl / ours_l / 1e9, 1),
                "cudnn_fp16_channels_last_us": round(cud_l * 1e3, 2),
                "nhwc_parity_ok": sample_parity(name, x, conv.weight, yl.contiguous())["ok"]}
            del x, y, xl, yl, g_ours, g_cud, g_ours_l, g_cud_l
    return grid


def gemm_sustained(gm, flops, device, peaks, seconds=1.5, per_graph=25):
    """The GEMM back to back for about `seconds` (CUDA graphs of `per_graph`
    launches, after half a second of the same load), with the SM clock and power
    sampled meanwhile: the sustained rate, against the sustained peak."""
    import torch
    g = graph_of(lambda: [gm() for _ in range(per_graph)])
    g.replay()
    torch.cuda.synchronize()
    t0 = time.time()
    g.replay()
    torch.cuda.synchronize()
    n = max(10, int(seconds / max(time.time() - t0, 1e-4)))
    uuid = str(torch.cuda.get_device_properties(device).uuid)
    sampler = ClockSampler(uuid if uuid.startswith("GPU-") else f"GPU-{uuid}")
    sampler.start()
    for _ in range(n // 3):
        g.replay()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(n):
        g.replay()
    e.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = s.elapsed_time(e) / (n * per_graph)
    tf = flops / ms / 1e9
    del g
    return {"launches": n * per_graph, "gemm_us": round(ms * 1e3, 2), "tflops": round(tf, 1),
            "frac_of_sustained_peak": round(tf / peaks["bf16_tflops_sustained"], 4),
            "sustained_peak": peaks["bf16_tflops_sustained"], "clocks": clocks,
            "l2": "warm (operands partly L2-resident back to back)"}


def gemm_stage_b256(device, flush, peaks, reps=20):
    """The north star's batch-256 GEMM stage: the tcgen05 GEMM alone (stage
    entry nova_batched_gemm_v2, L2 flushed) at batch 256 for conv2_x, conv4_x
    and conv5_x, with its fraction of the measured dense peak (burst figure:
    the kernel is timed alone).  The same layers' whole forward at batch 256
    is parity-checked on sampled images."""
    import torch
    from nova_winograd import ops
    lib = ops.get_lib()
    shapes = [l for l in LAYERS if l[0] in ("conv2_x", "conv4_x", "conv5_x")]
    out = {}
    for name, C, H, conv, x in build_layers(256, device, shapes):
        nt = live_tiles(H)
        BP = 256 * nt * nt
        with torch.no_grad():
            y = conv(x)
        V = torch.empty(64, BP, C, dtype=torch.float16, device=device)
        M = torch.empty(64, BP, C, dtype=torch.float16, device=device)
        s = ops.stream_ptr()
        ops.check(lib.nova_input_transform_v2(ops.ptr(x), ops.ptr(V), 256, C, H, H, 1, nt, nt, BP,
                                              s), "input_transform")
        h = conv._handle

        def gm():
            ops.check(lib.nova_batched_gemm_v2(h, ops.ptr(V), ops.ptr(M), BP, s), "gemm")

        ms = time_kernel(gm, reps, flush)
        flops = 2.0 * 64 * C * C * BP
        tf = flops / ms / 1e9
        # Calibration, not a product path: cuBLAS (torch.bmm, FP16 in and out)
        # on the same 64 GEMMs of [BP, C] x [C, K], timed the same way.
        Ut = torch.randn(64, C, C, dtype=torch.float16, device=device).transpose(1, 2)
        Mc = torch.empty_like(M)
        ms_cb = time_kernel(lambda: torch.bmm(V, Ut, out=Mc), reps, flush)
        del Ut, Mc
        def gm_cur():  # on the current stream at call time (capturable)
            ops.check(lib.nova_batched_gemm_v2(h, ops.ptr(V), ops.ptr(M), BP, ops.stream_ptr()),
                      "gemm")

        sustained = gemm_sustained(gm_cur, flops, device, peaks) if C == 512 else None
        out[name] = {"gemm_us": round(ms * 1e3, 2), "tflops": round(tf, 1),
                     "sustained_loop": sustained,
                     "cublas_bmm_us": round(ms_cb * 1e3, 2),
                     "cublas_bmm_tflops": round(flops / ms_cb / 1e9, 1),
                     "frac_of_peak": round(tf / peaks["bf16_tflops"], 4),
                     "peak": peaks["bf16_tflops"], "peak_kind": "dense bf16 burst (" +
                     peaks["source"] + ")",
                     "gemm_bytes": 2 * 64 * BP * C * 2 + 64 * C * C * 2,
                     "parity": sample_parity(name, x, conv.weight, y)}
        del V, M, x, y
    return out


def run_nova(args):
    import torch
    world, rank, local, dist = setup_dist()
    device = torch.device("cuda", local)
    peaks = load_peaks()
    batch = args.batch
    layers = build_layers(batch, device)
    flops_step = sum(direct_flops(batch, C, C, H) for _, C, H in LAYERS)
    flush = make_flush(device)

    def step():
        for _, _, _, conv, x in layers:
            conv(x)

    for _ in range(args.warmup):
        step()
    barrier(dist)
    uuid = str(torch.cuda.get_device_properties(device).uuid)
    sampler = ClockSampler(uuid if uuid.startswith("GPU-") else f"GPU-{uuid}")
    sampler.start()
    time.sleep(0.3)
    evs = []
    for _ in range(args.steps):
        flush()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        step()
        e.record()
        evs.append((s, e))
    torch.cuda.synchronize()
    barrier(dist)
    clocks = sampler.stop()
    step_ms = [s.elapsed_time(e) for s, e in evs]
    total_ms = max_over_ranks(dist, sum(step_ms))
    ms_per_step = total_ms / args.steps
    value = world * flops_step * args.steps / (total_ms / 1e3) / 1e12
    from nova_winograd import ops
    launches = 3 * len(LAYERS) * args.steps  # input transform, GEMM, output transform

    # End to end through the public module API: pinned host input -> device,
    # forward, output -> pinned host, every step.
    hx = [x.cpu().pin_memory() for _, _, _, _, x in layers]
    hy = [torch.empty(batch, C, H, H, dtype=torch.float16).pin_memory() for _, C, H, _, _ in layers]
    dx = [torch.empty_like(x) for _, _, _, _, x in layers]
    h2d = sum(t.numel() * 2 for t in hx)
    d2h = sum(t.numel() * 2 for t in hy)

    def e2e_step():
        for i, (_, _, _, conv, _) in enumerate(layers):
            dx[i].copy_(hx[i], non_blocking=True)
            hy[i].copy_(conv(dx[i]), non_blocking=True)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    barrier(dist)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        e2e_step()
    e.record()
    torch.cuda.synchronize()
    serial_ms = max_over_ranks(dist, s.elapsed_time(e))

    # The same work with the copies overlapped on their own streams; its last
    # step's host outputs must equal a fresh forward bit for bit, else the
    # serial figure stands.
    # No collective runs inside the try: the ranks (aligned by the reduction
    # above) agree on the outcome afterwards, every rank taking part.
    convs = [conv for _, _, _, conv, _ in layers]
    e2e_mode, e2e_note = "serial (one stream)", None
    pipe_ms, ok = 0.0, False
    try:
        cu = _TorchCuda()
        e2e_pipelined(hx, dx, hy, convs, max(1, args.warmup), cu)
        pipe_ms = e2e_pipelined(hx, dx, hy, convs, args.steps, cu)
        ok = all(torch.equal(hy[i], conv(hx[i].to(device)).cpu())
                 for i, conv in enumerate(convs))
        if not ok:
            e2e_note = "overlapped run's outputs differed; serial figure reported"
    except Exception as ex:  # pragma: no cover - reported, never fatal
        e2e_note = f"overlapped run failed: {ex!r}; serial figure reported"
    all_ok = max_over_ranks(dist, 0.0 if ok else 1.0) == 0.0
    pipe_ms = max_over_ranks(dist, pipe_ms)
    if not all_ok and e2e_note is None:
        e2e_note = "another rank's overlapped run failed; serial figure reported"
    e2e_ms, e2e_mode, e2e_note = choose_e2e(serial_ms, pipe_ms, all_ok, e2e_note)
    e2e_value = world * flops_step * args.steps / (e2e_ms / 1e3) / 1e12

    # Parity of what was timed: sampled images of every layer's output on the
    # timed inputs, against the oracle (after the timed region).
    parity = None
    if rank == 0:
        with torch.no_grad():
            parity = {name: sample_parity(name, x, conv.weight, conv(x))
                      for name, C, H, conv, x in layers}

    stages = roofline = lat = cpu = vendor = grid = b256 = stages_nhwc = None
    if rank == 0:
        stages = stage_profile(layers, batch, flush)
        roofline = roofline_from_stages(stages, peaks, batch)
        if not args.quick:
            stages_nhwc = [
                {"layer": st["layer"], "kernel": st["kernel"], "ms": round(st["ms"], 5),
                 "bytes": st["bytes"], "gbs": round(st["gbs"], 1),
                 "frac_of_hbm": round(st["gbs"] / peaks["hbm_gbs"], 3)}
                for st in stage_profile(layers, batch, flush, nhwc=True) if "nhwc" in st["kernel"]]
        lat = b1_latency(device, nhwc=not args.quick)
        vendor = vendor_layer_times(layers, flush, channels_last=not args.quick)
        if not args.quick:
            grid = config2_grid(device, flush)
            b256 = gemm_stage_b256(device, flush, peaks)
        if world == 1 and not args.no_cpu:
            v, threads, sample, extra = cpu_nova_sample(args.cpu_batch)
            cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample,
                   "cpu_model": cpu_model()}
            cpu.update(extra)
    barrier(dist)
    # BASELINE config 3 on every rank (batch 256 per GPU), so the 1..N GPU
    # runs record model images/s too.
    r50 = None
    if not args.quick:
        del layers
        torch.cuda.empty_cache()
        r50 = resnet50_measure(256, max(3, args.steps // 2), 3, device, dist, world, rank)
    barrier(dist)
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded N(0,1) FP16 inputs, Kaiming-normal FP32 weights)",
            "config": {"workload": "resnet50_3x3_sweep", "layers": [l[0] for l in LAYERS],
                       "batch_per_gpu": batch, "parallelism": f"dp{world} (batch-partitioned)",
                       "l2": "flushed between steps (write then read 2x L2)"},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms / args.steps,
                    "mode": e2e_mode, "serial_ms_per_step": serial_ms / args.steps,
                    "overlapped_ms_per_step": (pipe_ms / args.steps) if all_ok else None,
                    **({"note": e2e_note} if e2e_note else {})},
            "gpu_launches": launches,
            "roofline": roofline,
            "clocks": clocks,
            "cpu_baseline": cpu,
            "stages": [{k: (round(v, 5) if isinstance(v, float) else v) for k, v in st.items()}
                       for st in stages],
            "parity": parity,
            "stages_nhwc": stages_nhwc,
            "b1_latency_us": lat,
            "per_layer_vs_cudnn": vendor,
            "config2_grid": grid,
            "stages_b256": b256,
            "resnet50": r50,
            "step_ms": [round(t, 4) for t in step_ms],
            "library": ops.get_lib().nova_version().decode(),
        }
        emit(line)
    if dist is not None:
        dist.destroy_process_group()


def run_unet_layers(args):
    """UNet 3x3 stride-1 layer shapes (UNET_LAYERS for SD 1.5, SDXL_LAYERS for
    SDXL) at --batch: one step is one forward of each, L2 flushed between steps,
    with the same layers through torch's FP16 conv2d (cuDNN) for context.
    Synthetic N(0,1) inputs and Kaiming-normal weights; one GPU."""
    import torch
    shapes = SDXL_LAYERS if args.workload == "sdxl_layers" else UNET_LAYERS
    model = "SDXL" if args.workload == "sdxl_layers" else "SD 1.5"
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    layers = build_layers(args.batch, device, shapes)
    flush = make_flush(device)
    flops_step = sum(direct_flops(args.batch, C, C, H) for _, C, H in shapes)

    def step():
        for _, _, _, conv, x in layers:
            conv(x)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    evs = []
    for _ in range(args.steps):
        flush()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        step()
        e.record()
        evs.append((s, e))
    torch.cuda.synchronize()
    total_ms = sum(s.elapsed_time(e) for s, e in evs)
    emit({
        "metric": f"F(6,3) conv eff. TFLOP/s (direct-conv FLOPs / time), {model} UNet 3x3 s1 shapes",
        "value": flops_step * args.steps / (total_ms / 1e3) / 1e12, "unit": "TFLOP/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded N(0,1) FP16 inputs, Kaiming-normal FP32 weights)",
        "config": {"workload": f"{args.workload.split('_')[0]}_unet_3x3_shapes", "layers": [l[0] for l in shapes],
                   "batch_per_gpu": args.batch,
                   "l2": "flushed between steps (write then read 2x L2)"},
        "per_layer_vs_cudnn": vendor_layer_times(layers, flush, channels_last=True),
        "library": __import__("nova_winograd").ops.get_lib().nova_version().decode(),
    })


def resnet50_measure(batch, steps, warmup, device, dist, world, rank):
    """torchvision ResNet-50 (random init, BN in eval mode
    with running mean 0 / var 1), FP16, 3x224x224 N(0,1) input; the 13 eligible
    3x3 stride-1 convs replaced by replace_conv2d_with_nova.  Data parallel by
    batch: every rank runs `batch` images per step (weak scaling), timed with
    CUDA events, max over ranks.  The same model without replacement (cuDNN) is
    timed alongside; the replaced model's logits are compared with it, and one
    image's output of every replaced conv with the CPU oracle.  All ranks call
    this; returns the record (meaningful on rank 0)."""
    import torch
    import torchvision
    from nova_winograd import NovaWinogradConv2d, replace_conv2d_with_nova
    torch.manual_seed(1234 + rank)
    ref = torchvision.models.resnet50().to(device).half().eval()
    model = torchvision.models.resnet50().to(device).half().eval()
    model.load_state_dict(ref.state_dict())
    n_rep = replace_conv2d_with_nova(model, verbose=False)
    x = torch.randn(batch, 3, 224, 224, device=device, dtype=torch.float16)

    def timed(m):
        with torch.no_grad():
            for _ in range(warmup):
                out = m(x)
            barrier(dist)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(steps):
                out = m(x)
            e.record()
            torch.cuda.synchronize()
        return max_over_ranks(dist, s.elapsed_time(e)), out

    ms, out = timed(model)
    ms_ref, out_ref = timed(ref)
    finite = bool(torch.isfinite(out).all().item())
    rel = float(((out.float() - out_ref.float()).norm() / out_ref.float().norm()).item())
    # End to end: pinned host images in, logits out, every step.
    hx = x.cpu().pin_memory()
    hy = torch.empty(batch, 1000, dtype=torch.float16).pin_memory()
    with torch.no_grad():
        for _ in range(max(1, warmup)):
            hy.copy_(model(hx.to(device, non_blocking=True)), non_blocking=True)
        barrier(dist)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(steps):
            hy.copy_(model(hx.to(device, non_blocking=True)), non_blocking=True)
        e.record()
        torch.cuda.synchronize()
    e2e_ms = max_over_ranks(dist, s.elapsed_time(e))
    rec = {
        "img_s": world * batch * steps / (ms / 1e3), "ms_per_step": ms / steps,
        "batch_per_gpu": batch, "n_gpus": world, "replaced_convs": n_rep,
        "e2e": {"value": world * batch * steps / (e2e_ms / 1e3), "unit": "img/s",
                "h2d_bytes_per_step": hx.numel() * 2, "d2h_bytes_per_step": hy.numel() * 2},
        "cudnn_same_model_img_s": world * batch * steps / (ms_ref / 1e3),
        "logits_finite": finite, "logits_rel_diff_vs_cudnn": rel,
        "gpu_launches": 3 * n_rep * steps,
    }
    if rank == 0:
        # Batch 1 (config 3's latency case): eager forwards, and the whole
        # network captured once in a CUDA graph and replayed (the module's
        # forward is capturable), NOVA and cuDNN.
        x1 = x[:1].clone()
        b1 = {}
        for label, m in (("nova", model), ("cudnn", ref)):
            with torch.no_grad():
                b1[label + "_eager_ms"] = round(back_to_back_us(lambda: m(x1), reps=50) / 1e3, 4)
                g = graph_of(lambda: m(x1))
                b1[label + "_graph_ms"] = round(back_to_back_us(g.replay, reps=50) / 1e3, 4)
                del g
        rec["batch1"] = b1
        # Every replaced conv's output for image 0, from the activations the
        # model feeds it, against the oracle (hooks outside the timed region).
        seen = []
        hooks = [mod.register_forward_hook(
            lambda mod, inp, outp: seen.append((mod, inp[0][:1].clone(), outp[:1].clone())))
            for mod in model.modules() if isinstance(mod, NovaWinogradConv2d)]
        with torch.no_grad():
            model(x[:1])
        for hk in hooks:
            hk.remove()
        worst = None
        for mod, xi, yi in seen:
            r = sample_parity("resnet50", xi, mod.weight, yi)
            if worst is None or r["rel_l2_vs_oracle"] > worst["rel_l2_vs_oracle"] or not r["ok"]:
                worst = dict(r, ok=r["ok"] and (worst is None or worst["ok"]))
        rec["conv_parity_image0"] = {"convs_checked": len(seen),
                                     "worst_rel_l2_vs_oracle": worst["rel_l2_vs_oracle"],
                                     "all_ok": worst["ok"]}
    # The same two models channels-last (weights and input): the replaced convs
    # run the NHWC kernels, the rest of the network cuDNN's channels-last
    # kernels.  All ranks, weak scaling as above.
    model = model.to(memory_format=torch.channels_last)
    ref = ref.to(memory_format=torch.channels_last)
    x = x.contiguous(memory_format=torch.channels_last)
    ms_cl, out_cl = timed(model)
    ms_ref_cl, out_ref_cl = timed(ref)
    rec["channels_last"] = {
        "img_s": world * batch * steps / (ms_cl / 1e3), "ms_per_step": ms_cl / steps,
        "cudnn_same_model_img_s": world * batch * steps / (ms_ref_cl / 1e3),
        "logits_finite": bool(torch.isfinite(out_cl).all().item()),
        "logits_rel_diff_vs_cudnn": float(((out_cl.float() - out_ref_cl.float()).norm() /
                                           out_ref_cl.float().norm()).item()),
        "logits_rel_diff_vs_nchw": float(((out_cl.float() - out.float()).norm() /
                                          out.float().norm()).item()),
    }
    if rank == 0:
        # Batch 1 channels-last, whole network captured in a CUDA graph.
        x1 = x[:1].contiguous(memory_format=torch.channels_last)
        for label, m in (("nova", model), ("cudnn", ref)):
            with torch.no_grad():
                g = graph_of(lambda: m(x1))
                rec["channels_last"][f"batch1_{label}_graph_ms"] = round(
                    back_to_back_us(g.replay, reps=50) / 1e3, 4)
                del g
    del model, ref, x
    torch.cuda.empty_cache()
    return rec


def run_resnet50(args):
    """--workload resnet50: the ResNet-50 record alone as the line."""
    world, rank, local, dist = setup_dist()
    import torch
    device = torch.device("cuda", local)
    uuid = str(torch.cuda.get_device_properties(device).uuid)
    sampler = ClockSampler(uuid if uuid.startswith("GPU-") else f"GPU-{uuid}")
    sampler.start()
    rec = resnet50_measure(args.batch, args.steps, args.warmup, device, dist, world, rank)
    clocks = sampler.stop()
    if rank == 0:
        emit({
            "metric": "ResNet-50 FP16 inference images/s (13 3x3 s1 convs on NOVA F(6,3))",
            "value": rec["img_s"], "unit": "img/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": rec["ms_per_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (N(0,1) images, random-init weights, BN eval mean 0 / var 1)",
            "config": {"workload": "resnet50", "batch_per_gpu": args.batch,
                       "parallelism": f"dp{world} (batch-partitioned)",
                       "replaced_convs": rec["replaced_convs"],
                       "l2": "activations far larger than L2"},
            "e2e": rec["e2e"], "gpu_launches": rec["gpu_launches"],
            "cudnn_same_model_img_s": rec["cudnn_same_model_img_s"],
            "logits_finite": rec["logits_finite"],
            "logits_rel_diff_vs_cudnn": rec["logits_rel_diff_vs_cudnn"],
            "conv_parity_image0": rec.get("conv_parity_image0"),
            "batch1": rec.get("batch1"),
            "channels_last": rec.get("channels_last"),
            "clocks": clocks,
        })
    if dist is not None:
        dist.destroy_process_group()


def run_unet_model(args):
    """BASELINE configs 4 and 5: one denoising step of a random-init UNet
    (unet_callers.SD15 on a 4x64x64 latent with a 77x768 context, or
    unet_callers.SDXL on 4x128x128 with 77x2048, pooled text and time ids),
    FP16, every eligible 3x3 stride-1 conv (49 / 38) replaced by
    replace_conv2d_with_nova.  Data parallel by batch: every rank runs --batch
    latents per step (weak scaling).  The same model without replacement
    (cuDNN) is timed alongside and its output compared."""
    import copy
    import torch
    import unet_callers as U
    from nova_winograd import replace_conv2d_with_nova
    world, rank, local, dist = setup_dist()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    spec, latent, name = ((U.SD15, 64, "SD 1.5") if args.workload == "sd15"
                          else (U.SDXL, 128, "SDXL"))
    torch.manual_seed(1234)  # the same weights on every rank
    with torch.device(device):
        ref = U.UNet(spec)
    ref = ref.half().eval()
    model = copy.deepcopy(ref)
    n_rep = replace_conv2d_with_nova(model, verbose=False)
    x, t, ctx, extra = U.make_inputs(spec, args.batch, latent, device, seed=100 + rank)

    def step(m, xs, ctxs, ex):
        return m(xs, t, ctxs, **ex)

    def timed(m):
        with torch.no_grad():
            for _ in range(args.warmup):
                out = step(m, x, ctx, extra)
            barrier(dist)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(args.steps):
                out = step(m, x, ctx, extra)
            e.record()
            torch.cuda.synchronize()
        return max_over_ranks(dist, s.elapsed_time(e)), out

    uuid = str(torch.cuda.get_device_properties(device).uuid)
    sampler = ClockSampler(uuid if uuid.startswith("GPU-") else f"GPU-{uuid}")
    sampler.start()
    ms, out = timed(model)
    clocks = sampler.stop()
    ms_ref, out_ref = timed(ref)
    finite = bool(torch.isfinite(out).all().item())
    rel = float(((out.float() - out_ref.float()).norm() / out_ref.float().norm()).item())
    # End to end: pinned host latent and conditioning in, predicted noise out.
    hx, hctx = x.cpu().pin_memory(), ctx.cpu().pin_memory()
    hextra = {k: v.cpu().pin_memory() for k, v in extra.items()}
    hy = torch.empty_like(out, device="cpu").pin_memory()
    h2d = hx.numel() * hx.element_size() + hctx.numel() * hctx.element_size() + sum(
        v.numel() * v.element_size() for v in hextra.values())

    def e2e_step():
        ex = {k: v.to(device, non_blocking=True) for k, v in hextra.items()}
        hy.copy_(step(model, hx.to(device, non_blocking=True), hctx.to(device, non_blocking=True),
                      ex), non_blocking=True)

    with torch.no_grad():
        for _ in range(max(1, args.warmup)):
            e2e_step()
        barrier(dist)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.steps):
            e2e_step()
        e.record()
        torch.cuda.synchronize()
    e2e_ms = max_over_ranks(dist, s.elapsed_time(e))
    # Both models channels-last (weights and latent): the replaced convs on the
    # NHWC kernels, the rest on cuDNN's channels-last kernels.
    model = model.to(memory_format=torch.channels_last)
    ref = ref.to(memory_format=torch.channels_last)
    x = x.contiguous(memory_format=torch.channels_last)
    ms_cl, out_cl = timed(model)
    ms_ref_cl, out_ref_cl = timed(ref)
    channels_last = {
        "latents_s": world * args.batch * args.steps / (ms_cl / 1e3),
        "ms_per_step": ms_cl / args.steps,
        "cudnn_same_model_latents_s": world * args.batch * args.steps / (ms_ref_cl / 1e3),
        "cudnn_same_model_ms_per_step": ms_ref_cl / args.steps,
        "output_finite": bool(torch.isfinite(out_cl).all().item()),
        "output_rel_diff_vs_nchw": float(((out_cl.float() - out.float()).norm() /
                                          out.float().norm()).item()),
        # The same comparison for the cuDNN model: how far the network itself
        # carries summation-order differences between the two layouts.
        "cudnn_output_rel_diff_channels_last_vs_nchw": float(
            ((out_ref_cl.float() - out_ref.float()).norm() / out_ref.float().norm()).item()),
    }
    if rank == 0:
        emit({
            "metric": f"{name} UNet FP16 denoising step, latents/s ({n_rep} 3x3 s1 convs on NOVA F(6,3))",
            "value": world * args.batch * args.steps / (ms / 1e3), "unit": "latents/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (N(0,1) latent and context, random timesteps, random-init weights)",
            "config": {"workload": f"{args.workload}_unet_step", "batch_per_gpu": args.batch,
                       "latent": [spec.in_ch, latent, latent],
                       "parallelism": f"dp{world} (batch-partitioned)", "replaced_convs": n_rep,
                       "l2": "activations and weights far larger than L2"},
            "e2e": {"value": world * args.batch * args.steps / (e2e_ms / 1e3), "unit": "latents/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": hy.numel() * hy.element_size()},
            "gpu_launches": 3 * n_rep * args.steps,
            "cudnn_same_model_latents_s": world * args.batch * args.steps / (ms_ref / 1e3),
            "cudnn_same_model_ms_per_step": ms_ref / args.steps,
            "output_finite": finite, "output_rel_diff_vs_cudnn": rel,
            "channels_last": channels_last,
            "clocks": clocks,
        })
    if dist is not None:
        dist.destroy_process_group()


def gemm_trace(args):
    """Wait breakdown of the tcgen05 GEMM's warp roles (library built with
    -DNOVA_GEMM_TRACE, which adds SM-clock counters around every mbarrier
    wait): per CTA, cycles the producer waits for a free stage, the MMA issuer
    for a drained accumulator and for landed operands, the epilogue
    warpgroups for a finished accumulator and for their slab's previous TMA
    store; and the CTA's whole time.  Printed as microseconds at the clock
    given by --trace-mhz, averaged over the CTAs and --steps launches, for
    every sweep layer at batch 128 and conv2_x, conv4_x and conv5_x at batch
    256, L2 flushed before each launch and warm."""
    import ctypes
    import numpy as np
    import torch
    from nova_winograd import ops
    lib = ops.get_lib()
    try:
        # NOVA_GEMM_PAIR=1 routes eligible launches to the SM-pair kernel.
        tr = (lib.nova_debug_gemm2_trace if os.environ.get("NOVA_GEMM_PAIR") == "1"
              else lib.nova_debug_gemm_trace)
    except AttributeError:
        raise SystemExit("gemm-trace: the library was built without -DNOVA_GEMM_TRACE")
    tr.restype = ctypes.c_int
    tr.argtypes = [ctypes.c_void_p, ctypes.c_int]
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    flush = make_flush(device)
    buf = np.zeros((1024, 8), dtype=np.uint64)
    cols = ["producer_wait_free_stage", "mma_wait_accumulator_drained", "mma_wait_operands",
            "epilogue0_wait_accumulator", "epilogue1_wait_accumulator",
            "epilogue0_wait_slab_store_read", "cta_total"]
    nsm = torch.cuda.get_device_properties(device).multi_processor_count
    if os.environ.get("NOVA_GEMM_PAIR") == "1":
        nsm -= nsm % 2  # one CTA per SM of the pairs
    out = {"unit": f"us at {args.trace_mhz} MHz (SM-clock cycles / MHz)"}
    for B, names in ((128, ("conv2_x", "conv3_x", "conv4_x", "conv5_x")),
                     (256, ("conv2_x", "conv4_x", "conv5_x"))):
        shapes = [l for l in LAYERS if l[0] in names]
        for name, C, H, conv, x in build_layers(B, device, shapes):
            nt = live_tiles(H)
            BP = B * nt * nt
            with torch.no_grad():
                conv(x)
            V = torch.empty(64, BP, C, dtype=torch.float16, device=device)
            M = torch.empty_like(V)
            s = ops.stream_ptr()
            ops.check(lib.nova_input_transform_v2(ops.ptr(x), ops.ptr(V), B, C, H, H, 1, nt, nt,
                                                  BP, s), "input_transform")
            h = conv._handle

            def gm():
                ops.check(lib.nova_batched_gemm_v2(h, ops.ptr(V), ops.ptr(M), BP, s), "gemm")

            for mode in ("flushed", "warm"):
                gm()
                torch.cuda.synchronize()
                tr(None, 1)
                torch.cuda.synchronize()
                for _ in range(args.steps):
                    if mode == "flushed":
                        flush()
                    gm()
                torch.cuda.synchronize()
                tr(buf.ctypes.data, 0)
                cyc = buf[:nsm].astype(np.float64).mean(axis=0) / args.steps
                rec = {c: round(float(v) / args.trace_mhz, 2) for c, v in zip(cols, cyc)}
                # Event-timed duration of the same launches; CTA cycles over it
                # bound the SM clock the kernel ran at from below.
                if mode == "flushed":
                    us = time_kernel(gm, args.steps, flush) * 1e3
                else:
                    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    ev0.record()
                    for _ in range(args.steps):
                        gm()
                    ev1.record()
                    torch.cuda.synchronize()
                    us = ev0.elapsed_time(ev1) * 1e3 / args.steps
                rec["kernel_us_events"] = round(us, 2)
                rec["sm_mhz_lower_bound"] = round(float(cyc[len(cols) - 1]) / us, 0)
                out[f"{name}_B{B}_{mode}"] = rec
            del V, M, x
    print(json.dumps(out))


def profile_stages(args):
    """Launch order: input transform, GEMM, output transform, repeated --steps
    times, for one sweep layer at --batch (reference counterpart:
    benchmarks/bench_profile_stages.py, which times the stages by subtraction)."""
    import torch
    from nova_winograd import ops
    name, C, H = next(l for l in LAYERS if l[0] == args.profile_stages)
    torch.cuda.set_device(0)
    layers = build_layers(args.batch, torch.device("cuda", 0))
    _, _, _, conv, x = next(l for l in layers if l[0] == name)
    lib = ops.get_lib()
    nt = live_tiles(H)
    BP = args.batch * nt * nt
    V = torch.empty(64, BP, C, dtype=torch.float16, device="cuda")
    M = torch.empty(64, BP, C, dtype=torch.float16, device="cuda")
    y = torch.empty(args.batch, C, H, H, dtype=torch.float16, device="cuda")
    conv(x)
    s = ops.stream_ptr()
    if args.fused:
        # The fused single kernel (path 3) on the same layer, --steps times.
        ops.check(lib.nova_set_path(conv._handle, ops.PATH_FUSED), "set_path(fused)")
        for _ in range(args.steps):
            ops.check(lib.nova_forward_v2(conv._handle, ops.ptr(x), ops.ptr(y), args.batch, H, H,
                                          1, s), "fused forward")
        torch.cuda.synchronize()
        print(f"profile-stages {name} batch {args.batch} (fused): ok")
        return
    if args.nhwc:
        # The channels-last stage entries on the same layer.
        xl = x.contiguous(memory_format=torch.channels_last)
        yl = y.contiguous(memory_format=torch.channels_last)
        for _ in range(args.steps):
            ops.check(lib.nova_input_transform_nhwc_v2(ops.ptr(xl), ops.ptr(V), args.batch, C, H,
                                                       H, 1, nt, nt, BP, s), "input_transform_nhwc")
            ops.check(lib.nova_batched_gemm_v2(conv._handle, ops.ptr(V), ops.ptr(M), BP, s), "gemm")
            ops.check(lib.nova_output_transform_nhwc_v2(ops.ptr(M), ops.ptr(yl), args.batch, C, H,
                                                        H, nt, nt, BP, s), "output_transform_nhwc")
        torch.cuda.synchronize()
        print(f"profile-stages {name} batch {args.batch} (nhwc): ok")
        return
    for _ in range(args.steps):
        ops.check(lib.nova_input_transform_v2(ops.ptr(x), ops.ptr(V), args.batch, C, H, H, 1,
                                              nt, nt, BP, s), "input_transform")
        ops.check(lib.nova_batched_gemm_v2(conv._handle, ops.ptr(V), ops.ptr(M), BP, s), "gemm")
        ops.check(lib.nova_output_transform_v2(ops.ptr(M), ops.ptr(y), args.batch, C, H, H, nt,
                                               nt, BP, s), "output_transform")
    torch.cuda.synchronize()
    print(f"profile-stages {name} batch {args.batch}: ok")


_JSON_OUT = None


def emit(line):
    """The one JSON line on the original stdout; everything else (libraries
    included, e.g. NCCL's version banner) goes to stderr."""
    out = _JSON_OUT or sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def main():
    global _JSON_OUT
    sys.stdout.flush()
    _JSON_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=None,
                    help="per-GPU batch; default 128 for sweep and resnet50, 8 for the UNet "
                         "workloads")
    ap.add_argument("--cpu-batch", type=int, default=1,
                    help="images of each layer the CPU legs time per pass (a sample of --batch)")
    ap.add_argument("--impl", choices=["nova", "reference"], default="nova")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--quick", action="store_true",
                    help="sweep only: skip the batch 1/8/32 grid, the batch-256 GEMM stage, the "
                         "ResNet-50 record and the channels-last records")
    ap.add_argument("--workload",
                    choices=["sweep", "resnet50", "sd15", "sdxl", "sd15_layers", "sdxl_layers"],
                    default="sweep",
                    help="sweep: ResNet-50 3x3 layer sweep (BASELINE config 2, default); "
                         "resnet50: whole model images/s (config 3); sd15 / sdxl: one UNet "
                         "denoising step (configs 4 and 5); sd15_layers / sdxl_layers: their "
                         "3x3 conv shapes one layer at a time against cuDNN")
    ap.add_argument("--fused", action="store_true",
                    help="with --profile-stages: run the fused single kernel instead (C, K <= 64)")
    ap.add_argument("--nhwc", action="store_true",
                    help="with --profile-stages: the channels-last stage entries")
    ap.add_argument("--gemm-trace", action="store_true",
                    help="wait breakdown of the GEMM's warp roles (library built with "
                         "-DNOVA_GEMM_TRACE)")
    ap.add_argument("--trace-mhz", type=float, default=1965.0)
    ap.add_argument("--profile-stages", metavar="LAYER", default=None,
                    help="only run the three stage entries of one sweep layer (--steps times "
                         "each, no timing output): the driver for ncu captures")
    args = ap.parse_args()
    if args.batch is None:
        args.batch = 128 if args.workload in ("sweep", "resnet50") else 8
    if args.profile_stages:
        profile_stages(args)
        return
    if args.gemm_trace:
        gemm_trace(args)
        return
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "resnet50":
        args.warmup = max(3, args.warmup)
        run_resnet50(args)
    elif args.workload in ("sd15_layers", "sdxl_layers"):
        args.warmup = max(3, args.warmup)
        run_unet_layers(args)
    elif args.workload in ("sd15", "sdxl"):
        args.warmup = max(3, args.warmup)
        run_unet_model(args)
    else:
        args.warmup = max(3, args.warmup)
        run_nova(args)


if __name__ == "__main__":
    main()
