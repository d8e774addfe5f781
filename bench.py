"""Benchmark of the sparse submanifold-conv hot path (driver contract).

Workload (the one the headline metric is quoted on):
the 512^3 shell (R=200, half width 0.5) -> 503,562 voxels, a chain of four
SubMConv3d(64->64) + SiLU layers in bf16 with f32 accumulation. A step is one
pass of the four-layer chain with the neighbour map built (the reference's
own benchmark times warm-cache convs; the map build is reported separately).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl t2sc|reference]

N > 1 (under torchrun): the voxel set is cut into z-slabs of equal voxel
count, one per rank; each rank convolves its slab with a one-voxel halo
received from its z-neighbours over NCCL before every layer.
`--impl reference` times the reference algorithm on the host cores (the
CPU restatement in oracle/, all host threads, bounded samples).
"""
import argparse
import ctypes
import json
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "trellis2-mojo_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

METRIC = "SubM-conv3d effective TFLOP/s & Mvoxel/s, 512³ C=64, 1/2/4/8 B200 vs CPU"
UNIT = "TFLOP/s"
LAYERS, C = 4, 64
WORKLOAD = "cfg4: 512^3 seeded shell R=200 h=0.5 (503,562 voxels), 4 x SubMConv3d(64->64)+SiLU, bf16 in/f32 acc"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["bf16_tflops"], p["hbm_gbs"], "measured"
    except Exception:
        return 1590.0, 6650.0, "fallback"


def inputs():
    import t2sc
    S = t2sc.synth
    coords = S.shell(*S.SHELLS["cfg4"])
    n = len(coords)
    x = S.normal(400, (n, C))
    ws = [S.normal(401 + 3 * i, (C, 3, 3, 3, C), std=(1.0 / (27 * C)) ** 0.5) for i in range(LAYERS)]
    bs = [S.normal(402 + 3 * i, (C,), std=0.1) for i in range(LAYERS)]
    return coords, x, ws, bs


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, device):
        self.device = device
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), "--query-gpu=clocks.sm,clocks.max.sm,power.draw,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.summary = None
        if not self.proc:
            return
        self.proc.terminate()
        out, _ = self.proc.communicate()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [s.strip() for s in line.split(",")]
            try:
                sm.append(float(f[0]))
                mx = float(f[1])
            except (ValueError, IndexError):
                continue
            for nm, v in zip(names, f[3:7]):
                if v.lower() == "active":
                    reasons.add(nm)
        if sm:
            self.summary = {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons),
                            "samples": len(sm)}


def dram_traffic_per_launch():
    """DRAM bytes per conv launch from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "conv_tc_cfg4.txt")
    try:
        for line in open(p):
            if line.startswith("dram_bytes_per_launch:"):
                return float(line.split(":")[1])
    except OSError:
        pass
    return None


def cpu_baseline_sample(coords, x, w, b, target_s=10.0, nthreads=None):
    """The reference algorithm (oracle, Co-chunks of 8 as conv.mojo:166-194)
    on a bounded prefix of the layer's edge list; returns TFLOP/s."""
    from oracle import oracle as O
    O.build()
    src, tgt, kidx = O.neighbor_map(coords)
    e_total = len(src)
    nthreads = nthreads or 0  # 0: one thread per Co chunk, the reference's own parallelism
    ne = min(e_total, 100_000)
    t0 = time.perf_counter()
    O.conv(x, w, b, (src[:ne], tgt[:ne], kidx[:ne]), nthreads=nthreads)
    dt = time.perf_counter() - t0
    ne2 = int(min(e_total, max(ne, ne * target_s / max(dt, 1e-6))))
    t0 = time.perf_counter()
    O.conv(x, w, b, (src[:ne2], tgt[:ne2], kidx[:ne2]), nthreads=nthreads)
    dt = time.perf_counter() - t0
    flops = 2.0 * ne2 * C * C
    return flops / dt / 1e12, ne2, e_total, dt


def run_reference(args):
    """`--impl reference`: the reference's CPU algorithm on all host threads."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle as O
    O.build()
    coords, x, ws, bs = inputs()
    n = len(coords)
    src, tgt, kidx = O.neighbor_map(coords)
    rs, ss, ks = O.csr(n, src, tgt, kidx)
    cores = os.cpu_count() or 1
    # each step: one layer over a bounded block of target rows (all cores,
    # rows split across threads; per-row sums in the reference's order)
    rows = min(n, 20000)
    times, flops = [], 0.0
    for s in range(-args.warmup, args.steps):
        r0 = ((s + args.warmup) * rows) % max(1, n - rows)
        sub = (rs[r0:r0 + rows + 1] - rs[r0]).astype(np.int64)
        e0, e1 = rs[r0], rs[r0 + rows]
        t0 = time.perf_counter()
        y = np.empty((rows, C), np.float32)
        O.lib().orc_conv_forward_rows(
            O._p(np.ascontiguousarray(x)), rows, C, O._p(ws[0]), O._p(bs[0]), C, 27, O._p(sub),
            O._p(np.ascontiguousarray(ss[e0:e1])), O._p(np.ascontiguousarray(ks[e0:e1])), O._p(y), cores)
        if s >= 0:
            times.append(time.perf_counter() - t0)
            flops += 2.0 * (e1 - e0) * C * C
    t = sum(times)
    v = flops / t / 1e12
    mvox = args.steps * rows / t / 1e6
    line = {"metric": METRIC, "value": v, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "mvoxel_per_s": mvox,
            "config": {"workload": WORKLOAD, "voxels": n, "edges": len(src), "layers": LAYERS,
                       "sample": f"{rows} target rows of layer 1 per step"},
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": f"{rows} target rows x all their edges per step, {cores} threads"},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="t2sc", choices=["t2sc", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--overlap", action="store_true",
                    help="N>1: convolve interior rows while the halo is in flight (measured slower at N=4 and 8: "
                         "the second launch per layer costs more than the hidden exchange)")
    ap.add_argument("--op", default="conv", choices=["conv", "layernorm"],
                    help="layernorm: time the LayerNorm+SiLU glue kernel alone (not the headline metric)")
    args = ap.parse_args()
    if args.op == "layernorm":
        return run_layernorm(args)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.gpus > 1 or int(os.environ.get("WORLD_SIZE", "1")) > 1:
        return run_distributed(args)
    return run_single(args)


def run_layernorm(args, rows=8_000_000, c=64):
    """LayerNorm(eps 1e-6, affine) + SiLU over bf16 [rows, 64] features in
    place of the decoder's norm -> activation pairs; 1 GB in and out (larger
    than L2), so no flush is needed. Algorithmic bytes per launch:
    2 * rows * c * 2 (+ 512 B of weights)."""
    import torch

    import t2sc
    from t2sc import _lib
    ctx = t2sc.Context.default(0)
    stream = torch.cuda.Stream()
    ctx.set_stream(stream.cuda_stream)
    g = torch.Generator(device="cuda:0").manual_seed(0)
    x = torch.randn(rows, c, device="cuda:0", generator=g).to(torch.bfloat16)
    y = torch.empty_like(x)
    w = torch.randn(c, device="cuda:0", generator=g)
    b = torch.randn(c, device="cuda:0", generator=g)
    torch.cuda.synchronize()

    def launch():
        _lib.check(_lib.lib.t2sc_layernorm_device(ctx.handle, ctypes.c_void_p(x.data_ptr()),
                                                  ctypes.c_void_p(y.data_ptr()), rows, c,
                                                  ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(b.data_ptr()),
                                                  1e-6, _lib.SILU, _lib.DT_BF16), ctx.handle)

    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            launch()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        stream.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            launch()
        e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    alg = 2 * rows * c * 2 + 2 * c * 4
    _, hbm, src = peaks()
    gbs = alg / (ms * 1e-3) / 1e9
    print(json.dumps({"metric": "LayerNorm+SiLU bandwidth, bf16 [8M, 64]", "value": round(gbs, 1), "unit": "GB/s",
                      "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": round(ms, 4),
                      "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
                      "config": {"workload": f"layernorm_vec_kernel, rows={rows}, C={c}, eps=1e-6, affine, SiLU",
                                 "l2": "inputs larger than L2"},
                      "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "peak_source": src,
                                   "unit": "GB/s", "frac": round(gbs / hbm, 3)}}))


def run_single(args):
    import torch

    import t2sc
    from t2sc import _lib

    dev = 0
    torch.cuda.set_device(dev)
    ctx = t2sc.Context.default(dev)
    # a dedicated (non-default) stream shared by torch and the library, so
    # the CUDA events below time exactly the library's kernels
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    coords, x, ws, bs = inputs()
    n = len(coords)
    convs = [t2sc.SparseConv3d(w, b, dtype="bf16", ctx=ctx) for w, b in zip(ws, bs)]
    cdev = t2sc.Coords(ctx, coords)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    E = cdev.build_map()
    torch.cuda.synchronize()
    map_ms = 1e3 * (time.perf_counter() - t0)

    xd = torch.from_numpy(x).to("cuda").to(torch.bfloat16)
    bufs = [torch.empty((n, C), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    L = _lib.lib

    def step(evs=None):
        cur = xd
        for i, cv in enumerate(convs):
            out = bufs[i & 1]
            if evs is not None:
                evs[i][0].record(stream)
            rc = L.t2sc_conv_forward_device(cv.handle, cdev.handle, ctypes.c_void_p(cur.data_ptr()),
                                            ctypes.c_void_p(out.data_ptr()), _lib.SILU, None)
            if evs is not None:
                evs[i][1].record(stream)
            _lib.check(rc, ctx.handle)
            cur = out
        return cur

    for _ in range(args.warmup):
        step()
    ctx.synchronize()
    torch.cuda.synchronize()
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    step_times, layer_times = [], []
    launches0 = ctx.launch_count()
    clk = Clocks(dev).__enter__()
    time.sleep(0.3)
    if True:
        for _ in range(args.steps):
            flush.zero_()  # 256 MiB write: L2 (126 MB) holds nothing of the previous step
            evs = [(ev(), ev()) for _ in range(LAYERS)]
            s0, s1 = ev(), ev()
            torch.cuda.synchronize()
            s0.record(stream)
            step(evs)
            s1.record(stream)
            torch.cuda.synchronize()
            step_times.append(s0.elapsed_time(s1))
            layer_times += [a.elapsed_time(b) for a, b in evs]
    launches = ctx.launch_count() - launches0
    ctx.synchronize()
    # keep the GPU under the same load (untimed) until the clock sampler has
    # seen at least ~1 s of it
    t_load = time.perf_counter()
    while time.perf_counter() - t_load < 1.0:
        for _ in range(20):
            step()
        torch.cuda.synchronize()
    clk.__exit__()
    ms = float(np.sum(step_times)) / args.steps
    flops_layer = 2.0 * E * C * C
    value = LAYERS * flops_layer / (ms * 1e-3) / 1e12
    mvox = LAYERS * n / (ms * 1e-3) / 1e6
    peak_tf, peak_bw, peak_kind = peaks()
    layer_ms = float(np.mean(layer_times))
    achieved = flops_layer / (layer_ms * 1e-3) / 1e12
    bytes_layer = n * C * 2 * 2 + 27 * C * C * 2  # x in + y out (bf16) + weights
    traffic = dram_traffic_per_launch()

    # e2e through the public C ABI with pinned host buffers: upload, 4 layers, download
    xh = torch.from_numpy(x).pin_memory()
    yh = torch.empty((n, C), dtype=torch.float32).pin_memory()
    arr = (ctypes.c_void_p * LAYERS)(*[cv.handle.value for cv in convs])
    fl = (ctypes.c_int * LAYERS)(*([_lib.SILU] * LAYERS))
    for _ in range(2):
        _lib.check(L.t2sc_conv_chain_forward(arr, LAYERS, cdev.handle, ctypes.c_void_p(xh.data_ptr()),
                                             ctypes.c_void_p(yh.data_ptr()), fl), ctx.handle)
    e2e_t = []
    for _ in range(args.steps):
        flush.zero_()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        _lib.check(L.t2sc_conv_chain_forward(arr, LAYERS, cdev.handle, ctypes.c_void_p(xh.data_ptr()),
                                             ctypes.c_void_p(yh.data_ptr()), fl), ctx.handle)
        e2e_t.append(time.perf_counter() - t0)
    e2e_s = float(np.mean(e2e_t))

    cpu = None
    if not args.no_cpu_baseline:
        v, ne, etot, dt = cpu_baseline_sample(coords, x, ws[0], bs[0])
        cpu = {"value": v, "unit": UNIT, "cores": min(os.cpu_count() or 1, C // 8), "kind": "port",
               "sample": f"layer 1, first {ne} of {etot} edges (kernel-offset-major), reference Co-chunk "
                         f"parallelism ({C // 8} threads), {dt:.1f} s"}
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "mvoxel_per_s": mvox, "map_build_ms": map_ms,
            "config": {"workload": WORKLOAD, "voxels": n, "edges": E, "layers": LAYERS, "channels": C,
                       "l2": "flushed between steps (256 MiB write)", "parallelism": "single GPU"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": achieved / peak_tf, "traffic": traffic, "peak_source": peak_kind,
                         "kernel": "conv_tc_kernel (one layer)", "kernel_ms": layer_ms,
                         "algorithmic_bytes": bytes_layer,
                         "hbm_frac": bytes_layer / (layer_ms * 1e-3) / 1e9 / peak_bw},
            "e2e": {"value": LAYERS * flops_layer / e2e_s / 1e12, "unit": UNIT, "h2d_bytes_per_step": n * C * 4,
                    "d2h_bytes_per_step": n * C * 4, "ms_per_step": 1e3 * e2e_s},
            "gpu_launches": launches,
            "clocks": clk.summary,
            "cpu_baseline": cpu}
    print(json.dumps(line))


def run_distributed(args):
    """One rank per GPU (torchrun): the cfg4 shell is cut into z-slabs
    (t2sc.dist); before every layer each rank receives its one-voxel halo
    from its z-neighbours over NCCL, then convolves (own + halo) rows with
    outputs for its own rows. Total work is fixed as N grows (strong
    scaling); `value` is the whole job's TFLOP/s over the slowest rank."""
    import torch
    import torch.distributed as tdist

    import t2sc
    from t2sc import _lib, dist

    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    torch.cuda.set_device(local)
    tdist.init_process_group("nccl", device_id=torch.device("cuda", local))
    ctx = t2sc.Context.default(local)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    coords, x, ws, bs = inputs()
    slab = dist.partition(coords, world)[rank]
    rows = slab.rows
    n_own, n_loc = slab.n_own, len(rows)
    convs = [t2sc.SparseConv3d(w, b, dtype="bf16", ctx=ctx) for w, b in zip(ws, bs)]
    n_int = slab.n_int
    # interior targets [0, n_int) need no halo; boundary targets [n_int, n_own) do
    c_int = t2sc.Coords(ctx, coords[rows], targets=(0, n_int))
    c_bnd = t2sc.Coords(ctx, coords[rows], targets=(n_int, n_own))
    c_all = t2sc.Coords(ctx, coords[rows], n_targets=n_own) if (not args.overlap) else None
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e_loc = c_int.build_map() + c_bnd.build_map()
    if c_all is not None:
        c_all.build_map()
    torch.cuda.synchronize()
    map_ms = 1e3 * (time.perf_counter() - t0)
    e_all = torch.tensor([e_loc], dtype=torch.int64, device="cuda")
    tdist.all_reduce(e_all)
    E = int(e_all.item())

    xin = torch.zeros((n_loc, C), dtype=torch.bfloat16, device="cuda")
    xin[:n_own] = torch.from_numpy(x[slab.own]).to("cuda").to(torch.bfloat16)
    bufs = [torch.zeros((n_loc, C), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    L = _lib.lib

    def step():
        cur = xin
        for i, cv in enumerate(convs):
            pending = dist.start_halo(cur, slab, tdist)  # halo rows of this layer's input
            out = bufs[i & 1]
            if (not args.overlap):
                for q in pending:
                    q.wait()
                _lib.check(L.t2sc_conv_forward_device(cv.handle, c_all.handle, ctypes.c_void_p(cur.data_ptr()),
                                                      ctypes.c_void_p(out.data_ptr()), _lib.SILU, None), ctx.handle)
                cur = out
                continue
            # interior rows while the halo is in flight, boundary rows after it lands
            _lib.check(L.t2sc_conv_forward_device(cv.handle, c_int.handle, ctypes.c_void_p(cur.data_ptr()),
                                                  ctypes.c_void_p(out.data_ptr()), _lib.SILU, None), ctx.handle)
            for q in pending:
                q.wait()
            if n_own > n_int:
                _lib.check(L.t2sc_conv_forward_device(
                    cv.handle, c_bnd.handle, ctypes.c_void_p(cur.data_ptr()),
                    ctypes.c_void_p(out.data_ptr() + n_int * C * out.element_size()), _lib.SILU, None), ctx.handle)
            cur = out
        return cur

    for _ in range(args.warmup):
        step()
    ctx.synchronize()
    torch.cuda.synchronize()
    # The step (4 x (halo exchange + conv)) is captured once in a CUDA graph:
    # at 4-8 ranks a layer is ~20 us of GPU work, less than the host needs
    # to issue it eagerly. Falls back to eager launches if capture fails.
    graph = g = None
    launches_per_step = len(convs) * (2 if n_own > n_int and not (not args.overlap) else 1)
    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step()
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        graph = g
    except Exception as exc:  # noqa: BLE001
        if rank == 0:
            print(f"# graph capture failed, timing eager steps: {exc}", file=sys.stderr)
        torch.cuda.synchronize()
    run = graph.replay if graph is not None else step
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    times = []
    launches0 = ctx.launch_count()
    clk = Clocks(local).__enter__() if rank == 0 else None
    time.sleep(0.3)
    for _ in range(args.steps):
        flush.zero_()
        torch.cuda.synchronize()
        tdist.barrier()
        s0, s1 = ev(), ev()
        s0.record(stream)
        run()
        s1.record(stream)
        torch.cuda.synchronize()
        times.append(s0.elapsed_time(s1))
    launches = ctx.launch_count() - launches0 if graph is None else launches_per_step * args.steps
    t_load = time.perf_counter()
    while time.perf_counter() - t_load < 1.0:
        for _ in range(10):
            run()
        torch.cuda.synchronize()
    if clk:
        clk.__exit__()
    tt = torch.tensor(times, dtype=torch.float64, device="cuda")
    tdist.all_reduce(tt, op=tdist.ReduceOp.MAX)  # per step, the slowest rank
    ms = float(tt.sum().item()) / args.steps

    # e2e: each rank uploads its own rows from pinned host f32, runs the
    # chain with halo exchanges, downloads its own outputs as f32
    xh = torch.from_numpy(np.ascontiguousarray(x[slab.own])).pin_memory()
    yh = torch.empty((n_own, C), dtype=torch.float32).pin_memory()
    e2e = []
    for s in range(args.steps + 2):
        torch.cuda.synchronize()
        tdist.barrier()
        t0 = time.perf_counter()
        xin[:n_own].copy_(xh.to("cuda", non_blocking=True))
        run()
        out = bufs[(len(convs) - 1) & 1]
        yh.copy_(out[:n_own].float(), non_blocking=True)
        torch.cuda.synchronize()
        if s >= 2:
            e2e.append(time.perf_counter() - t0)
    et = torch.tensor(e2e, dtype=torch.float64, device="cuda")
    tdist.all_reduce(et, op=tdist.ReduceOp.MAX)
    e2e_s = float(et.sum().item()) / args.steps
    if rank == 0:
        flops = LAYERS * 2.0 * E * C * C
        n = len(coords)
        line = {"metric": METRIC, "value": flops / (ms * 1e-3) / 1e12, "unit": UNIT, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "mvoxel_per_s": LAYERS * n / (ms * 1e-3) / 1e6, "map_build_ms": map_ms,
                "config": {"workload": WORKLOAD, "voxels": n, "edges": E, "layers": LAYERS, "channels": C,
                           "l2": "flushed between steps (256 MiB write)",
                           "parallelism": f"z-slab x{world}, one-voxel halo over NCCL send/recv"
                                          + (" overlapped with the interior rows' conv" if args.overlap else ""),
                           "rank0_rows": n_own, "rank0_halo_rows": n_loc - n_own,
                           "cuda_graph": graph is not None},
                "e2e": {"value": flops / e2e_s / 1e12, "unit": UNIT, "h2d_bytes_per_step": n * C * 4,
                        "d2h_bytes_per_step": n * C * 4, "ms_per_step": 1e3 * e2e_s},
                "gpu_launches": launches, "clocks": clk.summary if clk else None, "cpu_baseline": None}
        print(json.dumps(line))
    # Release the captured graph (it references the NCCL communicator) before
    # the final barrier, then leave without tearing the communicators down:
    # destroying a process group whose NCCL comm was captured in a graph can
    # block, and the process is done.
    run = graph = g = None  # noqa: F841
    torch.cuda.synchronize()
    tdist.barrier()
    torch.cuda.synchronize()
    sys.stdout.flush()
    sys.stderr.flush()
    os._exit(0)


if __name__ == "__main__":
    main()
