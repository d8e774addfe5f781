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
CPU restatement in oracle/, all host threads) on the same four-layer step.
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


C5, C5_LAYERS, CFG5_SEEDS = 32, 2, (0, 1, 2, 3)
CFG5 = ("cfg5: 4 shapes (seeds 0-3), each a 512^3 shell R=200 h=0.5 subdivided with a Bernoulli(0.5) child mask "
        "(~2.0M voxels at 1024^3), 2 x SubMConv3d(32->32)+SiLU, bf16 in/f32 acc")


def cfg5_layers():
    """Weights of the cfg5 chain (one model shared by the four shapes)."""
    import t2sc
    S = t2sc.synth
    return [(S.normal(521 + 3 * i, (C5, 3, 3, 3, C5), std=(1.0 / (27 * C5)) ** 0.5), S.normal(522 + 3 * i, (C5,), std=0.1))
            for i in range(C5_LAYERS)]


def cfg5_coords(ctx, seed):
    """Child coordinates of one cfg5 shape: the seeded 512^3 parent shell
    subdivided on the GPU with a seeded Bernoulli(0.5) child mask."""
    import t2sc
    S = t2sc.synth
    parents = S.shell(*S.SHELLS["cfg5_parent"], seed=seed)
    mask = S.bernoulli(500 + seed, (len(parents), 8))
    x0 = np.zeros((len(parents), 8), np.float32)
    return t2sc.SparseUpsample(2).forward_subdivision(t2sc.SparseTensor(x0, parents, ctx=ctx), mask).coords


def conv_launch(L, _lib, ctx, cv, coords_handle, x, y, flags=1, residual=None):
    _lib.check(L.t2sc_conv_forward_device(cv.handle, coords_handle, ctypes.c_void_p(x.data_ptr()),
                                          ctypes.c_void_p(y.data_ptr()), flags,
                                          ctypes.c_void_p(residual.data_ptr()) if residual is not None else None),
               ctx.handle)


def timed(stream, fn, steps, warmup, flush):
    """W untimed calls, then K calls each bracketed by CUDA events on the
    launch stream with the L2 flushed before; returns the per-call ms list."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    out = []
    for _ in range(steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        fn()
        e1.record(stream)
        torch.cuda.synchronize()
        out.append(e0.elapsed_time(e1))
    return out


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


def reference_inputs():
    """The same seeded cfg4 inputs as inputs(), generated by the oracle's own
    restatement of the project RNG, so the CPU reference never loads the
    product library."""
    from oracle import oracle as O
    O.build()
    coords = O.synth_shell(*O.SHELLS["cfg4"])
    n = len(coords)
    x = O.synth_normal(400, (n, C))
    ws = [O.synth_normal(401 + 3 * i, (C, 3, 3, 3, C), std=(1.0 / (27 * C)) ** 0.5) for i in range(LAYERS)]
    bs = [O.synth_normal(402 + 3 * i, (C,), std=0.1) for i in range(LAYERS)]
    return coords, x, ws, bs


def run_reference(args):
    """`--impl reference`: the reference's CPU algorithm (the restatement of
    sparse/conv.mojo:56-199 in oracle/) on every host thread. One step is the
    whole GPU-arm step: the four SubMConv3d(64->64)+SiLU layers over all
    503,562 voxels, in f32 (the reference's CPU arithmetic), with the
    neighbour map built once beforehand as the reference caches it. Rows are
    split across threads; each row sums its edges in the reference's order."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle as O
    coords, x, ws, bs = reference_inputs()
    n = len(coords)
    src, tgt, kidx = O.neighbor_map(coords)
    E = len(src)
    rs, ss, ks = O.csr(n, src, tgt, kidx)
    del src, tgt, kidx
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)

    def step():
        h = x
        for w, b in zip(ws, bs):
            h = O.conv_rows(h, w, b, (rs, ss, ks), cores)
            O.lib().orc_silu(O._p(h), h.size)
        return h

    times = []
    for s in range(-args.warmup, args.steps):
        t0 = time.perf_counter()
        step()
        if s >= 0:
            times.append(time.perf_counter() - t0)
    t = float(np.sum(times))
    flops = LAYERS * 2.0 * E * C * C
    v = flops * args.steps / t / 1e12
    line = {"metric": METRIC, "value": v, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "mvoxel_per_s": LAYERS * n * args.steps / t / 1e6,
            "config": {"workload": WORKLOAD, "voxels": n, "edges": E, "layers": LAYERS, "channels": C,
                       "sample": "the whole step: 4 layers over all voxels (map built once, untimed)"},
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "nproc": os.cpu_count(), "threads": cores,
                             "kind": "port",
                             "sample": f"whole 4-layer cfg4 chain per step, f32, {cores} threads, rows split "
                                       f"across threads (oracle/t2sc_oracle.c orc_conv_forward_rows)"},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="t2sc", choices=["t2sc", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the cfg5 and cfg2 extra keys")
    ap.add_argument("--op", default="conv", choices=["conv", "layernorm", "map", "subdiv", "glue"],
                    help="layernorm / map / subdiv / glue: time the LayerNorm+SiLU glue kernel, the coordinate "
                         "hash + neighbour-map build (cfg4), the subdivision (cfg5 parents) or the pipeline glue "
                         "(trilinear sampler, cascade coordinates, FlexiDualGrid head) alone (not the headline)")
    args = ap.parse_args()
    if args.op == "layernorm":
        return run_layernorm(args)
    if args.op == "map":
        return run_map(args)
    if args.op == "subdiv":
        return run_subdiv(args)
    if args.op == "glue":
        return run_glue(args)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.gpus > 1 or int(os.environ.get("WORLD_SIZE", "1")) > 1:
        return run_distributed(args)
    return run_single(args)


def run_map(args):
    """Coordinate hash + 27-offset neighbour map of the cfg4 shell from
    device coordinates, as a decoder level pays it when its coordinates
    change: t2sc_coords_create_device (hash insert + range check) and
    t2sc_coords_build_map (row masks, mask sort, sorted neighbour rows, edge
    count). Algorithmic bytes (the survey's B_map): N*16 coords in +
    N*27*4 map out + 2*cap*12 hash (key + row, written then read; cap = the
    power of two >= 2N, a half-full table, independent of the library's own
    sparser table)."""
    import torch

    import t2sc
    ctx = t2sc.Context.default(0)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    coords, _, _, _ = inputs()
    n = len(coords)
    dc = torch.from_numpy(coords).cuda()
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    res = {}

    def once():
        c = t2sc.Coords(ctx, n=n, device_ptr=dc.data_ptr())
        res["E"] = c.build_map()
        del c

    ms = float(np.mean(timed(stream, once, args.steps, max(args.warmup, 3), flush)))
    cap = 1024
    while cap < 2 * n:
        cap *= 2
    alg = n * 16 + n * 27 * 4 + 2 * cap * 12
    _, hbm, src = peaks()
    gbs = alg / (ms * 1e-3) / 1e9
    print(json.dumps({"metric": "coordinate hash + neighbour-map build, cfg4 shell", "value": round(ms, 4),
                      "unit": "ms", "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3),
                      "higher_is_better": False, "dtype": "int32", "data": "synthetic",
                      "config": {"workload": f"cfg4 shell, {n} voxels, {res['E']} edges, 3x3x3, from device coords",
                                 "l2": "flushed between steps (256 MiB write)",
                                 "includes": "two host synchronisations (hash range check, edge count)"},
                      "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "peak_source": src,
                                   "unit": "GB/s", "frac": round(gbs / hbm, 4), "algorithmic_bytes": alg}}))


def run_subdiv(args):
    """2x subdivision of one cfg5 parent shell (seed 0, 503,562 parents,
    Bernoulli(0.5) child mask) with the parents' bf16 C=32 feature rows
    copied to the ~2M children (t2sc_subdivide_device, one host
    synchronisation to read M). Algorithmic bytes (the survey's B_sub):
    N*(16 + 8*4) + M*16 + M*C*2 (+ the N*C*2 parent rows read)."""
    import torch

    import t2sc
    from t2sc import _lib
    ctx = t2sc.Context.default(0)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    S = t2sc.synth
    parents = S.shell(*S.SHELLS["cfg5_parent"], seed=0)
    n = len(parents)
    dc = torch.from_numpy(parents).cuda()
    sub = torch.from_numpy(S.bernoulli(500, (n, 8))).cuda()
    x = torch.randn((n, C5), device="cuda").to(torch.bfloat16)
    oc = torch.empty((8 * n, 4), dtype=torch.int32, device="cuda")
    of = torch.empty((8 * n, C5), dtype=torch.bfloat16, device="cuda")
    par = torch.empty(8 * n, dtype=torch.int32, device="cuda")
    sidx = torch.empty(8 * n, dtype=torch.int32, device="cuda")
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    m = ctypes.c_int64()
    P = ctypes.c_void_p

    def once():
        _lib.check(_lib.lib.t2sc_subdivide_device(ctx.handle, P(dc.data_ptr()), n, P(sub.data_ptr()), _lib.SUB_NONZERO,
                                                  P(x.data_ptr()), C5, _lib.FEATS_UPSAMPLE, _lib.DT_BF16,
                                                  P(oc.data_ptr()), P(of.data_ptr()), P(par.data_ptr()),
                                                  P(sidx.data_ptr()), ctypes.byref(m)), ctx.handle)

    ms = float(np.mean(timed(stream, once, args.steps, max(args.warmup, 3), flush)))
    M = m.value
    alg = n * (16 + 8 * 4) + M * 16 + M * C5 * 2 + n * C5 * 2
    _, hbm, src = peaks()
    gbs = alg / (ms * 1e-3) / 1e9
    print(json.dumps({"metric": "subdivision upsample, cfg5 parent shell", "value": round(ms, 4), "unit": "ms",
                      "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3), "higher_is_better": False,
                      "dtype": "int32 + bf16 rows", "data": "synthetic",
                      "config": {"workload": f"{n} parents -> {M} children, C={C5} bf16 feature rows",
                                 "l2": "flushed between steps (256 MiB write)",
                                 "includes": "one host synchronisation (child count)"},
                      "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "peak_source": src,
                                   "unit": "GB/s", "frac": round(gbs / hbm, 4), "algorithmic_bytes": alg}}))


def run_glue(args):
    """The pipeline glue kernels, one JSON line each, with the oracle timed on
    the same inputs on one host thread (kind "port"):
      grid_sample: the cfg4 shell's 503,562 voxels (C = 6 f32 features, the
        texture decoder's PBR channels) sampled at 2M points near the surface;
        the coordinate hash is the handle's, built before timing.
        Algorithmic bytes: L*12 query + L*C*4 out + N*C*4 features + hash.
      cascade: 1,007,124 coordinates at resolution 512 (the cfg4 shell in two
        batches) -> 64^3 tokens (lr 512, target 1024, budget 49152); includes
        the two host read-backs. Algorithmic bytes: n*16 in + T*16 out.
      fdg_head: 2M rows of 7 f32 channels. Algorithmic bytes: T*7*4 + T*7*4."""
    import torch

    import t2sc
    from oracle import oracle as O
    ctx = t2sc.Context.default(0)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    S = t2sc.synth
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    _, hbm, src = peaks()
    W = max(args.warmup, 3)

    def line(name, ms, alg, workload, extra, cpu_s, cpu_sample):
        gbs = alg / (ms * 1e-3) / 1e9
        print(json.dumps({"metric": name, "value": round(ms, 4), "unit": "ms", "n_gpus": 1, "steps": args.steps,
                          "warmup": W, "higher_is_better": False, "dtype": "f32 / int32", "data": "synthetic",
                          "config": {"workload": workload, "l2": "flushed between steps (256 MiB write)", **extra},
                          "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "peak_source": src,
                                       "unit": "GB/s", "frac": round(gbs / hbm, 4), "algorithmic_bytes": alg},
                          "cpu_baseline": {"value": round(cpu_s * 1e3, 2), "unit": "ms", "cores": 1, "kind": "port",
                                           "sample": cpu_sample}}), flush=True)

    # ---- trilinear sampler ----
    c = S.shell(*S.SHELLS["cfg4"])
    n, C, L = len(c), 6, 2_000_000
    xyz = np.ascontiguousarray(c[:, 1:])
    feats = S.normal(42, (n, C))
    rng = np.random.default_rng(1)
    q = (xyz[rng.integers(0, n, L)] + rng.uniform(-1, 2, size=(L, 3))).astype(np.float32)
    coords = t2sc.Coords(ctx, c)
    df, dq = torch.from_numpy(feats).cuda(), torch.from_numpy(q).cuda()
    ms = float(np.mean(timed(stream, lambda: t2sc.grid_sample_trilinear_device(coords, df, 512, dq), args.steps,
                             W, flush)))
    hcap = 1 << int(np.ceil(np.log2(max(2 * n, 1024))))  # a half-full table, whatever the library's
    t0 = time.perf_counter()
    O.grid_sample_trilinear(feats, xyz, 512, q[:200_000])
    cpu = (time.perf_counter() - t0) * L / 200_000
    line("trilinear sampler, cfg4 shell", ms, L * 12 + L * C * 4 + n * C * 4 + hcap * 16,
         f"{n} voxels x {C} f32 channels sampled at {L} points", {"queries": L}, cpu,
         "oracle on the first 200,000 queries, scaled to 2M")
    # ---- cascade coordinates ----
    c2 = c.copy()
    c2[:, 0] = 1
    c2[:, 1:] = (c2[:, 1:] + 37) % 512
    hr = np.concatenate([c, c2])
    dh = torch.from_numpy(hr).cuda()
    res = {}

    def cas():
        res["out"] = t2sc.cascade_coords_device(dh, 512, 1024, 49152, ctx)

    ms = float(np.mean(timed(stream, cas, args.steps, W, flush)))
    T = len(res["out"][0])
    t0 = time.perf_counter()
    O.cascade_coords(hr, 512, 1024, 49152)
    cpu = time.perf_counter() - t0
    line("cascade coordinates, 512 -> 64^3 tokens", ms, len(hr) * 16 + T * 16,
         f"{len(hr)} coordinates at 512 (2 batches) -> {T} tokens, target 1024, budget 49152",
         {"includes": "two host read-backs (maximum q, token count)"}, cpu, "oracle on the whole input")
    # ---- FlexiDualGrid head ----
    Tn = 2_000_000
    f7 = torch.from_numpy(S.normal(43, (Tn, 7), 4.0)).cuda()
    ms = float(np.mean(timed(stream, lambda: t2sc.fdg_head_device(f7, 0.5, ctx), args.steps, W, flush)))
    f7h = f7.cpu().numpy()
    t0 = time.perf_counter()
    O.fdg_head(f7h, 0.5)
    cpu = time.perf_counter() - t0
    line("FlexiDualGrid head", ms, Tn * 7 * 4 * 2, f"{Tn} rows x 7 f32 channels", {}, cpu,
         "oracle on the whole input")


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


def extra_single(args, ctx, stream, flush):
    """cfg5 (the 1024^3 cascade: all four shapes on this GPU) and cfg2's
    f32 / f16 layers, timed like the headline (CUDA events on the launch
    stream, L2 flushed between steps). Reported as extra keys."""
    import torch

    import t2sc
    from t2sc import _lib
    L = _lib.lib
    out = {}
    peak_tf, peak_bw, _ = peaks()
    # ---- cfg5: 4 shapes x 2 layers ----
    convs = [t2sc.SparseConv3d(w, b, dtype="bf16", ctx=ctx) for w, b in cfg5_layers()]
    shapes, flops, vox = [], 0.0, 0
    for sd in CFG5_SEEDS:
        coords = cfg5_coords(ctx, sd)
        cd = t2sc.Coords(ctx, coords)
        e = cd.build_map()
        g = torch.Generator(device="cuda").manual_seed(520 + sd)
        x = torch.randn((len(coords), C5), device="cuda", generator=g).to(torch.bfloat16)
        bufs = [torch.empty_like(x) for _ in range(2)]
        shapes.append((cd, x, bufs))
        flops += C5_LAYERS * 2.0 * e * C5 * C5
        vox += len(coords)

    def step5():
        for cd, x, bufs in shapes:
            cur = x
            for i, cv in enumerate(convs):
                conv_launch(L, _lib, ctx, cv, cd.handle, cur, bufs[i & 1])
                cur = bufs[i & 1]

    ms = float(np.mean(timed(stream, step5, args.steps, args.warmup, flush)))
    out.update({"cfg5_tflops": flops / (ms * 1e-3) / 1e12, "cfg5_ms_per_step": ms, "cfg5_voxels": vox,
                "cfg5_mvoxel_per_s": C5_LAYERS * vox / (ms * 1e-3) / 1e6, "cfg5_frac": flops / (ms * 1e-3) / 1e12 / peak_tf,
                "cfg5_workload": CFG5})
    del shapes
    # ---- cfg2: one SubMConv3d(256->256) layer in f32 (split-TF32) and f16 ----
    S = t2sc.synth
    coords = S.shell(*S.SHELLS["cfg2"])
    n, c = len(coords), 256
    cd = t2sc.Coords(ctx, coords)
    e = cd.build_map()
    w = S.normal(201, (c, 3, 3, 3, c), std=(1.0 / (27 * c)) ** 0.5)
    b = S.normal(202, (c,), std=0.1)
    g = torch.Generator(device="cuda").manual_seed(200)
    x32 = torch.randn((n, c), device="cuda", generator=g)
    f = 2.0 * e * c * c
    for key, dt, wt, tdt, peak, label in (
            ("f32", "f32", w, torch.float32, peak_tf / 6, "TF32x3 = measured bf16 peak / 6"),
            ("f16", "f16", w, torch.float16, peak_tf, "measured bf16 peak")):
        cv = t2sc.SparseConv3d(wt, b, dtype=dt, ctx=ctx)
        xin = x32.to(tdt)
        y = torch.empty_like(xin)
        ms2 = float(np.mean(timed(stream, lambda: conv_launch(L, _lib, ctx, cv, cd.handle, xin, y, 0),
                                  args.steps, args.warmup, flush)))
        out[f"cfg2_{key}_layer_ms"] = ms2
        out[f"cfg2_{key}_tflops"] = f / (ms2 * 1e-3) / 1e12
        out[f"cfg2_{key}_frac"] = out[f"cfg2_{key}_tflops"] / peak
        out[f"cfg2_{key}_peak"] = label
    return out


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
    map_first_ms = 1e3 * (time.perf_counter() - t0)  # includes one-time kernel module loading
    # the map build as a decoder level pays it when its coordinates change:
    # hash + map of a fresh coordinate handle (host wall clock, synchronised)
    dcoords = torch.from_numpy(coords).cuda()
    warm = []
    for _ in range(3):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        c2 = t2sc.Coords(ctx, n=n, device_ptr=dcoords.data_ptr())
        c2.build_map()
        torch.cuda.synchronize()
        warm.append(1e3 * (time.perf_counter() - t0))
        del c2
    map_ms = float(np.median(warm))

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

    extra = {} if args.no_extra else extra_single(args, ctx, stream, flush)
    cpu = None
    if not args.no_cpu_baseline:
        v, ne, etot, dt = cpu_baseline_sample(coords, x, ws[0], bs[0])
        cpu = {"value": v, "unit": UNIT, "cores": min(os.cpu_count() or 1, C // 8), "threads": C // 8,
               "nproc": os.cpu_count(), "kind": "port",
               "sample": f"layer 1, first {ne} of {etot} edges (kernel-offset-major), reference Co-chunk "
                         f"parallelism ({C // 8} threads), {dt:.1f} s"}
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "mvoxel_per_s": mvox, "map_build_ms": map_ms, "map_build_first_ms": map_first_ms,
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
    line.update(extra)
    print(json.dumps(line))


def run_distributed(args):
    """One rank per GPU (torchrun). cfg4 (the headline): the shell is cut
    into z-slabs by the library (t2sc_partition_zslab); once per step each
    rank receives a 4-plane halo from its z-neighbours through the library's
    own NCCL communicator (t2sc_halo_exchange_device), then runs the four
    layers on all its rows (own + halo): the halo rows' results are right
    one plane less deep after every layer, the own rows after all four. Total work is
    fixed as N grows (strong scaling); `value` is the whole job's TFLOP/s
    over the slowest rank. cfg5 (extra keys): the four shapes are spread
    over the ranks (data parallel), and at N = 8 each shape is z-sharded
    over a group of two ranks with its own communicator. torch.distributed
    carries only the plumbing (unique-id broadcast, barriers, max/sum of
    the timings)."""
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
    L = _lib.lib
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")

    # one unique id per communicator: [0] the cfg4 slab group (all ranks),
    # [1..4] the cfg5 shape groups
    ids = [dist.Comm.unique_id() for _ in range(1 + len(CFG5_SEEDS))] if rank == 0 else [None]
    obj = [ids]
    tdist.broadcast_object_list(obj, src=0)
    ids = obj[0]

    # ------------------------------- cfg4 -------------------------------
    coords, x, ws, bs = inputs()
    comm = dist.Comm(ctx, ids[0], world, rank)
    # a halo LAYERS planes deep, exchanged once per step: layer l is right on
    # the own rows and the first LAYERS - l halo planes, so after the last
    # layer the own rows equal the global chain (no exchange between layers)
    slab = dist.NativeSlab(coords, world, rank, depth=LAYERS)
    rows, n_own = slab.rows, slab.n_own
    n_loc = len(rows)
    convs = [t2sc.SparseConv3d(w, b, dtype="bf16", ctx=ctx) for w, b in zip(ws, bs)]
    c_all = t2sc.Coords(ctx, coords[rows])  # every local row is a target
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    c_all.build_map()
    torch.cuda.synchronize()
    map_ms = 1e3 * (time.perf_counter() - t0)
    # useful work = the edges of the own rows (the halo rows' convs are redundant)
    e_loc = t2sc.Coords(ctx, coords[rows], n_targets=n_own).build_map()
    e_all = torch.tensor([e_loc], dtype=torch.int64, device="cuda")
    tdist.all_reduce(e_all)
    E = int(e_all.item())
    xin = torch.zeros((n_loc, C), dtype=torch.bfloat16, device="cuda")
    xin[:n_own] = torch.from_numpy(x[slab.own]).to("cuda").to(torch.bfloat16)
    bufs = [torch.zeros((n_loc, C), dtype=torch.bfloat16, device="cuda") for _ in range(2)]

    def step():
        cur = xin
        comm.exchange(cur, slab.counts)  # the step input's deep halo
        for i, cv in enumerate(convs):
            out = bufs[i & 1]
            conv_launch(L, _lib, ctx, cv, c_all.handle, cur, out)
            cur = out
        return cur

    for _ in range(args.warmup):
        step()
    comm.wait()
    # The step (4 x (halo exchange + conv)) is captured once in a CUDA graph:
    # at 4-8 ranks a layer is ~20 us of GPU work, less than the host needs
    # to issue it eagerly. Falls back to eager launches if capture fails.
    graph = None
    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step()
        torch.cuda.synchronize()
        g.replay()
        comm.wait()
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
    tok = torch.zeros(1, device="cuda")
    for _ in range(args.steps):
        flush.zero_()
        torch.cuda.synchronize()
        tdist.barrier()
        # the host barrier releases the ranks microseconds to ~0.1 ms apart; a
        # one-element all-reduce ordered before the start event aligns them
        # on the device, so that no rank's timed step includes waiting for a
        # peer that has not launched yet
        tdist.all_reduce(tok)
        s0, s1 = ev(), ev()
        s0.record(stream)
        run()
        s1.record(stream)
        torch.cuda.synchronize()
        times.append(s0.elapsed_time(s1))
    launches = ctx.launch_count() - launches0 if graph is None else len(convs) * args.steps
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
    for s_ in range(args.steps + 2):
        torch.cuda.synchronize()
        tdist.barrier()
        t0 = time.perf_counter()
        xin[:n_own].copy_(xh.to("cuda", non_blocking=True))
        run()
        out = bufs[(len(convs) - 1) & 1]
        yh.copy_(out[:n_own].float(), non_blocking=True)
        torch.cuda.synchronize()
        if s_ >= 2:
            e2e.append(time.perf_counter() - t0)
    et = torch.tensor(e2e, dtype=torch.float64, device="cuda")
    tdist.all_reduce(et, op=tdist.ReduceOp.MAX)
    e2e_s = float(et.sum().item()) / args.steps
    graph = g = None  # noqa: F841  (the graph holds NCCL work of `comm`)
    torch.cuda.synchronize()

    # ------------------------------- cfg5 -------------------------------
    extra = {}
    if not args.no_extra:
        extra = run_cfg5_distributed(args, ctx, stream, flush, ids, rank, world)

    if rank == 0:
        flops = LAYERS * 2.0 * E * C * C
        n = len(coords)
        line = {"metric": METRIC, "value": flops / (ms * 1e-3) / 1e12, "unit": UNIT, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "mvoxel_per_s": LAYERS * n / (ms * 1e-3) / 1e6, "map_build_ms": map_ms,
                "config": {"workload": WORKLOAD, "voxels": n, "edges": E, "layers": LAYERS, "channels": C,
                           "l2": "flushed between steps (256 MiB write)",
                           "parallelism": f"z-slab x{world}, {LAYERS}-plane halo over the library's NCCL send/recv once per "
                                          "step, every layer on own + halo rows",
                           "rank0_rows": n_own, "rank0_halo_rows": n_loc - n_own,
                           "cuda_graph": run is not step},
                "e2e": {"value": flops / e2e_s / 1e12, "unit": UNIT, "h2d_bytes_per_step": n * C * 4,
                        "d2h_bytes_per_step": n * C * 4, "ms_per_step": 1e3 * e2e_s},
                "gpu_launches": launches, "clocks": clk.summary if clk else None, "cpu_baseline": None,
                "gpus_active": world}
        line.update(extra)
        print(json.dumps(line))
    sys.stdout.flush()
    teardown(tdist, comm, rank)


def teardown(tdist, comm, rank):
    """Ends a distributed run: the library's communicator is finalised and
    destroyed (bounded inside the library), then torch's process group. Its
    teardown has blocked at exit on this pool after the run's work was done,
    so a watchdog ends the process 10 s after the results were printed if it
    does not return; each step is logged to stderr with its time."""
    import threading

    t0 = time.perf_counter()

    def log(msg):
        print(f"# rank {rank} teardown +{time.perf_counter() - t0:.2f}s: {msg}", file=sys.stderr, flush=True)

    def watchdog():
        time.sleep(10)
        log("process-group teardown did not return within 10 s; exiting")
        os._exit(0)

    threading.Thread(target=watchdog, daemon=True).start()
    tdist.barrier()
    comm.close()
    log("library communicator destroyed")
    tdist.destroy_process_group()
    log("process group destroyed")


def run_cfg5_distributed(args, ctx, stream, flush, ids, rank, world):
    """cfg5 over `world` ranks: shapes round-robin when world <= 4, else
    groups of world // 4 ranks per shape with a z-slab split and a halo
    exchange of a two-plane halo per shape and step on the group's own
    communicator."""
    import torch
    import torch.distributed as tdist

    import t2sc
    from t2sc import _lib, dist
    L = _lib.lib
    convs = [t2sc.SparseConv3d(w, b, dtype="bf16", ctx=ctx) for w, b in cfg5_layers()]
    nshape = len(CFG5_SEEDS)
    gs = world // nshape if world > nshape and world % nshape == 0 else 1
    if gs == 1:
        mine = [i for i in range(nshape) if i % world == rank]
    else:
        mine = [rank // gs]
    work, comms = [], []
    e_loc, vox = 0, 0
    for i in mine:
        coords = cfg5_coords(ctx, CFG5_SEEDS[i])
        g = torch.Generator(device="cuda").manual_seed(520 + CFG5_SEEDS[i])
        xg = torch.randn((len(coords), C5), device="cuda", generator=g).to(torch.bfloat16)
        if gs == 1:
            cd = t2sc.Coords(ctx, coords)
            x, counts, comm = xg, None, None
        else:
            comm = dist.Comm(ctx, ids[1 + i], gs, rank % gs)
            comms.append(comm)
            # a C5_LAYERS-plane halo exchanged once per shape and step; both
            # layers run on own + halo rows (see the cfg4 split above)
            sl = dist.NativeSlab(coords, gs, rank % gs, depth=C5_LAYERS)
            cd = t2sc.Coords(ctx, coords[sl.rows])
            x = torch.zeros((len(sl.rows), C5), dtype=torch.bfloat16, device="cuda")
            x[:sl.n_own] = xg[torch.from_numpy(sl.own).cuda()]
            counts = sl.counts
        cd.build_map()
        own = cd if gs == 1 else t2sc.Coords(ctx, coords[sl.rows], n_targets=sl.n_own)
        e_loc += own.build_map()  # useful work: the own rows' edges
        vox += cd.n if gs == 1 else sl.n_own
        bufs = [torch.zeros_like(x) for _ in range(2)]
        work.append((cd, x, bufs, comm, counts))

    def step5():
        for cd, x, bufs, comm, counts in work:
            cur = x
            if comm is not None:
                comm.exchange(cur, counts)
            for j, cv in enumerate(convs):
                conv_launch(L, _lib, ctx, cv, cd.handle, cur, bufs[j & 1])
                cur = bufs[j & 1]

    for _ in range(args.warmup):
        step5()
    torch.cuda.synchronize()
    tok = torch.zeros(1, device="cuda")
    times = []
    for _ in range(args.steps):
        flush.zero_()
        torch.cuda.synchronize()
        tdist.barrier()
        tdist.all_reduce(tok)  # device-side alignment of the ranks (as for cfg4)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        step5()
        e1.record(stream)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    tt = torch.tensor(times, dtype=torch.float64, device="cuda")
    tdist.all_reduce(tt, op=tdist.ReduceOp.MAX)
    ms = float(tt.sum().item()) / args.steps
    tot = torch.tensor([e_loc, vox], dtype=torch.int64, device="cuda")
    tdist.all_reduce(tot)
    E5, V5 = int(tot[0].item()), int(tot[1].item())
    flops = C5_LAYERS * 2.0 * E5 * C5 * C5
    peak_tf, _, _ = peaks()
    for comm in comms:
        comm.close()
    return {"cfg5_tflops": flops / (ms * 1e-3) / 1e12, "cfg5_ms_per_step": ms, "cfg5_voxels": V5,
            "cfg5_mvoxel_per_s": C5_LAYERS * V5 / (ms * 1e-3) / 1e6,
            "cfg5_frac": flops / (ms * 1e-3) / 1e12 / peak_tf / world, "cfg5_workload": CFG5,
            "cfg5_parallelism": (f"shapes round-robin over {world} ranks" if gs == 1 else
                                 f"{nshape} groups of {gs} ranks, z-slab + halo inside a group"),
            "cfg5_scaling": "strong"}


if __name__ == "__main__":
    main()
