"""The library's own NCCL data plane (t2sc_comm_*, t2sc_halo_exchange_device)
on two GPUs: two processes, one per GPU, partition the cfg1 shell with
t2sc_partition_zslab, exchange the halo of a feature matrix through libt2sc
and run the slab conv; every rank's outputs equal the single-GPU conv on its
own rows. Skipped on a box with fewer than two GPUs (the host logic is
covered on CPU by test_dist_host.py)."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

WORKER = r'''
import ctypes, os, sys
sys.path[:0] = [ROOT, ROOT + "/trellis2-mojo_b200", ROOT + "/tests"]
import numpy as np, torch
import t2sc
from t2sc import _lib, dist
from _cases import conv_inputs, rel_err
rank, world, uid_path = int(sys.argv[1]), int(sys.argv[2]), sys.argv[3]
torch.cuda.set_device(rank)
ctx = t2sc.Context(rank)
S = t2sc.synth
coords = S.shell(*S.SHELLS["cfg1"])
x, w, b = conv_inputs(S, len(coords), 64, 64, seed=91)
conv = t2sc.SparseConv3d(w, b, dtype="bf16", ctx=ctx)
ref = conv.forward(t2sc.SparseTensor(x, coords, ctx=ctx), silu=True).feats
uid = open(uid_path, "rb").read()
comm = dist.Comm(ctx, uid, world, rank, timeout_ms=60000)
sl = dist.NativeSlab(coords, world, rank)
xd = torch.zeros((len(sl.rows), 64), dtype=torch.bfloat16, device=f"cuda:{rank}")
xd[:sl.n_own] = torch.from_numpy(x[sl.own]).to(xd.device).to(torch.bfloat16)
torch.cuda.synchronize()
comm.exchange(xd, sl.counts)
comm.wait(30000)
halo = xd[sl.n_own:].float().cpu().numpy()
want = torch.from_numpy(x[sl.rows[sl.n_own:]]).to(torch.bfloat16).float().numpy()
assert np.array_equal(halo, want), "halo rows differ"
cd = t2sc.Coords(ctx, coords[sl.rows], n_targets=sl.n_own)
y = torch.empty((sl.n_own, 64), dtype=torch.bfloat16, device=xd.device)
_lib.check(_lib.lib.t2sc_conv_forward_device(conv.handle, cd.handle, ctypes.c_void_p(xd.data_ptr()),
                                             ctypes.c_void_p(y.data_ptr()), _lib.SILU, None), ctx.handle)
ctx.synchronize()
err = rel_err(y.float().cpu().numpy(), ref[sl.own])
assert err <= 1e-2, err
comm.close()
print("rank", rank, "ok", err)
'''


def test_two_gpu_halo_exchange_and_slab_conv(tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    sys.path[:0] = [os.path.join(ROOT, "trellis2-mojo_b200")]
    from t2sc import dist
    uid = tmp_path / "uid.bin"
    uid.write_bytes(dist.Comm.unique_id())
    script = tmp_path / "worker.py"
    script.write_text(f"ROOT = {ROOT!r}\n" + WORKER)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, str(script), str(r), "2", str(uid)], env=env,
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True) for r in range(2)]
    outs = []
    for p in procs:
        try:
            outs.append(p.communicate(timeout=300)[0])
        except subprocess.TimeoutExpired:
            p.kill()
            outs.append(p.communicate()[0])
    for p, o in zip(procs, outs):
        assert p.returncode == 0, o[-3000:]
