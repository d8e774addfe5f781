"""z-slab partition on one GPU: each rank's conv on (own + halo) rows,
outputs for own rows only (t2sc_coords_create_halo), equals the global conv
on those rows. The NCCL exchange itself is covered by the gloo test and
by bench.py under torchrun."""
import ctypes

import numpy as np
import pytest

from _cases import F16_TOL, conv_inputs, rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world,dtype", [(2, "bf16"), (4, "bf16"), (3, "f32")])
def test_slabs_equal_global_conv(t2sc, world, dtype):
    from t2sc import _lib, dist
    S = t2sc.synth
    ctx = t2sc.Context.default(0)
    coords = S.shell(*S.SHELLS["cfg1"])
    x, w, b = conv_inputs(S, len(coords), 64, 64, seed=77)
    conv = t2sc.SparseConv3d(w, b, dtype=dtype, ctx=ctx)
    ref = conv.forward(t2sc.SparseTensor(x, coords, ctx=ctx), silu=True).feats
    for sl in dist.partition(coords, world):
        rows = sl.rows
        c = t2sc.Coords(ctx, coords[rows], n_targets=sl.n_own)
        y = np.empty((sl.n_own, 64), np.float32)
        xl = np.ascontiguousarray(x[rows])
        _lib.check(_lib.lib.t2sc_conv_forward(conv.handle, c.handle, xl.ctypes.data_as(ctypes.c_void_p),
                                              y.ctypes.data_as(ctypes.c_void_p), _lib.SILU, None), ctx.handle)
        assert rel_err(y, ref[sl.own]) <= (1e-6 if dtype == "f32" else F16_TOL)
        # interior and boundary target ranges computed separately fill the same rows
        y2 = np.empty((sl.n_own, 64), np.float32)
        for t0, t1 in ((0, sl.n_int), (sl.n_int, sl.n_own)):
            if t1 == t0:
                continue
            cr = t2sc.Coords(ctx, coords[rows], targets=(t0, t1))
            part = np.empty((t1 - t0, 64), np.float32)
            _lib.check(_lib.lib.t2sc_conv_forward(conv.handle, cr.handle, xl.ctypes.data_as(ctypes.c_void_p),
                                                  part.ctypes.data_as(ctypes.c_void_p), _lib.SILU, None), ctx.handle)
            y2[t0:t1] = part
        assert rel_err(y2, ref[sl.own]) <= (1e-6 if dtype == "f32" else F16_TOL)


@pytest.mark.parametrize("world", [2, 4])
def test_deep_halo_four_layers_equal_global_chain(t2sc, world):
    """One exchange of a 4-plane halo per 4-layer step: every layer runs on
    all local rows (own + halo), each layer's results are right one plane
    further in, so after four layers the own rows equal the global chain."""
    import torch
    from t2sc import _lib, dist
    S = t2sc.synth
    ctx = t2sc.Context.default(0)
    ctx.set_stream(1)  # the legacy default stream: ordered with torch's default-stream work
    try:
        _deep_halo_case(t2sc, ctx, S, world)
    finally:
        ctx.set_stream(None)


def _deep_halo_case(t2sc, ctx, S, world):
    import torch
    from t2sc import _lib, dist
    coords = S.shell(*S.SHELLS["cfg1"])
    n, c = len(coords), 64
    x, _, _ = conv_inputs(S, n, c, c, seed=78)
    layers = [conv_inputs(S, 1, c, c, seed=79 + i)[1:] for i in range(4)]
    convs = [t2sc.SparseConv3d(w, b, dtype="bf16", ctx=ctx) for w, b in layers]

    def chain(crd, xd):
        cur = xd
        for cv in convs:
            out = torch.empty_like(cur)
            _lib.check(_lib.lib.t2sc_conv_forward_device(cv.handle, crd.handle, ctypes.c_void_p(cur.data_ptr()),
                                                         ctypes.c_void_p(out.data_ptr()), _lib.SILU, None),
                       ctx.handle)
            cur = out
        torch.cuda.synchronize()
        return cur.float().cpu().numpy()

    xg = torch.from_numpy(x).cuda().to(torch.bfloat16)
    ref = chain(t2sc.Coords(ctx, coords), xg)
    for r in range(world):
        sl = dist.NativeSlab(coords, world, r, depth=4)
        xl = xg[torch.from_numpy(sl.rows).cuda()].contiguous()  # own rows + the exchanged 4-plane halo
        y = chain(t2sc.Coords(ctx, coords[sl.rows]), xl)
        assert rel_err(y[:sl.n_own], ref[sl.own]) <= F16_TOL
