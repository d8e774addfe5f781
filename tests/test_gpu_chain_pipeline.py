"""The conv chain over host buffers (t2sc_conv_chain_forward) on a large
coordinate set ordered by (batch, x) runs as overlapped slabs (uploads,
slab chains and downloads on three streams, each slab with a halo as deep
as the chain's reach). Every output row must equal the same layers run
unsplit on the device: the slab split changes which rows share a tile, not
any row's arithmetic, so the comparison is exact."""
import ctypes

import numpy as np
import pytest

from _cases import conv_inputs

pytestmark = pytest.mark.gpu


def _unsplit(t2sc, convs, coords, x, flags, tdt):
    import torch
    from t2sc import _lib
    ctx = convs[0].ctx
    ctx.set_stream(1)
    try:
        cd = t2sc.Coords(ctx, coords)
        x0 = torch.from_numpy(x).cuda().to(tdt)
        cur = x0
        for cv, f in zip(convs, flags):
            out = torch.empty((len(coords), cv.out_channels), dtype=tdt, device="cuda")
            res = x0 if f & _lib.RESIDUAL else None
            _lib.check(_lib.lib.t2sc_conv_forward_device(cv.handle, cd.handle, ctypes.c_void_p(cur.data_ptr()),
                                                         ctypes.c_void_p(out.data_ptr()), f,
                                                         ctypes.c_void_p(res.data_ptr()) if res is not None else None),
                       ctx.handle)
            cur = out
        torch.cuda.synchronize()
        return cur.float().cpu().numpy()
    finally:
        ctx.set_stream(None)


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_pipelined_chain_equals_unsplit_cfg4(t2sc, dtype):
    import torch
    from t2sc import _lib
    S = t2sc.synth
    ctx = t2sc.Context.default(0)
    coords = S.shell(*S.SHELLS["cfg4"])  # lexicographic (batch, x, y, z): pipelined
    n, c = len(coords), 64
    x, _, _ = conv_inputs(S, n, c, c, seed=90)
    layers = [conv_inputs(S, 1, c, c, seed=91 + i)[1:] for i in range(4)]
    convs = [t2sc.SparseConv3d(w, b, dtype=dtype, ctx=ctx) for w, b in layers]
    flags = [_lib.SILU, _lib.SILU, _lib.SILU, _lib.SILU | _lib.RESIDUAL]
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    if dtype == "bf16":
        x = torch.from_numpy(x).to(torch.bfloat16).float().numpy()  # the same inputs on both sides
    y = t2sc.conv_chain(convs, t2sc.SparseTensor(x, coords, ctx=ctx), flags).feats
    ref = _unsplit(t2sc, convs, coords, x, flags, tdt)
    assert np.array_equal(y, ref)
    y2 = t2sc.conv_chain(convs, t2sc.SparseTensor(x, coords, ctx=ctx), flags).feats  # cached plan
    assert np.array_equal(y2, ref)


def test_unordered_and_small_sets_run_unsplit(t2sc):
    import torch
    from t2sc import _lib
    S = t2sc.synth
    ctx = t2sc.Context.default(0)
    coords = S.shell(*S.SHELLS["cfg4"])
    rng = np.random.default_rng(3)
    shuffled = coords[rng.permutation(len(coords))]  # not ordered by x: one unsplit run
    small = S.shell(*S.SHELLS["cfg1"])
    for crd in (shuffled, small):
        n = len(crd)
        x, w, b = conv_inputs(S, n, 32, 32, seed=95)
        x = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
        convs = [t2sc.SparseConv3d(w, b, dtype="bf16", ctx=ctx) for _ in range(2)]
        y = t2sc.conv_chain(convs, t2sc.SparseTensor(x, crd, ctx=ctx), [_lib.SILU, _lib.SILU]).feats
        ref = _unsplit(t2sc, convs, crd, x, [_lib.SILU, _lib.SILU], torch.bfloat16)
        assert np.array_equal(y, ref)
