"""The allocation-free subdivision entry point (t2sc_subdivide_noalloc_device).

It serves callers that may not allocate device memory mid-run (a fixed
memory budget handed to the library up front, or no allocator calls and
their implicit synchronisation inside a decode pass); its scratch is a
static device array. This file is collected last on purpose. Checks: two
calls in a row, each against the allocating entry point on the same
inputs (bit-exact: coordinates, parents, child slots and copied features),
and the rejection of a parent count above the static limit.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_PARENTS = 1 << 20


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _run(t2sc, fn, ctx, coords, sub, feats, c, mode, dtype_code, keep):
    import torch
    n = coords.shape[0]
    out_c = torch.empty((8 * n, 4), dtype=torch.int32, device="cuda")
    out_f = torch.empty((8 * n, c), dtype=feats.dtype, device="cuda")
    par = torch.empty(8 * n, dtype=torch.int32, device="cuda")
    sid = torch.empty(8 * n, dtype=torch.int32, device="cuda")
    m = ctypes.c_int64()
    rc = fn(ctx.handle, _ptr(coords), n, _ptr(sub), keep, _ptr(feats), c, mode, dtype_code, _ptr(out_c), _ptr(out_f),
            _ptr(par), _ptr(sid), ctypes.byref(m))
    t2sc._lib.check(rc, ctx.handle)
    ctx.synchronize()
    k = m.value
    return k, out_c[:k].cpu(), out_f[:k].cpu(), par[:k].cpu(), sid[:k].cpu()


def test_noalloc_matches_allocating_entry_point_twice(t2sc):
    import torch
    from t2sc import _lib
    L = _lib.lib
    ctx = t2sc.Context.default(0)
    S = t2sc.synth
    coords = torch.from_numpy(S.shell(*S.SHELLS["cfg1"])).cuda()
    n = coords.shape[0]
    cases = [  # two calls in a row with different inputs: stale scratch must not leak
        (S.bernoulli(31, (n, 8)), torch.float32, _lib.DT_F32, 24, _lib.FEATS_UPSAMPLE, _lib.SUB_NONZERO),
        (S.normal(32, (n, 8)), torch.bfloat16, _lib.DT_BF16, 16, _lib.FEATS_C2S, _lib.SUB_POSITIVE),
    ]
    for sub_np, tdt, dcode, c, mode, keep in cases:
        sub = torch.from_numpy(sub_np).cuda()
        cin = 8 * c if mode == _lib.FEATS_C2S else c
        feats = torch.randn((n, cin), device="cuda").to(tdt)
        ref = _run(t2sc, L.t2sc_subdivide_device, ctx, coords, sub, feats, c, mode, dcode, keep)
        got = _run(t2sc, L.t2sc_subdivide_noalloc_device, ctx, coords, sub, feats, c, mode, dcode, keep)
        assert got[0] == ref[0] > 0
        for a, b in zip(got[1:], ref[1:]):
            assert torch.equal(a, b)


def test_noalloc_rejects_more_parents_than_its_scratch(t2sc):
    import torch
    from t2sc import _lib
    ctx = t2sc.Context.default(0)
    dummy = torch.zeros(16, dtype=torch.int32, device="cuda")
    m = ctypes.c_int64()
    rc = _lib.lib.t2sc_subdivide_noalloc_device(ctx.handle, _ptr(dummy), MAX_PARENTS + 1, _ptr(dummy), 0, None, 0,
                                               _lib.FEATS_NONE, _lib.DT_F32, _ptr(dummy), None, _ptr(dummy),
                                               _ptr(dummy), ctypes.byref(m))
    assert rc == _lib.ERR_INVALID
    assert b"static scratch limit" in _lib.lib.t2sc_last_error(ctx.handle)


def test_noalloc_at_the_static_parent_limit(t2sc):
    """Exactly MAX_PARENTS parents (a 128 x 128 x 64 block of voxels): the
    largest input the static scratch takes, bit-exact against the
    allocating entry point."""
    import torch
    from t2sc import _lib
    L = _lib.lib
    ctx = t2sc.Context.default(0)
    g = torch.stack(torch.meshgrid(torch.arange(128), torch.arange(128), torch.arange(64), indexing="ij"), -1)
    g = g.reshape(-1, 3).to(torch.int32)
    coords = torch.cat([torch.zeros((g.shape[0], 1), dtype=torch.int32), g], 1).contiguous().cuda()
    assert coords.shape[0] == MAX_PARENTS
    sub = torch.from_numpy(t2sc.synth.bernoulli(33, (MAX_PARENTS, 8))).cuda()
    feats = torch.randn((MAX_PARENTS, 8), device="cuda").to(torch.bfloat16)
    args = (ctx, coords, sub, feats, 8, _lib.FEATS_UPSAMPLE, _lib.DT_BF16, _lib.SUB_NONZERO)
    ref = _run(t2sc, L.t2sc_subdivide_device, *args)
    got = _run(t2sc, L.t2sc_subdivide_noalloc_device, *args)
    assert got[0] == ref[0] > 3 * MAX_PARENTS
    for a, b in zip(got[1:], ref[1:]):
        assert torch.equal(a, b)
