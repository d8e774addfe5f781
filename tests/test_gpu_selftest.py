"""Failure detection without a GPU fault: a device wait on a barrier that
nothing completes gives up after its short bound and reports a timeout
status; the context then still runs convs correctly."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives(t2sc, oracle):
    from _cases import F16_TOL, conv_inputs, oracle_conv, rel_err
    ctx = t2sc.Context.default(0)
    for wait_us in (50, 2000):
        ctx.selftest(wait_us)  # raises unless the wait reported its timeout
    ctx.synchronize()          # the timeout flag was consumed by the self-test, not left behind
    S = t2sc.synth
    coords = S.shell(32, 12.0, 1.0)
    x, w, b = conv_inputs(S, len(coords), 64, 64, seed=3)
    y = t2sc.SparseConv3d(w, b, dtype="bf16", ctx=ctx).forward(t2sc.SparseTensor(x, coords, ctx=ctx)).feats
    assert rel_err(y, oracle_conv(oracle, coords, x, w, b, round_mode="bf16")) <= F16_TOL


def test_selftest_rejects_bad_limit(t2sc):
    ctx = t2sc.Context.default(0)
    with pytest.raises(t2sc.T2SCError):
        ctx.selftest(0)
