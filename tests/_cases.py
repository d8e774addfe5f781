"""Shared helpers for the GPU parity tests (inputs and error measures)."""
import numpy as np


def rel_err(got, ref):
    """max |got - ref| / max |ref|: the max-relative-error measure of the
    parity bar (f32 <= 1e-4, f16/bf16 <= 1e-2)."""
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    den = max(np.max(np.abs(ref)), 1e-30) if ref.size else 1.0
    return float(np.max(np.abs(got - ref)) / den) if ref.size else 0.0


F32_TOL = 1e-4
F16_TOL = 1e-2


def conv_inputs(synth, n, ci, co, seed):
    x = synth.normal(seed, (n, ci))
    w = synth.normal(seed + 1, (co, 3, 3, 3, ci), std=(1.0 / (27 * ci)) ** 0.5)
    b = synth.normal(seed + 2, (co,), std=0.1)
    return x, w, b


def oracle_conv(O, coords, x, w, b, dil=1, silu=False, residual=None, round_mode=None, edges=None):
    """The reference's conv (+ optional SiLU / residual) on the oracle; with
    round_mode the inputs and weights are first rounded to bf16/f16 (what
    the 16-bit GPU modes consume)."""
    if round_mode:
        x, w = O.round16(x, round_mode), O.round16(w, round_mode)
        if residual is not None:
            residual = O.round16(residual, round_mode)
    if edges is None:
        edges = O.neighbor_map(coords, kernel=tuple(w.shape[1:4]), dilation=dil)
    y = O.conv(x, w, b, edges)
    if silu:
        y = O.silu(y)
    if residual is not None:
        y = y + residual
    return y
