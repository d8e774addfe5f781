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


def oracle_chain(O, n, x, layers, csr, round_mode=None, residual_last=None):
    """The reference's conv chain on the oracle with every host thread:
    layers is a list of (w, b, silu); with round_mode the chain input, the
    weights and every intermediate are rounded to the 16-bit type the GPU
    chain keeps between layers. residual_last is added after the last layer
    (the identity residual of a residual block)."""
    import os
    nt = os.cpu_count() or 1
    h = O.round16(x, round_mode) if round_mode else x
    for i, (w, b, silu) in enumerate(layers):
        wr = O.round16(w, round_mode) if round_mode else w
        h = O.conv_rows(h, wr, b, csr, nt)
        if silu:
            h = O.silu(h)
        if i == len(layers) - 1 and residual_last is not None:
            r = O.round16(residual_last, round_mode) if round_mode else residual_last
            h = h + r
        if round_mode and i < len(layers) - 1:
            h = O.round16(h, round_mode)
    return h
