"""GPU SparseLinear (tcgen05 / CUDA-core conv kernels over an identity row
map) against the oracle's linear (trellis2_mojo/modules/nn.mojo:27-266),
with the SiLU / residual epilogue; and the ConvNeXt block of the decoder
(conv -> LayerNorm -> lin1/SiLU -> lin2 + x, models/sc_vaes/
sparse_unet_vae.mojo:38-64) end to end. Tolerances: max-rel 1e-4 for
"f32" (split-TF32), 1e-2 for 16-bit (inputs and weights rounded)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _round(a, mode):
    import torch
    dt = {"bf16": torch.bfloat16, "f16": torch.float16}[mode]
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dt).float().numpy()


@pytest.mark.parametrize("dtype,ci,co,rows", [("f32", 64, 256, 20011), ("bf16", 64, 256, 100003),
                                              ("f16", 256, 64, 4097), ("bf16", 128, 128, 1),
                                              ("f32", 64, 8, 3001), ("bf16", 12, 40, 777)])
def test_linear(t2sc, oracle, dtype, ci, co, rows):
    """Co = 8 (to_subdiv) and Ci = 12 take the CUDA-core kernel; the rest tcgen05."""
    from _cases import F16_TOL, F32_TOL, rel_err
    S = t2sc.synth
    x = S.normal(41, (rows, ci))
    w = S.normal(42, (co, ci)) * (1.0 / np.sqrt(ci))
    b = S.normal(43, (co,))
    res = S.normal(44, (rows, co))
    lin = t2sc.SparseLinear(w, b, dtype=dtype)
    tol = F32_TOL if dtype == "f32" else F16_TOL
    xr, wr = (x, w) if dtype == "f32" else (_round(x, dtype), _round(w, dtype))
    got = lin.forward(x)
    assert rel_err(got, oracle.linear(xr, wr, b)) < tol
    got = lin.forward(x, silu=True, residual=res)
    resr = res if dtype == "f32" else _round(res, dtype)
    assert rel_err(got, oracle.linear(xr, wr, b, silu=True, residual=resr)) < tol


def test_linear_row_count_change_and_errors(t2sc, oracle):
    import torch
    from _cases import F32_TOL, rel_err
    S = t2sc.synth
    w = S.normal(51, (32, 16))
    lin = t2sc.SparseLinear(w, None, dtype="f32")
    for rows in (300, 129, 300, 128):   # the identity map is rebuilt when the count changes
        x = S.normal(rows, (rows, 16))
        assert rel_err(lin.forward(x), oracle.linear(x, w)) < F32_TOL
    xt = torch.zeros((0, 16), device="cuda:0")
    assert lin.forward_device(xt).shape == (0, 32)
    conv = t2sc.SparseConv3d(S.normal(52, (16, 3, 3, 3, 16)), None)
    xt = torch.zeros((4, 16), device="cuda:0")
    yt = torch.empty((4, 16), device="cuda:0")
    with pytest.raises(t2sc.T2SCError):   # a 3x3x3 conv handle is not a linear layer
        t2sc._lib.check(t2sc.lib.t2sc_linear_forward_device(conv.handle, xt.data_ptr(), yt.data_ptr(), 4,
                                                            0, None), conv.ctx.handle)


def test_convnext_block_f32(t2sc, oracle):
    """h = conv(x); h = LN(h); h = lin2(silu(lin1(h))) + x on the cfg1 shell, C = 64, MLP 4x."""
    from _cases import F32_TOL, oracle_conv, rel_err
    S = t2sc.synth
    coords = S.shell(*S.SHELLS["cfg1"])
    n, c = len(coords), 64
    x = S.normal(61, (n, c))
    wc, bc = S.normal(62, (c, 3, 3, 3, c)) * 0.05, S.normal(63, (c,))
    ln = t2sc.LayerNorm32(c, eps=1e-6)
    ln.load(S.normal(64, (c,)), S.normal(65, (c,)))
    w1, b1 = S.normal(66, (4 * c, c)) * 0.125, S.normal(67, (4 * c,))
    w2, b2 = S.normal(68, (c, 4 * c)) * 0.0625, S.normal(69, (c,))
    xs = t2sc.SparseTensor(x, coords)
    h = t2sc.SparseConv3d(wc, bc).forward(xs)
    h = ln.forward(h)
    h = t2sc.SparseLinear(w1, b1).forward(h, silu=True)
    out = t2sc.SparseLinear(w2, b2).forward(h, residual=xs)
    r = oracle_conv(oracle, coords, x, wc, bc)
    r = oracle.layernorm(r, ln.weight, ln.bias, 1e-6)
    r = oracle.linear(r, w1, b1, silu=True)
    r = oracle.linear(r, w2, b2, residual=x)
    assert rel_err(out.feats, r) < F32_TOL
