"""GPU LayerNorm (+ fused SiLU) against the oracle's restatement of
LayerNorm32.forward (trellis2_mojo/modules/nn.mojo:313-370) and the SiLU
activation (nn.mojo:614-621). Tolerances: f32 1e-5 absolute on outputs of
order 1 (reduction order differs: warp tree vs 8-lane tree + tail); 16-bit
1e-2 relative to max |y| (one output rounding)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

F32_ATOL = 1e-5
LOW_TOL = 1e-2


@pytest.mark.parametrize("c,affine,silu,eps", [(64, True, True, 1e-6), (64, False, True, 1e-6),
                                               (128, True, False, 1e-5), (7, True, True, 1e-6),
                                               (1024, False, False, 1e-6), (200, True, True, 1e-6)])
def test_layernorm_f32(t2sc, oracle, c, affine, silu, eps):
    S = t2sc.synth
    x = S.normal(11, (4099, c)) * 2.5 + 0.7
    ln = t2sc.LayerNorm32(c, eps=eps, affine=affine)
    if affine:
        ln.load(S.normal(12, (c,)), S.normal(13, (c,)))
    got = ln.forward(x, silu=silu)
    ref = oracle.layernorm(x, ln.weight, ln.bias, eps, silu)
    assert np.max(np.abs(got - ref)) < F32_ATOL * max(1.0, np.abs(ref).max())


@pytest.mark.parametrize("dtype,c", [("bfloat16", 64), ("float16", 64), ("bfloat16", 12), ("float16", 520)])
def test_layernorm_16bit_inplace(t2sc, oracle, dtype, c):
    """C = 64 / 520: 16-byte vector kernel; C = 12 (24-byte rows): scalar kernel."""
    import torch
    S = t2sc.synth
    x = S.normal(21, (100003, c))
    ln = t2sc.LayerNorm32(c, eps=1e-6, affine=True)
    ln.load(S.normal(22, (c,)), S.normal(23, (c,)))
    xt = torch.from_numpy(x).to("cuda:0", getattr(torch, dtype))
    x_rounded = xt.float().cpu().numpy()
    ln.forward_device(xt, y=xt, silu=True)     # in place
    got = xt.float().cpu().numpy()
    ref = oracle.layernorm(x_rounded, ln.weight, ln.bias, 1e-6, True)
    assert np.max(np.abs(got - ref)) < LOW_TOL * np.abs(ref).max()


def test_layernorm_edges(t2sc, oracle):
    import torch
    ln = t2sc.LayerNorm32(16, eps=1e-6, affine=False)
    # zero rows: no launch, no error
    ln.forward_device(torch.empty((0, 16), device="cuda:0"))
    # constant rows normalise to exactly 0
    got = ln.forward(np.full((5, 16), 3.25, np.float32))
    assert np.all(got == 0)
    # a view 4 bytes off 16-byte alignment takes the scalar kernel
    x = np.random.default_rng(0).standard_normal((301, 17)).astype(np.float32)
    xt = torch.from_numpy(x).to("cuda:0")
    ln16 = t2sc.LayerNorm32(16, eps=1e-6, affine=False)
    view = xt.view(-1)[1:1 + 300 * 16].view(300, 16)
    out = torch.empty(300 * 16 + 1, device="cuda:0")[1:].view(300, 16)
    ln16.forward_device(view, y=out)
    ref = oracle.layernorm(view.cpu().numpy(), eps=1e-6)
    assert np.max(np.abs(out.cpu().numpy() - ref)) < F32_ATOL * max(1.0, np.abs(ref).max())
    with pytest.raises(t2sc.T2SCError):
        t2sc._lib.check(t2sc.lib.t2sc_layernorm_device(ln.ctx.handle, None, None, 1, 2048, None, None,
                                                       1e-6, 0, 0), ln.ctx.handle)


def test_decoder_glue_chain(t2sc, oracle):
    """norm1/SiLU -> SubM conv, the upsample block's first half
    (sparse_unet_vae.mojo:118-119), f32 end to end."""
    from _cases import F32_TOL, oracle_conv, rel_err
    S = t2sc.synth
    coords = S.shell(*S.SHELLS["cfg1"])
    n, c = len(coords), 64
    x = S.normal(31, (n, c))
    ln = t2sc.LayerNorm32(c, eps=1e-6)
    ln.load(S.normal(32, (c,)), S.normal(33, (c,)))
    w = S.normal(34, (c, 3, 3, 3, c)) * 0.05
    b = S.normal(35, (c,))
    h = ln.forward(t2sc.SparseTensor(x, coords), silu=True)
    y = t2sc.SparseConv3d(w, b).forward(h).feats
    h_ref = oracle.layernorm(x, ln.weight, ln.bias, 1e-6, True)
    y_ref = oracle_conv(oracle, coords, h_ref, w, b)
    assert rel_err(y, y_ref) < F32_TOL


def test_layernorm_rejects_bad_y(t2sc):
    import torch
    ln = t2sc.LayerNorm32(16)
    x = torch.zeros((4, 16), device="cuda:0")
    for y in (torch.zeros((3, 16), device="cuda:0"),                      # too small
              torch.zeros((4, 16), device="cuda:0", dtype=torch.bfloat16),  # wrong dtype
              torch.zeros((16, 4), device="cuda:0").t(),                  # not contiguous
              torch.zeros((4, 16))):                                      # host memory
        with pytest.raises(ValueError):
            ln.forward_device(x, y=y)
    with pytest.raises(ValueError):
        ln.forward_device(torch.zeros((4, 16)))


def test_linear_rejects_host_residual(t2sc):
    import torch
    lin = t2sc.SparseLinear(np.zeros((16, 16), np.float32))
    x = torch.zeros((4, 16), device="cuda:0")
    with pytest.raises(ValueError):
        lin.forward_device(x, residual=torch.zeros((4, 16)))
    with pytest.raises(ValueError):
        lin.forward_device(torch.zeros((4, 16)))
