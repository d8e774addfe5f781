"""ctypes wrapper of the CPU restatement (liboracle, t2sc_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg as the checker and the timed CPU reference.
Parity status: follows the reference source (file:line in t2sc_oracle.c);
values are unpinned beyond code-following, edge counts are pinned to the
reference's published dense-blob table.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_build", "libt2sc_oracle.so")


def build():
    src = [os.path.join(HERE, f) for f in ("t2sc_oracle.c", "t2sc_oracle.h", "Makefile")]
    if not os.path.exists(LIB) or any(os.path.getmtime(s) > os.path.getmtime(LIB) for s in src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = ctypes.CDLL(LIB)
        P, I, I64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
        L.orc_pack_key.restype = I64
        L.orc_pack_key.argtypes = [I64, I64, I64, I64]
        L.orc_neighbor_map.restype = I64
        L.orc_neighbor_map.argtypes = [P, I64, I, I, I, I, P, P, P, I64]
        L.orc_csr.restype = None
        L.orc_csr.argtypes = [I64, I64, P, P, P, P, P, P]
        L.orc_conv_forward.restype = None
        L.orc_conv_forward.argtypes = [P, I64, I, P, P, I, I, P, P, P, I64, P, I]
        L.orc_conv_forward_rows.restype = None
        L.orc_conv_forward_rows.argtypes = [P, I64, I, P, P, I, I, P, P, P, P, I]
        L.orc_silu.restype = None
        L.orc_silu.argtypes = [P, I64]
        L.orc_add.restype = None
        L.orc_add.argtypes = [P, P, I64]
        L.orc_round16.restype = None
        L.orc_round16.argtypes = [P, I64, I]
        L.orc_linear.restype = None
        L.orc_linear.argtypes = [P, I64, I, P, P, I, I, P, P]
        L.orc_layernorm.restype = None
        L.orc_layernorm.argtypes = [P, I64, I, P, P, ctypes.c_float, I, P]
        L.orc_subdivide.restype = I64
        L.orc_subdivide.argtypes = [P, I64, P, I, P, P, P]
        L.orc_select_rows.restype = None
        L.orc_select_rows.argtypes = [P, I, P, I64, P]
        L.orc_c2s_unfold.restype = None
        L.orc_c2s_unfold.argtypes = [P, I, P, P, I64, P]
        L.orc_synth_shell.restype = I64
        L.orc_synth_shell.argtypes = [I, ctypes.c_double, ctypes.c_double, ctypes.c_uint64, I, P, I64]
        L.orc_synth_normal.restype = None
        L.orc_synth_normal.argtypes = [ctypes.c_uint64, ctypes.c_float, P, I64]
        L.orc_synth_bernoulli.restype = None
        L.orc_synth_bernoulli.argtypes = [ctypes.c_uint64, ctypes.c_double, P, I64]
        L.orc_fdg_head.restype = None
        L.orc_fdg_head.argtypes = [P, I64, ctypes.c_double, P, P, P]
        L.orc_grid_sample_trilinear.restype = I
        L.orc_grid_sample_trilinear.argtypes = [P, I64, I, P, I, P, I64, P]
        L.orc_cascade_coords.restype = I64
        L.orc_cascade_coords.argtypes = [P, I64, I, I, I64, P, ctypes.POINTER(ctypes.c_int)]
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def neighbor_map(coords, kernel=(3, 3, 3), dilation=1):
    coords = np.ascontiguousarray(coords, np.int32)
    n = coords.shape[0]
    e = lib().orc_neighbor_map(_p(coords), n, *kernel, dilation, None, None, None, 0)
    src, tgt, kidx = (np.empty(e, np.int64) for _ in range(3))
    lib().orc_neighbor_map(_p(coords), n, *kernel, dilation, _p(src), _p(tgt), _p(kidx), e)
    return src, tgt, kidx


def csr(n, src, tgt, kidx):
    e = len(src)
    rs = np.empty(n + 1, np.int64)
    ss, ks = np.empty(e, np.int64), np.empty(e, np.int64)
    lib().orc_csr(n, e, _p(src), _p(tgt), _p(kidx), _p(rs), _p(ss), _p(ks))
    return rs, ss, ks


def conv(x, weight, bias, edges, nthreads=0):
    """SparseConv3d.forward's CPU loop; weight [Co,Kd,Kh,Kw,Ci]."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(weight, np.float32)
    co, ci = w.shape[0], w.shape[4]
    ks = w.shape[1] * w.shape[2] * w.shape[3]
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    src, tgt, kidx = edges
    out = np.empty((x.shape[0], co), np.float32)
    lib().orc_conv_forward(_p(x), x.shape[0], ci, _p(w), _p(b), co, ks, _p(src), _p(tgt), _p(kidx), len(src),
                           _p(out), nthreads)
    return out


def conv_rows(x, weight, bias, csr_arrays, nthreads):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(weight, np.float32)
    co, ci = w.shape[0], w.shape[4]
    ks = w.shape[1] * w.shape[2] * w.shape[3]
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    rs, ss, kk = csr_arrays
    out = np.empty((x.shape[0], co), np.float32)
    lib().orc_conv_forward_rows(_p(x), x.shape[0], ci, _p(w), _p(b), co, ks, _p(rs), _p(ss), _p(kk), _p(out),
                                nthreads)
    return out


def silu(v):
    v = np.ascontiguousarray(v, np.float32).copy()
    lib().orc_silu(_p(v), v.size)
    return v


def round16(v, mode):
    """mode 'bf16' or 'f16': round to nearest even."""
    v = np.ascontiguousarray(v, np.float32).copy()
    lib().orc_round16(_p(v), v.size, 2 if mode == "bf16" else 1)
    return v


def subdivide(coords, sub, positive=False):
    coords = np.ascontiguousarray(coords, np.int32)
    sub = np.ascontiguousarray(sub, np.float32)
    n = coords.shape[0]
    idx, sidx = np.empty(8 * n, np.int64), np.empty(8 * n, np.int64)
    nc = np.empty((8 * n, 4), np.int32)
    m = lib().orc_subdivide(_p(coords), n, _p(sub), int(positive), _p(idx), _p(sidx), _p(nc))
    return idx[:m].copy(), sidx[:m].copy(), nc[:m].copy()


def select_rows(x, idx):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty((len(idx), x.shape[1]), np.float32)
    lib().orc_select_rows(_p(x), x.shape[1], _p(np.ascontiguousarray(idx, np.int64)), len(idx), _p(out))
    return out


def c2s_unfold(x, idx, subidx):
    x = np.ascontiguousarray(x, np.float32)
    cout = x.shape[1] // 8
    out = np.empty((len(idx), cout), np.float32)
    lib().orc_c2s_unfold(_p(x), cout, _p(np.ascontiguousarray(idx, np.int64)),
                         _p(np.ascontiguousarray(subidx, np.int64)), len(idx), _p(out))
    return out


def layernorm(x, w=None, b=None, eps=1e-6, silu=False):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    w = None if w is None else np.ascontiguousarray(w, np.float32)
    b = None if b is None else np.ascontiguousarray(b, np.float32)
    lib().orc_layernorm(_p(x), x.shape[0], x.shape[1], _p(w), _p(b), eps, int(silu), _p(out))
    return out


def linear(x, w, b=None, silu=False, residual=None):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    co, ci = w.shape
    out = np.empty((x.shape[0], co), np.float32)
    b = None if b is None else np.ascontiguousarray(b, np.float32)
    res = None if residual is None else np.ascontiguousarray(residual, np.float32)
    lib().orc_linear(_p(x), x.shape[0], ci, _p(w), _p(b), co, int(silu), _p(res), _p(out))
    return out


# Seeded inputs of the benchmark configurations, generated here so that the
# CPU reference never loads the product library. name -> (grid, radius, h).
SHELLS = {
    "cfg1": (64, 24.0, 1.0),
    "cfg2": (128, 48.0, 1.75),
    "cfg3_parent": (128, 48.0, 0.9),
    "cfg4": (512, 200.0, 0.5),
    "cfg5_parent": (512, 200.0, 0.5),
}


def synth_shell(g, radius, h, seed=0, batch=0):
    n = lib().orc_synth_shell(g, radius, h, seed, batch, None, 0)
    out = np.empty((n, 4), np.int32)
    lib().orc_synth_shell(g, radius, h, seed, batch, _p(out), n)
    return out


def synth_normal(seed, shape, std=1.0):
    out = np.empty(shape, np.float32)
    lib().orc_synth_normal(seed, std, _p(out), out.size)
    return out


def synth_bernoulli(seed, shape, p=0.5):
    out = np.empty(shape, np.float32)
    lib().orc_synth_bernoulli(seed, p, _p(out), out.size)
    return out


def c2s_block(coords, x, norm1, conv1, conv2, out_channels, to_subdiv=None, subdiv=None):
    """SparseResBlockC2S3d._core / forward (trellis2_mojo/models/sc_vaes/
    sparse_unet_vae.mojo:103-133) composed from the restated pieces:
    subdiv = to_subdiv(x) (pred path, :126); h = conv1(SiLU(LN1(x))) (:118-119);
    mask = subdiv > 0 (_binarize, :30-37); h = C2S(h, mask), x2 = C2S(x, mask)
    (:120-122); h = conv2(SiLU(LN2(h))) (:123-124, LN2 without affine);
    return h + repeat_interleave(x2) (_skip, :103-115). Returns (coords, h, subdiv)."""
    x = np.ascontiguousarray(x, np.float32)
    if subdiv is None:
        subdiv = linear(x, *to_subdiv)
    h = layernorm(x, norm1[0], norm1[1], eps=1e-6, silu=True)
    h = conv(h, conv1[0], conv1[1], neighbor_map(coords))
    idx, sidx, nc = subdivide(coords, subdiv, positive=True)
    h = c2s_unfold(h, idx, sidx)
    x2 = c2s_unfold(x, idx, sidx)
    h = layernorm(h, None, None, eps=1e-6, silu=True)
    h = conv(h, conv2[0], conv2[1], neighbor_map(nc))
    k = out_channels // x2.shape[1]
    skip = np.repeat(x2, k, axis=1)  # out[r, c*k + j] = x2[r, c]
    return nc, h + skip, subdiv


def convnext_block(coords, x, conv_wb, norm_wb, lin1_wb, lin2_wb, edges=None):
    """SparseConvNeXtBlock3d.forward (sparse_unet_vae.mojo:60-64): conv ->
    LayerNorm(affine, eps 1e-6) -> lin2(SiLU(lin1(h))) -> + x."""
    h = conv(x, conv_wb[0], conv_wb[1], edges if edges is not None else neighbor_map(coords))
    h = layernorm(h, norm_wb[0], norm_wb[1], eps=1e-6)
    h = linear(h, lin1_wb[0], lin1_wb[1], silu=True)
    return linear(h, lin2_wb[0], lin2_wb[1], residual=x)


def decoder(sd, model_channels, num_blocks, coords, x, guide_subs=None, pred_subdiv=True):
    """SparseUnetVaeDecoder.forward / forward_guided (sparse_unet_vae.mojo:
    172-206, weights named as sparse_unet_vae_decoder_from, :255-284):
    from_latent -> per stage its ConvNeXt blocks, then (except the last
    stage) the C2S up block -> LayerNorm (eps 1e-5, no affine) ->
    output_layer. With guide_subs the up blocks use them (forward_guided);
    with pred_subdiv the predicted subdivisions are returned as well.
    Returns (coords, feats, subs)."""
    g = lambda n: (sd[n + ".weight"], sd.get(n + ".bias"))  # noqa: E731
    h = linear(x, *g("from_latent"))
    subs = []
    for s in range(len(num_blocks)):
        edges = neighbor_map(coords)
        for j in range(num_blocks[s]):
            p = f"blocks.{s}.{j}"
            h = convnext_block(coords, h, g(p + ".conv"), g(p + ".norm"), g(p + ".mlp.0"), g(p + ".mlp.2"), edges)
        if s < len(num_blocks) - 1:
            p = f"blocks.{s}.{num_blocks[s]}"
            given = None if guide_subs is None else guide_subs[s]
            pred = linear(h, *g(p + ".to_subdiv")) if pred_subdiv else None   # forward, :126-130
            use = given if given is not None else pred
            coords, h, _ = c2s_block(coords, h, g(p + ".norm1"), g(p + ".conv1"), g(p + ".conv2"),
                                     model_channels[s + 1], subdiv=use)
            subs.append(pred if pred_subdiv else use)
    h = layernorm(h, None, None, eps=1e-5)
    return coords, linear(h, *g("output_layer")), subs


def fdg_head(feats, voxel_margin=0.5):
    """(vertices [T,3], intersected [T,3], quad_lerp [T,1]) of decoded [T,7]
    features (models/sc_vaes/fdg_vae.mojo:17-50)."""
    f = np.ascontiguousarray(feats, np.float32)
    t = f.shape[0]
    v, i, q = np.empty((t, 3), np.float32), np.empty((t, 3), np.float32), np.empty((t, 1), np.float32)
    lib().orc_fdg_head(_p(f), t, voxel_margin, _p(v), _p(i), _p(q))
    return v, i, q


def grid_sample_trilinear(feats, coords_xyz, grid_size, query):
    """[L, C] trilinear samples (meshing/vertex_attrs.mojo:46-104)."""
    f = np.ascontiguousarray(feats, np.float32)
    xyz = np.ascontiguousarray(coords_xyz, np.int32)
    qy = np.ascontiguousarray(query, np.float32)
    out = np.empty((qy.shape[0], f.shape[1]), np.float32)
    rc = lib().orc_grid_sample_trilinear(_p(f), f.shape[0], f.shape[1], _p(xyz), grid_size, _p(qy), qy.shape[0],
                                         _p(out))
    assert rc == 0
    return out


def cascade_coords(hr_coords, lr_resolution, resolution, max_num_tokens):
    """(coords [T,4] int32, hr_resolution) (pipelines/image_to_3d.mojo:219-270)."""
    hr = np.ascontiguousarray(hr_coords, np.int32)
    out = np.empty((max(hr.shape[0], 1), 4), np.int32)
    res = ctypes.c_int()
    t = lib().orc_cascade_coords(_p(hr), hr.shape[0], lr_resolution, resolution, max_num_tokens, _p(out),
                                 ctypes.byref(res))
    if t < 0:
        raise ValueError("cascade_coords: token budget never met" if t == -2 else "allocation failed")
    return out[:t].copy(), res.value
