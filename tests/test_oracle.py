"""The CPU restatement (oracle) against everything that pins it: the
reference's published dense-blob edge counts, hand-computed known answers
for the map / CSR / subdivision order, and the committed golden fixtures."""
import numpy as np
import pytest


def blob(side):
    z, y, x = np.meshgrid(np.arange(side), np.arange(side), np.arange(side), indexing="ij")
    out = np.zeros((side ** 3, 4), np.int32)
    out[:, 1], out[:, 2], out[:, 3] = x.ravel() + 4, y.ravel() + 4, z.ravel() + 4
    return out


# docs/benchmarks/RESULTS.md:363-365 of the reference: N -> E for dense blobs
@pytest.mark.parametrize("side,n,e", [(23, 12167, 300763), (38, 54872, 1404928), (60, 216000, 5639752)])
def test_published_edge_counts(oracle, side, n, e):
    c = blob(side)
    assert len(c) == n
    src, tgt, kidx = oracle.neighbor_map(c)
    assert len(src) == e == (3 * side - 2) ** 3


def test_pack_key(oracle):
    L = oracle.lib()
    assert L.orc_pack_key(0, 0, 0, 0) == ((512 * 2048) + 512) * 2048 + 512
    assert L.orc_pack_key(1, 2, 3, 4) == ((1 * 2048 + 2 + 512) * 2048 + 3 + 512) * 2048 + 4 + 512


def test_map_order_known_answer(oracle):
    # two voxels adjacent along column 3 (+z in the kx slot)
    c = np.array([[0, 5, 5, 5], [0, 5, 5, 6]], np.int32)
    src, tgt, kidx = oracle.neighbor_map(c)
    # k = kz*9+ky*3+kx, offsets (kz-1, ky-1, kx-1) on columns 1,2,3
    # row1 sees row0 at offset col3 -1 -> k = 9+3+0 = 12; self at k = 13;
    # row0 sees row1 at offset col3 +1 -> k = 14
    assert list(kidx) == [12, 13, 13, 14]
    assert list(tgt) == [1, 0, 1, 0]
    assert list(src) == [0, 0, 1, 1]
    rs, ss, ks = oracle.csr(2, src, tgt, kidx)
    assert list(rs) == [0, 2, 4]
    assert list(ks) == [13, 14, 12, 13]
    assert list(ss) == [0, 1, 0, 1]


def test_duplicates_last_row_wins(oracle):
    c = np.array([[0, 1, 1, 1], [0, 1, 1, 1]], np.int32)
    src, tgt, kidx = oracle.neighbor_map(c)
    assert list(src) == [1, 1] and list(tgt) == [0, 1] and list(kidx) == [13, 13]


def test_batches_do_not_mix(oracle):
    c = np.array([[0, 1, 1, 1], [1, 1, 1, 2]], np.int32)
    src, tgt, kidx = oracle.neighbor_map(c)
    assert list(kidx) == [13, 13]


def test_dilation(oracle):
    c = np.array([[0, 0, 0, 0], [0, 2, 0, 0], [0, 1, 0, 0]], np.int32)
    src, tgt, kidx = oracle.neighbor_map(c, dilation=2)
    pairs = sorted(zip(src.tolist(), tgt.tolist(), kidx.tolist()))
    # rows 0 and 1 are two apart along column 1 -> offsets kz = 0/2 (k = 4 / 22)
    assert (0, 1, 4) in pairs and (1, 0, 22) in pairs and (2, 2, 13) in pairs
    assert len(pairs) == 5


def test_conv_matches_float64(oracle):
    rng = np.random.default_rng(0)
    c = blob(5)
    n, ci, co = len(c), 24, 40
    x = rng.standard_normal((n, ci)).astype(np.float32)
    w = (rng.standard_normal((co, 3, 3, 3, ci)) * 0.1).astype(np.float32)
    b = rng.standard_normal(co).astype(np.float32)
    e = oracle.neighbor_map(c)
    y = oracle.conv(x, w, b, e)
    src, tgt, kidx = e
    ref = np.zeros((n, co))
    wk = w.reshape(co, 27, ci).astype(np.float64)
    for s, t, k in zip(src, tgt, kidx):
        ref[t] += wk[:, k, :] @ x[s].astype(np.float64)
    ref += b
    assert np.max(np.abs(y - ref)) / np.max(np.abs(ref)) < 1e-6


def test_conv_row_parallel_is_bit_identical(oracle):
    rng = np.random.default_rng(1)
    c = blob(6)
    x = rng.standard_normal((len(c), 20)).astype(np.float32)
    w = rng.standard_normal((16, 3, 3, 3, 20)).astype(np.float32)
    b = rng.standard_normal(16).astype(np.float32)
    e = oracle.neighbor_map(c)
    y1 = oracle.conv(x, w, b, e, nthreads=1)
    y2 = oracle.conv(x, w, b, e, nthreads=0)
    y3 = oracle.conv_rows(x, w, b, oracle.csr(len(c), *e), nthreads=4)
    assert np.array_equal(y1, y2) and np.array_equal(y1, y3)


def test_subdivision_known_answer(oracle):
    c = np.array([[0, 1, 2, 3], [0, 4, 4, 4]], np.int32)
    sub = np.zeros((2, 8), np.float32)
    sub[0, [0, 5, 7]] = 1.0
    sub[1, 3] = -0.5  # nonzero -> kept by forward_subdivision, dropped by binarize
    idx, sidx, nc = oracle.subdivide(c, sub)
    assert list(idx) == [0, 0, 0, 1] and list(sidx) == [0, 5, 7, 3]
    assert nc.tolist() == [[0, 2, 4, 6], [0, 3, 4, 7], [0, 3, 5, 7], [0, 9, 9, 8]]
    idx, sidx, nc = oracle.subdivide(c, sub, positive=True)
    assert list(idx) == [0, 0, 0]
    x = np.arange(2 * 16, dtype=np.float32).reshape(2, 16)
    out = oracle.c2s_unfold(x, [0, 1], [5, 3])
    assert out.tolist() == [x[0, 10:12].tolist(), x[1, 6:8].tolist()]
    assert oracle.select_rows(x, [1, 0]).tolist() == [x[1].tolist(), x[0].tolist()]


def test_silu_formula(oracle):
    v = np.linspace(-20, 20, 101).astype(np.float32)
    ref = v.astype(np.float64) / (1 + np.exp(-v.astype(np.float64)))
    assert np.allclose(oracle.silu(v), ref, rtol=1e-6, atol=1e-7)


def test_round16(oracle):
    import torch
    v = np.random.default_rng(2).standard_normal(10000).astype(np.float32) * 100
    v[:4] = [65519.0, 65520.0, 1e-8, -3e-5]
    for mode, dt in (("bf16", torch.bfloat16), ("f16", torch.float16)):
        ref = torch.from_numpy(v).to(dt).float().numpy()
        assert np.array_equal(oracle.round16(v, mode), ref), mode


def test_golden_fixtures(oracle):
    import os
    d = os.path.join(os.path.dirname(__file__), "golden")
    g = np.load(os.path.join(d, "small_cases.npz"))
    for case in ("shell16", "blob4d2"):
        c = g[case + "_coords"]
        dil = int(g[case + "_dil"])
        src, tgt, kidx = oracle.neighbor_map(c, dilation=dil)
        assert np.array_equal(src, g[case + "_src"]) and np.array_equal(tgt, g[case + "_tgt"])
        assert np.array_equal(kidx, g[case + "_kidx"])
        y = oracle.conv(g[case + "_x"], g[case + "_w"], g[case + "_b"], (src, tgt, kidx))
        assert np.array_equal(y, g[case + "_y"])
    idx, sidx, nc = oracle.subdivide(g["sub_coords"], g["sub_mask"])
    assert np.array_equal(nc, g["sub_out_coords"]) and np.array_equal(idx, g["sub_idx"])


@pytest.mark.parametrize("c,affine,silu,eps", [(64, True, True, 1e-6), (13, False, False, 1e-5), (1024, True, False, 1e-6)])
def test_layernorm_oracle(oracle, c, affine, silu, eps):
    """orc_layernorm (nn.mojo:313-370) against the float64 definition."""
    rng = np.random.default_rng(c)
    x = (rng.standard_normal((97, c)) * 3 + 1.5).astype(np.float32)
    w = rng.standard_normal(c).astype(np.float32) if affine else None
    b = rng.standard_normal(c).astype(np.float32) if affine else None
    got = oracle.layernorm(x, w, b, eps, silu)
    xd = x.astype(np.float64)
    m = xd.mean(1, keepdims=True)
    v = ((xd - m) ** 2).mean(1, keepdims=True)
    ref = (xd - m) / np.sqrt(v + eps)
    if affine:
        ref = ref * w + b
    if silu:
        ref = ref / (1 + np.exp(-ref))
    assert np.max(np.abs(got - ref)) < 2e-5 * max(1.0, np.abs(ref).max())


def test_layernorm_known_answer(oracle):
    # constant row -> 0 (variance 0, eps keeps it finite); [1, 3] -> [-1, 1] * 1/sqrt(1 + eps)
    x = np.array([[2, 2, 2, 2], [1, 3, 1, 3]], np.float32)
    got = oracle.layernorm(x, eps=1e-6)
    assert np.all(got[0] == 0)
    assert np.allclose(got[1], np.array([-1, 1, -1, 1]) / np.sqrt(1 + 1e-6), atol=1e-7)


def test_linear_oracle(oracle):
    """orc_linear (nn.mojo:27-266) against the float64 definition, with SiLU and residual."""
    rng = np.random.default_rng(5)
    x = rng.standard_normal((131, 24)).astype(np.float32)
    w = rng.standard_normal((40, 24)).astype(np.float32)
    b = rng.standard_normal(40).astype(np.float32)
    res = rng.standard_normal((131, 40)).astype(np.float32)
    z = x.astype(np.float64) @ w.T.astype(np.float64) + b
    ref = z / (1 + np.exp(-z)) + res
    got = oracle.linear(x, w, b, silu=True, residual=res)
    assert np.max(np.abs(got - ref)) < 1e-4
    assert np.max(np.abs(oracle.linear(x, w) - x.astype(np.float64) @ w.T.astype(np.float64))) < 1e-4


def test_oracle_inputs_match_the_library_generator(oracle, t2sc):
    """The oracle's own seeded-input generator (used by the CPU reference
    arm) and the library's give the same shells, normals and masks."""
    for name in ("cfg1", "cfg2", "cfg3_parent"):
        for seed in (0, 3):
            a = oracle.synth_shell(*oracle.SHELLS[name], seed=seed)
            b = t2sc.synth.shell(*t2sc.synth.SHELLS[name], seed=seed)
            assert np.array_equal(a, b), (name, seed)
    assert np.array_equal(oracle.synth_normal(401, (27, 64), 0.1), t2sc.synth.normal(401, (27, 64), std=0.1))
    assert np.array_equal(oracle.synth_bernoulli(500, (1000, 8)), t2sc.synth.bernoulli(500, (1000, 8)))


def test_pipeline_glue_hand_cases(oracle):
    """The oracle's pipeline glue against cases worked by hand from
    fdg_vae.mojo:17-50, vertex_attrs.mojo:46-104 and image_to_3d.mojo:219-270."""
    f = np.zeros((3, 7), np.float32)
    f[:, 6] = [20.5, 0.0, -3.0]
    f[:, 3] = [1.0, 0.0, -1.0]
    v, i, q = oracle.fdg_head(f, 0.5)
    assert np.all(v == 0.5)  # (1 + 2m) * sigmoid(0) - m
    assert i[:, 0].tolist() == [1.0, 0.0, 0.0]
    np.testing.assert_allclose(q.ravel(), [20.5, np.log(2.0), np.log1p(np.exp(-3.0))], rtol=1e-6)

    xyz = np.array([[1, 1, 1], [1, 2, 1], [2, 1, 1], [1, 1, 1]], np.int32)
    feats = np.array([[0, 1], [2, 3], [4, 5], [6, 7]], np.float32)  # (1,1,1) resolves to its last row
    q = np.array([[1.5, 1.5, 1.5], [1.5, 2.0, 1.5], [0.2, 0.2, 0.2], [9, 9, 9], [-0.9, 1.5, 1.5]], np.float32)
    out = oracle.grid_sample_trilinear(feats, xyz, 4, q)
    assert out[0].tolist() == [6.0, 7.0]
    assert out[1].tolist() == [4.0, 5.0]  # half way between (1,1,1) and (1,2,1)
    assert out[2].tolist() == [0.0, 0.0] and out[3].tolist() == [0.0, 0.0]
    # x = -0.9: -1.4 truncates to -1 (a miss), -0.4 to 0 (absent): nothing found
    assert out[4].tolist() == [0.0, 0.0]

    hr = np.array([[0, 5, 5, 5], [0, 5, 5, 4], [0, 0, 0, 0], [1, 0, 0, 0], [0, 5, 5, 5]], np.int32)
    c, res = oracle.cascade_coords(hr, 8, 1024, 100)  # k = 64: q = int((v + 0.5) * 8)
    assert res == 1024
    assert c.tolist() == [[0, 4, 4, 4], [0, 44, 44, 36], [0, 44, 44, 44], [1, 4, 4, 4]]
    c, res = oracle.cascade_coords(hr, 8, 1536, 4)  # 4 tokens at every resolution: walks down to 1024
    assert res == 1024
    c, res = oracle.cascade_coords(hr, 8, 1536, 5)  # fits at once
    assert res == 1536 and len(c) == 4
