"""The whole SLat decoder on the device (SparseUnetVaeDecoder,
sparse_unet_vae.mojo:140-284) against the oracle's composition of the
restated blocks (oracle.decoder), f32, three stages (64 -> 32 -> 16
channels, one ConvNeXt block each, two C2S up blocks) from a 64^3 latent
shell. The shape decoder's predicted subdivisions are compared within the
f32 bar and then drive the oracle (so both sides unfold the same
children); the texture decoder runs guided by them. Coordinates bit-exact,
features max-rel-err <= 1e-4."""
import numpy as np
import pytest

from _cases import F32_TOL, rel_err

pytestmark = pytest.mark.gpu

CH, NB = [64, 32, 16], [1, 1, 1]


def _state_dict(S, latent, out, seed):
    sd, k = {}, [seed]

    def nrm(shape, std):
        k[0] += 1
        return S.normal(k[0], shape, std=std)

    sd["from_latent.weight"], sd["from_latent.bias"] = nrm((CH[0], latent), latent ** -0.5), nrm((CH[0],), 0.1)
    for s, c in enumerate(CH):
        for j in range(NB[s]):
            p = f"blocks.{s}.{j}"
            sd[p + ".conv.weight"], sd[p + ".conv.bias"] = nrm((c, 3, 3, 3, c), (27 * c) ** -0.5), nrm((c,), 0.1)
            sd[p + ".norm.weight"], sd[p + ".norm.bias"] = 1 + nrm((c,), 0.1), nrm((c,), 0.1)
            sd[p + ".mlp.0.weight"], sd[p + ".mlp.0.bias"] = nrm((4 * c, c), c ** -0.5), nrm((4 * c,), 0.1)
            sd[p + ".mlp.2.weight"], sd[p + ".mlp.2.bias"] = nrm((c, 4 * c), (4 * c) ** -0.5), nrm((c,), 0.1)
        if s < len(CH) - 1:
            p, co = f"blocks.{s}.{NB[s]}", CH[s + 1]
            sd[p + ".norm1.weight"], sd[p + ".norm1.bias"] = 1 + nrm((c,), 0.1), nrm((c,), 0.1)
            sd[p + ".conv1.weight"], sd[p + ".conv1.bias"] = nrm((8 * co, 3, 3, 3, c), (27 * c) ** -0.5), nrm((8 * co,), 0.1)
            sd[p + ".conv2.weight"], sd[p + ".conv2.bias"] = nrm((co, 3, 3, 3, co), (27 * co) ** -0.5), nrm((co,), 0.1)
            sd[p + ".to_subdiv.weight"], sd[p + ".to_subdiv.bias"] = nrm((8, c), c ** -0.5), nrm((8,), 0.1)
    sd["output_layer.weight"], sd["output_layer.bias"] = nrm((out, CH[-1]), CH[-1] ** -0.5), nrm((out,), 0.1)
    return sd


def test_shape_then_texture_decoder_f32(t2sc, oracle):
    S = t2sc.synth
    coords = S.shell(32, 10.0, 1.0)
    x = S.normal(950, (len(coords), 8))
    sd_shape = _state_dict(S, 8, 7, 1000)
    dec = t2sc.SparseUnetVaeDecoder(sd_shape, CH, NB, pred_subdiv=True)
    y, subs = dec.forward(t2sc.SparseTensor(x, coords))
    gsubs = [s.feats for s in subs]
    oc, oy, osubs = oracle.decoder(sd_shape, CH, NB, coords, x, guide_subs=gsubs, pred_subdiv=True)
    for a, b in zip(gsubs, osubs):
        assert rel_err(a, b) <= F32_TOL
    assert np.array_equal(y.coords, oc)
    assert rel_err(y.feats, oy) <= F32_TOL
    assert len(y.coords) > 4 * len(coords)
    # the coordinates after one up block
    c1 = dec.upsample_coords(t2sc.SparseTensor(x, coords), 1)
    assert np.array_equal(c1, subs[1].coords)
    # texture decoder guided by the shape decoder's subdivisions
    sd_tex = _state_dict(S, 8, 6, 2000)
    tex = t2sc.SparseUnetVaeDecoder(sd_tex, CH, NB, pred_subdiv=False)
    yt = tex.forward_guided(t2sc.SparseTensor(x, coords), subs)
    tc, ty, _ = oracle.decoder(sd_tex, CH, NB, coords, x, guide_subs=gsubs, pred_subdiv=False)
    assert np.array_equal(yt.coords, tc) and rel_err(yt.feats, ty) <= F32_TOL


def test_decode_shape_and_tex(t2sc, oracle):
    """decode_shape = forward + fdg_head (pipelines/image_to_3d.mojo:206-216),
    decode_tex = forward_guided * 0.5 + 0.5 (:288-297), against the oracle's
    decoder followed by its fdg_head."""
    S = t2sc.synth
    coords = S.shell(32, 10.0, 1.0)
    x = S.normal(951, (len(coords), 8))
    sd_shape = _state_dict(S, 8, 7, 1100)
    dec = t2sc.SparseUnetVaeDecoder(sd_shape, CH, NB, pred_subdiv=True)
    v, i, q, subs = t2sc.decode_shape(dec, t2sc.SparseTensor(x, coords), 0.5)
    gsubs = [s.feats for s in subs]
    oc, oy, _ = oracle.decoder(sd_shape, CH, NB, coords, x, guide_subs=gsubs, pred_subdiv=True)
    ov, oi, oq = oracle.fdg_head(oy, 0.5)
    assert np.array_equal(v.coords, oc)
    # the heads are smooth in the decoder output except the > 0 threshold:
    # compare intersected where the decoder outputs are not within the f32 bar of 0
    assert rel_err(v.feats, ov) <= F32_TOL and rel_err(q.feats, oq) <= F32_TOL
    clear = np.abs(oy[:, 3:6]) > 1e-3 * np.abs(oy).max()
    assert np.array_equal(i.feats[clear], oi[clear])
    sd_tex = _state_dict(S, 8, 6, 2100)
    tex = t2sc.SparseUnetVaeDecoder(sd_tex, CH, NB, pred_subdiv=False)
    yt = t2sc.decode_tex(tex, t2sc.SparseTensor(x, coords), subs)
    _, ty, _ = oracle.decoder(sd_tex, CH, NB, coords, x, guide_subs=gsubs, pred_subdiv=False)
    assert rel_err(yt.feats, ty * np.float32(0.5) + np.float32(0.5)) <= F32_TOL
