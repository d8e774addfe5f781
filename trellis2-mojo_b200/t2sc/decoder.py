"""The SLat decoder on the device: SparseUnetVaeDecoder
(trellis2_mojo/models/sc_vaes/sparse_unet_vae.mojo:140-284) over libt2sc's
block entry points. Features stay on the GPU from the latent to the output
layer; each stage's coordinates are a device handle whose neighbour map is
built once and shared by every conv of the stage; the up blocks return the
children's handle with its map already built.

  forward(x)                 pred_subdiv decoder -> (decoded, subs)       :172-190
  forward_guided(x, subs)    texture decoder guided by the shape subs     :192-206
  upsample_coords(x, times)  coordinates after `times` up blocks          :208-224

Weights come from a state dict with the checkpoint's names
(sparse_unet_vae_decoder_from, :255-284): from_latent, blocks.{s}.{j}.conv /
.norm / .mlp.0 / .mlp.2, blocks.{s}.{num_blocks[s]}.norm1 / .conv1 / .conv2 /
.to_subdiv, output_layer; conv weights [Co, Kd, Kh, Kw, Ci] (conv_none).
"""
import ctypes

import numpy as np

from . import _lib
from ._lib import check, lib
from .sparse import _DTYPES, Context, Coords, SparseLinear, SparseTensor


def _f(a):
    return None if a is None else np.ascontiguousarray(a, np.float32)


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def _dp(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _on_torch_stream(ctx, device):
    """Runs the context's work on torch's current stream of `device`, so the
    library's kernels are ordered with the torch tensors they read and write
    without any host synchronisation."""
    import torch
    handle = torch.cuda.current_stream(device).cuda_stream
    # torch's default stream has handle 0, which the C ABI reads as "the
    # context's own stream": name the legacy default stream (cudaStreamLegacy)
    ctx.set_stream(handle if handle else 1)


class SparseConvNeXtBlock3d:
    """conv3 -> LayerNorm(affine, 1e-6) -> Linear/SiLU/Linear -> + x
    (sparse_unet_vae.mojo:40-64), one t2sc_convnext_block_forward_device call."""

    def __init__(self, channels, conv, norm, lin1, lin2, dtype="f32", ctx=None):
        self.ctx = ctx or Context.default()
        self.channels, self.hidden = channels, int(np.shape(lin1[0])[0])
        self._keep = [_f(conv[0]), _f(conv[1]), _f(norm[0]), _f(norm[1]), _f(lin1[0]), _f(lin1[1]), _f(lin2[0]),
                      _f(lin2[1])]
        h = ctypes.c_void_p()
        check(lib.t2sc_convnext_block_create(self.ctx.handle, channels, self.hidden, *[_p(a) for a in self._keep],
                                             _DTYPES[dtype], ctypes.byref(h)), self.ctx.handle)
        self.handle = h

    def forward_device(self, coords, x):
        import torch
        _on_torch_stream(self.ctx, x.device)
        y = torch.empty_like(x)
        check(lib.t2sc_convnext_block_forward_device(self.handle, coords.handle, _dp(x), _dp(y)), self.ctx.handle)
        return y

    def __del__(self):
        h = getattr(self, "handle", None)
        if h and self.ctx.handle:
            lib.t2sc_convnext_block_destroy(h)
            self.handle = None


class _UpBlock:
    """SparseResBlockC2S3d through t2sc_c2s_block_forward_device with device tensors."""

    def __init__(self, channels, out_channels, pred_subdiv, norm1, conv1, conv2, to_subdiv, dtype, ctx):
        self.ctx, self.out_channels, self.pred_subdiv = ctx, out_channels, pred_subdiv
        self._keep = [_f(norm1[0]), _f(norm1[1]), _f(conv1[0]), _f(conv1[1]), _f(conv2[0]), _f(conv2[1]),
                      _f(to_subdiv[0]) if to_subdiv else None, _f(to_subdiv[1]) if to_subdiv else None]
        h = ctypes.c_void_p()
        check(lib.t2sc_c2s_block_create(ctx.handle, channels, out_channels, int(pred_subdiv),
                                        *[_p(a) for a in self._keep], _DTYPES[dtype], ctypes.byref(h)), ctx.handle)
        self.handle = h

    def forward_device(self, coords, x, subdiv=None):
        """-> (child Coords, child device coords [M, 4], h [M, Cout], subdiv [N, 8] f32)."""
        import torch
        n = coords.n
        dev = x.device
        _on_torch_stream(self.ctx, dev)
        sd = torch.empty((n, 8), dtype=torch.float32, device=dev) if subdiv is None else subdiv.contiguous()
        oc = torch.empty((8 * max(n, 1), 4), dtype=torch.int32, device=dev)
        of = torch.empty((8 * max(n, 1), self.out_channels), dtype=x.dtype, device=dev)
        m = ctypes.c_int64()
        child = ctypes.c_void_p()
        check(lib.t2sc_c2s_block_forward_device(self.handle, coords.handle, _dp(x), _dp(sd), _dp(oc), _dp(of),
                                                ctypes.byref(m), ctypes.byref(child)), self.ctx.handle)
        m = m.value
        return Coords.from_handle(self.ctx, child), oc[:m], of[:m], sd

    def __del__(self):
        h = getattr(self, "handle", None)
        if h and self.ctx.handle:
            lib.t2sc_c2s_block_destroy(h)
            self.handle = None


class SparseUnetVaeDecoder:
    def __init__(self, state_dict, model_channels, num_blocks, pred_subdiv, dtype="f32", ctx=None):
        sd = state_dict
        self.ctx = ctx or Context.default()
        self.dtype, self.pred_subdiv = dtype, bool(pred_subdiv)
        self.model_channels, self.num_blocks = list(model_channels), list(num_blocks)
        g = lambda name: (sd[name + ".weight"], sd.get(name + ".bias"))  # noqa: E731
        self.from_latent = SparseLinear(*g("from_latent"), dtype=dtype, ctx=self.ctx)
        self.stages, self.ups = [], []
        ns = len(num_blocks)
        for s in range(ns):
            c = model_channels[s]
            blocks = []
            for j in range(num_blocks[s]):
                p = f"blocks.{s}.{j}"
                blocks.append(SparseConvNeXtBlock3d(c, g(p + ".conv"), g(p + ".norm"), g(p + ".mlp.0"),
                                                    g(p + ".mlp.2"), dtype=dtype, ctx=self.ctx))
            self.stages.append(blocks)
            if s < ns - 1:
                p = f"blocks.{s}.{num_blocks[s]}"
                self.ups.append(_UpBlock(c, model_channels[s + 1], self.pred_subdiv, g(p + ".norm1"), g(p + ".conv1"),
                                         g(p + ".conv2"), g(p + ".to_subdiv") if self.pred_subdiv else None, dtype,
                                         self.ctx))
        self.output_layer = SparseLinear(*g("output_layer"), dtype=dtype, ctx=self.ctx)

    def _run(self, x, guide_subs=None, stop_at=None):
        import torch
        dev = f"cuda:{self.ctx.device}"
        tdt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[self.dtype]
        coords = x.device_coords
        dcoords = torch.from_numpy(np.ascontiguousarray(x.coords)).to(dev)
        h = self.from_latent.forward_device(torch.from_numpy(x.feats).to(dev, tdt))
        subs = []
        for s, blocks in enumerate(self.stages):
            if stop_at is not None and s == stop_at:
                return dcoords.cpu().numpy(), None
            for blk in blocks:
                h = blk.forward_device(coords, h)
            if s < len(self.stages) - 1:
                g = None if guide_subs is None else torch.from_numpy(np.ascontiguousarray(
                    guide_subs[s].feats if isinstance(guide_subs[s], SparseTensor) else guide_subs[s],
                    np.float32)).to(dev)
                child, dc, h, sd = self.ups[s].forward_device(coords, h, g)
                subs.append(SparseTensor(sd.cpu().numpy(), dcoords.cpu().numpy(), x.batch_size, self.ctx))
                coords, dcoords = child, dc
        if stop_at is not None:
            return dcoords.cpu().numpy(), None
        # final LayerNorm (eps 1e-5, no affine) then the output layer (:167-170)
        c = h.shape[1]
        _on_torch_stream(self.ctx, h.device)
        check(lib.t2sc_layernorm_device(self.ctx.handle, _dp(h), _dp(h), h.shape[0], c, None, None, 1e-5, 0,
                                        _DTYPES[self.dtype]), self.ctx.handle)
        y = self.output_layer.forward_device(h)
        out = SparseTensor(y.float().cpu().numpy(), dcoords.cpu().numpy(), x.batch_size, self.ctx)
        out._cache["coords"] = coords
        return out, subs

    def forward(self, x):
        if not self.pred_subdiv:
            raise ValueError("SparseUnetVaeDecoder: use forward_guided when pred_subdiv=False")
        return self._run(x)

    def forward_guided(self, x, guide_subs):
        if self.pred_subdiv:
            raise ValueError("SparseUnetVaeDecoder: use forward when pred_subdiv=True")
        if len(guide_subs) < len(self.stages) - 1:
            raise ValueError("SparseUnetVaeDecoder: one guide subdivision per up block")
        return self._run(x, guide_subs)[0]

    def upsample_coords(self, x, upsample_times):
        if not self.pred_subdiv:
            raise ValueError("SparseUnetVaeDecoder: upsample_coords needs pred_subdiv=True")
        return self._run(x, stop_at=upsample_times)[0]
