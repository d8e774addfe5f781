"""Pipeline glue around the decoder, on the device:

  fdg_head(h, voxel_margin)                        models/sc_vaes/fdg_vae.mojo:17-50
  decode_shape(decoder, slat, voxel_margin)        pipelines/image_to_3d.mojo:206-216
  decode_tex(decoder, slat, guide_subs)            pipelines/image_to_3d.mojo:288-297
  cascade_coords(hr, lr_res, res, max_tokens)      pipelines/image_to_3d.mojo:219-270
  grid_sample_trilinear(feats, xyz, grid, query)   meshing/vertex_attrs.mojo:46-104

Each has a host form with the reference's arguments and results (numpy /
SparseTensor) and a *_device form over torch CUDA tensors that runs on
torch's current stream.
"""
import ctypes

import numpy as np

from ._lib import check, lib
from .sparse import Context, Coords, SparseTensor, _check_on_ctx_device


def _dp(t):
    return ctypes.c_void_p(t.data_ptr())


def _on_torch_stream(ctx, device):
    import torch
    h = torch.cuda.current_stream(device).cuda_stream
    ctx.set_stream(h if h else 1)  # 0 would mean the context's own stream


def fdg_head_device(feats, voxel_margin=0.5, ctx=None):
    """Device f32 [T, 7] -> (vertices [T, 3], intersected [T, 3], quad_lerp [T, 1])."""
    import torch
    ctx = ctx or Context.default(feats.device.index or 0)
    _check_on_ctx_device(feats, ctx, "fdg_head: feats")
    if feats.dtype != torch.float32 or feats.dim() != 2 or feats.shape[1] != 7:
        raise ValueError("fdg_head: expected f32 [T, 7] features")
    f = feats.contiguous()
    t = f.shape[0]
    v = torch.empty((t, 3), dtype=torch.float32, device=f.device)
    i = torch.empty((t, 3), dtype=torch.float32, device=f.device)
    q = torch.empty((t, 1), dtype=torch.float32, device=f.device)
    _on_torch_stream(ctx, f.device)
    check(lib.t2sc_fdg_head_device(ctx.handle, _dp(f), t, float(voxel_margin), _dp(v), _dp(i), _dp(q)), ctx.handle)
    return v, i, q


def fdg_head(h, voxel_margin=0.5):
    """SparseTensor [T, 7] -> three SparseTensors on the same coordinates."""
    import torch
    if h.feats.shape[1] != 7:
        raise ValueError("fdg_head: expected 7 channels")
    ctx = h.ctx
    f = torch.from_numpy(h.feats).to(f"cuda:{ctx.device}")
    v, i, q = fdg_head_device(f, voxel_margin, ctx)
    return h.replace(v.cpu().numpy()), h.replace(i.cpu().numpy()), h.replace(q.cpu().numpy())


def decode_shape(decoder, slat, voxel_margin=0.5):
    """-> (vertices, intersected, quad_lerp, subs): the shape decoder's
    forward followed by the FlexiDualGrid head."""
    h, subs = decoder.forward(slat)
    v, i, q = fdg_head(h, voxel_margin)
    return v, i, q, subs


def decode_tex(decoder, slat, guide_subs):
    """Guided texture decode, then * 0.5 + 0.5 into colour space."""
    h = decoder.forward_guided(slat, guide_subs)
    return h.replace(h.feats * np.float32(0.5) + np.float32(0.5))


def cascade_coords_device(hr_coords, lr_resolution, resolution, max_num_tokens, ctx=None):
    """Device int32 [n, 4] -> (device int32 [T, 4] tokens, hr_resolution)."""
    import torch
    ctx = ctx or Context.default(hr_coords.device.index or 0)
    _check_on_ctx_device(hr_coords, ctx, "cascade_coords: hr_coords")
    if hr_coords.dtype != torch.int32 or hr_coords.dim() != 2 or hr_coords.shape[1] != 4:
        raise ValueError("cascade_coords: expected int32 [n, 4] coordinates")
    hc = hr_coords.contiguous()
    n = hc.shape[0]
    out = torch.empty((max(n, 1), 4), dtype=torch.int32, device=hc.device)
    t, res = ctypes.c_int64(), ctypes.c_int()
    _on_torch_stream(ctx, hc.device)
    check(lib.t2sc_cascade_coords_device(ctx.handle, _dp(hc), n, int(lr_resolution), int(resolution),
                                         int(max_num_tokens), _dp(out), ctypes.byref(t), ctypes.byref(res)),
          ctx.handle)
    return out[:t.value], res.value


def cascade_coords(hr_coords, lr_resolution, resolution, max_num_tokens, ctx=None):
    """Host int32 [n, 4] -> (int32 [T, 4], hr_resolution), as the reference returns them."""
    import torch
    ctx = ctx or Context.default()
    hc = torch.from_numpy(np.ascontiguousarray(hr_coords, np.int32)).to(f"cuda:{ctx.device}")
    out, res = cascade_coords_device(hc, lr_resolution, resolution, max_num_tokens, ctx)
    return out.cpu().numpy(), res


def grid_sample_trilinear_device(coords, feats, grid_size, query):
    """coords: a Coords handle (batch 0 rows) whose row order feats [n, C]
    (device f32) follows; query device f32 [L, 3] in voxel units -> [L, C]."""
    import torch
    ctx = coords.ctx
    _check_on_ctx_device(feats, ctx, "grid_sample: feats")
    _check_on_ctx_device(query, ctx, "grid_sample: query")
    if feats.dtype != torch.float32 or feats.dim() != 2 or feats.shape[0] != coords.n:
        raise ValueError("grid_sample: feats must be f32 [n, C] in the handle's row order")
    if query.dtype != torch.float32 or query.dim() != 2 or query.shape[1] != 3:
        raise ValueError("grid_sample: query must be f32 [L, 3]")
    f, q = feats.contiguous(), query.contiguous()
    out = torch.empty((q.shape[0], f.shape[1]), dtype=torch.float32, device=f.device)
    _on_torch_stream(ctx, f.device)
    check(lib.t2sc_grid_sample_trilinear_device(coords.handle, _dp(f), f.shape[1], int(grid_size), _dp(q),
                                                q.shape[0], _dp(out)), ctx.handle)
    return out


def grid_sample_trilinear(feats, coords_xyz, grid_size, query, ctx=None):
    """The reference's signature: feats [N, C], voxel coords [N, 3] (batch
    column stripped), query [L, 3] -> [L, C] (numpy)."""
    import torch
    ctx = ctx or Context.default()
    feats = np.ascontiguousarray(feats, np.float32)
    xyz = np.ascontiguousarray(coords_xyz, np.int32)
    if feats.shape[0] != xyz.shape[0]:
        raise ValueError("grid_sample_trilinear: feats/coords row mismatch")
    query = np.ascontiguousarray(query, np.float32)
    if query.ndim != 2 or query.shape[1] != 3:
        raise ValueError("grid_sample_trilinear: query must be [L, 3]")
    c4 = np.concatenate([np.zeros((xyz.shape[0], 1), np.int32), xyz], 1)
    coords = Coords(ctx, c4)
    dev = f"cuda:{ctx.device}"
    out = grid_sample_trilinear_device(coords, torch.from_numpy(feats).to(dev), grid_size,
                                       torch.from_numpy(query).to(dev))
    return out.cpu().numpy()
