"""Host-side mirror of the TRELLIS.2-Mojo sparse operator API over libt2sc.

Same names, argument meaning and error behaviour as the reference:
  SparseTensor                 trellis2_mojo/sparse/basic.mojo:296-339 (batch-order contract)
  SparseConv3d                 trellis2_mojo/sparse/conv.mojo:19-199
  sparse_conv3d_from           trellis2_mojo/loaders.mojo:43-50
  SparseUpsample               trellis2_mojo/sparse/spatial/basic.mojo:121-174
  SparseChannel2Spatial        trellis2_mojo/sparse/spatial/spatial2channel.mojo:80-145
  binarize                     trellis2_mojo/models/sc_vaes/sparse_unet_vae.mojo:30-37
  LayerNorm32                  trellis2_mojo/modules/nn.mojo:297-375 (+ fused SiLU, nn.mojo:614-621)
  SparseLinear                 trellis2_mojo/modules/nn.mojo:268-293 (linear, nn.mojo:27-266)

Every operator runs on the GPU through the C ABI; there is no CPU path.
Features are host numpy f32 arrays (the reference's Tensor[F32]); the
coordinate hash and neighbour maps live on the device in a handle shared by
every tensor derived through ``replace`` (the reference's spatial cache).
"""
import ctypes

import numpy as np

from . import _lib
from ._lib import check, lib

_DTYPES = {"f32": _lib.DT_F32, "f16": _lib.DT_F16, "bf16": _lib.DT_BF16}


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


class Context:
    """One per device; replaces GpuContext (trellis2_mojo/gpu/context.mojo:116-165)."""

    _default = {}

    def __init__(self, device=0):
        h = ctypes.c_void_p()
        rc = lib.t2sc_ctx_create(device, ctypes.byref(h))
        check(rc)
        self.handle = h
        self.device = device

    @classmethod
    def default(cls, device=0):
        if device not in cls._default:
            cls._default[device] = cls(device)
        return cls._default[device]

    def selftest(self, wait_us=2000):
        """Compute check + a bounded device wait that must time out cleanly."""
        check(lib.t2sc_ctx_selftest(self.handle, wait_us), self.handle)

    def synchronize(self):
        check(lib.t2sc_ctx_synchronize(self.handle), self.handle)

    def launch_count(self):
        v = ctypes.c_int64()
        check(lib.t2sc_ctx_launch_count(self.handle, ctypes.byref(v)), self.handle)
        return v.value

    def set_stream(self, stream_ptr):
        check(lib.t2sc_ctx_set_stream(self.handle, ctypes.c_void_p(stream_ptr) if stream_ptr else None),
              self.handle)

    def close(self):
        if self.handle:
            lib.t2sc_ctx_destroy(self.handle)
            self.handle = None


class Coords:
    """Device coordinates + hash + cached neighbour maps (the spatial cache)."""

    def __init__(self, ctx, coords=None, n=None, device_ptr=None, n_targets=None, targets=None):
        """n_targets: only the first n_targets rows receive conv outputs; the
        rest are halo rows that act as sources (t2sc_coords_create_halo)."""
        self.ctx = ctx
        h = ctypes.c_void_p()
        if targets is not None:  # target rows [t0, t1); all rows are sources
            coords = np.ascontiguousarray(coords, dtype=np.int32)
            rc = lib.t2sc_coords_create_range(ctx.handle, _p(coords), coords.shape[0], int(targets[0]), int(targets[1]),
                                              0, ctypes.byref(h))
        elif n_targets is not None:
            coords = np.ascontiguousarray(coords, dtype=np.int32)
            rc = lib.t2sc_coords_create_halo(ctx.handle, _p(coords), coords.shape[0], n_targets, 0, ctypes.byref(h))
        elif device_ptr is not None:
            rc = lib.t2sc_coords_create_device(ctx.handle, ctypes.c_void_p(device_ptr), n, ctypes.byref(h))
        else:
            coords = np.ascontiguousarray(coords, dtype=np.int32)
            rc = lib.t2sc_coords_create(ctx.handle, _p(coords), coords.shape[0], ctypes.byref(h))
        check(rc, ctx.handle)
        self.handle = h
        v = ctypes.c_int64()
        check(lib.t2sc_coords_count(h, ctypes.byref(v)))
        self.n = v.value

    @classmethod
    def from_handle(cls, ctx, handle):
        """Wraps a coordinate handle the library returned (owned from now on)."""
        self = cls.__new__(cls)
        self.ctx, self.handle = ctx, handle
        v = ctypes.c_int64()
        check(lib.t2sc_coords_count(handle, ctypes.byref(v)))
        self.n = v.value
        return self

    def build_map(self, kernel=(3, 3, 3), dilation=1):
        e = ctypes.c_int64()
        check(lib.t2sc_coords_build_map(self.handle, *kernel, dilation, ctypes.byref(e)), self.ctx.handle)
        return e.value

    def neighbor_map(self, kernel=(3, 3, 3), dilation=1):
        """(src, tgt, kidx) int64 edge lists in the reference order (conv.mojo:56-96)."""
        e = self.build_map(kernel, dilation)
        src, tgt, kidx = (np.empty(e, np.int64) for _ in range(3))
        ne = ctypes.c_int64()
        check(lib.t2sc_neighbor_map_export(self.handle, *kernel, dilation, _p(src), _p(tgt), _p(kidx), e,
                                           ctypes.byref(ne)), self.ctx.handle)
        return src, tgt, kidx

    def csr(self, kernel=(3, 3, 3), dilation=1):
        """(row_start, src_s, kidx_s) as conv.mojo:117-147 builds them."""
        e = self.build_map(kernel, dilation)
        rs = np.empty(self.n + 1, np.int64)
        src, kidx = np.empty(e, np.int64), np.empty(e, np.int64)
        ne = ctypes.c_int64()
        check(lib.t2sc_csr_export(self.handle, *kernel, dilation, _p(rs), _p(src), _p(kidx), e, ctypes.byref(ne)),
              self.ctx.handle)
        return rs, src, kidx

    def __del__(self):
        h = getattr(self, "handle", None)
        if h and self.ctx.handle:
            lib.t2sc_coords_destroy(h)
            self.handle = None


class SparseTensor:
    """feats f32 [N, C] + coords int32 [N, 4] (b, x, y, z); batches ordered
    (the contract SparseTensor._cal_offsets enforces, basic.mojo:320-339)."""

    def __init__(self, feats, coords, batch_size=-1, ctx=None, _cache=None):
        feats = np.ascontiguousarray(feats, dtype=np.float32)
        coords = np.ascontiguousarray(coords, dtype=np.int32)
        if coords.ndim != 2 or coords.shape[1] != 4:
            raise ValueError("SparseTensor: coords must be [N, 4]")
        if feats.shape[0] != coords.shape[0]:
            raise ValueError("SparseTensor: feats/coords row mismatch")
        b = coords[:, 0]
        if batch_size < 0:
            batch_size = int(b.max()) + 1 if len(b) else 0
        if len(b) and np.any(np.diff(b) < 0):
            raise ValueError("SparseTensor: batches must be ordered/contiguous")
        if len(b) and (b.min() < 0 or b.max() >= batch_size):
            raise ValueError("SparseTensor: batch index out of range")
        self.feats = feats
        self.coords = coords
        self.batch_size = batch_size
        self.offsets = np.concatenate([[0], np.cumsum(np.bincount(b, minlength=batch_size))]).astype(np.int64)
        self._ctx = ctx
        # shared by every tensor derived through replace(), like the
        # reference's ArcPointer spatial cache
        self._cache = _cache if _cache is not None else {}

    def seqlen(self, b):
        """Rows of batch b (basic.mojo:378-379)."""
        return int(self.offsets[b + 1] - self.offsets[b])

    def seqlen_list(self):
        return [self.seqlen(b) for b in range(self.batch_size)]

    def batch_broadcast_map(self):
        """Row index -> batch index (basic.mojo:149-155, 384-385)."""
        return np.repeat(np.arange(self.batch_size), np.diff(self.offsets)).tolist()

    def spatial_shape(self):
        """Per spatial axis, the largest coordinate + 1, cached with the
        coordinates like the reference's "shape" entry (basic.mojo:387-395)."""
        if "shape" not in self._cache:
            self._cache["shape"] = [int(self.coords[:, c].max()) + 1 if len(self.coords) else 0 for c in (1, 2, 3)]
        return list(self._cache["shape"])

    @property
    def ctx(self):
        if self._ctx is None:
            self._ctx = Context.default()
        return self._ctx

    @property
    def device_coords(self):
        if "coords" not in self._cache:
            self._cache["coords"] = Coords(self.ctx, self.coords)
        return self._cache["coords"]

    def replace(self, feats):
        """New feats, same coords and spatial cache (basic.mojo:399-404)."""
        return SparseTensor(feats, self.coords, self.batch_size, self._ctx, self._cache)

    def __add__(self, other):
        return self.replace(self.feats + other.feats)


class SparseConv3d:
    """Submanifold conv, stride 1. weight [Co, Kd, Kh, Kw, Ci] (conv_none
    layout), bias [Co]. dtype: "f32" (f32-accurate), "f16" or "bf16"
    (16-bit inputs and weights, f32 accumulation). The weights are uploaded
    once here (GpuSparseConv.try_build, gpu/conv.mojo:264-329, without its
    Co % 64 gate: every shape runs on the GPU)."""

    def __init__(self, weight, bias=None, has_bias=True, dilation=1, dtype="f32", ctx=None):
        weight = np.ascontiguousarray(weight, dtype=np.float32)
        if weight.ndim != 5:
            raise ValueError("SparseConv3d: weight must be [Co, Kd, Kh, Kw, Ci]")
        self.out_channels = weight.shape[0]
        self.in_channels = weight.shape[4]
        self.kernel_size = tuple(weight.shape[1:4])
        self.dilation = dilation
        self.has_bias = has_bias and bias is not None
        self.weight = weight
        self.bias = np.ascontiguousarray(bias, dtype=np.float32) if self.has_bias else None
        self.dtype = dtype
        self.ctx = ctx or Context.default()
        h = ctypes.c_void_p()
        kd, kh, kw = self.kernel_size
        check(lib.t2sc_conv_create(self.ctx.handle, _p(weight), _p(self.bias), self.out_channels, kd, kh, kw,
                                   self.in_channels, dilation, _DTYPES[dtype], ctypes.byref(h)), self.ctx.handle)
        self.handle = h

    def forward(self, x, silu=False, residual=None):
        """SparseConv3d.forward (conv.mojo:98-199); optional fused SiLU and
        residual add (the decoder's activation / `h + x`)."""
        if x.feats.shape[1] != self.in_channels:
            raise ValueError("SparseConv3d: in_features mismatch")
        y = np.empty((x.feats.shape[0], self.out_channels), np.float32)
        flags = (_lib.SILU if silu else 0) | (_lib.RESIDUAL if residual is not None else 0)
        res = None
        if residual is not None:
            res = np.ascontiguousarray(residual.feats if isinstance(residual, SparseTensor) else residual,
                                       dtype=np.float32)
            if res.shape != y.shape:
                raise ValueError("SparseConv3d: residual shape mismatch")
        check(lib.t2sc_conv_forward(self.handle, x.device_coords.handle, _p(x.feats), _p(y), flags, _p(res)),
              self.ctx.handle)
        return x.replace(y)

    __call__ = forward

    def __del__(self):
        h = getattr(self, "handle", None)
        if h and self.ctx.handle:
            lib.t2sc_conv_destroy(h)
            self.handle = None


def conv_chain(convs, x, flags):
    """Several convs on the same coordinates with device-resident
    intermediates (one upload, one download)."""
    n = x.feats.shape[0]
    y = np.empty((n, convs[-1].out_channels), np.float32)
    arr = (ctypes.c_void_p * len(convs))(*[c.handle.value for c in convs])
    fl = (ctypes.c_int * len(convs))(*flags)
    check(lib.t2sc_conv_chain_forward(arr, len(convs), x.device_coords.handle, _p(x.feats), _p(y), fl),
          convs[0].ctx.handle)
    return x.replace(y)


def sparse_conv3d_from(state_dict, prefix, dilation=1, dtype="f32", ctx=None):
    """loaders.mojo:43-50: the conv_none weight is already [Co, Kd, Kh, Kw, Ci]."""
    return SparseConv3d(state_dict[prefix + ".weight"], state_dict.get(prefix + ".bias"), dilation=dilation,
                        dtype=dtype, ctx=ctx)


class Binarized:
    """A subdivision tensor to be read as `sub > 0` on the device
    (the decoder's _binarize, sparse_unet_vae.mojo:30-37)."""

    def __init__(self, subdiv):
        self.subdiv = subdiv


def binarize(subdiv):
    """Marks `subdiv` for the `> 0` test; the comparison itself runs in the
    subdivision kernel (T2SC_SUB_POSITIVE)."""
    return Binarized(subdiv)


def _subdivide(x, subdivision, feats_mode, keep_mode):
    if isinstance(subdivision, Binarized):
        subdivision, keep_mode = subdivision.subdiv, _lib.SUB_POSITIVE
    sub = np.ascontiguousarray(subdivision.feats if isinstance(subdivision, SparseTensor) else subdivision,
                               dtype=np.float32)
    n = x.coords.shape[0]
    if sub.shape != (n, 8):
        raise ValueError("subdivision feats must be [N, 8]")
    c_in = x.feats.shape[1]
    if feats_mode == _lib.FEATS_C2S:
        if c_in % 8:
            raise ValueError("SparseChannel2Spatial: channels must be divisible by 8")
        c = c_in // 8
    else:
        c = c_in
    out_coords = np.empty((8 * n, 4), np.int32)
    out_feats = np.empty((8 * n, c), np.float32)
    parent = np.empty(8 * n, np.int64)
    subidx = np.empty(8 * n, np.int64)
    m = ctypes.c_int64()
    ctx = x.ctx
    check(lib.t2sc_subdivide(ctx.handle, _p(x.coords), n, _p(sub), keep_mode, _p(x.feats), c, feats_mode,
                             _p(out_coords), _p(out_feats), _p(parent), _p(subidx), ctypes.byref(m)), ctx.handle)
    m = m.value
    out = SparseTensor(out_feats[:m].copy(), out_coords[:m].copy(), x.batch_size, ctx)
    out.parent_idx, out.subidx = parent[:m].copy(), subidx[:m].copy()
    return out


class SparseUpsample:
    def __init__(self, factor=2):
        if factor != 2:
            raise ValueError("SparseUpsample: only factor 2 (subdivision) is supported")
        self.factor = factor

    def forward_subdivision(self, x, subdivision):
        """Children where sub != 0, parent feats copied (spatial/basic.mojo:144-174)."""
        return _subdivide(x, subdivision, _lib.FEATS_UPSAMPLE, _lib.SUB_NONZERO)


class SparseChannel2Spatial:
    def __init__(self, factor=2):
        if factor != 2:
            raise ValueError("SparseChannel2Spatial: only factor 2 is supported")
        self.factor = factor

    def forward_subdivision(self, x, subdivision):
        """Children where sub != 0, feats = channel slice c*C:(c+1)*C
        (spatial2channel.mojo:97-145)."""
        return _subdivide(x, subdivision, _lib.FEATS_C2S, _lib.SUB_NONZERO)


class LayerNorm32:
    """LayerNorm over the channel dim, statistics in f32 (nn.mojo:297-375),
    optionally followed by SiLU (the decoder's norm -> activation(ACT_SILU)
    pairs, sparse_unet_vae.mojo:118,123) in the same kernel."""

    def __init__(self, num_channels, eps=1e-5, affine=True, ctx=None):
        if num_channels < 1 or num_channels > 1024:
            raise ValueError("LayerNorm32: 1 <= num_channels <= 1024")
        self.num_channels, self.eps, self.affine = num_channels, float(eps), affine
        self.weight = np.ones(num_channels, np.float32) if affine else None   # nn.mojo:311-312
        self.bias = np.zeros(num_channels, np.float32) if affine else None
        self.ctx = ctx or Context.default()
        self._dev_wb = None

    def load(self, weight, bias):
        self.weight = np.ascontiguousarray(weight, np.float32).reshape(self.num_channels)
        self.bias = np.ascontiguousarray(bias, np.float32).reshape(self.num_channels)
        self._dev_wb = None

    def _wb(self):
        import torch
        if not self.affine:
            return None, None
        if self._dev_wb is None:
            dev = f"cuda:{self.ctx.device}"
            self._dev_wb = (torch.from_numpy(self.weight).to(dev), torch.from_numpy(self.bias).to(dev))
        return self._dev_wb

    def forward_device(self, x, y=None, silu=False):
        """x: CUDA tensor [rows, C] (float32/float16/bfloat16); y defaults to
        a new tensor (y may be x). Runs on the context's stream, which is
        ordered after torch's current stream at entry and before it on return."""
        import torch
        _check_on_ctx_device(x, self.ctx, "LayerNorm32: x")
        if x.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            raise ValueError("LayerNorm32: x must be float32, float16 or bfloat16")
        dt = _torch_dtype_code(x.dtype)
        if x.dim() != 2 or x.shape[1] != self.num_channels or not x.is_contiguous():
            raise ValueError("LayerNorm32: x must be contiguous [rows, num_channels]")
        if y is None:
            y = torch.empty_like(x)
        else:
            _check_on_ctx_device(y, self.ctx, "LayerNorm32: y")
            if y.shape != x.shape or y.dtype != x.dtype or not y.is_contiguous():
                raise ValueError("LayerNorm32: y must be a contiguous tensor of x's shape and dtype")
        w, b = self._wb()
        torch.cuda.current_stream(x.device).synchronize()
        check(lib.t2sc_layernorm_device(self.ctx.handle, ctypes.c_void_p(x.data_ptr()),
                                        ctypes.c_void_p(y.data_ptr()), x.shape[0], self.num_channels,
                                        ctypes.c_void_p(w.data_ptr()) if w is not None else None,
                                        ctypes.c_void_p(b.data_ptr()) if b is not None else None,
                                        self.eps, _lib.SILU if silu else 0, dt), self.ctx.handle)
        self.ctx.synchronize()
        return y

    def forward(self, feats, silu=False):
        """feats: host f32 [N, C] or a SparseTensor (then returns x.replace)."""
        import torch
        st = feats if isinstance(feats, SparseTensor) else None
        f = np.ascontiguousarray(st.feats if st is not None else feats, np.float32)
        y = self.forward_device(torch.from_numpy(f).to(f"cuda:{self.ctx.device}"), silu=silu).cpu().numpy()
        return st.replace(y) if st is not None else y

    __call__ = forward


def _check_on_ctx_device(t, ctx, what):
    """A device buffer handed to the library must live on the context's GPU:
    a host tensor or one on another GPU would be read or written through
    the wrong address space by the kernels."""
    if not getattr(t, "is_cuda", False) or t.device.index != ctx.device:
        raise ValueError(f"{what} must be a CUDA tensor on cuda:{ctx.device}")


def _torch_dtype_code(t):
    import torch
    return {torch.float32: _lib.DT_F32, torch.float16: _lib.DT_F16, torch.bfloat16: _lib.DT_BF16}[t]


class SparseLinear:
    """y = x @ weight.T + bias over the channel dim (nn.mojo:268-293), on the
    conv kernels with a 1x1x1 kernel over an identity row map. weight
    [Co, Ci], bias [Co]. dtype as SparseConv3d ("f32" f32-accurate, "f16" /
    "bf16" 16-bit inputs, f32 accumulation). SiLU and a residual add fuse
    into the epilogue (the ConvNeXt block's lin1/SiLU and lin2 + x)."""

    def __init__(self, weight, bias=None, has_bias=True, dtype="f32", ctx=None):
        weight = np.ascontiguousarray(weight, dtype=np.float32)
        if weight.ndim != 2:
            raise ValueError("SparseLinear: weight must be [Co, Ci]")
        self.out_features, self.in_features = weight.shape
        self.has_bias = has_bias and bias is not None
        self.weight = weight
        self.bias = np.ascontiguousarray(bias, dtype=np.float32) if self.has_bias else None
        self.dtype = dtype
        self.ctx = ctx or Context.default()
        h = ctypes.c_void_p()
        check(lib.t2sc_linear_create(self.ctx.handle, _p(weight), _p(self.bias), self.out_features,
                                     self.in_features, _DTYPES[dtype], ctypes.byref(h)), self.ctx.handle)
        self.handle = h

    def forward_device(self, x, silu=False, residual=None):
        """x: CUDA tensor [rows, Ci] of the layer's dtype (float32 for "f32");
        returns a new [rows, Co] tensor. Runs on the context's stream, ordered
        after torch's current stream at entry and before it on return."""
        import torch
        _check_on_ctx_device(x, self.ctx, "SparseLinear: x")
        if residual is not None:
            _check_on_ctx_device(residual, self.ctx, "SparseLinear: residual")
        if x.dim() != 2 or x.shape[1] != self.in_features or not x.is_contiguous():
            raise ValueError("SparseLinear: x must be contiguous [rows, in_features]")
        if x.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            raise ValueError("SparseLinear: x dtype does not match the layer's dtype")
        if _torch_dtype_code(x.dtype) != _DTYPES[self.dtype]:
            raise ValueError("SparseLinear: x dtype does not match the layer's dtype")
        y = torch.empty((x.shape[0], self.out_features), dtype=x.dtype, device=x.device)
        flags = (_lib.SILU if silu else 0) | (_lib.RESIDUAL if residual is not None else 0)
        if residual is not None and (residual.shape != y.shape or residual.dtype != y.dtype
                                     or not residual.is_contiguous()):
            raise ValueError("SparseLinear: residual must be a contiguous [rows, out_features] tensor of x's dtype")
        torch.cuda.current_stream(x.device).synchronize()
        check(lib.t2sc_linear_forward_device(self.handle, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()),
                                             x.shape[0], flags,
                                             ctypes.c_void_p(residual.data_ptr()) if residual is not None else None),
              self.ctx.handle)
        self.ctx.synchronize()
        return y

    def forward(self, x, silu=False, residual=None):
        """x: host f32 [N, Ci] or a SparseTensor (then returns x.replace);
        residual: host f32 [N, Co] / SparseTensor or None."""
        import torch
        st = x if isinstance(x, SparseTensor) else None
        f = np.ascontiguousarray(st.feats if st is not None else x, np.float32)
        if f.ndim != 2 or f.shape[1] != self.in_features:
            raise ValueError("SparseLinear: in_features mismatch")
        tdt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[self.dtype]
        dev = f"cuda:{self.ctx.device}"
        res = None
        if residual is not None:
            r = residual.feats if isinstance(residual, SparseTensor) else residual
            res = torch.from_numpy(np.ascontiguousarray(r, np.float32)).to(dev, tdt)
        y = self.forward_device(torch.from_numpy(f).to(dev, tdt), silu=silu, residual=res)
        y = y.float().cpu().numpy()
        return st.replace(y) if st is not None else y

    __call__ = forward

    def __del__(self):
        h = getattr(self, "handle", None)
        if h and self.ctx.handle:
            lib.t2sc_conv_destroy(h)
            self.handle = None


class SparseResBlockC2S3d:
    """The decoder's up block (sparse_unet_vae.mojo:67-133) on the device in
    one C-ABI call per forward: LN1/SiLU -> conv1 (C -> 8*Cout) -> C2S by the
    binarized subdivision -> LN2/SiLU -> conv2 + repeat-interleaved C2S of
    x. Weights as the checkpoint holds them (host f32): norm1 (weight,
    bias) [C], conv1 [8*Cout, 3, 3, 3, C] + [8*Cout], conv2
    [Cout, 3, 3, 3, Cout] + [Cout], to_subdiv [8, C] + [8] (pred_subdiv)."""

    def __init__(self, channels, out_channels, pred_subdiv, norm1, conv1, conv2, to_subdiv=None, dtype="f32",
                 ctx=None):
        self.channels, self.out_channels, self.pred_subdiv = channels, out_channels, bool(pred_subdiv)
        self.dtype = dtype
        self.ctx = ctx or Context.default()
        f = lambda a: None if a is None else np.ascontiguousarray(a, np.float32)  # noqa: E731
        self._keep = [f(norm1[0]), f(norm1[1]), f(conv1[0]), f(conv1[1]), f(conv2[0]), f(conv2[1]),
                      f(to_subdiv[0]) if to_subdiv else None, f(to_subdiv[1]) if to_subdiv else None]
        if self.pred_subdiv and to_subdiv is None:
            raise ValueError("SparseResBlockC2S3d: pred_subdiv needs to_subdiv weights")
        h = ctypes.c_void_p()
        check(lib.t2sc_c2s_block_create(self.ctx.handle, channels, out_channels, int(self.pred_subdiv),
                                        *[_p(a) for a in self._keep], _DTYPES[dtype], ctypes.byref(h)),
              self.ctx.handle)
        self.handle = h

    def _run(self, x, subdiv=None):
        import torch
        if x.feats.shape[1] != self.channels:
            raise ValueError("SparseResBlockC2S3d: in_features mismatch")
        n = x.feats.shape[0]
        dev = f"cuda:{self.ctx.device}"
        tdt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[self.dtype]
        xd = torch.from_numpy(x.feats).to(dev, tdt)
        if subdiv is None:
            sd = torch.empty((n, 8), dtype=torch.float32, device=dev)
        else:
            sub = np.ascontiguousarray(subdiv.feats if isinstance(subdiv, SparseTensor) else subdiv, np.float32)
            if sub.shape != (n, 8):
                raise ValueError("SparseResBlockC2S3d: subdivision must be [N, 8]")
            sd = torch.from_numpy(sub).to(dev)
        oc = torch.empty((8 * max(n, 1), 4), dtype=torch.int32, device=dev)
        of = torch.empty((8 * max(n, 1), self.out_channels), dtype=tdt, device=dev)
        m = ctypes.c_int64()
        torch.cuda.synchronize(dev)
        check(lib.t2sc_c2s_block_forward_device(self.handle, x.device_coords.handle, ctypes.c_void_p(xd.data_ptr()),
                                                ctypes.c_void_p(sd.data_ptr()), ctypes.c_void_p(oc.data_ptr()),
                                                ctypes.c_void_p(of.data_ptr()), ctypes.byref(m), None),
              self.ctx.handle)
        self.ctx.synchronize()
        m = m.value
        out = SparseTensor(of[:m].float().cpu().numpy(), oc[:m].cpu().numpy(), x.batch_size, self.ctx)
        return out, sd.cpu().numpy()

    def forward(self, x):
        """pred_subdiv path: returns (h, subdiv)."""
        if not self.pred_subdiv:
            raise ValueError("SparseResBlockC2S3d: use forward_guided when pred_subdiv=False")
        return self._run(x)

    def forward_guided(self, x, subdiv):
        """guide_subs path: the subdivision comes from the shape decoder."""
        return self._run(x, subdiv)[0]

    def __del__(self):
        h = getattr(self, "handle", None)
        if h and self.ctx.handle:
            lib.t2sc_c2s_block_destroy(h)
            self.handle = None
