"""t2sc: B200-native sparse submanifold convolution for TRELLIS.2-Mojo.

The product is the C-ABI library libt2sc.so (include/t2sc.h); this package
is its Python host binding, mirroring the reference's operator API.
"""
from ._lib import LIB_PATH, T2SCError, lib  # noqa: F401  (raises if the library is missing)
from .sparse import (Binarized, Context, LayerNorm32, Coords, SparseChannel2Spatial, SparseConv3d, SparseLinear,  # noqa: F401
                     SparseResBlockC2S3d, SparseTensor,
                     SparseUpsample, binarize, conv_chain, sparse_conv3d_from)
from . import synth  # noqa: F401
from .decoder import SparseConvNeXtBlock3d, SparseUnetVaeDecoder  # noqa: F401
from .pipeline import (cascade_coords, cascade_coords_device, decode_shape, decode_tex, fdg_head,  # noqa: F401
                       fdg_head_device, grid_sample_trilinear, grid_sample_trilinear_device)

__version__ = "0.1"
