"""ctypes binding of libt2sc.so (the C ABI declared in include/t2sc.h).

The shared library is built in-tree by ``trellis2-mojo_b200/build.py``. There
is no fallback: if the library is missing, importing this module raises.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libt2sc.so")

OK = 0
ERR_INVALID, ERR_CUDA, ERR_OOM, ERR_RANGE, ERR_TIMEOUT, ERR_UNSUPPORTED, ERR_CAPACITY = 1, 2, 3, 4, 5, 6, 7
DT_F32, DT_F16, DT_BF16 = 0, 1, 2
SILU, RESIDUAL = 1, 2
SUB_NONZERO, SUB_POSITIVE = 0, 1
FEATS_NONE, FEATS_UPSAMPLE, FEATS_C2S = 0, 1, 2

_NAMES = {ERR_INVALID: "invalid argument", ERR_CUDA: "CUDA error", ERR_OOM: "out of memory",
          ERR_RANGE: "coordinate out of range", ERR_TIMEOUT: "device wait timed out",
          ERR_UNSUPPORTED: "unsupported", ERR_CAPACITY: "buffer too small"}

# symbol -> (restype, argtypes); every symbol include/t2sc.h declares
P, I32, I64, U64, D, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_uint64, ctypes.c_double, ctypes.c_float
PP = ctypes.POINTER(ctypes.c_void_p)
PI64 = ctypes.POINTER(ctypes.c_int64)
SIGNATURES = {
    "t2sc_ctx_create": (I32, [I32, PP]),
    "t2sc_ctx_destroy": (I32, [P]),
    "t2sc_ctx_set_stream": (I32, [P, P]),
    "t2sc_ctx_synchronize": (I32, [P]),
    "t2sc_last_error": (ctypes.c_char_p, [P]),
    "t2sc_ctx_launch_count": (I32, [P, PI64]),
    "t2sc_version": (ctypes.c_char_p, []),
    "t2sc_ctx_selftest": (I32, [P, I32]),
    "t2sc_coords_create": (I32, [P, P, I64, PP]),
    "t2sc_coords_create_device": (I32, [P, P, I64, PP]),
    "t2sc_coords_create_halo": (I32, [P, P, I64, I64, I32, PP]),
    "t2sc_coords_create_range": (I32, [P, P, I64, I64, I64, I32, PP]),
    "t2sc_coords_destroy": (I32, [P]),
    "t2sc_coords_count": (I32, [P, PI64]),
    "t2sc_coords_build_map": (I32, [P, I32, I32, I32, I32, PI64]),
    "t2sc_neighbor_map_export": (I32, [P, I32, I32, I32, I32, P, P, P, I64, PI64]),
    "t2sc_csr_export": (I32, [P, I32, I32, I32, I32, P, P, P, I64, PI64]),
    "t2sc_conv_create": (I32, [P, P, P, I32, I32, I32, I32, I32, I32, I32, PP]),
    "t2sc_conv_destroy": (I32, [P]),
    "t2sc_conv_forward": (I32, [P, P, P, P, I32, P]),
    "t2sc_conv_forward_device": (I32, [P, P, P, P, I32, P]),
    "t2sc_conv_chain_forward": (I32, [P, I32, P, P, P, P]),
    "t2sc_subdivide": (I32, [P, P, I64, P, I32, P, I32, I32, P, P, P, P, PI64]),
    "t2sc_subdivide_device": (I32, [P, P, I64, P, I32, P, I32, I32, I32, P, P, P, P, PI64]),
    "t2sc_subdivide_noalloc_device": (I32, [P, P, I64, P, I32, P, I32, I32, I32, P, P, P, P, PI64]),
    "t2sc_linear_create": (I32, [P, P, P, I32, I32, I32, PP]),
    "t2sc_linear_forward_device": (I32, [P, P, P, I64, I32, P]),
    "t2sc_layernorm_device": (I32, [P, P, P, I64, I32, P, P, F, I32, I32]),
    "t2sc_fdg_head_device": (I32, [P, P, I64, D, P, P, P]),
    "t2sc_cascade_coords_device": (I32, [P, P, I64, I32, I32, I64, P, PI64, ctypes.POINTER(ctypes.c_int)]),
    "t2sc_grid_sample_trilinear_device": (I32, [P, P, I32, I32, P, I64, P]),
    "t2sc_convnext_block_create": (I32, [P, I32, I32, P, P, P, P, P, P, P, P, I32, PP]),
    "t2sc_convnext_block_destroy": (I32, [P]),
    "t2sc_convnext_block_forward_device": (I32, [P, P, P, P]),
    "t2sc_c2s_block_create": (I32, [P, I32, I32, I32, P, P, P, P, P, P, P, P, I32, PP]),
    "t2sc_c2s_block_destroy": (I32, [P]),
    "t2sc_c2s_block_forward_device": (I32, [P, P, P, P, P, P, PI64, PP]),
    "t2sc_partition_zslab": (I32, [P, I64, I32, I32, I32, P, I64, P]),
    "t2sc_comm_unique_id": (I32, [P]),
    "t2sc_comm_create": (I32, [P, P, I32, I32, I32, PP]),
    "t2sc_comm_destroy": (I32, [P]),
    "t2sc_comm_abort": (I32, [P]),
    "t2sc_halo_exchange_device": (I32, [P, P, I64, P]),
    "t2sc_comm_wait": (I32, [P, I32]),
    "t2sc_synth_shell": (I32, [I32, D, D, U64, I32, P, I64, PI64]),
    "t2sc_synth_normal": (I32, [U64, F, P, I64]),
    "t2sc_synth_bernoulli": (I32, [U64, D, P, I64]),
}


class T2SCError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"t2sc: {_NAMES.get(code, code)}: {msg}")
        self.code = code


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"libt2sc.so not built ({LIB_PATH}); run trellis2-mojo_b200/build.py")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def check(rc, ctx=None):
    if rc != OK:
        msg = lib.t2sc_last_error(ctx).decode() if ctx else ""
        raise T2SCError(rc, msg)
