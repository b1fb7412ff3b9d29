"""ctypes binding of libmxq.so (include/mxq.h).

The shared library is the product: there is no CPU or PyTorch fallback.  If
the library is missing the import fails loudly; if no sm_100a device is
present, creating a context fails with MXQ_ERR_UNSUPPORTED / CUDA errors.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmxq.so")

MXQ_OK = 0
MXQ_ERR_INVALID_ARGUMENT = -1
MXQ_ERR_CUDA = -2
MXQ_ERR_TIMEOUT = -3
MXQ_ERR_OUT_OF_MEMORY = -4
MXQ_ERR_UNSUPPORTED = -5

FMT_INT4 = 4
FMT_INT8 = 8
ACT_NONE = 0
ACT_SILU = 1
PATH_AUTO = 0
PATH_GEMV = 1
PATH_GEMM = 2
PEER_HANDLE_BYTES = 64

_vp = ctypes.c_void_p
_sz = ctypes.c_size_t
_i = ctypes.c_int
_f = ctypes.c_float

# name -> argtypes (restype is int for all but mxq_last_error)
SIGNATURES = {
    "mxq_abi_version": [],
    "mxq_create": [_i, ctypes.POINTER(_vp)],
    "mxq_destroy": [_vp],
    "mxq_set_stream": [_vp, _vp],
    "mxq_set_path": [_vp, _i],
    "mxq_reserve": [_vp, _sz, _sz],
    "mxq_synchronize": [_vp],
    "mxq_last_error": [_vp],
    "mxq_launch_count": [_vp, ctypes.POINTER(ctypes.c_uint64)],
    "mxq_weight_create": [_vp, _i, _sz, _sz, _vp, _vp, _i, ctypes.POINTER(_vp)],
    "mxq_weight_create_bsr": [_vp, _i, _sz, _sz, _vp, _vp, _vp, _i, ctypes.POINTER(_vp)],
    "mxq_weight_destroy": [_vp],
    "mxq_weight_shape": [_vp, ctypes.POINTER(_i), ctypes.POINTER(_sz), ctypes.POINTER(_sz)],
    "mxq_quantize_x": [_vp, _vp, _sz, _sz, _i, _vp, _vp],
    "mxq_swiglu_quantize": [_vp, _vp, _vp, _sz, _sz, _vp, _vp],
    "mxq_gemv": [_vp, _vp, _vp, _vp, _sz, _vp],
    "mxq_gather_dot": [_vp, _vp, _vp, _vp, _sz, _vp, _sz, _vp],
    "mxq_block_dots": [_vp, _vp, _vp, _sz, _vp],
    "mxq_linear": [_vp, _vp, _vp, _sz, _vp],
    "mxq_linear_host": [_vp, _vp, _vp, _sz, _vp],
    "mxq_linear_pair": [_vp, _vp, _vp, _vp, _sz, _vp],
    "mxq_linear_pair_host": [_vp, _vp, _vp, _vp, _sz, _vp],
    "mxq_peers_create": [_vp, _i, _i, _sz, _sz, ctypes.POINTER(_vp), _vp],
    "mxq_peers_connect": [_vp, _vp],
    "mxq_peers_set_wait_limit": [_vp, ctypes.c_uint32],
    "mxq_peers_destroy": [_vp],
    "mxq_linear_pair_sharded": [_vp, _vp, _vp, _vp, _vp, _vp],
    "mxq_debug_peer_stall": [_vp, _vp, _vp, ctypes.c_uint32],
    "mxq_mlp_swiglu": [_vp, _vp, _vp, _vp, _vp, _sz, _vp],
    "mxq_linear_noalloc": [_vp, _vp, _vp, _sz, _vp],
    "mxq_debug_gemm_stall": [_vp, _vp, _vp, _sz, _vp, ctypes.c_uint32],
    "mxq_route_topk": [_vp, _vp, _sz, _sz, _sz, _vp, _vp],
    "mxq_decoder_create": [_vp, _vp, ctypes.c_uint64, ctypes.POINTER(_vp)],
    "mxq_decoder_create_sharded": [_vp, _vp, ctypes.c_uint64, _i, _i, ctypes.POINTER(_vp), _vp],
    "mxq_decoder_connect": [_vp, _vp],
    "mxq_decoder_set_wait_limit": [_vp, ctypes.c_uint32],
    "mxq_decoder_destroy": [_vp],
    "mxq_decoder_reset": [_vp],
    "mxq_decoder_length": [_vp, ctypes.POINTER(_i)],
    "mxq_decoder_prefill": [_vp, _vp, _sz, _sz, _vp],
    "mxq_decoder_decode": [_vp, _vp, _sz, _vp],
    "mxq_decoder_score": [_vp, _vp, _sz, _sz, _vp, _vp],
    "mxq_decoder_weight": [_vp, _i, _i, ctypes.POINTER(_vp)],
    "mxq_decoder_embedding": [_vp, _sz, _sz, _vp],
    "mxq_decoder_set_trace": [_vp, _i],
    "mxq_decoder_get_trace": [_vp, _i, _vp, _sz],
    "mxq_weight_download": [_vp, _vp, _vp],
    "mxq_weight_save": [_vp, ctypes.c_char_p],
    "mxq_update_gaussian_moment": [_vp, _vp, _vp, _vp, _f],
    "mxq_activation_norm": [_vp, _vp, _vp, _sz, _sz, _vp],
    "mxq_micro_moe": [_vp, _vp, _vp, _vp, _sz, _sz, _vp, _vp, _vp, _sz, _sz, _vp],
    "mxq_weight_load": [_vp, ctypes.c_char_p, ctypes.POINTER(_vp)],
    "mxq_quantize_w": [_vp, _i, _vp, _sz, _sz, _vp, _vp, _vp],
    "mxq_weight_quantize": [_vp, _i, _sz, _sz, _vp, _i, ctypes.POINTER(_vp)],
    "mxq_halting_step_host": [_vp, _vp, _vp, _vp, _f, _vp, _vp, _vp],
    "mxq_rank16_dot_ptrs": [_vp, _vp, _sz, _vp, _vp, _sz, _vp],
    "mxq_halting_step": [_vp, _vp, _vp, _vp, _sz, _f, _vp, _vp, _vp],
    "mxq_hashed_route": [_vp, _vp, _sz, _sz, _sz, _sz, _sz, ctypes.c_uint64, _vp, _vp],
    "mxq_hashed_route_host": [_vp, _vp, _sz, _sz, _sz, _sz, _sz, ctypes.c_uint64, _vp, _vp],
    "mxq_moe_swiglu": [_vp, _vp, _vp, _vp, _sz, _vp, _vp, _sz, _sz, _vp],
    "mxq_moe_group_create": [_vp, _i, _i, _sz, _sz, _sz, ctypes.POINTER(_vp), _vp],
    "mxq_moe_group_connect": [_vp, _vp],
    "mxq_moe_group_set_wait_limit": [_vp, ctypes.c_uint32],
    "mxq_moe_group_destroy": [_vp],
    "mxq_moe_swiglu_sharded": [_vp, _vp, _vp, _vp, _vp, _sz, _vp, _vp, _sz, _sz, _vp],
    "mxq_policy_head": [_vp, _vp, _vp, _sz, _sz, _vp, _vp, _vp],
    "mxq_gae": [_vp, _vp, _vp, _vp, _vp, _sz, _sz, _f, _f, _vp, _vp],
    "mxq_gae_ring": [_vp, _vp, _vp, _vp, _vp, _sz, _sz, _sz, _sz, _sz, _f, _f, _vp, _vp],
}

_lib = None


def load():
    """Load libmxq.so once; raise ImportError if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            "libmxq.so is not built (expected at %s); run `python -m cpu_model_b200.build`" % LIB_PATH)
    lib = ctypes.CDLL(LIB_PATH)
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = ctypes.c_char_p if name == "mxq_last_error" else ctypes.c_int
    _lib = lib
    return lib


class MXError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__("%s (status %d)" % (msg, code))
        self.code = code


def check(rc, ctx_handle=None):
    """Raise on a negative status: ValueError for invalid arguments (the
    reference operators throw std::invalid_argument), MXError otherwise."""
    if rc == MXQ_OK:
        return
    msg = load().mxq_last_error(ctx_handle)
    msg = msg.decode() if msg else "error"
    if rc == MXQ_ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    raise MXError(rc, msg)
