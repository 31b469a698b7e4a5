"""ctypes binding to libdsmoe.so (the C ABI in include/dsmoe.h).

Mirrors the reference's native binding style (dsv41/ref/fp4lib.py:5-11): ``ctypes.CDLL`` of an
in-tree shared library, raw pointers and integer sizes, the caller owns every buffer. Unlike the
reference binding, every call returns a status that is turned into an exception here.

There is no fallback: if the library is missing, importing this module raises.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdsmoe.so")

OK, ERR_ARG, ERR_ALIGN, ERR_CUDA, ERR_WORKSPACE, ERR_TIMEOUT, ERR_UNSUPPORTED = 0, -1, -2, -3, -4, -5, -6
FMT_FP8, FMT_FP4 = 0, 1
LAYOUT_FRAG, LAYOUT_TC = 0, 1
SCORE_SIGMOID, SCORE_SQRTSOFTPLUS = 0, 1
DTYPE_F32, DTYPE_BF16, DTYPE_E4M3 = 0, 1, 2
MAX_DECODE_TOKENS = 64
COMM_HANDLE_BYTES = 64
SLOT_TOKENS = 8

FMT_NAMES = {"fp8": FMT_FP8, "fp4": FMT_FP4}
SCORE_NAMES = {"sigmoid": SCORE_SIGMOID, "sqrtsoftplus": SCORE_SQRTSOFTPLUS}


class DsmoeError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"dsmoe error {code}: {msg}")
        self.code = code


class Store(ctypes.Structure):
    _fields_ = [("w13", ctypes.c_void_p), ("w2", ctypes.c_void_p),
                ("w13_expert_bytes", ctypes.c_longlong), ("w2_expert_bytes", ctypes.c_longlong),
                ("fmt", ctypes.c_int), ("n_experts", ctypes.c_int), ("layout", ctypes.c_int), ("row0", ctypes.c_int)]


class Layer(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int), ("inter_local", ctypes.c_int), ("n_experts", ctypes.c_int),
                ("topk", ctypes.c_int), ("score_func", ctypes.c_int), ("route_scale", ctypes.c_float),
                ("gate_w", ctypes.c_void_p), ("gate_bias", ctypes.c_void_p), ("gate_bias_vl", ctypes.c_void_p),
                ("routed", Store), ("shared", Store)]


_P, _I, _LL, _F = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_float
_SIGS = {
    "dsmoe_version": ([], _I),
    "dsmoe_fp8_block_dequant": ([_P, _P, _LL, _LL, _I, _P, _I, _P], _I),
    "dsmoe_fp4_dequant": ([_P, _P, _LL, _LL, _P, _I, _P], _I),
    "dsmoe_fp8_gemm": ([_P, _I, _P, _LL, _LL, _P, _P, _LL, _P, _I, _P], _I),
    "dsmoe_fp4_gemm": ([_P, _I, _P, _LL, _LL, _P, _P, _LL, _P, _I, _P], _I),
    "dsmoe_act_quant": ([_P, _I, _LL, _LL, _I, _I, _P, _P, _P], _I),
    "dsmoe_store_expert_bytes": ([_I, _I, _I, ctypes.POINTER(_LL), ctypes.POINTER(_LL)], _I),
    "dsmoe_store_pack_expert": ([_I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P], _I),
    "dsmoe_store_unpack_expert": ([_I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P], _I),
    "dsmoe_store_tc_expert_bytes": ([_I, _I, _I, _I, _I, ctypes.POINTER(_LL), ctypes.POINTER(_LL)], _I),
    "dsmoe_store_tc_pack_expert": ([_I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P], _I),
    "dsmoe_store_tc_unpack_expert": ([_I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P], _I),
    "dsmoe_moe_workspace_bytes": ([ctypes.POINTER(Layer), _I], ctypes.c_size_t),
    "dsmoe_router": ([ctypes.POINTER(Layer), _P, _I, _P, _P, _P, _P, _P, ctypes.c_size_t, _P], _I),
    "dsmoe_router_noalloc": ([ctypes.POINTER(Layer), _P, _I, _P, _P, _P, _P, _P], _I),
    "dsmoe_moe_decode": ([ctypes.POINTER(Layer), _P, _I, _P, _P, _I, _P, _P, _P, _P, ctypes.c_size_t, _P], _I),
    "dsmoe_moe_decode_profiled": ([ctypes.POINTER(Layer), _P, _I, _P, _P, _I, _P, _P, _P, _P, ctypes.c_size_t, _P,
                                   ctypes.POINTER(_P)], _I),
    "dsmoe_moe_check": ([ctypes.POINTER(Layer), _I, _P, ctypes.c_size_t, _P], _I),
    "dsmoe_f32_to_bf16": ([_P, _P, _LL, _P], _I),
    "dsmoe_copy_async": ([_P, _P, _LL, _P], _I),
    "dsmoe_moe_prefill_workspace_bytes": ([ctypes.POINTER(Layer), _I], ctypes.c_size_t),
    "dsmoe_moe_prefill": ([ctypes.POINTER(Layer), _P, _I, _P, _P, _P, _I, _P, ctypes.c_size_t, _P], _I),
    "dsmoe_moe_prefill_check": ([ctypes.POINTER(Layer), _I, _P, ctypes.c_size_t, _P], _I),
    "dsmoe_comm_create": ([_I, _I, _I, ctypes.POINTER(_P), _P], _I),
    "dsmoe_comm_open": ([_P, _P], _I),
    "dsmoe_comm_destroy": ([_P], _I),
    "dsmoe_moe_allreduce_supported": ([ctypes.POINTER(Layer), _P, _P, _I], _I),
    "dsmoe_allreduce_rows": ([_P, _P, _I, _I, _P, _I, _P], _I),
    "dsmoe_comm_check": ([_P, _P], _I),
    "dsmoe_moe_decode_allreduce": ([ctypes.POINTER(Layer), _P, _P, _I, _P, _P, _I, _P, _P, _P, _P, ctypes.c_size_t,
                                    _P], _I),
}


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it first (python __graft_entry__.py build, or make -C csrc)")
    lib = ctypes.CDLL(LIB_PATH)
    lib.dsmoe_last_error.argtypes = []
    lib.dsmoe_last_error.restype = ctypes.c_char_p
    for name, (args, res) in _SIGS.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    return lib


lib = _load()


def check(code: int) -> None:
    if code != OK:
        raise DsmoeError(code, lib.dsmoe_last_error().decode(errors="replace"))


def call(name: str, *args) -> None:
    check(getattr(lib, name)(*args))


def ptr(t) -> int:
    """Device (or host) address of a tensor's first element; None -> NULL."""
    return None if t is None else t.data_ptr()


def stream_of(t=None) -> int:
    import torch
    dev = t.device if t is not None else torch.device("cuda")
    return torch.cuda.current_stream(dev).cuda_stream
