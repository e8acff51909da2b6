"""ctypes binding of the C ABI declared in include/chronos_moe.h (and the
expert-parallel, lookahead and attention headers beside it).

The library is ``project_chronos_b200/libchronos_moe.so`` (built in-tree by
``project_chronos_b200.build``).  Loading fails loudly: there is no other
implementation of this layer to fall back to.
"""
from __future__ import annotations

import ctypes
import os
import threading

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libchronos_moe.so")

CHRONOS_OK = 0
CHRONOS_ERR_INVALID_ARG = 1
CHRONOS_ERR_WORKSPACE_TOO_SMALL = 2
CHRONOS_ERR_CUDA = 3
CHRONOS_ERR_EXPERT_NOT_READY = 4
CHRONOS_ERR_NCCL = 5
CHRONOS_ERR_PIPELINE_TIMEOUT = 6

ERROR_NAMES = {
    CHRONOS_ERR_INVALID_ARG: "CHRONOS_ERR_INVALID_ARG",
    CHRONOS_ERR_WORKSPACE_TOO_SMALL: "CHRONOS_ERR_WORKSPACE_TOO_SMALL",
    CHRONOS_ERR_CUDA: "CHRONOS_ERR_CUDA",
    CHRONOS_ERR_EXPERT_NOT_READY: "CHRONOS_ERR_EXPERT_NOT_READY",
    CHRONOS_ERR_NCCL: "CHRONOS_ERR_NCCL",
    CHRONOS_ERR_PIPELINE_TIMEOUT: "CHRONOS_ERR_PIPELINE_TIMEOUT",
}

DTYPE_BF16 = 0
DTYPE_FP16 = 1
DTYPE_FP32 = 2

FLAG_PREROUTED = 0x1
FLAG_AVAIL_MASK = 0x2
FLAG_ACC_OUT = 0x4

ABI_VERSION = 2

# Functions declared in include/chronos_moe.h (checked against the header by the tests).
EXPORTS = ("chronos_moe_workspace_size", "chronos_moe_forward", "chronos_moe_route",
           "chronos_moe_last_error", "chronos_moe_abi_version", "chronos_moe_args_size",
           "chronos_moe_profile_begin", "chronos_moe_profile_end",
           "chronos_moe_kernel_launches", "chronos_moe_forward_noalloc", "chronos_moe_set_option",
           "chronos_ep_dispatch", "chronos_ep_combine", "chronos_ep_dispatch_args_size",
           "chronos_ep_combine_args_size", "chronos_lookahead_forward", "chronos_lookahead_args_size",
           "chronos_mla_decode", "chronos_sw_decode", "chronos_add_rmsnorm", "chronos_attn_args_size",
           "chronos_norm_args_size", "chronos_argmax_rows")

EP_MAX_RANKS = 32  # CHRONOS_EP_MAX_RANKS

NOALLOC_SCRATCH_BYTES = 16 << 20  # CHRONOS_NOALLOC_SCRATCH_BYTES

STAGES = ("route", "plan", "scatter", "gateup", "act", "down", "finalize")


class ChronosMoeShape(ctypes.Structure):
    _fields_ = [
        ("num_tokens", ctypes.c_int64),
        ("hidden", ctypes.c_int32),
        ("num_experts", ctypes.c_int32),
        ("top_k", ctypes.c_int32),
        ("ffn", ctypes.c_int32),
        ("num_shared", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
    ]


class ChronosMoeArgs(ctypes.Structure):
    _fields_ = [
        ("shape", ChronosMoeShape),
        ("norm_topk", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("x", ctypes.c_void_p),
        ("router_w", ctypes.c_void_p),
        ("router_bias", ctypes.c_void_p),
        ("w_gate", ctypes.c_void_p),
        ("w_up", ctypes.c_void_p),
        ("w_down", ctypes.c_void_p),
        ("pool_slots", ctypes.c_int32),
        ("slot_of_expert", ctypes.c_void_p),
        ("w_shared_gate", ctypes.c_void_p),
        ("w_shared_up", ctypes.c_void_p),
        ("w_shared_down", ctypes.c_void_p),
        ("avail", ctypes.c_void_p),
        ("ready_flags", ctypes.c_void_p),
        ("ready_epoch", ctypes.c_int32),
        ("spin_limit_ns", ctypes.c_int64),
        ("y", ctypes.c_void_p),
        ("router_probs", ctypes.c_void_p),
        ("topk_idx", ctypes.c_void_p),
        ("topk_weight", ctypes.c_void_p),
        ("expert_counts", ctypes.c_void_p),
        ("expert_mass", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("status", ctypes.c_void_p),
        ("max_ctas", ctypes.c_int32),
    ]


class ChronosEpDispatchArgs(ctypes.Structure):
    """Mirror of include/chronos_ep.h ChronosEpDispatchArgs."""
    _fields_ = [
        ("num_tokens", ctypes.c_int64),
        ("hidden", ctypes.c_int32),
        ("num_experts", ctypes.c_int32),
        ("top_k", ctypes.c_int32),
        ("world_size", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("num_chunks", ctypes.c_int32),
        ("meta_pairs", ctypes.c_int32),
        ("x", ctypes.c_void_p),
        ("topk_idx", ctypes.c_void_p),
        ("topk_weight", ctypes.c_void_p),
        ("avail", ctypes.c_void_p),
        ("send_counts", ctypes.c_void_p),
        ("send_x", ctypes.c_void_p),
        ("send_meta", ctypes.c_void_p),
        ("pair_slot", ctypes.c_void_p),
        ("shared_weight", ctypes.c_void_p),
        ("scratch", ctypes.c_void_p),
        ("seg_rows", ctypes.c_int64),
    ]


class ChronosEpCombineArgs(ctypes.Structure):
    """Mirror of include/chronos_ep.h ChronosEpCombineArgs."""
    _fields_ = [
        ("num_tokens", ctypes.c_int64),
        ("hidden", ctypes.c_int32),
        ("top_k", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("y_shared", ctypes.c_void_p),
        ("recv_y", ctypes.c_void_p),
        ("pair_slot", ctypes.c_void_p),
        ("y", ctypes.c_void_p),
    ]


class ChronosLookaheadArgs(ctypes.Structure):
    """Mirror of include/chronos_lookahead.h ChronosLookaheadArgs."""
    _fields_ = [
        ("num_tokens", ctypes.c_int64),
        ("hidden", ctypes.c_int32),
        ("inner", ctypes.c_int32),
        ("num_experts", ctypes.c_int32),
        ("steps", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("x", ctypes.c_void_p),
        ("w1", ctypes.c_void_p),
        ("w2", ctypes.c_void_p),
        ("probs", ctypes.c_void_p),
    ]


class ChronosAttnArgs(ctypes.Structure):
    """include/chronos_attention.h"""
    _fields_ = [
        ("batch", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("rope_dim", ctypes.c_int32),
        ("latent", ctypes.c_int32),
        ("window", ctypes.c_int32),
        ("max_len", ctypes.c_int32),
        ("table_len", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("eps", ctypes.c_float),
        ("pos", ctypes.c_void_p),
        ("proj", ctypes.c_void_p),
        ("norm_q", ctypes.c_void_p),
        ("norm_q2", ctypes.c_void_p),
        ("norm_kv", ctypes.c_void_p),
        ("w_krope", ctypes.c_void_p),
        ("w_knope", ctypes.c_void_p),
        ("w_v", ctypes.c_void_p),
        ("cos", ctypes.c_void_p),
        ("sin", ctypes.c_void_p),
        ("cache_a", ctypes.c_void_p),
        ("cache_b", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
    ]


class ChronosNormArgs(ctypes.Structure):
    """include/chronos_attention.h"""
    _fields_ = [
        ("rows", ctypes.c_int64),
        ("width", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("eps", ctypes.c_float),
        ("x_fp32", ctypes.c_int32),
        ("x", ctypes.c_void_p),
        ("residual", ctypes.c_void_p),
        ("sum_out", ctypes.c_void_p),
        ("weight", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
    ]


_lib = None
_lock = threading.Lock()


class ChronosMoeError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{ERROR_NAMES.get(code, code)}: {message}")
        self.code = code


def load_library(path: str = LIB_PATH):
    """Load (once) and return the extension; raises if it is missing or stale."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(
                f"chronos MoE CUDA extension not found at {path}; build it with "
                "`python -m project_chronos_b200.build` (nvcc, sm_100a)")
        lib = ctypes.CDLL(path)
        lib.chronos_moe_workspace_size.argtypes = [ctypes.POINTER(ChronosMoeShape)]
        lib.chronos_moe_workspace_size.restype = ctypes.c_size_t
        lib.chronos_moe_forward.argtypes = [ctypes.POINTER(ChronosMoeArgs), ctypes.c_void_p]
        lib.chronos_moe_forward.restype = ctypes.c_int
        lib.chronos_moe_route.argtypes = [ctypes.POINTER(ChronosMoeArgs), ctypes.c_void_p]
        lib.chronos_moe_route.restype = ctypes.c_int
        lib.chronos_moe_last_error.argtypes = []
        lib.chronos_moe_last_error.restype = ctypes.c_char_p
        lib.chronos_moe_abi_version.argtypes = []
        lib.chronos_moe_abi_version.restype = ctypes.c_int
        lib.chronos_moe_args_size.argtypes = []
        lib.chronos_moe_args_size.restype = ctypes.c_size_t
        lib.chronos_moe_profile_begin.argtypes = [ctypes.c_int]
        lib.chronos_moe_profile_begin.restype = ctypes.c_int
        lib.chronos_moe_profile_end.argtypes = [ctypes.POINTER(ctypes.c_float),
                                                ctypes.POINTER(ctypes.c_int32), ctypes.c_int]
        lib.chronos_moe_profile_end.restype = ctypes.c_int
        lib.chronos_moe_kernel_launches.argtypes = []
        lib.chronos_moe_kernel_launches.restype = ctypes.c_uint64
        lib.chronos_moe_forward_noalloc.argtypes = [ctypes.POINTER(ChronosMoeArgs),
                                                    ctypes.c_void_p]
        lib.chronos_moe_forward_noalloc.restype = ctypes.c_int
        lib.chronos_moe_set_option.argtypes = [ctypes.c_char_p, ctypes.c_int64]
        lib.chronos_moe_set_option.restype = ctypes.c_int
        lib.chronos_ep_dispatch.argtypes = [ctypes.POINTER(ChronosEpDispatchArgs), ctypes.c_void_p]
        lib.chronos_ep_dispatch.restype = ctypes.c_int
        lib.chronos_ep_combine.argtypes = [ctypes.POINTER(ChronosEpCombineArgs), ctypes.c_void_p]
        lib.chronos_ep_combine.restype = ctypes.c_int
        lib.chronos_ep_dispatch_args_size.argtypes = []
        lib.chronos_ep_dispatch_args_size.restype = ctypes.c_size_t
        lib.chronos_ep_combine_args_size.argtypes = []
        lib.chronos_ep_combine_args_size.restype = ctypes.c_size_t
        lib.chronos_lookahead_forward.argtypes = [ctypes.POINTER(ChronosLookaheadArgs), ctypes.c_void_p]
        lib.chronos_lookahead_forward.restype = ctypes.c_int
        lib.chronos_lookahead_args_size.argtypes = []
        lib.chronos_lookahead_args_size.restype = ctypes.c_size_t
        for fn, st in (("chronos_mla_decode", ChronosAttnArgs), ("chronos_sw_decode", ChronosAttnArgs),
                       ("chronos_add_rmsnorm", ChronosNormArgs)):
            getattr(lib, fn).argtypes = [ctypes.POINTER(st), ctypes.c_void_p]
            getattr(lib, fn).restype = ctypes.c_int
        lib.chronos_argmax_rows.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                            ctypes.c_void_p, ctypes.c_void_p]
        lib.chronos_argmax_rows.restype = ctypes.c_int
        lib.chronos_attn_args_size.argtypes = []
        lib.chronos_attn_args_size.restype = ctypes.c_size_t
        lib.chronos_norm_args_size.argtypes = []
        lib.chronos_norm_args_size.restype = ctypes.c_size_t
        if (lib.chronos_attn_args_size() != ctypes.sizeof(ChronosAttnArgs)
                or lib.chronos_norm_args_size() != ctypes.sizeof(ChronosNormArgs)):
            raise RuntimeError("attention args layout mismatch between the library and the binding")
        if lib.chronos_lookahead_args_size() != ctypes.sizeof(ChronosLookaheadArgs):
            raise RuntimeError("lookahead args layout mismatch between the library and the binding")
        if (lib.chronos_ep_dispatch_args_size() != ctypes.sizeof(ChronosEpDispatchArgs)
                or lib.chronos_ep_combine_args_size() != ctypes.sizeof(ChronosEpCombineArgs)):
            raise RuntimeError("expert-parallel args layout mismatch between the library and the binding")
        if lib.chronos_moe_abi_version() != ABI_VERSION:
            raise RuntimeError("chronos MoE extension ABI version mismatch; rebuild it")
        if lib.chronos_moe_args_size() != ctypes.sizeof(ChronosMoeArgs):
            raise RuntimeError("ChronosMoeArgs layout mismatch between the library and the binding")
        _lib = lib
        return lib


def check(rc: int) -> None:
    if rc != CHRONOS_OK:
        msg = load_library().chronos_moe_last_error().decode(errors="replace")
        raise ChronosMoeError(rc, msg)
