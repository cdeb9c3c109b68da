"""ctypes binding of libmorph_b200.so (declared in include/morph_b200.h).

The library is the only compute path: if it is missing the import fails with
instructions to build it; there is no CPU or eager-PyTorch fallback.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmorph_b200.so")

MB_OK = 0
MB_ERR_ARG = 1
MB_ERR_ALIGN = 2
MB_ERR_CUDA = 3
MB_ERR_OVERFLOW_MIN_SCALE = 4
MB_ERR_NONFINITE = 5
MB_ERR_TIMEOUT = 6
# a statistics pass that gave up reports its nonfinite count as at least 2^40
# (mb_adamw.cu kTimeoutMark): the step is refused as a time-out
TIMEOUT_MARK = float(1 << 40)
MB_ERR_INDEX = 7
MB_ERR_UNREPRESENTABLE = 8
MB_ERR_TOO_LARGE = 9

MB_F32, MB_F16, MB_BF16, MB_NONE = 0, 1, 2, 3
MB_MUON_MAX_BATCH = 64

MB_FAULT_APPLY, MB_FAULT_STATS, MB_FAULT_GEMM = 1, 2, 4

MB_FIN_LOSS_SCALE = 1
MB_FIN_GATE = 2
MB_FIN_CLIP_TORCH = 4
MB_FIN_CLIP_DISK = 8

_p = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f = ctypes.c_float
_d = ctypes.c_double


class Segment(ctypes.Structure):
    _fields_ = [("w", _p), ("m", _p), ("v", _p), ("g", _p), ("out", _p), ("numel", _i64),
                ("tile_begin", _i64), ("clock", _i32), ("group", _i32)]


class Group(ctypes.Structure):
    _fields_ = [("lr", _d), ("cwd", _f), ("omb1", _f), ("beta2", _f), ("omb2", _f), ("eps", _f),
                ("table", _i32)]


class StepState(ctypes.Structure):
    _fields_ = [("sumsq", _d), ("nonfinite", _d), ("scale", _d), ("step_scale", _d),
                ("good_steps", _i64), ("growth_interval", _i64), ("max_scale", _d), ("norm", _d),
                ("clip_coef", _f), ("skip", _i32), ("status", _i32), ("steps_applied", _i32),
                ("steps_skipped", _i32), ("reserved", _i32 * 3)]


class FinalizeOpts(ctypes.Structure):
    _fields_ = [("flags", _i32), ("reserved", _i32), ("max_norm", _d), ("backoff", _d), ("growth", _d)]


class Plan(ctypes.Structure):
    _fields_ = [("segs", _p), ("groups", _p), ("bc", _p), ("clocks", _p), ("workspace", _p), ("state", _p),
                ("n_tiles", _i64), ("bc_len", _i64), ("n_segs", _i32), ("n_groups", _i32),
                ("grad_dtype", _i32), ("out_dtype", _i32)]


class MuonArgs(ctypes.Structure):
    _fields_ = [("beta_lerp", _f), ("nesterov", _f), ("ns_a", _f), ("ns_b", _f), ("ns_c", _f),
                ("ns_steps", _i32), ("shape_scale", _f), ("cwd", _f), ("neg_lr", _f), ("ns_dtype", _i32),
                ("skip", _p), ("max_sms", _i32)]


class HostScalars(ctypes.Structure):
    _fields_ = [(n, _f) for n in ("cwd", "omb1", "beta2", "omb2", "bc2s", "eps", "nss", "scale", "coef")]


assert ctypes.sizeof(Segment) == 64 and ctypes.sizeof(Group) == 32
assert ctypes.sizeof(StepState) == 96 and ctypes.sizeof(FinalizeOpts) == 32

# name -> (restype, argtypes); the C-ABI surface, checked against the header by tests.
SIGNATURES = {
    "mb_version": (ctypes.c_int, []),
    "mb_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "mb_segments_plan": (ctypes.c_int, [_p, _i32, ctypes.POINTER(_i64)]),
    "mb_workspace_bytes": (ctypes.c_size_t, [_i32]),
    "mb_step_state_init": (ctypes.c_int, [_p, _d, _i64]),
    "mb_grad_stats": (ctypes.c_int, [_p, _p, _p]),
    "mb_step_finalize": (ctypes.c_int, [_p, _p, _p]),
    "mb_adamw_apply": (ctypes.c_int, [_p, _p]),
    "mb_adamw_apply_tiles": (ctypes.c_int, [_p, _i64, _i64, _i32, _p]),
    "mb_adamw_step": (ctypes.c_int, [_p, _p, _p]),
    "mb_adamw_step_noalloc": (ctypes.c_int, [_p, _p, _p]),
    "mb_adamw_update": (ctypes.c_int, [_p, _p, _p, _p, _i32, _p, _i32, _i64, _p, _p]),
    "mb_sparse_rows_update": (ctypes.c_int, [_p, _p, _p, _i64, _i64, _p, _i64, _p, _i32, _p, _p, _p]),
    "mb_cast_f32": (ctypes.c_int, [_p, _p, _i32, _i64, _i32, _p, _p]),
    "mb_fp8_pack": (ctypes.c_int, [_p, _i64, _p, _p, _p]),
    "mb_fp8_unpack": (ctypes.c_int, [_p, _p, _i64, _p, _i32, _p]),
    "mb_offload_rows_step": (ctypes.c_int, [_p, _p, _p, _i64, _i64, _p, _i64, _p, _i32, _p, _p, _p, _i64, _p, _p,
                                            _p, _p]),
    "mb_stream_wait": (ctypes.c_int, [_p, _i64]),
    "mb_accumulate_workspace_bytes": (ctypes.c_size_t, []),
    "mb_grad_accumulate": (ctypes.c_int, [_p, _p, _i32, _i64, ctypes.c_float, _i32, _p, _p, _p]),
    "mb_export_f16": (ctypes.c_int, [_p, _i64, _p, _p, _p]),
    "mb_adamw_apply_tiles_peers": (ctypes.c_int, [_p, _i64, _i64, _i32, _p, _i32, _p]),
    "mb_ipc_alloc": (ctypes.c_int, [ctypes.c_size_t, _p, _p]),
    "mb_ipc_free": (ctypes.c_int, [_p]),
    "mb_ipc_open": (ctypes.c_int, [_p, _p]),
    "mb_ipc_close": (ctypes.c_int, [_p]),
    "mb_muon_workspace_bytes": (ctypes.c_size_t, [_i64, _i64]),
    "mb_muon_batch_workspace_bytes": (ctypes.c_size_t, [_i32, _i64, _i64]),
    "mb_newton_schulz": (ctypes.c_int, [_p, _i64, _i64, _i32, _p, _i32, _p, _p, ctypes.c_size_t, _p, _p]),
    "mb_muon_step": (ctypes.c_int, [_p, _p, _p, _i32, _p, _i32, _i64, _i64, _p, _p, ctypes.c_size_t, _p, _p]),
    "mb_muon_step_batched": (ctypes.c_int, [_p, _p, _p, _i32, _p, _i32, _i32, _i64, _i64, _p, _p, ctypes.c_size_t,
                                            _p, _p]),
    "mb_debug_arm_fault": (ctypes.c_int, [_i32, _i64, _i64]),
    "mb_gemm16": (ctypes.c_int, [_i32, _p, _i64, _p, _i64, _i64, _i64, _i64, _f, _f, _p, _i64, _p, _i64, _p, _i64,
                                 _p, _i64, _p, _p]),
}

_LIB = None


def lib() -> ctypes.CDLL:
    """Load the library once; raise ImportError if it has not been built."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m morph_b200.csrc.build` "
                              "(morph_b200 has no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def status_string(rc: int) -> str:
    return lib().mb_status_string(rc).decode()


def check(rc: int, what: str = "") -> None:
    """Map a C-ABI status to the reference's exception types."""
    if rc == MB_OK:
        return
    msg = status_string(rc) + (f" ({what})" if what else "")
    if rc in (MB_ERR_ARG, MB_ERR_ALIGN, MB_ERR_UNREPRESENTABLE, MB_ERR_TOO_LARGE):
        raise ValueError(msg)
    if rc in (MB_ERR_OVERFLOW_MIN_SCALE, MB_ERR_NONFINITE):
        raise FloatingPointError(msg)
    if rc == MB_ERR_INDEX:
        raise IndexError(msg)
    if rc == MB_ERR_TIMEOUT:
        raise TimeoutError(msg)
    raise RuntimeError(msg)


def dtype_code(dtype) -> int:
    import torch
    codes = {torch.float32: MB_F32, torch.float16: MB_F16, torch.bfloat16: MB_BF16}
    if dtype is None:
        return MB_NONE
    if dtype not in codes:
        raise ValueError(f"unsupported dtype {dtype}")
    return codes[dtype]


def stream_handle(stream=None) -> ctypes.c_void_p:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def ptr(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())
