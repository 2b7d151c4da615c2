"""ctypes binding of libqi.so (include/qi.h).

The library is built in-tree by `python -m qweninfer_b200.csrc.build` (or
`__graft_entry__.build()`). There is no fallback: if the library is missing or the
GPU is not an sm_100 part, `lib()` raises.
"""

from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libqi.so"

QI_OK = 0
QI_ERR_ARG = 1001
QI_ERR_TIMEOUT = 1002
QI_ERR_DEVICE = 1003
QI_ERR_TOO_LARGE = 1004
QI_ERR_INDEX = 1005
# launch kinds of qi_forward_launch_times
LAUNCH_KINDS = ("embed", "qkv", "attention", "o_proj", "gate_up", "down", "head")

vp = C.c_void_p
i32 = C.c_int
i64 = C.c_longlong
f32 = C.c_float


class QiLayer(C.Structure):
    _fields_ = [("ln1", vp), ("w_qkv", vp), ("b_qkv", vp), ("w_o", vp), ("ln2", vp),
                ("w_gate_up", vp), ("w_down", vp)]


class QiModel(C.Structure):
    _fields_ = [("num_layers", i32), ("vocab", i32), ("max_seq", i32), ("eps", f32),
                ("embed", vp), ("norm", vp), ("rope_cos", vp), ("rope_sin", vp),
                ("layers", C.POINTER(QiLayer))]


class QiCache(C.Structure):
    _fields_ = [("k", vp), ("v", vp), ("cache_rows", i32), ("max_len", i32), ("page_table", vp),
                ("page_size", i32), ("pages_per_row", i32), ("n_pages", i32)]


class QiWorkspace(C.Structure):
    _fields_ = [("x", vp), ("q", vp), ("attn", vp), ("h", vp), ("attn_part", vp),
                ("attn_counters", vp), ("max_tokens", i32), ("max_splits", i32),
                ("split_keys", i32), ("err", vp), ("use_tc", i32), ("act_x", vp), ("act_attn", vp),
                ("act_h", vp), ("ss", vp), ("ss_ld", i32), ("tc_scratch", vp), ("tc_scratch_floats", i64),
                ("tc_counters", vp), ("tc_counters_len", i32), ("query_run", i32)]


# name -> (restype, argtypes), exactly the declarations of include/qi.h
SIGNATURES = {
    "qi_version": (i32, []),
    "qi_init": (i32, [i32]),
    "qi_tile_offset": (i64, [i32, i32, i32]),
    "qi_embed": (i32, [vp, i32, vp, i32, vp, vp, vp, vp]),
    "qi_qkv_rope_append": (i32, [vp, vp, f32, vp, vp, vp, vp, vp, vp, i32, vp, vp, i32, vp, vp, vp]),
    "qi_attention": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, i32, vp, vp, vp, vp, vp]),
    "qi_attention_noalloc": (i32, [vp, vp, vp, vp, vp, i32, i32, vp, vp, vp]),
    "qi_o_proj_residual": (i32, [vp, vp, i32, vp, vp, vp]),
    "qi_gate_up_swiglu": (i32, [vp, vp, f32, vp, i32, vp, vp, vp]),
    "qi_down_residual": (i32, [vp, vp, i32, vp, vp, vp]),
    "qi_lm_head_argmax": (i32, [vp, i64, vp, f32, vp, i32, i32, vp, i32, i64, vp, vp, vp]),
    "qi_rmsnorm": (i32, [vp, vp, f32, i32, vp, vp]),
    "qi_rope": (i32, [vp, i32, vp, i32, i32, i32, vp, vp, vp, vp]),
    "qi_move_rows": (i32, [vp, vp, i32, i32, i32, C.POINTER(i32), i32, vp]),
    "qi_forward": (i32, [C.POINTER(QiModel), C.POINTER(QiCache), C.POINTER(QiWorkspace), vp, vp, vp,
                         i32, i32, i32, i32, vp, i32, i64, vp, vp]),
    "qi_forward_launch_times": (i32, [C.POINTER(QiModel), C.POINTER(QiCache), C.POINTER(QiWorkspace), vp, vp, vp,
                                      i32, i32, i32, i32, vp, i32, i64, vp, vp, vp, vp, i32, vp]),
    "qi_act_tiles": (i32, [vp, vp, i32, i32, i32, vp, vp, i32, vp]),
    "qi_tc_linear": (i32, [vp, i32, i32, vp, i32, i32, vp, i32, f32, vp, i32, vp, i64, vp, i32, i32, vp, vp]),
    "qi_tc_gate_up_swiglu": (i32, [vp, vp, i32, i32, vp, i32, f32, vp, vp, i64, vp, i32, i32, vp, vp]),
}

_lock = threading.Lock()
_lib: C.CDLL | None = None
_inited: set[int] = set()


class QiError(RuntimeError):
    pass


def load_library(path: Path = LIB_PATH) -> C.CDLL:
    """Load libqi.so and declare every entry point (no GPU needed)."""
    if not path.exists():
        raise QiError(f"{path} is missing: build it with `python -m qweninfer_b200.csrc.build`")
    lib = C.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def lib() -> C.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            _lib = load_library()
    return _lib


def check(code: int, what: str) -> None:
    if code != QI_OK:
        names = {QI_ERR_ARG: "invalid argument", QI_ERR_TIMEOUT: "device wait timed out",
                 QI_ERR_DEVICE: "not an sm_100 (B200) device",
                 QI_ERR_TOO_LARGE: "size beyond the entry point's fixed capacity",
                 QI_ERR_INDEX: "a position or cache row outside the cache"}
        raise QiError(f"{what} failed: {names.get(code, f'CUDA error {code}')}")


_current = [-1]


def ensure_device(device: torch.device) -> None:
    """Make `device` the library's current device (its CUDA runtime keeps its own
    per-thread current device, separate from PyTorch's); raises unless it is a CUDA
    sm_100 device."""
    if device.type != "cuda":
        raise QiError(f"qweninfer_b200 runs on CUDA (sm_100) devices only, got {device}")
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if _current[0] == idx:
        return
    check(lib().qi_init(idx), "qi_init")
    _current[0] = idx
    _inited.add(idx)


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream
