"""ctypes bindings of the in-tree native libraries.

The CUDA library is the only compute path: if it is missing or fails to load,
every GPU entry point raises; nothing falls back to the CPU.
"""
from __future__ import annotations

import ctypes
import os
import re
import threading

from . import build as _build

_lock = threading.Lock()
_gpu = None
_synth = None

c_u32, c_i32, c_u64, c_f32, c_vp, c_int = (ctypes.c_uint32, ctypes.c_int32, ctypes.c_uint64, ctypes.c_float,
                                           ctypes.c_void_p, ctypes.c_int)


class Stats(ctypes.Structure):
    _fields_ = [("kernels_launched", c_u32), ("tokens", c_u32), ("unique_experts", c_u32),
                ("max_segment", c_u32), ("expert_loads", c_u64), ("layer_runs", c_u64)]


class GgufBlock(ctypes.Structure):
    _fields_ = [("kind", c_u32), ("D", c_u32), ("E", c_u32), ("K", c_u32), ("I", c_u32), ("eps", c_f32),
                ("has_bias", c_int), ("has_norm", c_int), ("down_type", c_u32)]


class KernelTime(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 32), ("launches", c_u32), ("total_ms", ctypes.c_double)]


# (name, restype, argtypes) for every entry point of include/lfm_gpu_moe.h
GPU_API = [
    ("lfm_gpu_moe_create", c_int, [ctypes.POINTER(c_vp), c_int]),
    ("lfm_gpu_moe_destroy", None, [c_vp]),
    ("lfm_gpu_moe_last_error", ctypes.c_char_p, [c_vp]),
    ("lfm_gpu_moe_upload_layer", c_int, [c_vp, c_u32, c_u32, c_u32, c_u32, c_u32, c_f32, c_vp, c_vp, c_vp, c_vp,
                                         c_vp, c_vp, c_u32, c_int, c_f32]),
    ("lfm_gpu_moe_upload_layer_typed", c_int, [c_vp, c_u32, c_u32, c_u32, c_u32, c_u32, c_f32, c_vp, c_vp, c_vp,
                                               c_vp, c_vp, c_vp, c_u32, c_u32, c_int, c_f32]),
    ("lfm_gpu_moe_upload_dense", c_int, [c_vp, c_u32, c_u32, c_u32, c_f32, c_vp, c_vp, c_vp, c_vp, c_u32]),
    ("lfm_gpu_moe_synth_layer", c_int, [c_vp, c_u32, c_u32, c_u32, c_u32, c_u32, c_f32, ctypes.POINTER(c_u64),
                                        c_f32, c_f32, c_f32, c_vp]),
    ("lfm_gpu_moe_upload_layer_shard", c_int, [c_vp, c_u32, c_u32, c_u32, c_u32, c_u32, c_f32, c_vp, c_vp, c_vp,
                                               c_vp, c_vp, c_vp, c_u32, c_int, c_f32, c_u32, c_u32]),
    ("lfm_gpu_moe_synth_layer_shard", c_int, [c_vp, c_u32, c_u32, c_u32, c_u32, c_u32, c_f32,
                                              ctypes.POINTER(c_u64), c_f32, c_f32, c_f32, c_vp, c_u32, c_u32]),
    ("lfm_gpu_moe_ep_route", c_int, [c_vp, c_u32, c_vp, c_u32, c_vp, c_vp, c_vp, c_vp]),
    ("lfm_gpu_moe_ep_experts", c_int, [c_vp, c_u32, c_vp, c_u32, c_vp, c_vp, c_vp]),
    ("lfm_gpu_moe_ep_combine", c_int, [c_vp, c_u32, c_vp, c_u32, c_vp, c_vp, c_vp]),
    ("lfm_gpu_moe_ep_p2p_attach", c_int, [c_vp, c_int, c_int, c_u32, c_u32, c_u32, c_u32, c_u32, c_u32, c_vp]),
    ("lfm_gpu_moe_ep_p2p_connect", c_int, [c_vp, c_vp]),
    ("lfm_gpu_moe_ep_p2p_forward", c_int, [c_vp, c_u32, c_vp, c_u32, c_vp]),
    ("lfm_gpu_moe_ep_p2p_forward_stack", c_int, [c_vp, c_u32, c_u32, c_vp, c_u32, c_vp]),
    ("lfm_gpu_moe_ep_p2p_wait_check", c_int, [c_vp, c_vp]),
    ("lfm_gpu_moe_ep_p2p_detach", c_int, [c_vp]),
    ("lfm_gpu_moe_gguf_describe", c_int, [ctypes.c_char_p, c_u32, c_vp, ctypes.POINTER(c_u32)]),
    ("lfm_gpu_moe_gguf_last_error", ctypes.c_char_p, []),
    ("lfm_gpu_moe_upload_gguf", c_int, [c_vp, ctypes.c_char_p, c_u32, c_u32, c_u32, c_u32, ctypes.POINTER(c_u32)]),
    ("lfm_gpu_moe_reserve", c_int, [c_vp, c_u32]),
    ("lfm_gpu_moe_forward", c_int, [c_vp, c_u32, c_vp, c_u32, c_int, c_vp]),
    ("lfm_gpu_moe_forward_stack", c_int, [c_vp, c_u32, c_u32, c_vp, c_u32, c_int, c_vp]),
    ("lfm_gpu_moe_forward_noalloc", c_int, [c_vp, c_u32, c_vp, c_u32, c_vp]),
    ("lfm_gpu_moe_debug_route", c_int, [c_vp, c_u32, c_vp, c_u32, c_vp, c_vp, c_vp]),
    ("lfm_gpu_moe_debug_q4k_rows", c_int, [c_vp, c_vp, c_u32, c_u32, c_vp, c_u32, c_vp, c_vp, c_vp, c_vp]),
    ("lfm_gpu_moe_debug_read_layer", c_int, [c_vp, c_u32, c_u32, c_vp, ctypes.c_size_t]),
    ("lfm_gpu_moe_debug_read_layer_range", c_int, [c_vp, c_u32, c_u32, ctypes.c_size_t, c_vp, ctypes.c_size_t]),
    ("lfm_gpu_moe_sync", c_int, [c_vp]),
    ("lfm_gpu_moe_last_stats", c_int, [c_vp, ctypes.POINTER(Stats)]),
    ("lfm_gpu_moe_profile", c_int, [c_vp, c_int]),
    ("lfm_gpu_moe_profile_read", c_int, [c_vp, ctypes.POINTER(KernelTime), c_u32, ctypes.POINTER(c_u32)]),
]

SYNTH_API = [
    ("lfm_synth_u64", c_u64, [c_u64, c_u64]),
    ("lfm_synth_normal", ctypes.c_double, [c_u64, c_u64]),
    ("lfm_synth_log", ctypes.c_double, [ctypes.c_double]),
    ("lfm_synth_float_to_half", ctypes.c_uint16, [c_f32]),
    ("lfm_synth_half_to_float", c_f32, [ctypes.c_uint16]),
    ("lfm_synth_fill_normal_f32", None, [c_vp, c_u64, c_u64, c_u64, c_f32, c_f32, c_int]),
    ("lfm_synth_fill_q4k_normal", None, [c_vp, c_u64, c_u64, c_u64, c_f32, c_int]),
    ("lfm_synth_quantize_q4k", c_int, [c_vp, c_vp, c_u64]),
    ("lfm_synth_dequantize_q4k", None, [c_vp, c_vp, c_u64]),
]


def header_functions() -> list:
    """Names of the functions include/lfm_gpu_moe.h declares."""
    path = os.path.join(_build.ROOT, "include", "lfm_gpu_moe.h")
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(lfm_gpu_moe_\w+)\s*\(", text)))


def _bind(lib, api):
    for name, res, args in api:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def load_gpu(build_if_missing: bool = True):
    """The CUDA library.  Raises if it cannot be built or loaded."""
    global _gpu
    with _lock:
        if _gpu is None:
            if build_if_missing:
                _build.build_gpu()
            if not os.path.exists(_build.GPU_SO):
                raise RuntimeError(f"CUDA library missing: {_build.GPU_SO} (run python -m laii_b200.build)")
            _gpu = _bind(ctypes.CDLL(_build.GPU_SO), GPU_API)
        return _gpu


def bind_synth(lib):
    """Bind the generator entry points on an already loaded build of csrc/lfm_synth.c."""
    return _bind(lib, SYNTH_API)


def load_synth(build_if_missing: bool = True):
    global _synth
    with _lock:
        if _synth is None:
            if build_if_missing:
                _build.build_synth()
            _synth = _bind(ctypes.CDLL(_build.SYNTH_SO), SYNTH_API)
        return _synth
