"""Python host API over the C-ABI of liblfm_gpu_moe.so (include/lfm_gpu_moe.h).

Mirrors the reference's MoE-FFN boundary: ``forward(layer, x)`` is
``lfm2_forward_moe_ffn_1x4`` (tools/lfm2_moe_checkpoint.c:312) batched over
the rows of x -- x is updated in place, x += MoE(x) -- and ``upload_layer``
takes the tensors ``lfm2_bind_moe_layer`` binds (:70-102) in GGUF layout.
Errors come back as ``MoEError`` carrying the library's status code; there is
no CPU fallback.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import numpy as np

from . import _native
from .synth import DenseLayer, MoELayer, Q8K_BYTES

GGML_TYPE_Q4_K = 12
GGML_TYPE_Q6_K = 14

STATUS = {0: "OK", -1: "INVALID_ARG", -2: "UNSUPPORTED", -3: "NOT_READY", -4: "OOM", -7: "CUDA", -8: "COMM",
          -9: "TIMEOUT", -10: "DEVICE_CHECK"}


class MoEError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"lfm_gpu_moe status {status} ({STATUS.get(status, '?')}): {message}")
        self.status = status


def _ptr(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def gguf_describe(path: str, block: int) -> Tuple[dict, int]:
    """The FFN of GGUF block `block` as the library binds it, and the file's block count (no GPU needed)."""
    lib = _native.load_gpu()
    out = _native.GgufBlock()
    n = ctypes.c_uint32()
    st = lib.lfm_gpu_moe_gguf_describe(str(path).encode(), block, ctypes.byref(out), ctypes.byref(n))
    if st != 0:
        raise MoEError(st, lib.lfm_gpu_moe_gguf_last_error().decode(errors="replace"))
    kind = {0: "none", 1: "dense", 2: "moe"}[out.kind]
    return ({"kind": kind, "D": out.D, "E": out.E, "K": out.K, "I": out.I, "eps": out.eps,
             "has_bias": bool(out.has_bias), "has_norm": bool(out.has_norm), "down_type": out.down_type}, n.value)


class GpuMoE:
    """One handle on one CUDA device (owns weights and scratch in HBM)."""

    def __init__(self, device: int = 0):
        self._lib = _native.load_gpu()
        h = ctypes.c_void_p()
        st = self._lib.lfm_gpu_moe_create(ctypes.byref(h), device)
        if st != 0:
            raise MoEError(st, f"cannot create a handle on device {device}")
        self._h = h
        self.device = device
        self.layers = {}

    # -- lifecycle -------------------------------------------------------
    def close(self):
        if getattr(self, "_h", None):
            self._lib.lfm_gpu_moe_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, st: int):
        if st != 0:
            raise MoEError(st, self._lib.lfm_gpu_moe_last_error(self._h).decode(errors="replace"))

    # -- weights ---------------------------------------------------------
    def upload_layer(self, layer: int, L: MoELayer):
        """Copy L into HBM; a layer whose down tensor is Q6_K (L.down_type 14) goes through
        lfm_gpu_moe_upload_layer_typed."""
        keep = [np.ascontiguousarray(a) for a in (L.ffn_norm, L.router_w, L.gate, L.up, L.down)]
        bias = None if L.bias is None else np.ascontiguousarray(L.bias, dtype=np.float32)
        down_type = int(getattr(L, "down_type", GGML_TYPE_Q4_K))
        if down_type == GGML_TYPE_Q4_K:
            self._check(self._lib.lfm_gpu_moe_upload_layer(
                self._h, layer, L.D, L.E, L.K, L.I, L.eps, _ptr(keep[0]), _ptr(keep[1]), _ptr(bias), _ptr(keep[2]),
                _ptr(keep[3]), _ptr(keep[4]), GGML_TYPE_Q4_K, int(L.norm_topk_prob), L.routed_scale))
        else:
            self._check(self._lib.lfm_gpu_moe_upload_layer_typed(
                self._h, layer, L.D, L.E, L.K, L.I, L.eps, _ptr(keep[0]), _ptr(keep[1]), _ptr(bias), _ptr(keep[2]),
                _ptr(keep[3]), _ptr(keep[4]), GGML_TYPE_Q4_K, down_type, int(L.norm_topk_prob), L.routed_scale))
        self.layers[layer] = ("moe", L.D, L.E, L.K, L.I)

    def upload_dense(self, layer: int, L: DenseLayer):
        keep = [np.ascontiguousarray(a) for a in (L.ffn_norm, L.gate, L.up, L.down)]
        self._check(self._lib.lfm_gpu_moe_upload_dense(self._h, layer, L.D, L.I, L.eps, *[_ptr(k) for k in keep],
                                                       GGML_TYPE_Q4_K))
        self.layers[layer] = ("dense", L.D, 0, 0, L.I)

    def synth_layer(self, layer: int, D: int, E: int, K: int, I: int, seeds, w_std=0.02, router_std=0.02,
                    bias_std=0.1, bias: Optional[np.ndarray] = None, eps: float = 1e-5):
        arr = (ctypes.c_uint64 * 5)(*[int(s) & 0xFFFFFFFFFFFFFFFF for s in seeds])
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        self._check(self._lib.lfm_gpu_moe_synth_layer(self._h, layer, D, E, K, I, eps, arr, w_std, router_std,
                                                      bias_std, _ptr(b)))
        self.layers[layer] = ("moe", D, E, K, I)

    # -- expert parallelism (laii_b200.ep) --------------------------------
    def upload_layer_shard(self, layer: int, L: MoELayer, first: int, count: int):
        """Full router; only experts [first, first+count) of L's expert tensors."""
        per_gu = L.I * (L.D // 256) * 144
        per_dn = L.D * (L.I // 256) * 144
        g = np.ascontiguousarray(L.gate.reshape(-1)[first * per_gu:(first + count) * per_gu])
        u = np.ascontiguousarray(L.up.reshape(-1)[first * per_gu:(first + count) * per_gu])
        d = np.ascontiguousarray(L.down.reshape(-1)[first * per_dn:(first + count) * per_dn])
        keep = [np.ascontiguousarray(a) for a in (L.ffn_norm, L.router_w)]
        bias = None if L.bias is None else np.ascontiguousarray(L.bias, dtype=np.float32)
        self._check(self._lib.lfm_gpu_moe_upload_layer_shard(
            self._h, layer, L.D, L.E, L.K, L.I, L.eps, _ptr(keep[0]), _ptr(keep[1]), _ptr(bias), _ptr(g), _ptr(u),
            _ptr(d), GGML_TYPE_Q4_K, int(L.norm_topk_prob), L.routed_scale, first, count))
        self.layers[layer] = ("moe-shard", L.D, L.E, L.K, L.I)

    def synth_layer_shard(self, layer: int, D: int, E: int, K: int, I: int, seeds, first: int, count: int,
                          w_std=0.02, router_std=0.02, bias_std=0.1, bias: Optional[np.ndarray] = None,
                          eps: float = 1e-5):
        arr = (ctypes.c_uint64 * 5)(*[int(s) & 0xFFFFFFFFFFFFFFFF for s in seeds])
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        self._check(self._lib.lfm_gpu_moe_synth_layer_shard(self._h, layer, D, E, K, I, eps, arr, w_std, router_std,
                                                            bias_std, _ptr(b), first, count))
        self.layers[layer] = ("moe-shard", D, E, K, I)

    def ep_route(self, layer: int, x_ptr: int, T: int, idx_ptr: int, w_ptr: int, q8_ptr: int, stream: int = 0):
        self._check(self._lib.lfm_gpu_moe_ep_route(self._h, layer, ctypes.c_void_p(x_ptr), T, ctypes.c_void_p(idx_ptr),
                                                   ctypes.c_void_p(w_ptr), ctypes.c_void_p(q8_ptr),
                                                   ctypes.c_void_p(stream or None)))

    def ep_experts(self, layer: int, q8_ptr: int, n: int, ids_ptr: int, y_ptr: int, stream: int = 0):
        self._check(self._lib.lfm_gpu_moe_ep_experts(self._h, layer, ctypes.c_void_p(q8_ptr), n,
                                                     ctypes.c_void_p(ids_ptr), ctypes.c_void_p(y_ptr),
                                                     ctypes.c_void_p(stream or None)))

    def ep_combine(self, layer: int, x_ptr: int, T: int, w_ptr: int, y_ptr: int, stream: int = 0):
        self._check(self._lib.lfm_gpu_moe_ep_combine(self._h, layer, ctypes.c_void_p(x_ptr), T, ctypes.c_void_p(w_ptr),
                                                     ctypes.c_void_p(y_ptr), ctypes.c_void_p(stream or None)))

    # -- expert parallelism over peer memory (one process per GPU) --------
    IPC_HANDLE_BYTES = 128  # LFM_GPU_MOE_IPC_HANDLE_BYTES

    def ep_p2p_attach(self, rank: int, world: int, max_tokens: int, D: int, E: int, K: int, I: int,
                      wait_ms: int = 0) -> bytes:
        """Allocate this rank's exchange arena; returns its IPC handle for the other ranks."""
        buf = ctypes.create_string_buffer(self.IPC_HANDLE_BYTES)
        self._check(self._lib.lfm_gpu_moe_ep_p2p_attach(self._h, rank, world, max_tokens, D, E, K, I, wait_ms, buf))
        return buf.raw

    def ep_p2p_connect(self, handles) -> None:
        """Map the other ranks' arenas; handles[r] = rank r's attach result."""
        blob = b"".join(bytes(h) for h in handles)
        if len(blob) != self.IPC_HANDLE_BYTES * len(handles):
            raise ValueError("every IPC handle is %d bytes" % self.IPC_HANDLE_BYTES)
        buf = ctypes.create_string_buffer(blob, len(blob))
        self._check(self._lib.lfm_gpu_moe_ep_p2p_connect(self._h, buf))

    def ep_p2p_forward(self, layer: int, x_ptr: int, T: int, stream: int = 0):
        self._check(self._lib.lfm_gpu_moe_ep_p2p_forward(self._h, layer, ctypes.c_void_p(x_ptr or None), T,
                                                         ctypes.c_void_p(stream or None)))

    def ep_p2p_forward_stack(self, first: int, n: int, x_ptr: int, T: int, stream: int = 0):
        """Layers [first, first + n): MoE shards as peer-memory steps, dense layers whole (CUDA graph replay)."""
        self._check(self._lib.lfm_gpu_moe_ep_p2p_forward_stack(self._h, first, n, ctypes.c_void_p(x_ptr or None), T,
                                                               ctypes.c_void_p(stream or None)))

    def ep_p2p_wait_check(self, stream: int = 0):
        self._check(self._lib.lfm_gpu_moe_ep_p2p_wait_check(self._h, ctypes.c_void_p(stream or None)))

    def ep_p2p_detach(self):
        self._check(self._lib.lfm_gpu_moe_ep_p2p_detach(self._h))

    def upload_gguf(self, path: str, first_block: int = 0, n_blocks: int = 0, expert_first: int = 0,
                    n_local: int = 0) -> int:
        """Blocks [first_block, +n_blocks) of a GGUF checkpoint into layer slots 0, 1, ... (n_local > 0: that
        expert shard of every MoE block); returns the number of layers uploaded."""
        n = ctypes.c_uint32()
        st = self._lib.lfm_gpu_moe_upload_gguf(self._h, str(path).encode(), first_block, n_blocks, expert_first,
                                               n_local, ctypes.byref(n))
        if st != 0:
            raise MoEError(st, self._lib.lfm_gpu_moe_gguf_last_error().decode(errors="replace"))
        for i in range(n_blocks or n.value):
            self.layers[i] = ("gguf", first_block + i)
        return n.value

    def reserve(self, max_tokens: int):
        self._check(self._lib.lfm_gpu_moe_reserve(self._h, max_tokens))

    # -- compute ---------------------------------------------------------
    def forward(self, layer: int, x: np.ndarray) -> np.ndarray:
        """x[T, D] (host, fp32, C-contiguous) += MoE(x), in place; returns x."""
        if x.dtype != np.float32 or not x.flags.c_contiguous:
            raise ValueError("x must be a C-contiguous float32 array")
        T = x.shape[0] if x.ndim == 2 else 1
        self._check(self._lib.lfm_gpu_moe_forward(self._h, layer, _ptr(x), T, 0, None))
        return x

    def forward_stack(self, first: int, n: int, x: np.ndarray) -> np.ndarray:
        if x.dtype != np.float32 or not x.flags.c_contiguous:
            raise ValueError("x must be a C-contiguous float32 array")
        T = x.shape[0] if x.ndim == 2 else 1
        self._check(self._lib.lfm_gpu_moe_forward_stack(self._h, first, n, _ptr(x), T, 0, None))
        return x

    def forward_device(self, layer: int, x_dev_ptr: int, T: int, stream: int = 0, n_layers: int = 1):
        """Asynchronous forward on a device pointer (e.g. a torch tensor's data_ptr())."""
        self._check(self._lib.lfm_gpu_moe_forward_stack(self._h, layer, n_layers, ctypes.c_void_p(x_dev_ptr), T, 1,
                                                        ctypes.c_void_p(stream) if stream else None))

    def sync(self):
        self._check(self._lib.lfm_gpu_moe_sync(self._h))

    def debug_route(self, layer: int, x: np.ndarray) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
        x = np.ascontiguousarray(x, dtype=np.float32)
        T, D = x.shape
        K = self.layers[layer][3]
        idx = np.zeros((T, K), np.uint32)
        w = np.zeros((T, K), np.float32)
        q8 = np.zeros(T * (D // 256) * Q8K_BYTES, np.uint8)
        self._check(self._lib.lfm_gpu_moe_debug_route(self._h, layer, _ptr(x), T, _ptr(idx), _ptr(w), _ptr(q8)))
        return idx, w, q8

    def debug_q4k_rows(self, w: np.ndarray, n_rows: int, n_cols: int, xq: np.ndarray, n_vec: int):
        nb = n_cols // 256
        sub = np.zeros((n_vec, n_rows, nb, 8), np.int32)
        acc = np.zeros((n_vec, n_rows, nb), np.int32)
        mins = np.zeros((n_vec, n_rows, nb), np.int32)
        out = np.zeros((n_vec, n_rows), np.float32)
        w = np.ascontiguousarray(w, dtype=np.uint8)
        xq = np.ascontiguousarray(xq, dtype=np.uint8)
        self._check(self._lib.lfm_gpu_moe_debug_q4k_rows(self._h, _ptr(w), n_rows, n_cols, _ptr(xq), n_vec,
                                                         _ptr(sub), _ptr(acc), _ptr(mins), _ptr(out)))
        return sub, acc, mins, out

    TENSORS = ("ffn_norm", "router_w", "exp_probs_b", "gate", "up", "down")

    def read_layer(self, layer: int, which: str, nbytes: int, offset: int = 0, out: Optional[np.ndarray] = None
                   ) -> np.ndarray:
        """Bytes [offset, offset + nbytes) of one device tensor of an uploaded layer (see TENSORS),
        into `out` (a contiguous uint8 buffer of nbytes) when given."""
        if out is None:
            out = np.zeros(nbytes, np.uint8)
        self._check(self._lib.lfm_gpu_moe_debug_read_layer_range(self._h, layer, self.TENSORS.index(which), offset,
                                                                 _ptr(out), nbytes))
        return out

    def profile(self, enable: bool = True):
        self._check(self._lib.lfm_gpu_moe_profile(self._h, int(enable)))

    def profile_read(self) -> dict:
        """{kernel name: (launches, total ms)} since the last read; clears the records."""
        buf = (_native.KernelTime * 16)()
        n = ctypes.c_uint32()
        self._check(self._lib.lfm_gpu_moe_profile_read(self._h, buf, 16, ctypes.byref(n)))
        return {buf[i].name.decode(): (buf[i].launches, buf[i].total_ms) for i in range(min(n.value, 16))}

    def last_stats(self) -> dict:
        s = _native.Stats()
        self._check(self._lib.lfm_gpu_moe_last_stats(self._h, ctypes.byref(s)))
        return {f: getattr(s, f) for f, _ in _native.Stats._fields_}
