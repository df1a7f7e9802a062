"""Seeded synthetic lfm2moe layers and inputs (host side).

Every tensor is a pure function of (seed, element index): see
``csrc/lfm_synth_core.h``.  The device generator (``lfm_gpu_moe_synth_*`` in
the CUDA library) evaluates the same arithmetic, so a layer filled on the GPU
is byte-identical to one built here.

The benchmark configurations (shapes, distributions, seeds) are the five of the
lfm2moe MoE-FFN metric: a single layer at T=1 / T=8 / T=2048 (skewed routing),
the LFM2-8B-A1B-shaped stack and the 24B-A2B-scale stack.
"""
from __future__ import annotations

import ctypes
import dataclasses
import hashlib
import os
from typing import Optional

import numpy as np

from . import _native

Q4K_BYTES = 144
Q6K_BYTES = 210
GGML_Q4_K = 12  # GGUF tensor type ids (ggml_type)
GGML_Q6_K = 14
Q8K_BYTES = 292
QK = 256

# One fixed seed per tensor kind; a layer index is mixed in with a multiply so
# layers of a stack get independent streams.
SEED_X = 0x1F3D_5A79_0000_0001
SEED_ROUTER = 0x1F3D_5A79_0000_0002
SEED_BIAS = 0x1F3D_5A79_0000_0003
SEED_GATE = 0x1F3D_5A79_0000_0004
SEED_UP = 0x1F3D_5A79_0000_0005
SEED_DOWN = 0x1F3D_5A79_0000_0006
SEED_DENSE_GATE = 0x1F3D_5A79_0000_0007
SEED_DENSE_UP = 0x1F3D_5A79_0000_0008
SEED_DENSE_DOWN = 0x1F3D_5A79_0000_0009
LAYER_STRIDE = 0x9E37_79B9


def layer_seed(base: int, layer: int) -> int:
    return (base + layer * LAYER_STRIDE) & 0xFFFF_FFFF_FFFF_FFFF


_gen = None  # a generator library chosen by use_generator_library()


def use_generator_library(path: str) -> None:
    """Generate with the build of csrc/lfm_synth.c at `path` instead of the package's own
    liblfm_synth.so (the bench's CPU reference arm uses the oracle's build, so that it maps
    no library of the GPU package).  Both builds compute the same bytes."""
    global _gen
    _gen = _native.bind_synth(ctypes.CDLL(path))


def _lib():
    return _gen if _gen is not None else _native.load_synth()


def normal_f32(n: int, seed: int, first: int = 0, mean: float = 0.0, std: float = 1.0,
               threads: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    _lib().lfm_synth_fill_normal_f32(out.ctypes.data_as(ctypes.c_void_p), ctypes.c_uint64(n),
                                     ctypes.c_uint64(first), ctypes.c_uint64(seed),
                                     ctypes.c_float(mean), ctypes.c_float(std),
                                     ctypes.c_int(threads or os.cpu_count() or 1))
    return out


def q4k_normal(n_blocks: int, seed: int, std: float, first_block: int = 0, threads: int = 0) -> np.ndarray:
    """Q4_K blocks [first_block, first_block+n_blocks) of an N(0, std) tensor, as uint8 bytes."""
    out = np.empty(n_blocks * Q4K_BYTES, dtype=np.uint8)
    _lib().lfm_synth_fill_q4k_normal(out.ctypes.data_as(ctypes.c_void_p), ctypes.c_uint64(n_blocks),
                                     ctypes.c_uint64(first_block), ctypes.c_uint64(seed),
                                     ctypes.c_float(std), ctypes.c_int(threads or os.cpu_count() or 1))
    return out


def quantize_q4k(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    if x.size % QK:
        raise ValueError("Q4_K quantisation needs a multiple of 256 values")
    out = np.empty(x.size // QK * Q4K_BYTES, dtype=np.uint8)
    _lib().lfm_synth_quantize_q4k(x.ctypes.data_as(ctypes.c_void_p), out.ctypes.data_as(ctypes.c_void_p),
                                  ctypes.c_uint64(x.size))
    return out


def dequantize_q4k(blocks: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(blocks, dtype=np.uint8).ravel()
    nb = b.size // Q4K_BYTES
    out = np.empty(nb * QK, dtype=np.float32)
    _lib().lfm_synth_dequantize_q4k(b.ctypes.data_as(ctypes.c_void_p), out.ctypes.data_as(ctypes.c_void_p),
                                    ctypes.c_uint64(nb))
    return out


def quantize_q6k(x: np.ndarray) -> np.ndarray:
    """fp32 -> GGUF Q6_K blocks (210 bytes per 256 values), our own quantiser.

    Per 16-value sub-block the scale is amax/31 (so codes q = rint(x/scale) lie in
    [-32, 31]); the super-block d = max scale / 127 is stored as fp16 and each
    sub-block keeps the int8 sc = rint(scale/d).  Codes are stored as q + 32 in
    the GGUF bit layout: value i (half = i/128, m = (i/32)%4, l = i%32) keeps its
    low nibble in ql[64*half + 32*(m%2) + l] (high nibble when m >= 2) and its top
    two bits at bits 2m..2m+1 of qh[32*half + l]; then int8 scales[16], fp16 d.
    """
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    if x.size % QK:
        raise ValueError("Q6_K quantisation needs a multiple of 256 values")
    step = 1 << 24  # values per piece: bounds the float64 temporaries
    if x.size > step:
        return np.concatenate([quantize_q6k(x[i:i + step]) for i in range(0, x.size, step)])
    nb = x.size // QK
    v = x.reshape(nb, 16, 16).astype(np.float64)
    scale = np.abs(v).max(axis=2) / 31.0                       # [nb, 16]
    d = (scale.max(axis=1) / 127.0).astype(np.float16)         # [nb]
    d32 = d.astype(np.float64)
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d32[:, None] > 0, np.rint(scale / d32[:, None]), 0.0)
    sc = np.clip(sc, -128, 127).astype(np.int8)
    eff = d32[:, None] * sc.astype(np.float64)                 # effective sub-block scale
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(eff[:, :, None] > 0, np.rint(v / eff[:, :, None]), 0.0)
    u = (np.clip(q, -32, 31) + 32).astype(np.uint8).reshape(nb, 2, 4, 32)  # [b, half, m, l]
    ql = np.empty((nb, 2, 64), np.uint8)
    ql[:, :, :32] = (u[:, :, 0] & 15) | ((u[:, :, 2] & 15) << 4)
    ql[:, :, 32:] = (u[:, :, 1] & 15) | ((u[:, :, 3] & 15) << 4)
    qh = (u[:, :, 0] >> 4) | ((u[:, :, 1] >> 4) << 2) | ((u[:, :, 2] >> 4) << 4) | ((u[:, :, 3] >> 4) << 6)
    out = np.empty((nb, Q6K_BYTES), np.uint8)
    out[:, :128] = ql.reshape(nb, 128)
    out[:, 128:192] = qh.reshape(nb, 64)
    out[:, 192:208] = sc.view(np.uint8)
    out[:, 208:210] = d.reshape(nb, 1).view(np.uint8)
    return out.ravel()


def dequantize_q6k(blocks: np.ndarray) -> np.ndarray:
    """GGUF Q6_K blocks -> fp32: d * sc[i/16] * (q_i - 32)."""
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1, Q6K_BYTES)
    nb = b.shape[0]
    ql = b[:, :128].reshape(nb, 2, 64)
    qh = b[:, 128:192].reshape(nb, 2, 32)
    sc = b[:, 192:208].copy().view(np.int8).astype(np.float32)
    d = b[:, 208:210].copy().view(np.float16).astype(np.float32).reshape(nb)
    u = np.empty((nb, 2, 4, 32), np.int32)
    u[:, :, 0] = (ql[:, :, :32] & 15) | ((qh & 3) << 4)
    u[:, :, 1] = (ql[:, :, 32:] & 15) | (((qh >> 2) & 3) << 4)
    u[:, :, 2] = (ql[:, :, :32] >> 4) | (((qh >> 4) & 3) << 4)
    u[:, :, 3] = (ql[:, :, 32:] >> 4) | (((qh >> 6) & 3) << 4)
    q = (u.reshape(nb, 256) - 32).astype(np.float32)
    return (d[:, None] * np.repeat(sc, 16, axis=1) * q).ravel()


@dataclasses.dataclass
class MoELayer:
    """Host copy of one lfm2moe layer, in GGUF layout.

    gate/up: Q4_K [E][I][D/256] blocks; down: [E][D][I/256] blocks of Q4_K
    (down_type 12) or Q6_K (down_type 14);
    router_w: fp32 [E, D]; bias (exp_probs_b): fp32 [E] or None; ffn_norm: fp32 [D].
    """
    D: int
    E: int
    K: int
    I: int
    ffn_norm: np.ndarray
    router_w: np.ndarray
    bias: Optional[np.ndarray]
    gate: np.ndarray
    up: np.ndarray
    down: np.ndarray
    eps: float = 1e-5
    norm_topk_prob: bool = True
    routed_scale: float = 1.0
    down_type: int = GGML_Q4_K

    def digest(self) -> str:
        h = hashlib.sha256()
        for a in (self.ffn_norm, self.router_w, self.bias, self.gate, self.up, self.down):
            if a is not None:
                h.update(np.ascontiguousarray(a).tobytes())
        return h.hexdigest()


@dataclasses.dataclass
class DenseLayer:
    """Host copy of a dense SwiGLU FFN layer: Q4_K gate/up [I][D/256], down [D][I/256]."""
    D: int
    I: int
    ffn_norm: np.ndarray
    gate: np.ndarray
    up: np.ndarray
    down: np.ndarray
    eps: float = 1e-5


def make_moe_layer(D: int, E: int, K: int, I: int, layer: int = 0, w_std: float = 0.02,
                   router_std: float = 0.02, bias_std: float = 0.1, bias: Optional[np.ndarray] = None,
                   threads: int = 0, down_type: int = GGML_Q4_K) -> MoELayer:
    """A synthetic lfm2moe layer: expert weights N(0, w_std) -> Q4_K (down: Q6_K when
    down_type is 14), router N(0, router_std), exp_probs_b N(0, bias_std) (or the given
    bias), ffn_norm = 1 (as the reference's MoE bench)."""
    if D % QK or I % QK:
        raise ValueError("D and I must be multiples of 256")
    if down_type not in (GGML_Q4_K, GGML_Q6_K):
        raise ValueError(f"down_type {down_type}: only Q4_K (12) and Q6_K (14)")
    gate = q4k_normal(E * I * D // QK, layer_seed(SEED_GATE, layer), w_std, threads=threads)
    up = q4k_normal(E * I * D // QK, layer_seed(SEED_UP, layer), w_std, threads=threads)
    if down_type == GGML_Q6_K:
        down = quantize_q6k(normal_f32(E * D * I, layer_seed(SEED_DOWN, layer), std=w_std, threads=threads))
    else:
        down = q4k_normal(E * D * I // QK, layer_seed(SEED_DOWN, layer), w_std, threads=threads)
    router = normal_f32(E * D, layer_seed(SEED_ROUTER, layer), std=router_std, threads=threads).reshape(E, D)
    if bias is None:
        bias = normal_f32(E, layer_seed(SEED_BIAS, layer), std=bias_std)
    return MoELayer(D=D, E=E, K=K, I=I, ffn_norm=np.ones(D, np.float32), router_w=router,
                    bias=np.ascontiguousarray(bias, dtype=np.float32), gate=gate, up=up, down=down,
                    down_type=down_type)


def make_dense_layer(D: int, I: int, layer: int = 0, w_std: float = 0.02, threads: int = 0) -> DenseLayer:
    gate = q4k_normal(I * D // QK, layer_seed(SEED_DENSE_GATE, layer), w_std, threads=threads)
    up = q4k_normal(I * D // QK, layer_seed(SEED_DENSE_UP, layer), w_std, threads=threads)
    down = q4k_normal(D * I // QK, layer_seed(SEED_DENSE_DOWN, layer), w_std, threads=threads)
    return DenseLayer(D=D, I=I, ffn_norm=np.ones(D, np.float32), gate=gate, up=up, down=down)


def make_hidden(T: int, D: int, seed_offset: int = 0) -> np.ndarray:
    """T rows of N(0,1) hidden states (row t uses normals [(t+off)*D, (t+off+1)*D))."""
    return normal_f32(T * D, SEED_X, first=seed_offset * D).reshape(T, D)


def zipf_bias(layer: MoELayer, s: float = 1.1, calib_tokens: int = 512, iters: int = 60,
              seed_offset: int = 1 << 20) -> np.ndarray:
    """exp_probs_b chosen so that expert popularity under top-K routing follows
    Zipf(s) over the E experts (rank r gets a share proportional to r^-s, capped
    at one selection per token).  Calibrated on `calib_tokens` seeded hidden
    rows by a fixed number of multiplicative updates in float64; deterministic.
    """
    E, K = layer.E, layer.K
    x = make_hidden(calib_tokens, layer.D, seed_offset=seed_offset).astype(np.float64)
    xb = x / np.sqrt((x * x).mean(axis=1, keepdims=True) + layer.eps)
    z = xb @ layer.router_w.astype(np.float64).T
    sig = 1.0 / (1.0 + np.exp(-z))
    target = np.arange(1, E + 1, dtype=np.float64) ** (-s)
    target = target / target.sum() * K
    target = np.minimum(target, 1.0)
    target = target / target.sum() * K
    b = np.zeros(E)
    for _ in range(iters):
        sel = sig + b
        top = np.argpartition(-sel, K - 1, axis=1)[:, :K]
        counts = np.bincount(top.ravel(), minlength=E) / calib_tokens
        b += 0.05 * (np.log(target + 1e-9) - np.log(counts + 1e-3))
    return b.astype(np.float32)


# ---------------------------------------------------------------------------
# The five benchmark configurations of the MoE-FFN metric.
# ---------------------------------------------------------------------------
CONFIGS = {
    1: dict(name="lfm2moe-layer-decode-T1", D=2048, E=32, K=4, I=1792, T=1, layers=1, dense=0),
    2: dict(name="lfm2moe-layer-verify-T8", D=2048, E=32, K=4, I=1792, T=8, layers=1, dense=0),
    3: dict(name="lfm2moe-layer-prefill-T2048-zipf1.1", D=2048, E=32, K=4, I=1792, T=2048, layers=1,
            dense=0, zipf=1.1),
    4: dict(name="lfm2-8b-a1b-stack-decode-64seq", D=2048, E=32, K=4, I=1792, T=64, layers=22, dense=2,
            dense_I=7168),
    5: dict(name="lfm2-24b-a2b-scale-stack-prefill-T4096", D=2048, E=64, K=4, I=1536, T=4096, layers=38,
            dense=0),
}
