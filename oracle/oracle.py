"""TEST INFRASTRUCTURE ONLY -- ctypes access to the CPU oracle.

  Oracle     our scalar restatement of the reference path (lfm_oracle.c)
  Reference  the reference's own CPU code built from its sources
             (oracle/_ref/libref_moe.so, see ref_harness.c); may be absent

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "liblfm_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libref_moe.so")
GEN_SO = os.path.join(HERE, "_build", "liblfm_gen.so")

ORDER_VNNI = 0
ORDER_AVX2 = 1

_vp, _u32, _f32, _int = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_float, ctypes.c_int


def build(ref_dir: Optional[str] = None) -> None:
    """Compile the oracle (and the reference harness when its sources exist)."""
    cmd = ["make", "-s", "-C", HERE]
    if ref_dir:
        cmd.append(f"REF={ref_dir}")
    subprocess.run(cmd, check=True)


def _p(a):
    return None if a is None else a.ctypes.data_as(_vp)


class Oracle:
    def __init__(self):
        if not os.path.exists(ORACLE_SO):
            build()
        lib = ctypes.CDLL(ORACLE_SO)
        lib.orc_dot_f32.restype = _f32
        lib.orc_dot_f32.argtypes = [_vp, _vp, _u32]
        lib.orc_quantize_q8k.argtypes = [_vp, _vp, _u32]
        lib.orc_rmsnorm_q8k.argtypes = [_vp, _vp, _u32, _f32, _vp, _vp]
        lib.orc_route.argtypes = [_vp, _vp, _vp, _u32, _u32, _u32, _int, _f32, _vp, _vp, _vp, _vp]
        lib.orc_q4k_rows.argtypes = [_int, _vp, _u32, _u32, _u32, _vp, _vp]
        lib.orc_q4k_row_ints.argtypes = [_vp, _vp, _u32, _vp, _vp, _vp]
        lib.orc_moe_forward.restype = _int
        lib.orc_q6k_rows.argtypes = [_int, _vp, _u32, _u32, _u32, _vp, _vp]
        lib.orc_q6k_row_ints.argtypes = [_vp, _vp, _u32, _vp, _vp, _vp]
        lib.orc_moe_forward.argtypes = [_int, _vp, _u32, _u32, _u32, _u32, _u32, _f32, _vp, _vp, _vp, _vp, _vp,
                                        _vp, _u32, _int, _f32, _vp, _vp, _vp, _vp]
        lib.orc_kat_router_inputs.argtypes = [_vp, _vp, _vp, _u32, _u32]
        lib.orc_kat_q8k_inputs.argtypes = [_vp, _u32]
        lib.orc_dense_ffn_forward.restype = _int
        lib.orc_dense_ffn_forward.argtypes = [_int, _vp, _u32, _u32, _u32, _f32, _vp, _vp, _vp, _vp]
        lib.orc_expert_rows.restype = _int
        lib.orc_expert_rows.argtypes = [_int, _u32, _u32, _vp, _vp, _vp, _vp, _vp, _u32, _vp]
        lib.orc_ep_combine.argtypes = [_vp, _u32, _u32, _u32, _vp, _vp]
        self.lib = lib

    def quantize_q8k(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32).ravel()
        out = np.zeros(x.size // 256 * 292, np.uint8)
        self.lib.orc_quantize_q8k(_p(x), _p(out), x.size)
        return out

    def kat_router_inputs(self, D=2048, E=32):
        """Inputs of the reference's router known-answer test (tests/test_moe_checkpoint.c:138-218)."""
        xb = np.zeros(D, np.float32)
        w = np.zeros((E, D), np.float32)
        b = np.zeros(E, np.float32)
        self.lib.orc_kat_router_inputs(_p(xb), _p(w), _p(b), D, E)
        return xb, w, b

    def kat_q8k_inputs(self, n=2048):
        """Input of the reference's Q8_K parity test (tests/test_cpuid_quants.c:69-111)."""
        x = np.zeros(n, np.float32)
        self.lib.orc_kat_q8k_inputs(_p(x), n)
        return x

    def rmsnorm_q8k(self, x: np.ndarray, norm_w: Optional[np.ndarray], eps: float):
        x = np.ascontiguousarray(x, np.float32)
        D = x.size
        xb = np.zeros(D, np.float32)
        xq = np.zeros(D // 256 * 292, np.uint8)
        nw = None if norm_w is None else np.ascontiguousarray(norm_w, np.float32)
        self.lib.orc_rmsnorm_q8k(_p(x), _p(nw), D, eps, _p(xb), _p(xq))
        return xb, xq

    def route(self, router_w, bias, xb, K, norm_topk=True, routed_scale=1.0):
        router_w = np.ascontiguousarray(router_w, np.float32)
        E, D = router_w.shape
        xb = np.ascontiguousarray(xb, np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        idx = np.zeros(K, np.uint32)
        w = np.zeros(K, np.float32)
        logits = np.zeros(E, np.float32)
        sel = np.zeros(E, np.float32)
        self.lib.orc_route(_p(router_w), _p(b), _p(xb), D, E, K, int(norm_topk), routed_scale, _p(idx), _p(w),
                           _p(logits), _p(sel))
        return idx, w, logits, sel

    def q4k_rows(self, W, n_cols, n_rows, xq, order=ORDER_VNNI, r0=0):
        out = np.zeros(n_rows, np.float32)
        self.lib.orc_q4k_rows(order, _p(np.ascontiguousarray(W)), n_cols, r0, n_rows,
                              _p(np.ascontiguousarray(xq)), _p(out))
        return out

    def q6k_rows(self, W, n_cols, n_rows, xq, order=ORDER_VNNI, r0=0):
        out = np.zeros(n_rows, np.float32)
        self.lib.orc_q6k_rows(order, _p(np.ascontiguousarray(W)), n_cols, r0, n_rows, _p(np.ascontiguousarray(xq)),
                              _p(out))
        return out

    def q6k_row_ints(self, row, xq, n_cols):
        """Per super-block (acc, off, total = acc - 32*off) of one Q6_K row against Q8_K xq."""
        nb = n_cols // 256
        acc, off, tot = (np.zeros(nb, np.int32) for _ in range(3))
        self.lib.orc_q6k_row_ints(_p(np.ascontiguousarray(row)), _p(np.ascontiguousarray(xq)), n_cols, _p(acc),
                                  _p(off), _p(tot))
        return acc, off, tot

    def q4k_row_ints(self, row, xq, n_cols):
        nb = n_cols // 256
        sub = np.zeros((nb, 8), np.int32)
        acc = np.zeros(nb, np.int32)
        mins = np.zeros(nb, np.int32)
        self.lib.orc_q4k_row_ints(_p(np.ascontiguousarray(row)), _p(np.ascontiguousarray(xq)), n_cols, _p(sub),
                                  _p(acc), _p(mins))
        return sub, acc, mins

    # -- expert-parallel pieces (host-logic tests of laii_b200.ep) ----------
    def ep_route(self, L, x: np.ndarray):
        """x[T, D] -> idx[T, K] (global ids), w[T, K], q8[T, D/256*292] (block_q8_K rows)."""
        T = x.shape[0]
        idx = np.zeros((T, L.K), np.int32)
        w = np.zeros((T, L.K), np.float32)
        q8 = np.zeros((T, L.D // 256 * 292), np.uint8)
        for t in range(T):
            xb, q8[t] = self.rmsnorm_q8k(x[t], L.ffn_norm, L.eps)
            i, wt, _, _ = self.route(L.router_w, L.bias, xb, L.K, L.norm_topk_prob, L.routed_scale)
            idx[t], w[t] = i.astype(np.int32), wt
        return idx, w, q8

    def ep_expert_rows(self, L, first: int, count: int, q8: np.ndarray, ids: np.ndarray, order=ORDER_VNNI):
        """Rows of global experts ids (all in [first, first+count)) -> y[n, D], unweighted."""
        n = ids.shape[0]
        per_gu = L.I * (L.D // 256) * 144
        per_dn = L.D * (L.I // 256) * 144
        g = np.ascontiguousarray(L.gate.reshape(-1)[first * per_gu:(first + count) * per_gu])
        u = np.ascontiguousarray(L.up.reshape(-1)[first * per_gu:(first + count) * per_gu])
        dn = np.ascontiguousarray(L.down.reshape(-1)[first * per_dn:(first + count) * per_dn])
        local = np.ascontiguousarray(ids.astype(np.int64) - first, np.uint32)
        assert np.all((ids >= first) & (ids < first + count)), "row routed to a foreign expert"
        y = np.zeros((n, L.D), np.float32)
        if n:
            st = self.lib.orc_expert_rows(order, L.D, L.I, _p(g), _p(u), _p(dn), _p(np.ascontiguousarray(q8)),
                                          _p(local), n, _p(y))
            if st != 0:
                raise RuntimeError(f"oracle expert_rows status {st}")
        return y

    def ep_combine(self, x: np.ndarray, w: np.ndarray, y: np.ndarray):
        """x[T, D] in place: x[t] = fmaf(w[t, k], y[t*K + k], x[t]) for k in order."""
        T, D = x.shape
        K = w.shape[1]
        self.lib.orc_ep_combine(_p(x), T, D, K, _p(np.ascontiguousarray(w, np.float32)),
                                _p(np.ascontiguousarray(y, np.float32)))
        return x

    def moe_forward(self, L, x: np.ndarray, order=ORDER_VNNI, want_h=False):
        """x[T, D] -> (x_out, idx[T,K], w[T,K], xq bytes, h[T,K,I] or None); x is not modified."""
        x = np.array(x, np.float32, copy=True, order="C")
        T = x.shape[0]
        idx = np.zeros((T, L.K), np.uint32)
        w = np.zeros((T, L.K), np.float32)
        xq = np.zeros(T * (L.D // 256) * 292, np.uint8)
        h = np.zeros((T, L.K, L.I), np.float32) if want_h else None
        st = self.lib.orc_moe_forward(order, _p(x), T, L.D, L.E, L.K, L.I, L.eps, _p(L.ffn_norm), _p(L.router_w),
                                      _p(L.bias), _p(L.gate), _p(L.up), _p(L.down), int(getattr(L, "down_type", 12)),
                                      int(L.norm_topk_prob), L.routed_scale, _p(idx), _p(w), _p(xq), _p(h))
        if st != 0:
            raise RuntimeError(f"oracle moe_forward status {st}")
        return x, idx, w, xq, h

    def dense_forward(self, L, x: np.ndarray, order=ORDER_VNNI):
        x = np.array(x, np.float32, copy=True, order="C")
        st = self.lib.orc_dense_ffn_forward(order, _p(x), x.shape[0], L.D, L.I, L.eps, _p(L.ffn_norm), _p(L.gate),
                                            _p(L.up), _p(L.down))
        if st != 0:
            raise RuntimeError(f"oracle dense_forward status {st}")
        return x


class Reference:
    """The reference's own CPU lfm2moe path (tools/lfm2_moe_checkpoint.c), built from source."""

    def __init__(self, n_threads: int = 1):
        if not os.path.exists(REF_SO):
            raise FileNotFoundError(REF_SO)
        lib = ctypes.CDLL(REF_SO)
        lib.ref_init.restype = _int
        lib.ref_init.argtypes = [_int]
        lib.ref_isa_name.restype = ctypes.c_char_p
        lib.ref_cpu_brand.restype = ctypes.c_char_p
        lib.ref_quantize_q8k.argtypes = [_vp, _vp, _u32]
        lib.ref_rmsnorm_q8k.argtypes = [_vp, _vp, _u32, _f32, _vp, _vp]
        lib.ref_route.argtypes = [_vp, _vp, _vp, _u32, _u32, _u32, _vp, _vp]
        lib.ref_q4k_rows.argtypes = [_vp, _u32, _u32, _u32, _u32, _vp, _vp]
        lib.ref_moe_forward.restype = _int
        lib.ref_moe_forward.argtypes = [_vp, _u32, _u32, _u32, _u32, _u32, _f32, _vp, _vp, _vp, _vp, _vp, _vp,
                                        _u32, _vp, _vp, _vp]
        lib.ref_dense_ffn_forward.restype = _int
        lib.ref_dense_ffn_forward.argtypes = [_vp, _u32, _u32, _u32, _f32, _vp, _vp, _vp, _vp]
        self.lib = lib
        self.n_threads = lib.ref_init(n_threads)

    def set_threads(self, n: int) -> int:
        self.n_threads = self.lib.ref_init(n)
        return self.n_threads

    @property
    def isa(self) -> str:
        return self.lib.ref_isa_name().decode()

    @property
    def cpu(self) -> str:
        return self.lib.ref_cpu_brand().decode().strip()

    @property
    def order(self) -> int:
        return ORDER_VNNI if "VNNI" in self.isa else ORDER_AVX2

    def quantize_q8k(self, x):
        x = np.ascontiguousarray(x, np.float32).ravel()
        out = np.zeros(x.size // 256 * 292, np.uint8)
        self.lib.ref_quantize_q8k(_p(x), _p(out), x.size)
        return out

    def rmsnorm_q8k(self, x, norm_w, eps):
        x = np.ascontiguousarray(x, np.float32)
        D = x.size
        xb = np.zeros(D, np.float32)
        xq = np.zeros(D // 256 * 292, np.uint8)
        nw = None if norm_w is None else np.ascontiguousarray(norm_w, np.float32)
        self.lib.ref_rmsnorm_q8k(_p(x), _p(nw), D, eps, _p(xb), _p(xq))
        return xb, xq

    def route(self, router_w, bias, xb, K):
        router_w = np.ascontiguousarray(router_w, np.float32)
        E, D = router_w.shape
        idx = np.zeros(K, np.uint32)
        w = np.zeros(K, np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        self.lib.ref_route(_p(router_w), _p(b), _p(np.ascontiguousarray(xb, np.float32)), D, E, K, _p(idx), _p(w))
        return idx, w

    def q4k_rows(self, W, n_cols, total_rows, xq, r0=0, n_rows=None):
        n_rows = total_rows if n_rows is None else n_rows
        out = np.zeros(n_rows, np.float32)
        self.lib.ref_q4k_rows(_p(np.ascontiguousarray(W)), n_cols, total_rows, r0, n_rows,
                              _p(np.ascontiguousarray(xq)), _p(out))
        return out

    def moe_forward(self, L, x, capture=True):
        x = np.array(x, np.float32, copy=True, order="C")
        T = x.shape[0]
        idx = np.zeros((T, L.K), np.uint32) if capture else None
        w = np.zeros((T, L.K), np.float32) if capture else None
        xq = np.zeros(T * (L.D // 256) * 292, np.uint8) if capture else None
        st = self.lib.ref_moe_forward(_p(x), T, L.D, L.E, L.K, L.I, L.eps, _p(L.ffn_norm), _p(L.router_w),
                                      _p(L.bias), _p(L.gate), _p(L.up), _p(L.down), int(getattr(L, "down_type", 12)), _p(idx), _p(w),
                                      _p(xq))
        if st != 0:
            raise RuntimeError(f"reference moe_forward status {st}")
        return x, idx, w, xq

    def dense_forward(self, L, x):
        x = np.array(x, np.float32, copy=True, order="C")
        st = self.lib.ref_dense_ffn_forward(_p(x), x.shape[0], L.D, L.I, L.eps, _p(L.ffn_norm), _p(L.gate),
                                            _p(L.up), _p(L.down))
        if st != 0:
            raise RuntimeError(f"reference dense_forward status {st}")
        return x


def q8k_fields(buf: np.ndarray, nblocks: int):
    """Split 292-byte block_q8_K records into (d[n], qs[n,256], bsums[n,16])."""
    rec = np.frombuffer(np.ascontiguousarray(buf).tobytes(), dtype=np.dtype(
        [("d", "<f4"), ("qs", "i1", 256), ("bs", "<i2", 16)]), count=nblocks)
    return rec["d"].copy(), rec["qs"].copy(), rec["bs"].copy()
