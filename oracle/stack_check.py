"""TEST INFRASTRUCTURE ONLY -- layer-by-layer parity of a GPU FFN stack against the CPU checker.

The GPU runs a stack of lfm2moe / dense FFN layers; for a subset of tokens the
caller records each layer's input and output rows.  Every layer is then re-run
on the CPU from the GPU's own input rows, so an error cannot hide behind the
layers after it, and the rows are compared under the parity bars of the path:

  - Q8_K of the normalised input (from lfm_gpu_moe_debug_route): bit-exact;
  - expert ids identical, except near-ties: a differing id is accepted only
    where the oracle's biased scores of the two experts differ by < 1e-6
    (tools/lfm2_moe_checkpoint.c:166-240 is the routing restated);
  - combine weights within 1e-6 relative;
  - layer outputs over the tokens whose routing matched: relative L2 <= 1e-3
    and max-abs <= 5e-3 (the reference path, tools/lfm2_moe_checkpoint.c:312-365
    per token; dense layers tools/lfm2_decode_1x4.c:1070-1104).

The CPU side is the reference's own code built from its sources (oracle/_ref)
where it was built, else the scalar restatement (oracle/lfm_oracle.c); the two
are pinned bit-exact against each other by tests/test_oracle_ref.py.  Expert
weights are read back from the device only for the experts the checked tokens
are routed to: a layer's other experts stay untouched zero pages.

Only tests/ and bench.py's parity block (after its timed region) use this.
"""
from __future__ import annotations

import os
from typing import Callable, Dict, Optional

import numpy as np

from .oracle import REF_SO, Oracle, Reference

REL_L2 = 1e-3
MAX_ABS = 5e-3
NEAR_TIE = 1e-6
Q4K = 144
TENSORS = ("ffn_norm", "router_w", "exp_probs_b", "gate", "up", "down")


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


class _Layer:
    """Host copy of an lfm2moe layer with the attribute names the oracle reads."""

    def __init__(self, D, E, K, I, ffn_norm, router_w, bias, gate, up, down, eps, down_type=12):
        self.D, self.E, self.K, self.I = D, E, K, I
        self.ffn_norm, self.router_w, self.bias = ffn_norm, router_w, bias
        self.gate, self.up, self.down = gate, up, down
        self.eps, self.norm_topk_prob, self.routed_scale, self.down_type = eps, True, 1.0, down_type


def routing_mismatch_ok(sel_row, idx_gpu, idx_orc, K) -> bool:
    """A routing difference is acceptable only if it is a near-tie in the oracle's scores."""
    s = np.sort(sel_row)[::-1]
    for k in range(K):
        if idx_gpu[k] != idx_orc[k]:
            nxt = s[k + 1] if k + 1 < len(s) else -np.inf
            prv = s[k - 1] if k > 0 else np.inf
            if min(abs(s[k] - nxt), abs(prv - s[k])) >= NEAR_TIE:
                return False
    return True


class StackChecker:
    """CPU re-run of single layers on given input rows, compared with the GPU's output rows."""

    def __init__(self, n_threads: int = 0):
        self.oracle = Oracle()
        self.ref = Reference(n_threads) if os.path.exists(REF_SO) else None
        self.kind = "reference (oracle/_ref)" if self.ref else "scalar oracle port"

    def _moe(self, L, x):
        if self.ref is not None:
            return self.ref.moe_forward(L, x)[0]
        return self.oracle.moe_forward(L, x)[0]

    def _dense(self, L, x):
        return (self.ref or self.oracle).dense_forward(L, x)

    def host_moe_layer(self, read: Callable, D: int, E: int, K: int, I: int, x_in: np.ndarray,
                       eps: float = 1e-5, down_type: int = 12):
        """The layer as the oracle reads it, with only the experts that x_in's tokens route to
        filled in.  read(which, offset, nbytes) -> uint8 bytes of a device tensor.  down_type:
        12 (Q4_K, 144-byte blocks) or 14 (Q6_K, 210-byte blocks)."""
        norm = read("ffn_norm", 0, 4 * D).view(np.float32).copy()
        router = read("router_w", 0, 4 * E * D).view(np.float32).reshape(E, D).copy()
        bias = read("exp_probs_b", 0, 4 * E).view(np.float32).copy()
        per_gu, per_dn = I * (D // 256) * Q4K, D * (I // 256) * (210 if down_type == 14 else Q4K)
        gate = np.zeros(E * per_gu, np.uint8)
        up = np.zeros(E * per_gu, np.uint8)
        down = np.zeros(E * per_dn, np.uint8)
        L = _Layer(D, E, K, I, norm, router, bias, gate, up, down, eps, down_type)
        sel_rows, want = [], set()
        for t in range(x_in.shape[0]):
            xb, _ = self.oracle.rmsnorm_q8k(x_in[t], norm, eps)
            idx, _, _, sel = self.oracle.route(router, bias, xb, K)
            sel_rows.append(sel)
            want.update(int(e) for e in idx)
        for e in sorted(want):
            for name, arr, per in (("gate", gate, per_gu), ("up", up, per_gu), ("down", down, per_dn)):
                arr[e * per:(e + 1) * per] = read(name, e * per, per)
        return L, np.array(sel_rows), sorted(want)

    def check_moe(self, L, sel, x_in, x_out, gpu_route: Optional[tuple] = None) -> Dict:
        """Compare the GPU's output rows of one MoE layer with the CPU's re-run of x_in.
        gpu_route = (idx[T,K], w[T,K], q8 bytes) from lfm_gpu_moe_debug_route on x_in, if available."""
        T = x_in.shape[0]
        xo = self._moe(L, x_in)
        out = {"tokens": T, "near_ties": 0, "routing_miss": 0, "q8_exact": None, "w_rel": None}
        match = np.ones(T, bool)
        if gpu_route is not None:
            ig, wg, qg = gpu_route
            io, wo, qo = self._route_only(L, x_in)
            out["q8_exact"] = bool(np.array_equal(qg, qo))
            match = np.all(ig == io, axis=1)
            for t in np.nonzero(~match)[0]:
                if routing_mismatch_ok(sel[t], ig[t], io[t], L.K):
                    out["near_ties"] += 1
                else:
                    out["routing_miss"] += 1
            if match.any():
                out["w_rel"] = float(np.max(np.abs(wg[match] - wo[match]) / np.maximum(np.abs(wo[match]), 1e-30)))
        out.update(self._compare(x_out[match], xo[match]))
        out["ok"] = bool(out["ok"] and out["routing_miss"] == 0 and out["q8_exact"] is not False
                         and (out["w_rel"] is None or out["w_rel"] <= NEAR_TIE))
        return out

    def _route_only(self, L, x_in):
        """(idx, w, q8) of x_in by the oracle's routing (no expert compute)."""
        T = x_in.shape[0]
        idx = np.zeros((T, L.K), np.uint32)
        w = np.zeros((T, L.K), np.float32)
        q8 = []
        for t in range(T):
            xb, q = self.oracle.rmsnorm_q8k(x_in[t], L.ffn_norm, L.eps)
            i, wt, _, _ = self.oracle.route(L.router_w, L.bias, xb, L.K)
            idx[t], w[t] = i, wt
            q8.append(q)
        return idx, w, np.concatenate(q8) if q8 else np.zeros(0, np.uint8)

    def check_dense(self, L, x_in, x_out) -> Dict:
        xo = self._dense(L, x_in)
        out = {"tokens": int(x_in.shape[0])}
        out.update(self._compare(x_out, xo))
        return out

    @staticmethod
    def _compare(got, want) -> Dict:
        if got.size == 0:
            return {"rel_l2": 0.0, "max_abs": 0.0, "ok": True}
        r = rel_l2(got, want)
        m = float(np.abs(np.asarray(got, np.float64) - want).max())
        return {"rel_l2": r, "max_abs": m, "ok": bool(np.isfinite(got).all() and r <= REL_L2 and m <= MAX_ABS)}


def summarise(per_layer) -> Dict:
    """One parity record for a stack: worst layer figures, counts, and the verdict."""
    moe = [p for p in per_layer if "near_ties" in p]
    return {"layers": len(per_layer),
            "tokens": max((p["tokens"] for p in per_layer), default=0),
            "rel_l2": max((p["rel_l2"] for p in per_layer), default=0.0),
            "max_abs": max((p["max_abs"] for p in per_layer), default=0.0),
            "ids_match": all(p["routing_miss"] == 0 for p in moe),
            "near_ties": sum(p["near_ties"] for p in moe),
            "q8_exact": all(p["q8_exact"] is not False for p in moe),
            "ok": all(p["ok"] for p in per_layer)}
