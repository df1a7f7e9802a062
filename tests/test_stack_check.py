"""The layer-by-layer stack checker (oracle/stack_check.py) and the bench's CPU reference arm.

The checker is what the bench's parity block and the stack tests rely on, so it
is pinned here on the CPU: rows the oracle itself produced pass; a planted
output error, a wrong expert id or a flipped Q8_K byte fails.  The reference
arm must describe the workload exactly as the GPU arm does and must map no
library of the GPU package.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from laii_b200 import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
D, E, K, I, DI = 512, 8, 2, 512, 768


def _reader(L):
    arrays = {"ffn_norm": L.ffn_norm, "router_w": L.router_w, "exp_probs_b": L.bias, "gate": L.gate, "up": L.up,
              "down": L.down}

    def read(which, off, nb):
        return np.ascontiguousarray(arrays[which]).view(np.uint8).reshape(-1)[off:off + nb].copy()
    return read


@pytest.fixture(scope="module")
def stack():
    from oracle.stack_check import StackChecker
    chk = StackChecker(1)
    dense = synth.make_dense_layer(D, DI, layer=0)
    moe = synth.make_moe_layer(D, E, K, I, layer=1)
    x = synth.make_hidden(6, D, seed_offset=21)
    return chk, dense, moe, x


def test_checker_accepts_the_oracles_own_rows(stack):
    from oracle.stack_check import summarise
    chk, dense, moe, x = stack
    x1 = chk.oracle.dense_forward(dense, x)
    x2, idx, w, q8, _ = chk.oracle.moe_forward(moe, x1)
    Lh, sel, want = chk.host_moe_layer(_reader(moe), D, E, K, I, x1)
    assert set(want) == set(int(e) for e in idx.ravel())
    # only the routed experts were read: the others stay zero
    per = I * (D // 256) * 144
    for e in range(E):
        assert bool(Lh.gate[e * per:(e + 1) * per].any()) == (e in want)
    p_dense = chk.check_dense(dense, x, x1)
    p_moe = chk.check_moe(Lh, sel, x1, x2, (idx.astype(np.int32), w, q8))
    assert p_dense["ok"] and p_moe["ok"], (p_dense, p_moe)
    s = summarise([p_dense, p_moe])
    assert s["ok"] and s["ids_match"] and s["q8_exact"] and s["rel_l2"] == 0.0


def test_checker_catches_planted_mistakes(stack):
    chk, dense, moe, x = stack
    x2, idx, w, q8, _ = chk.oracle.moe_forward(moe, x)
    Lh, sel, _ = chk.host_moe_layer(_reader(moe), D, E, K, I, x)
    route = (idx.astype(np.int32), w, q8)
    bad = x2.copy()
    bad[2, 7] += 1e-2                                           # an output error above max-abs
    assert not chk.check_moe(Lh, sel, x, bad, route)["ok"]
    bad_ids = idx.astype(np.int32).copy()
    bad_ids[1, 0] = (bad_ids[1, 0] + 1) % E if (bad_ids[1, 0] + 1) % E not in bad_ids[1] else (bad_ids[1, 0] + 2) % E
    r = chk.check_moe(Lh, sel, x, x2, (bad_ids, w, q8))         # a wrong expert, not a near-tie
    assert r["routing_miss"] == 1 and not r["ok"]
    bad_q8 = q8.copy()
    bad_q8[10] ^= 1                                              # one Q8_K byte
    assert not chk.check_moe(Lh, sel, x, x2, (idx.astype(np.int32), w, bad_q8))["ok"]
    assert not chk.check_dense(dense, x, x * 1.01)["ok"]


def test_reference_arm_maps_no_gpu_package_library(tmp_path):
    """The CPU reference arm of the bench generates its inputs with the oracle's build of the
    generator and runs the reference's CPU path: no laii_b200/_lib library is loaded."""
    from oracle.oracle import GEN_SO
    if not os.path.exists(GEN_SO):
        pytest.skip("oracle not built")
    code = (
        "import sys, json; sys.argv=['bench.py','--impl','reference','--config','1','--steps','1','--warmup','0',"
        "'--prefill-config','0']\n"
        "import bench; bench.main()\n"
        "maps=open('/proc/self/maps').read()\n"
        "print(json.dumps({'gpu_pkg_libs': sorted({l.split()[-1] for l in maps.splitlines() "
        "if 'laii_b200/_lib' in l})}))\n")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [json.loads(ln) for ln in r.stdout.splitlines() if ln.startswith("{")]
    line, maps = lines[0], lines[1]
    assert maps["gpu_pkg_libs"] == []
    assert line["impl"] == "reference" and line["value"] > 0
    import bench
    from laii_b200.synth import CONFIGS
    assert line["config"] == bench.workload(1, dict(CONFIGS[1]))   # the GPU arm prints the same dict


def test_both_generator_builds_make_the_same_bytes():
    from oracle.oracle import GEN_SO
    if not os.path.exists(GEN_SO):
        pytest.skip("oracle not built")
    a = synth.q4k_normal(64, 1234, 0.02, first_block=5)
    code = ("import sys; sys.path.insert(0, %r)\n"
            "from laii_b200 import synth; synth.use_generator_library(%r)\n"
            "sys.stdout.buffer.write(synth.q4k_normal(64, 1234, 0.02, first_block=5).tobytes())\n") % (ROOT, GEN_SO)
    r = subprocess.run([sys.executable, "-c", code], stdout=subprocess.PIPE, timeout=120)
    assert r.returncode == 0
    assert np.array_equal(np.frombuffer(r.stdout, np.uint8), a)
