"""Generate the golden fixtures in this directory by running the REFERENCE's own
CPU path (oracle/_ref/libref_moe.so, built from the reference sources by
oracle/Makefile) -- not our oracle.  Run once where the reference sources are
available:

    make -C oracle && python tests/golden/make_golden.py            # every fixture
    make -C oracle && python tests/golden/make_golden.py moe_q6k    # only the named lfm2moe cases

Fixtures (all small):
  router_kat.npz   the reference's router known-answer test inputs
                   (tests/test_moe_checkpoint.c:138-218) -> expert ids, weights
  q8k_kat.npz      the reference's Q8_K test input (tests/test_cpuid_quants.c:69-111)
                   and an all-zero row -> block_q8_K bytes
  moe_*.npz        lfm2moe layers on seeded synthetic weights -> x_out, ids,
                   weights, Q8_K(x); the weights are regenerated from their
                   seeds at test time and pinned by a SHA-256 digest
                   (moe_q6k: ffn_down_exps stored as Q6_K, down_type 14)
  dense_small.npz  a dense SwiGLU layer -> x_out
  meta.json        ISA the reference selected, thread count, digests
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from laii_b200 import synth  # noqa: E402
from oracle.oracle import Oracle, Reference  # noqa: E402

MOE_CASES = {
    "moe_small": dict(D=512, E=8, K=2, I=512, T=4, layer=3, seed_offset=1),
    "moe_cfg1": dict(D=2048, E=32, K=4, I=1792, T=1, layer=0, seed_offset=0),
    "moe_cfg2": dict(D=2048, E=32, K=4, I=1792, T=8, layer=0, seed_offset=0),
    "moe_e64": dict(D=2048, E=64, K=4, I=1536, T=2, layer=1, seed_offset=2),
    "moe_q6k": dict(D=512, E=8, K=2, I=512, T=4, layer=5, seed_offset=6, down_type=14),
}
DENSE_CASE = dict(D=512, I=1024, T=3, layer=0, seed_offset=4)


def moe_case(ref, name, c, meta):
    L = synth.make_moe_layer(c["D"], c["E"], c["K"], c["I"], layer=c["layer"], down_type=c.get("down_type", 12))
    x = synth.make_hidden(c["T"], c["D"], seed_offset=c["seed_offset"])
    xo, ii, ww, xq = ref.moe_forward(L, x)
    np.savez(os.path.join(HERE, name + ".npz"), x_out=xo, idx=ii, w=ww, xq=xq)
    meta["digests"][name] = {"layer": L.digest(), "x": __import__("hashlib").sha256(x.tobytes()).hexdigest()}


def main(only=()):
    ref = Reference(1)
    orc = Oracle()
    meta = {"isa": ref.isa, "cpu": ref.cpu, "threads": ref.n_threads, "digests": {}}
    if only:  # regenerate the named lfm2moe cases; keep the other fixtures as they are
        meta = json.load(open(os.path.join(HERE, "meta.json")))
        if meta["isa"] != ref.isa:
            raise SystemExit(f"fixtures were made with {meta['isa']}, this host selects {ref.isa}")
        for name in only:
            moe_case(ref, name, MOE_CASES[name], meta)
        meta["cases"]["moe"] = MOE_CASES
        json.dump(meta, open(os.path.join(HERE, "meta.json"), "w"), indent=1, sort_keys=True)
        print("wrote", ", ".join(only), "with reference ISA:", ref.isa)
        return

    xb, w, b = orc.kat_router_inputs(2048, 32)
    idx, wt = ref.route(w, b, xb, 4)
    np.savez(os.path.join(HERE, "router_kat.npz"), idx=idx, w=wt)

    x = orc.kat_q8k_inputs(2048)
    q = ref.quantize_q8k(x)
    qz = ref.quantize_q8k(np.zeros(512, np.float32))
    np.savez(os.path.join(HERE, "q8k_kat.npz"), q8=q, q8_zero=qz)

    for name, c in MOE_CASES.items():
        moe_case(ref, name, c, meta)

    c = DENSE_CASE
    Ld = synth.make_dense_layer(c["D"], c["I"], layer=c["layer"])
    x = synth.make_hidden(c["T"], c["D"], seed_offset=c["seed_offset"])
    np.savez(os.path.join(HERE, "dense_small.npz"), x_out=ref.dense_forward(Ld, x))
    meta["cases"] = {"moe": MOE_CASES, "dense": DENSE_CASE}
    json.dump(meta, open(os.path.join(HERE, "meta.json"), "w"), indent=1, sort_keys=True)
    print("wrote fixtures with reference ISA:", ref.isa)


if __name__ == "__main__":
    main(tuple(sys.argv[1:]))
