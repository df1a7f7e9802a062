"""Full-depth stacks on the GPU against the reference CPU path, layer by layer.

Config 4 (2 dense SwiGLU layers, I=7168, then 22 lfm2moe layers, D=2048, E=32,
top-4, I=1792; 64 tokens) and a 4-layer slice of config 5 (E=64, I=1536) at
T=4096.  The stack runs through forward_stack (one captured CUDA graph); the
same layers run once more one call at a time, recording a token subset's rows
before and after every layer; the graph's final rows must equal that chain's
bit for bit, and every layer is re-run on the CPU (the reference's
tools/lfm2_moe_checkpoint.c:312-365 per token, dense layers
tools/lfm2_decode_1x4.c:1070-1104) from the GPU's own input rows and compared
under the parity bars: ids equal except near-ties, Q8_K bit-exact, weights
within 1e-6, rows within rel-L2 1e-3 and max-abs 5e-3.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _seeds(layer):
    from laii_b200 import synth
    return [synth.layer_seed(s, layer) for s in (synth.SEED_GATE, synth.SEED_UP, synth.SEED_DOWN,
                                                   synth.SEED_ROUTER, synth.SEED_BIAS)]


def _run_stack(cfg, n_moe, T, sub):
    torch = pytest.importorskip("torch")
    from laii_b200 import synth
    from laii_b200.moe import GpuMoE
    from oracle.stack_check import StackChecker, summarise
    D, E, K, I = cfg["D"], cfg["E"], cfg["K"], cfg["I"]
    n_dense = cfg.get("dense", 0)
    layers = [("dense", l) for l in range(n_dense)] + [("moe", n_dense + m) for m in range(n_moe)]
    dense_host = {}
    x0 = synth.make_hidden(T, D, seed_offset=3)
    with GpuMoE(0) as g:
        for kind, l in layers:
            if kind == "dense":
                dense_host[l] = synth.make_dense_layer(D, cfg["dense_I"], layer=l)
                g.upload_dense(l, dense_host[l])
            else:
                g.synth_layer(l, D, E, K, I, _seeds(l))
        g.reserve(T)
        x = torch.from_numpy(x0.copy()).cuda()
        s = torch.cuda.current_stream().cuda_stream
        g.forward_device(0, x.data_ptr(), T, stream=s, n_layers=len(layers))   # captures the graph
        x.copy_(torch.from_numpy(x0))
        g.forward_device(0, x.data_ptr(), T, stream=s, n_layers=len(layers))   # replays it
        torch.cuda.synchronize()
        graph_out = x.cpu().numpy()
        x.copy_(torch.from_numpy(x0))
        rows = []
        for kind, l in layers:
            xin = x.cpu().numpy()[sub]
            g.forward_device(l, x.data_ptr(), T, stream=s)
            torch.cuda.synchronize()
            rows.append((kind, l, xin, x.cpu().numpy()[sub]))
        assert np.array_equal(graph_out, x.cpu().numpy()), "graph replay differs from the layer-by-layer chain"
        g.sync()
        chk = StackChecker(0)
        per_layer = []
        for kind, l, xin, xout in rows:
            if kind == "dense":
                per_layer.append(chk.check_dense(dense_host[l], xin, xout))
                continue
            Lh, sel, _ = chk.host_moe_layer(lambda w, o, n, l=l: g.read_layer(l, w, n, offset=o), D, E, K, I, xin)
            per_layer.append(chk.check_moe(Lh, sel, xin, xout, g.debug_route(l, np.ascontiguousarray(xin))))
    bad = [(i, p) for i, p in enumerate(per_layer) if not p["ok"]]
    assert not bad, bad[:3]
    return summarise(per_layer)


def test_config4_stack_against_reference_layer_by_layer():
    from laii_b200.synth import CONFIGS
    cfg = CONFIGS[4]
    sub = np.arange(0, 64, 8)
    s = _run_stack(cfg, cfg["layers"], cfg["T"], sub)
    assert s["layers"] == 24 and s["ids_match"] and s["q8_exact"]


def test_config5_slice_at_T4096_against_reference_layer_by_layer():
    from laii_b200.synth import CONFIGS
    cfg = CONFIGS[5]
    sub = np.linspace(0, 4095, 16).astype(np.int64)
    s = _run_stack(cfg, 4, cfg["T"], sub)
    assert s["layers"] == 4 and s["ids_match"] and s["q8_exact"]
