"""GPU parity of the CUDA MoE-FFN path against the CPU oracle (through the C-ABI).

Bars (from the task's parity contract):
  - Q8_K of the normalised input: bit-exact (same reduction order as the reference);
  - expert ids identical except near-ties, |score_k - score_{k+1}| < 1e-6 in the
    oracle's biased scores (exp() may differ by an ulp between glibc and CUDA);
  - combine weights within 1e-6 relative;
  - Q4_K x Q8_K integer partial sums (per sub-block dots, per super-block
    sum sc*dot and sum m*bsum): bit-exact; fp32 row results: bit-exact with the
    reference's AVX-VNNI evaluation order;
  - layer outputs: relative L2 <= 1e-3 and max-abs <= 5e-3, on x and on the
    MoE delta (x_out - x_in), over tokens whose routing matched.
"""
import numpy as np
import pytest

from conftest import cached_dense, cached_layer, rel_l2

pytestmark = pytest.mark.gpu

REL_L2 = 1e-3
MAX_ABS = 5e-3
NEAR_TIE = 1e-6


@pytest.fixture(scope="module")
def gpu():
    from laii_b200.moe import GpuMoE
    g = GpuMoE(0)
    yield g
    g.close()


def oracle_scores(oracle, L, x):
    """Oracle xb and biased selection scores per token."""
    out = []
    for t in range(x.shape[0]):
        xb, _ = oracle.rmsnorm_q8k(x[t], L.ffn_norm, L.eps)
        _, _, _, sel = oracle.route(L.router_w, L.bias, xb, L.K)
        out.append(sel)
    return np.array(out)


def routing_mismatch_ok(sel_row, idx_gpu, idx_orc, K):
    """A routing difference is acceptable only if it is a near-tie in the oracle's scores."""
    order = np.argsort(-sel_row, kind="stable")
    s = sel_row[order]
    for k in range(K):
        if idx_gpu[k] != idx_orc[k]:
            nxt = s[k + 1] if k + 1 < len(s) else -np.inf
            prv = s[k - 1] if k > 0 else np.inf
            if min(abs(s[k] - nxt), abs(prv - s[k])) >= NEAR_TIE:
                return False
    return True


TIGHT = 1e-5  # rel-L2 of the MoE output (the layer's delta) against the reference: 100x inside the bar


def compare_layer(oracle, gpu, L, x, layer_id):
    from laii_b200 import synth  # noqa: F401
    gpu.upload_layer(layer_id, L)
    xg = np.array(x, np.float32, copy=True)
    gpu.forward(layer_id, xg)
    xo, io, wo, qo, _ = oracle.moe_forward(L, x)
    ig, wg, qg = gpu.debug_route(layer_id, x)
    assert np.array_equal(qg, qo), "Q8_K of normalised input must be bit-exact"
    match = np.all(ig == io, axis=1)
    if not match.all():
        sel = oracle_scores(oracle, L, x)
        for t in np.nonzero(~match)[0]:
            assert routing_mismatch_ok(sel[t], ig[t], io[t], L.K), f"token {t}: routing differs beyond a near-tie"
    assert match.mean() >= 0.95
    m = match
    np.testing.assert_allclose(wg[m], wo[m], rtol=NEAR_TIE, atol=0)
    assert np.isfinite(xg).all()
    assert rel_l2(xg[m], xo[m]) <= REL_L2
    assert np.abs(xg[m] - xo[m]).max() <= MAX_ABS
    dg, do = xg[m] - x[m], xo[m] - x[m]
    assert rel_l2(dg, do) <= REL_L2
    return xg, xo, match


SHAPES = [
    (512, 8, 2, 512, 5),
    (512, 8, 2, 512, 33),
    (2048, 32, 4, 1792, 1),   # config 1
    (2048, 32, 4, 1792, 8),   # config 2
    (2048, 64, 4, 1536, 16),  # config 5 layer shape
]


@pytest.mark.parametrize("D,E,K,I,T", [
    (1024, 16, 4, 768, 1),     # decode: route, gate|up GEMV, h -> Q8_K, Q6_K down
    (1024, 16, 4, 768, 8),
    (1024, 16, 4, 768, 40),
    (1024, 16, 4, 768, 300),   # prefill-sized: mma.sync gate/up GEMM, then the Q6_K down
    (2048, 8, 4, 1792, 8),     # config-1/2 row lengths (D=2048, I=1792: 7 Q6_K super-blocks)
])
def test_q6k_down_layer_parity(oracle, gpu, D, E, K, I, T):
    """Q6_K ffn_down_exps (upload_layer_typed): same bars as the Q4_K layers."""
    from laii_b200 import synth
    L = cached_layer(D, E, K, I, down_type=14)
    x = synth.make_hidden(T, D, seed_offset=11)
    xg, xo, match = compare_layer(oracle, gpu, L, x, 1)
    # exact integers and the reference's fp32 order: only the exp of SiLU (CUDA's expf, within 2 ulp of
    # glibc's) moves the layer's output, far inside the tolerance
    assert rel_l2(xg[match] - x[match], xo[match] - x[match]) <= TIGHT
    assert gpu.last_stats()["tokens"] == T


def test_q6k_down_layer_refused_where_q4k_only(gpu):
    """The no-allocate entry point takes Q4_K layers only: a Q6_K-down layer is an
    error status with a message, not a wrong result."""
    import ctypes
    torch = pytest.importorskip("torch")
    from laii_b200 import _native, synth
    lib = _native.load_gpu()
    gpu.upload_layer(2, cached_layer(1024, 16, 4, 768, down_type=14))
    xt = torch.from_numpy(synth.make_hidden(4, 1024, seed_offset=3)).cuda()
    st = lib.lfm_gpu_moe_forward_noalloc(gpu._h, 2, ctypes.c_void_p(xt.data_ptr()), 4, None)
    assert st != 0 and b"Q6_K" in lib.lfm_gpu_moe_last_error(gpu._h)
    gpu.sync()


@pytest.mark.parametrize("D,E,K,I,T", SHAPES)
def test_moe_layer_parity(oracle, gpu, D, E, K, I, T):
    from laii_b200 import synth
    L = cached_layer(D, E, K, I)
    x = synth.make_hidden(T, D, seed_offset=7)
    xg, xo, match = compare_layer(oracle, gpu, L, x, 0)
    # the integer path is exact and the fp32 order is the reference's: only exp() ulps (the router's
    # sigmoid, SiLU's single-precision expf) move the MoE output, far inside the tolerance
    assert rel_l2(xg[match] - x[match], xo[match] - x[match]) <= TIGHT


@pytest.mark.parametrize("D,E,K,I,T", [(512, 8, 2, 512, 64), (2048, 32, 4, 1792, 64)])
def test_route_parity(oracle, gpu, D, E, K, I, T):
    from laii_b200 import synth
    from oracle.oracle import q8k_fields
    L = cached_layer(D, E, K, I)
    gpu.upload_layer(1, L)
    x = synth.make_hidden(T, D, seed_offset=11)
    ig, wg, qg = gpu.debug_route(1, x)
    sel = oracle_scores(oracle, L, x)
    for t in range(T):
        xb, qo = oracle.rmsnorm_q8k(x[t], L.ffn_norm, L.eps)
        io, wo, _, _ = oracle.route(L.router_w, L.bias, xb, K)
        nb = D // 256
        assert np.array_equal(qg[t * nb * 292:(t + 1) * nb * 292], qo)
        if not np.array_equal(ig[t], io):
            assert routing_mismatch_ok(sel[t], ig[t], io, K)
        else:
            np.testing.assert_allclose(wg[t], wo, rtol=NEAR_TIE, atol=0)
    d, qs, bs = q8k_fields(qg, T * (D // 256))
    assert np.all(np.abs(qs) <= 127)
    assert np.array_equal(bs, qs.reshape(-1, 16, 16).sum(axis=2).astype(np.int16))


@pytest.mark.parametrize("n_cols,n_rows,n_vec", [(256, 8, 1), (2048, 64, 3), (1792, 40, 2), (4096, 16, 2)])
def test_q4k_integer_sums_bit_exact(oracle, gpu, n_cols, n_rows, n_vec):
    from laii_b200 import synth
    nb = n_cols // 256
    W = synth.q4k_normal(n_rows * nb, seed=1234 + n_cols, std=0.02)
    xs = synth.normal_f32(n_vec * n_cols, seed=99 + n_rows).reshape(n_vec, n_cols)
    if n_vec > 1:
        xs[1, :256] = 0.0  # a zero block: d8 == 0, skipped by the fp32 update
    xq = np.concatenate([oracle.quantize_q8k(v) for v in xs])
    sub, acc, mins, rows = gpu.debug_q4k_rows(W, n_rows, n_cols, xq, n_vec)
    Wr = W.reshape(n_rows, nb * 144)
    for v in range(n_vec):
        xv = xq[v * nb * 292:(v + 1) * nb * 292]
        ref_rows = oracle.q4k_rows(W, n_cols, n_rows, xv)
        assert np.array_equal(rows[v], ref_rows), "fp32 rows must follow the reference order exactly"
        for r in range(n_rows):
            s, a, m = oracle.q4k_row_ints(Wr[r], xv, n_cols)
            assert np.array_equal(sub[v, r], s)
            assert np.array_equal(acc[v, r], a)
            assert np.array_equal(mins[v, r], m)


def test_dense_layer_parity(oracle, gpu):
    from laii_b200 import synth
    L = cached_dense(2048, 7168)
    gpu.upload_dense(2, L)
    x = synth.make_hidden(4, 2048, seed_offset=3)
    xg = gpu.forward(2, np.array(x, copy=True))
    xo = oracle.dense_forward(L, x)
    assert rel_l2(xg, xo) <= REL_L2 and np.abs(xg - xo).max() <= MAX_ABS
    assert rel_l2(xg - x, xo - x) <= TIGHT  # only SiLU's exp ulps move the FFN's output


def test_prefill_zipf_subset(oracle, gpu):
    """Config 3 (T=2048, Zipf(1.1) expert popularity): all tokens on the GPU, a
    subset re-run on the oracle (tokens are independent)."""
    from laii_b200 import synth
    L = cached_layer(2048, 32, 4, 1792, zipf=1.1)
    x = synth.make_hidden(2048, 2048, seed_offset=100)
    gpu.upload_layer(3, L)
    xg = gpu.forward(3, np.array(x, copy=True))
    st = gpu.last_stats()
    assert st["tokens"] == 2048 and st["unique_experts"] >= 16
    sub = np.arange(0, 2048, 64)
    xo, io, _, _, _ = oracle.moe_forward(L, x[sub])
    ig, _, _ = gpu.debug_route(3, x[sub])
    m = np.all(ig == io, axis=1)
    assert m.mean() >= 0.9
    assert rel_l2(xg[sub][m], xo[m]) <= REL_L2
    assert np.abs(xg[sub][m] - xo[m]).max() <= MAX_ABS


@pytest.mark.parametrize("D,E,K,I,T", [(512, 8, 2, 512, 256), (2048, 32, 4, 1792, 512)])
def test_prefill_gemm_equals_gemv(monkeypatch, D, E, K, I, T):
    """The tensor-core GEMM path (prefill-sized T) and the dp4a GEMV path form the
    same exact integer sums and the same fp32 update order: identical outputs."""
    from laii_b200 import synth
    from laii_b200.moe import GpuMoE
    L = cached_layer(D, E, K, I, layer=2)
    x = synth.make_hidden(T, D, seed_offset=41)
    with GpuMoE(0) as g:
        g.upload_layer(0, L)
        a = g.forward(0, np.array(x, copy=True))
    monkeypatch.setenv("LFM_GPU_MOE_NO_GEMM", "1")
    with GpuMoE(0) as g:
        g.upload_layer(0, L)
        b = g.forward(0, np.array(x, copy=True))
    assert np.array_equal(a, b)


@pytest.mark.parametrize("D,E,K,I,T,zipf", [(2048, 32, 4, 1792, 2048, 1.1), (2048, 64, 4, 1536, 1024, None),
                                             (2048, 32, 4, 1792, 64, None), (2048, 32, 4, 1792, 24, None),
                                             (2048, 32, 4, 1792, 200, None)])
def test_prefill_tcgen05_equals_mma_sync_and_gemv(monkeypatch, D, E, K, I, T, zipf):
    """The tcgen05 GEMM (k_umma.cu: A from shared memory for large token blocks,
    from tensor memory for small ones), the mma.sync GEMM (k_gemm.cu) and the
    dp4a GEMV form the same exact integer sums and the same fp32 update order:
    identical outputs."""
    from laii_b200 import synth
    from laii_b200.moe import GpuMoE
    L = cached_layer(D, E, K, I, layer=4, zipf=zipf)
    x = synth.make_hidden(T, D, seed_offset=57)
    outs = []
    for env in ({}, {"LFM_GPU_MOE_NO_UMMA": "1"}, {"LFM_GPU_MOE_NO_GEMM": "1"}):
        for k, v in env.items():
            monkeypatch.setenv(k, v)
        with GpuMoE(0) as g:
            g.upload_layer(0, L)
            g.profile(True)
            outs.append(g.forward(0, np.array(x, copy=True)))
            prof = g.profile_read()
            g.profile(False)
        if not env:
            assert "xt_gather" in prof and "gemm_gateup" in prof, prof
    assert np.array_equal(outs[0], outs[1])
    assert np.array_equal(outs[0], outs[2])


def test_prefill_gemm_path_is_taken_and_dense_matches_oracle(oracle, gpu):
    """A dense layer at T=64 goes through the GEMM path (per-kernel profile) and matches the oracle."""
    from laii_b200 import synth
    L = cached_dense(2048, 7168)
    gpu.upload_dense(6, L)
    x = synth.make_hidden(64, 2048, seed_offset=9)
    gpu.profile(True)
    xg = gpu.forward(6, np.array(x, copy=True))
    prof = gpu.profile_read()
    gpu.profile(False)
    assert ("gemm_gateup" in prof or "gemm_gate" in prof) and "gemm_down" in prof
    xo = oracle.dense_forward(L, x)
    assert rel_l2(xg, xo) <= REL_L2 and np.abs(xg - xo).max() <= MAX_ABS


def test_device_synth_matches_host(gpu):
    """A layer generated on the device equals the host-generated one, byte for byte."""
    from laii_b200 import synth
    D, E, K, I = 512, 8, 2, 512
    L = cached_layer(D, E, K, I, layer=5)
    seeds = [synth.layer_seed(s, 5) for s in (synth.SEED_GATE, synth.SEED_UP, synth.SEED_DOWN, synth.SEED_ROUTER,
                                               synth.SEED_BIAS)]
    gpu.upload_layer(4, L)
    gpu.synth_layer(5, D, E, K, I, seeds)
    host = {"ffn_norm": L.ffn_norm, "router_w": L.router_w, "exp_probs_b": L.bias, "gate": L.gate, "up": L.up,
            "down": L.down}
    for name, arr in host.items():
        b = np.ascontiguousarray(arr).view(np.uint8).ravel()
        d = gpu.read_layer(5, name, b.size)
        bad = np.nonzero(d != b)[0]
        assert bad.size == 0, f"{name}: {bad.size} bytes differ, first at {bad[:8]}"
        assert np.array_equal(gpu.read_layer(4, name, b.size), b), f"upload of {name} altered bytes"
    x = synth.make_hidden(6, D, seed_offset=5)
    a = gpu.forward(4, np.array(x, copy=True))
    b = gpu.forward(5, np.array(x, copy=True))
    assert np.array_equal(a, b)


def test_edge_cases(oracle, gpu):
    from laii_b200 import synth
    from laii_b200.moe import MoEError
    D, E, K, I = 512, 8, 2, 512
    L = cached_layer(D, E, K, I)
    gpu.upload_layer(6, L)
    # empty batch is a no-op
    gpu.forward(6, np.zeros((0, D), np.float32))
    # an all-zero row stays zero (RMSNorm of 0 is 0, Q8_K block d = 0, experts skip it)
    x = synth.make_hidden(3, D, seed_offset=9)
    x[1] = 0.0
    xg = gpu.forward(6, np.array(x, copy=True))
    xo, _, _, _, _ = oracle.moe_forward(L, x)
    assert np.array_equal(xg[1], np.zeros(D, np.float32))
    assert rel_l2(xg, xo) <= REL_L2
    # every token forced onto one expert (one large segment)
    Lb = cached_layer(D, E, K, I)
    bias = np.array(Lb.bias, copy=True)
    bias[3] += 10.0
    from dataclasses import replace
    Lf = replace(Lb, bias=bias)
    gpu.upload_layer(7, Lf)
    x = synth.make_hidden(40, D, seed_offset=13)
    xg = gpu.forward(7, np.array(x, copy=True))
    xo, io, _, _, _ = oracle.moe_forward(Lf, x)
    assert np.all(io[:, 0] == 3)
    assert rel_l2(xg, xo) <= REL_L2
    # errors are statuses, not crashes
    with pytest.raises(MoEError) as ei:
        gpu.forward(40, np.zeros((1, D), np.float32))
    assert ei.value.status == -3
    with pytest.raises(MoEError) as ei:
        gpu.upload_layer(8, replace(L, D=500))
    assert ei.value.status == -1


def test_device_pointer_forward_matches_host(gpu):
    torch = pytest.importorskip("torch")
    from laii_b200 import synth
    D, E, K, I = 2048, 32, 4, 1792
    L = cached_layer(D, E, K, I)
    gpu.upload_layer(9, L)
    x = synth.make_hidden(8, D, seed_offset=21)
    a = gpu.forward(9, np.array(x, copy=True))
    xt = torch.from_numpy(np.array(x, copy=True)).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    gpu.forward_device(9, xt.data_ptr(), 8, stream=stream)
    torch.cuda.synchronize()
    assert np.array_equal(xt.cpu().numpy(), a)
