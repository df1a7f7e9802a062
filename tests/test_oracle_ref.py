"""The oracle restatement against the reference CPU path built from its sources
(oracle/_ref/libref_moe.so), bit for bit, on fresh seeded inputs and edge
cases.  Skipped where the reference was never built."""
import numpy as np
import pytest

from conftest import cached_layer
from oracle.oracle import q8k_fields


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_q8k_random_and_edges(oracle, reference, seed):
    from laii_b200 import synth
    x = synth.normal_f32(4096, seed=seed, std=3.0)
    x[:256] = 0.0                          # all-zero block
    x[256:512] = 1e-30                     # tiny block (denormal products under FTZ)
    x[512] = 1e6                           # one large value dominating a block
    x[768:1024] = np.float32(0.5) * np.sign(x[768:1024])  # many exact .5 ties after scaling
    assert np.array_equal(oracle.quantize_q8k(x), reference.quantize_q8k(x))


@pytest.mark.parametrize("D", [256, 512, 2048, 4096])
def test_rmsnorm_q8k(oracle, reference, D):
    from laii_b200 import synth
    x = synth.normal_f32(D, seed=D, std=1.7)
    nw = synth.normal_f32(D, seed=D + 1, mean=1.0, std=0.1)
    for norm in (None, nw):
        xb_o, q_o = oracle.rmsnorm_q8k(x, norm, 1e-5)
        xb_r, q_r = reference.rmsnorm_q8k(x, norm, 1e-5)
        assert np.array_equal(xb_o, xb_r) and np.array_equal(q_o, q_r)


@pytest.mark.parametrize("E,K", [(8, 2), (32, 4), (64, 4), (64, 8)])
def test_route(oracle, reference, E, K):
    from laii_b200 import synth
    D = 2048
    w = synth.normal_f32(E * D, seed=E * 10 + K, std=0.02).reshape(E, D)
    b = synth.normal_f32(E, seed=E * 10 + K + 1, std=0.1)
    for t in range(8):
        xb = synth.normal_f32(D, seed=500 + t)
        i_o, w_o, _, _ = oracle.route(w, b, xb, K)
        i_r, w_r = reference.route(w, b, xb, K)
        assert np.array_equal(i_o, i_r) and np.array_equal(w_o, w_r)
    # no bias tensor (exp_probs_b absent) and an exact tie: equal rows tie, lowest index wins
    w2 = np.array(w, copy=True)
    w2[5] = w2[3]
    i_o, w_o, _, _ = oracle.route(w2, None, xb, K)
    i_r, w_r = reference.route(w2, None, xb, K)
    assert np.array_equal(i_o, i_r) and np.array_equal(w_o, w_r)


@pytest.mark.parametrize("n_cols", [256, 1792, 2048])
def test_q4k_rows(oracle, reference, n_cols):
    from laii_b200 import synth
    n_rows = 16
    W = synth.q4k_normal(n_rows * n_cols // 256, seed=n_cols, std=0.02)
    x = synth.normal_f32(n_cols, seed=n_cols + 7)
    xq = oracle.quantize_q8k(x)
    r = reference.q4k_rows(W, n_cols, n_rows, xq)
    o = oracle.q4k_rows(W, n_cols, n_rows, xq, order=reference.order)
    assert np.array_equal(o, r)


@pytest.mark.parametrize("D,E,K,I,T", [(512, 8, 2, 512, 3), (1024, 16, 4, 768, 5), (2048, 64, 4, 1536, 2)])
def test_moe_layer(oracle, reference, D, E, K, I, T):
    from laii_b200 import synth
    L = cached_layer(D, E, K, I)
    x = synth.make_hidden(T, D, seed_offset=31)
    xr, ir, wr, qr = reference.moe_forward(L, x)
    xo, io, wo, qo, _ = oracle.moe_forward(L, x, order=reference.order)
    assert np.array_equal(ir, io) and np.array_equal(wr, wo) and np.array_equal(qr, qo)
    assert np.array_equal(xr, xo)


@pytest.mark.parametrize("D,E,K,I,T", [(512, 8, 2, 512, 3), (1024, 16, 4, 768, 5)])
def test_moe_layer_q6k_down(oracle, reference, D, E, K, I, T):
    """Q6_K ffn_down_exps (Q4_K_M checkpoints): the reference selects its Q6_K x Q8_K
    kernel by tensor type (tools/lfm2_decode_1x4.c:618-630); bit for bit."""
    from laii_b200 import synth
    L = cached_layer(D, E, K, I, down_type=14)
    x = synth.make_hidden(T, D, seed_offset=33)
    xr, ir, wr, qr = reference.moe_forward(L, x)
    xo, io, wo, qo, _ = oracle.moe_forward(L, x, order=reference.order)
    assert np.array_equal(ir, io) and np.array_equal(wr, wo) and np.array_equal(qr, qo)
    assert np.array_equal(xr, xo)
    # the Q6_K layer is a different layer from its Q4_K twin, not a relabelled one
    assert not np.array_equal(xo, oracle.moe_forward(cached_layer(D, E, K, I), x, order=reference.order)[0])


def test_dense_layer(oracle, reference):
    from conftest import cached_dense
    from laii_b200 import synth
    L = cached_dense(512, 1024)
    x = synth.make_hidden(3, 512, seed_offset=8)
    assert np.array_equal(reference.dense_forward(L, x), oracle.dense_forward(L, x, order=reference.order))


def test_q8k_fields_layout(oracle):
    from laii_b200 import synth
    x = synth.normal_f32(512, seed=77)
    d, qs, bs = q8k_fields(oracle.quantize_q8k(x), 2)
    np.testing.assert_allclose(d, np.abs(x.reshape(2, 256)).max(axis=1) / 127, rtol=1e-6)
    assert np.array_equal(bs, qs.reshape(2, 16, 16).sum(axis=2))
