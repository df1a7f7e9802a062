"""The seeded generator: determinism, distribution, and the fp16/Q4_K helpers."""
import math

import numpy as np
import pytest

from laii_b200 import _native, synth


def test_counter_rng_is_splitmix64_stream():
    lib = _native.load_synth()
    # splitmix64 stepped sequentially from state s
    s = 12345
    mask = (1 << 64) - 1
    for ctr in range(4):
        s = (s + 0x9E3779B97F4A7C15) & mask
        z = s
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & mask
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & mask
        z ^= z >> 31
        assert lib.lfm_synth_u64(12345, ctr) == z


def test_log_accuracy():
    lib = _native.load_synth()
    for v in [1e-30, 1e-5, 0.1, 0.5, 0.7071, 1.0, 1.4143, 2.0, 3.7, 1e10]:
        assert abs(lib.lfm_synth_log(v) - math.log(v)) <= 4e-16 * max(1.0, abs(math.log(v)))


def test_normals_are_standard():
    x = synth.normal_f32(200_000, seed=42).astype(np.float64)
    assert abs(x.mean()) < 0.01 and abs(x.std() - 1.0) < 0.01
    assert abs(np.mean(np.abs(x) < 1.0) - 0.6827) < 0.005


def test_generation_is_deterministic_and_thread_count_free():
    a = synth.normal_f32(10_000, seed=7, threads=1)
    b = synth.normal_f32(10_000, seed=7, threads=8)
    c = synth.normal_f32(5_000, seed=7, first=5_000, threads=3)
    assert np.array_equal(a, b) and np.array_equal(a[5000:], c)
    q1 = synth.q4k_normal(64, seed=9, std=0.02, threads=1)
    q2 = synth.q4k_normal(64, seed=9, std=0.02, threads=5)
    assert np.array_equal(q1, q2)


def test_fp16_conversion_matches_ieee():
    lib = _native.load_synth()
    vals = np.concatenate([synth.normal_f32(2000, seed=3, std=1e-3), synth.normal_f32(2000, seed=4, std=100.0),
                           np.array([0.0, -0.0, 6.1e-5, 5.96e-8, 2.98e-8, 65504.0, 65520.0, 1e9, np.inf],
                                    np.float32)])
    for v in vals:
        h = lib.lfm_synth_float_to_half(float(v))
        assert h == int(np.float32(v).astype(np.float16).view(np.uint16))
        back = lib.lfm_synth_half_to_float(h)
        assert back == float(np.float16(np.uint16(h).view(np.float16)).astype(np.float32)) or math.isnan(back)


def test_q4k_quantiser_roundtrip():
    x = synth.normal_f32(256 * 64, seed=11, std=0.02)
    q = synth.quantize_q4k(x)
    assert q.size == 64 * 144
    y = synth.dequantize_q4k(q)
    err = np.abs(y - x).reshape(64, 8, 32)
    rng = (x.reshape(64, 8, 32).max(axis=2) - np.minimum(x.reshape(64, 8, 32).min(axis=2), 0))
    # a 4-bit step is range/15; allow a little for the 6-bit scale codes
    assert np.all(err.max(axis=2) <= rng / 15 * 0.75 + 1e-4)
    assert np.corrcoef(x, y)[0, 1] > 0.99


def test_layer_shapes_and_sizes():
    L = synth.make_moe_layer(512, 8, 2, 512)
    assert L.gate.size == 8 * 512 * 2 * 144 and L.down.size == 8 * 512 * 2 * 144
    assert L.router_w.shape == (8, 512) and L.bias.shape == (8,)
    with pytest.raises(ValueError):
        synth.make_moe_layer(500, 8, 2, 512)


def test_zipf_bias_skews_popularity(oracle):
    from conftest import cached_layer
    L = cached_layer(512, 8, 2, 512, zipf=1.1)
    x = synth.make_hidden(256, 512, seed_offset=3)
    counts = np.zeros(8)
    for t in range(256):
        xb, _ = oracle.rmsnorm_q8k(x[t], L.ffn_norm, L.eps)
        idx, _, _, _ = oracle.route(L.router_w, L.bias, xb, 2)
        counts[idx] += 1
    c = np.sort(counts)[::-1]
    assert c[0] > 2.5 * c[-1]


def test_q6k_quantiser_layout_and_oracle_integer_sums(oracle):
    """Our Q6_K quantiser round-trips within 6-bit error, and the oracle's exact
    super-block integers equal a direct numpy restatement over the dequantised
    codes: total = sum_i sc[i/16] * (q_i - 32) * q8_i (GGUF Q6_K layout)."""
    from laii_b200 import synth
    from oracle.oracle import q8k_fields
    x = synth.normal_f32(256 * 16, seed=77, std=0.02)
    x[:256] = 0.0                                  # all-zero super-block: d = 0
    blocks = synth.quantize_q6k(x)
    assert blocks.size == 16 * synth.Q6K_BYTES
    y = synth.dequantize_q6k(blocks)
    assert np.array_equal(y[:256], np.zeros(256, np.float32))
    assert np.linalg.norm(y - x) / np.linalg.norm(x) < 0.03
    v = synth.normal_f32(256 * 16, seed=78, std=1.0)
    xq = oracle.quantize_q8k(v)
    acc, off, tot = oracle.q6k_row_ints(blocks, xq, x.size)
    _, qs, bs = q8k_fields(xq, 16)
    b = blocks.reshape(16, synth.Q6K_BYTES)
    sc = b[:, 192:208].copy().view(np.int8).astype(np.int64)
    d = b[:, 208:210].copy().view(np.float16).astype(np.float64).reshape(16)
    with np.errstate(invalid="ignore", divide="ignore"):
        codes = np.where(d[:, None] > 0, y.reshape(16, 256) / (d[:, None] * np.repeat(sc, 16, axis=1)), 0)
    q = np.rint(codes).astype(np.int64)            # q_i - 32
    want = (np.repeat(sc, 16, axis=1) * q * qs.astype(np.int64)).sum(axis=1)
    assert np.array_equal(tot.astype(np.int64), want)
    assert np.array_equal(off.astype(np.int64), (sc * bs.astype(np.int64)).sum(axis=1))
    assert np.array_equal(tot, acc - 32 * off)
