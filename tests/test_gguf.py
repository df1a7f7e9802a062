"""GGUF checkpoints: the library's own GGUF v3 reader binds blocks as the
reference's loader + lfm2_bind_moe_layer do (tools/lfm2_loader.c,
tools/lfm2_moe_checkpoint.c:70-102).

CPU: files written with the gguf package (a dense block, a MoE block with
exp_probs_b.bias, a MoE block with the bare exp_probs_b name) are described
without a GPU; malformed files are refused.  GPU: the uploaded layers compute
bit for bit what upload_layer/upload_dense of the same arrays compute, and an
expert shard holds the same bytes as that slice of the full layer.
"""
import numpy as np
import pytest

from laii_b200 import synth
from laii_b200.moe import GpuMoE, MoEError, gguf_describe

D, E, K, I, DI = 512, 8, 2, 512, 768


def _layers():
    dense = synth.make_dense_layer(D, DI, layer=1)
    m1 = synth.make_moe_layer(D, E, K, I, layer=2)
    m2 = synth.make_moe_layer(D, E, K, I, layer=3)
    return dense, m1, m2


def _write(path, dense, m1, m2, drop=None, eps=1e-5):
    gguf = pytest.importorskip("gguf")
    Q4K = gguf.GGMLQuantizationType.Q4_K
    Q6K = gguf.GGMLQuantizationType.Q6_K
    w = gguf.GGUFWriter(str(path), "lfm2moe")
    w.add_uint32("lfm2moe.block_count", 3)
    w.add_uint32("lfm2moe.expert_count", E)
    w.add_uint32("lfm2moe.expert_used_count", K)
    w.add_float32("lfm2moe.attention.layer_norm_rms_epsilon", eps)
    w.add_string("general.note", "synthetic lfm2moe FFN stack")

    def q4k(name, arr, shape):
        if name != drop:
            w.add_tensor(name, np.ascontiguousarray(arr, dtype=np.uint8).reshape(shape), raw_dtype=Q4K)

    def f32(name, arr):
        if name != drop:
            w.add_tensor(name, np.ascontiguousarray(arr, dtype=np.float32))

    def down_exps(name, m):  # Q4_K, or Q6_K as Q4_K_M files store some ffn_down_exps
        if name == drop:
            return
        if m.down_type == 14:
            w.add_tensor(name, np.ascontiguousarray(m.down, dtype=np.uint8).reshape(E, D, I // 256 * 210),
                         raw_dtype=Q6K)
        else:
            q4k(name, m.down, (E, D, I // 256 * 144))

    nb, nbi, nbd = D // 256 * 144, I // 256 * 144, DI // 256 * 144
    f32("blk.0.ffn_norm.weight", dense.ffn_norm)
    q4k("blk.0.ffn_gate.weight", dense.gate, (DI, nb))
    q4k("blk.0.ffn_up.weight", dense.up, (DI, nb))
    q4k("blk.0.ffn_down.weight", dense.down, (D, nbd))
    for l, m, bias_name in ((1, m1, "exp_probs_b.bias"), (2, m2, "exp_probs_b")):
        f32(f"blk.{l}.ffn_norm.weight", m.ffn_norm)
        f32(f"blk.{l}.ffn_gate_inp.weight", m.router_w)
        f32(f"blk.{l}.{bias_name}", m.bias)
        q4k(f"blk.{l}.ffn_gate_exps.weight", m.gate, (E, I, nb))
        q4k(f"blk.{l}.ffn_up_exps.weight", m.up, (E, I, nb))
        down_exps(f"blk.{l}.ffn_down_exps.weight", m)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


@pytest.fixture(scope="module")
def stack(tmp_path_factory):
    dense, m1, m2 = _layers()
    path = tmp_path_factory.mktemp("gguf") / "lfm2moe-ffn.gguf"
    _write(path, dense, m1, m2)
    return path, dense, m1, m2


def test_describe_binds_dense_and_moe_blocks(stack):
    path = stack[0]
    b0, n = gguf_describe(path, 0)
    assert n == 3
    assert b0 == {"kind": "dense", "D": D, "E": 1, "K": 1, "I": DI, "eps": pytest.approx(1e-5), "has_bias": False,
                  "has_norm": True, "down_type": 12}
    for l in (1, 2):  # exp_probs_b.bias and the bare exp_probs_b name both bind
        b, _ = gguf_describe(path, l)
        assert (b["kind"], b["D"], b["E"], b["K"], b["I"], b["has_bias"]) == ("moe", D, E, K, I, True)
    b3, _ = gguf_describe(path, 3)
    assert b3["kind"] == "none"


def test_describe_refuses_incomplete_and_truncated_files(tmp_path):
    dense, m1, m2 = _layers()
    p = tmp_path / "no-up.gguf"
    _write(p, dense, m1, m2, drop="blk.1.ffn_up_exps.weight")
    with pytest.raises(MoEError) as ei:
        gguf_describe(p, 1)
    assert ei.value.status == -2 and "incomplete MoE" in str(ei.value)
    good = tmp_path / "good.gguf"
    _write(good, dense, m1, m2)
    cut = tmp_path / "cut.gguf"
    cut.write_bytes(good.read_bytes()[:-1000])
    with pytest.raises(MoEError) as ei:
        gguf_describe(cut, 1)
    assert ei.value.status == -1
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"NOTGGUF" + bytes(64))
    with pytest.raises(MoEError):
        gguf_describe(bad, 0)


@pytest.fixture(scope="module")
def stack_q6k(tmp_path_factory):
    """Block 2's ffn_down_exps stored as Q6_K."""
    dense, m1, _ = _layers()
    m2 = synth.make_moe_layer(D, E, K, I, layer=3, down_type=14)
    path = tmp_path_factory.mktemp("gguf") / "lfm2moe-ffn-q6k.gguf"
    _write(path, dense, m1, m2)
    return path, dense, m1, m2


def test_describe_binds_q6k_down_experts(stack_q6k):
    path = stack_q6k[0]
    b1, _ = gguf_describe(path, 1)
    b2, _ = gguf_describe(path, 2)
    assert (b1["kind"], b1["down_type"]) == ("moe", 12)
    assert (b2["kind"], b2["D"], b2["E"], b2["I"], b2["down_type"]) == ("moe", D, E, I, 14)


@pytest.mark.gpu
def test_upload_gguf_q6k_down_matches_upload_of_the_same_arrays(stack_q6k):
    path, dense, m1, m2 = stack_q6k
    x = synth.make_hidden(24, D, seed_offset=5)
    with GpuMoE(0) as ref:
        ref.upload_dense(0, dense)
        ref.upload_layer(1, m1)
        ref.upload_layer(2, m2)
        want = ref.forward_stack(0, 3, np.array(x, copy=True))
    with GpuMoE(0) as g:
        assert g.upload_gguf(path) == 3
        got = g.forward_stack(0, 3, np.array(x, copy=True))
        with pytest.raises(MoEError, match="Q4_K down"):
            g.upload_gguf(path, first_block=2, n_blocks=1, expert_first=0, n_local=4)
    assert np.array_equal(got, want)


@pytest.mark.gpu
def test_upload_gguf_matches_upload_of_the_same_arrays(stack):
    path, dense, m1, m2 = stack
    x = synth.make_hidden(24, D, seed_offset=4)
    with GpuMoE(0) as ref:
        ref.upload_dense(0, dense)
        ref.upload_layer(1, m1)
        ref.upload_layer(2, m2)
        want = ref.forward_stack(0, 3, np.array(x, copy=True))
        want1 = ref.forward(1, np.array(x[:3], copy=True))
    with GpuMoE(0) as g:
        assert g.upload_gguf(path) == 3
        got = g.forward_stack(0, 3, np.array(x, copy=True))
        got1 = g.forward(1, np.array(x[:3], copy=True))
    assert np.array_equal(got, want)
    assert np.array_equal(got1, want1)


@pytest.mark.gpu
def test_upload_gguf_expert_shard_holds_the_slice(stack):
    path, dense, m1, m2 = stack
    per_gu = I * (D // 256) * 144
    with GpuMoE(0) as g:
        assert g.upload_gguf(path, first_block=1, n_blocks=1, expert_first=3, n_local=2) == 1
        part = g.read_layer(0, "gate", 2 * per_gu)
        assert np.array_equal(part, m1.gate.reshape(-1)[3 * per_gu:5 * per_gu])


def _raw_gguf(path, ne, offset=0, type_=12):
    """A GGUF v3 file with one tensor "blk.0.attn_q.weight" of the given dims, type and data offset."""
    import struct
    name = b"blk.0.attn_q.weight"
    b = b"GGUF" + struct.pack("<IQQ", 3, 1, 0)
    b += struct.pack("<Q", len(name)) + name + struct.pack("<I", len(ne)) + struct.pack(f"<{len(ne)}Q", *ne)
    b += struct.pack("<IQ", type_, offset)
    b += bytes((-len(b)) % 32) + bytes(4096)
    path.write_bytes(b)
    return path


def test_describe_refuses_shapes_and_offsets_that_wrap(tmp_path):
    """Dims and offsets come from the file: a product or a sum that wraps 64 bits
    must not pass the end-of-file check."""
    cases = {
        "wrap.gguf": ([(1 << 32) - 256, (1 << 32) - 1, (1 << 32) - 1], 0),   # Q4_K bytes wrap
        "huge-dim.gguf": ([256, 1 << 40], 0),                                # a dim above 2^32
        "zero-dim.gguf": ([256, 0], 0),
        "offset.gguf": ([256, 1], (1 << 64) - 16),                           # data0 + offset wraps
    }
    for name, (ne, off) in cases.items():
        p = _raw_gguf(tmp_path / name, ne, off)
        with pytest.raises(MoEError) as ei:
            gguf_describe(p, 0)
        assert ei.value.status == -1, name
    ok = _raw_gguf(tmp_path / "ok.gguf", [256, 16])   # 16 rows x 144 B fit in the 4 KiB of data
    b, n = gguf_describe(ok, 0)
    assert (b["kind"], n) == ("none", 1)
