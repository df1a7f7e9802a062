"""lfm_gpu_moe_forward_noalloc (fixed static scratch, no allocation) through the C-ABI.

Collected last on purpose: it must pass alone and after every other test has
used (and grown) the handle's regular scratch on the same device.
"""
import ctypes

import numpy as np
import pytest

from conftest import cached_dense, cached_layer, rel_l2

pytestmark = pytest.mark.gpu

REL_L2, MAX_ABS = 1e-3, 5e-3


def _noalloc(lib, handle, layer, xt, T, stream):
    return lib.lfm_gpu_moe_forward_noalloc(handle, layer, ctypes.c_void_p(xt.data_ptr()), T, ctypes.c_void_p(stream))


@pytest.mark.parametrize("T", [1, 8, 58])
def test_noalloc_matches_forward_twice_in_a_row(T):
    torch = pytest.importorskip("torch")
    from laii_b200 import _native, synth
    from laii_b200.moe import GpuMoE
    lib = _native.load_gpu()
    D, E, K, I = 2048, 32, 4, 1792
    with GpuMoE(0) as g:
        g.upload_layer(0, cached_layer(D, E, K, I))
        x0 = synth.make_hidden(T, D, seed_offset=77)
        stream = torch.cuda.current_stream().cuda_stream
        ref = torch.from_numpy(np.array(x0, copy=True)).cuda()
        out = torch.from_numpy(np.array(x0, copy=True)).cuda()
        for _ in range(2):  # two calls in a row, each compared after the step
            g.forward_device(0, ref.data_ptr(), T, stream=stream)
            st = _noalloc(lib, g._h, 0, out, T, stream)
            assert st == 0, lib.lfm_gpu_moe_last_error(g._h)
            torch.cuda.synchronize()
            g.sync()
            a, b = out.cpu().numpy(), ref.cpu().numpy()
            assert rel_l2(a, b) <= REL_L2
            assert float(np.abs(a - b).max()) <= MAX_ABS


def test_noalloc_dense_layer():
    torch = pytest.importorskip("torch")
    from laii_b200 import _native, synth
    from laii_b200.moe import GpuMoE
    lib = _native.load_gpu()
    D, I, T = 2048, 7168, 4
    with GpuMoE(0) as g:
        g.upload_dense(1, cached_dense(D, I))
        x0 = synth.make_hidden(T, D, seed_offset=78)
        stream = torch.cuda.current_stream().cuda_stream
        ref = torch.from_numpy(np.array(x0, copy=True)).cuda()
        out = torch.from_numpy(np.array(x0, copy=True)).cuda()
        for _ in range(2):
            g.forward_device(1, ref.data_ptr(), T, stream=stream)
            assert _noalloc(lib, g._h, 1, out, T, stream) == 0, lib.lfm_gpu_moe_last_error(g._h)
            torch.cuda.synchronize()
            g.sync()
            a, b = out.cpu().numpy(), ref.cpu().numpy()
            assert rel_l2(a, b) <= REL_L2
            assert float(np.abs(a - b).max()) <= MAX_ABS


def test_noalloc_rejects_scratch_above_its_limit():
    torch = pytest.importorskip("torch")
    from laii_b200 import _native
    from laii_b200.moe import GpuMoE
    lib = _native.load_gpu()
    D, E, K, I = 2048, 32, 4, 1792
    with GpuMoE(0) as g:
        g.upload_layer(0, cached_layer(D, E, K, I))
        xt = torch.zeros(64, D, device="cuda")
        st = _noalloc(lib, g._h, 0, xt, 64, 0)  # 64 tokens need ~4.6 MB > 4 MiB
        assert st == -2
        assert b"above its fixed" in lib.lfm_gpu_moe_last_error(g._h)
        assert _noalloc(lib, g._h, 5, xt, 1, 0) == -3   # layer not uploaded
        assert float(xt.abs().sum()) == 0.0             # nothing ran


def test_noalloc_refuses_an_expert_shard():
    """A shard layer keeps the full router but only its own experts' weights, so
    routing it here would read past the shard: the call refuses it on the host."""
    torch = pytest.importorskip("torch")
    from laii_b200 import _native, synth
    from laii_b200.moe import GpuMoE
    lib = _native.load_gpu()
    D, E, K, I, T = 512, 8, 2, 512, 4
    L = synth.make_moe_layer(D, E, K, I, layer=0)
    with GpuMoE(0) as g:
        g.upload_layer_shard(3, L, 2, 4)
        x0 = synth.make_hidden(T, D, seed_offset=79)
        xt = torch.from_numpy(np.array(x0, copy=True)).cuda()
        st = _noalloc(lib, g._h, 3, xt, T, 0)
        assert st == -2
        assert b"expert shard" in lib.lfm_gpu_moe_last_error(g._h)
        torch.cuda.synchronize()
        assert np.array_equal(xt.cpu().numpy(), x0)      # x untouched
