"""The C shim of INTEGRATION.md, as laii would compile and call it.

CPU: the shim block compiles as C11 against the reference's own sources
(tools/lfm2_moe_checkpoint.c, tools/lfm2_prefill_batch.c) with the warnings that
would mean a wrong signature or type turned into errors, and the check library
the oracle build links with liblfm_gpu_moe.so exports its calls.
GPU: through the shim only -- lfm2_gpu_moe_bind, the drop-in
lfm2_forward_moe_ffn_gpu (one call per token, the signature of
lfm2_forward_moe_ffn_1x4, tools/lfm2_moe_checkpoint.c:312-320) and the batched
slot lfm2_forward_moe_ffn_batch_gpu on an LFM2BatchState (tools/lfm2_prefill_batch.c:1100-1120,
the B = 1 + K speculative-verify batch of tools/lfm2_speculative_pld.c:508) --
against the reference's CPU path on the same layer and rows: rel-L2 <= 1e-3,
max-abs <= 5e-3.
"""
import ctypes
import os
import subprocess

import numpy as np
import pytest

from conftest import ROOT, cached_dense, cached_layer, rel_l2

SHIM_SO = os.path.join(ROOT, "oracle", "_ref", "libshim_check.so")
REL_L2, MAX_ABS = 1e-3, 5e-3


def _reference_dir():
    import __graft_entry__
    return __graft_entry__.reference_dir()


def test_shim_block_compiles_against_the_reference(tmp_path):
    ref = _reference_dir()
    if not ref:
        pytest.skip("reference sources absent")
    from oracle.extract_shim import shim_source
    (tmp_path / "lfm_gpu_moe_shim.c").write_text(shim_source())
    cmd = ["gcc", "-std=c11", "-O0", "-mavx2", "-mfma", "-mf16c", "-D_GNU_SOURCE", "-fsyntax-only",
           "-Wno-unused-function", "-Wno-unused-variable", "-Wno-unused-but-set-variable",
           "-Werror=implicit-function-declaration", "-Werror=incompatible-pointer-types", "-Werror=int-conversion",
           f"-I{ref}", f"-I{ref}/include", f"-I{ROOT}/include", f"-I{tmp_path}",
           os.path.join(ROOT, "oracle", "shim_harness.c")]
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    assert r.returncode == 0, r.stdout[-3000:]


def test_shim_check_library_exports_its_calls():
    if not os.path.exists(SHIM_SO):
        pytest.skip("oracle/_ref/libshim_check.so not built (reference sources absent)")
    out = subprocess.run(["nm", "-D", "--defined-only", SHIM_SO], stdout=subprocess.PIPE, text=True).stdout
    names = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert {"shim_bind", "shim_forward_1x4", "shim_forward_batch", "shim_release"} <= names
    lib = ctypes.CDLL(SHIM_SO)
    lib.shim_max_batch.restype = ctypes.c_int
    assert lib.shim_max_batch() >= 8


def _shim():
    if not os.path.exists(SHIM_SO):
        pytest.skip("oracle/_ref/libshim_check.so not built")
    lib = ctypes.CDLL(SHIM_SO)
    vp, u32, f32 = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_float
    lib.shim_bind.restype = ctypes.c_int
    lib.shim_bind.argtypes = [u32, u32, u32, u32, u32, f32, vp, vp, vp, vp, vp, vp, u32]
    lib.shim_forward_1x4.argtypes = [u32, vp, u32, u32, f32]
    lib.shim_forward_batch.restype = ctypes.c_int
    lib.shim_forward_batch.argtypes = [u32, vp, u32]
    return lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _close(got, want):
    assert np.isfinite(got).all()
    assert rel_l2(got, want) <= REL_L2
    assert float(np.abs(got.astype(np.float64) - want).max()) <= MAX_ABS


@pytest.mark.gpu
def test_shim_drop_in_and_batched_slot_against_reference(reference):
    from laii_b200 import synth
    lib = _shim()
    D, E, K, I = 2048, 32, 4, 1792
    L = cached_layer(D, E, K, I)
    Ld = cached_dense(D, 7168)
    try:
        assert lib.shim_bind(3, D, E, K, I, L.eps, _p(L.ffn_norm), _p(L.router_w), _p(L.bias), _p(L.gate),
                             _p(L.up), _p(L.down), 12) == 1
        assert lib.shim_bind(0, D, 0, 0, 7168, Ld.eps, _p(Ld.ffn_norm), None, None, _p(Ld.gate), _p(Ld.up),
                             _p(Ld.down), 12) == 1
        x = synth.make_hidden(8, D, seed_offset=91)
        want = reference.moe_forward(L, x)[0]
        # the drop-in, one call per token as the decode loop makes them
        got1 = np.array(x[:2], copy=True)
        lib.shim_forward_1x4(3, _p(got1), 2, D, L.eps)
        _close(got1, want[:2])
        # the batched slot: a speculative-verify batch of 8 rows in one call
        gotb = np.array(x, copy=True)
        assert lib.shim_forward_batch(3, _p(gotb), 8) == 1
        _close(gotb, want)
        # a dense layer bound and run through the same drop-in
        gotd = np.array(x[:3], copy=True)
        lib.shim_forward_1x4(0, _p(gotd), 3, D, Ld.eps)
        _close(gotd, reference.dense_forward(Ld, x[:3]))
    finally:
        lib.shim_release()
