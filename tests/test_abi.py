"""The C-ABI library: it loads without a GPU and exports exactly what the header declares."""
import ctypes
import os
import subprocess

import pytest

from laii_b200 import _native, build


def test_library_builds_for_sm100a_and_loads():
    so = build.build_gpu()
    assert os.path.exists(so)
    lib = _native.load_gpu()
    assert lib is not None


def test_exports_every_header_function():
    lib = _native.load_gpu()
    declared = _native.header_functions()
    assert len(declared) >= 12
    for name in declared:
        assert hasattr(lib, name), name
    bound = {n for n, _, _ in _native.GPU_API}
    assert set(declared) <= bound, "every declared entry point has a ctypes binding"
    out = subprocess.run(["nm", "-D", "--defined-only", build.GPU_SO], stdout=subprocess.PIPE, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert {n for n in exported if n.startswith("lfm_gpu_moe")} == set(declared)


def test_no_cpu_fallback_without_gpu():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = _native.load_gpu()
    h = ctypes.c_void_p()
    assert lib.lfm_gpu_moe_create(ctypes.byref(h), 0) == -1
    assert not h.value
    from laii_b200.moe import GpuMoE, MoEError
    with pytest.raises(MoEError):
        GpuMoE(0)


def test_null_handle_is_an_error_not_a_crash():
    lib = _native.load_gpu()
    assert lib.lfm_gpu_moe_forward(None, 0, None, 1, 0, None) == -1
    assert lib.lfm_gpu_moe_sync(None) == -1
    assert lib.lfm_gpu_moe_last_error(None) == b"null handle"
    lib.lfm_gpu_moe_destroy(None)


def test_header_compiles_as_c11(tmp_path):
    src = tmp_path / "t.c"
    src.write_text('#include "lfm_gpu_moe.h"\nint main(void){lfm_gpu_moe_t *h = 0; (void)h; return LFM_GPU_OK;}\n')
    inc = os.path.join(build.ROOT, "include")
    r = subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I", inc, "-c", str(src), "-o", str(tmp_path / "t.o")],
                       stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    assert r.returncode == 0, r.stdout
