"""The C-ABI library loads and exports every symbol include/ds4f/gpu_cuda.h
declares (no GPU needed; no compute calls)."""
import ctypes as C
import os
import subprocess

import pytest

from tests._lib import ROOT, ds4f_cuda, gpu_available

dc = ds4f_cuda()


def test_library_exports_every_header_symbol():
    names = dc.header_symbols()
    assert len(names) >= 25
    L = C.CDLL(dc.LIB_PATH)
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_reference_shim_symbols_present():
    # the four symbols of the reference's include/ds4f/gpu.h:22-52
    L = C.CDLL(dc.LIB_PATH)
    for n in ("ds4f_gpu_init", "ds4f_gpu_free", "ds4f_gpu_mlx4_matvec",
              "ds4f_gpu_mlx4_batch"):
        assert hasattr(L, n)


def test_header_compiles_as_c99(tmp_path):
    src = tmp_path / "t.c"
    src.write_text('#include "ds4f/gpu_cuda.h"\nint main(void){return 0;}\n')
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-c",
                    "-I", os.path.join(ROOT, "include"), str(src), "-o",
                    str(tmp_path / "t.o")], check=True)


def test_sm100a_code_only():
    out = subprocess.run(["cuobjdump", "--list-elf", dc.LIB_PATH],
                         capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("cuobjdump unavailable")
    assert "sm_100a" in out.stdout


@pytest.mark.skipif(gpu_available(), reason="checks the no-GPU error path")
def test_init_fails_loudly_without_gpu():
    L = dc.lib()
    assert L.ds4f_gpu_init() == -1
    assert b"CUDA" in L.ds4f_gpu_last_error() or b"device" in L.ds4f_gpu_last_error()
