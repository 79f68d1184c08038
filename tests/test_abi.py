"""The C ABI without a GPU: libemugemm.so loads, exports every function include/emugemm.h declares, keeps the
reference's struct layouts, and fails loudly (never falls back to the CPU) when no sm_100 device exists.
The tile-table loader's arch rejection (src/emugemm.cpp:107-128) is exercised with an explicit arch."""
from __future__ import annotations

import ctypes
import pathlib
import subprocess
import sys

import pytest

import emugemm


def test_library_exports_every_header_function():
    names = emugemm.header_functions()
    assert len(names) >= 25
    lib = emugemm.lib()
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_reference_symbols_present():
    lib = emugemm.lib()
    for n in ("emugemm_init", "emugemm_shutdown", "emugemm_plan", "emugemm_sgemm", "emugemm_model_err",
              "emugemm_model_err_rho", "emugemm_estimate_rho", "emugemm_model_speed"):
        assert hasattr(lib, n)


def test_struct_layouts_match_reference():
    # src/emugemm.h:46-71: {double,int}, {float,float,int,float,int}, {enum,int,double,double,char*}.
    assert ctypes.sizeof(emugemm.EmuRequest) == 16
    assert ctypes.sizeof(emugemm.EmuHints) == 20
    assert emugemm.EmuPlan.predicted_err.offset == 8
    assert emugemm.EmuPlan.reason.offset == 24
    assert ctypes.sizeof(emugemm.EmuPlan) == 32


def test_header_compiles_as_c_and_cpp(tmp_path):
    src = tmp_path / "t.c"
    src.write_text('#define EMUGEMM_ROCBLAS_COMPAT\n#include "emugemm.h"\n'
                   'int main(void){ emu_plan_t p; rocblas_handle h = 0; (void)h; p.chunks = 1; return p.chunks - 1; }\n')
    inc = str(emugemm.HEADER.parent)
    for cc, extra in (("gcc", ["-x", "c"]), ("g++", ["-x", "c++"])):
        r = subprocess.run([f"/usr/bin/{cc}", *extra, "-Wall", "-Werror", "-I", inc, "-c", str(src), "-o",
                            str(tmp_path / f"t_{cc}.o")], capture_output=True, text=True)
        assert r.returncode == 0, r.stderr


def test_status_strings():
    lib = emugemm.lib()
    assert lib.emugemm_status_string(0) == b"success"
    assert lib.emugemm_status_string(101) == b"device wait timed out"


def test_no_cpu_fallback_without_sm100():
    """Without a B200 the library refuses to create a handle; it never computes on the host."""
    code = ("import sys; sys.path.insert(0, %r); import emugemm, ctypes\n"
            "h = ctypes.c_void_p()\n"
            "print(emugemm.lib().emugemm_create_handle(ctypes.byref(h)))\n" % str(emugemm.HERE))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    import torch

    if torch.cuda.is_available() and torch.cuda.get_device_capability(0) == (10, 0):
        pytest.skip("an sm_100 device is present")
    assert r.returncode == 0, r.stderr
    assert int(r.stdout.strip().splitlines()[-1]) in (6, 100)   # INTERNAL_ERROR (no device) or ARCH_MISMATCH


def test_sgemm_rejects_null_handle():
    lib = emugemm.lib()
    req = emugemm.EmuRequest(1e-5, 0)
    assert lib.emugemm_sgemm(None, 4, 4, 4, 0, 0, 0, ctypes.byref(req), None, None) == 1


def test_tune_table_arch_rejection(tmp_path):
    lib = emugemm.lib()
    csv = tmp_path / "tiles.csv"
    csv.write_text(
        "arch,cuda_version,M,N,K,dtype,tile,best_ms,default_ms,gain\n"
        "sm_100a,12.9,8192,8192,8192,bf16,2,2.5,2.6,1.04\n"
        "sm_100a,12.9,256,256,262144,fp32,64,1.0,1.2,1.2\n"
        "sm_90a,12.9,8192,8192,8192,bf16,1,2.5,2.6,1.04\n"
        "gfx90a:sramecc+:xnack-,5.2.0,8192,8192,8192,bf16,-606629811,8.0,8.1,1.01\n"
        "garbage line\n")
    assert lib.emugemm_init_for_arch(str(csv).encode(), b"sm_100a") == 0
    assert lib.emugemm_tune_rows() == 2
    assert lib.emugemm_tune_lookup(8192, 8192, 8192, 1) == 2
    assert lib.emugemm_tune_lookup(6000, 8192, 8192, 1) == 2      # within log2 distance 1
    assert lib.emugemm_tune_lookup(1024, 1024, 1024, 1) == 0      # too far: built-in choice
    assert lib.emugemm_tune_lookup(256, 256, 262144, 0) == 64
    assert lib.emugemm_init_for_arch(str(csv).encode(), b"gfx90a:sramecc+:xnack-") == 0
    assert lib.emugemm_tune_rows() == 1
    assert lib.emugemm_init_for_arch(str(tmp_path / "missing.csv").encode(), b"sm_100a") == 0
    assert lib.emugemm_tune_rows() == 0
    lib.emugemm_shutdown()


def test_reference_table_is_rejected_on_b200():
    """The reference's own gfx90a table (820 rows) must be refused wholesale for sm_100a."""
    import pathlib

    from conftest import REF_ROOT

    ref_csv = REF_ROOT / "data" / "tune_table.csv"
    if not ref_csv.exists():
        pytest.skip("reference tree not present")
    lib = emugemm.lib()
    assert lib.emugemm_init_for_arch(str(ref_csv).encode(), b"sm_100a") == 0
    assert lib.emugemm_tune_rows() == 0
    assert lib.emugemm_init_for_arch(str(ref_csv).encode(), b"gfx90a:sramecc+:xnack-") == 0
    assert lib.emugemm_tune_rows() == 820
    lib.emugemm_shutdown()


def test_committed_b200_tile_table():
    """The per-shape B200 table that tune_tiles.py measured: every row valid for sm_100a, rejected for another
    arch, and the lookup returns the measured winners."""
    lib = emugemm.lib()
    table = str(pathlib.Path(__file__).resolve().parent.parent / "emugemm-cdna_b200" / "tiles_b200.csv")
    try:
        assert lib.emugemm_init_for_arch(table.encode(), b"sm_100a") == 0
        assert lib.emugemm_tune_rows() == 261
        assert lib.emugemm_tune_lookup(1024, 1024, 1024, 1) == 4         # bf16x3: A split into TMEM
        assert lib.emugemm_tune_lookup(1024, 1024, 16384, 1) == 2        # bf16x3: CTA pairs
        assert lib.emugemm_tune_lookup(8192, 8192, 4096, 2) == 2         # fp16x3: CTA pairs (scaled accumulator)
        assert lib.emugemm_tune_lookup(1024, 1024, 4096, 2) == 1         # fp16x3, 16 pair tiles: single CTA
        assert lib.emugemm_tune_lookup(1024, 2048, 4096, 0) == 128       # FP32 tile edge
        assert lib.emugemm_init_for_arch(table.encode(), b"sm_90a") == 0
        assert lib.emugemm_tune_rows() == 0
    finally:
        lib.emugemm_shutdown()
