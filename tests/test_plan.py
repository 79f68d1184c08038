"""Planner parity: emugemm_plan must reproduce the reference planner (src/emugemm.cpp:216-282) exactly when
given the reference's constants (model "ref_mi250"): same chosen scheme, chunk count, reason string, and
bitwise-equal predicted_err / predicted_speedup. Also the plan invariants of bench/emugemm_test.cpp:35-61,
checked for both constant tables. No GPU needed."""
from __future__ import annotations

import csv
import ctypes
import math
import pathlib
import random

import pytest

import emugemm
import oracle

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "plan_ref_mi250.csv"


@pytest.fixture
def ref_model():
    emugemm.set_model("ref_mi250")
    yield
    emugemm.set_model("b200")


def _rows():
    with GOLDEN.open() as f:
        yield from csv.DictReader(f)


def _our_plan(M, N, K, tgt, force, a, b, rho, hints):
    req = emugemm.EmuRequest(tgt, force)
    hn = emugemm.EmuHints(a, b, 0, rho, 0)
    return emugemm.lib().emugemm_plan(M, N, K, ctypes.byref(req), ctypes.byref(hn) if hints else None)


def test_golden_fixture_present():
    rows = list(_rows())
    assert len(rows) > 1000
    reasons = {r["reason"] for r in rows}
    assert any(r.startswith("TARGET UNREACHABLE") for r in reasons)
    assert "robust, target above bf16x3 floor" in reasons


def test_plans_match_reference_golden(ref_model):
    mismatches = []
    for r in _rows():
        M, N, K = int(r["M"]), int(r["N"]), int(r["K"])
        tgt = float.fromhex(r["tgt"])
        a, b, rho = float.fromhex(r["a_absmax"]), float.fromhex(r["b_absmax"]), float.fromhex(r["rho"])
        p = _our_plan(M, N, K, tgt, int(r["force"]), a, b, rho, int(r["hints"]))
        got = (p.chosen, p.chunks, p.predicted_err.hex(), p.predicted_speedup.hex(), p.reason.decode())
        want = (int(r["chosen"]), int(r["chunks"]), r["predicted_err"], r["predicted_speedup"], r["reason"])
        if got != want:
            mismatches.append((r, got))
    assert not mismatches, f"{len(mismatches)} plan mismatches, first: {mismatches[:3]}"


@pytest.mark.skipif(not oracle.ref_available(), reason="reference planner not built (make -C oracle ref)")
def test_plans_match_live_reference_random(ref_model):
    rnd = random.Random(7)
    for _ in range(3000):
        M = rnd.choice([1, 17, 256, 1000, 2048, 4096, 8192, 30000])
        N = rnd.choice([1, 33, 256, 1024, 4096, 8192])
        K = rnd.choice([1, 7, 64, 1000, 4096, 8192, 60000, 262144, 1 << 20])
        tgt = 10 ** rnd.uniform(-8, -2) if rnd.random() < 0.9 else rnd.choice([0.0, -1.0])
        force = 0 if rnd.random() < 0.85 else rnd.randrange(1, 6)
        a = rnd.choice([-1.0, 0.0, 5e-5, 7e-5, 1.0, 65503.0, 65504.0, 1e6, 10 ** rnd.uniform(-6, 7)])
        b = rnd.choice([-1.0, 0.0, 1.0, 65504.0, 10 ** rnd.uniform(-6, 7)])
        rho = rnd.choice([-1.0, 0.0, 10 ** rnd.uniform(0, 6.5)])
        hints = rnd.random() < 0.95
        ref = oracle.ref_plan(M, N, K, tgt, force, a, b, rho, hints=hints)
        p = _our_plan(M, N, K, tgt, force, a, b, rho, hints)
        assert (p.chosen, p.chunks, p.reason.decode()) == (ref["chosen"], ref["chunks"], ref["reason"])
        assert p.predicted_err.hex() == ref["predicted_err"].hex()
        assert p.predicted_speedup.hex() == ref["predicted_speedup"].hex()


@pytest.mark.skipif(not oracle.ref_available(), reason="reference planner not built")
def test_model_functions_match_reference(ref_model):
    r = oracle.rlib()
    for s in range(1, 6):
        for K in (1, 100, 4096, 65536, 262144, 1 << 20):
            for c in (0, 1, 2, 4, 16, 64, 256, 1024):
                assert emugemm.lib().emugemm_model_err(s, K, c).hex() == r.emugemm_model_err(s, K, c).hex()
                for rho in (-1.0, 0.0, 3.5, 1e4):
                    assert (emugemm.lib().emugemm_model_err_rho(s, K, c, rho).hex() ==
                            r.emugemm_model_err_rho(s, K, c, rho).hex())
            for c in (1, 3, 4, 5, 16, 17, 64, 65, 256, 257):
                assert emugemm.lib().emugemm_model_speed(s, c).hex() == r.emugemm_model_speed(s, c).hex()
    assert math.isnan(emugemm.lib().emugemm_model_err(9, 10, 1))


# The named rows of the planner table quoted for the benchmark configurations (reference constants).
KNOWN = [
    ((1024, 1024, 1024), 1e-5, (1.0, 1.0, 24.0), 0, "NATIVE_FP32", 1, 6.7125e-07, "native fp32 suffices"),
    ((1024, 1024, 1024), 1e-5, (1.0, 1.0, 24.0), 3, "BF16X3", 1, 5.2087e-06, "forced"),
    ((8192, 8192, 8192), 1e-5, (4.19e6, 1.0, -1.0), 0, "BF16X3", 1, 4.5089e-06, "robust, target above bf16x3 floor"),
    ((8192, 8192, 8192), 1e-5, (1.0, 1.0, -1.0), 0, "BF16X3", 1, 4.5089e-06, "robust, target above bf16x3 floor"),
    ((256, 256, 65536), 1e-7, (1.0, 1.0, 192.0), 0, "FP32_CHUNKED", 256, 3.3563e-07, "TARGET UNREACHABLE"),
    ((256, 256, 262144), 1e-6, (1.0, 1.0, 384.0), 0, "FP32_CHUNKED", 128, 9.4929e-07, "target below bf16x3 floor"),
    ((2048, 2048, 8192), 1e-5, (4.0, 4.0, 1e4), 0, "FP32_CHUNKED", 256, 1.7480e-05, "TARGET UNREACHABLE"),
    ((4096, 4096, 1048576), 1e-5, (5.0, 5.0, -1.0), 0, "FP16X3", 1, 9.1719e-06, "fp16 range safe"),
]


@pytest.mark.parametrize("case", KNOWN, ids=[f"{c[0]}-{c[4]}" for c in KNOWN])
def test_known_plans(ref_model, case):
    (M, N, K), tgt, (a, b, rho), force, chosen, chunks, perr, reason = case
    p = emugemm.plan(M, N, K, tgt, force, a, b, rho)
    assert emugemm.SCHEME_NAMES[p.chosen] == chosen
    assert p.chunks == chunks
    assert p.predicted_err == pytest.approx(perr, rel=1e-4)
    assert p.reason.decode().startswith(reason)


@pytest.mark.parametrize("model", ["ref_mi250", "b200"])
def test_plan_invariants(model):
    """bench/emugemm_test.cpp:35-61: no plan claims an error above the target unless it says UNREACHABLE;
    no plan is slower than native when native meets the target; bf16x3 never below its floor."""
    emugemm.set_model(model)
    try:
        bad = 0
        for K in (4096, 65536, 262144):
            for tg in (1e-4, 1e-5, 4e-6, 1e-6, 1e-7):
                p = emugemm.plan(4096, 4096, K, tg, 0, 1.0, 1.0, 0.0)
                unreachable = b"UNREACHABLE" in p.reason
                if not unreachable and p.predicted_err > tg * 1.0001:
                    bad += 1
                native_ok = emugemm.lib().emugemm_model_err(emugemm.NATIVE_FP32, K, 1) <= tg
                if native_ok and p.predicted_speedup < 0.999:
                    bad += 1
        p = emugemm.plan(4096, 4096, 262144, 1e-6, 0, 1e6, 1e6, 0.0)
        assert p.chosen != emugemm.BF16X3
        assert bad == 0
    finally:
        emugemm.set_model("b200")


def test_set_model_rejects_unknown():
    with pytest.raises(emugemm.EmuGemmError):
        emugemm.set_model("mi300")
    assert emugemm.get_model() == "b200"
