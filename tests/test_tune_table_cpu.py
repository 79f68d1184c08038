"""The tile tuner's table bookkeeping (no GPU): rows already present are skipped on resume, and --replace drops the
rows of the dtypes being measured again while the header and every other row stay in place."""
from __future__ import annotations

import importlib.util
import pathlib

ROOT = pathlib.Path(__file__).resolve().parent.parent


def _tuner():
    spec = importlib.util.spec_from_file_location("tune_tiles", ROOT / "emugemm-cdna_b200" / "tune_tiles.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_drop_rows_keeps_header_and_other_dtypes(tmp_path):
    tt = _tuner()
    table = tmp_path / "tiles.csv"
    rows = ["sm_100a,12.8,1024,1024,1024,bf16,4,0.04,0.041,1.02\n",
            "sm_100a,12.8,1024,1024,1024,fp16,1,0.06,0.06,1.00\n",
            "sm_100a,12.8,1024,1024,1024,fp32,64,0.09,0.087,0.96\n",
            "sm_100a,12.8,2048,1024,4096,bf16,2,0.09,0.09,1.00\n"]
    table.write_text(tt.HEADER + "".join(rows))
    assert tt.existing_keys(table) == {(1024, 1024, 1024, "bf16"), (1024, 1024, 1024, "fp16"),
                                       (1024, 1024, 1024, "fp32"), (2048, 1024, 4096, "bf16")}
    tt.drop_rows(table, {"bf16", "fp16"})
    assert table.read_text() == tt.HEADER + rows[2]
    assert tt.existing_keys(table) == {(1024, 1024, 1024, "fp32")}
    tt.append_row(table, rows[0])
    assert table.read_text() == tt.HEADER + rows[2] + rows[0]


def test_append_row_writes_header_once(tmp_path):
    tt = _tuner()
    table = tmp_path / "new.csv"
    tt.append_row(table, "sm_100a,12.8,1,1,1,bf16,1,0.1,0.1,1.0\n")
    tt.append_row(table, "sm_100a,12.8,2,2,2,bf16,2,0.1,0.1,1.0\n")
    lines = table.read_text().splitlines()
    assert lines[0] + "\n" == tt.HEADER and len(lines) == 3


def test_committed_table_rows_are_valid():
    """Every row of the committed B200 table: the arch of this build, a known dtype and a tile code its kernels have."""
    tt = _tuner()
    path = ROOT / "emugemm-cdna_b200" / "tiles_b200.csv"
    keys = tt.existing_keys(path)
    assert len(keys) == 261
    codes = {"bf16": {1, 2, 3, 4}, "fp16": {1, 2, 3}, "fp32": {16, 32, 64, 128, 3264}}
    for line in path.read_text().splitlines()[1:]:
        f = line.split(",")
        assert f[0] == "sm_100a" and f[5] in codes and int(f[6]) in codes[f[5]], line
