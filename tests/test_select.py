"""The B200 selection table (tilec_b200/mm_select.json) and its loader (CPU only)."""
import json
import os

import pytest

from tilec_b200 import _native, select, tune


def test_committed_table_is_valid_and_fp32_class():
    rows = select.load_table(select.TABLE_PATH)
    assert rows, "mm_select.json is missing or empty"
    names = {_native.VARIANT_NAMES[r[6]] for r in rows}
    assert names <= set(tune.FP32_CLASS), "AUTO may only pick fp32-accurate variants"
    with open(select.TABLE_PATH) as f:
        doc = json.load(f)
    assert doc["heldout"]["shapes"] > 0
    # the grid covers every log2 size up to 2^63 in each dimension
    for m, n, k in [(1, 1, 1), (512, 64, 4096), (65536, 8192, 8192), (3, 777, 3001), (2 ** 40, 2, 2)]:
        assert select.lookup(rows, m, n, k) is not None


def test_lookup_first_match_wins(tmp_path):
    p = tmp_path / "t.json"
    p.write_text(json.dumps({"rows": [[0, 4, 0, 64, 0, 64, "simt", 0], [0, 64, 0, 64, 0, 64, "3xtf32", 2]]}))
    rows = select.load_table(str(p))
    assert select.lookup(rows, 8, 100, 100) == ("simt", 0)
    assert select.lookup(rows, 16, 100, 100) == ("3xtf32", 2)


@pytest.mark.parametrize("bad", [
    {"rows": [[0, 1, 0, 1, 0, 1, "nope", 0]]},
    {"rows": [[0, 1, 0, 1, 0, 1, "simt"]]},
    {"rows": [[2, 1, 0, 1, 0, 1, "simt", 0]]},
    {"rows": [[0, 1, 0, 1, 0, 1, "simt", -1]]},
])
def test_malformed_tables_rejected(tmp_path, bad):
    p = tmp_path / "bad.json"
    p.write_text(json.dumps(bad))
    with pytest.raises(ValueError):
        select.load_table(str(p))


def test_fit_on_committed_sweep():
    rows = tune.load(tune.DEFAULT_CSV)
    table = tune.fit(rows)
    assert len(table) == (len(tune.GRID_EDGES) - 1) ** 3
    assert all(r[6] in tune.FP32_CLASS and r[7] == 0 for r in table)
    assert os.path.basename(tune.DEFAULT_CSV) == "mm_bench_b200.csv"
