"""The B200 selection table (tilec_b200/mm_select.json) and its loader (CPU only)."""
import json
import os

import pytest

from tilec_b200 import _native, select, tune


def test_committed_table_is_valid_and_fp32_class():
    """The table holds rows only where the sweep beat the built-in rules by a margin (it may
    be empty: then AUTO is the built-in rules), each fp32-accurate, and it records its
    held-out and cross-validated reports: a fit that cross-validation rates worse than the
    rules ships no rows."""
    rows = select.load_table(select.TABLE_PATH)
    names = {_native.VARIANT_NAMES[r[6]] for r in rows}
    assert names <= set(tune.FP32_CLASS), "AUTO may only pick fp32-accurate variants"
    with open(select.TABLE_PATH) as f:
        doc = json.load(f)
    assert doc["heldout"]["shapes"] > 0 and doc["shapes"] >= 64
    cv = doc["cross_validation"]
    if doc.get("fitted_table_kept", True):
        assert cv["selector_x_of_best"] <= cv["builtin_x_of_best"] + 1e-9
    else:  # the fit lost to the rules under cross-validation, so none of it ships
        assert rows == []
    for m, n, k in [(1, 1, 1), (512, 64, 4096), (65536, 8192, 8192), (3, 777, 3001), (2 ** 40, 2, 2)]:
        hit = select.lookup(rows, m, n, k)
        assert hit is None or hit[0] in tune.FP32_CLASS


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
    assert len({(r["M"], r["K"], r["N"]) for r in rows}) == 64
    for margin in (1.0, 1.05, 1.10):
        table = tune.fit(rows, margin=margin)
        assert len(table) <= (len(tune.GRID_EDGES) - 1) ** 3
        assert all(r[6] in tune.FP32_CLASS and r[7] == 0 for r in table)
    # a lower bar admits more override rows
    assert len(tune.fit(rows, margin=1.0)) >= len(tune.fit(rows, margin=1.10))
    assert os.path.basename(tune.DEFAULT_CSV) == "mm_bench_b200.csv"


def test_fit_overrides_only_where_builtin_loses():
    """Synthetic sweep: around small shapes SIMT beats the built-in choice by 2x, elsewhere
    the built-in choice is best; the fit emits rows only for the former."""
    rows = []
    for i, (m, k, n) in enumerate([(2, 2, 2), (3, 2, 3), (2, 3, 3), (4096, 4096, 4096), (3000, 5000, 4000),
                                   (5000, 3000, 6000)]):
        small = m < 100
        t_builtin = 2.0 if small else 1.0
        rows.append({"device": "x", "M": m, "K": k, "N": n, "variant": "builtin", "split_k": 0, "ms": t_builtin})
        rows.append({"device": "x", "M": m, "K": k, "N": n, "variant": "simt", "split_k": 0,
                     "ms": 1.0 if small else 5.0})
        rows.append({"device": "x", "M": m, "K": k, "N": n, "variant": "3xtf32", "split_k": 0,
                     "ms": 2.0 if small else 1.0})
    table = tune.fit(rows)
    assert table and all(r[6] == "simt" for r in table)
    assert select.lookup([t[:6] + [_native.VARIANTS[t[6]], t[7]] for t in table], 2, 2, 2) == ("simt", 0)
    assert select.lookup([t[:6] + [_native.VARIANTS[t[6]], t[7]] for t in table], 4096, 4096, 4096) is None


def test_train_ships_a_table_only_when_cross_validation_prefers_it(tmp_path, monkeypatch):
    """`train` writes the fitted rows only if cross-validation rates them better than the
    built-in rules; otherwise the table is empty (AUTO stays the built-in rules)."""
    import csv
    path = tmp_path / "sweep.csv"
    with open(path, "w", newline="") as f:
        w = csv.writer(f)
        w.writerow(tune.FIELDS)
        for m, k, n in [(2, 2, 2), (3, 2, 3), (2, 3, 3), (4096, 4096, 4096), (3000, 5000, 4000), (5000, 3000, 6000)]:
            small = m < 100
            w.writerow(["x", m, k, n, "builtin", 0, 2.0 if small else 1.0])
            w.writerow(["x", m, k, n, "simt", 0, 1.0 if small else 5.0])
            w.writerow(["x", m, k, n, "3xtf32", 0, 2.0 if small else 1.0])
    base = {"folds": 5, "shuffles": 3, "selector_worst": 1.0, "builtin_worst": 1.0}
    out = tmp_path / "table.json"
    monkeypatch.setattr(tune, "cross_validate", lambda rows: dict(base, selector_x_of_best=1.2, builtin_x_of_best=1.0))
    doc = tune.train(str(path), str(out))
    assert doc["rows"] == [] and doc["fitted_table_kept"] is False
    assert json.loads(out.read_text())["rows"] == []
    monkeypatch.setattr(tune, "cross_validate", lambda rows: dict(base, selector_x_of_best=0.9, builtin_x_of_best=1.0))
    doc = tune.train(str(path), str(out))
    assert doc["rows"] and doc["fitted_table_kept"] is True
    assert all(r[6] == "simt" for r in doc["rows"])
