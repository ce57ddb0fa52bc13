"""The autotuner's table writer and the two committed tables (host only)."""
from __future__ import annotations

import os

from depthwise_conv_b200 import tune

FIELDS_PER_ROW = 6 + len(tune.FIELDS)


def _rows(path):
    return [ln.strip() for ln in open(path) if ln.startswith("{")]


def _plan(**over):
    p = dict(cols_per_thread=16, rows_per_thread=1, tile_h=2, tile_w=32, ring_rows=6, ring_wrows=0, grid=0,
             row_splits=1, load_schedule=0, band_tiles=0)
    p.update(over)
    return p


def test_committed_tables_parse():
    for path in (tune.TABLE, tune.TABLE_RES):
        rows = _rows(path)
        assert rows, path
        keys = set()
        for r in rows:
            vals = [int(v) for v in r.strip("{},").split(",")]
            assert len(vals) in (FIELDS_PER_ROW - 1, FIELDS_PER_ROW), r  # older rows omit band_tiles
            key = tuple(vals[:6])
            assert key not in keys, f"duplicate entry {key} in {os.path.basename(path)}"
            keys.add(key)
            assert vals[5] in (0, 1) and vals[4] % 2 == 1


def test_write_table_merges_into_its_base_and_keeps_its_header(tmp_path):
    out = tmp_path / "res.inc"
    tune.write_table([((3, 32, 32, 768, 7, 1), _plan(ring_rows=8, load_schedule=1))], str(out), tune.TABLE_RES)
    text = open(out).read()
    head = [ln for ln in text.splitlines() if ln.startswith("//")]
    assert head == [ln.rstrip("\n") for ln in open(tune.TABLE_RES) if ln.startswith("//")]
    rows = _rows(out)
    assert len(rows) == len(_rows(tune.TABLE_RES)) + 1
    assert "{3, 32, 32, 768, 7, 1, 16, 1, 2, 32, 8, 0, 0, 1, 1, 0}," in rows
    # a row for an existing key replaces it
    key_row = _rows(tune.TABLE_RES)[0]
    B, H, W, C, K, acc = (int(v) for v in key_row.strip("{},").split(",")[:6])
    tune.write_table([((B, H, W, C, K, acc), _plan(tile_h=4))], str(out), tune.TABLE_RES)
    rows = _rows(out)
    assert len(rows) == len(_rows(tune.TABLE_RES))
    assert any(r.startswith("{%d, %d, %d, %d, %d, %d, 16, 1, 4," % (B, H, W, C, K, acc)) for r in rows)


def test_write_table_default_base_is_the_main_table(tmp_path):
    out = tmp_path / "main.inc"
    tune.write_table([], str(out))
    assert _rows(out) == sorted(_rows(tune.TABLE), key=lambda r: tuple(int(v) for v in r.strip("{},").split(",")[:6]))
