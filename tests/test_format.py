"""Trie format: the engine's builder writes the reference's bytes, and
load -> save round-trips (golden: tests/golden/format.json, generated from the
unmodified reference by tests/golden/make_golden.py)."""
import os
import sys

import pytest

from helpers import REPO, file_sha, load_json

sys.path.insert(0, os.path.join(REPO, "tests", "golden"))


@pytest.fixture(scope="module")
def ft(built):
    import flashtrie
    return flashtrie


def test_builder_matches_reference_bytes(ft, tmp_path):
    import make_golden
    golden = {c["name"]: c for c in load_json("format.json")["cases"]}
    for name, rows in make_golden.format_cases():
        g = golden[name]
        t = ft.Trie()
        t.build(token_rows=rows)
        p = str(tmp_path / (name + ".bin"))
        t.save(p)
        assert os.path.getsize(p) == g["bytes"], name
        assert file_sha(p) == g["sha256"], name
        assert t.num_keys() == g["num_keys"] and t.num_nodes() == g["num_nodes"], name
        assert t.total_size() == g["total_size"], name
        assert t.io_size() == g["bytes"], name


def test_load_save_roundtrip(ft, tmp_path):
    import make_golden
    rows = dict(make_golden.format_cases())["small-random"]
    a = ft.Trie()
    a.build(token_rows=rows)
    p1, p2, p3 = (str(tmp_path / n) for n in ("a.bin", "b.bin", "c.bin"))
    a.save(p1)
    b = ft.Trie()
    b.load(p1)
    b.save(p2)
    c = ft.Trie()
    c.mmap(p1)
    c.save(p3)
    assert open(p1, "rb").read() == open(p2, "rb").read() == open(p3, "rb").read()
    assert b.num_keys() == a.num_keys() and c.num_nodes() == a.num_nodes()


def test_numpy_rows_build(ft, tmp_path):
    import numpy as np
    rows = np.array([[3, 1, 2], [3, 1, 5], [7, 7, 7]], dtype=np.uint32)
    a, b = ft.Trie(), ft.Trie()
    a.build(token_rows=rows)
    b.build(token_rows=rows.tolist())
    pa, pb = str(tmp_path / "a"), str(tmp_path / "b")
    a.save(pa)
    b.save(pb)
    assert open(pa, "rb").read() == open(pb, "rb").read()


def test_errors(ft, tmp_path):
    t = ft.Trie()
    with pytest.raises(RuntimeError, match="STATE_ERROR"):
        t.num_keys()
    with pytest.raises(RuntimeError, match="STATE_ERROR"):
        t.save(str(tmp_path / "x"))
    with pytest.raises(RuntimeError, match="IO_ERROR"):
        t.load(str(tmp_path / "missing.bin"))
    bad = tmp_path / "bad.bin"
    bad.write_bytes(b"We hate Marisa.\0" + b"\0" * 64)
    with pytest.raises(RuntimeError, match="FORMAT_ERROR"):
        t.load(str(bad))
    # truncated file
    good = ft.Trie()
    good.build(token_rows=[[1, 2, 3], [1, 2, 4]])
    p = str(tmp_path / "good.bin")
    good.save(p)
    data = open(p, "rb").read()
    (tmp_path / "trunc.bin").write_bytes(data[: len(data) // 2])
    with pytest.raises(RuntimeError, match="IO_ERROR"):
        t.load(str(tmp_path / "trunc.bin"))
    t.build(token_rows=[[1]])
    t.clear()
    with pytest.raises(RuntimeError, match="STATE_ERROR"):
        t.num_keys()
    with pytest.raises(TypeError):
        t.build(token_rows=[[1, -2]])
