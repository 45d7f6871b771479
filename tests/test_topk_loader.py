"""`flashtrie.load_topk_keys_and_scores` against the reference loader.

The fixture holds a seeded top-k dataset directory (tools/beam-search-helper.h
reads `topk_keys.txt` and `topk_scores.txt` from it) and what the unmodified
reference's loader returned for it: depth-0 rows in file order, deeper rows
sorted by id with their scores permuted alongside, duplicate ids, short rows
padded with UINT32_MAX / -FLT_MAX, long rows truncated, ids written as floats.
The engine's loader must return the same lists, scores bit for bit.
"""
import os
import sys

import pytest

from helpers import REPO, load_json


def _write_dir(d, keys_txt, scores_txt):
    with open(os.path.join(d, "topk_keys.txt"), "w") as f:
        f.write(keys_txt)
    with open(os.path.join(d, "topk_scores.txt"), "w") as f:
        f.write(scores_txt)
    return str(d)


def test_loader_matches_reference_fixture(built, tmp_path):
    import flashtrie
    g = load_json("topk_loader.json")
    keys, scores = flashtrie.load_topk_keys_and_scores(_write_dir(tmp_path, g["topk_keys_txt"], g["topk_scores_txt"]))
    assert keys == g["ref_keys"]
    assert scores == g["ref_scores"]
    # The fixture exercises what it claims to: padding, truncation to topk,
    # an all-padding row and a deeper row that was out of id order.
    topk = int(g["topk_keys_txt"].split()[2])
    rows = [row for req in keys for row in req]
    assert all(len(row) == topk for row in rows)
    assert any(row[-1] == 0xFFFFFFFF and row[0] != 0xFFFFFFFF for row in rows)
    assert any(all(x == 0xFFFFFFFF for x in row) for row in rows)
    first_lines = g["topk_keys_txt"].splitlines()[1:]
    assert any(len(line.split()) > topk for line in first_lines)


def test_loader_matches_reference_module_live(built, tmp_path):
    """Where the reference module is built (oracle/_ref), the same directory
    through both loaders."""
    ref_dir = os.path.join(REPO, "oracle", "_ref")
    if not (os.path.isdir(ref_dir) and any(f.startswith("flashtrie_ref") for f in os.listdir(ref_dir))):
        pytest.skip("reference module not built")
    sys.path.insert(0, ref_dir)
    os.environ.setdefault("MARISA_MANAGED_ALLOC", "0")
    import flashtrie
    import flashtrie_ref
    sys.path.insert(0, os.path.join(REPO, "tests", "golden"))
    from make_golden import topk_loader_texts
    d = _write_dir(tmp_path, *topk_loader_texts())
    assert flashtrie.load_topk_keys_and_scores(d) == flashtrie_ref.load_topk_keys_and_scores(d)


def test_loader_errors(built, tmp_path):
    """A missing file raises (the reference prints and calls exit(1)); rows of
    ids and scores that differ in length raise (the reference asserts, which
    release builds compile out, and then reads past the shorter row)."""
    import flashtrie
    with pytest.raises(RuntimeError, match="topk keys"):
        flashtrie.load_topk_keys_and_scores(str(tmp_path / "absent"))
    d = _write_dir(tmp_path, "1 1 2\n5 6\n", "1 1 2\n-1.0\n")
    with pytest.raises(RuntimeError, match="differ in length"):
        flashtrie.load_topk_keys_and_scores(d)
    d2 = tmp_path / "hdr"
    d2.mkdir()
    _write_dir(d2, "1 1 2\n5 6\n", "1 2 2\n-1.0 -2.0\n")
    with pytest.raises(RuntimeError, match="headers differ"):
        flashtrie.load_topk_keys_and_scores(str(d2))
