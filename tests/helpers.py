"""Shared helpers for the test suite (paths, fixtures, comparisons)."""
import hashlib
import json
import os

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(REPO, "tests", "golden")


def load_json(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def file_sha(path):
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


def same_result(a_sent, a_lpn, b_sent, b_lpn):
    """Ordered lists equal and scores bit-identical."""
    return [list(s) for s in a_sent] == [list(s) for s in b_sent] and list(a_lpn) == list(b_lpn)


def same_result_tol(a_sent, a_lpn, b_sent, b_lpn, rtol=1e-5):
    """Sequences identical and in the same order; scores within rtol."""
    if [list(s) for s in a_sent] != [list(s) for s in b_sent]:
        return False
    return bool(np.allclose(np.asarray(a_lpn, float), np.asarray(b_lpn, float), rtol=rtol, atol=0.0))
