"""Generates the golden fixtures in tests/golden/ from the UNMODIFIED reference.

Run in a container that has the reference sources and the module built by
oracle/ref.mk (`make -f oracle/ref.mk`):

    python tests/golden/make_golden.py

Fixtures (JSON):
  format.json   for seeded key sets: sha256 and size of the file the reference
                `Trie.build(...).save()` writes (the engine's builder must write
                the same bytes), plus num_keys/num_nodes/total_size/io_size.
  search_c1.json
                config-1 trie (100k keys) and seeded requests: the reference
                CPU `tbs(use_gpu=False)` output for each, whether that output
                holds beams that are not keys (the reference CPU link-node bug),
                and a sha256 of the generated inputs so generator drift fails
                loudly instead of comparing different inputs.
  search_hand.json
                hand-built tries and requests covering links, internal link
                nodes, terminal link nodes, thresholds, ties, duplicate ids,
                unsorted rows and zero-width beams.
  lookup_c1.json
                key ids the reference's own lookup tool (tools/marisa-lookup.cc,
                built by oracle/ref.mk) reports on the config-1 trie for keys,
                prefixes of keys and random sequences (-1: not a key).
  search_c2.json, search_c3.json
                the request shapes of configs 2 (K=256, L=16, beam 100) and 3
                (K=1000, L=20, beam 1000) on 200k-key tries of their key
                distributions: reference CPU `tbs` outputs.
  topk_loader.json
                a seeded top-k dataset directory (its two text files) and what
                the reference's `load_topk_keys_and_scores` returns for it.
  api_surface.json
                the signature line of every public function and Trie method
                of the reference module (names, keyword names, defaults).
This script and the fixture generation run only where the reference sources
are (the reference's module is built from them by oracle/ref.mk); the GPU-side
tests read the committed JSON files and never the reference itself.

    python tests/golden/make_golden.py           # all fixtures
    python tests/golden/make_golden.py lookup    # lookup_c1.json only
    python tests/golden/make_golden.py topk      # topk_loader.json only
    python tests/golden/make_golden.py api       # api_surface.json only
    python tests/golden/make_golden.py shape [2 3]  # search_c2.json / search_c3.json only
"""
import hashlib
import json
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "oracle", "_ref"))
os.environ.setdefault("MARISA_MANAGED_ALLOC", "0")

import workload as W  # noqa: E402

THR = (W.TOKEN_LOGP_THRESHOLD, W.SENT_LOGP_THRESHOLD, W.LENGTH_NORM)


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def file_sha(path):
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


def format_cases():
    rng = np.random.default_rng(7)
    cases = []
    for name, n, V, lo, hi in [("tiny-random", 40, 6, 1, 4), ("small-random", 3000, 40, 1, 7),
                                ("mid-random", 20000, 70000, 2, 9), ("wide-labels", 5000, 2**31 - 1, 1, 6)]:
        rows = [rng.integers(0, V, size=int(rng.integers(lo, hi + 1))).tolist() for _ in range(n)]
        cases.append((name, rows))
    tok, off = W.gen_keys(100_000, 32_000, 2, 8, 1.1, seed=1)
    cases.append(("config1-keys", W.key_rows(tok, off)))
    cases.append(("empty", []))
    cases.append(("empty-key", [[]]))
    cases.append(("duplicates", [[5], [5], [5, 6], [5, 6], [9, 9, 9]]))
    return cases


def c1_reference_trie():
    import flashtrie_ref as ref
    cfg = W.CONFIGS[1]
    tok, off = W.gen_keys(cfg["keys"], cfg["vocab"], cfg["len_lo"], cfg["len_hi"], cfg["zipf"], seed=1)
    t = ref.Trie()
    t.build(token_rows=W.key_rows(tok, off))
    path = "/tmp/golden_c1.bin"
    t.save(path)
    return t, tok, off, path


def lookup_golden(tok, off, path):
    rng = np.random.default_rng(17)
    n = len(off) - 1
    queries = []
    for i in rng.choice(n, size=300, replace=False):
        key = tok[off[i]:off[i + 1]].tolist()
        queries.append(key)
        if len(key) > 1:
            queries.append(key[:int(rng.integers(1, len(key)))])  # a prefix: a key or not
    for _ in range(100):
        queries.append(rng.integers(0, W.CONFIGS[1]["vocab"], size=int(rng.integers(1, 6))).tolist())
    tool = os.path.join(REPO, "oracle", "_ref", "marisa-lookup")
    inp = "".join(" ".join(str(x) for x in q) + "\n" for q in queries)
    res = subprocess.run([tool, path], input=inp, capture_output=True, text=True, check=True,
                         env=dict(os.environ, MARISA_MANAGED_ALLOC="0"))
    ids = [int(line.split("\t")[0]) for line in res.stdout.splitlines()]
    assert len(ids) == len(queries)
    with open(os.path.join(HERE, "lookup_c1.json"), "w") as f:
        json.dump({"trie_sha256": file_sha(path), "queries": queries, "ids": ids}, f)


def topk_loader_texts():
    """The two text files of a seeded top-k dataset directory in the layout the
    reference loader reads (tools/beam-search-helper.h:28-126): a header line
    `num_requests max_output_len topk` in each file, then one line per
    (request, depth) of ids / log-probabilities.  Rows cover the cases the
    loader treats differently: depth 0 (kept in file order), deeper rows out
    of id order (sorted by id, scores permuted with them), duplicate ids,
    rows shorter than topk (padded with UINT32_MAX / -FLT_MAX), rows longer
    than topk (truncated after sorting), ids written as floats ("12.0",
    "12e0"), and an empty row."""
    rng = np.random.default_rng(23)
    n_req, max_len, topk = 4, 5, 6
    k_lines = ["%d %d %d" % (n_req, max_len, topk)]
    s_lines = ["%d %d %d" % (n_req, max_len, topk)]
    for r in range(n_req):
        for d in range(max_len):
            width = [topk, topk - 2, topk + 3, 0, topk][(r + d) % 5]
            ids = rng.integers(0, 400, size=width).tolist()
            if width > 2 and d % 2 == 1:
                ids[1] = ids[0]  # a duplicate id in the row
            lp = np.sort(rng.normal(-3.0, 2.0, size=width).astype(np.float32))[::-1]
            words = []
            for j, x in enumerate(ids):
                words.append("%d.0" % x if j % 4 == 1 else "%de0" % x if j % 4 == 3 else str(x))
            k_lines.append(" ".join(words))
            s_lines.append(" ".join(repr(float(v)) for v in lp))
    return "\n".join(k_lines) + "\n", "\n".join(s_lines) + "\n"


def topk_loader_golden():
    import tempfile
    import flashtrie_ref as ref
    keys_txt, scores_txt = topk_loader_texts()
    with tempfile.TemporaryDirectory() as d:
        with open(os.path.join(d, "topk_keys.txt"), "w") as f:
            f.write(keys_txt)
        with open(os.path.join(d, "topk_scores.txt"), "w") as f:
            f.write(scores_txt)
        keys, scores = ref.load_topk_keys_and_scores(d)
    with open(os.path.join(HERE, "topk_loader.json"), "w") as f:
        json.dump({"topk_keys_txt": keys_txt, "topk_scores_txt": scores_txt, "ref_keys": keys,
                   "ref_scores": scores}, f)


# Request shapes of configs 2 and 3 on 200k-key tries of their key
# distributions: (config, keys, requests, fixture).
SHAPES = {2: (200_000, 48, "search_c2.json"), 3: (200_000, 24, "search_c3.json")}


def shape_golden(cfg_id):
    """A configuration's request shape (its K, L, beam, vocabulary and key
    distribution) on a 200k-key trie: the reference CPU `tbs` output for
    seeded requests."""
    import flashtrie_ref as ref
    from oracle.oracle import OracleTrie
    n_keys, n_req, name = SHAPES[cfg_id]
    cfg = dict(W.CONFIGS[cfg_id], keys=n_keys)
    tok, off = W.gen_keys(cfg["keys"], cfg["vocab"], cfg["len_lo"], cfg["len_hi"], cfg["zipf"], seed=cfg_id)
    t = ref.Trie()
    t.build(token_rows=W.key_rows(tok, off))
    path = "/tmp/golden_c%d.bin" % cfg_id
    t.save(path)
    orc = OracleTrie(path)
    beams, ids, lp = W.gen_requests(cfg_id, tok, off, n_req, cfg=cfg)
    reqs = []
    for r in range(n_req):
        sent, lpn, _ = ref.tbs(t, beams[r].tolist(), ids[r].tolist(), lp[r].tolist(), *THR, False, False)
        invalid = [i for i, s in enumerate(sent) if not orc.lookup(s)]
        reqs.append({"index": r, "inputs_sha256": sha(beams[r], ids[r], lp[r]), "ref_sent": sent, "ref_lpn": lpn,
                     "ref_invalid": invalid})
    with open(os.path.join(HERE, name), "w") as f:
        json.dump({"config": cfg_id, "keys": n_keys, "key_seed": cfg_id, "keys_sha256": sha(tok, off),
                   "trie_sha256": file_sha(path), "thresholds": THR, "requests": reqs}, f)


def api_golden():
    """The first (signature) line of every public function and Trie method's
    docstring in the reference module, as pybind11 writes it."""
    import flashtrie_ref as ref

    def sig(obj):
        return (obj.__doc__ or "").strip().split("\n")[0]

    surface = {"functions": {n: sig(getattr(ref, n)) for n in dir(ref) if not n.startswith("_") and n != "Trie"},
               "Trie": {n: sig(getattr(ref.Trie, n)) for n in dir(ref.Trie) if not n.startswith("_")}}
    with open(os.path.join(HERE, "api_surface.json"), "w") as f:
        json.dump(surface, f, indent=1)


def main():
    import flashtrie_ref as ref
    from oracle.oracle import OracleTrie

    out = {"generator": "tests/golden/make_golden.py", "cases": []}
    for name, rows in format_cases():
        t = ref.Trie()
        t.build(token_rows=rows)
        path = "/tmp/golden_%s.bin" % name
        t.save(path)
        out["cases"].append({"name": name, "sha256": file_sha(path), "bytes": os.path.getsize(path),
                             "num_keys": t.num_keys(), "num_nodes": t.num_nodes(), "total_size": t.total_size()})
    with open(os.path.join(HERE, "format.json"), "w") as f:
        json.dump(out, f, indent=1)

    # ---- config 1 search goldens
    cfg = W.CONFIGS[1]
    tok, off = W.gen_keys(cfg["keys"], cfg["vocab"], cfg["len_lo"], cfg["len_hi"], cfg["zipf"], seed=1)
    t = ref.Trie()
    t.build(token_rows=W.key_rows(tok, off))
    path = "/tmp/golden_c1.bin"
    t.save(path)
    orc = OracleTrie(path)
    reqs = []
    n_req = 160
    beams, ids, lp = W.gen_requests(1, tok, off, n_req)
    for r in range(n_req):
        ee = r >= 120  # the last 40 use early exit
        sent, lpn, _ = ref.tbs(t, beams[r].tolist(), ids[r].tolist(), lp[r].tolist(), *THR, ee, False)
        invalid = [i for i, s in enumerate(sent) if not orc.lookup(s)]
        reqs.append({"index": r, "seed": 1000 + r, "inputs_sha256": sha(beams[r], ids[r], lp[r]),
                     "early_exit": ee, "ref_sent": sent, "ref_lpn": lpn, "ref_invalid": invalid})
    with open(os.path.join(HERE, "search_c1.json"), "w") as f:
        json.dump({"config": 1, "key_seed": 1, "keys_sha256": sha(tok, off), "trie_sha256": file_sha(path),
                   "thresholds": THR, "requests": reqs}, f)

    # ---- hand-built tries
    hand = []
    keysets = {
        # links, an internal link node ([20,21,22] is a link node with a child),
        # a terminal internal link node, a single-label key
        "links": [[1, 2, 3, 4], [1, 2, 3, 5], [20, 21, 22], [20, 21, 22, 23], [7]],
        "deep": [[1, 2, 3, 4, 5, 6, 7, 8], [1, 2, 3, 4, 5, 6, 7, 9], [1, 2, 9], [1, 2], [1], [3, 3, 3, 3]],
        "fan": [[i, j] for i in range(1, 6) for j in range(0, 40, 3)] + [[100 + i] for i in range(50)],
    }
    rng = np.random.default_rng(11)
    for name, keys in keysets.items():
        t = ref.Trie()
        t.build(token_rows=keys)
        for q in range(24):
            L = int(rng.integers(1, 9))
            K = int(rng.integers(1, 12))
            vocab = sorted({k for key in keys for k in key} | {0, 99, 1000})
            rows_i, rows_l = [], []
            for _ in range(L):
                row = rng.choice(vocab, size=K, replace=bool(q % 5 == 4)).tolist()
                if q % 3 != 2:
                    row = sorted(row)
                rows_i.append([int(x) for x in row])
                # coarse values so that exact ties occur
                rows_l.append([float(np.float32(-0.5 * int(rng.integers(0, 6)))) for _ in range(K)])
            B = int(rng.integers(1, 6))
            beams_q = [B] * L
            # (A zero width before the last position crashes the reference CPU
            # path: Candidates::push reads top() of an empty heap,
            # candidates.h:223.  Zero widths are covered by the oracle tests.)
            tt, st = (-10.0, -40.0) if q % 4 else (-1.6, -3.1)
            ln = [0.0, 1.0, 5.0][q % 3]
            ee = bool(q % 8 == 7)
            sent, lpn, _ = ref.tbs(t, beams_q, rows_i, rows_l, tt, st, ln, ee, False)
            # The oracle has its own trie loader; check on the same file bytes.
            t.save("/tmp/golden_hand.bin")
            orc = OracleTrie("/tmp/golden_hand.bin")
            invalid = [i for i, s in enumerate(sent) if not orc.lookup(s)]
            hand.append({"trie": name, "beams": beams_q, "topk_id": rows_i, "topk_logp": rows_l,
                         "token_logp_threshold": tt, "sents_logp_threshold": st, "length_norm": ln,
                         "early_exit": ee, "ref_sent": sent, "ref_lpn": lpn, "ref_invalid": invalid})
    with open(os.path.join(HERE, "search_hand.json"), "w") as f:
        json.dump({"keysets": keysets, "requests": hand}, f)
    print("wrote", os.listdir(HERE))


if __name__ == "__main__":
    if sys.argv[1:] == ["lookup"]:
        _, tok, off, path = c1_reference_trie()
        lookup_golden(tok, off, path)
    elif sys.argv[1:] == ["topk"]:
        topk_loader_golden()
    elif sys.argv[1:] == ["api"]:
        api_golden()
    elif sys.argv[1:2] == ["shape"]:
        for c in sys.argv[2:] or SHAPES:
            shape_golden(int(c))
    else:
        main()
        _, tok, off, path = c1_reference_trie()
        lookup_golden(tok, off, path)
        topk_loader_golden()
        api_golden()
        for c in SHAPES:
            shape_golden(c)
