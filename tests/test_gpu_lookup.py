"""Device lookup (ft_lookup_batch_device / flashtrie_device.lookup): key ids of
token sequences, compared with the oracle's lookup_id (itself pinned against
the reference's own lookup tool) on keys, their prefixes and extensions,
perturbed keys and random sequences, over tries with hashed nodes, link
nodes, text and binary tails.  Device reverse lookup
(ft_reverse_lookup_batch_device / flashtrie_device.reverse_lookup): every key
id of a trie gives back exactly the trie's keys, each one the key the
oracle's lookup_id maps to that id."""
import numpy as np
import pytest

import workload as W
from helpers import load_json

pytestmark = pytest.mark.gpu


def _queries(rng, keys, vocab, n_random=200):
    q = [[]]
    for k in keys:
        k = list(k)
        q.append(k)
        if len(k) > 1:
            q.append(k[:-1])
            q.append(k[:int(rng.integers(1, len(k)))])
            bad = list(k)
            bad[int(rng.integers(0, len(k)))] = int(rng.integers(0, vocab + 2))
            q.append(bad)
        q.append(k + [int(rng.integers(0, vocab + 2))])
    for _ in range(n_random):
        q.append(rng.integers(0, vocab + 2, size=int(rng.integers(1, 10))).tolist())
    return q


def _check(trie, path, queries):
    import torch
    import flashtrie_device as fd
    from oracle.oracle import OracleTrie
    o = OracleTrie(path)
    lens = np.array([len(x) for x in queries], np.int64)
    off = np.zeros(len(queries) + 1, np.int64)
    np.cumsum(lens, out=off[1:])
    flat = np.array([t for x in queries for t in x], np.uint32)
    dev = torch.device("cuda:0")
    tok = torch.from_numpy(flat.view(np.int32)).to(dev) if flat.size else torch.zeros(0, dtype=torch.int32, device=dev)
    ids = fd.lookup(trie, tok, torch.from_numpy(off).to(dev)).cpu().numpy().view(np.uint32)
    want = np.array([o.lookup_id(x) for x in queries], np.int64)
    want = np.where(want < 0, 0xFFFFFFFF, want).astype(np.uint32)
    bad = np.flatnonzero(ids != want)
    assert bad.size == 0, [(queries[i], int(ids[i]), int(want[i])) for i in bad[:5]]
    return int((want != 0xFFFFFFFF).sum())


def _trie(tmp_path, keys, name):
    import flashtrie
    t = flashtrie.Trie()
    t.build(token_rows=keys)
    p = str(tmp_path / (name + ".bin"))
    t.save(p)
    t.init_tbs_gpu(1, max_num_topk=8, max_num_outpos=8, max_num_out_beams=8)
    return t, p


def test_lookup_config1_trie(built, tmp_path):
    cfg = dict(W.CONFIGS[1])
    tok, off = W.gen_keys(30000, cfg["vocab"], cfg["len_lo"], cfg["len_hi"], cfg["zipf"], seed=51)
    keys = W.key_rows(tok, off)
    t, p = _trie(tmp_path, keys, "c1")
    rng = np.random.default_rng(5)
    sample = [keys[i] for i in rng.choice(len(keys), 800, replace=False)]
    found = _check(t, p, _queries(rng, sample, cfg["vocab"]))
    assert found >= 800


def test_lookup_hand_and_random_tries(built, tmp_path):
    g = load_json("search_hand.json")
    rng = np.random.default_rng(9)
    for name, keys in g["keysets"].items():
        t, p = _trie(tmp_path, keys, name)
        _check(t, p, _queries(rng, keys, 64, n_random=50))
    special = [[0xFFFFFFFF, 3, 4], [1, 2, 3], [1, 2, 4], [], [5] * 9]  # binary tail, empty key
    t, p = _trie(tmp_path, special, "special")
    _check(t, p, _queries(rng, special, 8, n_random=50) + [[0xFFFFFFFF], [0xFFFFFFFF, 3]])
    for vocab in (3, 300, 5000):
        keys = [rng.integers(0, vocab, size=int(rng.integers(1, 12))).tolist() for _ in range(3000)]
        t, p = _trie(tmp_path, keys, "r%d" % vocab)
        _check(t, p, _queries(rng, keys[:600], vocab))


def test_lookup_agrees_with_search_key_ids(built, tmp_path):
    import flashtrie
    cfg = dict(W.CONFIGS[1])
    tok, off = W.gen_keys(20000, cfg["vocab"], cfg["len_lo"], cfg["len_hi"], cfg["zipf"], seed=53)
    t = flashtrie.Trie()
    t.build_flat(tok, off)
    p = str(tmp_path / "s.bin")
    t.save(p)
    beams, ids, lp = W.gen_requests(1, tok, off, 8, cfg=cfg)
    t.init_tbs_gpu(8, max_num_topk=cfg["K"], max_num_outpos=cfg["L"], max_num_out_beams=cfg["beam"])
    sents, _, _, _, keys = flashtrie.bs_tbs_gpu(t, 8, beams, ids, lp, -10.0, -40.0, 5.0, False, return_key_ids=True)
    flat_s = [s for r in sents for s in r]
    flat_k = [k for r in keys for k in r]
    assert flat_s
    import torch
    import flashtrie_device as fd
    lens = np.array([len(s) for s in flat_s], np.int64)
    o = np.zeros(len(flat_s) + 1, np.int64)
    np.cumsum(lens, out=o[1:])
    tk = torch.from_numpy(np.array([x for s in flat_s for x in s], np.uint32).view(np.int32)).cuda()
    got = fd.lookup(t, tk, torch.from_numpy(o).cuda()).cpu().numpy().view(np.uint32)
    assert got.tolist() == flat_k


def test_lookup_rejects_bad_offsets(built, tmp_path):
    import torch
    import flashtrie_device as fd
    t, p = _trie(tmp_path, [[1, 2], [3]], "b")
    tok = torch.tensor([1, 2, 3], dtype=torch.int32, device="cuda")
    with pytest.raises(RuntimeError):
        fd.lookup(t, tok, torch.tensor([0, 2, 1], dtype=torch.int64, device="cuda"))  # decreasing
    with pytest.raises(RuntimeError):
        fd.lookup(t, tok, torch.tensor([0, 5], dtype=torch.int64, device="cuda"))  # past the end
    assert fd.device_status(t) == 0
    ok = fd.lookup(t, tok, torch.tensor([0, 2, 3, 3], dtype=torch.int64, device="cuda")).cpu().tolist()
    assert ok[0] != -1 and ok[1] != -1 and ok[2] == -1  # [1,2], [3], [] (not a key)
    with pytest.raises(TypeError):
        fd.lookup(t, tok.cpu(), torch.tensor([0, 1], dtype=torch.int64, device="cuda"))


def _check_reverse(trie, path, keys, max_len):
    import torch
    import flashtrie_device as fd
    from oracle.oracle import OracleTrie
    o = OracleTrie(path)
    n_keys = o.num_keys()
    ids = np.arange(n_keys + 2, dtype=np.uint32)
    ids[-1] = 0xFFFFFFFF  # not key ids: n_keys and 2^32 - 1
    toks, lens = fd.reverse_lookup(trie, torch.from_numpy(ids.view(np.int32)).cuda(), max_len)
    toks, lens = toks.cpu().numpy().view(np.uint32), lens.cpu().numpy()
    assert lens[-1] == -1 and lens[-2] == -1
    got = []
    for i in range(n_keys):
        assert 0 <= lens[i], i
        if lens[i] > max_len:
            continue
        seq = toks[i, :lens[i]].tolist()
        assert o.lookup_id(seq) == i, (i, seq)
        got.append(tuple(seq))
    want = {tuple(k) for k in keys if len(k) <= max_len}
    assert set(got) == want and len(got) == len(want)
    assert int((lens[:n_keys] > max_len).sum()) == len({tuple(k) for k in keys if len(k) > max_len})


def test_reverse_lookup_returns_every_key(built, tmp_path):
    cfg = dict(W.CONFIGS[1])
    tok, off = W.gen_keys(30000, cfg["vocab"], cfg["len_lo"], cfg["len_hi"], cfg["zipf"], seed=57)
    keys = W.key_rows(tok, off)
    t, p = _trie(tmp_path, keys, "rc1")
    _check_reverse(t, p, keys, 8)
    _check_reverse(t, p, keys, 5)  # longer keys report their length only
    g = load_json("search_hand.json")
    for name, ks in g["keysets"].items():
        t, p = _trie(tmp_path, ks, "rh_" + name)
        _check_reverse(t, p, ks, 16)
    special = [[0xFFFFFFFF, 3, 4], [1, 2, 3], [1, 2, 4], [], [5] * 9]
    t, p = _trie(tmp_path, special, "rspecial")
    _check_reverse(t, p, special, 12)
    rng = np.random.default_rng(61)
    for vocab in (3, 5000):
        ks = [rng.integers(0, vocab, size=int(rng.integers(1, 14))).tolist() for _ in range(4000)]
        t, p = _trie(tmp_path, ks, "rr%d" % vocab)
        _check_reverse(t, p, ks, 14)
