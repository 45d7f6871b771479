"""The seeded synthetic workloads the bench measures on (no GPU): key sets and
requests have the shapes and value distributions the configurations name,
and the same seed gives the same data."""
import numpy as np
import pytest

import workload as W


def test_keys_distinct_lengths_and_vocab():
    cfg = W.CONFIGS[1]
    tok, off = W.gen_keys(5000, cfg["vocab"], cfg["len_lo"], cfg["len_hi"], cfg["zipf"], seed=3)
    assert len(off) == 5001 and off[0] == 0 and off[-1] == len(tok)
    lens = np.diff(off)
    assert lens.min() >= cfg["len_lo"] and lens.max() <= cfg["len_hi"]
    assert tok.max() < cfg["vocab"]
    keys = {tuple(tok[off[i]:off[i + 1]]) for i in range(5000)}
    assert len(keys) == 5000
    # Zipf: the most frequent id is 0, far above the median id's frequency.
    counts = np.bincount(tok, minlength=cfg["vocab"])
    assert counts.argmax() == 0 and counts[0] > 20 * max(1, counts[cfg["vocab"] // 2])


def test_keys_deterministic():
    a = W.gen_keys(2000, 1000, 2, 6, 1.1, seed=5)
    b = W.gen_keys(2000, 1000, 2, 6, 1.1, seed=5)
    c = W.gen_keys(2000, 1000, 2, 6, 1.1, seed=6)
    assert all(np.array_equal(x, y) for x, y in zip(a, b))
    assert not np.array_equal(a[0][:100], c[0][:100])


def test_torch_generator_cpu():
    tok, off = W.gen_keys_torch(3000, 5000, 3, 9, 1.05, seed=2, device="cpu")
    lens = np.diff(off)
    assert len(off) == 3001 and lens.min() >= 3 and lens.max() <= 9 and tok.max() < 5000
    assert len({tuple(tok[off[i]:off[i + 1]]) for i in range(3000)}) == 3000
    tok2, off2 = W.gen_keys_torch(3000, 5000, 3, 9, 1.05, seed=2, device="cpu")
    assert np.array_equal(tok, tok2) and np.array_equal(off, off2)


@pytest.mark.parametrize("cfg_id", [1, 5])
def test_requests_shape_and_rows(cfg_id):
    cfg = dict(W.CONFIGS[cfg_id], keys=3000, vocab=4000, K=32, L=6)
    tok, off = W.gen_keys(cfg["keys"], cfg["vocab"], 4, 8, cfg["zipf"], seed=9)
    beams, ids, lp = W.gen_requests(cfg_id, tok, off, 12, cfg=cfg)
    assert beams.shape == (12, 6) and ids.shape == (12, 6, 32) and lp.shape == (12, 6, 32)
    assert (beams == cfg["beam"]).all()
    for i in range(12):
        for t in range(6):
            row = ids[i, t]
            assert (np.diff(row.astype(np.int64)) > 0).all()  # sorted, distinct
            # log-softmax of the row: probabilities sum to one
            assert abs(np.exp(lp[i, t].astype(np.float64)).sum() - 1.0) < 1e-4
    again = W.gen_requests(cfg_id, tok, off, 12, cfg=cfg)
    assert all(np.array_equal(x, y) for x, y in zip((beams, ids, lp), again))


def test_target_key_is_proposed():
    """Config 1: one proposal per position is a token of a real key, the
    target, boosted; its prefix is therefore always searchable."""
    cfg = dict(W.CONFIGS[1])
    tok, off = W.gen_keys(4000, cfg["vocab"], cfg["len_lo"], cfg["len_hi"], cfg["zipf"], seed=1)
    keys = {tuple(tok[off[i]:off[i + 1]].tolist()) for i in range(4000)}
    beams, ids, lp = W.gen_requests(1, tok, off, 20, cfg=cfg)
    found = 0
    for i in range(20):
        # some key must have every token proposed at its position
        for k in keys:
            if len(k) <= cfg["L"] and all(k[t] in set(ids[i, t].tolist()) for t in range(len(k))):
                found += 1
                break
    assert found == 20


def test_torch_keys_sorted_and_length_weights():
    """sort=True returns the same key set in lexicographic order (a key before
    the keys it prefixes); len_weights draws lengths with those weights
    before duplicates are dropped."""
    tok, off = W.gen_keys_torch(4000, 400, 1, 5, 1.0, seed=4, device="cpu", sort=True)
    rows = [tuple(tok[off[i]:off[i + 1]].tolist()) for i in range(len(off) - 1)]
    assert rows == sorted(rows) and len(set(rows)) == len(rows) == 4000
    tok2, off2 = W.gen_keys_torch(4000, 400, 1, 5, 1.0, seed=4, device="cpu")
    assert sorted(tuple(tok2[off2[i]:off2[i + 1]].tolist()) for i in range(4000)) == rows
    cfg = W.resolve(4, keys=20000)
    assert cfg["keyset"] == "ref-lengths" and (cfg["len_lo"], cfg["len_hi"]) == (1, 8)
    tok3, off3 = W.gen_keys_torch(20000, cfg["vocab"], cfg["len_lo"], cfg["len_hi"], cfg["zipf"], seed=4,
                                  device="cpu", len_weights=cfg["len_weights"], sort=True)
    lens = np.bincount(np.diff(off3).astype(np.int64), minlength=9)
    assert lens[0] == 0 and lens[3] == lens.max()  # length 3 carries the largest weight
    with pytest.raises(ValueError):
        W.gen_keys_torch(10, 100, 1, 3, 1.0, seed=1, device="cpu", len_weights=[1, 2])
