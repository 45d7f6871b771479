"""The size-independent result checks of the full-size GPU tests
(tests/test_gpu_fullsize.py: check_properties), run on the oracle's own
results here (no GPU): they pass on correct results and catch each kind of
planted mistake."""
import copy

import numpy as np
import pytest

import workload as W
from test_gpu_fullsize import check_properties


@pytest.fixture(scope="module")
def case(built, tmp_path_factory):
    import flashtrie
    from oracle.oracle import OracleTrie
    cfg = dict(W.CONFIGS[1])
    tok, off = W.gen_keys(30000, cfg["vocab"], cfg["len_lo"], cfg["len_hi"], cfg["zipf"], seed=41)
    t = flashtrie.Trie()
    t.build_flat(tok, off)
    p = str(tmp_path_factory.mktemp("props") / "p.bin")
    t.save(p)
    o = OracleTrie(p)
    beams, ids, lp = W.gen_requests(1, tok, off, 6, cfg=cfg)
    out = []
    for i in range(6):
        s, l = o.tbs(beams[i], ids[i], lp[i], W.TOKEN_LOGP_THRESHOLD, W.SENT_LOGP_THRESHOLD, W.LENGTH_NORM, False)
        out.append((s, l, [o.lookup_id(x) for x in s]))
    i = max(range(6), key=lambda j: len(out[j][0]))
    assert len(out[i][0]) >= 3
    return o, beams[i], ids[i], lp[i], out[i], tok, off


def test_oracle_results_pass(case):
    o, beams, ids, lp, (s, l, k), _, _ = case
    check_properties(o, beams, ids, lp, s, l, k)


def _plant(case, how):
    o, beams, ids, lp, (s, l, k), tok, off = case
    s, l, k = copy.deepcopy(s), list(l), list(k)
    if how == "score":
        l[1] = np.nextafter(l[1], 0.0)
    elif how == "order":
        s[0], s[1], l[0], l[1], k[0], k[1] = s[1], s[0], l[1], l[0], k[1], k[0]
    elif how == "duplicate":
        s[1], l[1], k[1] = list(s[0]), l[0], k[0]
        l = sorted(l)
    elif how == "key_id":
        k[0] = (k[0] + 1) & 0xFFFFFFFF
    elif how == "not_proposed":
        bad = int(ids[0].max()) + 1  # no proposal of position 0 has this id
        s[0] = [bad] + list(s[0][1:])
    elif how == "too_many":
        beams = beams.copy()
        beams[-1] = len(s) - 1
    return o, beams, ids, lp, s, l, k


@pytest.mark.parametrize("how", ["score", "order", "duplicate", "key_id", "not_proposed", "too_many"])
def test_planted_mistakes_are_caught(case, how):
    with pytest.raises(AssertionError):
        check_properties(*_plant(case, how))
