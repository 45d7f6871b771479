"""Key ids of the results (LoudsTrie::lookup's id): every result beam's id
equals the oracle's lookup_id of its token sequence, itself pinned against the
reference's own lookup tool (tests/test_oracle_golden.py)."""
import numpy as np
import pytest

import workload as W

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def trie_and_oracle(built, tmp_path_factory):
    import flashtrie
    from oracle.oracle import OracleTrie
    cfg = dict(W.CONFIGS[1])
    tok, off = W.gen_keys(40000, cfg["vocab"], cfg["len_lo"], cfg["len_hi"], cfg["zipf"], seed=31)
    t = flashtrie.Trie()
    t.build_flat(tok, off)
    p = str(tmp_path_factory.mktemp("k") / "k.bin")
    t.save(p)
    return t, OracleTrie(p), tok, off, cfg


def test_host_path_key_ids(trie_and_oracle):
    import flashtrie
    t, o, tok, off, cfg = trie_and_oracle
    n = 40  # 40 * 10 * 8 token slots: the one-copy path
    beams, ids, lp = W.gen_requests(1, tok, off, n, cfg=cfg)
    t.init_tbs_gpu(n, max_num_topk=cfg["K"], max_num_outpos=cfg["L"], max_num_out_beams=64)
    sents, lpns, _, _, keys = flashtrie.bs_tbs_gpu(t, n, beams, ids, lp, -10.0, -40.0, 5.0, False,
                                                    return_key_ids=True)
    plain = flashtrie.bs_tbs_gpu(t, n, beams, ids, lp, -10.0, -40.0, 5.0, False)
    assert len(plain) == 4 and plain[0] == sents and plain[1] == lpns
    total = 0
    for i in range(n):
        assert len(keys[i]) == len(sents[i])
        for s, k in zip(sents[i], keys[i]):
            assert k == o.lookup_id(s), (i, s)
            total += 1
    assert total > 0
    s1, l1, _, k1 = flashtrie.tbs(t, beams[0], ids[0], lp[0], -10.0, -40.0, 5.0, False, True, return_key_ids=True)
    assert k1 == keys[0] and s1 == sents[0]


def test_large_batch_key_ids(trie_and_oracle):
    """Compact two-phase result path with key ids."""
    import flashtrie
    t, o, tok, off, cfg = trie_and_oracle
    cfg = dict(cfg, beam=200)
    n = 48
    beams, ids, lp = W.gen_requests(1, tok, off, n, start=500, cfg=cfg)
    t.init_tbs_gpu(n, max_num_topk=cfg["K"], max_num_outpos=cfg["L"], max_num_out_beams=200)
    sents, _, _, _, keys = flashtrie.bs_tbs_gpu(t, n, beams, ids, lp, -10.0, -40.0, 5.0, False,
                                                 return_key_ids=True)
    for i in range(n):
        assert keys[i] == [o.lookup_id(s) for s in sents[i]], i


def test_device_path_key_ids(trie_and_oracle):
    import torch
    import flashtrie_device as fd
    t, o, tok, off, cfg = trie_and_oracle
    n = 8
    beams, ids, lp = W.gen_requests(1, tok, off, n, start=900, cfg=cfg)
    t.init_tbs_gpu(n, max_num_topk=cfg["K"], max_num_outpos=cfg["L"], max_num_out_beams=cfg["beam"])
    dev = torch.device("cuda:0")
    out = fd.bs_tbs_device(t, torch.from_numpy(beams.astype(np.int32)).to(dev),
                           torch.from_numpy(ids.view(np.int32)).to(dev), torch.from_numpy(lp).to(dev),
                           -10.0, -40.0, 5.0, False, key_ids=True)
    sents, _, keys = fd.to_lists(out)
    for i in range(n):
        assert keys[i] == [o.lookup_id(s) for s in sents[i]], i
