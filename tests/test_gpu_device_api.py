"""The device-tensor API (flashtrie_device) and beam widths above 1024."""
import numpy as np
import pytest

import workload as W
from helpers import same_result

pytestmark = pytest.mark.gpu


def _trie(tmp_path, n_keys=30000, seed=21, cfg_id=1):
    import flashtrie
    cfg = dict(W.CONFIGS[cfg_id])
    tok, off = W.gen_keys(n_keys, cfg["vocab"], cfg["len_lo"], cfg["len_hi"], cfg["zipf"], seed=seed)
    t = flashtrie.Trie()
    t.build_flat(tok, off)
    p = str(tmp_path / "d.bin")
    t.save(p)
    return p, tok, off, cfg


def test_device_tensors_match_host_path(built, tmp_path):
    import torch
    import flashtrie
    import flashtrie_device as fd
    p, tok, off, cfg = _trie(tmp_path)
    n = 12
    beams, ids, lp = W.gen_requests(1, tok, off, n, cfg=cfg)
    # Half of the rows unsorted: the kernel sorts them in shared memory.
    rng = np.random.default_rng(3)
    for i in range(0, n, 2):
        for t_ in range(ids.shape[1]):
            perm = rng.permutation(ids.shape[2])
            ids[i, t_] = ids[i, t_, perm]
            lp[i, t_] = lp[i, t_, perm]
    t = flashtrie.Trie()
    t.load(p)
    t.init_tbs_gpu(n, max_num_topk=cfg["K"], max_num_outpos=cfg["L"], max_num_out_beams=cfg["beam"])
    dev = torch.device("cuda:0")
    out = fd.bs_tbs_device(t, torch.from_numpy(beams.astype(np.int32)).to(dev),
                           torch.from_numpy(ids.view(np.int32)).to(dev), torch.from_numpy(lp).to(dev),
                           -10.0, -40.0, 5.0, False)
    d_sents, d_lpns = fd.to_lists(out)
    h_sents, h_lpns, _, _ = flashtrie.bs_tbs_gpu(t, n, beams, ids, lp, -10.0, -40.0, 5.0, False)
    for i in range(n):
        assert same_result(d_sents[i], d_lpns[i], h_sents[i], h_lpns[i]), i


def test_device_search_on_a_side_stream(built, tmp_path):
    """A search on a stream other than the current one: its outputs are
    allocated and cleared on that stream, so it returns what the same search
    on the current stream returns, twice in a row (the second reuses freed
    blocks of the first)."""
    import torch
    import flashtrie
    import flashtrie_device as fd
    p, tok, off, cfg = _trie(tmp_path, seed=23)
    n = 10
    beams, ids, lp = W.gen_requests(1, tok, off, n, cfg=cfg)
    t = flashtrie.Trie()
    t.load(p)
    t.init_tbs_gpu(n, max_num_topk=cfg["K"], max_num_outpos=cfg["L"], max_num_out_beams=cfg["beam"])
    dev = torch.device("cuda:0")
    d_in = (torch.from_numpy(beams.astype(np.int32)).to(dev), torch.from_numpy(ids.view(np.int32)).to(dev),
            torch.from_numpy(lp).to(dev))
    want = fd.to_lists(fd.bs_tbs_device(t, *d_in, -10.0, -40.0, 5.0, False, key_ids=True))
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))  # the inputs were written on the current stream
    for _ in range(2):
        out = fd.bs_tbs_device(t, *d_in, -10.0, -40.0, 5.0, False, stream=side, check=False, key_ids=True)
        side.synchronize()
        assert fd.device_status(t) == 0
        assert fd.to_lists(out) == want
        del out


def test_device_tensor_validation(built, tmp_path):
    import torch
    import flashtrie
    import flashtrie_device as fd
    p, tok, off, cfg = _trie(tmp_path, n_keys=2000)
    t = flashtrie.Trie()
    t.load(p)
    t.init_tbs_gpu(2, max_num_topk=8, max_num_outpos=4, max_num_out_beams=4)
    dev = torch.device("cuda:0")
    beams = torch.full((2, 4), 4, dtype=torch.int32, device=dev)
    ids = torch.zeros((2, 4, 8), dtype=torch.int32, device=dev)
    lp = torch.zeros((2, 4, 8), dtype=torch.float32, device=dev)
    with pytest.raises(TypeError):
        fd.bs_tbs_device(t, beams.cpu(), ids, lp, -10.0, -40.0, 1.0, False)
    with pytest.raises(ValueError):
        fd.bs_tbs_device(t, beams, ids.to(torch.int64), lp, -10.0, -40.0, 1.0, False)
    # A beam width beyond the workspace is refused by the kernel and reported.
    with pytest.raises(RuntimeError):
        fd.bs_tbs_device(t, torch.full((2, 4), 9, dtype=torch.int32, device=dev), ids, lp, -10.0, -40.0, 1.0,
                         False, capacity=9)
    assert fd.device_status(t) == 0


def test_beam_width_above_1024_matches_oracle(built, tmp_path):
    """Exact selection at any width: the reference's radix path above 1024
    beams is broken (candidates-gpu.h:165-316), the engine's is not."""
    import flashtrie
    from oracle.oracle import OracleTrie
    cfg = dict(W.CONFIGS[1], vocab=300, beam=2000, K=64, L=6)
    tok, off = W.gen_keys(60000, cfg["vocab"], cfg["len_lo"], cfg["len_hi"], cfg["zipf"], seed=23)
    tb = flashtrie.Trie()
    tb.build_flat(tok, off)
    p = str(tmp_path / "wide.bin")
    tb.save(p)
    beams, ids, lp = W.gen_requests(1, tok, off, 3, cfg=cfg)
    t = flashtrie.Trie()
    t.load(p)
    t.init_tbs_gpu(3, max_num_topk=64, max_num_outpos=6, max_num_out_beams=2000)
    o = OracleTrie(p)
    for thr in [(-10.0, -40.0), (-30.0, -200.0)]:
        sents, lpns, _, _ = flashtrie.bs_tbs_gpu(t, 3, beams, ids, lp, thr[0], thr[1], 5.0, False)
        for i in range(3):
            o_s, o_l = o.tbs(beams[i], ids[i], lp[i], thr[0], thr[1], 5.0, False)
            assert same_result(sents[i], lpns[i], o_s, o_l), (i, thr)
        assert max(len(s) for s in sents) > 1024  # results wider than 1024 beams


def test_device_calls_with_changing_shape_and_length_norm(built, tmp_path):
    """The device path reuses its uploaded meta and factor tables while the
    batch shape and length norm stay the same: every change must show."""
    import torch
    import flashtrie
    import flashtrie_device as fd
    p, tok, off, cfg = _trie(tmp_path, n_keys=20000, seed=27)
    beams, ids, lp = W.gen_requests(1, tok, off, 10, cfg=cfg)
    t = flashtrie.Trie()
    t.load(p)
    t.init_tbs_gpu(10, max_num_topk=cfg["K"], max_num_outpos=cfg["L"], max_num_out_beams=cfg["beam"])
    dev = torch.device("cuda:0")
    for n, L, ln in [(10, 8, 5.0), (10, 8, 5.0), (10, 8, 1.0), (4, 8, 1.0), (10, 8, 1.0), (6, 5, 1.0), (6, 5, 0.0)]:
        b, i_, l_ = beams[:n, :L].copy(), ids[:n, :L].copy(), lp[:n, :L].copy()
        out = fd.bs_tbs_device(t, torch.from_numpy(b.astype(np.int32)).to(dev),
                               torch.from_numpy(i_.view(np.int32)).to(dev), torch.from_numpy(l_).to(dev),
                               -10.0, -40.0, ln, False)
        d_sents, d_lpns = fd.to_lists(out)
        h_sents, h_lpns, _, _ = flashtrie.bs_tbs_gpu(t, n, b, i_, l_, -10.0, -40.0, ln, False)
        for r in range(n):
            assert same_result(d_sents[r], d_lpns[r], h_sents[r], h_lpns[r]), (n, L, ln, r)
