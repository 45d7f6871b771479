"""GPU parity: the B200 engine (through the drop-in module and the C ABI)
against the C oracle, bit-exact on sequences, lengths and scores, and against
the reference's own CPU outputs (golden) wherever the reference paths agree."""
import ctypes
import math
import os

import numpy as np
import pytest

import workload as W
from helpers import REPO, file_sha, load_json, same_result, sha

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ft(built):
    import flashtrie
    return flashtrie


@pytest.fixture(scope="module")
def c1(ft, tmp_path_factory):
    from oracle.oracle import OracleTrie
    g = load_json("search_c1.json")
    cfg = W.CONFIGS[1]
    tok, off = W.gen_keys(cfg["keys"], cfg["vocab"], cfg["len_lo"], cfg["len_hi"], cfg["zipf"], seed=g["key_seed"])
    t = ft.Trie()
    t.build(token_rows=W.key_rows(tok, off))
    p = str(tmp_path_factory.mktemp("c1") / "c1.bin")
    t.save(p)
    assert file_sha(p) == g["trie_sha256"]
    t.init_tbs_gpu(16, max_num_topk=64, max_num_outpos=8, max_num_out_beams=64)
    return t, OracleTrie(p), tok, off, g


def run_one(ft, trie, beams, ids, lp, thr, ee):
    sent, lpn, _ = ft.tbs(trie, list(map(int, beams)), np.asarray(ids, np.uint32), np.asarray(lp, np.float32),
                          thr[0], thr[1], thr[2], ee, True)
    return sent, lpn


def test_c1_single_requests_match_oracle_and_reference(ft, c1):
    trie, oracle, tok, off, g = c1
    reqs = g["requests"]
    beams, ids, lp = W.gen_requests(1, tok, off, len(reqs))
    ref_exact = 0
    for r in reqs:
        i = r["index"]
        assert sha(beams[i], ids[i], lp[i]) == r["inputs_sha256"]
        sent, lpn = run_one(ft, trie, beams[i], ids[i], lp[i], g["thresholds"], r["early_exit"])
        o_sent, o_lpn = oracle.tbs(beams[i], ids[i], lp[i], *g["thresholds"], r["early_exit"])
        assert same_result(sent, lpn, o_sent, o_lpn), "request %d differs from the oracle" % i
        if same_result(sent, lpn, r["ref_sent"], r["ref_lpn"]):
            ref_exact += 1
        else:
            assert r["ref_invalid"] or r["early_exit"]
    assert ref_exact >= 119


def check_config_shape(search, tmp_path, cfg_id):
    """The request shape of config `cfg_id` on the 200k-key trie of its
    golden fixture: `search(trie_path, beams, ids, lp, thresholds, cfg)` must
    return, for every request, exactly the oracle's result and exactly the
    unmodified reference CPU's (every request of these fixtures is one where
    the reference paths agree)."""
    import flashtrie
    from oracle.oracle import OracleTrie
    g = load_json("search_c%d.json" % cfg_id)
    cfg = dict(W.CONFIGS[cfg_id], keys=g["keys"])
    tok, off = W.gen_keys(cfg["keys"], cfg["vocab"], cfg["len_lo"], cfg["len_hi"], cfg["zipf"], seed=g["key_seed"])
    t = flashtrie.Trie()
    t.build_flat(tok, off)
    p = str(tmp_path / "shape.bin")
    t.save(p)
    assert file_sha(p) == g["trie_sha256"]
    reqs = g["requests"]
    beams, ids, lp = W.gen_requests(cfg_id, tok, off, len(reqs), cfg=cfg)
    for r in reqs:
        assert sha(beams[r["index"]], ids[r["index"]], lp[r["index"]]) == r["inputs_sha256"]
    sents, lpns = search(p, beams, ids, lp, g["thresholds"], cfg)
    o = OracleTrie(p)
    for r in reqs:
        i = r["index"]
        o_sent, o_lpn = o.tbs(beams[i], ids[i], lp[i], *g["thresholds"], False)
        assert same_result(sents[i], lpns[i], o_sent, o_lpn), "request %d differs from the oracle" % i
        assert same_result(sents[i], lpns[i], r["ref_sent"], r["ref_lpn"]), "request %d differs from the reference" % i


@pytest.mark.parametrize("cfg_id", [2, 3])
def test_config_shapes_match_reference(ft, tmp_path, cfg_id):
    """Configs 2 and 3's request shapes (K=256, L=16, beam 100; K=1000,
    L=20, beam 1000), the whole fixture as one batch through bs_tbs_gpu:
    identical to the oracle and to the reference CPU's own outputs."""
    def search(path, beams, ids, lp, thr, cfg):
        t = ft.Trie()
        t.load(path)
        n = beams.shape[0]
        t.init_tbs_gpu(n, max_num_topk=cfg["K"], max_num_outpos=cfg["L"], max_num_out_beams=cfg["beam"])
        sents, lpns, _, _ = ft.bs_tbs_gpu(t, n, beams, ids, lp, thr[0], thr[1], thr[2], False)
        return sents, lpns
    check_config_shape(search, tmp_path, cfg_id)


def test_c1_batched_matches_single(ft, c1):
    trie, oracle, tok, off, g = c1
    beams, ids, lp = W.gen_requests(1, tok, off, 16, start=200)
    for ee in (False, True):
        sents, lpns, ms, phases = ft.bs_tbs_gpu(trie, 16, beams.tolist(), ids.tolist(), lp.tolist(),
                                                *g["thresholds"], ee)
        assert len(phases) == 16 and all(len(p) == 5 for p in phases)
        for i in range(16):
            o_sent, o_lpn = oracle.tbs(beams[i], ids[i], lp[i], *g["thresholds"], ee)
            assert same_result(sents[i], lpns[i], o_sent, o_lpn), (ee, i)
        # numpy fast path gives the same answer
        s2, l2, _, _ = ft.bs_tbs_gpu(trie, 16, beams, ids, lp, *g["thresholds"], ee)
        assert s2 == sents and l2 == lpns


def test_hand_tries_match_oracle(ft, tmp_path):
    from oracle.oracle import OracleTrie
    g = load_json("search_hand.json")
    tries = {}
    for name, keys in g["keysets"].items():
        t = ft.Trie()
        t.build(token_rows=keys)
        p = str(tmp_path / (name + ".bin"))
        t.save(p)
        t.init_tbs_gpu(1, max_num_topk=16, max_num_outpos=8, max_num_out_beams=8)
        tries[name] = (t, OracleTrie(p))
    for r in g["requests"]:
        t, o = tries[r["trie"]]
        args = (r["beams"], r["topk_id"], r["topk_logp"], r["token_logp_threshold"], r["sents_logp_threshold"],
                r["length_norm"], r["early_exit"])
        sent, lpn, _ = ft.tbs(t, *args, True)
        o_sent, o_lpn = o.tbs(*args)
        assert same_result(sent, lpn, o_sent, o_lpn), r


def random_case(rng, n_keys, vocab, max_len, L, K, B, dup_rows=False, unsorted=False):
    keys = [rng.integers(0, vocab, size=int(rng.integers(1, max_len + 1))).tolist() for _ in range(n_keys)]
    ids = np.zeros((L, K), np.uint32)
    for t in range(L):
        row = rng.choice(vocab, size=K, replace=dup_rows or K > vocab)
        ids[t] = row if unsorted else np.sort(row)
    lp = (-rng.exponential(1.5, size=(L, K))).astype(np.float32)
    beams = [B] * L
    return keys, beams, ids, lp


@pytest.mark.parametrize("seed", range(12))
def test_random_tries_match_oracle(ft, tmp_path, seed):
    from oracle.oracle import OracleTrie
    rng = np.random.default_rng(100 + seed)
    vocab = int(rng.choice([3, 16, 300, 5000]))
    L = int(rng.integers(1, 10))
    K = int(rng.choice([1, 7, 64, 300, 1024]))
    B = int(rng.choice([1, 5, 50, 400]))
    keys, beams, ids, lp = random_case(rng, int(rng.choice([10, 2000, 30000])), vocab, 9, L, K, B,
                                       dup_rows=seed % 3 == 0, unsorted=seed % 4 == 1)
    t = ft.Trie()
    t.build(token_rows=keys)
    p = str(tmp_path / "r.bin")
    t.save(p)
    o = OracleTrie(p)
    t.init_tbs_gpu(1, max_num_topk=max(K, 1), max_num_outpos=L, max_num_out_beams=B)
    for ln, ee, thr in [(0.0, False, (-10.0, -40.0)), (5.0, seed % 2 == 0, (-1.0, -6.0)), (1.0, False, (-30, -100))]:
        sent, lpn, _ = ft.tbs(t, beams, ids, lp, thr[0], thr[1], ln, ee, True)
        o_sent, o_lpn = o.tbs(beams, ids, lp, thr[0], thr[1], ln, ee)
        assert same_result(sent, lpn, o_sent, o_lpn), (seed, ln, ee, thr)


def test_edge_cases(ft, tmp_path):
    from oracle.oracle import OracleTrie
    t = ft.Trie()
    keys = [[1, 2, 3, 4], [1, 2, 3, 5], [20, 21, 22], [20, 21, 22, 23], [7], [7, 8]]
    t.build(token_rows=keys)
    p = str(tmp_path / "e.bin")
    t.save(p)
    o = OracleTrie(p)
    t.init_tbs_gpu(2, max_num_topk=8, max_num_outpos=6, max_num_out_beams=8)
    ids = [[1, 7, 20, 4294967295], [2, 8, 21, 4294967295], [3, 22, 4294967295, 4294967295],
           [4, 5, 23, 4294967295]]
    fm = -3.4028234663852886e38
    lp = [[-1.0, -2.0, -0.5, fm], [-1.0, -0.25, -0.125, fm], [-0.5, -0.75, fm, fm], [-1.0, -2.0, -3.0, fm]]
    cases = [
        ([4, 4, 4, 4], False),
        ([1, 1, 1, 1], False),
        ([4, 0, 4, 4], False),       # zero width mid-way: nothing survives
        ([4, 4, 4, 0], False),       # final beam 0: empty result
        ([2, 2, 2, 2], True),
        ([4], False),                # one position
    ]
    for beams, ee in cases:
        L = len(beams)
        sent, lpn, _ = ft.tbs(t, beams, ids[:L], lp[:L], -10.0, -40.0, 1.0, ee, True)
        o_sent, o_lpn = o.tbs(beams, ids[:L], lp[:L], -10.0, -40.0, 1.0, ee)
        assert same_result(sent, lpn, o_sent, o_lpn), beams
        if beams[-1] == 0:
            assert sent == [] and lpn == []
    # thresholds are strict (<= drops): a logp exactly at the token threshold
    sent, lpn, _ = ft.tbs(t, [4], [[7]], [[-2.0]], -2.0, -40.0, 1.0, False, True)
    assert sent == []
    sent, lpn, _ = ft.tbs(t, [4], [[7]], [[-1.5]], -2.0, -40.0, 1.0, False, True)
    assert sent == [[7]]
    # K = 0 rows
    sent, lpn, _ = ft.tbs(t, [4, 4], [[], []], [[], []], -10.0, -40.0, 1.0, False, True)
    assert sent == []
    # limits are enforced
    with pytest.raises(ValueError):
        ft.tbs(t, [9], [[7]], [[-1.0]], -10.0, -40.0, 1.0, False, True)
    with pytest.raises(ValueError):
        ft.tbs(t, [], [], [], -10.0, -40.0, 1.0, False, True)


def test_empty_and_single_key_tries(ft, tmp_path):
    from oracle.oracle import OracleTrie
    for keys in ([], [[]], [[5]], [[0xFFFFFFFF, 3, 4], [1, 2, 3], [1, 2, 4]]):
        t = ft.Trie()
        t.build(token_rows=keys)
        p = str(tmp_path / "k.bin")
        t.save(p)
        o = OracleTrie(p)
        ids = [[0, 1, 5, 0xFFFFFFFF], [2, 3, 4, 5], [3, 4, 5, 6]]
        lp = [[-1.0, -1.0, -1.0, -1.0]] * 3
        sent, lpn, _ = ft.tbs(t, [3, 3, 3], ids, lp, -10.0, -40.0, 1.0, False, True)
        o_sent, o_lpn = o.tbs([3, 3, 3], ids, lp, -10.0, -40.0, 1.0, False)
        assert same_result(sent, lpn, o_sent, o_lpn), keys


def test_device_entry_point_matches_host(ft, c1, tmp_path):
    """ft_tbs_batch_device on torch device buffers == the host entry point."""
    import torch
    trie, oracle, tok, off, g = c1
    n = 8
    beams, ids, lp = W.gen_requests(1, tok, off, n, start=300)
    lib = ctypes.CDLL(os.path.join(REPO, "flash-trie_b200", "libftcore.so"))

    class Params(ctypes.Structure):
        _fields_ = [("token_logp_threshold", ctypes.c_float), ("reserved", ctypes.c_float),
                    ("sent_logp_threshold", ctypes.c_double), ("length_norm", ctypes.c_double),
                    ("early_exit", ctypes.c_int32), ("reserved2", ctypes.c_int32)]

    class Batch(ctypes.Structure):
        _fields_ = [("n", ctypes.c_uint32), ("num_outpos", ctypes.c_uint32), ("topk", ctypes.c_uint32),
                    ("out_capacity", ctypes.c_uint32)] + [(f, ctypes.c_void_p) for f in
                                                          ("beams", "topk_id", "topk_logp", "out_count", "out_lpn",
                                                           "out_len", "out_tok", "out_key")]

    dev = torch.device("cuda:0")
    d_beams = torch.from_numpy(beams.astype(np.int32)).to(dev)
    d_ids = torch.from_numpy(ids.view(np.int32)).to(dev)
    d_lp = torch.from_numpy(lp).to(dev)
    L, K, cap = beams.shape[1], ids.shape[2], int(beams[0, -1])
    out_count = torch.zeros(n, dtype=torch.int32, device=dev)
    out_lpn = torch.zeros(n * cap, dtype=torch.float64, device=dev)
    out_len = torch.zeros(n * cap, dtype=torch.int32, device=dev)
    out_tok = torch.zeros(n * cap * L, dtype=torch.int32, device=dev)
    b = Batch(n, L, K, cap, d_beams.data_ptr(), d_ids.data_ptr(), d_lp.data_ptr(), out_count.data_ptr(),
              out_lpn.data_ptr(), out_len.data_ptr(), out_tok.data_ptr())
    prm = Params(g["thresholds"][0], 0.0, g["thresholds"][1], g["thresholds"][2], 0, 0)
    # The Python trie object wraps an ft_trie*; reach it through a fresh C-ABI handle instead.
    h = ctypes.c_void_p()
    assert lib.ft_trie_create(ctypes.byref(h)) == 0
    path = str(tmp_path / "c1_dev.bin")
    trie.save(path)
    assert lib.ft_trie_load(h, path.encode()) == 0
    assert lib.ft_trie_init_tbs_gpu(h, ctypes.c_uint64(n), ctypes.c_uint64(K), ctypes.c_uint64(L),
                                    ctypes.c_uint64(cap), ctypes.c_uint64(cap * L), ctypes.c_uint64(cap * L),
                                    ctypes.c_uint64(1024)) == 0
    stream = torch.cuda.current_stream(dev)
    assert lib.ft_tbs_batch_device(h, ctypes.byref(b), ctypes.byref(prm), ctypes.c_void_p(stream.cuda_stream)) == 0
    torch.cuda.synchronize()
    st = ctypes.c_uint32(99)
    assert lib.ft_trie_device_status(h, ctypes.byref(st)) == 0 and st.value == 0
    cnt = out_count.cpu().numpy()
    lpn_h = out_lpn.cpu().numpy().reshape(n, cap)
    len_h = out_len.cpu().numpy().reshape(n, cap)
    tok_h = out_tok.cpu().numpy().view(np.uint32).reshape(n, cap, L)
    for i in range(n):
        o_sent, o_lpn = oracle.tbs(beams[i], ids[i], lp[i], *g["thresholds"], False)
        sent = [tok_h[i, j, :len_h[i, j]].tolist() for j in range(cnt[i])]
        assert same_result(sent, lpn_h[i, :cnt[i]].tolist(), o_sent, o_lpn), i
    lib.ft_trie_destroy(h)
