"""Batch sharding on GPUs: the sharded search returns exactly what one search
of the whole batch returns (world size 1 on one GPU; world size 2 over NCCL
when the box has two GPUs), and large batches (compact result tokens, two-
phase copy) agree with the oracle request by request."""
import os
import socket

import numpy as np
import pytest

import workload as W
from helpers import same_result

pytestmark = pytest.mark.gpu


def _small_trie(tmp_path, n_keys=20000, seed=5):
    import flashtrie
    cfg = dict(W.CONFIGS[1])
    tok, off = W.gen_keys(n_keys, cfg["vocab"], cfg["len_lo"], cfg["len_hi"], cfg["zipf"], seed=seed)
    t = flashtrie.Trie()
    t.build_flat(tok, off)
    p = str(tmp_path / "m.bin")
    t.save(p)
    return p, tok, off, cfg


def test_sharded_world1_equals_plain(built, tmp_path):
    import flashtrie
    import flashtrie_shard as fs
    p, tok, off, cfg = _small_trie(tmp_path)
    beams, ids, lp = W.gen_requests(1, tok, off, 9, cfg=cfg)
    t = flashtrie.Trie()
    t.load(p)
    t.init_tbs_gpu(9, max_num_topk=cfg["K"], max_num_outpos=cfg["L"], max_num_out_beams=cfg["beam"])
    a = flashtrie.bs_tbs_gpu(t, 9, beams, ids, lp, -10.0, -40.0, 5.0, False)
    b = fs.bs_tbs_sharded(t, beams, ids, lp, -10.0, -40.0, 5.0, False)
    assert a[0] == b[0] and a[1] == b[1]


def test_large_batch_matches_oracle(built, tmp_path):
    """A batch whose strided token region exceeds the one-copy limit takes the
    compact two-phase result path; every request must match the oracle."""
    import flashtrie
    from oracle.oracle import OracleTrie
    p, tok, off, cfg = _small_trie(tmp_path, n_keys=50000, seed=7)
    cfg = dict(cfg, beam=200, K=64, L=8)
    n = 48  # 48 * 200 * 8 * 4 bytes of token slots > 256 KB
    beams, ids, lp = W.gen_requests(1, tok, off, n, cfg=cfg)
    t = flashtrie.Trie()
    t.load(p)
    t.init_tbs_gpu(n, max_num_topk=64, max_num_outpos=8, max_num_out_beams=200)
    sents, lpns, _, _ = flashtrie.bs_tbs_gpu(t, n, beams, ids, lp, -10.0, -40.0, 5.0, False)
    o = OracleTrie(p)
    for i in range(n):
        o_s, o_l = o.tbs(beams[i], ids[i], lp[i], -10.0, -40.0, 5.0, False)
        assert same_result(sents[i], lpns[i], o_s, o_l), i


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, path, q):
    import datetime
    import torch
    import torch.distributed as dist
    import flashtrie
    import flashtrie_shard as fs
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        cfg = dict(W.CONFIGS[1])
        tok = np.load(path + ".tok.npy")
        off = np.load(path + ".off.npy")
        beams, ids, lp = W.gen_requests(1, tok, off, 7, cfg=cfg)
        t = flashtrie.Trie()
        t.load(path)
        t.init_tbs_gpu(7, max_num_topk=cfg["K"], max_num_outpos=cfg["L"], max_num_out_beams=cfg["beam"])
        got = fs.bs_tbs_sharded(t, beams, ids, lp, -10.0, -40.0, 5.0, False)
        want = flashtrie.bs_tbs_gpu(t, 7, beams, ids, lp, -10.0, -40.0, 5.0, False)
        q.put((rank, got[0] == want[0] and got[1] == want[1]))
    finally:
        dist.destroy_process_group()


def test_sharded_world2_nccl(built, tmp_path):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    p, tok, off, cfg = _small_trie(tmp_path)
    np.save(p + ".tok.npy", tok)
    np.save(p + ".off.npy", off)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, p, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(300)
        assert pr.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(2))
    assert all(ok for _, ok in res), res


@pytest.mark.parametrize("dense", ["0", "1"])
def test_batch_beyond_sm_count_matches_oracle(built, tmp_path, monkeypatch, dense):
    """300 requests: more than one per SM, so one-CTA teams take requests in
    turn; with FT_DENSE=1 the two-CTAs-per-SM kernel instance runs them."""
    import flashtrie
    from oracle.oracle import OracleTrie
    monkeypatch.setenv("FT_DENSE", dense)
    p, tok, off, cfg = _small_trie(tmp_path, n_keys=30000, seed=11)
    n = 300
    beams, ids, lp = W.gen_requests(1, tok, off, n, cfg=cfg)
    t = flashtrie.Trie()
    t.load(p)
    t.init_tbs_gpu(n, max_num_topk=cfg["K"], max_num_outpos=cfg["L"], max_num_out_beams=cfg["beam"])
    sents, lpns, _, _ = flashtrie.bs_tbs_gpu(t, n, beams, ids, lp, -10.0, -40.0, 5.0, False)
    o = OracleTrie(p)
    for i in range(n):
        o_s, o_l = o.tbs(beams[i], ids[i], lp[i], -10.0, -40.0, 5.0, False)
        assert same_result(sents[i], lpns[i], o_s, o_l), i
