"""Multi-rank host logic on CPU (gloo, world size 2): batch sharding, the
result gather, max-over-ranks timing and the bench's reference arm under
torchrun.  The search itself needs a GPU; here a deterministic stand-in
search checks that sharding and gathering preserve request order."""
import json
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

from helpers import REPO

import flashtrie_shard as fs


def test_shard_range_partitions_every_batch():
    for n in range(0, 40):
        for world in range(1, 9):
            spans = [fs.shard_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        fs.shard_range(4, 2, 2)


def fake_search(trie, n, beams, ids, lps, tt, st, ln, ee):
    """Stands in for bs_tbs_gpu: one result per request derived from it."""
    assert n == len(beams) == len(ids) == len(lps)
    sents = [[[int(ids[i][0][0]), int(beams[i][0])]] for i in range(n)]
    lpns = [[float(lps[i][0][0]) * ln] for i in range(n)]
    phases = [[0.0, 0.0, 0.0, 0.0, float(ids[i][1][1])] for i in range(n)]
    return sents, lpns, 0.5 + n, phases


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n, q):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        rng = np.random.default_rng(7)
        beams = rng.integers(1, 50, size=(n, 3)).astype(np.uint32)
        ids = rng.integers(0, 1000, size=(n, 3, 4)).astype(np.uint32)
        lps = -rng.random((n, 3, 4)).astype(np.float32)
        got = fs.bs_tbs_sharded(None, beams, ids, lps, -10.0, -40.0, 2.0, False, search=fake_search)
        want = fake_search(None, n, beams, ids, lps, -10.0, -40.0, 2.0, False)
        lo, hi = fs.shard_range(n, rank, world)
        own = fs.bs_tbs_sharded(None, beams, ids, lps, -10.0, -40.0, 2.0, False, search=fake_search, gather=False)
        mx = fs.max_over_ranks([float(rank), 10.0 - rank])
        q.put((rank, got[0] == want[0], got[1] == want[1], got[3] == want[3], len(own[0]) == hi - lo,
               got[2], mx))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [5, 1, 8])
def test_sharded_search_gathers_in_request_order(n):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(world))
    for rank, s_ok, l_ok, p_ok, own_ok, ms, mx in res:
        assert s_ok and l_ok and p_ok and own_ok, rank
        # ms is the slowest rank's: the rank with the larger slice
        assert ms == 0.5 + fs.shard_range(n, 0, world)[1]
        assert mx == [1.0, 10.0]


def failing_search(trie, n, beams, ids, lps, tt, st, ln, ee):
    """Raises when its slice holds a request marked bad (beam width -1)."""
    if any(int(b[0]) == -1 for b in beams):
        raise ValueError("tbs: beam width exceeds max_num_out_beams")
    return fake_search(trie, n, beams, ids, lps, tt, st, ln, ee)


def _failing_worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        n = 6
        beams = np.ones((n, 3), dtype=np.int64)
        beams[n - 1, 0] = -1  # a bad request in the last rank's slice
        ids = np.zeros((n, 3, 4), dtype=np.uint32)
        lps = -np.ones((n, 3, 4), dtype=np.float32)
        try:
            fs.bs_tbs_sharded(None, beams, ids, lps, -10.0, -40.0, 2.0, False, search=failing_search)
            q.put((rank, "returned"))
        except ValueError as e:
            q.put((rank, "ValueError: %s" % e))
        except RuntimeError as e:
            q.put((rank, "RuntimeError: %s" % e))
        # The group is still usable: every rank took the same collective steps.
        got = fs.bs_tbs_sharded(None, np.ones((n, 3), dtype=np.int64), ids, lps, -10.0, -40.0, 2.0, False,
                                search=fake_search)
        q.put((rank, "after: %d" % len(got[0])))
    finally:
        dist.destroy_process_group()


def test_sharded_search_failure_raises_on_every_rank():
    """A search that raises on one rank makes every rank raise, with no rank
    left waiting in the gather: the failing rank its own error, the others a
    RuntimeError naming it; the process group stays usable."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(2 * world))
    assert res == [(0, "RuntimeError: bs_tbs_sharded: the search failed on rank 1 "
                       "(ValueError: tbs: beam width exceeds max_num_out_beams)"),
                   (0, "after: 6"),
                   (1, "ValueError: tbs: beam width exceeds max_num_out_beams"),
                   (1, "after: 6")], res


def test_bench_reference_arm_under_torchrun(tmp_path):
    """Two ranks, CPU: rank 0 alone runs the reference CPU arm and prints one
    JSON line; rank 1 exits 0 without work."""
    ref = os.path.join(REPO, "oracle", "_ref")
    if not (os.path.isdir(ref) and any(f.startswith("flashtrie_ref") for f in os.listdir(ref))):
        pytest.skip("oracle/_ref not built (reference sources absent)")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(REPO, "bench.py"), "--impl", "reference", "--gpus", "2", "--steps", "3", "--warmup", "3",
           "--config", "1", "--keys", "20000", "--requests", "4", "--cpu-budget", "0.5",
           "--trie-dir", str(tmp_path)]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env, cwd=str(tmp_path))
    assert r.returncode == 0, r.stderr[-3000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["value"] > 0 and d["cpu_baseline"]["kind"] == "reference"
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["n_gpus"] == 2
    # The arm searched a trie the reference's own builder wrote, and never
    # loaded the engine.
    assert d["config"]["trie_built_by"].startswith("reference builder"), d["config"]
    assert d["engine_modules_loaded"] == [] and d["steps"] == 3
