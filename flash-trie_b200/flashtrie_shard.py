"""Batch sharding of trie-constrained beam search over the GPUs of one node.

The trie is read-only and the requests of a batch are independent, so every
rank (one process per GPU) keeps its own replica of the device trie and
searches a contiguous slice of the batch; nothing crosses NVLink while the
search runs.  The reference searches on device 0 only
(lib/marisa/grimoire/trie/tbs-kernels.cu:599-648 allocates every workspace on
the current device); this module is the multi-GPU layer on top of the same
`bs_tbs_gpu` entry point.

    import torch.distributed as dist, flashtrie, flashtrie_shard as fs
    dist.init_process_group("nccl")            # one process per GPU
    torch.cuda.set_device(local_rank)
    trie = flashtrie.Trie(); trie.load(path)   # replica on this GPU
    trie.init_tbs_gpu(per_rank_batch, ...)
    sents, lpns, ms, phases = fs.bs_tbs_sharded(trie, beams, ids, logps, -10.0, -40.0, 5.0, False)

Every rank passes the whole batch (or the same arrays) and gets the whole
batch's results back in request order; `gather=False` returns only the
rank's own slice.
"""
import torch
import torch.distributed as dist


def shard_range(n, rank, world):
    """Contiguous slice [lo, hi) of n requests for `rank`; the first n % world
    ranks take one extra request."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank %d out of range for world size %d" % (rank, world))
    base, extra = divmod(int(n), world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def _world(group):
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


def bs_tbs_sharded(trie, batch_beams, batch_topk_id, batch_topk_logp, token_logp_threshold,
                   sents_logp_threshold, length_norm, early_exit, group=None, gather=True, search=None):
    """Searches this rank's slice of the batch with `search` (default
    `flashtrie.bs_tbs_gpu`) and, with `gather`, returns the results of the
    whole batch on every rank: (sents, logp_norms, ms, phase_times), where
    ms is the slowest rank's call time.

    With `gather`, a search that raises on one rank still takes part in the
    gather (carrying its error instead of results), and then every rank
    raises: the failing rank its own exception, the others a RuntimeError
    naming the failed rank.  No rank is left waiting in the collective."""
    if search is None:
        import flashtrie
        search = flashtrie.bs_tbs_gpu
    rank, world = _world(group)
    n = len(batch_beams)
    lo, hi = shard_range(n, rank, world)
    collective = gather and world > 1
    error, local = None, None
    try:
        if hi > lo:
            sents, lpns, ms, phases = search(trie, hi - lo, batch_beams[lo:hi], batch_topk_id[lo:hi],
                                             batch_topk_logp[lo:hi], token_logp_threshold, sents_logp_threshold,
                                             length_norm, early_exit)
        else:
            sents, lpns, ms, phases = [], [], 0.0, []
        local = (list(sents), list(lpns), float(ms), list(phases))
    except Exception as e:
        if not collective:
            raise
        error = e
    if not collective:
        return local
    parts = [None] * world
    msg = None if error is None else "%s: %s" % (type(error).__name__, error)
    dist.all_gather_object(parts, (msg, local), group=group)
    if error is not None:
        raise error
    failed = [(r, m) for r, (m, _) in enumerate(parts) if m is not None]
    if failed:
        raise RuntimeError("bs_tbs_sharded: the search failed on rank %d (%s)" % failed[0])
    out_s, out_l, out_p = [], [], []
    for _, (s, l, _, p) in parts:
        out_s.extend(s)
        out_l.extend(l)
        out_p.extend(p)
    return out_s, out_l, max(part[2] for _, part in parts), out_p


def max_over_ranks(values, group=None, device=None):
    """Element-wise maximum of a list of floats over the ranks (timings are
    reported as the slowest rank's); identity without a process group."""
    vals = [float(v) for v in values]
    rank, world = _world(group)
    if world == 1:
        return vals
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" \
            else torch.device("cpu")
    t = torch.tensor(vals, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return [float(x) for x in t.cpu()]
