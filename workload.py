"""Seeded synthetic workloads for the five configurations the reference's
metric is quoted on (keys and per-request top-K proposals).

The paper's production requests and the NQ-Open/KILT setup are not available,
so these stand in for them with the shapes and value distributions the
configurations name:
  keys      N distinct keys, length uniform in [lo, hi], tokens i.i.d. Zipf(s)
            over ids 0..V-1 (id = rank-1, P(rank) proportional to rank^-s),
            key seed = config id;
  requests  a target key drawn uniformly; at position i < len(target) the row
            holds target[i]; the row is filled to K distinct ids with Zipf(s)
            draws without replacement; logits ~ N(0, 2) with the target +3;
            logp = log_softmax(logits) in f64, stored as f32; rows sorted by
            id; request seed = 1000 * config + request index.
  config 5  30% of requests are off-trie: their boosted token at position 0
            is resampled from ids that are not root children, later positions
            from uniform ids.
Used by bench.py and tests; the engine itself never imports it.
"""
import numpy as np

CONFIGS = {
    1: dict(keys=100_000, vocab=32_000, len_lo=2, len_hi=8, zipf=1.1, K=64, L=8, beam=10,
            batch=1, early_exit=False, off_trie=0.0),
    2: dict(keys=10_000_000, vocab=500_000, len_lo=3, len_hi=16, zipf=1.05, K=256, L=16, beam=100,
            batch=1, early_exit=False, off_trie=0.0),
    3: dict(keys=200_000_000, vocab=2_200_000, len_lo=4, len_hi=20, zipf=1.0, K=1000, L=20, beam=1000,
            batch=1, early_exit=False, off_trie=0.0),
    4: dict(keys=800_000_000, vocab=2_200_000, len_lo=4, len_hi=24, zipf=1.0, K=1000, L=24, beam=1000,
            batch=64, early_exit=False, off_trie=0.0),
    5: dict(keys=800_000_000, vocab=2_200_000, len_lo=4, len_hi=24, zipf=1.0, K=1000, L=24, beam=1000,
            batch=64, early_exit=True, off_trie=0.3),
}
# Key-length distributions.  "spec" is the configuration's own (uniform in
# [len_lo, len_hi]).  Configs 4 and 5 as written (800M keys, lengths 4-24)
# need about 11G tail labels, beyond the 2^32-label tail of the trie format
# (lib/marisa/grimoire/trie/tail.cc:221), so at 800M keys they use
# "ref-lengths": lengths 1-8 drawn with the reference's example-generator
# weights 2,10,45,25,10,5,2,1 (examples/make_example_data.py:57), the
# distribution behind the reference's 800M-key index figure; vocabulary and
# Zipf exponent stay the configuration's.
KEYSETS = {
    "spec": {},
    "ref-lengths": dict(len_lo=1, len_hi=8, len_weights=(2, 10, 45, 25, 10, 5, 2, 1)),
}
DEFAULT_KEYSET = {1: "spec", 2: "spec", 3: "spec", 4: "ref-lengths", 5: "ref-lengths"}


def resolve(cfg_id, keyset=None, **overrides):
    """The configuration's parameters with its key-length distribution
    (`keyset`, default per config) and any overrides applied."""
    cfg = dict(CONFIGS[cfg_id])
    ks = keyset or DEFAULT_KEYSET[cfg_id]
    cfg.update(KEYSETS[ks])
    cfg["keyset"] = ks
    cfg.setdefault("len_weights", None)
    for k, v in overrides.items():
        if v:
            cfg[k] = v
    return cfg


TOKEN_LOGP_THRESHOLD = -10.0
SENT_LOGP_THRESHOLD = -40.0
LENGTH_NORM = 5.0


class Zipf:
    """Inverse-CDF sampler for Zipf(s) over ids 0..V-1."""

    def __init__(self, vocab, s):
        w = np.arange(1, vocab + 1, dtype=np.float64) ** (-float(s))
        self.cdf = np.cumsum(w)
        self.cdf /= self.cdf[-1]
        self.vocab = vocab

    def draw(self, rng, n):
        u = rng.random(n)
        ids = np.searchsorted(self.cdf, u, side="right")
        return np.minimum(ids, self.vocab - 1).astype(np.uint32)


def _row_hash(mat, lens):
    h = np.full(mat.shape[0], np.uint64(1469598103934665603), dtype=np.uint64)
    prime = np.uint64(1099511628211)
    with np.errstate(over="ignore"):
        for c in range(mat.shape[1]):
            h = (h ^ mat[:, c].astype(np.uint64)) * prime
        h = (h ^ lens.astype(np.uint64)) * prime
    return h


def gen_keys(n, vocab, len_lo, len_hi, zipf_s, seed, chunk=4_000_000):
    """Returns (tokens u32[total], offsets u64[n+1]) of n distinct keys."""
    rng = np.random.default_rng(seed)
    z = Zipf(vocab, zipf_s)
    width = len_hi
    mats, lens_all, hashes = [], [], []
    have = 0
    while have < n:
        m = int(min(chunk, (n - have) * 1.2 + 1024))
        lens = rng.integers(len_lo, len_hi + 1, size=m).astype(np.uint32)
        mat = z.draw(rng, m * width).reshape(m, width)
        mask = np.arange(width)[None, :] >= lens[:, None]
        mat[mask] = 0
        h = _row_hash(mat, lens)
        mats.append(mat)
        lens_all.append(lens)
        hashes.append(h)
        allh = np.concatenate(hashes)
        _, first = np.unique(allh, return_index=True)
        have = len(first)
    mat = np.concatenate(mats)
    lens = np.concatenate(lens_all)
    allh = np.concatenate(hashes)
    _, first = np.unique(allh, return_index=True)
    first = np.sort(first)[:n]
    mat = mat[first]
    lens = lens[first]
    offsets = np.zeros(n + 1, np.uint64)
    np.cumsum(lens, out=offsets[1:])
    mask = np.arange(width)[None, :] < lens[:, None]
    tokens = mat[mask].astype(np.uint32)
    return tokens, offsets


def key_rows(tokens, offsets):
    return [tokens[offsets[i]:offsets[i + 1]].tolist() for i in range(len(offsets) - 1)]


def gen_request(tokens, offsets, vocab, K, L, zipf_s, seed, zipf=None, off_trie=False, root_children=None):
    """One request: (beams placeholder-free ids u32[L,K], logp f32[L,K])."""
    rng = np.random.default_rng(seed)
    z = zipf or Zipf(vocab, zipf_s)
    n = len(offsets) - 1
    t = int(rng.integers(0, n))
    target = tokens[offsets[t]:offsets[t + 1]]
    ids = np.zeros((L, K), np.uint32)
    logp = np.zeros((L, K), np.float32)
    for i in range(L):
        tgt = None
        if i < len(target):
            tgt = int(target[i])
            if off_trie:
                if i == 0 and root_children is not None:
                    while True:
                        c = int(rng.integers(0, vocab))
                        if c not in root_children:
                            tgt = c
                            break
                else:
                    tgt = int(rng.integers(0, vocab))
        row = [] if tgt is None else [tgt]
        chosen = set(row)
        while len(row) < K:
            need = K - len(row)
            for c in z.draw(rng, max(2 * need, 64)).tolist():
                if c not in chosen:
                    chosen.add(c)
                    row.append(c)
                    if len(row) == K:
                        break
            if len(chosen) >= vocab:
                break
        row = np.array(row[:K], dtype=np.uint32)
        logits = rng.normal(0.0, 2.0, size=len(row))
        if tgt is not None:
            logits[0] += 3.0
        m = logits.max()
        lse = m + np.log(np.exp(logits - m).sum())
        lp = (logits - lse).astype(np.float32)
        order = np.argsort(row, kind="stable")
        ids[i, :len(row)] = row[order]
        logp[i, :len(row)] = lp[order]
    return ids, logp


def gen_requests(cfg_id, tokens, offsets, n_requests, start=0, cfg=None, root_children=None):
    cfg = cfg or CONFIGS[cfg_id]
    z = Zipf(cfg["vocab"], cfg["zipf"])
    out_ids, out_lp = [], []
    for r in range(start, start + n_requests):
        seed = 1000 * cfg_id + r
        off = False
        if cfg.get("off_trie", 0.0) > 0:
            off = np.random.default_rng(10_000_000 + seed).random() < cfg["off_trie"]
        ids, lp = gen_request(tokens, offsets, cfg["vocab"], cfg["K"], cfg["L"], cfg["zipf"], seed,
                              zipf=z, off_trie=off, root_children=root_children)
        out_ids.append(ids)
        out_lp.append(lp)
    beams = np.full((n_requests, cfg["L"]), cfg["beam"], np.uint32)
    return beams, np.stack(out_ids), np.stack(out_lp)


def gen_keys_torch(n, vocab, len_lo, len_hi, zipf_s, seed, device="cuda", len_weights=None, sort=False):
    """Same distribution as gen_keys, drawn with torch on `device` (seconds for
    10^7-10^8 keys on a GPU instead of minutes with numpy).  Deterministic for
    a given seed and device type; returns numpy (tokens u32, offsets u64).

    len_weights: relative frequencies of the lengths len_lo..len_hi instead of
    a uniform length (the reference's example generator draws lengths 1..8
    with weights 2,10,45,25,10,5,2,1, examples/make_example_data.py:57);
    duplicates are dropped after drawing, so short keys end up rarer than
    their weight where their distinct count runs out.
    sort: return the keys in lexicographic order (a shorter key before the
    keys it prefixes), the order every trie builder sorts them into; the
    key set is the same either way."""
    import torch
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(int(seed))
    w = torch.arange(1, vocab + 1, dtype=torch.float64, device=dev).pow(-float(zipf_s))
    cdf = torch.cumsum(w, 0)
    cdf /= cdf[-1].clone()
    width = len_hi
    cols = torch.arange(width, device=dev)
    if len_weights is not None:
        lw = torch.tensor([float(x) for x in len_weights], dtype=torch.float64, device=dev)
        if lw.numel() != len_hi - len_lo + 1 or bool((lw < 0).any()) or float(lw.sum()) <= 0:
            raise ValueError("len_weights needs one non-negative weight per length %d..%d" % (len_lo, len_hi))
        lw /= lw.sum()
    mats, lens_l, hashes = [], [], []
    keep = None
    m = int(n * 1.1) + 4096
    chunk = 32 << 20  # rows drawn per call; bounds the f64 scratch at 10^8+ keys
    while True:
        for c0 in range(0, m, chunk):
            mc = min(chunk, m - c0)
            if len_weights is None:
                lens = torch.randint(len_lo, len_hi + 1, (mc,), generator=g, device=dev)
            else:
                lens = torch.multinomial(lw, mc, replacement=True, generator=g) + len_lo
            u = torch.rand(mc * width, generator=g, device=dev, dtype=torch.float64)
            mat = torch.searchsorted(cdf, u, right=True).clamp_(max=vocab - 1).view(mc, width)
            del u
            mat.masked_fill_(cols[None, :] >= lens[:, None], 0)
            h = lens.to(torch.int64) * 1000003
            for c in range(width):
                h = (h ^ mat[:, c]) * 1099511628211 + 7
            mats.append(mat.to(torch.int32))
            lens_l.append(lens.to(torch.int32))
            hashes.append(h)
            del mat
        h = torch.cat(hashes)
        hs, perm = torch.sort(h, stable=True)
        del h
        first = torch.ones_like(hs, dtype=torch.bool)
        first[1:] = hs[1:] != hs[:-1]
        del hs
        keep = torch.sort(perm[first]).values
        del perm, first
        if keep.numel() >= n:
            break
        m = int((n - keep.numel()) * 1.3) + 4096
    keep = keep[:n]
    allm = torch.cat(mats) if len(mats) > 1 else mats[0]
    mats.clear()
    alll = torch.cat(lens_l)
    mat = allm[keep]
    del allm
    lens = alll[keep].to(torch.int64)
    if sort:
        # LSD: stable sorts by column from the last to the first; a position
        # past a key's end sorts before every token (token + 1 vs 0).
        perm = torch.arange(n, device=dev)
        for c in range(width - 1, -1, -1):
            col = torch.where(lens[perm] > c, mat[perm, c].to(torch.int64) + 1, 0)
            perm = perm[torch.sort(col, stable=True).indices]
            del col
        mat = mat[perm]
        lens = lens[perm]
        del perm
    offsets = torch.zeros(n + 1, dtype=torch.int64, device=dev)
    torch.cumsum(lens, 0, out=offsets[1:])
    tokens = mat[cols[None, :] < lens[:, None]]
    out = tokens.cpu().numpy().view(np.uint32), offsets.cpu().numpy().astype(np.uint64)
    del tokens, mat, lens, offsets, keep, alll, cdf, w, cols, g
    if dev.type == "cuda":
        torch.cuda.empty_cache()  # the scratch of 10^8+ keys is tens of GB; hand it back
    return out
