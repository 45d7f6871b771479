"""Benchmark of the B200 trie-constrained beam search (TBS) engine.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C]
                    [--batch B] [--beam B] [--keys N] [--keyset spec|ref-lengths]
                    [--impl b200|reference|reference-gpu]

Default workload: config 3 of the reference's metric (200M keys over a 2.2M
vocabulary, K=1000 proposals per position, L=20 positions, beam 1000,
batch 1 per GPU).  A step is one batch of requests searched against that
trie.

The trie file is cached in --trie-dir.  When it is absent, the reference
arm builds it with the reference's own builder (oracle/_ref/ref_build: the
unmodified marisa Keyset + Trie::build + save) and the b200 arm with the
engine's builder, whose files are byte-identical; the line names which one
wrote the file the run searched.  Keys come from the seeded generator in
workload.py (drawn with torch, sorted), requests likewise.

Arms:
  b200       value = q/s with inputs resident in HBM (device entry point
             ft_tbs_batch_device, CUDA events on the launching stream);
             e2e = q/s through the drop-in `flashtrie.bs_tbs_gpu` with numpy
             host buffers (H2D of the inputs, D2H of the results inside the
             timed region).  Extra fields: latency by beam (100/500/1000,
             batch 1), q/s at batch 8 (the reference's peak point) and at
             batches 296 and 1184 with the roofline fraction, the total batch
             of 64 split over the N ranks (strong scaling), the reference
             kernel (its sources compiled for sm_100a) on the same requests,
             the reference CPU `tbs` on one pinned core (cpu_baseline), and on
             one GPU the north star's point on config 4's 800M-key trie
             (north_star, a child process).
  reference  the reference's CPU `tbs(use_gpu=False)` (the unmodified
             reference built from its sources by oracle/ref.mk), one worker
             process per host core, each pinned to its core; a step is one
             request.  Rank 0 only.

Multi-GPU (torchrun): the trie is replicated on every rank and each rank
searches its own batch (weak scaling for `value`, no collective on the data
path); times are the max over ranks.
"""
import argparse
import ctypes
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "flash-trie_b200")
for _p in (REPO, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import workload as W  # noqa: E402
from flashtrie_shard import max_over_ranks  # noqa: E402

METRIC = ("trie-search q/s at batch 1 (latency mean/p99 ms at beam 100/500/1000 and peak q/s alongside); "
          "beam search over the synthetic trie of the named config")
UNIT = "requests/s"
STRONG_TOTAL_BATCH = 64  # north-star split: a total batch of 64 over 1/2/4/8 GPUs
SWEEP_BEAMS = (100, 500, 1000)
PEAK_BATCH = 8  # the reference's published peak q/s point (README.md:62-64)
BIG_BATCH = 296  # two requests per SM on the 148-SM B200: one per resident team
HUGE_BATCH = 1184  # eight per SM: each resident team takes four requests in turn


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=3)
    ap.add_argument("--keyset", default=None, choices=sorted(W.KEYSETS),
                    help="key-length distribution (default: the config's, see workload.KEYSETS)")
    ap.add_argument("--batch", type=int, default=0, help="requests per step per GPU (default: the config's)")
    ap.add_argument("--beam", type=int, default=0, help="override the config's beam width")
    ap.add_argument("--keys", type=int, default=0, help="override the config's key count")
    ap.add_argument("--requests", type=int, default=32, help="distinct requests of the headline loop")
    ap.add_argument("--impl", default="b200", choices=["b200", "reference", "reference-gpu"])
    ap.add_argument("--cpu-budget", type=float, default=25.0,
                    help="seconds of reference CPU work in cpu_baseline (at least one request runs; 0: skip)")
    ap.add_argument("--no-extras", action="store_true", help="headline and e2e only (quick runs)")
    ap.add_argument("--trie-dir", default="/tmp")
    ap.add_argument("--nonempty-only", action="store_true",
                    help="reference-gpu: search only requests the oracle gives at least one result")
    ap.add_argument("--with-ref-gpu", action="store_true",
                    help="add the reference kernel's line (reference_gpu) also with --no-extras")
    ap.add_argument("--no-north-star", action="store_true",
                    help="skip the north_star field (config 4, 800M keys, measured in a child process)")
    return ap.parse_args()


# ----------------------------------------------------------------- setup
def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def workload_cfg(args):
    cfg = W.resolve(args.config, args.keyset, batch=args.batch, beam=args.beam, keys=args.keys)
    if cfg["keyset"] != "spec" and (cfg["len_lo"], cfg["len_hi"]) != (W.CONFIGS[args.config]["len_lo"],
                                                                       W.CONFIGS[args.config]["len_hi"]):
        cfg["key_lengths"] = "%d-%d, weights %s (reference example generator)" % (
            cfg["len_lo"], cfg["len_hi"], ",".join(str(x) for x in cfg["len_weights"]))
    else:
        cfg["key_lengths"] = "uniform %d-%d" % (cfg["len_lo"], cfg["len_hi"])
    return cfg


def trie_base(args, cfg):
    return os.path.join(args.trie_dir, "ft_bench_c%d_%s_k%d" % (args.config, cfg["keyset"], cfg["keys"]))


def trie_path(args, cfg):
    return trie_base(args, cfg) + ".bin"


def trie_meta(args, cfg):
    """Sidecar of a finished trie file (written last): who built it, when."""
    try:
        with open(trie_base(args, cfg) + ".meta.json") as f:
            return json.load(f)
    except (OSError, ValueError):
        return None


def gen_keys(args, cfg, device):
    """The config's keys (torch, seeded by the config id, sorted), written as
    raw .u32 tokens and .u64 offsets beside the trie file."""
    t0 = time.time()
    tok, off = W.gen_keys_torch(cfg["keys"], cfg["vocab"], cfg["len_lo"], cfg["len_hi"], cfg["zipf"],
                                seed=args.config, device=device, len_weights=cfg["len_weights"], sort=True)
    base = trie_base(args, cfg)
    tok.tofile(base + ".u32.tmp")
    off.tofile(base + ".u64.tmp")
    os.replace(base + ".u32.tmp", base + ".u32")
    os.replace(base + ".u64.tmp", base + ".u64")
    return tok, off, time.time() - t0


def load_keys(args, cfg):
    """The keys, memory-mapped: requests touch only their target keys, and
    the ranks of one box share the page cache."""
    base = trie_base(args, cfg)
    return np.memmap(base + ".u32", np.uint32, mode="r"), np.memmap(base + ".u64", np.uint64, mode="r")


def finish_trie(args, cfg, built_by, gen_s, build_s):
    meta = {"built_by": built_by, "keys": cfg["keys"], "keyset": cfg["keyset"], "gen_keys_s": round(gen_s, 1),
            "build_s": round(build_s, 1), "file_bytes": os.path.getsize(trie_path(args, cfg))}
    base = trie_base(args, cfg)
    with open(base + ".meta.json.tmp", "w") as f:
        json.dump(meta, f)
    os.replace(base + ".meta.json.tmp", base + ".meta.json")
    return meta


def build_with_reference(args, cfg, device):
    """The reference's own builder (oracle/_ref/ref_build) writes the trie."""
    tok, off, gen_s = gen_keys(args, cfg, device)
    del tok, off
    base = trie_base(args, cfg)
    t0 = time.time()
    env = dict(os.environ, MARISA_MANAGED_ALLOC="0")
    subprocess.run([os.path.join(REPO, "oracle", "_ref", "ref_build"), base + ".u32", base + ".u64",
                    trie_path(args, cfg) + ".tmp"], check=True, env=env, stdout=subprocess.DEVNULL)
    os.replace(trie_path(args, cfg) + ".tmp", trie_path(args, cfg))
    return finish_trie(args, cfg, "reference builder (oracle/_ref/ref_build: marisa Keyset + Trie::build)",
                       gen_s, time.time() - t0)


def build_with_engine(args, cfg, device):
    import flashtrie
    tok, off, gen_s = gen_keys(args, cfg, device)
    t0 = time.time()
    t = flashtrie.Trie()
    t.build_flat(tok, off)
    del tok, off
    t.save(trie_path(args, cfg) + ".tmp")
    os.replace(trie_path(args, cfg) + ".tmp", trie_path(args, cfg))
    return finish_trie(args, cfg, "engine builder (flashtrie.Trie.build_flat; byte-identical to the reference's)",
                       gen_s, time.time() - t0)


def wait_for_trie(args, cfg, limit_s=5400):
    t_end = time.time() + limit_s
    while trie_meta(args, cfg) is None:
        if time.time() > t_end:
            raise RuntimeError("rank 0 did not finish the trie file within %d s" % limit_s)
        time.sleep(1.0)
    return trie_meta(args, cfg)


def root_children(tok, off):
    return set(np.unique(tok[off[:-1][np.diff(off) > 0].astype(np.int64)]).tolist())


def gen_requests(args, cfg, tok, off, n, start):
    rc = root_children(tok, off) if cfg.get("off_trie", 0.0) > 0 else None
    return W.gen_requests(args.config, tok, off, n, start=start, cfg=cfg, root_children=rc)


def config_dict(args, cfg, world, meta):
    """The config object both arms print."""
    return {"workload": "config%d" % args.config, "keys": cfg["keys"], "vocab": cfg["vocab"],
            "key_lengths": cfg["key_lengths"], "zipf": cfg["zipf"], "K": cfg["K"], "L": cfg["L"],
            "beam": cfg["beam"], "batch_per_gpu": cfg["batch"], "early_exit": cfg["early_exit"],
            "off_trie": cfg.get("off_trie", 0.0),
            "parallelism": "replicated trie, batch sharded over %d GPU(s)" % world,
            "l2": "not flushed; trie file %.2f GB > 126 MB L2" % (meta["file_bytes"] / 1e9 if meta else 0.0),
            "trie_built_by": meta["built_by"] if meta else None}


class Clocks:
    """Samples SM clocks and throttle reasons with nvidia-smi during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.FIELDS,
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.th = threading.Thread(target=self._read, daemon=True)
            self.th.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


# ------------------------------------------------------------- C ABI view
class Params(ctypes.Structure):
    _fields_ = [("token_logp_threshold", ctypes.c_float), ("reserved", ctypes.c_float),
                ("sent_logp_threshold", ctypes.c_double), ("length_norm", ctypes.c_double),
                ("early_exit", ctypes.c_int32), ("reserved2", ctypes.c_int32)]


class DeviceBatch(ctypes.Structure):
    _fields_ = [("n", ctypes.c_uint32), ("num_outpos", ctypes.c_uint32), ("topk", ctypes.c_uint32),
                ("out_capacity", ctypes.c_uint32)] + [(f, ctypes.c_void_p) for f in
                                                      ("beams", "topk_id", "topk_logp", "out_count", "out_lpn",
                                                       "out_len", "out_tok", "out_key")]


# ncu captures of the search kernel summarised under profiles/ (one launch
# each): (config, keyset, keys, batch, beam) -> summary file holding the
# measured dram__bytes_read.sum + dram__bytes_write.sum of that launch.
PROFILED = {
    (2, "spec", 10_000_000, 1, 100): "tbs_search_kernel_config2_batch1.md",
    (3, "spec", 200_000_000, 1, 1000): "tbs_search_kernel_config3_beam1000_batch1.md",
    (3, "spec", 50_000_000, 1, 1000): "tbs_search_kernel_config3_50m_beam1000_batch1.md",
    (3, "spec", 50_000_000, 296, 100): "tbs_search_kernel_config3_50m_beam100_batch296.md",
}


def measured_traffic(args, cfg):
    """DRAM bytes per launch from the profile summary of this workload, or
    (None, None) when it was not captured."""
    name = PROFILED.get((args.config, cfg["keyset"], cfg["keys"], cfg["batch"], cfg["beam"]))
    if not name:
        return None, None
    try:
        with open(os.path.join(REPO, "profiles", name)) as f:
            for line in f:
                if line.startswith("dram_bytes_per_launch:"):
                    return int(line.split(":")[1]), "profiles/" + name
    except OSError:
        pass
    return None, None


def oracle_pass(path, beams, ids, lp, cfg):
    """Per-request algorithmic bytes from the oracle's byte model and the
    oracle's results (test infrastructure, used as the counter and the
    checker only)."""
    from oracle.oracle import OracleTrie
    o = OracleTrie(path)
    out, results = [], []
    for i in range(len(beams)):
        sent, lpn, st = o.tbs(beams[i], ids[i], lp[i], W.TOKEN_LOGP_THRESHOLD, W.SENT_LOGP_THRESHOLD,
                              W.LENGTH_NORM, cfg["early_exit"], stats=True)
        out.append(st.bytes_alg)
        results.append(([list(x) for x in sent], list(lpn)))
    return np.array(out, dtype=np.float64), results


def _a16(x):
    return (x + 15) & ~15


def host_copy_bytes(nb, L, K, cap, tok_total):
    """Bytes the host path of bs_tbs_gpu moves for a batch of nb requests of
    one shape: one H2D copy of [meta | length-norm factors | beams | ids |
    logp | status words], then the result headers and tokens D2H (one copy
    when the token slots fit in kOneCopyTokenBytes, else headers plus only
    the tokens produced)."""
    h2d = _a16(24 * nb) + _a16(8 * (L + 1)) + _a16(4 * nb * L) + 2 * _a16(4 * nb * L * K) + 16
    q_tok = 16 + _a16(4 * nb) + _a16(40 * nb) + _a16(8 * nb * cap) + _a16(4 * nb * cap) + _a16(8 * nb)
    tok_bytes_max = 4 * nb * cap * L
    d2h = q_tok + (tok_bytes_max if tok_bytes_max <= 256 * 1024 else 4 * tok_total)
    return h2d, d2h


def reference_cpu_sample(path, beams, ids, lp, cfg, budget_s, procs=1, n_target=None):
    """Times the reference CPU tbs.  procs == 1: one worker pinned to core 0
    runs requests until budget_s is spent (at least one).  procs > 1: one
    worker per core, each pinned, sharing n_target requests round-robin.
    Returns (q/s, per-request ms list, requests, wall seconds)."""
    if procs <= 1:
        return _ref_worker((path, beams, ids, lp, cfg["early_exit"], budget_s, 0, 1, None))
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    with ctx.Pool(procs) as pool:
        parts = pool.map(_ref_worker, [(path, beams, ids, lp, cfg["early_exit"], budget_s, r, procs, n_target)
                                       for r in range(procs)])
    done = sum(p[2] for p in parts)
    wall = max(p[3] for p in parts)
    ms = [m for p in parts for m in p[1]]
    return done / wall if wall > 0 else 0.0, ms, done, wall


def _ref_worker(a):
    path, beams, ids, lp, ee, budget, rank, procs, n_target = a
    cores = sorted(os.sched_getaffinity(0))
    os.sched_setaffinity(0, {cores[rank % len(cores)]})
    os.environ["MARISA_MANAGED_ALLOC"] = "0"
    sys.path.insert(0, os.path.join(REPO, "oracle", "_ref"))
    import flashtrie_ref as ref
    t = ref.Trie()
    t.mmap(path)
    lists = {}
    ms = []
    start = time.perf_counter()
    i = rank
    while (n_target is None and (not ms or time.perf_counter() - start < budget)) or \
            (n_target is not None and i < n_target):
        j = i % len(beams)
        if j not in lists:
            lists[j] = (beams[j].tolist(), ids[j].tolist(), lp[j].tolist())
        a0 = time.perf_counter()
        ref.tbs(t, *lists[j], W.TOKEN_LOGP_THRESHOLD, W.SENT_LOGP_THRESHOLD, W.LENGTH_NORM, ee, False)
        ms.append((time.perf_counter() - a0) * 1e3)
        i += procs
    wall = time.perf_counter() - start
    return len(ms) / wall if wall > 0 else 0.0, ms, len(ms), wall


def ref_built():
    d = os.path.join(REPO, "oracle", "_ref")
    return os.path.isdir(d) and any(f.startswith("flashtrie_ref") for f in os.listdir(d)) and \
        os.path.exists(os.path.join(d, "ref_build"))


# --------------------------------------------------------------- arms
def run_reference(args, cfg):
    rank, world, local = dist_env()
    if rank != 0:
        return
    if not ref_built():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref was not built (reference sources absent)"}))
        return
    import torch
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    meta = trie_meta(args, cfg)
    if meta is None:
        meta = build_with_reference(args, cfg, dev)
        if dev == "cuda":
            torch.cuda.empty_cache()
    path = trie_path(args, cfg)
    tok, off = load_keys(args, cfg)
    n_req = max(args.requests, args.warmup + args.steps)
    beams, ids, lp = gen_requests(args, cfg, tok, off, n_req, start=0)
    del tok, off
    procs = max(1, len(os.sched_getaffinity(0)))
    # Warm-up steps (page cache, module load) untimed, then exactly K steps;
    # a step is one request of the workload.
    if args.warmup:
        reference_cpu_sample(path, beams[:args.warmup], ids[:args.warmup], lp[:args.warmup], cfg, 0.0,
                             min(procs, args.warmup), n_target=args.warmup)
    sl = slice(args.warmup, args.warmup + args.steps)
    qps, ms, done, wall = reference_cpu_sample(path, beams[sl], ids[sl], lp[sl], cfg, 0.0,
                                               min(procs, args.steps), n_target=args.steps)
    ms_arr = np.array(ms)
    cores_used = min(procs, args.steps)
    line = {
        "impl": "reference", "metric": METRIC, "value": qps, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * wall / max(done, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u32 ids / f64 scores",
        "data": "synthetic (seeded generator, workload.py)",
        "config": config_dict(args, cfg, world, meta),
        "latency_ms": {"mean": float(ms_arr.mean()) if len(ms) else None,
                       "p99": float(np.percentile(ms_arr, 99)) if len(ms) else None,
                       "per": "request, one pinned core per worker"},
        "cpu_baseline": {"value": qps, "unit": UNIT, "cores": cores_used, "kind": "reference",
                         "sample": "%d requests of config %d in %.1f s wall on %d worker processes, each pinned to "
                                   "its own core (reference tbs, use_gpu=False, trie mmap'd)"
                                   % (done, args.config, wall, cores_used)},
        "e2e": {"value": qps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "setup_s": {"trie": meta},
        # This arm runs the reference alone: the engine's modules stay unloaded.
        "engine_modules_loaded": sorted(m for m in ("flashtrie", "flashtrie_device") if m in sys.modules),
    }
    print(json.dumps(line))


def run_reference_gpu(args, cfg):
    """The reference's own GPU kernel (its sources compiled unmodified for
    sm_100a by oracle/ref.mk), one request per call (batch 1, one cooperative
    grid at a time), timed the way the reference reports it: the `ms` its
    `tbs` binding returns (tools/bindings.cpp:54-64).  Not a driver arm; the
    b200 arm runs it in a child process and reports it beside its own line.
    With --nonempty-only, requests whose oracle result is empty are skipped:
    the reference's output path reads out_sent_offset[num_beams - 1] with
    num_beams == 0 (tbs-kernels.cu:445, :815)."""
    rank, world, local = dist_env()
    if rank != 0:
        return
    # The reference kernel reads the trie through managed memory
    # (vector.h:222-235, 484-492); host-malloc'd arrays would be host pointers.
    os.environ["MARISA_MANAGED_ALLOC"] = "1"
    sys.path.insert(0, os.path.join(REPO, "oracle", "_ref"))
    import flashtrie_ref as ref
    import torch
    from oracle.oracle import OracleTrie
    meta = trie_meta(args, cfg)
    if meta is None:
        print(json.dumps({"impl": "reference-gpu", "unavailable": "no cached trie file"}))
        return
    path = trie_path(args, cfg)
    tok, off = load_keys(args, cfg)
    beams, ids, lp = gen_requests(args, cfg, tok, off, max(args.requests, args.steps), start=0)
    del tok, off
    B, L, K = cfg["beam"], cfg["L"], cfg["K"]
    o = OracleTrie(path)
    args_t = (W.TOKEN_LOGP_THRESHOLD, W.SENT_LOGP_THRESHOLD, W.LENGTH_NORM, cfg["early_exit"])
    expect, skipped = {}, 0
    for i in range(len(beams)):
        s_, l_ = o.tbs(beams[i], ids[i], lp[i], *args_t)
        if args.nonempty_only and not s_:
            skipped += 1
            continue
        expect[i] = (s_, l_)
    del o
    use = sorted(expect)
    if not use:
        print(json.dumps({"impl": "reference-gpu", "unavailable": "every request has an empty result"}))
        return
    t = ref.Trie()
    t.load(path)
    # Buffers sized well above one step's worst case (B*K candidates) and the
    # history (max_num_inter_beams) above 1 + L*B saved beams.
    t.init_tbs_gpu(1, max_num_topk=K, max_num_outpos=L, max_num_out_beams=4 * B,
                   max_num_out_tokens=4 * B * L, max_num_inter_beams=4 * B * L + 64)
    lists = {i: (beams[i].tolist(), ids[i].tolist(), lp[i].tolist()) for i in use}
    for s in range(args.warmup):
        ref.tbs(t, *lists[use[s % len(use)]], *args_t, True)
    torch.cuda.synchronize()
    ms, same_sets = [], 0
    for s in range(args.steps):
        i = use[s % len(use)]
        sent, lpn, m = ref.tbs(t, *lists[i], *args_t, True)
        ms.append(m)
        a = sorted(zip(map(tuple, sent), [round(x, 9) for x in lpn]))
        b = sorted(zip(map(tuple, expect[i][0]), [round(x, 9) for x in expect[i][1]]))
        same_sets += int(a == b)
    ms = np.array(ms)
    print(json.dumps({"impl": "reference-gpu", "metric": METRIC, "value": 1e3 / ms.mean(), "unit": UNIT,
                      "latency_ms": {"mean": float(ms.mean()), "p50": float(np.percentile(ms, 50)),
                                     "p99": float(np.percentile(ms, 99)),
                                     "per": "request, the reference binding's own ms (2-decimal truncation)"},
                      "steps": args.steps, "warmup": args.warmup,
                      "config": {"workload": "config%d" % args.config, "keys": cfg["keys"], "K": K, "L": L,
                                 "beam": B, "batch": 1},
                      "requests": len(use), "skipped_empty": skipped,
                      "result_sets_equal_to_oracle": "%d of %d" % (same_sets, args.steps)}))


class Device:
    """The engine's device entry point over resident inputs of one shape."""

    def __init__(self, lib, handle, dev, stream, beams, ids, lp, cap, L, K, prm):
        import torch
        self.lib, self.handle, self.stream, self.prm = lib, handle, stream, prm
        self.R = len(beams)
        self.L, self.K, self.cap = L, K, cap
        self.out_cap = cap  # the output capacity a call declares: its beam width
        self.d_beams = torch.from_numpy(np.ascontiguousarray(beams).astype(np.int32)).to(dev)
        self.d_ids = torch.from_numpy(np.ascontiguousarray(ids).view(np.int32)).to(dev)
        self.d_lp = torch.from_numpy(np.ascontiguousarray(lp)).to(dev)
        self.dev = dev
        self.outs = {}

    def set_beam(self, beam):
        self.d_beams.fill_(int(beam))
        self.out_cap = min(int(beam), self.cap)

    def _outs(self, nb):
        import torch
        if nb not in self.outs:
            dev, cap, L = self.dev, self.cap, self.L
            self.outs[nb] = (torch.zeros(nb, dtype=torch.int32, device=dev),
                             torch.zeros(nb * cap, dtype=torch.float64, device=dev),
                             torch.zeros(nb * cap, dtype=torch.int32, device=dev),
                             torch.zeros(nb * cap * L, dtype=torch.int32, device=dev))
        return self.outs[nb]

    def launch(self, step, nb):
        """Batch of nb requests starting at a rotating offset into the
        resident requests (consecutive batches use different requests)."""
        s = (step * nb) % max(1, self.R - nb + 1) if self.R > nb else 0
        oc, ol, on, ot = self._outs(nb)
        b = DeviceBatch(nb, self.L, self.K, self.out_cap, self.d_beams[s].data_ptr(), self.d_ids[s].data_ptr(),
                        self.d_lp[s].data_ptr(), oc.data_ptr(), ol.data_ptr(), on.data_ptr(), ot.data_ptr())
        rc = self.lib.ft_tbs_batch_device(self.handle, ctypes.byref(b), ctypes.byref(self.prm),
                                          ctypes.c_void_p(self.stream.cuda_stream))
        if rc != 0:
            raise RuntimeError(self.lib.ft_last_error().decode())
        return s

    def timed(self, nb, steps, warmup, barrier=None):
        """warmup untimed launches, then `steps` launches, each bracketed by
        CUDA events on the launching stream.  Returns (total ms, per-step ms
        array, first requests used)."""
        import torch
        for s in range(warmup):
            self.launch(s, nb)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if barrier:
            barrier()
        torch.cuda.synchronize()
        used = []
        t0.record(self.stream)
        for s in range(steps):
            ev[s][0].record(self.stream)
            used.append(self.launch(warmup + s, nb))
            ev[s][1].record(self.stream)
        t1.record(self.stream)
        torch.cuda.synchronize()
        if barrier:
            barrier()
        return t0.elapsed_time(t1), np.array([a.elapsed_time(b) for a, b in ev]), used

    def check_status(self):
        st = ctypes.c_uint32()
        assert self.lib.ft_trie_device_status(self.handle, ctypes.byref(st)) == 0 and st.value == 0, \
            "device status %d" % st.value


def run_b200(args, cfg):
    import torch
    import flashtrie

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        barrier = lambda: dist.barrier()  # noqa: E731
    else:
        barrier = lambda: None  # noqa: E731

    # The north star's point runs first, in a child process, while this
    # process holds no device memory (its key generation and device image
    # need most of the GPU).
    north_star = None
    if world == 1 and args.config == 3 and not (args.no_extras or args.no_north_star):
        north_star = north_star_subprocess(args)

    t_setup = time.time()
    meta = trie_meta(args, cfg)
    if meta is None:
        if rank == 0:
            meta = build_with_engine(args, cfg, str(dev))
            torch.cuda.empty_cache()
        else:
            meta = wait_for_trie(args, cfg)
    barrier()
    path = trie_path(args, cfg)
    B, L, K, nb = cfg["beam"], cfg["L"], cfg["K"], cfg["batch"]
    tok, off = load_keys(args, cfg)
    # Each rank its own seeded requests (weak scaling): enough distinct ones
    # for the largest batch of the extras.
    big = 0 if args.no_extras else HUGE_BATCH
    n_req = max(args.requests, nb) if args.no_extras else max(args.requests, nb, big, STRONG_TOTAL_BATCH)
    beams, ids, lp = gen_requests(args, cfg, tok, off, n_req, start=rank * n_req)
    del tok, off
    trie = flashtrie.Trie()
    trie.mmap(path)  # parsed from the page cache the ranks share; no private copy of the file
    free0 = torch.cuda.mem_get_info(dev)[0]
    t_init = time.time()
    max_batch = nb if args.no_extras else max(nb, big, PEAK_BATCH, -(-STRONG_TOTAL_BATCH // world))
    cap = max([B] + ([] if args.no_extras else list(SWEEP_BEAMS)))
    trie.init_tbs_gpu(max_batch, max_num_topk=K, max_num_outpos=L, max_num_out_beams=cap,
                      max_num_out_tokens=cap * L, max_num_inter_beams=cap * L)
    init_s = time.time() - t_init
    device_gb = (free0 - torch.cuda.mem_get_info(dev)[0]) / 1e9  # device image + search workspace
    lib = ctypes.CDLL(os.path.join(PKG, "libftcore.so"))
    lib.ft_last_error.restype = ctypes.c_char_p
    handle = ctypes.c_void_p(trie.ft_handle())
    prm = Params(W.TOKEN_LOGP_THRESHOLD, 0.0, W.SENT_LOGP_THRESHOLD, W.LENGTH_NORM, int(cfg["early_exit"]), 0)
    stream = torch.cuda.Stream(dev)
    head_R = min(args.requests, n_req)
    head = Device(lib, handle, dev, stream, beams[:head_R], ids[:head_R], lp[:head_R], cap, L, K, prm)
    head.set_beam(B)
    setup_s = time.time() - t_setup

    with torch.cuda.stream(stream):
        for s in range(args.warmup):
            head.launch(s, nb)
    torch.cuda.synchronize()
    head.check_status()

    # Clocks are sampled by nvidia-smi (100 ms period) from before until after
    # the timed region; a short sustained loop of the same step on each side
    # keeps the GPU under load for the sampler when the timed region itself
    # is shorter than a sampling period.
    clocks = Clocks(local)
    clocks.start()

    def sustained(seconds):
        t_end = time.time() + seconds
        k = 0
        while time.time() < t_end:
            for _ in range(16):
                head.launch(k, nb)
                k += 1
            stream.synchronize()

    sustained(0.6)
    elapsed_ms, step_ms, used = head.timed(nb, args.steps, 0, barrier)
    sustained(0.4)
    clk = clocks.stop()
    head.check_status()

    extras = {}
    if not args.no_extras:
        # Latency by beam at batch 1 (the metric's beam 100/500/1000 points).
        by_beam = {}
        for bw in SWEEP_BEAMS:
            head.set_beam(bw)
            _, ms_b, _ = head.timed(1, max(args.steps, 20), 3)
            by_beam[str(bw)] = {"mean": float(ms_b.mean()), "p50": float(np.percentile(ms_b, 50)),
                                "p99": float(np.percentile(ms_b, 99))}
        extras["latency_ms_by_beam"] = dict(by_beam, per="device time of one request (batch 1), CUDA events, "
                                                          "%d steps each" % max(args.steps, 20))
        # Peak q/s: batch 8 (the reference's published peak point) and a large
        # batch, every beam; whole box = all ranks' requests over the slowest.
        big_dev = Device(lib, handle, dev, stream, beams, ids, lp, cap, L, K, prm)
        peak = {}
        for bw in SWEEP_BEAMS:
            big_dev.set_beam(bw)
            for bb in (PEAK_BATCH, BIG_BATCH, HUGE_BATCH):
                steps_b = 10 if bb >= BIG_BATCH else max(args.steps, 20)
                tot, _, _ = big_dev.timed(bb, steps_b, 3, barrier)
                tot = max_over_ranks([tot], device=dev)[0] if world > 1 else tot
                peak["beam%d_batch%d" % (bw, bb)] = world * bb * steps_b / (tot / 1e3)
        extras["peak_qps"] = dict(peak, per="whole box (%d GPU(s)), device-resident inputs, batch per GPU" % world)
        # Strong scaling: the north star's total batch of 64 split over the
        # ranks, at the headline beam.
        big_dev.set_beam(B)
        per_rank = -(-STRONG_TOTAL_BATCH // world)
        tot, ms_s, _ = big_dev.timed(per_rank, max(args.steps, 20), 3, barrier)
        tot = max_over_ranks([tot], device=dev)[0] if world > 1 else tot
        extras["strong_scaling"] = {"total_batch": per_rank * world, "batch_per_gpu": per_rank, "beam": B,
                                    "qps": per_rank * world * max(args.steps, 20) / (tot / 1e3),
                                    "ms_per_step": tot / max(args.steps, 20),
                                    "scaling": "strong (fixed total batch of %d)" % STRONG_TOTAL_BATCH}
        big_dev.check_status()
        del big_dev
    head.set_beam(B)

    # e2e through the drop-in module with host buffers, on the batches the
    # headline loop searched.
    e2e_steps = args.steps
    for s in range(min(args.warmup, 3)):
        i = used[s % len(used)]
        flashtrie.bs_tbs_gpu(trie, nb, beams[i:i + nb], ids[i:i + nb], lp[i:i + nb], W.TOKEN_LOGP_THRESHOLD,
                             W.SENT_LOGP_THRESHOLD, W.LENGTH_NORM, cfg["early_exit"])
    # Per-call results are kept as returned and examined after the timed
    # loop, so the loop holds the API call and nothing else.
    outs = []
    barrier()
    t0 = time.perf_counter()
    for s in range(e2e_steps):
        i = used[s % len(used)]
        outs.append((i, flashtrie.bs_tbs_gpu(trie, nb, beams[i:i + nb], ids[i:i + nb], lp[i:i + nb],
                                             W.TOKEN_LOGP_THRESHOLD, W.SENT_LOGP_THRESHOLD, W.LENGTH_NORM,
                                             cfg["early_exit"])))
    e2e_s = time.perf_counter() - t0
    phase_sum = np.zeros(5)
    binding_ms, h2d_total, d2h_total, e2e_res = [], 0, 0, {}
    for i, (sents, lpns, bms, phases) in outs:
        binding_ms.append(bms)
        phase_sum += np.asarray(phases, dtype=np.float64).sum(axis=0)
        h2d, d2h = host_copy_bytes(nb, L, K, cap, sum(len(x) for ss in sents for x in ss))
        h2d_total += h2d
        d2h_total += d2h
        for k in range(nb):
            e2e_res[i + k] = ([list(x) for x in sents[k]], list(lpns[k]))

    elapsed_ms, e2e_s = max_over_ranks([elapsed_ms, e2e_s], device=dev) if world > 1 else (elapsed_ms, e2e_s)

    if rank == 0:
        total_req = args.steps * nb * world
        value = total_req / (elapsed_ms / 1e3)
        e2e_value = e2e_steps * nb * world / e2e_s
        # Roofline of the search kernel: algorithmic bytes per launch over the
        # mean launch time (CUDA events on the launching stream).
        first = sorted(set(used))
        idx = sorted({i + k for i in first for k in range(nb)})
        per_req_bytes, o_res = oracle_pass(path, beams[idx], ids[idx], lp[idx], cfg)
        by_req = dict(zip(idx, per_req_bytes))
        counts = [len(r[0]) for r in o_res]
        same = sum(int(e2e_res.get(i) == r) for i, r in zip(idx, o_res))
        bytes_per_launch = float(np.mean([sum(by_req[i + k] for k in range(nb)) for i in used]))
        peak_bw, peak_kind = measured_peaks()
        achieved = bytes_per_launch / (float(step_ms.mean()) / 1e3) / 1e9
        traffic, traffic_src = measured_traffic(args, cfg)
        if "peak_qps" in extras:
            # Large-batch roofline: the headline requests' mean bytes per
            # request (same distribution) times the batch's q/s.
            fr = {bb: extras["peak_qps"]["beam%d_batch%d" % (B, bb)] / world * float(per_req_bytes.mean()) / 1e9
                  for bb in (BIG_BATCH, HUGE_BATCH)}
            best = max(fr, key=fr.get)
            a_big = fr[best]
            extras["peak_roofline"] = {"batch": best, "beam": B, "achieved": a_big, "peak": peak_bw,
                                       "unit": "GB/s", "frac": a_big / peak_bw,
                                       "frac_by_batch": {str(bb): v / peak_bw for bb, v in fr.items()},
                                       "bytes_per_request": float(per_req_bytes.mean()),
                                       "per": "one GPU; bytes per request from the oracle's byte model over the "
                                              "headline requests"}
        cpu = None
        if world == 1 and ref_built() and args.cpu_budget > 0:
            cpu_qps, cpu_ms, cpu_n, cpu_wall = reference_cpu_sample(path, beams[idx], ids[idx], lp[idx], cfg,
                                                                    args.cpu_budget, 1)
            cpu = {"value": cpu_qps, "unit": UNIT, "cores": 1, "kind": "reference",
                   "sample": "%d request(s) of config %d, %.1f s, reference tbs(use_gpu=False), one process "
                             "pinned to one core" % (cpu_n, args.config, cpu_wall),
                   "ms_per_request": float(np.mean(cpu_ms))}
        if world == 1 and ref_built() and (args.with_ref_gpu or not args.no_extras):
            extras["reference_gpu"] = reference_gpu_subprocess(args, cfg)
        if north_star is not None:
            extras["north_star"] = north_star
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u32 ids / f64 scores",
            "data": "synthetic (seeded generator, workload.py)",
            "config": config_dict(args, cfg, world, meta),
            "latency_ms": {"mean": float(step_ms.mean()), "p50": float(np.percentile(step_ms, 50)),
                           "p99": float(np.percentile(step_ms, 99)), "per": "step (batch of %d)" % nb},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": int(h2d_total / max(e2e_steps, 1)),
                    "d2h_bytes_per_step": int(d2h_total / max(e2e_steps, 1)),
                    "path": "flashtrie.bs_tbs_gpu (numpy host buffers)",
                    "binding_ms": {"mean": float(np.mean(binding_ms)), "p99": float(np.percentile(binding_ms, 99))}},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak_bw, "unit": "GB/s",
                         "frac": achieved / peak_bw, "traffic": traffic, "traffic_source": traffic_src,
                         "peak_source": peak_kind, "bytes_alg_per_launch": bytes_per_launch},
            "cpu_baseline": cpu,
            "phase_ms_per_request": dict(zip(["expansion", "validation(fused)", "selection", "overhead", "kernel"],
                                              (phase_sum / max(e2e_steps * nb, 1)).round(5).tolist())),
            "clocks": clk,
            "gpu_launches": args.steps,
            "results_per_request": float(np.mean(counts)),
            "parity_vs_oracle": {"requests": len(idx), "identical": same,
                                 "what": "rank 0's e2e results (sequences, order, f64 scores) against the C oracle "
                                         "(oracle/tbs_oracle.c) on the same requests, bit for bit"},
            "setup_s": {"trie": meta, "load_and_requests": round(setup_s - init_s, 1), "init_tbs_gpu": init_s,
                        "device_gb_image_and_workspace": round(device_gb, 2), "max_batch": max_batch,
                        "num_nodes": trie.num_nodes(), "num_keys": trie.num_keys()},
        }
        line.update(extras)
        print(json.dumps(line))
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def reference_gpu_subprocess(args, cfg):
    """The reference kernel on the same trie and requests, in a child process
    (the reference module keeps its own CUDA state); its JSON or a reason."""
    cmd = [sys.executable, os.path.abspath(__file__), "--impl", "reference-gpu", "--config", str(args.config),
           "--steps", "20", "--warmup", "3", "--requests", str(min(args.requests, 20)), "--trie-dir", args.trie_dir,
           "--nonempty-only"]
    for k in ("keyset", "beam", "keys", "batch"):
        v = getattr(args, k)
        if v:
            cmd += ["--" + k, str(v)]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
        for ln in r.stdout.splitlines()[::-1]:
            if ln.startswith("{"):
                return json.loads(ln)
        return {"unavailable": "reference-gpu exited %d: %s" % (r.returncode, r.stderr[-300:])}
    except subprocess.TimeoutExpired:
        return {"unavailable": "reference-gpu took more than 900 s"}


def north_star_subprocess(args):
    """The north star's own point, beam 1000 at batch 1 on config 4's trie
    (800M keys), in a child process: its latency, oracle parity and the
    reference kernel on the same requests.  The child builds (or reuses) the
    trie file in the same directory."""
    cmd = [sys.executable, os.path.abspath(__file__), "--config", "4", "--batch", "1", "--steps", "20", "--warmup",
           "5", "--no-extras", "--cpu-budget", "0", "--trie-dir", args.trie_dir]
    if ref_built():
        cmd.append("--with-ref-gpu")
    t0 = time.time()
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=1200)
    except subprocess.TimeoutExpired:
        return {"unavailable": "config 4 took more than 1200 s"}
    child = None
    for ln in r.stdout.splitlines()[::-1]:
        if ln.startswith("{"):
            child = json.loads(ln)
            break
    if child is None:
        return {"unavailable": "config 4 exited %d: %s" % (r.returncode, r.stderr[-300:])}
    keep = ("value", "unit", "ms_per_step", "config", "latency_ms", "e2e", "roofline", "clocks", "gpu_launches",
            "results_per_request", "parity_vs_oracle", "reference_gpu")
    out = {k: child[k] for k in keep if k in child}
    out["setup_s"] = {k: child["setup_s"].get(k) for k in ("trie", "device_gb_image_and_workspace", "num_nodes",
                                                         "num_keys")}
    out["wall_s"] = round(time.time() - t0, 1)
    out["what"] = ("north star: 800M-key, V=2.2M trie (config 4, the reference generator's key lengths), beam "
                   "1000, batch 1, target p99 <= 1.5 ms; `python bench.py --config 4 --batch 1 --no-extras "
                   "--cpu-budget 0 --with-ref-gpu` in a child process")
    return out


def main():
    args = parse()
    cfg = workload_cfg(args)
    if args.impl == "reference":
        run_reference(args, cfg)
    elif args.impl == "reference-gpu":
        run_reference_gpu(args, cfg)
    else:
        run_b200(args, cfg)


if __name__ == "__main__":
    main()
