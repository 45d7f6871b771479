"""The no-allocation entry point, ft_tbs_batch_device_noalloc.

Some callers cannot allocate device memory while they search (their host
framework owns every device allocation, or their request threads must not
stall on cudaMalloc/cudaFree).  This entry point runs the same search as
ft_tbs_batch_device with its scratch in a fixed array inside the library.
The test calls it through the C ABI twice in a row and checks both results
against the allocating entry point's (exact equality: the search is
deterministic and bit-exact).  It lives in its own file so that pytest
collects it last.
"""
import ctypes
import os

import numpy as np
import pytest

import workload as W
from helpers import REPO

pytestmark = pytest.mark.gpu


class Params(ctypes.Structure):
    _fields_ = [("token_logp_threshold", ctypes.c_float), ("reserved", ctypes.c_float),
                ("sent_logp_threshold", ctypes.c_double), ("length_norm", ctypes.c_double),
                ("early_exit", ctypes.c_int32), ("reserved2", ctypes.c_int32)]


class Batch(ctypes.Structure):
    _fields_ = [("n", ctypes.c_uint32), ("num_outpos", ctypes.c_uint32), ("topk", ctypes.c_uint32),
                ("out_capacity", ctypes.c_uint32)] + [(f, ctypes.c_void_p) for f in
                                                      ("beams", "topk_id", "topk_logp", "out_count", "out_lpn",
                                                       "out_len", "out_tok", "out_key")]


def _setup(lib, n, L, K, cap, beams_cap=None):
    cfg = W.CONFIGS[1]
    tok, off = W.gen_keys(cfg["keys"], cfg["vocab"], cfg["len_lo"], cfg["len_hi"], cfg["zipf"], seed=1)
    h = ctypes.c_void_p()
    assert lib.ft_trie_create(ctypes.byref(h)) == 0
    assert lib.ft_trie_build(h, tok.ctypes.data_as(ctypes.c_void_p), off.ctypes.data_as(ctypes.c_void_p),
                             ctypes.c_uint64(len(off) - 1)) == 0
    assert lib.ft_trie_init_tbs_gpu(h, *map(ctypes.c_uint64, (n, K, L, cap, cap * L, cap * L, 1024))) == 0, \
        lib.ft_last_error()
    return h, tok, off


def _runner(lib, h, n, L, K, cap, d_beams, d_ids, d_lp, prm):
    import torch
    dev = d_beams.device
    stream = torch.cuda.current_stream(dev)

    def run(fn, expect_rc=0):
        outs = (torch.zeros(n, dtype=torch.int32, device=dev), torch.zeros(n * cap, dtype=torch.float64, device=dev),
                torch.zeros(n * cap, dtype=torch.int32, device=dev),
                torch.zeros(n * cap * L, dtype=torch.int32, device=dev))
        b = Batch(n, L, K, cap, d_beams.data_ptr(), d_ids.data_ptr(), d_lp.data_ptr(),
                  *[o.data_ptr() for o in outs])
        rc = fn(h, ctypes.byref(b), ctypes.byref(prm), ctypes.c_void_p(stream.cuda_stream))
        assert rc == expect_rc, (rc, lib.ft_last_error())
        torch.cuda.synchronize()
        cnt, lpn, ln, tk = (o.cpu().numpy() for o in outs)
        res = []
        for i in range(n):
            c = int(cnt[i])
            sents = [tk.view(np.uint32).reshape(n, cap, L)[i, j, :ln.reshape(n, cap)[i, j]].tolist()
                     for j in range(c)]
            res.append((sents, lpn.reshape(n, cap)[i, :c].tolist()))
        return res

    return run


def _check_same(n, got, expected):
    for i in range(n):
        assert got[i][0] == expected[i][0], i
        np.testing.assert_allclose(got[i][1], expected[i][1], rtol=1e-5, atol=0)
        assert got[i][1] == expected[i][1], i


def _lib():
    lib = ctypes.CDLL(os.path.join(REPO, "flash-trie_b200", "libftcore.so"))
    lib.ft_last_error.restype = ctypes.c_char_p
    return lib


def test_no_alloc_entry_point_matches_allocating_one(built, tmp_path):
    import torch
    lib = _lib()
    n = 6
    cfg = W.CONFIGS[1]
    L, K, cap = cfg["L"], cfg["K"], cfg["beam"]
    h, tok, off = _setup(lib, n, L, K, cap)
    beams, ids, lp = W.gen_requests(1, tok, off, n, start=500)
    assert beams.shape[1] == L and ids.shape[2] == K and int(beams[0, -1]) == cap

    dev = torch.device("cuda:0")
    d_beams = torch.from_numpy(beams.astype(np.int32)).to(dev)
    d_ids = torch.from_numpy(ids.view(np.int32)).to(dev)
    d_lp = torch.from_numpy(lp).to(dev)
    prm = Params(W.TOKEN_LOGP_THRESHOLD, 0.0, W.SENT_LOGP_THRESHOLD, W.LENGTH_NORM, 0, 0)
    run = _runner(lib, h, n, L, K, cap, d_beams, d_ids, d_lp, prm)

    expected = run(lib.ft_tbs_batch_device)
    assert any(r[0] for r in expected)
    first = run(lib.ft_tbs_batch_device_noalloc)
    second = run(lib.ft_tbs_batch_device_noalloc)
    _check_same(n, first, expected)
    _check_same(n, second, expected)

    # Batches beyond the fixed scratch are refused with a clear error, on the
    # host, before anything is launched.
    stream = torch.cuda.current_stream(dev)
    out = torch.zeros(16, dtype=torch.int32, device=dev)
    p_out = out.data_ptr()
    big = Batch(4096, L, 8192, 8192, d_beams.data_ptr(), d_ids.data_ptr(), d_lp.data_ptr(),
                p_out, p_out, p_out, p_out, 0)
    rc = lib.ft_tbs_batch_device_noalloc(h, ctypes.byref(big), ctypes.byref(prm), ctypes.c_void_p(stream.cuda_stream))
    assert rc == -20 and b"scratch" in lib.ft_last_error()
    lib.ft_trie_destroy(h)


def test_no_alloc_more_requests_than_scratch_slots(built):
    """Wide beams make one request's scratch ~2.4 MiB, so the 8 MiB array holds
    three slots and six requests take turns in them; results still equal the
    allocating entry point's."""
    import torch
    lib = _lib()
    n, cap = 6, 400
    cfg = W.CONFIGS[1]
    L, K = cfg["L"], cfg["K"]
    h, tok, off = _setup(lib, n, L, K, cap)
    beams, ids, lp = W.gen_requests(1, tok, off, n, start=700)
    beams[:] = cap
    dev = torch.device("cuda:0")
    d_beams = torch.from_numpy(beams.astype(np.int32)).to(dev)
    d_ids = torch.from_numpy(ids.view(np.int32)).to(dev)
    d_lp = torch.from_numpy(lp).to(dev)
    prm = Params(W.TOKEN_LOGP_THRESHOLD, 0.0, W.SENT_LOGP_THRESHOLD, W.LENGTH_NORM, 0, 0)
    run = _runner(lib, h, n, L, K, cap, d_beams, d_ids, d_lp, prm)
    expected = run(lib.ft_tbs_batch_device)
    assert sum(len(r[0]) for r in expected) > n
    _check_same(n, run(lib.ft_tbs_batch_device_noalloc), expected)
    _check_same(n, run(lib.ft_tbs_batch_device_noalloc), expected)
    lib.ft_trie_destroy(h)


def test_no_alloc_shape_and_length_norm_change_between_calls(built):
    """A call with another L, K and length norm after a first call: the
    per-call metadata and length-norm factors in the shared array are
    rewritten, and both calls match the allocating entry point."""
    import torch
    lib = _lib()
    n = 5
    cfg = W.CONFIGS[1]
    L, K, cap = cfg["L"], cfg["K"], cfg["beam"]
    h, tok, off = _setup(lib, n, L, K, cap)
    beams, ids, lp = W.gen_requests(1, tok, off, n, start=900)
    dev = torch.device("cuda:0")
    for (L2, K2, ln) in ((L, K, W.LENGTH_NORM), (L - 3, K // 2, 1.0), (L, K, W.LENGTH_NORM)):
        # Rows stay sorted by id when truncated to their first K2 columns.
        b2 = np.ascontiguousarray(beams[:, :L2])
        i2 = np.ascontiguousarray(ids[:, :L2, :K2])
        l2 = np.ascontiguousarray(lp[:, :L2, :K2])
        d_beams = torch.from_numpy(b2.astype(np.int32)).to(dev)
        d_ids = torch.from_numpy(i2.view(np.int32)).to(dev)
        d_lp = torch.from_numpy(l2).to(dev)
        prm = Params(W.TOKEN_LOGP_THRESHOLD, 0.0, W.SENT_LOGP_THRESHOLD, ln, 0, 0)
        run = _runner(lib, h, n, L2, K2, cap, d_beams, d_ids, d_lp, prm)
        expected = run(lib.ft_tbs_batch_device)
        assert any(r[0] for r in expected)
        _check_same(n, run(lib.ft_tbs_batch_device_noalloc), expected)
    lib.ft_trie_destroy(h)


def test_no_alloc_width_above_capacity_is_refused_by_the_kernel(built):
    """A beam width above out_capacity is not checked on the host (the widths
    live in device memory); the kernel checks every width before it writes
    anything but the request's zero count, and the call reports FT_ERR_DEVICE."""
    import torch
    lib = _lib()
    n = 3
    cfg = W.CONFIGS[1]
    L, K, cap = cfg["L"], cfg["K"], cfg["beam"]
    h, tok, off = _setup(lib, n, L, K, cap)
    beams, ids, lp = W.gen_requests(1, tok, off, n, start=950)
    beams[1, 2] = cap + 1
    dev = torch.device("cuda:0")
    d_beams = torch.from_numpy(beams.astype(np.int32)).to(dev)
    d_ids = torch.from_numpy(ids.view(np.int32)).to(dev)
    d_lp = torch.from_numpy(lp).to(dev)
    prm = Params(W.TOKEN_LOGP_THRESHOLD, 0.0, W.SENT_LOGP_THRESHOLD, W.LENGTH_NORM, 0, 0)
    run = _runner(lib, h, n, L, K, cap, d_beams, d_ids, d_lp, prm)
    got = run(lib.ft_tbs_batch_device_noalloc, expect_rc=-22)  # FT_ERR_DEVICE
    assert b"status 0x" in lib.ft_last_error()
    assert got[1] == ([], [])
    # The next good call starts from a clean status word.
    beams[1, 2] = cap
    d_beams.copy_(torch.from_numpy(beams.astype(np.int32)))
    expected = run(lib.ft_tbs_batch_device)
    _check_same(n, run(lib.ft_tbs_batch_device_noalloc), expected)
    lib.ft_trie_destroy(h)
