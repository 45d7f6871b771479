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


def test_no_alloc_entry_point_matches_allocating_one(built, tmp_path):
    import torch
    lib = ctypes.CDLL(os.path.join(REPO, "flash-trie_b200", "libftcore.so"))
    lib.ft_last_error.restype = ctypes.c_char_p
    cfg = W.CONFIGS[1]
    tok, off = W.gen_keys(cfg["keys"], cfg["vocab"], cfg["len_lo"], cfg["len_hi"], cfg["zipf"], seed=1)
    n = 6
    beams, ids, lp = W.gen_requests(1, tok, off, n, start=500)
    L, K, cap = beams.shape[1], ids.shape[2], int(beams[0, -1])

    h = ctypes.c_void_p()
    assert lib.ft_trie_create(ctypes.byref(h)) == 0
    assert lib.ft_trie_build(h, tok.ctypes.data_as(ctypes.c_void_p), off.ctypes.data_as(ctypes.c_void_p),
                             ctypes.c_uint64(len(off) - 1)) == 0
    assert lib.ft_trie_init_tbs_gpu(h, *map(ctypes.c_uint64, (n, K, L, cap, cap * L, cap * L, 1024))) == 0, \
        lib.ft_last_error()

    dev = torch.device("cuda:0")
    d_beams = torch.from_numpy(beams.astype(np.int32)).to(dev)
    d_ids = torch.from_numpy(ids.view(np.int32)).to(dev)
    d_lp = torch.from_numpy(lp).to(dev)
    prm = Params(W.TOKEN_LOGP_THRESHOLD, 0.0, W.SENT_LOGP_THRESHOLD, W.LENGTH_NORM, 0, 0)
    stream = torch.cuda.current_stream(dev)

    def run(fn):
        outs = (torch.zeros(n, dtype=torch.int32, device=dev), torch.zeros(n * cap, dtype=torch.float64, device=dev),
                torch.zeros(n * cap, dtype=torch.int32, device=dev),
                torch.zeros(n * cap * L, dtype=torch.int32, device=dev))
        b = Batch(n, L, K, cap, d_beams.data_ptr(), d_ids.data_ptr(), d_lp.data_ptr(),
                  *[o.data_ptr() for o in outs])
        rc = fn(h, ctypes.byref(b), ctypes.byref(prm), ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0, lib.ft_last_error()
        torch.cuda.synchronize()
        cnt, lpn, ln, tk = (o.cpu().numpy() for o in outs)
        res = []
        for i in range(n):
            c = int(cnt[i])
            sents = [tk.view(np.uint32).reshape(n, cap, L)[i, j, :ln.reshape(n, cap)[i, j]].tolist()
                     for j in range(c)]
            res.append((sents, lpn.reshape(n, cap)[i, :c].tolist()))
        return res

    expected = run(lib.ft_tbs_batch_device)
    assert any(r[0] for r in expected)
    first = run(lib.ft_tbs_batch_device_noalloc)
    second = run(lib.ft_tbs_batch_device_noalloc)
    for i in range(n):
        assert first[i][0] == expected[i][0] and second[i][0] == expected[i][0], i
        np.testing.assert_allclose(first[i][1], expected[i][1], rtol=1e-5, atol=0)
        np.testing.assert_allclose(second[i][1], expected[i][1], rtol=1e-5, atol=0)
        assert first[i][1] == expected[i][1] == second[i][1]

    # Batches beyond the fixed scratch are refused with a clear error.
    big = Batch(4096, L, 8192, 8192, d_beams.data_ptr(), d_ids.data_ptr(), d_lp.data_ptr(), 0, 0, 0, 0)
    rc = lib.ft_tbs_batch_device_noalloc(h, ctypes.byref(big), ctypes.byref(prm), ctypes.c_void_p(stream.cuda_stream))
    assert rc == -20 and b"scratch" in lib.ft_last_error()
    lib.ft_trie_destroy(h)
