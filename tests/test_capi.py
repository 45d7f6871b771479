"""The C-ABI library loads and exports every entry point include/*.h declares
(no device calls: this runs without a GPU)."""
import ctypes
import glob
import os
import re

from helpers import REPO


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(REPO, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\*?\s*(ft_[A-Za-z0-9_]+)\s*\(", src, re.M):
            names.add(m.group(1))
    return names


def test_library_exports_declared_symbols(built):
    lib = ctypes.CDLL(os.path.join(REPO, "flash-trie_b200", "libftcore.so"))
    names = declared_symbols()
    assert len(names) >= 14
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing


def test_host_entry_points_without_gpu(built, tmp_path):
    lib = ctypes.CDLL(os.path.join(REPO, "flash-trie_b200", "libftcore.so"))
    lib.ft_last_error.restype = ctypes.c_char_p
    h = ctypes.c_void_p()
    assert lib.ft_trie_create(ctypes.byref(h)) == 0
    toks = (ctypes.c_uint32 * 5)(1, 2, 3, 1, 2)
    offs = (ctypes.c_uint64 * 3)(0, 3, 5)
    assert lib.ft_trie_build(h, toks, offs, ctypes.c_uint64(2)) == 0
    p = str(tmp_path / "t.bin").encode()
    assert lib.ft_trie_save(h, p) == 0
    assert lib.ft_trie_load(h, b"/nonexistent/trie.bin") == -9  # FT_ERR_IO
    assert b"IO_ERROR" in lib.ft_last_error()
    # A device lookup needs a GPU workspace: refused before any device call.
    lib.ft_lookup_batch_device.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p,
                                           ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p]
    assert lib.ft_lookup_batch_device(h, 1, None, None, 0, None, None) == -1  # FT_ERR_STATE
    assert b"init_tbs_gpu" in lib.ft_last_error()
    lib.ft_reverse_lookup_batch_device.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p,
                                                   ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p,
                                                   ctypes.c_void_p]
    assert lib.ft_reverse_lookup_batch_device(h, 1, None, 4, None, None, None) == -1  # FT_ERR_STATE
    lib.ft_trie_destroy(h)


class _Params(ctypes.Structure):
    _fields_ = [("token_logp_threshold", ctypes.c_float), ("reserved", ctypes.c_float),
                ("sent_logp_threshold", ctypes.c_double), ("length_norm", ctypes.c_double),
                ("early_exit", ctypes.c_int32), ("reserved2", ctypes.c_int32)]


_BATCH_PTRS = ("beams", "topk_id", "topk_logp", "out_count", "out_lpn", "out_len", "out_tok", "out_key")


class _Batch(ctypes.Structure):
    _fields_ = [("n", ctypes.c_uint32), ("num_outpos", ctypes.c_uint32), ("topk", ctypes.c_uint32),
                ("out_capacity", ctypes.c_uint32)] + [(f, ctypes.c_void_p) for f in _BATCH_PTRS]


def test_device_entry_points_refuse_null_pointers(built):
    """Both device entry points refuse a non-empty batch with a NULL required
    pointer before anything reaches the device (no GPU involved: the checks
    run on the host and return FT_ERR_NULL first)."""
    lib = ctypes.CDLL(os.path.join(REPO, "flash-trie_b200", "libftcore.so"))
    lib.ft_last_error.restype = ctypes.c_char_p
    h = ctypes.c_void_p()
    assert lib.ft_trie_create(ctypes.byref(h)) == 0
    toks = (ctypes.c_uint32 * 5)(1, 2, 3, 1, 2)
    offs = (ctypes.c_uint64 * 3)(0, 3, 5)
    assert lib.ft_trie_build(h, toks, offs, ctypes.c_uint64(2)) == 0
    prm = _Params(-10.0, 0.0, -40.0, 5.0, 0, 0)
    # Stand-in addresses: never dereferenced, since every call below is
    # refused on the host before any launch or copy.
    fake = {f: 0x1000 * (i + 1) for i, f in enumerate(_BATCH_PTRS)}
    required = [f for f in _BATCH_PTRS if f != "out_key"]
    for entry in ("ft_tbs_batch_device", "ft_tbs_batch_device_noalloc"):
        fn = getattr(lib, entry)
        for missing in required:
            ptrs = dict(fake, **{missing: None})
            b = _Batch(2, 3, 4, 8, *[ptrs[f] for f in _BATCH_PTRS])
            rc = fn(h, ctypes.byref(b), ctypes.byref(prm), None)
            assert rc == -2, (entry, missing, rc)  # FT_ERR_NULL
            assert missing.encode() in lib.ft_last_error(), (entry, missing)
        # An empty batch needs no pointers: nothing to check, nothing to do
        # (the allocating entry point still needs a workspace first).
        empty = _Batch(0, 3, 4, 8, *([None] * len(_BATCH_PTRS)))
        rc = fn(h, ctypes.byref(empty), ctypes.byref(prm), None)
        assert rc in (0, -1), (entry, rc)
    lib.ft_trie_destroy(h)


def test_device_api_rejects_host_tensors(built):
    """flashtrie_device validates its inputs before touching a device."""
    import pytest
    import torch
    import flashtrie
    import flashtrie_device as fd
    t = flashtrie.Trie()
    t.build(token_rows=[[1, 2], [1, 3]])
    beams = torch.ones((1, 2), dtype=torch.int32)
    ids = torch.zeros((1, 2, 4), dtype=torch.int32)
    lp = torch.zeros((1, 2, 4), dtype=torch.float32)
    with pytest.raises(TypeError):
        fd.bs_tbs_device(t, beams, ids, lp, -10.0, -40.0, 1.0, False)
    with pytest.raises(TypeError):
        fd.lookup(t, torch.zeros(3, dtype=torch.int32), torch.zeros(2, dtype=torch.int64))
    with pytest.raises(TypeError):
        fd.reverse_lookup(t, torch.zeros(3, dtype=torch.int32), 4)
