"""TEST INFRASTRUCTURE ONLY - ctypes front end of the C search oracle.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg use this
module, and only as the checker.  The product never imports it.
"""
import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = os.path.join(_HERE, "liboracle.so")
_lib = None


class OracleStats(ctypes.Structure):
    _fields_ = [
        ("steps_run", ctypes.c_uint32),
        ("parents_inlink", ctypes.c_uint64 * 256),
        ("parents_branch", ctypes.c_uint64 * 256),
        ("degree_sum", ctypes.c_uint64 * 256),
        ("next_pushes", ctypes.c_uint64 * 256),
        ("sel_pushes", ctypes.c_uint64 * 256),
        ("bytes_alg", ctypes.c_uint64),
        ("ties_at_cut", ctypes.c_uint32),
    ]


def build():
    """Compile liboracle.so (gcc) if it is missing or stale."""
    src = os.path.join(_HERE, "tbs_oracle.c")
    if (not os.path.exists(_LIB)) or os.path.getmtime(_LIB) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", _HERE])


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB)
        L.oracle_load.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p, ctypes.c_int]
        L.oracle_load.restype = ctypes.c_int
        L.oracle_free.argtypes = [ctypes.c_void_p]
        L.oracle_num_nodes.argtypes = [ctypes.c_void_p]
        L.oracle_num_nodes.restype = ctypes.c_uint64
        L.oracle_num_keys.argtypes = [ctypes.c_void_p]
        L.oracle_num_keys.restype = ctypes.c_uint64
        L.oracle_lookup.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32]
        L.oracle_lookup.restype = ctypes.c_int
        L.oracle_lookup_id.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32]
        L.oracle_lookup_id.restype = ctypes.c_int64
        L.oracle_tbs.argtypes = [
            ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p,
            ctypes.c_void_p, ctypes.c_float, ctypes.c_double, ctypes.c_double, ctypes.c_int,
            ctypes.c_uint32, ctypes.c_uint32, ctypes.POINTER(ctypes.c_uint32), ctypes.c_void_p,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(OracleStats)]
        L.oracle_tbs.restype = ctypes.c_int
        _lib = L
    return _lib


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


class OracleTrie:
    def __init__(self, path):
        self._h = ctypes.c_void_p()
        err = ctypes.create_string_buffer(256)
        rc = lib().oracle_load(path.encode(), ctypes.byref(self._h), err, 256)
        if rc != 0:
            raise RuntimeError("oracle_load failed: " + err.value.decode())

    def __del__(self):
        if getattr(self, "_h", None):
            lib().oracle_free(self._h)
            self._h = None

    def num_nodes(self):
        return lib().oracle_num_nodes(self._h)

    def num_keys(self):
        return lib().oracle_num_keys(self._h)

    def lookup(self, key):
        a = np.ascontiguousarray(key, dtype=np.uint32)
        return bool(lib().oracle_lookup(self._h, _ptr(a), len(a)))

    def lookup_id(self, key):
        """Key id (reference LoudsTrie::lookup), or -1."""
        a = np.ascontiguousarray(key, dtype=np.uint32)
        return int(lib().oracle_lookup_id(self._h, _ptr(a), len(a)))

    def tbs(self, beams, topk_id, topk_logp, token_logp_threshold, sents_logp_threshold,
            length_norm, early_exit, stats=False):
        """One request.  Returns (list of token lists, list of logp_norm)
        ascending, like the reference `tbs` binding (tools/bindings.cpp:45-69),
        plus an OracleStats when stats=True."""
        beams = np.ascontiguousarray(beams, dtype=np.uint32)
        ids = np.ascontiguousarray(topk_id, dtype=np.uint32)
        lp = np.ascontiguousarray(topk_logp, dtype=np.float32)
        L = len(beams)
        K = ids.shape[1] if ids.ndim == 2 else 0
        assert ids.shape == lp.shape and (ids.ndim != 2 or ids.shape[0] == L)
        cap = max(int(beams[-1]) if L else 1, 1)
        out_n = ctypes.c_uint32()
        out_lpn = np.zeros(cap, np.float64)
        out_len = np.zeros(cap, np.uint32)
        out_tok = np.zeros(cap * max(L, 1), np.uint32)
        st = OracleStats()
        rc = lib().oracle_tbs(self._h, L, K, _ptr(beams), _ptr(ids), _ptr(lp),
                              float(token_logp_threshold), float(sents_logp_threshold),
                              float(length_norm), int(bool(early_exit)), cap, max(L, 1),
                              ctypes.byref(out_n), _ptr(out_lpn), _ptr(out_len), _ptr(out_tok),
                              ctypes.byref(st))
        if rc != 0:
            raise RuntimeError("oracle_tbs failed with %d" % rc)
        n = out_n.value
        sents = [out_tok[i * max(L, 1): i * max(L, 1) + out_len[i]].tolist() for i in range(n)]
        res = (sents, out_lpn[:n].tolist())
        return res + (st,) if stats else res
