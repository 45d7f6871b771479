"""Trie-constrained beam search on inputs that already live in device memory.

For callers whose proposals come out of a model on the GPU (the top-k of the
logits at each position): the search reads them where they are and writes
its results to device tensors, on the caller's CUDA stream, with no host
copy in between.  This is the C-ABI entry point `ft_tbs_batch_device`
(include/flashtrie_b200.h); the reference has no counterpart (its
`bs_tbs_gpu` always stages host lists, tools/bindings.cpp:71-119).

    import torch, flashtrie, flashtrie_device as fd
    trie = flashtrie.Trie(); trie.load("trie.bin")
    trie.init_tbs_gpu(64, max_num_topk=1000, max_num_outpos=20, max_num_out_beams=1000)
    out = fd.bs_tbs_device(trie, beams, topk_id, topk_logp, -10.0, -40.0, 5.0, False)
    sents, lpns = fd.to_lists(out)        # host lists, only when needed
    ids = fd.lookup(trie, tokens, offsets)  # key ids of token sequences on the device
    toks, lens = fd.reverse_lookup(trie, ids, max_len=20)  # and back

Inputs (contiguous, on one CUDA device): beams int32 [n, L]; topk_id int32
[n, L, K] (token ids, read as unsigned); topk_logp float32 [n, L, K].  Rows
need not be sorted by id.  The search runs on `stream` (default: the current
stream); inputs written on another stream must be ordered before it by the
caller (an event, or stream.wait_stream), and the outputs are allocated on
`stream`.  Outputs: count int32 [n]; logp_norm float64
[n, cap] ascending; lengths int32 [n, cap]; tokens int32 [n, cap, L], beam j
of request i in tokens[i, j, :lengths[i, j]]; with key_ids=True also key ids
int32 [n, cap] (LoudsTrie::lookup's id of each result, read as unsigned).
"""
import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None


class _Params(ctypes.Structure):
    _fields_ = [("token_logp_threshold", ctypes.c_float), ("reserved", ctypes.c_float),
                ("sent_logp_threshold", ctypes.c_double), ("length_norm", ctypes.c_double),
                ("early_exit", ctypes.c_int32), ("reserved2", ctypes.c_int32)]


class _Batch(ctypes.Structure):
    _fields_ = [("n", ctypes.c_uint32), ("num_outpos", ctypes.c_uint32), ("topk", ctypes.c_uint32),
                ("out_capacity", ctypes.c_uint32)] + [(f, ctypes.c_void_p) for f in
                                                      ("beams", "topk_id", "topk_logp", "out_count", "out_lpn",
                                                       "out_len", "out_tok", "out_key")]


def _lib():
    global _LIB
    if _LIB is None:
        lib = ctypes.CDLL(os.path.join(_HERE, "libftcore.so"))
        lib.ft_tbs_batch_device.argtypes = [ctypes.c_void_p, ctypes.POINTER(_Batch), ctypes.POINTER(_Params),
                                            ctypes.c_void_p]
        lib.ft_tbs_batch_device.restype = ctypes.c_int
        lib.ft_lookup_batch_device.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p,
                                               ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p]
        lib.ft_lookup_batch_device.restype = ctypes.c_int
        lib.ft_reverse_lookup_batch_device.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p,
                                                       ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p,
                                                       ctypes.c_void_p]
        lib.ft_reverse_lookup_batch_device.restype = ctypes.c_int
        lib.ft_trie_device_status.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32)]
        lib.ft_trie_device_status.restype = ctypes.c_int
        lib.ft_last_error.restype = ctypes.c_char_p
        _LIB = lib
    return _LIB


def _check(rc):
    if rc != 0:
        raise RuntimeError(_lib().ft_last_error().decode())


def _want(t, name, dtype, ndim, device):
    if not isinstance(t, torch.Tensor) or t.device.type != "cuda":
        raise TypeError("%s must be a CUDA tensor" % name)
    if t.dtype != dtype or t.dim() != ndim or not t.is_contiguous():
        raise ValueError("%s must be a contiguous %s tensor with %d dimensions" % (name, dtype, ndim))
    if device is not None and t.device != device:
        raise ValueError("%s is on %s, expected %s" % (name, t.device, device))


def device_status(trie):
    """Synchronises the device and returns (and clears) the status bits of the
    device-resident searches since the last call (0: all searches passed their
    self-checks)."""
    st = ctypes.c_uint32(0)
    _check(_lib().ft_trie_device_status(ctypes.c_void_p(trie.ft_handle()), ctypes.byref(st)))
    return st.value


def bs_tbs_device(trie, beams, topk_id, topk_logp, token_logp_threshold, sents_logp_threshold, length_norm,
                  early_exit, capacity=None, stream=None, check=True, key_ids=False):
    """Searches n requests whose inputs are CUDA tensors; returns
    (count, logp_norm, lengths, tokens[, keys]) as CUDA tensors on the same
    device (keys with key_ids=True).

    capacity: result slots per request (>= every final beam width); default
    beams[:, -1].max(), which reads one value back from the device.
    stream: a torch.cuda.Stream (default: the current stream of the device).
    check: synchronise after the search and raise if a self-check failed or a
    request exceeded the workspace; with check=False the call is asynchronous
    and device_status() reports later."""
    _want(beams, "beams", torch.int32, 2, None)
    dev = beams.device
    _want(topk_id, "topk_id", torch.int32, 3, dev)
    _want(topk_logp, "topk_logp", torch.float32, 3, dev)
    n, L = beams.shape
    if topk_id.shape[:2] != (n, L) or topk_logp.shape != topk_id.shape:
        raise ValueError("topk_id and topk_logp must be [n, L, K] with n, L matching beams")
    K = topk_id.shape[2]
    if capacity is None:
        capacity = int(beams[:, -1].max().item()) if n and L else 1
    capacity = max(int(capacity), 1)
    if stream is None:
        stream = torch.cuda.current_stream(dev)
    # The outputs are allocated and filled on the search's stream, so the
    # fills come before the search writes them whatever stream is current.
    with torch.cuda.stream(stream):
        count = torch.zeros(n, dtype=torch.int32, device=dev)
        lpn = torch.empty((n, capacity), dtype=torch.float64, device=dev)
        lens = torch.zeros((n, capacity), dtype=torch.int32, device=dev)
        toks = torch.empty((n, capacity, max(L, 1)), dtype=torch.int32, device=dev)
        keys = torch.full((n, capacity), -1, dtype=torch.int32, device=dev) if key_ids else None
    out = (count, lpn, lens, toks) + ((keys,) if key_ids else ())
    if n == 0:
        return out
    b = _Batch(n, L, K, capacity, beams.data_ptr(), topk_id.data_ptr(), topk_logp.data_ptr(), count.data_ptr(),
               lpn.data_ptr(), lens.data_ptr(), toks.data_ptr(), keys.data_ptr() if key_ids else None)
    prm = _Params(float(token_logp_threshold), 0.0, float(sents_logp_threshold), float(length_norm),
                  int(bool(early_exit)), 0)
    with torch.cuda.device(dev):
        _check(_lib().ft_tbs_batch_device(ctypes.c_void_p(trie.ft_handle()), ctypes.byref(b), ctypes.byref(prm),
                                          ctypes.c_void_p(stream.cuda_stream)))
    if check:
        st = device_status(trie)
        if st:
            raise RuntimeError("device search failed its self-checks or exceeded the workspace (status 0x%x)" % st)
    return out


def lookup(trie, tokens, offsets, stream=None, check=True):
    """Key ids of n token sequences on the device: LoudsTrie::lookup for a
    batch (C ABI ft_lookup_batch_device).  tokens: int32 CUDA tensor [T]
    (ids read as unsigned); offsets: int64 CUDA tensor [n + 1], key i being
    tokens[offsets[i]:offsets[i + 1]].  Returns an int32 tensor [n] of key
    ids (the ids key_ids=True reports; read as unsigned), -1 where the
    sequence is not a key.  check: synchronise and raise if the kernel
    reported bad offsets or an inconsistent trie."""
    _want(tokens, "tokens", torch.int32, 1, None)
    dev = tokens.device
    _want(offsets, "offsets", torch.int64, 1, dev)
    n = offsets.numel() - 1
    if n < 0:
        raise ValueError("offsets must have n + 1 >= 1 entries")
    if stream is None:
        stream = torch.cuda.current_stream(dev)
    with torch.cuda.stream(stream):
        out = torch.empty(n, dtype=torch.int32, device=dev)
    if n == 0:
        return out
    with torch.cuda.device(dev):
        _check(_lib().ft_lookup_batch_device(ctypes.c_void_p(trie.ft_handle()), n, ctypes.c_void_p(tokens.data_ptr()),
                                             ctypes.c_void_p(offsets.data_ptr()), tokens.numel(),
                                             ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(stream.cuda_stream)))
    if check:
        st = device_status(trie)
        if st:
            raise RuntimeError("device lookup reported bad offsets or an inconsistent trie (status 0x%x)" % st)
    return out


def reverse_lookup(trie, ids, max_len, stream=None, check=True):
    """Token sequences of key ids on the device: LoudsTrie::reverse_lookup
    for a batch (C ABI ft_reverse_lookup_batch_device).  ids: int32 CUDA
    tensor [n] (read as unsigned).  Returns (tokens int32 [n, max_len],
    lengths int32 [n]): key i is tokens[i, :lengths[i]] when lengths[i] <=
    max_len (longer keys report their length and write no tokens); -1 marks
    an id that is not a key id.  The first call derives the trie's parent
    links on the device once."""
    _want(ids, "ids", torch.int32, 1, None)
    dev = ids.device
    n = ids.numel()
    max_len = int(max_len)
    if max_len < 0:
        raise ValueError("max_len must be >= 0")
    if stream is None:
        stream = torch.cuda.current_stream(dev)
    with torch.cuda.stream(stream):
        toks = torch.zeros((n, max(max_len, 1)), dtype=torch.int32, device=dev)
        lens = torch.empty(n, dtype=torch.int32, device=dev)
    if n == 0:
        return toks[:, :max_len], lens
    with torch.cuda.device(dev):
        _check(_lib().ft_reverse_lookup_batch_device(ctypes.c_void_p(trie.ft_handle()), n,
                                                     ctypes.c_void_p(ids.data_ptr()), max_len,
                                                     ctypes.c_void_p(toks.data_ptr()), ctypes.c_void_p(lens.data_ptr()),
                                                     ctypes.c_void_p(stream.cuda_stream)))
    if check:
        st = device_status(trie)
        if st:
            raise RuntimeError("device reverse lookup found an inconsistent trie (status 0x%x)" % st)
    return toks[:, :max_len], lens


def to_lists(out):
    """(count, logp_norm, lengths, tokens[, keys]) -> (sentences, logp_norms
    [, key_ids]) as host lists in the layout bs_tbs_gpu returns."""
    host = [t.cpu() for t in out]
    count, lpn, lens, toks = host[:4]
    sents, lpns, keys = [], [], []
    for i in range(count.shape[0]):
        c = int(count[i])
        sents.append([(toks[i, j, :int(lens[i, j])].numpy().view("uint32")).tolist() for j in range(c)])
        lpns.append(lpn[i, :c].tolist())
        if len(host) > 4:
            keys.append(host[4][i, :c].numpy().view("uint32").tolist())
    return (sents, lpns, keys) if len(host) > 4 else (sents, lpns)
