"""The module `flashtrie` offers the reference module's surface.

The fixture holds the signature line pybind11 writes for every public
function and `Trie` method of the unmodified reference module
(tools/bindings.cpp:24-122).  For each of them the engine's module must have
the same name, the same parameter names in the same order (a caller may pass
any of them by keyword, as examples/flashtrie_bench.py:222-248 does) and the
same defaults; parameters the engine adds come after them and all have
defaults.  Parameters the reference leaves unnamed (`arg0`) are positional
only there, so any name is accepted for them here.
"""
import pytest

from helpers import load_json


def split_params(sig):
    """[(name, default or None)] of a pybind11 signature line
    `name(a: T, b: T = d, *, c: T = e) -> R`, with the type annotations
    (which contain commas inside brackets) skipped."""
    parts, depth, cur = [], 0, ""
    for ch in sig[sig.index("(") + 1:]:
        if ch in "[(":
            depth += 1
        elif ch in "])":
            depth -= 1
            if depth < 0:  # the parameter list's closing parenthesis
                break
        if ch == "," and depth == 0:
            parts.append(cur.strip())
            cur = ""
        else:
            cur += ch
    if cur.strip():
        parts.append(cur.strip())
    out = []
    for p in parts:
        if p in ("*", "/"):
            out.append((p, None))
            continue
        name = p.split(":")[0].split("=")[0].strip()
        default = p.split("=", 1)[1].strip() if "=" in p else None
        out.append((name, default))
    return out


def test_signature_parser():
    got = split_params("f(self: X, a: dict[str, int], b: typing.Sequence[int] = 3, *, c: bool = False) -> None")
    assert got == [("self", None), ("a", None), ("b", "3"), ("*", None), ("c", "False")]


def _check(ours_sig, ref_sig, what):
    ref_p = [p for p in split_params(ref_sig) if p[0] != "self"]
    ours_p = [p for p in split_params(ours_sig) if p[0] != "self"]
    ours_named = [p for p in ours_p if p[0] not in ("*", "/")]
    assert len(ours_named) >= len(ref_p), what
    for (rn, rd), (on, od) in zip(ref_p, ours_named):
        if not rn.startswith("arg"):
            assert on == rn, "%s: parameter %s is called %s" % (what, rn, on)
        assert od == rd, "%s: default of %s is %s, the reference's %s" % (what, rn, od, rd)
    for on, od in ours_named[len(ref_p):]:
        assert od is not None, "%s: added parameter %s has no default" % (what, on)


def test_module_surface_matches_reference(built):
    import flashtrie
    g = load_json("api_surface.json")
    for name, ref_sig in g["functions"].items():
        assert hasattr(flashtrie, name), name
        _check(getattr(flashtrie, name).__doc__.strip().split("\n")[0], ref_sig, name)
    for name, ref_sig in g["Trie"].items():
        assert hasattr(flashtrie.Trie, name), "Trie." + name
        _check(getattr(flashtrie.Trie, name).__doc__.strip().split("\n")[0], ref_sig, "Trie." + name)


@pytest.mark.parametrize("bad", [
    "tbs(trie: T, beams: X, topk_id: Y, topk_logp: Z, token_logp_threshold: F, sents_logp_threshold: F, "
    "length_norm: F, early_exit: bool, use_gpu: bool = True) -> tuple",
    "tbs(trie: T, beams: X, topk_ids: Y, topk_logp: Z, token_logp_threshold: F, sents_logp_threshold: F, "
    "length_norm: F, early_exit: bool, use_gpu: bool = False) -> tuple",
    "tbs(trie: T, beams: X, topk_id: Y, topk_logp: Z, token_logp_threshold: F, sents_logp_threshold: F, "
    "length_norm: F, early_exit: bool, use_gpu: bool = False, extra: int) -> tuple",
])
def test_surface_check_catches_drift(bad):
    """A changed default, a renamed keyword and an added required parameter
    are each reported."""
    g = load_json("api_surface.json")
    with pytest.raises(AssertionError):
        _check(bad, g["functions"]["tbs"], "tbs")
