"""The Julia ccall bindings shown in INTEGRATION.md match the C header: every
bound name is declared, and each call's argument-type tuple and argument list
have the prototype's length, with Julia types that agree with the C ones."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _prototypes():
    text = open(os.path.join(ROOT, "include", "reels_lowvram.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    out = {}
    for m in re.finditer(r"\b(reels_\w+)\s*\(([^)]*)\)\s*;", text):
        params = m.group(2).strip()
        out[m.group(1)] = [] if params in ("", "void") else [p.strip() for p in params.split(",")]
    return out


def _balanced(s, i):
    depth = 0
    for j in range(i, len(s)):
        depth += {"(": 1, ")": -1}.get(s[j], 0)
        if depth == 0:
            return s[i:j + 1]
    raise ValueError("unbalanced parentheses")


def _split_top(s):
    out, depth, cur = [], 0, ""
    for ch in s:
        depth += {"(": 1, "{": 1, ")": -1, "}": -1}.get(ch, 0)
        if ch == "," and depth == 0:
            out.append(cur.strip())
            cur = ""
        else:
            cur += ch
    if cur.strip():
        out.append(cur.strip())
    return out


def _ccalls():
    doc = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    for m in re.finditer(r"ccall\(\(:(\w+),", doc):
        parts = _split_top(_balanced(doc, m.start() + len("ccall"))[1:-1])
        yield m.group(1), parts[2], parts[3:]


def _agrees(jl, c):
    ctype = c.rsplit(" ", 1)[0] if " " in c else c
    ptr = "*" in c
    rules = {"Cint": lambda: ctype.strip() == "int", "Int64": lambda: "int64_t" in ctype and not ptr,
             "Csize_t": lambda: "size_t" in ctype and not ptr, "Cfloat": lambda: ctype.strip() == "float",
             "UInt64": lambda: "uint64_t" in ctype and not ptr}
    if jl.startswith(("CuPtr", "Ptr")):
        return ptr
    return rules[jl]()


def test_julia_bindings_match_the_header():
    protos = _prototypes()
    calls = list(_ccalls())
    assert len(calls) >= 10
    for name, types, args in calls:
        assert name in protos, name
        tys = _split_top(types.strip()[1:-1])
        assert len(tys) == len(protos[name]) == len(args), (name, len(tys), len(protos[name]), len(args))
        for jl, c in zip(tys, protos[name]):
            assert _agrees(jl, c), (name, jl, c)
