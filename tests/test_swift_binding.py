"""The Swift wrapper (source only: no Swift toolchain here) stays in step with
the C header: every dr_* call in it names a declared entry point and passes as
many arguments as the declaration has parameters."""
import os
import re

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "diffrast.h")
SWIFT = os.path.join(ROOT, "mlx-swift-diffrast_b200", "swift", "Sources", "DiffRast", "DiffRast.swift")


def _split_top(args: str):
    depth, cur, out = 0, "", []
    for ch in args:
        if ch in "([{":
            depth += 1
        elif ch in ")]}":
            depth -= 1
        if ch == "," and depth == 0:
            out.append(cur)
            cur = ""
        else:
            cur += ch
    if cur.strip():
        out.append(cur)
    return out


def _calls(src: str, name_re: str):
    for m in re.finditer(name_re, src):
        i, depth = m.end(), 1
        while depth:
            depth += {"(": 1, ")": -1}.get(src[i], 0)
            i += 1
        yield m.group(1), src[m.end():i - 1]


def test_swift_calls_match_header_arity():
    hdr = open(HEADER).read()
    decl = {name: (0 if args.strip() in ("", "void") else len(_split_top(args)))
            for name, args in _calls(hdr, r"\bDR_API\s+[\w\s\*]*?\b(dr_\w+)\s*\(")}
    src = open(SWIFT).read()
    seen = 0
    for name, args in _calls(src, r"\b(dr_\w+)\("):
        assert name in decl, f"{name} is not declared in include/diffrast.h"
        n = 0 if not args.strip() else len(_split_top(args))
        assert n == decl[name], f"{name}: Swift passes {n} arguments, header declares {decl[name]}"
        seen += 1
    assert seen >= 12
