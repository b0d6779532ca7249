"""Static check of the programmatic-dependent-launch rule (CPU, no device).

Kernels launched with programmatic stream serialization (`launch_pdl` and
`launch_pdl_cluster` in reels_b200/csrc/lowvram.cu) may be scheduled before the kernel ahead of them
in the stream has finished.  Each must therefore execute
`griddepcontrol.wait` (griddep_wait) before touching global memory, and must
execute it on every path: a kernel whose CTAs could all exit without waiting
would complete before its predecessor and release the kernel after it too
early, breaking the stream's order transitively.  This test finds every
kernel passed to launch_pdl and checks that its body calls griddep_wait()
before any `return` and before its first global-memory access by pointer
argument."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "reels_b200", "csrc")


def _sources():
    out = {}
    for f in sorted(os.listdir(CSRC)):
        if f.endswith((".cu", ".cuh")):
            out[f] = open(os.path.join(CSRC, f)).read()
    return out


def _kernel_body(src, name):
    m = re.search(r"__global__\s+void\s+(?:__launch_bounds__\([^)]*\)\s*)?" + re.escape(name) + r"\s*\(", src)
    if not m:
        return None
    i = src.index("{", m.end())
    depth, j = 0, i
    while True:
        if src[j] == "{":
            depth += 1
        elif src[j] == "}":
            depth -= 1
            if depth == 0:
                return src[i:j + 1]
        j += 1


def test_every_pdl_kernel_waits_before_anything_else():
    srcs = _sources()
    launcher = srcs["lowvram.cu"]
    names = set(re.findall(r"launch_pdl(?:_cluster)?\(\s*([A-Za-z_][A-Za-z_0-9]*)", launcher))
    names -= {"kern", "void"}
    assert names, "no launch_pdl call sites found"
    checked = 0
    for name in sorted(names):
        body = None
        for src in srcs.values():
            body = _kernel_body(src, name)
            if body:
                break
        assert body is not None, f"kernel {name} not found"
        w = body.find("griddep_wait()")
        assert w >= 0, f"{name} is launched with programmatic serialization but never waits"
        before = body[:w]
        assert "return" not in before, f"{name} can return before griddep_wait()"
        checked += 1
    assert checked >= 10
