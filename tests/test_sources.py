"""Source-level checks of the CUDA code that need no GPU.

Kernels launched through `launch_pdl` (programmatic stream serialization)
may start before the previous kernel of the stream has finished; they are
correct only if they wait (`pdl_enter`, which runs `griddepcontrol.wait`)
before touching global memory. This test finds every kernel passed to
`launch_pdl` and checks that its body starts with that call."""
import os
import re

CSRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "musapy_b200", "csrc")


def _sources():
    out = {}
    for name in sorted(os.listdir(CSRC)):
        if name.endswith((".cu", ".cuh", ".h")):
            with open(os.path.join(CSRC, name)) as f:
                out[name] = f.read()
    return out


def _kernel_body_start(text, kernel):
    """The first statement of __global__ function `kernel`, or None."""
    m = re.search(r"__global__[^;{]*?\b" + re.escape(kernel) + r"\s*\(", text)
    if not m:
        return None
    depth, i = 0, m.end() - 1
    while i < len(text):  # skip the parameter list
        if text[i] == "(":
            depth += 1
        elif text[i] == ")":
            depth -= 1
            if depth == 0:
                break
        i += 1
    brace = text.index("{", i)
    body = text[brace + 1:]
    body = re.sub(r"^\s*(//[^\n]*\n\s*)*", "", body)
    return body.split(";", 1)[0].strip()


def test_every_pdl_launched_kernel_waits_first():
    src = _sources()
    launched = set()
    for text in src.values():
        for m in re.finditer(r"launch_pdl\(\s*(k_[A-Za-z0-9_]*)", text):
            launched.add(m.group(1))
    assert {"k_ew_contig", "k_ew_rows", "k_red_row_block", "k_red_combine", "k_red_col_v"} <= launched
    for k in sorted(launched):
        firsts = [s for s in (_kernel_body_start(t, k) for t in src.values()) if s is not None]
        assert firsts, f"kernel {k} passed to launch_pdl but not defined in csrc/"
        for first in firsts:
            assert first == "pdl_enter()", f"kernel {k} is launched with launch_pdl but starts with {first!r}"


def test_kernels_that_start_with_pdl_enter():
    """The kernels that start with pdl_enter are exactly the ones launched
    with launch_pdl (in a kernel launched the plain way it would return at
    once; the list keeps a new use deliberate)."""
    src = _sources()
    users = set()
    for text in src.values():
        for m in re.finditer(r"__global__[^;{]*?\b(k_[A-Za-z0-9_]*)\s*\(", text):
            if _kernel_body_start(text, m.group(1)) == "pdl_enter()":
                users.add(m.group(1))
    assert users == {"k_ew_contig", "k_ew_rows", "k_red_row_warp", "k_red_row_block", "k_red_col", "k_red_col_v",
                     "k_red_combine", "k_red_gen"}
