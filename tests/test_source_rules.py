"""Static checks of the CUDA sources (CPU).

* Every kernel launched with programmatic stream serialisation (``launch_pdl`` /
  ``MHMOE_LAUNCH_PDL``) must begin with ``pdl_wait()``: such a kernel may be scheduled
  before its predecessor finishes, and anything it read before the wait could be stale.
* No bulk or tensor copy may load with cluster multicast (the library runs on multi-GPU
  boxes, where such a load of peer memory is not allowed).
"""
import re
from pathlib import Path

CSRC = Path(__file__).resolve().parents[1] / "magi-2-preview_b200" / "csrc"


def _sources():
    return {p.name: p.read_text() for p in sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh"))}


def _pdl_launched(srcs):
    names = set()
    for text in srcs.values():
        # call sites only: the first argument (a kernel, maybe with template arguments) then a comma
        for m in re.finditer(r"(?:MHMOE_LAUNCH_PDL|launch_pdl)\(\s*([A-Za-z_]\w*)\s*(?:<[^<>]*>)?\s*,", text):
            names.add(m.group(1))
    return names


def _kernel_body_start(text, name):
    """First statement of each __global__ definition named `name` (templates included)."""
    out = []
    for m in re.finditer(r"__global__[^;{]*?\b" + re.escape(name) + r"\s*\(", text, re.S):
        depth, i = 0, m.end() - 1
        while True:
            if text[i] == "(":
                depth += 1
            elif text[i] == ")":
                depth -= 1
                if depth == 0:
                    break
            i += 1
        j = text.index("{", i)
        out.append(text[j + 1:j + 200].strip().split(";")[0])
    return out


def test_pdl_kernels_wait_first():
    srcs = _sources()
    launched = _pdl_launched(srcs)
    # the macro's own body and the router launch a function-pointer variable named `kernel`;
    # the router's kernel is checked by name
    launched.discard("kernel")
    launched.add("router_tc_kernel")
    assert len(launched) >= 15, launched
    for name in sorted(launched):
        starts = [s for text in srcs.values() for s in _kernel_body_start(text, name)]
        assert starts, f"no __global__ definition found for {name}"
        for s in starts:
            assert s.startswith("pdl_wait()"), f"{name} does not start with pdl_wait(): {s!r}"


def test_no_multicast_loads():
    for fname, text in _sources().items():
        for ln, line in enumerate(text.splitlines(), 1):
            if "cp.async.bulk" in line and "multicast" in line:
                raise AssertionError(f"{fname}:{ln}: bulk/tensor load with cluster multicast")
