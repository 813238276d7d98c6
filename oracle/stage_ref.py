"""Stage the reference's own ``inference/flash_mh_moe`` package into ``oracle/_ref/``.

    python oracle/stage_ref.py [--src <reference root>]

Test and comparison infrastructure only.  The reference path is Python + Triton
(``route.py`` in plain torch, ``triton/mh_moe_fwd.py`` JIT-compiled for the GPU it runs
on), so "building" it means placing its unmodified source files where the GPU box can
import them: ``oracle/_ref/flash_mh_moe/`` (git-ignored; it travels with the working
tree).  ``bench.py --impl reference`` imports it from there to time the reference's own
layer path — its CPU route/sort, and its Triton kernel on the B200 at the shapes that
kernel compiles (power-of-two d_head).  Nothing in the product package imports it.

Files copied verbatim (their paths within the reference project):
  inference/flash_mh_moe/__init__.py, fwd.py, route.py,
  inference/flash_mh_moe/triton/__init__.py, triton/mh_moe_fwd.py
"""
from __future__ import annotations

import argparse
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
DEST = HERE / "_ref" / "flash_mh_moe"
FILES = ("__init__.py", "fwd.py", "route.py", "triton/__init__.py", "triton/mh_moe_fwd.py")
DEFAULT_SRC = Path("/root/reference")


def stage(src_root: Path = DEFAULT_SRC, quiet: bool = False) -> Path | None:
    """Copy the reference package into oracle/_ref; returns the package dir, or None when
    the reference tree is absent (e.g. on a GPU box, where a staged copy is used as is)."""
    src = Path(src_root) / "inference" / "flash_mh_moe"
    if not src.is_dir():
        if not quiet:
            print(f"reference package not found at {src}; nothing staged", file=sys.stderr)
        return DEST if (DEST / "__init__.py").exists() else None
    for rel in FILES:
        s, d = src / rel, DEST / rel
        d.parent.mkdir(parents=True, exist_ok=True)
        if not d.exists() or d.read_bytes() != s.read_bytes():
            shutil.copyfile(s, d)
    (DEST.parent / "README").write_text(
        "Unmodified copy of the reference's inference/flash_mh_moe package, staged by "
        "oracle/stage_ref.py for comparison timing. Not product code; git-ignored.\n")
    if not quiet:
        print(f"staged {len(FILES)} files into {DEST}")
    return DEST


def import_ref():
    """Import the staged reference package as ``ref_flash_mh_moe`` (raises ImportError when
    it was never staged)."""
    import importlib.util
    init = DEST / "__init__.py"
    if not init.exists():
        raise ImportError("reference flash_mh_moe is not staged under oracle/_ref (run oracle/stage_ref.py)")
    name = "ref_flash_mh_moe"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, init, submodule_search_locations=[str(DEST)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--src", default=str(DEFAULT_SRC))
    a = ap.parse_args()
    stage(Path(a.src))
