"""CPU: libmhmoe.so loads and exports every symbol include/mhmoe.h declares, and the
ctypes table matches the header.  No device calls (there is no GPU here)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "mhmoe.h"


def declared_symbols():
    txt = HEADER.read_text()
    return sorted(set(re.findall(r"^MHMOE_API\s+[\w\s\*]+?\b(mhmoe_\w+)\(", txt, flags=re.M)))


def _lib_path():
    from flash_mh_moe import _lib
    return _lib.LIB_PATH


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ["mhmoe_topk", "mhmoe_global_sort", "mhmoe_ffn_nvfp4", "mhmoe_pack_weights_nvfp4",
              "mhmoe_router_logits"]:
        assert s in syms


def test_library_exports_all_declared_symbols():
    p = _lib_path()
    if not p.exists():
        pytest.fail(f"{p} is not built (run magi-2-preview_b200/build.py)")
    lib = ctypes.CDLL(str(p))
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_ctypes_table_covers_header():
    from flash_mh_moe import _lib
    assert sorted(_lib.SIGNATURES) == declared_symbols()


def test_host_only_calls():
    from flash_mh_moe import _lib
    L = _lib.lib()
    assert L.mhmoe_version() >= 1
    assert L.mhmoe_status_string(0) == b"ok"
    assert L.mhmoe_max_mtiles(131072, 128) == 1024 + 128
    assert L.mhmoe_global_sort_workspace_bytes(1, 16384, 8, 128) > 0
    assert L.mhmoe_ffn_workspace_bytes(131072, 16384, 1, 3072, 1024, 128) > 131072 * 3072 * 2


def test_cuda_calls_refuse_without_device():
    """Every compute entry point fails loudly (no CPU fallback) when no sm_100 is present."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("device present")
    from flash_mh_moe import _lib
    L = _lib.lib()
    rc = L.mhmoe_topk(1, None, 1, 1, 8, 2, 0, 1, 0, 1, 1e-12, 1.0, 1, 1, None)
    assert rc != 0
