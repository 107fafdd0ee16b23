"""The C-ABI library loads without a GPU and exports every entry point of include/q3t.h.

No compute call is made: loading resolves symbols only. The ctypes signature
table used by the Python host must name exactly the header's entry points.
"""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "q3t.h"


def declared():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(q3t_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_engine_entry_points():
    names = declared()
    for required in ("q3t_linear", "q3t_decode_attention", "q3t_sample", "q3t_kv_write", "q3t_tick_gather",
                     "q3t_tick_commit", "q3t_code_ring_read", "q3t_pcm16", "q3t_rvq_gather",
                     "q3t_decode_attention_noalloc"):
        assert required in names


def test_library_exports_every_declared_symbol():
    from qwen3_tts_b200 import _lib
    if not _lib.LIBRARY_PATH.exists():
        pytest.skip("libq3t_b200.so not built (run __graft_entry__.build())")
    lib = ctypes.CDLL(str(_lib.LIBRARY_PATH))
    missing = [name for name in declared() if not hasattr(lib, name)]
    assert not missing, missing


def test_ctypes_table_matches_header():
    from qwen3_tts_b200 import _lib
    assert sorted(_lib.SIGNATURES) == declared()
