"""The C-ABI library loads and exports every entry point include/layerstream.h declares (no GPU needed:
nothing here launches a kernel)."""

import os
import re
import subprocess

import pytest

import layerstream_b200 as ls

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "layerstream.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ls_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_verify_path_entry_points():
    names = declared_functions()
    for must in ["ls_model_open", "ls_forward", "ls_forward_multi", "ls_verify", "ls_truncate", "ls_speculative_greedy",
                 "ls_quantize_model", "ls_last_error"]:
        assert must in names


def test_library_loads_and_exports_every_declared_symbol():
    L = ls.lib()
    missing = [n for n in declared_functions() if not hasattr(L, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", ls.LIB_PATH], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r" T (ls_\w+)", out))
    assert set(declared_functions()) <= exported
    # nothing else leaks out of the library's C ABI
    assert exported <= set(declared_functions())


def test_binding_covers_every_declared_symbol():
    assert set(declared_functions()) == set(ls.SYMBOLS)


def test_errors_are_values_not_crashes():
    # a missing file is an error status with a message, raised as LayerstreamError (no GPU touched)
    with pytest.raises(ls.LayerstreamError) as e:
        ls.Model("/nonexistent/model.lsq")
    assert "nonexistent" in str(e.value) or "open" in str(e.value)
