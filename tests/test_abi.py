"""The C-ABI library loads and exports every function include/*.h declares
(no device work: these run without a GPU)."""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in ("sam3_cuda.h", "sam3_synth.h"):
        text = open(os.path.join(ROOT, "include", h)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^\s*(?:[\w\s\*]+?)\b((?:cb|sam3)_\w+)\s*\(", text, re.M):
            if "static inline" in text[max(0, m.start() - 40):m.start() + 40]:
                continue
            names.add(m.group(1))
    return sorted(n for n in names if not n.startswith("sam3_mix") and
                  n not in ("sam3_stream_base", "sam3_normal_at", "sam3_u8_at"))


def test_library_builds_and_exports_every_declared_symbol(sb):
    import ctypes
    lib = sb.lib()
    names = declared_functions()
    assert len(names) > 40
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(sb.EXPORTS) == set(names)


def test_status_strings_and_no_device_init(sb):
    import ctypes
    lib = sb.lib()
    assert lib.cb_errstr(0) == b"success"
    assert b"argument" in lib.cb_errstr(3)
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if has_gpu:
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    assert lib.cb_init(ctypes.byref(h), 0) == 1  # CB_ENODEV


def test_host_generator_matches_oracle_copy(sb, ob):
    import numpy as np
    n = 4096
    a = np.empty(n, np.float32)
    sb.lib().sam3_synth_normal(9, 4, n, 0.0, 0.02, a.ctypes.data)
    assert np.array_equal(a, ob.normal(9, 4, (n,), 0.0, 0.02))
