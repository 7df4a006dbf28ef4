"""The C-ABI library loads and exports every entry point the header declares.
CPU only: no compute call is made."""
import ctypes
import os
import re

import pytest

from tinylm_c_b200 import _lib
from tinylm_c_b200.zero1 import zero1_layout

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    inc = os.path.join(ROOT, "include")
    for f in os.listdir(inc):
        if f.endswith(".h"):
            src = open(os.path.join(inc, f)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names |= set(re.findall(r"\b(tl_\w+)\s*\(", src))
    return names


def test_library_loads_and_exports_header():
    L = _lib.lib()
    names = declared_symbols()
    assert len(names) >= 25
    for n in sorted(names):
        assert hasattr(L, n), f"{n} declared in include/ but not exported"


def test_binding_table_covers_header():
    assert declared_symbols() == set(_lib.SIGNATURES), "ctypes table and header disagree"


def test_exports_are_c_abi_only():
    """No C++-mangled public symbols leak from the library."""
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    public = [l.split()[-1] for l in out.splitlines() if " T " in l]
    assert all(not s.startswith("_Z") for s in public), [s for s in public if s.startswith("_Z")][:5]


@pytest.mark.parametrize("n,world", [(0, 1), (1, 1), (976000, 1), (976000, 2), (188777472, 8), (4096 * 8, 8), (4096 * 8 + 1, 8)])
def test_zero1_layout_matches_library(n, world):
    n_pad, shard = zero1_layout(n, world)
    assert _lib.lib().tl_zero1_padded(n, world) == n_pad
    assert n_pad >= n and n_pad % (world * 4096) == 0 and shard * world == n_pad
    assert n_pad - n < world * 4096


def test_calls_before_init_return_status_not_crash():
    """Without tl_init (and here without any GPU) a compute call reports
    TL_ENOINIT through the status code and tl_last_error."""
    L = _lib.lib()
    rc = L.tl_matmul(None, None, None, 4, 4, 4)
    assert rc == _lib.TL_ENOINIT
    assert b"tl_init" in L.tl_last_error()
    assert L.tl_set_gemm_engine(7) == _lib.TL_EINVAL
    assert L.tl_set_gemm_engine(-1) == _lib.TL_EINVAL
    for e in range(6):   # 0 automatic ... 5 the hybrid split: per-thread settings, no device needed
        assert L.tl_set_gemm_engine(e) == _lib.TL_OK
    assert L.tl_set_gemm_engine(0) == _lib.TL_OK


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "nope.so"))
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(ImportError):
        _lib.lib()
