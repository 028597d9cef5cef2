"""The C-ABI library builds for sm_100a, loads without a GPU and exports every
symbol the public header declares (no compute calls here)."""
import ctypes
import os
import re

from aideen_b200 import backend, build
from aideen_b200.layout import all_weights_len

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    src = open(os.path.join(ROOT, "include", "aideen_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(aideen_[a-z_]+)\s*\(", src)))


def test_library_exports_every_header_symbol():
    build.build()
    lib = ctypes.CDLL(build.LIB)
    names = header_functions()
    assert len(names) >= 25
    for n in names:
        assert hasattr(lib, n), n
    # the Python mirror declares the same set
    assert set(backend.exported_symbols()) == set(names)


def test_all_weights_len_host_function():
    lib = backend.load_library()
    for d, h in [(128, 4), (512, 8), (1024, 16)]:
        assert lib.aideen_all_weights_len(d, h) == all_weights_len(d, h)


def test_header_constants_match_the_python_mirror():
    """The aideen_cfg flag bit and the constants the Python mirror passes through
    the C ABI are the header's."""
    src = open(os.path.join(ROOT, "include", "aideen_b200.h")).read()
    defs = dict(re.findall(r"#define\s+(AIDEEN_\w+)\s+(\d+)u?", src))
    assert int(defs["AIDEEN_CFG_ASSOC"]) == backend.CFG_ASSOC
    assert int(defs["AIDEEN_UNIQUE_ID_BYTES"]) == 128
