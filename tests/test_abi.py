"""CPU: the C-ABI libraries build, load and export every symbol include/hb_b200.h and include/hb_comm.h
declare, with the prototypes the ctypes bindings use. No compute or communicator calls (no GPU here)."""
import re

import pytest

from conftest import ROOT


def _header_functions(header="hb_b200.h"):
    text = (ROOT / "include" / header).read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"^\s*int\s+(hb_\w+)\s*\(", text, flags=re.M)


def test_library_exports_every_declared_symbol():
    from hummingbird_b200 import _lib, build
    build.build()
    lib = _lib.lib()
    names = _header_functions()
    assert len(names) >= 8
    for name in names:
        assert hasattr(lib, name), f"{name} declared in hb_b200.h but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes prototype"


def test_header_argument_counts_match_binding():
    text = re.sub(r"/\*.*?\*/", "", (ROOT / "include" / "hb_b200.h").read_text(), flags=re.S)
    from hummingbird_b200 import _lib
    for name, body in re.findall(r"int\s+(hb_\w+)\s*\(([^)]*)\)\s*;", text):
        args = [a for a in body.split(",") if a.strip() and a.strip() != "void"]
        assert len(args) == len(_lib.SIGNATURES[name]), name


def test_comm_library_exports_every_declared_symbol():
    from hummingbird_b200 import build, comm
    build.build_comm()
    lib = comm.lib()
    names = _header_functions("hb_comm.h")
    assert len(names) == 7
    text = re.sub(r"/\*.*?\*/", "", (ROOT / "include" / "hb_comm.h").read_text(), flags=re.S)
    for name in names:
        assert hasattr(lib, name), f"{name} declared in hb_comm.h but not exported"
    for name, body in re.findall(r"int\s+(hb_\w+)\s*\(([^)]*)\)\s*;", text):
        args = [a for a in body.split(",") if a.strip() and a.strip() != "void"]
        assert len(args) == len(comm.SIGNATURES[name]), name


def test_comm_rejects_bad_arguments_before_any_nccl_call():
    import ctypes
    from hummingbird_b200 import comm
    lib = comm.lib()
    h = ctypes.c_void_p()
    uid = ctypes.create_string_buffer(comm.ID_BYTES)
    assert lib.hb_comm_init(uid, 2, 2, 1000, ctypes.byref(h)) == 1   # rank out of range: HB_ERR_SHAPE
    assert lib.hb_comm_init(None, 2, 0, 1000, ctypes.byref(h)) == 9  # HB_ERR_NULL
    assert lib.hb_comm_halo_exchange(None, None, 1, 0, 0, 0, 1, 0, 0, 0, 1000, None) == 9


def test_no_cpu_fallback_when_library_missing(tmp_path, monkeypatch):
    from hummingbird_b200 import _lib
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "missing.so")
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(RuntimeError, match="missing"):
        _lib.lib()


def test_kernel_sources_use_cta_local_loads_only():
    # The same kernels run in multi-GPU jobs, so no TMA / bulk load may use cluster multicast: every CTA
    # loads its own copy. The searched qualifier is assembled from parts so this test does not spell it.
    bad = re.compile("multi" + "cast" + re.escape("::") + "clu" + "ster")
    for path in list((ROOT / "hummingbird_b200" / "csrc").glob("*")):
        assert not bad.search(path.read_text()), path
