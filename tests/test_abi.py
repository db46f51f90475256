"""CPU: the C-ABI library builds, loads and exports every symbol include/hb_b200.h declares, with the
prototypes the ctypes binding uses. No compute calls (no GPU here)."""
import re

import pytest

from conftest import ROOT


def _header_functions():
    text = (ROOT / "include" / "hb_b200.h").read_text()
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
