"""CPU: ``__graft_entry__.build()`` compiles the library (when nvcc is present) and
accepts it -- an ABI bump in the header must not break the build entry point."""
import os
import shutil
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(shutil.which("nvcc") is None and not os.path.exists("/usr/local/cuda/bin/nvcc"),
                    reason="needs nvcc")
def test_build_entry_point_builds_and_loads():
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    import __graft_entry__

    from detkernels_b200 import _lib
    __graft_entry__.build()
    assert _lib.load().dk_abi_version() == _lib.ABI_VERSION


def test_loader_reports_a_stale_library(tmp_path, monkeypatch):
    """A library without the declared entry points is refused with the rebuild message."""
    import subprocess

    from detkernels_b200 import _lib
    src = tmp_path / "stale.c"
    src.write_text("int dk_abi_version(void) { return %d; }\n" % _lib.ABI_VERSION)
    so = tmp_path / "libstale.so"
    subprocess.run(["gcc", "-shared", "-fPIC", "-o", str(so), str(src)], check=True)
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "library_path", lambda: str(so))
    with pytest.raises(_lib.DetKernelsError, match="stale build"):
        _lib.load()
    src.write_text("int dk_abi_version(void) { return 1; }\n")
    subprocess.run(["gcc", "-shared", "-fPIC", "-o", str(so) + "1", str(src)], check=True)
    monkeypatch.setattr(_lib, "library_path", lambda: str(so) + "1")
    with pytest.raises(_lib.DetKernelsError, match="ABI version 1"):
        _lib.load()
