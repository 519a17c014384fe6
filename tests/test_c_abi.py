"""The C ABI from a C host: tests/c/abi_check.c is compiled with the system C compiler against
include/htrc_flat.h, linked to libhtrc_flat.so and run (no GPU: argument validation and workspace
sizing only)."""
import os
import shutil
import subprocess
from pathlib import Path

import pytest

from htrc_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


def test_c_host_compiles_links_and_runs(tmp_path):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lib_dir = _lib.LIB_PATH.parent
    exe = tmp_path / "abi_check"
    subprocess.run([cc, "-std=c99", "-Wall", "-Werror", "-I", str(ROOT / "include"), str(ROOT / "tests" / "c" / "abi_check.c"),
                    "-L", str(lib_dir), "-lhtrc_flat", f"-Wl,-rpath,{lib_dir}", "-o", str(exe)], check=True)
    env = dict(os.environ, LD_LIBRARY_PATH=f"{lib_dir}:{os.environ.get('LD_LIBRARY_PATH', '')}")
    r = subprocess.run([str(exe)], capture_output=True, text=True, env=env, timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.startswith("ok ")
    # the ctypes mirror of the argument struct has the C layout's size
    import ctypes
    assert int(r.stdout.split()[-1]) == ctypes.sizeof(_lib.HtrcFlatArgs)
