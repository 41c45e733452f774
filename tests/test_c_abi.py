"""The C ABI from C and C++: ``tests/c_abi/abi_smoke.c`` includes only
``include/constellation_b200.h``, links ``libconstellation_b200.so`` and round-trips an
expert-node request through the library's codec and request handler (no GPU needed)."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
LIBDIR = ROOT / "constellation_b200"
SRC = Path(__file__).resolve().parent / "c_abi" / "abi_smoke.c"


@pytest.mark.parametrize("compiler,flags", [("gcc", ["-std=c99", "-x", "c"]), ("g++", ["-std=c++17", "-x", "c++"])])
def test_header_compiles_links_and_runs(tmp_path, compiler, flags):
    if shutil.which(compiler) is None:
        pytest.skip(f"{compiler} not installed")
    if not (LIBDIR / "libconstellation_b200.so").is_file():
        pytest.fail("libconstellation_b200.so is not built")
    exe = tmp_path / "abi_smoke"
    cmd = [compiler, *flags, "-Wall", "-Wextra", "-Werror", "-I", str(ROOT / "include"), str(SRC), "-x", "none",
           "-L", str(LIBDIR), "-lconstellation_b200", f"-Wl,-rpath,{LIBDIR}", "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0 and out.stdout.strip() == "OK", out.stdout + out.stderr
