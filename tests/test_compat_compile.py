"""CPU: the reference engine's own call sites compile unchanged against the
C ABI through include/smoe_cuda_compat.h.

The reference's src/ tree is mirrored into a temporary directory of
symbolic links, except compute/metal_bridge.h, which becomes a one-line file
including smoe_cuda_compat.h; then g++ checks decode.cpp, prefill.cpp,
main.cpp and scout/scout.cpp (the files that call smoe_metal_*) with
-fsyntax-only. Two force-included standard headers stand in for what Apple's
libc++ pulls in transitively (common.hpp uses posix_memalign, free and
std::sqrt without including <cstdlib>/<cmath>); nothing of the reference is
edited. The reference tree is found through SMOE_REFERENCE_SRC or next to
this repository (../reference/src); the test skips when it is absent.
engine.cpp is not checked: it includes <mach/mach.h> (macOS only) and makes
no smoe_metal_* call."""
import os
import shutil
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def reference_src():
    p = os.environ.get("SMOE_REFERENCE_SRC") or os.path.join(os.path.dirname(ROOT), "reference", "src")
    return p if os.path.isfile(os.path.join(p, "compute", "metal_bridge.h")) else None


@pytest.mark.parametrize("unit", ["decode.cpp", "prefill.cpp", "main.cpp", "scout/scout.cpp"])
def test_reference_call_sites_compile_against_compat_header(unit, tmp_path):
    src = reference_src()
    if src is None:
        pytest.skip("reference source tree not present")
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    for dirpath, _, files in os.walk(src):
        rel = os.path.relpath(dirpath, src)
        os.makedirs(tmp_path / rel, exist_ok=True)
        for f in files:
            if os.path.join(rel, f) == os.path.join("compute", "metal_bridge.h"):
                continue
            os.symlink(os.path.join(dirpath, f), tmp_path / rel / f)
    (tmp_path / "compute" / "metal_bridge.h").write_text('#include "smoe_cuda_compat.h"\n')
    r = subprocess.run(["g++", "-std=c++20", "-fsyntax-only", "-include", "cstdlib", "-include", "cmath",
                        "-I", os.path.join(ROOT, "include"), str(tmp_path / unit)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]


def test_compat_header_is_plain_c():
    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        with open(c, "w") as f:
            f.write('#include "smoe_cuda_compat.h"\nint main(void) { return 0; }\n')
        r = subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-fsyntax-only", "-I",
                            os.path.join(ROOT, "include"), c], capture_output=True, text=True)
        assert r.returncode == 0, r.stderr
