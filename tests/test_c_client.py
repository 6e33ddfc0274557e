# SPDX-License-Identifier: MIT
"""CPU: the C-ABI from C. tests/c/abi_client.c includes every public header
as C17 (the reference's language), links libqh200.so the way a maintainer
would, and exercises the host-side entry points (status codes on bad
arguments, layout queries, synthetic data, GGUF write/read, sampler seeding)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(shutil.which(os.environ.get("CC", "gcc")) is None, reason="no C compiler")
def test_c_client_builds_and_runs(qh, tmp_path):
    lib_dir = os.path.dirname(qh.LIB_PATH)
    exe = str(tmp_path / "abi_client")
    cc = os.environ.get("CC", "gcc")
    subprocess.run([cc, "-std=c17", "-Wall", "-Wextra", "-Werror", f"-I{os.path.join(ROOT, 'include')}",
                    os.path.join(ROOT, "tests", "c", "abi_client.c"), f"-L{lib_dir}", "-lqh200",
                    f"-Wl,-rpath,{lib_dir}", "-o", exe], check=True)
    r = subprocess.run([exe, str(tmp_path / "m.gguf")], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == "ok"
