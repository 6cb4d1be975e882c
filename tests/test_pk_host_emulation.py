"""CPU check of the 32-bit-key addressing kernel (sdmchat_b200/csrc/pk_address.cu): its device code compiled as host
C++ (tests/pk_host/make_host.py) and run thread by thread, against a brute-force combine, against its own forced
exact path, and for per-thread ownership of every shared-memory byte it writes (tests/pk_host/check_pk_host.cpp)."""
import os
import shutil
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_pk_fast_kernel_logic_on_host(tmp_path):
    hdr = tmp_path / "pk_host.h"
    subprocess.run([sys.executable, os.path.join(HERE, "pk_host", "make_host.py"), str(hdr)], check=True)
    exe = tmp_path / "check_pk_host"
    subprocess.run(["g++", "-O2", "-std=c++17", f'-DPK_HOST_HEADER="{hdr}"',
                    os.path.join(HERE, "pk_host", "check_pk_host.cpp"), "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
