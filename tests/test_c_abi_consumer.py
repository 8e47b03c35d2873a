"""The C ABI from a plain C99 program (tests/c_abi/consumer.c), compiled with gcc
against include/mhc_pre.h and linked with the library the way a host program that
called the reference's aclnn pair would link it.  Without a GPU it checks the ABI
version, status strings and shape rejects; on a B200 it also runs a split-K, a
small-batch and a decode shape through mhcPreRun / mhcPreRunPrepared, and each
through mhcPostPreRun (the post step fused with the next MhcPre), and compares them
with the C oracle on the same inputs."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
CUDA = Path("/usr/local/cuda")


def _build(tmp_path: Path) -> Path:
    import mhcpre_review_b200 as mp
    from oracle import ref
    mp.lib()
    ref.build()
    exe = tmp_path / "consumer"
    lib_dirs = [ROOT / "mhcpre_review_b200", ROOT / "oracle", CUDA / "lib64"]
    cmd = ["gcc", "-std=c99", "-O2", "-Wall", "-Werror", "-I", str(ROOT / "include"), "-I", str(ROOT / "oracle"),
           "-I", str(CUDA / "include"), str(ROOT / "tests" / "c_abi" / "consumer.c"), "-o", str(exe)]
    for d in lib_dirs:
        cmd += ["-L", str(d), f"-Wl,-rpath,{d}"]
    cmd += ["-lmhcpre_b200", "-lmhc_oracle", "-lcudart", "-lm"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_c_consumer_without_gpu(tmp_path):
    exe = _build(tmp_path)
    r = subprocess.run([str(exe), "--no-gpu"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "OK (0 failures)" in r.stdout


@pytest.mark.gpu
def test_c_consumer_on_gpu(tmp_path):
    exe = _build(tmp_path)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "path 0" in r.stdout and "path 2" in r.stdout and "path 4" in r.stdout
