"""The C ABI from a plain-C host program (gcc, no Python, no GPU): the header compiles as C,
the library links, and version, size queries and argument errors behave as declared."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
LIBDIR = ROOT / "qwen3-tts-rsi-engine_b200" / "qwen3_tts_b200"


@pytest.mark.skipif(shutil.which("gcc") is None or not (LIBDIR / "libq3t_b200.so").exists(),
                    reason="gcc or the built library is missing")
def test_plain_c_host(tmp_path):
    exe = tmp_path / "abi_host_checks"
    build = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", str(ROOT / "include"),
                            str(ROOT / "tests" / "abi" / "abi_host_checks.c"), "-L", str(LIBDIR), "-lq3t_b200",
                            f"-Wl,-rpath,{LIBDIR}", "-o", str(exe)], capture_output=True, text=True)
    assert build.returncode == 0, build.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "FAIL" not in run.stdout and run.stdout.count("ok") >= 12
