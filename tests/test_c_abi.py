"""The C ABI from plain C: tests/c_abi/abi_smoke.c compiled with the system C compiler against include/ud.h and
linked to the in-tree libud.so (no Python or PyTorch in the program). Without a device the program checks the
defaults, status strings and argument validation and reports the missing device as UD_ERR_CUDA; on a B200 it
also brings an engine up, opens and closes a stream, and shuts it down."""

import shutil
import subprocess
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
LIBDIR = ROOT / "universal-dictator_b200"


def _build(tmp_path) -> Path:
    cc = shutil.which("cc") or shutil.which("gcc")
    if cc is None:
        pytest.skip("no C compiler")
    exe = tmp_path / "abi_smoke"
    subprocess.run([cc, "-std=c99", "-Wall", "-Werror", "-I", str(ROOT / "include"),
                    str(ROOT / "tests" / "c_abi" / "abi_smoke.c"), "-L", str(LIBDIR), "-lud",
                    f"-Wl,-rpath,{LIBDIR}", "-o", str(exe)], check=True, capture_output=True, text=True)
    return exe


def test_c_program_without_a_device(tmp_path):
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    r = subprocess.run([str(_build(tmp_path))], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.startswith("no engine: CUDA error")


@pytest.mark.gpu
def test_c_program_on_a_device(tmp_path):
    r = subprocess.run([str(_build(tmp_path))], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.strip() == "engine ok"
