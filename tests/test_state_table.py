"""Host version registry (csrc/state_table.h): directed and randomised checks
of the StateId contract the reference's native/state_table.h:11-38 defines,
compiled with the host C++ compiler (no GPU)."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(shutil.which("g++") is None, reason="no host C++ compiler")
def test_state_registry_model_check(tmp_path):
    exe = tmp_path / "state_table_check"
    subprocess.run(["g++", "-std=c++17", "-O1", "-fsanitize=address,undefined", "-o", str(exe),
                    str(ROOT / "tests" / "state_table_check.cpp")], check=True)
    for seed in (1, 2, 3):
        out = subprocess.run([str(exe), str(seed)], check=True, capture_output=True, text=True).stdout
        assert out.startswith("PASS"), out
