"""The rapier_serve binary (built with the library) refuses bad command lines before touching a GPU."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "rapier_b200", "rapier_serve")


@pytest.mark.parametrize("argv", [[], ["--serve"], ["--synthetic", "tiny"], ["--model", "x.gguf", "--synthetic", "tiny", "--serve"],
                                  ["--synthetic", "huge", "--serve"], ["--synthetic", "tiny", "--bogus"]])
def test_usage_errors(argv):
    if not os.path.exists(EXE):
        pytest.skip("rapier_serve not built")
    r = subprocess.run([EXE, *argv], capture_output=True, text=True, timeout=60)
    assert r.returncode == 2 and "usage:" in r.stderr
