"""The plain C example (ark_b200/examples/step_from_c.c) runs on the GPU."""
import subprocess

import pytest

from test_abi_cpu import build_c_example

pytestmark = pytest.mark.gpu


def test_plain_c_caller_runs(tmp_path):
    out = subprocess.run([str(build_c_example(tmp_path))], capture_output=True, text=True,
                         timeout=120)
    assert out.returncode == 0, out.stderr
    assert "fused step: opt_step=3 loss_scale=1024" in out.stdout
