"""Every GEMV shape through each tensor-core kernel.

By default the library sends gate/up pairs and launches of at least 48 MB of
weights to the N = 256 kernel (weights as the wide MMA operand) and the rest
to the M = 128 kernel.  These tests rerun the GEMV, LM-head, MLP and engine
parity suites in a child process with the choice forced one way:
QWEN_TCW_MIN_MB=0 (every eligible launch on the N = 256 kernel, K-split and
small segments included) and QWEN_GEMV_PATH=tc128 (every launch, pairs and
the LM head included, on the M = 128 kernel).
"""

import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
SUITES = ["test_gemv_gpu.py", "test_lm_head_gpu.py", "test_mlp_norm_gpu.py", "test_engine_gpu.py"]


@pytest.mark.parametrize("env", [{"QWEN_TCW_MIN_MB": "0"}, {"QWEN_GEMV_PATH": "tc128"}],
                         ids=["all_wide", "all_m128"])
def test_suites_with_forced_gemv_kernel(env):
    full_env = dict(os.environ, **env)
    cmd = [sys.executable, "-m", "pytest", "-x", "-q", "-m", "gpu", "-p", "no:cacheprovider"] + \
          [os.path.join(HERE, s) for s in SUITES]
    r = subprocess.run(cmd, cwd=os.path.dirname(HERE), env=full_env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
