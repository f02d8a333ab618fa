"""The streaming batch-1 kernel (dq_stream.cu) on the plain split / INT4 GEMV.

The plain entry points run the block kernel of dq_gemv.cu unless DQ_STREAM=1
is in the environment when the library first decides (once per process), so
the parity, full-size and determinism tests of test_gpu_parity.py run again
here in a child process with that setting: the streaming kernel then serves
every call it supports (native layout; for the split GEMV also the
column-major mirror) and must meet the same oracle tolerances.
"""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def test_parity_suite_on_the_streaming_kernel():
    env = dict(os.environ, DQ_STREAM="1")
    sel = "split_gemv or int4_gemv or device_error"
    r = subprocess.run([sys.executable, "-m", "pytest", os.path.join(HERE, "test_gpu_parity.py"), "-m", "gpu", "-q",
                        "-x", "-k", sel, "-p", "no:cacheprovider"], env=env, cwd=os.path.dirname(HERE),
                       capture_output=True, text=True, timeout=1200)
    tail = "\n".join((r.stdout + r.stderr).splitlines()[-30:])
    assert r.returncode == 0, tail
    assert " passed" in r.stdout, tail
