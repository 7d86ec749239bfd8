"""The forward kernel's named-barrier MMA issuer (``HCP_FWD_NAMED_BARRIERS=1``)
must give the same answers as the default issuer: the whole forward parity
suite (``test_fwd_gpu.py``) runs again in a child process with the switch
set (the library reads it once per process)."""

import os
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.gpu
def test_named_barrier_issuer_passes_the_forward_parity_suite():
    env = dict(os.environ, HCP_FWD_NAMED_BARRIERS="1")
    cmd = [sys.executable, "-m", "pytest", os.path.join(HERE, "test_fwd_gpu.py"), "-q", "-x", "-m", "gpu",
           "-p", "no:cacheprovider"]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600, cwd=os.path.dirname(HERE))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert " passed" in r.stdout and "failed" not in r.stdout
