"""Every variant of the forward kernel besides the default (5) must give the
default's answers: the forward parity suite (``test_fwd_gpu.py``, without
its 131072-token case) runs again in a child process per variant, the
variant chosen by ``HCP_FWD_VARIANT`` (the library reads it once per
process).

0 - mbarrier MMA issuer on 320 threads; 1 - named-barrier MMA issuer; 2 - 1
with a quarter of the exponentials on the FMA pipe; 3, 4 (and the default 5)
- 384 threads with the registers split by setmaxnreg and packed softmax
math, with a quarter, three eighths (none) of the exponentials on the FMA
pipe; 6 - the named-barrier issuer on 384 threads with the setmaxnreg
split."""

import os
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.gpu
@pytest.mark.parametrize("variant", ["0", "1", "2", "3", "4", "6"])  # 5 is the default
def test_forward_variant_passes_the_forward_parity_suite(variant):
    env = dict(os.environ, HCP_FWD_VARIANT=variant)
    cmd = [sys.executable, "-m", "pytest", os.path.join(HERE, "test_fwd_gpu.py"), "-q", "-x", "-m", "gpu",
           "-k", "not cfg3", "-p", "no:cacheprovider"]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600, cwd=os.path.dirname(HERE))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert " passed" in r.stdout and "failed" not in r.stdout
