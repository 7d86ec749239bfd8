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
split; 7 - variant 5 as a persistent kernel (one CTA per SM running a
static list of 256-row blocks: every mbarrier keeps counting across them)."""

import os
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.gpu
@pytest.mark.parametrize("variant", ["0", "1", "2", "3", "4", "6", "7"])  # 5 is the default
def test_forward_variant_passes_the_forward_parity_suite(variant):
    env = dict(os.environ, HCP_FWD_VARIANT=variant)
    cmd = [sys.executable, "-m", "pytest", os.path.join(HERE, "test_fwd_gpu.py"), "-q", "-x", "-m", "gpu",
           "-k", "not cfg3", "-p", "no:cacheprovider"]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600, cwd=os.path.dirname(HERE))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert " passed" in r.stdout and "failed" not in r.stdout


@pytest.mark.gpu
def test_persistent_variant_matches_the_default_on_many_blocks_per_cta(tmp_path):
    """Variant 7 runs many 256-row blocks per CTA (every mbarrier keeps
    counting across them), which the small parity cases above do not reach:
    its outputs on launches of 448 to 14336 blocks x heads
    (``fwd_variant_outputs.py``) must equal the default variant's to within
    one bf16 step (the per-block arithmetic is the same, so they are expected
    to be bit-identical), and its LSE to 1e-5."""
    import torch

    paths = {}
    for variant in ("5", "7"):
        paths[variant] = str(tmp_path / f"v{variant}.pt")
        env = dict(os.environ, HCP_FWD_VARIANT=variant)
        r = subprocess.run([sys.executable, os.path.join(HERE, "fwd_variant_outputs.py"), paths[variant]], env=env,
                           capture_output=True, text=True, timeout=600, cwd=os.path.dirname(HERE))
        assert r.returncode == 0, f"variant {variant}: " + r.stdout[-2000:] + r.stderr[-3000:]
    want, got = torch.load(paths["5"]), torch.load(paths["7"])
    assert sorted(want) == sorted(got)
    for name in want:
        (wo, wl), (go, gl) = want[name], got[name]
        wo, go = wo.float(), go.float()
        step = torch.exp2(torch.floor(torch.log2(wo.abs().clamp_min(2.0 ** -14))) - 7)
        bad = (go - wo).abs() > step * 1.0001
        same = float((go == wo).float().mean())
        assert not bool(bad.any()), f"{name}: {int(bad.sum())} elements beyond one bf16 step of the default"
        assert float((gl - wl).abs().max()) <= 1e-5, f"{name}: lse differs from the default"
        print(f"{name}: {same:.6f} of the output elements bit-identical to the default")
