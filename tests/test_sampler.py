"""The flow-matching samplers (coda-wan-dit_b200/sampler.py) against the fp64 oracle
restatement (oracle/sampler_ref.py), on CPU in float64: a nonlinear velocity field exercises
the order-2 predictor and corrector terms (agreement to 1e-10 relative), and a field whose data
prediction is constant must land exactly on it (UniPC's exponential integrator and Euler are
exact there). Parity with upstream Wan's scheduler is unpinned (not vendored in the reference)."""
import numpy as np
import pytest
import torch

from oracle import sampler_ref


def _field(x, sigma):
    return 0.3 * x + 0.2 * np.sin(3.0 * x) - 0.5 * sigma


def _run(sched, x):
    for t in sched.timesteps:
        sigma = t / 1000.0
        v = torch.from_numpy(_field(x.numpy(), sigma))
        x = sched.step(v, x)
    return x


@pytest.mark.parametrize("steps,shift", [(1, 5.0), (2, 5.0), (8, 5.0), (25, 3.0)])
def test_unipc_matches_oracle(pkg, steps, shift):
    x0 = np.random.default_rng(0).standard_normal((3, 4, 5))
    got = _run(pkg.sampler.FlowUniPC(steps, shift), torch.from_numpy(x0.copy())).numpy()
    want = sampler_ref.unipc_sample(_field, x0, steps, shift)
    assert np.linalg.norm(got - want) / np.linalg.norm(want) < 1e-10


def test_euler_matches_oracle(pkg):
    x0 = np.random.default_rng(1).standard_normal((2, 7))
    got = _run(pkg.sampler.FlowEuler(10, 5.0), torch.from_numpy(x0.copy())).numpy()
    want = sampler_ref.euler_sample(_field, x0, 10, 5.0)
    assert np.allclose(got, want, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("solver", ["unipc", "euler"])
def test_exact_for_a_constant_data_prediction(pkg, solver):
    rng = np.random.default_rng(2)
    target = rng.standard_normal((4, 6))
    x = torch.from_numpy(rng.standard_normal((4, 6)))
    sched = pkg.sampler.FlowUniPC(12, 5.0) if solver == "unipc" else pkg.sampler.FlowEuler(12, 5.0)
    for t in sched.timesteps:
        sigma = t / 1000.0
        v = (x - torch.from_numpy(target)) / sigma  # x0 = x - sigma v = target at every step
        x = sched.step(v, x)
    assert np.allclose(x.numpy(), target, rtol=0, atol=1e-10)


def test_schedule(pkg):
    s = pkg.sampler.flow_sigmas(50, 5.0)
    assert len(s) == 51 and 0.999 < s[0] < 1.0 and s[-1] == 0.0
    assert all(a > b for a, b in zip(s, s[1:]))
    assert np.allclose(s, sampler_ref.flow_sigmas(50, 5.0), rtol=0, atol=1e-15)
