"""TEST INFRASTRUCTURE ONLY (imported by tests/, never by the product path).

fp64 NumPy restatement of the flow-matching multistep UniPC sampler (Zhao et al. 2023, "UniPC",
B(h) = expm1(-h), data prediction, order <= 2 with first-order warm-up and final step, UniC
corrector after every step but the first) and of the Euler flow step, written from the
published algorithm in its general form (the order conditions R rho = b solved with
np.linalg.solve; the order-2 predictor uses the algorithm's fixed rho = 1/2). It checks the
device sampler in coda-wan-dit_b200/sampler.py, which uses closed forms.

Parity unpinned: the reference drives upstream Wan's FlowUniPCMultistepScheduler
(generate_video.py:371-403), which is not vendored in the reference tree, so no golden vectors
of the upstream scheduler exist here.
"""
from __future__ import annotations

import math

import numpy as np


def flow_sigmas(steps: int, shift: float) -> np.ndarray:
    u = (1.0 - 1.0 / 1000.0) * (1.0 - np.arange(steps) / steps)
    s = shift * u / (1.0 + (shift - 1.0) * u)
    return np.concatenate([s, [0.0]])


def _alpha_sigma(s: float):
    return 1.0 - s, s


def _lam(s: float) -> float:
    a, sg = _alpha_sigma(s)
    return math.log(a) - math.log(sg) if sg > 0 else math.inf


def _rb(rks, h, order):
    hh = -h
    h_phi_1 = math.expm1(hh)
    h_phi_k = h_phi_1 / hh - 1.0
    bh = math.expm1(hh)
    fac = 1
    R, b = [], []
    for i in range(1, order + 1):
        R.append(np.power(rks, i - 1))
        b.append(h_phi_k * fac / bh)
        fac *= i + 1
        h_phi_k = h_phi_k / hh - 1.0 / fac
    return np.stack(R), np.array(b), h_phi_1, bh


def unipc_sample(model, x: np.ndarray, steps: int, shift: float = 5.0, order: int = 2) -> np.ndarray:
    """model(x, sigma) -> flow velocity v; returns the sample at sigma = 0."""
    sig = flow_sigmas(steps, shift)
    outs, sigs = [], []
    last_x, last_order = None, 1
    x = x.astype(np.float64)
    for i in range(steps):
        s = float(sig[i])
        m = x - s * model(x, s)
        if i > 0:
            # corrector (UniC) at sigma_i from sigma_{i-1}
            s0, t = sigs[-1], s
            a_t, sg_t = _alpha_sigma(t)
            h = _lam(t) - _lam(s0)
            rks, d1s = [], []
            for k in range(1, last_order):
                rk = (_lam(sigs[-(k + 1)]) - _lam(s0)) / h
                rks.append(rk)
                d1s.append((outs[-(k + 1)] - outs[-1]) / rk)
            rks.append(1.0)
            R, b, hp1, bh = _rb(np.array(rks), h, last_order)
            rhos = np.array([0.5]) if last_order == 1 else np.linalg.solve(R, b)
            xt = sg_t / s0 * last_x - a_t * hp1 * outs[-1]
            corr = sum(rhos[k] * d1s[k] for k in range(len(d1s))) if d1s else 0.0
            x = xt - a_t * bh * (corr + rhos[-1] * (m - outs[-1]))
        outs = (outs + [m])[-order:]
        sigs = (sigs + [s])[-order:]
        this_order = min(order, len(outs), steps - i)
        last_x, last_order = x, this_order
        # predictor (UniP) from sigma_i to sigma_{i+1}
        t = float(sig[i + 1])
        a_t, sg_t = _alpha_sigma(t)
        if t == 0.0:
            x = outs[-1].copy()  # sigma_t = 0: e^{-h} = 0, the step lands on the data prediction
            continue
        h = _lam(t) - _lam(s)
        rks, d1s = [], []
        for k in range(1, this_order):
            rk = (_lam(sigs[-(k + 1)]) - _lam(s)) / h
            rks.append(rk)
            d1s.append((outs[-(k + 1)] - outs[-1]) / rk)
        rks.append(1.0)
        R, b, hp1, bh = _rb(np.array(rks), h, this_order)
        xt = sg_t / s * x - a_t * hp1 * outs[-1]
        if d1s:
            rhos = np.array([0.5]) if this_order == 2 else np.linalg.solve(R[:-1, :-1], b[:-1])
            xt = xt - a_t * bh * sum(rhos[k] * d1s[k] for k in range(len(d1s)))
        x = xt
    return x


def euler_sample(model, x: np.ndarray, steps: int, shift: float = 5.0) -> np.ndarray:
    sig = flow_sigmas(steps, shift)
    x = x.astype(np.float64)
    for i in range(steps):
        x = x + (sig[i + 1] - sig[i]) * model(x, float(sig[i]))
    return x
