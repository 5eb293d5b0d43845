"""Sampling loop around the fused DiT forward (the reference's generation loop,
generate_video.py:371-403, without the text encoder and VAE, which are out of scope).

Per step: one CFG batch-2 forward of `FusedWanModel` (conditional and unconditional entries
share the latent and the timestep, so every block folds its adaLN modulation into its weights
once per step for both), the guidance combine v = v_u + g (v_c - v_u), and a flow-matching
update of the latent:

* ``FlowUniPC``: multistep UniPC, B(h) = expm1(-h) ("bh2"), data prediction, solver order 2
  with a first-order warm-up and a first-order final step, the UniC corrector after every step
  but the first. Published algorithm: Zhao et al., "UniPC: A Unified Predictor-Corrector
  Framework for Fast Sampling of Diffusion Models" (2023); flow matching uses alpha = 1 - sigma,
  lambda = log(alpha / sigma) and x0 = x - sigma v.
* ``FlowEuler``: x <- x + (sigma_next - sigma) v.

The schedule (`flow_sigmas`) is sigma_i = s u_i / (1 + (s - 1) u_i) over u = linspace(0.999,
0, steps + 1)[:-1] with shift s (Wan's timestep shift), then a final sigma of 0; the model's
timestep is 1000 sigma. All scheduler arithmetic runs on the GPU in fp32 on the latent tensor;
the per-step coefficients are host scalars.
"""
from __future__ import annotations

import math

import torch


SIGMA_MAX = 1.0 - 1.0 / 1000.0  # top of a 1000-step training schedule (alpha > 0, finite lambda)


def flow_sigmas(steps: int, shift: float) -> list[float]:
    """steps + 1 decreasing noise levels ending at exactly 0."""
    if steps < 1:
        raise ValueError("steps must be >= 1")
    out = []
    for i in range(steps):
        u = SIGMA_MAX * (1.0 - i / steps)
        out.append(shift * u / (1.0 + (shift - 1.0) * u))
    out.append(0.0)
    return out


class FlowEuler:
    def __init__(self, steps: int, shift: float = 5.0):
        self.sigmas = flow_sigmas(steps, shift)
        self.i = 0

    @property
    def timesteps(self) -> list[float]:
        return [1000.0 * s for s in self.sigmas[:-1]]

    def step(self, v: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
        s, s_next = self.sigmas[self.i], self.sigmas[self.i + 1]
        self.i += 1
        return x + (s_next - s) * v


def _lam(sigma: float) -> float:
    return math.log(1.0 - sigma) - math.log(sigma)


class FlowUniPC:
    """Multistep UniPC (bh2, data prediction, order <= 2) on a flow-matching schedule."""

    def __init__(self, steps: int, shift: float = 5.0, order: int = 2):
        if order not in (1, 2):
            raise ValueError("order 1 or 2")
        self.sigmas = flow_sigmas(steps, shift)
        self.order = order
        self.i = 0
        self.x0s: list[torch.Tensor] = []  # data predictions of the last steps (newest last)
        self.sig_hist: list[float] = []    # their noise levels
        self.last_x: torch.Tensor | None = None
        self.last_order = 1

    @property
    def timesteps(self) -> list[float]:
        return [1000.0 * s for s in self.sigmas[:-1]]

    @staticmethod
    def _coeffs(s0: float, t: float):
        """alpha_t, sigma_t / sigma_s0, h, h_phi_1 = expm1(-h), B(h) for a step s0 -> t."""
        if t <= 0.0:
            # final step to sigma = 0: alpha = 1, the update returns the data prediction blend
            return 1.0, 0.0, math.inf, -1.0, -1.0
        h = _lam(t) - _lam(s0)
        hp1 = math.expm1(-h)
        return 1.0 - t, t / s0, h, hp1, hp1

    def _predict(self, x: torch.Tensor, order: int) -> torch.Tensor:
        s0, t = self.sig_hist[-1], self.sigmas[self.i + 1]
        m0 = self.x0s[-1]
        alpha_t, ratio, h, hp1, bh = self._coeffs(s0, t)
        x_t = ratio * x - alpha_t * hp1 * m0
        if order == 2 and math.isfinite(h):
            s1 = self.sig_hist[-2]
            rk = (_lam(s1) - _lam(s0)) / h
            d1 = (self.x0s[-2] - m0) / rk
            x_t = x_t - alpha_t * bh * 0.5 * d1  # rho = 1/2 for the order-2 predictor
        return x_t

    def _correct(self, x_prev: torch.Tensor, m_t: torch.Tensor, order: int) -> torch.Tensor:
        """UniC: refine the sample at sigma_t using its own data prediction m_t."""
        s0, t = self.sig_hist[-1], self.sigmas[self.i]
        m0 = self.x0s[-1]
        alpha_t, ratio, h, hp1, bh = self._coeffs(s0, t)
        x_t = ratio * x_prev - alpha_t * hp1 * m0
        d1_t = m_t - m0
        if order == 1:
            return x_t - alpha_t * bh * 0.5 * d1_t
        # order 2: solve [[1, 1], [rk, 1]] rho = [b1, b2] with the bh2 right-hand side
        s1 = self.sig_hist[-2]
        rk = (_lam(s1) - _lam(s0)) / h
        hh = -h
        phi = hp1 / hh - 1.0
        b1 = phi / bh
        b2 = (phi / hh - 0.5) * 2.0 / bh
        rho1 = (b2 - b1) / (rk - 1.0)  # coefficient of D1 (previous step's difference)
        rho_t = b1 - rho1              # coefficient of the current difference
        d1 = (self.x0s[-2] - m0) / rk
        return x_t - alpha_t * bh * (rho1 * d1 + rho_t * d1_t)

    def step(self, v: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
        sigma = self.sigmas[self.i]
        m = x - sigma * v  # data prediction
        if self.i > 0 and self.last_x is not None:
            x = self._correct(self.last_x, m, self.last_order)
        self.x0s = (self.x0s + [m])[-2:]
        self.sig_hist = (self.sig_hist + [sigma])[-2:]
        remaining = len(self.sigmas) - 1 - self.i
        order = min(self.order, len(self.x0s), remaining)
        self.last_x = x
        self.last_order = order
        x_next = self._predict(x, order)
        self.i += 1
        return x_next


@torch.no_grad()
def sample(model, noise: list[torch.Tensor], context: list[torch.Tensor], context_null: list[torch.Tensor],
           seq_len: int, steps: int = 50, guide_scale: float = 5.0, shift: float = 5.0, solver: str = "unipc",
           input_dtype: torch.dtype = torch.bfloat16, callback=None) -> list[torch.Tensor]:
    """Denoise `noise` (one latent per prompt) with classifier-free guidance.

    Each step runs one forward over [x_0..x_{n-1}, x_0..x_{n-1}] with the prompt contexts
    followed by the null contexts (one batch of 2n; the shared timestep keeps one weight fold
    per block and step). Returns the final latents (fp32).
    """
    n = len(noise)
    sched = FlowUniPC(steps, shift) if solver == "unipc" else FlowEuler(steps, shift)
    xs = [z.float().clone() for z in noise]
    ctx = list(context) + list(context_null)
    for i, t in enumerate(sched.timesteps):
        inp = [x.to(input_dtype) for x in xs]
        out = model(inp + inp, torch.full((2 * n,), float(t)), ctx, seq_len)
        new = []
        for j in range(n):
            v_c, v_u = out[j], out[n + j]
            v = v_u + guide_scale * (v_c - v_u)
            new.append(v)
        stacked = sched.step(torch.stack(new), torch.stack(xs))
        xs = list(stacked.unbind(0))
        if callback is not None:
            callback(i, t, xs)
    return xs
