"""TEST INFRASTRUCTURE ONLY: numpy f32 restatement of the reference's DDIM
scheduler (src/scheduler.rs:19-98,155-169) and DPM-Solver++(2M)
(src/scheduler.rs:100-152), pinned on its test values (src/scheduler.rs:181-255)."""
from __future__ import annotations

import math

import numpy as np

TRAIN_STEPS = 1000
BETA_START = 0.00085
BETA_END = 0.012
f32 = np.float32


def alphas_cumprod():
    """linspace(√β0, √β1, 1000, f32)² → cumprod(1 − β), torch's two-ended CPU linspace."""
    start, end = f32(np.sqrt(BETA_START)), f32(np.sqrt(BETA_END))
    n = TRAIN_STEPS
    step = (end - start) / f32(n - 1)
    out = np.empty(n, np.float32)
    acc = f32(1.0)
    for i in range(n):
        s = start + step * f32(i) if i < n // 2 else end - step * f32(n - 1 - i)
        acc = f32(acc * (f32(1.0) - s * s))
        out[i] = acc
    return out


class Ddim:
    def __init__(self, steps: int, strength: float, trailing: bool = False):
        assert 1 <= steps <= TRAIN_STEPS
        self.ac = alphas_cumprod()
        self.step_ratio = TRAIN_STEPS // steps
        if trailing:
            r = TRAIN_STEPS / steps
            allt = [int(round(TRAIN_STEPS - i * r)) - 1 for i in range(steps)]
        else:
            allt = [i * self.step_ratio for i in reversed(range(steps))]
        init = min(int(steps * strength), steps)
        self.timesteps = allt[steps - init:]
        self.pure_noise_start = strength >= 1.0

    def add_noise(self, x0, noise, t):
        a = self.ac[t]
        sa, sb = f32(np.sqrt(a)), f32(np.sqrt(f32(1.0) - a))
        return (sa * np.asarray(x0, np.float32) + sb * np.asarray(noise, np.float32)).astype(np.float32)

    def step(self, eps, t, sample):
        a_t = self.ac[t]
        a_prev = self.ac[t - self.step_ratio] if t >= self.step_ratio else f32(1.0)
        sqrt_b_t, sqrt_a_t = f32(np.sqrt(f32(1.0) - a_t)), f32(np.sqrt(a_t))
        sqrt_a_prev, sqrt_b_prev = f32(np.sqrt(a_prev)), f32(np.sqrt(f32(1.0) - a_prev))
        eps = np.asarray(eps, np.float32)
        x0 = (np.asarray(sample, np.float32) - sqrt_b_t * eps) / sqrt_a_t
        return (sqrt_a_prev * x0 + sqrt_b_prev * eps).astype(np.float32)


def dpm_coefficients(ddim: Ddim, t: int):
    """alpha_t, sigma_t, lambda_t = ln(alpha_t / sigma_t) in f64 (src/scheduler.rs:100-105)."""
    a = float(ddim.ac[t])
    alpha, sigma = math.sqrt(a), math.sqrt(1.0 - a)
    return alpha, sigma, math.log(alpha) - math.log(sigma)


class Dpm2M:
    """DPM-Solver++(2M) (src/scheduler.rs:107-152): first order on the first step and after
    restart(), second order after that, and the last step lands on the data prediction."""

    def __init__(self):
        self.prev = None

    def restart(self):
        self.prev = None

    def step(self, ddim: Ddim, eps, i: int, sample):
        steps = ddim.timesteps
        alpha, sigma, lam = dpm_coefficients(ddim, steps[i])
        inv_alpha, sigma_f = f32(1.0 / alpha), f32(sigma)
        x = np.asarray(sample, np.float32)
        x0 = ((x - sigma_f * np.asarray(eps, np.float32)) * inv_alpha).astype(np.float32)
        if i + 1 >= len(steps):
            return x0
        alpha_n, sigma_n, lam_n = dpm_coefficients(ddim, steps[i + 1])
        h = lam_n - lam
        keep = f32(sigma_n / sigma)
        phi = alpha_n * (1.0 - math.exp(-h))
        if self.prev is None:
            out = keep * x + f32(phi) * x0
        else:
            x0_prev, lam_prev = self.prev
            r = (lam - lam_prev) / h
            c0, c1 = f32(phi * (1.0 + 0.5 / r)), f32(phi * 0.5 / r)
            out = keep * x + c0 * x0 - c1 * x0_prev
        self.prev = (x0, lam)
        return out.astype(np.float32)
