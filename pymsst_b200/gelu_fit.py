"""Coefficients of the normal-CDF approximation used by the 16-bit GELU kernels (csrc/gelu.cuh).

The kernels evaluate Phi(x) = 1 / (1 + 2^(-x * H(x^2 / C^2))) for |x| <= C = 5.5 with H a degree-9
polynomial, and saturate Phi to 0 / 1 beyond C (where fp32 erf has already rounded to -1 / 1).  H is
fitted here to the base-2 logit of the normal CDF divided by x, log2(Phi / (1 - Phi)) / x, by weighted
least squares on Chebyshev nodes of [0, C] with the weights raised at the worst points a few times
(Lawson's iteration toward the minimax fit).  The weight x makes the fitted quantity the exponent
x * H itself, so the relative error of min(Phi, 1 - Phi) -- and with it the relative error of
x * Phi(x) on both sides of zero -- is uniform.  The logistic form keeps the saturation out of the
polynomial, which is why a low degree suffices.

``python -m pymsst_b200.gelu_fit`` prints the coefficients (as C float literals) and the result of an
fp32 emulation of the kernel arithmetic over every finite bf16 and fp16 input, compared with the exact
GELU (float64) rounded to the same type.  Needs scipy; the library itself does not import this module.
"""
from __future__ import annotations

import numpy as np

C = 5.5
DEGREE = 9


def fit(degree: int = DEGREE, nodes: int = 6000, iterations: int = 8) -> np.ndarray:
    from scipy.special import log_ndtr

    k = np.arange(nodes)
    x = C * (0.5 + 0.5 * np.cos(np.pi * (k + 0.5) / nodes))
    x = np.concatenate([x, [1e-6]])
    target = (log_ndtr(x) - log_ndtr(-x)) / np.log(2) / x
    v = np.vander(x * x / (C * C), degree + 1, increasing=True)
    weight = x.copy()
    w = weight.copy()
    coef = None
    for _ in range(iterations):
        coef, *_ = np.linalg.lstsq(v * w[:, None], target * w, rcond=None)
        err = np.abs((v @ coef - target) * weight)
        w = w * (1 + 10 * err / err.max())
    return coef.astype(np.float32)


def phi_fp32(x: np.ndarray, coef: np.ndarray) -> np.ndarray:
    """fp32 emulation of the kernel's Phi (exact exp2 and reciprocal, rounded to fp32)."""
    with np.errstate(over="ignore", invalid="ignore"):
        x = x.astype(np.float32)
        t = (x * x).astype(np.float32)
        s = (t * np.float32(1 / (C * C))).astype(np.float32)
        h = coef[-1]
        for c in coef[-2::-1]:
            h = (h * s + c).astype(np.float32)
        h = np.where(t > np.float32(C * C), np.float32(1e4), h)
        e = np.exp2((-x * h).astype(np.float64)).astype(np.float32)
        return (np.float32(1) / (np.float32(1) + e)).astype(np.float32)


def check(coef: np.ndarray) -> dict:
    import torch
    from scipy.special import ndtr

    out = {}
    for name, dtype in (("bf16", torch.bfloat16), ("fp16", torch.float16)):
        xs = torch.arange(0, 65536, dtype=torch.int32).to(torch.int16).view(dtype).float()
        xs = xs[torch.isfinite(xs)]
        xd = xs.double().numpy()
        exact = np.where(np.abs(xd) > C, np.where(xd > 0, xd, 0.0), xd * ndtr(xd))
        ref = torch.from_numpy(exact).to(torch.float32).to(dtype).float()
        y = torch.from_numpy((xs.numpy() * phi_fp32(xs.numpy(), coef)).astype(np.float32)).to(dtype).float()
        out[name] = (int((y != ref).sum()), xs.numel())
    return out


def main() -> None:
    coef = fit()
    print("static constexpr float kPhiH[%d] = {%s};" % (len(coef), ", ".join("%.9ef" % c for c in coef)))
    for name, (bad, n) in check(coef).items():
        print(f"{name}: {bad} of {n} finite inputs differ from the exact GELU rounded to {name}")


if __name__ == "__main__":
    main()
