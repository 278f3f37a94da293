"""Fits the cubic used by the attention kernels to evaluate 2^f on FMA units.

Method: Cody-Waite style range reduction x = n + f with n = rint(x) and
f in [-1/2, 1/2], so 2^x = 2^n * 2^f; 2^n is applied by adding n to the
float exponent field and 2^f is approximated by a degree-3 polynomial. The
polynomial is the minimax fit in *relative* error, computed here with the
Remez exchange algorithm starting from Chebyshev extrema.

    python miowtion_b200/csrc/fit_exp2_poly.py

prints the coefficients (as float32 hex literals for csrc/exp2_poly.cuh) and
the max relative error of the float32 Horner evaluation.
"""

from __future__ import annotations

import numpy as np

DEGREE = 3
LO, HI = -0.5, 0.5


def remez(degree: int = DEGREE, iters: int = 60) -> np.ndarray:
    """Minimax p(f) = c0 + c1 f + ... + cd f^d for 2^f in relative error."""
    # Unknowns c0..cd and the levelled error E: d + 2 unknowns and nodes.
    m = degree + 2
    k = np.arange(m)
    nodes = np.sort(0.5 * (LO + HI)
                    + 0.5 * (HI - LO) * np.cos(np.pi * k / (m - 1)))
    grid = np.linspace(LO, HI, 400001)
    coef = None
    for _ in range(iters):
        # (sum c_i x^i - 2^x) / 2^x = (-1)^j E  at every node
        a = np.zeros((m, m))
        b = np.zeros(m)
        for j, x in enumerate(nodes):
            t = 2.0 ** x
            a[j, :degree + 1] = [x ** i / t for i in range(degree + 1)]
            a[j, degree + 1] = -((-1) ** j)
            b[j] = 1.0
        sol = np.linalg.solve(a, b)
        coef = sol[:degree + 1]
        err = np.polyval(coef[::-1], grid) / 2.0 ** grid - 1.0
        # new nodes: the extremum of |err| inside each run of equal sign
        sign = np.sign(err)
        cuts = np.nonzero(np.diff(sign))[0]
        bounds = np.concatenate([[0], cuts + 1, [grid.size]])
        ext = np.array([lo + np.argmax(np.abs(err[lo:hi]))
                        for lo, hi in zip(bounds[:-1], bounds[1:])
                        if hi > lo])
        while ext.size > m:
            mags = np.abs(err[ext])
            ext = np.delete(ext, 0 if mags[0] < mags[-1] else ext.size - 1)
        if ext.size < m:
            break
        nodes = grid[ext]
    return coef


def f32_horner(coef: np.ndarray, f: np.ndarray) -> np.ndarray:
    c = coef.astype(np.float32)
    f = f.astype(np.float32)
    acc = np.full_like(f, c[-1])
    for ci in c[-2::-1]:
        acc = (acc * f + ci).astype(np.float32)
    return acc


# Lower clamp of the argument in exp2_poly.cuh (masked keys give ~0).
CLAMP = -125.0


def exp2_emulated(x: np.ndarray, coef: np.ndarray) -> np.ndarray:
    """The kernel's evaluation, in float32: clamp, round, poly, exponent."""
    x = np.maximum(x.astype(np.float32), np.float32(CLAMP))
    n = np.rint(x).astype(np.float32)
    f = (x - n).astype(np.float32)
    p = f32_horner(coef, f)
    bits = p.view(np.int32) + (n.astype(np.int32) << 23)
    return bits.view(np.float32)


def main() -> None:
    coef = remez()
    grid = np.linspace(-0.5, 0.5, 1 << 20)
    rel = np.abs(f32_horner(coef, grid) / 2.0 ** grid - 1.0).max()
    x = np.linspace(-100.0, 8.0, 1 << 22).astype(np.float32)
    full = np.abs(exp2_emulated(x, coef) / 2.0 ** x.astype(np.float64) - 1)
    print('coefficients c0..c3:', [float(np.float32(c)) for c in coef])
    print('hex:', [hex(np.float32(c).view(np.uint32)) for c in coef])
    print(f'max relative error on [-1/2, 1/2]: {rel:.3e}; '
          f'on [-100, 8]: {full.max():.3e}')


if __name__ == '__main__':
    main()
