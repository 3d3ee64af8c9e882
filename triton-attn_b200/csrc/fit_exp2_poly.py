"""Derive the polynomials used by the kernels' FMA-pipe exp2 (``exp2_poly_x2``, degree 3, and
``exp2_poly4_x2``, degree 4, in common.cuh).

Method: Cody-Waite style range reduction x = j + f, j = round(x), f in [-0.5, 0.5], so 2^x = 2^j * 2^f;
2^f is approximated by the polynomial of the given degree that minimises the maximum *relative* error
on [-0.5, 0.5], found with the Remez exchange algorithm. Printed per degree: the coefficients (fp32, with
their bit patterns) and the max relative error of an fp32 Horner evaluation (about 7.5e-5 for degree 3,
below the 4.9e-4 half-ulp of the fp16 P it feeds; 2.7e-6 for degree 4). Run:
python triton-attn_b200/csrc/fit_exp2_poly.py
"""

import numpy as np


def remez_rel(deg: int = 3, a: float = -0.5, b: float = 0.5, iters: int = 30) -> tuple[np.ndarray, float]:
    n = deg + 2
    x = (a + b) / 2 + (b - a) / 2 * np.cos(np.pi * np.arange(n)[::-1] / (n - 1))  # Chebyshev extrema
    grid = np.linspace(a, b, 200001)
    c = np.zeros(deg + 1)
    for _ in range(iters):
        A = np.zeros((n, n))
        for i in range(n):  # p(x_i) + (-1)^i E 2^{x_i} = 2^{x_i}
            A[i, : deg + 1] = x[i] ** np.arange(deg + 1)
            A[i, deg + 1] = (-1) ** i * np.exp2(x[i])
        sol = np.linalg.solve(A, np.exp2(x))
        c = sol[: deg + 1]
        err = np.polyval(c[::-1], grid) / np.exp2(grid) - 1
        ext = [0] + [i for i in range(1, len(grid) - 1) if (err[i] - err[i - 1]) * (err[i + 1] - err[i]) <= 0]
        ext.append(len(grid) - 1)
        alt: list[int] = []
        for i in ext:  # alternating extrema, largest of each sign run
            if not alt or np.sign(err[i]) != np.sign(err[alt[-1]]):
                alt.append(i)
            elif abs(err[i]) > abs(err[alt[-1]]):
                alt[-1] = i
        while len(alt) > n:
            alt.pop(0 if abs(err[alt[0]]) < abs(err[alt[-1]]) else -1)
        if len(alt) != n:
            break
        x = grid[alt]
    return c, float(np.abs(err).max())


def main() -> None:
    for deg in (3, 4):
        c, e = remez_rel(deg)
        c32 = c.astype(np.float32)
        g = np.linspace(-0.5, 0.5, 1000001).astype(np.float32)
        p = np.float32(c32[deg])
        for k in range(deg - 1, -1, -1):
            p = (p * g + c32[k]).astype(np.float32)
        e32 = float(np.abs(p.astype(np.float64) / np.exp2(g.astype(np.float64)) - 1).max())
        print(f"degree {deg}: minimax rel err {e:.3e}; fp32 Horner rel err {e32:.3e}")
        for i, v in enumerate(c32):
            print(f"  c{i} = {float(v)!r}f  // 0x{int(v.view(np.uint32)):08x}")


if __name__ == "__main__":
    main()
