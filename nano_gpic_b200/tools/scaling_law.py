"""Scaling-law fit of held-out loss against model and data size (reference tools/fit/scaling_law.py:1-128).

    L(N, D) = E + (A / N^alpha + B / D^beta)^k

N = image parameters (18 x image layers x width^2), D = image tokens seen (256 per image), C = 6 N D. The fit is a
weighted least-squares on the relative error, in the variables x = ln(N/1e8), y = ln(D/1e10):
    L = E + exp(c + k * logaddexp(-alpha x, r - beta y))      (c = k ln A', r = ln(B'/A') in scaled units)
from several random starts within bounds, the best kept. Run weights: exp(-d^2 / (2 * 0.4^2)) * sqrt(C / C0), d = ln N
minus the vertex of a quadratic fit of L in ln N over the runs of the same budget (runs far from their budget's
minimum count less); --equal-weights gives every run weight 1. Compute-optimal size for a budget C:
    N* = G (C/6)^(beta/(alpha+beta)),  D* = C / (6 N*),  G = (alpha A / (beta B))^(1/(alpha+beta)).

    python -m nano_gpic_b200.tools.scaling_law [--csv runs.csv] [--boot 200] [--equal-weights]
The CSV has columns flops, image_params, image_tokens, heldout_loss (the reference's final_ladder_runs.csv, read from
the reference tree by default).
"""
import argparse
import csv
import math
import os

import numpy as np

C0 = 3.567e18  # the smallest ladder budget; budgets are C0 * 2^j
# name, lower, upper, range of random starts
PARAMS = [("E", 0.0, 0.0645, (0.055, 0.064)), ("c", -25.0, 5.0, (-9.0, -3.0)), ("alpha", 0.005, 3.0, (0.05, 1.5)),
          ("beta", 0.005, 3.0, (0.05, 1.5)), ("r", -15.0, 15.0, (-3.0, 3.0)), ("k", 0.005, 3.0, (0.05, 1.2))]


def model(th, x, y):
    E, c, a, b, r, k = th
    return E + np.exp(c + k * np.logaddexp(-a * x, r - b * y))


def fit(x, y, L, w, starts=48, seed=1, init=()):
    from scipy.optimize import least_squares
    lo = np.array([p[1] for p in PARAMS])
    hi = np.array([p[2] for p in PARAMS])
    rng = np.random.default_rng(seed)
    cand = list(init) + [np.array([rng.uniform(*p[3]) for p in PARAMS]) for _ in range(starts)]
    sw = np.sqrt(w)
    best, best_cost = None, np.inf
    for th0 in cand:
        th0 = np.clip(th0, lo + 1e-9 * (hi - lo), hi - 1e-9 * (hi - lo))
        try:
            with np.errstate(all="ignore"):
                res = least_squares(lambda th: sw * (model(th, x, y) / L - 1.0), th0, bounds=(lo, hi), method="trf",
                                    x_scale="jac", max_nfev=4000, ftol=1e-12, xtol=1e-12, gtol=1e-12)
        except (ValueError, FloatingPointError):
            continue
        cost = float(np.sum(res.fun ** 2))
        if np.isfinite(cost) and cost < best_cost:
            best, best_cost = res.x, cost
    return best


def budget_vertex_distance(N, L, C):
    j = np.round(np.log2(C / C0)).astype(int)
    d = np.zeros(len(N))
    for b in np.unique(j):
        i = j == b
        if i.sum() < 3:
            continue
        q2, q1, _ = np.polyfit(np.log(N[i]), L[i], 2)
        d[i] = np.log(N[i]) + q1 / (2 * q2)
    return d


def constants(th):
    """(E, A, B, alpha, beta, k) in unscaled units."""
    E, c, a, b, r, k = th
    K = math.exp(c / k)
    return {"E": E, "A": K * 1e8 ** a, "B": K * math.exp(r) * 1e10 ** b, "alpha": a, "beta": b, "k": k}


def optimum(p, C):
    G = (p["alpha"] * p["A"] / (p["beta"] * p["B"])) ** (1.0 / (p["alpha"] + p["beta"]))
    N = G * (C / 6.0) ** (p["beta"] / (p["alpha"] + p["beta"]))
    return N, C / (6.0 * N)


def loss_at(p, N, D):
    return p["E"] + (p["A"] / N ** p["alpha"] + p["B"] / D ** p["beta"]) ** p["k"]


def load(path):
    with open(path) as f:
        rows = list(csv.DictReader(f))
    col = lambda k: np.array([float(r[k]) for r in rows])
    return rows, col("image_params"), col("image_tokens"), col("heldout_loss"), col("flops")


def run(N, D, L, C, equal_weights=False, boot=0):
    x, y = np.log(N / 1e8), np.log(D / 1e10)
    d = budget_vertex_distance(N, L, C)
    w = np.ones(len(N)) if equal_weights else np.exp(-d ** 2 / (2 * 0.4 ** 2)) * np.sqrt(C / C0)
    th = fit(x, y, L, w)
    p = constants(th)
    err = model(th, x, y) / L - 1
    out = {"params": p, "rms_rel_err": float(np.sqrt(np.mean(err ** 2))), "max_rel_err": float(np.max(np.abs(err))),
           "N_exponent": p["beta"] / (p["alpha"] + p["beta"])}
    if boot:
        rng = np.random.default_rng(7)
        ex = []
        for _ in range(boot):
            i = rng.choice(len(N), len(N))
            tb = fit(x[i], y[i], L[i], w[i], starts=4, seed=int(rng.integers(1 << 30)), init=[th])
            pb = constants(tb)
            ex.append(pb["beta"] / (pb["alpha"] + pb["beta"]))
        out["N_exponent_90"] = [float(v) for v in np.percentile(ex, [5, 95])]
    return out


def default_csv():
    here = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    return os.path.join(here, "baseline", "_ref", "tools", "fit", "final_ladder_runs.csv")


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--csv", default=default_csv())
    ap.add_argument("--boot", type=int, default=0)
    ap.add_argument("--equal-weights", action="store_true")
    a = ap.parse_args(argv)
    rows, N, D, L, C = load(a.csv)
    res = run(N, D, L, C, a.equal_weights, a.boot)
    p = res["params"]
    print(f"{len(rows)} runs; L = E + (A/N^alpha + B/D^beta)^k")
    print("  " + ", ".join(f"{k} {v:.4g}" for k, v in p.items()))
    print(f"  relative loss error: RMS {100 * res['rms_rel_err']:.3f}%, largest {100 * res['max_rel_err']:.3f}%;"
          f" N* ~ C^{res['N_exponent']:.3f}")
    for Cb in [C0 * 2 ** j for j in range(7)] + [1e21]:
        n, dd = optimum(p, Cb)
        mlr = 1.36e-2 * (Cb / C0) ** -0.5
        print(f"  C {Cb:.3g}: N* {n / 1e6:8.0f}M  D* {dd / 1e9:8.1f}B  D/N {dd / n:6.1f}  L {loss_at(p, n, dd):.5f}"
              f"  Muon lr {mlr:.2e}  Muon wd {5 / (mlr * dd / (1024 * 256)):.4f}")
    if "N_exponent_90" in res:
        print(f"  bootstrap N* exponent 90% interval {res['N_exponent_90']}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
