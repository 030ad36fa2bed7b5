"""Distribution metrics between generated and reference image features (the metrics of the reference's gpic_eval:
gpic_eval/metrics/fd.py, prdc.py, mmd.py), written from their published definitions:

    frechet_distance   Heusel et al. 2017 (FID's distance between Gaussians):
                       |mu1 - mu2|^2 + Tr(S1 + S2 - 2 (S1 S2)^(1/2)); when the matrix square root is not finite, eps
                       is added to both diagonals (the TTUR reference implementation's fallback); imaginary parts below
                       1e-3 are dropped.
    prdc               Naeem et al. 2020: precision, recall, density, coverage with k-nearest-neighbour balls
                       (radius = distance to the k-th neighbour other than the point itself).
    polynomial_mmd     Binkowski et al. 2018 (KID): unbiased MMD^2 with the kernel (gamma x.y + coef0)^degree,
                       gamma = 1/dim, averaged over random subsets.
Features are float arrays [n, dim]; computations in float64.
"""
import numpy as np


def statistics(feats):
    f = np.asarray(feats, dtype=np.float64)
    return f.mean(0), np.cov(f, rowvar=False)


def frechet_distance(mu1, sigma1, mu2, sigma2, eps=1e-6):
    from scipy import linalg
    mu1, mu2 = np.atleast_1d(mu1).astype(np.float64), np.atleast_1d(mu2).astype(np.float64)
    s1, s2 = np.atleast_2d(sigma1).astype(np.float64), np.atleast_2d(sigma2).astype(np.float64)
    diff = mu1 - mu2
    covmean = linalg.sqrtm(s1 @ s2)
    if not np.isfinite(covmean).all():
        off = np.eye(s1.shape[0]) * eps
        covmean = linalg.sqrtm((s1 + off) @ (s2 + off))
    if np.iscomplexobj(covmean):
        if not np.allclose(np.diagonal(covmean).imag, 0, atol=1e-3):
            raise ValueError(f"imaginary component {np.max(np.abs(covmean.imag))}")
        covmean = covmean.real
    return float(diff @ diff + np.trace(s1) + np.trace(s2) - 2 * np.trace(covmean))


def _pairwise(a, b=None):
    a = np.asarray(a, dtype=np.float64)
    b = a if b is None else np.asarray(b, dtype=np.float64)
    d2 = (a * a).sum(1)[:, None] + (b * b).sum(1)[None, :] - 2 * a @ b.T
    return np.sqrt(np.maximum(d2, 0.0))


def _knn_radii(feats, k):
    d = _pairwise(feats)
    return np.partition(d, k, axis=1)[:, k]  # index 0 is the point itself (distance 0)


def prdc(real, fake, k=5):
    rr = _knn_radii(real, k)
    fr = _knn_radii(fake, k)
    d = _pairwise(real, fake)  # [n_real, n_fake]
    precision = float((d < rr[:, None]).any(axis=0).mean())
    recall = float((d < fr[None, :]).any(axis=1).mean())
    density = float((d < rr[:, None]).sum(axis=0).mean() / k)
    coverage = float((d.min(axis=1) < rr).mean())
    return {"precision": precision, "recall": recall, "density": density, "coverage": coverage}


def _poly_kernel(a, b, degree, gamma, coef0):
    return (gamma * (a @ b.T) + coef0) ** degree


def mmd2_unbiased(x, y, degree=3, gamma=None, coef0=1.0):
    x, y = np.asarray(x, dtype=np.float64), np.asarray(y, dtype=np.float64)
    gamma = 1.0 / x.shape[1] if gamma is None else gamma
    m = x.shape[0]
    kxx = _poly_kernel(x, x, degree, gamma, coef0)
    kyy = _poly_kernel(y, y, degree, gamma, coef0)
    kxy = _poly_kernel(x, y, degree, gamma, coef0)
    sxx = (kxx.sum() - np.trace(kxx)) / (m * (m - 1))
    syy = (kyy.sum() - np.trace(kyy)) / (m * (m - 1))
    return float(sxx + syy - 2 * kxy.mean())


def polynomial_mmd(real, fake, n_subsets=100, subset_size=1000, seed=0, **kw):
    rng = np.random.default_rng(seed)
    m = min(len(real), len(fake), subset_size)
    vals = [mmd2_unbiased(real[rng.choice(len(real), m, replace=False)],
                          fake[rng.choice(len(fake), m, replace=False)], **kw) for _ in range(n_subsets)]
    return float(np.mean(vals)), float(np.std(vals))


def evaluate(fake, real=None, ref_mu=None, ref_sigma=None, k=5, prdc_max=10000, seed=0):
    """All metrics of generated features `fake` against reference features and/or reference statistics."""
    out = {"n": int(len(fake))}
    mu, sigma = statistics(fake)
    if ref_mu is None and real is not None:
        ref_mu, ref_sigma = statistics(real)
    if ref_mu is not None:
        out["fd"] = frechet_distance(mu, sigma, ref_mu, ref_sigma)
    if real is not None:
        rng = np.random.default_rng(seed)
        r = real if len(real) <= prdc_max else real[rng.choice(len(real), prdc_max, replace=False)]
        f = fake if len(fake) <= prdc_max else fake[rng.choice(len(fake), prdc_max, replace=False)]
        out.update(prdc(r, f, k))
        out["mmd"], out["mmd_std"] = polynomial_mmd(real, fake, seed=seed)
    return out
