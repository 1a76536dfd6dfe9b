"""Seeded synthetic base sets and codebooks with the shapes of the benchmark configurations.

The reference's benchmark configurations point at SIFT1M / Deep1M / GIST1M files that are not
available here; these generators stand in for them with the shapes and value ranges stated for
each configuration (numpy ``default_rng(seed)``):

* ``sift_like``   D=128, Gaussian mixture around centres uniform in [0,255]^D, per-cluster sigma
                  uniform in [10, 40], rounded and clipped to [0, 255] (configs 0, 3, 4).
* ``deep_like``   D=96, anisotropic Gaussian mixture (random orthogonal basis per component,
                  eigenvalues decaying as 1/i), each point L2-normalised (config 1).
* ``gist_like``   D=960, Dirichlet-like centres plus N(0, 0.05^2), clipped to [0, 1] (config 2).

Codebooks: the reference freezes them from its own trainer, which is outside the encode path.
``train_rvq`` is a seeded stand-in: residual k-means (one K-centre k-means per layer on the
residual of the previous layers), run on a subsample.
"""
from __future__ import annotations

import numpy as np


def sift_like(n: int, d: int = 128, seed: int = 0, n_centres: int = 1000, dtype=np.float32,
              start: int = 0) -> np.ndarray:
    """Rows are vectors.  ``start`` skips that many points of the same stream (slices of a larger set)."""
    rng = np.random.default_rng(seed)
    centres = rng.uniform(0.0, 255.0, size=(n_centres, d)).astype(np.float32)
    sigma = rng.uniform(10.0, 40.0, size=n_centres).astype(np.float32)
    out = np.empty((n, d), dtype=dtype)
    chunk = 1 << 18
    # Each chunk of the stream has its own generator so any slice can be produced on its own.
    first = start // chunk
    pos = 0
    c = first
    while pos < n:
        g = np.random.default_rng([seed, 7, c])
        lab = g.integers(0, n_centres, size=chunk)
        pts = centres[lab] + g.standard_normal((chunk, d), dtype=np.float32) * sigma[lab, None]
        pts = np.clip(np.rint(pts), 0.0, 255.0)
        lo = (start - c * chunk) if c == first else 0
        take = min(chunk - lo, n - pos)
        out[pos:pos + take] = pts[lo:lo + take].astype(dtype)
        pos += take
        c += 1
    return out


def deep_like(n: int, d: int = 96, seed: int = 1, n_comp: int = 4096) -> np.ndarray:
    rng = np.random.default_rng(seed)
    means = rng.standard_normal((n_comp, d)).astype(np.float32)
    lam = (1.0 / np.arange(1, d + 1, dtype=np.float32)).astype(np.float32)
    lab = rng.integers(0, n_comp, size=n)
    out = np.empty((n, d), np.float32)
    order = np.argsort(lab, kind="stable")
    bounds = np.searchsorted(lab[order], np.arange(n_comp + 1))
    for c in range(n_comp):
        idx = order[bounds[c]:bounds[c + 1]]
        if idx.size == 0:
            continue
        g = np.random.default_rng([seed, c])
        q, _ = np.linalg.qr(g.standard_normal((d, d)))
        z = g.standard_normal((idx.size, d)).astype(np.float32) * np.sqrt(lam)
        out[idx] = means[c] + z @ q.T.astype(np.float32)
    out /= np.linalg.norm(out, axis=1, keepdims=True)
    return out.astype(np.float32)


def gist_like(n: int, d: int = 960, seed: int = 2, n_centres: int = 2000) -> np.ndarray:
    rng = np.random.default_rng(seed)
    centres = rng.dirichlet(np.full(d, 0.5), size=n_centres).astype(np.float32) * (d / 4.0)
    centres = np.clip(centres, 0.0, 1.0)
    lab = rng.integers(0, n_centres, size=n)
    out = np.empty((n, d), np.float32)
    chunk = 65536
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        out[s:e] = np.clip(centres[lab[s:e]] + rng.standard_normal((e - s, d), dtype=np.float32) * 0.05, 0.0, 1.0)
    return out


def train_rvq(X: np.ndarray, m: int, k: int, iters: int = 8, seed: int = 0, device: str | None = None):
    """Residual k-means codebooks.  Returns a list of m arrays of shape (k, D) (one row per codeword).

    Runs on torch (``device`` = "cuda" when given and available, else CPU) for speed; the result only
    seeds the encoder's inputs, it is not part of the measured path.
    """
    import torch

    dev = torch.device(device if device else "cpu")
    g = torch.Generator(device="cpu").manual_seed(seed)
    R = torch.as_tensor(np.ascontiguousarray(X, np.float32)).to(dev)
    books = []
    for _ in range(m):
        idx = torch.randperm(R.shape[0], generator=g)[:k]
        C = R[idx.to(dev)].clone()
        for _ in range(iters):
            d2 = (C * C).sum(1)[None, :] - 2.0 * (R @ C.T)
            lab = d2.argmin(1)
            # Centroid sums through a one-hot matmul: deterministic on the GPU (no atomics).
            onehot = torch.nn.functional.one_hot(lab, k).to(R.dtype)
            S = onehot.T @ R
            cnt = onehot.sum(0)
            nz = cnt > 0
            C[nz] = S[nz] / cnt[nz, None]
        d2 = (C * C).sum(1)[None, :] - 2.0 * (R @ C.T)
        lab = d2.argmin(1)
        R = R - C[lab]
        books.append(C.cpu().numpy().astype(np.float32))
    return books


def flatten_books(books) -> np.ndarray:
    """C_all as an (H, D) array: row h is flat codeword h (the reference's C_all column h)."""
    return np.ascontiguousarray(np.concatenate(books, axis=0), dtype=np.float32)
