"""Seeded synthetic inputs with the shapes of the SemanticLogKV flush-and-attend workloads.

No dataset is read: keys come from an isotropic Gaussian mixture around
per-group centres (the reference's own benchmark harnesses use the same kind
of clustered synthetic keys), with a fraction of orphan tokens at a fixed
distance from every centre and planted outlier spans.  Everything is numpy
and deterministic for a given seed, so tests, the golden-fixture generator and
the benchmark all see identical inputs.
"""
from __future__ import annotations

import numpy as np


def rope_tables(length: int, n_elem: int, base: float = 10000.0):
    """cos/sin tables of shape [length, n_elem] in the rotate-half convention.

    Frequencies are ``base ** (-2i / n_elem)`` for ``i < n_elem // 2`` repeated
    twice along the feature axis, evaluated in float32.
    """
    inv = (1.0 / (base ** (np.arange(0, n_elem, 2, dtype=np.float32) / np.float32(n_elem)))).astype(np.float32)
    ang = (np.arange(length, dtype=np.float32)[:, None] * inv[None, :]).astype(np.float32)
    ang = np.concatenate([ang, ang], axis=1)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def apply_rope(x: np.ndarray, pos: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Rotate-half RoPE of ``x[..., T, D]`` at integer positions ``pos[..., T]`` (float32)."""
    half = x.shape[-1] // 2
    c = cos[pos]
    s = sin[pos]
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    return (x * c + rot * s).astype(np.float32)


class MixtureKeys:
    """Pre-RoPE keys drawn around ``clusters`` centres per KV group."""

    def __init__(self, rng: np.random.Generator, groups: int, dim: int, clusters: int,
                 sigma: float = 0.3, orphan_frac: float = 0.05, centre_scale: float = 1.0):
        self.rng = rng
        self.groups, self.dim, self.clusters = groups, dim, clusters
        self.sigma, self.orphan_frac = sigma, orphan_frac
        self.centres = (rng.standard_normal((groups, clusters, dim)) * centre_scale).astype(np.float32)

    def draw(self, batch: int, tokens: int) -> np.ndarray:
        rng, G, D = self.rng, self.groups, self.dim
        z = rng.integers(0, self.clusters, size=(batch, G, tokens))
        base = self.centres[np.arange(G)[None, :, None], z]
        noise = rng.standard_normal((batch, G, tokens, D)).astype(np.float32) * self.sigma
        orphan = rng.random((batch, G, tokens)) < self.orphan_frac
        u = rng.standard_normal((batch, G, tokens, D)).astype(np.float32)
        u /= np.linalg.norm(u, axis=-1, keepdims=True)
        far = u * np.float32(4.0 * self.sigma * np.sqrt(D))
        return np.where(orphan[..., None], base + far, base + noise).astype(np.float32)

    def plant_outlier_span(self, keys: np.ndarray, b: int, start: int, length: int, scale: float) -> None:
        """Overwrite one contiguous span (all groups) with a shared far-away direction."""
        u = self.rng.standard_normal((self.groups, self.dim)).astype(np.float32)
        u /= np.linalg.norm(u, axis=-1, keepdims=True)
        keys[b, :, start:start + length] = (u[:, None, :] * np.float32(scale)
                                            + self.rng.standard_normal((self.groups, length, self.dim)).astype(np.float32)
                                            * np.float32(self.sigma))


def boundary_pattern(rng: np.random.Generator, rows: int, tokens: int, kind: str) -> np.ndarray:
    """Span-end flags per row: every 23rd token ('mod23'), every 3rd ('mod3') or random p=0.2."""
    if kind == "mod23":
        row = (np.arange(tokens) % 23) == 22
        return np.broadcast_to(row, (rows, tokens)).copy()
    if kind == "mod3":
        row = (np.arange(tokens) % 3) == 2
        return np.broadcast_to(row, (rows, tokens)).copy()
    return rng.random((rows, tokens)) < 0.2


class StressMixture:
    """Keys of the unified-route stress workload: per (stream, group) a ``components``-centre
    Gaussian mixture (centres ~ N(0, I)) with per-component sigma ~ U[0.1, 0.6] and a fraction of
    orphan tokens placed 4 sigma sqrt(D) from their centre in a random direction."""

    def __init__(self, rng: np.random.Generator, streams: int, groups: int, dim: int, components: int = 48,
                 orphan_frac: float = 0.10):
        self.rng = rng
        self.shape = (streams, groups, dim)
        self.orphan_frac = orphan_frac
        self.centres = rng.standard_normal((streams, groups, components, dim)).astype(np.float32)
        self.sigma = rng.uniform(0.1, 0.6, (streams, groups, components)).astype(np.float32)

    def draw(self, tokens: int) -> np.ndarray:
        rng = self.rng
        S, G, D = self.shape
        z = rng.integers(0, self.centres.shape[2], size=(S, G, tokens))
        si, gi = np.arange(S)[:, None, None], np.arange(G)[None, :, None]
        base = self.centres[si, gi, z]
        sig = self.sigma[si, gi, z][..., None]
        x = base + sig * rng.standard_normal((S, G, tokens, D)).astype(np.float32)
        u = rng.standard_normal((S, G, tokens, D)).astype(np.float32)
        u /= np.linalg.norm(u, axis=-1, keepdims=True)
        far = base + u * (4.0 * sig * np.float32(np.sqrt(D)))
        orphan = rng.random((S, G, tokens)) < self.orphan_frac
        return np.where(orphan[..., None], far, x).astype(np.float32)
