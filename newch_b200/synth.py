"""Seeded synthetic inputs for the benchmark configurations (no datasets are downloaded).

Each generator is a pure function of (seed, shape), so a workload trace stores the generator spec
instead of the bytes and any machine regenerates the identical array. MNIST-shaped images stand in
for MNIST, N(0,1) images for the MobileNet-style input, uniform token ids for the text corpus.
"""

from __future__ import annotations

import hashlib

import numpy as np

VERSION = 1
_REGISTRY: dict = {}


def _register(arr: np.ndarray, spec: list) -> np.ndarray:
    arr = np.ascontiguousarray(arr)
    _REGISTRY[hashlib.sha256(arr.tobytes()).hexdigest()] = spec
    return arr


def uniform_u8(seed: int, shape) -> np.ndarray:
    """uint8 pixels uniform in [0, 255]."""
    shape = tuple(int(s) for s in shape)
    a = np.random.default_rng(seed).integers(0, 256, size=shape, dtype=np.uint8)
    return _register(a, ["uniform_u8", int(seed), list(shape)])


def uniform_f32(seed: int, shape) -> np.ndarray:
    """float32 uniform in [0, 1)."""
    shape = tuple(int(s) for s in shape)
    a = np.random.default_rng(seed).random(size=shape, dtype=np.float32)
    return _register(a, ["uniform_f32", int(seed), list(shape)])


def normal_f32(seed: int, shape) -> np.ndarray:
    """float32 N(0, 1)."""
    shape = tuple(int(s) for s in shape)
    a = np.random.default_rng(seed).standard_normal(size=shape, dtype=np.float32)
    return _register(a, ["normal_f32", int(seed), list(shape)])


def labels(seed: int, n: int, classes: int) -> np.ndarray:
    """int32 class indices uniform in [0, classes)."""
    a = np.random.default_rng(seed + 7919).integers(0, classes, size=(int(n),), dtype=np.int32)
    return _register(a, ["labels", int(seed), int(n), int(classes)])


def spec_for(data: bytes):
    """The generator spec that produced exactly these bytes, or None."""
    return _REGISTRY.get(hashlib.sha256(data).hexdigest())


def generate(spec) -> np.ndarray:
    kind = spec[0]
    if kind == "uniform_u8":
        return uniform_u8(spec[1], spec[2])
    if kind == "uniform_f32":
        return uniform_f32(spec[1], spec[2])
    if kind == "normal_f32":
        return normal_f32(spec[1], spec[2])
    if kind == "labels":
        return labels(spec[1], spec[2], spec[3])
    raise ValueError(f"unknown synthetic generator {kind!r}")


def with_seed_offset(spec, offset: int):
    """Same generator and shape, another seed (per-rank data shards)."""
    spec = list(spec)
    spec[1] = int(spec[1]) + int(offset)
    return spec
