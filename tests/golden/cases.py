"""Seeded inputs on which the reference engine is run to pin the oracle.

Each case is chosen to drive one path of the reference dispatcher
(python_interface/frnn_engine.cu:195-250) and keeps every point inside
[0, 1) so the reference's grid drops nothing (insert_points.cu:74-87): a
dropped point would leave stale entries the reference's kernels index with.
"""

import numpy as np

from frnn_cuda import datagen


def _clip(p):
    return np.clip(p, 0.0, np.float32(0.999999)).astype(np.float32)


def cases():
    """Yield (name, points (N, D) float32, K, radius)."""
    u3 = datagen.generate("uniform", 4096, 3, seed=21)
    yield "grid_aos3_d3", u3, 16, datagen.uniform_radius(4096, 3, 16)
    u2 = datagen.generate("uniform", 4096, 2, seed=22)
    yield "grid_nd_d2", u2, 8, datagen.uniform_radius(4096, 2, 10)
    u4 = datagen.generate("uniform", 4096, 4, seed=23)
    yield "grid_nd_d4", u4, 16, datagen.uniform_radius(4096, 4, 16)
    u5 = datagen.generate("uniform", 4096, 5, seed=24)
    yield "grid_nd_d5", u5, 16, datagen.uniform_radius(4096, 5, 16)
    l12 = _clip(datagen.generate("lowrank4", 4096, 12, seed=25))
    yield "firstd_d12", l12, 32, datagen.calibrate_radius(l12, 24, sample=512)
    l16 = _clip(datagen.generate("lowrank6", 4096, 16, seed=26))
    yield "firstd_d16", l16, 64, datagen.calibrate_radius(l16, 48, sample=512)
    m3 = _clip(datagen.generate("mixture", 4096, 3, seed=27))
    yield "grid_aos3_mixture", m3, 32, datagen.calibrate_radius(m3, 24, sample=512)
    yield "bf_fallback_d3", m3, 32, 0.0099
    s128 = datagen.generate("sphere", 2048, 128, seed=28)
    yield "bf_fallback_d128", s128, 128, datagen.calibrate_radius(s128, 64, sample=512)
    yield "bf_fallback_d12", l12[:3000], 16, 0.55
    t3 = datagen.generate("uniform", 300, 3, seed=29)
    yield "bf_small_d3", t3, 8, 0.2
