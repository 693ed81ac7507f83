"""Integer random streams of the GPU kernels, restated in numpy.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

- pcg_hash / uniform_pm: the reset generator carried inside every reference
  step kernel (cartpole_metal.py:40-51): the PCG hash of Jarzynski & Olano
  (JCGT 2020) of seed ^ (i * 0x9E3779B9) plus a row offset, top 24 bits to a
  float in [-bound, bound). Reset values are therefore bit-exact functions of
  (seed, env index, row) and the oracle reproduces them exactly.
- philox4x32_10 / normal: this build's counter-based ES noise (Philox-4x32-10,
  Salmon et al. SC 2011, then Box-Muller). The integer words are exact; the
  normals agree with the GPU to float32 rounding of log/sqrt/sin/cos.
"""

import numpy as np

M32 = np.uint64(0xFFFFFFFF)
GOLDEN = 0x9E3779B9
ROW_STRIDE = 0x85EBCA6B
CLASSIC_ROW_OFFSETS = (0, 0x85EBCA6B, 0xC2B2AE35, 0x27D4EB2F)  # cartpole_metal.py:90-93


def _u32(x):
    return np.asarray(x, dtype=np.uint64) & M32


def pcg_hash(v):
    """PCG hash of uint32 values (any integer array); returns uint32."""
    v = _u32(v)
    s = (v * np.uint64(747796405) + np.uint64(2891336453)) & M32
    shift = (s >> np.uint64(28)) + np.uint64(4)
    w = (((s >> shift) ^ s) * np.uint64(277803737)) & M32
    return ((w >> np.uint64(22)) ^ w).astype(np.uint32)


def env_hash(seed, index):
    """seed ^ (index * 0x9E3779B9) mod 2^32 for an array of global env indices."""
    idx = _u32(np.asarray(index, dtype=np.int64).astype(np.uint64))
    return (_u32(seed) ^ ((idx * np.uint64(GOLDEN)) & M32)).astype(np.uint32)


def uniform_pm(h, bound):
    """Top 24 bits of a hash to float32 in [-bound, bound): exact up to the final product."""
    t = (np.asarray(h, dtype=np.uint32) >> np.uint32(8)).astype(np.float32) * np.float32(1.0 / 16777216.0)
    t = t * np.float32(2.0) - np.float32(1.0)
    return (t * np.float32(bound)).astype(np.float32)


def reset_rows(seed, n, rows, bound, index_offset=0, offsets=None, center=None):
    """(rows, n) fresh values: row r of env i is uniform_pm(pcg_hash(env_hash + offset_r), bound)
    (+ center[r], one float32 add). offsets default to r * 0x85EBCA6B (pendulum_metal.py:86-90)."""
    h = env_hash(seed, np.arange(n, dtype=np.int64) + index_offset).astype(np.uint64)
    out = np.empty((rows, n), dtype=np.float32)
    for r in range(rows):
        off = offsets[r] if offsets is not None else (r * ROW_STRIDE) & 0xFFFFFFFF
        u = uniform_pm(pcg_hash(h + np.uint64(off)), bound)
        out[r] = u if center is None else (np.float32(center[r]) + u).astype(np.float32)
    return out


# ---- Philox-4x32-10 + Box-Muller -------------------------------------------

_PH_M0, _PH_M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
_PH_W0, _PH_W1 = np.uint64(0x9E3779B9), np.uint64(0xBB67AE85)


def philox4x32_10(c0, c1, c2, c3, k0, k1):
    """Ten Philox rounds on arrays of uint32 counter words; returns four uint32 arrays."""
    c0, c1, c2, c3 = (_u32(c) for c in (c0, c1, c2, c3))
    k0, k1 = _u32(k0), _u32(k1)
    for _ in range(10):
        p0 = _PH_M0 * c0
        p1 = _PH_M1 * c2
        c0, c1, c2, c3 = ((p1 >> np.uint64(32)) ^ c1 ^ k0) & M32, p1 & M32, ((p0 >> np.uint64(32)) ^ c3 ^ k1) & M32, p0 & M32
        k0 = (k0 + _PH_W0) & M32
        k1 = (k1 + _PH_W1) & M32
    return tuple(c.astype(np.uint32) for c in (c0, c1, c2, c3))


def noise(seed, gen, pairs, d):
    """(len(pairs), d) standard normals: element (pair, j) from Philox counter (j // 4, pair,
    gen lo, gen hi), key (seed lo, seed hi ^ pair hi), Box-Muller on word pairs (0, 1) and (2, 3)."""
    pairs = np.asarray(pairs, dtype=np.int64)
    nb = (d + 3) // 4
    blk = np.broadcast_to(np.arange(nb, dtype=np.int64)[None, :], (len(pairs), nb))
    pr = np.broadcast_to(pairs[:, None], blk.shape).astype(np.uint64)
    seed, gen = int(seed), int(gen)
    r = philox4x32_10(blk.astype(np.uint64), pr & M32, gen & 0xFFFFFFFF, (gen >> 32) & 0xFFFFFFFF,
                      seed & 0xFFFFFFFF, ((seed >> 32) & 0xFFFFFFFF) ^ (pr >> np.uint64(32)))
    inv24 = np.float32(1.0 / 16777216.0)
    u1a = ((r[0] >> np.uint32(8)) + np.uint32(1)).astype(np.float32) * inv24
    u2a = (r[1] >> np.uint32(8)).astype(np.float32) * inv24
    u1b = ((r[2] >> np.uint32(8)) + np.uint32(1)).astype(np.float32) * inv24
    u2b = (r[3] >> np.uint32(8)).astype(np.float32) * inv24
    ra = np.sqrt(np.float32(-2.0) * np.log(u1a))
    rb = np.sqrt(np.float32(-2.0) * np.log(u1b))
    # sincospi(2u): angle pi * (2u) evaluated in float64 then rounded, the exact function value
    ang_a, ang_b = np.pi * (2.0 * u2a.astype(np.float64)), np.pi * (2.0 * u2b.astype(np.float64))
    out = np.stack([ra * np.cos(ang_a).astype(np.float32), ra * np.sin(ang_a).astype(np.float32),
                    rb * np.cos(ang_b).astype(np.float32), rb * np.sin(ang_b).astype(np.float32)], axis=-1)
    return out.reshape(len(pairs), nb * 4)[:, :d].astype(np.float32)
