"""Seeded synthetic MX data (numpy PCG64), shared by the tests and the
benchmark so every arm sees identical bytes.

Weights: int8 uniform in [-127, 127] or int4 uniform in [-8, 7] (packed two
per byte, element 2i in the low nibble), E8M0 block exponents uniform in
[emin, emax].  Activations: fp32 N(0, 1).
"""
import numpy as np


def rng(seed):
    return np.random.Generator(np.random.PCG64(seed))


def pack_int4(vals):
    """int8 array [..., K] with values in [-8, 7] -> uint8 [..., K/2]."""
    v = (vals.astype(np.int16) & 0xF).astype(np.uint8)
    return (v[..., 0::2] | (v[..., 1::2] << 4)).astype(np.uint8)


def unpack_int4(packed):
    lo = (packed & 0xF).astype(np.int8)
    hi = (packed >> 4).astype(np.int8)
    lo = np.where(lo >= 8, lo - 16, lo).astype(np.int8)
    hi = np.where(hi >= 8, hi - 16, hi).astype(np.int8)
    out = np.empty(packed.shape[:-1] + (packed.shape[-1] * 2,), dtype=np.int8)
    out[..., 0::2] = lo
    out[..., 1::2] = hi
    return out


def weights(fmt, n, k, emin, emax, seed):
    """(data, scales): data int8 [n, k] (fmt 8) or uint8 packed [n, k/2]
    (fmt 4); scales uint8 [n, k/32] = exponent + 127."""
    g = rng(seed)
    if fmt == 8:
        data = g.integers(-127, 128, size=(n, k), dtype=np.int8)
    else:
        data = pack_int4(g.integers(-8, 8, size=(n, k), dtype=np.int8))
    scales = (g.integers(emin, emax + 1, size=(n, k // 32), dtype=np.int16) + 127).astype(np.uint8)
    return data, scales


def normal(shape, seed):
    return rng(seed).standard_normal(size=shape, dtype=np.float32)


def block_mask(n, k, density, seed, block=64):
    """uint8 [ceil(n/64)][k/64]: each 64x64 block present with probability
    `density` (uniform-random mask, as the block-sparse MoE layer uses)."""
    g = rng(seed)
    return (g.random(((n + block - 1) // block, k // block)) < density).astype(np.uint8)


def apply_block_mask(fmt, data, mask, block=64):
    """Copy of `data` ([n][k] int8, or [n][k/2] packed int4) with every
    masked-out 64x64 block set to zero weights."""
    out = data.copy()
    nb, kb = mask.shape
    per = block // 2 if fmt == 4 else block   # bytes of one block row
    for br in range(nb):
        for bc in range(kb):
            if not mask[br, bc]:
                out[br * block:(br + 1) * block, bc * per:(bc + 1) * per] = 0
    return out
