"""Threefry-2x32 counter PRNG and the normal sampler used by the CP norm estimate.

Oracle (test infrastructure).  The reference seeds its power iteration with
``jax.random.split(jax.random.PRNGKey(seed), batch)`` and
``jax.random.normal(key, (n,), dtype)`` (``src/purin/solvers/chambolle_pock/
kernels.py:54-55``).  Those live in the third-party dependency ``jax`` (pinned
``jax==0.6.2`` in ``.github/constraints/jax-baseline.txt:2``), which is not
vendored.  This module restates the published algorithms:

* Threefry-2x32 with 20 rounds (Salmon, Moraes, Dror, Shaw, "Parallel random
  numbers: as easy as 1, 2, 3", SC'11), key-schedule constant 0x1BD11BDA and
  rotation constants (13,15,26,6 / 17,29,16,24);
* JAX's key derivation with ``jax_threefry_partitionable`` on (the default
  since JAX 0.5): a 64-bit flat counter split into (hi, lo) words, key from
  seed ``s`` = (s >> 32, s & 0xffffffff), split child ``i`` = threefry(key,
  (0, i)), and per-element bits = threefry(key, (0, j)) combined as
  ``(hi << 32) | lo`` for 64-bit draws or ``hi ^ lo`` for 32-bit draws;
* uniform draws built by filling the mantissa of a float in [1, 2), and
  normals as ``sqrt(2) * erfinv(u)`` with ``u`` in (-1, 1).

It is pinned by the Random123 known-answer vectors (tests/test_oracle_prng.py).
"""

from __future__ import annotations

import numpy as np
from scipy.special import erfinv

_ROT0 = (13, 15, 26, 6)
_ROT1 = (17, 29, 16, 24)
_PARITY = np.uint32(0x1BD11BDA)


def _rounds(x0, x1, rotations):
    for r in rotations:
        x0 = x0 + x1
        x1 = (x1 << np.uint32(r)) | (x1 >> np.uint32(32 - r))
        x1 = x0 ^ x1
    return x0, x1


def threefry2x32(k0, k1, c0, c1):
    """Threefry-2x32-20 block function on uint32 arrays (broadcasting)."""
    k0 = np.asarray(k0, dtype=np.uint32)
    k1 = np.asarray(k1, dtype=np.uint32)
    x0 = np.array(c0, dtype=np.uint32, copy=True)
    x1 = np.array(c1, dtype=np.uint32, copy=True)
    x0, x1 = np.broadcast_arrays(x0, x1)
    x0 = x0.copy()
    x1 = x1.copy()
    ks = (k0, k1, k0 ^ k1 ^ _PARITY)
    with np.errstate(over="ignore"):
        x0 = x0 + ks[0]
        x1 = x1 + ks[1]
        x0, x1 = _rounds(x0, x1, _ROT0)
        x0 = x0 + ks[1]
        x1 = x1 + ks[2] + np.uint32(1)
        x0, x1 = _rounds(x0, x1, _ROT1)
        x0 = x0 + ks[2]
        x1 = x1 + ks[0] + np.uint32(2)
        x0, x1 = _rounds(x0, x1, _ROT0)
        x0 = x0 + ks[0]
        x1 = x1 + ks[1] + np.uint32(3)
        x0, x1 = _rounds(x0, x1, _ROT1)
        x0 = x0 + ks[1]
        x1 = x1 + ks[2] + np.uint32(4)
        x0, x1 = _rounds(x0, x1, _ROT0)
        x0 = x0 + ks[2]
        x1 = x1 + ks[0] + np.uint32(5)
    return x0.astype(np.uint32), x1.astype(np.uint32)


def prng_key(seed: int) -> np.ndarray:
    """Key for an integer seed: (seed >> 32, seed & 0xffffffff)."""
    seed = int(seed)
    return np.array([(seed >> 32) & 0xFFFFFFFF, seed & 0xFFFFFFFF], dtype=np.uint32)


def split(key, count: int, offset: int = 0) -> np.ndarray:
    """Child keys ``offset .. offset+count-1`` of ``key`` (fold-like split)."""
    idx = np.arange(offset, offset + count, dtype=np.uint64)
    hi = (idx >> np.uint64(32)).astype(np.uint32)
    lo = (idx & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    b0, b1 = threefry2x32(key[0], key[1], hi, lo)
    return np.stack([b0, b1], axis=-1)


def random_bits(key, n: int, width: int) -> np.ndarray:
    """Per-element random bits of ``width`` (32 or 64) for a flat draw of size n."""
    idx = np.arange(n, dtype=np.uint64)
    hi = (idx >> np.uint64(32)).astype(np.uint32)
    lo = (idx & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    b0, b1 = threefry2x32(key[0], key[1], hi, lo)
    if width == 64:
        return (b0.astype(np.uint64) << np.uint64(32)) | b1.astype(np.uint64)
    if width == 32:
        return b0 ^ b1
    raise ValueError("width must be 32 or 64")


def uniform(key, n: int, dtype, minval, maxval) -> np.ndarray:
    """Uniform draws in [minval, maxval) by mantissa filling, in ``dtype``."""
    dtype = np.dtype(dtype)
    finfo = np.finfo(dtype)
    nbits, nmant = finfo.bits, finfo.nmant
    bits = random_bits(key, n, nbits)
    utype = np.uint64 if nbits == 64 else np.uint32
    one_bits = np.array(1.0, dtype=dtype).view(utype)
    float_bits = (bits.astype(utype) >> utype(nbits - nmant)) | one_bits
    floats = float_bits.view(dtype) - dtype.type(1.0)
    minval = dtype.type(minval)
    maxval = dtype.type(maxval)
    return np.maximum(minval, floats * (maxval - minval) + minval)


def normal(key, n: int, dtype) -> np.ndarray:
    """Standard normal draws ``sqrt(2) * erfinv(u)``, u uniform in (-1, 1)."""
    dtype = np.dtype(dtype)
    lo = np.nextafter(np.array(-1.0, dtype), np.array(0.0, dtype))
    u = uniform(key, n, dtype, lo, 1.0)
    value = erfinv(u.astype(np.float64)).astype(dtype)
    return (dtype.type(np.sqrt(2.0)) * value).astype(dtype)


def _threefry_blocks_original(key, count: np.ndarray):
    """Legacy ``threefry_2x32(key, count)``: halves of the counter as (x0, x1)."""
    count = np.asarray(count, dtype=np.uint32).ravel()
    odd = count.size % 2
    if odd:
        count = np.concatenate([count, np.zeros(1, np.uint32)])
    half = count.size // 2
    y0, y1 = threefry2x32(key[0], key[1], count[:half], count[half:])
    out = np.concatenate([y0, y1])
    return out[:-1] if odd else out


def split_original(key, count: int) -> np.ndarray:
    """Legacy (non-partitionable) split: threefry over iota(2*count)."""
    out = _threefry_blocks_original(key, np.arange(2 * count, dtype=np.uint32))
    return out.reshape(count, 2)


def random_bits_original(key, n: int, width: int) -> np.ndarray:
    """Legacy bit generation: threefry over iota(ceil(width*n/32))."""
    words = (width * n + 31) // 32
    bits = _threefry_blocks_original(key, np.arange(words, dtype=np.uint32))
    if width == 64:
        hi, lo = bits[: words // 2], bits[words // 2 :]
        return (hi.astype(np.uint64) << np.uint64(32)) | lo.astype(np.uint64)
    return bits


def normal_from_bits(bits, dtype) -> np.ndarray:
    """``sqrt(2) * erfinv(u)`` for mantissa-filled uniforms u in (nextafter(-1, 0), 1)."""
    dtype = np.dtype(dtype)
    finfo = np.finfo(dtype)
    nbits, nmant = finfo.bits, finfo.nmant
    utype = np.uint64 if nbits == 64 else np.uint32
    one_bits = np.array(1.0, dtype=dtype).view(utype)
    float_bits = (np.asarray(bits).astype(utype) >> utype(nbits - nmant)) | one_bits
    floats = float_bits.view(dtype) - dtype.type(1.0)
    lo = np.nextafter(np.array(-1.0, dtype), np.array(0.0, dtype))
    u = np.maximum(lo, floats * (dtype.type(1.0) - lo) + lo)
    value = erfinv(u.astype(np.float64)).astype(dtype)
    return (dtype.type(np.sqrt(2.0)) * value).astype(dtype)


def batch_normals(
    seed: int,
    batch: int,
    n: int,
    dtype,
    offset: int = 0,
    total: int | None = None,
    partitionable: bool = True,
) -> np.ndarray:
    """Rows ``normal(split(PRNGKey(seed), total)[offset + b], (n,))`` for b < batch.

    ``partitionable`` selects JAX's ``jax_threefry_partitionable`` key scheme
    (default on since JAX 0.5); ``False`` restates the legacy scheme, whose
    child keys depend on the total split count ``total`` (the global batch).
    """
    width = np.finfo(np.dtype(dtype)).bits
    total = offset + batch if total is None else int(total)
    if partitionable:
        keys = split(prng_key(seed), batch, offset)
        bits = [random_bits(keys[b], n, width) for b in range(batch)]
    else:
        keys = split_original(prng_key(seed), total)[offset : offset + batch]
        bits = [random_bits_original(keys[b], n, width) for b in range(batch)]
    return np.stack([normal_from_bits(b, dtype) for b in bits], axis=0)
