"""Pin the oracle's Threefry PRNG and normal sampler against published values."""

import numpy as np

from oracle.prng import (
    batch_normals,
    normal_from_bits,
    prng_key,
    random_bits,
    random_bits_original,
    split,
    threefry2x32,
)


def _hex(pair):
    return tuple(hex(int(x)) for x in pair)


def test_threefry_random123_known_answers():
    """Known-answer vectors of Threefry-2x32-20 (Random123 test suite)."""
    assert _hex(threefry2x32(0, 0, 0, 0)) == ("0x6b200159", "0x99ba4efe")
    assert _hex(threefry2x32(0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF)) == (
        "0x1cb996fc", "0xbb002be7")
    assert _hex(threefry2x32(0x13198A2E, 0x03707344, 0x243F6A88, 0x85A308D3)) == (
        "0xc4923a9c", "0x483df7a0")


def test_prng_key_layout():
    np.testing.assert_array_equal(prng_key(42), [0, 42])
    np.testing.assert_array_equal(prng_key(2**33 + 5), [2, 5])


def test_legacy_normal_matches_published_draws():
    """``jax.random.normal(PRNGKey(0), (10,))`` in float32 as printed in JAX's quickstart,
    and the scalar draw ``normal(PRNGKey(0))``; agreement to the last bit of erfinv."""
    key = prng_key(0)
    got = normal_from_bits(random_bits_original(key, 10, 32), np.float32)
    published = [-0.3721109, 0.26423115, -0.18252768, -0.7368197, -0.44030377, -0.1521442,
                 -0.67135346, -0.5908641, 0.73168886, 0.5673026]
    np.testing.assert_allclose(got, published, rtol=2e-7, atol=0)
    scalar = normal_from_bits(random_bits_original(key, 1, 32), np.float32)
    np.testing.assert_allclose(scalar, [-0.20584226], rtol=2e-7)


def test_partitionable_scheme_counter_layout():
    """Split child i and element j use the 64-bit counter (0, i) / (0, j)."""
    key = prng_key(42)
    keys = split(key, 3)
    for i in range(3):
        np.testing.assert_array_equal(keys[i], threefry2x32(key[0], key[1], 0, i))
    bits64 = random_bits(keys[1], 4, 64)
    x0, x1 = threefry2x32(keys[1][0], keys[1][1], 0, 3)
    assert int(bits64[3]) == (int(x0) << 32) | int(x1)
    bits32 = random_bits(keys[1], 4, 32)
    assert int(bits32[3]) == int(x0) ^ int(x1)


def test_batch_normals_shard_offsets_reproduce_full_batch():
    full = batch_normals(42, 6, 5, np.float64)
    part = batch_normals(42, 3, 5, np.float64, offset=3, total=6)
    np.testing.assert_array_equal(full[3:], part)
    full_legacy = batch_normals(42, 6, 5, np.float32, partitionable=False)
    part_legacy = batch_normals(42, 2, 5, np.float32, offset=4, total=6, partitionable=False)
    np.testing.assert_array_equal(full_legacy[4:], part_legacy)


def test_normals_are_standard():
    x = batch_normals(0, 4, 20000, np.float64)
    assert abs(x.mean()) < 0.02 and abs(x.std() - 1) < 0.02
