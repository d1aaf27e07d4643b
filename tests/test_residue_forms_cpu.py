"""The extraction's residue arithmetic, restated on the CPU and checked
exhaustively over its input range: the quotient umulhi(v, ceil(2^32 / p)) is
exact for every pre-sum v the kernel can form, the stored byte
((v + 128) mod p) - 128 is congruent to the biased integer and within int8,
and a modular dot product of such residues equals the one of the reference's
symmetric balanced residues modulo p while staying inside int32."""
import numpy as np
import pytest

PRIMES = [256, 255, 253, 251, 247, 241, 239, 233, 229, 227, 223, 217, 211, 199,
          197, 193, 191, 181, 179, 173]


def bytes_weights(p):
    return [(1 << (8 * j)) % p for j in range(7)]


@pytest.mark.parametrize("p", PRIMES)
def test_quotient_exact_over_the_presum_range(p):
    # v = dp4a over the 7 bytes (<= 7 * 255 * 255) + cb (< 257) + 128
    vmax = 7 * 255 * 255 + 256 + 128
    v = np.arange(vmax + 1, dtype=np.uint64)
    mex = np.uint64(-(-(1 << 32) // p))
    q = (v * mex) >> np.uint64(32)
    assert np.array_equal(q, v // np.uint64(p))
    r = v - q * np.uint64(p)
    assert int(r.max()) < p


@pytest.mark.parametrize("p", PRIMES)
def test_stored_byte_congruent_and_in_int8(p):
    rng = np.random.default_rng(p)
    be = int(rng.integers(16, 54))
    w = bytes_weights(p)
    cb = p - (1 << be) % p
    for _ in range(2000):
        T = int(rng.integers(-(1 << be), (1 << be) + 1))   # the scaling keeps |T| <= 2^b
        u = (T + (1 << be)) % (1 << 64)              # biased two's complement, as the kernel forms it
        assert u < (1 << 56)
        v = sum(((u >> (8 * j)) & 0xFF) * w[j] for j in range(7)) + cb + 128
        r = v - ((v * -(-(1 << 32) // p)) >> 32) * p
        byte = (r ^ 0x80) & 0xFF
        stored = byte - 256 if byte >= 128 else byte  # int8 value of the byte
        assert -128 <= stored <= min(127, p - 129)
        assert (stored - T) % p == 0


@pytest.mark.parametrize("p", [256, 255, 217, 173])
def test_dot_products_agree_modulo_p_within_int32(p):
    rng = np.random.default_rng(7)
    K = 131071                                        # the single-launch K bound
    x = rng.integers(-(1 << 40), 1 << 40, size=(2, K))
    sym = ((x + p // 2) % p) - p // 2                 # symmetric balanced residues
    if p == 256:
        sym = np.where(sym == 128, -128, sym)
    off = ((x % p + 128) % p) - 128                   # the stored form
    assert off.min() >= -128 and off.max() <= 127
    d_sym = int(np.dot(sym[0], sym[1]))
    d_off = int(np.dot(off[0], off[1]))
    assert (d_sym - d_off) % p == 0
    assert abs(d_off) <= K * 128 * 128 < 2 ** 31
