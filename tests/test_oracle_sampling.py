"""The oracle's sampling restatement (crates/arcqml-sim/src/statevector/api/measurement.rs:18-60).

Pins: the ChaCha block function against RFC 7539's test vectors (section 2.3.2 and appendix
A.1 #1, ChaCha20) and against OpenSSL's ChaCha20 for random keys and 64-bit counter and stream
words; the reference's own sampling tests (Bell state, 1000 shots, seed 42: only
"00" and "11", counts summing to 1000 — run_tests.rs:280-295, python/tests/api/single.rs:140-166);
and the oracle's bisection against a literal restatement of the reference's per-shot linear scan.
StdRng's seed expansion and stream layout come from crates the reference does not ship
(rand 0.10.2, rand_core 0.10.1, chacha20 0.10.2): bit-exact counts against Rust are unpinned.
"""
import math

import numpy as np


def test_chacha20_rfc7539_vectors(oracle):
    blk = oracle.chacha_block([0] * 8, 0, 0, 20)
    out = b"".join(x.to_bytes(4, "little") for x in blk)
    assert out.hex() == ("76b8e0ada0f13d90405d6ae55386bd28bdd219b8a08ded1aa836efcc8b770dc7"
                         "da41597c5157488d7724e03fb8d84a376a43b8f41518a11cc387b669b2ee6586")
    # section 2.3.2: key 00..1f, nonce 00:00:00:09:00:00:00:4a:00:00:00:00, block counter 1;
    # the 32-bit counter + 96-bit nonce words are words 12-15 of the same state
    key = [int.from_bytes(bytes(range(4 * i, 4 * i + 4)), "little") for i in range(8)]
    blk = oracle.chacha_block(key, 1 | (0x09000000 << 32), 0x4A000000, 20)
    out = b"".join(x.to_bytes(4, "little") for x in blk)
    assert out.hex()[:64] == "10f1e7e4d13b5915500fdd1fa32071c4c7d1f4c733c068030422aa9ac3d46c4e"


def test_chacha20_matches_openssl_for_random_keys_and_64_bit_words(oracle):
    """An independent ChaCha20 (OpenSSL through the cryptography package, whose 16-byte IV is
    state words 12-15) agrees block for block, with counter and stream words above 2^32."""
    import struct

    import pytest
    algs = pytest.importorskip("cryptography.hazmat.primitives.ciphers")
    rng = np.random.Generator(np.random.PCG64(77))
    for _ in range(64):
        key = [int(x) for x in rng.integers(0, 2**32, 8, dtype=np.uint64)]
        ctr, stream = (int(x) for x in rng.integers(0, 2**63, 2, dtype=np.uint64))
        iv = struct.pack("<4I", ctr & 0xFFFFFFFF, ctr >> 32, stream & 0xFFFFFFFF, stream >> 32)
        enc = algs.Cipher(algs.algorithms.ChaCha20(struct.pack("<8I", *key), iv), mode=None)
        words = list(struct.unpack("<16I", enc.encryptor().update(bytes(64))))
        assert words == oracle.chacha_block(key, ctr, stream, 20)


def test_bell_state_counts_like_reference_test(oracle):
    s = 1.0 / math.sqrt(2.0)
    amps = np.array([s, 0, 0, s], dtype=np.complex128)
    counts = oracle.sample_counts(amps, 2, 1000, 42)
    assert sum(counts.values()) == 1000
    assert set(counts) <= {"00", "11"}
    assert list(counts) == sorted(counts)


def literal_scan(amps, shots, seed, oracle):
    """The reference's sample_basis_index, line by line (measurement.rs:44-59)."""
    probs = [a.real * a.real + a.imag * a.imag for a in amps]
    total = 0.0
    for p in probs:
        total += p
    out = []
    for s in range(shots):
        target = float(oracle.stdrng_u64(seed, s) >> 11) * 2.0 ** -53 * total
        cum = 0.0
        for i, p in enumerate(probs):
            cum += p
            if target < cum:
                out.append(i)
                break
        else:
            out.append(len(probs) - 1)
    return out


def test_bisection_equals_linear_scan(oracle):
    rng = np.random.Generator(np.random.PCG64(5))
    for n, seed in [(1, 0), (3, 7), (6, 2 ** 63 + 11), (8, 123456789)]:
        a = rng.normal(size=1 << n) + 1j * rng.normal(size=1 << n)
        a[rng.uniform(size=a.size) < 0.3] = 0  # zero-probability entries
        a /= np.linalg.norm(a)
        got = oracle.sample_indices(a, n, 300, seed)
        assert list(map(int, got)) == literal_scan(a, 300, seed, oracle)


def test_generator_is_counter_based(oracle):
    """Shot s reads words 2s, 2s+1 of block s // 8: blocks can be generated independently."""
    seed = 99
    key = oracle.stdrng_key(seed)
    for s in (0, 1, 7, 8, 15, 1000):
        blk = oracle.chacha_block(key, s // 8, 0, 12)
        w = (s % 8) * 2
        assert oracle.stdrng_u64(seed, s) == blk[w] | (blk[w + 1] << 32)
