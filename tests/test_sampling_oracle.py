"""The oracle's seeded sampler (src/sampling.rs) on the CPU: its ChaCha
block function pinned to published test vectors, and the reference's own
sampling tests (tests/sampling.rs) restated on it."""
import math

import numpy as np
import pytest

from oracle import oracle as O

# RFC 7539 section 2.3.2: key 00..1f, block counter 1, nonce
# 00:00:00:09:00:00:00:4a:00:00:00:00; 20 rounds.
RFC_IN = [0x61707865, 0x3320646E, 0x79622D32, 0x6B206574,
          0x03020100, 0x07060504, 0x0B0A0908, 0x0F0E0D0C,
          0x13121110, 0x17161514, 0x1B1A1918, 0x1F1E1D1C,
          0x00000001, 0x09000000, 0x4A000000, 0x00000000]
RFC_OUT = [0xE4E7F110, 0x15593BD1, 0x1FDD0F50, 0xC47120A3,
           0xC7F4D1C7, 0x0368C033, 0x9AAA2204, 0x4E6CD4C3,
           0x466482D2, 0x09AA9F07, 0x05D7C214, 0xA2028BD9,
           0xD19C12B5, 0xB94E16DE, 0xE883D0CB, 0x4E3C50A2]

# RFC 7539 appendix A.1, test vectors 1 and 2: all-zero key and nonce,
# block counters 0 and 1 (the first two blocks of the zero-key stream).
ZERO_KEY_BLOCKS = [
    [0xADE0B876, 0x903DF1A0, 0xE56A5D40, 0x28BD8653, 0xB819D2BD, 0x1AED8DA0, 0xCCEF36A8, 0xC70D778B,
     0x7C5941DA, 0x8D485751, 0x3FE02477, 0x374AD8B8, 0xF4B8436A, 0x1CA11815, 0x69B687C3, 0x8665EEB2],
    [0xBEE7079F, 0x7A385155, 0x7C97BA98, 0x0D082D73, 0xA0290FCB, 0x6965E348, 0x3E53C612, 0xED7AEE32,
     0x7621B729, 0x434EE69C, 0xB03371D5, 0xD539D874, 0x281FED31, 0x45FB0A51, 0x1F0AE1AC, 0x6F4D794B],
]

# ChaCha with 8 rounds, all-zero 256-bit key and IV: the first 64 keystream
# bytes of the published reduced-round test vectors.
CHACHA8_ZERO = bytes.fromhex(
    "3e00ef2f895f40d67f5bb8e81f09a5a12c840ec3ce9a7f3b181be188ef711a1e"
    "984ce172b9216f419f445367456d5619314a42a3da86b001387bfdb80e0cfe42")

CONST = [0x61707865, 0x3320646E, 0x79622D32, 0x6B206574]


def test_chacha20_block_rfc7539():
    assert [int(v) for v in O.chacha_block(RFC_IN, 20)] == RFC_OUT


def test_zero_key_stream_layout():
    # Blocks 0 and 1 of the zero-key stream, through the block function and
    # through the generator's four-block buffer (64-bit counter in words
    # 12-13, stream in words 14-15).
    for c, want in enumerate(ZERO_KEY_BLOCKS):
        assert [int(v) for v in O.chacha_block(CONST + [0] * 8 + [c, 0, 0, 0], 20)] == want
    # The generator runs 8 rounds; the same layout with 8 rounds gives the
    # published ChaCha8 stream.
    words = O.Rng(key=bytes(32)).next_u32_words(16)
    assert b"".join(w.to_bytes(4, "little") for w in words) == CHACHA8_ZERO


def test_rng_buffer_crosses_blocks_in_order():
    # 4 blocks per refill: words 0..127 of the stream equal blocks 0..7.
    key = bytes(range(32))
    kw = [int.from_bytes(key[4 * i:4 * i + 4], "little") for i in range(8)]
    words = O.Rng(key=key).next_u32_words(128)
    for b in range(8):
        blk = O.chacha_block(CONST + kw + [b, 0, 0, 0], 8)
        assert words[16 * b:16 * b + 16] == [int(v) for v in blk]


def test_seed_from_u64_pcg_expansion():
    # rand_core's seed_from_u64: 8 PCG32 outputs, little-endian, form the key.
    def pcg_key(seed):
        out, st = bytearray(), seed
        for _ in range(8):
            st = (st * 6364136223846793005 + 11634580027462260723) & (2**64 - 1)
            xs = (((st >> 18) ^ st) >> 27) & 0xFFFFFFFF
            rot = st >> 59
            x = ((xs >> rot) | (xs << ((32 - rot) & 31))) & 0xFFFFFFFF
            out += x.to_bytes(4, "little")
        return bytes(out)
    for seed in [0, 1, 42, 2**64 - 1]:
        a, b = O.Rng(seed=seed), O.Rng(key=pcg_key(seed))
        assert [a.next_u64() for _ in range(40)] == [b.next_u64() for _ in range(40)]


def test_random_f64_takes_top_53_bits():
    a, b = O.Rng(seed=7), O.Rng(seed=7)
    for _ in range(100):
        v = a.random_f64()
        assert v == (b.next_u64() >> 11) * 2.0 ** -53 and 0.0 <= v < 1.0


def _random():
    return O.Sampler(temperature=1.0, top_k=2, seed=42)


def test_tie_and_membership_rules():
    # tests/sampling.rs:10-24
    assert O.Sampler().sample([2.0, 2.0, 1.0]) == (O.OK, 0)
    assert O.Sampler(temperature=1.0, top_k=1, seed=42).sample([-0.0, 0.0]) == (O.OK, 0)
    for _ in range(100):
        st, i = _random().sample([-10.0, 0.0, 3.0, 4.0])
        assert st == O.OK and i >= 2


def test_reproducible_and_errors_do_not_advance():
    # tests/sampling.rs:26-47
    a, b = _random(), _random()
    assert a.sample([float("nan"), 0.0]) == (O.NONFINITE, None)
    seq = [a.sample([0.0, 1.0])[1] for _ in range(64)]
    assert seq == [b.sample([0.0, 1.0])[1] for _ in range(64)]
    a.reset()
    assert seq == [a.sample([0.0, 1.0])[1] for _ in range(64)]
    assert 0 in seq and 1 in seq


def test_two_class_mass():
    # tests/sampling.rs:49-58: P(1) = 3/4.
    s = _random()
    count = sum(s.sample([0.0, math.log(3.0)])[1] == 1 for _ in range(10000))
    assert 7350 <= count <= 7650, count


def test_bad_parameters_empty_and_nonfinite():
    # tests/sampling.rs:60-100
    for t in [0.0, -1.0, float("nan"), float("inf")]:
        with pytest.raises(ValueError) as e:
            O.Sampler(temperature=t, top_k=1, seed=0)
        assert e.value.args[0] == O.INVALID_PARAMETERS
    with pytest.raises(ValueError):
        O.Sampler(temperature=1.0, top_k=0, seed=0)
    assert _random().sample([]) == (O.EMPTY_LOGITS, None)
    assert _random().sample([0.0]) == (O.INVALID_PARAMETERS, None)
    for bad in [float("inf"), float("-inf")]:
        assert _random().sample([bad, 0.0]) == (O.NONFINITE, None)
    tiny = np.array([1], dtype=np.uint32).view(np.float32)[0]
    fmax = float(np.finfo(np.float32).max)
    assert O.Sampler(temperature=tiny, top_k=2, seed=42).sample([-fmax, fmax]) == (O.OK, 1)


def test_walk_matches_restatement():
    # The walk over the top-k in (logit desc, id asc) order, restated in
    # Python with the same draws: identical ids on a vocabulary with ties.
    rng = np.random.default_rng(5)
    lg = rng.integers(-40, 40, 3000).astype(np.float32) / 8
    for k, t in [(1, 1.0), (7, 0.7), (64, 1.3), (3000, 2.0)]:
        s, r = O.Sampler(temperature=t, top_k=k, seed=11), O.Rng(seed=11)
        order = sorted(range(lg.size), key=lambda i: (-float(lg[i]), i))[:k]
        mx = float(lg.max())
        for _ in range(20):
            mass = [math.exp((float(lg[i]) - mx) / float(np.float32(t))) for i in order]
            total = 0.0
            for m in mass:
                total += m
            target, cum, want = r.random_f64() * total, 0.0, None
            for i, m in zip(order, mass):
                cum += m
                if target < cum:
                    want = i
                    break
            assert s.sample(lg) == (O.OK, want)
