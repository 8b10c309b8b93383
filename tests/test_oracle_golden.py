"""The CPU oracle against every golden vector of the reference's tests.

The vectors were recorded by the reference (tests/golden/make_golden.py extracts
them from tests/testthat/test-prng.R, test-random.R, test-scipy-special.R and the
fixtures stateful_rng.json, lax_x32.json, lax_x64.json).  Integer and key data
must agree exactly.  Floats are held to the reference's own rule (16 ulp, or the
relative tolerance of the fixture) and, tighter, to 0 ulp: the oracle reproduces
every recorded float bit for bit, except the log-transform samplers, whose recorded
float32 values carry XLA's own float32 logarithm; those are held to the case's
"max_ulp" (3, and 16 for gumbel mode "high"; see make_golden._log_allowance).
"""

import numpy as np
import pytest

from golden_cases import OracleBackend, check, evaluate, expected, load_cases, max_ulp

CASES = load_cases()


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_oracle_matches_reference_golden(case):
    got = evaluate(case, OracleBackend())
    ok, detail = check(case, got)
    assert ok, f"{case['name']} ({case['source']}): {detail}"
    want = expected(case)
    if want.dtype.kind == "f":
        assert max_ulp(np.asarray(got).astype(want.dtype), want) <= case.get("max_ulp", 0), \
            case["source"]


def test_golden_covers_the_path():
    ops = {c["op"] for c in CASES}
    assert {"threefry_2x32", "seed", "split", "fold_in", "bits", "uniform", "normal",
            "bernoulli", "vmap_split", "vmap_fold_in", "vmap_uniform", "vmap_normal",
            "erf_inv", "randint", "exponential", "gumbel", "laplace", "logistic",
            "truncated_normal", "permutation", "choice", "rbg_bits", "rbg_split",
            "rbg_fold_in", "rbg_vmap_bits"} <= ops
    # both layouts and x64 are pinned
    assert any(c["args"].get("partitionable") is False for c in CASES)
    assert any(c["args"].get("x64") for c in CASES)


def test_unfused_uniform_differs_from_reference():
    """The reference's recorded uniforms need the fused affine map: the unfused form
    misses test-random.R:43 by 4 ulp (f32) and :160 by 8 ulp (f64)."""
    for name in ("uniform_42_23_m", "x64_uniform_42_23_m"):
        case = next(c for c in CASES if c["name"] == name)
        got = evaluate(case, OracleBackend(mul_add_fma=False))
        assert max_ulp(np.asarray(got), expected(case)) > 0


def test_threefry_known_answers(oracle):
    # Random123 known-answer vectors, tests/testthat/test-prng.R:61-63
    assert oracle.threefry2x32(0, 0, 0, 0) == (0x6B200159, 0x99BA4EFE)
    m = 0xFFFFFFFF
    assert oracle.threefry2x32(m, m, m, m) == (0x1CB996FC, 0xBB002BE7)
    assert oracle.threefry2x32(0x13198A2E, 0x03707344, 0x243F6A88, 0x85A308D3) == (
        0xC4923A9C, 0x483DF7A0)


def test_bits_bulk_matches_elementwise(oracle):
    key = oracle.seed(123)
    n = 1 << 12
    for part in (True, False):
        for bw in (8, 16, 32, 64):
            bulk = oracle.random_bits(key, bw, n, part)
            idx = [0, 1, 2, 3, n // 2 - 1, n // 2, n - 2, n - 1]
            assert np.array_equal(bulk[idx], oracle.bits_at(key, bw, n, part, idx))
    # a range is a slice of the whole request
    whole = oracle.random_bits(key, 32, n, True)
    assert np.array_equal(oracle.random_bits(key, 32, n, True, begin=1000, count=77),
                          whole[1000:1077])


def test_original_layout_segments(oracle):
    """Original-layout requests of 2^32-1 words or more split the key and hash
    iota(2^32-1) per sub-key (R/prng.R:233-245)."""
    key = oracle.seed(0)
    size = (1 << 32) + 5  # nblocks = 1, rem = 6
    sub = oracle.split(key, 2, partitionable=False)
    # word 0 of the first segment: block 0 of iota(2^32-1) hashes (0, 2^31)
    assert oracle.bits_at(key, 32, size, False, [0])[0] == oracle.threefry2x32(
        int(sub[0][0]), int(sub[0][1]), 0, 1 << 31)[0]
    # the last word of the first segment is x1 of block 2^31-2, counts (2^31-2, 2^32-2)
    assert oracle.bits_at(key, 32, size, False, [(1 << 32) - 2])[0] == oracle.threefry2x32(
        int(sub[0][0]), int(sub[0][1]), (1 << 31) - 2, (1 << 32) - 2)[1]
    last = oracle.random_bits(sub[1], 32, 6, False)
    got = oracle.bits_at(key, 32, size, False, [(1 << 32) - 1 + i for i in range(6)])
    assert np.array_equal(got, last)


def test_philox_known_answers(oracle):
    # Random123's published known-answer vectors for philox4x32-10 (the first is also the
    # reference's rbg_bits, test-prng.R:50)
    assert oracle.philox4x32([0, 0, 0, 0], [0, 0]) == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C,
                                                       0x9B00DBD8]
    m = 0xFFFFFFFF
    assert oracle.philox4x32([m, m, m, m], [m, m]) == [0x408F276D, 0x41C83B0E, 0xA20BC7C6,
                                                       0x6D5451FD]
    assert oracle.philox4x32([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344],
                             [0xA4093822, 0x299F31D0]) == [0xD16CFE09, 0x94FDCCEB, 0x5001E420,
                                                           0x24126EA1]


def test_rbg_stream_layout(oracle):
    """32-bit element e is word e % 4 of block e / 4; the 128-bit counter carries across
    words; 8/16-bit elements are the low bits of the 32-bit ones."""
    q = [0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF, 7]
    w = oracle.rbg_bits(q, 32, 12)
    for b in range(3):
        c = ((0xFFFFFFFF | 0xFFFFFFFF << 32 | 0xFFFFFFFF << 64 | 7 << 96) + b) % (1 << 128)
        want = oracle.philox4x32([(c >> (32 * i)) & 0xFFFFFFFF for i in range(4)], q[:2])
        assert list(w[4 * b:4 * b + 4]) == want
    assert np.array_equal(oracle.rbg_bits(q, 8, 12), (w & 0xFF).astype(np.uint8))
    assert np.array_equal(oracle.rbg_bits(q, 16, 12), (w & 0xFFFF).astype(np.uint16))
    w64 = oracle.rbg_bits(q, 64, 6)
    assert np.array_equal(w64, w.astype(np.uint64)[0::2] | w.astype(np.uint64)[1::2] << 32)


def test_rbg_shuffle_under_vmap_reduces_to_the_key_of_lane_zero(oracle):
    """The vmap restatement of rnd_shuffle with rbg / unsafe_rbg keys: lane 0 is the
    unbatched shuffle of the first key (row 0 of the batched request is the unbatched
    request), every lane is a permutation, and the lanes differ."""
    import numpy as np
    q = oracle.rbg_seed(5)
    for impl in ("rbg", "unsafe_rbg"):
        lanes = oracle.shuffle_rbg_lanes(q, impl, 3, 1, 3000, 1)
        key, cur = np.asarray(q, dtype=np.uint32), np.arange(3000)
        for _ in range(2):  # 3000 elements: two rounds
            sp = oracle.rbg_split(key, 2) if impl == "rbg" else oracle.rbg_unsafe_split(key, 2)
            key = sp[0]
            cur = cur[np.argsort(oracle.rbg_bits(sp[1], 32, 3000), kind="stable")]
        assert np.array_equal(lanes[0], cur), impl
        for r in lanes:
            assert np.array_equal(np.sort(r), np.arange(3000))
        assert not np.array_equal(lanes[1], lanes[0]) and not np.array_equal(lanes[2], lanes[1])
