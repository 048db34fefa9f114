"""The CPU oracle against the reference's own known answers (tests/golden)
and against independent numpy restatements.  No GPU."""
import numpy as np
import pytest

from tests.golden_util import DT, OPS, cases_of_kind, input_array

pytestmark = []


@pytest.mark.parametrize("case_id", cases_of_kind("reduce_full", "reduce_full_prepared"))
def test_full_reduction_fixture(oracle, golden, case_id):
    c = golden[case_id]
    a = input_array(c)
    lay = c["layout"]
    if "error" in c:
        return  # output-shape errors are planner behaviour (test_planner.py)
    got = oracle.reduce_full(a, lay["shape"], lay["strides"], lay["offset"], op=OPS[c["op"]])
    np.testing.assert_array_equal(np.array([got], dtype=a.dtype), np.array(c["expected"], dtype=a.dtype))
    if "rewrite" in c:
        b = np.array(c["rewrite"], dtype=a.dtype)
        got = oracle.reduce_full(b, lay["shape"], lay["strides"], lay["offset"], op=OPS[c["op"]])
        assert got == c["expected_after_rewrite"][0]


@pytest.mark.parametrize("case_id", cases_of_kind("reduce_axis", "reduce_axis_prepared"))
def test_axis_reduction_fixture(oracle, golden, case_id):
    c = golden[case_id]
    a = input_array(c)
    lay = c["layout"]
    if "error" in c or "error_prefix" in c:
        if c.get("error", "").startswith(("axis 2", "min_axis")):
            with pytest.raises(ValueError):
                oracle.reduce_axis(a, lay["shape"], c["axis"], op=OPS[c["op"]],
                                   in_strides=lay["strides"], in_offset=lay["offset"])
        return
    got = oracle.reduce_axis(a, lay["shape"], c["axis"], op=OPS[c["op"]], in_strides=lay["strides"],
                             in_offset=lay["offset"])
    np.testing.assert_array_equal(got, np.array(c["expected"], dtype=a.dtype))


@pytest.mark.parametrize("case_id", cases_of_kind("scan", "scan_prepared"))
def test_scan_fixture(oracle, golden, case_id):
    c = golden[case_id]
    a = input_array(c)
    lay = c["layout"]
    if "error" in c or "error_prefix" in c:
        if c.get("error", "").startswith("scan axis 2"):
            with pytest.raises(ValueError):
                oracle.scan_axis(a, lay["shape"], c["axis"], op=OPS[c["op"]], in_strides=lay["strides"])
        return
    out_lay = c.get("out_layout")
    out_strides = out_lay["strides"] if out_lay else lay["strides"]
    n = int(np.prod(lay["shape"]))
    got = oracle.scan_axis(a, lay["shape"], c["axis"], op=OPS[c["op"]], reverse=c["reverse"],
                           in_strides=lay["strides"], in_offset=lay["offset"],
                           out_storage=np.zeros(max(n, len(a)), a.dtype) if out_lay is None else np.zeros(n, a.dtype),
                           out_strides=out_strides)
    np.testing.assert_array_equal(got[:n] if out_lay else got[:len(c["expected"])],
                                  np.array(c["expected"], dtype=a.dtype))


def test_exclusive_scan_matches_shifted_inclusive(oracle):
    rng = np.random.default_rng(7)
    for dt in (np.uint32, np.int32, np.int64):
        a = rng.integers(-50, 50, size=1000).astype(dt)
        inc = oracle.scan_axis(a, [1000], 0)
        exc = oracle.scan_axis(a, [1000], 0, exclusive=True)
        np.testing.assert_array_equal(exc[1:], inc[:-1])
        assert exc[0] == 0
        rexc = oracle.scan_axis(a, [1000], 0, reverse=True, exclusive=True)
        rinc = oracle.scan_axis(a, [1000], 0, reverse=True)
        np.testing.assert_array_equal(rexc[:-1], rinc[1:])
        with np.errstate(over="ignore"):
            np.testing.assert_array_equal(inc, np.cumsum(a, dtype=dt))


def test_argmax_lowest_index_wins(oracle):
    x = np.array([[1, 5, 5, 2], [7, 7, 7, 7], [-1, -3, -1, -3]], dtype=np.float32).ravel()
    v, i = oracle.arg_reduce_axis(x, [3, 4], 1, op=oracle.MAX)
    np.testing.assert_array_equal(i, [1, 0, 0])
    np.testing.assert_array_equal(v, [5, 7, -1])
    v, i = oracle.arg_reduce_axis(x, [3, 4], 1, op=oracle.MIN)
    np.testing.assert_array_equal(i, [0, 0, 1])
    v, i = oracle.arg_reduce_axis(x, [3, 4], 0, op=oracle.MAX)
    np.testing.assert_array_equal(i, [1, 1, 1, 1])


def test_identities_match_reference_tokens(oracle):
    # ops.rs:926-984 and the CudaC tokens ops.rs:1033-1060: +/-3.402823466e+38f, not inf.
    empty = np.zeros(0, np.float32)
    assert oracle.reduce_full(empty, [0], op=oracle.MIN) == np.float32(3.402823466e38)
    assert oracle.reduce_full(empty, [0], op=oracle.MAX) == np.float32(-3.402823466e38)
    assert oracle.reduce_full(np.zeros(0, np.uint32), [0], op=oracle.MIN) == 0xFFFFFFFF
    assert oracle.reduce_full(np.zeros(0, np.int32), [0], op=oracle.MAX) == -2**31
    assert oracle.reduce_full(np.zeros(0, np.int32), [0], op=oracle.PROD) == 1


def test_integer_folds_wrap(oracle):
    a = np.array([2**31 - 1, 1, 5], dtype=np.int32)
    assert oracle.reduce_full(a, [3]) == np.int32(-2**31 + 5)
    b = np.array([2**31 - 1, 1], dtype=np.int32)
    assert oracle.reduce_full(b, [2], out_dtype=np.int64) == 2**31


def test_generators_match_their_definition(oracle):
    # SplitMix64 of (seed<<32 ^ i), restated in Python integers.
    M = (1 << 64) - 1

    def sm(x):
        z = (x + 0x9E3779B97F4A7C15) & M
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
        return z ^ (z >> 31)

    for seed in (0, 1, 4):
        for i in (0, 1, 12345, 2**32 + 7):
            assert oracle.hash64(seed, i) == sm(((seed << 32) ^ i) & M)
    u = oracle.generate(oracle.GEN_U32_LOW4, 1, 100)
    assert u.max() <= 15 and u.dtype == np.uint32
    f = oracle.generate(oracle.GEN_F32_UNIFORM_PM1, 0, 1000)
    assert f.min() >= -1 and f.max() < 1
    i32 = oracle.generate(oracle.GEN_I32_PM1000, 4, 10000)
    assert i32.min() >= -1000 and i32.max() <= 1000
    d = oracle.generate(oracle.GEN_F64_UNIT, 3, 1000)
    assert d.min() >= 0 and d.max() < 1
    z = oracle.generate(oracle.GEN_F32_NORMAL, 2, 100000)
    assert abs(float(z.mean())) < 0.02 and abs(float(z.std()) - 1) < 0.02


def test_mt_baselines_agree_with_sequential(oracle):
    a = oracle.generate(oracle.GEN_U32_LOW4, 1, 100003)
    out = np.empty_like(a)
    oracle.exclusive_scan_u32_mt(a, out, 0, 4)
    np.testing.assert_array_equal(out, oracle.scan_axis(a, [a.size], 0, exclusive=True))
    b = oracle.generate(oracle.GEN_I32_PM1000, 4, 100003)
    outb = np.empty_like(b)
    oracle.inclusive_scan_i32_mt(b, outb, 5, 3)
    ref = oracle.scan_axis(b, [b.size], 0)
    np.testing.assert_array_equal(outb, ref + 5)
    assert oracle.sum_i32_to_i64_mt(b, 3) == int(b.astype(np.int64).sum())
    m = oracle.generate(oracle.GEN_F32_NORMAL, 2, 64 * 100)
    v, i = oracle.row_argmax_f32_mt(m, 64, 100, 2)
    v2, i2 = oracle.arg_reduce_axis(m, [64, 100], 1)
    np.testing.assert_array_equal(i, i2)
    c = oracle.generate(oracle.GEN_F64_UNIT, 3, 50 * 300)
    np.testing.assert_allclose(oracle.col_sum_f64_mt(c, 50, 300, 2),
                               oracle.reduce_axis(c, [50, 300], 0).ravel(), rtol=1e-12)


MAPS = {"dot": 0, "trace": 1, "norm_l1": 2, "norm_l2": 3, "norm_max": 4}


@pytest.mark.parametrize("case_id", cases_of_kind("map"))
def test_map_reduction_fixture(oracle, golden, case_id):
    c = golden[case_id]
    a = input_array(c)
    lay = c["layout"]
    if "error_prefix" in c:
        return  # planner behaviour, checked on the GPU path
    b = np.array(c["input_b"], dtype=a.dtype) if "input_b" in c else None
    lb = c.get("layout_b", lay)
    got = oracle.map_reduce(MAPS[c["map"]], a, lay["shape"], lay["strides"], lay["offset"], b=b,
                            b_strides=lb["strides"], b_offset=lb["offset"])
    assert abs(float(got) - c["expected"][0]) <= c.get("tolerance", 0.0), c["source"]
