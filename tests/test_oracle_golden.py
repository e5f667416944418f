"""Pin the CPU oracle against fixtures produced by the reference's own kernels
(tests/golden/make_golden.py). CPU only."""
import numpy as np
import pytest

import oracle as O
from conftest import FRO_TOL, MAX_REL_TOL, rel_errors

BITS = (2, 4, 6, 8)
DTYPES = ("bf16", "f16")


def _f32(g, key, dtype):
    return O.to_f32(g[key], dtype)


@pytest.mark.parametrize("b", BITS)
def test_pack_words_bit_exact(golden, b):
    a = golden["pack_in_u8"]
    out = O.pack_words(a.view(np.uint32), b)
    np.testing.assert_array_equal(out, golden[f"pack_out_b{b}"])
    # storage = K*N*b/8 bytes (tests/test_grinqh_ops.py:76)
    assert out.nbytes == a.size * b // 8


@pytest.mark.parametrize("b", BITS)
def test_unpack_bit_exact(golden, b):
    rec = O.unpack(golden[f"pack_out_b{b}"], b, golden["pack_in_u8"].shape[1] // 4)
    np.testing.assert_array_equal(rec, golden[f"unpack_out_b{b}"])
    np.testing.assert_array_equal(rec, golden["pack_in_u8"] >> (8 - b))


@pytest.mark.parametrize("b", BITS)
def test_pack_codes_bit_exact(golden, b):
    np.testing.assert_array_equal(O.pack_codes(golden[f"codes_b{b}"], b), golden[f"packed_b{b}"])
    np.testing.assert_array_equal(O.pack_codes(golden[f"dense_codes_b{b}"], b), golden[f"dense_packed_b{b}"])
    n = golden[f"codes_b{b}"].shape[1]
    np.testing.assert_array_equal(O.unpack_codes(golden[f"packed_b{b}"], b, n // 4), golden[f"codes_b{b}"])


def test_shuffle_roundtrip():
    w = np.arange(5 * 48, dtype=np.int32).reshape(5, 48)
    np.testing.assert_array_equal(O.postshuffle(O.preshuffle(w)), w)
    with pytest.raises(ValueError):
        O.preshuffle(np.zeros((2, 24)))


def test_bias_table():
    # kernel.py:73-82: b=8 deltas 32,-24,-6,-2; all zones -> 0; b=2 -> always 0
    t8 = O.bias_table(8)
    assert t8[0b0001] == 32 and t8[0b0011] == 8 and t8[0b0111] == 2 and t8[0b1111] == 0
    assert t8[0b0010] == -24  # independent zones (non-prefix masks are legal)
    assert (O.bias_table(2) == 0).all()
    t4 = O.bias_table(4)
    assert t4[1] == 2 and t4[3] == 0 and t4[0b1100] == 0  # zones >= b/2 never count


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("b", BITS)
@pytest.mark.parametrize("q", ["spread", "all_or_nothing", "mild", "aggressive", "skip_all", "dense"])
def test_graded_gemv_matches_reference_kernel(golden, dtype, b, q):
    key = f"gemv_{dtype}_b{b}_{q}"
    x = _f32(golden, f"gemv_x_{dtype}", dtype)[0]
    s = _f32(golden, f"gemv_s_{dtype}", dtype)
    y = O.graded_gemv(x, golden[f"codes_b{b}"], s, golden[key + "_th"], b, 128)
    y_store = O.round_to_dtype(y, dtype)
    ref = _f32(golden, key + "_y", dtype)[0]
    mx, fro = rel_errors(O.to_f32(y_store, dtype), ref)
    assert mx <= 4e-3 and fro <= 1e-3, (mx, fro)
    # the reference rounds an fp32 accumulation: almost every element must agree exactly
    assert np.mean(O.to_f32(y_store, dtype) == ref) > 0.97


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("b", BITS)
@pytest.mark.parametrize("m", [2, 3, 5, 8])
@pytest.mark.parametrize("t", ["dense", "spread"])
def test_union_gemv_matches_reference_kernel(golden, dtype, b, m, t):
    key = f"union_{dtype}_m{m}_b{b}_{t}"
    x = _f32(golden, f"union_x_{dtype}_m{m}", dtype)
    s = _f32(golden, f"union_s_{dtype}_m{m}", dtype)
    y = O.union_gemv(x, golden[f"codes_b{b}"], s, golden[key + "_th"], b, 128)
    ref = _f32(golden, key + "_y", dtype)
    mx, fro = rel_errors(O.to_f32(O.round_to_dtype(y, dtype), dtype), ref)
    assert mx <= 4e-3 and fro <= 1e-3, (mx, fro)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("b", BITS)
def test_dense_matches_reference(golden, dtype, b):
    key = f"dense_{dtype}_b{b}"
    x = _f32(golden, key + "_x", dtype)
    s = _f32(golden, key + "_s", dtype)
    y = O.dense(x, golden[f"dense_codes_b{b}"], s, 128, dtype)
    ref = _f32(golden, key + "_y", dtype)
    mx, fro = rel_errors(O.to_f32(O.round_to_dtype(y, dtype), dtype), ref)
    assert mx <= MAX_REL_TOL / 4 and fro <= FRO_TOL / 4, (mx, fro)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows", [1, 4])
def test_op_with_bias_matches_reference(golden, dtype, rows):
    key = f"bias_{dtype}_m{rows}"
    x = _f32(golden, key + "_x", dtype)
    s = _f32(golden, key + "_s", dtype)
    bias = _f32(golden, key + "_bias", dtype)
    y = O.gemm_or_gemv(x, golden["codes_b8"], s, bias, 8, 128, golden[key + "_th"], dtype)
    ref = _f32(golden, key + "_y", dtype)
    mx, fro = rel_errors(O.to_f32(y, dtype), ref)
    assert mx <= 4e-3 and fro <= 1.5e-3, (mx, fro)


def test_config_like_case(golden):
    x = O.to_f32(golden["cfg_x"], "bf16")[0]
    s = O.to_f32(golden["cfg_s"], "bf16")
    np.testing.assert_array_equal(O.pack_codes(golden["cfg_codes"], 8), golden["cfg_packed"])
    y = O.graded_gemv(x, golden["cfg_codes"], s, golden["cfg_th"], 8, 128)
    ref = O.to_f32(golden["cfg_y"], "bf16")[0]
    mx, fro = rel_errors(O.to_f32(O.round_to_dtype(y, "bf16"), "bf16"), ref)
    assert mx <= 4e-3 and fro <= 1e-3


@pytest.mark.parametrize("b", BITS)
@pytest.mark.parametrize("case", ["spread", "lowest", "highest", "70_20_10", "non_monotone"])
def test_graded_rows_equals_looped_gemv(b, case):
    """The many-row evaluation of per-token grading (used at configs[2] sizes) equals
    the reference-pinned one-row GEMV looped over the rows."""
    rng = np.random.default_rng(b * 13 + len(case))
    K, N, M = 384, 96, 7
    codes = rng.integers(-(1 << (b - 1)), 1 << (b - 1), size=(K, N)).astype(np.int8)
    s = O.to_f32(O.round_to_dtype(rng.random((K // 128, N)) * 0.02 + 1e-3, "bf16"), "bf16")
    x, _ = O.make_activations(rng, M, K, dist="t3")
    x = O.to_f32(O.round_to_dtype(x, "bf16"), "bf16")
    ax = np.abs(x)
    th = {"spread": O.quantile_thresholds(ax, [0.2, 0.4, 0.6, 0.8]),
          "lowest": [-1.0, float("inf"), float("inf"), float("inf")],
          "highest": [-1.0] * 4,
          "70_20_10": [-1.0] + O.quantile_thresholds(ax, [0.7, 0.9, 0.9]),
          "non_monotone": O.quantile_thresholds(ax, [0.5, 0.1, 0.9, 0.3])}[case]
    np.testing.assert_allclose(O.graded_rows(x, codes, s, th, b, 128, k_chunk=128),
                               O.looped_gemv(x, codes, s, th, b, 128), rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("b", BITS)
def test_checkpoint_codec(golden, b):
    codes = golden[f"ct_codes_b{b}"]
    np.testing.assert_array_equal(O.ct_pack_to_int32(codes, b), golden[f"ct_packed_b{b}"])
    np.testing.assert_array_equal(O.ct_unpack_from_int32(golden[f"ct_packed_b{b}"], b, codes.shape), codes)


def test_grade_is_strict_fp32():
    x = np.array([0.5, -0.5, 0.25, 1.0, np.nan], dtype=np.float32)
    m = O.grade(x, [0.5, 0.25, 0.0, 2.0], 8)
    # |x| > t strictly; NaN is never active
    assert list(m) == [0b0110, 0b0110, 0b0100, 0b0111, 0]
    assert (O.grade(x, [-1.0] * 4, 4) <= 0b0011).all()
