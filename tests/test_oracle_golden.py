"""Pin the CPU oracle to the reference: constants and code choice on the
reference's own outputs (tests/golden/reference_golden.npz, made by running the
reference's host-side functions, see tests/golden/make_golden.py), plus the
known-answer tests of the reference's test suite restated on the oracle
(tests/test_quantize.py:90-131 in the reference)."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from helpers import bits, host_input


def test_constants_match_reference(golden):
    assert np.array_equal(bits(O.NF4_TABLE), bits(golden["nf4_table"]))
    assert np.array_equal(bits(O.NF4_THRESHOLDS), bits(golden["nf4_thresholds"]))


@pytest.mark.parametrize("kw, key", [
    ({}, "dynamic_map"),
    ({"signed": False}, "dynamic_map_unsigned"),
    ({"max_exponent_bits": 3, "total_bits": 4}, "dynamic_map_4bit"),
])
def test_create_dynamic_map_bitwise(golden, kw, key):
    assert np.array_equal(bits(O.create_dynamic_map(**kw)), bits(golden[key]))


def test_package_dynamic_map_bitwise(golden):
    import bnb_b200
    m = bnb_b200.create_dynamic_map().numpy()
    assert np.array_equal(bits(m), bits(golden["dynamic_map"]))


def test_nf4_code_choice_matches_reference(golden):
    got = O.codes_nf4(golden["nf4_code_in"])
    assert np.array_equal(got, golden["nf4_code_out"])


@pytest.mark.parametrize("which", ["dmap", "user"])
def test_8bit_code_choice_matches_reference(golden, which):
    code, xin, xout = ((golden["dynamic_map"], golden["q8_code_in"], golden["q8_code_out"])
                       if which == "dmap" else
                       (golden["q8_user_code"], golden["q8_user_in"], golden["q8_user_out"]))
    assert np.array_equal(O.codes_8bit(code, xin), xout)
    # the threshold-count restatement the CUDA kernel evaluates
    T = O.q8_thresholds(code)
    assert T is not None and np.all(np.diff(T) >= 0)
    assert np.array_equal(O.codes_8bit_count(T, xin), xout)


def test_blocksize_validation_matches_reference(golden):
    from bnb_b200.kernels.dequantize import _log2_blocksize
    for bs, l2 in zip(golden["log2_blocksizes"], golden["log2_values"]):
        assert _log2_blocksize(int(bs)) == int(l2)
    for bs in golden["log2_rejected"]:
        with pytest.raises(ValueError, match="power of two"):
            _log2_blocksize(int(bs))


def test_gemv_constants_match_reference(golden):
    from bnb_b200.kernels import gemv
    assert gemv.GEMV_MAX_M == int(golden["gemv_max_m"])
    assert [gemv._rows_per_warp(m) for m in range(1, 21)] == golden["rows_per_warp"].tolist()


# ---- the reference test suite's known answers, restated on the oracle ----

def test_kat_nf4_thresholds():
    """Values on and one ulp either side of each threshold, in blocks whose
    absmax is 1, so the scaled value is the value itself (reference
    tests/test_quantize.py:90-99). rcp(1) = 1 is exact."""
    t = O.NF4_THRESHOLDS
    vals = np.concatenate([t, np.nextafter(t, np.float32(np.inf)), np.nextafter(t, np.float32(-np.inf))])
    x = np.zeros(128, np.float32)
    x[:len(vals)] = vals
    x[63] = x[127] = 1.0
    q, am = O.quantize_nf4(x, O.F32, 64, rcp=np.ones(2, np.float32))
    assert np.array_equal(am, [1.0, 1.0])
    codes = np.empty(128, np.uint8)
    codes[0::2], codes[1::2] = q >> 4, q & 15
    j = np.arange(15)
    assert np.array_equal(codes[:15], j)          # on the threshold: not above it
    assert np.array_equal(codes[15:30], j + 1)    # one ulp above
    assert np.array_equal(codes[30:45], j)        # one ulp below
    assert codes[63] == 15 and codes[127] == 15


def test_kat_8bit_midpoints():
    """Values on and one ulp either side of each codebook midpoint
    (reference tests/test_quantize.py:102-114): codes follow the reference's
    search exactly."""
    code = O.create_dynamic_map()
    mid = ((code[1:] + code[:-1]) * np.float32(0.5)).astype(np.float32)
    vals = np.concatenate([code, mid, np.nextafter(mid, np.float32(np.inf)),
                           np.nextafter(mid, np.float32(-np.inf))])
    bs = 256
    x = np.zeros(-(-len(vals) // (bs - 1)) * bs, np.float32)
    for i, start in enumerate(range(0, len(vals), bs - 1)):
        chunk = vals[start:start + bs - 1]
        x[i * bs:i * bs + len(chunk)] = chunk
        x[(i + 1) * bs - 1] = 1.0
    nb = len(x) // bs
    q, am = O.quantize_8bit(x, O.F32, bs, code, rcp=np.ones(nb, np.float32))
    assert np.all(am == 1.0)
    assert np.array_equal(q, O.codes_8bit(code, x))
    # each codebook entry maps to itself
    assert np.array_equal(O.codes_8bit(code, code), np.arange(256))


@pytest.mark.parametrize("nf4", [True, False])
def test_kat_special_values(nf4):
    """All-zero blocks, denormal-only blocks, huge and tiny values, -0.0
    (reference tests/test_quantize.py:117-131)."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal(64 * 6).astype(np.float32)
    x[0:64] = 0.0
    x[64:128] = (rng.standard_normal(64) * 1e-39).astype(np.float32)  # float32 denormals
    x[128:192] *= np.float32(1e30)
    x[192:256] = -x[192:256] * np.float32(1e-30)
    x[256] = -0.0
    if nf4:
        q, am, amb = O.quantize_nf4(x, O.F32, 64, want_ambiguous=True)
        codes = np.empty(x.size, np.uint8)
        codes[0::2], codes[1::2] = q >> 4, q & 15
        # zero and denormal-only blocks: absmax 0, r = inf, 0 * inf = NaN -> code 0
        assert am[0] == 0.0 and am[1] == 0.0
        assert np.all(codes[:128] == 0)
        assert codes[256] == 7  # -0.0 in a normal block decodes to the 0.0 code
    else:
        code = O.create_dynamic_map()
        q, am, amb = O.quantize_8bit(x, O.F32, 64, code, want_ambiguous=True)
        assert am[0] == 0.0 and am[1] == 0.0
        assert np.all(q[:128] == 0)  # NaN walks the search down to code 0
        assert q[256] == 127         # -0.0 -> the codebook's 0.0
    assert amb.mean() < 0.02


@pytest.mark.parametrize("dtype", [O.F32, O.F16, O.BF16])
def test_oracle_roundtrip_idempotent(dtype):
    """dequantize(quantize(x)) re-quantizes to the same codes and absmax."""
    x = host_input(np.random.default_rng(3).standard_normal(3 * 64 + 5).astype(np.float32), dtype)
    q, am = O.quantize_nf4(x, dtype, 64)
    y = O.dequantize_nf4(q, am, x.size, 64, O.F32)
    q2, am2 = O.quantize_nf4(y, O.F32, 64)
    assert np.array_equal(bits(am), bits(am2))
    assert np.array_equal(q, q2)


def test_oracle_nested_chain_equals_two_steps():
    """The fused nested decode equals 8-bit dequantize(f32) + offset, then
    NF4 with the decoded scales (reference array.py:95-108)."""
    rng = np.random.default_rng(5)
    am = np.abs(rng.standard_normal(1000)).astype(np.float32) * np.float32(0.05)
    off = O.mean_f32(am)
    code = O.create_dynamic_map()
    q2, am2 = O.quantize_8bit(am, O.F32, 256, code, offset=off)
    step = O.dequantize_8bit(q2, am2, code, 256, O.F32, offset=off)
    fused = O.nested_absmax(q2, am2, code, off, 256)
    assert np.array_equal(bits(step), bits(fused))
    assert np.max(np.abs(fused - am)) < 0.05 * np.max(am)
