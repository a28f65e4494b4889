"""The lookup formulations the CUDA quantize kernels evaluate, checked on the
CPU against the reference's literal algorithms (restated in the oracle, which
test_oracle_golden pins to the reference's own outputs)."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from helpers import GEMV_ATOL, GEMV_RTOL


def test_nf4_bucket_lookup_exhaustive():
    """code = base[i] + (s > thr[i]) with i = bits(fma(max(s,-1), 16, 2^23+16)) & 63
    equals the 15-compare count for EVERY float32 s in [-1.01, 1.01], NaN and -inf."""
    thr, base = O.nf4_bucket_tables()
    assert np.sum(np.isfinite(thr)) == 15  # one bucket per threshold
    assert O.check_nf4_buckets(stride=1) == 0


def _random_codebooks(n, seed):
    rng = np.random.default_rng(seed)
    books = []
    for i in range(n):
        c = np.sort(rng.uniform(-1.0, 1.0, 256).astype(np.float32))
        c = np.unique(c)
        while c.size < 256:
            c = np.unique(np.concatenate([c, rng.uniform(-1, 1, 256 - c.size).astype(np.float32)]))
        if i % 2:
            c = np.sort(np.sign(c) * np.abs(c) ** 3).astype(np.float32)  # dense near 0
        books.append(c)
    return books


def test_q8_bucket_table_dynamic_map():
    """The 8-bit kernel's one-lookup code choice (a threshold per bucket of
    sign, exponent and mb mantissa bits; code = (E +- low bits) >> 24) == the
    reference's binary search, dynamic map, every 3rd float32 bit pattern in
    [-1.01, 1.01], every threshold +-3 ulp, NaN, infinities, zeros."""
    bad, mb = O.check_q8_buckets(O.create_dynamic_map(), stride=3)
    assert bad == 0
    assert mb == 7


def _common_codebooks():
    """Codebooks of the bitsandbytes family besides the signed dynamic map:
    the unsigned dynamic map, a linear map and a normal-quantile map."""
    from statistics import NormalDist
    lin = np.linspace(-1.0, 1.0, 256).astype(np.float32)
    nd = NormalDist()
    q = np.array([nd.inv_cdf((i + 0.5) / 256) for i in range(256)])
    quant = (q / np.abs(q).max()).astype(np.float32)
    return {"dynamic_unsigned": O.create_dynamic_map(False).astype(np.float32), "linear": lin, "quantile": quant}


@pytest.mark.parametrize("name", ["dynamic_unsigned", "linear", "quantile"])
def test_q8_bucket_table_common_codebooks(name):
    code = _common_codebooks()[name]
    bad, mb = O.check_q8_buckets(code, stride=97)
    assert bad == 0 and mb >= 5, (bad, mb)


@pytest.mark.parametrize("seed", [1, 2])
def test_q8_bucket_table_random_codebooks(seed):
    """Uniformly random codebooks: exact where the table applies; where two
    thresholds are closer than the finest bucket it is declined (the kernel
    then runs the literal search, checked on the GPU)."""
    for code in _random_codebooks(2, seed):
        bad, mb = O.check_q8_buckets(code, stride=97)
        assert bad == 0 or (bad == -1 and mb == -1), (bad, mb)


def test_q8_bucket_table_declines_crowded_codebooks():
    """Thresholds closer than the finest bucket (here: codes 1 ulp apart) ->
    the table formulation is refused; the kernel runs the literal search."""
    code = O.create_dynamic_map().astype(np.float32).copy()
    code[200] = np.nextafter(code[201], np.float32(-np.inf))
    code[199] = np.nextafter(code[200], np.float32(-np.inf))
    assert np.all(np.diff(code) > 0)
    bad, mb = O.check_q8_buckets(code, stride=1 << 20)
    assert bad == -1 and mb == -1


def test_q8_thresholds_reject_unsorted():
    code = O.create_dynamic_map().copy()
    code[10], code[11] = code[11], code[10]
    assert O.q8_thresholds(code) is None
    code = O.create_dynamic_map().copy()
    code[-1] = np.inf
    assert O.q8_thresholds(code) is None


def test_q8_count_equals_search_near_every_threshold():
    code = O.create_dynamic_map()
    T = O.q8_thresholds(code)
    vals = [T]
    up, dn = T.copy(), T.copy()
    for _ in range(4):
        up = np.nextafter(up, np.float32(np.inf))
        dn = np.nextafter(dn, np.float32(-np.inf))
        vals += [up, dn]
    v = np.concatenate(vals).astype(np.float32)
    assert np.array_equal(O.codes_8bit_count(T, v), O.codes_8bit(code, v))


def test_ambiguity_is_rare_and_absent_with_device_rcp():
    """Without the device's reciprocals only a small fraction of codes depend
    on rcp.approx's exact value; with them (here: stand-in values) none do."""
    x = np.random.default_rng(7).standard_normal(1 << 16).astype(np.float32)
    _, am, amb = O.quantize_nf4(x, O.F32, 64, want_ambiguous=True)
    assert amb.mean() < 1e-3
    r = np.empty_like(am)
    O.lib().or_rcp_ieee_ftz(O._p(am), O._p(r), am.size)
    _, _, amb2 = O.quantize_nf4(x, O.F32, 64, rcp=r, want_ambiguous=True)
    assert not amb2.any()


def test_gemv_reference_numerics_close_to_f64():
    """The reference GEMV's float32 numerics against the float64 product."""
    rng = np.random.default_rng(11)
    n, k = 64, 1024
    w = rng.standard_normal(n * k).astype(np.float32)
    q, am = O.quantize_nf4(w, O.F32, 64)
    x = O.f32_to_bf16(rng.standard_normal((3, k)).astype(np.float32)).reshape(3, k)
    y64, yabs = O.gemv_f64(x, O.BF16, q, n, 64, am)
    yref = O.bf16_to_f32(O.gemv_ref(x, O.BF16, q, n, 64, am)).reshape(3, n)
    assert np.all(np.abs(yref - y64) <= GEMV_RTOL * np.abs(y64) + GEMV_ATOL * yabs)
