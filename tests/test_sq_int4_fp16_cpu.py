"""INT4 and FP16 scalar quantization on the host: the oracle's INT4 codes and
QuantizedDistance against the reference's own test values
(quantization_test.go:66-79, 95-135) and the binary16 conversion of the
library's FP16 kind (quantize_fp16) against the oracle's restatement of
utility.Float32ToFloat16Bits."""
import json
import os

import numpy as np
import pytest

from oracle.oracle import COSINE, IP, L2, MIPSL2, OK

FIX = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_fixtures.json")))


def int4_decode(packed, p, d):
    codes = np.empty(d, np.int32)
    codes[0::2] = packed & 0x0F
    codes[1::2] = packed >> 4
    codes[codes >= 8] -= 16
    return np.float32(p.inverse_scale) * codes.astype(np.float32) + np.float32(p.offset)


def test_int4_decoded_fixture(oracle):
    f = FIX["int4"]
    st, packed, p = oracle.quantize_int4(f["input"])
    assert st == OK
    assert np.allclose(int4_decode(packed, p, 4), np.float32(f["decoded"]), atol=1e-6)


def test_int4_distance_matches_decoded(oracle):
    f = FIX["quantized_vs_decoded"]
    st, lc, lp = oracle.quantize_int4(f["left"])
    st2, rc, rp = oracle.quantize_int4(f["right"])
    assert st == OK and st2 == OK
    ldec, rdec = int4_decode(lc, lp, 4), int4_decode(rc, rp, 4)
    for metric in (L2, IP, COSINE, MIPSL2):
        _, want = oracle.metric_compute(metric, ldec, rdec)
        st, got = oracle.quantized_distance_int4(metric, lc, lp, rc, rp, 4)
        assert st == OK
        assert abs(float(got) - float(want)) <= 2e-5 * max(1, abs(float(want)))


def test_int4_zero_vectors_and_odd_dimension(oracle):
    """quantization_test.go:119-135 and :210-213."""
    _, zc, zp = oracle.quantize_int4([0, 0])
    _, uc, up = oracle.quantize_int4([1, 0])
    for metric, left, right, want in ((COSINE, (zc, zp), (zc, zp), 0.0),
                                      (COSINE, (zc, zp), (uc, up), 1.0),
                                      (MIPSL2, (zc, zp), (zc, zp), 0.0)):
        st, got = oracle.quantized_distance_int4(metric, left[0], left[1], right[0], right[1], 2)
        assert st == OK and got == want
    st, _, _ = oracle.quantize_int4([1.0])
    assert st != OK
    _, _, p = oracle.quantize_int4([3.5, 3.5])
    assert p.inverse_scale == 0 and p.offset == 3.5


def test_int4_search_matches_brute_force(oracle):
    """xo_sq4_search equals scoring every row with QuantizedDistanceToFloat."""
    rng = np.random.default_rng(3)
    x = rng.standard_normal((300, 12)).astype(np.float32)
    q = rng.standard_normal((4, 12)).astype(np.float32)
    keys = rng.permutation(1 << 16)[:300].astype(np.uint64)
    packed, params = oracle.quantize_int4_batch(x)
    for metric in (L2, IP, COSINE, MIPSL2):
        st, ok, os_, oc, _ = oracle.sq4_search(metric, packed, params, x, keys, q, 7)
        assert st == OK
        for qi in range(4):
            _, qc, qp = oracle.quantize_int4(q[qi])
            from oracle.oracle import SQParams
            sc = []
            for r in range(300):
                rp = SQParams(*params[r].tolist())
                sc.append(oracle.quantized_distance_int4(metric, packed[r], rp, qc, qp, 12)[1])
            sc = np.array(sc, np.float32)
            order = sorted(range(300), key=lambda r: ((-sc[r]) if metric == IP else sc[r], keys[r]))
            assert list(ok[qi, :7]) == [keys[r] for r in order[:7]]
            assert np.array_equal(os_[qi, :7], sc[order[:7]])


def test_quantize_fp16_reference_values(oracle):
    """TestQuantizeFP16 (quantization_test.go:28-47) and the overflow case
    (:206-209)."""
    import xvec_b200
    f = FIX["fp16"]
    half, st = xvec_b200.quantize_fp16(L2, np.float32([f["input"]]))
    assert st[0] == OK
    assert list(half[0].astype("<u2").view(np.uint8)) == f["code_bytes"]
    _, st = xvec_b200.quantize_fp16(L2, np.float32([[np.finfo(np.float32).max, 0]]))
    assert st[0] == xvec_b200.OVERFLOW


def test_quantize_fp16_matches_oracle(oracle):
    import xvec_b200
    rng = np.random.default_rng(11)
    v = (rng.standard_normal((64, 40)) * rng.choice([1e-7, 1e-3, 1, 300, 3e4], (64, 1))).astype(
        np.float32)
    v[3, 5] = 65519.0     # rounds down to 65504
    v[4, 6] = 65520.0     # rounds to infinity: ErrQuantizationOverflow
    v[5, 7] = np.nan      # rejected by the metric validation first
    v[6, 8] = 2.98e-8     # below half the smallest subnormal: +0
    for metric in (L2, IP):
        half, st = xvec_b200.quantize_fp16(metric, v)
        assert st[4] == xvec_b200.OVERFLOW and st[5] == xvec_b200.NON_FINITE
        finite = np.isfinite(v).all(axis=1)
        big = (np.abs(v) >= 65520.0).any(axis=1)
        assert np.array_equal(st == xvec_b200.OVERFLOW, finite & big)
        ok = np.flatnonzero(st == OK)
        assert 3 in ok and 6 in ok
        want = oracle.f32_to_f16(v[ok].reshape(-1)).reshape(ok.size, -1)
        assert np.array_equal(half[ok], want)
    _, st = xvec_b200.quantize_fp16(IP, np.full((1, 4), 3e19, np.float32))
    assert st[0] == xvec_b200.NON_FINITE      # metric.Compute(v, v) overflows first
    _, st = xvec_b200.quantize_fp16(L2, np.full((1, 4), 3e19, np.float32))
    assert st[0] == xvec_b200.OVERFLOW
