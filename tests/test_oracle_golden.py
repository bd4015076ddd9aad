"""Pins the CPU oracle to the reference: its known-answer tests (tests/golden/
reference_fixtures.json, transcribed from the Go test sources) and its own
AVX-512/AVX C kernels compiled in place (oracle/_ref)."""
import json
import math
import os

import numpy as np
import pytest

from oracle.oracle import COSINE, IP, L2, MIPSL2, NON_FINITE, OK, ReferenceFloats

FIX = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_fixtures.json")))


def test_flat_metrics_fixture(oracle):
    f = FIX["flat_metrics"]
    keys = np.array([c[0] for c in f["candidates"]], np.uint64)
    rows = np.array([c[1] for c in f["candidates"]], np.float32)
    for metric, want in f["want"].items():
        st, k, s, c, _ = oracle.flat_search(int(metric), rows, keys, np.array([f["query"]]), f["k"])
        assert st == OK
        got = [[int(k[0, i]), float(s[0, i])] for i in range(c[0])]
        assert got == want, (metric, got)


def test_metric_values(oracle):
    for metric, left, right, want, tol in FIX["metric_values"]["cases"]:
        st, s = oracle.metric_compute(metric, left, right)
        assert st == OK
        assert abs(float(s) - want) <= tol


def test_zero_vectors(oracle):
    for metric, left, right, want in FIX["zero_vectors"]["cases"]:
        st, s = oracle.metric_compute(metric, left, right)
        assert st == OK and float(s) == want


def test_cosine_extremes(oracle):
    for left, right, want in FIX["cosine_extremes"]["cases"]:
        st, s = oracle.metric_compute(COSINE, left, right)
        assert st == OK and abs(float(s) - want) <= 1e-6


def test_validation_errors(oracle):
    st, _ = oracle.metric_compute(IP, [np.float32(np.nan)], [1])
    assert st == NON_FINITE
    big = np.float32(3.4028235e38)
    st, _ = oracle.metric_compute(IP, [big, big], [big, big])
    assert st == NON_FINITE


def test_float32_accumulation(oracle):
    f = FIX["float32_accumulation"]
    assert oracle.inner_product(*f["ip_zero"]) == 0.0
    assert oracle.inner_product(*f["two_pow_24"]) == float(1 << 24)
    dn = oracle.dot_norms(*f["two_pow_24"])
    assert list(dn) == [float(1 << 24)] * 3


def test_fp16_fixture(oracle):
    f = FIX["fp16"]
    bits = oracle.f32_to_f16(f["input"])
    assert list(bits.astype("<u2").view(np.uint8)) == f["code_bytes"]
    assert list(oracle.f16_to_f32(bits)) == f["decoded"]


def test_fp16_matches_numpy_round_to_nearest_even(oracle):
    rng = np.random.default_rng(5)
    vals = np.concatenate([rng.standard_normal(2000).astype(np.float32) * 10,
                           np.float32([6.1e-5, 5.96e-8, 2.98e-8, 2.99e-8, 65504, 65520, 1e-9])])
    ours = oracle.f32_to_f16(vals)
    with np.errstate(over="ignore"):
        want = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(ours, want)
    back = oracle.f16_to_f32(ours)
    assert np.array_equal(back, ours.view(np.float16).astype(np.float32))


def test_int8_fixture(oracle):
    f = FIX["int8"]
    st, codes, p = oracle.quantize_int8(f["input"])
    assert st == OK
    assert list(codes.view(np.uint8)) == f["code_bytes"]
    assert abs(p.inverse_scale - f["inverse_scale"]) <= 1e-8
    assert p.offset == f["offset"]


def test_int4_fixture(oracle):
    f = FIX["int4"]
    st, packed, p = oracle.quantize_int4(f["input"])
    assert st == OK and list(packed) == f["code_bytes"]


def test_constant_vector(oracle):
    f = FIX["constant_vector"]
    st, codes, p = oracle.quantize_int8(f["input"])
    assert st == OK and p.inverse_scale == 0 and p.offset == 3.5 and not codes.any()


def test_quantized_distance_matches_decoded(oracle):
    f = FIX["quantized_vs_decoded"]
    st, lc, lp = oracle.quantize_int8(f["left"])
    st2, rc, rp = oracle.quantize_int8(f["right"])
    assert st == OK and st2 == OK
    ldec = np.float32(lp.inverse_scale) * lc.astype(np.float32) + np.float32(lp.offset)
    rdec = np.float32(rp.inverse_scale) * rc.astype(np.float32) + np.float32(rp.offset)
    for metric in (L2, IP, COSINE, MIPSL2):
        _, want = oracle.metric_compute(metric, ldec, rdec)
        st, got = oracle.quantized_distance_int8(metric, lc, lp, rc, rp)
        assert st == OK
        assert abs(float(got) - float(want)) <= 2e-5 * max(1, abs(float(want)))


def _pq_fixture(metric):
    pivots = np.zeros((256, 4), np.float32)
    for c in range(256):
        if metric == L2:
            pivots[c, 0] = c
            pivots[c, 3] = c
        else:
            pivots[c, 0] = 1
            pivots[c, 2] = 1
    if metric == IP:
        pivots.reshape(-1)[4:8] = [0, 1, 0, 1]
    return pivots, np.array([0, 2, 4], np.int32)


def test_pq_l2_fixture(oracle):
    f = FIX["pq_l2"]
    pivots, offsets = _pq_fixture(L2)
    st, code = oracle.pq_encode(L2, pivots, offsets, f["vector"])
    assert st == OK and list(code) == f["code"]
    st, table = oracle.pq_distance_table(L2, pivots, offsets, f["query"])
    assert st == OK
    for idx, val in f["table_entries"]:
        assert table[idx] == val
    st, score = oracle.pq_lookup(table, code)
    assert st == OK and score == f["lookup"]


def test_pq_ip_fixture(oracle):
    f = FIX["pq_ip"]
    pivots, offsets = _pq_fixture(IP)
    st, table = oracle.pq_distance_table(IP, pivots, offsets, f["query"])
    for vec, want_code, want_score in zip(f["vectors"], f["codes"], f["scores"]):
        st, code = oracle.pq_encode(IP, pivots, offsets, vec)
        assert st == OK and list(code) == want_code
        st, score = oracle.pq_lookup(table, code)
        assert st == OK and score == want_score


def test_pq_chunk_offsets_wider_first(oracle):
    assert list(oracle.pq_chunk_offsets(10, 4)) == [0, 3, 6, 8, 10]
    assert list(oracle.pq_chunk_offsets(128, 32)) == list(range(0, 129, 4))


def test_kmeans_reservoir_fixture(oracle):
    f = FIX["kmeans_reservoir"]
    idx = oracle.kmeans_reservoir(len(f["vectors"]), f["clusters"], f["seed"])
    assert [f["vectors"][i] for i in idx] == f["centroids"]


def test_kmeans_tie_lower_index(oracle):
    f = FIX["kmeans_tie"]
    st, labels, scores = oracle.kmeans_assign(L2, np.array([f["vector"]]), np.array(f["centroids"]))
    assert st == OK and labels[0] == f["label"] and scores[0] == f["score"]


def test_fht_rotator_fixture(oracle):
    f = FIX["fht_rotator"]
    st, out = oracle.fht_rotate(f["signs"], f["input"])
    assert st == OK
    assert np.allclose(out, f["rotated"], atol=1e-6)


def test_rabitq_pinned_library_fixture(oracle):
    f = FIX["rabitq_pinned"]
    idx = np.arange(64)
    vec = ((idx * 17 % 29) - 14).astype(np.float32) * np.float32(0.125)
    cen = ((idx * 5 % 11) - 5).astype(np.float32) * np.float32(0.05)
    for metric, want in f["factors"].items():
        st, binary, extra, fac = oracle.rabitq_quantize(vec, cen, 0, f["total_bits"],
                                                        f["extra_scale"], int(metric) == IP)
        assert st == OK
        eb = f["total_bits"] - 1
        bits = np.unpackbits(binary, bitorder="little")
        ebits = np.unpackbits(extra, bitorder="little")
        values = [int(sum(int(ebits[i * eb + b]) << b for b in range(eb)) | (int(bits[i]) << eb))
                  for i in range(64)]
        assert values == f["values"]
        got = [fac.coarse_add, fac.coarse_rescale, fac.coarse_error, fac.full_add, fac.full_rescale]
        for g, w in zip(got, want):
            assert abs(g - w) <= 2e-6 * max(1, abs(w))


@pytest.mark.skipif(not ReferenceFloats.available(), reason="reference kernels not built or no AVX-512")
def test_restated_kernels_bit_identical_to_reference_c():
    """floats_test.go:26-51 dims, unaligned; bit-identical against the compiled reference C."""
    from oracle.oracle import Oracle
    ref = ReferenceFloats()
    ora = Oracle()
    for d in [8, 9, 15, 16, 17, 31, 127, 128, 129, 768, 960, 1024, 1536]:
        rng = np.random.default_rng(d)
        buf_a = rng.uniform(-1, 1, d + 1).astype(np.float32)
        buf_b = rng.uniform(-1, 1, d + 1).astype(np.float32)
        a, b = buf_a[1:], buf_b[1:]
        assert ref.l2_squared(a, b) == ora.l2_squared(a, b), d
        assert ref.inner_product(a, b) == ora.inner_product(a, b), d
        assert np.array_equal(ref.dot_norms(a, b), ora.dot_norms(a, b)), d


def test_flat_search_brute_force_equivalence(oracle):
    """Ranking rules of topk.go:105-166 against a direct float64-free sort."""
    rng = np.random.default_rng(3)
    rows = rng.standard_normal((500, 24)).astype(np.float32)
    rows[100] = rows[7]  # exact duplicate: tie broken by key
    keys = rng.permutation(10_000)[:500].astype(np.uint64)
    q = rng.standard_normal((3, 24)).astype(np.float32)
    q[0] = rows[7]
    for metric in (L2, IP, COSINE, MIPSL2):
        st, ok, os_, oc, _ = oracle.flat_search(metric, rows, keys, q, 20)
        assert st == OK
        for qi in range(3):
            scores = [oracle.metric_compute(metric, rows[i], q[qi])[1] for i in range(500)]
            sign = -1 if metric == IP else 1
            order = sorted(range(500), key=lambda i: (sign * float(scores[i]), int(keys[i])))[:20]
            assert [int(keys[i]) for i in order] == [int(x) for x in ok[qi]]


def test_merge_results_order_independent(oracle):
    """query_test.go:113-136: merging is independent of batch order."""
    rng = np.random.default_rng(9)
    keys = rng.permutation(1000)[:200].astype(np.uint64)
    scores = rng.integers(0, 20, 200).astype(np.float32)
    a = oracle.merge_results(L2, 15, keys, scores)
    perm = rng.permutation(200)
    b = oracle.merge_results(L2, 15, keys[perm], scores[perm])
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


@pytest.mark.skipif(not ReferenceFloats.available(), reason="reference kernels not built or no AVX-512")
def test_flat_search_same_with_reference_kernels():
    from oracle.oracle import Oracle
    ora = Oracle()
    rng = np.random.default_rng(8)
    rows = rng.standard_normal((800, 96)).astype(np.float32)
    keys = np.arange(800, dtype=np.uint64)
    q = rng.standard_normal((5, 96)).astype(np.float32)
    a = ora.flat_search(COSINE, rows, keys, q, 10)
    ora.use_reference_kernels(ReferenceFloats())
    try:
        b = ora.flat_search(COSINE, rows, keys, q, 10)
    finally:
        ora.use_reference_kernels(None)
    assert np.array_equal(a[1], b[1]) and np.array_equal(a[2], b[2])


@pytest.mark.parametrize("metric", [L2, IP, COSINE, MIPSL2])
def test_ivf_sq8_is_sq8_over_the_probed_lists(oracle, metric):
    """ScalarQuantizedIVFIndex.search (ivf_quantized.go:135-192) is the SQ8
    search (quantized_index.go:313-335) restricted to the positions of the
    probed lists: per query, the SQ8 search with a filter holding exactly
    those positions gives the same keys and scores (refine included)."""
    rng = np.random.default_rng(40 + metric)
    n, d, nlist = 700, 20, 9
    rows = rng.standard_normal((n, d)).astype(np.float32)
    keys = rng.permutation(50_000)[:n].astype(np.uint64)
    queries = rng.standard_normal((6, d)).astype(np.float32)
    centroids = rows[:nlist].copy()
    st, labels, _ = oracle.kmeans_assign(metric, rows, centroids)
    assert st == OK
    offsets = np.cumsum(np.concatenate([[0], np.bincount(labels, minlength=nlist)])).astype(np.int64)
    positions = np.argsort(labels, kind="stable").astype(np.int64)
    codes, params = oracle.quantize_int8_batch(rows)
    for nprobe, scale in ((3, 0.0), (3, 2.5), (nlist, 0.0)):
        st, ok, os_, oc, ost = oracle.ivf_sq8_search(metric, codes, params, rows, keys, centroids,
                                                     offsets, positions, queries, 12, nprobe,
                                                     refine_scale=scale)
        assert st == OK and (ost == 0).all()
        for q in range(queries.shape[0]):
            lists = oracle.ivf_probe(metric, centroids, queries[q], nprobe)
            bitmap = np.zeros((n + 31) // 32, np.uint32)
            for li in lists:
                for p in positions[offsets[li]:offsets[li + 1]]:
                    bitmap[p >> 5] |= np.uint32(1 << int(p & 31))
            _, fk, fs, fc, _ = oracle.sq8_search(metric, codes, params, rows, keys,
                                                 queries[q:q + 1], 12, refine_scale=scale,
                                                 bitmap=bitmap)
            assert oc[q] == fc[0]
            assert np.array_equal(ok[q, :oc[q]], fk[0, :fc[0]])
            assert np.array_equal(os_[q, :oc[q]].view(np.uint32), fs[0, :fc[0]].view(np.uint32))


@pytest.mark.parametrize("metric", [L2, IP])
def test_rabitq_full_estimate(oracle, metric):
    """Estimate (rabitq.go:434-446) on multi-bit codes: the oracle against a
    direct numpy evaluation of raBitQFullCodeDot and the estimate formula, and
    the estimate tracking the true distance more closely as TotalBits grows."""
    rng = np.random.default_rng(11 + metric)
    d, n = 96, 200
    cents = rng.standard_normal((4, d)).astype(np.float32)
    rows = (cents[rng.integers(0, 4, n)] + 0.4 * rng.standard_normal((n, d))).astype(np.float32)
    q = (cents[1] + 0.4 * rng.standard_normal(d)).astype(np.float32)
    padded = oracle.rabitq_padded_dimension(d)
    signs = rng.integers(0, 256, 4 * padded // 8, dtype=np.uint8)
    st, rot, qsum, gadd, gerr = oracle.rabitq_prepare_query(metric, cents, signs, q)
    assert st == OK
    errs = {}
    for tb, scale in ((1, 0.0), (4, 5.2), (7, 15.75)):
        codes, extra, fac = oracle.rabitq_encode_batch(metric, cents, signs, rows, tb, scale)
        eb = tb - 1
        est = np.zeros(n)
        for i in range(n):
            st, e = oracle.rabitq_estimate(rot, qsum, gadd, gerr, tb, codes[i],
                                           extra[i] if eb else None, fac[i])
            assert st == OK
            est[i] = e
            if eb:
                bits = np.unpackbits(codes[i], bitorder="little")[:padded]
                xb = np.unpackbits(extra[i], bitorder="little")
                vals = [int(sum(int(xb[j * eb + b]) << b for b in range(eb))) | (int(bits[j]) << eb)
                        for j in range(padded)]
                dot = 0.0
                for j in range(padded):
                    dot += float(vals[j]) * float(rot[j])
                center = -((1 << eb) - 0.5)
                c = int(fac[i]["cluster"])
                want = fac[i]["full_add"] + gadd[c] + fac[i]["full_rescale"] * (dot + center * qsum)
                assert e == np.float32(want), (tb, i)
        truth = ((rows - q) ** 2).sum(1) if metric == L2 else 1.0 - rows @ q
        errs[tb] = np.abs(est - truth).mean()
    assert errs[7] < errs[4] < errs[1], errs


def test_pq_kmc2_seed_fixture(oracle):
    """TestPQKMC2SeedFixture (pq_test.go:59-66)."""
    st, cents = oracle.pq_kmc2(L2, np.arange(6, dtype=np.float32)[:, None], 3, 0)
    assert st == OK
    assert cents[:, 0].tolist() == [1.0, 5.0, 3.0]


def test_pq_train_prefix_and_padding(oracle):
    """TrainPQ (pq.go:107-179): the codebook depends only on the first
    MaxTrainSamples rows; each chunk is KMC2-seeded k-means with its own seed;
    with fewer than 256 samples the remaining pivots repeat centroid 0."""
    rng = np.random.default_rng(2)
    v = rng.standard_normal((700, 8)).astype(np.float32)
    st, a = oracle.pq_train(L2, v, 4, max_train_samples=500, max_iterations=5, seed=9)
    assert st == OK
    w = v.copy()
    w[500:] = rng.standard_normal((200, 8))
    st, b = oracle.pq_train(L2, w, 4, max_train_samples=500, max_iterations=5, seed=9)
    assert st == OK and np.array_equal(a, b)
    offsets = oracle.pq_chunk_offsets(8, 4)
    for c in range(4):
        lo, hi = offsets[c], offsets[c + 1]
        seed = 9 ^ (0x70716b6d00000000 + c)
        st, init = oracle.pq_kmc2(L2, v[:500, lo:hi], 256, seed)
        st, cents, _ = oracle.kmeans_train_init(L2, v[:500, lo:hi], init, 5)
        assert np.array_equal(a[:, lo:hi], cents)
    st, small = oracle.pq_train(IP, v[:100], 4, max_iterations=3, seed=1)
    assert st == OK
    assert np.array_equal(small[100:], np.repeat(small[:1], 156, axis=0))


@pytest.mark.parametrize("metric", [L2, IP, COSINE, MIPSL2])
def test_ivf_full_probe_matches_flat(oracle, metric):
    """TestIVFFullProbeMatchesFlat (ivf_test.go:324-345): probing every list
    returns exactly the Flat top-k (cosine with cached magnitudes included)."""
    keys = np.array([9, 2, 7, 4, 1, 8], np.uint64)
    vecs = np.array([[-2, 1, 0], [1, 0, 2], [0, 3, -1], [2, 2, 2], [-1, -1, 1], [4, 0, -2]],
                    np.float32)
    q = np.array([[1, 2, 0.5]], np.float32)
    cents = vecs[[0, 2, 5]].copy()
    st, labels, _ = oracle.kmeans_assign(metric, vecs, cents)
    assert st == OK
    offsets = np.cumsum(np.concatenate([[0], np.bincount(labels, minlength=3)])).astype(np.int64)
    positions = np.argsort(labels, kind="stable").astype(np.int64)
    _, ik, isc, ic, _ = oracle.ivf_flat_search(metric, vecs, keys, cents, offsets, positions, q, 6, 3)
    _, fk, fs, fc, _ = oracle.flat_search(metric, vecs, keys, q, 6)
    assert ic[0] == fc[0] == 6
    assert np.array_equal(ik, fk)
    assert np.array_equal(isc.view(np.uint32), fs.view(np.uint32))
