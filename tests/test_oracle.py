"""CPU tests of the oracle (test infrastructure): pinned against the
reference's own output, plus known-answer tests and layout checks."""

import hashlib
import json
import os

import numpy as np
import pytest

import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _manifest():
    with open(os.path.join(GOLDEN, "smoke_golden.json")) as f:
        return json.load(f)["cases"]


@pytest.fixture(scope="module")
def golden_arrays():
    return np.load(os.path.join(GOLDEN, "smoke_golden.npz"))


_WEIGHTS = {}


def _weights(n, k, seed):
    if (n, k, seed) not in _WEIGHTS:
        _WEIGHTS.clear()
        _WEIGHTS[(n, k, seed)] = oracle.gen_weight_smoke(n, k, seed)
    return _WEIGHTS[(n, k, seed)]


@pytest.mark.parametrize("case", _manifest(), ids=lambda c: c["name"])
def test_oracle_matches_reference_golden(case, golden_arrays):
    """Generators by hash and the GEMM bit-for-bit against fixtures produced by
    the reference's kernels/smoke_test.cu host code."""
    w, ws = _weights(case["N"], case["K"], case["weight_seed"])
    assert _sha(w) == case["sha_weight"]
    assert _sha(ws) == case["sha_weight_scales"]
    a, as_ = oracle.gen_activation_smoke(case["M"], case["K"], case["act_seed"])
    assert _sha(a) == case["sha_act"]
    assert _sha(as_) == case["sha_act_scales"]
    out = oracle.compute_reference(a, as_, w, ws, threads=8)
    want = oracle.bf16_bits_to_f32(golden_arrays[case["name"]])
    assert np.array_equal(out.view(np.uint32), want.view(np.uint32))


def test_act_seed_mix_matches_reference_formula():
    # kernels/smoke_test.cu:523: seed ^ (0x9e3779b97f4a7c15 * m), 64-bit wrap
    assert oracle.smoke_act_seed(0x5EED1234, 1) == 0x5EED1234 ^ 0x9E3779B97F4A7C15
    assert oracle.smoke_act_seed(0, 2) == (0x9E3779B97F4A7C15 * 2) & (2**64 - 1)


@pytest.mark.parametrize("n,k,m,seed", [(130, 256, 2, 3), (384, 512, 5, 0xABCDEF01)])
def test_oracle_matches_reference_build(n, k, m, seed):
    """Direct comparison with the reference build when it is present."""
    ref = oracle.load_ref()
    if ref is None:
        pytest.skip("oracle/_ref not built (reference checkout absent)")
    w1, s1 = oracle.gen_weight_smoke(n, k, seed)
    w2, s2 = oracle.gen_weight_smoke(n, k, seed, lib=ref)
    assert np.array_equal(w1, w2) and np.array_equal(s1, s2)
    a1, as1 = oracle.gen_activation_smoke(m, k, seed + 1)
    a2, as2 = oracle.gen_activation_smoke(m, k, seed + 1, lib=ref)
    assert np.array_equal(a1, a2) and np.array_equal(as1, as2)
    o1 = oracle.compute_reference(a1, as1, w1, s1)
    o2 = oracle.compute_reference(a1, as1, w1, s1, lib=ref)
    assert np.array_equal(o1.view(np.uint32), o2.view(np.uint32))


def test_fp8_lut_known_values():
    lut = oracle.fp8_lut()
    assert lut[0x00] == 0.0 and lut[0x38] == 1.0 and lut[0xB8] == -1.0
    assert lut[0x7E] == 448.0 and lut[0xFE] == -448.0
    assert lut[0x7F] == 0.0 and lut[0xFF] == 0.0          # NaN patterns -> 0 (smoke_test.cu:67)
    assert lut[0x01] == 2.0 ** -9                          # smallest subnormal


def test_quant_round_trip_on_representable_values():
    lib = oracle.load()
    lut = oracle.fp8_lut()
    for b in range(256):
        if b in (0x7F, 0xFF, 0x80):
            continue
        assert lib.orc_quant_e4m3(float(lut[b])) == b


def test_kat_ones_weights_power_of_two_activations():
    """Known answer (kernels/README.md:576-584): W all 1.0, activation value
    2^j in k_block j, unit scales -> out = 128 * sum_j 2^j exactly."""
    n, k, m = 256, 512, 3
    one = 0x38
    w = np.full((n, k), one, np.uint8)
    a = np.zeros((m, k), np.uint8)
    codes = {1.0: 0x38, 2.0: 0x40, 4.0: 0x48, 8.0: 0x50}
    for kb, v in enumerate((1.0, 2.0, 4.0, 8.0)):
        a[:, kb * 128:(kb + 1) * 128] = codes[v]
    ws = np.ones(((n + 127) // 128, k // 128), np.float32)
    as_ = np.ones((m, k // 128), np.float32)
    out = oracle.compute_reference(a, as_, w, ws)
    assert np.all(out == 128.0 * 15.0)
    # per-block scales enter linearly
    ws2 = ws.copy()
    ws2[1, :] = 0.5
    out2 = oracle.compute_reference(a, as_, w, ws2)
    assert np.all(out2[:, :128] == 1920.0) and np.all(out2[:, 128:] == 960.0)


def test_multithreaded_reference_is_bit_identical():
    w, ws = oracle.gen_weight_smoke(640, 1024, 21)
    a, as_ = oracle.gen_activation_smoke(4, 1024, 22)
    o1 = oracle.compute_reference(a, as_, w, ws, threads=1)
    o8 = oracle.compute_reference(a, as_, w, ws, threads=7)
    assert np.array_equal(o1.view(np.uint32), o8.view(np.uint32))


@pytest.mark.parametrize("bm", [32, 48, 56, 64, 128])
def test_prepack_layout_formula(bm):
    """kernels/weight_prepack.cuh:13-19: packed[((t*KB+kb)*BM+r)*128+k%128] = W[t*BM+r][k]."""
    n, k = 200, 384
    rng = np.random.default_rng(bm)
    w = rng.integers(0, 256, (n, k), dtype=np.uint8)
    packed = oracle.prepack(w, bm)
    tiles = (n + bm - 1) // bm
    kb_count = k // 128
    view = packed.reshape(tiles, kb_count, bm, 128)
    for t in range(tiles):
        for kb in range(kb_count):
            rows = w[t * bm:min(n, (t + 1) * bm), kb * 128:(kb + 1) * 128]
            assert np.array_equal(view[t, kb, :rows.shape[0]], rows)
            assert not view[t, kb, rows.shape[0]:].any()


def test_swizzled_prepack_is_permutation_of_packed():
    n, k, bm = 136, 256, 64
    rng = np.random.default_rng(5)
    w = rng.integers(0, 256, (n, k), dtype=np.uint8)
    plain = oracle.prepack(w, bm).reshape(-1, 8, 16)       # [rows][chunk][16]
    sw = oracle.prepack(w, bm, swizzled=True).reshape(-1, 8, 16)
    for r in range(plain.shape[0]):
        for c in range(8):
            assert np.array_equal(sw[r, c ^ (r % 8)], plain[r, c])


def test_pertensor_generator_properties():
    q, s, scale = oracle.gen_pertensor(300, 512, 1234, scale_rows=3, threads=3)
    q2, s2, scale2 = oracle.gen_pertensor(300, 512, 1234, scale_rows=3, threads=1)
    assert np.array_equal(q, q2) and scale == scale2           # thread-count independent
    assert np.all(s == scale) and s.shape == (3, 4)
    lut = oracle.fp8_lut()
    vals = lut[q]
    assert np.abs(vals).max() == 448.0                          # amax maps to 448
    assert 0.5 < float(np.std(vals * scale)) < 2.0              # N(0,1) draws
    q3, _, _ = oracle.gen_pertensor(300, 512, 1235, scale_rows=3)
    assert not np.array_equal(q, q3)


def test_bench_generators_shapes_and_padding():
    w, s = oracle.gen_weight_bench(200, 256, oracle.BENCH_SEED)
    assert w.shape == (256, 256) and s.shape == (3, 2)
    assert not w[200:].any()                                    # pad rows are zero
    assert np.all(s[2] == 0.0)                                  # guard scale row
    a, sa = oracle.gen_activation_bench(3, 256, oracle.BENCH_SEED)
    assert a.shape == (3, 256) and np.all(sa > 0)


def test_elementwise_check_floor():
    want = np.array([[1.0, -1.0, 0.0, 1e-6]], np.float32)
    ok, worst = oracle.elementwise_ok(want * (1 + 5e-3), want)
    assert ok
    ok, _ = oracle.elementwise_ok(want * 1.05, want)
    assert not ok


def test_quantize_rows_matches_reference_formula_and_torch_e4m3():
    """orc_quantize_rows (bench/bench_decode.cu:459-467): scale =
    max(amax, 1e-4)/448 per row and 128-block, bytes = RN e4m3 of the clamped
    quotient -- cross-checked against torch's float8_e4m3fn conversion, with a
    zero block (scale = 1e-4/448) and large magnitudes."""
    import torch
    rng = np.random.default_rng(3)
    x = rng.standard_normal((6, 512)).astype(np.float32) * np.float32(3.0)
    x[1, 128:256] = 0.0
    x[2, :128] *= np.float32(1e4)
    x = torch.from_numpy(x).bfloat16().float().numpy()
    q, s = oracle.quantize_rows(x)
    blocks = x.reshape(6, 4, 128)
    amax = np.abs(blocks).max(-1)
    assert np.array_equal(s, (np.maximum(amax, np.float32(1e-4)) / np.float32(448)).astype(np.float32))
    assert s[1, 1] == np.float32(np.float32(1e-4) / np.float32(448))
    want = torch.from_numpy(np.clip(blocks / s[..., None], -448, 448).astype(np.float32)) \
        .to(torch.float8_e4m3fn).view(torch.uint8).numpy().reshape(6, 512)
    assert np.array_equal(q, want)
