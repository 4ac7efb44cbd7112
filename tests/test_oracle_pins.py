"""Pins the CPU oracle before it is trusted as the checker (CPU only).

Against fixtures the reference's own code produced (tests/golden/reference_*,
made by tests/golden/make_golden.py from oracle/_ref), against the reference
compiled in this container when oracle/_ref is present, and against the known
answers of the reference's tests: Tests/Kernels/Int8BlocksTests.cpp:89-243,
ArgmaxTests.cpp:107-245, GeGLUTests.cpp:242-267.
"""
import os

import numpy as np
import pytest

import oracle_bindings as ob

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def golden(name):
    return np.load(os.path.join(GOLDEN, name))


# ---- fp16 and the generator ------------------------------------------------

def test_half_conversion_matches_ieee_round_to_nearest_even():
    rng = np.random.default_rng(7)
    values = (rng.standard_normal(50000) * 10.0 ** rng.integers(-9, 6, 50000)).astype(np.float32)
    edges = np.array([65504, 65519.996, 65520, 1e-8, 5.9604645e-08, 2.9802322e-08, 2.9802326e-08, -0.0,
                      6.1035156e-05, 6.1035152e-05, np.inf, -np.inf], dtype=np.float32)
    lib = ob.oracle()
    with np.errstate(over="ignore"):
        for v in np.concatenate([values, edges]):
            expected = int(np.float32(v).astype(np.float16).view(np.uint16))
            assert lib.oracle_half_from_float(float(v)) == expected, v
    for bits in range(0, 1 << 16, 7):
        if (bits & 0x7C00) == 0x7C00 and bits & 0x3FF:
            continue  # NaN payloads
        expected = float(np.uint16(bits).view(np.float16))
        got = lib.oracle_half_to_float(bits)
        assert got == expected or (np.isnan(got) and np.isnan(expected))


def test_mt19937_matches_the_reference_library():
    fixture = golden("reference_mt19937.npz")
    for key in fixture.files:
        seed = int(key.split("_")[1])
        out = np.empty(2000, dtype=np.uint32)
        ob.oracle().oracle_mt19937_raw(seed, 2000, ob.p(out))
        np.testing.assert_array_equal(out, fixture[key])


def test_spread_values_follows_the_reference_formula():
    raw = golden("reference_mt19937.npz")["seed_8181"]
    expected = (3.0 * ((raw[:1280] % 2001).astype(np.float32) / np.float32(1000.0) - np.float32(1.0))).astype(
        np.float32)
    np.testing.assert_array_equal(ob.spread_values(1280, 8181, 3.0), expected)


# ---- Q8_0 quantizer ------------------------------------------------------------

@pytest.mark.parametrize("case", ["roundtrip", "magnitudes", "pieces", "gemma_like", "ties"])
def test_quantizer_matches_reference_fixture(case):
    fixture = golden("reference_int8_blocks.npz")
    values = fixture[f"{case}_values"]
    np.testing.assert_array_equal(ob.quantize(values), fixture[f"{case}_bytes"])
    np.testing.assert_array_equal(ob.dequantize(fixture[f"{case}_bytes"], values.size),
                                  fixture[f"{case}_dequantized"])


@pytest.mark.skipif(not ob.ref_available(), reason="oracle/_ref not built (needs the reference tree)")
def test_quantizer_matches_compiled_reference_on_random_tensors():
    rng = np.random.default_rng(11)
    for scale in (1e-6, 1e-3, 0.02, 1.0, 300.0, 7e4):
        values = (rng.standard_normal(32 * 777 + 32) * scale).astype(np.float32)
        values[:32] = 0.0
        np.testing.assert_array_equal(ob.quantize(values), ob.ref_quantize(values))


def test_int8_blocks_sizes_and_shapes():
    lib = ob.oracle()
    assert lib.oracle_int8_blocks_byte_count(64) == 68
    assert lib.oracle_int8_blocks_byte_count(2048 * 2048) == 2048 * 2048 + 2048 * 2048 // 16
    assert lib.oracle_quantizes_as_int8_blocks(2048, 2048 * 2048)
    assert lib.oracle_quantizes_as_int8_blocks(16384, 2048 * 16384)
    assert lib.oracle_quantizes_as_int8_blocks(2048, 256000 * 2048)
    assert lib.oracle_quantizes_as_int8_blocks(32, 64)
    assert not lib.oracle_quantizes_as_int8_blocks(48, 32 * 48)
    assert not lib.oracle_quantizes_as_int8_blocks(32, 32 * 3)
    assert not lib.oracle_quantizes_as_int8_blocks(0, 0)


def test_round_trip_is_exact_to_the_scale():
    """Int8BlocksTests.cpp:89-120: every value comes back as scale * k, |k| <= 127."""
    values = ob.spread_values(32 * 40, 8181, 3.0)
    recovered = ob.dequantize(ob.quantize(values), values.size)
    for block in range(40):
        v = values[32 * block: 32 * block + 32]
        r = recovered[32 * block: 32 * block + 32]
        scale = np.float32(np.float16(np.max(np.abs(v)) / np.float32(127.0)))
        assert scale > 0
        steps = np.rint(r / scale)
        assert np.all(np.abs(steps) <= 127)
        np.testing.assert_array_equal(r, (scale * steps.astype(np.float32)).astype(np.float32))
        assert np.all(np.abs(r - v) <= 0.5 * scale)


def test_blocks_follow_their_own_magnitude():
    """Int8BlocksTests.cpp:126-187, including the zero block and the block too
    small for any fp16 scale (stored as zeroes)."""
    magnitudes = np.array([1.0e-2, 1.0e3, 0.0, 1.0, 6.0e-8, 1.0e4], dtype=np.float32)
    values = (ob.spread_values(6 * 32, 1717, 1.0).reshape(6, 32) * magnitudes[:, None]).reshape(-1)
    recovered = ob.dequantize(ob.quantize(values), values.size).reshape(6, 32)
    values = values.reshape(6, 32)
    for b, m in enumerate(magnitudes):
        if m == 0.0 or m < 1e-7:
            assert np.all(recovered[b] == 0.0)
        else:
            assert np.all(np.abs(recovered[b] - values[b]) <= 0.5 * m / 127.0)


def test_quantizing_in_pieces_equals_whole():
    """Int8BlocksTests.cpp:222-243."""
    values = ob.spread_values(32 * 20, 5150, 2.0)
    whole = ob.quantize(values)
    pieces = np.zeros_like(whole)
    for first in range(0, values.size, 4 * 32):
        chunk = np.ascontiguousarray(values[first: first + 128])
        ob.oracle().oracle_quantize_int8_blocks(ob.p(chunk), first, 128, values.size, ob.p(pieces))
    np.testing.assert_array_equal(pieces, whole)


# ---- argmax ------------------------------------------------------------------

def test_argmax_matches_reference_fixture():
    fixture = golden("reference_argmax.npz")
    for row, expected in zip(fixture["hand_rows"], fixture["hand_expected"]):
        assert ob.argmax(row) == expected
    assert list(fixture["hand_expected"]) == [0, 18, 36, 5]  # ArgmaxTests.cpp:107-121
    for row, expected in zip(fixture["spread_rows"], fixture["spread_expected"]):
        assert ob.argmax(row, fixture["spread_mask"]) == expected
    vocab = ob.spread_values(256000, 256000, 4.0)
    vocab[137425] = 900.0
    vocab[318] = 800.0
    mask = np.zeros(256000, dtype=np.float32)
    mask[137425] = 1.0
    assert [ob.argmax(vocab), ob.argmax(vocab, mask)] == list(fixture["vocab_expected"]) == [137425, 318]


def test_argmax_all_masked_is_zero_and_ties_take_the_lowest_index():
    row = np.array([3.0, 7.0, 7.0, 1.0], dtype=np.float32)
    assert ob.argmax(row) == 1
    assert ob.argmax(row, np.ones(4, dtype=np.float32)) == 0
    only = np.array([1.0, 1.0, 0.0, 1.0], dtype=np.float32)
    assert ob.argmax(np.array([1000.0, 999.0, -1000.0, 997.0], dtype=np.float32), only) == 2


@pytest.mark.skipif(not ob.ref_available(), reason="oracle/_ref not built (needs the reference tree)")
def test_argmax_matches_compiled_sampler():
    ref = ob.ref()
    rng = np.random.default_rng(3)
    for _ in range(50):
        row = rng.integers(-5, 5, 257).astype(np.float32)  # many ties
        mask = (rng.random(257) < 0.3).astype(np.float32)
        expected = ref.ref_sampler_argmax(ob.p(row), ob.p(mask), row.size)
        assert ob.argmax(row, mask) == expected


# ---- scalar pieces --------------------------------------------------------------

def test_tanh_gelu_tails_stay_finite():
    """GeGLUTests.cpp:242-267: +-30 and +-1000 saturate rather than NaN."""
    lib = ob.oracle()
    for x in (30.0, -30.0, 1000.0, -1000.0):
        y = lib.oracle_tanh_gelu_float(x)
        assert np.isfinite(y)
        assert abs(y - (x if x > 0 else 0.0)) <= 1e-3 * abs(x)
    for x in np.linspace(-8, 8, 97):
        assert abs(lib.oracle_tanh_gelu_float(float(x)) - lib.oracle_tanh_gelu_double(float(x))) <= 1e-6 * (1 + abs(x))


def test_rotary_table_matches_its_definition():
    cos = np.empty(64 * 8, dtype=np.float32)
    sin = np.empty(64 * 8, dtype=np.float32)
    ob.oracle().oracle_rotary_table(64, 16, 10000.0, ob.p(cos), ob.p(sin))
    pos = np.arange(64)[:, None].astype(np.float64)
    inv = 1.0 / np.power(10000.0, 2.0 * np.arange(8) / 16.0)
    np.testing.assert_array_equal(cos.reshape(64, 8), np.cos(pos * inv).astype(np.float32))
    np.testing.assert_array_equal(sin.reshape(64, 8), np.sin(pos * inv).astype(np.float32))


# ---- the forward pass -------------------------------------------------------------

def _small_model(precision):
    from huggingfaceeacp_b200 import native

    shape = native.SMALL_INT8
    tensors = {}
    for tensor, layer in native.model_tensors(shape):
        tensors[(tensor, layer)] = native.synthetic_tensor(shape, tensor, layer, seed=11)
    return shape, tensors, ob.OracleModel(shape, tensors, precision=precision)


def test_cached_steps_equal_the_full_recompute():
    """The oracle's KV cache is exact against the reference's full recompute
    (ReferenceDecoder.h:283-375): stepping token by token gives the same rows."""
    shape, tensors, whole = _small_model("double")
    prompt = np.array([5, 41, 3, 17, 28, 9, 60], dtype=np.uint32)
    hidden, logits = whole.step(prompt)
    _, _, stepped = _small_model("double")
    for i, tok in enumerate(prompt):
        h, lg = stepped.step([tok])
        np.testing.assert_array_equal(h[0], hidden[i])
        np.testing.assert_array_equal(lg[0], logits[i])


def test_float_oracle_tracks_double_oracle():
    _, _, double = _small_model("double")
    _, _, single = _small_model("float")
    prompt = np.array([5, 41, 3, 17, 28, 9, 60], dtype=np.uint32)
    hd, ld = double.step(prompt)
    hf, lf = single.step(prompt)
    assert ob.worst_error(lf, ld) <= 5e-6
    assert ob.worst_error(hf, hd) <= 5e-6


def test_window_refusal_leaves_the_position():
    _, _, model = _small_model("double")
    model.step(np.arange(16, dtype=np.uint32) % 64)
    assert model.position == 16
    with pytest.raises(AssertionError):
        model.step([1])
    assert model.position == 16
