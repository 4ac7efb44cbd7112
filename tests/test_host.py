"""The product's host side (libhf_host.so) and the C-ABI surface (CPU only).

The product quantizer must write the reference's bytes (Int8Blocks.cpp:
176-199): checked against the reference's own fixtures, against the pinned
oracle, and against the compiled reference when present. The C-ABI libraries
must load and export every entry point include/*.h declares.
"""
import os
import re

import numpy as np
import pytest

import oracle_bindings as ob
from huggingfaceeacp_b200 import native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")


@pytest.mark.parametrize("case", ["roundtrip", "magnitudes", "pieces", "gemma_like", "ties"])
def test_product_quantizer_writes_the_reference_bytes(case):
    fixture = np.load(os.path.join(GOLDEN, "reference_int8_blocks.npz"))
    values = fixture[f"{case}_values"]
    np.testing.assert_array_equal(native.quantize(values), fixture[f"{case}_bytes"])
    np.testing.assert_array_equal(native.dequantize(fixture[f"{case}_bytes"], values.size),
                                  fixture[f"{case}_dequantized"])


def test_product_quantizer_equals_oracle_on_model_tensors():
    for tensor, layer in [(native.QUERY, 0), (native.DOWN, 3)]:
        shape = native.SMALL_INT8.replace(width=256, intermediate=512)
        count = int(np.prod(shape.tensor_shape(tensor)))
        values = native.synthetic_normal(5, tensor, layer, count, 0.02)
        np.testing.assert_array_equal(native.quantize(values), ob.quantize(values))
    rng = np.random.default_rng(1)
    for scale in (1e-7, 1e-4, 1.0, 6e4):
        values = (rng.standard_normal(32 * 300) * scale).astype(np.float32)
        np.testing.assert_array_equal(native.quantize(values), ob.quantize(values))


def test_threaded_quantize_equals_single_thread_and_pieces():
    values = native.synthetic_normal(9, 1, 0, 32 * 70001 + 32, 0.02)
    whole = native.quantize(values, threads=1)
    np.testing.assert_array_equal(native.quantize(values, threads=8), whole)
    pieces = np.zeros_like(whole)
    lib = native.host()
    step = 32 * 9999
    for first in range(0, values.size, step):
        n = min(step, values.size - first)
        chunk = np.ascontiguousarray(values[first:first + n])
        assert lib.hf_quantize_int8_blocks(native._ptr(chunk), first, n, values.size, native._ptr(pieces), 3) == 0
    np.testing.assert_array_equal(pieces, whole)


def test_quantizer_refuses_ragged_pieces():
    lib = native.host()
    values = np.zeros(64, dtype=np.float32)
    out = np.zeros(68, dtype=np.uint8)
    assert lib.hf_quantize_int8_blocks(native._ptr(values), 0, 48, 64, native._ptr(out), 1) == native.HF_E_INVALID
    assert lib.hf_quantize_int8_blocks(native._ptr(values), 16, 32, 64, native._ptr(out), 1) == native.HF_E_INVALID
    assert not out.any()
    assert native.int8_blocks_byte_count(64) == 68
    assert native.quantizes_as_int8_blocks(2048, 2048 * 2048)
    assert not native.quantizes_as_int8_blocks(48, 32 * 48)


def test_half_narrowing_matches_numpy():
    lib = native.host()
    rng = np.random.default_rng(5)
    with np.errstate(over="ignore"):
        for v in (rng.standard_normal(5000) * 10.0 ** rng.integers(-8, 6, 5000)).astype(np.float32):
            assert lib.hf_half_from_float(float(v)) == int(np.float32(v).astype(np.float16).view(np.uint16))


def test_generator_is_counter_based_and_normal():
    a = native.synthetic_normal(3, 7, 2, 100001, 0.02)
    b = native.synthetic_normal(3, 7, 2, 100001, 0.02, threads=1)
    np.testing.assert_array_equal(a, b)
    tail = native.synthetic_normal(3, 7, 2, 1000, 0.02, first=50000)
    np.testing.assert_array_equal(tail, a[50000:51000])
    assert abs(float(a.mean())) < 3e-4 and abs(float(a.std()) - 0.02) < 3e-4
    assert not np.array_equal(a[:1000], native.synthetic_normal(3, 7, 3, 1000, 0.02))
    tokens = native.synthetic_tokens(0, 16, 256000)
    assert tokens[0] == 2 and np.all(tokens[1:] >= 3) and np.all(tokens < 256000)
    np.testing.assert_array_equal(tokens, native.synthetic_tokens(0, 16, 256000))


def _declared(header):
    text = open(os.path.join(ROOT, "include", header)).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(hf_[a-z0-9_]+)\s*\(", text)))


@pytest.mark.parametrize("header,library", [("hf_cuda.h", "libhf_cuda.so"), ("hf_host.h", "libhf_host.so")])
def test_libraries_load_and_export_every_declared_symbol(header, library):
    import ctypes

    names = _declared(header)
    assert len(names) > 5
    lib = ctypes.CDLL(os.path.join(native.LIB_DIR, library))
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_cuda_library_reports_devices_without_failing():
    assert native.device_count() >= 0


def test_decode_byte_accounting_matches_the_survey():
    # 2,662,727,680 B of Q8_0 weights per batch-1 token (layers + tied logits).
    assert native.weight_bytes(native.GEMMA_2B) == 2_662_727_680
