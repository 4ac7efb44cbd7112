"""Pins oracle.c's restatement of the seeded generator (CPU only).

The BASELINE configs' random-init weights and prompts come from the
counter-based generator of the product's host library (hf_synthetic_normal,
hf_synthetic_tokens in include/hf_host.h). The bench's reference arm builds
its model from oracle.c alone, so that arm loads none of the product's
libraries; these tests require the two to agree bit for bit: normal values
(whole tensors, odd counts, pieces at an even offset), token ids, and the
Q8_0 bytes of whole tensors.
"""
import numpy as np
import pytest

import oracle_bindings as ob
from huggingfaceeacp_b200 import native


@pytest.mark.parametrize("seed,tensor,layer,count", [(0, native.QUERY, 3, 2048 * 64), (7, native.EMBEDDING, -1, 99_999),
                                                     (3, native.INPUT_NORM, 17, 2048), (123456789, native.DOWN, 0, 1)])
def test_normals_equal_the_host_library(seed, tensor, layer, count):
    stddev = 0.1 if tensor == native.INPUT_NORM else 0.02
    expected = native.synthetic_normal(seed, tensor, layer, count, stddev)
    np.testing.assert_array_equal(ob.synthetic_normal(seed, tensor, layer, count, stddev), expected)


def test_a_piece_at_an_even_offset_equals_the_same_slice():
    whole = ob.synthetic_normal(5, native.GATE_UP, 2, 300_001, 0.02)
    out = np.empty(1001, dtype=np.float32)
    lib = ob.oracle()
    assert lib.oracle_synthetic_normal(5, lib.oracle_synthetic_stream(native.GATE_UP, 2), 150_000, 1001, 0.02,
                                       ob.p(out), 3) == 0
    np.testing.assert_array_equal(out, whole[150_000:151_001])


@pytest.mark.parametrize("seed,count,vocab", [(0, 16, 256000), (2, 8064, 256000), (3 + 63, 512, 8192), (9, 1, 4)])
def test_tokens_equal_the_host_library(seed, count, vocab):
    np.testing.assert_array_equal(ob.synthetic_tokens(seed, count, vocab), native.synthetic_tokens(seed, count, vocab))


def test_model_bytes_equal_the_host_library():
    shape = native.GEMMA_2B.replace(layers=1, vocab=1024)
    ours = ob.synthetic_model(shape, seed=4)
    for (tensor, layer), data in ours.items():
        np.testing.assert_array_equal(data, native.synthetic_tensor(shape, tensor, layer, 4))
