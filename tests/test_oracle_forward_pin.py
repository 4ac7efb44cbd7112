"""Pins the oracle's double forward pass against the reference's own (CPU only).

The reference checks its GPU decoder against referenceDecode, a scalar
double-precision restatement of GemmaForCausalLM.forward with full causal
recompute (Tests/Decoder/ReferenceDecoder.h:294-375). oracle/build_ref.sh
compiles that header unchanged into oracle/_ref; these tests require oracle.c's
double model, which runs incrementally over a KV cache, to equal it on:

- the reference's own synthetic checkpoint and prompt (Tests/Decoder/Common.h:
  179-237 at the int8 shape; DecoderTests.cpp:51-54), in one step, token by
  token and as a continuation, with the Gemma embedding scale and with 1;
- a Gemma-width one-layer model (2048 wide, 8 query heads of 256 over one KV
  head, a 16384-wide feed-forward) with N(0, 0.02) weights.

Both sides read the same Q8_0 weights: the reference through its own
Int8Blocks round trip (quantizedReferenceModel, :79-103), the oracle through
oracle.c's quantizer (itself pinned bit for bit to the reference's). The
fixture tests/golden/reference_decode_small.npz holds the reference's outputs
for the first case, so the pin also runs where oracle/_ref is absent.
"""
import os

import numpy as np
import pytest

import oracle_bindings as ob
from huggingfaceeacp_b200 import native

# Relative agreement required of two double-precision evaluations of the same
# arithmetic that differ only in summation order.
PIN_TOLERANCE = 1e-12
PROMPT = [5, 41, 3, 17, 28, 9, 60]
needs_ref = pytest.mark.skipif(not ob.ref_available(), reason="oracle/_ref not built (needs the reference tree)")


def oracle_rows(shape, tensors, tokens, split):
    """The oracle's hidden and logit rows for `tokens`, fed in steps of the given sizes."""
    model = ob.OracleModel(shape, tensors, precision="double")
    hidden, logits, at = [], [], 0
    for size in split:
        h, lg = model.step(tokens[at:at + size])
        hidden.append(h)
        logits.append(lg)
        at += size
    model.close()
    return np.concatenate(hidden), np.concatenate(logits)


def test_oracle_equals_reference_decode_fixture():
    fixture = np.load(os.path.join(ob.GOLDEN_DIR, "reference_decode_small.npz"))
    shape = native.SMALL_INT8
    tensors = ob.q8_model_tensors(ob.reference_synthetic_raw(shape))
    prompt = [int(t) for t in fixture["prompt"]]
    for name, s in (("scaled", shape), ("unit", shape.replace(embed_scale=1.0))):
        for split in ([len(prompt)], [1] * len(prompt), [4, 3]):
            hidden, logits = oracle_rows(s, tensors, prompt, split)
            assert ob.worst_error(hidden, fixture[f"{name}_hidden"]) <= PIN_TOLERANCE, (name, split)
            assert ob.worst_error(logits, fixture[f"{name}_logits"]) <= PIN_TOLERANCE, (name, split)


@needs_ref
@pytest.mark.parametrize("embed_scale", [None, 1.0])
def test_oracle_equals_compiled_reference_decode(embed_scale):
    shape = native.SMALL_INT8.replace(embed_scale=embed_scale)
    raw = ob.reference_synthetic_raw(shape)
    tensors = ob.q8_model_tensors(raw)
    ref_hidden, ref_logits = ob.ref_decode(shape, raw, PROMPT)
    for split in ([7], [1] * 7, [2, 1, 4]):
        hidden, logits = oracle_rows(shape, tensors, PROMPT, split)
        assert ob.worst_error(hidden, ref_hidden) <= PIN_TOLERANCE, split
        assert ob.worst_error(logits, ref_logits) <= PIN_TOLERANCE, split
    # Quantization is visible at this tolerance: the unquantized reference differs.
    _, plain_logits = ob.ref_decode(shape, raw, PROMPT, quantize=False)
    assert ob.worst_error(plain_logits, ref_logits) > 1e-4


@needs_ref
def test_oracle_equals_compiled_reference_decode_at_gemma_width():
    shape = native.GEMMA_2B.replace(layers=1, vocab=512, max_positions=16)
    w, q, kv, f = shape.width, shape.query_width, shape.kv_width, shape.intermediate
    streams = iter(range(100))

    def normal(count, stddev):
        return native.synthetic_normal(91, next(streams), 0, count, stddev)

    raw = {"embedding": normal(shape.vocab * w, 0.02), "final_norm": normal(w, 0.1),
           "layers": [{"input_norm": normal(w, 0.1), "query": normal(q * w, 0.02), "key": normal(kv * w, 0.02),
                       "value": normal(kv * w, 0.02), "output": normal(w * q, 0.02), "gate": normal(f * w, 0.02),
                       "up": normal(f * w, 0.02), "down": normal(w * f, 0.02), "post_norm": normal(w, 0.1)}]}
    tokens = [2, 401, 17, 299, 3]
    ref_hidden, ref_logits = ob.ref_decode(shape, raw, tokens)
    hidden, logits = oracle_rows(shape, ob.q8_model_tensors(raw), tokens, [3, 1, 1])
    assert ob.worst_error(hidden, ref_hidden) <= PIN_TOLERANCE
    assert ob.worst_error(logits, ref_logits) <= PIN_TOLERANCE
