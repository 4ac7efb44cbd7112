"""Failure detection on the device, in the forms this pool allows: nothing
faults, traps or hangs. A bounded wait whose arrival never comes must give up
after its poll limit, set its bit in the context's error word and let the
kernel return; hf_cuda_sync then reports HF_E_DEVICE naming the wait and
clears the word, and the context goes on decoding exactly. Likewise a top-p
draw whose set needs more than the device sampler's 1,024 candidates is
reported, not silently truncated. The reference's analogue is the refusal
that leaves the decoder usable (Tests/Decoder/ReferenceDecoder.h:418-446).
"""
import numpy as np
import pytest

import oracle_bindings as ob
from huggingfaceeacp_b200 import native

pytestmark = pytest.mark.gpu

SHAPE = native.DecoderShape(width=2048, heads=8, kv_heads=1, head_width=256, layers=1, intermediate=16384,
                            vocab=8192, max_positions=64, max_step_rows=16, embed_scale=1.0)
PROMPT = np.array([2, 5, 41, 3, 17, 28, 9, 60], dtype=np.uint32)


@pytest.fixture(scope="module")
def model():
    ctx = native.Context(SHAPE)
    tensors = ctx.load_synthetic(seed=7, keep=True)
    yield ctx, tensors
    ctx.close()


@pytest.mark.parametrize("kind,words", [(native.PROBE_STAGE_WAIT, "stage wait"),
                                        (native.PROBE_GRID_BARRIER, "grid barrier")])
def test_a_wait_that_never_completes_is_reported_and_the_context_recovers(model, kind, words):
    ctx, tensors = model
    expected = ob.greedy_reference(SHAPE, tensors, PROMPT, 6)
    ctx.probe_wait_timeout(kind)
    with pytest.raises(native.HFError) as reported:
        ctx.sync()
    assert reported.value.code == native.HF_E_DEVICE
    assert words in str(reported.value)
    ctx.sync()  # the word was cleared
    for path in (native.DECODE_PERSISTENT, native.DECODE_GRAPH):
        ctx.set_decode_path(path)
        assert list(ctx.generate(PROMPT, 6)) == expected


def test_a_top_p_set_beyond_the_device_sampler_is_reported(model):
    ctx, tensors = model
    flat = np.zeros(SHAPE.vocab, dtype=np.float32)  # every token equally likely: p = 0.9 needs 7,373 of them
    with pytest.raises(native.HFError) as reported:
        ctx.sample(flat, temperature=1.0, top_p=0.9, seed=3)
    assert reported.value.code == native.HF_E_DEVICE
    assert "1024 candidates" in str(reported.value)
    row = ob.spread_values(SHAPE.vocab, 99, 8.0)
    assert list(ctx.sample(row, temperature=0.7, top_p=0.9, seed=3, draws=4)) == list(
        ob.ref_sample(row, None, 0.7, 0, 0.9, 3, 4))
