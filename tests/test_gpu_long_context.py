"""Long-context decode (BASELINE config 2's shape of work: an 8,064-token prompt,
then decode steps up to an 8,192-position window) on a two-layer Gemma-width
model: the whole-loop decode kernel (128 context splits and its merge phase)
against the independent graph path (mqa_fast splits + mqa_merge), token by
token, at the decoder tolerance (DecoderTests.cpp:41). Both paths are checked
against the double oracle at short contexts in test_gpu_decoder.py; here they
must agree where the oracle would take minutes."""
import numpy as np
import pytest

import oracle_bindings as ob
from huggingfaceeacp_b200 import native

pytestmark = pytest.mark.gpu

TOLERANCE = 5e-6
SHAPE = native.DecoderShape(width=2048, heads=8, kv_heads=1, head_width=256, layers=2, intermediate=16384,
                            vocab=8192, max_positions=8192, max_step_rows=512, embed_scale=1.0)


def test_whole_loop_and_graph_decode_agree_at_the_end_of_an_8192_window():
    with native.Context(SHAPE) as ctx:
        ctx.load_synthetic(seed=2)
        prompt = native.synthetic_tokens(2, 8064, SHAPE.vocab)
        rows = {}
        for path in (native.DECODE_PERSISTENT, native.DECODE_GRAPH):
            ctx.set_decode_path(path)
            ctx.begin_sequence()
            ctx.prefill_async(prompt)
            ctx.decode_async(100)
            generated = ctx.read_slots(8065, 100)
            rows[path] = (generated, [ctx.step([int(t)]) for t in (5, 17, 99)])
            assert ctx.position == 8167
        assert np.array_equal(rows[native.DECODE_PERSISTENT][0], rows[native.DECODE_GRAPH][0])
        for (lp, hp), (lg, hg) in zip(rows[native.DECODE_PERSISTENT][1], rows[native.DECODE_GRAPH][1]):
            assert ob.worst_error(lp, lg) <= TOLERANCE
            assert ob.worst_error(hp, hg) <= TOLERANCE
