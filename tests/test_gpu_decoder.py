"""Decoder and generation parity on the B200, through the C-ABI.

Mirrors Tests/Decoder/DecoderTests.cpp and Tests/Generation/GenerationTests.cpp
on the reference's own synthetic int8 decoder shape (vocab 64, width 32, ffn 64,
2 layers, 2 heads over 1 KV head of 16, window 16; Tests/Decoder/Common.h:38-72,
prompt {5, 41, 3, 17, 28, 9, 60}; DecoderTests.cpp:51-54), which runs the
generic kernels, and on Gemma-width models (width 2048, 8 heads of 256 over one
KV head) that run the sm_100a streaming path, each against the double-precision
oracle over the same Q8_0 bytes at the reference's 5e-6 tolerance
(DecoderTests.cpp:41, 61-75).
"""
import numpy as np
import pytest

import oracle_bindings as ob
from huggingfaceeacp_b200 import native

pytestmark = pytest.mark.gpu

TOLERANCE = 5e-6
PROMPT = np.array([5, 41, 3, 17, 28, 9, 60], dtype=np.uint32)

# Gemma widths with few layers: the streaming kernels' shapes, an oracle that
# finishes in seconds. `varied` shrinks the embedding scale so greedy decoding
# leaves the self-copying fixed point random tied embeddings fall into.
MINI = native.DecoderShape(width=2048, heads=8, kv_heads=1, head_width=256, layers=2, intermediate=4096, vocab=8192,
                           max_positions=320, max_step_rows=64)
MINI_WIDE_FFN = MINI.replace(intermediate=16384, layers=1, max_positions=64)
VARIED = MINI.replace(embed_scale=1.0)


class Pair:
    """A GPU context and a CPU oracle over the same bytes."""

    def __init__(self, shape, seed=11):
        self.shape = shape
        self.ctx = native.Context(shape)
        self.tensors = self.ctx.load_synthetic(seed=seed, keep=True)
        self.oracle = ob.OracleModel(shape, self.tensors, precision="double")

    def fresh_oracle(self):
        return ob.OracleModel(self.shape, self.tensors, precision="double")

    def step(self, tokens):
        logits, hidden = self.ctx.step(tokens)
        ref_hidden, ref_logits = self.oracle.step(tokens)
        return max(ob.worst_error(logits, ref_logits), ob.worst_error(hidden, ref_hidden))

    def close(self):
        self.ctx.close()
        self.oracle.close()


@pytest.fixture(scope="module", params=["small", "mini"])
def pair(request):
    shape = native.SMALL_INT8 if request.param == "small" else MINI
    p = Pair(shape)
    yield p
    p.close()


def test_fast_path_selection(pair):
    assert pair.ctx.fast_path == (pair.shape.width == 2048)


def test_prompt_matches_reference(pair):
    pair.ctx.begin_sequence()
    pair.oracle.begin_sequence()
    assert pair.step(PROMPT) <= TOLERANCE
    assert pair.ctx.position == len(PROMPT)


def test_cached_steps_match_reference(pair):
    pair.ctx.begin_sequence()
    pair.oracle.begin_sequence()
    worst = 0.0
    for i, token in enumerate(PROMPT):
        worst = max(worst, pair.step([token]))
        assert pair.ctx.position == i + 1
    assert worst <= TOLERANCE


def test_prompt_in_two_blocks_matches_reference(pair):
    pair.ctx.begin_sequence()
    pair.oracle.begin_sequence()
    assert max(pair.step(PROMPT[:4]), pair.step(PROMPT[4:])) <= TOLERANCE
    assert pair.ctx.position == len(PROMPT)


def test_begin_sequence_resets_the_sequence_exactly(pair):
    pair.ctx.begin_sequence()
    pair.ctx.step([11, 22, 33, 44, 55])
    pair.ctx.begin_sequence()
    assert pair.ctx.position == 0
    first = pair.ctx.step(PROMPT)
    pair.ctx.begin_sequence()
    second = pair.ctx.step(PROMPT)
    np.testing.assert_array_equal(first[0], second[0])
    np.testing.assert_array_equal(first[1], second[1])


def _refuses_leaving_logits_untouched(ctx, tokens, code):
    """ReferenceDecoder.h:418-446: a refused step records nothing."""
    before = ctx.position
    logits = np.full((len(tokens), ctx.shape.vocab), -12345.0, dtype=np.float32)
    rc = ctx.lib.hf_cuda_step(ctx.handle, native._ptr(np.asarray(tokens, dtype=np.uint32)), len(tokens),
                              native._ptr(logits), None)
    assert rc == code
    assert ctx.position == before
    assert np.all(logits == -12345.0)


def test_step_past_the_window_is_refused(pair):
    ctx = pair.ctx
    ctx.begin_sequence()
    P = pair.shape.max_positions
    cap = pair.shape.max_step_rows or P
    whole = (np.arange(P) % pair.shape.vocab).astype(np.uint32)
    for first in range(0, P, cap):
        ctx.step(whole[first:first + cap], want_logits=False, want_hidden=False)
    assert ctx.position == P
    _refuses_leaving_logits_untouched(ctx, [1], native.HF_E_WINDOW)
    ctx.begin_sequence()
    for first in range(0, P - 1, cap):
        ctx.step(whole[first:min(first + cap, P - 1)], want_logits=False, want_hidden=False)
    _refuses_leaving_logits_untouched(ctx, [1, 2], native.HF_E_WINDOW)


def test_bad_token_and_empty_step_are_refused(pair):
    pair.ctx.begin_sequence()
    _refuses_leaving_logits_untouched(pair.ctx, [pair.shape.vocab], native.HF_E_TOKEN)
    rc = pair.ctx.lib.hf_cuda_step(pair.ctx.handle, native._ptr(PROMPT), 0, None, None)
    assert rc == native.HF_E_INVALID


def test_short_step_capacity_matches_reference_and_refuses_more():
    """DecoderTests.cpp:187-248: a four-row capacity feeds a prompt in blocks."""
    shape = native.SMALL_INT8.replace(max_step_rows=4)
    p = Pair(shape)
    try:
        assert max(p.step(PROMPT[:4]), p.step(PROMPT[4:])) <= TOLERANCE
        assert p.step([12]) <= TOLERANCE
        p.ctx.begin_sequence()
        _refuses_leaving_logits_untouched(p.ctx, [5, 41, 3, 17, 28], native.HF_E_CAPACITY)
        p.ctx.step([5, 41, 3, 17])
        assert p.ctx.position == 4
    finally:
        p.close()


def test_unprepared_decoder_is_refused():
    with native.Context(native.SMALL_INT8) as ctx:
        assert not ctx.prepared
        ctx.upload(native.EMBEDDING, -1, native.synthetic_tensor(native.SMALL_INT8, native.EMBEDDING, -1, 1))
        _refuses_leaving_logits_untouched(ctx, [1], native.HF_E_NOT_READY)
        with pytest.raises(native.HFError) as err:
            ctx.upload(native.QUERY, 0, np.zeros(10, dtype=np.uint8))
        assert err.value.code == native.HF_E_SHAPE


def test_invalid_shapes_are_refused():
    for bad in (native.SMALL_INT8.replace(head_width=18), native.SMALL_INT8.replace(heads=3),
                native.SMALL_INT8.replace(max_step_rows=17), native.SMALL_INT8.replace(width=0),
                native.SMALL_INT8.replace(head_width=512)):
        with pytest.raises(native.HFError) as err:
            native.Context(bad)
        assert err.value.code == native.HF_E_SHAPE


def test_wide_feed_forward_on_the_streaming_path():
    """intermediate 16384: the down projection's 8-warp row split."""
    p = Pair(MINI_WIDE_FFN)
    try:
        assert p.step(PROMPT) <= TOLERANCE
        for token in (100, 200, 300):
            assert p.step([token]) <= TOLERANCE
    finally:
        p.close()


def test_split_context_attention_matches_reference():
    """Positions past 64 use the split (flash-decoding) attention and its merge;
    crossing 64, 128 and 256 keys exercises 1, 2, 4 and 8 splits."""
    p = Pair(MINI, seed=3)
    try:
        prompt = native.synthetic_tokens(3, 60, MINI.vocab)
        worst = p.step(prompt)
        for i in range(220):
            token = int(prompt[i % 60])
            err = p.step([token])
            worst = max(worst, err)
        assert worst <= TOLERANCE, worst
    finally:
        p.close()


# ---- generation (GenerationTests.cpp:192-233, 556-596) ------------------------

@pytest.mark.parametrize("shape", [native.SMALL_INT8, MINI, VARIED], ids=["small", "mini", "varied"])
def test_greedy_generation_equals_the_host_driven_reference_loop(shape):
    with native.Context(shape) as ctx:
        tensors = ctx.load_synthetic(seed=5, keep=True)
        prompt = PROMPT % shape.vocab
        count = min(24, shape.max_positions - len(prompt))
        expected, margins = ob.greedy_reference(shape, tensors, prompt, count, with_margins=True)
        got = ctx.generate(prompt, count)
        assert list(got) == expected, (list(got), expected, margins)
        if shape is VARIED:
            assert len(set(expected)) > 3  # the feedback path sees real token changes


@pytest.mark.parametrize("capacity,length", [(64, 70), (4, 10), (1, 5)])
def test_prompt_longer_than_a_step_generates_like_the_reference(capacity, length):
    """A prompt fed in several blocks (Gemma.cpp:341-380): every block but the
    last leaves the next prompt token in its slot; only the last one samples."""
    shape = MINI.replace(intermediate=16384, embed_scale=1.0, max_positions=96, max_step_rows=capacity)
    with native.Context(shape) as ctx:
        tensors = ctx.load_synthetic(seed=41, keep=True)
        prompt = native.synthetic_tokens(100, length, shape.vocab)
        expected = ob.greedy_reference(shape, tensors, prompt, 12)
        assert list(ctx.generate(prompt, 12)) == expected


def test_generation_stops_at_end_of_sequence_and_at_the_window():
    shape = VARIED
    with native.Context(shape) as ctx:
        tensors = ctx.load_synthetic(seed=5, keep=True)
        full = ob.greedy_reference(shape, tensors, PROMPT, 24)
        eos = full[10]
        first = full.index(eos)
        assert list(ctx.generate(PROMPT, 24, eos=eos)) == full[:first]
        window = ctx.generate(PROMPT, 10 ** 6)
        assert len(window) == shape.max_positions - len(PROMPT)
        assert list(window[:24]) == full
    with native.Context(native.SMALL_INT8) as ctx:
        ctx.load_synthetic(seed=5)
        assert len(ctx.generate(np.arange(16, dtype=np.uint32), 5)) == 0
        with pytest.raises(native.HFError) as err:
            ctx.generate(np.arange(17, dtype=np.uint32), 5)
        assert err.value.code == native.HF_E_WINDOW
        with pytest.raises(native.HFError):
            ctx.generate(np.array([], dtype=np.uint32), 5)


def test_decoding_is_deterministic_across_runs():
    with native.Context(MINI) as ctx:
        ctx.load_synthetic(seed=9)
        a = [ctx.step(PROMPT)[0]] + [ctx.step([t])[0] for t in (7, 8, 9)]
        ctx.begin_sequence()
        b = [ctx.step(PROMPT)[0]] + [ctx.step([t])[0] for t in (7, 8, 9)]
        for x, y in zip(a, b):
            np.testing.assert_array_equal(x, y)


# ---- the two fast decode paths -----------------------------------------------

MINI_PERSISTENT = MINI.replace(intermediate=16384)


def test_persistent_path_matches_reference_across_context_splits():
    """The whole-loop kernel (one cooperative launch per call) on a shape it
    serves, token by token across 1 to 8 attention splits, past 128 keys
    eight splits of two and three double-buffered 16-key tiles."""
    p = Pair(MINI_PERSISTENT, seed=13)
    try:
        assert p.ctx.decode_path == native.DECODE_PERSISTENT
        prompt = native.synthetic_tokens(13, 60, MINI_PERSISTENT.vocab)
        worst = p.step(prompt)
        for i in range(210):
            worst = max(worst, p.step([int(prompt[(7 * i) % 60])]))
        assert worst <= TOLERANCE, worst
    finally:
        p.close()


def test_persistent_path_matches_reference_across_the_merge_phase():
    """Up to 512 keys eight splits of up to four tiles, folded while o_proj
    stages its input; past 512 one 16-key split per CTA and a merge phase:
    a 496-token prompt, then token by token from 497 to 536 keys."""
    shape = MINI_PERSISTENT.replace(max_positions=544, max_step_rows=512)
    p = Pair(shape, seed=17)
    try:
        assert p.ctx.decode_path == native.DECODE_PERSISTENT
        prompt = native.synthetic_tokens(17, 496, shape.vocab)
        worst = p.step(prompt)
        for i in range(40):
            worst = max(worst, p.step([int(prompt[(5 * i) % 496])]))
        assert worst <= TOLERANCE, worst
    finally:
        p.close()


def test_graph_and_persistent_paths_agree():
    with native.Context(MINI_PERSISTENT) as ctx:
        ctx.load_synthetic(seed=21)
        rows = {}
        for path in (native.DECODE_GRAPH, native.DECODE_PERSISTENT):
            ctx.set_decode_path(path)
            ctx.begin_sequence()
            out = [ctx.step(PROMPT)]
            out += [ctx.step([t]) for t in (3, 1, 4, 1, 5, 9, 2, 6)]
            rows[path] = out
        for (lg, hd), (lp, hp) in zip(rows[native.DECODE_GRAPH], rows[native.DECODE_PERSISTENT]):
            assert ob.worst_error(lp, lg) <= TOLERANCE
            assert ob.worst_error(hp, hd) <= TOLERANCE


def test_persistent_multi_step_launches_feed_tokens_back():
    """decode_async with many steps per launch: the token each step writes is
    the one the next step embeds, inside the kernel."""
    shape = MINI_PERSISTENT.replace(embed_scale=1.0)
    with native.Context(shape) as ctx:
        tensors = ctx.load_synthetic(seed=5, keep=True)
        assert ctx.decode_path == native.DECODE_PERSISTENT
        expected = ob.greedy_reference(shape, tensors, PROMPT, 40)
        assert len(set(expected)) > 3
        assert list(ctx.generate(PROMPT, 40)) == expected
        ctx.prefill_async(PROMPT)
        ctx.decode_async(39)  # one launch
        assert ctx.decode_launches(5) == 1
        assert list(ctx.read_slots(len(PROMPT), 40)) == expected
