"""Batched greedy decode of independent sequences through the C-ABI:
hf_cuda_create_batch, hf_cuda_prefill_batch_async, hf_cuda_decode_batch_async,
hf_cuda_read_batch_slots, hf_cuda_generate_batch.

Every sequence of a batch must produce exactly the tokens the host-driven
reference loop (Tests/Generation/Common.h:248-300) produces for that sequence
alone, on a Gemma-shaped decoder whose embedding scale is 1 so the greedy
sequences vary; the context's single-sequence calls use a window of their own.
"""
import numpy as np
import pytest

import oracle_bindings as ob
from huggingfaceeacp_b200 import native

pytestmark = pytest.mark.gpu

SHAPE = native.DecoderShape(width=2048, heads=8, kv_heads=1, head_width=256, layers=2, intermediate=16384,
                            vocab=8192, max_positions=128, max_step_rows=64, embed_scale=1.0)
SEED = 41
SEQUENCES = 5  # odd: the last pair of rows of a product block is half used
PROMPT = 70    # two prefill blocks; 71-82 keys: two attention splits per sequence
TOKENS = 12


@pytest.fixture(scope="module")
def batch():
    ctx = native.Context(SHAPE, sequences=SEQUENCES)
    tensors = ctx.load_synthetic(seed=SEED, keep=True)
    prompts = np.stack([native.synthetic_tokens(100 + q, PROMPT, SHAPE.vocab) for q in range(SEQUENCES)])
    yield ctx, tensors, prompts
    ctx.close()


def test_every_sequence_of_a_batch_matches_its_own_reference_loop(batch):
    ctx, tensors, prompts = batch
    out = ctx.generate_batch(prompts, TOKENS)
    assert out.shape == (SEQUENCES, TOKENS)
    distinct = set()
    for q in range(SEQUENCES):
        expected = ob.greedy_reference(SHAPE, tensors, prompts[q], TOKENS)
        assert list(out[q]) == expected, q
        distinct.update(expected)
    assert len(distinct) > SEQUENCES  # the sequences differ and vary


def test_batched_steps_continue_from_where_they_stopped(batch):
    ctx, tensors, prompts = batch
    ctx.prefill_batch_async(prompts)
    ctx.decode_batch_async(4)
    ctx.decode_batch_async(TOKENS - 5)
    out = ctx.read_batch_slots(PROMPT, TOKENS)
    assert np.array_equal(out, ctx.generate_batch(prompts, TOKENS))


def test_identical_prompts_give_identical_rows(batch):
    ctx, tensors, prompts = batch
    out = ctx.generate_batch(np.stack([prompts[3]] * SEQUENCES), 6)
    assert all(np.array_equal(row, out[0]) for row in out)


def test_single_sequence_calls_use_their_own_window(batch):
    ctx, tensors, prompts = batch
    ctx.prefill_batch_async(prompts)
    expected = ob.greedy_reference(SHAPE, tensors, prompts[2], 8)
    assert list(ctx.generate(prompts[2], 8)) == expected
    # The batched sequences are untouched by the single-sequence run.
    ctx.decode_batch_async(TOKENS - 1)
    assert np.array_equal(ctx.read_batch_slots(PROMPT, TOKENS), ctx.generate_batch(prompts, TOKENS))


def test_batch_refusals():
    with pytest.raises(native.HFError) as too_many:
        native.Context(SHAPE, sequences=SHAPE.max_step_rows + 1)
    assert too_many.value.code == native.HF_E_CAPACITY
    narrow = SHAPE.replace(intermediate=4096)  # not a shape the stage records serve
    with pytest.raises(native.HFError) as shape:
        native.Context(narrow, sequences=2)
    assert shape.value.code == native.HF_E_SHAPE
    with native.Context(SHAPE, sequences=2) as ctx:
        ctx.load_synthetic(seed=SEED)
        with pytest.raises(native.HFError) as empty:
            ctx.decode_batch_async(1)  # nothing prefilled
        assert empty.value.code == native.HF_E_INVALID
        with pytest.raises(native.HFError) as window:
            ctx.generate_batch(np.zeros((2, 100), np.uint32), 30)
        assert window.value.code == native.HF_E_WINDOW
