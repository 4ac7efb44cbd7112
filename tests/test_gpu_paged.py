"""Batched decode over the paged KV cache (hf_cuda_create_paged,
hf_cuda_admit_async, hf_cuda_release, hf_cuda_decode_batch_async).

The reference decodes one sequence over one contiguous cache per layer
(DecoderShape.h:105, Decoder.cpp:199-203). Here the batched sequences keep
their K/V rows in pages of 64 positions drawn from one pool, found through a
page table, so sequences of different lengths share a step and join and leave
between steps. Every active sequence must produce exactly the tokens of the
host-driven reference loop (Tests/Generation/Common.h:248-300) for its prompt
alone, whatever its neighbours do; the pool's accounting and refusals are
checked alongside. Gemma widths, two layers, embedding scale 1 (varied tokens).
"""
import numpy as np
import pytest

import oracle_bindings as ob
from huggingfaceeacp_b200 import native

pytestmark = pytest.mark.gpu

SHAPE = native.DecoderShape(width=2048, heads=8, kv_heads=1, head_width=256, layers=2, intermediate=16384,
                            vocab=8192, max_positions=320, max_step_rows=128, embed_scale=1.0)
SEED = 43
PAGE = native.PAGE_ROWS


def prompt(q, length):
    return native.synthetic_tokens(500 + q, length, SHAPE.vocab)


@pytest.fixture(scope="module")
def model():
    ctx = native.Context(SHAPE, sequences=6, pages=40)
    tensors = ctx.load_synthetic(seed=SEED, keep=True)
    yield ctx, tensors
    ctx.close()


def expected(tensors, q, length, tokens):
    return ob.greedy_reference(SHAPE, tensors, prompt(q, length), tokens)


def test_sequences_of_different_lengths_share_steps(model):
    ctx, tensors = model
    lengths = {0: 5, 1: 70, 2: 130, 3: 64, 4: 200, 5: 1}  # within a page, across pages, on page edges
    for q in range(6):
        if ctx.sequence_position(q) >= 0:
            ctx.release(q)
    assert ctx.free_pages == 40
    for q, n in lengths.items():
        ctx.admit_async(q, prompt(q, n))
    assert ctx.free_pages == 40 - sum((n + PAGE - 1) // PAGE for n in lengths.values())
    ctx.decode_batch_async(11)
    for q, n in lengths.items():
        assert ctx.sequence_position(q) == n + 11
        got = ctx.read_batch_slots(0, SHAPE.max_positions + 1)[q, n:n + 12]
        assert list(got) == expected(tensors, q, n, 12), q


def test_sequences_join_and_leave_between_steps(model):
    ctx, tensors = model
    for q in range(6):
        if ctx.sequence_position(q) >= 0:
            ctx.release(q)
    ctx.admit_async(0, prompt(0, 40))
    ctx.admit_async(3, prompt(3, 100))
    ctx.decode_batch_async(4)
    ctx.admit_async(5, prompt(5, 63))   # joins four steps later
    ctx.release(3)                      # leaves; its pages go back to the pool
    ctx.admit_async(2, prompt(2, 150))  # takes pages the released sequence held
    ctx.decode_batch_async(7)
    slots = ctx.read_batch_slots(0, SHAPE.max_positions + 1)
    assert list(slots[0, 40:52]) == expected(tensors, 0, 40, 12)
    assert list(slots[5, 63:71]) == expected(tensors, 5, 63, 8)
    assert list(slots[2, 150:158]) == expected(tensors, 2, 150, 8)
    assert list(slots[3, 100:105]) == expected(tensors, 3, 100, 5)  # what it made before it left
    assert ctx.sequence_position(3) == -1 and ctx.sequence_position(0) == 51


def test_pool_refusals_leave_the_batch_as_it_was():
    with native.Context(SHAPE, sequences=2, pages=4) as ctx:
        tensors = ctx.load_synthetic(seed=SEED, keep=True)
        with pytest.raises(native.HFError) as big:
            ctx.admit_async(0, prompt(0, 4 * PAGE + 1))  # five pages
        assert big.value.code == native.HF_E_CAPACITY
        assert ctx.free_pages == 4 and ctx.sequence_position(0) == -1
        ctx.admit_async(0, prompt(0, 2 * PAGE))      # two pages
        ctx.admit_async(1, prompt(1, PAGE + 10))     # two pages: the pool is empty
        assert ctx.free_pages == 0
        with pytest.raises(native.HFError) as again:
            ctx.admit_async(1, prompt(1, 3))
        assert again.value.code == native.HF_E_INVALID  # sequence 1 is active
        with pytest.raises(native.HFError) as grow:
            ctx.decode_batch_async(1)  # sequence 0 would need a third page
        assert grow.value.code == native.HF_E_CAPACITY
        assert ctx.sequence_position(0) == 2 * PAGE
        ctx.release(0)
        ctx.decode_batch_async(5)  # sequence 1 alone, inside its second page
        got = ctx.read_batch_slots(PAGE + 10, 6)[1]
        assert list(got) == ob.greedy_reference(SHAPE, tensors, prompt(1, PAGE + 10), 6)
        with pytest.raises(native.HFError) as window:
            ctx.admit_async(0, prompt(0, SHAPE.max_positions + 1))
        assert window.value.code == native.HF_E_WINDOW
