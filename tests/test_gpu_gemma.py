"""BASELINE config 0 on the B200: random-init Gemma-2B (seed 0), BOS + 15
prompt ids, 32 greedy decode steps, through the C-ABI.

Gates: greedy tokens bit-identical to the oracle
over 32 steps; logits max-abs <= 1e-2 x (max - min) and cosine >= 0.9999 per
step. The tokens and per-step top-64 logits are pinned in
tests/golden/gemma2b_config0.npz (tests/golden/make_golden.py, the double
oracle); the whole logits rows are checked against the double oracle run live
on the host over the same Q8_0 bytes.
"""
import os

import numpy as np
import pytest

import oracle_bindings as ob
from huggingfaceeacp_b200 import native

pytestmark = pytest.mark.gpu

LOGIT_RANGE_TOLERANCE = 1e-2
COSINE_FLOOR = 0.9999
STEPS = 32


@pytest.fixture(scope="module")
def gemma():
    golden = np.load(os.path.join(ob.GOLDEN_DIR, "gemma2b_config0.npz"))
    shape = native.GEMMA_2B.replace(max_step_rows=512)
    ctx = native.Context(shape)
    tensors = ctx.load_synthetic(seed=0, keep=True)
    yield ctx, tensors, golden
    ctx.close()


def test_config0_prompt_is_the_seeded_prompt(gemma):
    _, _, golden = gemma
    np.testing.assert_array_equal(native.synthetic_tokens(0, 16, 256000), golden["prompt"])


def test_config0_greedy_tokens_are_bit_identical(gemma):
    ctx, _, golden = gemma
    tokens = ctx.generate(golden["prompt"], STEPS)
    np.testing.assert_array_equal(tokens, golden["tokens"])


def test_config0_logits_within_tolerance_of_the_oracle(gemma):
    ctx, tensors, golden = gemma
    oracle = ob.OracleModel(native.GEMMA_2B.replace(max_positions=64), tensors, precision="double")
    ctx.begin_sequence()
    prompt = golden["prompt"]
    logits, _ = ctx.step(prompt, want_hidden=False)
    _, expected = oracle.step(prompt, last_row_only=True, want_hidden=False)
    row = logits[-1]
    worst_ratio, worst_cos = 0.0, 1.0
    for step in range(STEPS):
        ref = expected[-1]
        span = float(ref.max() - ref.min())
        ratio = float(np.max(np.abs(row.astype(np.float64) - ref))) / span
        cos = float(np.dot(row, ref) / (np.linalg.norm(row) * np.linalg.norm(ref)))
        worst_ratio, worst_cos = max(worst_ratio, ratio), min(worst_cos, cos)
        # the pinned top-64 of the fixture
        top = golden["top_index"][step]
        assert np.max(np.abs(row[top] - golden["top_value"][step])) <= LOGIT_RANGE_TOLERANCE * golden["logits_range"][step]
        token = int(np.argmax(row))  # first index of the maximum
        assert token == ob.argmax(ref) == int(golden["tokens"][step])
        if step + 1 < STEPS:
            logits, _ = ctx.step([token], want_hidden=False)
            row = logits[-1]
            _, expected = oracle.step([token], want_hidden=False)
    oracle.close()
    assert worst_ratio <= LOGIT_RANGE_TOLERANCE, worst_ratio
    assert worst_cos >= COSINE_FLOOR, worst_cos
