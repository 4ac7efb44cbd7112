"""Sampling on the device (hf_cuda_sample, hf_cuda_generate_sampled) against
the reference's own Sampler (Sampling/Sampler.cpp:78-215, compiled unchanged
into oracle/_ref by oracle/build_ref.sh): the same tokens, draw for draw, for
the reference's option order (temperature, top-k, top-p) on Gemma-sized
rows, with ties and suppressed tokens, and a sampled generation equal to the
host-driven loop (Gemma::generateBySampling, Gemma.cpp:545-592) that samples
the decoder's own logits with the reference Sampler."""
import numpy as np
import pytest

import oracle_bindings as ob
from huggingfaceeacp_b200 import native

pytestmark = pytest.mark.gpu

ROWS = native.GEMMA_2B.replace(layers=1, max_positions=128, max_step_rows=16)  # vocab 256000; no weights needed


@pytest.fixture(scope="module")
def rows_ctx():
    with native.Context(ROWS) as ctx:
        yield ctx


def _row(seed, peaked=False):
    rng = np.random.default_rng(seed)
    logits = rng.normal(0.0, 2.0, ROWS.vocab).astype(np.float32)
    logits[rng.integers(0, ROWS.vocab, 4000)] = np.float32(1.5)  # ties, broken by the lower token
    if peaked:
        logits[rng.integers(0, ROWS.vocab, 60)] += np.float32(14.0)  # a nucleus of a few dozen tokens
    return logits


CASES = [
    dict(temperature=0.7, top_k=40, top_p=1.0),
    dict(temperature=1.0, top_k=40, top_p=0.9),
    dict(temperature=1.3, top_k=1024, top_p=0.95),
    dict(temperature=0.5, top_k=5, top_p=0.5),
    dict(temperature=1.0, top_k=1, top_p=1.0),
    dict(temperature=0.8, top_k=0, top_p=0.9, peaked=True),
    dict(temperature=1.0, top_k=0, top_p=1.0),
    dict(temperature=2.0, top_k=300, top_p=1.0),
]


@pytest.mark.parametrize("case", CASES, ids=[str(i) for i in range(len(CASES))])
def test_device_draws_equal_the_reference_sampler(rows_ctx, case):
    case = dict(case)
    logits = _row(100 + CASES.index(case), peaked=case.pop("peaked", False))
    expected = ob.ref_sample(logits, None, seed=7, draws=64, **case)
    got = rows_ctx.sample(logits, seed=7, draws=64, **case)
    np.testing.assert_array_equal(got, expected)


def test_suppressed_tokens_and_all_suppressed(rows_ctx):
    logits = _row(5)
    mask = np.zeros(ROWS.vocab, np.float32)
    mask[np.argsort(logits)[-200:]] = 1.0  # the 200 best are out of the running
    for case in (dict(temperature=1.0, top_k=50, top_p=0.9), dict(temperature=0.9, top_k=0, top_p=1.0)):
        expected = ob.ref_sample(logits, mask, seed=11, draws=32, **case)
        np.testing.assert_array_equal(rows_ctx.sample(logits, seed=11, draws=32, mask=mask, **case), expected)
    everything = np.ones(ROWS.vocab, np.float32)  # no candidate: token 0 and no draw (Sampler.cpp:87-88)
    expected = ob.ref_sample(logits, everything, temperature=1.0, top_k=10, top_p=1.0, seed=3, draws=3)
    assert list(expected) == [0, 0, 0]
    np.testing.assert_array_equal(rows_ctx.sample(logits, temperature=1.0, top_k=10, seed=3, draws=3,
                                                  mask=everything), expected)


def test_zero_temperature_is_the_argmax(rows_ctx):
    logits = _row(9)
    assert list(rows_ctx.sample(logits, temperature=0.0, draws=2)) == [int(np.argmax(logits))] * 2


def test_refused_options(rows_ctx):
    logits = _row(1)
    for bad in (dict(temperature=-1.0), dict(temperature=1.0, top_k=-1), dict(temperature=1.0, top_p=0.0),
                dict(temperature=1.0, top_p=1.5), dict(temperature=1.0, top_k=2000)):
        with pytest.raises(native.HFError) as err:
            rows_ctx.sample(logits, **bad)
        assert err.value.code == native.HF_E_INVALID


def test_sampled_generation_equals_the_host_loop():
    """Gemma::generateBySampling: the decoder's logits, one reference draw per
    token, the token fed back. The host loop's logits come from hf_cuda_step
    and agree with the generation's to float rounding, so the fixed seed's
    draws are the same tokens unless a uniform lands within that rounding of
    a cumulative boundary."""
    shape = native.DecoderShape(width=2048, heads=8, kv_heads=1, head_width=256, layers=2, intermediate=16384,
                                vocab=8192, max_positions=64, max_step_rows=16, embed_scale=1.0)
    options = dict(temperature=0.9, top_k=40, top_p=0.95)
    with native.Context(shape) as ctx:
        ctx.load_synthetic(seed=31)
        prompt = native.synthetic_tokens(31, 17, shape.vocab)
        got = ctx.generate_sampled(prompt, 12, seed=5, **options)
        ctx.begin_sequence()
        ctx.step(prompt[:16], want_hidden=False)
        logits, _ = ctx.step(prompt[16:], want_hidden=False)
        expected = []
        for t in range(12):
            token = ob.ref_sample_at(logits[-1], seed=5, skip=t, **options)
            expected.append(token)
            if t + 1 < 12:
                logits, _ = ctx.step([token], want_hidden=False)
        assert list(got) == expected
        assert len(set(expected)) > 3  # the draws vary
