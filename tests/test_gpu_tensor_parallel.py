"""Tensor-parallel prefill over NCCL (hf_cuda_set_tensor_parallel) on two
GPUs of one box: two processes, one context per GPU, each holding the whole
model and running the feed-forward of every prefill block on its half, the
down partial sums added by one NCCL allreduce per layer. Both ranks' rows must
equal the double oracle's at the decoder tolerance (DecoderTests.cpp:41), equal
each other bit for bit (the allreduce hands every rank the same sums), and the
greedy continuation must equal the host-driven reference loop. Needs two
GPUs; skipped on one.
"""
import multiprocessing
import os
import socket

import numpy as np
import pytest

import oracle_bindings as ob

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOLERANCE = 5e-6
LAYERS, VOCAB, POSITIONS, STEP_ROWS = 2, 8192, 640, 256
PROMPT_LENGTH, TOKENS, SEED = 600, 6, 21


def _shape():
    from huggingfaceeacp_b200 import native

    return native.DecoderShape(width=2048, heads=8, kv_heads=1, head_width=256, layers=LAYERS, intermediate=16384,
                               vocab=VOCAB, max_positions=POSITIONS, max_step_rows=STEP_ROWS, embed_scale=1.0)


def _rank(rank: int, world: int, port: int, out):
    import datetime

    import torch.distributed as dist

    from huggingfaceeacp_b200 import native

    torch.cuda.set_device(rank)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        shape = _shape()
        with native.Context(shape, device=rank) as ctx:
            ctx.load_synthetic(seed=SEED)
            nccl_id = native.broadcast_bytes(dist, native.nccl_unique_id() if rank == 0 else None,
                                             native.NCCL_ID_BYTES)
            ctx.set_tensor_parallel(rank, world, nccl_id)
            prompt = native.synthetic_tokens(SEED, PROMPT_LENGTH, shape.vocab)
            ctx.begin_sequence()
            for first in range(0, PROMPT_LENGTH, STEP_ROWS):  # steps of 256, 256 and 88 rows
                logits, hidden = ctx.step(prompt[first:first + STEP_ROWS])
            tokens = ctx.generate(prompt, TOKENS)
            out.put((rank, logits[-8:].copy(), hidden.copy(), list(tokens)))
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="tensor-parallel prefill needs two GPUs")
def test_two_rank_prefill_equals_the_oracle():
    from huggingfaceeacp_b200 import native

    ctx = multiprocessing.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict((r, rest) for r, *rest in (out.get(timeout=600) for _ in procs))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    (l0, h0, t0), (l1, h1, t1) = got[0], got[1]
    assert np.array_equal(l0, l1) and np.array_equal(h0, h1) and t0 == t1
    shape = _shape()
    tensors = {k: native.synthetic_tensor(shape, k[0], k[1], SEED) for k in native.model_tensors(shape)}
    prompt = native.synthetic_tokens(SEED, PROMPT_LENGTH, shape.vocab)
    oracle = ob.OracleModel(shape, tensors, precision="double")
    ref_hidden, ref_logits = oracle.step(prompt)
    oracle.close()
    last = PROMPT_LENGTH - (PROMPT_LENGTH - 1) // STEP_ROWS * STEP_ROWS  # rows of the last step
    assert ob.worst_error(l0, ref_logits[-8:]) <= TOLERANCE
    assert ob.worst_error(h0, ref_hidden[-last:]) <= TOLERANCE
    assert t0 == ob.greedy_reference(shape, tensors, prompt, TOKENS)
