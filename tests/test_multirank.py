"""The multi-GPU host logic of bench.py on CPU: one process per rank over the
gloo backend (world size 2), as torchrun launches the bench on N GPUs.

- max_over_ranks: every rank gets the element-wise maximum of all ranks'
  device times (a multi-GPU time is the slowest rank's), at the same call on
  every rank;
- the reference arm: ranks other than 0 exit 0 without work, rank 0 alone
  times and prints.
"""
import multiprocessing
import os
import socket
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out):
    sys.path.insert(0, ROOT)
    import torch.distributed as dist

    import bench

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        # three timed regions in the bench's order, each rank its own times
        first = bench.max_over_ranks(dist, [10.0 + rank], device="cpu")
        pair = bench.max_over_ranks(dist, [5.0 - rank, 0.25 * (rank + 1)], device="cpu")
        last = bench.max_over_ranks(dist, [3.0 if rank == 1 else 1.0], device="cpu")
        out.put((rank, first, pair, last))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_with_two_gloo_ranks():
    ctx = multiprocessing.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    results = [out.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, first, pair, last in results:
        assert first == [11.0]
        assert pair == [5.0, 0.5]
        assert last == [3.0]


def test_max_over_ranks_in_one_process_is_the_identity():
    sys.path.insert(0, ROOT)
    import bench

    assert bench.max_over_ranks(None, [1.5, 2]) == [1.5, 2.0]


def test_reference_arm_rank_other_than_zero_does_no_work(monkeypatch, capsys):
    sys.path.insert(0, ROOT)
    import bench

    monkeypatch.setenv("RANK", "1")
    monkeypatch.setenv("WORLD_SIZE", "2")

    class Args:
        steps, warmup, gpus = 1, 3, 2

    assert bench.run_reference(Args()) == 0
    assert capsys.readouterr().out == ""


def _id_rank_main(rank: int, world: int, port: int, out):
    sys.path.insert(0, ROOT)
    import torch.distributed as dist

    from huggingfaceeacp_b200 import native

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        # rank 0's communicator id reaches every rank unchanged (the tensor-parallel
        # prefill's set-up; the id's bytes stand in for hf_cuda_nccl_unique_id's)
        payload = bytes((i * 37 + 11) % 256 for i in range(native.NCCL_ID_BYTES)) if rank == 0 else None
        out.put((rank, native.broadcast_bytes(dist, payload, native.NCCL_ID_BYTES)))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_id_reaches_every_rank():
    ctx = multiprocessing.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_id_rank_main, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(out.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    expected = bytes((i * 37 + 11) % 256 for i in range(128))
    assert got[0] == expected and got[1] == expected
