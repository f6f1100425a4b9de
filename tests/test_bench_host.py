"""Host logic of the batched multi-GPU bench line on CPU: two gloo ranks, each with its own
sequences' timings, combine into one job (all sequences' tokens over the slowest rank's wall and
device times), the same on every rank.  No GPU: batch_job_rates takes the collective as an argument."""
import multiprocessing as mp
import socket


def _local(rank: int) -> dict:
    # rank 1 is the slower one in wall time, rank 0 in device time
    return {"sequences": 8, "prompt": 128, "generated": 16,
            "prefill": {"tok_s": 0.0, "device_tok_s": 8 * 128 / (0.50 if rank == 0 else 0.40), "seconds": 0.6 + 0.1 * rank},
            "decode": {"tok_s": 0.0, "device_tok_s": 0.0, "seconds": 0.3 + 0.2 * rank, "ms_per_step": 20.0 - 2.0 * rank}}


def _rank(rank: int, world: int, port: int, out) -> None:
    import torch
    import torch.distributed as dist
    import bench
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        def slowest(v):
            t = torch.tensor(v, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return t.tolist()
        out.put((rank, bench.batch_job_rates(_local(rank), 16, 128, 16, slowest)))
    finally:
        dist.destroy_process_group()


def test_batch_job_rates_gloo_world2():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        got = dict(q.get(timeout=120) for _ in range(2))
        for p in procs:
            p.join(timeout=60)
            assert p.exitcode == 0
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
    assert got[0] == got[1]
    r = got[0]
    assert r["sequences"] == 16
    assert abs(r["prefill"]["seconds"] - 0.7) < 1e-12 and abs(r["prefill"]["tok_s"] - 16 * 128 / 0.7) < 1e-6
    assert abs(r["prefill"]["device_tok_s"] - 16 * 128 / 0.50) < 1e-6  # rank 0's device time is the longer
    assert abs(r["decode"]["seconds"] - 0.5) < 1e-12 and abs(r["decode"]["tok_s"] - 16 * 16 / 0.5) < 1e-6
    assert r["decode"]["ms_per_step"] == 20.0
    assert abs(r["decode"]["device_tok_s"] - 16 * 16 / (20.0 * 16 / 1e3)) < 1e-6
