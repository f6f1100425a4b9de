"""Host logic of expert parallelism on CPU: the handle exchange over a
world_size-2 gloo group (engine.connect_group) delivers every rank's handle
to every rank in rank order.  No GPU: the engine is a stand-in object."""
import multiprocessing as mp
import socket


class _FakeEngine:
    def __init__(self, rank: int):
        self.rank = rank
        self.got = None

    def ep_handle(self):
        return bytes([self.rank]) * 64, 1000 + self.rank

    def connect(self, handles):
        self.got = handles


def _rank(rank: int, world: int, port: int, out) -> None:
    import torch.distributed as dist
    from conftest import load_package  # noqa: F401
    from qwen30brust_b200 import engine as E
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        eng = _FakeEngine(rank)
        E.connect_group(eng)
        out.put((rank, eng.got))
    finally:
        dist.destroy_process_group()


def test_connect_group_gloo_world2():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        got = dict(out.get(timeout=120) for _ in range(2))
        for p in procs:
            p.join(timeout=60)
            assert p.exitcode == 0
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
    want = [(bytes([r]) * 64, 1000 + r) for r in range(2)]
    assert got[0] == want and got[1] == want
