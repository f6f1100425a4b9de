"""Expert parallelism: one engine per GPU, each holding experts/world of every
layer's experts, exchanging the partial MoE vectors over NVLink inside the
whole-token kernel.

Every rank must produce the same logits (each sums x' and the ranks' partials
in rank order) and match the CPU oracle within the north-star tolerance
(max-abs 2e-2, top-1), and greedy decoding must reproduce the golden tokens.
The ranks' sum order differs from the one-GPU combine, so agreement with the
one-GPU engine is up to fp32 reassociation, not bitwise."""
import multiprocessing as mp

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def _gpus() -> int:
    import torch
    return torch.cuda.device_count()


def _run_ranks(world: int, tokens, prompt_len: int, n_greedy: int):
    import _ep_worker
    ctx = mp.get_context("spawn")
    up = ctx.Queue()
    downs = [ctx.Queue() for _ in range(world)]
    procs = [ctx.Process(target=_ep_worker.run, args=(r, world, up, downs[r], tokens, prompt_len, n_greedy))
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        handles, done = {}, {}
        while len(done) < world:
            kind, rank, payload = up.get(timeout=300)
            assert kind != "error", f"rank {rank}:\n{payload}"
            if kind == "handle":
                handles[rank] = payload
                if len(handles) == world:
                    for q in downs:
                        q.put([handles[r] for r in range(world)])
            else:
                done[rank] = payload
        for p in procs:
            p.join(timeout=60)
        return [done[r] for r in range(world)]
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_expert_parallel_matches_oracle(oracle, tools, world):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    z = np.load(GOLDEN / "tiny_q_golden.npz")
    tokens, golden, n0 = z["tokens"].tolist(), z["logits"], int(z["prompt_len"])
    out = _run_ranks(world, tokens, n0, 32)
    m = oracle.Model(tools.synth_gguf(tools.TINY), 64)
    ref = [m.forward(int(t)) for t in tokens]
    for rank, (logits, toks, pos) in enumerate(out):
        for p, (g, o) in enumerate(zip(logits, ref)):
            assert np.array_equal(g, out[0][0][p]), (rank, p)  # the same bits on every rank
            err = float(np.abs(g - o).max())
            assert err < 2e-2 and err < 1e-4 * max(1.0, float(np.abs(o).max())), (rank, p, err)
            assert np.abs(g - golden[p]).max() < 2e-2
            assert int(np.argmax(g)) == oracle.sample_greedy(o), (rank, p)
        assert toks == tokens[n0:n0 + 32], rank
        assert pos == n0 + 32


def test_expert_parallel_refusals(cuda_engine, tools):
    """Host-side checks of the expert-parallel entry points (one GPU)."""
    img = tools.synth_gguf(tools.TINY)  # 8 experts
    E = cuda_engine.Engine
    with pytest.raises(cuda_engine.QwenCudaError, match="multiple of the world size"):
        E.expert_parallel(img, 16, 0, 0, 3)
    with pytest.raises(cuda_engine.QwenCudaError, match="rank < world"):
        E.expert_parallel(img, 16, 0, 2, 2)
    with pytest.raises(cuda_engine.QwenCudaError, match="world <= 8"):
        E.expert_parallel(img, 16, 0, 0, 16)
    e = E.expert_parallel(img, 16, 0, 0, 2)
    assert e.decode_path == (0, "")
    with pytest.raises(cuda_engine.QwenCudaError, match="not connected"):
        e.forward(1)
    with pytest.raises(cuda_engine.QwenCudaError, match="only the whole-token kernel"):
        e.set_decode_mode(1)
    h, dev = e.ep_handle()
    assert len(h) == 64
    with pytest.raises(cuda_engine.QwenCudaError, match="different GPUs"):  # both ranks on one GPU
        e.connect([(h, dev), (h, dev)])
    with pytest.raises(cuda_engine.QwenCudaError, match="not connected"):
        e.forward(1)
    single = E(img, 16)
    with pytest.raises(cuda_engine.QwenCudaError, match="not an expert-parallel engine"):
        single.ep_handle()


def test_peer_gone_times_out_and_gpu_stays_usable(cuda_engine):
    """A rank that stops between steps: the other rank's next token ends with the timeout error
    within a few seconds (bounded waits of 2 s, no GPU fault), its position resets, and the GPU
    still runs a fresh engine.  Host-side failure only; no NCCL, plain peer stores."""
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    import _ep_worker
    ctx = mp.get_context("spawn")
    up = ctx.Queue()
    downs = [ctx.Queue() for _ in range(2)]
    procs = [ctx.Process(target=_ep_worker.run_peer_gone, args=(r, 2, up, downs[r], [3, 1, 4]))
             for r in range(2)]
    for p in procs:
        p.start()
    try:
        handles, synced, done = {}, set(), {}
        while len(done) < 2:
            kind, rank, payload = up.get(timeout=300)
            assert kind != "error", f"rank {rank}:\n{payload}"
            if kind == "handle":
                handles[rank] = payload
                if len(handles) == 2:
                    for q in downs:
                        q.put([handles[r] for r in range(2)])
            elif kind == "synced":
                synced.add(rank)
                if len(synced) == 2:
                    downs[0].put("go")
            else:
                done[rank] = payload
                if rank == 0:
                    downs[1].put("finish")
        for p in procs:
            p.join(timeout=60)
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
    code, msg, seconds, pos, fresh_ok = done[0]
    assert code == cuda_engine.ERR_CUDA and "timed out" in msg, (code, msg)
    assert seconds < 30, seconds
    assert pos == 0  # a failed forward resets the cache, as model.rs:210-216 does
    assert fresh_ok
