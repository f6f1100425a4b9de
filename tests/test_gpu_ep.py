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


def _spawn(world: int, target, args_of, go_after_sync: bool = False):
    """Runs target(rank, world, up, down, *args_of(rank)) on `world` processes: relays the handles,
    and (go_after_sync) tells rank 0 to go on once every rank has synced, then rank 1 to finish once
    rank 0 is done.  Returns each rank's result."""
    ctx = mp.get_context("spawn")
    up = ctx.Queue()
    downs = [ctx.Queue() for _ in range(world)]
    procs = [ctx.Process(target=target, args=(r, world, up, downs[r], *args_of(r))) for r in range(world)]
    for p in procs:
        p.start()
    try:
        handles, synced, done = {}, set(), {}
        while len(done) < world:
            kind, rank, payload = up.get(timeout=300)
            assert kind != "error", f"rank {rank}:\n{payload}"
            if kind == "handle":
                handles[rank] = payload
                if len(handles) == world:
                    for q in downs:
                        q.put([handles[r] for r in range(world)])
            elif kind == "synced":
                synced.add(rank)
                if go_after_sync and len(synced) == world:
                    downs[0].put("go")
            else:
                done[rank] = payload
                if go_after_sync and rank == 0:
                    for q in downs[1:]:
                        q.put("finish")
        for p in procs:
            p.join(timeout=60)
        return [done[r] for r in range(world)]
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()


def _batch_calls(rank: int, vocab: int):
    """Rank `rank`'s calls for 3 sequences, with the same token counts on every rank: whole prompts
    (26 tokens), a 140-token call of two passes (100 + 40 tokens, interleaved), 4 decode steps in a
    shuffled order."""
    rng = np.random.default_rng(100 + rank)
    calls = []
    prompts = [rng.integers(0, vocab, n).tolist() for n in (5, 9, 12)]
    calls.append(([0] * 5 + [1] * 9 + [2] * 12, sum(prompts, [])))
    a, b = rng.integers(0, vocab, 100).tolist(), rng.integers(0, vocab, 40).tolist()
    seqs, toks = [], []
    for i in range(100):
        seqs.append(0)
        toks.append(a[i])
        if i < 40:
            seqs.append(1)
            toks.append(b[i])
    calls.append((seqs, toks))
    for _ in range(4):
        perm = rng.permutation(3).tolist()
        calls.append((perm, rng.integers(0, vocab, 3).tolist()))
    return calls


@pytest.mark.parametrize("world", [2, 4, 8])
def test_batched_expert_parallel_matches_oracle(oracle, tools, world):
    """BASELINE config 5's split on `world` GPUs: every rank's sequences against the oracle run on
    each sequence alone, and against a one-GPU batch of the same calls (logits within 1e-4 of its
    largest element; the device decode loop samples the same ids)."""
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    import _ep_worker
    spec = tools.TINY
    params = [(11, 0.7, 0, 0.9), (12, 1.0, 5, 1.0), (13, 0.0, 0, 1.0)]
    out = _spawn(world, _ep_worker.run_batch, lambda r: (_batch_calls(r, spec.vocab), params, 6))
    img = tools.synth_gguf(spec)
    worst = 0.0
    for rank, (rows, ids, pos, rows1, ids1) in enumerate(out):
        refs = [oracle.Model(img, 256) for _ in range(3)]
        for (seqs, toks), got, one in zip(_batch_calls(rank, spec.vocab), rows, rows1):
            last = {}
            for q, t in zip(seqs, toks):
                last[q] = refs[q].forward(t)
            order = list(dict.fromkeys(reversed(seqs)))[::-1]
            assert got.shape == (len(order), spec.vocab)
            for r, r1, q in zip(got, one, order):
                err = float(np.abs(r - last[q]).max())
                assert err < 2e-2 and int(np.argmax(r)) == int(np.argmax(last[q])), (rank, q, err)
                worst = max(worst, err)
                assert float(np.abs(r - r1).max()) <= 1e-4 * max(1.0, float(np.abs(r1).max())), (rank, q)
        assert ids.tolist() == ids1.tolist(), rank
        assert pos == [105 + 6 + 4 * 1, 49 + 6 + 4 * 1, 12 + 6 + 4 * 1], (rank, pos)
    assert worst < 1e-3, worst


def test_batched_expert_parallel_refusals(cuda_engine, tools):
    """Host-side checks of the batch exchange entry points (one GPU)."""
    img = tools.synth_gguf(tools.TINY)
    e = cuda_engine.Engine.expert_parallel(img, 16, 0, 0, 2)
    b = cuda_engine.Batch(e, 2, 16)
    with pytest.raises(cuda_engine.QwenCudaError, match="not connected"):
        b.forward([0], [1])
    h, dev = b.ep_handle()
    assert len(h) == 64
    with pytest.raises(cuda_engine.QwenCudaError, match="different GPUs"):
        b.connect([(h, dev), (h, dev)])
    with pytest.raises(cuda_engine.QwenCudaError, match="not connected"):
        b.forward([0], [1])
    single = cuda_engine.Batch(cuda_engine.Engine(img, 16), 2, 16)
    with pytest.raises(cuda_engine.QwenCudaError, match="not an expert-parallel engine"):
        single.ep_handle()
    q8 = tools.synth_gguf(tools.TINY.with_(kind_gate_up=tools.Q8_0))
    with pytest.raises(cuda_engine.QwenCudaError, match="need the tensor-core MoE path"):
        cuda_engine.Batch(cuda_engine.Engine.expert_parallel(q8, 16, 0, 0, 2), 2, 16)


def test_batched_peer_gone_times_out_and_gpu_stays_usable():
    """A rank that stops between calls: the other rank's next call ends with the barrier timeout
    (2 s, once: later waits of the call give up at once), its batch then refuses calls, and the GPU
    still runs a fresh engine.  Host-side failure only; plain peer loads and flags, no NCCL."""
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    import _ep_worker
    out = _spawn(2, _ep_worker.run_batch_peer_gone, lambda r: (), go_after_sync=True)
    code, msg, seconds, after, fresh_ok = out[0]
    assert "did not reach the barrier" in msg, msg
    assert 1.5 < seconds < 30, seconds
    assert "create a new batch" in after, after
    assert fresh_ok
