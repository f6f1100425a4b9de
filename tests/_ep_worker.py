"""Child process of the expert-parallel GPU tests: one rank on one GPU.

Handles travel through multiprocessing queues (the parent gathers every
rank's handle and sends the full list back), so the test needs neither
torch.distributed nor NCCL."""
import traceback


def run(rank: int, world: int, up, down, tokens, prompt_len: int, n_greedy: int) -> None:
    try:
        from conftest import load_package  # noqa: F401  (package on sys.path)
        from qwen30brust_b200 import engine as E, tools as T

        img = T.synth_gguf(T.TINY)
        eng = E.Engine.expert_parallel(img, 64, rank, rank, world)
        up.put(("handle", rank, eng.ep_handle()))
        eng.connect(down.get(timeout=120))
        logits = [eng.forward(int(t)) for t in tokens]
        eng.reset()
        eng.forward_tokens(tokens[:prompt_len], want_logits=False)
        toks, _ = eng.decode_greedy(n_greedy)
        up.put(("done", rank, (logits, toks.tolist(), eng.position)))
        eng.close()
    except Exception:  # reported to the parent, which fails the test
        up.put(("error", rank, traceback.format_exc()))


def run_peer_gone(rank: int, world: int, up, down, tokens) -> None:
    """Failure detection without a GPU fault: both ranks decode len(tokens) tokens in lockstep,
    then rank 1 stops calling forward (it has nothing in flight) and rank 0 runs one more token.
    Rank 0's kernel waits for rank 1's partial MoE vectors, which never come: its bounded waits end
    with the engine's timeout error, and the GPU stays usable (a fresh engine runs a token)."""
    import time
    try:
        from conftest import load_package  # noqa: F401  (package on sys.path)
        from qwen30brust_b200 import engine as E, tools as T

        img = T.synth_gguf(T.TINY)
        eng = E.Engine.expert_parallel(img, 64, rank, rank, world)
        up.put(("handle", rank, eng.ep_handle()))
        eng.connect(down.get(timeout=120))
        for t in tokens:
            eng.forward(int(t))
        up.put(("synced", rank, None))
        result = None
        if rank == 0:
            down.get(timeout=120)  # the other ranks are idle now
            t0 = time.time()
            try:
                eng.forward(int(tokens[0]))
                result = ("no error", time.time() - t0)
            except E.QwenCudaError as x:
                result = (x.code, x.msg, time.time() - t0, eng.position)
            fresh = E.Engine(img, 16)
            ok = fresh.forward(1)
            result = result + (bool(ok.size == T.TINY.vocab),)
            fresh.close()
        else:
            down.get(timeout=120)  # stay idle until rank 0 is done
        up.put(("done", rank, result))
        eng.close()
    except Exception:
        up.put(("error", rank, traceback.format_exc()))


def run_batch(rank: int, world: int, up, down, calls, params, steps: int) -> None:
    """Batched expert parallelism: this rank's 3 sequences on an expert-parallel engine's batch
    (its calls: (seq ids, tokens) with the same token counts on every rank), then the device decode
    loop with `params` samplers; the same calls on a one-GPU batch of the same GPU for comparison."""
    try:
        from conftest import load_package  # noqa: F401  (package on sys.path)
        from qwen30brust_b200 import engine as E, tools as T

        img = T.synth_gguf(T.TINY)
        eng = E.Engine.expert_parallel(img, 256, rank, rank, world)
        b = E.Batch(eng, 3, 256)
        up.put(("handle", rank, b.ep_handle()))
        b.connect(down.get(timeout=120))
        rows = [b.forward(s, t) for s, t in calls]
        ids = b.decode_sample([E.Sampler(*p, device=rank) for p in params], [0, 1, 2], steps)
        pos = [b.position(q) for q in range(3)]
        one = E.Engine(img, 256, rank)
        b1 = E.Batch(one, 3, 256)
        rows1 = [b1.forward(s, t) for s, t in calls]
        ids1 = b1.decode_sample([E.Sampler(*p, device=rank) for p in params], [0, 1, 2], steps)
        up.put(("done", rank, (rows, ids, pos, rows1, ids1)))
        b1.close()
        one.close()
        b.close()
        eng.close()
    except Exception:
        up.put(("error", rank, traceback.format_exc()))


def run_batch_peer_gone(rank: int, world: int, up, down) -> None:
    """As run_peer_gone for a batch of an expert-parallel engine: both ranks run two steps in
    lockstep, then rank 1 stops and rank 0 runs one more; rank 0's call ends with the barrier
    timeout, its batch refuses further calls, and the GPU still runs a fresh engine."""
    import time
    try:
        from conftest import load_package  # noqa: F401  (package on sys.path)
        from qwen30brust_b200 import engine as E, tools as T

        img = T.synth_gguf(T.TINY)
        eng = E.Engine.expert_parallel(img, 64, rank, rank, world)
        b = E.Batch(eng, 2, 64)
        up.put(("handle", rank, b.ep_handle()))
        b.connect(down.get(timeout=120))
        for t in ([3, 1], [4, 1]):
            b.forward([0, 1], t)
        up.put(("synced", rank, None))
        result = None
        if rank == 0:
            down.get(timeout=120)  # the other rank is idle now
            t0 = time.time()
            try:
                b.forward([0, 1], [5, 9])
                result = ("no error", time.time() - t0)
            except E.QwenCudaError as x:
                result = (x.code, x.msg, time.time() - t0)
            try:
                b.forward([0, 1], [2, 6])
                result = result + ("accepted",)
            except E.QwenCudaError as x:
                result = result + (x.msg,)
            fresh = E.Engine(img, 16)
            ok = fresh.forward(1)
            result = result + (bool(ok.size == T.TINY.vocab),)
            fresh.close()
        else:
            down.get(timeout=120)  # stay idle until rank 0 is done
        up.put(("done", rank, result))
        b.close()
        eng.close()
    except Exception:
        up.put(("error", rank, traceback.format_exc()))
