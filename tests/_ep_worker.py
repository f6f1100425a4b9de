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
