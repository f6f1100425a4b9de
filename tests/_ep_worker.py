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
