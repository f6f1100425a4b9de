"""Several sequences per step (qc_batch_*, BASELINE config 5) against the CPU oracle.

Each sequence of a batch must give, token for token, the logits Model::forward gives on that
sequence alone (model.rs:210-216), whatever else shares the step: prompt chunks and decode tokens
of other sequences, in any order.  Tolerances as for the single-sequence decode path: max-abs
2e-2 with top-1 agreement (north star); the gap is fp32 reassociation only in practice.  The MoE
half runs on the tcgen05 tensor-core path here (Q4_K gate/up, Q6_K down), the sampler on one block
per sequence."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _close(got, want, what):
    err = float(np.abs(got - want).max())
    assert err < 2e-2, (what, err)
    assert int(np.argmax(got)) == int(np.argmax(want)), what
    return err


def test_batch_mixed_prefill_and_decode_match_oracle(cuda_engine, oracle, tools):
    spec = tools.TINY
    img = tools.synth_gguf(spec)
    eng = cuda_engine.Engine(img, 128)
    b = cuda_engine.Batch(eng, 6, 128)
    refs = [oracle.Model(img, 128) for _ in range(6)]
    rng = np.random.default_rng(21)
    lens = [5, 1, 9, 3, 12, 7]
    prompts = [rng.integers(0, spec.vocab, n).tolist() for n in lens]
    worst = 0.0

    def ref_last(q, toks):
        out = None
        for t in toks:
            out = refs[q].forward(t)
        return out

    # call 1: whole prompts of sequences 0, 2, 4 back to back (rows in order of each one's last token)
    seqs = [0] * 5 + [2] * 9 + [4] * 12
    toks = prompts[0] + prompts[2] + prompts[4]
    rows = b.forward(seqs, toks)
    assert rows.shape == (3, spec.vocab)
    for r, q in zip(rows, (0, 2, 4)):
        worst = max(worst, _close(r, ref_last(q, prompts[q]), f"prompt of {q}"))
    # call 2: prompts of 1, 3, 5 interleaved token by token
    order, k = [], [0, 0, 0]
    while any(k[i] < lens[q] for i, q in enumerate((1, 3, 5))):
        for i, q in enumerate((1, 3, 5)):
            if k[i] < lens[q]:
                order.append((q, prompts[q][k[i]]))
                k[i] += 1
    rows = b.forward([q for q, _ in order], [t for _, t in order])
    last_order = list(dict.fromkeys(reversed([q for q, _ in order])))[::-1]
    for r, q in zip(rows, last_order):
        worst = max(worst, _close(r, ref_last(q, prompts[q]), f"interleaved prompt of {q}"))
    assert [b.position(q) for q in range(6)] == lens
    # decode steps: one token for every sequence, in a shuffled order each step
    for step in range(8):
        perm = rng.permutation(6).tolist()
        toks = rng.integers(0, spec.vocab, 6).tolist()
        rows = b.forward(perm, toks)
        for r, q, t in zip(rows, perm, toks):
            worst = max(worst, _close(r, refs[q].forward(t), f"step {step} seq {q}"))
    assert worst < 1e-3, worst
    # reset one sequence and start it again; the others are untouched
    b.reset(3)
    refs[3].reset()
    assert b.position(3) == 0 and b.position(4) == lens[4] + 8
    fresh = rng.integers(0, spec.vocab, 4).tolist()
    _close(b.forward([3] * 4, fresh)[0], ref_last(3, fresh), "after reset")
    _close(b.forward([4], [11])[0], refs[4].forward(11), "untouched sequence")
    # argument errors change nothing
    with pytest.raises(cuda_engine.QwenCudaError) as ei:
        b.forward([0], [spec.vocab])
    assert ei.value.code == cuda_engine.ERR_TOKEN
    with pytest.raises(cuda_engine.QwenCudaError) as ei:
        b.forward([1] * 200, [1] * 200)
    assert ei.value.code == cuda_engine.ERR_CONTEXT
    with pytest.raises(cuda_engine.QwenCudaError, match="sequence index"):
        b.forward([6], [1])
    assert b.position(1) == lens[1] + 8
    # the engine's own single-sequence state is separate
    assert eng.position == 0
    e0 = eng.forward(prompts[0][0])
    _close(e0, oracle.Model(img, 128).forward(prompts[0][0]), "engine beside a batch")
    b.close()
    eng.close()


def test_batch_30b_shapes_long_prompt_chunks(cuda_engine, oracle, tools):
    """The 30B-A3B shapes (32q/4kv x 128, 128 experts top-8, vocab 151,936) with 2 layers: 4
    sequences, prompts fed in chunks that cross the pass size (128 tokens), then decode steps."""
    spec = tools.QWEN3_30B_A3B.with_(layers=2)
    img = tools.synth_gguf(spec)
    eng = cuda_engine.Engine(img, 1024)
    b = cuda_engine.Batch(eng, 4, 1024)
    refs = [oracle.Model(img, 1024, fast=True) for _ in range(4)]
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, spec.vocab, n).tolist() for n in (300, 40, 129, 7)]
    # one call with the first 200 tokens of sequence 0 and all of 1 and 3; then the rest of 0 and 2
    seqs = [0] * 200 + [1] * 40 + [3] * 7
    rows = b.forward(seqs, prompts[0][:200] + prompts[1] + prompts[3])
    for q, toks in ((0, prompts[0][:200]), (1, prompts[1]), (3, prompts[3])):
        refs[q].prefill(toks[:-1])
    want = {q: refs[q].forward(prompts[q][-1] if q != 0 else prompts[0][199]) for q in (0, 1, 3)}
    for r, q in zip(rows, (0, 1, 3)):
        _close(r, want[q], f"chunk of {q}")
    rows = b.forward([2] * 129 + [0] * 100, prompts[2] + prompts[0][200:])
    refs[2].prefill(prompts[2][:-1])
    refs[0].prefill(prompts[0][200:-1])
    _close(rows[0], refs[2].forward(prompts[2][-1]), "prompt of 2")
    _close(rows[1], refs[0].forward(prompts[0][-1]), "rest of 0")
    for step in range(3):
        toks = rng.integers(0, spec.vocab, 4).tolist()
        rows = b.forward([0, 1, 2, 3], toks)
        for q in range(4):
            _close(rows[q], refs[q].forward(toks[q]), f"step {step} seq {q}")
    b.close()
    eng.close()


def test_batch_sampling_matches_oracle_samplers(cuda_engine, oracle, tools):
    """qc_batch_sample draws every sequence in one launch with its own sampler; qc_batch_decode_sample
    runs the chat loop for all of them on the device and gives the ids of a host-driven loop."""
    spec = tools.TINY.with_(vocab=20000)  # a vocabulary above the shared-memory set size too
    img = tools.synth_gguf(spec)
    eng = cuda_engine.Engine(img, 64)
    params = [(3, 0.7, 20, 0.9), (4, 1.0, 0, 1.0), (5, 0.0, 0, 1.0), (6, 0.8, 0, 0.95)]
    rng = np.random.default_rng(9)
    prompts = [rng.integers(0, spec.vocab, n).tolist() for n in (6, 3, 8, 5)]
    # a host-driven loop: forward all, sample all (batch), compare each draw with the oracle sampler
    b = cuda_engine.Batch(eng, 4, 64)
    seqs = [q for q in range(4) for _ in prompts[q]]
    rows = b.forward(seqs, sum(prompts, []))
    dev = [cuda_engine.Sampler(*p) for p in params]
    ora = [oracle.Sampler(*p) for p in params]
    manual = []
    for step in range(12):
        ids = b.sample(dev, [0, 1, 2, 3])
        for q in range(4):
            assert ids[q] == ora[q].sample(rows[q]), (step, q)
        manual.append(ids.tolist())
        rows = b.forward([0, 1, 2, 3], ids)
    # the same loop on the device, from the same prompts and seeds
    b2 = cuda_engine.Batch(eng, 4, 64)
    b2.forward(seqs, sum(prompts, []), want_logits=False)
    got = b2.decode_sample([cuda_engine.Sampler(*p) for p in params], [0, 1, 2, 3], 12)
    assert got.tolist() == manual
    assert [b2.position(q) for q in range(4)] == [len(p) + 12 for p in prompts]
    with pytest.raises(cuda_engine.QwenCudaError, match="distinct"):
        b2.decode_sample([dev[0], dev[1]], [0, 0], 1)
    b.close()
    b2.close()
    eng.close()


def test_batch_format_mix_matches_oracle(cuda_engine, oracle, tools):
    """Q6_K attention rows and a Q4_K output matrix on the tensor cores, a Q8_0 O projection on the
    CUDA-core batched matvec beside them, Q4_K expert down rows: per-sequence logits as the oracle's."""
    spec = tools.TINY.with_(kind_attn=tools.Q6_K, kind_attn_out=tools.Q8_0, kind_output=tools.Q4_K,
                            kind_down=tools.Q4_K)
    img = tools.synth_gguf(spec)
    eng = cuda_engine.Engine(img, 64)
    b = cuda_engine.Batch(eng, 3, 64)
    refs = [oracle.Model(img, 64) for _ in range(3)]
    rng = np.random.default_rng(13)
    prompts = [rng.integers(0, spec.vocab, n).tolist() for n in (9, 4, 30)]
    rows = b.forward([q for q in range(3) for _ in prompts[q]], sum(prompts, []))
    for q in range(3):
        want = None
        for t in prompts[q]:
            want = refs[q].forward(t)
        _close(rows[q], want, f"prompt of {q}")
    for step in range(4):
        toks = rng.integers(0, spec.vocab, 3).tolist()
        rows = b.forward([2, 0, 1], [toks[2], toks[0], toks[1]])
        for r, q in zip(rows, (2, 0, 1)):
            _close(r, refs[q].forward(toks[q]), f"step {step} seq {q}")
    b.close()
    eng.close()
