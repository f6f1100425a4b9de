"""The MoE half of a layer for a batch of tokens (qc_moe_layer) against the
oracle's per-token restatement of model.rs:245-287.

Path 1 runs the per-token decode kernels once per token; path 2 groups the tokens per expert and
runs gate/up and down as tcgen05 tensor-core GEMMs: the K-quant integers as exact fp16 operands,
one accumulator per 256-column super-block scaled by its d in the epilogue, activations as fp16
hi + lo.  Both must match the oracle's MoE output (out - x) within 5e-4 of its largest element
(two chained matvecs at the north star's 1e-4 each, plus SwiGLU), and each other."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _f32_tensor(tools, img, name):
    v, kind, dims = tools.tensor_view(img, name)
    assert kind == tools.F32
    return np.frombuffer(v.tobytes(), dtype=np.float32)


def _oracle_moe(oracle, tools, img, spec, layer, x):
    H, I, E, top = spec.hidden, spec.intermediate, spec.experts, spec.top
    b = f"blk.{layer}."
    norm = _f32_tensor(tools, img, b + "ffn_norm.weight")
    router, rk, _ = tools.tensor_view(img, b + "ffn_gate_inp.weight")
    stacks = {}
    for n in ("gate", "up", "down"):
        v, k, dims = tools.tensor_view(img, b + f"ffn_{n}_exps.weight")
        per = tools.row_bytes(k, dims[0]) * dims[1]
        stacks[n] = (v, k, per)
    out = np.empty_like(x)
    for t in range(x.shape[0]):
        h = oracle.rms(x[t], norm, spec.eps)
        logits = oracle.matvec(router, rk, E, H, h)
        moe = np.zeros(H, dtype=np.float32)
        for e, w in oracle.route(logits, top):
            def mv(n, rows, cols, vec):
                v, k, per = stacks[n]
                return oracle.matvec(v[e * per:(e + 1) * per], k, rows, cols, vec)
            g, u = mv("gate", I, H, h), mv("up", I, H, h)
            act = (g / (np.float32(1.0) + np.exp(-g))) * u
            moe = moe + np.float32(w) * mv("down", H, I, act.astype(np.float32))
        out[t] = x[t] + moe
    return out


def _check(got, ref, x, tol=5e-4):
    d_ref, d_got = ref - x, got - x
    scale = float(np.abs(d_ref).max())
    err = float(np.abs(d_got - d_ref).max())
    assert err <= tol * scale, (err, scale)
    return err / scale


SPECS = {
    "tiny": lambda tools: (tools.TINY, 0.0),
    "30b_layer": lambda tools: (tools.QWEN3_30B_A3B.with_(layers=1, vocab=512), 1.1),
    # the other formats Q4_K_M files give expert matrices: Q4_K down (the SwiGLU epilogue then writes
    # the down GEMM's min chunks), Q6_K gate/up (pair tiles of Q6_K rows)
    "tiny_q4k_down": lambda tools: (tools.TINY.with_(kind_down=tools.Q4_K), 0.0),
    "tiny_q6k_gate_up": lambda tools: (tools.TINY.with_(kind_gate_up=tools.Q6_K), 0.0),
    "30b_q4k_down": lambda tools: (tools.QWEN3_30B_A3B.with_(layers=1, vocab=512, kind_down=tools.Q4_K), 1.1),
}


@pytest.mark.parametrize("which,tokens", [("tiny", [1, 5, 40]), ("30b_layer", [1, 8, 32, 130]),
                                          ("tiny_q4k_down", [3, 33]), ("tiny_q6k_gate_up", [3, 33]),
                                          ("30b_q4k_down", [40])])
def test_moe_layer_paths_match_oracle(cuda_engine, oracle, tools, which, tokens):
    spec, skew = SPECS[which](tools)
    img = tools.synth_gguf(spec)
    if skew:
        tools.skew_router(img, 0, skew)
    e = cuda_engine.Engine(img, 16)
    rng = np.random.default_rng(3)
    worst = {1: 0.0, 2: 0.0}
    for T in tokens:
        x = rng.normal(size=(T, spec.hidden)).astype(np.float32)
        ref = _oracle_moe(oracle, tools, img, spec, 0, x)
        outs = {}
        for path in (1, 2):
            outs[path], ms = e.moe_layer(0, x, path)
            assert ms > 0
            worst[path] = max(worst[path], _check(outs[path], ref, x))
        _check(outs[2], outs[1], x)
    assert e.position == 0  # the KV cache and position are not touched
    print(which, "worst relative error per path:", worst)


def test_moe_layer_refusals(cuda_engine, tools):
    img = tools.synth_gguf(tools.TINY)
    e = cuda_engine.Engine(img, 16)
    x = np.zeros((2, tools.TINY.hidden), dtype=np.float32)
    with pytest.raises(cuda_engine.QwenCudaError, match="layer index"):
        e.moe_layer(5, x, 2)
    with pytest.raises(cuda_engine.QwenCudaError, match="path"):
        e.moe_layer(0, x, 3)
    q8 = tools.synth_gguf(tools.TINY.with_(kind_gate_up=tools.Q8_0))
    with pytest.raises(cuda_engine.QwenCudaError, match="takes Q4_K and Q6_K rows"):
        cuda_engine.Engine(q8, 16).moe_layer(0, x, 2)
    out, _ = cuda_engine.Engine(q8, 16).moe_layer(0, x, 1)  # the per-token kernels take any format
    assert out.shape == x.shape
