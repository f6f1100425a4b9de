"""Quantizers and the synthetic GGUF writer, checked with the oracle's decoder (no GPU)."""
import numpy as np
import pytest

KINDS = (0, 1, 2, 8, 12, 13, 14)


@pytest.mark.parametrize("kind", KINDS)
def test_quantize_roundtrip_error_is_bounded(oracle, tools, kind):
    x = tools.normal(7, 1234 + kind, 4096, std=0.02)
    q = tools.quantize(kind, x)
    assert q.size == tools.row_bytes(kind, 4096)
    y = oracle.decode(q, kind, 4096)
    err = np.abs(y - x)
    # step size of the format relative to the sub-block range; loose, format-aware bounds
    bound = {0: 0.0, 1: 6e-5, 2: 0.01, 8: 0.0005, 12: 0.006, 13: 0.003, 14: 0.002}[kind]
    assert err.max() <= bound + 1e-9, (kind, err.max())
    if kind in (12, 13, 14):
        assert np.corrcoef(x, y)[0, 1] > 0.99


def test_quantizers_exercise_every_field(tools, oracle):
    """Random blocks must use high scale bits, Q5_K fifth bits and both Q6_K scale signs."""
    x = tools.normal(3, 99, 256 * 64, std=0.02)
    q5 = tools.quantize(13, x).reshape(-1, 176)
    assert q5[:, 16:48].any(), "Q5_K qh bits never set"
    q4 = tools.quantize(12, x).reshape(-1, 144)
    assert (q4[:, 4:12] >> 6).any(), "Q4_K high scale bits never set"


def test_normal_stream_is_reproducible_and_seeded(tools):
    a = tools.normal(0, 5, 1000)
    b = tools.normal(0, 5, 1000)
    c = tools.normal(1, 5, 1000)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    assert abs(a.mean()) < 0.15 and abs(a.std() - 1) < 0.1
    tail = tools.normal(0, 5, 10, first=990)
    assert np.array_equal(tail, a[990:])


def test_random_matrix_matches_row_quantization(tools):
    kind, rows, cols = 12, 5, 512
    m = tools.random_matrix(kind, rows, cols, seed=4, stream=77, std=0.02, threads=3)
    x = tools.normal(4, 77, rows * cols, std=0.02)
    assert np.array_equal(m, tools.quantize(kind, x))


def test_synth_gguf_is_accepted_by_the_reference_parser(oracle, tools):
    img = tools.synth_gguf(tools.TINY)
    oracle.gguf_check(img.tobytes())
    m = oracle.Model(img, 32)
    c = m.config
    for k in ("hidden", "layers", "heads", "kvheads", "head_dim", "experts", "top", "intermediate", "vocab"):
        assert c[k] == getattr(tools.TINY, k)
    assert c["theta"] == 1e6


def test_synth_size_30b_matches_survey_arithmetic(tools):
    """The 30B-shape image: Q4_K attention/gate/up, Q6_K down/output, F16 router, Q8_0 embeddings."""
    n = tools.synth_size(tools.QWEN3_30B_A3B)
    per_layer = (4096 * 1152 + 2 * 512 * 1152 + 2048 * 2304 + 128 * 4096 + 2 * 128 * 768 * 1152
                 + 128 * 2048 * 630 + 2 * 2048 * 4 + 2 * 128 * 4)
    expected = 48 * per_layer + 151936 * 2176 + 151936 * 1680 + 2048 * 4
    assert expected < n < expected + 64 * 1024
