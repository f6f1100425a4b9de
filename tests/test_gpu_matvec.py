"""Dequant and dequant-fused matvec on the GPU against the CPU oracle (BASELINE config 2 shapes).

Tolerances: dequantized values bit-exact with quant.rs;
matvec outputs within rel 1e-4 of the reference's sequential fp32 fold,
measured as max|y - y_ref| <= 1e-4 * max|y_ref| over the output vector and,
per element, |y_i - y_ref_i| <= 1e-4 * |y_ref_i| + 1e-6 * max|y_ref|.
"""
import zlib

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu

KINDS = (0, 1, 2, 8, 12, 13, 14)
Q4_K, Q5_K, Q6_K, Q8_0, F16 = 12, 13, 14, 8, 1

# (name, cols, rows, kind): the Qwen3-30B-A3B matvec shapes of BASELINE config 2.
SHAPES = [
    ("q_proj", 2048, 4096, Q4_K), ("kv_proj", 2048, 512, Q4_K), ("o_proj", 4096, 2048, Q4_K),
    ("gate_up", 2048, 768, Q4_K), ("gate_up_q5", 2048, 768, Q5_K), ("down", 768, 2048, Q6_K),
    ("router", 2048, 128, F16), ("vocab", 2048, 151936, Q6_K),
]
SHAPES_Q8 = [(n + "_q8", c, r, Q8_0) for n, c, r, _ in SHAPES]


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def test_dequant_golden_blocks_bit_exact(cuda_engine, torch_cuda):
    """tests/core.rs:50-151 fixtures through the device layout and k_dequant."""
    torch = torch_cuda
    z = np.load(GOLDEN / "quant_blocks.npz")
    for kind in KINDS:
        b, expected = z[f"bytes_{kind}"], z[f"expected_{kind}"]
        m = cuda_engine.Matrix(kind, 1, expected.size, b)
        out = torch.empty(expected.size, dtype=torch.float32, device="cuda")
        m.dequant(out.data_ptr())
        torch.cuda.synchronize()
        assert np.array_equal(_bits(out.cpu().numpy()), _bits(expected)), f"kind={kind}"


@pytest.mark.parametrize("kind", KINDS)
def test_dequant_random_bit_exact(cuda_engine, oracle, tools, torch_cuda, kind):
    torch = torch_cuda
    rows, cols, experts = 37, 768, 3
    blocks = tools.random_matrix(kind, rows * experts, cols, seed=11, stream=kind, std=0.02)
    m = cuda_engine.Matrix(kind, rows, cols, blocks, experts=experts)
    rb = tools.row_bytes(kind, cols)
    for e in (0, 2):
        ref = oracle.decode_rows(blocks[e * rows * rb:(e + 1) * rows * rb], kind, rows, cols)
        out = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
        m.dequant(out.data_ptr(), expert=e)
        torch.cuda.synchronize()
        assert np.array_equal(_bits(out.cpu().numpy()), _bits(ref.ravel())), (kind, e)


def _check_rel(y, ref, what):
    scale = float(np.abs(ref).max())
    err = np.abs(y - ref)
    assert err.max() <= 1e-4 * scale, f"{what}: vector rel {err.max() / scale:.3e}"
    bad = err > 1e-4 * np.abs(ref) + 1e-6 * scale
    assert not bad.any(), f"{what}: {bad.sum()} elements beyond rel 1e-4 (worst {err[bad].max():.3e})"


@pytest.mark.parametrize("name,cols,rows,kind", SHAPES + SHAPES_Q8)
def test_matvec_matches_oracle(cuda_engine, oracle, tools, torch_cuda, name, cols, rows, kind):
    torch = torch_cuda
    blocks = tools.random_matrix(kind, rows, cols, seed=2, stream=zlib.crc32(name.encode()), std=0.02)
    x = tools.normal(2, 999, cols)  # x ~ N(0, 1)
    ref = oracle.matvec(blocks, kind, rows, cols, x, fast=rows > 100000)  # (identical results, faster)
    m = cuda_engine.Matrix(kind, rows, cols, blocks)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty(rows, dtype=torch.float32, device="cuda")
    m.matvec(xd.data_ptr(), yd.data_ptr())
    torch.cuda.synchronize()
    _check_rel(yd.cpu().numpy(), ref, name)


def test_matvec_experts_and_odd_shapes(cuda_engine, oracle, tools, torch_cuda):
    torch = torch_cuda
    for kind, rows, cols, experts in [(Q6_K, 2048, 768, 3), (Q4_K, 300, 256, 2), (0, 33, 7, 1), (1, 5, 40, 2),
                                      (2, 65, 96, 2), (Q8_0, 1, 32, 1), (Q5_K, 3, 512, 4)]:
        blocks = tools.random_matrix(kind, rows * experts, cols, seed=5, stream=kind + rows, std=0.02)
        m = cuda_engine.Matrix(kind, rows, cols, blocks, experts=experts)
        x = tools.normal(5, 7, cols)
        xd = torch.from_numpy(x).cuda()
        rb = tools.row_bytes(kind, cols)
        for e in range(experts):
            ref = oracle.matvec(blocks[e * rows * rb:(e + 1) * rows * rb], kind, rows, cols, x)
            yd = torch.empty(rows, dtype=torch.float32, device="cuda")
            m.matvec(xd.data_ptr(), yd.data_ptr(), expert=e)
            torch.cuda.synchronize()
            _check_rel(yd.cpu().numpy(), ref, f"kind={kind} rows={rows} cols={cols} e={e}")


def test_packed_matvec_golden_blocks(cuda_engine):
    """tests/core.rs:152-185: three copies of the golden blocks, tol 0.002 + 5e-5|y|, twice."""
    z = np.load(GOLDEN / "quant_blocks.npz")
    for kind in KINDS:
        b, decoded = z[f"bytes_{kind}"], z[f"expected_{kind}"]
        cols = decoded.size
        x = ((np.arange(cols) % 13).astype(np.float32) - 6.0) / 7.0
        expected = float(np.dot(x.astype(np.float64), decoded.astype(np.float64)))
        data = np.concatenate([b, b, b])
        for _ in range(2):
            y = cuda_engine.packed_matvec(kind, 3, cols, data, x)
            assert np.all(np.abs(y - expected) < 0.002 + abs(expected) * 5e-5), (kind, y, expected)


def test_large_grid(cuda_engine):
    """tests/core.rs:186-206: 70,001 rows of F32 [s, 2s] times [1.5, -0.5]."""
    rows = 70001
    x = np.array([1.5, -0.5], dtype=np.float32)
    for s in (1.0, 2.0, 3.0):
        data = np.tile(np.array([s, 2 * s], dtype=np.float32), rows).view(np.uint8)
        y = cuda_engine.packed_matvec(0, rows, 2, data, x)
        assert y.size == rows and np.all(np.abs(y - s * 0.5) < 1e-5)


def test_packed_matvec_rejects_bad_shapes(cuda_engine):
    with pytest.raises(cuda_engine.QwenCudaError, match="shape mismatch"):
        cuda_engine.packed_matvec(12, 2, 256, np.zeros(144, dtype=np.uint8), np.zeros(256, dtype=np.float32))
