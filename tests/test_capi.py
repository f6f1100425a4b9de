"""The C-ABI library loads, exports every declared symbol, and rejects bad
inputs before touching the GPU (no CUDA compute here)."""
import re
import struct

import pytest

from conftest import GOLDEN, ROOT


def _declared(header: str) -> set[str]:
    text = (ROOT / "include" / header).read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(q[ct]t?_[a-z0-9_]+)\s*\(", text))


def test_cuda_library_exports_every_declared_symbol(cuda_engine):
    names = _declared("qwen_cuda.h")
    assert len(names) >= 20
    L = cuda_engine.lib()
    for n in names:
        assert hasattr(L, n), n
    assert names == set(cuda_engine.EXPORTS)


def test_tools_library_exports_every_declared_symbol(tools):
    names = _declared("qwen_tools.h")
    L = tools.lib()
    for n in names:
        assert hasattr(L, n), n


def test_row_bytes_matches_reference(cuda_engine, oracle):
    """quant.rs:12-21 through the C ABI, including its errors (tests/core.rs:43-46)."""
    for kind, cols in [(0, 3), (1, 5), (2, 64), (8, 2048), (12, 2048), (13, 768), (14, 768), (14, 2048)]:
        assert cuda_engine.row_bytes(kind, cols) == oracle.row_bytes(kind, cols)
    with pytest.raises(cuda_engine.QwenCudaError, match="not divisible"):
        cuda_engine.row_bytes(12, 255)
    with pytest.raises(cuda_engine.QwenCudaError, match="not supported"):
        cuda_engine.row_bytes(99, 256)


def _create_err(cuda_engine, data: bytes, ctx: int = 4) -> str:
    with pytest.raises(cuda_engine.QwenCudaError) as ei:
        cuda_engine.Engine(data, ctx)
    assert ei.value.code == cuda_engine.ERR_INVALID
    return ei.value.msg


def test_malformed_headers_rejected_through_c_abi(cuda_engine):
    """tests/model.rs:71-97 against qc_engine_create_gguf (parsing precedes any device work)."""
    b = (GOLDEN / "tiny_f32.gguf").read_bytes()
    assert "failed to fill" in _create_err(cuda_engine, b[:10])
    assert "truncated tensor" in _create_err(cuda_engine, b[:-20])
    assert "not a GGUF" in _create_err(cuda_engine, b"NOPE" + b[4:])
    assert "version 999" in _create_err(cuda_engine, b[:4] + struct.pack("<I", 999) + b[8:])
    assert "exceeds limit" in _create_err(cuda_engine, b[:8] + struct.pack("<Q", 2**64 - 1) + b[16:])


def test_context_and_config_validation_through_c_abi(cuda_engine):
    """model.rs:176-180: context must be in 1..=max_context (32 in the fixture)."""
    b = (GOLDEN / "tiny_f32.gguf").read_bytes()
    assert "context must be in 1..=32" in _create_err(cuda_engine, b, 0)
    assert "context must be in 1..=32" in _create_err(cuda_engine, b, 33)
    # architecture check (model.rs:22-28): patch the arch string in place
    bad = b.replace(b"qwen3moe", b"qwen3mox", 1)
    assert "only qwen3moe" in _create_err(cuda_engine, bad)
