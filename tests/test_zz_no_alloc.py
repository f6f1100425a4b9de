"""qc_packed_matvec_noalloc, the allocation-free packed matvec.

It serves callers that may not allocate device memory (a host whose own
allocator has reserved the GPU's memory, or code that must not call cudaFree,
which may synchronize the device).  Its working memory is one static
__device__ array per GPU shared by every call, so these tests check that two
calls in a row — with different shapes before them, leaving other contents in
the array — agree with the CPU oracle (the reference's Cpu::matvec) and with
qc_packed_matvec within the matvec tolerance, that only the first call on a
device reserves memory (the array, when CUDA loads the code holding it) and no
later call allocates, and that oversized matrices are refused.  The file is
named to run last.
"""
import subprocess
import sys
import textwrap

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

# (kind, rows, cols): formats with padding (Q8_0/Q4_0 odd block counts, F16/F32 odd
# widths, row counts not a multiple of 8) after wider ones, so stale contents would show.
CASES = [(1, 96, 1000), (12, 300, 512), (14, 64, 768), (8, 33, 96), (2, 65, 96), (1, 5, 40), (0, 70, 7),
         (13, 17, 256)]


def _check_rel(y, ref, what):
    scale = float(np.abs(ref).max())
    err = np.abs(y - ref)
    assert err.max() <= 1e-4 * scale, f"{what}: vector rel {err.max() / scale:.3e}"
    assert not (err > 1e-4 * np.abs(ref) + 1e-6 * scale).any(), what


def test_noalloc_matches_oracle_and_packed_matvec_on_two_calls(cuda_engine, tools, oracle):
    for kind, rows, cols in CASES:
        blocks = tools.random_matrix(kind, rows, cols, seed=9, stream=kind * 1000 + rows, std=0.02)
        for call in range(2):
            x = tools.normal(9, 17 + call, cols)
            want = oracle.matvec(blocks, kind, rows, cols, x)
            ref = cuda_engine.packed_matvec(kind, rows, cols, blocks, x)
            got = cuda_engine.packed_matvec_noalloc(kind, rows, cols, blocks, x)
            what = f"kind={kind} rows={rows} cols={cols} call={call}"
            _check_rel(got, want, what + " vs oracle")
            _check_rel(got, ref, what + " vs qc_packed_matvec")


# Run in a fresh process, so the call below is the first one on the device whether this file runs
# alone or after every other test: free device memory before the first call (after the allocating
# matvec has loaded the shared kernels), after it, and after four more calls.
_MEMORY_PROBE = textwrap.dedent("""
    import sys
    sys.path.insert(0, {root!r})
    from __graft_entry__ import load_package
    load_package()
    import torch
    from qwen30brust_b200 import engine as E, tools as T
    torch.cuda.init()
    kind, rows, cols = 12, 256, 2048
    blocks = T.random_matrix(kind, rows, cols, seed=3, stream=5, std=0.02)
    x = T.normal(3, 6, cols)
    E.packed_matvec(kind, rows, cols, blocks, x)
    torch.cuda.synchronize()
    free = [torch.cuda.mem_get_info()[0]]
    E.packed_matvec_noalloc(kind, rows, cols, blocks, x)
    torch.cuda.synchronize()
    free.append(torch.cuda.mem_get_info()[0])
    for _ in range(4):
        E.packed_matvec_noalloc(kind, rows, cols, blocks, x)
    torch.cuda.synchronize()
    free.append(torch.cuda.mem_get_info()[0])
    print("FREE", *free)
""")


def test_noalloc_reserves_once_then_allocates_nothing(cuda_engine, torch_cuda):
    r = subprocess.run([sys.executable, "-c", _MEMORY_PROBE.format(root=str(ROOT))], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    line = next(ln for ln in r.stdout.splitlines() if ln.startswith("FREE"))
    before, first, after = (int(v) for v in line.split()[1:])
    array = 32 << 20
    assert 0 <= before - first <= array + (4 << 20), (before, first)  # the array (and its code), once
    assert after == first  # later calls allocate nothing


def test_noalloc_refuses_matrices_beyond_its_scratch(cuda_engine):
    rows, cols = 16384, 2048  # F16: 64 MiB of raw blocks alone
    blocks = np.zeros(rows * cols * 2, dtype=np.uint8)
    with pytest.raises(cuda_engine.QwenCudaError, match="at most"):
        cuda_engine.packed_matvec_noalloc(1, rows, cols, blocks, np.zeros(cols, dtype=np.float32))
    with pytest.raises(cuda_engine.QwenCudaError, match="shape mismatch"):
        cuda_engine.packed_matvec_noalloc(12, 2, 256, np.zeros(144, dtype=np.uint8), np.zeros(256, dtype=np.float32))
