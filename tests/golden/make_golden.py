#!/usr/bin/env python3
"""Regenerate the golden fixtures under tests/golden/ (run in the build container).

Sources, all from the reference project (K410Sh4/QWEN-30BRust):

* quant_blocks.npz — the two-block dequant fixtures of tests/core.rs:50-143:
  bytes ``(j*73 + block*29 + 19) % 256`` with d=0.125, dmin=0.0625 and the
  expected values from the test's own block-wise equations (restated here in
  NumPy, independently of any decoder).
* tiny_f32.gguf, tiny_f32_logits.json — tools/reference_fixture.py create()
  and reference() (the NumPy oracle), byte-identical to tests/data/ in the
  reference, plus the CPU parity errors it recorded (validation/parity-cpu.json).
* tiny_q_golden.npz: the quantized 2-layer hidden-256 model
  written by libqwen_tools (seed 0), its prompt (16 ids U[0,512) from seed 1),
  and 32 greedy steps, with logits at every position computed by the
  reference's NumPy forward (tools/reference_fixture.py:80-110) on the
  dequantized weights.  Dequantization uses the oracle, which quant_blocks.npz
  pins bit-exactly.

Usage: python tests/golden/make_golden.py --reference <path of the reference checkout>
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
REF = Path(".")  # the reference checkout, set from --reference by main()


def f16_bytes(v: float) -> bytes:
    return np.array([v], dtype=np.float16).tobytes()


def core_fixture(kind: int):
    """tests/core.rs:50-143 — two blocks per format and their expected values."""
    n, size = {0: (1, 4), 1: (1, 2), 2: (32, 18), 8: (32, 34), 12: (256, 144), 13: (256, 176),
               14: (256, 210)}[kind]
    b = bytearray(size * 2)
    expected: list[float] = []
    for block in range(2):
        p = block * size
        for j in range(size):
            b[p + j] = (j * 73 + block * 29 + 19) % 256
        if kind == 0:
            f = 0.75 if block == 0 else -1.25
            b[p:p + 4] = np.array([f], dtype=np.float32).tobytes()
            expected.append(f)
        elif kind == 1:
            f = 0.75 if block == 0 else -1.25
            b[p:p + 2] = f16_bytes(f)
            expected.append(f)
        elif kind in (2, 8):
            b[p:p + 2] = f16_bytes(0.125)
            if kind == 8:
                expected.extend(float(np.float32(np.int8(np.uint8(v))) * np.float32(0.125)) for v in b[p + 2:p + 34])
            else:
                for shift in (0, 4):
                    expected.extend(float(np.float32(((v >> shift) & 15) - 8) * np.float32(0.125))
                                    for v in b[p + 2:p + 18])
        elif kind in (12, 13):
            b[p:p + 2] = f16_bytes(0.125)
            b[p + 2:p + 4] = f16_bytes(0.0625)
            packed = b[p + 4:p + 16]
            ds, ms = [0] * 8, [0] * 8
            for j in range(4):
                ds[j] = packed[j] & 63
                ms[j] = packed[j + 4] & 63
                ds[j + 4] = (packed[j + 8] & 15) | ((packed[j] >> 6) * 16)
                ms[j + 4] = (packed[j + 8] >> 4) | ((packed[j + 4] >> 6) * 16)
            qs = p + (16 if kind == 12 else 48)
            for chunk in range(4):
                for upper in range(2):
                    for lane in range(32):
                        q = (b[qs + chunk * 32 + lane] >> (upper * 4)) & 15
                        g = chunk * 2 + upper
                        if kind == 13 and ((b[p + 16 + lane] >> g) & 1):
                            q += 16
                        # 0.125 * ds * q - 0.0625 * ms, each product rounded to f32 (core.rs:109)
                        a = np.float32(np.float32(0.125) * np.float32(ds[g])) * np.float32(q)
                        c = np.float32(0.0625) * np.float32(ms[g])
                        expected.append(float(np.float32(a - c)))
        elif kind == 14:
            b[p + 208:p + 210] = f16_bytes(0.125)
            out = [0.0] * 256
            for chunk in range(2):
                for lane in range(32):
                    low0 = b[p + chunk * 64 + lane]
                    low1 = b[p + chunk * 64 + 32 + lane]
                    hi = b[p + 128 + chunk * 32 + lane]
                    qv = [(low0 & 15) | ((hi & 3) << 4), (low1 & 15) | (((hi >> 2) & 3) << 4),
                          (low0 >> 4) | (((hi >> 4) & 3) << 4), (low1 >> 4) | (((hi >> 6) & 3) << 4)]
                    for quarter in range(4):
                        sc = np.float32(np.int8(np.uint8(b[p + 192 + chunk * 8 + quarter * 2 + lane // 16])))
                        out[chunk * 128 + quarter * 32 + lane] = float(
                            np.float32(np.float32(0.125) * sc) * np.float32(qv[quarter] - 32))
            expected.extend(out)
    assert len(expected) == n * 2
    return np.frombuffer(bytes(b), dtype=np.uint8), np.array(expected, dtype=np.float32)


def load_reference_fixture():
    spec = importlib.util.spec_from_file_location("reference_fixture", REF / "tools" / "reference_fixture.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main() -> None:
    # 1. quant.rs two-block goldens
    arrays = {}
    for kind in (0, 1, 2, 8, 12, 13, 14):
        blocks, expected = core_fixture(kind)
        arrays[f"bytes_{kind}"] = blocks
        arrays[f"expected_{kind}"] = expected
    np.savez(HERE / "quant_blocks.npz", **arrays)

    # 2. the reference's F32 tiny model and NumPy logits
    rf = load_reference_fixture()
    tmp = HERE / "tiny_f32.gguf"
    weights = rf.create(tmp)
    expected = rf.reference(weights, [1, 5, 2, 9])
    ref_gguf = (REF / "tests" / "data" / "tiny-qwen3moe.gguf").read_bytes()
    assert tmp.read_bytes() == ref_gguf, "regenerated fixture differs from the reference's tests/data copy"
    parity = json.loads((REF / "validation" / "parity-cpu.json").read_text())
    (HERE / "tiny_f32_logits.json").write_text(json.dumps({
        "tokens": [1, 5, 2, 9],
        "expected_logits": expected,
        "reference_cpu_max_abs_error_by_prefix": parity["max_absolute_error_by_prefix"],
        "source": "tools/reference_fixture.py create()/reference(); validation/parity-cpu.json",
    }, indent=1))

    # 3. config 1: quantized tiny model, NumPy reference forward on dequantized weights
    sys.path.insert(0, str(ROOT))
    from __graft_entry__ import load_package
    load_package()
    from qwen30brust_b200 import tools
    from oracle import oracle as O

    spec = tools.TINY
    img = tools.synth_gguf(spec)
    sha = hashlib.sha256(img.tobytes()).hexdigest()
    om = O.Model(img, 64)  # parses the image with the oracle's gguf.rs restatement
    del om
    w = dequantize_all(img, O)
    H, D, NH, NKV, E, TOP, FF, V, L = (spec.hidden, spec.head_dim, spec.heads, spec.kvheads, spec.experts,
                                        spec.top, spec.intermediate, spec.vocab, spec.layers)
    for k, v in dict(H=H, D=D, NH=NH, NKV=NKV, E=E, TOP=TOP, FF=FF, VOCAB=V, LAYERS=L, EPS=spec.eps,
                     THETA=spec.theta).items():
        setattr(rf, k, v)
    prompt = np.random.default_rng(1).integers(0, V, 16).tolist()
    tokens = list(prompt)
    for _ in range(32):  # greedy continuation, argmax ties to the lowest id (sampling.rs:31-35)
        last = rf.reference(w, tokens)[-1]
        tokens.append(int(np.argmax(np.array(last, dtype=np.float32))))
    logits = np.array(rf.reference(w, tokens), dtype=np.float32)  # every position, teacher-forced
    np.savez(HERE / "tiny_q_golden.npz", tokens=np.array(tokens, dtype=np.uint32),
             prompt_len=np.array(16), logits=logits, gguf_sha256=np.array(sha))
    print("tiny quantized model sha256", sha, "tokens", tokens)


def dequantize_all(img: np.ndarray, O) -> dict[str, np.ndarray]:
    """Every tensor of a GGUF image as float32 in NumPy orientation (rows, cols) / (E, rows, cols)."""
    import struct
    buf = img.tobytes()
    pos = 4 + 4
    nt, nk = struct.unpack_from("<QQ", buf, pos)
    pos += 16

    def rstr(p):
        n, = struct.unpack_from("<Q", buf, p)
        return buf[p + 8:p + 8 + n].decode(), p + 8 + n

    for _ in range(nk):
        _, pos = rstr(pos)
        t, = struct.unpack_from("<I", buf, pos)
        pos += 4
        if t == 8:
            _, pos = rstr(pos)
        else:
            pos += {4: 4, 6: 4}[t]
    infos = []
    for _ in range(nt):
        name, pos = rstr(pos)
        nd, = struct.unpack_from("<I", buf, pos)
        pos += 4
        dims = list(struct.unpack_from("<" + "Q" * nd, buf, pos))
        pos += 8 * nd
        kind, off = struct.unpack_from("<IQ", buf, pos)
        pos += 12
        infos.append((name, dims, kind, off))
    start = (pos + 31) // 32 * 32
    out = {}
    for name, dims, kind, off in infos:
        cols = dims[0]
        rows = int(np.prod(dims[1:])) if len(dims) > 1 else 1
        rb = O.row_bytes(kind, cols)
        data = img[start + off:start + off + rb * rows]
        vals = O.decode_rows(data, kind, rows, cols)
        out[name] = vals.reshape(list(reversed(dims))) if len(dims) > 1 else vals.reshape(cols)
    return out


if __name__ == "__main__":
    import argparse
    ap = argparse.ArgumentParser(description="regenerate tests/golden/ from the reference checkout")
    ap.add_argument("--reference", required=True, type=Path, help="path of the K410Sh4/QWEN-30BRust checkout")
    REF = ap.parse_args().reference.resolve()
    main()
