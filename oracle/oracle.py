"""ctypes bindings for the CPU oracle (test infrastructure only).

`liboracle.so` restates the reference crate's CPU path (quant.rs, backend.rs
Cpu::matvec, ops.rs, model.rs, gguf.rs, sampling.rs greedy).  Only the tests,
`__graft_entry__.smoke()` and bench.py's CPU-baseline arm use this module: it
is the checker, never the product.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

_lib = None


def build() -> Path:
    """Compile liboracle.so from oracle.cpp (make, in place)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        sz, u32, f32, vp = C.c_size_t, C.c_uint32, C.c_float, C.c_void_p
        fp = C.POINTER(C.c_float)
        L.or_last_error.restype = C.c_char_p
        L.or_layout.argtypes = [u32, C.POINTER(sz), C.POINTER(sz)]
        L.or_row_bytes.argtypes = [u32, sz, C.POINTER(sz)]
        L.or_decode.argtypes = [vp, sz, u32, sz, fp]
        L.or_decode_rows.argtypes = [vp, u32, sz, sz, fp]
        L.or_matvec.argtypes = [vp, sz, u32, sz, sz, fp, fp, C.c_int]
        L.or_rms.argtypes = [fp, fp, sz, f32]
        L.or_rope.argtypes = [fp, sz, sz, sz, f32]
        L.or_softmax.argtypes = [fp, sz]
        L.or_route.argtypes = [fp, sz, sz, C.POINTER(u32), fp]
        L.or_attention.argtypes = [fp, fp, fp, sz, sz, sz, sz, fp]
        L.or_sample_greedy.argtypes = [fp, sz, C.POINTER(u32)]
        L.or_model_open.argtypes = [C.c_char_p, sz, C.c_int]
        L.or_model_open.restype = vp
        L.or_model_from_memory.argtypes = [vp, sz, sz, C.c_int]
        L.or_model_from_memory.restype = vp
        L.or_model_forward.argtypes = [vp, u32, fp]
        L.or_model_reset.argtypes = [vp]
        L.or_model_prefill.argtypes = [vp, C.POINTER(u32), sz]
        L.or_model_set_fast.argtypes = [vp, C.c_int]
        L.or_model_set_fast.restype = None
        L.or_matvec_fast.argtypes = [vp, sz, u32, sz, sz, fp, fp, C.c_int]
        L.or_model_position.argtypes = [vp]
        L.or_model_position.restype = sz
        L.or_model_matvecs.argtypes = [vp]
        L.or_model_matvecs.restype = C.c_uint64
        L.or_model_config.argtypes = [vp, C.POINTER(sz), fp]
        L.or_model_free.argtypes = [vp]
        L.or_gguf_check.argtypes = [vp, sz]
        L.or_f16_to_f32.argtypes = [C.c_uint16]
        L.or_f16_to_f32.restype = f32
        L.or_chacha_block.argtypes = [C.POINTER(u32), C.c_int, C.POINTER(u32)]
        L.or_chacha_block.restype = None
        L.or_sampler_new.argtypes = [C.c_uint64, f32, sz, f32]
        L.or_sampler_new.restype = vp
        L.or_sampler_sample.argtypes = [vp, fp, sz, C.POINTER(u32)]
        L.or_sampler_next_u32.argtypes = [vp]
        L.or_sampler_next_u32.restype = u32
        L.or_sampler_key.argtypes = [vp, C.POINTER(u32)]
        L.or_sampler_key.restype = None
        L.or_sampler_free.argtypes = [vp]
        L.or_sampler_free.restype = None
        _lib = L
    return _lib


class OracleError(RuntimeError):
    pass


def _check(rc: int) -> None:
    if rc != 0:
        raise OracleError(lib().or_last_error().decode())


def _fp(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def layout(kind: int) -> tuple[int, int]:
    b, n = C.c_size_t(), C.c_size_t()
    _check(lib().or_layout(kind, C.byref(b), C.byref(n)))
    return b.value, n.value


def row_bytes(kind: int, cols: int) -> int:
    out = C.c_size_t()
    _check(lib().or_row_bytes(kind, cols, C.byref(out)))
    return out.value


def decode(blocks: bytes | np.ndarray, kind: int, cols: int) -> np.ndarray:
    b = np.frombuffer(bytes(blocks), dtype=np.uint8) if not isinstance(blocks, np.ndarray) else blocks
    b = np.ascontiguousarray(b, dtype=np.uint8)
    out = np.empty(cols, dtype=np.float32)
    _check(lib().or_decode(b.ctypes.data, b.size, kind, cols, _fp(out)))
    return out


def decode_rows(blocks: np.ndarray, kind: int, rows: int, cols: int) -> np.ndarray:
    b = np.ascontiguousarray(blocks, dtype=np.uint8)
    assert b.size >= row_bytes(kind, cols) * rows
    out = np.empty((rows, cols), dtype=np.float32)
    _check(lib().or_decode_rows(b.ctypes.data, kind, rows, cols, _fp(out)))
    return out


def matvec(blocks: np.ndarray, kind: int, rows: int, cols: int, x, threads: int = 0, fast: bool = False) -> np.ndarray:
    """backend.rs Cpu::matvec; `fast` decodes a block at a time (identical results, faster)."""
    b = np.ascontiguousarray(blocks, dtype=np.uint8)
    xx = _f32(x)
    assert xx.size == cols
    y = np.empty(rows, dtype=np.float32)
    fn = lib().or_matvec_fast if fast else lib().or_matvec
    _check(fn(b.ctypes.data, b.size, kind, rows, cols, _fp(xx), _fp(y), threads))
    return y


def rms(x, w, eps: float) -> np.ndarray:
    xx, ww = _f32(x).copy(), _f32(w)
    _check(lib().or_rms(_fp(xx), _fp(ww), xx.size, eps))
    return xx


def rope(x, head: int, pos: int, theta: float) -> np.ndarray:
    xx = _f32(x).copy()
    lib().or_rope(_fp(xx), xx.size, head, pos, theta)
    return xx


def softmax(x) -> np.ndarray:
    xx = _f32(x).copy()
    _check(lib().or_softmax(_fp(xx), xx.size))
    return xx


def route(logits, top: int) -> list[tuple[int, float]]:
    ll = _f32(logits)
    ids = (C.c_uint32 * max(top, 1))()
    w = np.empty(max(top, 1), dtype=np.float32)
    _check(lib().or_route(_fp(ll), ll.size, top, ids, _fp(w)))
    return [(int(ids[i]), float(w[i])) for i in range(top)]


def attention(q, k, v, heads: int, kvheads: int, d: int) -> np.ndarray:
    qq, kk, vv = _f32(q), _f32(k), _f32(v)
    time = kk.size // (kvheads * d)
    out = np.empty(heads * d, dtype=np.float32)
    _check(lib().or_attention(_fp(qq), _fp(kk), _fp(vv), heads, kvheads, d, time, _fp(out)))
    return out


def sample_greedy(logits) -> int:
    ll = _f32(logits)
    out = C.c_uint32()
    _check(lib().or_sample_greedy(_fp(ll), ll.size, C.byref(out)))
    return out.value


def gguf_check(buf: bytes) -> None:
    b = np.frombuffer(buf, dtype=np.uint8)
    _check(lib().or_gguf_check(b.ctypes.data if b.size else None, b.size))


CONFIG_KEYS = ("hidden", "layers", "heads", "kvheads", "head_dim", "experts", "top",
               "intermediate", "vocab", "max_context")


class Model:
    """model.rs Model with the Cpu backend: `forward(token) -> logits`, reset on error."""

    def __init__(self, source: str | os.PathLike | np.ndarray, context: int, threads: int = 0, fast: bool = False):
        """`fast`: block-decoding matvecs, bit-identical to the reference's per-element decode
        (the default, which the CPU baseline times); for tests that run many tokens."""
        L = lib()
        self._buf = None
        if isinstance(source, np.ndarray):
            self._buf = np.ascontiguousarray(source, dtype=np.uint8)
            h = L.or_model_from_memory(self._buf.ctypes.data, self._buf.size, context, threads)
        else:
            h = L.or_model_open(str(source).encode(), context, threads)
        if not h:
            raise OracleError(L.or_last_error().decode())
        self._h = h
        v = (C.c_size_t * 10)()
        et = np.empty(2, dtype=np.float32)
        L.or_model_config(h, v, _fp(et))
        self.config = dict(zip(CONFIG_KEYS, list(v)))
        self.config["eps"], self.config["theta"] = float(et[0]), float(et[1])
        L.or_model_set_fast(h, 1 if fast else 0)

    def forward(self, token: int, want_logits: bool = True) -> np.ndarray | None:
        """One token; with want_logits False the output projection is skipped (returns None)."""
        if not want_logits:
            _check(lib().or_model_forward(self._h, token, None))
            return None
        out = np.empty(self.config["vocab"], dtype=np.float32)
        _check(lib().or_model_forward(self._h, token, _fp(out)))
        return out

    def set_fast(self, fast: bool) -> None:
        """Block-decoding (True) or per-element (False, the reference's way) matvecs from now on."""
        lib().or_model_set_fast(self._h, 1 if fast else 0)

    def prefill(self, tokens) -> None:
        """Forwards of `tokens` without logits, computed layer by layer over all of them (each
        weight row decoded once per layer): the same KV cache and position as one forward per
        token, much faster.  Test and benchmark set-up only."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        _check(lib().or_model_prefill(self._h, t.ctypes.data_as(C.POINTER(C.c_uint32)), t.size))

    def reset(self) -> None:
        lib().or_model_reset(self._h)

    @property
    def position(self) -> int:
        return lib().or_model_position(self._h)

    @property
    def matvecs(self) -> int:
        return lib().or_model_matvecs(self._h)

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().or_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def chacha_block(state16, rounds: int) -> np.ndarray:
    """The ChaCha block function (input state of 16 words + state) with `rounds` rounds."""
    a = np.ascontiguousarray(state16, dtype=np.uint32)
    out = np.empty(16, dtype=np.uint32)
    lib().or_chacha_block(a.ctypes.data_as(C.POINTER(C.c_uint32)), rounds, out.ctypes.data_as(C.POINTER(C.c_uint32)))
    return out


class Sampler:
    """sampling.rs Sampler (StdRng = ChaCha12 seeded by seed_from_u64)."""

    def __init__(self, seed: int, temperature: float, top_k: int, top_p: float):
        h = lib().or_sampler_new(seed, temperature, top_k, top_p)
        if not h:
            raise OracleError(lib().or_last_error().decode())
        self._h = h

    def sample(self, logits) -> int:
        ll = np.ascontiguousarray(logits, dtype=np.float32)
        out = C.c_uint32()
        _check(lib().or_sampler_sample(self._h, _fp(ll), ll.size, C.byref(out)))
        return out.value

    def next_u32(self) -> int:
        return lib().or_sampler_next_u32(self._h)

    def key(self) -> np.ndarray:
        k = np.empty(8, dtype=np.uint32)
        lib().or_sampler_key(self._h, k.ctypes.data_as(C.POINTER(C.c_uint32)))
        return k

    def __del__(self):
        if getattr(self, "_h", None):
            lib().or_sampler_free(self._h)
            self._h = None
