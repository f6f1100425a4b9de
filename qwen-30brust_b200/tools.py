"""Host-side model tooling: GGML block quantizers and synthetic GGUF images.

ctypes bindings for libqwen_tools.so (include/qwen_tools.h).  The presets
below are the benchmark configurations: `TINY` is the 2-layer hidden-256 model
the reference's CPU path runs in seconds, `QWEN3_30B_A3B` the full
Qwen3-30B-A3B architecture with a Q4_K_M-style type mix.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, asdict, replace
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libqwen_tools.so"

F32, F16, Q4_0, Q8_0, Q4_K, Q5_K, Q6_K = 0, 1, 2, 8, 12, 13, 14
KIND_NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q8_0: "Q8_0", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K"}
BLOCK = {F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176),
         Q6_K: (256, 210)}


def row_bytes(kind: int, cols: int) -> int:
    block, size = BLOCK[kind]
    if cols <= 0 or cols % block:
        raise ValueError(f"row width {cols} is not divisible by block size {block}")
    return cols // block * size


class _Spec(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("hidden", "layers", "heads", "kvheads", "head_dim", "experts", "top",
                                           "intermediate", "vocab", "context_length")] + [
        ("eps", C.c_float), ("theta", C.c_float)] + [
        (n, C.c_uint32) for n in ("kind_embd", "kind_attn", "kind_attn_out", "kind_router", "kind_gate_up",
                                   "kind_down", "kind_output", "tied_output")] + [
        ("weight_std", C.c_float), ("norm_value", C.c_float), ("seed", C.c_uint64)]


@dataclass(frozen=True)
class ModelSpec:
    hidden: int
    layers: int
    heads: int
    kvheads: int
    head_dim: int
    experts: int
    top: int
    intermediate: int
    vocab: int
    context_length: int
    eps: float = 1e-6
    theta: float = 1e6
    kind_embd: int = Q8_0
    kind_attn: int = Q4_K
    kind_attn_out: int = Q4_K
    kind_router: int = F16
    kind_gate_up: int = Q4_K
    kind_down: int = Q6_K
    kind_output: int = Q6_K
    tied_output: int = 0
    weight_std: float = 0.02
    norm_value: float = 1.0
    seed: int = 0

    def with_(self, **kw) -> "ModelSpec":
        return replace(self, **kw)


# 2 layers, hidden 256, 4q/2kv x 64, 8 experts top-2, I=256, vocab 512, theta 1e6.
TINY = ModelSpec(hidden=256, layers=2, heads=4, kvheads=2, head_dim=64, experts=8, top=2, intermediate=256,
                 vocab=512, context_length=4096, eps=1e-6, theta=1e6)
# Qwen3-30B-A3B shape, Q4_K attention/gate/up, Q6_K down/output, F16 router.
QWEN3_30B_A3B = ModelSpec(hidden=2048, layers=48, heads=32, kvheads=4, head_dim=128, experts=128, top=8,
                          intermediate=768, vocab=151936, context_length=4096, eps=1e-6, theta=1e7)

_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is not built; run __graft_entry__.build()")
        L = C.CDLL(str(LIB_PATH))
        L.qct_quantize.argtypes = [C.c_uint32, C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t]
        L.qct_normal.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_float, C.c_float, C.c_void_p, C.c_size_t]
        L.qct_stream_of.argtypes = [C.c_char_p]
        L.qct_stream_of.restype = C.c_uint64
        L.qct_random_matrix.argtypes = [C.c_uint32, C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64, C.c_float,
                                        C.c_void_p, C.c_size_t, C.c_int]
        L.qct_synth_size.argtypes = [C.POINTER(_Spec), C.POINTER(C.c_uint64)]
        L.qct_synth_write.argtypes = [C.POINTER(_Spec), C.c_void_p, C.c_uint64, C.c_int]
        L.qct_f16_to_f32.argtypes = [C.c_uint16]
        L.qct_f16_to_f32.restype = C.c_float
        L.qct_f32_to_f16.argtypes = [C.c_float]
        L.qct_f32_to_f16.restype = C.c_uint16
        _lib = L
    return _lib


def quantize(kind: int, x) -> np.ndarray:
    xx = np.ascontiguousarray(x, dtype=np.float32).ravel()
    block, size = BLOCK[kind]
    out = np.empty(xx.size // block * size, dtype=np.uint8)
    rc = lib().qct_quantize(kind, xx.ctypes.data, xx.size, out.ctypes.data, out.size)
    if rc:
        raise ValueError(f"qct_quantize({kind}, n={xx.size}) failed: {rc}")
    return out


def normal(seed: int, stream: int, n: int, mean: float = 0.0, std: float = 1.0, first: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().qct_normal(seed, stream, first, mean, std, out.ctypes.data, n)
    return out


def stream_of(name: str) -> int:
    return lib().qct_stream_of(name.encode())


def random_matrix(kind: int, rows: int, cols: int, seed: int, stream: int, std: float = 0.02,
                  threads: int = 0, out: np.ndarray | None = None) -> np.ndarray:
    n = row_bytes(kind, cols) * rows
    if out is None:
        out = np.empty(n, dtype=np.uint8)
    assert out.size >= n and out.dtype == np.uint8
    rc = lib().qct_random_matrix(kind, rows, cols, seed, stream, std, out.ctypes.data, out.size, threads)
    if rc:
        raise ValueError(f"qct_random_matrix failed: {rc}")
    return out


def _spec(s: ModelSpec) -> _Spec:
    return _Spec(**asdict(s))


def synth_size(spec: ModelSpec) -> int:
    total = C.c_uint64()
    rc = lib().qct_synth_size(C.byref(_spec(spec)), C.byref(total))
    if rc:
        raise ValueError(f"invalid spec: {rc}")
    return total.value


def synth_gguf(spec: ModelSpec, threads: int = 0, out: np.ndarray | None = None) -> np.ndarray:
    """The GGUF image of a synthetic model as a uint8 array (identical to a file's bytes)."""
    n = synth_size(spec)
    if out is None:
        out = np.empty(n, dtype=np.uint8)
    assert out.size >= n
    rc = lib().qct_synth_write(C.byref(_spec(spec)), out.ctypes.data, out.size, threads)
    if rc:
        raise ValueError(f"qct_synth_write failed: {rc}")
    return out[:n]


def f16_to_f32(v: int) -> float:
    return lib().qct_f16_to_f32(v)


def f32_to_f16(v: float) -> int:
    return lib().qct_f32_to_f16(v)


def gguf_table(buf) -> tuple[dict, list, int]:
    """Walk a GGUF image's header (gguf.rs:102-195 layout): (metadata scalars and strings,
    [(name, dims, kind, offset relative to the data start)], data start)."""
    import struct
    buf = bytes(buf) if not isinstance(buf, (bytes, bytearray)) else buf
    pos = 8
    nt, nk = struct.unpack_from("<QQ", buf, pos)
    pos += 16

    def rstr(p):
        n, = struct.unpack_from("<Q", buf, p)
        return buf[p + 8:p + 8 + n].decode(), p + 8 + n

    sizes = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 10: 8, 11: 8, 12: 8}
    meta = {}
    for _ in range(nk):
        k, pos = rstr(pos)
        t, = struct.unpack_from("<I", buf, pos)
        pos += 4
        if t == 8:
            meta[k], pos = rstr(pos)
        elif t == 9:
            it, n = struct.unpack_from("<IQ", buf, pos)
            pos += 12
            for _ in range(n):
                if it == 8:
                    _, pos = rstr(pos)
                else:
                    pos += sizes[it]
        else:
            meta[k] = struct.unpack_from("<" + {4: "I", 6: "f"}.get(t, "I"), buf, pos)[0]
            pos += sizes[t]
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
    return meta, infos, start


def tensor_view(img: np.ndarray, name: str) -> tuple[np.ndarray, int, list]:
    """(the bytes of tensor `name` inside a GGUF image, as a writable view; kind; dims)."""
    _, infos, start = gguf_table(img[:1 << 22].tobytes() if img.size > (1 << 22) else img.tobytes())
    for n, dims, kind, off in infos:
        if n == name:
            nbytes = row_bytes(kind, dims[0]) * int(np.prod(dims[1:], dtype=np.int64))
            return img[start + off:start + off + nbytes], kind, dims
    raise KeyError(name)


def skew_router(img: np.ndarray, layer: int, s: float) -> None:
    """Scale row e of an F16 router (ffn_gate_inp) by (e + 1)^-s, in place: larger rows win the
    top-k more often, so the expert load falls off with the expert index (Zipf-like)."""
    v, kind, dims = tensor_view(img, f"blk.{layer}.ffn_gate_inp.weight")
    assert kind == F16
    w = v.view(np.float16).reshape(dims[1], dims[0])
    g = (np.arange(dims[1], dtype=np.float64) + 1.0) ** -s
    w[:] = (w.astype(np.float64) * g[:, None]).astype(np.float16)
