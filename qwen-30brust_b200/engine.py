"""ctypes bindings of the C ABI in include/qwen_cuda.h (libqwen_cuda.so).

This mirrors the reference crate's interface on the host side:
  Engine.forward(token)         ~ Model::forward (src/model.rs:210-216)
  Engine.forward_tokens(ids)    ~ the `logits` command's loop (src/main.rs:144-146)
  Engine.decode_greedy(n)       ~ the chat loop with temperature 0 (src/main.rs:261-282)
  packed_matvec(...)            ~ Vulkan::packed_matvec (src/backend.rs:174-261)
  Matrix                        ~ a resident weight matrix for Backend::matvec
Errors raise QwenCudaError with the engine's message and status code.  There is
no CPU fallback: if the library is missing, loading fails.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libqwen_cuda.so"

OK, ERR_INVALID, ERR_CUDA, ERR_CONTEXT, ERR_TOKEN, ERR_NONFINITE, ERR_NOMEM = range(7)

EXPORTS = (
    "qc_engine_create", "qc_engine_create_gguf", "qc_engine_open", "qc_engine_destroy", "qc_engine_error",
    "qc_last_error", "qc_engine_config", "qc_engine_set_stream", "qc_forward", "qc_forward_tokens",
    "qc_decode_greedy", "qc_decode_enqueue", "qc_sync", "qc_reset", "qc_position", "qc_get_stats",
    "qc_logits_device", "qc_row_bytes", "qc_matrix_create", "qc_matrix_matvec", "qc_matrix_dequant",
    "qc_matrix_bytes", "qc_matrix_destroy", "qc_packed_matvec", "qc_profile_step", "qc_packed_matvec_noalloc",
    "qc_engine_set_decode_mode", "qc_engine_decode_path", "qc_engine_create_gguf_ep", "qc_engine_ep_handle",
    "qc_engine_ep_connect", "qc_sampler_create", "qc_sampler_destroy", "qc_sampler_sample", "qc_sampler_words",
    "qc_engine_sample", "qc_decode_sample", "qc_moe_layer", "qc_batch_create", "qc_batch_destroy",
    "qc_batch_forward", "qc_batch_reset", "qc_batch_position", "qc_batch_logits_device", "qc_batch_sample",
    "qc_batch_decode_sample", "qc_batch_stats", "qc_batch_ep_handle", "qc_batch_ep_connect",
)


def connect_group(eng, group=None) -> None:
    """Connect an expert-parallel engine (or a Batch of one) to its peers:
    all-gather every rank's ep_handle() over torch.distributed (any backend;
    rank order of `group`), then .connect.  Each rank of the group must call it."""
    import torch.distributed as dist
    allh = [None] * dist.get_world_size(group)
    dist.all_gather_object(allh, eng.ep_handle(), group=group)
    eng.connect(allh)


class QwenCudaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code
        self.msg = msg


class Config(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("hidden", "layers", "heads", "kvheads", "head_dim", "experts", "top",
                                           "intermediate", "vocab", "max_context")] + [
        ("eps", C.c_float), ("theta", C.c_float)]

    def as_dict(self) -> dict:
        return {n: getattr(self, n) for n, _ in self._fields_}


class TensorDesc(C.Structure):
    _fields_ = [("name", C.c_char_p), ("kind", C.c_uint32), ("n_dims", C.c_uint32), ("dims", C.c_uint64 * 3),
                ("offset", C.c_uint64), ("len", C.c_uint64)]


PHASES = ("embed", "attn_in", "attention", "oproj", "router", "gateup", "down", "output")


class PhaseTimes(C.Structure):
    _fields_ = [(p + "_ms", C.c_double) for p in PHASES] + [("launches", C.c_uint32), ("token_ms", C.c_double)]


class Stats(C.Structure):
    _fields_ = [("matvecs", C.c_uint64), ("uploaded_bytes", C.c_uint64), ("cache_hits", C.c_uint64),
                ("matvec_ms", C.c_double), ("tokens", C.c_uint64), ("weight_bytes", C.c_uint64),
                ("kv_bytes", C.c_uint64)]

    def as_dict(self) -> dict:
        return {n: getattr(self, n) for n, _ in self._fields_}


_lib = None


def lib() -> C.CDLL:
    """Load libqwen_cuda.so (built by qwen-30brust_b200/build.py); fails loudly if absent."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is not built; run `python __graft_entry__.py` / build()")
        L = C.CDLL(str(LIB_PATH))
        vp, u32, u64, sz, i = C.c_void_p, C.c_uint32, C.c_uint64, C.c_size_t, C.c_int
        pp = C.POINTER(vp)
        L.qc_engine_create.argtypes = [C.POINTER(TensorDesc), sz, vp, sz, C.POINTER(Config), u32, i, pp]
        L.qc_engine_create_gguf.argtypes = [vp, sz, u32, i, pp]
        L.qc_engine_open.argtypes = [C.c_char_p, u32, i, pp]
        L.qc_engine_destroy.argtypes = [vp]
        L.qc_engine_destroy.restype = None
        L.qc_engine_error.argtypes = [vp]
        L.qc_engine_error.restype = C.c_char_p
        L.qc_last_error.restype = C.c_char_p
        L.qc_engine_config.argtypes = [vp, C.POINTER(Config)]
        L.qc_engine_set_stream.argtypes = [vp, vp]
        L.qc_forward.argtypes = [vp, u32, vp]
        L.qc_forward_tokens.argtypes = [vp, vp, sz, vp]
        L.qc_decode_greedy.argtypes = [vp, u32, vp, vp]
        L.qc_decode_enqueue.argtypes = [vp, u32]
        L.qc_sync.argtypes = [vp]
        L.qc_reset.argtypes = [vp]
        L.qc_position.argtypes = [vp, C.POINTER(u32)]
        L.qc_get_stats.argtypes = [vp, C.POINTER(Stats)]
        L.qc_logits_device.argtypes = [vp, pp]
        L.qc_row_bytes.argtypes = [u32, u64, C.POINTER(u64)]
        L.qc_matrix_create.argtypes = [u32, u64, u64, u64, vp, u64, i, pp]
        L.qc_matrix_matvec.argtypes = [vp, u32, vp, vp, vp]
        L.qc_matrix_dequant.argtypes = [vp, u32, vp, vp]
        L.qc_matrix_bytes.argtypes = [vp, C.POINTER(u64), C.POINTER(u64)]
        L.qc_matrix_destroy.argtypes = [vp]
        L.qc_matrix_destroy.restype = None
        L.qc_packed_matvec.argtypes = [u32, u64, u64, vp, u64, vp, vp]
        L.qc_profile_step.argtypes = [vp, C.POINTER(PhaseTimes)]
        L.qc_packed_matvec_noalloc.argtypes = [u32, u64, u64, vp, u64, vp, vp]
        L.qc_engine_set_decode_mode.argtypes = [vp, C.c_int]
        L.qc_engine_decode_path.argtypes = [vp, C.POINTER(C.c_int), C.POINTER(C.c_char_p)]
        L.qc_engine_create_gguf_ep.argtypes = [vp, sz, u32, i, u32, u32, pp]
        L.qc_engine_ep_handle.argtypes = [vp, vp, C.POINTER(C.c_int)]
        L.qc_engine_ep_connect.argtypes = [vp, vp, vp]
        L.qc_sampler_create.argtypes = [u64, C.c_float, u32, C.c_float, i, pp]
        L.qc_sampler_destroy.argtypes = [vp]
        L.qc_sampler_destroy.restype = None
        L.qc_sampler_sample.argtypes = [vp, vp, u32, vp, C.POINTER(u32)]
        L.qc_sampler_words.argtypes = [vp, u32, vp]
        L.qc_engine_sample.argtypes = [vp, vp, C.POINTER(u32)]
        L.qc_decode_sample.argtypes = [vp, vp, u32, vp, vp]
        L.qc_moe_layer.argtypes = [vp, u32, vp, u32, vp, i, C.POINTER(C.c_float)]
        L.qc_batch_create.argtypes = [vp, u32, u32, pp]
        L.qc_batch_destroy.argtypes = [vp]
        L.qc_batch_destroy.restype = None
        L.qc_batch_forward.argtypes = [vp, vp, vp, u32, vp]
        L.qc_batch_reset.argtypes = [vp, u32]
        L.qc_batch_position.argtypes = [vp, u32, C.POINTER(u32)]
        L.qc_batch_logits_device.argtypes = [vp, u32, pp]
        L.qc_batch_sample.argtypes = [vp, vp, vp, u32, vp]
        L.qc_batch_decode_sample.argtypes = [vp, vp, vp, u32, u32, vp]
        L.qc_batch_stats.argtypes = [vp, C.POINTER(Stats)]
        L.qc_batch_ep_handle.argtypes = [vp, vp, C.POINTER(C.c_int)]
        L.qc_batch_ep_connect.argtypes = [vp, vp, vp]
        _lib = L
    return _lib


def _global_check(rc: int) -> None:
    if rc != OK:
        raise QwenCudaError(rc, lib().qc_last_error().decode())


def row_bytes(kind: int, cols: int) -> int:
    out = C.c_uint64()
    _global_check(lib().qc_row_bytes(kind, cols, C.byref(out)))
    return out.value


def _u8(a) -> np.ndarray:
    if isinstance(a, (bytes, bytearray)):
        return np.frombuffer(bytes(a), dtype=np.uint8)
    return np.ascontiguousarray(a, dtype=np.uint8)


class Sampler:
    """sampling.rs Sampler on the device (qc_sampler_*): Sampler(seed, temperature, top_k, top_p)."""

    def __init__(self, seed: int, temperature: float, top_k: int, top_p: float, device: int = 0):
        h = C.c_void_p()
        _global_check(lib().qc_sampler_create(seed, temperature, top_k, top_p, device, C.byref(h)))
        self._h = h

    def sample_device(self, logits_ptr: int, n: int, stream_ptr: int | None = None) -> int:
        """Sampler::sample on n float32 logits at a device address."""
        t = C.c_uint32()
        _global_check(lib().qc_sampler_sample(self._h, logits_ptr, n, stream_ptr, C.byref(t)))
        return t.value

    def words(self, n: int) -> np.ndarray:
        out = np.empty(max(n, 1), dtype=np.uint32)
        _global_check(lib().qc_sampler_words(self._h, n, out.ctypes.data))
        return out[:n]

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().qc_sampler_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Engine:
    """A resident Qwen3-MoE model on one GPU (see include/qwen_cuda.h)."""

    def __init__(self, source, context: int, device: int = 0):
        L = lib()
        h = C.c_void_p()
        if isinstance(source, (str, os.PathLike)):
            rc = L.qc_engine_open(str(source).encode(), context, device, C.byref(h))
        else:
            img = _u8(source)
            rc = L.qc_engine_create_gguf(img.ctypes.data, img.size, context, device, C.byref(h))
        _global_check(rc)
        self._h = h
        cfg = Config()
        self._check(L.qc_engine_config(h, C.byref(cfg)))
        self.config = cfg.as_dict()
        self.vocab = cfg.vocab
        self.context = context

    @classmethod
    def from_tensors(cls, tensors: list[dict], base: np.ndarray, config: dict, context: int, device: int = 0):
        """qc_engine_create: a parsed tensor table over `base` (name, kind, dims, offset, len)."""
        L = lib()
        arr = (TensorDesc * len(tensors))()
        names = []
        for k, t in enumerate(tensors):
            nm = t["name"].encode()
            names.append(nm)
            arr[k].name = nm
            arr[k].kind = t["kind"]
            arr[k].n_dims = len(t["dims"])
            for j, d in enumerate(t["dims"]):
                arr[k].dims[j] = d
            arr[k].offset = t["offset"]
            arr[k].len = t["len"]
        cfg = Config(**{k: config[k] for k, _ in Config._fields_})
        b = _u8(base)
        h = C.c_void_p()
        _global_check(L.qc_engine_create(arr, len(tensors), b.ctypes.data, b.size, C.byref(cfg), context, device,
                                         C.byref(h)))
        self = cls.__new__(cls)
        self._h = h
        self.config = cfg.as_dict()
        self.vocab = cfg.vocab
        self.context = context
        return self

    @classmethod
    def expert_parallel(cls, image, context: int, device: int, rank: int, world: int):
        """qc_engine_create_gguf_ep: this rank's share of the experts (one process and GPU per rank).

        The engine is usable after connect() with every rank's handle."""
        L = lib()
        img = _u8(image)
        h = C.c_void_p()
        _global_check(L.qc_engine_create_gguf_ep(img.ctypes.data, img.size, context, device, rank, world,
                                                 C.byref(h)))
        self = cls.__new__(cls)
        self._h = h
        cfg = Config()
        self._check(L.qc_engine_config(h, C.byref(cfg)))
        self.config = cfg.as_dict()
        self.vocab = cfg.vocab
        self.context = context
        self.rank, self.world = rank, world
        return self

    def ep_handle(self) -> tuple[bytes, int]:
        """(64-byte IPC handle of this rank's exchange buffer, id of its GPU)."""
        buf = (C.c_uint8 * 64)()
        dev = C.c_int()
        self._check(lib().qc_engine_ep_handle(self._h, buf, C.byref(dev)))
        return bytes(buf), dev.value

    def connect(self, handles: list[tuple[bytes, int]]) -> None:
        """qc_engine_ep_connect with every rank's ep_handle() in rank order."""
        hb = np.frombuffer(b"".join(h for h, _ in handles), dtype=np.uint8).copy()
        ids = np.array([d for _, d in handles], dtype=np.int32)
        self._check(lib().qc_engine_ep_connect(self._h, hb.ctypes.data, ids.ctypes.data))

    def _check(self, rc: int) -> None:
        if rc != OK:
            raise QwenCudaError(rc, lib().qc_engine_error(self._h).decode())

    def forward(self, token: int, want_logits: bool = True) -> np.ndarray | None:
        out = np.empty(self.vocab, dtype=np.float32) if want_logits else None
        self._check(lib().qc_forward(self._h, token, out.ctypes.data if out is not None else None))
        return out

    def forward_into(self, token: int, out: np.ndarray) -> None:
        """qc_forward writing into a caller-owned (e.g. pinned) float32 buffer."""
        self._check(lib().qc_forward(self._h, token, out.ctypes.data))

    def forward_tokens(self, tokens, want_logits: bool = True) -> np.ndarray | None:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.empty(self.vocab, dtype=np.float32) if want_logits else None
        self._check(lib().qc_forward_tokens(self._h, t.ctypes.data, t.size,
                                            out.ctypes.data if out is not None else None))
        return out

    def decode_greedy(self, n: int, want_logits: bool = False):
        toks = np.empty(max(n, 1), dtype=np.uint32)
        out = np.empty(self.vocab, dtype=np.float32) if want_logits else None
        self._check(lib().qc_decode_greedy(self._h, n, toks.ctypes.data, out.ctypes.data if out is not None else None))
        return toks[:n], out

    def decode_enqueue(self, n: int) -> None:
        self._check(lib().qc_decode_enqueue(self._h, n))

    def sync(self) -> None:
        self._check(lib().qc_sync(self._h))

    def reset(self) -> None:
        self._check(lib().qc_reset(self._h))

    def set_stream(self, stream_ptr: int | None) -> None:
        self._check(lib().qc_engine_set_stream(self._h, stream_ptr))

    @property
    def position(self) -> int:
        p = C.c_uint32()
        self._check(lib().qc_position(self._h, C.byref(p)))
        return p.value

    def stats(self) -> dict:
        s = Stats()
        self._check(lib().qc_get_stats(self._h, C.byref(s)))
        return s.as_dict()

    def profile_step(self) -> dict:
        """Per-kernel-kind device ms of one real decode step (advances the position)."""
        t = PhaseTimes()
        self._check(lib().qc_profile_step(self._h, C.byref(t)))
        out = {p: getattr(t, p + "_ms") for p in PHASES}
        out["launches"] = t.launches
        out["token"] = t.token_ms
        return out

    def set_decode_mode(self, mode: int) -> None:
        """0: the whole-token kernel when the model fits it (default); 1: the per-phase kernels."""
        self._check(lib().qc_engine_set_decode_mode(self._h, mode))

    @property
    def decode_path(self) -> tuple[int, str]:
        """(0 whole-token kernel | 1 per-phase kernels, why the whole-token kernel is not used or "")."""
        path, why = C.c_int(), C.c_char_p()
        self._check(lib().qc_engine_decode_path(self._h, C.byref(path), C.byref(why)))
        return path.value, (why.value or b"").decode()

    def sample(self, sampler: "Sampler") -> int:
        """qc_engine_sample: Sampler::sample on the logits of the last step."""
        t = C.c_uint32()
        self._check(lib().qc_engine_sample(self._h, sampler._h, C.byref(t)))
        return t.value

    def decode_sample(self, sampler: "Sampler", n: int, want_logits: bool = False):
        """qc_decode_sample: n (sample, step) pairs on the device; returns the n sampled ids."""
        toks = np.empty(max(n, 1), dtype=np.uint32)
        out = np.empty(self.vocab, dtype=np.float32) if want_logits else None
        self._check(lib().qc_decode_sample(self._h, sampler._h, n, toks.ctypes.data,
                                           out.ctypes.data if out is not None else None))
        return toks[:n], out

    def moe_layer(self, layer: int, x, path: int) -> tuple[np.ndarray, float]:
        """qc_moe_layer: the MoE half of `layer` for a batch of token vectors x [T][hidden].
        path 1: per-token decode kernels; path 2: tensor-core grouped GEMMs.  Returns (out, device ms)."""
        xx = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty_like(xx)
        ms = C.c_float()
        self._check(lib().qc_moe_layer(self._h, layer, xx.ctypes.data, xx.shape[0], out.ctypes.data, path,
                                       C.byref(ms)))
        return out, ms.value

    def logits_device_ptr(self) -> int:
        p = C.c_void_p()
        self._check(lib().qc_logits_device(self._h, C.byref(p)))
        return p.value

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().qc_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


class Batch:
    """Several sequences on one engine (qc_batch_*): per-sequence KV caches and positions, any mix of
    their tokens per step (decode tokens of many sequences, prompt chunks of one)."""

    def __init__(self, engine: Engine, n_seqs: int, context: int):
        h = C.c_void_p()
        engine._check(lib().qc_batch_create(engine._h, n_seqs, context, C.byref(h)))
        self._h, self.engine, self.n_seqs, self.context = h, engine, n_seqs, context
        self.vocab = engine.vocab

    def _check(self, rc: int) -> None:
        self.engine._check(rc)

    def forward(self, seq_ids, tokens, want_logits: bool = True) -> np.ndarray | None:
        """qc_batch_forward: returns [rows][vocab], one row per sequence of the call (its last token),
        in call order, or None."""
        sq = np.ascontiguousarray(seq_ids, dtype=np.uint32)
        tk = np.ascontiguousarray(tokens, dtype=np.uint32)
        assert sq.size == tk.size
        rows = len(dict.fromkeys(reversed(sq.tolist())))
        out = np.empty((rows, self.vocab), dtype=np.float32) if want_logits else None
        self._check(lib().qc_batch_forward(self._h, sq.ctypes.data, tk.ctypes.data, sq.size,
                                           out.ctypes.data if out is not None else None))
        if out is not None:  # rows are in order of each sequence's last token
            return out
        return None

    def reset(self, seq: int = 0xFFFFFFFF) -> None:
        self._check(lib().qc_batch_reset(self._h, seq))

    def position(self, seq: int) -> int:
        p = C.c_uint32()
        self._check(lib().qc_batch_position(self._h, seq, C.byref(p)))
        return p.value

    def logits_device_ptr(self, seq: int) -> int:
        p = C.c_void_p()
        self._check(lib().qc_batch_logits_device(self._h, seq, C.byref(p)))
        return p.value

    def sample(self, samplers: list, seq_ids) -> np.ndarray:
        sq = np.ascontiguousarray(seq_ids, dtype=np.uint32)
        sp = (C.c_void_p * len(samplers))(*[s._h.value for s in samplers])
        out = np.empty(max(sq.size, 1), dtype=np.uint32)
        self._check(lib().qc_batch_sample(self._h, sp, sq.ctypes.data, sq.size, out.ctypes.data))
        return out[:sq.size]

    def decode_sample(self, samplers: list, seq_ids, steps: int) -> np.ndarray:
        """qc_batch_decode_sample: [steps][n] sampled ids."""
        sq = np.ascontiguousarray(seq_ids, dtype=np.uint32)
        sp = (C.c_void_p * len(samplers))(*[s._h.value for s in samplers])
        out = np.empty((max(steps, 1), sq.size), dtype=np.uint32)
        self._check(lib().qc_batch_decode_sample(self._h, sp, sq.ctypes.data, sq.size, steps, out.ctypes.data))
        return out[:steps]

    def stats(self) -> dict:
        s = Stats()
        self._check(lib().qc_batch_stats(self._h, C.byref(s)))
        return s.as_dict()

    def ep_handle(self) -> tuple[bytes, int]:
        """(64-byte IPC handle of this rank's exchange region, id of its GPU): batches of an
        expert-parallel engine."""
        buf = (C.c_uint8 * 64)()
        dev = C.c_int()
        self._check(lib().qc_batch_ep_handle(self._h, buf, C.byref(dev)))
        return bytes(buf), dev.value

    def connect(self, handles: list[tuple[bytes, int]]) -> None:
        """qc_batch_ep_connect with every rank's ep_handle() in rank order."""
        hb = np.frombuffer(b"".join(h for h, _ in handles), dtype=np.uint8).copy()
        ids = np.array([d for _, d in handles], dtype=np.int32)
        self._check(lib().qc_batch_ep_connect(self._h, hb.ctypes.data, ids.ctypes.data))

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().qc_batch_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Matrix:
    """`experts` stacked (rows x cols) GGML matrices resident in the device layout."""

    def __init__(self, kind: int, rows: int, cols: int, blocks, experts: int = 1, device: int = 0):
        b = _u8(blocks)
        h = C.c_void_p()
        _global_check(lib().qc_matrix_create(kind, rows, cols, experts, b.ctypes.data, b.size, device, C.byref(h)))
        self._h = h
        self.kind, self.rows, self.cols, self.experts = kind, rows, cols, experts

    def matvec(self, x_ptr: int, y_ptr: int, stream: int | None = None, expert: int = 0) -> None:
        _global_check(lib().qc_matrix_matvec(self._h, expert, x_ptr, y_ptr, stream))

    def dequant(self, out_ptr: int, stream: int | None = None, expert: int = 0) -> None:
        _global_check(lib().qc_matrix_dequant(self._h, expert, out_ptr, stream))

    def nbytes(self) -> tuple[int, int]:
        d, p = C.c_uint64(), C.c_uint64()
        _global_check(lib().qc_matrix_bytes(self._h, C.byref(d), C.byref(p)))
        return d.value, p.value

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().qc_matrix_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def packed_matvec(kind: int, rows: int, cols: int, blocks, x) -> np.ndarray:
    b = _u8(blocks)
    xx = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(rows, dtype=np.float32)
    _global_check(lib().qc_packed_matvec(kind, rows, cols, b.ctypes.data, b.size, xx.ctypes.data, y.ctypes.data))
    return y


def packed_matvec_noalloc(kind: int, rows: int, cols: int, blocks, x) -> np.ndarray:
    """qc_packed_matvec_noalloc: as packed_matvec, with no device allocation — for hosts
    whose allocator owns the GPU's memory or that must not call cudaFree.  Working memory
    is one static 32 MiB array per GPU shared by all calls (overlapping calls race)."""
    b = _u8(blocks)
    xx = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(rows, dtype=np.float32)
    _global_check(lib().qc_packed_matvec_noalloc(kind, rows, cols, b.ctypes.data, b.size, xx.ctypes.data,
                                                 y.ctypes.data))
    return y
