"""Python binding (ctypes) of the B200 Qwen3 library's C ABI (include/q3_b200.h).

Mirrors the reference's C++ surface (asriva32/Qwen3.cpp include/inference.h): ``Qwen3`` (load,
ForwardToken, Generate, ResetInference), ``Block`` (Block::forward, ResetCache, GetCache) and
the free kernels. Errors raise the Python counterparts of the reference's exception types:
``InvalidArgument`` (std::invalid_argument), ``OutOfRange`` (std::out_of_range) and
``Q3RuntimeError`` (std::runtime_error).

The CUDA library must be built (``python qwen3.cpp_b200/build.py``); loading fails loudly when it
is missing. There is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
# Q3B200_LIB selects another build of the library (e.g. one compiled with self-checks).
LIB_PATH = Path(os.environ.get("Q3B200_LIB", PKG / "lib" / "libq3b200.so"))

F32P = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
U16P = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
I32P = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")


class Q3Error(Exception):
    code = -1


class Q3RuntimeError(Q3Error, RuntimeError):
    code = 1


class InvalidArgument(Q3Error, ValueError):
    code = 2


class OutOfRange(Q3Error, IndexError):
    code = 3


class DeviceTimeout(Q3RuntimeError):
    code = 5


_ERRORS = {1: Q3RuntimeError, 2: InvalidArgument, 3: OutOfRange, 5: DeviceTimeout}


class Config(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "dim", "hidden_dim", "head_dim", "n_layers", "n_heads", "n_kv_heads", "vocab_size",
        "max_seq_len", "bos_token_id", "eos_token_id", "rotary_dim")] + [
        ("rope_theta", C.c_float), ("norm_eps", C.c_float)] + [
        (n, C.c_int32) for n in ("tie_word_embeddings", "attention_bias", "qk_norm")]

    def as_dict(self) -> dict:
        return {n: getattr(self, n) for n, _ in self._fields_}

    @classmethod
    def from_dict(cls, d: dict) -> "Config":
        c = cls()
        for n, _ in cls._fields_:
            if n in d:
                setattr(c, n, d[n])
        return c


class GenStats(C.Structure):
    _fields_ = [("prompt_tokens", C.c_size_t), ("generated_tokens", C.c_size_t),
                ("prefill_seconds", C.c_double), ("decode_seconds", C.c_double),
                ("stopped_on_eos", C.c_int32), ("reached_token_limit", C.c_int32)]


_lib = None


def lib() -> C.CDLL:
    """Load libq3b200.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise FileNotFoundError(
            f"{LIB_PATH} is missing: build it with `python qwen3.cpp_b200/build.py`")
    L = C.CDLL(str(LIB_PATH))
    vp, i32, sz = C.c_void_p, C.c_int32, C.c_size_t
    L.q3_last_error.restype = C.c_char_p
    L.q3_version.restype = C.c_char_p
    sig = {
        "q3_model_load": [C.c_char_p, C.c_int, C.c_int, C.POINTER(vp)],
        "q3_model_config": [vp, C.POINTER(Config)],
        "q3_model_tensor_count": [vp, C.POINTER(C.c_int)],
        "q3_reset": [vp],
        "q3_forward_token": [vp, i32, C.c_int, vp],
        "q3_forward_token_ref": [vp, i32, C.c_int, C.POINTER(C.POINTER(C.c_float))],
        "q3_forward_token_layers": [vp, i32, C.c_int, vp, vp],
        "q3_forward_token_greedy": [vp, i32, C.c_int, C.POINTER(C.POINTER(C.c_float)),
                                    C.POINTER(C.c_int32)],
        "q3_kv_row": [vp, C.c_int, C.c_int, U16P, U16P],
        "q3_prefill": [vp, I32P, C.c_int, C.c_int, vp, vp],
        "q3_prefill_layers": [vp, I32P, C.c_int, C.c_int, vp, vp, vp],
        "q3_model_set_prefill_path": [vp, C.c_int],
        "q3_model_prefill_path": [vp, C.POINTER(C.c_int)],
        "q3_model_set_prefill_precision": [vp, C.c_int],
        "q3_model_prefill_precision": [vp, C.POINTER(C.c_int)],
        "q3_gemm_bf16": [vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, vp],
        "q3_gemm_f16": [vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, vp],
        "q3_batch_create": [vp, C.c_int, C.c_int, C.POINTER(vp)],
        "q3_batch_add": [vp, I32P, C.c_int, C.POINTER(C.c_int), vp, vp],
        "q3_batch_add_many": [vp, I32P, I32P, C.c_int, C.POINTER(C.c_int), vp, vp],
        "q3_batch_size": [vp, C.POINTER(C.c_int)],
        "q3_batch_stream": [vp, C.POINTER(vp)],
        "q3_batch_decode": [vp, C.c_int, vp],
        "q3_batch_decode_forced": [vp, I32P, C.c_int, vp, vp],
        "q3_batch_kv_row": [vp, C.c_int, C.c_int, C.c_int, U16P, U16P],
        "q3_tp_create": [vp, C.c_int, C.c_int, C.POINTER(vp)],
        "q3_tp_ipc_handle": [vp, vp],
        "q3_tp_connect": [vp, vp],
        "q3_tp_stream": [vp, C.POINTER(vp)],
        "q3_tp_decode": [vp, i32, C.c_int, C.c_int, vp],
        "q3_tp_decode_forced": [vp, I32P, C.c_int, C.c_int, vp],
        "q3_tp_configure": [vp, C.c_int, C.c_longlong],
        "q3_tp_reset": [vp],
        "q3_tp_set_path": [vp, C.c_int],
        "q3_tp_path": [vp, C.POINTER(C.c_int)],
        "q3_tp_nccl_unique_id": [vp],
        "q3_tp_nccl_connect": [vp, vp],
        "q3_decode_greedy": [vp, i32, C.c_int, C.c_int, vp, vp],
        "q3_decode_forced": [vp, I32P, C.c_int, C.c_int, vp, vp],
        "q3_generate": [vp, vp, C.c_int, sz, C.c_int, vp, C.POINTER(sz), C.POINTER(GenStats)],
        "q3_model_stream": [vp, C.POINTER(vp)],
        "q3_model_set_decode_path": [vp, C.c_int],
        "q3_model_decode_path": [vp, C.POINTER(C.c_int)],
        "q3_model_fused_timeout_selftest": [vp, C.POINTER(C.c_int)],
        "q3_model_fused_profile": [vp, i32, C.c_int, vp, sz, C.POINTER(C.c_int),
                                   C.POINTER(C.c_int)],
        "q3_block_create": [C.POINTER(Config), C.POINTER(vp), C.POINTER(sz), C.c_int, C.POINTER(vp)],
        "q3_block_forward": [vp, F32P, C.c_int, C.c_int, C.c_int, C.c_int],
        "q3_block_reset_cache": [vp],
        "q3_block_get_cache": [vp, U16P, U16P],
        "q3_block_set_cache": [vp, U16P, U16P],
        "q3_rmsnorm": [vp, vp, vp, C.c_float, C.c_int, vp],
        "q3_softmax": [vp, vp, C.c_int, vp],
        "q3_matmul": [vp, vp, vp, C.c_int, C.c_int, vp],
        "q3_rope": [vp, C.c_int, C.c_int, C.c_int, C.c_float, C.c_int, vp],
        "q3_ffn": [vp, vp, vp, vp, vp, vp, vp, C.c_int, C.c_int, vp],
        "q3_attn": [vp, vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, vp],
        "q3_attn_noalloc": [vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, vp],
        "q3_greedy": [vp, C.c_int, vp, vp],
    }
    for name, args in sig.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = C.c_int
    L.q3_model_free.argtypes = [vp]
    L.q3_model_free.restype = None
    L.q3_block_free.argtypes = [vp]
    L.q3_block_free.restype = None
    L.q3_batch_free.argtypes = [vp]
    L.q3_batch_free.restype = None
    L.q3_tp_free.argtypes = [vp]
    L.q3_tp_free.restype = None
    L.q3_attn_workspace_size.argtypes = [C.c_int, C.c_int]
    L.q3_attn_workspace_size.restype = sz
    L.q3_attn_noalloc_max_scratch.argtypes = []
    L.q3_attn_noalloc_max_scratch.restype = sz
    _lib = L
    return L


def check(status: int) -> None:
    if status != 0:
        msg = lib().q3_last_error().decode(errors="replace")
        raise _ERRORS.get(status, Q3Error)(msg)


def _ptr(a) -> int | None:
    return None if a is None else a.ctypes.data


class Qwen3:
    """class Qwen3 (include/inference.h:227-264) on one GPU."""

    def __init__(self, path: str | os.PathLike, context_length: int = 512, device: int = 0):
        h = C.c_void_p()
        self._lib = lib()  # held so that close() still works during interpreter shutdown
        check(self._lib.q3_model_load(str(path).encode(), context_length, device, C.byref(h)))
        self._h = h
        cfg = Config()
        check(lib().q3_model_config(h, C.byref(cfg)))
        self.config = cfg.as_dict()
        n = C.c_int()
        check(lib().q3_model_tensor_count(h, C.byref(n)))
        self.tensor_count = n.value

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.q3_model_free(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    @property
    def stream(self) -> int:
        s = C.c_void_p()
        check(lib().q3_model_stream(self._h, C.byref(s)))
        return s.value or 0

    def reset(self) -> None:
        """ResetInference (src/inference.cpp:583-590)."""
        check(lib().q3_reset(self._h))

    PATH_LAYERWISE = 0
    PATH_FUSED = 1

    @property
    def decode_path(self) -> int:
        p = C.c_int()
        check(lib().q3_model_decode_path(self._h, C.byref(p)))
        return p.value

    @decode_path.setter
    def decode_path(self, path: int) -> None:
        check(lib().q3_model_set_decode_path(self._h, int(path)))

    def fused_profile(self, token: int, pos: int) -> np.ndarray:
        """globaltimer stamps of one fused decode step, [phases, grid, 4] (ns)."""
        c = self.config
        cap = (5 * c["n_layers"] + 2) * 1024 * 8
        buf = np.zeros(cap, np.uint64)
        nph, grid = C.c_int(), C.c_int()
        check(lib().q3_model_fused_profile(self._h, int(token), int(pos), buf.ctypes.data, cap,
                                           C.byref(nph), C.byref(grid)))
        return buf[: nph.value * grid.value * 8].reshape(nph.value, grid.value, 8)

    def fused_timeout_selftest(self) -> bool:
        t = C.c_int()
        check(lib().q3_model_fused_timeout_selftest(self._h, C.byref(t)))
        return bool(t.value)

    def forward_token(self, token: int, pos: int) -> np.ndarray:
        """ForwardToken (src/inference.cpp:592-637): logits of one token."""
        out = np.empty(self.config["vocab_size"], np.float32)
        check(lib().q3_forward_token(self._h, int(token), int(pos), out.ctypes.data))
        return out

    def forward_token_ref(self, token: int, pos: int) -> np.ndarray:
        """ForwardToken returning a read-only view of the model's pinned logits buffer, valid
        until the next call (the reference returns a reference to its logits vector)."""
        ptr = C.POINTER(C.c_float)()
        check(lib().q3_forward_token_ref(self._h, int(token), int(pos), C.byref(ptr)))
        view = np.ctypeslib.as_array(ptr, shape=(self.config["vocab_size"],))
        view.flags.writeable = False
        return view

    def forward_token_greedy(self, token: int, pos: int):
        """ForwardToken + Sampler::Greedy: (read-only view of the model's pinned logits buffer,
        valid until the next call; the greedy token computed on the device)."""
        ptr = C.POINTER(C.c_float)()
        nxt = C.c_int32()
        check(lib().q3_forward_token_greedy(self._h, int(token), int(pos), C.byref(ptr),
                                            C.byref(nxt)))
        view = np.ctypeslib.as_array(ptr, shape=(self.config["vocab_size"],))
        view.flags.writeable = False
        return view, int(nxt.value)

    def forward_token_layers(self, token: int, pos: int):
        c = self.config
        hid = np.empty((c["n_layers"] + 1, c["dim"]), np.float32)
        out = np.empty(c["vocab_size"], np.float32)
        check(lib().q3_forward_token_layers(self._h, int(token), int(pos), hid.ctypes.data,
                                            out.ctypes.data))
        return hid, out

    def kv_row(self, layer: int, kv_pos: int):
        kvd = self.config["n_kv_heads"] * self.config["head_dim"]
        k = np.empty(kvd, np.uint16)
        v = np.empty(kvd, np.uint16)
        check(lib().q3_kv_row(self._h, layer, kv_pos, k, v))
        return k, v

    def prefill(self, ids, pos0: int = 0, want_logits: bool = True):
        ids = np.ascontiguousarray(ids, np.int32)
        logits = np.empty(self.config["vocab_size"], np.float32) if want_logits else None
        nxt = np.zeros(1, np.int32)
        check(lib().q3_prefill(self._h, ids, ids.size, pos0, _ptr(logits), nxt.ctypes.data))
        return logits, int(nxt[0])

    def prefill_layers(self, ids, pos0: int = 0):
        """Prefill returning the last prompt token's hidden state before the first layer and
        after every layer, its logits and its greedy argmax."""
        c = self.config
        ids = np.ascontiguousarray(ids, np.int32)
        hid = np.empty((c["n_layers"] + 1, c["dim"]), np.float32)
        logits = np.empty(c["vocab_size"], np.float32)
        nxt = np.zeros(1, np.int32)
        check(lib().q3_prefill_layers(self._h, ids, ids.size, pos0, hid.ctypes.data,
                                      logits.ctypes.data, nxt.ctypes.data))
        return hid, logits, int(nxt[0])

    PREFILL_TOKENWISE, PREFILL_BATCHED = 0, 1

    @property
    def prefill_path(self) -> int:
        p = C.c_int()
        check(lib().q3_model_prefill_path(self._h, C.byref(p)))
        return p.value

    @prefill_path.setter
    def prefill_path(self, path: int) -> None:
        check(lib().q3_model_set_prefill_path(self._h, int(path)))

    PREFILL_BF16, PREFILL_F16 = 0, 1

    @property
    def prefill_precision(self) -> int:
        p = C.c_int()
        check(lib().q3_model_prefill_precision(self._h, C.byref(p)))
        return p.value

    @prefill_precision.setter
    def prefill_precision(self, precision: int) -> None:
        check(lib().q3_model_set_prefill_precision(self._h, int(precision)))

    def decode_greedy(self, first_token: int, pos0: int, n_steps: int, want_logits=False):
        toks = np.empty(max(n_steps, 1), np.int32)
        logits = np.empty(self.config["vocab_size"], np.float32) if want_logits else None
        check(lib().q3_decode_greedy(self._h, int(first_token), pos0, n_steps, toks.ctypes.data,
                                     _ptr(logits)))
        return toks[:n_steps], logits

    def decode_forced(self, tokens, pos0: int = 0, want_logits: bool = False):
        tokens = np.ascontiguousarray(tokens, np.int32)
        am = np.empty(max(tokens.size, 1), np.int32)
        logits = (np.empty((tokens.size, self.config["vocab_size"]), np.float32)
                  if want_logits else None)
        check(lib().q3_decode_forced(self._h, tokens, tokens.size, pos0, am.ctypes.data,
                                     _ptr(logits)))
        return am[:tokens.size], logits

    def generate(self, prompt_ids, max_new_tokens: int = 512, stop_on_eos: bool = True):
        """Generate (src/inference.cpp:639-700) on token IDs; returns (tokens, stats dict)."""
        p = np.ascontiguousarray(prompt_ids, np.int32)
        out = np.empty(max(max_new_tokens, 1), np.int32)
        n = C.c_size_t()
        st = GenStats()
        check(lib().q3_generate(self._h, _ptr(p) if p.size else None, p.size, max_new_tokens,
                                int(stop_on_eos), out.ctypes.data, C.byref(n), C.byref(st)))
        stats = {k: getattr(st, k) for k, _ in GenStats._fields_}
        return out[:n.value].copy(), stats


class Batch:
    """Independent sequences decoded together on the model's GPU (q3_batch_*)."""

    def __init__(self, model: "Qwen3", max_seqs: int, max_tokens: int):
        self._lib = lib()
        self.model = model  # the model must outlive the batch
        self.vocab = model.config["vocab_size"]
        self.kvd = model.config["n_kv_heads"] * model.config["head_dim"]
        h = C.c_void_p()
        check(self._lib.q3_batch_create(model._h, max_seqs, max_tokens, C.byref(h)))
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            self._lib.q3_batch_free(self._h)
            self._h = None

    def __del__(self):
        self.close()

    @property
    def size(self) -> int:
        n = C.c_int()
        check(self._lib.q3_batch_size(self._h, C.byref(n)))
        return n.value

    @property
    def stream(self) -> int:
        s = C.c_void_p()
        check(self._lib.q3_batch_stream(self._h, C.byref(s)))
        return s.value or 0

    def add(self, ids, want_logits: bool = False):
        """Adds a sequence (prefilling its prompt); returns (slot, next token, logits|None)."""
        ids = np.ascontiguousarray(ids, np.int32)
        slot = C.c_int()
        nxt = np.zeros(1, np.int32)
        lg = np.empty(self.vocab, np.float32) if want_logits else None
        check(self._lib.q3_batch_add(self._h, ids, ids.size, C.byref(slot), nxt.ctypes.data,
                                     _ptr(lg)))
        return slot.value, int(nxt[0]), lg

    def add_many(self, prompts, want_logits: bool = False):
        """Adds several sequences, prefilling their prompts together; returns (first slot, next
        tokens [n], logits [n, vocab] | None)."""
        lens = np.ascontiguousarray([len(p) for p in prompts], np.int32)
        ids = np.ascontiguousarray(np.concatenate([np.asarray(p, np.int32) for p in prompts]),
                                   np.int32)
        first = C.c_int()
        nxt = np.zeros(len(prompts), np.int32)
        lg = np.empty((len(prompts), self.vocab), np.float32) if want_logits else None
        check(self._lib.q3_batch_add_many(self._h, ids, lens, len(prompts), C.byref(first),
                                          nxt.ctypes.data, _ptr(lg)))
        return first.value, nxt, lg

    def decode(self, n_steps: int) -> np.ndarray:
        """n_steps greedy steps for every sequence: tokens [n_steps, n_seqs]."""
        out = np.empty((max(n_steps, 1), self.size), np.int32)
        check(self._lib.q3_batch_decode(self._h, n_steps, out.ctypes.data))
        return out[:n_steps]

    def decode_forced(self, tokens, want_logits: bool = False):
        """Teacher-forced steps on tokens [n_steps, n_seqs]: (argmax, logits|None)."""
        tokens = np.ascontiguousarray(tokens, np.int32)
        n = tokens.shape[0]
        am = np.empty(tokens.shape, np.int32)
        lg = np.empty(tokens.shape + (self.vocab,), np.float32) if want_logits else None
        check(self._lib.q3_batch_decode_forced(self._h, tokens, n, am.ctypes.data, _ptr(lg)))
        return am, lg

    def kv_row(self, slot: int, layer: int, pos: int):
        k = np.empty(self.kvd, np.uint16)
        v = np.empty(self.kvd, np.uint16)
        check(self._lib.q3_batch_kv_row(self._h, slot, layer, pos, k, v))
        return k, v


class TpDecoder:
    """Tensor-parallel decode (q3_tp_*): rank `rank` of `world`, on `model`'s GPU."""

    def __init__(self, model: "Qwen3", rank: int, world: int):
        self._lib = lib()
        self.model = model
        h = C.c_void_p()
        check(self._lib.q3_tp_create(model._h, rank, world, C.byref(h)))
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            self._lib.q3_tp_free(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def ipc_handle(self) -> bytes:
        buf = (C.c_uint8 * 64)()
        check(self._lib.q3_tp_ipc_handle(self._h, buf))
        return bytes(buf)

    def connect(self, handles) -> None:
        """handles: the 64-byte handles of every rank, in rank order."""
        blob = b"".join(handles)
        buf = (C.c_uint8 * len(blob)).from_buffer_copy(blob)
        check(self._lib.q3_tp_connect(self._h, buf))

    @property
    def stream(self) -> int:
        s = C.c_void_p()
        check(self._lib.q3_tp_stream(self._h, C.byref(s)))
        return s.value or 0

    def decode(self, first_token: int, pos0: int, n_steps: int) -> np.ndarray:
        out = np.empty(max(n_steps, 1), np.int32)
        check(self._lib.q3_tp_decode(self._h, int(first_token), pos0, n_steps, out.ctypes.data))
        return out[:n_steps]

    def decode_forced(self, tokens, pos0: int) -> np.ndarray:
        tokens = np.ascontiguousarray(tokens, np.int32)
        out = np.empty(max(tokens.size, 1), np.int32)
        check(self._lib.q3_tp_decode_forced(self._h, tokens, tokens.size, pos0, out.ctypes.data))
        return out[:tokens.size]

    def configure(self, solo_allreduce: bool = False, wait_cycles: int = 4_000_000_000) -> None:
        """solo_allreduce: at world 1, route the partials through the all-reduce kernel;
        wait_cycles: budget of each bounded flag wait (SM clock cycles)."""
        check(self._lib.q3_tp_configure(self._h, int(bool(solo_allreduce)), int(wait_cycles)))

    def reset(self) -> None:
        """Clears the state a timed-out step left (every rank resets before decoding again)."""
        check(self._lib.q3_tp_reset(self._h))

    FUSED, GRAPH, GRAPH_NCCL = 0, 1, 2  # Q3_TP_FUSED, Q3_TP_GRAPH, Q3_TP_GRAPH_NCCL

    @staticmethod
    def nccl_unique_id() -> bytes:
        """A new 128-byte NCCL unique id (one rank makes it; every rank connects with it)."""
        buf = (C.c_uint8 * 128)()
        check(lib().q3_tp_nccl_unique_id(buf))
        return bytes(buf)

    def nccl_connect(self, uid: bytes) -> None:
        """NCCL communicator for the GRAPH_NCCL comparison path."""
        buf = (C.c_uint8 * 128).from_buffer_copy(uid)
        check(self._lib.q3_tp_nccl_connect(self._h, buf))

    @property
    def path(self) -> int:
        v = C.c_int()
        check(self._lib.q3_tp_path(self._h, C.byref(v)))
        return v.value

    @path.setter
    def path(self, p: int) -> None:
        check(self._lib.q3_tp_set_path(self._h, int(p)))


class Block:
    """class Block (include/inference.h:178-202) on one GPU."""

    def __init__(self, cfg: dict, weights, device: int = 0):
        self.config = dict(cfg)
        self.weights = [np.ascontiguousarray(w, np.uint16) for w in weights]
        arr = (C.c_void_p * 11)(*[w.ctypes.data for w in self.weights])
        counts = (C.c_size_t * 11)(*[w.size for w in self.weights])
        c = Config.from_dict(cfg)
        h = C.c_void_p()
        self._lib = lib()
        check(self._lib.q3_block_create(C.byref(c), arr, counts, device, C.byref(h)))
        self._h = h
        self.kv_shape = (cfg["max_seq_len"], cfg["n_kv_heads"] * cfg["head_dim"])

    def close(self):
        if getattr(self, "_h", None):
            self._lib.q3_block_free(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def forward(self, x: np.ndarray, pos: int, num_sink: int, kv_pos: int, kv_len: int) -> None:
        """Block::forward, in place on the fp32 vector x."""
        if x.dtype != np.float32 or not x.flags.c_contiguous:
            raise TypeError("x must be a contiguous float32 array")
        check(lib().q3_block_forward(self._h, x, pos, num_sink, kv_pos, kv_len))

    def reset_cache(self):
        check(lib().q3_block_reset_cache(self._h))

    def get_cache(self):
        k = np.empty(self.kv_shape, np.uint16)
        v = np.empty(self.kv_shape, np.uint16)
        check(lib().q3_block_get_cache(self._h, k, v))
        return k, v

    def set_cache(self, k, v):
        check(lib().q3_block_set_cache(self._h, np.ascontiguousarray(k, np.uint16),
                                       np.ascontiguousarray(v, np.uint16)))


# ------------------------------------------------------------------ free kernels (device pointers)

def rmsnorm(out_ptr, x_ptr, w_ptr, eps, n, stream=None):
    check(lib().q3_rmsnorm(out_ptr, x_ptr, w_ptr, eps, n, stream))


def softmax(out_ptr, x_ptr, n, stream=None):
    check(lib().q3_softmax(out_ptr, x_ptr, n, stream))


def matmul(out_ptr, x_ptr, w_ptr, n, m, stream=None):
    check(lib().q3_matmul(out_ptr, x_ptr, w_ptr, n, m, stream))


def rope(x_ptr, d, head_dim, pos, theta, rotary_dim, stream=None):
    check(lib().q3_rope(x_ptr, d, head_dim, pos, theta, rotary_dim, stream))


def ffn(out_ptr, lin1_ptr, lin2_ptr, x_ptr, w1, w2, w3, hidden_dim, dim, stream=None):
    check(lib().q3_ffn(out_ptr, lin1_ptr, lin2_ptr, x_ptr, w1, w2, w3, hidden_dim, dim, stream))


def attn_workspace_size(head_dim: int, kv_len: int) -> int:
    return int(lib().q3_attn_workspace_size(head_dim, kv_len))


def attn(out_ptr, ws_ptr, q_ptr, k_ptr, v_ptr, head_dim, n_kv_heads, kv_len, stream=None):
    check(lib().q3_attn(out_ptr, ws_ptr, q_ptr, k_ptr, v_ptr, head_dim, n_kv_heads, kv_len,
                        stream))


def attn_noalloc(out_ptr, q_ptr, k_ptr, v_ptr, head_dim, n_kv_heads, kv_len, stream=None):
    """attn without a workspace: the scratch is a static device array inside the library, so the
    call allocates nothing (for callers that cannot allocate device memory). Calls that may
    overlap on the GPU share that array and must be ordered by the caller."""
    check(lib().q3_attn_noalloc(out_ptr, q_ptr, k_ptr, v_ptr, head_dim, n_kv_heads, kv_len,
                                stream))


def greedy(logits_ptr, n, out_ptr, stream=None):
    check(lib().q3_greedy(logits_ptr, n, out_ptr, stream))


GEMM_STORE_F32, GEMM_ADD_F32, GEMM_SWIGLU, GEMM_STORE_BF16 = 0, 1, 2, 3


def gemm_bf16(out: int, a: int, w: int, w3, M: int, N: int, K: int, epilogue: int, stream=None):
    """q3_gemm_bf16 on device pointers: out[M, N] = epilogue(A[M, K] . W[N, K]^T)."""
    check(lib().q3_gemm_bf16(out, a, w, w3, M, N, K, epilogue, stream))


def gemm_f16(out: int, a: int, w: int, w3, M: int, N: int, K: int, epilogue: int, stream=None):
    """q3_gemm_f16: as gemm_bf16 with fp16 operands (and fp16 SwiGLU / 16-bit stores)."""
    check(lib().q3_gemm_f16(out, a, w, w3, M, N, K, epilogue, stream))
