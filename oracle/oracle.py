"""Test infrastructure only: Python access to the two CPU oracles.

* ``PortModel`` / ``PortBlock`` / ``port_ops`` - the plain-C restatement (q3_oracle.c, built into
  oracle/_build/libq3oracle.so; needs only gcc, so it can be built wherever the tests run).
* ``RefModel`` / ``RefBlock`` / ``ref_ops`` - the unmodified reference engine compiled from its
  sources (oracle/_ref/libq3ref.so, built by oracle/Makefile where the reference tree exists; the
  prebuilt library travels with the repository snapshot).

Only tests/, the smoke check and bench.py's CPU-baseline leg import this module.

``read_qwen3_bin`` restates the reference loader (src/inference.cpp:445-481, helpers :20-263):
magic, version, metadata JSON parsed with the reference's naive ``"key":`` lookup, tensor
records with their byte-size and dtype checks.
"""
from __future__ import annotations

import ctypes as C
import json
import os
import struct
import subprocess
import threading
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PORT_LIB = HERE / "_build" / "libq3oracle.so"
REF_LIB = HERE / "_ref" / "libq3ref.so"
# The same sources built with the reference's -march=native resolved for the GPU hosts' CPU
# (-march=sapphirerapids); used for CPU timing where this host's CPU has those instructions.
REF_NATIVE_LIB = HERE / "_ref" / "libq3ref_spr.so"
NATIVE_FLAGS = ("avx512f", "avx512bw", "avx512vl", "avx512dq", "avx512cd", "avx512ifma",
                "avx512vbmi", "avx512_vbmi2", "avx512_vnni", "avx512_bitalg", "avx512_vpopcntdq",
                "avx512_bf16", "avx512_fp16", "avx_vnni", "amx_tile", "amx_bf16", "amx_int8")


def host_runs_native_build() -> bool:
    """True when this host's CPU has the instruction sets -march=sapphirerapids may use."""
    try:
        text = Path("/proc/cpuinfo").read_text()
    except OSError:
        return False
    flags = set()
    for line in text.splitlines():
        if line.startswith("flags"):
            flags = set(line.split(":", 1)[1].split())
            break
    return all(f in flags for f in NATIVE_FLAGS)
# The reference source tree (asriva32/Qwen3.cpp), when this machine has one: Q3_REFERENCE_TREE.
REFERENCE_TREE = (Path(os.environ["Q3_REFERENCE_TREE"]) if os.environ.get("Q3_REFERENCE_TREE")
                  else None)

_lock = threading.Lock()

# ------------------------------------------------------------------ Qwen3.bin reader

MAGIC = b"QWEN3CP\0"
DTYPE_SIZES = {1: 4, 3: 2, 4: 1, 5: 4}  # include/inference.h:23-28 (2 = f16 is rejected)
CONFIG_KEYS_STR = ("arch", "dtype", "act_type")
CONFIG_KEYS_INT = ("dim", "hidden_dim", "head_dim", "n_layers", "n_heads", "n_kv_heads",
                   "vocab_size", "max_seq_len", "bos_token_id", "eos_token_id", "rotary_dim")
CONFIG_KEYS_FLOAT = ("rope_theta", "norm_eps")
CONFIG_KEYS_BOOL = ("tie_word_embeddings", "attention_bias", "qk_norm")


class ModelFileError(RuntimeError):
    """std::runtime_error from the reference loader."""


def _json_value(js: str, key: str) -> str:
    # JsonValue, src/inference.cpp:97-124
    qk = '"' + key + '":'
    p = js.find(qk)
    if p < 0:
        raise ModelFileError("Missing metadata key: " + key)
    p += len(qk)
    while p < len(js) and js[p] == " ":
        p += 1
    if p >= len(js):
        raise ModelFileError("Malformed metadata value for: " + key)
    if js[p] == '"':
        e = js.find('"', p + 1)
        if e < 0:
            raise ModelFileError("Unterminated string metadata value for: " + key)
        return js[p + 1:e]
    e = min([i for i in (js.find(",", p), js.find("}", p)) if i >= 0], default=-1)
    if e < 0:
        raise ModelFileError("Unterminated metadata value for: " + key)
    return js[p:e]


def parse_config(js: str) -> dict:
    # ParseConfig + ValidateConfig, src/inference.cpp:145-182
    c: dict = {}
    for k in CONFIG_KEYS_STR:
        c[k] = _json_value(js, k)
    for k in CONFIG_KEYS_INT:
        c[k] = int(_json_value(js, k))
    for k in CONFIG_KEYS_FLOAT:
        c[k] = float(np.float32(float(_json_value(js, k))))
    for k in CONFIG_KEYS_BOOL:
        v = _json_value(js, k)
        if v not in ("true", "false"):
            raise ModelFileError("Metadata value is not bool for: " + k)
        c[k] = v == "true"
    if min(c["dim"], c["hidden_dim"], c["head_dim"], c["n_heads"], c["n_kv_heads"],
           c["max_seq_len"]) <= 0:
        raise ValueError("Block config dimensions must be positive")
    if c["n_heads"] % c["n_kv_heads"]:
        raise ValueError("Attention head count must be divisible by KV head count")
    if c["rotary_dim"] < 0 or c["rotary_dim"] > c["head_dim"] or c["rotary_dim"] % 2:
        raise ValueError("rotary_dim must be even and no larger than head_dim")
    return c


@dataclass
class TensorRecord:
    name: str
    dtype: int
    shape: tuple
    data_offset: int
    byte_size: int


def read_qwen3_bin(path) -> tuple[dict, dict[str, TensorRecord]]:
    """Header and tensor index of a Qwen3.bin (the constructor, src/inference.cpp:445-481)."""
    with open(path, "rb") as f:
        if f.read(8) != MAGIC:
            raise ModelFileError("Invalid Qwen3 model file magic")
        (version,) = struct.unpack("<I", f.read(4))
        if version != 1:
            raise ModelFileError("Unsupported Qwen3 model file version")
        (mlen,) = struct.unpack("<Q", f.read(8))
        cfg = parse_config(f.read(mlen).decode())
        if cfg["dtype"] != "bf16":
            raise ModelFileError("Only bf16 Qwen3.bin files are supported")
        (count,) = struct.unpack("<Q", f.read(8))
        recs: dict[str, TensorRecord] = {}
        for _ in range(count):
            (nl,) = struct.unpack("<I", f.read(4))
            name = f.read(nl).decode()
            dtype, ndim = struct.unpack("<II", f.read(8))
            shape = struct.unpack("<%dQ" % ndim, f.read(8 * ndim)) if ndim else ()
            (nbytes,) = struct.unpack("<Q", f.read(8))
            off = f.tell()
            if dtype not in DTYPE_SIZES:
                raise ModelFileError("Unknown tensor dtype")
            if int(np.prod(shape, dtype=np.int64)) * DTYPE_SIZES[dtype] != nbytes:
                raise ModelFileError("Tensor byte size mismatch for " + name)
            tok = name in ("tokenizer.json", "tokenizer.tokens", "tokenizer.offsets")
            if tok:
                ok = (dtype == 4 and name != "tokenizer.offsets") or (
                    dtype == 5 and name == "tokenizer.offsets")
                if not ok:
                    raise ModelFileError("Unsupported tokenizer tensor dtype for " + name)
            elif dtype != 3:
                raise ModelFileError("Only bf16 model tensors are supported: " + name)
            if name in recs:
                raise ModelFileError("Duplicate tensor record: " + name)
            recs[name] = TensorRecord(name, dtype, tuple(shape), off, nbytes)
            f.seek(nbytes, os.SEEK_CUR)
    return cfg, recs


class WeightFile:
    """Memory-mapped bf16 tensors of a Qwen3.bin."""

    def __init__(self, path):
        self.path = str(path)
        self.config, self.records = read_qwen3_bin(path)
        self._mm = np.memmap(self.path, dtype=np.uint8, mode="r")

    def tensor(self, name: str) -> np.ndarray:
        r = self.records[name]
        raw = self._mm[r.data_offset:r.data_offset + r.byte_size]
        return raw.view(np.uint16).reshape(r.shape)

    def layer(self, l: int) -> list[np.ndarray]:
        p = f"model.layers.{l}."
        return [self.tensor(p + s) for s in (
            "attn.norm.weight", "attn.q_norm.weight", "attn.k_norm.weight", "attn.wq.weight",
            "attn.wk.weight", "attn.wv.weight", "attn.wo.weight", "mlp.norm.weight",
            "mlp.w1.weight", "mlp.w2.weight", "mlp.w3.weight")]


# ------------------------------------------------------------------ library loading

def build_port() -> Path:
    with _lock:
        src = HERE / "q3_oracle.c"
        if not PORT_LIB.exists() or PORT_LIB.stat().st_mtime < src.stat().st_mtime:
            subprocess.run(["make", "-s", "-C", str(HERE), "_build/libq3oracle.so"], check=True)
    return PORT_LIB


def build_ref() -> Path | None:
    """Build oracle/_ref from the reference tree when it exists; else use a prebuilt copy."""
    with _lock:
        if REFERENCE_TREE is not None and REFERENCE_TREE.exists():
            subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REF={REFERENCE_TREE}"],
                           check=True)
    return REF_LIB if REF_LIB.exists() else None


def ref_available() -> bool:
    return REF_LIB.exists() or (REFERENCE_TREE is not None and REFERENCE_TREE.exists())


_port = None
_ref = {}
F32P = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
U16P = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")


class Q3OCfg(C.Structure):
    _fields_ = [("dim", C.c_int), ("hidden_dim", C.c_int), ("head_dim", C.c_int),
                ("n_heads", C.c_int), ("n_kv_heads", C.c_int), ("max_seq_len", C.c_int),
                ("rotary_dim", C.c_int), ("rope_theta", C.c_float), ("norm_eps", C.c_float)]


def port_lib():
    global _port
    if _port is None:
        lib = C.CDLL(str(build_port()))
        lib.q3o_block_create.restype = C.c_void_p
        lib.q3o_block_create.argtypes = [C.POINTER(Q3OCfg), C.POINTER(C.c_void_p)]
        lib.q3o_block_free.argtypes = [C.c_void_p]
        lib.q3o_block_reset.argtypes = [C.c_void_p]
        lib.q3o_block_forward.argtypes = [C.c_void_p, F32P, C.c_int, C.c_int, C.c_int, C.c_int]
        lib.q3o_block_k_cache.restype = C.c_void_p
        lib.q3o_block_k_cache.argtypes = [C.c_void_p]
        lib.q3o_block_v_cache.restype = C.c_void_p
        lib.q3o_block_v_cache.argtypes = [C.c_void_p]
        lib.q3o_model_create.restype = C.c_void_p
        lib.q3o_model_create.argtypes = [C.POINTER(Q3OCfg), C.c_int, C.c_int, C.c_void_p,
                                         C.c_void_p, C.POINTER(C.c_void_p)]
        lib.q3o_model_free.argtypes = [C.c_void_p]
        lib.q3o_model_reset.argtypes = [C.c_void_p]
        lib.q3o_model_forward.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
        lib.q3o_model_kv_row.argtypes = [C.c_void_p, C.c_int, C.c_int, U16P, U16P]
        lib.q3o_model_prefill.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                                          C.c_void_p, C.c_void_p, C.c_void_p]
        lib.q3o_rmsnorm.argtypes = [F32P, F32P, U16P, C.c_float, C.c_int]
        lib.q3o_softmax.argtypes = [F32P, F32P, C.c_int]
        lib.q3o_silu.restype = C.c_float
        lib.q3o_silu.argtypes = [C.c_float]
        lib.q3o_matmul.argtypes = [F32P, F32P, U16P, C.c_int, C.c_int]
        lib.q3o_rope.argtypes = [F32P, C.c_int, C.c_int, C.c_int, C.c_float, C.c_int]
        lib.q3o_ffn.argtypes = [F32P, F32P, F32P, F32P, U16P, U16P, U16P, C.c_int, C.c_int]
        lib.q3o_attn.argtypes = [F32P, F32P, F32P, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                 C.c_int]
        lib.q3o_greedy.argtypes = [F32P, C.c_int]
        lib.q3o_positions.argtypes = [C.c_int, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int),
                                      C.POINTER(C.c_int)]
        _port = lib
    return _port


def ref_lib(native: bool = False):
    """The reference engine library; native=True: its -march=native build for the GPU hosts'
    CPU (callers check host_runs_native_build() first)."""
    if native not in _ref:
        path = build_ref()
        if native:
            path = REF_NATIVE_LIB if REF_NATIVE_LIB.exists() else None
        if path is None:
            raise FileNotFoundError("oracle/_ref/libq3ref.so is not built")
        lib = C.CDLL(str(path))
        lib.q3ref_last_error.restype = C.c_char_p
        lib.q3ref_load.argtypes = [C.c_char_p, C.c_int, C.POINTER(C.c_void_p)]
        lib.q3ref_free.argtypes = [C.c_void_p]
        lib.q3ref_config.argtypes = [C.c_void_p, C.POINTER(C.c_int), C.POINTER(C.c_float)]
        lib.q3ref_tensor_count.argtypes = [C.c_void_p]
        lib.q3ref_reset.argtypes = [C.c_void_p]
        lib.q3ref_forward_token.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        lib.q3ref_forward_layers.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                                             C.c_void_p]
        lib.q3ref_kv_row.argtypes = [C.c_void_p, C.c_int, C.c_int, U16P, U16P]
        lib.q3ref_generate_ids.argtypes = [C.c_void_p, C.POINTER(C.c_int), C.c_int, C.c_int,
                                           C.POINTER(C.c_int), C.POINTER(C.c_double),
                                           C.POINTER(C.c_double)]
        lib.q3ref_block_create.argtypes = [C.POINTER(C.c_int), C.POINTER(C.c_float),
                                           C.POINTER(C.c_void_p), C.POINTER(C.c_void_p)]
        lib.q3ref_block_free.argtypes = [C.c_void_p]
        lib.q3ref_block_forward.argtypes = [C.c_void_p, F32P, C.c_int, C.c_int, C.c_int, C.c_int]
        lib.q3ref_block_reset.argtypes = [C.c_void_p]
        lib.q3ref_block_set_cache.argtypes = [C.c_void_p, U16P, U16P]
        lib.q3ref_block_get_cache.argtypes = [C.c_void_p, U16P, U16P]
        lib.q3ref_rmsnorm.argtypes = [F32P, F32P, U16P, C.c_float, C.c_int]
        lib.q3ref_softmax.argtypes = [F32P, F32P, C.c_int]
        lib.q3ref_silu.restype = C.c_float
        lib.q3ref_silu.argtypes = [C.c_float]
        lib.q3ref_matmul.argtypes = [F32P, F32P, U16P, C.c_int, C.c_int]
        lib.q3ref_rope.argtypes = [F32P, C.c_int, C.c_int, C.c_int, C.c_float, C.c_int]
        lib.q3ref_ffn.argtypes = [F32P, F32P, F32P, F32P, U16P, U16P, U16P, C.c_int, C.c_int]
        lib.q3ref_fastattn.argtypes = [F32P, F32P, F32P, C.c_void_p, C.c_void_p, C.c_int,
                                       C.c_int, C.c_int]
        lib.q3ref_greedy.argtypes = [F32P, C.c_int, C.POINTER(C.c_int)]
        _ref[native] = lib
    return _ref[native]


class OracleError(Exception):
    def __init__(self, code: int, msg: str = ""):
        super().__init__(f"oracle status {code}: {msg}")
        self.code = code


def _check_ref(st: int):
    if st:
        raise OracleError(st, ref_lib().q3ref_last_error().decode())


def _check_port(st: int):
    if st:
        raise OracleError(st, {2: "invalid_argument", 3: "out_of_range"}.get(st, "error"))


def positions(pos: int, ctx: int) -> tuple[int, int, int]:
    """(num_sink, kv_pos, kv_len) of src/inference.cpp:605-613, from the C restatement."""
    a, b, c = C.c_int(), C.c_int(), C.c_int()
    port_lib().q3o_positions(pos, ctx, C.byref(a), C.byref(b), C.byref(c))
    return a.value, b.value, c.value


# ------------------------------------------------------------------ models

def _block_cfg(cfg: dict) -> Q3OCfg:
    return Q3OCfg(cfg["dim"], cfg["hidden_dim"], cfg["head_dim"], cfg["n_heads"],
                  cfg["n_kv_heads"], cfg["max_seq_len"], cfg["rotary_dim"],
                  cfg["rope_theta"], cfg["norm_eps"])


class PortModel:
    """The C restatement of Qwen3 (ForwardToken and the per-layer hidden states)."""

    kind = "port"

    def __init__(self, path, ctx: int = 512):
        self.wf = WeightFile(path)
        cfg = dict(self.wf.config)
        if ctx <= 0 or ctx > cfg["max_seq_len"]:
            raise ValueError("Context length is outside the model's supported range")
        cfg["max_seq_len"] = ctx
        self.config = cfg
        lib = port_lib()
        self._keep = [self.wf.tensor("model.embed.weight"), self.wf.tensor("model.norm.weight")]
        ptrs = []
        for l in range(cfg["n_layers"]):
            for t in self.wf.layer(l):
                self._keep.append(t)
                ptrs.append(t.ctypes.data)
        arr = (C.c_void_p * len(ptrs))(*ptrs)
        c = _block_cfg(cfg)
        self._h = lib.q3o_model_create(C.byref(c), cfg["n_layers"], cfg["vocab_size"],
                                       self._keep[0].ctypes.data, self._keep[1].ctypes.data, arr)

    def __del__(self):
        if getattr(self, "_h", None):
            port_lib().q3o_model_free(self._h)
            self._h = None

    def reset(self):
        port_lib().q3o_model_reset(self._h)

    def forward(self, token: int, pos: int, layers: bool = False):
        c = self.config
        logits = np.empty(c["vocab_size"], np.float32)
        hid = np.empty((c["n_layers"] + 1, c["dim"]), np.float32) if layers else None
        _check_port(port_lib().q3o_model_forward(
            self._h, token, pos, hid.ctypes.data if layers else None, logits.ctypes.data))
        return (hid, logits) if layers else logits

    def kv_row(self, layer: int, kv_pos: int):
        kvd = self.config["n_kv_heads"] * self.config["head_dim"]
        k = np.empty(kvd, np.uint16)
        v = np.empty(kvd, np.uint16)
        _check_port(port_lib().q3o_model_kv_row(self._h, layer, kv_pos, k, v))
        return k, v

    def forward_many(self, tokens, pos0: int = 0, want=None, logits: bool = False,
                     layers: bool = False):
        """ForwardToken over tokens at positions pos0.. (no ring wrap), computed layer by layer
        over all tokens; bit-identical to calling forward() per token. want: boolean mask of the
        tokens whose logits are computed (default all). Returns a dict with 'argmax' ([n], -1
        where not wanted), 'logits' ([wanted, vocab], when logits) and 'hidden_last'
        ([(n_layers + 1), dim] of the last token, when layers)."""
        c = self.config
        toks = np.ascontiguousarray(tokens, np.int32)
        n = toks.size
        mask = (np.ones(n, np.uint8) if want is None
                else np.ascontiguousarray(np.asarray(want, bool), np.uint8))
        am = np.empty(n, np.int32)
        lg = np.empty((int(mask.sum()), c["vocab_size"]), np.float32) if logits else None
        hid = np.empty((c["n_layers"] + 1, c["dim"]), np.float32) if layers else None
        _check_port(port_lib().q3o_model_prefill(
            self._h, toks.ctypes.data, n, int(pos0), mask.ctypes.data,
            lg.ctypes.data if logits else None, am.ctypes.data,
            hid.ctypes.data if layers else None))
        out = {"argmax": am}
        if logits:
            out["logits"] = lg
        if layers:
            out["hidden_last"] = hid
        return out


class RefModel:
    """The reference engine itself (Qwen3::ForwardToken, or its per-layer restatement from
    public pieces for hidden states and KV rows)."""

    kind = "reference"

    def __init__(self, path, ctx: int = 512, native: bool = False):
        lib = self._lib = ref_lib(native)
        h = C.c_void_p()
        _check_ref(lib.q3ref_load(str(path).encode(), ctx, C.byref(h)))
        self._h = h
        ints = (C.c_int * 14)()
        fl = (C.c_float * 2)()
        _check_ref(lib.q3ref_config(h, ints, fl))
        keys = ("dim", "hidden_dim", "head_dim", "n_layers", "n_heads", "n_kv_heads",
                "vocab_size", "max_seq_len", "bos_token_id", "eos_token_id", "rotary_dim",
                "tie_word_embeddings", "qk_norm", "attention_bias")
        self.config = {k: int(v) for k, v in zip(keys, ints)}
        self.config["rope_theta"], self.config["norm_eps"] = float(fl[0]), float(fl[1])
        self._layered = False

    def __del__(self):
        if getattr(self, "_h", None):
            self._lib.q3ref_free(self._h)
            self._h = None

    def tensor_count(self) -> int:
        return self._lib.q3ref_tensor_count(self._h)

    def reset(self):
        _check_ref(self._lib.q3ref_reset(self._h))

    def forward(self, token: int, pos: int, layers: bool = False):
        c = self.config
        logits = np.empty(c["vocab_size"], np.float32)
        if layers:
            hid = np.empty((c["n_layers"] + 1, c["dim"]), np.float32)
            _check_ref(self._lib.q3ref_forward_layers(self._h, token, pos, hid.ctypes.data,
                                                      logits.ctypes.data))
            return hid, logits
        _check_ref(self._lib.q3ref_forward_token(self._h, token, pos, logits.ctypes.data))
        return logits

    def forward_layers(self, token: int, pos: int):
        return self.forward(token, pos, layers=True)

    def kv_row(self, layer: int, kv_pos: int):
        kvd = self.config["n_kv_heads"] * self.config["head_dim"]
        k = np.empty(kvd, np.uint16)
        v = np.empty(kvd, np.uint16)
        _check_ref(self._lib.q3ref_kv_row(self._h, layer, kv_pos, k, v))
        return k, v

    def generate_ids(self, prompt, steps: int):
        p = (C.c_int * len(prompt))(*[int(t) for t in prompt])
        out = (C.c_int * max(steps, 1))()
        ps, ds = C.c_double(), C.c_double()
        _check_ref(self._lib.q3ref_generate_ids(self._h, p, len(prompt), steps, out,
                                                C.byref(ps), C.byref(ds)))
        return list(out)[:steps], ps.value, ds.value


# ------------------------------------------------------------------ blocks

class _BlockBase:
    def __init__(self, cfg: dict, weights: list[np.ndarray]):
        self.config = dict(cfg)
        self.weights = [np.ascontiguousarray(w, dtype=np.uint16) for w in weights]
        self.kv_shape = (cfg["max_seq_len"], cfg["n_kv_heads"] * cfg["head_dim"])


class PortBlock(_BlockBase):
    kind = "port"

    def __init__(self, cfg, weights):
        super().__init__(cfg, weights)
        arr = (C.c_void_p * 11)(*[w.ctypes.data for w in self.weights])
        c = _block_cfg(cfg)
        self._h = port_lib().q3o_block_create(C.byref(c), arr)

    def __del__(self):
        if getattr(self, "_h", None):
            port_lib().q3o_block_free(self._h)
            self._h = None

    def forward(self, x: np.ndarray, pos, num_sink, kv_pos, kv_len):
        _check_port(port_lib().q3o_block_forward(self._h, x, pos, num_sink, kv_pos, kv_len))

    def reset(self):
        port_lib().q3o_block_reset(self._h)

    def _cache(self):
        n = self.kv_shape[0] * self.kv_shape[1]
        k = np.ctypeslib.as_array(C.cast(port_lib().q3o_block_k_cache(self._h),
                                         C.POINTER(C.c_uint16)), (n,))
        v = np.ctypeslib.as_array(C.cast(port_lib().q3o_block_v_cache(self._h),
                                         C.POINTER(C.c_uint16)), (n,))
        return k.reshape(self.kv_shape), v.reshape(self.kv_shape)

    def set_cache(self, k, v):
        ck, cv = self._cache()
        ck[...] = k
        cv[...] = v

    def get_cache(self):
        ck, cv = self._cache()
        return ck.copy(), cv.copy()


class RefBlock(_BlockBase):
    kind = "reference"

    def __init__(self, cfg, weights):
        super().__init__(cfg, weights)
        ints = (C.c_int * 7)(cfg["dim"], cfg["hidden_dim"], cfg["head_dim"], cfg["n_heads"],
                             cfg["n_kv_heads"], cfg["max_seq_len"], cfg["rotary_dim"])
        fl = (C.c_float * 2)(cfg["rope_theta"], cfg["norm_eps"])
        arr = (C.c_void_p * 11)(*[w.ctypes.data for w in self.weights])
        h = C.c_void_p()
        _check_ref(ref_lib().q3ref_block_create(ints, fl, arr, C.byref(h)))
        self._h = h

    def __del__(self):
        if getattr(self, "_h", None):
            ref_lib().q3ref_block_free(self._h)
            self._h = None

    def forward(self, x: np.ndarray, pos, num_sink, kv_pos, kv_len):
        _check_ref(ref_lib().q3ref_block_forward(self._h, x, pos, num_sink, kv_pos, kv_len))

    def reset(self):
        _check_ref(ref_lib().q3ref_block_reset(self._h))

    def set_cache(self, k, v):
        _check_ref(ref_lib().q3ref_block_set_cache(
            self._h, np.ascontiguousarray(k, np.uint16), np.ascontiguousarray(v, np.uint16)))

    def get_cache(self):
        k = np.empty(self.kv_shape, np.uint16)
        v = np.empty(self.kv_shape, np.uint16)
        _check_ref(ref_lib().q3ref_block_get_cache(self._h, k, v))
        return k, v


# ------------------------------------------------------------------ free functions

class _Ops:
    """The free functions of include/inference.h:308-315 plus Sampler::Greedy."""

    def __init__(self, kind: str):
        self.kind = kind

    @property
    def lib(self):
        return port_lib() if self.kind == "port" else ref_lib()

    def _f(self, name):
        return getattr(self.lib, ("q3o_" if self.kind == "port" else "q3ref_") + name)

    def rmsnorm(self, x, w, eps):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        self._f("rmsnorm")(out, x, np.ascontiguousarray(w, np.uint16), eps, x.size)
        return out

    def softmax(self, x):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        self._f("softmax")(out, x, x.size)
        return out

    def silu(self, x: float) -> float:
        return float(self._f("silu")(x))

    def matmul(self, x, w):
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.uint16)
        out = np.empty(w.shape[0], np.float32)
        self._f("matmul")(out, x, w, w.shape[0], w.shape[1])
        return out

    def rope(self, x, head_dim, pos, theta, rotary_dim):
        out = np.array(x, dtype=np.float32, copy=True)
        self._f("rope")(out, out.size, head_dim, pos, theta, rotary_dim)
        return out

    def ffn(self, x, w1, w2, w3):
        x = np.ascontiguousarray(x, np.float32)
        hidden, dim = w1.shape
        out = np.empty(dim, np.float32)
        l1 = np.empty(hidden, np.float32)
        l2 = np.empty(hidden, np.float32)
        self._f("ffn")(out, l1, l2, x, np.ascontiguousarray(w1, np.uint16),
                       np.ascontiguousarray(w2, np.uint16), np.ascontiguousarray(w3, np.uint16),
                       hidden, dim)
        return out

    def attn(self, q, k, v, head_dim, n_kv_heads, kv_len, head_offset=0):
        """FastAttn for one query head; k/v are [kv_len, n_kv_heads*head_dim] bf16 caches and
        head_offset selects the KV head's first column."""
        q = np.ascontiguousarray(q, np.float32)
        k = np.ascontiguousarray(k, np.uint16)
        v = np.ascontiguousarray(v, np.uint16)
        out = np.empty(head_dim, np.float32)
        scores = np.empty(max(kv_len, 1), np.float32)
        self._f("fastattn" if self.kind != "port" else "attn")(
            out, scores, q, k.ctypes.data + 2 * head_offset, v.ctypes.data + 2 * head_offset,
            head_dim, n_kv_heads, kv_len)
        return out

    def greedy(self, logits) -> int:
        logits = np.ascontiguousarray(logits, np.float32)
        if self.kind == "port":
            if logits.size == 0:
                raise ValueError("Cannot sample empty logits")
            return int(self.lib.q3o_greedy(logits, logits.size))
        out = C.c_int()
        _check_ref(self.lib.q3ref_greedy(logits, logits.size, C.byref(out)))
        return out.value


port_ops = _Ops("port")
ref_ops = _Ops("reference")
