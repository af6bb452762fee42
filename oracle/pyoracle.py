"""ctypes binding of the CPU oracle (liboracle.so) — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import
this module; the product library never does. Builds liboracle.so on first use
when a compiler is present (make -C oracle).
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"


def build() -> Path:
    srcs = [HERE / "oracle.cpp", HERE / "oracle.h", HERE / "Makefile"]
    if not LIB.exists() or LIB.stat().st_mtime < max(s.stat().st_mtime for s in srcs):
        subprocess.run(["make", "-C", str(HERE), "-s"], check=True)
    return LIB


class OrcShape(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("dim", "hidden_dim", "n_heads", "head_size", "n_kv_heads", "vocab_size",
                                          "n_layers", "ctx_len")] + [
        ("rms_norm_eps", C.c_float), ("rope_theta", C.c_float), ("group_size", C.c_uint32),
        ("rope_freq_scale", C.c_float), ("rope_ext_factor", C.c_float), ("rope_attn_factor", C.c_float),
        ("rope_original_ctx_len", C.c_uint32), ("attention_scale", C.c_float), ("weight_format", C.c_int32),
        ("rope_mode", C.c_int32), ("llama3_old_ctx", C.c_float), ("q4_mode", C.c_int32),
        ("untied_lm_head", C.c_int32), ("bos", C.c_uint32), ("eos", C.c_uint32)]


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(str(LIB))
        P = C.c_void_p
        sig = {
            "orc_set_threads": (None, [C.c_int]),
            "orc_get_threads": (C.c_int, []),
            "orc_set_probe": (None, [C.c_int]),
            "orc_quantize_q8": (None, [P, P, P, C.c_size_t, C.c_uint32]),
            "orc_quantize_q4_ref": (None, [P, P, P, C.c_size_t, C.c_uint32]),
            "orc_matmul_q8_slices": (None, [P, C.c_size_t, P, P, P, P, C.c_size_t, C.c_size_t, C.c_size_t]),
            "orc_matmul_f32": (None, [P, C.c_size_t, P, P, C.c_size_t, C.c_size_t]),
            "orc_block_dots": (None, [P, P, P, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t]),
            "orc_rmsnorm": (None, [P, P, P, C.c_size_t, C.c_float, C.c_int]),
            "orc_rms_norm_scalar": (None, [P, C.c_size_t, P, C.c_float, C.c_int]),
            "orc_silu": (None, [P, C.c_size_t]),
            "orc_rope": (None, [C.POINTER(OrcShape), P, P, C.c_uint32]),
            "orc_rope_gguf": (None, [C.POINTER(OrcShape), P, P, C.c_uint32]),
            "orc_fused_attention": (None, [P, P, P, P, P, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t,
                                           C.c_size_t, C.c_uint32, C.c_size_t, C.c_float]),
            "orc_argmax": (C.c_uint32, [P, C.c_size_t]),
            "orc_f16_to_f32": (C.c_float, [C.c_uint16]),
            "orc_model_load": (P, [C.c_char_p, C.c_uint32, C.c_int, C.c_int]),
            "orc_model_free": (None, [P]),
            "orc_last_error": (C.c_char_p, []),
            "orc_model_shape": (C.c_int, [P, C.POINTER(OrcShape)]),
            "orc_get_embeddings": (C.c_int, [P, C.c_uint32, P]),
            "orc_session_new": (P, [P]),
            "orc_session_free": (None, [P]),
            "orc_session_reset": (None, [P]),
            "orc_session_key_cache": (P, [P]),
            "orc_session_value_cache": (P, [P]),
            "orc_session_cache_len": (C.c_size_t, [P]),
            "orc_forward_x": (C.c_int, [P, P, P, C.c_size_t, C.c_uint32, P]),
        }
        for k, (r, a) in sig.items():
            f = getattr(L, k)
            f.restype = r
            f.argtypes = a
        _lib = L
    return _lib


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


def set_threads(n: int) -> None:
    lib().orc_set_threads(n)


def set_probe(flags: int) -> None:
    """0 = faithful restatement; 1 = rmsnorm sum of squares in f64 (a 1-ulp
    perturbation used to measure a test model's sensitivity)."""
    lib().orc_set_probe(flags)


def quantize_q8(x: np.ndarray, gs: int = 32):
    x = np.ascontiguousarray(x, np.float32)
    q = np.zeros(x.size, np.int8)
    s = np.zeros(x.size // gs, np.float32)
    lib().orc_quantize_q8(_p(q), _p(s), _p(x), x.size, gs)
    return q, s


def quantize_q4_ref(x: np.ndarray, gs: int = 32):
    x = np.ascontiguousarray(x, np.float32)
    q = np.zeros(x.size, np.int8)
    s = np.zeros(x.size // gs, np.float32)
    lib().orc_quantize_q4_ref(_p(q), _p(s), _p(x), x.size, gs)
    return q, s


def matmul_q8(out: np.ndarray, xq, xs, wq, ws, n: int, o: int, gs: int = 32) -> np.ndarray:
    """In-place like the reference (quad columns accumulate into `out`)."""
    arrs = [np.ascontiguousarray(a) for a in (xq, xs, wq, ws)]
    assert out.dtype == np.float32 and out.flags.c_contiguous
    lib().orc_matmul_q8_slices(_p(out), out.size, *map(_p, arrs), n, o, gs)
    return out


def matmul_f32(out: np.ndarray, x, w, n: int, o: int) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    lib().orc_matmul_f32(_p(out), out.size, _p(x), _p(w), n, o)
    return out


def block_dots(xq, wq, batch: int, n: int, o: int, gs: int = 32) -> np.ndarray:
    xq = np.ascontiguousarray(xq, np.int8)
    wq = np.ascontiguousarray(wq, np.int8)
    out = np.zeros((batch, o, n // gs), np.int32)
    lib().orc_block_dots(_p(out), _p(xq), _p(wq), batch, n, o, gs)
    return out


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    o = np.zeros_like(x)
    lib().orc_rmsnorm(_p(o), _p(x), _p(w), x.size, eps, 0)
    return o


def rms_norm_scalar(x: np.ndarray, w: np.ndarray, eps: float, add_unit_offset: bool = False) -> np.ndarray:
    x = np.array(x, np.float32, copy=True)
    w = np.ascontiguousarray(w, np.float32)
    lib().orc_rms_norm_scalar(_p(x), x.size, _p(w), eps, 1 if add_unit_offset else 0)
    return x


def silu(x: np.ndarray) -> np.ndarray:
    x = np.array(x, np.float32, copy=True)
    lib().orc_silu(_p(x), x.size)
    return x


def fused_attention(sq, key_cache, value_cache, seq_len: int, batch: int, n_heads: int, n_kv_heads: int,
                    head_size: int, start_pos: int, kv_dim: int, attn_scale: float) -> np.ndarray:
    sq = np.ascontiguousarray(sq, np.float32)
    kc = np.ascontiguousarray(key_cache, np.float32)
    vc = np.ascontiguousarray(value_cache, np.float32)
    out = np.zeros(batch * n_heads * head_size, np.float32)
    scores = np.zeros(n_heads * batch * seq_len, np.float32)
    lib().orc_fused_attention(_p(out), _p(scores), _p(sq), _p(kc), _p(vc), seq_len, batch, n_heads, n_kv_heads,
                              head_size, start_pos, kv_dim, attn_scale)
    return out


def rope(shape: "OrcShape", sq: np.ndarray, k: np.ndarray, pos: int):
    """The model's RoPE of one token's q [heads*hd] and k [kv_heads*hd] at
    `pos` (util.rs:589-635 `rope` for llama3 scaling, else util.rs:653-718
    `rope_gguf`), as forward.rs:154-175 applies it. Returns rotated copies."""
    q = np.array(sq, np.float32, copy=True)
    kk = np.array(k, np.float32, copy=True)
    fn = lib().orc_rope if shape.rope_mode == 1 else lib().orc_rope_gguf
    fn(C.byref(shape), _p(q), _p(kk), pos)
    return q, kk


def argmax(p: np.ndarray) -> int:
    p = np.ascontiguousarray(p, np.float32)
    return int(lib().orc_argmax(_p(p), p.size))


def f16_to_f32(h: int) -> float:
    return float(lib().orc_f16_to_f32(h))


Q4_GGML, Q4_REF = 0, 1
Q8_0, Q4_0, F16 = 0, 1, 2  # WeightFormat (weight_type.rs:17-22)
ROPE_GGUF, ROPE_LLAMA3 = 0, 1


class Model:
    """Oracle model loaded from a .gguf, .safetensors or .lmrs file (lib.rs:107-133 dispatch)."""

    def __init__(self, path: str, max_ctx_len: int = 0xFFFFFFFF, fmt_override: int = -1, q4_mode: int = Q4_GGML):
        self._h = lib().orc_model_load(str(path).encode(), max_ctx_len, fmt_override, q4_mode)
        if not self._h:
            raise RuntimeError(lib().orc_last_error().decode())
        self.shape = OrcShape()
        lib().orc_model_shape(self._h, C.byref(self.shape))

    def get_embeddings(self, token: int) -> np.ndarray:
        out = np.zeros(self.shape.dim, np.float32)
        lib().orc_get_embeddings(self._h, token, _p(out))
        return out

    def create_session(self) -> "Session":
        return Session(self)

    def forward_x(self, tokens, start_pos: int, session: "Session") -> np.ndarray:
        t = np.ascontiguousarray(tokens, np.uint32)
        logits = np.zeros(self.shape.vocab_size, np.float32)
        rc = lib().orc_forward_x(self._h, session._h, _p(t), t.size, start_pos, _p(logits))
        if rc != 0:
            raise RuntimeError(lib().orc_last_error().decode())
        return logits

    def __del__(self):
        if getattr(self, "_h", None):
            lib().orc_model_free(self._h)
            self._h = None


class Session:
    def __init__(self, model: Model):
        self.model = model
        self._h = lib().orc_session_new(model._h)
        self.pos = 0

    def reset(self) -> None:
        lib().orc_session_reset(self._h)
        self.pos = 0

    def kv(self):
        n = lib().orc_session_cache_len(self._h)
        k = np.ctypeslib.as_array((C.c_float * n).from_address(lib().orc_session_key_cache(self._h)))
        v = np.ctypeslib.as_array((C.c_float * n).from_address(lib().orc_session_value_cache(self._h)))
        return k, v

    def __del__(self):
        if getattr(self, "_h", None):
            lib().orc_session_free(self._h)
            self._h = None
