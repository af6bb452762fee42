"""Python mirror of the reference's API for the quantized forward path.

The reference crate (yallma3-mini-inference) exposes, for this path:
  * weight_type.rs:17-120  WeightFormat, QuantizedTensor, quantize, matmul,
                           new_workspace_buffer
  * quantization.rs:23-52  MutableQuantizedTensorQ8, quantize
  * transformer.rs:19-69   the Transformer trait (load_model, name, vocab_size,
                           get_embeddings[_batch], forward_x, create_session,
                           max_ctx_len, eos_token, bos_token)
  * base_transformer.rs:78-105  InferenceSession (caller advances `pos`)
  * lib.rs:107-152         load_transformer, load_transformer_ffi
This module keeps those names and argument meanings and forwards every call to
the C-ABI of libyallma3_b200.so (include/yallma3.h), which runs the sm_100a
kernels. There is no CPU fallback: without the built library, importing this
module raises. Where the reference panics (format/variant mismatch), these
functions raise YlError.

Device tensors are passed as torch CUDA tensors (or raw integer device
addresses); torch is only the allocator here.
"""
from __future__ import annotations

import ctypes as C
import enum
import os
from pathlib import Path
from typing import Optional, Sequence

import numpy as np

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libyallma3_b200.so"

if not LIB_PATH.exists():
    raise ImportError(f"{LIB_PATH} is not built; run `python {_PKG / 'build.py'}` (nvcc, sm_100a)")

_lib = C.CDLL(str(LIB_PATH))

# ---------------------------------------------------------------- structs --


class QTensorC(C.Structure):
    _fields_ = [("fmt", C.c_int32), ("scale_type", C.c_int32), ("len", C.c_uint64), ("gs", C.c_uint64),
                ("rows", C.c_uint64), ("cols", C.c_uint64), ("scale_stride", C.c_uint64),
                ("quant", C.c_void_p), ("scale", C.c_void_p), ("owned", C.c_int32), ("flags", C.c_int32)]


class ShapeC(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("dim", "hidden_dim", "n_heads", "head_size", "n_kv_heads", "vocab_size",
                                          "n_layers", "ctx_len")] + [
        ("rms_norm_eps", C.c_float), ("rope_theta", C.c_float), ("group_size", C.c_uint32),
        ("rope_freq_scale", C.c_float), ("rope_ext_factor", C.c_float), ("rope_attn_factor", C.c_float),
        ("rope_original_ctx_len", C.c_uint32), ("attention_scale", C.c_float), ("weight_format", C.c_int32),
        ("rope_mode", C.c_int32), ("untied_lm_head", C.c_int32), ("tp_rank", C.c_int32), ("tp_size", C.c_int32),
        ("_pad", C.c_int32)]


class TpSplitC(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("q_rows0", "q_rows", "kv_rows0", "kv_rows", "ffn_rows0", "ffn_rows",
                                          "vocab0", "vocab_rows")]


class SynthC(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "vocab_size",
                                          "context_length")] + [
        ("rope_theta", C.c_float), ("rms_norm_eps", C.c_float), ("weight_format", C.c_int32),
        ("tied", C.c_int32), ("llama3_scaling", C.c_int32), ("llama3_factor", C.c_float),
        ("llama3_low", C.c_float), ("llama3_high", C.c_float), ("llama3_orig_ctx", C.c_uint32),
        ("seed", C.c_uint64), ("weight_std", C.c_float), ("threads", C.c_int32)]


_P = C.c_void_p
_sigs = {
    "yl_last_error": (C.c_char_p, []),
    "yl_version": (C.c_char_p, []),
    "yl_qtensor_alloc": (C.c_int, [C.c_int, C.c_uint64, C.c_uint64, C.POINTER(QTensorC)]),
    "yl_qtensor_alloc_weight": (C.c_int, [C.c_int, C.c_int, C.c_uint64, C.c_uint64, C.c_uint64,
                                          C.POINTER(QTensorC)]),
    "yl_qtensor_free": (C.c_int, [C.POINTER(QTensorC)]),
    "yl_qtensor_upload": (C.c_int, [C.POINTER(QTensorC), _P, _P, _P]),
    "yl_qtensor_download": (C.c_int, [C.POINTER(QTensorC), _P, _P, _P]),
    "yl_quantize_q8_0": (C.c_int, [_P, _P, _P, C.c_uint64, C.c_uint32, _P]),
    "yl_quantize": (C.c_int, [C.c_int, C.POINTER(QTensorC), _P, C.c_uint64, C.c_uint32, _P]),
    "yl_matmul": (C.c_int, [_P, C.POINTER(QTensorC), C.POINTER(QTensorC), C.c_uint64, C.c_uint64, C.c_uint64,
                            C.c_uint64, C.c_int, _P]),
    "yl_fused_attention": (C.c_int, [_P, _P, _P, _P, C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64,
                                     C.c_uint32, C.c_uint64, C.c_float, _P]),
    "yl_fused_attention_static": (C.c_int, [_P, _P, _P, _P, C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64,
                                            C.c_uint64, C.c_uint32, C.c_uint64, C.c_float, _P]),
    "yl_load_transformer": (C.c_int, [C.c_char_p, C.c_int, C.c_uint32, C.c_int, C.POINTER(_P)]),
    "yl_load_transformer_tp": (C.c_int, [C.c_char_p, C.c_uint32, C.c_int, C.c_int, C.c_int, C.POINTER(_P)]),
    "yl_session_tp_handle": (C.c_int, [_P, C.c_char_p]),
    "yl_session_tp_connect": (C.c_int, [_P, C.c_char_p]),
    "yl_tp_plan": (C.c_int, [C.POINTER(ShapeC), C.c_int, C.c_int, C.POINTER(TpSplitC)]),
    "yl_model_free": (C.c_int, [_P]),
    "yl_model_name": (C.c_char_p, [_P]),
    "yl_model_vocab_size": (C.c_uint64, [_P]),
    "yl_model_max_ctx_len": (C.c_uint32, [_P]),
    "yl_model_eos_token": (C.c_uint32, [_P]),
    "yl_model_bos_token": (C.c_uint32, [_P]),
    "yl_model_shape": (C.c_int, [_P, C.POINTER(ShapeC)]),
    "yl_model_device_bytes": (C.c_uint64, [_P]),
    "yl_get_embeddings": (C.c_int, [_P, C.c_uint32, _P]),
    "yl_get_embeddings_batch": (C.c_int, [_P, _P, C.c_uint64, _P]),
    "yl_model_weight": (C.c_int, [_P, C.c_uint32, C.c_int, C.POINTER(QTensorC)]),
    "yl_create_session": (C.c_int, [_P, C.POINTER(_P)]),
    "yl_session_reset": (C.c_int, [_P]),
    "yl_session_free": (C.c_int, [_P]),
    "yl_session_pos": (C.c_uint32, [_P]),
    "yl_session_set_pos": (C.c_int, [_P, C.c_uint32]),
    "yl_session_kv": (C.c_int, [_P, C.POINTER(_P), C.POINTER(_P), C.POINTER(C.c_uint64)]),
    "yl_forward_x": (C.c_int, [_P, _P, _P, C.c_uint64, C.c_uint32, _P, _P]),
    "yl_decode_greedy": (C.c_int, [_P, _P, C.c_uint32, C.c_uint32, C.c_uint32, _P, _P, C.c_int]),
    "yl_decode_step_launches": (C.c_int, [_P, C.POINTER(C.c_uint32)]),
    "yl_config_set": (C.c_int, [C.c_char_p, C.c_int64]),
    "yl_batch_create": (C.c_int, [_P, C.c_uint32, C.POINTER(_P)]),
    "yl_batch_free": (C.c_int, [_P]),
    "yl_batch_forward": (C.c_int, [_P, C.POINTER(_P), C.c_uint32, _P, _P, _P, _P]),
    "yl_session_decode_graph_launches": (C.c_int, [_P, C.c_int, C.POINTER(C.c_uint32)]),
    "yl_model_attention_decode": (C.c_int, [_P, _P, _P, _P, C.c_uint32, _P, _P, _P, _P]),
    "yl_profile_decode_step": (C.c_int, [_P, _P, C.c_uint32, C.c_uint32, _P, C.c_uint32, C.POINTER(C.c_uint32)]),
    "yl_trace_decode_step": (C.c_int, [_P, _P, C.c_uint32, C.c_uint32, _P, C.c_uint64, C.POINTER(C.c_uint32)]),
    "load_transformer_ffi": (C.c_bool, [C.c_char_p]),
    "infer_ffi": (C.c_void_p, [C.c_char_p]),
    "free_string": (None, [C.c_void_p]),
    "yl_infer_config": (C.c_int, [C.c_float, C.c_float, C.c_uint64, C.c_uint32]),
    "yl_tokenizer_load": (C.c_int, [C.c_char_p, C.POINTER(_P)]),
    "yl_tokenizer_free": (C.c_int, [_P]),
    "yl_model_tokenizer": (C.c_int, [_P, C.POINTER(_P)]),
    "yl_tokenizer_info": (C.c_int, [_P, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32), C.POINTER(C.c_uint32),
                                    C.POINTER(C.c_int)]),
    "yl_tokenizer_encode": (C.c_int, [_P, C.c_char_p, C.c_int, C.c_int, _P, C.c_uint64, C.POINTER(C.c_uint64)]),
    "yl_tokenizer_decode": (C.c_int, [_P, _P, C.c_uint64, _P, C.c_uint64, C.POINTER(C.c_uint64)]),
    "yl_tokenizer_chat_prompt": (C.c_int, [_P, C.c_char_p, C.c_char_p, _P, C.c_uint64, C.POINTER(C.c_uint64)]),
    "yl_tokenizer_render_chat": (C.c_int, [_P, _P, _P, C.c_uint64, C.c_int, _P, C.c_uint64, C.POINTER(C.c_uint64)]),
    "yl_tokenizer_encode_wrap_n_header": (C.c_int, [_P, C.c_char_p, C.c_char_p, C.c_int, _P, C.c_uint64,
                                                    C.POINTER(C.c_uint64)]),
    "yl_tokenizer_set_chat_template": (C.c_int, [_P, C.c_char_p]),
    "yl_tokenizer_apply_system_template": (C.c_int, [_P, C.c_char_p, _P, C.c_uint64, C.POINTER(C.c_uint64)]),
    "yl_tokenizer_apply_turn_template": (C.c_int, [_P, C.c_char_p, C.c_int, _P, C.c_uint64, C.POINTER(C.c_uint64)]),
    "yl_chat_template_render": (C.c_int, [C.c_char_p, _P, _P, C.c_uint64, C.c_int, _P, C.c_uint64,
                                          C.POINTER(C.c_uint64)]),
    "yl_sampler_create": (C.c_int, [C.c_uint32, C.c_float, C.c_float, C.c_uint64, C.POINTER(_P)]),
    "yl_sampler_free": (C.c_int, [_P]),
    "yl_sampler_sample": (C.c_int, [_P, _P, _P, _P]),
    "yl_sampler_result": (C.c_int, [_P, C.POINTER(C.c_uint32)]),
    "yl_session_logits": (C.c_int, [_P, C.POINTER(_P)]),
    "yl_synth_write_gguf": (C.c_int, [C.c_char_p, C.POINTER(SynthC)]),
}
for _name, (_res, _args) in _sigs.items():
    _f = getattr(_lib, _name)
    _f.restype = _res
    _f.argtypes = _args

EXPORTED = tuple(_sigs)

# ------------------------------------------------------------------ errors --

STATUS = {0: "YL_OK", -1: "YL_ERR_ARG", -2: "YL_ERR_IO", -3: "YL_ERR_FORMAT", -4: "YL_ERR_CUDA",
          -5: "YL_ERR_OOM", -6: "YL_ERR_RANGE", -7: "YL_ERR_TIMEOUT", -8: "YL_ERR_UNSUPPORTED", -9: "YL_ERR_COMM"}


class YlError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS.get(code, code)}: {msg}")
        self.code = code


def _check(rc: int) -> None:
    if rc != 0:
        raise YlError(rc, _lib.yl_last_error().decode(errors="replace"))


def last_error() -> str:
    return _lib.yl_last_error().decode(errors="replace")


def config_set(key: str, value: int) -> None:
    """Process-wide device-path option (yl_config_set): gemm, gemm_tc, gemm_tc_min, gemm_f16_min."""
    _check(_lib.yl_config_set(key.encode(), int(value)))


def version() -> str:
    return _lib.yl_version().decode()


def raw_lib() -> C.CDLL:
    """The loaded C library (for direct C-ABI calls in tests and benchmarks)."""
    return _lib


def _ptr(t) -> Optional[int]:
    if t is None:
        return None
    if isinstance(t, int):
        return t
    if hasattr(t, "data_ptr"):
        return t.data_ptr()
    if isinstance(t, np.ndarray):
        return t.ctypes.data
    raise TypeError(f"cannot take a pointer of {type(t)}")


def _stream(stream) -> Optional[int]:
    if stream is None:
        try:
            import torch
            if torch.cuda.is_available():
                return torch.cuda.current_stream().cuda_stream
        except ImportError:
            pass
        return None
    return stream if isinstance(stream, int) else stream.cuda_stream


# ------------------------------------------------------ weight_type.rs ---

class WeightFormat(enum.IntEnum):
    """weight_type.rs:17-22"""
    Q8_0 = 0
    Q4_0 = 1
    F16 = 2


class QuantType(enum.IntEnum):
    """quantization.rs:15-21"""
    NONE = 0
    Q8_0 = 1
    Q4_0 = 2
    F16 = 3


SCALE_F32, SCALE_F16 = 0, 1


class QuantizedTensor:
    """A device-resident QuantizedTensor (weight_type.rs:30-50).

    Activation tensors (the reference's flat containers) come from
    `new_workspace_buffer`; weight matrices (repacked HBM layout) from
    `QuantizedTensor.weight`. Views of model weights are not owned."""

    def __init__(self, c: QTensorC):
        self.c = c

    @staticmethod
    def weight(fmt: WeightFormat, rows: int, cols: int, gs: int = 32, scale_type: int = SCALE_F16):
        c = QTensorC()
        _check(_lib.yl_qtensor_alloc_weight(int(fmt), scale_type, rows, cols, gs, C.byref(c)))
        return QuantizedTensor(c)

    @property
    def fmt(self) -> WeightFormat:
        return WeightFormat(self.c.fmt)

    @property
    def len(self) -> int:
        return self.c.len

    def upload(self, quant_vals=None, scale_factor=None, values=None) -> "QuantizedTensor":
        """Host data in the reference container layout (numpy): int8 values and
        f32 scales per group (Q4_0 weights: signed q-8), or f32 values (F16)."""
        q = None if quant_vals is None else np.ascontiguousarray(quant_vals, dtype=np.int8)
        s = None if scale_factor is None else np.ascontiguousarray(scale_factor, dtype=np.float32)
        v = None if values is None else np.ascontiguousarray(values, dtype=np.float32)
        _check(_lib.yl_qtensor_upload(C.byref(self.c), _ptr(q), _ptr(s), _ptr(v)))
        return self

    def download(self):
        n = self.c.len
        if self.c.fmt == WeightFormat.F16:
            v = np.empty(n, np.float32)
            _check(_lib.yl_qtensor_download(C.byref(self.c), None, None, _ptr(v)))
            return v
        q = np.empty(n, np.int8)
        s = np.empty(n // self.c.gs, np.float32)
        _check(_lib.yl_qtensor_download(C.byref(self.c), _ptr(q), _ptr(s), None))
        return q, s

    def free(self) -> None:
        if self.c.owned and self.c.quant:
            _lib.yl_qtensor_free(C.byref(self.c))

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def new_workspace_buffer(fmt: WeightFormat, len: int, gs: int) -> QuantizedTensor:
    """weight_type.rs:108-120"""
    c = QTensorC()
    _check(_lib.yl_qtensor_alloc(int(fmt), len, gs, C.byref(c)))
    return QuantizedTensor(c)


def quantize(fmt: WeightFormat, dst: QuantizedTensor, x, n: int, gs: int, stream=None) -> None:
    """weight_type.rs:76-90: quantize n values of device tensor `x` into `dst`."""
    _check(_lib.yl_quantize(int(fmt), C.byref(dst.c), _ptr(x), n, gs, _stream(stream)))


def quantize_q8_0(x, q, scale, n: int, gs: int = 32, stream=None) -> None:
    """quantization.rs:29-52 on device pointers / tensors (bit-exact)."""
    _check(_lib.yl_quantize_q8_0(_ptr(x), _ptr(q), _ptr(scale), n, gs, _stream(stream)))


def matmul(out, x: QuantizedTensor, w: QuantizedTensor, n: int, o: int, gs: int, batch: Optional[int] = None,
           accumulate: bool = True, stream=None) -> None:
    """weight_type.rs:92-106. batch defaults to out.numel() // o like the
    reference. accumulate=True reproduces the reference's `+=` on the first
    4*floor(o/4) columns."""
    if batch is None:
        batch = out.numel() // o
    _check(_lib.yl_matmul(_ptr(out), C.byref(x.c), C.byref(w.c), n, o, gs, batch, 1 if accumulate else 0,
                          _stream(stream)))


def fused_attention(output, sq, key_cache, value_cache, seq_len: int, batch: int, n_heads: int, n_kv_heads: int,
                    head_size: int, start_pos: int, kv_dim: int, attn_scale: float, stream=None) -> None:
    """forward.rs:299-400 on device tensors (queries rotated, caches filled)."""
    _check(_lib.yl_fused_attention(_ptr(output), _ptr(sq), _ptr(key_cache), _ptr(value_cache), seq_len, batch,
                                   n_heads, n_kv_heads, head_size, start_pos, kv_dim, attn_scale, _stream(stream)))


# -------------------------------------------------- transformer.rs ---

class InferenceSession:
    """base_transformer.rs:78-105: device KV cache; the caller advances pos."""

    def __init__(self, handle: int, model: "Transformer"):
        self._h = handle
        self._model = model
        self.pos = 0

    def reset(self) -> None:
        _check(_lib.yl_session_reset(self._h))
        self.pos = 0

    def tp_handle(self) -> bytes:
        """This rank's exchange-region handle (tensor-parallel sessions)."""
        buf = C.create_string_buffer(64)
        _check(_lib.yl_session_tp_handle(self._h, buf))
        return buf.raw

    def tp_connect(self, handles: Sequence[bytes]) -> None:
        """Maps every rank's exchange region (handles in rank order)."""
        blob = b"".join(handles)
        _check(_lib.yl_session_tp_connect(self._h, blob))

    def tp_connect_group(self, group=None) -> None:
        """Exchanges handles over torch.distributed (all ranks call this)."""
        import torch.distributed as dist
        hs = [None] * dist.get_world_size(group)
        dist.all_gather_object(hs, self.tp_handle(), group=group)
        self.tp_connect(hs)

    def kv_cache(self):
        k, v, n = _P(), _P(), C.c_uint64()
        _check(_lib.yl_session_kv(self._h, C.byref(k), C.byref(v), C.byref(n)))
        return k.value, v.value, n.value

    def close(self) -> None:
        if self._h:
            _lib.yl_session_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class SessionBatch:
    """Batched decode of independent sessions (yl_batch_forward): one step
    feeds one token to each of up to `max_sessions` sessions of one model."""

    def __init__(self, model: "Transformer", max_sessions: int):
        h = _P()
        _check(_lib.yl_batch_create(model._h, int(max_sessions), C.byref(h)))
        self._h = h.value
        self._model = model
        self.max_sessions = int(max_sessions)

    def forward(self, sessions: Sequence["InferenceSession"], tokens: Sequence[int], positions: Sequence[int],
                want_logits: bool = False):
        """One decode step; returns (ids [n], logits [n, vocab] or None). Each
        session's pos becomes positions[i] + 1."""
        n = len(sessions)
        hs = (_P * n)(*[se._h for se in sessions])
        t = np.ascontiguousarray(tokens, np.uint32)
        p = np.ascontiguousarray(positions, np.uint32)
        if t.size != n or p.size != n:
            raise ValueError("one token and one position per session")
        ids = np.empty(n, np.uint32)
        logits = np.empty((n, self._model.vocab_size()), np.float32) if want_logits else None
        _check(_lib.yl_batch_forward(self._h, hs, n, _ptr(t), _ptr(p), _ptr(logits) if logits is not None else None,
                                     _ptr(ids)))
        for i, se in enumerate(sessions):
            se.pos = int(p[i]) + 1
        return ids, logits

    def close(self) -> None:
        if self._h:
            _lib.yl_batch_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Transformer:
    """The Transformer trait (transformer.rs:19-69) over a device model."""

    def __init__(self, handle: int):
        self._h = handle

    @classmethod
    def load_model(cls, model_path: str, max_ctx_len: int = 0xFFFFFFFF) -> "Transformer":
        return load_transformer(model_path, False, max_ctx_len, None)

    def name(self) -> str:
        return _lib.yl_model_name(self._h).decode()

    def vocab_size(self) -> int:
        return int(_lib.yl_model_vocab_size(self._h))

    def max_ctx_len(self) -> int:
        return int(_lib.yl_model_max_ctx_len(self._h))

    def eos_token(self) -> int:
        return int(_lib.yl_model_eos_token(self._h))

    def bos_token(self) -> int:
        return int(_lib.yl_model_bos_token(self._h))

    def tokenizer(self) -> "Tokenizer":
        """Transformer::tokenizer(): loaded from the model file at the first call."""
        h = _P()
        _check(_lib.yl_model_tokenizer(self._h, C.byref(h)))
        return Tokenizer(h.value, owned=False, keep=self)

    def shape(self) -> ShapeC:
        s = ShapeC()
        _check(_lib.yl_model_shape(self._h, C.byref(s)))
        return s

    def device_bytes(self) -> int:
        return int(_lib.yl_model_device_bytes(self._h))

    def get_embeddings(self, token: int) -> np.ndarray:
        out = np.empty(self.shape().dim, np.float32)
        _check(_lib.yl_get_embeddings(self._h, token, _ptr(out)))
        return out

    def get_embeddings_batch(self, tokens: Sequence[int]) -> list:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        d = self.shape().dim
        out = np.empty((len(t), d), np.float32)
        _check(_lib.yl_get_embeddings_batch(self._h, _ptr(t), len(t), _ptr(out)))
        return [row for row in out]

    def create_session(self) -> InferenceSession:
        h = _P()
        _check(_lib.yl_create_session(self._h, C.byref(h)))
        return InferenceSession(h.value, self)

    def create_batch(self, max_sessions: int) -> SessionBatch:
        """Workspace for batched decode of up to max_sessions (<= 16) sessions."""
        return SessionBatch(self, max_sessions)

    def forward_x(self, tokens: Sequence[int], start_pos: int, session: InferenceSession) -> np.ndarray:
        """Logits of the last token (length vocab_size), like forward.rs:261-279."""
        logits, _ = self.forward_x_full(tokens, start_pos, session, want_logits=True)
        return logits

    def forward_x_full(self, tokens, start_pos: int, session: InferenceSession, want_logits: bool = True,
                       logits_out: Optional[np.ndarray] = None):
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        logits = None
        if want_logits:
            logits = logits_out if logits_out is not None else np.empty(self.vocab_size(), np.float32)
        am = np.zeros(1, np.uint32)
        _check(_lib.yl_forward_x(self._h, session._h, _ptr(t), len(t), start_pos, _ptr(logits), _ptr(am)))
        return logits, int(am[0])

    def decode_greedy(self, session: InferenceSession, first_token: int, start_pos: int, n_steps: int,
                      stream=None, sync: bool = True) -> Optional[np.ndarray]:
        """n_steps device-resident greedy steps (one CUDA graph launch each)."""
        out = np.empty(n_steps, np.uint32) if sync else None
        _check(_lib.yl_decode_greedy(self._h, session._h, first_token, start_pos, n_steps, _ptr(out),
                                     _stream(stream) if stream is not None else None, 1 if sync else 0))
        return out

    def decode_step_launches(self) -> int:
        n = C.c_uint32()
        _check(_lib.yl_decode_step_launches(self._h, C.byref(n)))
        return n.value

    def attention_decode(self, qkv, key_cache, value_cache, pos: int, out=None, out_q=None, out_s=None,
                         stream=None) -> None:
        """The decode step's fused RoPE + cache write + attention kernel for one
        token (device tensors): k/v rows written at `pos`, output into out (f32)
        and/or out_q/out_s (Q8_0 blocks)."""
        _check(_lib.yl_model_attention_decode(self._h, _ptr(qkv), _ptr(key_cache), _ptr(value_cache), pos,
                                              _ptr(out), _ptr(out_q), _ptr(out_s), _stream(stream)))

    def decode_graph_launches(self, session: InferenceSession, with_logits: bool = False) -> int:
        """Kernel nodes of the session's captured decode graph (counted in the graph)."""
        n = C.c_uint32()
        _check(_lib.yl_session_decode_graph_launches(session._h, 1 if with_logits else 0, C.byref(n)))
        return n.value

    def profile_decode_step(self, session: InferenceSession, token: int, pos: int) -> np.ndarray:
        """Per-launch device microseconds of one decode step launched kernel
        by kernel: [embed, (qkv, attention, wo, gate/up, down) x layers, lm_head]."""
        cap = 8 + 8 * self.shape().n_layers
        us = np.zeros(cap, np.float32)
        n = C.c_uint32()
        _check(_lib.yl_profile_decode_step(self._h, session._h, token, pos, _ptr(us), cap, C.byref(n)))
        return us[:n.value]

    def trace_decode_step(self, session: InferenceSession, token: int, pos: int) -> np.ndarray:
        """Global-timer stamps (ns) of one decode step run as the decode graph
        runs it: array [launch][cta][8] = (entry, activations staged / wait
        released, wait released / partials visible, done, rows loaded, norm
        factor ready, -, -); zeros where a launch has fewer CTAs or a point
        is not stamped (the embedding launch has none)."""
        n_max = 7 * self.shape().n_layers + 6
        out = np.zeros(n_max * 8192, np.uint64)
        n = C.c_uint32()
        _check(_lib.yl_trace_decode_step(self._h, session._h, token, pos, _ptr(out), out.size, C.byref(n)))
        return out[: n.value * 8192].reshape(n.value, 1024, 8)

    def weight(self, layer: int, which: int) -> QuantizedTensor:
        c = QTensorC()
        _check(_lib.yl_model_weight(self._h, layer, which, C.byref(c)))
        return QuantizedTensor(c)

    def close(self) -> None:
        if self._h:
            _lib.yl_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass



class Tokenizer:
    """tokenizer.rs's Tokenizer (byte-level BPE) through the C-ABI (host only)."""

    def __init__(self, handle: int, owned: bool = True, keep=None):
        self._h = handle
        self._owned = owned
        self._keep = keep  # the model that owns a borrowed tokenizer

    @classmethod
    def load(cls, model_path: str) -> "Tokenizer":
        h = _P()
        _check(_lib.yl_tokenizer_load(model_path.encode(), C.byref(h)))
        return cls(h.value)

    def info(self) -> dict:
        v, b, e, t = C.c_uint32(), C.c_uint32(), C.c_uint32(), C.c_int()
        _check(_lib.yl_tokenizer_info(self._h, C.byref(v), C.byref(b), C.byref(e), C.byref(t)))
        return {"vocab_size": v.value, "bos": b.value, "eos": e.value, "has_template": bool(t.value)}

    def _ids(self, fn, *args) -> list:
        n = C.c_uint64()
        cap = 256
        while True:
            buf = np.zeros(cap, np.uint32)
            rc = fn(self._h, *args, _ptr(buf), cap, C.byref(n))
            if rc == -6 and n.value > cap:  # YL_ERR_RANGE: retry with the reported size
                cap = n.value
                continue
            _check(rc)
            return [int(x) for x in buf[: n.value]]

    def encode(self, text: str, bos: bool = False, eos: bool = False) -> list:
        return self._ids(_lib.yl_tokenizer_encode, text.encode(), 1 if bos else 0, 1 if eos else 0)

    def decode(self, ids: Sequence[int]) -> str:
        t = np.ascontiguousarray(ids, dtype=np.uint32)
        n = C.c_uint64()
        cap = 64 + 16 * len(t)
        while True:
            buf = C.create_string_buffer(cap)
            rc = _lib.yl_tokenizer_decode(self._h, _ptr(t) if len(t) else None, len(t), buf, cap, C.byref(n))
            if rc == -6 and n.value + 1 > cap:
                cap = n.value + 1
                continue
            _check(rc)
            return buf.raw[: n.value].decode("utf-8")

    def chat_prompt(self, user: str, system: str = "") -> list:
        return self._ids(_lib.yl_tokenizer_chat_prompt, system.encode(), user.encode())

    def encode_wrap_n_header(self, text: str, header: str, begin_of_text_wrap: bool) -> list:
        return self._ids(_lib.yl_tokenizer_encode_wrap_n_header, text.encode(), header.encode(),
                         1 if begin_of_text_wrap else 0)

    def set_chat_template(self, template: str) -> None:
        _check(_lib.yl_tokenizer_set_chat_template(self._h, template.encode()))

    def apply_system_template(self, system: str) -> list:
        return self._ids(_lib.yl_tokenizer_apply_system_template, system.encode())

    def apply_turn_template(self, user: str, add_empty_assistant: bool) -> list:
        return self._ids(_lib.yl_tokenizer_apply_turn_template, user.encode(), 1 if add_empty_assistant else 0)

    def render_chat(self, messages: Sequence[tuple], add_generation_prompt: bool) -> list:
        """Tokenizer::render_chat_template: messages are (role, content) pairs."""
        roles, contents, keep = _message_arrays(messages)
        return self._ids(_lib.yl_tokenizer_render_chat, roles, contents, len(messages),
                         1 if add_generation_prompt else 0)

    def close(self) -> None:
        if self._h and self._owned:
            _lib.yl_tokenizer_free(self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Sampler:
    """sampler.rs's Sampler on the device: sample() takes a CUDA logits row."""

    def __init__(self, vocab_size: int, temperature: float, top_p: float, seed: int):
        h = _P()
        _check(_lib.yl_sampler_create(vocab_size, temperature, top_p, seed, C.byref(h)))
        self._h = h.value

    def sample(self, logits, stream=None) -> int:
        """Sampler::sample(&mut logits): logits (device, float32) is overwritten like the reference's slice."""
        out = C.c_uint32()
        _check(_lib.yl_sampler_sample(self._h, _ptr(logits), C.byref(out), _stream(stream)))
        return out.value

    def close(self) -> None:
        if self._h:
            _lib.yl_sampler_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _message_arrays(messages: Sequence[tuple]):
    enc = [(r.encode(), c.encode()) for r, c in messages]
    roles = (C.c_char_p * max(1, len(enc)))(*[r for r, _ in enc])
    contents = (C.c_char_p * max(1, len(enc)))(*[c for _, c in enc])
    return C.cast(roles, C.c_void_p), C.cast(contents, C.c_void_p), (roles, contents, enc)


def render_chat_template(template: str, messages: Sequence[tuple], add_generation_prompt: bool) -> str:
    """Renders chat-template source with {messages, add_generation_prompt}
    (the text step of Tokenizer::render_chat_template)."""
    roles, contents, keep = _message_arrays(messages)
    n = C.c_uint64()
    cap = 256 + 2 * len(template)
    while True:
        buf = C.create_string_buffer(cap)
        rc = _lib.yl_chat_template_render(template.encode(), roles, contents, len(messages),
                                          1 if add_generation_prompt else 0, buf, cap, C.byref(n))
        if rc == -6 and n.value + 1 > cap:
            cap = n.value + 1
            continue
        _check(rc)
        return buf.raw[: n.value].decode("utf-8")


def session_logits(session: InferenceSession) -> int:
    """Device address of the session's logits row (single-GPU models)."""
    p = _P()
    _check(_lib.yl_session_logits(session._h, C.byref(p)))
    return p.value


def infer_config(temperature: float = 0.7, top_p: float = 0.9, seed: int = 42, max_tokens: int = 0) -> None:
    _check(_lib.yl_infer_config(temperature, top_p, seed, max_tokens))


def infer_ffi(prompt: str) -> Optional[str]:
    """infer_ffi + free_string as a C host binds them (PoC_Bun_load.js:12-38)."""
    p = _lib.infer_ffi(prompt.encode())
    if not p:
        return None
    try:
        return C.string_at(p).decode("utf-8")
    finally:
        _lib.free_string(p)

def load_transformer(model_path: str, sequential: bool = False, max_ctx_len: int = 0xFFFFFFFF,
                     fmt_override: Optional[WeightFormat] = None) -> Transformer:
    """lib.rs:107-133"""
    h = _P()
    _check(_lib.yl_load_transformer(str(model_path).encode(), 1 if sequential else 0, max_ctx_len,
                                    -1 if fmt_override is None else int(fmt_override), C.byref(h)))
    return Transformer(h.value)


def load_transformer_tp(model_path: str, tp_rank: int, tp_size: int, max_ctx_len: int = 0xFFFFFFFF,
                        fmt_override: Optional[WeightFormat] = None) -> Transformer:
    """Rank tp_rank's shard of a tensor-parallel model on the current device
    (one process per GPU); its sessions need tp_connect / tp_connect_group."""
    h = _P()
    _check(_lib.yl_load_transformer_tp(str(model_path).encode(), max_ctx_len,
                                       -1 if fmt_override is None else int(fmt_override), tp_rank, tp_size,
                                       C.byref(h)))
    return Transformer(h.value)


def tp_plan(shape: ShapeC, tp_rank: int, tp_size: int) -> dict:
    """The tensor-parallel split of a shape (no GPU needed)."""
    out = TpSplitC()
    _check(_lib.yl_tp_plan(C.byref(shape), tp_rank, tp_size, C.byref(out)))
    return {n: getattr(out, n) for n, _ in TpSplitC._fields_}


def shape_of(**kw) -> ShapeC:
    """A ShapeC from keyword fields (others zero), e.g. for tp_plan."""
    sc = ShapeC()
    for k, v in kw.items():
        setattr(sc, k, v)
    return sc


def load_transformer_ffi(model_path: Optional[str]) -> bool:
    """lib.rs:135-152"""
    return bool(_lib.load_transformer_ffi(None if model_path is None else str(model_path).encode()))


# -------------------------------------------------- synthetic models ---

# Benchmark configurations: C1 SmolLM2-135M-shaped, C2/C3 Llama-3.2-1B-shaped (Q8_0 /
# Q4_0), C4 Llama-3-8B-shaped (untied lm_head); plus tiny shapes for tests.
PRESETS = {
    "c1": dict(dim=576, hidden_dim=1536, n_layers=30, n_heads=9, n_kv_heads=3, vocab_size=49152,
               context_length=2048, rope_theta=1e5, rms_norm_eps=1e-5, weight_format=WeightFormat.Q8_0, tied=True,
               seed=0),
    "c2": dict(dim=2048, hidden_dim=8192, n_layers=16, n_heads=32, n_kv_heads=8, vocab_size=128256,
               context_length=131072, rope_theta=5e5, rms_norm_eps=1e-5, weight_format=WeightFormat.Q8_0, tied=True,
               llama3_scaling=True, seed=1),
    "c3": dict(dim=2048, hidden_dim=8192, n_layers=16, n_heads=32, n_kv_heads=8, vocab_size=128256,
               context_length=131072, rope_theta=5e5, rms_norm_eps=1e-5, weight_format=WeightFormat.Q4_0, tied=True,
               llama3_scaling=True, seed=2),
    "c4": dict(dim=4096, hidden_dim=14336, n_layers=32, n_heads=32, n_kv_heads=8, vocab_size=128256,
               context_length=8192, rope_theta=5e5, rms_norm_eps=1e-5, weight_format=WeightFormat.Q8_0, tied=False,
               seed=3),
    "tiny": dict(dim=256, hidden_dim=512, n_layers=2, n_heads=4, n_kv_heads=2, vocab_size=512, context_length=256,
                 rope_theta=1e4, rms_norm_eps=1e-5, weight_format=WeightFormat.Q8_0, tied=True, seed=7),
    "tiny128": dict(dim=512, hidden_dim=1024, n_layers=2, n_heads=4, n_kv_heads=1, vocab_size=1000,
                    context_length=512, rope_theta=5e5, rms_norm_eps=1e-5, weight_format=WeightFormat.Q8_0,
                    tied=False, seed=8),
}


def synth_write_gguf(path: str, dim: int, hidden_dim: int, n_layers: int, n_heads: int, n_kv_heads: int,
                     vocab_size: int, context_length: int = 4096, rope_theta: float = 1e4, rms_norm_eps: float = 1e-5,
                     weight_format: WeightFormat = WeightFormat.Q8_0, tied: bool = True, llama3_scaling: bool = False,
                     llama3_factor: float = 32.0, llama3_low: float = 1.0, llama3_high: float = 4.0,
                     llama3_orig_ctx: int = 8192, seed: int = 0, weight_std: float = 0.02, threads: int = 0) -> str:
    """Writes a seeded random-init LLaMA GGUF v3 (weights ~ N(0, weight_std))."""
    c = SynthC(dim=dim, hidden_dim=hidden_dim, n_layers=n_layers, n_heads=n_heads, n_kv_heads=n_kv_heads,
               vocab_size=vocab_size, context_length=context_length, rope_theta=rope_theta,
               rms_norm_eps=rms_norm_eps, weight_format=int(weight_format), tied=1 if tied else 0,
               llama3_scaling=1 if llama3_scaling else 0, llama3_factor=llama3_factor, llama3_low=llama3_low,
               llama3_high=llama3_high, llama3_orig_ctx=llama3_orig_ctx, seed=seed, weight_std=weight_std,
               threads=threads)
    _check(_lib.yl_synth_write_gguf(str(path).encode(), C.byref(c)))
    return str(path)


def synth_preset(name: str, path: str, **overrides) -> str:
    cfg = dict(PRESETS[name])
    cfg.update(overrides)
    return synth_write_gguf(path, **cfg)


def prompt_ids(vocab: int, n: int, seed: int) -> np.ndarray:
    """Uniform random prompt ids (seeded)."""
    return np.random.default_rng(seed).integers(0, vocab, size=n, dtype=np.uint32)
