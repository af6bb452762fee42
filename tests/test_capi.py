"""CPU: the C-ABI library loads, exports every function include/yallma3.h
declares, and rejects bad inputs with status codes (no GPU needed)."""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_functions() -> list[str]:
    src = (ROOT / "include" / "yallma3.h").read_text()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\**\s*([A-Za-z_][A-Za-z0-9_]*)\s*\(", src, re.M)
    return sorted(set(n for n in names if n not in {"if", "return", "sizeof"}))


def test_header_symbols_exported(yl):
    lib = yl.raw_lib()
    names = declared_functions()
    assert "yl_matmul" in names and "load_transformer_ffi" in names and "yl_forward_x" in names
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # the Python mirror binds every declared function
    assert set(names) <= set(yl.EXPORTED), set(names) - set(yl.EXPORTED)


def test_version(yl):
    assert "sm_100a" in yl.version()


def test_load_errors_without_gpu(yl, tmp_path):
    with pytest.raises(yl.YlError) as e:
        yl.load_transformer(str(tmp_path / "missing.gguf"))
    assert e.value.code == -2  # YL_ERR_IO
    with pytest.raises(yl.YlError) as e:
        yl.load_transformer(str(tmp_path / "model.bin"))
    assert e.value.code == -1  # unsupported extension (lib.rs:131)
    with pytest.raises(yl.YlError) as e:  # no config.json beside it
        yl.load_transformer(str(tmp_path / "model.safetensors"))
    assert e.value.code == -2 and "config.json" in str(e.value)
    with pytest.raises(yl.YlError) as e:
        yl.load_transformer(str(tmp_path / "model.lmrs"))
    assert e.value.code == -2
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"NOTGGUF" + bytes(64))
    with pytest.raises(yl.YlError) as e:
        yl.load_transformer(str(bad))
    assert e.value.code == -3 and "magic" in str(e.value)
    v2 = tmp_path / "v2.gguf"
    v2.write_bytes(b"GGUF" + (2).to_bytes(4, "little") + bytes(16))
    with pytest.raises(yl.YlError) as e:
        yl.load_transformer(str(v2))
    assert e.value.code == -3 and "version 3" in str(e.value)


def test_truncated_gguf_rejected(yl, tmp_path, model_factory):
    data = Path(model_factory("tiny")).read_bytes()
    t = tmp_path / "trunc.gguf"
    t.write_bytes(data[:200])
    with pytest.raises(yl.YlError) as e:
        yl.load_transformer(str(t))
    assert e.value.code == -3


def test_ffi_returns_false_on_error(yl, tmp_path):
    assert yl.load_transformer_ffi(None) is False
    assert yl.load_transformer_ffi(str(tmp_path / "nope.gguf")) is False


def test_null_arguments(yl):
    lib = yl.raw_lib()
    assert lib.yl_matmul(None, None, None, 0, 0, 32, 0, 0, None) == -1
    assert lib.yl_quantize_q8_0(None, None, None, 64, 16, None) == -8  # group size 16 unsupported on device
    assert lib.yl_model_vocab_size(None) == 0


def test_synth_gguf_parsed_by_oracle(yl, orc, model_factory):
    for preset, fmt in (("tiny", 0), ("tiny128", 0)):
        m = orc.Model(model_factory(preset), 4096)
        cfg = yl.PRESETS[preset]
        assert m.shape.dim == cfg["dim"] and m.shape.vocab_size == cfg["vocab_size"]
        assert m.shape.head_size == cfg["dim"] // cfg["n_heads"]
        assert m.shape.untied_lm_head == (0 if cfg["tied"] else 1)
        assert m.shape.weight_format == fmt


def test_synth_deterministic(yl, tmp_path):
    a = yl.synth_preset("tiny", str(tmp_path / "a.gguf"), threads=1)
    b = yl.synth_preset("tiny", str(tmp_path / "b.gguf"), threads=7)
    assert Path(a).read_bytes() == Path(b).read_bytes()
    c = yl.synth_preset("tiny", str(tmp_path / "c.gguf"), seed=99)
    assert Path(a).read_bytes() != Path(c).read_bytes()


def test_synth_weight_statistics(yl, orc, model_factory):
    m = orc.Model(model_factory("tiny128"), 512)
    e = np.concatenate([m.get_embeddings(t) for t in range(64)])
    assert abs(float(e.std()) - 0.02) < 0.002 and abs(float(e.mean())) < 0.002


def test_infer_ffi_error_paths_without_gpu(tmp_path):
    """infer_ffi before any load_transformer_ffi returns NULL (no abort),
    free_string accepts NULL, yl_infer_config rejects a negative temperature.
    Run in a fresh process: the loaded-model slot is process-global."""
    import subprocess
    import sys
    code = (
        "import importlib, sys, ctypes as C\n"
        f"sys.path.insert(0, {str(ROOT)!r})\n"
        "yl = importlib.import_module('yallma3-mini-inference_b200')\n"
        "lib = yl.raw_lib()\n"
        "assert lib.infer_ffi(b'hello') is None\n"
        "assert 'no model loaded' in yl.last_error()\n"
        "lib.free_string(None)\n"
        "assert lib.yl_infer_config(C.c_float(-1.0), C.c_float(0.9), 42, 0) == -1\n"
        "assert lib.yl_infer_config(C.c_float(0.0), C.c_float(0.9), 42, 8) == 0\n"
        "print('ok')\n")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr


def test_matmul_size_checks_do_not_wrap(tmp_path):
    """yl_matmul checks batch * n against the activation length without 64-bit
    wrap-around and refuses batches beyond 32 bits, before any CUDA call: a
    batch whose product with n wraps to a small number gets YL_ERR_ARG. Run
    with no visible GPU on descriptors whose device pointers are placeholders
    (never dereferenced on this path)."""
    import os
    import subprocess
    import sys
    code = (
        "import importlib, sys, ctypes as C\n"
        f"sys.path.insert(0, {str(ROOT)!r})\n"
        "yl = importlib.import_module('yallma3-mini-inference_b200')\n"
        "lib = yl.raw_lib()\n"
        "n, o = 96, 64\n"
        "w = yl.QTensorC(fmt=0, scale_type=1, len=o * n, gs=32, rows=o, cols=n, scale_stride=n // 32,\n"
        "                quant=0x1000, scale=0x2000, owned=0, flags=0)\n"
        "x = yl.QTensorC(fmt=0, scale_type=1, len=4 * n, gs=32, rows=0, cols=0, scale_stride=0,\n"
        "                quant=0x3000, scale=0x4000, owned=0, flags=0)\n"
        "for batch in ((1 << 64) // n + 1, 1 << 32, (1 << 63) + 3, 5):\n"
        "    rc = lib.yl_matmul(C.c_void_p(0x5000), C.byref(x), C.byref(w), n, o, 32, batch, 0, None)\n"
        "    assert rc == -1, (batch, rc, yl.last_error())\n"
        "t = yl.QTensorC()\n"
        "for fmt in (0, 2):  # an activation length whose byte count would wrap\n"
        "    assert lib.yl_qtensor_alloc(fmt, (1 << 62) + 4, 32, C.byref(t)) == -1, yl.last_error()\n"
        "print('ok')\n")
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr


def test_config_set_keys(yl):
    """yl_config_set: the documented keys are accepted (and restored), an
    unknown key is YL_ERR_ARG; no GPU needed."""
    for key, value, default in (("gemm", 0, 1), ("gemm_tc", 1, 0), ("gemm_tc_min", 128, 96),
                                ("gemm_f16_min", 0, 16), ("gemm_f16_min", 32, 16)):
        yl.config_set(key, value)
        yl.config_set(key, default)
    import pytest
    with pytest.raises(yl.YlError) as e:
        yl.config_set("no_such_option", 1)
    assert e.value.code == -1
