"""CPU checks of the drop-in boundary: the C-ABI library loads, exports every
symbol include/cis2b.h declares, and reports argument / artifact / config
errors as status codes (the reference exits the process instead,
code/cis2-fp/gpu/cis2_model.h:296-360)."""
from __future__ import annotations

import ctypes
import json
import os
import shutil
import subprocess

import numpy as np
import pytest


def test_library_exports_every_header_symbol(pkg):
    L = pkg.lib()
    syms = pkg.header_symbols()
    assert "cis2b_load" in syms and "cis2b_generate" in syms and len(syms) >= 10
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", pkg.LIB_PATH], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert set(syms) <= exported


def test_no_torch_in_library(pkg):
    out = subprocess.run(["ldd", pkg.LIB_PATH], capture_output=True, text=True).stdout
    assert "torch" not in out and "python" not in out


def test_cli_built(pkg):
    assert os.access(pkg.CLI_PATH, os.X_OK)
    r = subprocess.run([pkg.CLI_PATH, "--bogus"], capture_output=True, text=True)
    assert r.returncode == 2 and "unknown CLI argument" in r.stderr


def _load_rc(pkg, path, **kw):
    o = pkg._Opts(**kw)
    h = ctypes.c_void_p()
    rc = pkg.lib().cis2b_load(path.encode(), ctypes.byref(o), ctypes.byref(h))
    return rc, pkg.lib().cis2b_last_error().decode(), h


def test_load_missing_dir_is_io_error(pkg, tmp_path):
    rc, msg, h = _load_rc(pkg, str(tmp_path / "nope"))
    assert rc == 2 and "cannot read" in msg and not h.value


def test_load_rejects_bad_options(pkg, tmp_path):
    rc, msg, _ = _load_rc(pkg, str(tmp_path), reduction=7)
    assert rc == 1 and "reduction" in msg
    rc, msg, _ = _load_rc(pkg, str(tmp_path), max_positions=-1)
    assert rc == 1


def _copy_model(synth, synth_root, tmp_path, name="tiny"):
    src = synth.ensure_model(name, synth_root)
    dst = tmp_path / name
    shutil.copytree(src, dst)
    return dst


def test_load_refuses_bad_configs(pkg, synth, synth_root, tmp_path):
    d = _copy_model(synth, synth_root, tmp_path)
    cfg = json.loads((d / "config.json").read_text())
    for patch, code, word in [({"rope_scaling": {"type": "linear", "factor": 2.0}}, 3, "rope_scaling"),
                              ({"num_key_value_heads": 3}, 3, "num_key_value_heads"),
                              ({"head_dim": 15}, 3, "head_dim")]:
        c = dict(cfg)
        c.update(patch)
        (d / "config.json").write_text(json.dumps(c))
        rc, msg, _ = _load_rc(pkg, str(d))
        assert rc == code and word in msg, (patch, rc, msg)
    # The architecture gate (code/cis2-fp/src/main.rs:545-644).
    for patch, word in [({"model_type": "mistral"}, "model_type"), ({"torch_dtype": "float16"}, "torch_dtype"),
                        ({"head_dim": 32}, "head_dim"), ({"partial_rotary_factor": 0.5}, "partial_rotary_factor"),
                        ({"use_sliding_window": True}, "use_sliding_window"),
                        ({"quantization_config": {"bits": 4}}, "quantization_config"),
                        ({"attention_multiplier": 0.5}, "attention_multiplier"),
                        ({"final_logit_softcapping": 30.0}, "final_logit_softcapping"),
                        ({"num_experts": 8}, "num_experts")]:
        c = dict(cfg)
        c.update(patch)
        (d / "config.json").write_text(json.dumps(c))
        rc, msg, _ = _load_rc(pkg, str(d))
        assert rc == 3 and word in msg, (patch, rc, msg)
    # Null-valued keys and the settings the gate allows pass it.
    c = dict(cfg)
    c.update({"rope_scaling": None, "quantization_config": None, "use_sliding_window": False,
              "partial_rotary_factor": 1.0, "model_type": "qwen2"})
    (d / "config.json").write_text(json.dumps(c))
    rc, msg, _ = _load_rc(pkg, str(d))
    assert rc != 3, msg
    c = dict(cfg)
    del c["vocab_size"]
    (d / "config.json").write_text(json.dumps(c))
    rc, msg, _ = _load_rc(pkg, str(d))
    assert rc == 3
    (d / "config.json").write_text("{not json")
    rc, msg, _ = _load_rc(pkg, str(d))
    assert rc == 2


def test_gate_runs_before_the_weights_are_read(pkg, synth, synth_root, tmp_path):
    """An unsupported checkpoint is refused by name even without its weights
    (code/cis2-fp/src/main.rs:812-823); the CLI prints the reference's
    CIS2_REF_UNSUPPORTED line and exits 2."""
    d = _copy_model(synth, synth_root, tmp_path)
    cfg = json.loads((d / "config.json").read_text())
    cfg["model_type"] = "gemma"
    (d / "config.json").write_text(json.dumps(cfg))
    (d / "model.safetensors").unlink()
    rc, msg, _ = _load_rc(pkg, str(d))
    assert rc == 3 and "model_type" in msg
    ids = tmp_path / "ids.txt"
    ids.write_text("1 2 3\n")
    p = subprocess.run([pkg.CLI_PATH, "--weights-dir", str(d), "--ids", str(ids), "--gen-toks", "2"],
                       capture_output=True, text=True, timeout=60)
    assert p.returncode == 2
    assert p.stderr.startswith("CIS2_REF_UNSUPPORTED reason=model_type="), p.stderr


def test_load_detects_corrupt_weights(pkg, synth, synth_root, tmp_path):
    d = _copy_model(synth, synth_root, tmp_path)
    p = d / "model.safetensors"
    b = bytearray(p.read_bytes())
    (d / "model.safetensors").write_bytes(bytes(b[: len(b) // 2]))  # truncated data section
    rc, msg, _ = _load_rc(pkg, str(d))
    assert rc == 2 and ("byte range" in msg or "header" in msg)
    p.write_bytes(b"\x05")
    rc, msg, _ = _load_rc(pkg, str(d))
    assert rc == 2


def test_op_entry_points_validate_before_device(pkg):
    L = pkg.lib()
    x = np.zeros(4, np.float32)
    assert L.cis2b_op_pinned_map(0, 9, x.ctypes.data, x.ctypes.data, 4) == 1
    assert L.cis2b_op_matmul(0, None, None, 1, 1, 8, 0, None) == 1
    W = np.zeros((2, 12), np.uint16)
    X = np.zeros((1, 12), np.float32)
    Y = np.zeros((1, 2), np.float32)
    assert L.cis2b_op_matmul(0, W.ctypes.data, X.ctypes.data, 1, 2, 12, 0, Y.ctypes.data) == 1
    out = ctypes.c_uint32()
    assert L.cis2b_op_sample(0, x.ctypes.data, 4, ctypes.c_float(0.0), ctypes.c_float(0.9), 1, 1,
                             ctypes.byref(out)) == 1


def test_generate_null_model_is_arg_error(pkg):
    L = pkg.lib()
    assert L.cis2b_generate(None, None, None, 1, 1, None, None, None, None, None) == 1
    assert "NULL" in L.cis2b_last_error().decode()


def test_last_error_is_thread_local(pkg):
    import threading
    L = pkg.lib()
    L.cis2b_generate(None, None, None, 1, 1, None, None, None, None, None)
    seen = {}

    def worker():
        seen["msg"] = L.cis2b_last_error().decode()

    t = threading.Thread(target=worker)
    t.start()
    t.join()
    assert seen["msg"] == ""
