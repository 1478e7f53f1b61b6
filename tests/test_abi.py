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


# ---------------------------------------------------------------- the reference's refusal suite

def reference_root() -> str | None:
    """The reference checkout: $CIS2_REFERENCE_ROOT, else `reference` beside
    this repository; None when neither exists (as on a GPU box)."""
    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    root = os.environ.get("CIS2_REFERENCE_ROOT") or os.path.join(os.path.dirname(here), "reference")
    return root if os.path.isdir(os.path.join(root, "code", "cis2-fp")) else None


def rust_gate_reason(cfg: dict) -> str | None:
    """The Rust reference's gate restated (code/cis2-fp/src/main.rs:545-644):
    the refusal reason it prints, or None when it admits the config."""
    def u64(v):
        return v if isinstance(v, int) and not isinstance(v, bool) and v >= 0 else None

    mt = cfg.get("model_type")
    if isinstance(mt, str) and mt not in ("llama", "qwen2"):
        return f'model_type="{mt}" is not in the CIS-2 specified subset ["llama", "qwen2"]'
    dt = cfg.get("torch_dtype")
    if isinstance(dt, str) and dt != "bfloat16":
        return f'torch_dtype="{dt}"; CIS-2 pins bf16-on-disk weights (\u00a73.5)'
    h, nh = u64(cfg.get("hidden_size")), u64(cfg.get("num_attention_heads"))
    if h is not None and nh is not None:
        if nh == 0:
            return "num_attention_heads=0"
        derived = h // nh
        ex = u64(cfg.get("head_dim"))
        if ex is not None and ex != derived:
            return (f"config declares head_dim={ex} but this implementation derives "
                    f"hidden_size/num_attention_heads={derived}; the decode path uses the derived value, "
                    "so the explicit one would be silently ignored")
        if derived % 2:
            return f"derived head_dim={derived} is odd; RoPE pairs require even"
    prf = cfg.get("partial_rotary_factor")
    if isinstance(prf, (int, float)) and not isinstance(prf, bool) and prf != 1.0:
        return f"partial_rotary_factor={prf!r}; only full rotary is specified"
    if cfg.get("rope_scaling") is not None:
        return "rope_scaling is set; only unscaled RoPE is specified"
    if cfg.get("use_sliding_window") is True:
        return "use_sliding_window=true; only full causal attention is specified"
    if cfg.get("quantization_config") is not None:
        return "quantization_config is present; CIS-2 reads unquantized bf16 weights"
    for k in ("attention_multiplier", "embedding_multiplier", "residual_multiplier", "logits_scaling",
              "attn_logit_softcapping", "final_logit_softcapping", "query_pre_attn_scalar"):
        if cfg.get(k) is not None:
            return (f"{k} is set; this implementation hardcodes rsqrt(head_dim) attention scaling and no logit "
                    "scaling, so the result would be silently wrong")
    for k in ("num_local_experts", "num_experts", "n_routed_experts", "moe_intermediate_size"):
        if cfg.get(k) is not None:
            return f"{k} is set; MoE routing is not specified"
    return None


def refusal_fixture_dirs() -> list[str]:
    root = reference_root()
    if root is None:
        return []
    base = os.path.join(root, "code", "cis2-fp", "tests", "fixtures")
    return sorted(os.path.join(base, s, d) for s in ("refusal", "refusal-deep")
                  if os.path.isdir(os.path.join(base, s)) for d in os.listdir(os.path.join(base, s)))


@pytest.mark.skipif(reference_root() is None, reason="reference checkout not present")
def test_reference_refusal_suite(pkg):
    """code/cis2-fp/tests/fixtures/run_refusal_suite.sh run through cis2b_ref:
    every checkpoint the Rust gate refuses is refused by name (exit 2, the
    reference's reason text, no digest); the ones it admits pass the gate
    and then fail on their absent weights (exit 101, as the reference's
    panic does).  The admitted set is exactly qwen2-1.5b: Qwen3 is refused
    by default, like the Rust reference, and admitted only through the
    qwen3-port gate."""
    dirs = refusal_fixture_dirs()
    assert len(dirs) >= 12
    admitted = []
    for d in dirs:
        with open(os.path.join(d, "config.json")) as f:
            cfg = json.load(f)
        want = rust_gate_reason(cfg)
        p = subprocess.run([pkg.CLI_PATH, "--weights-dir", d, "--gen-toks", "1"], capture_output=True, text=True,
                           timeout=60)
        assert "CIS2_REF digest=" not in p.stdout
        if want is None:
            admitted.append(os.path.basename(d))
            assert p.returncode == 101, (d, p.returncode, p.stderr)
            continue
        assert p.returncode == 2, (d, p.returncode, p.stderr)
        lines = p.stderr.splitlines()
        assert lines[0] == "CIS2_REF_UNSUPPORTED reason=" + want, (d, lines[0], want)
        assert lines[1] == "This checkpoint is outside the CIS-2 specified subset; no digest emitted."
        rc, msg, _ = _load_rc(pkg, d)
        assert rc == 3 and msg == want
    assert admitted == ["qwen25-1.5b"]
    q3 = [d for d in dirs if os.path.basename(d) == "qwen3-0.6b-base"][0]
    rc, msg, _ = _load_rc(pkg, q3, arch_gate=1)
    assert rc == 2 and "model.safetensors" in msg  # admitted by the port gate; no weights here
    p = subprocess.run([pkg.CLI_PATH, "--weights-dir", q3, "--gen-toks", "1", "--arch-gate", "qwen3-port"],
                       capture_output=True, text=True, timeout=60)
    assert p.returncode == 101 and "CIS2_REF_UNSUPPORTED" not in p.stderr


def test_qwen3_needs_the_port_gate(pkg, synth, synth_root):
    """A qwen3 config is refused by the default gate with the Rust reason and
    loads through CIS2B_GATE_QWEN3_PORT (up to the device, which this test
    does not need: on a machine without one the load fails after the gate)."""
    d = synth.ensure_model("tiny_qwen3", synth_root)
    rc, msg, _ = _load_rc(pkg, d)
    assert rc == 3 and msg == 'model_type="qwen3" is not in the CIS-2 specified subset ["llama", "qwen2"]'
    rc, msg, h = _load_rc(pkg, d, arch_gate=1)
    assert rc != 3, msg
    if rc == 0:
        pkg.lib().cis2b_free(h)
    rc, msg, _ = _load_rc(pkg, d, arch_gate=2)
    assert rc == 1 and "gate" in msg


def test_config_json_strings_and_numbers(pkg, synth, synth_root, tmp_path):
    """config.json reading: \\u escapes (a surrogate pair included) decode,
    and malformed JSON -- a bad number, a lone surrogate, a raw control
    character -- is an artifact error, never a silent default."""
    d = _copy_model(synth, synth_root, tmp_path)
    base = (d / "config.json").read_text().rstrip().rstrip("}")
    for extra, ok in [(', "note": "caf\\u00e9 \\ud83d\\ude00 \\"q\\" \\/"}', True),
                      (', "note": 1.5e-3}', True),
                      (', "note": 01}', False), (', "note": 1.}', False), (', "note": -}', False),
                      (', "note": "\\ud83d"}', False), (', "note": "a\tb"}', False),
                      (', "note": tru}', False)]:
        (d / "config.json").write_text(base + extra)
        rc, msg, h = _load_rc(pkg, str(d))
        if ok:
            assert rc not in (2, 3), (extra, msg)
            if rc == 0:
                pkg.lib().cis2b_free(h)
        else:
            assert rc == 2 and "config.json" in msg, (extra, rc, msg)


def test_matmul_shapes_reach_every_register_tile(pkg):
    """The bit-exact GEMM shapes (tests/test_gpu_kernels.py SHAPES) reach every
    tile of the register-tiled product; the tile choice is host code, so
    this runs without a device."""
    from test_gpu_kernels import BIG_TILES, SHAPES
    L = pkg.lib()
    L.cis2b_op_gemm_tile.argtypes = [ctypes.c_int32, ctypes.c_int32]
    seen = {int(L.cis2b_op_gemm_tile(m, n)) for m, n, _ in SHAPES if m >= 64}
    assert seen == set(range(len(BIG_TILES))), sorted(seen)
    assert L.cis2b_op_gemm_tile(63, 100) == -1


# (rows, n_out) -> the register tile (index into BIG_TILES) that measured fastest,
# or within 5 % of it, on B200 for the workloads' products (fp32 panels, 32-deep
# k stages): decode steps of C5 (256 rows) and C3 (300 rows), their lm_head, and
# the C2 prompt pass (4,096 rows).
MEASURED_TILE_CHOICES = {
    (256, 960): {2, 3}, (256, 576): {3, 4}, (256, 3072): {2, 3}, (300, 2304): {3}, (300, 768): {2, 3},
    (300, 6144): {2, 3}, (300, 32000): {1, 2}, (256, 49152): {0, 1}, (4096, 3072): {0, 1},
}


@pytest.mark.parametrize("rows,n", sorted(MEASURED_TILE_CHOICES))
def test_tile_choice_matches_measured_best(rows, n, pkg):
    """gemm_big_choice's cost model picks, for the workloads' product shapes,
    a tile that measured fastest (or within 5 %) in the standalone sweep."""
    L = pkg.lib()
    L.cis2b_op_gemm_tile.argtypes = [ctypes.c_int32, ctypes.c_int32]
    assert int(L.cis2b_op_gemm_tile(rows, n)) in MEASURED_TILE_CHOICES[(rows, n)]
