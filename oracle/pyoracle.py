"""oracle/pyoracle.py -- TEST INFRASTRUCTURE ONLY.

Python access to the two CPU checkers:
  * `PortOracle`: ctypes wrapper around oracle/libcis2oracle.so, our C11
    restatement of the CIS-2 path (oracle/cis2_oracle.c);
  * `run_refdrv`: runs the reference's own C++ port (compiled from the
    reference sources into oracle/_ref by oracle/Makefile) through
    oracle/refdrv.cpp and parses its JSON lines.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
this module, and only as the checker / the timed CPU arm.
"""
from __future__ import annotations

import ctypes
import hashlib
import json
import os
import struct
import subprocess
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libcis2oracle.so")
REF_DIR = os.path.join(HERE, "_ref")

SLOTS = ["input_layernorm.weight", "post_attention_layernorm.weight", "self_attn.q_proj.weight",
         "self_attn.k_proj.weight", "self_attn.v_proj.weight", "self_attn.o_proj.weight",
         "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight",
         "self_attn.q_norm.weight", "self_attn.k_norm.weight", "self_attn.q_proj.bias",
         "self_attn.k_proj.bias", "self_attn.v_proj.bias"]


class _Cfg(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int32), ("inter", ctypes.c_int32), ("n_layers", ctypes.c_int32),
                ("n_heads", ctypes.c_int32), ("n_kv_heads", ctypes.c_int32),
                ("head_dim", ctypes.c_int32), ("vocab", ctypes.c_int32), ("eps", ctypes.c_float),
                ("rope_theta", ctypes.c_double), ("tied", ctypes.c_int32), ("tree", ctypes.c_int32)]


class _Sample(ctypes.Structure):
    _fields_ = [("enabled", ctypes.c_int32), ("seed", ctypes.c_uint64),
                ("temperature", ctypes.c_float), ("top_p", ctypes.c_float), ("top_k", ctypes.c_uint32)]


def sample_struct(sample: dict | None) -> _Sample:
    """sample: None (greedy) or {"seed", "temperature", "top_p"} plus
    "scheme": "e23" (default) or "gumbel" (the CIS2-SAMPLE-1 clause, with "top_k")."""
    if not sample:
        return _Sample(0, 0, 0.8, 0.95, 0)
    scheme = 2 if sample.get("scheme", "e23") == "gumbel" else 1
    return _Sample(scheme, int(sample["seed"]), float(sample["temperature"]), float(sample["top_p"]),
                   int(sample.get("top_k", 0)))


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            subprocess.run(["make", "-s", "-C", HERE, "port"], check=True)
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.c_void_p
        L.cis2o_model_new.restype = P
        L.cis2o_model_new.argtypes = [ctypes.POINTER(_Cfg), P, P, P, ctypes.POINTER(P)]
        L.cis2o_model_free.argtypes = [P]
        L.cis2o_generate.argtypes = [P, P, P, ctypes.c_uint32, ctypes.c_uint32,
                                     ctypes.POINTER(_Sample), P, P, P, P, P, ctypes.c_char_p]
        L.cis2o_logits.argtypes = [P, P, ctypes.c_uint32, ctypes.c_uint32, P]
        L.cis2o_inv_freq.argtypes = [P, P, P]
        L.cis2o_table_digest.argtypes = [P]
        for f in ("exp", "sin", "cos", "ln", "silu", "rsqrt"):
            fn = getattr(L, "cis2o_" + f)
            fn.restype = ctypes.c_float
            fn.argtypes = [ctypes.c_float]
        L.cis2o_map.argtypes = [ctypes.c_int32, P, P, ctypes.c_size_t]
        L.cis2o_dot.restype = ctypes.c_float
        L.cis2o_dot.argtypes = [P, P, ctypes.c_int32, ctypes.c_int32]
        L.cis2o_sum.restype = ctypes.c_float
        L.cis2o_sum.argtypes = [P, ctypes.c_int32, ctypes.c_int32]
        L.cis2o_matmul_bf16.argtypes = [P, P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                        ctypes.c_int32, P]
        L.cis2o_softmax.argtypes = [P, ctypes.c_int32, ctypes.c_int32]
        L.cis2o_argmax.restype = ctypes.c_uint32
        L.cis2o_argmax.argtypes = [P, ctypes.c_int32]
        L.cis2o_math_sweep.restype = ctypes.c_size_t
        L.cis2o_math_sweep.argtypes = [P]
        L.cis2o_murmur3_32.restype = ctypes.c_uint32
        L.cis2o_murmur3_32.argtypes = [P, ctypes.c_size_t, ctypes.c_uint32]
        L.cis2o_gumbel_noise.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, P, P, P]
        L.cis2o_sample_gumbel.restype = ctypes.c_uint32
        L.cis2o_sample_gumbel.argtypes = [P, ctypes.c_int32, ctypes.c_float, ctypes.c_uint32, ctypes.c_float,
                                          ctypes.c_uint64, ctypes.c_uint32, P]
        L.cis2o_sample_pinned.restype = ctypes.c_uint32
        L.cis2o_sample_pinned.argtypes = [P, ctypes.c_int32, ctypes.c_float, ctypes.c_float,
                                          ctypes.c_uint64, ctypes.c_uint64]
        L.cis2o_rng_word.restype = ctypes.c_uint64
        L.cis2o_rng_word.argtypes = [ctypes.c_uint64, ctypes.c_uint64]
        L.cis2o_sha256.argtypes = [P, ctypes.c_size_t, P]
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


# ---------------------------------------------------------------- artifacts

def read_safetensors(path: str) -> dict[str, np.ndarray]:
    """name -> uint16 array (bf16 bits), memory-mapped."""
    with open(path, "rb") as f:
        (hlen,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(hlen))
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    base = 8 + hlen
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        assert info["dtype"] == "BF16", (name, info["dtype"])
        b, e = info["data_offsets"]
        out[name] = np.frombuffer(mm, dtype="<u2", count=(e - b) // 2, offset=base + b).reshape(
            info["shape"])
    return out


def read_config(weights_dir: str) -> dict:
    with open(os.path.join(weights_dir, "config.json")) as f:
        return json.load(f)


def artifact_hashes(weights_dir: str) -> bytes:
    """weights_sha256 || tokenizer_sha256 || config_sha256 (raw, 96 bytes)."""
    out = b""
    for fn in ("model.safetensors", "tokenizer.json", "config.json"):
        h = hashlib.sha256()
        with open(os.path.join(weights_dir, fn), "rb") as f:
            for chunk in iter(lambda: f.read(1 << 22), b""):
                h.update(chunk)
        out += h.digest()
    return out


def _flatten_prompts(prompts) -> tuple[np.ndarray, np.ndarray]:
    rows = [np.asarray(p, dtype=np.uint32).ravel() for p in prompts]
    lens = np.array([len(r) for r in rows], dtype=np.uint32)
    flat = np.ascontiguousarray(np.concatenate(rows) if rows else np.zeros(0, np.uint32))
    return flat, lens


class PortOracle:
    """Our C restatement bound to one weights directory and reduction mode."""

    def __init__(self, weights_dir: str, tree: bool = False, hashes: bytes | None = None):
        self.dir = weights_dir
        cfg = read_config(weights_dir)
        self.cfg = cfg
        self.t = read_safetensors(os.path.join(weights_dir, "model.safetensors"))
        H = int(cfg["hidden_size"])
        heads = int(cfg["num_attention_heads"])
        hd = int(cfg.get("head_dim", H // heads))
        tied = bool(cfg.get("tie_word_embeddings", True))
        c = _Cfg(hidden=H, inter=int(cfg["intermediate_size"]), n_layers=int(cfg["num_hidden_layers"]),
                 n_heads=heads, n_kv_heads=int(cfg["num_key_value_heads"]), head_dim=hd,
                 vocab=int(cfg["vocab_size"]), eps=float(np.float32(cfg["rms_norm_eps"])),
                 rope_theta=float(cfg["rope_theta"]), tied=1 if tied else 0, tree=1 if tree else 0)
        self.c = c
        self.vocab = c.vocab
        L = c.n_layers
        ptrs = (ctypes.c_void_p * (L * len(SLOTS)))()
        for li in range(L):
            for si, s in enumerate(SLOTS):
                a = self.t.get(f"model.layers.{li}.{s}")
                ptrs[li * len(SLOTS) + si] = None if a is None else _ptr(a)
        self._ptrs = ptrs
        lm = None if tied else _ptr(self.t["lm_head.weight"])
        self.h = lib().cis2o_model_new(ctypes.byref(c), _ptr(self.t["model.embed_tokens.weight"]),
                                       _ptr(self.t["model.norm.weight"]), lm, ptrs)
        self.hashes = hashes if hashes is not None else artifact_hashes(weights_dir)

    def __del__(self):
        if getattr(self, "h", None):
            lib().cis2o_model_free(self.h)
            self.h = None

    def generate(self, prompts, gen: int, sample: dict | None = None, trace_path: str | None = None,
                 step_digests: bool = True) -> dict:
        flat, lens = _flatten_prompts(prompts)
        n = len(lens)
        toks = np.zeros((n, gen), dtype=np.uint32)
        steps = np.zeros((n, gen, 32), dtype=np.uint8) if step_digests else None
        wit = np.zeros((n, 32), dtype=np.uint8)
        arg = np.zeros((n, 32), dtype=np.uint8)
        s = sample_struct(sample)
        hdr = np.frombuffer(self.hashes, dtype=np.uint8).copy()
        rc = lib().cis2o_generate(self.h, _ptr(flat), _ptr(lens), n, gen, ctypes.byref(s), _ptr(hdr),
                                  _ptr(toks), None if steps is None else _ptr(steps), _ptr(wit),
                                  _ptr(arg), trace_path.encode() if trace_path else None)
        assert rc == 0
        return {"tokens": toks, "step_digests": steps, "witness": wit, "argmax": arg}

    def logits(self, ids, n_prompt: int, n_rows: int) -> np.ndarray:
        ids = np.ascontiguousarray(np.asarray(ids, dtype=np.uint32))
        out = np.zeros((n_rows, self.vocab), dtype=np.float32)
        rc = lib().cis2o_logits(self.h, _ptr(ids), n_prompt, n_rows, _ptr(out))
        assert rc == 0
        return out

    def inv_freq(self) -> tuple[np.ndarray, bytes]:
        out = np.zeros(self.c.head_dim // 2, dtype=np.float32)
        d = np.zeros(32, dtype=np.uint8)
        lib().cis2o_inv_freq(self.h, _ptr(out), _ptr(d))
        return out, d.tobytes()


def table_digest() -> bytes:
    d = np.zeros(32, dtype=np.uint8)
    lib().cis2o_table_digest(_ptr(d))
    return d.tobytes()


def pinned_map(fn: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().cis2o_map(fn, _ptr(x), _ptr(y), x.size)
    return y


def matmul_bf16(W: np.ndarray, X: np.ndarray, tree: bool = False) -> np.ndarray:
    W = np.ascontiguousarray(W, dtype=np.uint16)
    X = np.ascontiguousarray(X, dtype=np.float32)
    rows, k = X.shape
    n = W.shape[0]
    Y = np.zeros((rows, n), dtype=np.float32)
    lib().cis2o_matmul_bf16(_ptr(W), _ptr(X), rows, n, k, 1 if tree else 0, _ptr(Y))
    return Y


# ---------------------------------------------------------------- reference binary

def refdrv_path(qwen3: bool = False, tree: bool = False) -> str:
    name = "refdrv" + ("_qwen3" if qwen3 else "") + ("_tree" if tree else "")
    return os.path.join(REF_DIR, name)


def have_refdrv() -> bool:
    return os.path.exists(refdrv_path())


def run_refdrv(weights_dir: str, prompts, gen: int, tree: bool = False, sample: dict | None = None,
               step_digests: bool = False, qwen3: bool | None = None, timeout: float | None = None,
               workers: int = 1) -> list[dict]:
    """Runs the reference port on each prompt; returns one dict per sequence."""
    if qwen3 is None:
        qwen3 = "head_dim" in read_config(weights_dir)
    exe = refdrv_path(qwen3=qwen3, tree=tree)
    prompts = [np.asarray(p, dtype=np.uint32).ravel() for p in prompts]
    with tempfile.TemporaryDirectory() as td:
        ids_path = os.path.join(td, "ids.txt")
        with open(ids_path, "w") as f:
            for p in prompts:
                f.write(" ".join(str(int(v)) for v in p) + "\n")
        n = len(prompts)
        workers = max(1, min(workers, n))
        chunks = [(i * n // workers, (i + 1) * n // workers) for i in range(workers)]
        procs = []
        for ci, (a, b) in enumerate(chunks):
            cmd = [exe, "--weights-dir", weights_dir, "--ids", ids_path, "--gen-toks", str(gen),
                   "--first", str(a), "--count", str(b - a), "--out", os.path.join(td, f"o{ci}.jsonl")]
            if step_digests:
                cmd.append("--step-digests")
            if sample:
                cmd += ["--sample", str(int(sample["seed"])), repr(float(sample["temperature"])),
                        repr(float(sample["top_p"]))]
            procs.append(subprocess.Popen(cmd, stderr=subprocess.DEVNULL))
        for p in procs:
            if p.wait(timeout=timeout) != 0:
                raise RuntimeError(f"refdrv failed rc={p.returncode}")
        out = []
        for ci in range(len(chunks)):
            with open(os.path.join(td, f"o{ci}.jsonl")) as f:
                for line in f:
                    d = json.loads(line)
                    if d["kind"] == "seq":
                        out.append(d)
        out.sort(key=lambda d: d["seq"])
        return out


def gumbel_noise(seed: int, step: int, index: int) -> tuple[int, int, int]:
    """(hash, u bits, g bits) of one (seed, step, index) of the CIS2-SAMPLE-1 noise."""
    h = ctypes.c_uint32()
    u = ctypes.c_float()
    g = ctypes.c_float()
    lib().cis2o_gumbel_noise(seed, step, index, ctypes.byref(h), ctypes.byref(u), ctypes.byref(g))
    ub = np.array([u.value], dtype=np.float32).view(np.uint32)[0]
    gb = np.array([g.value], dtype=np.float32).view(np.uint32)[0]
    return int(h.value), int(ub), int(gb)


def sample_gumbel(logits, temperature: float, top_k: int, top_p: float, seed: int, step: int):
    """(next_id, z[V]) of one CIS2-SAMPLE-1 draw."""
    x = np.ascontiguousarray(logits, dtype=np.float32)
    z = np.zeros_like(x)
    r = lib().cis2o_sample_gumbel(_ptr(x), x.size, temperature, top_k, top_p, seed, step, _ptr(z))
    return int(r), z


def math_sweep_inputs() -> np.ndarray:
    """The pinned-function sweep points (oracle/math_sweep.h), fp32."""
    n = lib().cis2o_math_sweep(None)
    x = np.zeros(n, dtype=np.float32)
    lib().cis2o_math_sweep(_ptr(x))
    return x


MATH_FUNCS = ("exp", "sin", "cos", "ln", "silu", "rsqrt")


def sweep_digests(x: np.ndarray, outs: dict) -> dict:
    """Digests of a sweep's outputs: NaNs canonicalised to 0x7FC00000 (their
    encoding differs between x86 SSE and the GPU for NaNs produced by
    arithmetic), plus the set of indices that are NaN."""
    import hashlib
    res = {"n": int(x.size), "inputs_sha256": hashlib.sha256(x.view(np.uint32).astype("<u4").tobytes()).hexdigest()}
    for f in MATH_FUNCS:
        y = np.ascontiguousarray(outs[f], dtype=np.float32).view(np.uint32).copy()
        nan = np.isnan(outs[f])
        y[nan] = 0x7FC00000
        res[f] = {"canon_sha256": hashlib.sha256(y.astype("<u4").tobytes()).hexdigest(),
                  "nan_count": int(nan.sum()),
                  "nan_index_sha256": hashlib.sha256(np.nonzero(nan)[0].astype("<u4").tobytes()).hexdigest()}
    return res


def read_refmath(path: str) -> tuple[np.ndarray, dict]:
    """Reads oracle/_ref/refmath output: (x, {fn: y})."""
    raw = open(path, "rb").read()
    assert raw[:8] == b"CIS2MSW1"
    n = int(np.frombuffer(raw[8:12], dtype="<u4")[0])
    rec = np.frombuffer(raw[12:12 + 28 * n], dtype="<u4").reshape(n, 7)
    x = rec[:, 0].copy().view(np.float32)
    return x, {f: rec[:, i + 1].copy().view(np.float32) for i, f in enumerate(MATH_FUNCS)}
