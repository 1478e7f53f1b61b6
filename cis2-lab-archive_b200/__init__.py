"""cis2-lab-archive_b200 -- B200 (sm_100a) CIS-2 deterministic fp32 decoder.

Python ctypes shim over libcis2b.so (C ABI in include/cis2b.h) for lab
harnesses: the reference's harnesses drive the decoder through a subprocess
and parse its stdout (code/cis2-llm/server/app/runner.py:48-88); this module
offers the same load / generate / witness surface in-process, and the
`cis2b_ref` binary next to it prints the reference's stdout lines.

The package imports no CUDA Python bindings; the compute path is the native
library only.  If libcis2b.so is missing, every entry point raises instead of
falling back to anything else.
"""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT_DIR = os.path.dirname(PKG_DIR)
LIB_PATH = os.path.join(PKG_DIR, "libcis2b.so")
CLI_PATH = os.path.join(PKG_DIR, "cis2b_ref")
HEADER_PATH = os.path.join(ROOT_DIR, "include", "cis2b.h")

SEQUENTIAL, TREE = 0, 1
OP_MATMUL_DECODE = 2  # CIS2B_OP_MATMUL_DECODE: sequential order through the decode-step kernel
OP_MATMUL_DECODE_TREE = 3  # CIS2B_OP_MATMUL_DECODE_TREE: tree order through the decode-step kernel
PINNED_FUNCS = {"exp": 0, "sin": 1, "cos": 2, "ln": 3, "silu": 4, "rsqrt": 5}


class Cis2Error(RuntimeError):
    """A libcis2b call returned a non-zero status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"cis2b error {code}: {msg}")
        self.code = code


class _Opts(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int32), ("reduction", ctypes.c_int32),
                ("max_positions", ctypes.c_int32), ("arch_gate", ctypes.c_int32),
                ("reserved", ctypes.c_int32 * 4)]


# CIS2B_GATE_*: "reference" is the Rust reference's architecture gate
# (model_type llama or qwen2); "qwen3-port" also admits model_type qwen3, as
# the lab's Qwen3 port of the C++ path does.
ARCH_GATES = {"reference": 0, "qwen3-port": 1}


class _Sample(ctypes.Structure):
    _fields_ = [("seed", ctypes.c_uint64), ("temperature", ctypes.c_float), ("top_p", ctypes.c_float),
                ("scheme", ctypes.c_uint32), ("top_k", ctypes.c_uint32)]


SAMPLE_E23, SAMPLE_GUMBEL = 0, 1  # CIS2B_SAMPLE_*


def _sample_struct(sample: dict) -> _Sample:
    """sample: {"seed", "temperature", "top_p"} plus "scheme": "e23" (default)
    or "gumbel" (the CIS2-SAMPLE-1 clause, which also takes "top_k")."""
    scheme = SAMPLE_GUMBEL if sample.get("scheme", "e23") == "gumbel" else SAMPLE_E23
    return _Sample(int(sample["seed"]), float(sample["temperature"]), float(sample["top_p"]), scheme,
                   int(sample.get("top_k", 0)))


class _Info(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int32), ("intermediate", ctypes.c_int32), ("n_layers", ctypes.c_int32),
                ("n_heads", ctypes.c_int32), ("n_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("vocab", ctypes.c_int32), ("tied", ctypes.c_int32), ("rms_norm_eps", ctypes.c_float),
                ("rope_theta", ctypes.c_double), ("reduction", ctypes.c_int32),
                ("max_positions", ctypes.c_int32),
                ("weights_sha256", ctypes.c_uint8 * 32), ("tokenizer_sha256", ctypes.c_uint8 * 32),
                ("config_sha256", ctypes.c_uint8 * 32), ("table_digest", ctypes.c_uint8 * 32),
                ("inv_freq_table_digest", ctypes.c_uint8 * 32)]


class _Timing(ctypes.Structure):
    _fields_ = [("total_ms", ctypes.c_double), ("prefill_ms", ctypes.c_double),
                ("decode_ms", ctypes.c_double), ("witness_tail_ms", ctypes.c_double),
                ("kernel_launches", ctypes.c_int64), ("h2d_bytes", ctypes.c_int64),
                ("d2h_bytes", ctypes.c_int64)]


class _KTime(ctypes.Structure):
    _fields_ = [("launches", ctypes.c_int64), ("total_ms", ctypes.c_double)]


PROF_CLASSES = {"lm_head": 1, "layer_gemm": 2, "attention": 4, "witness": 8}


_lib = None


def lib() -> ctypes.CDLL:
    """The loaded libcis2b.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is not built: run `make -C {PKG_DIR}` "
                           "(or __graft_entry__.build()); there is no fallback path")
    L = ctypes.CDLL(LIB_PATH)
    P, I32, U32, SZ = ctypes.c_void_p, ctypes.c_int32, ctypes.c_uint32, ctypes.c_size_t
    L.cis2b_last_error.restype = ctypes.c_char_p
    L.cis2b_load.argtypes = [ctypes.c_char_p, ctypes.POINTER(_Opts), ctypes.POINTER(P)]
    L.cis2b_info_get.argtypes = [P, ctypes.POINTER(_Info)]
    L.cis2b_generate.argtypes = [P, P, P, U32, U32, ctypes.POINTER(_Sample), P, P, P, P]
    L.cis2b_verify.argtypes = [P, P, P, U32, P, U32, ctypes.POINTER(_Sample), P, P, P, P, P]
    L.cis2b_last_timing.argtypes = [P, ctypes.POINTER(_Timing)]
    L.cis2b_logits.argtypes = [P, P, U32, U32, P]
    L.cis2b_profile.argtypes = [P, U32]
    L.cis2b_profile_read.argtypes = [P, U32, ctypes.POINTER(_KTime)]
    L.cis2b_free.argtypes = [P]
    L.cis2b_free.restype = None
    L.cis2b_op_pinned_map.argtypes = [I32, I32, P, P, SZ]
    L.cis2b_op_matmul.argtypes = [I32, P, P, I32, I32, I32, I32, P]
    L.cis2b_op_sha256_stream.argtypes = [I32, P, SZ, P, U32, U32, P]
    L.cis2b_op_argmax.argtypes = [I32, P, I32, I32, P]
    L.cis2b_op_sample.argtypes = [I32, P, I32, ctypes.c_float, ctypes.c_float, ctypes.c_uint64,
                                  ctypes.c_uint64, ctypes.POINTER(U32)]
    L.cis2b_op_sample_gumbel.argtypes = [I32, P, I32, ctypes.c_float, U32, ctypes.c_float, ctypes.c_uint64, U32,
                                         ctypes.POINTER(U32)]
    L.cis2b_op_sample_static.argtypes = [I32, P, I32, ctypes.c_float, ctypes.c_float, ctypes.c_uint64,
                                         ctypes.c_uint64, P, P]
    _lib = L
    return L


def header_symbols() -> list[str]:
    """Every function include/cis2b.h declares."""
    with open(HEADER_PATH) as f:
        text = f.read()
    return sorted(set(re.findall(r"^\s*(?:int|void|const char \*)\s*\*?\s*(cis2b_\w+)\s*\(", text, re.M)))


def _check(rc: int) -> None:
    if rc != 0:
        raise Cis2Error(rc, lib().cis2b_last_error().decode(errors="replace"))


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


class Model:
    """One loaded model on one device (reference: verify3 cis2_model_load)."""

    def __init__(self, weights_dir: str, device: int = 0, reduction: str | int = "sequential",
                 max_positions: int = 0, arch_gate: str | int = "reference"):
        red = {"sequential": SEQUENTIAL, "tree": TREE}.get(reduction, reduction)
        o = _Opts(device=device, reduction=int(red), max_positions=max_positions,
                  arch_gate=int(ARCH_GATES.get(arch_gate, arch_gate)))
        h = ctypes.c_void_p()
        _check(lib().cis2b_load(weights_dir.encode(), ctypes.byref(o), ctypes.byref(h)))
        self._h = h
        inf = _Info()
        _check(lib().cis2b_info_get(self._h, ctypes.byref(inf)))
        self.info = {k: (bytes(getattr(inf, k)) if isinstance(getattr(inf, k), ctypes.Array) else getattr(inf, k))
                     for k, _ in _Info._fields_}
        self.vocab = inf.vocab

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().cis2b_free(self._h)
            self._h = None

    __del__ = close

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def generate(self, prompts, gen: int, sample: dict | None = None, step_digests: bool = True) -> dict:
        rows = [np.asarray(p, dtype=np.uint32).ravel() for p in prompts]
        lens = np.array([len(r) for r in rows], dtype=np.uint32)
        flat = np.ascontiguousarray(np.concatenate(rows) if rows else np.zeros(0, np.uint32))
        n = len(rows)
        toks = np.zeros((n, gen), dtype=np.uint32)
        steps = np.zeros((n, gen, 32), dtype=np.uint8) if step_digests else None
        wit = np.zeros((n, 32), dtype=np.uint8)
        arg = np.zeros((n, 32), dtype=np.uint8)
        smp = ctypes.byref(_sample_struct(sample)) if sample else None
        _check(lib().cis2b_generate(self._h, _ptr(flat), _ptr(lens), n, gen, smp, _ptr(toks), _ptr(steps),
                                    _ptr(wit), _ptr(arg)))
        return {"tokens": toks, "step_digests": steps, "witness": wit, "argmax": arg}

    def verify(self, prompts, claimed, sample: dict | None = None, step_digests: bool = True) -> dict:
        """Teacher-forced receipt verification: claimed[i] is sequence i's
        generated id list (all the same length).  Returns the recomputed
        tokens, first_mismatch per sequence (-1 = none) and the digests."""
        rows = [np.asarray(p, dtype=np.uint32).ravel() for p in prompts]
        lens = np.array([len(r) for r in rows], dtype=np.uint32)
        flat = np.ascontiguousarray(np.concatenate(rows) if rows else np.zeros(0, np.uint32))
        cl = np.ascontiguousarray(np.asarray(claimed, dtype=np.uint32).reshape(len(rows), -1))
        n, gen = cl.shape
        toks = np.zeros((n, gen), dtype=np.uint32)
        first = np.zeros(n, dtype=np.int32)
        steps = np.zeros((n, gen, 32), dtype=np.uint8) if step_digests else None
        wit = np.zeros((n, 32), dtype=np.uint8)
        arg = np.zeros((n, 32), dtype=np.uint8)
        smp = ctypes.byref(_sample_struct(sample)) if sample else None
        _check(lib().cis2b_verify(self._h, _ptr(flat), _ptr(lens), n, _ptr(cl), gen, smp, _ptr(toks), _ptr(first),
                                  _ptr(steps), _ptr(wit), _ptr(arg)))
        return {"tokens": toks, "first_mismatch": first, "step_digests": steps, "witness": wit, "argmax": arg}

    def timing(self) -> dict:
        t = _Timing()
        _check(lib().cis2b_last_timing(self._h, ctypes.byref(t)))
        return {k: getattr(t, k) for k, _ in _Timing._fields_}

    def profile(self, classes) -> None:
        """Time every launch of the named kernel classes (see PROF_CLASSES)."""
        mask = 0
        for c in classes:
            mask |= PROF_CLASSES[c]
        _check(lib().cis2b_profile(self._h, mask))

    def profile_read(self, cls: str) -> dict:
        k = _KTime()
        _check(lib().cis2b_profile_read(self._h, PROF_CLASSES[cls], ctypes.byref(k)))
        return {"launches": k.launches, "total_ms": k.total_ms}

    def logits(self, ids, n_prompt: int, n_rows: int) -> np.ndarray:
        ids = np.ascontiguousarray(np.asarray(ids, dtype=np.uint32))
        out = np.zeros((n_rows, self.vocab), dtype=np.float32)
        _check(lib().cis2b_logits(self._h, _ptr(ids), n_prompt, n_rows, _ptr(out)))
        return out


# ---------------------------------------------------------------- kernel entry points

def pinned_map(fn: str | int, x: np.ndarray, device: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    _check(lib().cis2b_op_pinned_map(device, PINNED_FUNCS.get(fn, fn), _ptr(x), _ptr(y), x.size))
    return y


def matmul(W: np.ndarray, X: np.ndarray, tree: bool = False, device: int = 0, decode: bool = False) -> np.ndarray:
    """Y = X @ widen(W).T in the pinned order.  decode=True runs it through
    the few-row kernel of the decode steps (tree order needs k % 32 == 0)."""
    W = np.ascontiguousarray(W, dtype=np.uint16)
    X = np.ascontiguousarray(X, dtype=np.float32)
    rows, k = X.shape
    Y = np.zeros((rows, W.shape[0]), dtype=np.float32)
    if decode:
        mode = OP_MATMUL_DECODE_TREE if tree else OP_MATMUL_DECODE
    else:
        mode = TREE if tree else SEQUENTIAL
    _check(lib().cis2b_op_matmul(device, _ptr(W), _ptr(X), rows, W.shape[0], k, mode, _ptr(Y)))
    return Y


def sha256_stream(prefix: bytes, words: np.ndarray, chunk_words: int, device: int = 0) -> np.ndarray:
    words = np.ascontiguousarray(words, dtype=np.uint32)
    n_chunks = words.size // chunk_words if chunk_words else 0
    pre = np.frombuffer(prefix, dtype=np.uint8).copy() if prefix else None
    out = np.zeros((max(n_chunks, 1), 32), dtype=np.uint8)
    _check(lib().cis2b_op_sha256_stream(device, _ptr(pre), len(prefix), _ptr(words), chunk_words, n_chunks,
                                        _ptr(out)))
    return out


def argmax(logits: np.ndarray, device: int = 0) -> np.ndarray:
    """First index of the strict maximum of each row (the decode steps' kernel)."""
    x = np.ascontiguousarray(np.atleast_2d(logits), dtype=np.float32)
    out = np.zeros(x.shape[0], dtype=np.uint32)
    _check(lib().cis2b_op_argmax(device, _ptr(x), x.shape[0], x.shape[1], _ptr(out)))
    return out


def sample(logits: np.ndarray, temperature: float, top_p: float, seed: int, position: int,
           device: int = 0) -> int:
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    out = ctypes.c_uint32()
    _check(lib().cis2b_op_sample(device, _ptr(logits), logits.size, temperature, top_p, seed, position,
                                 ctypes.byref(out)))
    return int(out.value)


def sample_gumbel(logits: np.ndarray, temperature: float, top_k: int, top_p: float, seed: int, step: int,
                  device: int = 0) -> int:
    """One seeded Gumbel-max (CIS2-SAMPLE-1) draw on the device."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    out = ctypes.c_uint32()
    _check(lib().cis2b_op_sample_gumbel(device, _ptr(logits), logits.size, temperature, top_k, top_p, seed, step,
                                        ctypes.byref(out)))
    return int(out.value)
