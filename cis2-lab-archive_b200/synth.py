"""Seeded synthetic CIS-2 artifacts: bf16 safetensors, config.json, a stub
tokenizer.json and prompt token ids.

The reference publishes no benchmark data for its decode path; its five
benchmark configurations are model SHAPES with seeded random weights.  This
module is the one place those artifacts are made, so that the CUDA build, the
CPU oracle and the reference's own C++ port all read byte-identical files.

Layout follows what the reference loader expects:
  * tensor names and shapes: code/cis2-fp/gpu/cis2_host.cpp:134-159 (plus the
    Qwen3 q_norm/k_norm tensors of labs/w1x-qwen3/scripts/qwen3-port.diff:139-141);
  * safetensors container (8-byte LE header length, JSON header with
    dtype/shape/data_offsets, raw little-endian data):
    code/cis2-fp/gpu/cis2_model.h:296-326;
  * config keys read: code/cis2-fp/gpu/cis2_host.cpp:104-117 (+ "head_dim",
    qwen3-port.diff:109).

Values: projection/embedding matrices are N(0, 0.02) drawn as float32 from
NumPy's PCG64 (one independent stream per tensor, keyed by the model seed and
the tensor's index in the canonical order), multiplied by 0.02 in float32 and
rounded to bf16 with round-to-nearest-even on the fp32 bit pattern.  All norm
gains are exactly 1.0 (bf16 0x3F80).  Prompt ids are uniform in [0, vocab),
one PCG64 stream per sequence so that sequence i is the same whatever the
total number of sequences.
"""
from __future__ import annotations

import hashlib
import json
import os
import struct
from dataclasses import dataclass, field, asdict

import numpy as np


@dataclass(frozen=True)
class ModelShape:
    name: str
    hidden: int
    inter: int
    layers: int
    heads: int
    kv_heads: int
    vocab: int
    eps: str            # decimal text written into config.json (strtod'd by the loader)
    theta: str          # decimal text written into config.json
    tied: bool
    seed: int
    head_dim: int | None = None   # explicit head_dim key (Qwen3); None = hidden/heads
    qk_norm: bool = False         # per-head q_norm/k_norm tensors (Qwen3)
    qkv_bias: bool = False        # q/k/v bias tensors (Qwen2 family)
    model_type: str = "llama"
    coverage: bool = False        # lm_head rows rebuilt for the tie / subnormal clauses (below)

    @property
    def hd(self) -> int:
        return self.head_dim if self.head_dim is not None else self.hidden // self.heads

    @property
    def q_dim(self) -> int:
        return self.heads * self.hd

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.hd


MODELS: dict[str, ModelShape] = {
    # BASELINE configs 1, 2, 5: SmolLM2-135M shape.
    "smollm2": ModelShape("smollm2", 576, 1536, 30, 9, 3, 49152, "1e-05", "100000", True, 135),
    # llama-160m shape (MHA, untied head).
    "llama160m": ModelShape("llama160m", 768, 3072, 12, 12, 12, 32000, "1e-06", "10000", False, 160),
    # Qwen3-0.6B shape (explicit head_dim 128, QK-norm).
    "qwen3_0p6b": ModelShape("qwen3_0p6b", 1024, 3072, 28, 16, 8, 151936, "1e-06", "1000000", True, 600,
                             head_dim=128, qk_norm=True, model_type="qwen3"),
    # Small shapes for fast parity tests.  Each exercises a different branch.
    "tiny": ModelShape("tiny", 64, 128, 2, 4, 2, 512, "1e-05", "100000", True, 7),
    "tiny_mha_untied": ModelShape("tiny_mha_untied", 96, 160, 2, 3, 3, 384, "1e-06", "10000", False, 8),
    "tiny_qwen3": ModelShape("tiny_qwen3", 64, 96, 2, 4, 2, 640, "1e-06", "1000000", True, 9,
                             head_dim=32, qk_norm=True, model_type="qwen3"),
    "tiny_bias": ModelShape("tiny_bias", 64, 128, 2, 4, 1, 256, "1e-06", "1000000", True, 10,
                            qkv_bias=True, model_type="qwen2"),
    # Mid-size: SmolLM2 widths with fewer layers and a smaller vocab, so the
    # oracle finishes in seconds while the kernels see realistic K and N.
    "mid": ModelShape("mid", 576, 1536, 3, 9, 3, 4096, "1e-05", "100000", True, 11),
    # Constructed coverage vector (labs/w1x-coverage/plans/2026-10-16-w1x-coverage-PLAN.md:8-16):
    # hidden 64, 2 heads (head_dim 32), 2 layers, inter 128, vocab 32, untied.
    "coverage": ModelShape("coverage", 64, 128, 2, 2, 2, 32, "1e-05", "10000", False, 20261016,
                           coverage=True),
}

# The coverage model's clauses.  Rows TIE_A and TIE_B of lm_head are the
# same +-2.0 row, so every step's logits tie exactly between them and the
# strict-first argmax (code/cis2-fp/src/main.rs:1161-1169) must pick TIE_A.
# Row SUB holds one non-zero weight, +-2^-126 (the smallest normal bf16), at
# a column whose final-norm value at the last prompt position lies in
# [0.25, 0.75] in magnitude: its step-0 logit is then a positive subnormal,
# which the pinned FTZ/DAZ environment flushes to +0 before the witness
# hashes it (spec §1.3, code/cis2-fp/gpu/cis2_fpenv.h:62-135).
COVERAGE_TIE_A, COVERAGE_TIE_B, COVERAGE_SUB = 5, 17, 29
COVERAGE_PROMPT_SEED, COVERAGE_PROMPT_LEN = 20261016, 4


@dataclass(frozen=True)
class Workload:
    name: str
    model: str
    n_seq: int          # sequences per GPU (or total, see `sharded_total`)
    prompt_len: int
    gen: int
    prompt_seed: int
    sampled: bool = False
    seed: int = 0
    temperature: float = 0.8
    top_p: float = 0.95
    sharded_total: bool = False   # n_seq is the total over all GPUs


WORKLOADS: dict[str, Workload] = {
    "c1": Workload("c1", "smollm2", 1, 32, 256, 1001),
    "c2": Workload("c2", "smollm2", 64, 64, 256, 1002),
    "c3": Workload("c3", "llama160m", 300, 48, 128, 1003, sharded_total=True),
    "c4": Workload("c4", "qwen3_0p6b", 32, 64, 256, 1004, sampled=True, seed=20261201),
    "c5": Workload("c5", "smollm2", 256, 1024, 1024, 1005, sharded_total=True),
}


# ---------------------------------------------------------------- tensors

def tensor_specs(m: ModelShape) -> list[tuple[str, tuple[int, ...], str]]:
    """Canonical (name, shape, kind) list; kind is 'mat' or 'gain'."""
    H, I, V, QD, KV, HD = m.hidden, m.inter, m.vocab, m.q_dim, m.kv_dim, m.hd
    out: list[tuple[str, tuple[int, ...], str]] = [("model.embed_tokens.weight", (V, H), "mat")]
    for i in range(m.layers):
        p = f"model.layers.{i}."
        out += [
            (p + "input_layernorm.weight", (H,), "gain"),
            (p + "post_attention_layernorm.weight", (H,), "gain"),
            (p + "self_attn.q_proj.weight", (QD, H), "mat"),
            (p + "self_attn.k_proj.weight", (KV, H), "mat"),
            (p + "self_attn.v_proj.weight", (KV, H), "mat"),
            (p + "self_attn.o_proj.weight", (H, QD), "mat"),
            (p + "mlp.gate_proj.weight", (I, H), "mat"),
            (p + "mlp.up_proj.weight", (I, H), "mat"),
            (p + "mlp.down_proj.weight", (H, I), "mat"),
        ]
        if m.qk_norm:
            out += [(p + "self_attn.q_norm.weight", (HD,), "gain"),
                    (p + "self_attn.k_norm.weight", (HD,), "gain")]
        if m.qkv_bias:
            out += [(p + "self_attn.q_proj.bias", (QD,), "mat"),
                    (p + "self_attn.k_proj.bias", (KV,), "mat"),
                    (p + "self_attn.v_proj.bias", (KV,), "mat")]
    out.append(("model.norm.weight", (H,), "gain"))
    if not m.tied:
        out.append(("lm_head.weight", (V, H), "mat"))
    return out


def f32_to_bf16_rne(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bits, round to nearest even (inputs are finite)."""
    u = x.astype(np.float32).view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)
    return r.astype(np.uint16)


def make_tensor(m: ModelShape, index: int, shape: tuple[int, ...], kind: str) -> np.ndarray:
    n = int(np.prod(shape))
    if kind == "gain":
        return np.full(n, 0x3F80, dtype=np.uint16)
    rng = np.random.Generator(np.random.PCG64([m.seed, index]))
    z = rng.standard_normal(n, dtype=np.float32)
    z *= np.float32(0.02)
    return f32_to_bf16_rne(z)


def config_json_text(m: ModelShape) -> str:
    arch = {"llama": "LlamaForCausalLM", "qwen3": "Qwen3ForCausalLM",
            "qwen2": "Qwen2ForCausalLM"}[m.model_type]
    lines = [
        '{',
        f'  "architectures": ["{arch}"],',
        f'  "model_type": "{m.model_type}",',
        f'  "hidden_size": {m.hidden},',
        f'  "intermediate_size": {m.inter},',
        f'  "num_hidden_layers": {m.layers},',
        f'  "num_attention_heads": {m.heads},',
        f'  "num_key_value_heads": {m.kv_heads},',
    ]
    if m.head_dim is not None:
        lines.append(f'  "head_dim": {m.head_dim},')
    lines += [
        f'  "vocab_size": {m.vocab},',
        f'  "rms_norm_eps": {m.eps},',
        f'  "rope_theta": {m.theta},',
        f'  "tie_word_embeddings": {"true" if m.tied else "false"},',
        f'  "attention_bias": {"true" if m.qkv_bias else "false"},',
        '  "hidden_act": "silu",',
        '  "torch_dtype": "bfloat16",',
        '  "cis2_synthetic": "N(0,0.02) bf16 RNE, PCG64 per tensor, norm gains 1.0"',
        '}',
    ]
    return "\n".join(lines) + "\n"


TOKENIZER_STUB = ('{"version": "1.0", "model": {"type": "cis2-synthetic-stub"}, '
                  '"note": "token ids are supplied directly; this file only enters the witness by hash"}\n')


def write_safetensors(path: str, tensors: list[tuple[str, tuple[int, ...], np.ndarray]]) -> None:
    header: dict[str, object] = {"__metadata__": {"format": "pt", "generator": "cis2 synth"}}
    off = 0
    for name, shape, arr in tensors:
        nb = arr.size * 2
        header[name] = {"dtype": "BF16", "shape": list(shape), "data_offsets": [off, off + nb]}
        off += nb
    h = json.dumps(header, separators=(",", ":")).encode()
    pad = (8 - (len(h) % 8)) % 8
    h += b" " * pad
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for _, _, arr in tensors:
            f.write(arr.astype("<u2", copy=False).tobytes())
    os.replace(tmp, path)


def sha256_file(path: str) -> bytes:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            b = f.read(1 << 22)
            if not b:
                break
            h.update(b)
    return h.digest()


def _widen(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << np.uint32(16)).view(np.float32).astype(np.float64)


def _final_hidden_f64(m: ModelShape, t: dict[str, np.ndarray], ids: np.ndarray) -> np.ndarray:
    """Final-norm output of the last of `ids` in float64: the plain Llama
    forward (RMSNorm, rotate-half RoPE, causal GQA attention, SwiGLU) with no
    pinned order.  Only its signs and rough magnitudes are used, to place the
    coverage rows; nothing is checked against it."""
    H, HD, NH, NKV = m.hidden, m.hd, m.heads, m.kv_heads
    eps, theta = float(m.eps), float(m.theta)

    def rms(x, w):
        return x / np.sqrt((x * x).mean(-1, keepdims=True) + eps) * w

    def W(name, rows, cols):
        return _widen(t[name]).reshape(rows, cols)

    P = len(ids)
    h = W("model.embed_tokens.weight", m.vocab, H)[ids.astype(np.int64)]
    half = HD // 2
    ang = np.arange(P)[:, None] * theta ** (-np.arange(half) * 2.0 / HD)[None, :]
    cos, sin = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]

    def rope(x):  # [P, heads, HD]
        x1, x2 = x[..., :half], x[..., half:]
        return np.concatenate([x1 * cos - x2 * sin, x2 * cos + x1 * sin], axis=-1)

    for li in range(m.layers):
        p = f"model.layers.{li}."
        x = rms(h, _widen(t[p + "input_layernorm.weight"]))
        q = rope((x @ W(p + "self_attn.q_proj.weight", m.q_dim, H).T).reshape(P, NH, HD))
        k = rope((x @ W(p + "self_attn.k_proj.weight", m.kv_dim, H).T).reshape(P, NKV, HD))
        v = (x @ W(p + "self_attn.v_proj.weight", m.kv_dim, H).T).reshape(P, NKV, HD)
        att = np.zeros((P, NH, HD))
        for hh in range(NH):
            g = hh // (NH // NKV)
            s = q[:, hh, :] @ k[:, g, :].T / np.sqrt(HD)
            s = np.where(np.tril(np.ones((P, P), bool)), s, -np.inf)
            e = np.exp(s - s.max(-1, keepdims=True))
            att[:, hh, :] = (e / e.sum(-1, keepdims=True)) @ v[:, g, :]
        h = h + att.reshape(P, m.q_dim) @ W(p + "self_attn.o_proj.weight", H, m.q_dim).T
        x = rms(h, _widen(t[p + "post_attention_layernorm.weight"]))
        gt = x @ W(p + "mlp.gate_proj.weight", m.inter, H).T
        up = x @ W(p + "mlp.up_proj.weight", m.inter, H).T
        h = h + (gt / (1.0 + np.exp(-gt)) * up) @ W(p + "mlp.down_proj.weight", H, m.inter).T
    return rms(h, _widen(t["model.norm.weight"]))[-1]


def coverage_prompt() -> np.ndarray:
    return random_prompts("coverage", 1, COVERAGE_PROMPT_LEN, COVERAGE_PROMPT_SEED)[0]


def _apply_coverage_rows(m: ModelShape, tensors: list) -> None:
    t = {name: arr for name, _, arr in tensors}
    x = _final_hidden_f64(m, t, coverage_prompt())
    lm = t["lm_head.weight"].reshape(m.vocab, m.hidden)
    tie = np.where(x >= 0, 0x4000, 0xC000).astype(np.uint16)       # +-2.0 in bf16
    lm[COVERAGE_TIE_A] = tie
    lm[COVERAGE_TIE_B] = tie
    mag = np.abs(x)
    col = int(np.argmin(np.where((mag >= 0.25) & (mag <= 0.75), np.abs(mag - 0.5), np.inf)))
    assert 0.25 <= mag[col] <= 0.75, "no column with |x| in [0.25, 0.75]"
    lm[COVERAGE_SUB] = 0
    lm[COVERAGE_SUB, col] = 0x0080 if x[col] > 0 else 0x8080        # +-2^-126, product sign +


def coverage_column(weights_dir: str) -> int:
    """Column of the coverage model's single non-zero weight in row SUB."""
    with open(os.path.join(weights_dir, "model.safetensors"), "rb") as f:
        (hl,) = struct.unpack("<Q", f.read(8))
        hdr = json.loads(f.read(hl))
        b, e = hdr["lm_head.weight"]["data_offsets"]
        f.seek(8 + hl + b)
        lm = np.frombuffer(f.read(e - b), dtype="<u2").reshape(hdr["lm_head.weight"]["shape"])
    (nz,) = np.nonzero(lm[COVERAGE_SUB])
    return int(nz[0])


def ensure_model(m: ModelShape | str, root: str) -> str:
    """Write (once) the three artifacts of `m` under root/<name>/ and return the dir."""
    if isinstance(m, str):
        m = MODELS[m]
    d = os.path.join(root, m.name)
    stamp = os.path.join(d, ".complete")
    if os.path.exists(stamp):
        return d
    os.makedirs(d, exist_ok=True)
    specs = tensor_specs(m)
    tensors = [(name, shape, make_tensor(m, i, shape, kind)) for i, (name, shape, kind) in enumerate(specs)]
    if m.coverage:
        _apply_coverage_rows(m, tensors)
    write_safetensors(os.path.join(d, "model.safetensors"), tensors)
    with open(os.path.join(d, "config.json"), "w") as f:
        f.write(config_json_text(m))
    with open(os.path.join(d, "tokenizer.json"), "w") as f:
        f.write(TOKENIZER_STUB)
    with open(stamp, "w") as f:
        f.write("ok\n")
    return d


def prompt_ids(w: Workload | str, n_seq: int | None = None, first: int = 0,
               prompt_len: int | None = None) -> np.ndarray:
    """[n_seq, prompt_len] uint32 ids; row i uses PCG64([prompt_seed, first + i])."""
    if isinstance(w, str):
        w = WORKLOADS[w]
    m = MODELS[w.model]
    n = w.n_seq if n_seq is None else n_seq
    L = w.prompt_len if prompt_len is None else prompt_len
    out = np.empty((n, L), dtype=np.uint32)
    for i in range(n):
        rng = np.random.Generator(np.random.PCG64([w.prompt_seed, first + i]))
        out[i] = rng.integers(0, m.vocab, size=L, dtype=np.int64).astype(np.uint32)
    return out


def random_prompts(model: str, n_seq: int, prompt_len: int, seed: int, first: int = 0) -> np.ndarray:
    """Prompts for ad-hoc test cases (same generator as `prompt_ids`)."""
    m = MODELS[model]
    out = np.empty((n_seq, prompt_len), dtype=np.uint32)
    for i in range(n_seq):
        rng = np.random.Generator(np.random.PCG64([seed, first + i]))
        out[i] = rng.integers(0, m.vocab, size=prompt_len, dtype=np.int64).astype(np.uint32)
    return out


def write_ids_file(path: str, ids: np.ndarray) -> None:
    """One sequence per line, decimal ids separated by spaces."""
    with open(path, "w") as f:
        for row in np.atleast_2d(ids):
            f.write(" ".join(str(int(v)) for v in row) + "\n")


def default_root() -> str:
    return os.environ.get("CIS2B_SYNTH_DIR", os.path.join(os.path.dirname(os.path.dirname(
        os.path.abspath(__file__))), "_synth"))
