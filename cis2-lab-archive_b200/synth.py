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
}


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
