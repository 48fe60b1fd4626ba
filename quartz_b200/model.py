"""Decoder shapes and the seeded synthetic int8 weights of the decode workloads.

``ModelSpec`` holds what the device decode step needs from an HF-style config
(quartz/config.py: hidden size, heads, head_dim decoupled from hidden/heads,
RoPE base and llama3 scaling, tied embeddings). Two architectures are covered,
the two quartz ships (quartz/models/qwen3.py, quartz/models/llama.py): they
differ only in Qwen3's per-head q/k RMSNorm before RoPE.

``random_int8_weights`` draws the synthetic checkpoints the decode workloads run
on (there are no real checkpoints offline): every Linear and Embedding, in the
order quartz's leaf walker visits them (quartz/weights.py:70-82 over the module
tree of quartz/models/common.py:17-78), gets ``standard_normal(shape, float32)
* 0.02`` from one ``np.random.default_rng(seed)``, then the symmetric per-row
int8 quantiser (quartz/quantize.py:26-38). RMSNorm weights are ones. The same
recipe run through quartz itself produces bit-identical int8 tensors.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Iterator

import numpy as np

from .quantize import quantize_symmetric

ARCHS = ("Qwen3ForCausalLM", "LlamaForCausalLM")


@dataclass(frozen=True)
class ModelSpec:
    arch: str
    hidden: int
    layers: int
    n_heads: int
    n_kv: int
    head_dim: int
    inter: int
    vocab: int
    rope_theta: float
    tie: bool
    rope_scaling: dict | None = field(default=None, hash=False, compare=False)
    eps: float = 1e-6

    def __post_init__(self):
        if self.arch not in ARCHS:
            raise ValueError(f"unsupported architecture {self.arch!r}; expected one of {ARCHS}")
        if self.n_heads % self.n_kv:
            raise ValueError("query heads must be a multiple of kv heads")
        if self.head_dim % 2:
            raise ValueError("head_dim must be even (half-split RoPE)")

    @property
    def qk_norm(self) -> bool:
        """Qwen3 normalises each q/k head before RoPE (quartz/models/qwen3.py:27-34)."""
        return self.arch == "Qwen3ForCausalLM"

    @property
    def qkv_rows(self) -> int:
        return (self.n_heads + 2 * self.n_kv) * self.head_dim

    @classmethod
    def from_hf(cls, cfg: dict, arch: str | None = None) -> "ModelSpec":
        """From an HF config dict (the fields quartz/config.py:20-80 reads)."""
        arch = arch or (cfg.get("architectures") or [None])[0]
        hd = cfg.get("head_dim") or cfg["hidden_size"] // cfg["num_attention_heads"]
        return cls(arch=arch, hidden=cfg["hidden_size"], layers=cfg["num_hidden_layers"],
                   n_heads=cfg["num_attention_heads"],
                   n_kv=cfg.get("num_key_value_heads") or cfg["num_attention_heads"],
                   head_dim=hd, inter=cfg["intermediate_size"], vocab=cfg["vocab_size"],
                   rope_theta=float(cfg.get("rope_theta", 10000.0)),
                   tie=bool(cfg.get("tie_word_embeddings", False)),
                   rope_scaling=cfg.get("rope_scaling"),
                   eps=float(cfg.get("rms_norm_eps", 1e-6)))

    def int8_bytes_per_token(self) -> int:
        """Weight bytes one decode token streams: int8 matrices + fp32 row scales
        (the embedding gather reads one row; a tied lm_head reads the table)."""
        H, hd = self.hidden, self.head_dim
        per_layer_rows = [(self.qkv_rows, H), (H, self.n_heads * hd), (2 * self.inter, H),
                          (H, self.inter)]
        body = sum(n * k + 4 * n for n, k in per_layer_rows) * self.layers
        lm = self.vocab * H + 4 * self.vocab
        return body + lm

    def kv_bytes_per_token(self, ctx: int) -> int:
        """fp32 K and V bytes one decode token reads at context length ctx."""
        return 2 * 4 * self.layers * self.n_kv * ctx * self.head_dim


QWEN3_0P6B = ModelSpec(arch="Qwen3ForCausalLM", hidden=1024, layers=28, n_heads=16, n_kv=8,
                       head_dim=128, inter=3072, vocab=151936, rope_theta=1e6, tie=True)

LLAMA3_SCALING = dict(rope_type="llama3", factor=32.0, low_freq_factor=1.0,
                      high_freq_factor=4.0, original_max_position_embeddings=8192)

LLAMA_3P2_1B = ModelSpec(arch="LlamaForCausalLM", hidden=2048, layers=16, n_heads=32, n_kv=8,
                         head_dim=64, inter=8192, vocab=128256, rope_theta=5e5, tie=True,
                         rope_scaling=LLAMA3_SCALING)

QWEN3_8B = ModelSpec(arch="Qwen3ForCausalLM", hidden=4096, layers=36, n_heads=32, n_kv=8,
                     head_dim=128, inter=12288, vocab=151936, rope_theta=1e6, tie=False)


def rope_inv_freq(spec: ModelSpec) -> np.ndarray:
    """Per-pair inverse frequencies, fp32 [head_dim / 2] (quartz/rope.py:26-66).

    Plain: base ** (-(2j) / D) evaluated in fp32. llama3 scaling rescales the
    frequency denominators base ** (2j / D): long wavelengths are divided by
    ``factor``, short ones kept, the band between blended smoothly.
    """
    D, base = spec.head_dim, spec.rope_theta
    sc = spec.rope_scaling
    if sc and sc.get("rope_type") == "llama3":
        factor = sc["factor"]
        low = sc.get("low_freq_factor", 1.0)
        high = sc.get("high_freq_factor", 4.0)
        old = sc.get("original_max_position_embeddings", 8192)
        denom = base ** (np.arange(0, D, 2, dtype=np.float32) / D)
        wavelen = 2 * np.pi * denom
        denom = np.where(wavelen > old / low, denom * factor, denom)
        medium = (wavelen > old / high) & (wavelen < old / low)
        smooth = (old / wavelen - low) / (high - low)
        blended = denom / ((1 - smooth) / factor + smooth)
        denom = np.where(medium, blended, denom).astype(np.float32)
        return (1.0 / denom).astype(np.float32)
    return (base ** (-(np.arange(0, D, 2, dtype=np.float32) / D))).astype(np.float32)


def leaf_names(spec: ModelSpec) -> list[tuple[str, tuple[int, int]]]:
    """(name, (out, in)) of every Linear/Embedding in quartz's leaf-walk order:
    embedding, then per layer q, k, v, o, gate, up, down, then an untied lm_head."""
    H, hd = spec.hidden, spec.head_dim
    out = [("model.embed_tokens", (spec.vocab, H))]
    for i in range(spec.layers):
        p = f"model.layers.{i}."
        out += [(p + "self_attn.q_proj", (spec.n_heads * hd, H)),
                (p + "self_attn.k_proj", (spec.n_kv * hd, H)),
                (p + "self_attn.v_proj", (spec.n_kv * hd, H)),
                (p + "self_attn.o_proj", (H, spec.n_heads * hd)),
                (p + "mlp.gate_proj", (spec.inter, H)),
                (p + "mlp.up_proj", (spec.inter, H)),
                (p + "mlp.down_proj", (H, spec.inter))]
    if not spec.tie:
        out.append(("lm_head", (spec.vocab, H)))
    return out


def random_int8_weights(spec: ModelSpec, seed: int = 1234, std: float = 0.02,
                        group_size: int | None = None
                        ) -> Iterator[tuple[str, np.ndarray, np.ndarray]]:
    """Yield (name, q int8 [out, in], scale fp32 [out, ng]) in leaf order."""
    rng = np.random.default_rng(seed)
    for name, shape in leaf_names(spec):
        w = rng.standard_normal(shape, dtype=np.float32) * np.float32(std)
        q, s = quantize_symmetric(w, group_size)
        del w
        yield name, q, s


def cached_int8_weights(spec: ModelSpec, seed: int = 1234, std: float = 0.02,
                        cache_dir: str | None = None) -> list[tuple[str, np.ndarray, np.ndarray]]:
    """random_int8_weights(spec, seed, std) as a list, kept in a per-host cache
    file so that processes after the first (other ranks, later runs) load the
    int8 tensors instead of drawing them again (the fp32 draws dominate: about
    25 s for the Qwen3-0.6B checkpoint on one core). The first process to take
    the file lock draws and writes the file; the others wait for it and load
    it. Directory: `cache_dir`, else $QZ_CACHE_DIR, else the system temp dir."""
    import fcntl
    import hashlib
    import os
    import tempfile

    key = hashlib.sha256(repr((spec, seed, std)).encode()).hexdigest()[:20]
    root = cache_dir or os.environ.get("QZ_CACHE_DIR") or tempfile.gettempdir()
    os.makedirs(root, exist_ok=True)
    base = os.path.join(root, f"qz_int8_ckpt_{key}")
    shapes = leaf_names(spec)

    def load():
        # two flat files (all q bytes, all scales) mapped copy-on-write; the
        # tensors are views into them, in leaf order
        qb = np.load(base + "_q.npy", mmap_mode="c")
        sb = np.load(base + "_s.npy", mmap_mode="c")
        out, oq, os_ = [], 0, 0
        for name, (n, k) in shapes:
            if oq + n * k > qb.size or os_ + n > sb.size:
                raise ValueError("cache file shorter than the checkpoint")
            out.append((name, qb[oq:oq + n * k].reshape(n, k), sb[os_:os_ + n].reshape(n, 1)))
            oq += n * k
            os_ += n
        return out

    with open(base + ".lock", "w") as lk:
        fcntl.flock(lk, fcntl.LOCK_EX)
        try:
            if os.path.exists(base + "_s.npy"):
                try:
                    return load()
                except (OSError, ValueError):
                    pass                     # damaged or partial: draw again
            out = list(random_int8_weights(spec, seed, std))
            for suffix, parts in (("_q", [q.reshape(-1) for _, q, _ in out]),
                                  ("_s", [s_.reshape(-1) for _, _, s_ in out])):
                tmp = f"{base}{suffix}.{os.getpid()}.tmp.npy"
                np.save(tmp, np.concatenate(parts))
                os.replace(tmp, base + suffix + ".npy")   # the scales file last: it marks completion
            return out
        finally:
            fcntl.flock(lk, fcntl.LOCK_UN)


def norm_weights(spec: ModelSpec) -> dict[str, np.ndarray]:
    """The RMSNorm weights of the synthetic checkpoints: all ones."""
    H, hd = spec.hidden, spec.head_dim
    out = {"model.norm": np.ones(H, np.float32)}
    for i in range(spec.layers):
        p = f"model.layers.{i}."
        out[p + "input_layernorm"] = np.ones(H, np.float32)
        out[p + "post_attention_layernorm"] = np.ones(H, np.float32)
        if spec.qk_norm:
            out[p + "self_attn.q_norm"] = np.ones(hd, np.float32)
            out[p + "self_attn.k_norm"] = np.ones(hd, np.float32)
    return out


def seeded_kv(spec: ModelSpec, length: int, seed: int = 99, batch: int | None = None
              ) -> Iterator[tuple[np.ndarray, np.ndarray]]:
    """Per layer, (K, V) fp32 [n_kv, length, head_dim] of N(0, 1) draws from one
    default_rng(seed), K before V, layer by layer (the prefilled-cache start of
    the decode workload). With `batch` B, per layer [B, n_kv, length,
    head_dim] draws (the caches of B sequences decoded in lockstep)."""
    rng = np.random.default_rng(seed)
    shape = (batch or 1, spec.n_kv, length, spec.head_dim)
    for _ in range(spec.layers):
        k = rng.standard_normal(shape, dtype=np.float32)
        v = rng.standard_normal(shape, dtype=np.float32)
        yield (k[0], v[0]) if batch is None else (k, v)
