"""Decoder shapes for the weight-loading, KV and training-offload workloads.

``llama3_8b()``: 32 layers, hidden 4096, MLP 14336, 32 query / 8 KV heads of
128, vocab 128256, untied embeddings -> 8,030,261,248 parameters (16.06 GB
in bf16).  ``decoder_7b()``: the 7B decoder of the training-offload config
(32 layers, hidden 4096, MLP 11008, 32 heads, vocab 32000) ->
6,738,415,616 parameters.

``weight_manifest`` packs every tensor into one host image in a fixed
order, each tensor starting on a 4 KiB boundary so TMA / bulk copies and
fp8 row tiles (128 rows) can address it directly.  All 2-D matrices have
both dimensions divisible by 128, so the fp8 e4m3 128x128 block landing
covers them exactly; 1-D norm weights stay bf16.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass, field

ALIGN = 4096


@dataclass(frozen=True)
class DecoderConfig:
    name: str
    layers: int
    hidden: int
    intermediate: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    tie_embeddings: bool = False

    @property
    def q_dim(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim

    def as_dict(self) -> dict:
        return asdict(self)


def llama3_8b() -> DecoderConfig:
    return DecoderConfig("llama-3-8b", layers=32, hidden=4096, intermediate=14336, heads=32, kv_heads=8,
                         head_dim=128, vocab=128256)


def decoder_7b() -> DecoderConfig:
    return DecoderConfig("decoder-7b", layers=32, hidden=4096, intermediate=11008, heads=32, kv_heads=32,
                         head_dim=128, vocab=32000)


@dataclass(frozen=True)
class TensorSpec:
    name: str
    shape: tuple[int, ...]
    offset: int          # byte offset in the packed host image
    dtype: str = "bf16"

    @property
    def numel(self) -> int:
        n = 1
        for d in self.shape:
            n *= int(d)
        return n

    @property
    def nbytes(self) -> int:
        return self.numel * 2

    @property
    def is_matrix(self) -> bool:
        return len(self.shape) == 2


@dataclass(frozen=True)
class WeightManifest:
    config: DecoderConfig
    tensors: tuple[TensorSpec, ...] = field(default_factory=tuple)

    @property
    def total_bytes(self) -> int:
        last = self.tensors[-1]
        return _align(last.offset + last.nbytes)

    @property
    def param_count(self) -> int:
        return sum(t.numel for t in self.tensors)

    def by_name(self) -> dict[str, TensorSpec]:
        return {t.name: t for t in self.tensors}

    def matrices(self) -> list[TensorSpec]:
        return [t for t in self.tensors if t.is_matrix]

    def vectors(self) -> list[TensorSpec]:
        return [t for t in self.tensors if not t.is_matrix]


def _align(n: int, a: int = ALIGN) -> int:
    return (int(n) + a - 1) // a * a


def tensor_shapes(cfg: DecoderConfig) -> list[tuple[str, tuple[int, ...]]]:
    """(name, shape) in HF-style names and a layer-major order."""
    h, f = cfg.hidden, cfg.intermediate
    out = [("model.embed_tokens.weight", (cfg.vocab, h))]
    for i in range(cfg.layers):
        p = f"model.layers.{i}."
        out += [(p + "input_layernorm.weight", (h,)),
                (p + "self_attn.q_proj.weight", (cfg.q_dim, h)),
                (p + "self_attn.k_proj.weight", (cfg.kv_dim, h)),
                (p + "self_attn.v_proj.weight", (cfg.kv_dim, h)),
                (p + "self_attn.o_proj.weight", (h, cfg.q_dim)),
                (p + "post_attention_layernorm.weight", (h,)),
                (p + "mlp.gate_proj.weight", (f, h)),
                (p + "mlp.up_proj.weight", (f, h)),
                (p + "mlp.down_proj.weight", (h, f))]
    out.append(("model.norm.weight", (h,)))
    if not cfg.tie_embeddings:
        out.append(("lm_head.weight", (cfg.vocab, h)))
    return out


def weight_manifest(cfg: DecoderConfig) -> WeightManifest:
    off = 0
    specs = []
    for name, shape in tensor_shapes(cfg):
        t = TensorSpec(name, tuple(int(d) for d in shape), off)
        specs.append(t)
        off = _align(off + t.nbytes)
    return WeightManifest(cfg, tuple(specs))


__all__ = ["ALIGN", "DecoderConfig", "TensorSpec", "WeightManifest", "decoder_7b", "llama3_8b", "tensor_shapes",
           "weight_manifest"]
