"""Model configuration for the dense K8/V4 decoder family.

``DENSE_27B`` is the benchmark architecture: 64 layers, hidden 5120, 24 query
/ 4 KV heads of dim 128, SiLU-gated MLP 17408, RMSNorm, RoPE theta 1e6, vocab
151936, INT8 embedding and lm_head (per-row scaled), GPTQ INT4 g128 linears,
one MTP draft layer. Smaller presets keep the same structure for tests.
The reference serves the same shape (hidden 5120, its embedding partitions
``(124160, 5120)`` per TP2 rank, ``huggingface/swift-baked/README.md:88``;
MTP6 and the served flags at ``k8v4_v030/launch.sh:176-194``).
"""
from __future__ import annotations

import dataclasses
import json


@dataclasses.dataclass(frozen=True)
class ModelConfig:
    name: str = "dense-27b"
    num_layers: int = 64
    hidden: int = 5120
    num_heads: int = 24
    num_kv_heads: int = 4
    head_dim: int = 128
    intermediate: int = 17408
    vocab: int = 151936
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    max_position: int = 262144 + 8192
    group_size: int = 128
    mtp_layers: int = 1

    def __post_init__(self) -> None:
        if self.num_heads % self.num_kv_heads:
            raise ValueError("num_heads must be a multiple of num_kv_heads")
        for name in ("hidden", "intermediate"):
            if getattr(self, name) % self.group_size:
                raise ValueError("%s must be a multiple of the group size" % name)

    @property
    def gqa(self) -> int:
        return self.num_heads // self.num_kv_heads

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    def linear_params(self) -> int:
        """Parameters of the quantized linears of one layer."""
        h, i = self.hidden, self.intermediate
        return h * (self.q_size + 2 * self.kv_size) + self.q_size * h + h * 2 * i + i * h

    def to_json(self) -> str:
        return json.dumps(dataclasses.asdict(self), indent=2)

    @classmethod
    def from_dict(cls, d: dict) -> "ModelConfig":
        fields = {f.name for f in dataclasses.fields(cls)}
        return cls(**{k: v for k, v in d.items() if k in fields})

    def tp_shard(self, tp: int) -> "TPShape":
        return TPShape.make(self, tp)


@dataclasses.dataclass(frozen=True)
class TPShape:
    """Per-rank head and width split for tensor parallel degree ``tp``.

    Query heads split evenly. KV heads split evenly while ``tp`` divides them;
    beyond that they are replicated (each KV head shared by ``tp / hkv`` ranks),
    which makes the per-rank GQA ``hq_local / 1``.
    """

    tp: int
    hq_local: int
    hkv_local: int
    kv_replicas: int
    inter_local: int
    vocab_local: int

    @classmethod
    def make(cls, cfg: ModelConfig, tp: int) -> "TPShape":
        if tp < 1 or cfg.num_heads % tp:
            raise ValueError("tp %d does not divide %d query heads" % (tp, cfg.num_heads))
        if cfg.intermediate % (tp * cfg.group_size):
            raise ValueError("tp %d does not split the MLP on group boundaries" % tp)
        if cfg.vocab % tp:
            raise ValueError("tp %d does not divide the vocab" % tp)
        if tp <= cfg.num_kv_heads:
            if cfg.num_kv_heads % tp:
                raise ValueError("tp %d does not divide %d KV heads" % (tp, cfg.num_kv_heads))
            hkv, rep = cfg.num_kv_heads // tp, 1
        else:
            if tp % cfg.num_kv_heads:
                raise ValueError("tp %d is not a multiple of %d KV heads" % (tp, cfg.num_kv_heads))
            hkv, rep = 1, tp // cfg.num_kv_heads
        return cls(tp, cfg.num_heads // tp, hkv, rep, cfg.intermediate // tp, cfg.vocab // tp)

    @property
    def gqa_local(self) -> int:
        return self.hq_local // self.hkv_local

    def kv_heads_of(self, rank: int, num_kv_heads: int) -> list[int]:
        if self.kv_replicas == 1:
            return list(range(rank * self.hkv_local, (rank + 1) * self.hkv_local))
        return [rank // self.kv_replicas]


DENSE_27B = ModelConfig()
# Same structure, small sizes: unit tests and smoke runs.
TINY = ModelConfig(name="tiny", num_layers=2, hidden=512, num_heads=12, num_kv_heads=2, head_dim=128,
                   intermediate=1024, vocab=2048, max_position=8192)
SMALL = ModelConfig(name="small", num_layers=4, hidden=1024, num_heads=24, num_kv_heads=4, head_dim=128,
                    intermediate=2048, vocab=8192, max_position=65536)
PRESETS = {"dense-27b": DENSE_27B, "tiny": TINY, "small": SMALL}
