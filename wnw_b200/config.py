"""``WnWConfig``: the WnW head-class / chunk configuration.

Same JSON schema, fields, derived quantities and query methods as the
reference (src/algorithms/wnw/code/config.py:6-121), so a config file written
for the reference loads unchanged.
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field


@dataclass
class WnWConfig:
    chunk_size_s: float
    overlap_s: float
    token_rate: float
    class_a: list            # global q-head ids: layer * num_q_heads + q
    class_b: list            # global kv-head ids: layer * num_kv_heads + kv
    retention_ratios: list   # per (layer, kv head); None for class-A heads
    top_k_chunks: int
    eviction_lag: int
    prefill_score_mode: str
    prefill_global_topk: bool = False
    num_layers: int = 0
    num_kv_heads: int = 0
    num_q_heads: int = 0
    _class_a_set: set = field(default_factory=set, repr=False)
    _class_b_set: set = field(default_factory=set, repr=False)
    _class_a_kv_set: set = field(default_factory=set, repr=False)

    def __post_init__(self):
        self._class_a_set = set(self.class_a)
        self._class_b_set = set(self.class_b)
        if self.stride_tokens <= 0:
            raise ValueError(f"overlap_tokens {self.overlap_tokens} leaves no stride within chunks of "
                             f"{self.chunk_size_tokens} tokens (the overlap must be smaller than the chunk)")
        if self.chunk_size_tokens % self.stride_tokens != 0:
            raise ValueError(f"a chunk of {self.chunk_size_tokens} tokens is not a whole number of "
                             f"{self.stride_tokens}-token segments (the stride must divide the chunk size)")
        if self.num_q_heads > 0 and self.num_kv_heads > 0:
            self._rebuild_class_a_kv_set()

    def set_model_dims(self, num_layers, num_kv_heads, num_q_heads):
        self.num_layers, self.num_kv_heads, self.num_q_heads = num_layers, num_kv_heads, num_q_heads
        self._rebuild_class_a_kv_set()

    def _rebuild_class_a_kv_set(self):
        g = self.num_q_heads // self.num_kv_heads
        self._class_a_kv_set = {(gid // self.num_q_heads) * self.num_kv_heads + (gid % self.num_q_heads) // g
                                for gid in self.class_a}

    @property
    def chunk_size_tokens(self) -> int:
        return int(self.chunk_size_s * self.token_rate)

    @property
    def overlap_tokens(self) -> int:
        return int(self.overlap_s * self.token_rate)

    @property
    def stride_tokens(self) -> int:
        return self.chunk_size_tokens - self.overlap_tokens

    def get_layer_class_a(self, layer_idx):
        lo = layer_idx * self.num_q_heads
        return [gid - lo for gid in self.class_a if lo <= gid < lo + self.num_q_heads]

    def get_layer_class_b(self, layer_idx):
        lo = layer_idx * self.num_kv_heads
        return [gid - lo for gid in self.class_b if lo <= gid < lo + self.num_kv_heads]

    def get_retention(self, layer_idx, local_kv_head):
        return self.retention_ratios[layer_idx * self.num_kv_heads + local_kv_head]

    def is_class_a(self, layer_idx, q_head):
        return layer_idx * self.num_q_heads + q_head in self._class_a_set

    def is_class_a_kv_head(self, layer_idx, kv_head):
        return layer_idx * self.num_kv_heads + kv_head in self._class_a_kv_set

    def is_class_b(self, layer_idx, kv_head):
        return layer_idx * self.num_kv_heads + kv_head in self._class_b_set

    @classmethod
    def from_dict(cls, raw, num_layers=0, num_kv_heads=0, num_q_heads=0):
        chunk, heads, sel = raw["chunk"], raw["heads"], raw["selection"]
        score = raw.get("score", {})
        mode = score.get("prefill_mode", "mean_text")
        if mode not in ("last", "mean_text"):
            raise ValueError(f"unknown prefill_mode {mode!r}")
        return cls(chunk_size_s=chunk["size_s"], overlap_s=chunk["overlap_s"], token_rate=chunk["token_rate"],
                   class_a=heads["class_a"], class_b=heads["class_b"], retention_ratios=heads["retention_ratios"],
                   top_k_chunks=sel["top_k_chunks"], eviction_lag=sel["eviction_lag"], prefill_score_mode=mode,
                   prefill_global_topk=score.get("prefill_global_topk", False), num_layers=num_layers,
                   num_kv_heads=num_kv_heads, num_q_heads=num_q_heads)

    @classmethod
    def from_json(cls, path, num_layers=0, num_kv_heads=0, num_q_heads=0):
        with open(path) as f:
            return cls.from_dict(json.load(f), num_layers, num_kv_heads, num_q_heads)

    def to_dict(self):
        return {"chunk": {"size_s": self.chunk_size_s, "overlap_s": self.overlap_s, "token_rate": self.token_rate},
                "heads": {"class_a": list(self.class_a), "class_b": list(self.class_b),
                          "retention_ratios": list(self.retention_ratios)},
                "selection": {"top_k_chunks": self.top_k_chunks, "eviction_lag": self.eviction_lag},
                "score": {"prefill_mode": self.prefill_score_mode,
                          "prefill_global_topk": self.prefill_global_topk}}
