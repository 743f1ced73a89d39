"""Chunks: the unit of KV reuse (API of cacheblend-hf-v7 ``chunker.py``).

A chunk is a run of token ids with a stable id used as the KVStore key.  The id
format (first 16 hex digits of sha256(text | comma-joined ids)) is kept
identical to the reference so that stores keyed by either implementation agree.
"""
from __future__ import annotations

import hashlib
from dataclasses import dataclass

import torch


@dataclass
class Chunk:
    text: str
    token_ids: list[int]
    chunk_id: str
    is_cached: bool = False

    @property
    def length(self) -> int:
        return len(self.token_ids)


def _stable_id(text: str, token_ids: list[int]) -> str:
    """Reference chunker.py:32-38 id: sha256(text, b"|", "1,2,3")[:16]."""
    digest = hashlib.sha256()
    digest.update(text.encode("utf-8"))
    digest.update(b"|")
    digest.update(",".join(map(str, token_ids)).encode("utf-8"))
    return digest.hexdigest()[:16]


def chunk_texts(tokenizer, texts: list[str]) -> list[Chunk]:
    """Tokenise each text on its own (no special tokens) into a Chunk."""
    out = []
    for text in texts:
        ids = list(tokenizer(text, add_special_tokens=False)["input_ids"])
        out.append(Chunk(text=text, token_ids=ids, chunk_id=_stable_id(text, ids)))
    return out


def fused_input_ids(chunks: list[Chunk], device: torch.device | None = None) -> torch.Tensor:
    """(1, total_seq) int64 tensor of all chunks' ids in order."""
    ids = [t for c in chunks for t in c.token_ids]
    t = torch.tensor(ids, dtype=torch.long).unsqueeze(0)
    return t if device is None else t.to(device)


def chunk_offsets(chunks: list[Chunk]) -> list[tuple[int, int]]:
    """[(start, end)] of each chunk in the fused sequence."""
    spans, pos = [], 0
    for c in chunks:
        spans.append((pos, pos + c.length))
        pos += c.length
    return spans
