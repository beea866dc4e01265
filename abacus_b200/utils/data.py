"""Token data: the reference's pre-tokenised document files and a synthetic
uniform-random source of the same shape.

Document handling follows the examples (``examples/train_gpt_dp.py:34-81``):
documents are 1-D token tensors; batches are padded with -100 to the longest
document in the batch (optionally to a multiple, for sequence parallelism).
"""
from __future__ import annotations

from pathlib import Path

import torch


def load_documents(path: Path) -> tuple[list[torch.Tensor], int]:
    path = Path(path)
    if not path.is_file():
        raise FileNotFoundError(f"Missing {path}. Run: python -m abacus_b200.scripts.prep_data")
    saved = torch.load(path, weights_only=True)
    documents = saved["tokens"]
    if not documents:
        raise ValueError(f"{path} contains no documents")
    return documents, int(saved["vocab_size"])


def select_documents(documents, limit=None, rank: int = 0, world_size: int = 1):
    """Drop documents shorter than 2 tokens; with several ranks keep an equal,
    rank-strided share (DP)."""
    if limit is not None:
        documents = documents[:limit]
    kept = []
    for document in documents:
        if document.ndim != 1:
            raise ValueError(f"Expected a document of shape (L,), got {tuple(document.shape)}")
        if document.numel() < 2:
            continue
        kept.append(document)
    if world_size == 1:
        return kept
    usable = (len(kept) // world_size) * world_size
    if usable == 0:
        raise ValueError(f"Need at least {world_size} documents with 2 or more tokens, found {len(kept)}")
    return kept[:usable][rank::world_size]


def padded_batches(documents, batch_size: int, multiple_of: int = 1):
    usable = (len(documents) // batch_size) * batch_size
    if usable == 0:
        raise ValueError(f"Need at least {batch_size} documents with 2 or more tokens, found {len(documents)}")
    for start in range(0, usable, batch_size):
        group = documents[start : start + batch_size]
        length = max(d.numel() for d in group)
        if multiple_of > 1 and length % multiple_of != 0:
            length += multiple_of - (length % multiple_of)
        batch = torch.full((batch_size, length), -100, dtype=torch.long)
        for row, document in enumerate(group):
            batch[row, : document.numel()] = document
        yield batch


class SyntheticTokens:
    """Uniform-random int64 tokens in [0, vocab), seeded (the benchmark data).

    ``batch(step)`` is deterministic in (seed, rank, step). With ``pin`` the
    batches are returned in pinned host memory for asynchronous H2D copies.
    """

    def __init__(self, vocab_size: int, batch_size: int, seq_len: int, seed: int = 0, rank: int = 0, pin: bool = False):
        self.vocab_size = vocab_size
        self.batch_size = batch_size
        self.seq_len = seq_len
        self.seed = seed
        self.rank = rank
        self.pin = pin and torch.cuda.is_available()

    def batch(self, step: int) -> torch.Tensor:
        g = torch.Generator().manual_seed(self.seed + 1_000_003 * self.rank + step)
        t = torch.randint(0, self.vocab_size, (self.batch_size, self.seq_len), generator=g, dtype=torch.long)
        return t.pin_memory() if self.pin else t

    def __iter__(self):
        step = 0
        while True:
            yield self.batch(step)
            step += 1
