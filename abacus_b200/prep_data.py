"""Tokenise NeelNanda/pile-10k into the document file the examples read
(``scripts/prep_data.py`` in the reference): each document becomes
``<bos> tokens <eos>`` (at most 2048 tokens) and the file holds
``{"tokens": [Tensor(L)], "vocab_size": V}``.

    python -m abacus_b200.prep_data [--out data/pile-10k.pt] [--tokenizer NAME]

Needs network access and the ``datasets`` package; the benchmarks and tests
use synthetic tokens instead.
"""
from __future__ import annotations

import argparse
from pathlib import Path

import torch

DEFAULT_OUT = Path(__file__).resolve().parents[1] / "data" / "pile-10k.pt"


def main() -> None:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--out", type=Path, default=DEFAULT_OUT)
    p.add_argument("--tokenizer", default="meta-llama/Llama-2-7b-hf")
    p.add_argument("--max-tokens", type=int, default=2048)
    args = p.parse_args()
    try:
        from datasets import load_dataset
        from transformers import AutoTokenizer
    except ImportError as error:
        raise SystemExit("prep_data needs the `datasets` and `transformers` packages") from error
    tok = AutoTokenizer.from_pretrained(args.tokenizer)
    ds = load_dataset("NeelNanda/pile-10k", split="train")
    docs = []
    for row in ds:
        ids = tok(row["text"], add_special_tokens=False)["input_ids"][: args.max_tokens - 2]
        docs.append(torch.tensor([tok.bos_token_id, *ids, tok.eos_token_id], dtype=torch.long))
    args.out.parent.mkdir(parents=True, exist_ok=True)
    torch.save({"tokens": docs, "vocab_size": int(tok.vocab_size)}, args.out)
    print(f"wrote {len(docs)} documents to {args.out}")


if __name__ == "__main__":
    main()
