"""Build one small pre-training shard that ``PretrainDataset`` reads.

Behaviour of the reference's shard builder
(``scripts/build_small_pretrain_data.py:28-121``): stream documents from a
text source, drop those shorter than ``min_chars``, tokenize each without
special tokens, append the EOS id after every document, stop once
``target_tokens`` ids are collected, truncate to exactly that many and write
them as a 1-D ``torch.uint32`` tensor with ``torch.save`` to
``<out_dir>/shard_0000.bin``.

Sources: ``synthetic`` (deterministic generated prose, identical on every
run and machine), ``text:<path>`` (a local UTF-8 file, one document per
blank-line-separated paragraph) or ``hf:<dataset>`` (a Hugging Face dataset,
only if the ``datasets`` package and the data are available locally).
Tokenizers: any ``transformers`` tokenizer found locally, or ``bytes`` (UTF-8
bytes as ids 0-255 with EOS 256), which needs no files.

``python -m data.build_small_shard --source synthetic --tokenizer bytes
--target-tokens 200000 --out-dir data/pretrain_small``
"""
from __future__ import annotations

import argparse
import hashlib
import sys
from pathlib import Path
from typing import Callable, Iterable, Iterator, List, Tuple

import torch

_TOPICS = [
    "Routing each token to a few experts keeps the compute per token small while the parameter count grows.",
    "A latent key-value cache stores one compressed vector per position instead of full keys and values.",
    "Rotary position embeddings rotate pairs of query and key features by an angle that grows with position.",
    "Tensor cores multiply tiles held in shared memory and accumulate the products in dedicated memory.",
    "A draft head proposes the next token cheaply and the main model keeps it only when it agrees.",
    "Load balancing without an auxiliary loss nudges a per-expert bias after every optimizer step.",
    "Gradient clipping rescales all gradients together when their global norm exceeds a threshold.",
    "Peer-to-peer stores over the switch fabric move rows directly into another device's buffers.",
    "Warmup raises the learning rate linearly before a cosine schedule lowers it to a floor.",
    "Checkpoints written to a temporary file and renamed into place survive a crash mid-write.",
]


def synthetic_documents(n_docs: int) -> Iterator[str]:
    """Deterministic documents: each one mixes a hash-chosen set of topic
    sentences, repeated a hash-chosen number of times."""
    for i in range(n_docs):
        d = hashlib.blake2b(f"synthetic-document-{i}".encode(), digest_size=32).digest()
        sentences = []
        for j in range(3 + d[0] % 6):
            sentences.extend([_TOPICS[d[1 + j] % len(_TOPICS)]] * (1 + d[17 + j] % 2))
        yield " ".join(sentences)


def text_file_documents(path: str) -> Iterator[str]:
    with open(path, encoding="utf-8") as f:
        block: List[str] = []
        for line in f:
            if line.strip():
                block.append(line.rstrip("\n"))
            elif block:
                yield "\n".join(block)
                block = []
        if block:
            yield "\n".join(block)


def hf_documents(name: str) -> Iterator[str]:
    try:
        from datasets import load_dataset
    except ImportError as e:
        raise RuntimeError("the `datasets` package is not installed; use --source synthetic or text:<path>") from e
    ds = load_dataset(name, split="train", streaming=True)
    return (row["text"] for row in ds)


def open_source(source: str, n_docs: int = 100_000) -> Iterator[str]:
    if source == "synthetic":
        return synthetic_documents(n_docs)
    if source.startswith("text:"):
        return text_file_documents(source[len("text:"):])
    if source.startswith("hf:"):
        return hf_documents(source[len("hf:"):])
    raise ValueError(f"unknown source {source!r} (synthetic, text:<path>, hf:<dataset>)")


def open_tokenizer(name: str) -> Tuple[Callable[[str], List[int]], int, int]:
    """``(encode, eos_id, vocab_size)``; ``bytes`` needs no files, any other
    name is loaded with ``transformers`` from local files only."""
    if name == "bytes":
        return (lambda text: list(text.encode("utf-8"))), 256, 257
    from transformers import AutoTokenizer
    tok = AutoTokenizer.from_pretrained(name, local_files_only=True)
    eos = tok.eos_token_id if tok.eos_token_id is not None else tok.vocab_size - 1
    return (lambda text: tok.encode(text, add_special_tokens=False)), int(eos), int(tok.vocab_size)


def build_shard(out_dir: str, documents: Iterable[str], encode: Callable[[str], List[int]], eos_id: int,
                target_tokens: int = 200_000, min_chars: int = 200) -> Path:
    """Tokenize ``documents`` until ``target_tokens`` ids; write ``shard_0000.bin``."""
    ids: List[int] = []
    for text in documents:
        if len(text) < min_chars:
            continue
        doc = encode(text)
        if not doc:
            continue
        ids.extend(doc)
        ids.append(eos_id)
        if len(ids) >= target_tokens:
            break
    if not ids:
        raise RuntimeError("the text source produced no tokens")
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    path = out / "shard_0000.bin"
    torch.save(torch.tensor(ids[:target_tokens], dtype=torch.int64).to(torch.uint32), path)
    return path


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="Build a small pre-training token shard")
    ap.add_argument("--source", default="synthetic", help="synthetic | text:<path> | hf:<dataset>")
    ap.add_argument("--tokenizer", default="bytes", help="bytes, or a locally available transformers tokenizer")
    ap.add_argument("--target-tokens", type=int, default=200_000)
    ap.add_argument("--min-chars", type=int, default=200)
    ap.add_argument("--out-dir", default="data/pretrain_small")
    a = ap.parse_args(argv)
    encode, eos, vocab = open_tokenizer(a.tokenizer)
    path = build_shard(a.out_dir, open_source(a.source), encode, eos, a.target_tokens, a.min_chars)
    n = torch.load(path, weights_only=True).numel()
    print(f"[data] wrote {n:,} tokens (vocab {vocab}, eos {eos}) -> {path}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
