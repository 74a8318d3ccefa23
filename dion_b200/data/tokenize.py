"""Tokenize text documents into token files for :class:`~dion_b200.data.TokenFileLoader`.

    python -m dion_b200.data.tokenize --input 'c4/*.json.gz' --output data/c4 \\
        --tokenizer /path/to/hf_tokenizer_dir [--val-docs 1000] [--shard-tokens 500000000]

Each document becomes ``[bos] + ids + [eos]`` and the documents are
concatenated in input order, as torchtitan's text loader does before it cuts
windows (the reference trains through it on c4_test). Inputs: ``.jsonl`` /
``.json`` (one object per line with a text field, optionally gzip'd),
``.parquet`` (a text column) and ``.txt`` (one document per file).
Tokenizers: a local HuggingFace tokenizer directory (``transformers``,
offline) or ``byte`` (UTF-8 bytes, ids 0-255, BOS 256, EOS 257: vocabulary
258, no files needed). Output: ``<output>-00000.bin``... (train) and, with
``--val-docs N``, the first N documents as ``<output>-val-00000.bin``.
"""
from __future__ import annotations

import argparse
import glob
import gzip
import io
import json
import os
from typing import Iterable, Iterator, List, Optional, Sequence

import numpy as np

from . import write_token_file

__all__ = ["ByteTokenizer", "load_tokenizer", "iter_documents", "tokenize_to_files", "main"]


class ByteTokenizer:
    """UTF-8 bytes as ids (0-255) plus BOS = 256 and EOS = 257."""

    vocab_size = 258
    bos_id = 256
    eos_id = 257

    def encode(self, text: str) -> List[int]:
        return list(text.encode("utf-8"))

    def decode(self, ids: Sequence[int]) -> str:
        return bytes(i for i in ids if i < 256).decode("utf-8", errors="replace")


class _HFTokenizer:
    def __init__(self, path: str):
        from transformers import AutoTokenizer

        self.tok = AutoTokenizer.from_pretrained(path, local_files_only=True)
        self.vocab_size = len(self.tok)
        self.bos_id = self.tok.bos_token_id
        self.eos_id = self.tok.eos_token_id

    def encode(self, text: str) -> List[int]:
        return self.tok.encode(text, add_special_tokens=False)

    def decode(self, ids: Sequence[int]) -> str:
        return self.tok.decode(list(ids))


def load_tokenizer(spec: str):
    """``"byte"`` or a local HuggingFace tokenizer directory."""
    if spec == "byte":
        return ByteTokenizer()
    if not os.path.isdir(spec):
        raise FileNotFoundError(f"tokenizer {spec!r}: expected 'byte' or a local tokenizer directory")
    return _HFTokenizer(spec)


def _open_text(path: str):
    return io.TextIOWrapper(gzip.open(path, "rb"), encoding="utf-8") if path.endswith(".gz") else open(
        path, encoding="utf-8")


def iter_documents(paths: Iterable[str], text_field: str = "text") -> Iterator[str]:
    """Documents of the input files, in order."""
    for path in paths:
        base = path[:-3] if path.endswith(".gz") else path
        if base.endswith((".jsonl", ".json")):
            with _open_text(path) as f:
                head = f.read(1)
                f.seek(0)
                if head == "[":  # one JSON array of objects
                    for obj in json.load(f):
                        yield obj[text_field]
                else:
                    for line in f:
                        line = line.strip()
                        if line:
                            yield json.loads(line)[text_field]
        elif base.endswith(".parquet"):
            import pyarrow.parquet as pq

            table = pq.read_table(path, columns=[text_field])
            for batch in table.to_batches():
                yield from batch.column(0).to_pylist()
        elif base.endswith(".txt"):
            with _open_text(path) as f:
                yield f.read()
        else:
            raise ValueError(f"{path}: unsupported input (jsonl, json, parquet or txt, optionally .gz)")


class _ShardWriter:
    def __init__(self, prefix: str, shard_tokens: int):
        self.prefix, self.shard_tokens = prefix, shard_tokens
        self.buf: List[np.ndarray] = []
        self.n = 0
        self.files: List[str] = []
        self.total = 0

    def add(self, ids: List[int]) -> None:
        self.buf.append(np.asarray(ids, dtype=np.int64))
        self.n += len(ids)
        if self.shard_tokens and self.n >= self.shard_tokens:
            self.flush()

    def flush(self) -> None:
        if not self.buf:
            return
        path = f"{self.prefix}-{len(self.files):05d}.bin"
        write_token_file(path, np.concatenate(self.buf))
        self.files.append(path)
        self.total += self.n
        self.buf, self.n = [], 0


_WORKER_TOK = None


def _worker_init(spec: str) -> None:
    global _WORKER_TOK
    _WORKER_TOK = load_tokenizer(spec)


def _encode_doc(tok, text: str) -> List[int]:
    ids = tok.encode(text)
    if tok.bos_id is not None:
        ids = [tok.bos_id] + ids
    if tok.eos_id is not None:
        ids = ids + [tok.eos_id]
    return ids


def _worker_encode(text: str) -> List[int]:
    return _encode_doc(_WORKER_TOK, text)


def tokenize_to_files(inputs: Sequence[str], output: str, tokenizer="byte", text_field: str = "text",
                      val_docs: int = 0, shard_tokens: int = 0, max_docs: Optional[int] = None,
                      workers: int = 1) -> dict:
    """Tokenize ``inputs`` into token files under the prefix ``output``;
    returns the file lists, token counts and the tokenizer's vocabulary size.
    ``workers`` > 1 (with a tokenizer given by name or path) encodes the
    documents in that many processes, keeping their order."""
    tok = load_tokenizer(tokenizer) if isinstance(tokenizer, str) else tokenizer
    train = _ShardWriter(output, shard_tokens)
    val = _ShardWriter(output + "-val", shard_tokens)
    docs = 0
    texts = iter_documents(inputs, text_field)
    if max_docs is not None:
        import itertools

        texts = itertools.islice(texts, max_docs)
    pool = None
    if workers > 1 and isinstance(tokenizer, str):
        import multiprocessing as mp

        pool = mp.get_context("spawn").Pool(workers, initializer=_worker_init, initargs=(tokenizer,))
        encoded = pool.imap(_worker_encode, texts, chunksize=64)
    else:
        encoded = (_encode_doc(tok, t) for t in texts)
    try:
        for ids in encoded:
            (val if docs < val_docs else train).add(ids)
            docs += 1
    finally:
        if pool is not None:
            pool.close()
            pool.join()
    train.flush()
    val.flush()
    return {"train": train.files, "val": val.files, "train_tokens": train.total, "val_tokens": val.total,
            "documents": docs, "vocab_size": tok.vocab_size}


def main(argv: Optional[Sequence[str]] = None) -> dict:
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("--input", nargs="+", required=True, help="input files or glob patterns")
    p.add_argument("--output", required=True, help="output prefix (files <prefix>-00000.bin ...)")
    p.add_argument("--tokenizer", default="byte", help="'byte' or a local HuggingFace tokenizer directory")
    p.add_argument("--text-field", default="text")
    p.add_argument("--val-docs", type=int, default=0, help="first N documents go to the validation files")
    p.add_argument("--shard-tokens", type=int, default=0, help="start a new file after this many tokens")
    p.add_argument("--max-docs", type=int, default=None)
    p.add_argument("--workers", type=int, default=1, help="tokenizer processes (document order is kept)")
    a = p.parse_args(argv)
    inputs: List[str] = []
    for pat in a.input:
        found = sorted(glob.glob(pat)) if any(c in pat for c in "*?[") else [pat]
        if not found:
            raise SystemExit(f"no input matches {pat!r}")
        inputs.extend(found)
    res = tokenize_to_files(inputs, a.output, a.tokenizer, a.text_field, a.val_docs, a.shard_tokens, a.max_docs,
                            a.workers)
    print(json.dumps(res))
    return res


if __name__ == "__main__":
    main()
