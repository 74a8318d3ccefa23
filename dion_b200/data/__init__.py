"""Training data: token files read by the native loader, text tokenized on
the fly, and synthetic tokens.

The reference trains through torchtitan's HuggingFace loader (c4_test;
ada_dion/integration/config_registry.py:161-168 names the dataset), which
tokenizes documents on the fly, concatenates them and cuts the stream into
non-overlapping windows of ``seq_len + 1`` tokens. Here documents are
tokenized once into token files (:mod:`dion_b200.data.tokenize`), and
:class:`TokenFileLoader` reads windows from the memory-mapped files with a
C++ prefetch thread (``dion_b200/csrc/io/token_loader.cpp``), so the
training loop never waits on tokenization or file reads.
:class:`TextStreamLoader` (``--dataloader.dataset text:<files>``) keeps
torchtitan's on-the-fly form for small corpora.

The loaders hand out pinned int64 ``(tokens, labels)`` pairs of shape
``[local_batch, seq_len]``, fresh buffers per step (the caching host
allocator reuses a buffer only after its asynchronous copy has finished),
and expose ``state_dict`` / ``load_state_dict`` with the number of global
samples consumed, which checkpoints store.
"""
from __future__ import annotations

import glob
import os
from typing import Dict, Iterator, List, Optional, Sequence, Tuple, Union

import numpy as np
import torch

__all__ = ["TokenFileLoader", "TextStreamLoader", "SyntheticTokens", "write_token_file", "token_file_info", "expand_paths",
           "build_loader", "HEADER_BYTES", "MAGIC"]

MAGIC = b"DB2TOKN1"
HEADER_BYTES = 32
_VERSION = 1


def _io():
    try:
        from .. import _io as mod
    except ImportError as e:  # the loader is native; there is no Python fallback
        raise RuntimeError("dion_b200._io is not built: run `python setup.py build_ext --inplace`") from e
    return mod


def _pinned(shape) -> torch.Tensor:
    return torch.empty(shape, dtype=torch.int64, pin_memory=torch.cuda.is_available())


def write_token_file(path: str, tokens: Union[np.ndarray, torch.Tensor, Sequence[int]],
                     bytes_per_token: Optional[int] = None) -> str:
    """Write ``tokens`` as a token file (32-byte header + little-endian ids).
    ``bytes_per_token`` defaults to 2 when every id fits in 16 bits, else 4."""
    if isinstance(tokens, torch.Tensor):
        tokens = tokens.detach().cpu().numpy()
    arr = np.asarray(tokens).reshape(-1)
    if arr.size and arr.min() < 0:
        raise ValueError("token ids must be non-negative")
    top = int(arr.max()) if arr.size else 0
    bpt = bytes_per_token or (2 if top < 2 ** 16 else 4)
    if bpt not in (2, 4) or top >= 2 ** (8 * bpt):
        raise ValueError(f"ids up to {top} do not fit in {bpt} bytes per token")
    data = arr.astype("<u2" if bpt == 2 else "<u4")
    header = np.zeros(HEADER_BYTES, dtype=np.uint8)
    header[:8] = np.frombuffer(MAGIC, dtype=np.uint8)
    header[8:12] = np.frombuffer(np.uint32(_VERSION).tobytes(), dtype=np.uint8)
    header[12:16] = np.frombuffer(np.uint32(bpt).tobytes(), dtype=np.uint8)
    header[16:24] = np.frombuffer(np.uint64(data.size).tobytes(), dtype=np.uint8)
    d = os.path.dirname(os.path.abspath(path))
    os.makedirs(d, exist_ok=True)
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(header.tobytes())
        f.write(data.tobytes())
    os.replace(tmp, path)
    return path


def token_file_info(path: str, bytes_per_token: int = 0) -> Dict[str, int]:
    """Token count, bytes per token and header size of a token file (a raw
    file needs ``bytes_per_token``)."""
    n, bpt, hdr = _io().file_info(path, bytes_per_token)
    return {"tokens": int(n), "bytes_per_token": int(bpt), "header_bytes": int(hdr)}


TEXT_SUFFIXES = (".jsonl", ".json", ".parquet", ".txt", ".jsonl.gz", ".json.gz", ".txt.gz")


def expand_paths(spec: Union[str, Sequence[str]], suffixes: Sequence[str] = (".bin",)) -> List[str]:
    """Files named by ``spec``: a comma-separated list of files, directories
    (every file inside ending in one of ``suffixes``, sorted) or glob
    patterns, in the order given."""
    items = spec.split(",") if isinstance(spec, str) else list(spec)
    out: List[str] = []
    for item in (i.strip() for i in items):
        if not item:
            continue
        if os.path.isdir(item):
            found = sorted(f for f in glob.glob(os.path.join(item, "*")) if f.endswith(tuple(suffixes)))
        elif any(c in item for c in "*?["):
            found = sorted(glob.glob(item))
        else:
            found = [item]
        if not found:
            raise FileNotFoundError(f"no token files match {item!r}")
        out.extend(found)
    return out


class TokenFileLoader:
    """Batches of ``local_batch`` windows of ``seq_len + 1`` tokens from token
    files, for one data-parallel rank.

    Global sample ``g`` reads window ``perm_e(g mod W)`` of epoch ``e``
    (``W`` windows; a keyed permutation per epoch when ``shuffle``, else the
    identity); the batch at position ``p`` gives rank ``r`` the samples
    ``p + r * local_batch + i``, and the position advances by
    ``world * local_batch`` per step. ``vocab`` (when > 0) is checked on the
    host for every token."""

    def __init__(self, paths: Union[str, Sequence[str]], seq_len: int, local_batch: int, rank: int = 0,
                 world: int = 1, seed: int = 0, shuffle: bool = True, prefetch: int = 4, vocab: int = 0,
                 bytes_per_token: int = 0, position: int = 0, timeout_s: float = 120.0):
        self.paths = expand_paths(paths)
        self.seq_len, self.local_batch = int(seq_len), int(local_batch)
        self.rank, self.world = int(rank), int(world)
        self._impl = _io().TokenLoader(self.paths, self.seq_len, self.local_batch, self.rank, self.world,
                                       int(seed) & (2 ** 64 - 1), bool(shuffle), int(prefetch), int(vocab),
                                       int(bytes_per_token), int(position), float(timeout_s))

    @property
    def windows(self) -> int:
        return self._impl.windows

    @property
    def total_tokens(self) -> int:
        return self._impl.total_tokens

    @property
    def position(self) -> int:
        """Global samples consumed so far (the next batch starts here)."""
        return self._impl.position

    def window_of(self, sample: int) -> int:
        return self._impl.window_of(sample)

    def next(self) -> Tuple[torch.Tensor, torch.Tensor]:
        t = _pinned((self.local_batch, self.seq_len))
        l = _pinned((self.local_batch, self.seq_len))
        self._impl.next(t, l)
        return t, l

    def __iter__(self) -> Iterator[Tuple[torch.Tensor, torch.Tensor]]:
        while True:
            yield self.next()

    def state_dict(self) -> Dict[str, int]:
        return {"samples": int(self.position)}

    def load_state_dict(self, sd: Dict[str, int]) -> None:
        self._impl.seek(int(sd["samples"]))


class SyntheticTokens:
    """Uniform random tokens over the vocabulary from a fixed seed, drawn on
    the host (one [global_batch, seq + 1] draw per step; each rank keeps its
    slice) into pinned memory."""

    def __init__(self, vocab: int, seq_len: int, local_batch: int, seed: int, rank: int = 0, world: int = 1):
        self.vocab, self.seq, self.lb = vocab, seq_len, local_batch
        self.rank, self.world = rank, world
        self.seed = seed
        self.gen = torch.Generator().manual_seed(seed)
        self.steps = 0

    def _draw(self) -> torch.Tensor:
        self.steps += 1
        return torch.randint(0, self.vocab, (self.lb * self.world, self.seq + 1), generator=self.gen)

    def next(self) -> Tuple[torch.Tensor, torch.Tensor]:
        full = self._draw()
        mine = full[self.rank * self.lb : (self.rank + 1) * self.lb]
        pin = torch.cuda.is_available()
        t = mine[:, :-1].contiguous().pin_memory() if pin else mine[:, :-1].contiguous()
        l = mine[:, 1:].contiguous().pin_memory() if pin else mine[:, 1:].contiguous()
        return t, l

    def __iter__(self) -> Iterator[Tuple[torch.Tensor, torch.Tensor]]:
        while True:
            yield self.next()

    def state_dict(self) -> Dict[str, int]:
        return {"samples": self.steps * self.lb * self.world}

    def load_state_dict(self, sd: Dict[str, int]) -> None:
        """Replay the generator to the saved point (same global batch size)."""
        steps = int(sd["samples"]) // (self.lb * self.world)
        self.gen = torch.Generator().manual_seed(self.seed)
        self.steps = 0
        for _ in range(steps):
            self._draw()


class TextStreamLoader:
    """Text documents tokenized on the fly, as torchtitan's HuggingFace text
    loader does (the reference trains through it): rank ``r`` of ``world``
    takes documents ``r, r + world, ...`` of the input files (in order,
    re-read after the last), encodes each as ``[BOS] + ids + [EOS]``,
    concatenates them and cuts non-overlapping windows of ``seq_len + 1``
    tokens. A background thread prepares ``prefetch`` batches ahead.

    The state is the number of windows this rank has consumed; loading it
    re-reads the documents up to that point (use token files and
    :class:`TokenFileLoader` for large corpora: they resume in O(1) and
    need no tokenizer at training time)."""

    def __init__(self, paths: Union[str, Sequence[str]], tokenizer, seq_len: int, local_batch: int, rank: int = 0,
                 world: int = 1, text_field: str = "text", vocab: int = 0, prefetch: int = 4, position: int = 0):
        from .tokenize import load_tokenizer

        self.paths = expand_paths(paths, TEXT_SUFFIXES)
        self.tok = load_tokenizer(tokenizer) if isinstance(tokenizer, str) else tokenizer
        self.seq_len, self.local_batch = int(seq_len), int(local_batch)
        self.rank, self.world = int(rank), int(world)
        self.text_field, self.vocab, self.prefetch = text_field, int(vocab), max(1, int(prefetch))
        if self.vocab and self.tok.vocab_size > self.vocab:
            raise ValueError(f"the tokenizer's vocabulary ({self.tok.vocab_size}) exceeds the model's ({self.vocab})")
        self._start(int(position))

    def _windows(self):
        from .tokenize import _encode_doc, iter_documents

        L = self.seq_len + 1
        buf: List[int] = []
        while True:
            any_doc = False
            for i, text in enumerate(iter_documents(self.paths, self.text_field)):
                if i % self.world != self.rank:
                    continue
                any_doc = True
                buf.extend(_encode_doc(self.tok, text))
                while len(buf) >= L:
                    yield buf[:L]
                    del buf[:L]
            if not any_doc:
                raise ValueError(f"rank {self.rank} of {self.world} gets no document from {self.paths}")

    def _start(self, position: int) -> None:
        import queue
        import threading

        self._windows_used = position
        q: "queue.Queue" = queue.Queue(maxsize=self.prefetch)
        stop = threading.Event()
        self._q, self._stop = q, stop  # the thread keeps its own queue and flag across a restart

        def work():
            try:
                it = self._windows()
                for _ in range(position):  # resume: skip the windows already used
                    next(it)
                while not stop.is_set():
                    rows = [next(it) for _ in range(self.local_batch)]
                    t = torch.tensor(rows, dtype=torch.int64)
                    while not stop.is_set():
                        try:
                            q.put(t, timeout=0.1)
                            break
                        except queue.Full:
                            continue
            except BaseException as e:  # surfaces in next()
                q.put(e)

        self._thread = threading.Thread(target=work, daemon=True)
        self._thread.start()

    def next(self) -> Tuple[torch.Tensor, torch.Tensor]:
        item = self._q.get(timeout=600)
        if isinstance(item, BaseException):
            raise item
        self._windows_used += self.local_batch
        t, l = _pinned((self.local_batch, self.seq_len)), _pinned((self.local_batch, self.seq_len))
        t.copy_(item[:, :-1])
        l.copy_(item[:, 1:])
        return t, l

    def __iter__(self) -> Iterator[Tuple[torch.Tensor, torch.Tensor]]:
        while True:
            yield self.next()

    def close(self) -> None:
        self._stop.set()
        self._thread.join(timeout=5)

    def state_dict(self) -> Dict[str, int]:
        # windows used per rank (the same on every rank: each step takes local_batch)
        return {"samples": int(self._windows_used)}

    def load_state_dict(self, sd: Dict[str, int]) -> None:
        self.close()
        self._start(int(sd["samples"]))


def build_loader(dataset: str, *, vocab: int, seq_len: int, local_batch: int, seed: int, rank: int, world: int,
                 shuffle: bool = True, prefetch: int = 4, bytes_per_token: int = 0, tokenizer: str = "byte",
                 text_field: str = "text"):
    """``"synthetic"`` -> :class:`SyntheticTokens`; ``"text:<files>"``
    (jsonl / json / parquet / txt) -> :class:`TextStreamLoader` with
    ``tokenizer``; anything else names token files (see
    :func:`expand_paths`) -> :class:`TokenFileLoader`."""
    if dataset in ("", "synthetic"):
        return SyntheticTokens(vocab, seq_len, local_batch, seed, rank, world)
    if dataset.startswith("text:"):
        return TextStreamLoader(dataset[len("text:"):], tokenizer, seq_len, local_batch, rank=rank, world=world,
                                text_field=text_field, vocab=vocab, prefetch=prefetch)
    return TokenFileLoader(dataset, seq_len, local_batch, rank=rank, world=world, seed=seed, shuffle=shuffle,
                           prefetch=prefetch, vocab=vocab, bytes_per_token=bytes_per_token)
