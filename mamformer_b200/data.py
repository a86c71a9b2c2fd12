"""Training data: pre-tokenised ``.bin`` shards, synthetic tokens, pinned-memory prefetch.

Reference: ``scripts/train.py:48-128`` (``TextDataset``) and ``scripts/prepare_data.py:77-180``
(shard writer).  The shard format is the reference's - flat little-endian token ids, uint16
(uint32 when the vocabulary has 65536 entries or more), described by ``metadata.json`` with
``dtype``, ``seq_len``, ``total_tokens``, ``vocab_size``, ``num_shards`` - so data prepared by
either framework trains in the other.  Sequences are windows of ``seq_len + 1`` tokens with a
stride of ``seq_len`` (one token of overlap carries the next-token target across windows).

Differences: shards are memory-mapped instead of read whole into Python lists; the file order
is reshuffled every epoch and split across data-parallel ranks; the synthetic fallback uses the
model's vocabulary; and the training input is ``(input_ids, labels)`` with ``labels ==
input_ids`` - the model shifts internally (the reference's loader pre-shifts its labels and the
model shifts them again, so it trains on the token two positions ahead).
"""

from __future__ import annotations

import json
import queue
import random
import threading
from pathlib import Path
from typing import Iterator, Optional

import numpy as np
import torch


def _shard_dtype(data_dir: Path):
    meta = data_dir / "metadata.json"
    if meta.exists():
        info = json.loads(meta.read_text())
        return np.uint32 if info.get("dtype") == "uint32" else np.uint16
    return np.uint16


class TokenShardDataset(torch.utils.data.IterableDataset):
    def __init__(self, data_dir: str, seq_len: int = 8192, seed: int = 42, rank: int = 0, world: int = 1,
                 vocab_size: int = 32000):
        self.dir = Path(data_dir) if data_dir else Path("/nonexistent")
        self.seq_len, self.seed, self.rank, self.world = seq_len, seed, rank, world
        self.vocab_size = vocab_size
        self.files = sorted(self.dir.glob("*.bin")) if self.dir.exists() else []
        self.synthetic = not self.files
        self.dtype = _shard_dtype(self.dir) if self.files else np.uint16

    def __iter__(self) -> Iterator[torch.Tensor]:
        if self.synthetic:
            g = torch.Generator().manual_seed(self.seed + self.rank)
            while True:
                yield torch.randint(0, self.vocab_size, (self.seq_len,), generator=g)
        rng = random.Random(self.seed)
        W = self.seq_len + 1
        carry = np.zeros(0, dtype=np.int64)
        k = 0
        while True:
            files = list(self.files)
            rng.shuffle(files)
            for f in files:
                data = np.memmap(f, dtype=self.dtype, mode="r")
                if carry.size:
                    data = np.concatenate([carry, np.asarray(data, dtype=np.int64)])
                pos = 0
                while pos + W <= data.shape[0]:
                    if k % self.world == self.rank:
                        yield torch.from_numpy(np.asarray(data[pos:pos + W - 1], dtype=np.int64))
                    k += 1
                    pos += self.seq_len
                carry = np.asarray(data[pos:], dtype=np.int64)[-self.seq_len:]


# reference-compatible name
TextDataset = TokenShardDataset


class PinnedBatchLoader:
    """Background thread: stacks ``batch`` sequences into pinned host memory and (on CUDA)
    starts the host-to-device copy on a side stream, ``prefetch`` batches ahead.  ``next()``
    returns a device tensor whose copy the current stream has been made to wait for."""

    def __init__(self, dataset, batch: int, device="cuda", prefetch: int = 2):
        self.it = iter(dataset)
        self.batch = batch
        self.device = torch.device(device)
        self.cuda = self.device.type == "cuda"
        self.q: "queue.Queue" = queue.Queue(maxsize=max(1, prefetch))
        self.stream = torch.cuda.Stream(self.device) if self.cuda else None
        self._stop = False
        self.t = threading.Thread(target=self._work, daemon=True)
        self.t.start()

    def _work(self):
        while not self._stop:
            rows = [next(self.it) for _ in range(self.batch)]
            host = torch.stack(rows)
            if self.cuda:
                host = host.pin_memory()
                with torch.cuda.stream(self.stream):
                    dev = host.to(self.device, non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(self.stream)
                self.q.put((dev, ev, host))
            else:
                self.q.put((host, None, host))

    def __iter__(self):
        return self

    def __next__(self) -> torch.Tensor:
        dev, ev, host = self.q.get()
        if ev is not None:
            torch.cuda.current_stream(self.device).wait_event(ev)
            dev.record_stream(torch.cuda.current_stream(self.device))
        return dev

    def close(self):
        self._stop = True


def write_shards(token_stream, out_dir: str, seq_len: int, vocab_size: int, num_shards: int = 64) -> dict:
    """Write an iterable of token-id lists as ``num_shards`` round-robin ``.bin`` shards of
    ``seq_len + 1``-token chunks plus ``metadata.json`` (the layout of ``prepare_data.py``)."""
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    dt = np.uint16 if vocab_size < 65536 else np.uint32
    handles = {}
    buf, total, shard = [], 0, 0
    W = seq_len + 1

    def flush(chunk):
        nonlocal shard, total
        h = handles.get(shard)
        if h is None:
            h = handles[shard] = open(out / f"shard_{shard:05d}.bin", "wb")
        np.asarray(chunk, dtype=dt).tofile(h)
        total += len(chunk)
        shard = (shard + 1) % num_shards

    for ids in token_stream:
        buf.extend(ids)
        while len(buf) >= W:
            flush(buf[:W])
            buf = buf[W:]
    if buf:
        flush(buf)
    for h in handles.values():
        h.close()
    meta = {"dtype": "uint16" if dt is np.uint16 else "uint32", "seq_len": seq_len, "total_tokens": total,
            "vocab_size": vocab_size, "num_shards": len(handles)}
    (out / "metadata.json").write_text(json.dumps(meta, indent=2))
    return meta
