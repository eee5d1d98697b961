"""Training data path: pre-tokenised token shards, packed sequences, pinned-host prefetch.

The reference streams FineWeb through HF `datasets`, tokenises on the fly and packs the token stream into
max_seq_len chunks (dataset.py:9-42); its collate gives {"src": ids, "tgt": ids} (dataset.py:45-51). Here
the tokenising happens once, offline (`write_token_shard` from any iterable of token lists, e.g. a GPT-2
tokenizer's output), and training reads fixed-size windows straight out of a memory-mapped shard:

  TokenShard            a flat uint16/uint32 token file + its length; window(i) = tokens[i*L, (i+1)*L)
  PackedTokenDataset    the reference's packing of a document stream into max_seq_len chunks, as a
                        torch IterableDataset over token lists (no tokenizer inside)
  ShardLoader           batches of windows, sharded over data-parallel ranks, gathered on a background
                        thread into pinned host buffers and copied to the GPU on a side stream, so the
                        host->device copy of batch i+1 overlaps step i; yields {"src", "tgt"} as the
                        reference's collate does
  hellaswag_collate_fn  the reference's multiple-choice collate (dataset.py:71-153) over any tokenizer
                        with encode(); scoring lives in the Trainer

No dataset files ship with this package (the benchmark uses uniform random token ids).
"""
from __future__ import annotations

import queue
import threading
from typing import Iterable, Iterator, List, Optional

import numpy as np
import torch
from torch.utils.data import IterableDataset

_MAGIC = b"RGPTTOK1"
_HEADER = 32  # magic (8) | dtype code (8) | token count (8) | reserved (8)


def write_token_shard(path: str, docs: Iterable[List[int]], vocab_size: int) -> int:
    """Concatenate token lists into one shard file; returns the token count. uint16 storage when the
    vocabulary fits (GPT-2's 50257 / 50304 does), else uint32."""
    dt = np.uint16 if vocab_size <= 65536 else np.uint32
    n = 0
    with open(path, "wb") as f:
        f.write(b"\0" * _HEADER)
        for doc in docs:
            a = np.asarray(doc, dtype=np.int64)
            if a.size and (a.min() < 0 or a.max() >= vocab_size):
                raise ValueError(f"token id outside [0, {vocab_size})")
            f.write(a.astype(dt).tobytes())
            n += a.size
        f.seek(0)
        f.write(_MAGIC + np.array([np.dtype(dt).itemsize, n, 0], dtype=np.int64).tobytes())
    return n


class TokenShard:
    """Read-only memory map of a token shard written by write_token_shard."""

    def __init__(self, path: str):
        with open(path, "rb") as f:
            head = f.read(_HEADER)
        if len(head) != _HEADER or head[:8] != _MAGIC:
            raise ValueError(f"{path} is not a token shard")
        itemsize, n, _ = np.frombuffer(head[8:], dtype=np.int64)
        self.dtype = {2: np.uint16, 4: np.uint32}[int(itemsize)]
        self.n_tokens = int(n)
        self.tokens = np.memmap(path, dtype=self.dtype, mode="r", offset=_HEADER, shape=(self.n_tokens,))

    def n_windows(self, length: int) -> int:
        return self.n_tokens // length

    def window(self, i: int, length: int) -> np.ndarray:
        return self.tokens[i * length:(i + 1) * length]


class PackedTokenDataset(IterableDataset):
    """Packs a stream of token lists into max_seq_len chunks, carrying the remainder of each document into
    the next chunk (the packing of dataset.py:30-42, without the tokenizer). Yields int64 tensors."""

    def __init__(self, docs: Iterable[List[int]], max_seq_len: int):
        self.docs, self.max_seq_len = docs, max_seq_len

    def __iter__(self) -> Iterator[torch.Tensor]:
        buf: List[int] = []
        L = self.max_seq_len
        for doc in self.docs:
            buf.extend(doc)
            while len(buf) >= L:
                yield torch.tensor(buf[:L], dtype=torch.long)
                buf = buf[L:]


def fineweb_collate_fn(batch: List[torch.Tensor]) -> dict:
    """{"src": ids, "tgt": ids} (dataset.py:45-51): the trainer shifts them into inputs and labels."""
    ids = torch.stack(batch)
    return {"src": ids, "tgt": ids}


class ShardLoader:
    """Batches of seq_len-token windows from a TokenShard, for data-parallel rank `rank` of `world`.

    Each epoch visits a permutation of the windows (seeded, identical on every rank); rank r takes every
    world-th batch, so ranks see disjoint data. A background thread gathers each batch from the memory
    map into a pinned host buffer; the copy to `device` runs on a side stream, and the consumer's stream
    waits on the copy's event, so the copy of the next batch overlaps the current step. Yields
    {"src": ids, "tgt": ids} int64 [batch_size, seq_len] device tensors (the reference's collate)."""

    def __init__(self, shard: TokenShard | str, batch_size: int, seq_len: int, device=None, rank: int = 0,
                 world: int = 1, seed: int = 0, shuffle: bool = True, prefetch: int = 2):
        self.shard = shard if isinstance(shard, TokenShard) else TokenShard(shard)
        self.B, self.T = int(batch_size), int(seq_len)
        self.rank, self.world = int(rank), int(world)
        self.seed, self.shuffle, self.prefetch = int(seed), bool(shuffle), max(1, int(prefetch))
        self.device = torch.device(device) if device is not None else None
        self.epoch = 0
        nw = self.shard.n_windows(self.T)
        self.n_batches_total = nw // self.B
        if self.n_batches_total < self.world:
            raise ValueError(f"{nw} windows of {self.T} tokens are too few for {self.world} ranks x batch {self.B}")
        self.n_batches = self.n_batches_total // self.world  # per rank (equal on every rank)

    def __len__(self) -> int:
        return self.n_batches

    def set_epoch(self, epoch: int) -> None:
        self.epoch = int(epoch)

    def _order(self) -> np.ndarray:
        nw = self.n_batches_total * self.B
        if not self.shuffle:
            return np.arange(nw)
        return np.random.default_rng((self.seed, self.epoch)).permutation(nw)

    def host_batch(self, windows: np.ndarray, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Gather windows into an int64 [B, T] host tensor (pinned when `out` is)."""
        if out is None:
            out = torch.empty(len(windows), self.T, dtype=torch.long)
        view = out.numpy()
        for j, w in enumerate(windows):
            view[j] = self.shard.window(int(w), self.T)
        return out

    def __iter__(self):
        order = self._order()
        mine = [order[(k * self.world + self.rank) * self.B:(k * self.world + self.rank + 1) * self.B]
                for k in range(self.n_batches)]
        self.epoch += 1
        if self.device is None or self.device.type != "cuda":
            for w in mine:
                ids = self.host_batch(w)
                yield {"src": ids, "tgt": ids}
            return
        yield from self._device_iter(mine)

    def _device_iter(self, mine):
        dev = self.device
        nbuf = self.prefetch + 1
        pinned = [torch.empty(self.B, self.T, dtype=torch.long).pin_memory() for _ in range(nbuf)]
        free: "queue.Queue[int]" = queue.Queue()
        for i in range(nbuf):
            free.put(i)
        ready: "queue.Queue" = queue.Queue()
        stop = threading.Event()

        def gather():
            try:
                for w in mine:
                    slot = free.get()
                    if stop.is_set():
                        return
                    self.host_batch(w, pinned[slot])
                    ready.put(slot)
            except Exception as e:  # surfaced to the consumer
                ready.put(e)
            ready.put(None)

        th = threading.Thread(target=gather, daemon=True)
        th.start()
        copy_stream = torch.cuda.Stream(device=dev)
        pending = []  # (slot, event) of host buffers whose copies may still be reading them
        try:
            while True:
                item = ready.get()
                if item is None:
                    break
                if isinstance(item, Exception):
                    raise item
                slot = item
                consumer = torch.cuda.current_stream(dev)
                with torch.cuda.stream(copy_stream):
                    ids = torch.empty(self.B, self.T, dtype=torch.long, device=dev)
                    ids.copy_(pinned[slot], non_blocking=True)
                    done = torch.cuda.Event()
                    done.record(copy_stream)
                consumer.wait_event(done)
                ids.record_stream(consumer)
                pending.append((slot, done))
                while pending and pending[0][1].query():  # host buffers whose copies have finished
                    free.put(pending.pop(0)[0])
                if len(pending) >= nbuf:  # every buffer in flight: wait for the oldest copy
                    s, ev = pending.pop(0)
                    ev.synchronize()
                    free.put(s)
                yield {"src": ids, "tgt": ids}
        finally:
            stop.set()
            for s, ev in pending:
                ev.synchronize()
                free.put(s)
            for _ in range(nbuf):
                free.put(0)
            th.join(timeout=5)


def hellaswag_collate_fn(batch: List[dict], tokenizer, max_seq_len: int) -> dict:
    """Multiple-choice batch of HellaSwag-style items ({"context", "endings", "label"}) for scoring by
    per-token loss (dataset.py:71-153): each (context, ending) pair becomes BOS + context + ending + EOS,
    truncated from the left to max_seq_len and right-padded with the pad id (EOS when the tokenizer has
    no pad); labels copy the ids with the context and the padding set to -100. Returns input_ids and
    labels [n_items * n_endings, max_seq_len], example_indices (item of each row) and correct_labels."""
    pad = tokenizer.pad_token_id
    if pad is None:
        pad = tokenizer.eos_token_id
        if pad is None:
            raise ValueError("Tokenizer must have a pad_token_id or eos_token_id defined.")
    bos = tokenizer.bos_token_id if tokenizer.bos_token_id is not None else getattr(tokenizer, "cls_token_id", None)
    eos = tokenizer.eos_token_id if tokenizer.eos_token_id is not None else getattr(tokenizer, "sep_token_id", None)
    head = [bos] if bos is not None else []
    tail = [eos] if eos is not None else []
    ids_rows, label_rows, owner, correct = [], [], [], []
    for i, item in enumerate(batch):
        ctx = tokenizer.encode(item["context"], add_special_tokens=False)
        for ending in item["endings"]:
            end = tokenizer.encode(ending, add_special_tokens=False)
            seq = (head + ctx + end + tail)[-max_seq_len:]
            n = len(seq)
            row = torch.full((max_seq_len,), pad, dtype=torch.long)
            row[:n] = torch.tensor(seq, dtype=torch.long)
            lab = row.clone()
            scored = len(end) + len(tail)  # the ending and EOS are scored; the context is not
            if n - scored > 0:
                lab[:n - scored] = -100
            lab[n:] = -100
            ids_rows.append(row)
            label_rows.append(lab)
            owner.append(i)
        correct.append(int(item["label"]))
    return {"input_ids": torch.stack(ids_rows).contiguous(), "labels": torch.stack(label_rows).contiguous(),
            "example_indices": torch.tensor(owner, dtype=torch.long),
            "correct_labels": torch.tensor(correct, dtype=torch.long)}

