"""Data path on the CPU: token shards, packing, rank sharding, and the multiple-choice collate.

The collate is pinned to the reference's own hellaswag_collate_fn (dataset.py:71-153): the fixture
tests/golden/hellaswag_collate.pt holds its output for synthetic items and a one-id-per-character toy
tokenizer (tests/golden/gen_golden.py), and the restatement here must reproduce it exactly.
"""
import os

import numpy as np
import torch

from rgpt_b200.data import (PackedTokenDataset, ShardLoader, TokenShard, fineweb_collate_fn, hellaswag_collate_fn,
                            write_token_shard)

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


class ToyTokenizer:
    pad_token_id = None
    eos_token_id = 1
    bos_token_id = 2

    def encode(self, text, add_special_tokens=True):
        return [3 + (ord(c) % 97) for c in text]


def test_hellaswag_collate_matches_reference():
    g = torch.load(os.path.join(GOLD, "hellaswag_collate.pt"), weights_only=False)
    out = hellaswag_collate_fn(g["items"], ToyTokenizer(), g["max_seq_len"])
    assert set(out) == set(g["out"])
    for k, v in g["out"].items():
        assert torch.equal(out[k], v), k


def test_packing_matches_reference_rule():
    docs = [list(range(i * 100, i * 100 + n)) for i, n in enumerate([5, 13, 2, 30, 7])]
    chunks = list(PackedTokenDataset(docs, 8))
    flat = [t for d in docs for t in d]
    assert len(chunks) == len(flat) // 8
    for i, c in enumerate(chunks):
        assert c.tolist() == flat[8 * i:8 * i + 8]
    b = fineweb_collate_fn(chunks[:3])
    assert b["src"].shape == (3, 8) and b["src"] is b["tgt"]


def test_token_shard_roundtrip_and_rank_sharding(tmp_path):
    rng = np.random.default_rng(0)
    docs = [rng.integers(0, 50304, size=int(n)).tolist() for n in rng.integers(1, 400, size=60)]
    path = str(tmp_path / "tokens.bin")
    n = write_token_shard(path, docs, vocab_size=50304)
    shard = TokenShard(path)
    flat = np.concatenate([np.asarray(d) for d in docs])
    assert shard.n_tokens == n == flat.size and shard.dtype == np.uint16
    assert np.array_equal(np.asarray(shard.tokens), flat)
    T, B, world = 17, 3, 4
    seen = []
    for rank in range(world):
        loader = ShardLoader(shard, B, T, rank=rank, world=world, seed=5)
        batches = list(loader)
        assert len(batches) == len(loader) == (shard.n_windows(T) // B) // world
        for b in batches:
            ids = b["src"]
            assert ids.shape == (B, T) and ids.dtype == torch.long and b["tgt"] is ids
            for row in ids:
                # every row is one aligned window of the token stream
                starts = [i for i in range(shard.n_windows(T)) if np.array_equal(flat[i * T:(i + 1) * T], row.numpy())]
                assert starts
                seen.append(starts[0])
    assert len(seen) == len(set(seen))  # ranks and batches never repeat a window within an epoch


def test_shard_loader_epochs_reshuffle(tmp_path):
    path = str(tmp_path / "t.bin")
    write_token_shard(path, [list(range(1000))], vocab_size=1000)
    loader = ShardLoader(path, 2, 10, seed=1)
    e0 = torch.cat([b["src"] for b in loader])
    e1 = torch.cat([b["src"] for b in loader])
    assert not torch.equal(e0, e1)
    assert sorted(e0[:, 0].tolist()) == sorted(e1[:, 0].tolist())


def test_token_shard_rejects_out_of_range(tmp_path):
    import pytest

    with pytest.raises(ValueError):
        write_token_shard(str(tmp_path / "bad.bin"), [[0, 5, 70000]], vocab_size=50304)
