"""Synthetic training data.

``DummyDataset`` has the reference's sample semantics (utils/datasets.py:111-158):
random ``input_ids`` in [1, vocab), a right-padded boolean attention mask
whose valid length is uniform in [S/3, S-1), and labels equal to the ids
except -100 on padding and on a random "instruction" prefix of
10..min(100, S/5) tokens.  ``UniformTokens`` is the benchmark data: ids
uniform in [0, vocab), no padding, labels = ids.
"""
from __future__ import annotations

import torch
from torch.utils.data import Dataset


class DummyDataset(Dataset):
    def __init__(self, size: int = 1000, tokenizer=None, max_length: int = 512,
                 vocab_size: int = 32000, seed: int = 0):
        self.size = size
        self.max_length = max_length
        self.vocab_size = getattr(tokenizer, "vocab_size", None) or vocab_size
        self.seed = seed

    def __len__(self):
        return self.size

    def __getitem__(self, idx):
        g = torch.Generator().manual_seed(self.seed * 1_000_003 + idx)
        S = self.max_length
        ids = torch.randint(1, self.vocab_size, (S,), generator=g)
        valid = int(torch.randint(S // 3, max(S // 3 + 1, S - 1), (1,), generator=g))
        mask = torch.zeros(S, dtype=torch.bool)
        mask[:valid] = True
        labels = ids.clone()
        labels[~mask] = -100
        hi = max(11, min(100, S // 5))
        prefix = int(torch.randint(10, hi, (1,), generator=g))
        labels[:prefix] = -100
        return {"input_ids": ids, "attention_mask": mask, "labels": labels}


class UniformTokens(Dataset):
    def __init__(self, size: int, seq_len: int, vocab_size: int, seed: int = 0):
        self.size, self.seq_len, self.vocab_size, self.seed = size, seq_len, vocab_size, seed

    def __len__(self):
        return self.size

    def __getitem__(self, idx):
        g = torch.Generator().manual_seed(self.seed * 1_000_003 + idx)
        ids = torch.randint(0, self.vocab_size, (self.seq_len,), generator=g)
        return {"input_ids": ids, "attention_mask": torch.ones(self.seq_len, dtype=torch.bool),
                "labels": ids.clone()}
