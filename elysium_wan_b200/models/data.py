"""Deterministic batches: a pure function of (data_seed, step, microbatch).

Same rule as the reference (src/wantrain/model/data.py:13-66), so any process
regenerates identical tokens without a broadcast: a CPU torch.Generator seeded
with data_seed*1_000_003 + step*1_009 + mb draws randint(0, vocab,
(mb_size, seq_len + 1)); inputs are [:, :-1], targets [:, 1:]. With a dataset,
windows into the pretokenised stream (logical shard mb % data_shards).
"""

from __future__ import annotations

import numpy as np
import torch


def batch_seed(data_seed: int, step: int, mb: int) -> int:
    return data_seed * 1_000_003 + step * 1_009 + mb


def make_batch(data_seed: int, step: int, mb: int, mb_size: int, seq_len: int, vocab_size: int,
               dataset: str | None = None, data_shards: int = 1):
    g = torch.Generator()
    g.manual_seed(batch_seed(data_seed, step, mb))
    span = seq_len + 1
    if dataset is None:
        toks = torch.randint(0, vocab_size, (mb_size, span), generator=g)
    else:
        from . import dataset as ds

        meta = ds.read_manifest(dataset)
        total, dtype = meta["total_tokens"], meta["dtype"]
        if data_shards > 1:
            shard = mb % data_shards
            lo = (total * shard) // data_shards
            hi = (total * (shard + 1)) // data_shards
            arr, base = ds.shard_view(dataset, shard, data_shards, total, dtype)
            max_start = (hi - lo) - span - 1
            if max_start <= 0:
                raise ValueError(f"shard {shard}/{data_shards} holds {hi - lo} tokens, too few")
            starts = torch.randint(0, max_start, (mb_size,), generator=g)
            rows = [torch.from_numpy(arr[lo - base + s: lo - base + s + span].astype(np.int64))
                    for s in starts.tolist()]
        else:
            arr = ds.token_array(dataset, dtype)
            max_start = total - span - 1
            if max_start <= 0:
                raise ValueError(f"dataset holds {total} tokens, too few for a {span}-token window")
            starts = torch.randint(0, max_start, (mb_size,), generator=g)
            rows = [torch.from_numpy(arr[s: s + span].astype(np.int64)) for s in starts.tolist()]
        toks = torch.stack(rows)
    return toks[:, :-1].contiguous(), toks[:, 1:].contiguous()
