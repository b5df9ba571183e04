"""Dataset preparation: a corpus tokenised into a flat token stream plus a
manifest pinning tokenizer, vocabulary size, element dtype, token count and the
sha256 of the stream and of each logical shard.

Same manifest format as the reference (src/wantrain/model/dataset.py:1-285):
`<dataset>.meta.json` = {tokenizer, vocab_size, total_tokens, n_shards, dtype,
sha256, eot_token, source, source_type[, shard_sha256]}, uint16 for
vocabularies up to 65536 tokens and uint32 above. Tokenizers: "bytes" (UTF-8
bytes, vocab 256, always available), or a tiktoken encoding / HF tokenizer
when those packages are installed.
"""

from __future__ import annotations

import hashlib
import json
import os

import numpy as np

DTYPES = {"uint16": np.uint16, "uint32": np.uint32}


def dtype_for_vocab(vocab_size: int) -> str:
    return "uint16" if vocab_size <= 2 ** 16 else "uint32"


def manifest_path(dataset: str) -> str:
    return f"{dataset}.meta.json"


def file_digest(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for b in iter(lambda: f.read(1 << 20), b""):
            h.update(b)
    return h.hexdigest()


def write_manifest(dataset, tokenizer, vocab_size, total_tokens, n_shards, dtype=None, extra=None):
    m = dict(tokenizer=tokenizer, vocab_size=vocab_size, total_tokens=total_tokens,
             n_shards=n_shards, dtype=dtype or dtype_for_vocab(vocab_size), **(extra or {}))
    with open(manifest_path(dataset), "w") as f:
        json.dump(m, f, indent=2)
    return m


def read_manifest(dataset: str) -> dict:
    p = manifest_path(dataset)
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    n = os.path.getsize(dataset) // 2  # legacy: a bare uint16 stream
    return dict(tokenizer="unknown", vocab_size=65536, total_tokens=n, n_shards=1, dtype="uint16")


def check_compatible(dataset: str, vocab_size: int) -> dict:
    m = read_manifest(dataset)
    if m["vocab_size"] > vocab_size:
        raise ValueError(f"dataset vocabulary {m['vocab_size']} exceeds the model's {vocab_size}")
    return m


def token_array(dataset: str, dtype: str):
    return np.memmap(dataset, dtype=DTYPES[dtype], mode="r")


def shard_bounds(total: int, k: int, n: int):
    return (total * k) // n, (total * (k + 1)) // n


def shard_view(dataset: str, shard: int, n_shards: int, total: int, dtype: str):
    """(array, base offset) holding logical shard `shard`: a `<dataset>.shard{k}of{n}`
    slice when present, else the whole stream."""
    p = f"{dataset}.shard{shard}of{n_shards}"
    if os.path.exists(p):
        lo, _ = shard_bounds(total, shard, n_shards)
        return np.memmap(p, dtype=DTYPES[dtype], mode="r"), lo
    return token_array(dataset, dtype), 0


def shard_digests(path: str, total: int, n_shards: int, dtype: str) -> list:
    isz = np.dtype(DTYPES[dtype]).itemsize
    out = []
    with open(path, "rb") as f:
        for k in range(n_shards):
            lo, hi = shard_bounds(total, k, n_shards)
            f.seek(lo * isz)
            out.append(hashlib.sha256(f.read((hi - lo) * isz)).hexdigest())
    return out


def _load_tokenizer(name: str):
    if name == "bytes":
        return (lambda text: list(text.encode("utf-8"))), 256, 0
    try:
        import tiktoken

        enc = tiktoken.get_encoding(name)
        return (lambda text: enc.encode_ordinary(text)), enc.n_vocab, enc.eot_token
    except ImportError:
        pass
    try:
        from transformers import AutoTokenizer

        tok = AutoTokenizer.from_pretrained(name)
        eot = tok.eos_token_id if tok.eos_token_id is not None else 0
        return (lambda text: tok.encode(text, add_special_tokens=False)), len(tok), eot
    except Exception as e:
        raise ValueError(f"tokenizer {name!r} is not available here ({e!r}); use 'bytes'") from e


def _iter_texts(source: str, source_type: str, text_key: str):
    st = source_type
    if st == "auto":
        st = "jsonl" if source.endswith((".jsonl", ".json")) else "txt"
    with open(source, encoding="utf-8") as f:
        if st == "jsonl":
            for line in f:
                line = line.strip()
                if line:
                    yield json.loads(line)[text_key]
        else:
            for para in f.read().split("\n\n"):
                if para.strip():
                    yield para


def prepare(source: str, out: str, tokenizer: str = "gpt2", source_type: str = "auto",
            text_key: str = "text", n_shards: int = 1, limit_tokens: int | None = None,
            eot_token: int | None = None) -> dict:
    enc, vocab, eot = _load_tokenizer(tokenizer)
    eot = eot if eot_token is None else eot_token
    dtype = dtype_for_vocab(vocab)
    total = 0
    with open(out, "wb") as f:
        for text in _iter_texts(source, source_type, text_key):
            arr = np.asarray(enc(text) + [eot], dtype=DTYPES[dtype])
            f.write(arr.tobytes())
            total += arr.size
            if limit_tokens and total >= limit_tokens:
                break
    extra = dict(sha256=file_digest(out), eot_token=eot, source=source, source_type=source_type)
    if n_shards > 1:
        extra["shard_sha256"] = shard_digests(out, total, n_shards, dtype)
        arr = token_array(out, dtype)
        for k in range(n_shards):
            lo, hi = shard_bounds(total, k, n_shards)
            np.asarray(arr[lo:hi]).tofile(f"{out}.shard{k}of{n_shards}")
    return write_manifest(out, tokenizer, vocab, total, n_shards, dtype, extra=extra)
