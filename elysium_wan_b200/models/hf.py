"""Hugging Face checkpoints: a validating safetensors reader / writer, the
checkpoint digest, and importers that load Llama-family and GPT-2
checkpoints into this engine's flat parameter names.

Reference: src/wantrain/model/hf.py:1-166 (the reader, which validates every
header entry before reading a tensor byte, and `checkpoint_digest`). Only
safetensors is read: a .bin checkpoint is a pickle, and unpickling a
downloaded file executes whatever it contains. The importers are this
engine's own: the reference runs transformers' module trees instead
(arch "hf"), which this engine does not build; a Llama or GPT-2 checkpoint
instead becomes a config plus a state dict for the built-in decoder.

Llama's rotary embedding in Hugging Face layout rotates the two halves of a
head (rotate_half); this engine rotates adjacent pairs (the original layout),
so q and k projection rows are permuted on import (per head, half-split ->
interleaved), which makes the two computations identical.
"""

from __future__ import annotations

import hashlib
import json
import os
import struct

import torch

DTYPES = {"F64": torch.float64, "F32": torch.float32, "F16": torch.float16,
          "BF16": torch.bfloat16, "I64": torch.int64, "I32": torch.int32, "I16": torch.int16,
          "I8": torch.int8, "U8": torch.uint8, "BOOL": torch.bool,
          "F8_E4M3": torch.float8_e4m3fn, "F8_E5M2": torch.float8_e5m2}
CODES = {v: k for k, v in DTYPES.items()}
INDEX = "model.safetensors.index.json"
_MAX_HEADER = 100 * 2**20


def _esize(dtype) -> int:
    return torch.empty((), dtype=dtype).element_size()


def read_header(file: str) -> tuple[dict, int]:
    """({name: {dtype, shape, data_offsets}}, data offset); every entry is
    validated (known dtype, non-negative integer dims, offsets inside the
    data and equal to the shape's byte size) before any tensor is read."""
    with open(file, "rb") as fh:
        raw = fh.read(8)
        if len(raw) != 8:
            raise ValueError(f"{file}: not a safetensors file (no header length)")
        (n,) = struct.unpack("<Q", raw)
        if n > _MAX_HEADER:
            raise ValueError(f"{file}: safetensors header of {n} bytes refused")
        header = json.loads(fh.read(n))
        data_len = os.fstat(fh.fileno()).st_size - 8 - n
    if not isinstance(header, dict) or data_len < 0:
        raise ValueError(f"{file}: not a safetensors file (bad header)")
    header.pop("__metadata__", None)
    for name, info in header.items():
        if not isinstance(info, dict) or info.get("dtype") not in DTYPES:
            raise ValueError(f"{file}: tensor {name} has an unsupported dtype")
        shape, offs = info.get("shape"), info.get("data_offsets")
        if not isinstance(shape, list) or not all(type(d) is int and d >= 0 for d in shape):
            raise ValueError(f"{file}: tensor {name} has an invalid shape {shape!r}")
        if (not isinstance(offs, list) or len(offs) != 2 or not all(type(o) is int for o in offs)
                or not 0 <= offs[0] <= offs[1] <= data_len):
            raise ValueError(f"{file}: tensor {name} has invalid data_offsets {offs!r}")
        numel = 1
        for d in shape:
            numel *= d
        if offs[1] - offs[0] != numel * _esize(DTYPES[info["dtype"]]):
            raise ValueError(f"{file}: tensor {name}'s data_offsets do not match its shape")
    return header, 8 + n


def read_tensor(file: str, info: dict, base: int) -> torch.Tensor:
    dtype = DTYPES[info["dtype"]]
    start, end = info["data_offsets"]
    shape = tuple(info["shape"])
    with open(file, "rb") as fh:
        fh.seek(base + start)
        raw = bytearray(fh.read(end - start))
    if len(raw) != end - start:
        raise ValueError(f"{file}: truncated tensor data")
    if end == start:
        return torch.empty(shape, dtype=dtype)
    return torch.frombuffer(raw, dtype=torch.uint8).view(dtype).reshape(shape).clone()


def shard_files(path: str) -> list[str]:
    if not os.path.isdir(path):
        return [path]
    idx = os.path.join(path, INDEX)
    if os.path.exists(idx):
        with open(idx) as fh:
            names = set(json.load(fh)["weight_map"].values())
        out = []
        for v in sorted(names):
            if os.path.basename(v) != v:
                raise ValueError(f"{idx}: shard name {v!r} is not a file of the checkpoint")
            out.append(os.path.join(path, v))
        return out
    return sorted(os.path.join(path, f) for f in os.listdir(path) if f.endswith(".safetensors"))


def index(path: str) -> dict:
    """{name: (file, info, base)} over every shard; a name in two shards is
    refused."""
    files = shard_files(path)
    if not files:
        raise FileNotFoundError(f"no .safetensors under {path} (only safetensors is read: a .bin "
                                f"checkpoint is a pickle and unpickling executes code)")
    out: dict = {}
    for f in files:
        header, base = read_header(f)
        for name, info in header.items():
            if name in out:
                raise ValueError(f"tensor {name} appears in two shards of {path}")
            out[name] = (f, info, base)
    return out


def load_state(path: str) -> dict:
    return {n: read_tensor(f, i, b) for n, (f, i, b) in index(path).items()}


def save_file(tensors: dict, file: str, metadata: dict | None = None):
    """Write a safetensors file (tensors in name order, 8-byte aligned header)."""
    header, off, blobs = {}, 0, []
    for name in sorted(tensors):
        t = tensors[name].detach().cpu().contiguous()
        b = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": CODES[t.dtype], "shape": list(t.shape),
                        "data_offsets": [off, off + len(b)]}
        off += len(b)
        blobs.append(b)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(file, "wb") as fh:
        fh.write(struct.pack("<Q", len(h)))
        fh.write(h)
        for b in blobs:
            fh.write(b)


def checkpoint_digest(path: str) -> str:
    """sha256 over the names, shapes and fp32 values of every tensor, in name
    order: stages that downloaded different weights are refused."""
    h = hashlib.sha256()
    for name, (f, info, base) in sorted(index(path).items()):
        t = read_tensor(f, info, base)
        h.update(name.encode())
        h.update(str(tuple(t.shape)).encode())
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes() if t.dtype == torch.uint8
                 else t.contiguous().float().numpy().tobytes())
    return h.hexdigest()


# ------------------------------------------------------------------ importers
def _hf_config(path: str) -> dict:
    cfg = os.path.join(path, "config.json") if os.path.isdir(path) else None
    if cfg is None or not os.path.exists(cfg):
        raise FileNotFoundError(f"{path}: config.json is needed to import a checkpoint")
    with open(cfg) as fh:
        return json.load(fh)


def config_from_hf(hf: dict, seq_len: int | None = None, **overrides):
    """GPTConfig of a Llama-family or GPT-2 config.json."""
    from .config import GPTConfig

    mt = hf.get("model_type")
    if mt in ("llama", "mistral", "qwen2"):
        if hf.get("rope_scaling"):
            raise NotImplementedError("rope_scaling is not implemented")
        d = dict(vocab_size=hf["vocab_size"], n_layer=hf["num_hidden_layers"],
                 n_head=hf["num_attention_heads"],
                 n_kv_head=hf.get("num_key_value_heads") or hf["num_attention_heads"],
                 d_model=hf["hidden_size"], d_ff=hf["intermediate_size"],
                 seq_len=seq_len or min(2048, hf.get("max_position_embeddings", 2048)),
                 norm="rmsnorm", mlp="swiglu", pos="rope", bias=bool(hf.get("attention_bias")),
                 rms_eps=float(hf.get("rms_norm_eps", 1e-6)),
                 rope_theta=float(hf.get("rope_theta", 10000.0)),
                 tie_embeddings=bool(hf.get("tie_word_embeddings", False)), init_scheme="gpt2")
        if d["bias"] and mt != "qwen2":
            raise NotImplementedError("attention_bias on o_proj is not mapped")
    elif mt == "gpt2":
        d = dict(vocab_size=hf["vocab_size"], n_layer=hf["n_layer"], n_head=hf["n_head"],
                 d_model=hf["n_embd"], d_ff=hf.get("n_inner") or 4 * hf["n_embd"],
                 seq_len=seq_len or hf.get("n_positions", 1024), tie_embeddings=True,
                 ln_eps=float(hf.get("layer_norm_epsilon", 1e-5)), init_scheme="gpt2")
    else:
        raise NotImplementedError(f"model_type {mt!r} is not importable (llama, mistral, qwen2, "
                                  f"gpt2 are)")
    d.update(overrides)
    return GPTConfig(**d).validate()


def _half_to_pairs(w: torch.Tensor, heads: int) -> torch.Tensor:
    """Rows of a q / k projection from half-split rotary order to adjacent
    pairs, per head: row j < hd/2 -> 2j, row hd/2 + j -> 2j + 1."""
    out_f = w.shape[0]
    hd = out_f // heads
    return w.reshape(heads, 2, hd // 2, *w.shape[1:]).transpose(1, 2).reshape(w.shape)


def llama_state(cfg, hf_state: dict) -> dict:
    """This engine's parameter names -> tensors from a Llama-family state."""
    n, H, Hk = cfg.n_layer, cfg.n_head, cfg.kv_heads
    out = {"0.tok.weight": hf_state["model.embed_tokens.weight"]}
    for i in range(n):
        e, p = i + 1, f"model.layers.{i}."
        q = _half_to_pairs(hf_state[p + "self_attn.q_proj.weight"], H)
        k = _half_to_pairs(hf_state[p + "self_attn.k_proj.weight"], Hk)
        v = hf_state[p + "self_attn.v_proj.weight"]
        out[f"{e}.ln1.weight"] = hf_state[p + "input_layernorm.weight"]
        if Hk == H:
            out[f"{e}.qkv.weight"] = torch.cat([q, k, v])
        else:
            out[f"{e}.q.weight"] = q
            out[f"{e}.kv.weight"] = torch.cat([k, v])
        if cfg.bias:
            qb = _half_to_pairs(hf_state[p + "self_attn.q_proj.bias"], H)
            kb = _half_to_pairs(hf_state[p + "self_attn.k_proj.bias"], Hk)
            vb = hf_state[p + "self_attn.v_proj.bias"]
            if Hk == H:
                out[f"{e}.qkv.bias"] = torch.cat([qb, kb, vb])
            else:
                out[f"{e}.q.bias"], out[f"{e}.kv.bias"] = qb, torch.cat([kb, vb])
            out[f"{e}.proj.bias"] = hf_state.get(p + "self_attn.o_proj.bias",
                                                 torch.zeros(cfg.d_model))
            for k_ in ("gate", "up", "down"):
                out[f"{e}.mlp.{k_}.bias"] = hf_state.get(
                    p + f"mlp.{k_}_proj.bias",
                    torch.zeros(cfg.d_model if k_ == "down" else cfg.ff))
        out[f"{e}.proj.weight"] = hf_state[p + "self_attn.o_proj.weight"]
        out[f"{e}.ln2.weight"] = hf_state[p + "post_attention_layernorm.weight"]
        for k_ in ("gate", "up", "down"):
            out[f"{e}.mlp.{k_}.weight"] = hf_state[p + f"mlp.{k_}_proj.weight"]
    out[f"{n + 1}.ln_f.weight"] = hf_state["model.norm.weight"]
    if not cfg.tie_embeddings:
        out[f"{n + 1}.out.weight"] = hf_state["lm_head.weight"]
    return out


def gpt2_state(cfg, hf_state: dict) -> dict:
    """GPT-2 (Conv1D weights stored [in, out]) -> this engine's names."""
    g = lambda k: hf_state[k if k in hf_state else "transformer." + k]  # noqa: E731
    n = cfg.n_layer
    out = {"0.tok.weight": g("wte.weight"), "0.pos.weight": g("wpe.weight")[:cfg.seq_len]}
    for i in range(n):
        e, p = i + 1, f"h.{i}."
        out[f"{e}.ln1.weight"], out[f"{e}.ln1.bias"] = g(p + "ln_1.weight"), g(p + "ln_1.bias")
        out[f"{e}.qkv.weight"] = g(p + "attn.c_attn.weight").t()
        out[f"{e}.qkv.bias"] = g(p + "attn.c_attn.bias")
        out[f"{e}.proj.weight"] = g(p + "attn.c_proj.weight").t()
        out[f"{e}.proj.bias"] = g(p + "attn.c_proj.bias")
        out[f"{e}.ln2.weight"], out[f"{e}.ln2.bias"] = g(p + "ln_2.weight"), g(p + "ln_2.bias")
        out[f"{e}.mlp.fc1.weight"] = g(p + "mlp.c_fc.weight").t()
        out[f"{e}.mlp.fc1.bias"] = g(p + "mlp.c_fc.bias")
        out[f"{e}.mlp.fc2.weight"] = g(p + "mlp.c_proj.weight").t()
        out[f"{e}.mlp.fc2.bias"] = g(p + "mlp.c_proj.bias")
    out[f"{n + 1}.ln_f.weight"], out[f"{n + 1}.ln_f.bias"] = g("ln_f.weight"), g("ln_f.bias")
    return out


def import_checkpoint(path: str, seq_len: int | None = None, **overrides):
    """(GPTConfig, {engine name: fp32 tensor}) of a Hugging Face checkpoint
    directory (config.json + safetensors)."""
    hf = _hf_config(path)
    cfg = config_from_hf(hf, seq_len, **overrides)
    st = load_state(path)
    conv = llama_state if hf.get("model_type") != "gpt2" else gpt2_state
    return cfg, {k: v.float().contiguous() for k, v in conv(cfg, st).items()}


def load_into(model, state: dict, strict: bool = True):
    """Copy an imported state into a StageModel's slice (its entries only)."""
    names = model.store.names()
    missing = [n for n in names if n not in state]
    if strict and missing:
        raise KeyError(f"checkpoint lacks {missing[:5]}")
    for n in names:
        if n in state:
            t = state[n]
            want = tuple(model.store.index[n][1])
            if tuple(t.shape) != want:
                raise ValueError(f"{n}: checkpoint shape {tuple(t.shape)} != {want}")
            model.store.set_initial(n, t.to(model.store.device, torch.float32))
    model.store.sync_work()


_IMPORTED: dict = {}


def init_from_spec(model, spec):
    """Load spec.init_from into a StageModel when the spec names one (after
    its seeded init); checks spec.init_sha256 when set."""
    if not getattr(spec, "init_from", None):
        return
    key = os.path.abspath(spec.init_from)
    if key not in _IMPORTED:
        if spec.init_sha256 and checkpoint_digest(spec.init_from) != spec.init_sha256:
            raise ValueError(f"{spec.init_from}: digest does not match init_sha256")
        _IMPORTED[key] = import_checkpoint(spec.init_from, seq_len=spec.model.seq_len)[1]
    load_into(model, _IMPORTED[key])
