"""A small GGUF (version 3) writer for the tests: the container the model
loader reads (csrc/host/b200_gguf.c), with LLaMA-family metadata keys and
tensor names. Test infrastructure only.
"""
from __future__ import annotations

import struct

import numpy as np

U32, F32, STR, ARR, U64 = 4, 6, 8, 9, 10
GGML_F32 = 0


def _s(b: bytes) -> bytes:
    return struct.pack("<Q", len(b)) + b


def kv(key: str, vtype: int, value, elem_type: int | None = None) -> bytes:
    out = _s(key.encode()) + struct.pack("<I", vtype)
    if vtype == U32:
        return out + struct.pack("<I", value)
    if vtype == F32:
        return out + struct.pack("<f", value)
    if vtype == U64:
        return out + struct.pack("<Q", value)
    if vtype == STR:
        return out + _s(value.encode())
    if vtype == ARR:
        out += struct.pack("<IQ", elem_type, len(value))
        if elem_type == STR:
            return out + b"".join(_s(v.encode()) for v in value)
        return out + b"".join(struct.pack("<I", v) for v in value)
    raise ValueError(vtype)


def container(kvs: list[bytes], tensors: list[tuple], align: int = 32, version: int = 3,
              magic: bytes = b"GGUF", n_tensors: int | None = None) -> bytes:
    """tensors: (name, extents with ne0 first, ggml type, data bytes)."""
    head = magic + struct.pack("<IQQ", version, len(tensors) if n_tensors is None else n_tensors, len(kvs))
    head += b"".join(kvs)
    off, infos, blobs = 0, b"", []
    for name, dims, t, data in tensors:
        infos += _s(name.encode()) + struct.pack("<I", len(dims))
        infos += b"".join(struct.pack("<Q", d) for d in dims) + struct.pack("<IQ", t, off)
        pad = (-len(data)) % align
        blobs.append(bytes(data) + b"\0" * pad)
        off += len(data) + pad
    head += infos
    return head + b"\0" * ((-len(head)) % align) + b"".join(blobs)


def llama_tensors(cfg: dict, w: dict, tied: bool = False) -> list[tuple]:
    """The GGUF tensors of a model given as the oracle's weight dict (ggml
    blocks per matrix, f32 norms)."""
    E, F, V = cfg["n_embd"], cfg["n_ff"], cfg["vocab"]
    qd, kd = cfg["n_head"] * cfg["head_dim"], cfg["n_head_kv"] * cfg["head_dim"]
    wt, et = cfg["wtype"], cfg["etype"]
    ts = [("token_embd.weight", (E, V), et, np.asarray(w["tok_embd"], np.uint8).tobytes())]
    names = [("attn_norm", "attn_norm", (E,), GGML_F32), ("attn_q", "wq", (E, qd), wt),
             ("attn_k", "wk", (E, kd), wt), ("attn_v", "wv", (E, kd), wt),
             ("attn_output", "wo", (qd, E), wt), ("ffn_norm", "ffn_norm", (E,), GGML_F32),
             ("ffn_gate", "wgate", (E, F), wt), ("ffn_up", "wup", (E, F), wt),
             ("ffn_down", "wdown", (F, E), wt)]
    for layer in range(cfg["n_layer"]):
        for gname, key, dims, t in names:
            data = np.ascontiguousarray(w[key][layer])
            ts.append((f"blk.{layer}.{gname}.weight", dims, t, data.tobytes()))
    ts.append(("output_norm.weight", (E,), GGML_F32, np.asarray(w["output_norm"], np.float32).tobytes()))
    if not tied:
        ts.append(("output.weight", (E, V), et, np.asarray(w["output"], np.uint8).tobytes()))
    return ts


def llama_kvs(cfg: dict, arch: str = "llama", ctx: int = 4096, drop: tuple = (),
              n_rot: int | None = None) -> list[bytes]:
    items = [("general.architecture", STR, arch), ("general.name", STR, "synthetic"),
             (f"{arch}.block_count", U32, cfg["n_layer"]), (f"{arch}.context_length", U32, ctx),
             (f"{arch}.embedding_length", U32, cfg["n_embd"]),
             (f"{arch}.feed_forward_length", U32, cfg["n_ff"]),
             (f"{arch}.attention.head_count", U32, cfg["n_head"]),
             (f"{arch}.attention.head_count_kv", U32, cfg["n_head_kv"]),
             (f"{arch}.rope.freq_base", F32, cfg["rope_theta"]),
             (f"{arch}.attention.layer_norm_rms_epsilon", F32, 1e-6)]
    if n_rot is not None:
        items.append((f"{arch}.rope.dimension_count", U32, n_rot))
    out = [kv(k, t, v) for k, t, v in items if k.split(".", 1)[-1] not in drop and k not in drop]
    if "tokenizer.ggml.tokens" not in drop:
        out.append(kv("tokenizer.ggml.tokens", ARR, [f"t{i}" for i in range(cfg["vocab"])], STR))
    return out


def write_llama(path, cfg: dict, w: dict, tied: bool = False, **kw) -> None:
    with open(path, "wb") as f:
        f.write(container(llama_kvs(cfg, **kw), llama_tensors(cfg, w, tied)))
