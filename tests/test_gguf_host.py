"""GGUF import on the host, no GPU (csrc/host/b200_gguf.c).

- pai_b200_gguf_inspect reads the configuration adapters/llama/llama.c:
  304-375 reads (keys, defaults, the tied lm head) from a LLaMA GGUF file;
- on the same files the reference's own parser (adapters/llama/gguf.c, in
  oracle/_ref) reads the same keys, tensor extents and types, and its
  dequantisation of each stored tensor equals the oracle's dequantisation
  of the blocks that were written (the bytes reach the loader unchanged);
- malformed containers give the reference parser's status codes, and the
  LLaMA-level checks give the reference importer's (llama.c:299-375);
- a file above the reference's 2 GiB import cap (llama.c:279) is accepted:
  the file is mapped, not read.
"""
import ctypes as C
import os
import struct

import numpy as np
import pytest

import gguf_writer as gw
from oracle import py_oracle as po
from prosperoai_b200.api import PaiError, gguf_inspect

CFG = dict(n_layer=2, n_embd=256, n_head=2, n_head_kv=1, head_dim=128, n_ff=512, vocab=300,
           eps=1e-5, rope_theta=500000.0, wtype=po.Q4_0, etype=po.Q8_0)
PROTOCOL, UNSUPPORTED, MISMATCH, IO = -10, -3, -6, -7


def weights(cfg, seed=3):
    rng = np.random.default_rng(seed)
    E, F, V = cfg["n_embd"], cfg["n_ff"], cfg["vocab"]
    qd, kd = cfg["n_head"] * cfg["head_dim"], cfg["n_head_kv"] * cfg["head_dim"]

    def q(t, rows, cols):
        return po.quantize(t, (rng.standard_normal(rows * cols) * 0.02).astype(np.float32))

    w = {"tok_embd": q(cfg["etype"], V, E), "output": q(cfg["etype"], V, E),
         "output_norm": rng.uniform(0.5, 1.5, E).astype(np.float32)}
    for key, rows, cols in (("wq", qd, E), ("wk", kd, E), ("wv", kd, E), ("wo", E, qd),
                            ("wgate", F, E), ("wup", F, E), ("wdown", E, F)):
        w[key] = [q(cfg["wtype"], rows, cols) for _ in range(cfg["n_layer"])]
    for key in ("attn_norm", "ffn_norm"):
        w[key] = [rng.uniform(0.5, 1.5, E).astype(np.float32) for _ in range(cfg["n_layer"])]
    return w


def status_of(path):
    try:
        gguf_inspect(str(path))
        return 0
    except PaiError as e:
        return e.status


def ref_open(data: bytes):
    R = po.ref()
    buf = C.create_string_buffer(data, len(data))
    f = po.Gguf()
    st = R.pai_gguf_open(buf, len(data), C.byref(f))
    return st, f, buf


@pytest.mark.parametrize("tied", [False, True])
def test_inspect_reads_llama_configuration(tmp_path, tied):
    w = weights(CFG)
    p = tmp_path / "m.gguf"
    gw.write_llama(p, CFG, w, tied=tied, ctx=8192)
    info = gguf_inspect(str(p))
    c = info["cfg"]
    for k in ("n_layer", "n_embd", "n_head", "n_head_kv", "head_dim", "n_ff", "vocab", "wtype", "etype"):
        assert c[k] == CFG[k], k
    assert c["rope_theta"] == np.float32(CFG["rope_theta"])
    assert c["eps"] == np.float32(1e-5)  # the executor's default, not the file's 1e-6 (llama.c:674)
    assert info["architecture"] == "llama" and info["version"] == 3 and info["context_length"] == 8192
    assert info["n_rot"] == 128 and info["tied_output"] == tied
    want = sum(np.asarray(a).nbytes for k, v in w.items() if k != "output" or not tied
               for a in (v if isinstance(v, list) else [v]))
    assert info["weight_bytes"] == want


def test_defaults_of_optional_keys(tmp_path):
    """head_count_kv absent -> head_count; freq_base absent -> 10000; rope
    dimension_count 0 or odd -> head_dim (llama.c:336-374)."""
    cfg = dict(CFG, n_head_kv=CFG["n_head"])
    p = tmp_path / "m.gguf"
    kvs = gw.llama_kvs(cfg, drop=("attention.head_count_kv", "rope.freq_base"), n_rot=0)
    p.write_bytes(gw.container(kvs, gw.llama_tensors(cfg, weights(cfg))))
    info = gguf_inspect(str(p))
    assert info["cfg"]["n_head_kv"] == cfg["n_head"] and info["cfg"]["rope_theta"] == 10000.0
    assert info["n_rot"] == 128


@pytest.mark.skipif(po.ref() is None, reason="reference build (oracle/_ref) not present")
def test_reference_parser_reads_the_same_file(tmp_path):
    w = weights(CFG)
    p = tmp_path / "m.gguf"
    gw.write_llama(p, CFG, w)
    data = p.read_bytes()
    R = po.ref()
    st, f, buf = ref_open(data)
    assert st == 0
    info = gguf_inspect(str(p))
    assert f.version == info["version"] and f.tensor_count == info["tensor_count"]
    for key, field in (("llama.block_count", "n_layer"), ("llama.embedding_length", "n_embd"),
                       ("llama.feed_forward_length", "n_ff"), ("llama.attention.head_count", "n_head"),
                       ("llama.attention.head_count_kv", "n_head_kv")):
        v = C.c_uint32()
        assert R.pai_gguf_get_u32(C.byref(f), key.encode(), C.byref(v)) == 0
        assert v.value == info["cfg"][field], key
    th = C.c_float()
    assert R.pai_gguf_get_f32(C.byref(f), b"llama.rope.freq_base", C.byref(th)) == 0
    assert th.value == info["cfg"]["rope_theta"]
    # every tensor: the reference's dequantisation of the stored bytes equals
    # the oracle's dequantisation of what was written
    for name, dims, t, raw in gw.llama_tensors(CFG, w):
        rt = R.pai_gguf_find_tensor(C.byref(f), name.encode())
        assert rt, name
        assert rt.contents.type == t and list(rt.contents.dims[:len(dims)]) == list(dims)
        out = C.POINTER(C.c_float)()
        n = po.U64()
        assert R.pai_gguf_dequant(C.byref(f), rt, C.byref(out), C.byref(n)) == 0
        got = np.ctypeslib.as_array(out, (n.value,)).copy()
        C.CDLL(None).free(C.cast(out, C.c_void_p))
        want = (np.frombuffer(raw, np.float32) if t == 0 else
                po.dequant(t, np.frombuffer(raw, np.uint8), n.value))
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), name
    R.pai_gguf_close(C.byref(f))


def _malformed(cfg, w):
    kvs = gw.llama_kvs(cfg)
    ts = gw.llama_tensors(cfg, w)
    good = gw.container(kvs, ts)
    bad_name = [("x" * 200, (4,), 0, b"\0" * 16)]
    yield "magic", gw.container(kvs, ts, magic=b"GGUX")
    yield "version 4", gw.container(kvs, ts, version=4)
    yield "version 0", gw.container(kvs, ts, version=0)
    yield "1025 tensors", gw.container(kvs, [], n_tensors=1025)
    yield "truncated metadata", good[:200]
    yield "short", good[:20]
    yield "long name", gw.container(kvs, bad_name)
    yield "5 dims", gw.container(kvs, [("t", (1, 1, 1, 1, 1), 0, b"\0" * 4)])
    yield "huge extent", gw.container(kvs, [("t", (1 << 27,), 0, b"")])
    yield "alignment 3", gw.container(kvs + [gw.kv("general.alignment", gw.U32, 3)], ts)
    yield "unknown value type", gw.container([gw._s(b"k") + struct.pack("<I", 13) + b"\0" * 8], ts)


@pytest.mark.skipif(po.ref() is None, reason="reference build (oracle/_ref) not present")
def test_malformed_containers_match_reference_codes(tmp_path):
    w = weights(CFG)
    for what, data in _malformed(CFG, w):
        p = tmp_path / "bad.gguf"
        p.write_bytes(data)
        st_ref, f, buf = ref_open(data)
        if st_ref == 0:
            po.ref().pai_gguf_close(C.byref(f))
        assert st_ref in (PROTOCOL, UNSUPPORTED), what
        assert status_of(p) == st_ref, what


def test_llama_level_errors(tmp_path):
    w = weights(CFG)
    cases = {
        "gpt2": (gw.container(gw.llama_kvs(CFG, arch="gpt2"), gw.llama_tensors(CFG, w)), UNSUPPORTED),
        "no block_count": (gw.container(gw.llama_kvs(CFG, drop=("block_count",)), gw.llama_tensors(CFG, w)),
                           MISMATCH),
        "no tokens": (gw.container(gw.llama_kvs(CFG, drop=("tokenizer.ggml.tokens",)),
                                   gw.llama_tensors(CFG, w)), MISMATCH),
        "missing tensor": (gw.container(gw.llama_kvs(CFG), gw.llama_tensors(CFG, w)[:-3]), MISMATCH),
        # 4 heads of 64 and 2 kv heads: the same tensor shapes, a head size the backend does not run
        "head_dim 64": (gw.container(gw.llama_kvs(dict(CFG, n_head=4, n_head_kv=2)), gw.llama_tensors(CFG, w)),
                        UNSUPPORTED),
        "partial rotary": (gw.container(gw.llama_kvs(CFG, n_rot=64), gw.llama_tensors(CFG, w)), UNSUPPORTED),
    }
    for what, (data, want) in cases.items():
        p = tmp_path / "m.gguf"
        p.write_bytes(data)
        assert status_of(p) == want, what
    # a tensor whose bytes run past the end of the file
    p = tmp_path / "m.gguf"
    p.write_bytes(gw.container(gw.llama_kvs(CFG), gw.llama_tensors(CFG, w))[:-4096])
    assert status_of(p) == PROTOCOL
    # mixed matrix types
    w2 = dict(w)
    w2["wk"] = [po.quantize(po.Q8_0, np.zeros(128 * 256, np.float32))] + w["wk"][1:]
    ts = gw.llama_tensors(CFG, w2)
    ts = [(n, d, po.Q8_0 if n == "blk.0.attn_k.weight" else t, b) for n, d, t, b in ts]
    p.write_bytes(gw.container(gw.llama_kvs(CFG), ts))
    assert status_of(p) == UNSUPPORTED
    assert status_of(tmp_path / "absent.gguf") == IO


def test_file_above_two_gib_is_mapped(tmp_path):
    """The reference refuses files over 2 GiB (llama.c:279); the loader maps
    the file, so a model whose data lies past 2 GiB inspects normally
    (sparse file: the padding takes no disk)."""
    w = weights(CFG)
    kvs = gw.llama_kvs(CFG)
    ts = gw.llama_tensors(CFG, w)
    gap = (5 << 29)  # 2.5 GiB of zeros before the first tensor's data
    off, infos = gap, b""
    for name, dims, t, data in ts:
        infos += gw._s(name.encode()) + struct.pack("<I", len(dims))
        infos += b"".join(struct.pack("<Q", x) for x in dims) + struct.pack("<IQ", t, off)
        off += len(data) + (-len(data)) % 32
    pre = b"GGUF" + struct.pack("<IQQ", 3, len(ts), len(kvs)) + b"".join(kvs) + infos
    pre += b"\0" * ((-len(pre)) % 32)
    p = tmp_path / "big.gguf"
    with open(p, "wb") as f:
        f.write(pre)
        f.seek(len(pre) + gap)
        for _, _, _, data in ts:
            f.write(data + b"\0" * ((-len(data)) % 32))
    assert os.path.getsize(p) > (2 << 30)
    info = gguf_inspect(str(p))
    assert info["cfg"]["n_layer"] == CFG["n_layer"]


@pytest.mark.parametrize("version", [1, 2])
def test_older_container_versions_read_like_the_reference(tmp_path, version):
    """Versions 1-3 are accepted with one layout (adapters/llama/gguf.c:148-152
    reads 64-bit counts for all of them); both parsers read the same file."""
    w = weights(CFG)
    data = gw.container(gw.llama_kvs(CFG), gw.llama_tensors(CFG, w), version=version)
    p = tmp_path / "m.gguf"
    p.write_bytes(data)
    info = gguf_inspect(str(p))
    assert info["version"] == version and info["cfg"]["n_layer"] == CFG["n_layer"]
    if po.ref() is not None:
        st, f, buf = ref_open(data)
        assert st == 0 and f.version == version and f.tensor_count == info["tensor_count"]
        po.ref().pai_gguf_close(C.byref(f))


def test_mistral_architecture_is_read(tmp_path):
    """llama.c:309-313 accepts "llama" and "mistral" (keys prefixed by the name)."""
    w = weights(CFG)
    p = tmp_path / "m.gguf"
    p.write_bytes(gw.container(gw.llama_kvs(CFG, arch="mistral"), gw.llama_tensors(CFG, w)))
    info = gguf_inspect(str(p))
    assert info["architecture"] == "mistral" and info["cfg"]["n_embd"] == CFG["n_embd"]
