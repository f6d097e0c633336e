"""Version-2 .pai containers holding ggml blocks, on the host (no GPU).

A GGUF file converted by pai_b200_pai_from_gguf:
- reads back through pai_b200_pai_inspect with the configuration the GGUF
  reader reports;
- decodes, with an independent reader in this file, into a header whose
  section table carries u64 offsets and sizes, a manifest whose entries
  carry the pai_ir_quant_t of the ggml block kind, and weights whose bytes
  are the GGUF tensors' bytes unchanged;
- is refused by the reference's own version-1 reader (pai/pai.c
  pai_pai_open, compiled in oracle/_ref), so the versions never mix;
- with a corrupted manifest fails its CRC (PAI_ERR_PROTOCOL).
The ggml block kind of pai_ir_quant_t round-trips for Q4_0, Q8_0 and Q4_K.
"""
import ctypes as C
import struct

import numpy as np
import pytest

import gguf_writer as gw
from oracle import py_oracle as po
from prosperoai_b200 import _native
from prosperoai_b200.api import PaiError, gguf_inspect, pai_from_gguf, pai_inspect
from test_gguf_host import CFG, weights

PROTOCOL = -10


class IrQuant(C.Structure):
    """pai_ir_quant_t (ir/ir.h:95-103)."""
    _fields_ = [("present", C.c_uint8), ("bit_width", C.c_uint8), ("scale_repr", C.c_uint8),
                ("zero_point_repr", C.c_uint8), ("is_signed", C.c_uint8),
                ("block_structure", C.c_uint8), ("group_size", C.c_uint16)]


def read_pai(data: bytes):
    magic, version, flags, nsec, crc = struct.unpack_from("<IHHII", data, 0)
    secs = {}
    for i in range(nsec):
        t, f, off, size = struct.unpack_from("<IIQQ", data, 16 + 24 * i)
        secs[t] = (off, size, f)
    off, size, _ = secs[2]
    man = data[off:off + size]
    (count,), p, entries = struct.unpack_from("<I", man, 0), 4, {}
    for _ in range(count):
        (ln,) = struct.unpack_from("<H", man, p)
        name = man[p + 2:p + 2 + ln].decode()
        p += 2 + ln
        vid, dtype, rank = struct.unpack_from("<IBB", man, p)
        p += 8
        shape = struct.unpack_from("<6Q", man, p)
        p += 48
        woff, wsize = struct.unpack_from("<QQ", man, p)
        p += 16
        q = IrQuant.from_buffer_copy(man[p:p + 8])
        p += 8
        entries[name] = dict(dtype=dtype, rank=rank, shape=shape, off=woff, size=wsize, q=q)
    return dict(magic=magic, version=version, flags=flags, secs=secs, entries=entries)


@pytest.fixture
def model_files(tmp_path):
    cfg = dict(CFG)
    w = weights(cfg, seed=11)
    g = tmp_path / "m.gguf"
    gw.write_llama(g, cfg, w)
    p = tmp_path / "m.pai"
    pai_from_gguf(str(g), str(p))
    return cfg, w, g, p


def test_pai_v2_round_trip(model_files):
    cfg, w, g, p = model_files
    gi, pi = gguf_inspect(str(g)), pai_inspect(str(p))
    assert pi["version"] == 2 and pi["cfg"] == gi["cfg"] and pi["weight_bytes"] == gi["weight_bytes"]
    assert pi["n_rot"] == gi["n_rot"] and pi["tied_output"] == gi["tied_output"]
    data = p.read_bytes()
    f = read_pai(data)
    assert f["magic"] == 0x43494150 and f["version"] == 2 and f["flags"] == 0
    assert set(f["secs"]) == {1, 2, 3, 0x100}
    woff = f["secs"][3][0]
    assert woff % 256 == 0
    for name, blob in (("token_embd.weight", w["tok_embd"]), ("output.weight", w["output"]),
                       ("blk.1.attn_q.weight", w["wq"][1]), ("blk.0.ffn_down.weight", w["wdown"][0])):
        e = f["entries"][name]
        t = cfg["etype"] if name in ("token_embd.weight", "output.weight") else cfg["wtype"]
        assert e["dtype"] == 8 and e["rank"] == 2  # PAI_DTYPE_U8: bytes of ggml blocks
        assert e["q"].present == 1 and e["q"].block_structure == 3  # PAI_IR_QUANT_BLOCK_GGML
        assert e["q"].group_size == (256 if t == po.Q4_K else 32)
        assert data[woff + e["off"]:woff + e["off"] + e["size"]] == np.asarray(blob, np.uint8).tobytes()
    n = f["entries"]["blk.0.attn_norm.weight"]
    assert n["dtype"] == 0 and n["rank"] == 1 and n["q"].present == 0
    got = np.frombuffer(data[woff + n["off"]:woff + n["off"] + n["size"]], np.float32)
    assert np.array_equal(got, w["attn_norm"][0])


def test_pai_v2_refused_by_the_reference_v1_reader(model_files):
    R = po.ref()
    if R is None:
        pytest.skip("reference build (oracle/_ref) not present")
    _, _, _, p = model_files
    data = p.read_bytes()

    class Container(C.Structure):  # pai_pai_container_t (pai/pai.h:82-93), opaque room here
        _fields_ = [("raw", C.c_uint8 * 256)]

    R.pai_pai_open.restype = C.c_int32
    R.pai_pai_open.argtypes = [C.c_char_p, C.c_uint32, C.c_void_p]
    c = Container()
    assert R.pai_pai_open(data, len(data), C.byref(c)) == PROTOCOL


def test_pai_v2_crc_guards_the_manifest(model_files, tmp_path):
    _, _, _, p = model_files
    data = bytearray(p.read_bytes())
    f = read_pai(bytes(data))
    off = f["secs"][2][0]
    data[off + 10] ^= 0x5A
    bad = tmp_path / "bad.pai"
    bad.write_bytes(bytes(data))
    with pytest.raises(PaiError) as e:
        pai_inspect(str(bad))
    assert e.value.status == PROTOCOL


@pytest.mark.parametrize("t,bits,group,signed", [(po.Q4_0, 4, 32, 1), (po.Q8_0, 8, 32, 1),
                                                 (po.Q4_K, 4, 256, 0)])
def test_ir_quant_ggml_kind_round_trip(t, bits, group, signed):
    L = _native.load()
    q = IrQuant()
    assert L.pai_b200_ir_quant_ggml(t, C.byref(q)) == 0
    assert (q.present, q.bit_width, q.group_size, q.is_signed, q.block_structure) == (1, bits, group, signed, 3)
    back = C.c_uint32()
    assert L.pai_b200_ir_quant_ggml_type(C.byref(q), C.byref(back)) == 0 and back.value == t
    q.block_structure = 2  # PAI_IR_QUANT_BLOCK_GROUP: not a ggml kind
    assert L.pai_b200_ir_quant_ggml_type(C.byref(q), C.byref(back)) == -3
