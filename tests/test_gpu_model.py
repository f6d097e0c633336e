"""Decoder parity: greedy tokens of the CUDA decode equal the composed
reference decode (oracle session, llama.c:669-797 op order over the
pai_ref_* restatements) for 64 steps, with the same synthetic weights.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import py_oracle as po
from prosperoai_b200 import _native
from prosperoai_b200.api import Model, Session

pytestmark = pytest.mark.gpu

SMALL = dict(n_layer=2, n_embd=512, n_head=4, n_head_kv=2, head_dim=128, n_ff=1024,
             vocab=2048, eps=1e-5, rope_theta=500000.0, wtype=po.Q4_0, etype=po.Q8_0)

KINDS = {"tok_embd": _native.T_TOK_EMBD, "output": _native.T_OUTPUT, "wq": _native.T_WQ,
         "wk": _native.T_WK, "wv": _native.T_WV, "wo": _native.T_WO, "wgate": _native.T_WGATE,
         "wup": _native.T_WUP, "wdown": _native.T_WDOWN}


def shape(cfg, name):
    E, qd, kd = cfg["n_embd"], cfg["n_head"] * cfg["head_dim"], cfg["n_head_kv"] * cfg["head_dim"]
    return {"tok_embd": (cfg["vocab"], E, cfg["etype"]), "output": (cfg["vocab"], E, cfg["etype"]),
            "wq": (qd, E, cfg["wtype"]), "wk": (kd, E, cfg["wtype"]), "wv": (kd, E, cfg["wtype"]),
            "wo": (E, qd, cfg["wtype"]), "wgate": (cfg["n_ff"], E, cfg["wtype"]),
            "wup": (cfg["n_ff"], E, cfg["wtype"]), "wdown": (E, cfg["n_ff"], cfg["wtype"])}[name]


def synth_weights(dev, cfg, seed):
    """The blocks pai_b200_model_synthesize generates, downloaded for the oracle."""
    L = _native.load()
    out = {"attn_norm": [], "ffn_norm": []}
    for name, kind in KINDS.items():
        layers = [0] if name in ("tok_embd", "output") else range(cfg["n_layer"])
        for layer in layers:
            rows, cols, t = shape(cfg, name)
            tmp = dev.alloc(rows * cols * 4)
            blk = dev.alloc(po.row_bytes(t, cols) * rows)
            s = L.pai_b200_tensor_seed(seed, kind, layer)
            _native.check(L.pai_b200_synth_blocks(dev.ctx, t, rows, cols, s, 0.02, tmp.ptr, blk.ptr),
                          "synth_blocks")
            b = blk.download(np.uint8)
            if name in ("tok_embd", "output"):
                out[name] = b
            else:
                out.setdefault(name, []).append(b)
    for _ in range(cfg["n_layer"]):
        out["attn_norm"].append(np.ones(cfg["n_embd"], np.float32))
        out["ffn_norm"].append(np.ones(cfg["n_embd"], np.float32))
    out["output_norm"] = np.ones(cfg["n_embd"], np.float32)
    return out


def oracle_generate(cfg, w, prompt, steps, max_ctx, threads=8):
    s = po.Session(cfg, w, max_ctx, threads=threads)
    tok = None
    for t in prompt:
        tok = s.step(int(t))
    out = [tok]
    for _ in range(steps - 1):
        out.append(s.step(out[-1]))
    hidden = s.hidden()
    s.close()
    return out, hidden


def gpu_generate(sess, prompt, steps):
    tok = None
    for t in prompt:
        tok = sess.step(np.array([t], np.int32))
    out = [int(tok[0])]
    for _ in range(steps - 1):
        out.append(int(sess.step(np.array([out[-1]], np.int32))[0]))
    return out


@pytest.mark.parametrize("wtype", [po.Q4_0, po.Q4_K, po.Q8_0])
def test_greedy_tokens_match_reference_for_64_steps(dev, wtype):
    cfg = dict(SMALL, wtype=wtype)
    seed = 1234 + wtype
    w = synth_weights(dev, cfg, seed)
    prompt = np.random.default_rng(seed).integers(0, cfg["vocab"], 8)
    ref_tokens, ref_hidden = oracle_generate(cfg, w, prompt, 64, 96)
    m = Model(dev, cfg)
    m.synthesize(seed)
    sess = Session(m, 1, 96)
    got = gpu_generate(sess, prompt, 64)
    hidden = sess.hidden()
    sess.close()
    m.close()
    assert got == ref_tokens
    assert np.max(np.abs(hidden - ref_hidden)) <= 1e-3 * np.max(np.abs(ref_hidden))


def test_set_tensor_equals_synthesize(dev):
    cfg = SMALL
    w = synth_weights(dev, cfg, 77)
    m1 = Model(dev, cfg)
    m1.synthesize(77)
    m2 = Model(dev, cfg)
    for name, kind in KINDS.items():
        if name in ("tok_embd", "output"):
            m2.set_tensor(kind, 0, w[name])
        else:
            for layer in range(cfg["n_layer"]):
                m2.set_tensor(kind, layer, w[name][layer])
    for layer in range(cfg["n_layer"]):
        m2.set_tensor(_native.T_ATTN_NORM, layer, w["attn_norm"][layer])
        m2.set_tensor(_native.T_FFN_NORM, layer, w["ffn_norm"][layer])
    m2.set_tensor(_native.T_OUTPUT_NORM, 0, w["output_norm"])
    outs = []
    for m in (m1, m2):
        s = Session(m, 1, 32)
        outs.append([int(s.step(np.array([t], np.int32))[0]) for t in (5, 9, 100, 3)])
        outs.append(s.hidden())
        s.close()
        m.close()
    assert outs[0] == outs[2]
    assert np.array_equal(outs[1], outs[3])


def test_device_resident_run_equals_host_steps(dev):
    m = Model(dev, SMALL)
    m.synthesize(5)
    s = Session(m, 1, 64)
    host = gpu_generate(s, [1, 2, 3], 20)
    s.reset()
    for t in (1, 2):
        s.step(np.array([t], np.int32))
    s.set_tokens(np.array([3], np.int32))
    dev_tokens = []
    for _ in range(20):
        s.run(1)
        dev_tokens.append(int(s.tokens()[0]))
    assert dev_tokens == host
    s.close()
    m.close()


@pytest.mark.parametrize("batch", [2, 4, 8])
def test_batched_sequences_are_independent(dev, batch):
    m = Model(dev, SMALL)
    m.synthesize(9)
    prompts = np.random.default_rng(batch).integers(0, SMALL["vocab"], (batch, 4))
    singles = []
    s1 = Session(m, 1, 64)
    for b in range(batch):
        s1.reset()
        singles.append(gpu_generate(s1, prompts[b], 12))
    s1.close()
    sb = Session(m, batch, 64)
    tok = None
    for p in range(4):
        tok = sb.step(prompts[:, p].astype(np.int32))
    seqs = [[int(t)] for t in tok]
    for _ in range(11):
        tok = sb.step(np.array([s[-1] for s in seqs], np.int32))
        for b in range(batch):
            seqs[b].append(int(tok[b]))
    sb.close()
    m.close()
    assert seqs == singles


def test_session_bounds(dev):
    from prosperoai_b200 import PaiError
    m = Model(dev, SMALL)
    m.synthesize(1)
    s = Session(m, 1, 4)
    with pytest.raises(PaiError) as e:
        s.step(np.array([SMALL["vocab"]], np.int32))
    assert e.value.status == -1
    for _ in range(128):  # max_ctx 4 is rounded up to one 128-position cache block
        s.step(np.array([1], np.int32))
    with pytest.raises(PaiError) as e:
        s.step(np.array([1], np.int32))
    assert e.value.status == -2  # PAI_ERR_NOMEM, as pai_kv_cache_reserve (kv_cache.c:135-137)
    s.close()
    m.close()


@pytest.mark.parametrize("wtype", [po.Q4_0, po.Q4_K, po.Q8_0])
@pytest.mark.parametrize("batch", [1, 4])
def test_persistent_kernel_agrees_with_one_launch_per_op(dev, wtype, batch, monkeypatch):
    """The persistent decode kernel (one cooperative launch for every layer)
    and the one-launch-per-op step compute the same decode: the same greedy
    tokens, hidden states within 1e-4 max-abs-rel (the RMSNorm sums and
    split-K partials are added in different orders)."""
    cfg = dict(SMALL, wtype=wtype)
    m = Model(dev, cfg)
    m.synthesize(31 + wtype)
    monkeypatch.setenv("PAI_B200_PERSISTENT", "0")
    s_op = Session(m, batch, 64)
    monkeypatch.setenv("PAI_B200_PERSISTENT", "1")
    s_pk = Session(m, batch, 64)
    assert s_pk.step_kernels == 4 and s_op.step_kernels > 4
    tok = np.random.default_rng(batch).integers(0, cfg["vocab"], batch).astype(np.int32)
    t_op, t_pk = tok.copy(), tok.copy()
    for i in range(24):
        t_op = s_op.step(t_op)
        t_pk = s_pk.step(t_pk)
        assert np.array_equal(t_op, t_pk), i
        h_op, h_pk = s_op.hidden(), s_pk.hidden()
        assert np.max(np.abs(h_op - h_pk)) <= 1e-4 * np.max(np.abs(h_op)), i
    s_pk.run_layers(2)  # timing entry point: launches only the layer kernel
    dev.sync()
    s_op.close()
    s_pk.close()
    m.close()
