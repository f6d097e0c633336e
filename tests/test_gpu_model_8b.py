"""Decoder parity at the benchmark's shapes.

- The Llama-3-8B-shaped Q4_0 model of the headline benchmark (32 layers,
  n_embd 4096, 32/8 heads, n_ff 14336, vocab 128256, Q8_0 embedding and
  lm head): 64 greedy tokens of the CUDA decode equal the oracle's composed
  reference decode (the op order of adapters/llama/llama.c:669-797, greedy
  rule of models/sampler.c:89-99) on the same synthetic weights. The
  oracle's top-1/top-2 logit gap of every step is printed, so a mismatch
  can be told apart from a near tie.
- One decoder layer of that shape (benchmark config 4) over a cache of 4096
  past positions drawn N(0, 1) in fp16: the hidden state after each of 8
  steps is within 1e-3 max-abs-rel of the oracle's, and the tokens agree.
- KV-cache position accounting with the reference's pai_kv_cache_reserve
  semantics (cache/kv_cache.c:125-152).
"""
import os

import numpy as np
import pytest

from oracle import py_oracle as po
from prosperoai_b200 import PaiError
from prosperoai_b200.api import Model, Session
from test_gpu_model import SMALL, gpu_generate, synth_weights

pytestmark = pytest.mark.gpu

CFG_8B = dict(n_layer=32, n_embd=4096, n_head=32, n_head_kv=8, head_dim=128, n_ff=14336,
              vocab=128256, eps=1e-5, rope_theta=500000.0, wtype=po.Q4_0, etype=po.Q8_0)
THREADS = max(8, os.cpu_count() or 8)


def top2_gap(logits):
    i = int(np.argmax(logits))
    rest = np.delete(logits, i)
    return float(logits[i] - np.max(rest))


@pytest.fixture(scope="module")
def oracle_8b_run(dev):
    """The oracle's 64 greedy tokens, top-1/top-2 gaps and final hidden state
    for the 8B-shaped model (computed once for both step paths)."""
    cfg, seed, steps = CFG_8B, 88, 64
    prompt = [int(t) for t in np.random.default_rng(seed).integers(0, cfg["vocab"], 8)]
    max_ctx = len(prompt) + steps
    w = synth_weights(dev, cfg, seed)
    ref = po.Session(cfg, w, max_ctx, threads=THREADS)
    want, gaps = [], []
    tok = None
    for t in prompt:
        tok, logits = ref.step(t, want_logits=True)
    want.append(tok)
    gaps.append(top2_gap(logits))
    for _ in range(steps - 1):
        tok, logits = ref.step(want[-1], want_logits=True)
        want.append(tok)
        gaps.append(top2_gap(logits))
    ref_hidden = ref.hidden()
    ref.close()
    print(f"oracle top-1/top-2 logit gaps: min {min(gaps):.3e}, median {np.median(gaps):.3e}")
    return dict(cfg=cfg, seed=seed, prompt=prompt, max_ctx=max_ctx, want=want, gaps=gaps, hidden=ref_hidden)


@pytest.mark.parametrize("persistent", [False, True])
def test_8b_shape_greedy_tokens_match_reference_for_64_steps(dev, oracle_8b_run, persistent, monkeypatch):
    o = oracle_8b_run
    monkeypatch.setenv("PAI_B200_PERSISTENT", "1" if persistent else "0")
    m = Model(dev, o["cfg"])
    m.synthesize(o["seed"])
    s = Session(m, 1, o["max_ctx"])
    assert (s.step_kernels == 4) == persistent
    got = gpu_generate(s, o["prompt"], 64)
    hidden = s.hidden()
    s.close()
    m.close()
    want, gaps = o["want"], o["gaps"]
    first_bad = next((i for i, (a, b) in enumerate(zip(got, want)) if a != b), None)
    assert got == want, f"first mismatch at step {first_bad}, oracle gap there {gaps[first_bad]:.3e}"
    assert np.max(np.abs(hidden - o["hidden"])) <= 1e-3 * np.max(np.abs(o["hidden"]))


@pytest.mark.parametrize("persistent", [False, True])
def test_config4_layer_over_4096_position_cache(dev, persistent, monkeypatch):
    monkeypatch.setenv("PAI_B200_PERSISTENT", "1" if persistent else "0")
    cfg = dict(CFG_8B, n_layer=1, vocab=2048)
    seed, past, steps = 404, 4096, 8
    max_ctx = past + 128
    w = synth_weights(dev, cfg, seed)
    rng = np.random.default_rng(seed)
    hk, hd = cfg["n_head_kv"], cfg["head_dim"]
    k = rng.standard_normal((hk, past, hd)).astype(np.float16)
    v = rng.standard_normal((hk, past, hd)).astype(np.float16)
    ref = po.Session(cfg, w, max_ctx, threads=THREADS)
    ref.set_kv(0, k.view(np.uint16), v.view(np.uint16))
    ref.seek(past)
    m = Model(dev, cfg)
    m.synthesize(seed)
    s = Session(m, 1, max_ctx)
    assert s.kv_reserve(past) == 0
    s.write_kv(0, 0, k, v)
    tok_ref = tok_gpu = 17
    for i in range(steps):
        tok_ref = ref.step(tok_ref)
        tok_gpu = int(s.step(np.array([tok_gpu], np.int32))[0])
        h_ref, h_gpu = ref.hidden(), s.hidden()
        err = float(np.max(np.abs(h_gpu - h_ref)) / np.max(np.abs(h_ref)))
        assert err <= 1e-3, (i, err)
        assert tok_gpu == tok_ref, i
    assert s.pos == past + steps
    s.close()
    m.close()
    ref.close()


def test_kv_reserve_semantics(dev):
    m = Model(dev, SMALL)
    m.synthesize(3)
    s = Session(m, 2, 130)
    info = s.kv_info()
    assert info["capacity_tokens"] == 256 and info["block_tokens"] == 128  # whole blocks
    assert info["positions"] == 0 and info["batch"] == 2
    assert info["head_stride"] == 256 * 128 and info["seq_stride"] == 2 * 256 * 128
    with pytest.raises(PaiError) as e:
        s.kv_reserve(0)
    assert e.value.status == -1  # PAI_ERR_INVALID_ARG
    assert s.kv_reserve(100) == 0
    assert s.kv_reserve(28) == 100
    with pytest.raises(PaiError) as e:
        s.kv_reserve(129)
    assert e.value.status == -2  # PAI_ERR_NOMEM, as pai_kv_cache_reserve
    assert s.kv_info()["positions"] == 128 and s.kv_info()["stats_blocks"] == 2
    s.step(np.array([1, 2], np.int32))  # a decode step reserves its position
    assert s.pos == 129 and s.kv_info()["stats_blocks"] == 3
    s.reset()
    assert s.kv_info()["positions"] == 0 and s.kv_info()["stats_blocks"] == 0
    s.close()
    m.close()
