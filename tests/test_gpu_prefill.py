"""Prompt prefill (pai_b200_session_prefill): the prompt appended in one
pass per layer (GEMMs over all rows, RoPE + fp16 K/V append for every
position, causal attention over the cache) is equivalent to stepping it.

- with the layer matrices on the batched GEMV (PAI_B200_PREFILL_GEMM=0),
  whose per-row arithmetic is the decode step's: the token after the prompt
  and 24 greedy decode steps after it equal the oracle's stepped decode, for
  1 and 2 sequences (Q8_0, Q4_K layers);
- a prompt prefilled in two calls, and one longer than a pass (several
  passes attending over the cache earlier passes filled), give the tokens
  of the oracle (the same GEMV path: these check the prefill's positions,
  cache layout and passes);
- the default path, the tcgen05 GEMM with bf16 tiles, for Q4_0, Q8_0 and
  Q4_K layers: the hidden state after the prompt is within 2e-2
  (max-abs-rel) of the oracle's, and the next token is the oracle's
  wherever the oracle's top-two logit gap exceeds the error bound.
"""
import numpy as np
import pytest

from oracle import py_oracle as po
from prosperoai_b200.api import Model, Session
from test_gpu_model import SMALL, synth_weights

pytestmark = pytest.mark.gpu


def oracle_run(cfg, w, prompt, steps, max_ctx, want_logits=False):
    s = po.Session(cfg, w, max_ctx, threads=8)
    tok, logits = None, None
    for t in prompt:
        if want_logits:
            tok, logits = s.step(int(t), want_logits=True)
        else:
            tok = s.step(int(t))
    hidden = s.hidden()
    out = [tok]
    for _ in range(steps):
        out.append(s.step(out[-1]))
    s.close()
    return out, hidden, logits


def gpu_decode(sess, first, steps):
    out = [list(first)]
    for _ in range(steps):
        out.append(list(sess.step(np.array(out[-1], np.int32))))
    return out


@pytest.mark.parametrize("wtype,batch", [(po.Q8_0, 1), (po.Q4_K, 2)])
def test_prefill_then_decode_matches_stepped_oracle(dev, wtype, batch, monkeypatch):
    monkeypatch.setenv("PAI_B200_PREFILL_GEMM", "0")
    cfg = dict(SMALL, wtype=wtype)
    seed = 5100 + wtype
    w = synth_weights(dev, cfg, seed)
    rng = np.random.default_rng(seed)
    P, steps, max_ctx = 37, 24, 80
    prompts = rng.integers(0, cfg["vocab"], (batch, P))
    m = Model(dev, cfg)
    m.synthesize(seed)
    sess = Session(m, batch, max_ctx)
    first = sess.prefill(prompts)
    assert sess.pos == P
    got = gpu_decode(sess, first, steps)
    sess.close()
    m.close()
    for b in range(batch):
        want, _, _ = oracle_run(cfg, w, prompts[b], steps, max_ctx)
        assert [t[b] for t in got] == want, f"sequence {b}"


def test_prefill_in_parts_and_in_several_passes(dev, monkeypatch):
    monkeypatch.setenv("PAI_B200_PREFILL_GEMM", "0")
    cfg = dict(SMALL, wtype=po.Q8_0)
    seed = 5200
    w = synth_weights(dev, cfg, seed)
    rng = np.random.default_rng(seed)
    m = Model(dev, cfg)
    m.synthesize(seed)
    # two calls: 13 then 21 positions
    prompt = rng.integers(0, cfg["vocab"], 34)
    sess = Session(m, 1, 64)
    sess.prefill(prompt[None, :13])
    first = sess.prefill(prompt[None, 13:])
    got = gpu_decode(sess, first, 8)
    sess.close()
    want, _, _ = oracle_run(cfg, w, prompt, 8, 64)
    assert [t[0] for t in got] == want
    # 8 sequences of 300 positions: 2400 rows, more than one pass holds
    prompts = rng.integers(0, cfg["vocab"], (8, 300))
    sess = Session(m, 8, 310)
    first = sess.prefill(prompts)
    sess.close()
    m.close()
    for b in (0, 5, 7):
        want, _, _ = oracle_run(cfg, w, prompts[b], 0, 310)
        assert first[b] == want[0], f"sequence {b}"


@pytest.mark.parametrize("wtype", [po.Q4_0, po.Q8_0, po.Q4_K])
def test_prefill_gemm_within_bf16_bound(dev, wtype):
    cfg = dict(SMALL, wtype=wtype)
    seed = 5300 + wtype
    w = synth_weights(dev, cfg, seed)
    rng = np.random.default_rng(seed)
    P, max_ctx = 96, 128
    prompt = rng.integers(0, cfg["vocab"], P)
    m = Model(dev, cfg)
    m.synthesize(seed)
    sess = Session(m, 1, max_ctx)
    first = sess.prefill(prompt[None, :])
    hidden = sess.hidden()
    sess.close()
    m.close()
    want, want_hidden, logits = oracle_run(cfg, w, prompt, 0, max_ctx, want_logits=True)
    err = float(np.max(np.abs(hidden - want_hidden)) / np.max(np.abs(want_hidden)))
    assert err <= 2e-2, err
    top = np.sort(logits)[-2:]
    if top[1] - top[0] > 4 * err * np.max(np.abs(logits)):
        assert first[0] == want[0]
