"""A model loaded from a GGUF file (pai_b200_model_load_gguf: blocks as
stored, no dequantisation at import) decodes the same 64 greedy tokens as
the oracle's composed reference decode of the same blocks, with non-unit
norm gains; an untied and a tied lm head (output.weight absent: the
embedding, adapters/llama/llama.c:445-470). The same file converted to a
version-2 .pai container (ggml blocks kept, pai_b200_pai_from_gguf) and
loaded from it (pai_b200_model_load_pai) decodes the same tokens."""
import numpy as np
import pytest

import gguf_writer as gw
from oracle import py_oracle as po
from prosperoai_b200.api import Model, Session, gguf_inspect, pai_from_gguf
from test_gpu_model import SMALL, gpu_generate, oracle_generate, synth_weights

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("wtype,etype,tied", [(po.Q4_0, po.Q8_0, False), (po.Q4_K, po.Q4_0, True)])
def test_gguf_model_matches_oracle(dev, tmp_path, wtype, etype, tied):
    cfg = dict(SMALL, wtype=wtype, etype=etype)
    seed = 4100 + wtype + etype
    w = synth_weights(dev, cfg, seed)
    rng = np.random.default_rng(seed)
    for key in ("attn_norm", "ffn_norm"):
        w[key] = [rng.uniform(0.5, 1.5, cfg["n_embd"]).astype(np.float32) for _ in range(cfg["n_layer"])]
    w["output_norm"] = rng.uniform(0.5, 1.5, cfg["n_embd"]).astype(np.float32)
    if tied:
        w["output"] = w["tok_embd"]
    path = tmp_path / "model.gguf"
    gw.write_llama(path, cfg, w, tied=tied)
    info = gguf_inspect(str(path))
    assert info["tied_output"] == tied and info["cfg"]["wtype"] == wtype
    prompt = rng.integers(0, cfg["vocab"], 6)
    want, want_hidden = oracle_generate(cfg, w, prompt, 64, 80)
    m = Model.from_gguf(dev, str(path))
    sess = Session(m, 1, 80)
    got = gpu_generate(sess, prompt, 64)
    hidden = sess.hidden()
    sess.close()
    m.close()
    assert got == want
    assert np.max(np.abs(hidden - want_hidden)) <= 1e-3 * np.max(np.abs(want_hidden))
    pai = tmp_path / "model.pai"
    pai_from_gguf(str(path), str(pai))
    m = Model.from_pai(dev, str(pai))
    sess = Session(m, 1, 80)
    got_pai = gpu_generate(sess, prompt, 64)
    hidden_pai = sess.hidden()
    sess.close()
    m.close()
    assert got_pai == want
    assert np.array_equal(hidden_pai, hidden)  # the same blocks reach the device
