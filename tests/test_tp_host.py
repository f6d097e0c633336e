"""Host side of tensor parallelism, on CPU with 2 gloo ranks (no GPU).

- the communicator id made on rank 0 reaches every rank unchanged;
- the sharding plan of the model loader (csrc/host/b200_model.c
  pack_tensor: q/k/v rows by head block, o and down by input columns,
  gate/up rows, lm head by vocabulary rows) plus the two exchange steps
  (sum of the row-parallel partial outputs, merge of per-shard
  (maximum, index) pairs in rank order) reproduces the unsharded layer and
  the first index of the global maximum, here in float64 numpy;
- a rank that raises before joining makes the others fail at their next
  collective within the process-group timeout instead of hanging.
"""
import datetime
import multiprocessing as mp
import os
import socket

import numpy as np

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn(fn, *args, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=fn, args=(r, port, q) + args) for r in range(WORLD)]
    for p in ps:
        p.start()
    out = {}
    try:
        for _ in range(WORLD):
            r = q.get(timeout=timeout)
            out[r["rank"]] = r
    finally:
        for p in ps:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
                p.join()
    return out


def _init(rank, port, seconds=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=seconds))
    return dist


def _id_worker(rank, port, q):
    dist = _init(rank, port)
    from prosperoai_b200.api import share_tp_id
    got = share_tp_id(rank, lambda: bytes((i * 7 + 3) % 256 for i in range(128)))
    dist.destroy_process_group()
    q.put({"rank": rank, "id": got})


def test_unique_id_reaches_every_rank():
    res = _spawn(_id_worker)
    want = bytes((i * 7 + 3) % 256 for i in range(128))
    for r in range(WORLD):
        assert res[r]["id"] == want


def _rmsnorm(x, eps=1e-5):
    return x / np.sqrt(np.mean(x * x) + eps)


def _layer_full(x, W, cfg):
    """One decoder MLP + attention-output block at position 0 (attention over
    a single position returns v), unsharded, float64."""
    hd, H, HK = cfg["hd"], cfg["H"], cfg["HK"]
    xn = _rmsnorm(x)
    q, k, v = W["wq"] @ xn, W["wk"] @ xn, W["wv"] @ xn
    att = np.concatenate([v[(h // (H // HK)) * hd:(h // (H // HK) + 1) * hd] for h in range(H)])
    x = x + W["wo"] @ att
    xn = _rmsnorm(x)
    g, u = W["wgate"] @ xn, W["wup"] @ xn
    x = x + W["wdown"] @ (g / (1 + np.exp(-g)) * u)
    return x, W["out"] @ _rmsnorm(x)


def _shard(W, cfg, r, n):
    hd, H, HK, F, V = cfg["hd"], cfg["H"], cfg["HK"], cfg["F"], cfg["V"]
    hl, hkl, fl, vl = H // n, HK // n, F // n, V // n
    return {"wq": W["wq"][r * hl * hd:(r + 1) * hl * hd], "wk": W["wk"][r * hkl * hd:(r + 1) * hkl * hd],
            "wv": W["wv"][r * hkl * hd:(r + 1) * hkl * hd], "wo": W["wo"][:, r * hl * hd:(r + 1) * hl * hd],
            "wgate": W["wgate"][r * fl:(r + 1) * fl], "wup": W["wup"][r * fl:(r + 1) * fl],
            "wdown": W["wdown"][:, r * fl:(r + 1) * fl], "out": W["out"][r * vl:(r + 1) * vl], "v0": r * vl}


def _model(seed):
    cfg = dict(hd=8, H=4, HK=2, E=32, F=64, V=96)
    rng = np.random.default_rng(seed)
    E, hd, H, HK, F, V = cfg["E"], cfg["hd"], cfg["H"], cfg["HK"], cfg["F"], cfg["V"]
    W = {"wq": rng.normal(0, 0.3, (H * hd, E)), "wk": rng.normal(0, 0.3, (HK * hd, E)),
         "wv": rng.normal(0, 0.3, (HK * hd, E)), "wo": rng.normal(0, 0.3, (E, H * hd)),
         "wgate": rng.normal(0, 0.3, (F, E)), "wup": rng.normal(0, 0.3, (F, E)),
         "wdown": rng.normal(0, 0.3, (E, F)), "out": rng.normal(0, 0.3, (V, E))}
    return cfg, W, rng.normal(0, 1, E)


def _decomp_worker(rank, port, q):
    dist = _init(rank, port)
    import torch
    cfg, W, x = _model(11)
    S = _shard(W, cfg, rank, WORLD)
    hd, hl, hkl = cfg["hd"], cfg["H"] // WORLD, cfg["HK"] // WORLD
    g = hl // hkl
    xn = _rmsnorm(x)
    v = S["wv"] @ xn  # this rank's kv heads; q/k unused at one position
    att = np.concatenate([v[(h // g) * hd:(h // g + 1) * hd] for h in range(hl)])
    t = torch.from_numpy(S["wo"] @ att)  # row-parallel partial
    dist.all_reduce(t)
    x = x + t.numpy()
    xn = _rmsnorm(x)
    gg, uu = S["wgate"] @ xn, S["wup"] @ xn
    t = torch.from_numpy(S["wdown"] @ (gg / (1 + np.exp(-gg)) * uu))
    dist.all_reduce(t)
    x = x + t.numpy()
    logits = S["out"] @ _rmsnorm(x)
    i = int(np.argmax(logits))
    pair = torch.tensor([logits[i], float(i + S["v0"])], dtype=torch.float64)
    pairs = [torch.zeros(2, dtype=torch.float64) for _ in range(WORLD)]
    dist.all_gather(pairs, pair)
    best, bidx = -np.inf, -1
    for p in pairs:  # ranks in order: a later shard wins only with a larger value
        if bidx < 0 or p[0].item() > best:
            best, bidx = p[0].item(), int(p[1].item())
    dist.destroy_process_group()
    q.put({"rank": rank, "x": x, "tok": bidx})


def test_tp_decomposition_matches_unsharded():
    cfg, W, x = _model(11)
    want_x, want_logits = _layer_full(x, W, cfg)
    res = _spawn(_decomp_worker)
    for r in range(WORLD):
        np.testing.assert_allclose(res[r]["x"], want_x, rtol=1e-12, atol=1e-12)
        assert res[r]["tok"] == int(np.argmax(want_logits))


def _fail_worker(rank, port, q):
    dist = _init(rank, port, seconds=5)
    import torch
    try:
        if rank == 1:
            raise RuntimeError("rank 1 fails before the collective")
        t = torch.ones(4)
        dist.all_reduce(t)
        q.put({"rank": rank, "outcome": "completed"})
    except RuntimeError as e:
        q.put({"rank": rank, "outcome": "error", "msg": str(e)[:200]})


def test_failed_rank_surfaces_as_error():
    res = _spawn(_fail_worker, timeout=90)
    assert res[1]["outcome"] == "error"
    assert res[0]["outcome"] == "error"  # the collective timed out instead of hanging
