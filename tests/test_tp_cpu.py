"""The tensor-parallel partition on CPU ranks (gloo, world sizes 2 and 4): each rank runs the decode math
of its shard (yalm_b200.tp.shard — the engine's own slice table, read through the C ABI's
yb_tp_shard, host arithmetic only), the wo / w2 partial sums are
exchanged and added in rank order as the engine's kernels do, the logits are gathered, and the
result must equal the unsharded forward pass."""
import os
import socket

import numpy as np
import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _f16(t, y):
    return t.array(y).view(np.float16).astype(np.float32)


def _rms(x, w, eps):
    return x * (1.0 / np.sqrt(np.mean(x.astype(np.float64) ** 2) + eps)).astype(np.float32) * w


def _rope(v, hd, pos, theta):
    out = v.copy()
    for i in range(0, v.size, 2):
        j = i % hd
        f = 1.0 / theta ** (j / hd)
        c, s = np.cos(pos * f), np.sin(pos * f)
        out[i], out[i + 1] = v[i] * c - v[i + 1] * s, v[i] * s + v[i + 1] * c
    return out


def _forward(y, c, toks, rank, world, exchange):
    """Decode math of one rank's shard; exchange(kind, array) -> list of per-rank arrays."""
    from yalm_b200.tp import shard
    sh = shard(c, rank, world)
    t = y.tensors
    hd, gq = c.head_dim, c.n_heads // c.n_kv_heads
    emb = _f16(t["model.embed.weight"], y)
    kc = [[] for _ in range(c.n_layers)]
    vc = [[] for _ in range(c.n_layers)]
    outs = []
    for pos, tok in enumerate(toks):
        x = emb[tok].copy()
        for l in range(c.n_layers):
            p = f"model.layers.{l}."
            xb = _rms(x, t[p + "attn.norm.weight"].array(y), c.norm_eps)
            q = _f16(t[p + "attn.wq.weight"], y)[sh.q_rows] @ xb
            k = _f16(t[p + "attn.wk.weight"], y)[sh.kv_rows] @ xb
            v = _f16(t[p + "attn.wv.weight"], y)[sh.kv_rows] @ xb
            q, k = _rope(q, hd, pos, c.rope_theta), _rope(k, hd, pos, c.rope_theta)
            kc[l].append(k.astype(np.float16).astype(np.float32))
            vc[l].append(v.astype(np.float16).astype(np.float32))
            K, V = np.stack(kc[l]), np.stack(vc[l])
            att = np.zeros_like(q)
            for h in range(q.size // hd):
                g = h // gq
                s = K[:, g * hd:(g + 1) * hd] @ q[h * hd:(h + 1) * hd] / np.sqrt(hd)
                pr = np.exp(s - s.max())
                pr /= pr.sum()
                att[h * hd:(h + 1) * hd] = pr @ V[:, g * hd:(g + 1) * hd]
            part = _f16(t[p + "attn.wo.weight"], y)[:, sh.q_rows] @ att
            for pr_ in exchange("wo", part):
                x = x + pr_
            xb = _rms(x, t[p + "mlp.norm.weight"].array(y), c.norm_eps)
            g1 = _f16(t[p + "mlp.w1.weight"], y)[sh.hidden] @ xb
            g3 = _f16(t[p + "mlp.w3.weight"], y)[sh.hidden] @ xb
            hb = g1 / (1 + np.exp(-g1)) * g3
            part = _f16(t[p + "mlp.w2.weight"], y)[:, sh.hidden] @ hb
            for pr_ in exchange("w2", part):
                x = x + pr_
        xn = _rms(x, t["model.norm.weight"].array(y), c.norm_eps)
        lg = _f16(t["model.output.weight"], y)[sh.vocab] @ xn
        outs.append(np.concatenate(exchange("logits", lg)))
    return np.stack(outs)


def _rank_main(rank, world, port, path, toks, q):
    import torch.distributed as dist
    import torch
    from yalm_b200 import Config, YALMData
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        y = YALMData(path)
        c = Config.from_yalm(y)

        def exchange(kind, a):
            buf = [torch.zeros(a.size, dtype=torch.float32) for _ in range(world)]
            dist.all_gather(buf, torch.from_numpy(np.ascontiguousarray(a, np.float32)))
            return [b.numpy() for b in buf]  # rank order, as the kernels add them

        out = _forward(y, c, toks, rank, world, exchange)
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,kv_heads", [(2, 2), (4, 4)])
def test_tensor_parallel_partition_gloo(tiny_yalm, world, kv_heads):
    import torch.multiprocessing as mp
    from yalm_b200 import Config, YALMData, synth
    # a 2-layer slice of the tiny architecture keeps the numpy reference fast; 4 ranks need 4 kv
    # heads (each GQA group stays whole on one rank)
    path = synth.write_yalm(tiny_yalm.replace(".yalm", f"_2l_kv{kv_heads}.yalm"),
                            synth.shape_with("tiny", n_layers=2, n_kv_heads=kv_heads), seed=0)
    toks = [5, 77, 1200, 3]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, path, toks, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    y = YALMData(path)
    c = Config.from_yalm(y)
    full = _forward(y, c, toks, 0, 1, lambda kind, a: [a])
    for r in range(world):
        assert np.array_equal(res[r], res[0])  # every rank holds identical logits
    # fp32 reassociation of the split dot products only
    assert np.abs(res[0] - full).max() < 2e-4


def test_partition_covers_every_row_once_and_rejects_uneven_worlds():
    """The slices of all ranks tile Wq / Wk / Wv / W1 / W3 / classifier rows exactly once, in rank
    order; a world size that would split a GQA group or the hidden units unevenly is refused."""
    from yalm_b200 import Config, YalmB200Error, synth
    from yalm_b200.tp import shard

    for name in ("mistral-7b", "llama-70b"):
        shp = synth.SHAPES[name]
        c = Config(dim=shp.dim, hidden_dim=shp.hidden_dim, head_dim=shp.head_dim, n_layers=shp.n_layers,
                   n_heads=shp.n_heads, n_kv_heads=shp.n_kv_heads, vocab_size=shp.vocab_size,
                   max_seq_len=4096, rope_theta=shp.rope_theta, rotary_dim=shp.head_dim, act=1)
        for world in (1, 2, 4, 8):
            parts = [shard(c, r, world) for r in range(world)]
            for field, total in (("q_rows", c.n_heads * c.head_dim), ("kv_rows", c.n_kv_heads * c.head_dim),
                                 ("hidden", c.hidden_dim), ("vocab", c.vocab_size)):
                sl = [getattr(p, field) for p in parts]
                assert sl[0].start == 0 and sl[-1].stop == total
                assert all(a.stop == b.start for a, b in zip(sl, sl[1:]))
            # the q heads of a rank are exactly the GQA groups of its kv heads
            gq = c.n_heads // c.n_kv_heads
            for p in parts:
                assert p.q_rows.start == p.kv_rows.start * gq and p.q_rows.stop == p.kv_rows.stop * gq
        with pytest.raises(YalmB200Error):
            shard(c, 0, 16)  # 8 kv heads cannot go to 16 ranks
        with pytest.raises(YalmB200Error):
            shard(c, 0, 3)
