"""The tensor-parallel shard arithmetic on CPU: two `gloo` ranks each keep the
block of every tensor that tmg_tp_shard (the split the library's loader
applies after tmg_tp_init) assigns them, run forward_token (src/model.rs:
392-491) on their shard with the oracle's kernels, sum the row-split o and
down partials with an allreduce (the two per layer the GPU path issues over
NCCL, at the residual adds of src/model.rs:461-464 and 477-479), gather the
vocab-split logits, and must reproduce the unsharded oracle's logits.

Bar: logits within 1e-4 absolute of the oracle's at every step (the only
change is the order of the o/down sums across the two shards).
"""
import ctypes
import os
import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")
mp = pytest.importorskip("torch.multiprocessing")

ROOT = Path(__file__).resolve().parent.parent
STEPS = 10


def _setup():
    from tinyminigo_b200 import synth

    cfg = synth.CONFIGS["c1"]
    return cfg, synth.make_weights(cfg, 321), synth.random_prompt(cfg["vocab_size"], STEPS, 8)


def shard(cfg, name, rank, world):
    from tinyminigo_b200._lib import Config, check, lib

    c = Config(cfg["hidden_size"], cfg["num_hidden_layers"], cfg["num_attention_heads"],
               cfg["num_key_value_heads"], cfg["head_dim"], cfg["intermediate_size"],
               cfg["vocab_size"], cfg["rms_norm_eps"], cfg["rope_theta"], 0, 0)
    out = (ctypes.c_int64 * 4)()
    check(lib().tmg_tp_shard(ctypes.byref(c), name.encode(), rank, world, out))
    return tuple(out)


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist

    from oracle import oracle as orc
    from tinyminigo_b200 import synth

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg, w, toks = _setup()
        h, d, eps, theta = cfg["hidden_size"], cfg["head_dim"], cfg["rms_norm_eps"], cfg["rope_theta"]
        nq, nkv = cfg["num_attention_heads"] // world, cfg["num_key_value_heads"] // world

        def block(name):
            r0, nr, c0, nc = shard(cfg, name, rank, world)
            a = w[name]
            return np.ascontiguousarray(a.reshape(a.shape[0], -1)[r0:r0 + nr, c0:c0 + nc])

        def allreduce(v):
            t = torch.from_numpy(np.ascontiguousarray(v, np.float32))
            dist.all_reduce(t)
            return t.numpy()

        f32 = synth.bf16_to_f32
        L = cfg["num_hidden_layers"]
        mats = {}
        for layer in range(L):
            p = f"model.layers.{layer}."
            for n in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                      "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"):
                mats[p + n] = block(p + n + ".weight")
        lm = block("lm_head.weight")
        emb = w["model.embed_tokens.weight"]
        ones = np.ones(h, np.float32)  # norm weights of the synthetic model
        kc = [np.zeros((0, nkv * d), np.float32) for _ in range(L)]
        vc = [np.zeros((0, nkv * d), np.float32) for _ in range(L)]
        all_logits = []
        for pos, tok in enumerate(toks):
            x = f32(emb[int(tok)]).copy()
            for layer in range(L):
                p = f"model.layers.{layer}."
                xn = orc.rms_norm(x, ones, eps)
                qv = orc.rope_table_rotate(orc.matmul_w(xn, mats[p + "self_attn.q_proj"]), nq, d, pos, theta)
                kv = orc.rope_table_rotate(orc.matmul_w(xn, mats[p + "self_attn.k_proj"]), nkv, d, pos, theta)
                vv = orc.matmul_w(xn, mats[p + "self_attn.v_proj"])
                kc[layer] = np.vstack([kc[layer], kv[None]])
                vc[layer] = np.vstack([vc[layer], vv[None]])
                att = orc.attention_batch(qv, kc[layer], vc[layer], nq, nkv, d, pos)[0]
                x = x + allreduce(orc.matmul_w(att, mats[p + "self_attn.o_proj"]))
                xn = orc.rms_norm(x, ones, eps)
                g = orc.matmul_w(xn, mats[p + "mlp.gate_proj"])
                u = orc.matmul_w(xn, mats[p + "mlp.up_proj"])
                act = np.array([orc.silu(float(a)) for a in g], np.float32) * u
                x = x + allreduce(orc.matmul_w(act, mats[p + "mlp.down_proj"]))
            part = torch.from_numpy(orc.matmul_w(orc.rms_norm(x, ones, eps), lm))
            parts = [torch.zeros_like(part) for _ in range(world)]
            dist.all_gather(parts, part)
            all_logits.append(torch.cat(parts).numpy())
        q.put((rank, np.stack(all_logits)))
    finally:
        dist.destroy_process_group()


def test_shard_layout_is_the_documented_split():
    cfg, _, _ = _setup()
    h, d, I = cfg["hidden_size"], cfg["head_dim"], cfg["intermediate_size"]
    qd, kd = cfg["num_attention_heads"] * d, cfg["num_key_value_heads"] * d
    V = cfg["vocab_size"]
    for rank in range(2):
        assert shard(cfg, "model.layers.1.self_attn.q_proj.weight", rank, 2) == (rank * qd // 2, qd // 2, 0, h)
        assert shard(cfg, "model.layers.1.self_attn.v_proj.weight", rank, 2) == (rank * kd // 2, kd // 2, 0, h)
        assert shard(cfg, "model.layers.0.self_attn.o_proj.weight", rank, 2) == (0, h, rank * qd // 2, qd // 2)
        assert shard(cfg, "model.layers.0.mlp.up_proj.weight", rank, 2) == (rank * I // 2, I // 2, 0, h)
        assert shard(cfg, "model.layers.0.mlp.down_proj.weight", rank, 2) == (0, h, rank * I // 2, I // 2)
        assert shard(cfg, "lm_head.weight", rank, 2) == (rank * V // 2, V // 2, 0, h)
        assert shard(cfg, "model.embed_tokens.weight", rank, 2) == (0, V, 0, h)
        assert shard(cfg, "model.norm.weight", rank, 2) == (0, h, 0, 1)
    # a world that does not divide the heads is refused
    from tinyminigo_b200._lib import TmgError

    with pytest.raises(TmgError):
        shard(cfg, "lm_head.weight", 0, 3)


def test_two_gloo_ranks_reproduce_the_oracle(orc):
    world, port = 2, 29547
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(60)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    cfg, w, toks = _setup()
    om = orc.OracleModel(cfg, w)
    ref = np.stack([om.forward_token(int(t)) for t in toks])
    for r in range(world):
        assert res[r].shape == ref.shape
        assert np.max(np.abs(res[r] - ref)) < 1e-4, (r, float(np.max(np.abs(res[r] - ref))))
