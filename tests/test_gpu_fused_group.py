"""Greedy decode of one sequence spread over 2, 4 or 8 GPUs by the fused decode
kernel (tmg_fused_group_init): the row groups and attention items of every
phase are dealt over all the GPUs' SMs, and every exchanged value, KV-cache
row and argmax candidate is written into every GPU's memory over NVLink.

Each rank is a process with its own context holding the full weights; rank
0's NCCL unique id reaches the other ranks through the spawning test.  Each
output row is computed whole on one GPU, so the tokens must be identical,
bit for bit, to the same decode on one GPU (which each rank runs first on
a cache of its own), and the same on every rank; the single-GPU tokens are
checked against the CPU oracle (generate's argmax loop, src/model.rs:
614-663) with conftest.GreedyCheck.  Shapes: the 8B-class instance (C4
shape, 2 layers, on 2, 4 and 8 GPUs as the box has them) and the 1B-class
one (c2 shape, 2 layers, 2 GPUs: its O phase has 256 row groups, so each
GPU runs 128 CTAs).
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available() or torch.cuda.device_count() < 2:  # pragma: no cover
    pytest.skip("needs 2 GPUs", allow_module_level=True)

STEPS = 40
PROMPT = 40


def _setup(which):
    from tinyminigo_b200 import synth

    cfg = synth.with_layers(synth.CONFIGS[which], 2)
    return cfg, synth.random_prompt(cfg["vocab_size"], PROMPT, 61)


def _rank(which, rank, world, uid, q):
    try:
        import torch as t_

        t_.cuda.set_device(rank)
        from tinyminigo_b200 import synth
        from tinyminigo_b200.model import Model, ModelConfig

        cfg, prompt = _setup(which)
        w = synth.make_weights(cfg, 62, device="cuda")
        mc = ModelConfig(cfg["hidden_size"], cfg["num_hidden_layers"], cfg["num_attention_heads"],
                         cfg["num_key_value_heads"], cfg["head_dim"], cfg["intermediate_size"],
                         cfg["rms_norm_eps"], cfg["rope_theta"], cfg["vocab_size"], [], 0)
        m = Model.from_tensors(mc, w, device=rank)
        cap = PROMPT + 2 * STEPS + 8
        # the same decode on this GPU alone first
        solo = m.new_cache(cap)
        tok0 = int(np.argmax(m.forward_seq(prompt, solo)))
        ids_solo = m.decode([tok0], solo, STEPS)[0].tolist()
        solo.close()
        cache = m.new_cache(cap)
        m.forward_seq(prompt, cache)
        m.fused_group(cache, uid, rank, world)
        ids_a = m.decode([tok0], cache, STEPS // 2)[0].tolist()  # two launches in a row
        ids_b = m.decode([ids_a[-1]], cache, STEPS - STEPS // 2)[0].tolist()
        q.put((rank, tok0, ids_solo, ids_a + ids_b))
        cache.close()
        m.close()
    except Exception as e:  # pragma: no cover - reported by the parent
        q.put((rank, None, repr(e), None))


@pytest.mark.parametrize("which,world", [("c4", 2), ("c2", 2), ("c4", 4), ("c4", 8)])
def test_fused_group_matches_one_gpu(orc, greedy, which, world):
    from tinyminigo_b200 import synth
    from tinyminigo_b200._lib import check, lib

    if torch.cuda.device_count() < world:  # pragma: no cover
        pytest.skip(f"needs {world} GPUs")
    uid = (ctypes.c_uint8 * 128)()
    check(lib().tmg_tp_unique_id(uid))
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(which, r, world, bytes(uid), q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            rank, tok0, solo, grp = q.get(timeout=600)
            res[rank] = (tok0, solo, grp)
    finally:
        for p in procs:
            p.join(120)
            if p.is_alive():  # pragma: no cover
                p.kill()
    for r in range(world):
        assert res[r][0] is not None, f"rank {r} failed: {res[r][1]}"
    for r in range(world):
        tok0, solo, grp = res[r]
        assert grp == solo, f"rank {r}: the {world}-GPU decode differs from one GPU's"
        assert res[r] == res[0]
    cfg, prompt = _setup(which)
    w = synth.make_weights(cfg, 62, device="cuda")
    ids, margins, second, _ = greedy.oracle(orc.OracleModel(cfg, w), prompt, STEPS + 1)
    tok0, solo, _ = res[0]
    greedy.agree(f"{which} shape, 2 layers, fused on {world} GPUs", [tok0] + solo, ids, margins,
                 second)
