"""Tensor parallelism (the 8B config's sharding) on 2 GPUs of one node.

Each rank is a process with its own context and GPU; rank 0's NCCL unique
id reaches the other rank through the spawning test.  q/k/v and gate/up are
split by heads and rows, o/down by input columns with one allreduce per
sublayer, the LM head by vocabulary rows with an allgather of the logits.
The model is the c2 shape cut to 2 layers (head counts, intermediate size
and vocabulary all divide by 2).

Bar: every rank produces the same greedy ids as the CPU oracle; the
partial sums of o/down change the summation order, so a step whose top-2
logits differ by less than 1e-3 may flip (the ids must then agree up to
that step and the pick must be the oracle's runner-up; conftest.GreedyCheck
reports the smallest margin met and whether that allowance fired);
first-step logits within 1e-3 relative / 1e-2 absolute.
"""
import ctypes
import json
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available() or torch.cuda.device_count() < 2:  # pragma: no cover
    pytest.skip("needs 2 GPUs", allow_module_level=True)

GOLD = Path(__file__).resolve().parent / "golden"
STEPS = 24


def _setup():
    from tinyminigo_b200 import synth
    d = json.loads((GOLD / "hf_c2_l2.json").read_text())
    cfg = synth.with_layers(synth.CONFIGS["c2"], d["layers"])
    return d, cfg, synth.make_weights(cfg, d["weight_seed"])


def _rank(rank, world, uid, q):
    try:
        import torch as t_

        t_.cuda.set_device(rank)
        from tinyminigo_b200.model import GenParams, Model, ModelConfig, generate

        d, cfg, w = _setup()
        mc = ModelConfig(cfg["hidden_size"], cfg["num_hidden_layers"], cfg["num_attention_heads"],
                         cfg["num_key_value_heads"], cfg["head_dim"], cfg["intermediate_size"],
                         cfg["rms_norm_eps"], cfg["rope_theta"], cfg["vocab_size"], [], 0)
        m = Model.from_tensors(mc, w, device=rank, tp=(uid, rank, world))
        out = generate(m, d["prompt"], GenParams(max_tokens=STEPS))
        q.put((rank, out.tokens, out.logits_first_step))
        m.close()
    except Exception as e:  # pragma: no cover - reported by the parent
        q.put((rank, repr(e), None))


def test_tp2_greedy_matches_oracle(orc, greedy):
    from tinyminigo_b200._lib import check, lib

    uid = (ctypes.c_uint8 * 128)()
    check(lib().tmg_tp_unique_id(uid))
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    world = 2
    procs = [ctx.Process(target=_rank, args=(r, world, bytes(uid), q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, toks, first = q.get(timeout=600)
        res[rank] = (toks, first)
    for p in procs:
        p.join(120)
    for r in range(world):
        assert res[r][1] is not None, f"rank {r} failed: {res[r][0]}"

    d, cfg, w = _setup()
    om = orc.OracleModel(cfg, w)
    ids, margins, second, ref_first = greedy.oracle(om, d["prompt"], STEPS)

    for r in range(world):
        toks, first = res[r]
        assert np.all(np.abs(first - ref_first) <= 1e-2 + 1e-3 * np.abs(ref_first))
        greedy.agree(f"TP2 rank {r}, c2 2-layer", toks, ids, margins, second)
    assert res[0][0] == res[1][0]  # both ranks hold the same (allgathered) result
