"""Failure detection without a GPU fault.

1. A bounded device-side wait gives up.  Every wait of the fused decode
   kernel is bounded and ends the launch with the context's timeout error
   word.  The test option TMG_TEST_FUSED_STALL=<phase> makes the next fused
   launch of a context wait, in that phase of its first step, for a tag that
   no phase writes (TMG_TEST_FUSED_POLL_MS bounds the poll).  generate must
   return TMG_ERR_TIMEOUT quickly, every CTA must leave (the call returns),
   and the same context must then decode correctly.
2. A peer never joins.  tmg_tp_init on rank 0 of a world of 2 whose rank 1
   never starts must return TMG_ERR_NCCL within TMG_TP_TIMEOUT_S instead of
   blocking (the communicator is non-blocking; nothing runs on the GPU).
   It runs in a child process so the aborted NCCL state stays there.

Reference: errors surface as anyhow::Result (src/main.rs:19-24).
"""
import ctypes
import json
import os
import time
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a GPU", allow_module_level=True)

from tinyminigo_b200 import synth  # noqa: E402
from tinyminigo_b200._lib import TmgError  # noqa: E402
from tinyminigo_b200.model import GenParams, Model, ModelConfig, generate  # noqa: E402

GOLD = Path(__file__).resolve().parent / "golden"
TMG_ERR_TIMEOUT = -6
TMG_ERR_NCCL = -7


def cfg_obj(cfg):
    return ModelConfig(cfg["hidden_size"], cfg["num_hidden_layers"], cfg["num_attention_heads"],
                       cfg["num_key_value_heads"], cfg["head_dim"], cfg["intermediate_size"],
                       cfg["rms_norm_eps"], cfg["rope_theta"], cfg["vocab_size"], [], 0)


def test_fused_wait_gives_up_and_the_context_recovers(orc, greedy):
    d = json.loads((GOLD / "hf_c2_l2.json").read_text())
    cfg = synth.with_layers(synth.CONFIGS["c2"], d["layers"])
    t = synth.make_weights(cfg, d["weight_seed"])
    os.environ["TMG_TEST_FUSED_STALL"] = "2"  # layer 0's O phase (its att gather)
    os.environ["TMG_TEST_FUSED_POLL_MS"] = "50"
    try:
        m = Model.from_tensors(cfg_obj(cfg), t)
    finally:
        del os.environ["TMG_TEST_FUSED_STALL"]
        del os.environ["TMG_TEST_FUSED_POLL_MS"]
    t0 = time.perf_counter()
    with pytest.raises(TmgError) as ei:
        generate(m, d["prompt"], GenParams(max_tokens=8))
    waited = time.perf_counter() - t0
    assert ei.value.code == TMG_ERR_TIMEOUT, str(ei.value)
    assert waited < 30.0, waited
    # the next call on the same context runs normally
    out = generate(m, d["prompt"], GenParams(max_tokens=8))
    ids, margins, second, _ = greedy.oracle(orc.OracleModel(cfg, t), d["prompt"], 8)
    greedy.agree("after a timed-out fused launch", out.tokens, ids, margins, second)
    m.close()


def _lonely_rank(q):
    try:
        os.environ["TMG_TP_TIMEOUT_S"] = "3"
        from tinyminigo_b200._lib import Config, lib

        L = lib()
        cfg = Config(64, 2, 4, 2, 16, 128, 32000, 1e-6, 10000.0, 0, 0)
        ctx = ctypes.c_void_p()
        rc = L.tmg_create(0, ctypes.byref(cfg), ctypes.byref(ctx))
        if rc != 0:
            q.put(("create", rc, "", 0.0, 0))
            return
        uid = (ctypes.c_uint8 * 128)()
        rc = L.tmg_tp_unique_id(uid)
        if rc != 0:
            q.put(("unique id", rc, "", 0.0, 0))
            return
        t0 = time.perf_counter()
        rc = L.tmg_tp_init(ctx, uid, 0, 2)  # rank 1 never starts
        waited = time.perf_counter() - t0
        msg = L.tmg_last_error(ctx).decode()
        q.put(("init", rc, msg, waited, L.tmg_destroy(ctx)))
    except Exception as e:  # pragma: no cover - reported by the parent
        q.put(("exception", -100, repr(e), 0.0, 0))


def test_tp_init_without_peer_times_out():
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely_rank, args=(q,))
    p.start()
    try:
        what, rc, msg, waited, destroyed = q.get(timeout=240)
    finally:
        p.join(60)
        if p.is_alive():  # pragma: no cover - a host-side hang; nothing runs on the GPU
            p.kill()
    assert what == "init", (what, rc, msg)
    assert rc == TMG_ERR_NCCL, (rc, msg)
    assert "did not join" in msg, msg
    assert 2.5 < waited < 60.0, waited
    assert destroyed == 0
