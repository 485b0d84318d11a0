"""The fused batch-1 decode kernel (decode_fused.cu) through the C ABI.

Greedy generate and tmg_decode on one stream run every step inside
decode_fused_kernel (one persistent launch per call), so these tests pin
that kernel against the HF golden vectors of the c2 shape (2 layers), the
CPU oracle over a long context (many attention splits and merges), the
plain per-step forward path, EOS handling, and the shape of its trace.

Bar: greedy ids identical; the first-step logits within 1e-3 relative /
1e-2 absolute.  A greedy step whose top-2 logits differ by less than 1e-3
(in the oracle) is decided by summation order, which the GPU's parallel
sums change; the sequences must then agree up to that step, and the GPU's
pick there must be the oracle's runner-up (conftest.GreedyCheck, which
reports every comparison's smallest margin and whether that allowance
fired).
"""
import json
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a GPU", allow_module_level=True)

from tinyminigo_b200 import synth  # noqa: E402
from tinyminigo_b200.model import GenParams, Model, ModelConfig, generate  # noqa: E402

GOLD = Path(__file__).resolve().parent / "golden"


def cfg_obj(cfg, eos=()):
    return ModelConfig(cfg["hidden_size"], cfg["num_hidden_layers"], cfg["num_attention_heads"],
                       cfg["num_key_value_heads"], cfg["head_dim"], cfg["intermediate_size"],
                       cfg["rms_norm_eps"], cfg["rope_theta"], cfg["vocab_size"], list(eos), 0)


@pytest.fixture(scope="module")
def c2l2():
    d = json.loads((GOLD / "hf_c2_l2.json").read_text())
    cfg = synth.with_layers(synth.CONFIGS["c2"], d["layers"])
    t = synth.make_weights(cfg, d["weight_seed"])  # CPU draws, as the golden file
    return d, cfg, t


def first_divergence(a, b):
    return next((i for i, (x, y) in enumerate(zip(a, b)) if x != y), None)


def test_fused_generate_matches_hf_golden(orc, greedy, c2l2):
    d, cfg, t = c2l2
    m = Model.from_tensors(cfg_obj(cfg), t)
    n = len(d["greedy"])
    out = generate(m, d["prompt"], GenParams(max_tokens=n))
    ids, margins, second, _ = greedy.oracle(orc.OracleModel(cfg, t), d["prompt"], n)
    assert ids == d["greedy"]  # the oracle reproduces the HF golden ids
    greedy.agree("c2 2-layer HF golden (fused)", out.tokens, ids, margins, second)
    top5 = np.argsort(-out.logits_first_step)[:5].tolist()
    assert top5 == d["top5_ids"]
    assert np.allclose(out.logits_first_step[:16], d["first_logits_head"], rtol=1e-3, atol=1e-2)
    m.close()


def test_fused_long_context_matches_oracle(orc, greedy, c2l2):
    # 64-token prompt + 300 greedy steps: up to 364 positions, so the kernel
    # goes from 3 to 12 attention splits per kv head with merges
    d, cfg, t = c2l2
    prompt = synth.random_prompt(cfg["vocab_size"], 64, 3)
    om = orc.OracleModel(cfg, t)
    steps = 300
    ids, margins, second, _ = greedy.oracle(om, prompt, steps)
    m = Model.from_tensors(cfg_obj(cfg), t)
    out = generate(m, prompt, GenParams(max_tokens=steps))
    greedy.agree("c2 2-layer 300 steps (fused)", out.tokens, ids, margins, second)
    m.close()


def test_fused_decode_matches_plain_forward(c2l2):
    # tmg_decode (fused kernel) against forward_token + argmax (per-step
    # graph of separate kernels) from the same prefilled cache
    d, cfg, t = c2l2
    m = Model.from_tensors(cfg_obj(cfg), t)
    prompt = synth.random_prompt(cfg["vocab_size"], 40, 5)
    steps = 64
    c1 = m.new_cache(256)
    tok0 = int(np.argmax(m.forward_seq(prompt, c1)))
    fused = m.decode([tok0], c1, steps)[0].tolist()
    c2 = m.new_cache(256)
    m.forward_seq(prompt, c2)
    plain, tok = [], tok0
    for _ in range(steps):
        logits = m.forward_token(tok, c2)
        tok = int(np.argmax(logits))
        plain.append(tok)
    i = first_divergence(fused, plain)
    assert i is None, f"fused and plain diverged at step {i}: {fused[i]} vs {plain[i]}"
    c1.close()
    c2.close()
    m.close()


def test_fused_stops_on_eos_like_reference(orc, c2l2):
    d, cfg, t = c2l2
    eos = d["greedy"][4]  # the 5th greedy token (steps 0-4 have clear margins)
    om = orc.OracleModel(cfg, t)
    ref, _, _, _ = om.generate(d["prompt"], 12, eos=[eos])
    m = Model.from_tensors(cfg_obj(cfg, eos=[eos]), t)
    out = generate(m, d["prompt"], GenParams(max_tokens=12))
    assert out.tokens == ref.tolist()
    assert out.tokens[-1] == eos and len(out.tokens) == 5
    m.close()


def test_fused_trace_is_well_formed(c2l2):
    d, cfg, t = c2l2
    m = Model.from_tensors(cfg_obj(cfg), t)
    cache = m.new_cache(128)
    tok = int(np.argmax(m.forward_seq(d["prompt"], cache)))
    tr = m.trace_fused(tok, cache)
    L = cfg["num_hidden_layers"]
    n_ctas, nph, words = tr.shape
    assert nph == 5 * L + 1 and words == 12 and n_ctas >= 1
    # every CTA enters every phase, in order
    entry = tr[:, :, 0].astype(np.int64)
    assert np.all(entry > 0)
    assert np.all(np.diff(entry, axis=1) >= 0)
    # the GEMV phases deal all row groups: QKV (3072 rows / 8), O (2048 / 8),
    # GU (8192 / 4), DOWN (2048 / 2), LM head (vocab / 8)
    groups = tr[:, :, 7].astype(np.int64).sum(axis=0)
    V = cfg["vocab_size"]
    for layer in range(L):
        assert groups[5 * layer + 0] == 3072 // 8
        assert groups[5 * layer + 2] == 2048 // 8
        assert groups[5 * layer + 3] == 8192 // 4
        assert groups[5 * layer + 4] == 2048 // 2
    assert groups[5 * L] == (V + 7) // 8
    cache.close()
    m.close()


def test_fused_head_dim_128_matches_oracle(orc, greedy):
    # the head-dim-128 kernel instance: 16 query heads of 128 over 4 kv heads
    # (n_q * d = hidden = 2048), 2 layers, a 40-token prompt and 48 greedy
    # steps against the oracle
    cfg = dict(synth.CONFIGS["c2"])
    cfg.update(num_attention_heads=16, num_key_value_heads=4, head_dim=128,
               vocab_size=32000, num_hidden_layers=2)
    t = synth.make_weights(cfg, 11)
    prompt = synth.random_prompt(cfg["vocab_size"], 40, 12)
    steps = 48
    ids, margins, second, _ = greedy.oracle(orc.OracleModel(cfg, t), prompt, steps)
    m = Model.from_tensors(cfg_obj(cfg), t)
    out = generate(m, prompt, GenParams(max_tokens=steps))
    greedy.agree("head dim 128, 2 layers (fused)", out.tokens, ids, margins, second)
    c = m.new_cache(128)
    tok0 = int(np.argmax(m.forward_seq(prompt, c)))
    tr = m.trace_fused(tok0, c)  # the fused kernel ran for this shape
    assert tr.shape[1] == 5 * 2 + 1
    c.close()
    m.close()


def test_fused_8b_shape_matches_oracle(orc, greedy):
    # the 8B-class kernel instance (hidden 4096, head dim 128, 32 / 8 heads,
    # intermediate 14336: 4 rows per stage, the down rows one per stage, act
    # gathered in two pieces), 2 layers of the C4 shape, 48 greedy steps
    cfg = synth.with_layers(synth.CONFIGS["c4"], 2)
    t = synth.make_weights(cfg, 44, device="cuda")
    prompt = synth.random_prompt(cfg["vocab_size"], 40, 45)
    steps = 48
    ids, margins, second, first = greedy.oracle(orc.OracleModel(cfg, t), prompt, steps)
    m = Model.from_tensors(cfg_obj(cfg), t)
    out = generate(m, prompt, GenParams(max_tokens=steps))
    greedy.agree("C4 shape, 2 layers (fused, 8B instance)", out.tokens, ids, margins, second)
    c = m.new_cache(128)
    tok0 = int(np.argmax(m.forward_seq(prompt, c)))
    tr = m.trace_fused(tok0, c)  # the fused kernel ran for this shape
    assert tr.shape[1] == 5 * 2 + 1
    groups = tr[:, :, 7].astype(np.int64).sum(axis=0)
    # QKV 6144 rows / 4, O 4096 / 4, GU 14336 / 2, DOWN 4096 / 1
    assert list(groups[:5]) == [6144 // 4, 0, 4096 // 4, 14336 // 2, 4096]
    c.close()
    m.close()
