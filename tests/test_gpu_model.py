"""Model-level parity of the CUDA token loop (through the C ABI) with the
CPU oracle, on the benchmark configurations' shapes.

The bar (north star): greedy token sequences identical to the reference's;
logits within 1e-3 relative / 1e-2 absolute, i.e. |a - b| <= 1e-2 + 1e-3 |b|.
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
from tinyminigo_b200.model import GenParams, Model, ModelConfig, generate, generate_batch  # noqa: E402

GOLD = Path(__file__).resolve().parent / "golden"


def close(a, b):
    return np.all(np.abs(a - b) <= 1e-2 + 1e-3 * np.abs(b))


def margin(logits):
    s = np.sort(logits)
    return float(s[-1] - s[-2])


def cfg_obj(cfg, eos=()):
    return ModelConfig(cfg["hidden_size"], cfg["num_hidden_layers"], cfg["num_attention_heads"],
                       cfg["num_key_value_heads"], cfg["head_dim"], cfg["intermediate_size"],
                       cfg["rms_norm_eps"], cfg["rope_theta"], cfg["vocab_size"], list(eos), 0)


@pytest.fixture(scope="module")
def c1():
    d = json.loads((GOLD / "hf_c1.json").read_text())
    cfg = synth.CONFIGS["c1"]
    t = synth.make_weights(cfg, d["weight_seed"])
    return d, cfg, t


@pytest.fixture(scope="module")
def c2():
    cfg = synth.CONFIGS["c2"]
    t = synth.make_weights(cfg, 2024, device="cuda")
    return cfg, t


def test_c1_generate_matches_oracle_and_hf(orc, c1):
    d, cfg, t = c1
    om = orc.OracleModel(cfg, t)
    ref_toks, ref_first, _, _ = om.generate(d["prompt"], 40)
    assert ref_toks.tolist() == d["greedy"]
    m = Model.from_tensors(cfg_obj(cfg), t)
    out = generate(m, d["prompt"], GenParams(max_tokens=40))
    assert out.tokens == d["greedy"]
    assert close(out.logits_first_step, ref_first)
    assert np.max(np.abs(out.logits_first_step - ref_first)) < 1e-4


def test_c1_load_from_file_and_stepwise_logits(orc, c1, tmp_path):
    d, cfg, t = c1
    path = synth.write_model(tmp_path, cfg, t)
    m = Model.load(path)
    assert m.config.vocab_size == 32000 and m.config.head_dim == 16
    om = orc.OracleModel(cfg, t)
    cache = m.new_cache(128)
    a = m.prefill(d["prompt"][:9], cache)
    b = om.forward_seq(d["prompt"][:9])
    assert close(a, b)
    for tok in d["prompt"][9:] + d["greedy"][:6]:
        a = m.forward_token(tok, cache)
        b = om.forward_token(tok)
        assert close(a, b) and np.max(np.abs(a - b)) < 1e-4
    assert cache.len(0) == om.kv_len(0) == 16 + 6
    for layer in range(cfg["num_hidden_layers"]):
        kr, vr = om.kv_read(layer)
        assert np.allclose(cache.keys_flat(layer), kr, atol=1e-5, rtol=1e-5)
        assert np.allclose(cache.values_flat(layer), vr, atol=1e-5, rtol=1e-5)
    cache.reset()
    assert cache.len(0) == 0


@pytest.mark.parametrize("tied", [False, True])
def test_c1_load_from_tmb_repack(orc, c1, tmp_path, tied):
    # load_model_tmb (src/model.rs:108-179): the repacked file gives the same
    # greedy ids and first-step logits as the tensors it was written from
    from tinyminigo_b200 import tmb

    d, cfg, t = c1
    if tied:
        t = {k: v for k, v in t.items() if k != "lm_head.weight"}
        cfg = dict(cfg, tie_word_embeddings=True)
    p = tmp_path / "m.tmb"
    tmb.write(p, dict(cfg, eos_token_ids=[d["greedy"][3]]), t)
    m = Model.load(p)
    assert m.config.eos_token_ids == []  # the repack's EOS key is not read back
    ref = Model.from_tensors(cfg_obj(cfg), t)
    a = generate(m, d["prompt"], GenParams(max_tokens=20))
    b = generate(ref, d["prompt"], GenParams(max_tokens=20))
    assert a.tokens == b.tokens
    assert np.max(np.abs(a.logits_first_step - b.logits_first_step)) <= 1e-6
    if not tied:
        assert a.tokens == d["greedy"][:20]
    m.close()
    ref.close()


def test_tmb_load_refusals(c1, tmp_path):
    import ctypes

    from tinyminigo_b200 import tmb
    from tinyminigo_b200._lib import TmgError, check, lib

    d, cfg, t = c1
    # an f32 embedding that is not a widened BF16 cannot go to the BF16 table
    t2 = dict(t)
    t2["model.embed_tokens.weight"] = synth.bf16_to_f32(t["model.embed_tokens.weight"]) * np.float32(1.0001)
    p = tmp_path / "f32.tmb"
    tmb.write(p, cfg, t2)
    with pytest.raises(TmgError, match="not a BF16 value"):
        Model.load(p)
    # the file's shape must be the context's
    q = tmp_path / "ok.tmb"
    tmb.write(q, cfg, t)
    other = Model(cfg_obj(dict(cfg, intermediate_size=256)))
    with pytest.raises(TmgError, match="does not match"):
        check(lib().tmg_load_tmb(other._h, str(q).encode()), other._h, "load")
    other.close()


def test_c1_eos_stops_like_reference(orc, c1):
    d, cfg, t = c1
    eos = d["greedy"][5]
    om = orc.OracleModel(cfg, t)
    ref, _, _, _ = om.generate(d["prompt"], 40, eos=[eos])
    m = Model.from_tensors(cfg_obj(cfg, [eos]), t)
    seen = []
    out = generate(m, d["prompt"], GenParams(max_tokens=40), on_token=seen.append)
    assert out.tokens == ref.tolist() == d["greedy"][:6]
    assert seen == out.tokens
    assert m._gen_cache.len(0) == om.kv_len(0) == 16 + 5


def test_c1_sampled_matches_oracle(orc, c1):
    d, cfg, t = c1
    om = orc.OracleModel(cfg, t)
    m = Model.from_tensors(cfg_obj(cfg), t)
    p = GenParams(max_tokens=30, temperature=0.8, top_k=40, top_p=0.95, repetition_penalty=1.1,
                  seed=7)
    u = orc.stdrng_uniforms(7, 30)
    ref, _, _, _ = om.generate(d["prompt"], 30, 0.8, 40, 0.95, 1.1, 7, uniforms=u)
    out = generate(m, d["prompt"], p)  # uniforms from the library's StdRng restatement
    assert out.tokens == ref.tolist()


def test_c1_greedy_with_penalty(orc, c1):
    d, cfg, t = c1
    om = orc.OracleModel(cfg, t)
    m = Model.from_tensors(cfg_obj(cfg), t)
    ref, _, _, _ = om.generate(d["prompt"], 20, 0.0, 0, 1.0, 1.3)
    out = generate(m, d["prompt"], GenParams(max_tokens=20, repetition_penalty=1.3))
    assert out.tokens == ref.tolist()


def test_c2_generate_256_full_depth(orc, greedy, c2):
    # BASELINE config C2 as stated: the 1B shape at full depth (16 layers,
    # tied head), a 64-token random prompt, then 256 greedy steps through
    # generate (every step inside the fused decode kernel), against the
    # oracle's generate loop (src/model.rs:614-663)
    cfg, t = c2
    prompt = synth.random_prompt(cfg["vocab_size"], 64, 11)
    om = orc.OracleModel(cfg, t)
    steps = 256
    ids, margins, second, ref_first = greedy.oracle(om, prompt, steps)
    m = Model.from_tensors(cfg_obj(cfg), t)
    out = generate(m, prompt, GenParams(max_tokens=steps))
    assert close(out.logits_first_step, ref_first), np.max(np.abs(out.logits_first_step - ref_first))
    greedy.agree("C2 1B, 16 layers, 64-token prompt, 256 steps (fused)", out.tokens, ids, margins,
                 second)
    m.close()


def test_c4_8b_shape_on_one_gpu(orc, greedy):
    # BASELINE config C4's model (hidden 4096, 32 layers, 32 q / 8 kv heads of
    # 128, intermediate 14336, vocab 128256, untied) on one GPU: a 128-token
    # random prompt, first-step logits within 1e-3 rel / 1e-2 abs of the
    # oracle's, then 16 greedy steps
    cfg = synth.CONFIGS["c4"]
    t = synth.make_weights(cfg, 4048, device="cuda")
    prompt = synth.random_prompt(cfg["vocab_size"], 128, 17)
    steps = 16
    om = orc.OracleModel(cfg, t)
    ids, margins, second, ref_first = greedy.oracle(om, prompt, steps)
    m = Model.from_tensors(cfg_obj(cfg), t)
    out = generate(m, prompt, GenParams(max_tokens=steps))
    assert close(out.logits_first_step, ref_first), np.max(np.abs(out.logits_first_step - ref_first))
    greedy.agree("C4 8B shape, 1 GPU, 128-token prompt, 16 steps", out.tokens, ids, margins, second)
    m.close()
    del om


def test_c2_batched_streams_match_single(orc, c2):
    cfg, t = c2
    m = Model.from_tensors(cfg_obj(cfg), t)
    prompts = np.stack([synth.random_prompt(cfg["vocab_size"], 16, s) for s in range(4)])
    outs = generate_batch(m, prompts, [GenParams(max_tokens=8)] * 4)
    for s in range(4):
        single = generate(m, prompts[s], GenParams(max_tokens=8))
        assert outs[s] == single.tokens
    m.close()


def test_capacity_and_bad_tokens_are_errors(c1):
    d, cfg, t = c1
    m = Model.from_tensors(cfg_obj(cfg), t)
    cache = m.new_cache(4)
    with pytest.raises(Exception, match="capacity"):
        m.prefill(list(range(5)), cache)
    with pytest.raises(Exception, match="out of range"):
        m.forward_token(10**6, cache)
    with pytest.raises(ValueError):
        m.prefill([], cache)
    with pytest.raises(Exception, match="top_k"):
        generate(m, d["prompt"], GenParams(max_tokens=3, temperature=0.7, top_k=0))


def test_batched_long_prompts_match_single_streams(c2):
    # 16 streams with 2048-token prompts: the batched decode attention splits
    # each context into multi-tile ranges, and the position being decoded
    # can sit in any tile of the last range; every stream must match its
    # own single-stream run (which decodes through a different kernel)
    cfg, t = c2
    cfg2 = synth.with_layers(cfg, 2)
    t2 = {k: v for k, v in t.items() if not k.startswith("model.layers.")
          or int(k.split(".")[2]) < 2}
    m = Model.from_tensors(cfg_obj(cfg2), t2)
    M, T, steps = 16, 2048, 12
    prompts = np.stack([synth.random_prompt(cfg["vocab_size"], T, 50 + s) for s in range(M)])
    outs = generate_batch(m, prompts, [GenParams(max_tokens=steps)] * M)
    for s in range(M):
        single = generate(m, prompts[s], GenParams(max_tokens=steps))
        assert outs[s] == single.tokens, f"stream {s}"
    m.close()


def test_bench_c5_host_leg_on_a_small_case():
    # bench.py's C5 host leg (oracle decode from the GPU-prefilled KV cache,
    # logits compared per step) on 3 streams of a 2-layer c2 shape
    import bench

    cfg = synth.with_layers(synth.CONFIGS["c2"], 2)
    w = synth.make_weights(cfg, 5)
    m = Model.from_tensors(cfg_obj(cfg), w)
    M, T = 3, 300
    prompts = [synth.random_prompt(cfg["vocab_size"], T, 40 + i) for i in range(M)]
    cache = m.new_cache(T + 16, n_streams=M)
    for i in range(M):
        m.forward_seq(prompts[i], cache, stream=i, want_logits=False)
    res = bench.c5_cpu_leg(m, cache, cfg, w, T, [int(p[-1]) for p in prompts], n_steps=4)
    assert res["parity"]["logits_within_1e-3_rel_1e-2_abs"], res["parity"]
    assert res["cpu_baseline"]["value"] > 0 and res["cpu_baseline"]["kind"] == "port"
    assert cache.len(0, 0) == T + 4
    cache.close()
    m.close()


def test_cache_destroyed_after_its_context(c1):
    # a KV cache and a WMat handle that outlive their context (garbage
    # collection can order the destructors either way) are released with
    # the context; their own destroy calls afterwards are safe
    import ctypes

    from tinyminigo_b200._lib import check, lib

    d, cfg, t = c1
    m = Model.from_tensors(cfg_obj(cfg), t)
    cache = m.new_cache(64)
    w = np.zeros((16, 16), np.uint16)
    wm = ctypes.c_void_p()
    check(lib().tmg_wmat_upload_bf16(m._h, w.ctypes.data_as(ctypes.c_void_p), 16, 16,
                                     ctypes.byref(wm)), m._h)
    check(lib().tmg_destroy(m._h))
    m._h = None
    m._caches = []
    assert lib().tmg_kv_destroy(cache._h) == 0
    cache._h = None
    assert lib().tmg_wmat_free(wm) == 0
