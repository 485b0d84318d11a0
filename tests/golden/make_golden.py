"""Generate the golden fixtures that pin the CPU oracle at model level.

The reference validates its engine against HF transformers'
LlamaForCausalLM run in f32 (scripts/hf_reference.py, tests/numerical.rs:
top-5 ids and first logits of the first step, then a greedy sequence).  The
checkpoint those goldens use is not available here, so this script replays
the same method on seeded synthetic weights (tinyminigo_b200.synth) and saves
HF's outputs as small JSON fixtures.  tests/test_oracle_golden.py checks the
oracle against them.

Run from the repo root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from tinyminigo_b200 import synth  # noqa: E402

# (fixture name, base config, layers override, weight seed, prompt seed, prompt len, greedy steps)
CASES = [
    ("c1", "c1", None, 1234, 99, 16, 40),
    ("c2_l2", "c2", 2, 4321, 7, 16, 12),
]


def hf_model(cfg: dict, tensors: dict):
    from transformers import LlamaConfig, LlamaForCausalLM

    hc = LlamaConfig(
        vocab_size=cfg["vocab_size"], hidden_size=cfg["hidden_size"],
        intermediate_size=cfg["intermediate_size"], num_hidden_layers=cfg["num_hidden_layers"],
        num_attention_heads=cfg["num_attention_heads"],
        num_key_value_heads=cfg["num_key_value_heads"], head_dim=cfg["head_dim"],
        rms_norm_eps=cfg["rms_norm_eps"], max_position_embeddings=4096,
        rope_parameters={"rope_type": "default", "rope_theta": cfg["rope_theta"]},
        tie_word_embeddings=cfg["tie_word_embeddings"], attention_bias=False, mlp_bias=False,
        hidden_act="silu", bos_token_id=0, eos_token_id=None, pad_token_id=None,
    )
    hc._attn_implementation = "eager"
    m = LlamaForCausalLM(hc).to(torch.float32).eval()
    sd = {k: torch.from_numpy(synth.bf16_to_f32(v).reshape(v.shape).copy()) for k, v in tensors.items()}
    if cfg["tie_word_embeddings"]:
        sd["lm_head.weight"] = sd["model.embed_tokens.weight"]
    missing, unexpected = m.load_state_dict(sd, strict=False)
    assert not unexpected, unexpected
    assert all("rotary" in k for k in missing), missing
    return m


def run_case(name, base, layers, wseed, pseed, plen, steps):
    cfg = synth.CONFIGS[base] if layers is None else synth.with_layers(synth.CONFIGS[base], layers)
    tensors = synth.make_weights(cfg, wseed)
    prompt = synth.random_prompt(cfg["vocab_size"], plen, pseed)
    m = hf_model(cfg, tensors)
    ids = torch.tensor(prompt.astype(np.int64))[None]
    with torch.no_grad():
        logits = m(ids).logits[0, -1].float().numpy()
        gen = m.generate(ids, max_new_tokens=steps, do_sample=False, min_new_tokens=steps,
                         pad_token_id=0)
    greedy = gen[0, plen:].tolist()
    top5 = np.argsort(-logits, kind="stable")[:5]
    return {
        "name": name, "config": base, "layers": cfg["num_hidden_layers"], "weight_seed": wseed,
        "prompt_seed": pseed, "prompt": prompt.tolist(),
        "first_logits_head": [float(v) for v in logits[:16]],
        "top5_ids": [int(i) for i in top5], "top5_vals": [float(logits[i]) for i in top5],
        "logits_sum": float(logits.astype(np.float64).sum()),
        "logits_sumsq": float((logits.astype(np.float64) ** 2).sum()),
        "greedy": greedy,
        "source": "HF transformers LlamaForCausalLM, f32, eager attention",
        "transformers": __import__("transformers").__version__,
    }


def main():
    out = Path(__file__).resolve().parent
    for case in CASES:
        d = run_case(*case)
        (out / f"hf_{d['name']}.json").write_text(json.dumps(d, indent=1))
        print(d["name"], d["top5_ids"], d["greedy"][:8])


if __name__ == "__main__":
    main()
