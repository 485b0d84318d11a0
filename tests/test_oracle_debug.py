"""The oracle's TMG_DEBUG lines (src/model.rs:406-409, 468-470, 480-482),
on the host: one forward_token of the C1 shape in a child process with
TMG_DEBUG set prints `embed first8: [...]`, then per layer `L<i> attn_out
first8: [...]` and `L<i> out first8: [...]`, the embedding values being the
token's BF16 embedding row widened exactly; without TMG_DEBUG nothing is
printed.  (tests/test_gpu_debug.py compares the GPU's lines with these.)"""
import os
import re
import subprocess
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]

CHILD = r'''
import sys
sys.path.insert(0, {root!r})
from tinyminigo_b200 import synth
from oracle import oracle as orc
orc.build()
cfg = synth.CONFIGS["c1"]
w = synth.make_weights(cfg, 91)
om = orc.OracleModel(cfg, w)
om.reset()
om.forward_token(1234)
'''

LINE = re.compile(r"^(embed|L\d+ attn_out|L\d+ out) first8: \[(.*)\]$")


def run(debug):
    env = dict(os.environ)
    env.pop("TMG_DEBUG", None)
    if debug:
        env["TMG_DEBUG"] = "1"
    r = subprocess.run([sys.executable, "-c", CHILD.format(root=str(ROOT))], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    return [ln for ln in r.stderr.splitlines() if LINE.match(ln.strip())]


def test_oracle_prints_the_reference_debug_lines():
    from tinyminigo_b200 import synth

    lines = run(True)
    labels = [LINE.match(ln).group(1) for ln in lines]
    assert labels == ["embed", "L0 attn_out", "L0 out", "L1 attn_out", "L1 out"]
    cfg = synth.CONFIGS["c1"]
    emb = synth.bf16_to_f32(synth.make_weights(cfg, 91)["model.embed_tokens.weight"])
    emb = emb.reshape(cfg["vocab_size"], cfg["hidden_size"])[1234, :8]
    got = np.array([float(v) for v in LINE.match(lines[0]).group(2).split(",")], np.float32)
    assert np.array_equal(got, emb)
    assert run(False) == []
