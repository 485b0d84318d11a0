"""TMG_DEBUG: the per-token forward prints the reference's debug lines
(src/model.rs:406-409, 468-470, 480-482): the first 8 values of the
embedding, then per layer of the residual stream after attention and after
the MLP.  A child process with TMG_DEBUG=1 runs one forward_token of the C1
shape on the GPU and the same token through the CPU oracle (which prints
the same lines); the labels must match line for line, the embedding values
exactly (BF16 widened) and the rest within 1e-4 relative / 1e-5 absolute.
"""
import os
import re
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover - CPU box
    pytest.skip("needs a GPU", allow_module_level=True)

ROOT = Path(__file__).resolve().parents[1]

CHILD = r'''
import sys
sys.path.insert(0, {root!r})
from tinyminigo_b200 import synth
from tinyminigo_b200.model import Model, ModelConfig
from oracle import oracle as orc
orc.build()
cfg = synth.CONFIGS["c1"]
w = synth.make_weights(cfg, 91)
mc = ModelConfig(cfg["hidden_size"], cfg["num_hidden_layers"], cfg["num_attention_heads"],
                 cfg["num_key_value_heads"], cfg["head_dim"], cfg["intermediate_size"],
                 cfg["rms_norm_eps"], cfg["rope_theta"], cfg["vocab_size"], [], 0)
m = Model.from_tensors(mc, w)
cache = m.new_cache(16)
print("=== gpu", file=sys.stderr, flush=True)
m.forward_token(1234, cache)
print("=== oracle", file=sys.stderr, flush=True)
om = orc.OracleModel(cfg, w)
om.reset()
om.forward_token(1234)
print("=== end", file=sys.stderr, flush=True)
cache.close()
m.close()
'''

LINE = re.compile(r"^(embed|L\d+ attn_out|L\d+ out) first8: \[(.*)\]$")


def parse(block):
    out = []
    for ln in block:
        mt = LINE.match(ln.strip())
        if mt:
            out.append((mt.group(1), [float(v) for v in mt.group(2).split(",")]))
    return out


def test_debug_lines_match_the_oracle():
    code = CHILD.format(root=str(ROOT))
    env = dict(os.environ, TMG_DEBUG="1")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    err = r.stderr.splitlines()
    gi, oi, ei = err.index("=== gpu"), err.index("=== oracle"), err.index("=== end")
    gpu, ref = parse(err[gi + 1:oi]), parse(err[oi + 1:ei])
    layers = 2
    assert [k for k, _ in ref] == ["embed"] + [f"L{i} {w}" for i in range(layers)
                                               for w in ("attn_out", "out")]
    assert [k for k, _ in gpu] == [k for k, _ in ref]
    for (k, g), (_, o) in zip(gpu, ref):
        assert len(g) == len(o) == 8
        for a, b in zip(g, o):
            if k == "embed":
                assert a == b
            else:
                assert abs(a - b) <= 1e-5 + 1e-4 * abs(b), (k, g, o)
