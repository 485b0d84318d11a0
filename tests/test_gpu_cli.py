"""The command line end to end on the GPU (src/main.rs): a C1 checkpoint
with a word-level tokenizer ("t<id>" for every id) and a template that
passes the prompt through; the streamed text is the tokens generate()
returns, and the --dump-first-logits file holds its first-step logits."""
import json
import re

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover - CPU box
    pytest.skip("needs a GPU", allow_module_level=True)

from tinyminigo_b200 import cli, synth  # noqa: E402
from tinyminigo_b200.model import GenParams, Model, generate  # noqa: E402


def word_tokenizer(path, vocab):
    from tokenizers import Tokenizer, models, pre_tokenizers, decoders

    t = Tokenizer(models.WordLevel({f"t{i}": i for i in range(vocab)}, unk_token="t0"))
    t.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    t.decoder = decoders.WordPiece(prefix="##")  # joins tokens with spaces
    t.save(str(path))


@pytest.mark.parametrize("sampled", [False, True])
def test_cli_generates_like_the_api(tmp_path, capsys, sampled):
    cfg = synth.CONFIGS["c1"]
    w = synth.make_weights(cfg, 11)
    model_path = synth.write_model(tmp_path, cfg, w)
    word_tokenizer(tmp_path / "tokenizer.json", cfg["vocab_size"])
    (tmp_path / "t.jinja").write_text("{{ messages[0].content }}")
    prompt = [5, 17, 300, 31999, 4, 4, 123]
    flags = ["--temperature", "0.8", "--top-k", "40", "--top-p", "0.9", "--seed", "7"] if sampled else []
    rc = cli.main(["-m", str(model_path), "--template", str(tmp_path / "t.jinja"),
                   "--max-tokens", "12", "--dump-first-logits", str(tmp_path / "d.json"), *flags,
                   " ".join(f"t{i}" for i in prompt)])
    out = capsys.readouterr()
    assert rc == 0, out.err
    assert f"prompt tokens: {len(prompt)} {prompt}" in out.err
    m = Model.load(model_path)
    p = GenParams(max_tokens=12, temperature=0.8, top_k=40, top_p=0.9, seed=7) if sampled \
        else GenParams(max_tokens=12)
    res = generate(m, prompt, p)
    m.close()
    # each token is decoded alone and printed as it comes (no separator)
    got = [int(v) for v in re.findall(r"t(\d+)", out.out)]
    assert got == res.tokens
    d = json.loads((tmp_path / "d.json").read_text())
    assert d["top5_ids"] == [int(i) for i in np.argsort(-res.logits_first_step, kind="stable")[:5]]
    assert np.allclose(d["first8"], res.logits_first_step[:8], rtol=1e-6, atol=1e-6)
