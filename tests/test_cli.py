"""The reference's command line (src/cli.rs, src/main.rs) and its host-side
helpers (src/template.rs, src/tokenizer.rs), without a GPU: flags and
defaults, the template and tokenizer-path known answers of the reference's
own tests, the --dump-first-logits format, --repack, and the errors."""
import json

import numpy as np
import pytest

from tinyminigo_b200 import cli, synth, tmb


def test_flags_and_defaults():  # src/cli.rs:5-54
    a = cli.parse_args(["-m", "m.safetensors", "--template", "t.jinja", "hello"])
    assert (a.model, a.template, a.tokenizer, a.prompt) == ("m.safetensors", "t.jinja", None, "hello")
    assert (a.max_tokens, a.temperature, a.top_k, a.top_p, a.repetition_penalty, a.seed) == \
        (256, 0.0, 0, 1.0, 1.0, 42)
    assert a.dump_first_logits is None and a.repack is None
    b = cli.parse_args(["--model", "x", "--template", "t", "--tokenizer", "tk.json",
                        "--max-tokens", "7", "--temperature", "0.8", "--top-k", "40",
                        "--top-p", "0.95", "--repetition-penalty", "1.1", "--seed", "9",
                        "--dump-first-logits", "d.json", "--repack", "o.tmb", "p"])
    assert (b.tokenizer, b.max_tokens, b.temperature, b.top_k, b.top_p, b.repetition_penalty,
            b.seed, b.dump_first_logits, b.repack) == \
        ("tk.json", 7, 0.8, 40, 0.95, 1.1, 9, "d.json", "o.tmb")
    with pytest.raises(SystemExit):
        cli.parse_args(["--template", "t", "p"])  # --model is required
    with pytest.raises(SystemExit):
        cli.parse_args(["-m", "x", "--template", "t", "--max-tokens", "-1", "p"])


def test_resolve_tokenizer_path():  # src/tokenizer.rs:44-64
    assert str(cli.resolve_tokenizer_path("/x/t.json", "/y/m.safetensors")) == "/x/t.json"
    assert str(cli.resolve_tokenizer_path(None, "/y/m.safetensors")) == "/y/tokenizer.json"


def test_render_chat_template_known_answer(tmp_path):  # src/template.rs:31-43
    p = tmp_path / "t.jinja"
    p.write_text("{{ bos_token }}{% for m in messages %}<|im_start|>{{ m.role }}\n{{ m.content }}"
                 "<|im_end|>\n{% endfor %}{% if add_generation_prompt %}<|im_start|>assistant\n"
                 "{% endif %}")
    out = cli.render_chat_template(p, "Hi", "<s>")
    assert out == "<s><|im_start|>user\nHi<|im_end|>\n<|im_start|>assistant\n"


def test_template_python_string_methods(tmp_path):
    # HF templates call Python string methods (minijinja-contrib pycompat there)
    p = tmp_path / "t.jinja"
    p.write_text("{% for m in messages %}{{ m.content.strip().upper() }}"
                 "{% if m.role.startswith('us') %}|u{% endif %}{% endfor %}{{ eos_token }}")
    assert cli.render_chat_template(p, "  hey ", "<s>") == "HEY|u</s>"
    with pytest.raises(RuntimeError, match="reading chat template"):
        cli.render_chat_template(tmp_path / "missing.jinja", "x", "<s>")


def test_first_logits_dump_format():  # src/main.rs:107-123
    lg = np.array([0.5, 2.0, -1.0, 2.0, 0.1, 3.25, 0.5, 1.0, 7.0], np.float32)
    d = json.loads(cli.first_logits_dump(lg))
    assert list(d) == ["first8", "top5_ids", "top5_vals"]
    assert d["top5_ids"] == [8, 5, 1, 3, 7]  # a tie keeps the lower id first (stable sort)
    assert d["top5_vals"] == [7.0, 3.25, 2.0, 2.0, 1.0]
    assert np.array_equal(np.float32(d["first8"]), lg[:8])
    assert json.loads(cli.first_logits_dump(np.float32([0.1] * 8)))["first8"][0] == 0.1


def test_repack_flag(tmp_path):  # src/main.rs:29-35
    cfg = synth.CONFIGS["c1"]
    src = synth.write_model(tmp_path / "m", cfg, synth.make_weights(cfg, 3))
    out = tmp_path / "m.tmb"
    assert cli.main(["-m", str(src), "--template", "unused", "--repack", str(out), "x"]) == 0
    ref = tmp_path / "ref.tmb"
    tmb.repack(src, ref)
    assert out.read_bytes() == ref.read_bytes()


def test_errors_exit_1(tmp_path, capsys):
    assert cli.main(["-m", str(tmp_path / "nope.safetensors"), "--template", "t", "x"]) == 1
    assert "error: model file not found" in capsys.readouterr().err
    assert cli.main(["-m", str(tmp_path / "nope.safetensors"), "--template", "t",
                     "--repack", str(tmp_path / "o.tmb"), "x"]) == 1
    assert "config.json not found" in capsys.readouterr().err
