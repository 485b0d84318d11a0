"""The reference engine's command line (src/cli.rs, src/main.rs) over the B200
library: the same flags and defaults, the same flow.

    python -m tinyminigo_b200 -m dir/model.safetensors --template chat.jinja \\
        [--tokenizer tokenizer.json] [--max-tokens 256] [--temperature 0] \\
        [--top-k 0] [--top-p 1] [--repetition-penalty 1] [--seed 42] \\
        [--dump-first-logits out.json] [--repack out.tmb] "prompt"

`--repack` writes a TMB1 file and exits (src/main.rs:29-35); otherwise the
model goes to HBM (a TMB1 file or safetensors + config.json), the prompt is
rendered through the chat template (src/template.rs:6-29, jinja2 in place of
minijinja + its Python-method compatibility), encoded with the HF tokenizer
(src/tokenizer.rs, the `tokenizers` package in place of the crate), and
generate() streams each new token's text to stdout.  Host-side text work
only: every forward runs in the CUDA library.  TMG_THREADS (the reference's
CPU thread count) has nothing to set here and is ignored.
"""
from __future__ import annotations

import argparse
import json
import sys
import time
from pathlib import Path

import numpy as np


def parse_args(argv=None) -> argparse.Namespace:
    """Args, src/cli.rs:5-54 (clap): the same names, value names and defaults."""
    ap = argparse.ArgumentParser(
        prog="tinyminigo",
        description="tinyminigo — a minimal inference engine for MiniCPM5 (Llama-style "
                    "decoder), on the B200 library")
    ap.add_argument("-m", "--model", metavar="FILE", required=True,
                    help="Path to the model weights (safetensors file)")
    ap.add_argument("--template", metavar="FILE", required=True,
                    help="Path to the Jinja chat template file")
    ap.add_argument("--tokenizer", metavar="FILE", default=None,
                    help="Path to the tokenizer (defaults to tokenizer.json next to the model)")
    ap.add_argument("--max-tokens", metavar="N", type=int, default=256,
                    help="Maximum number of new tokens to generate")
    ap.add_argument("--temperature", metavar="T", type=float, default=0.0,
                    help="Sampling temperature (0 = greedy)")
    ap.add_argument("--top-k", metavar="K", type=int, default=0,
                    help="Top-k sampling (0 = disabled)")
    ap.add_argument("--top-p", metavar="P", type=float, default=1.0,
                    help="Top-p (nucleus) sampling threshold (1.0 = disabled)")
    ap.add_argument("--repetition-penalty", metavar="R", type=float, default=1.0,
                    help="Repetition penalty (1.0 = disabled)")
    ap.add_argument("--seed", metavar="SEED", type=int, default=42,
                    help="Random seed for sampling")
    ap.add_argument("prompt", help="The user prompt")
    ap.add_argument("--dump-first-logits", metavar="FILE", default=None,
                    help=argparse.SUPPRESS)
    ap.add_argument("--repack", metavar="FILE", default=None, help=argparse.SUPPRESS)
    a = ap.parse_args(argv)
    if a.max_tokens < 0 or a.top_k < 0 or a.seed < 0:
        ap.error("--max-tokens, --top-k and --seed take non-negative integers (usize/u64)")
    return a


def resolve_tokenizer_path(explicit, model_path) -> Path:
    """resolve_tokenizer_path, src/tokenizer.rs:44-53."""
    if explicit is not None:
        return Path(explicit)
    return Path(model_path).parent / "tokenizer.json"


def render_chat_template(template_path, user_prompt: str, bos_token: str) -> str:
    """render_chat_template, src/template.rs:6-29: one user message, the
    generation prompt on, the reference's bos/eos/pad strings."""
    import jinja2

    try:
        src = Path(template_path).read_text()
    except OSError as e:
        raise RuntimeError(f"reading chat template {template_path}: {e}") from e
    env = jinja2.Environment(keep_trailing_newline=True)
    try:
        tmpl = env.from_string(src)
    except jinja2.TemplateError as e:
        raise RuntimeError(f"parsing chat template {template_path}: {e}") from e
    return tmpl.render(messages=[{"role": "user", "content": user_prompt}],
                       add_generation_prompt=True, bos_token=bos_token, eos_token="</s>",
                       pad_token="</s>")


def first_logits_dump(logits: np.ndarray) -> str:
    """The --dump-first-logits file, src/main.rs:107-123: the 5 largest logits
    (a stable sort by value, descending: ties keep the lower id first), their
    values and the first 8 logits, as pretty JSON with serde_json's key order."""
    lg = np.asarray(logits, np.float32)
    top = np.argsort(-lg, kind="stable")[:5]
    f32 = lambda v: float(str(np.float32(v)))  # noqa: E731  (shortest f32 decimal, as serde_json)
    dump = {"top5_ids": [int(i) for i in top], "top5_vals": [f32(lg[i]) for i in top],
            "first8": [f32(v) for v in lg[:8]]}
    return json.dumps(dump, indent=2, sort_keys=True)


def main(argv=None) -> int:
    try:
        return _run(parse_args(argv))
    except Exception as e:  # noqa: BLE001  (main.rs prints `error: {e:#}` and exits 1)
        print(f"error: {e}", file=sys.stderr)
        return 1


def _run(args) -> int:
    from . import tmb

    model_path = Path(args.model)
    if args.repack is not None:
        if not (model_path.parent / "config.json").exists():
            raise RuntimeError(f"config.json not found next to {model_path}")
        tmb.repack(model_path, args.repack)
        return 0
    if not model_path.exists():
        raise RuntimeError(f"model file not found: {model_path}")

    from .model import GenParams, Model, generate

    print(f"loading model {model_path} ...", file=sys.stderr)
    t0 = time.perf_counter()
    m = Model.load(model_path)
    c = m.config
    print(f"loaded in {time.perf_counter() - t0:.2f}s: layers={c.num_hidden_layers} "
          f"hidden={c.hidden_size} heads={c.num_attention_heads} kv_heads={c.num_key_value_heads} "
          f"head_dim={c.head_dim} vocab={c.vocab_size}", file=sys.stderr)

    tok_path = resolve_tokenizer_path(args.tokenizer, model_path)
    if not tok_path.exists():
        raise RuntimeError(f"tokenizer not found at {tok_path} (pass --tokenizer to specify)")
    from tokenizers import Tokenizer

    tok = Tokenizer.from_file(str(tok_path))
    rendered = render_chat_template(args.template, args.prompt, "<s>")
    print(f"--- rendered prompt ---\n{rendered}\n-----------------------", file=sys.stderr)
    ids = tok.encode(rendered, add_special_tokens=False).ids
    print(f"prompt tokens: {len(ids)} {ids}", file=sys.stderr)

    params = GenParams(max_tokens=args.max_tokens, temperature=args.temperature,
                       top_k=args.top_k, top_p=args.top_p,
                       repetition_penalty=args.repetition_penalty, seed=args.seed)

    def on_token(t: int):
        sys.stdout.write(tok.decode([t], skip_special_tokens=True))
        sys.stdout.flush()

    t_start = time.perf_counter()
    res = generate(m, ids, params, on_token=on_token)
    if args.dump_first_logits is not None:
        Path(args.dump_first_logits).write_text(first_logits_dump(res.logits_first_step))
    print()
    elapsed = time.perf_counter() - t_start
    n_gen = len(res.tokens)
    dec = max(n_gen - 1, 0)  # the last generated step belongs to prefill + 1 forward
    pf = max(res.prefill_secs, 1e-9)
    print(f"\n[{n_gen} tokens generated in {elapsed:.2f}s | prefill: {len(ids)} tok in "
          f"{res.prefill_secs:.2f}s ({len(ids) / pf:.1f} tok/s) | decode: ~{dec} tok in "
          f"{elapsed - res.prefill_secs:.2f}s ({dec / max(elapsed - res.prefill_secs, 1e-9):.2f} "
          f"tok/s)]", file=sys.stderr)
    m.close()
    return 0
