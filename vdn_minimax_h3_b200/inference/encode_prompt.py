"""Encode t2va prompts into prompt caches (reference src/inference/encode_prompt.py).

    python -m vdn_minimax_h3_b200.inference.encode_prompt --prompt "..." --out prompts/p.pt
    python -m vdn_minimax_h3_b200.inference.encode_prompt --jsonl prompts.jsonl --take 4 \
        --out_dir prompts --name prompt [--rows 0 7 9]

The prompt is encoded verbatim (no chat template, no special tokens); every row is tagged
TEXT. With --model_root (a MiniMax-H3 snapshot holding processor/ and text_encoder/) the
Qwen3-VL conditioner runs; without it the weight-free stand-in writes caches of the same
format (offline runs, tests). Batch mode loads the conditioner once for all rows; output
names keep the jsonl row index (<name>_<row>.pt).
"""
import argparse
import json
import os
import sys

from vdn_minimax_h3_b200.inference.encoders import TEXT_TAG, make_conditioner
from vdn_minimax_h3_b200.inference.prompt_cache import save_prompt


def encode_one(cond, prompt, out):
    ids = cond.tokenize(prompt)
    emb = cond.encode(ids)
    save_prompt(out, prompt, emb, [TEXT_TAG] * len(ids))
    print(f"wrote {out}: {len(ids)} tokens, embeds {tuple(emb.shape)}", flush=True)
    return out


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--prompt", type=str)
    p.add_argument("--out", type=str)
    p.add_argument("--jsonl", type=str, help="one JSON object per line with a 'prompt' field")
    p.add_argument("--take", type=int, default=4, help="jsonl: encode the first N rows")
    p.add_argument("--rows", type=int, nargs="*", default=None,
                   help="jsonl: encode exactly these row indices (names keep the index)")
    p.add_argument("--out_dir", type=str, default="prompts")
    p.add_argument("--name", type=str, default="prompt")
    p.add_argument("--model_root", type=str, default=None,
                   help="MiniMax-H3 snapshot with processor/ and text_encoder/; "
                        "default: the weight-free stand-in conditioner")
    p.add_argument("--device", type=str, default="cuda:0")
    p.add_argument("--seed", type=int, default=0, help="stand-in conditioner seed")
    args = p.parse_args(argv)
    if not args.jsonl and not (args.prompt and args.out):
        p.error("pass --jsonl, or both --prompt and --out")
    cond = make_conditioner(args.model_root, args.device, args.seed)
    written = []
    if args.jsonl:
        with open(args.jsonl) as f:
            rows = [json.loads(line) for line in f if line.strip()]
        picked = (list(enumerate(rows))[:args.take] if args.rows is None
                  else [(i, rows[i]) for i in args.rows])
        for i, r in picked:
            written.append(encode_one(cond, r["prompt"],
                                      os.path.join(args.out_dir, f"{args.name}_{i}.pt")))
    else:
        written.append(encode_one(cond, args.prompt, args.out))
    return written


if __name__ == "__main__":
    main()
    sys.exit(0)
