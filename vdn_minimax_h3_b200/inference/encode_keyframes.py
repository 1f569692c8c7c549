"""Encode a keyframe (i2va / l2va / fl2va) or reference (ref2va) request into one prompt
cache (reference src/inference/encode_keyframes.py:158-243).

    python -m vdn_minimax_h3_b200.inference.encode_keyframes --prompt "..." \
        --first first.png [--last last.png] --out prompts/mine.pt
    python -m vdn_minimax_h3_b200.inference.encode_keyframes --prompt "..." \
        --refs a.png b.png [--ref_size 768] --out prompts/mine.pt

Keyframes: the canvas follows the first keyframe (768 short edge, sides multiples of 32,
area <= 768 x 1344); the first is stretched onto it, the last cover-cropped. References:
each on its own `--ref_size` short edge; the render canvas is 16:9. The presentation is
`"<Picture i>: "` + vision block per image, then the prompt (vision rows tagged VIDEO);
each image is VAE-encoded under seed 42. The cache carries prompt, prompt_embeds,
text_token_tags, keyframe_anchors, keyframe_files, condition_latents, height, width (and
reference_size for references). Without --model_root / --vae_root the weight-free
stand-ins produce the same format.
"""
import argparse
import sys

from vdn_minimax_h3_b200.inference.encoders import (REFERENCE_SHORT_EDGE, VIDEO_TAG,
                                                    KEYFRAME_INSTRUCTIONS, KeyframeVaeStandIn,
                                                    build_presentation, check_instruction,
                                                    make_conditioner, normalize_references,
                                                    put_on_canvas, resolve_canvas_size)
from vdn_minimax_h3_b200.inference.prompt_cache import (REFERENCE_ANCHOR, conditioning_mode,
                                                        save_prompt)


def main(argv=None):
    from PIL import Image
    p = argparse.ArgumentParser()
    p.add_argument("--prompt", type=str, required=True)
    p.add_argument("--first", type=str, help="keyframe the video starts from")
    p.add_argument("--last", type=str, help="keyframe the video ends on")
    p.add_argument("--refs", type=str, nargs="+", metavar="IMAGE",
                   help="reference images in <Picture i> order (ref2va-like request)")
    p.add_argument("--ref_size", type=int, default=REFERENCE_SHORT_EDGE)
    p.add_argument("--out", type=str, required=True)
    p.add_argument("--model_root", type=str, default=None,
                   help="MiniMax-H3 snapshot with processor/ and text_encoder/; default: "
                        "the weight-free stand-in conditioner")
    p.add_argument("--device", type=str, default="cuda:0")
    p.add_argument("--seed", type=int, default=0, help="stand-in seeds")
    args = p.parse_args(argv)
    if bool(args.refs) == bool(args.first or args.last):
        p.error("pass --first and/or --last, or --refs (neither is t2va: use encode_prompt)")
    if args.refs:
        pairs = [(REFERENCE_ANCHOR, path) for path in args.refs]
        anchors = [a for a, _ in pairs]
        images = normalize_references([Image.open(path) for _, path in pairs], args.ref_size)
        height, width = resolve_canvas_size(16, 9)
    else:
        pairs = [(a, path) for a, path in (("first", args.first), ("last", args.last)) if path]
        anchors = [a for a, _ in pairs]
        if not check_instruction(args.prompt, anchors):
            print(f"warning: {conditioning_mode(anchors)} keyframes, but the prompt does not "
                  f"open with the mode's instruction line:\n    "
                  f"{KEYFRAME_INSTRUCTIONS[tuple(anchors)][1]}\nEncoding the prompt as given.",
                  file=sys.stderr, flush=True)
        images, height, width = put_on_canvas([Image.open(path) for _, path in pairs])
    mode = conditioning_mode(anchors)
    print(f"{mode}: canvas {width}x{height}; images {[im.size for im in images]}", flush=True)
    cond = make_conditioner(args.model_root, args.device, args.seed)
    ids, tags = build_presentation(cond, args.prompt, images)
    emb = cond.encode(ids, images)
    vae = KeyframeVaeStandIn(args.seed)
    latents = [vae.encode(im) for im in images]
    extra = {"keyframe_files": [path for _, path in pairs], "height": height, "width": width}
    if args.refs:
        extra["reference_size"] = args.ref_size
    save_prompt(args.out, args.prompt, emb, tags, anchors, latents, **extra)
    print(f"wrote {args.out}: {len(ids)} tokens ({tags.count(VIDEO_TAG)} vision rows), "
          f"{len(images)} images {[tuple(c.shape) for c in latents]}", flush=True)
    return args.out


if __name__ == "__main__":
    main()
    sys.exit(0)
