"""AR vs STD per-sample benchmark with the reference CLI's decode flags.

    python -m std_b200.benchmark_std --eval-num 2 --frame-num 32 --max-new-tokens 128 \
        --gamma 9 --target-k-plus-text 1024 --ignore-eos --strict-equality --output metrics.jsonl

Mirrors scripts/benchmark_std.py:455-760 of the reference: for each sample, AR
then STD through the public entry points (ar_generate_qwen25vl /
std_generate_qwen25vl), a token-equality check (--strict-equality aborts on a
mismatch, optional first-divergence records in --mismatch-output) and one
JSONL record per sample with the reference's field names where they apply.

The reference reads Video-MME / MLVU / VideoDetailCaption through the
Qwen2.5-VL processor and vision tower; neither the datasets, the weights nor
the vision tower are part of this decode path.  Samples here are synthetic:
a random-init Qwen2.5-VL-7B-shaped decoder (std 0.02, --weights-seed) and,
per sample i, frame_num x 512 visual embeddings N(0,1) followed by
--text-len text ids U[0, 151643) (seed 100 + i) -- the configs' layout.
Flags of the reference that select paths this build does not have
(--dataset other than synthetic, --sparse-attn-mode other than b200,
--verify-fallback other than none, --verify-attn-backend other than default,
--no-copy-sparse-prefill) are rejected.
"""

from __future__ import annotations

import argparse
import json
import sys
import time
from pathlib import Path

import torch

VIDEO_TOKEN_ID = 151656
TOKENS_PER_FRAME = 512


def _args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--dataset", choices=["synthetic"], default="synthetic")
    ap.add_argument("--config", choices=["7b", "tiny"], default="7b", help="decoder shape (tiny: a 2-layer test model)")
    ap.add_argument("--weights-seed", type=int, default=2)
    ap.add_argument("--eval-num", type=int, default=1)
    ap.add_argument("--skip-samples", type=int, default=0)
    ap.add_argument("--frame-num", type=int, default=32)
    ap.add_argument("--text-len", type=int, default=128)
    ap.add_argument("--max-new-tokens", type=int, default=64)
    ap.add_argument("--gamma", type=int, default=9)
    ap.add_argument("--target-k-plus-text", type=int, default=1024)
    ap.add_argument("--k", type=int, default=None)
    ap.add_argument("--verify-mode", choices=["parallel", "sequential"], default="parallel")
    ap.add_argument("--verify-fallback", choices=["none"], default="none")
    ap.add_argument("--verify-attn-backend", choices=["default"], default="default")
    ap.add_argument("--sparse-attn-mode", choices=["b200"], default="b200")
    ap.add_argument("--sparse-cache", choices=["compact", "indexed"], default="compact")
    ap.add_argument("--strict-equality", action="store_true", help="Abort if STD generated tokens differ from AR.")
    ap.add_argument("--ignore-eos", action="store_true",
                    help="Performance mode: continue after EOS so AR and STD both emit exactly max-new-tokens.")
    ap.add_argument("--eos-token-id", type=int, default=151645)
    ap.add_argument("--output", default="results/std_b200/metrics.jsonl")
    ap.add_argument("--mismatch-output", default=None, help="Optional JSONL path for first-divergence diagnostics.")
    return ap.parse_args(argv)


def _sample(i: int, frames: int, text_len: int, hidden: int, vocab: int, device):
    V = frames * TOKENS_PER_FRAME
    g = torch.Generator().manual_seed(100 + i)
    ids = torch.full((1, V + text_len), VIDEO_TOKEN_ID, dtype=torch.int64)
    ids[0, V:] = torch.randint(0, min(151643, vocab), (text_len,), generator=g)
    gd = torch.Generator(device=device).manual_seed(100 + i)
    vis = torch.randn(1, V, hidden, generator=gd, device=device).to(torch.bfloat16)
    return {"input_ids": ids, "visual_embeds": vis}


def _agreement(a: torch.Tensor, b: torch.Tensor):
    """token_level_agreement and common_prefix_length of two generated suffixes."""
    a, b = a.flatten().tolist(), b.flatten().tolist()
    n = min(len(a), len(b))
    prefix = next((i for i in range(n) if a[i] != b[i]), n)
    mism = sum(1 for i in range(n) if a[i] != b[i]) + abs(len(a) - len(b))
    denom = max(len(a), len(b))
    return {"token_level_agreement": 1.0 - mism / denom if denom else 1.0, "common_prefix_length": prefix}


def main(argv=None) -> int:
    args = _args(argv)
    from .model import QWEN25_VL_7B, TINY, Qwen25VLDecoder
    from .std_qwen25vl import ar_generate_qwen25vl, generated_suffix, std_generate_qwen25vl, tokens_equal

    cfg = QWEN25_VL_7B if args.config == "7b" else TINY
    model = Qwen25VLDecoder(cfg, seed=args.weights_seed)
    out_path = Path(args.output)
    out_path.parent.mkdir(parents=True, exist_ok=True)
    mismatch = open(args.mismatch_output, "w", encoding="utf-8") if args.mismatch_output else None
    speedups = []
    try:
        with out_path.open("w", encoding="utf-8") as f:
            for i in range(args.skip_samples, args.skip_samples + args.eval_num):
                inputs = _sample(i, args.frame_num, args.text_len, cfg.hidden_size, cfg.vocab_size, model.device)
                prompt_len = int(inputs["input_ids"].shape[1])
                eos = -1 if args.ignore_eos else args.eos_token_id
                t0 = time.time()
                ar = ar_generate_qwen25vl(model, inputs, VIDEO_TOKEN_ID, eos, max_new_tokens=args.max_new_tokens,
                                          ignore_eos=args.ignore_eos)
                ar_dt = time.time() - t0
                t0 = time.time()
                std, sel = std_generate_qwen25vl(model, inputs, VIDEO_TOKEN_ID, eos,
                                                 max_new_tokens=args.max_new_tokens, gamma=args.gamma,
                                                 target_k_plus_text=args.target_k_plus_text, explicit_k=args.k,
                                                 verify_mode=args.verify_mode, ignore_eos=args.ignore_eos,
                                                 sparse_cache=args.sparse_cache)
                std_dt = time.time() - t0
                a_gen, s_gen = generated_suffix(ar.output_ids, prompt_len), generated_suffix(std.output_ids, prompt_len)
                equal = tokens_equal(a_gen, s_gen)
                agree = _agreement(a_gen, s_gen)
                if not equal and mismatch is not None:
                    mismatch.write(json.dumps({"sample_index": i, **agree,
                                               "ar_tokens": a_gen.flatten().tolist(),
                                               "std_tokens": s_gen.flatten().tolist()}) + "\n")
                if args.strict_equality and not equal:
                    raise RuntimeError(f"STD token mismatch on sample {i}.")
                speedup = ar.decoding_time / std.decoding_time if std.decoding_time > 0 else 0.0
                speedups.append(speedup)
                rec = {
                    "dataset": args.dataset, "sample_index": i, "sample_id": f"synthetic-{100 + i}",
                    "frame_num": args.frame_num, "prompt_len": prompt_len, "visual_len": sel.visual_len,
                    "text_len": sel.text_len, "k": sel.k, "gamma": args.gamma, "verify_mode": args.verify_mode,
                    "verify_fallback": args.verify_fallback, "verify_attn_backend": args.verify_attn_backend,
                    "sparse_attn_mode": args.sparse_attn_mode, "sparse_cache": args.sparse_cache,
                    "copy_sparse_prefill": True, "max_new_tokens": args.max_new_tokens,
                    "ignore_eos": args.ignore_eos, "token_equal": equal, **agree,
                    "ar_generate_len": ar.generate_len, "std_generate_len": std.generate_len,
                    "ar_inference_time": ar.inference_time, "std_inference_time": std.inference_time,
                    "ar_decoding_time": ar.decoding_time, "std_decoding_time": std.decoding_time,
                    "speedup": speedup,
                    "inference_speedup": ar.inference_time / std.inference_time if std.inference_time else 0.0,
                    "ar_tokens_per_second": ar.generate_len / ar.decoding_time if ar.decoding_time else 0.0,
                    "std_tokens_per_second": std.generate_len / std.decoding_time if std.decoding_time else 0.0,
                    "accepted_draft_tokens": std.accepted_draft_tokens,
                    "proposed_draft_tokens": std.proposed_draft_tokens, "acceptance_rate": std.acceptance_rate,
                    "mean_accept_length": std.mean_accept_length, "decode_rounds": std.decode_rounds,
                    "committed_tokens_per_round": std.generate_len / std.decode_rounds if std.decode_rounds else 0.0,
                    "accept_lengths": std.accept_lengths, "ar_prefill_time": ar.prefill_time,
                    "std_prefill_time": std.prefill_time, "std_selection_time": std.selection_time,
                    "std_sparse_cache_time": std.sparse_cache_time, "ar_wall_time": ar_dt, "std_wall_time": std_dt,
                }
                f.write(json.dumps(rec) + "\n")
                f.flush()
                print(f"  [{i}] prompt_len={prompt_len} AR={ar.decoding_time:.2f}s STD={std.decoding_time:.2f}s "
                      f"speedup={speedup:.2f}x accept={std.acceptance_rate:.2f} match={'yes' if equal else 'NO'}",
                      flush=True)
    finally:
        if mismatch is not None:
            mismatch.close()
    if speedups:
        print(f"average speedup {sum(speedups) / len(speedups):.2f}x over {len(speedups)} sample(s)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
