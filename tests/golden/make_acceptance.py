"""Record the reference's STD / AR decoding on the reduced decoder of
acceptance_case.py (CPU, fp16 -- the reference's selection path needs fp16),
with its acceptance, tokens, timing and thread count:

    STD_REFERENCE=<path to the mcy1123/STD checkout> python tests/golden/make_acceptance.py

The reference's modules are built from its own Qwen2_5_VLConfig and loaded
with acceptance_case.state_dict(); a thin wrapper feeds the visual
embeddings at the video-token positions (the vision tower is outside the
path) and the reference's std_generate_qwen25vl / ar_generate_qwen25vl run
unmodified.  Writes tests/golden/acceptance_reduced.npz."""

from __future__ import annotations

import os
import sys
import time
from types import SimpleNamespace

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import acceptance_case as case  # noqa: E402
from make_golden import import_reference  # noqa: E402


def reference_model(qm):
    from specvlm.models.configuration_qwen2_5_vl import Qwen2_5_VLConfig

    config = Qwen2_5_VLConfig(vocab_size=case.VOCAB, hidden_size=case.HIDDEN, intermediate_size=case.INTER,
                              num_hidden_layers=case.LAYERS, num_attention_heads=case.HEADS,
                              num_key_value_heads=case.KV_HEADS, max_position_embeddings=32768,
                              rope_theta=1000000.0, rms_norm_eps=1e-6,
                              rope_scaling={"type": "mrope", "mrope_section": [16, 24, 24]})
    config._attn_implementation = "sdpa"
    for name, val in [("pad_token_id", None), ("output_attentions", False), ("output_hidden_states", False),
                      ("use_return_dict", True), ("use_cache", True)]:
        if not hasattr(config, name):
            setattr(config, name, val)

    class ReducedLM(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.config = config
            self.model = qm.Qwen2_5_VLModel(config)
            self.lm_head = torch.nn.Linear(config.hidden_size, config.vocab_size, bias=False)
            self.visual = None  # [V, H] embeddings for the video-token positions

        @property
        def dtype(self):
            return self.model.embed_tokens.weight.dtype

        def forward(self, input_ids=None, **kwargs):
            emb = self.model.embed_tokens(input_ids)
            mask = input_ids == case.VIDEO_TOKEN_ID
            n = int(mask.sum())
            if n:
                emb = emb.clone()
                emb[mask] = self.visual[:n].to(emb.dtype)
            out = self.model(inputs_embeds=emb, **kwargs)
            return SimpleNamespace(logits=self.lm_head(out.last_hidden_state),
                                   attentions=getattr(out, "attentions", None))

    m = ReducedLM()
    missing, unexpected = m.load_state_dict(case.state_dict(), strict=False)
    assert not unexpected, unexpected
    assert all("rotary" in k or "inv_freq" in k for k in missing), missing
    return m.eval().to(torch.float16)


def main():
    qm, sq = import_reference()
    torch.manual_seed(0)
    model = reference_model(qm)
    rec = {"threads": torch.get_num_threads(), "torch": torch.__version__}
    std_acc, std_tok, ar_tok, std_time, ar_time, prefill = [], [], [], [], [], []
    for i in range(len(case.REQUEST_SEEDS)):
        ids, vis = case.request(i)
        model.visual = vis.to(torch.float16)
        with torch.inference_mode():
            t0 = time.time()
            std, sel = sq.std_generate_qwen25vl(model, {"input_ids": ids}, video_token_id=case.VIDEO_TOKEN_ID,
                                                eos_token_id=-1, max_new_tokens=case.MAX_NEW, gamma=case.GAMMA,
                                                target_k_plus_text=case.K_PLUS_TEXT, ignore_eos=True)
            t1 = time.time()
            ar = sq.ar_generate_qwen25vl(model, {"input_ids": ids}, video_token_id=case.VIDEO_TOKEN_ID,
                                         eos_token_id=-1, max_new_tokens=case.MAX_NEW, ignore_eos=True)
            t2 = time.time()
        P = ids.shape[1]
        std_acc.append(list(std.accept_lengths))
        std_tok.append(std.output_ids[0, P:].numpy())
        ar_tok.append(ar.output_ids[0, P:].numpy())
        std_time.append(std.decoding_time)
        ar_time.append(ar.decoding_time)
        prefill.append(t1 - t0 - std.decoding_time)
        print(f"request {i}: k={sel.k} accept {std.accept_lengths} rate {std.acceptance_rate:.3f} "
              f"std==ar {np.array_equal(std_tok[-1], ar_tok[-1])} std {std.decoding_time:.1f}s ar "
              f"{ar.decoding_time:.1f}s total {t2 - t0:.1f}s", flush=True)
    rounds = max(len(a) for a in std_acc)
    acc = np.full((len(std_acc), rounds), -1, dtype=np.int64)
    for i, a in enumerate(std_acc):
        acc[i, : len(a)] = a
    np.savez_compressed(os.path.join(HERE, "acceptance_reduced.npz"), accept_lengths=acc,
                        std_tokens=np.stack(std_tok), ar_tokens=np.stack(ar_tok),
                        std_decoding_s=np.array(std_time), ar_decoding_s=np.array(ar_time),
                        std_prefill_s=np.array(prefill), threads=np.int64(rec["threads"]), torch=str(rec["torch"]),
                        k=np.int64(sel.k))
    print("wrote acceptance_reduced.npz", rec)


if __name__ == "__main__":
    main()
