"""The reference's own Python path, timed on the host cores.

BASELINE INFRASTRUCTURE ONLY.  The product (the CUDA library under
``jalapenos-at-home_b200/``) never imports this module; ``bench.py``'s
reference arm and ``tests/`` do.

The reference's Python baseline (``python/speculative_decoding.py:1-47``,
``python/check_mxfp4.py:27-79``) runs transformers ``Qwen3ForCausalLM``:
the draft proposes with ``generate`` and the target checks the proposals with
one forward over the whole sequence.  Here the same models run in float32
with eager attention on the CPU, loaded with the seeded synthetic weights
(MXFP4 projections dequantized, as ``check_mxfp4.py:44-61`` does), and the
loop keeps both models' KV caches between rounds (a restatement of
``speculative_decoding.py:21-47`` with the caches the Rust engine keeps,
``engine/src/speculative.rs:43-143``): the draft proposes k tokens one at a
time, the target checks them in one forward, both caches are cropped back
to the accepted prefix, and the draft catches up on the accepted tokens.
The oracle-draft override (``oracle.oracle_draft_token``) replaces each
proposal as in the benchmark's workload.
"""
from __future__ import annotations

import time

import numpy as np

import oracle as O


def hf_model(cfg: O.Config, model: O.Model, meta: bool = True):
    """transformers ``Qwen3ForCausalLM`` (float32, eager attention) holding
    ``model``'s weights (MXFP4 matrices dequantized exactly).  With ``meta``
    the module is built without initialising its parameters, which are then
    assigned from the oracle's tensors (full-size models build in seconds)."""
    import torch
    from transformers import Qwen3Config, Qwen3ForCausalLM

    hc = Qwen3Config(
        vocab_size=cfg.vocab, hidden_size=cfg.hidden, intermediate_size=cfg.inter,
        num_hidden_layers=cfg.layers, num_attention_heads=cfg.q_heads,
        num_key_value_heads=cfg.kv_heads, head_dim=O.HEAD_DIM, rms_norm_eps=1e-6,
        rope_theta=1000000.0, max_position_embeddings=cfg.max_positions,
        tie_word_embeddings=cfg.tied, eos_token_id=cfg.eos, attention_bias=False,
        use_sliding_window=False,
    )
    hc._attn_implementation = "eager"
    t = model.tensors
    sd = {"model.embed_tokens.weight": t["embed"].values(),
          "model.norm.weight": O.bf16_to_f32(t["norm"])}
    if not cfg.tied:
        sd["lm_head.weight"] = t["lm_head"].values()
    for layer in range(cfg.layers):
        for name in O.PROJECTIONS:
            sd[f"model.layers.{layer}.{O.HF_NAMES[name]}"] = t[f"{layer}.{name}"].values()
        for name in O.NORM_CODE:
            sd[f"model.layers.{layer}.{O.HF_NAMES[name]}"] = O.bf16_to_f32(t[f"{layer}.{name}"])
    state = {k: torch.from_numpy(np.ascontiguousarray(v, dtype=np.float32)) for k, v in sd.items()}
    if meta:
        with torch.device("meta"):
            m = Qwen3ForCausalLM(hc)
        missing, unexpected = m.load_state_dict(state, strict=False, assign=True)
        # buffers outside the state dict (the rotary frequencies) are rebuilt
        m.model.rotary_emb = type(m.model.rotary_emb)(config=hc)
    else:
        m = Qwen3ForCausalLM(hc)
        missing, unexpected = m.load_state_dict(state, strict=False)
    missing = [k for k in missing if not (cfg.tied and k == "lm_head.weight")]
    assert not missing and not unexpected, (missing, unexpected)
    if cfg.tied:
        m.lm_head.weight = m.model.embed_tokens.weight
    return m.to(torch.float32).eval()


def speculative(target, draft, prompt, count: int, gamma: int, eos: int, vocab: int,
                oracle_stream=None, oracle_p: float = 0.0, oracle_seed: int = 0,
                max_rounds: int | None = None):
    """Greedy speculative decoding with both models' KV caches kept between
    rounds (the control flow of ``engine/src/speculative.rs:43-143``, which
    ``oracle.generate_scheduled`` restates for the oracle's models).  Returns
    (tokens, accepted, drafted, rounds, marks) with ``marks`` = (seconds
    since the end of both prefills, tokens) after each round."""
    import torch
    from transformers import DynamicCache

    def run(model, ids, cache):
        out = model(input_ids=torch.tensor([ids]), past_key_values=cache, use_cache=True)
        return out.logits[0].argmax(dim=-1).tolist()

    def override(tok, position):
        if oracle_stream is None:
            return tok
        return O.oracle_draft_token(oracle_stream, oracle_p, oracle_seed, position, vocab, tok)

    tokens = list(prompt)
    limit = len(prompt) + count
    tc, dc = DynamicCache(), DynamicCache()
    with torch.inference_mode():
        first = run(target, tokens, tc)[-1]
        draft_next = override(run(draft, tokens, dc)[-1], dc.get_seq_length())
        accepted_total = drafted_total = rounds = 0
        pending = None
        marks = []
        t0 = time.perf_counter()
        while len(tokens) < limit:
            if max_rounds is not None and rounds >= max_rounds:
                break
            start = len(tokens)
            budget = min(gamma, limit - start)
            proposed = []
            for i in range(budget):
                proposed.append(draft_next)
                if i + 1 == budget or draft_next == eos:
                    break
                draft_next = override(run(draft, [draft_next], dc)[-1], dc.get_seq_length())
            checked = run(target, ([pending] if pending is not None else []) + proposed, tc)
            predictions = ([first] if first is not None else []) + checked
            first = None
            accepted = 0
            nxt = predictions[0]
            while accepted < len(proposed) and proposed[accepted] == nxt:
                accepted += 1
                nxt = predictions[accepted]
            rounds += 1
            drafted_total += len(proposed)
            accepted_total += accepted
            tokens.extend(proposed[:accepted])
            if (tokens[-1] == eos and accepted > 0) or len(tokens) == limit:
                marks.append((time.perf_counter() - t0, len(tokens)))
                break
            tc.crop(start + accepted)
            dc.crop(min(start + accepted, dc.get_seq_length()))
            tokens.append(nxt)
            if nxt == eos or len(tokens) == limit:
                marks.append((time.perf_counter() - t0, len(tokens)))
                break
            pending = nxt
            tail = tokens[dc.get_seq_length():]
            draft_next = override(run(draft, tail, dc)[-1], dc.get_seq_length())
            marks.append((time.perf_counter() - t0, len(tokens)))
    return tokens, accepted_total, drafted_total, rounds, marks
