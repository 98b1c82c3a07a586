"""Generates the golden fixtures in tests/golden/ from the reference itself.

Run where a checkout of the reference project is available; its path is the
required first argument.  The fixtures it writes are committed, so tests
never need the reference at run time.

* mxfp4_quantize.npz -- inputs and outputs of the reference's own
  ``quantize`` / ``dequantize`` (python/quantize_mxfp4.py:18-49) on seeded
  matrices and hand-picked edge cases (midpoints, signed zeros, tiny and huge
  blocks, all-zero blocks).
* forward_<model>.npz -- the reference's Python oracle pattern
  (python/check_mxfp4.py:38-62): transformers ``Qwen3ForCausalLM`` in float32
  with eager attention, loaded with seeded synthetic weights (dequantized
  MXFP4 where quantized), producing hidden_1, logits and greedy tokens.
* synth.npz -- first values and checksums of the seeded weight stream, so the
  generator definition cannot drift.

Usage: python tests/golden/make_golden.py <path to the reference checkout>
"""
from __future__ import annotations

import importlib.util
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO / "oracle"))
import oracle as O  # noqa: E402


def load_reference_quantizer(ref: Path):
    spec = importlib.util.spec_from_file_location("quantize_mxfp4", ref / "python" / "quantize_mxfp4.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def quantize_cases(rng: np.random.Generator) -> dict[str, np.ndarray]:
    cases = {}
    cases["normal_002"] = (rng.standard_normal((32, 256)) * 0.02).astype(np.float32)
    cases["normal_1"] = rng.standard_normal((16, 256)).astype(np.float32)
    # bf16-rounded weights: what the converter actually feeds quantize()
    w = (rng.standard_normal((32, 512)) * 0.02).astype(np.float32)
    cases["bf16_weights"] = O.bf16_to_f32(O.f32_to_bf16(w)).reshape(w.shape)
    cases["tiny"] = (rng.standard_normal((8, 128)) * 1e-38).astype(np.float32)
    cases["subnormal"] = (rng.standard_normal((4, 64)) * 1e-44).astype(np.float32)
    cases["huge"] = (rng.standard_normal((8, 128)) * 1e37).astype(np.float32)
    cases["mixed_scales"] = (rng.standard_normal((16, 256)) *
                             np.exp2(rng.integers(-40, 40, (16, 256)))).astype(np.float32)
    levels = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], np.float32)
    codes = np.tile(np.concatenate([levels, -levels]), 2)[None, :]
    cases["all_codes"] = codes.astype(np.float32)
    mids = np.zeros((4, 32), np.float32)
    mids[0, :8] = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0]
    mids[1, :8] = -mids[0, :8]
    mids[1, 8] = 6.0
    mids[2, :] = -0.0
    mids[3, :16] = np.linspace(-6, 6, 16) * 2.0 ** -30
    cases["midpoints"] = mids
    blocks = np.zeros((2, 64), np.float32)
    blocks[0, :32] = 6
    blocks[0, 32:] = -0.75
    cases["per_block"] = blocks
    # exact midpoints at many scales (ties to even), plus values just off them
    ties = np.zeros((8, 32), np.float32)
    for r in range(8):
        e = float(2.0 ** (r * 7 - 20))
        ties[r, 0] = 6 * e
        ties[r, 1:8] = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32) * e
        ties[r, 8:15] = np.nextafter(ties[r, 1:8], np.float32(np.inf))
        ties[r, 15:22] = np.nextafter(ties[r, 1:8], np.float32(0))
    cases["ties"] = ties
    return cases


def make_quantize(ref: Path) -> None:
    q = load_reference_quantizer(ref)
    rng = np.random.default_rng(20261201)
    out = {}
    for name, values in quantize_cases(rng).items():
        packed, scales = q.quantize(values)
        out[f"{name}.values"] = values
        out[f"{name}.packed"] = packed
        out[f"{name}.scales"] = scales
        out[f"{name}.dequantized"] = q.dequantize(packed, scales)
    np.savez_compressed(HERE / "mxfp4_quantize.npz", **out)
    print("mxfp4_quantize.npz:", len(out) // 4, "cases")


def hf_model(cfg: O.Config, model: O.Model):
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
    m = Qwen3ForCausalLM(hc).to(torch.float32).eval()
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
    state = {k: torch.from_numpy(np.array(v, dtype=np.float32)) for k, v in sd.items()}
    missing, unexpected = m.load_state_dict(state, strict=False)
    missing = [k for k in missing if not (cfg.tied and k == "lm_head.weight")]
    assert not missing and not unexpected, (missing, unexpected)
    if cfg.tied:
        m.tie_weights()
    return m


def make_forward(name: str, preset: str, seed: int, mxfp4: bool, prompt_len: int, new: int,
                 full_logits: bool) -> None:
    import torch
    import transformers

    torch.set_num_threads(8)
    cfg = O.PRESETS[preset]
    model = O.Model.synthetic(cfg, seed, mxfp4=mxfp4)
    prompt = O.prompt_ids(prompt_len, cfg.vocab, 2)
    m = hf_model(cfg, model)
    ids = torch.tensor([prompt])
    with torch.inference_mode():
        out = m(ids, output_hidden_states=True)
        gen = m.generate(ids, max_new_tokens=new, do_sample=False, eos_token_id=None,
                         pad_token_id=0)
    logits = out.logits[0].float().numpy()
    rec = {
        "prompt": np.array(prompt, np.int64),
        "hidden_1": out.hidden_states[1][0].float().numpy(),
        "tokens": gen[0].numpy().astype(np.int64),
        "meta": np.array(json.dumps({
            "preset": preset, "seed": seed, "mxfp4": mxfp4, "torch": torch.__version__,
            "transformers": transformers.__version__, "attn": "eager", "dtype": "float32"})),
    }
    if full_logits:
        rec["logits"] = logits
        rec["last_logits"] = logits[-1]
    else:
        top = np.argsort(-logits, axis=1)[:, :16]
        rec["top_ids"] = top.astype(np.int64)
        rec["top_logits"] = np.take_along_axis(logits, top, axis=1)
    np.savez_compressed(HERE / f"forward_{name}.npz", **rec)
    print(f"forward_{name}.npz:", rec["tokens"][prompt_len:].tolist())


def make_synth() -> None:
    rec = {}
    for seed in (0, 1):
        for idx in (0, 1, 5, 12):
            rec[f"s{seed}_t{idx}_head"] = O.synth_bf16(seed, idx, 64)
            rec[f"s{seed}_t{idx}_mid"] = O.synth_bf16(seed, idx, 37, first=1_000_003)
    blob = O.synth_bf16(0, 3, 1 << 20)
    rec["s0_t3_sum_f64"] = np.array(O.bf16_to_f32(blob).astype(np.float64).sum())
    rec["s0_t3_bits_xor"] = np.array(np.bitwise_xor.reduce(blob.astype(np.uint64) *
                                                           np.arange(1, blob.size + 1, dtype=np.uint64)))
    rec["prompt_32_seed2"] = np.array(O.prompt_ids(32, 151936, 2), np.int64)
    np.savez_compressed(HERE / "synth.npz", **rec)
    print("synth.npz")


def main() -> None:
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <path to the reference checkout>")
    ref = Path(sys.argv[1])
    make_quantize(ref)
    make_synth()
    make_forward("tiny", "tiny", 0, False, 12, 16, True)
    make_forward("tiny_untied", "tiny-untied", 0, False, 12, 16, True)
    make_forward("tiny_mxfp4", "tiny", 0, True, 12, 16, True)
    make_forward("qwen3_0_6b", "qwen3-0.6b", 1, False, 8, 4, False)
    make_forward("qwen3_0_6b_mxfp4", "qwen3-0.6b", 1, True, 8, 4, False)


if __name__ == "__main__":
    main()
