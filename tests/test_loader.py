"""The product's safetensors loader (jl_weights_load) against the rules of
the reference loader, engine/src/lib.rs:89-202.  Host only: no GPU needed."""
import json
import struct

import numpy as np
import pytest

import checkpoint as CK
import jalapeno as J
import oracle as O


@pytest.fixture(scope="module")
def tiny():
    return O.Model.synthetic("tiny-draft", 3), O.Model.synthetic("tiny-draft", 3, mxfp4=True)


def test_bf16_checkpoint_round_trips(tmp_path, tiny):
    model, _ = tiny
    CK.write_model(model, tmp_path, quantized=False)
    w = J.load(tmp_path)
    # embed, norm, 11 per layer; tied: no lm_head
    assert len(w) == 2 + 11 * model.cfg.layers
    t = w.tensor("model.layers.0.mlp.up_proj.weight")
    assert t["dtype"] == "bf16" and t["shape"] == (256, 128)
    np.testing.assert_array_equal(t["bf16"], model.tensors["0.up"].bf16.reshape(-1))


def test_mxfp4_checkpoint_pairs_packed_and_scales(tmp_path, tiny):
    _, q = tiny
    CK.write_model(q, tmp_path, quantized=True)
    w = J.load(tmp_path)
    t = w.tensor("model.layers.0.self_attn.q_proj.weight")
    assert t["dtype"] == "mxfp4" and t["shape"] == (256, 128)
    np.testing.assert_array_equal(t["packed"], q.tensors["0.q"].packed.reshape(-1))
    np.testing.assert_array_equal(t["scales"], q.tensors["0.q"].scales.reshape(-1))
    norm = w.tensor("model.layers.0.input_layernorm.weight")
    assert norm["dtype"] == "bf16" and (norm["bf16"] == 0x3F80).all()
    emb = w.tensor("model.embed_tokens.weight")
    assert emb["dtype"] == "bf16"


def raw_file(path, header: dict, data: bytes, header_len=None):
    text = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(text) if header_len is None else header_len))
        f.write(text)
        f.write(data)


def expect_error(tmp_path, match, status=J.JL_ERR_FORMAT):
    with pytest.raises(J.JlError) as e:
        J.load(tmp_path)
    assert e.value.status == status, e.value
    assert match in e.value.message, e.value.message
    # Model::load checks every header before it reads a payload or touches a
    # GPU: the same status and message, here without a device
    cfg = tmp_path / "config.json"
    if not cfg.exists():
        cfg.write_text(json.dumps({"num_hidden_layers": 1, "max_position_embeddings": 64,
                                   "eos_token_id": 0}))
    with pytest.raises(J.JlError) as m:
        J.Model.load(tmp_path)
    assert (m.value.status, m.value.message) == (e.value.status, e.value.message)


def entry(dtype, shape, start, end):
    return {"dtype": dtype, "shape": shape, "data_offsets": [start, end]}


def test_empty_directory(tmp_path):
    expect_error(tmp_path, "no safetensors files")


def test_header_length_checks(tmp_path):
    raw_file(tmp_path / "a.safetensors", {}, b"", header_len=100_000_001)
    expect_error(tmp_path, "invalid safetensors header length")


def test_offsets_out_of_range(tmp_path):
    raw_file(tmp_path / "a.safetensors", {"w": entry("BF16", [2], 0, 8)}, b"\0" * 4)
    expect_error(tmp_path, "invalid tensor offsets")


def test_non_bf16_tensor_rejected(tmp_path):
    raw_file(tmp_path / "a.safetensors", {"w": entry("F32", [2], 0, 8)}, b"\0" * 8)
    expect_error(tmp_path, "expected BF16 tensor")


def test_u16_only_in_quantized_files(tmp_path):
    raw_file(tmp_path / "a.safetensors", {"w": entry("U16", [2], 0, 4)}, b"\0" * 4)
    expect_error(tmp_path, "expected BF16 tensor")


def test_duplicate_across_files(tmp_path):
    raw_file(tmp_path / "a.safetensors", {"w": entry("BF16", [2], 0, 4)}, b"\0" * 4)
    raw_file(tmp_path / "b.safetensors", {"w": entry("BF16", [2], 0, 4)}, b"\0" * 4)
    expect_error(tmp_path, "duplicate tensor")


def q_header(extra=None, scale_shape=(1, 1), packed_shape=(1, 16), packed_len=16, scale_len=1):
    h = {"__metadata__": {"format": "jalapenos-mxfp4-v1"},
         "m.mxfp4_packed": entry("U8", list(packed_shape), 0, packed_len),
         "m.mxfp4_scales": entry("U8", list(scale_shape), packed_len, packed_len + scale_len)}
    h.update(extra or {})
    return h


def test_orphaned_scales(tmp_path):
    h = {"__metadata__": {"format": "jalapenos-mxfp4-v1"}, "m.mxfp4_scales": entry("U8", [1, 1], 0, 1)}
    raw_file(tmp_path / "a.safetensors", h, b"\x7f")
    expect_error(tmp_path, "MXFP4 scales have no matching packed weights")


def test_missing_scales(tmp_path):
    h = {"__metadata__": {"format": "jalapenos-mxfp4-v1"}, "m.mxfp4_packed": entry("U8", [1, 16], 0, 16)}
    raw_file(tmp_path / "a.safetensors", h, b"\0" * 16)
    expect_error(tmp_path, "missing MXFP4 scales")


def test_nan_scale(tmp_path):
    raw_file(tmp_path / "a.safetensors", q_header(), b"\0" * 16 + b"\xff")
    expect_error(tmp_path, "NaN scale")


def test_bad_mxfp4_shape(tmp_path):
    raw_file(tmp_path / "a.safetensors", q_header(scale_shape=(1, 2), scale_len=2), b"\0" * 16 + b"\x7f\x7f")
    expect_error(tmp_path, "invalid MXFP4 tensor shape")


def test_unexpected_u8(tmp_path):
    h = {"__metadata__": {"format": "jalapenos-mxfp4-v1"}, "m": entry("U8", [4], 0, 4)}
    raw_file(tmp_path / "a.safetensors", h, b"\0" * 4)
    expect_error(tmp_path, "unexpected U8 tensor")


def test_u8_in_plain_file_is_not_bf16(tmp_path):
    raw_file(tmp_path / "a.safetensors", {"m.mxfp4_packed": entry("U8", [1, 16], 0, 16)}, b"\0" * 16)
    expect_error(tmp_path, "expected BF16 tensor")


def test_valid_minimal_mxfp4(tmp_path):
    raw_file(tmp_path / "a.safetensors", q_header(), bytes(range(16)) + b"\x7f")
    w = J.load(tmp_path)
    t = w.tensor("m")
    assert t["shape"] == (1, 32)
    np.testing.assert_array_equal(t["packed"], np.arange(16, dtype=np.uint8))


def test_config_requires_reference_fields(tmp_path, tiny):
    model, _ = tiny
    CK.write_model(model, tmp_path, quantized=False)
    cfg = json.loads((tmp_path / "config.json").read_text())
    del cfg["eos_token_id"]
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    with pytest.raises(J.JlError) as e:
        J.Model.load(tmp_path)
    # no GPU here: the config is read before the device is touched
    assert e.value.status in (J.JL_ERR_FORMAT, J.JL_ERR_NO_DEVICE)
