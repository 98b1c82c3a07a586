"""Fuzzing the product's safetensors loader (jl_weights_load, the rules of
engine/src/lib.rs:89-202): whatever bytes a checkpoint holds, loading either
succeeds or fails with a status and a message; it never crashes, hangs or
reads outside the file.  Host only."""
import json
import struct

import pytest
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

import checkpoint as CK
import jalapeno as J
import oracle as O

SETTINGS = settings(max_examples=150, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])


@pytest.fixture(scope="module")
def valid_bytes(tmp_path_factory):
    """One shard of a tiny MXFP4 checkpoint (packed/scales pairs and U16 norms)."""
    d = tmp_path_factory.mktemp("valid")
    CK.write_model(O.Model.synthetic("tiny-draft", 3, mxfp4=True), d, quantized=True, shards=1)
    return (d / "model-00001-of-00001.safetensors").read_bytes(), (d / "config.json").read_text()


def load_or_error(directory):
    try:
        J.load(directory)
    except J.JlError as e:
        assert e.status in (J.JL_ERR_FORMAT, J.JL_ERR_INVALID_ARG, J.JL_ERR_OOM, J.JL_ERR_IO), e
        assert e.message
        return False
    return True


def write(directory, name, data):
    directory.mkdir(parents=True, exist_ok=True)
    (directory / name).write_bytes(data)


def test_valid_file_loads(tmp_path, valid_bytes):
    raw, _ = valid_bytes
    write(tmp_path, "a.safetensors", raw)
    assert load_or_error(tmp_path)


@SETTINGS
@given(data=st.data())
def test_mutated_bytes(tmp_path_factory, valid_bytes, data):
    raw, _ = valid_bytes
    b = bytearray(raw)
    hlen = struct.unpack("<Q", raw[:8])[0]
    # flip bytes anywhere (header-heavy), then maybe truncate or extend
    for _ in range(data.draw(st.integers(1, 8))):
        at = data.draw(st.integers(0, min(len(b) - 1, 8 + hlen + 64)))
        b[at] = data.draw(st.integers(0, 255))
    cut = data.draw(st.sampled_from([None, 0, 4, 8, 8 + hlen // 2, 8 + hlen, len(b) - 1]))
    if cut is not None:
        del b[cut:]
    if data.draw(st.booleans()):
        b += bytes(data.draw(st.binary(max_size=64)))
    load_or_error(tmp_path_factory.mktemp("m"))  # empty directory: an error, not a crash
    d = tmp_path_factory.mktemp("m")
    write(d, "a.safetensors", bytes(b))
    load_or_error(d)


DTYPES = ["BF16", "U8", "U16", "F32", "F16", "I64", "BOOL", "", "bf16"]


@st.composite
def headers(draw):
    n = draw(st.integers(0, 4))
    header = {}
    size = draw(st.integers(0, 4096))
    for i in range(n):
        name = draw(st.sampled_from(["model.norm.weight", "w.mxfp4_packed", "w.mxfp4_scales",
                                     "model.embed_tokens.weight", "x", "lm_head.weight"]))
        shape = draw(st.lists(st.integers(-2, 70000), max_size=3))
        a = draw(st.integers(-5, size + 100))
        b = draw(st.integers(-5, size + 100))
        offs = draw(st.sampled_from([[a, b], [a], [], "x", [a, b, 0]]))
        header[name + ("" if i == 0 else str(i))] = {"dtype": draw(st.sampled_from(DTYPES)), "shape": shape,
                                                     "data_offsets": offs}
    if draw(st.booleans()):
        header["__metadata__"] = {"format": draw(st.sampled_from(["pt", "jalapenos-mxfp4-v1", "other"]))}
    return header, size


@SETTINGS
@given(h=headers(), declared=st.sampled_from([None, 0, 1, 7, 10**9, 2**63]))
def test_random_headers(tmp_path_factory, h, declared):
    header, size = h
    text = json.dumps(header).encode()
    raw = struct.pack("<Q", len(text) if declared is None else declared) + text + bytes(size)
    d = tmp_path_factory.mktemp("h")
    write(d, "a.safetensors", raw)
    load_or_error(d)


def test_garbage_json_and_lengths(tmp_path):
    for i, body in enumerate([b"", b"\xff" * 16, b"{", b"[]", b'{"a": 1}', b'{"a": {"dtype": "BF16"}}',
                              b'{"a": {"dtype": "BF16", "shape": [2], "data_offsets": [0, 4]}}']):
        d = tmp_path / str(i)
        write(d, "a.safetensors", struct.pack("<Q", len(body)) + body)
        load_or_error(d)
