"""Model::load streams checkpoint payloads from the files to the GPU.

`jl_model_load` validates every safetensors header first (the checks of
engine/src/lib.rs:85-202), then copies each tensor's bytes from its file to
device memory through two pinned chunks, so the checkpoint is never whole in
host memory.  These tests hold it to the in-memory loader (`jl_weights_load`,
the reference's `load`): the same bytes for every tensor, with tensors larger
than a staging chunk and split over two files, and the same tied-head rule
(a lm_head equal to the embedding table is stored once, gpu.rs:340-357).
"""
import numpy as np
import pytest

import checkpoint as CK
import jalapeno as J
import oracle as O

pytestmark = pytest.mark.gpu

# embed and lm_head are 40000 x 256 bf16 = 20.5 MB each: more than one 16 MB chunk
BIG = O.Config("stream-test", 2, 256, 2, 1, 512, 40000, False)


def _device_bytes(model, t):
    if t["dtype"] == "mxfp4":
        want = np.concatenate([t["packed"], t["scales"]])
    else:
        want = t["bf16"].view(np.uint8)
    return model.read_tensor(t["name"], want.size), want


@pytest.mark.parametrize("quantized", [False, True])
def test_streamed_tensors_equal_the_host_loader(tmp_path, quantized):
    ref = O.Model.synthetic(BIG, 7, mxfp4=quantized)
    CK.write_model(ref, tmp_path, quantized=quantized, shards=2)
    host = J.load(tmp_path)
    model = J.Model.load(tmp_path, kv_pool_tokens=256)
    assert model.info.tied == 0
    names = host.names()
    assert "lm_head.weight" in names and len(names) == 3 + 11 * BIG.layers
    for name in names:
        t = dict(host.tensor(name), name=name)
        got, want = _device_bytes(model, t)
        np.testing.assert_array_equal(got, want, err_msg=name)


def test_head_equal_to_embedding_is_tied(tmp_path):
    cfg = O.Config("stream-tied", 1, 256, 2, 1, 512, 40000, True)
    ref = O.Model.synthetic(cfg, 9)
    ref.tensors["lm_head"] = ref.tensors["embed"]
    CK.write_model(ref, tmp_path, quantized=False)
    model = J.Model.load(tmp_path, kv_pool_tokens=256)
    assert model.info.tied == 1
    prompt = O.prompt_ids(8, cfg.vocab, 2)
    synth = J.Model.from_config(cfg, 9, kv_pool_tokens=256)
    a = model.predict(prompt, model.cache(), all=True, logits=True)[1]
    b = synth.predict(prompt, synth.cache(), all=True, logits=True)[1]
    np.testing.assert_array_equal(a, b)
