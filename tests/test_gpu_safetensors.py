"""hf_cuda_load_safetensors: a Gemma checkpoint read from safetensors shards,
its projection weights widened and quantized on the device. The bar is the
reference's loader (TensorLoader.cpp:162-347): widen F16/BF16/F64 exactly
(F64 rounded to nearest), quantize with quantizeInt8Blocks, stack gate over
up. The same float values quantized by the host quantizer (whose bytes equal
the reference's own Int8Blocks.cpp, tests/test_oracle_pins.py) and uploaded
tensor by tensor must give a decoder whose logits and hidden states are
bit-identical, so the device bytes are the host bytes."""
import os

import numpy as np
import pytest

import safetensors_files as stf
from huggingfaceeacp_b200 import native

pytestmark = pytest.mark.gpu

SHAPE = native.DecoderShape(width=2048, heads=8, kv_heads=1, head_width=256, layers=2, intermediate=4096, vocab=8192,
                            max_positions=64, max_step_rows=16, embed_scale=1.0)
PROMPT = np.array([2, 41, 3, 17, 28, 9, 60, 1000, 4097], dtype=np.uint32)


def _shards(tmp_path, tensors, count=2):
    names = sorted(tensors)
    paths = []
    for i in range(count):
        path = os.path.join(tmp_path, f"model-{i + 1:05d}-of-{count:05d}.safetensors")
        stf.write(path, {n: tensors[n] for n in names[i::count]}, metadata={"format": "pt"})
        paths.append(path)
    return paths


def _same_decoder(a: native.Context, b: native.Context, steps: int = 4):
    for ctx in (a, b):
        ctx.begin_sequence()
    la, ha = a.step(PROMPT)
    lb, hb = b.step(PROMPT)
    assert np.array_equal(la, lb) and np.array_equal(ha, hb)
    token = int(np.argmax(la[-1]))
    for _ in range(steps):
        la, ha = a.step([token])
        lb, hb = b.step([token])
        assert np.array_equal(la, lb) and np.array_equal(ha, hb)
        token = int(np.argmax(la[-1]))


def test_checkpoint_equals_host_quantized_upload(tmp_path):
    overrides = {"model.layers.0.self_attn.v_proj.weight": "F16", "model.layers.1.self_attn.o_proj.weight": "F64",
                 "model.layers.1.mlp.up_proj.weight": "F32"}
    tensors, widened = stf.gemma_checkpoint(SHAPE, seed=21, overrides=overrides)
    paths = _shards(tmp_path, tensors)
    with native.Context(SHAPE) as loaded, native.Context(SHAPE) as uploaded:
        assert not loaded.prepared
        loaded.load_safetensors(paths)
        assert loaded.prepared
        stf.upload_widened(uploaded, SHAPE, widened)
        _same_decoder(loaded, uploaded)
        loaded.begin_sequence()
        uploaded.begin_sequence()
        assert list(loaded.generate(PROMPT, 8)) == list(uploaded.generate(PROMPT, 8))


def test_wide_feed_forward_checkpoint_on_the_whole_loop_kernel(tmp_path):
    """The 16384-wide feed-forward: single-token steps run the persistent
    kernel over the stage records and down slices built from the loaded bytes."""
    shape = SHAPE.replace(intermediate=16384, layers=1)
    tensors, widened = stf.gemma_checkpoint(shape, seed=22, dtype="F16")
    paths = _shards(tmp_path, tensors, count=1)
    with native.Context(shape) as loaded, native.Context(shape) as uploaded:
        loaded.load_safetensors(paths)
        stf.upload_widened(uploaded, shape, widened)
        _same_decoder(loaded, uploaded, steps=3)


def test_refusals_leave_the_decoder_unprepared(tmp_path):
    tensors, _ = stf.gemma_checkpoint(SHAPE.replace(layers=1), seed=23)
    shape = SHAPE.replace(layers=1)

    def refused(tensor_map, code, reason, count=1, extra=None):
        sub = os.path.join(tmp_path, str(len(os.listdir(tmp_path))))
        os.makedirs(sub)
        paths = _shards(sub, tensor_map, count)
        if extra:
            paths.append(extra)
        with native.Context(shape) as ctx:
            with pytest.raises(native.HFError) as err:
                ctx.load_safetensors(paths)
            assert err.value.code == code and reason in str(err.value)
            assert not ctx.prepared

    missing = dict(tensors)
    del missing["model.layers.0.mlp.down_proj.weight"]
    refused(missing, native.HF_E_INVALID, "'model.layers.0.mlp.down_proj.weight', and the checkpoint has none")
    wrong = dict(tensors)
    wrong["model.norm.weight"] = ("F32", np.zeros(2047, np.float32))
    refused(wrong, native.HF_E_SHAPE, "tensor 'model.norm.weight' is [2047]")
    integer = dict(tensors)
    integer["model.layers.0.self_attn.k_proj.weight"] = ("I32", np.zeros((256, 2048), np.int32))
    refused(integer, native.HF_E_INVALID, "not a float type")
    dup = os.path.join(tmp_path, "dup.safetensors")
    stf.write(dup, {"model.norm.weight": tensors["model.norm.weight"]})
    refused(tensors, native.HF_E_INVALID, "in more than one shard", extra=dup)
    bad = os.path.join(tmp_path, "bad.safetensors")
    with open(bad, "wb") as f:
        f.write(stf.assemble("{not json"))
    refused(tensors, native.HF_E_INVALID, "not valid JSON", extra=bad)
