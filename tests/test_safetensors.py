"""The safetensors reader (huggingfaceeacp_b200/host/safetensors.h) through
hf_safetensors_describe, on the cases Tests/Model/SafeTensorsTests.cpp holds
the reference's reader to: what a well-formed header lists, and every
malformed header refused with a reason rather than read past its end."""
import os
import struct

import numpy as np
import pytest

import safetensors_files as stf
from huggingfaceeacp_b200 import native


def _file(tmp_path, image: bytes, name="m.safetensors"):
    path = os.path.join(tmp_path, name)
    with open(path, "wb") as f:
        f.write(image)
    return path


def _refused(tmp_path, image: bytes) -> str:
    with pytest.raises(native.SafeTensorsError) as err:
        native.describe_safetensors(_file(tmp_path, image))
    return str(err.value)


def test_single_tensor(tmp_path):
    """SafeTensorsTests.cpp:43-62."""
    blob = np.arange(1, 7, dtype=np.float32).tobytes()
    path = _file(tmp_path, stf.assemble('{"weight":{"dtype":"F32","shape":[2,3],"data_offsets":[0,24]}}', blob))
    d = native.describe_safetensors(path)
    assert d == {"tensors": [("weight", "F32", (2, 3), 0, 24)], "metadata": {}}


def test_multiple_tensors_and_metadata(tmp_path):
    """SafeTensorsTests.cpp:167-191: every tensor, its dtype, shape and range; metadata kept apart."""
    path = os.path.join(tmp_path, "multi.safetensors")
    stf.write(path, {"a": ("F32", np.zeros((4, 8), np.float32)), "b": ("BF16", np.zeros(5, np.uint16)),
                     "c": ("F16", np.zeros((2, 2, 2), np.float16)), "d": ("F64", np.zeros(3, np.float64))},
              metadata={"format": "pt", "note": "tab-free"})
    d = native.describe_safetensors(path)
    assert [(t[0], t[1], t[2]) for t in d["tensors"]] == [("a", "F32", (4, 8)), ("b", "BF16", (5,)),
                                                          ("c", "F16", (2, 2, 2)), ("d", "F64", (3,))]
    assert d["tensors"][1][3:] == (128, 138)
    assert d["metadata"] == {"format": "pt", "note": "tab-free"}


def test_integer_tensors_are_listed(tmp_path):
    """SafeTensorsTests.cpp:192-202: an integer tensor is a legal entry (only widening refuses it)."""
    path = _file(tmp_path, stf.assemble('{"w":{"dtype":"I32","shape":[2],"data_offsets":[0,8]}}',
                                        np.array([1, 2], np.int32).tobytes()))
    assert native.describe_safetensors(path)["tensors"] == [("w", "I32", (2,), 0, 8)]


def test_malformed_headers(tmp_path):
    """SafeTensorsTests.cpp:213-239."""
    assert "shorter than its length prefix" in _refused(tmp_path, bytes(7))
    assert "runs past the end" in _refused(tmp_path, stf.assemble("{}", length=3))
    assert "runs past the end" in _refused(tmp_path, stf.assemble("{}", length=(1 << 64) - 1))
    for header in ("{not json", "[1,2,3]", "", '{"w":42}', '{"w":{"dtype":"F32","shape":[1],"data_offsets":[0,4]}} x',
                   '{"a":{},"a":{}}'):
        _refused(tmp_path, stf.assemble(header, bytes(4)))


def test_missing_fields_and_unknown_dtype(tmp_path):
    """SafeTensorsTests.cpp:241-264."""
    for header, reason in (('{"w":{"shape":[1],"data_offsets":[0,4]}}', "dtype"),
                           ('{"w":{"dtype":"F32","data_offsets":[0,4]}}', "shape"),
                           ('{"w":{"dtype":"F32","shape":[1]}}', "data_offsets"),
                           ('{"w":{"dtype":"F8_E4M3","shape":[1],"data_offsets":[0,1]}}', "unknown dtype")):
        assert reason in _refused(tmp_path, stf.assemble(header, bytes(4)))


def test_shape_disagrees_with_range(tmp_path):
    """SafeTensorsTests.cpp:266-307: a shape and a byte range that disagree, a
    range past the blob, a reversed range and a negative dimension."""
    blob = np.array([1.0, 2.0], np.float32).tobytes()
    cases = (('{"w":{"dtype":"F32","shape":[3],"data_offsets":[0,8]}}', "disagrees"),
             ('{"w":{"dtype":"BF16","shape":[2],"data_offsets":[0,8]}}', "disagrees"),
             ('{"w":{"dtype":"F32","shape":[4],"data_offsets":[0,16]}}', "past the end of the blob"),
             ('{"w":{"dtype":"F32","shape":[1],"data_offsets":[8,4]}}', "reversed"),
             ('{"w":{"dtype":"F32","shape":[-1],"data_offsets":[0,0]}}', "negative"))
    for header, reason in cases:
        assert reason in _refused(tmp_path, stf.assemble(header, blob))


def test_metadata_must_be_strings(tmp_path):
    """SafeTensorsTests.cpp:309-315."""
    assert "not a string" in _refused(tmp_path, stf.assemble('{"__metadata__":{"format":7}}'))
    assert "not an object" in _refused(tmp_path, stf.assemble('{"__metadata__":7}'))


def test_empty_tensor_is_legal(tmp_path):
    """SafeTensorsTests.cpp:317-324."""
    path = _file(tmp_path, stf.assemble('{"empty":{"dtype":"F32","shape":[0,4],"data_offsets":[0,0]}}'))
    assert native.describe_safetensors(path)["tensors"] == [("empty", "F32", (0, 4), 0, 0)]


def test_missing_file_is_an_error(tmp_path):
    """SafeTensorsTests.cpp:326-337."""
    with pytest.raises(native.SafeTensorsError) as err:
        native.describe_safetensors(os.path.join(tmp_path, "no", "such", "model.safetensors"))
    assert "cannot be opened" in str(err.value)


def test_escaped_names_and_large_offsets(tmp_path):
    """JSON escapes in a tensor name and a 64-bit offset beyond 2^53 (refused as past the blob, not mis-read)."""
    blob = np.zeros(1, np.float32).tobytes()
    path = _file(tmp_path, stf.assemble('{"a\\u00e9\\n\\"b":{"dtype":"F32","shape":[1],"data_offsets":[0,4]}}', blob))
    assert native.describe_safetensors(path)["tensors"][0][0] == 'aé\n"b'.replace("\n", "\n")
    big = 9007199254740993  # 2^53 + 1: not representable as a double
    assert "past the end" in _refused(tmp_path, stf.assemble(
        '{"w":{"dtype":"U8","shape":[1],"data_offsets":[%d,%d]}}' % (big, big + 1), blob))


def test_checkpoint_writer_round_trip(tmp_path):
    """The Gemma checkpoint the GPU loader test builds is one the reader accepts, name for name."""
    shape = native.DecoderShape(width=64, heads=2, kv_heads=1, head_width=32, layers=1, intermediate=128, vocab=96,
                                max_positions=16)
    tensors, widened = stf.gemma_checkpoint(shape, seed=3)
    path = os.path.join(tmp_path, "gemma.safetensors")
    stf.write(path, tensors)
    listed = {t[0]: t for t in native.describe_safetensors(path)["tensors"]}
    assert set(listed) == set(tensors)
    assert listed["model.layers.0.mlp.gate_proj.weight"][1:3] == ("BF16", (128, 64))
    assert listed["model.norm.weight"][1:3] == ("F32", (64,))
    # bf16 rounding is to nearest even and widens back exactly
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5e-3], np.float32)
    assert np.array_equal(stf.bf16_widen(stf.bf16_bits(x)), np.array([1.0, 1.0, 1.015625, -0.0025024414], np.float32))
    assert struct.unpack("<Q", open(path, "rb").read(8))[0] > 0
