"""Writing safetensors files for the tests: well-formed ones from numpy
arrays, malformed ones from a header string, and a Gemma checkpoint of the
synthetic random-init model (the layout GemmaTensors.cpp:25-62 names)."""
import json
import struct

import numpy as np

from huggingfaceeacp_b200 import native

NUMPY_DTYPE = {"F32": np.float32, "F64": np.float64, "F16": np.float16, "I32": np.int32, "U8": np.uint8}


def bf16_bits(values: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns, rounded to nearest even (finite inputs)."""
    bits = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_widen(bits: np.ndarray) -> np.ndarray:
    """bfloat16 bit patterns -> float32, exactly (the top half of a float)."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def assemble(header: str, blob: bytes = b"", length: int | None = None) -> bytes:
    """A file image: 8-byte little-endian header length (`length` overrides it), header, blob."""
    head = header.encode()
    return struct.pack("<Q", len(head) if length is None else length) + head + blob


def write(path, tensors: dict, metadata: dict | None = None):
    """tensors: name -> (dtype name, array). BF16 arrays are uint16 bit patterns."""
    header, blob, at = {}, bytearray(), 0
    for name, (dtype, array) in tensors.items():
        raw = np.ascontiguousarray(array).tobytes()
        header[name] = {"dtype": dtype, "shape": list(array.shape), "data_offsets": [at, at + len(raw)]}
        blob += raw
        at += len(raw)
    if metadata is not None:
        header["__metadata__"] = metadata
    with open(path, "wb") as f:
        f.write(assemble(json.dumps(header), bytes(blob)))


def gemma_checkpoint(shape: native.DecoderShape, seed: int, dtype: str = "BF16", overrides: dict | None = None):
    """The synthetic model's float tensors as a Gemma checkpoint: name ->
    (dtype, array), projection weights in `dtype` (norms F32; `overrides`
    maps a name to another dtype), and name -> the float32 values a loader
    widens them to."""
    tensors, widened = {}, {}
    overrides = overrides or {}

    def add(name, values, as_dtype):
        as_dtype = overrides.get(name, as_dtype)
        if as_dtype == "BF16":
            bits = bf16_bits(values)
            tensors[name], widened[name] = ("BF16", bits), bf16_widen(bits)
        else:
            arr = values.astype(NUMPY_DTYPE[as_dtype])
            tensors[name], widened[name] = (as_dtype, arr), arr.astype(np.float32)

    def normal(tensor, layer, dims, stddev):
        count = int(np.prod(dims))
        return native.synthetic_normal(seed, tensor, layer, count, stddev).reshape(dims)

    W, I = shape.width, shape.intermediate
    add("model.embed_tokens.weight", normal(native.EMBEDDING, -1, (shape.vocab, W), native.LINEAR_STDDEV), dtype)
    for l in range(shape.layers):
        p = f"model.layers.{l}."
        for tensor, suffix in ((native.QUERY, "self_attn.q_proj.weight"), (native.KEY, "self_attn.k_proj.weight"),
                               (native.VALUE, "self_attn.v_proj.weight"), (native.OUTPUT, "self_attn.o_proj.weight"),
                               (native.DOWN, "mlp.down_proj.weight")):
            add(p + suffix, normal(tensor, l, shape.tensor_shape(tensor), native.LINEAR_STDDEV), dtype)
        gate_up = normal(native.GATE_UP, l, (2 * I, W), native.LINEAR_STDDEV)
        add(p + "mlp.gate_proj.weight", gate_up[:I], dtype)
        add(p + "mlp.up_proj.weight", gate_up[I:], dtype)
        add(p + "input_layernorm.weight", normal(native.INPUT_NORM, l, (W,), native.NORM_STDDEV), "F32")
        add(p + "post_attention_layernorm.weight", normal(native.POST_NORM, l, (W,), native.NORM_STDDEV), "F32")
    add("model.norm.weight", normal(native.FINAL_NORM, -1, (W,), native.NORM_STDDEV), "F32")
    return tensors, widened


def upload_widened(ctx: native.Context, shape: native.DecoderShape, widened: dict):
    """The same model through the host path: the widened values quantized by
    the host quantizer (quantizeInt8Blocks' bytes) and uploaded per tensor."""
    ctx.upload(native.EMBEDDING, -1, native.quantize(widened["model.embed_tokens.weight"].reshape(-1)))
    ctx.upload(native.FINAL_NORM, -1, widened["model.norm.weight"])
    for l in range(shape.layers):
        p = f"model.layers.{l}."
        for tensor, suffix in ((native.QUERY, "self_attn.q_proj.weight"), (native.KEY, "self_attn.k_proj.weight"),
                               (native.VALUE, "self_attn.v_proj.weight"), (native.OUTPUT, "self_attn.o_proj.weight"),
                               (native.DOWN, "mlp.down_proj.weight")):
            ctx.upload(tensor, l, native.quantize(widened[p + suffix].reshape(-1)))
        stacked = np.concatenate([widened[p + "mlp.gate_proj.weight"].reshape(-1),
                                  widened[p + "mlp.up_proj.weight"].reshape(-1)])
        ctx.upload(native.GATE_UP, l, native.quantize(stacked))
        ctx.upload(native.INPUT_NORM, l, widened[p + "input_layernorm.weight"])
        ctx.upload(native.POST_NORM, l, widened[p + "post_attention_layernorm.weight"])
