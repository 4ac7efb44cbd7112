"""Test-side ctypes bindings to the CPU oracle (oracle/_build/liboracle.so) and
to the reference's own compiled sources (oracle/_ref/libhf_ref.so).

TEST INFRASTRUCTURE: only tests/, __graft_entry__.smoke() and bench.py's CPU
legs use this module; the product never imports it.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_LIB = os.path.join(ROOT, "oracle", "_build", "liboracle.so")
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libhf_ref.so")
GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")

_vp = ctypes.c_void_p
_oracle = None
_ref = None


class OracleShape(ctypes.Structure):
    _fields_ = [
        ("width", ctypes.c_int), ("heads", ctypes.c_int), ("kv_heads", ctypes.c_int),
        ("head_width", ctypes.c_int), ("layers", ctypes.c_int), ("intermediate", ctypes.c_int),
        ("vocab", ctypes.c_int), ("max_positions", ctypes.c_int), ("rms_eps", ctypes.c_float),
        ("rope_theta", ctypes.c_double), ("embed_scale", ctypes.c_float),
    ]


def oracle() -> ctypes.CDLL:
    global _oracle
    if _oracle is None:
        if not os.path.exists(ORACLE_LIB):
            raise ImportError(f"{ORACLE_LIB} is not built (oracle/build.sh)")
        lib = ctypes.CDLL(ORACLE_LIB)
        lib.oracle_half_from_float.restype = ctypes.c_uint16
        lib.oracle_half_from_float.argtypes = [ctypes.c_float]
        lib.oracle_half_to_float.restype = ctypes.c_float
        lib.oracle_half_to_float.argtypes = [ctypes.c_uint16]
        lib.oracle_int8_blocks_byte_count.restype = ctypes.c_int64
        lib.oracle_int8_blocks_byte_count.argtypes = [ctypes.c_int64]
        lib.oracle_quantizes_as_int8_blocks.argtypes = [ctypes.c_int64, ctypes.c_int64]
        lib.oracle_quantize_int8_blocks.argtypes = [_vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _vp]
        lib.oracle_dequantize_int8_blocks.argtypes = [_vp, ctypes.c_int64, _vp]
        lib.oracle_spread_values.argtypes = [ctypes.c_int, ctypes.c_uint32, ctypes.c_float, _vp]
        lib.oracle_mt19937_raw.argtypes = [ctypes.c_uint32, ctypes.c_int, _vp]
        lib.oracle_rotary_table.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_double, _vp, _vp]
        lib.oracle_tanh_gelu_double.restype = ctypes.c_double
        lib.oracle_tanh_gelu_double.argtypes = [ctypes.c_double]
        lib.oracle_tanh_gelu_float.restype = ctypes.c_float
        lib.oracle_tanh_gelu_float.argtypes = [ctypes.c_float]
        lib.oracle_argmax.restype = ctypes.c_uint32
        lib.oracle_argmax.argtypes = [_vp, _vp, ctypes.c_int64]
        lib.oracle_argmax_double.restype = ctypes.c_uint32
        lib.oracle_argmax_double.argtypes = [_vp, _vp, ctypes.c_int64]
        lib.oracle_model_create.restype = _vp
        lib.oracle_model_create.argtypes = [ctypes.POINTER(OracleShape), ctypes.c_int, ctypes.c_int]
        lib.oracle_model_destroy.argtypes = [_vp]
        lib.oracle_model_set_q8.argtypes = [_vp, ctypes.c_int, ctypes.c_int, _vp]
        lib.oracle_model_set_f32.argtypes = [_vp, ctypes.c_int, ctypes.c_int, _vp]
        lib.oracle_begin_sequence.argtypes = [_vp]
        lib.oracle_position.argtypes = [_vp]
        lib.oracle_threads.argtypes = [_vp]
        lib.oracle_step.argtypes = [_vp, _vp, ctypes.c_int, _vp, _vp, ctypes.c_int]
        lib.oracle_synthetic_stream.restype = ctypes.c_uint64
        lib.oracle_synthetic_stream.argtypes = [ctypes.c_int, ctypes.c_int]
        lib.oracle_synthetic_normal.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int64, ctypes.c_int64,
                                                ctypes.c_double, _vp, ctypes.c_int]
        lib.oracle_synthetic_tokens.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.c_int, _vp]
        _oracle = lib
    return _oracle


def ref_available() -> bool:
    return os.path.exists(REF_LIB)


def ref() -> ctypes.CDLL:
    """The reference's own Int8Blocks.cpp and Sampler.cpp (oracle/build_ref.sh)."""
    global _ref
    if _ref is None:
        lib = ctypes.CDLL(REF_LIB)
        lib.ref_int8_blocks_byte_count.restype = ctypes.c_longlong
        lib.ref_int8_blocks_byte_count.argtypes = [ctypes.c_longlong]
        lib.ref_quantizes_as_int8_blocks.argtypes = [ctypes.c_longlong, ctypes.c_longlong]
        lib.ref_quantize_int8_blocks.argtypes = [_vp, ctypes.c_longlong, ctypes.c_longlong, ctypes.c_longlong, _vp]
        lib.ref_dequantize_int8_blocks.argtypes = [_vp, ctypes.c_longlong, _vp]
        lib.ref_sampler_argmax.argtypes = [_vp, _vp, ctypes.c_longlong]
        lib.ref_mt19937_raw.argtypes = [ctypes.c_uint, ctypes.c_int, _vp]
        lib.ref_sampler_sample.argtypes = [_vp, _vp, ctypes.c_longlong, ctypes.c_float, ctypes.c_int, ctypes.c_float,
                                           ctypes.c_ulonglong, ctypes.c_int, _vp]
        lib.ref_sampler_sample_at.argtypes = [_vp, ctypes.c_longlong, ctypes.c_float, ctypes.c_int, ctypes.c_float,
                                              ctypes.c_ulonglong, ctypes.c_int, _vp]
        lib.ref_reference_decode.argtypes = [_vp, ctypes.c_float, ctypes.c_double, ctypes.c_float, _vp, ctypes.c_int,
                                             _vp, ctypes.c_int, _vp, _vp]
        lib.ref_tokenizer_from_json.restype = _vp
        lib.ref_tokenizer_from_json.argtypes = [ctypes.c_char_p, ctypes.c_size_t]
        lib.ref_tokenizer_free.argtypes = [_vp]
        lib.ref_tokenizer_vocabulary.argtypes = [_vp]
        lib.ref_tokenizer_encode.argtypes = [_vp, ctypes.c_char_p, ctypes.c_size_t, ctypes.c_int, _vp, ctypes.c_int]
        lib.ref_tokenizer_decode.restype = ctypes.c_longlong
        lib.ref_tokenizer_decode.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_char_p, ctypes.c_longlong]
        _ref = lib
    return _ref


class RefTokenizer:
    """The reference's own Tokenizer (Tokenizer/Tokenizer.h:32-124), compiled
    unchanged into oracle/_ref: fromJsonText, encode / encodeWithBos, decode,
    vocabularySize."""

    def __init__(self, json_text: bytes):
        self.lib = ref()
        self.handle = self.lib.ref_tokenizer_from_json(json_text, len(json_text))
        if not self.handle:
            raise ValueError("the reference tokenizer refused the tokenizer.json")

    def vocabulary(self) -> int:
        return int(self.lib.ref_tokenizer_vocabulary(self.handle))

    def encode(self, text: str, bos: bool = False) -> list[int]:
        data = text.encode()
        out = np.zeros(4 * len(data) + 8, dtype=np.int32)
        n = self.lib.ref_tokenizer_encode(self.handle, data, len(data), int(bos), p(out), len(out))
        if n < 0:
            raise ValueError("the reference tokenizer refused the text")
        return [int(t) for t in out[:n]]

    def decode(self, tokens) -> bytes:
        ids = np.ascontiguousarray(tokens, dtype=np.int32)
        cap = 64 * max(1, len(ids)) + 64
        buf = ctypes.create_string_buffer(cap)
        n = self.lib.ref_tokenizer_decode(self.handle, p(ids), len(ids), buf, cap)
        if n < 0 or n > cap:
            raise ValueError("the reference tokenizer refused the tokens")
        return buf.raw[:n]

    def close(self):
        if getattr(self, "handle", None):
            self.lib.ref_tokenizer_free(self.handle)
            self.handle = None

    def __del__(self):
        self.close()


SPACE_PIECE = "\u2581"  # a space as the vocabulary spells it (Tokenizer/Metaspace.h)


def synthetic_tokenizer_json(size: int = 384) -> tuple[str, dict]:
    """A small SentencePiece-BPE tokenizer.json in the form gemma-2b's file
    takes (added special tokens, a Replace(" " -> U+2581) normalizer, byte
    fallback, merges as "left right" strings), built here: pieces for a few
    words out of single letters, the 256 byte pieces, and unused pieces up to
    `size` tokens. Returns the JSON text and the vocabulary (piece -> id)."""
    import json

    vocab = {}

    def add(piece):
        if piece not in vocab:
            vocab[piece] = len(vocab)
        return piece

    for special in ("<pad>", "<eos>", "<bos>", "<unk>"):
        add(special)
    for b in range(256):
        add(f"<0x{b:02X}>")
    add(SPACE_PIECE)
    for c in "abcdefghijklmnopqrstuvwxyz":
        add(c)
    merges = []
    for word in ("the", "cat", "sat", "on", "mat", "hat", "and", "dog", "in", "a"):
        piece = word[0]
        for c in word[1:]:
            merges.append(f"{piece} {c}")
            piece = add(piece + c)
        merges.append(f"{SPACE_PIECE} {piece}")
        add(SPACE_PIECE + piece)
    k = 0
    while len(vocab) < size:
        add(f"<unused{k}>")
        k += 1
    added = [{"id": vocab[t], "content": t, "single_word": False, "lstrip": False, "rstrip": False,
              "normalized": False, "special": True} for t in ("<pad>", "<eos>", "<bos>", "<unk>")]
    doc = {"version": "1.0", "truncation": None, "padding": None, "added_tokens": added,
           "normalizer": {"type": "Replace", "pattern": {"String": " "}, "content": SPACE_PIECE},
           "pre_tokenizer": None, "post_processor": None, "decoder": None,
           "model": {"type": "BPE", "dropout": None, "unk_token": "<unk>", "continuing_subword_prefix": None,
                     "end_of_word_suffix": None, "fuse_unk": True, "byte_fallback": True, "vocab": vocab,
                     "merges": merges}}
    return json.dumps(doc, ensure_ascii=False), vocab


def p(a):
    return None if a is None else a.ctypes.data_as(_vp)


# ---- scalar helpers --------------------------------------------------------

def spread_values(count: int, seed: int, value_range: float) -> np.ndarray:
    """Tests/Kernels/Common.h:90-99."""
    out = np.empty(count, dtype=np.float32)
    oracle().oracle_spread_values(count, seed, value_range, p(out))
    return out


def quantize(values: np.ndarray) -> np.ndarray:
    values = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
    out = np.zeros(int(oracle().oracle_int8_blocks_byte_count(values.size)), dtype=np.uint8)
    oracle().oracle_quantize_int8_blocks(p(values), 0, values.size, values.size, p(out))
    return out


def quantize_threaded(values: np.ndarray, threads: int | None = None) -> np.ndarray:
    """quantize() over pieces of whole 32-element blocks on several threads
    (ctypes releases the GIL): the bytes are the same as one call's."""
    from concurrent.futures import ThreadPoolExecutor

    values = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
    out = np.zeros(int(oracle().oracle_int8_blocks_byte_count(values.size)), dtype=np.uint8)
    threads = threads or os.cpu_count() or 1
    piece = max(32, (values.size // threads + 31) // 32 * 32)

    def run(first):
        count = min(piece, values.size - first)
        oracle().oracle_quantize_int8_blocks(p(values[first:]), first, count, values.size, p(out))

    with ThreadPoolExecutor(threads) as pool:
        list(pool.map(run, range(0, values.size, piece)))
    return out


def dequantize(stored: np.ndarray, elements: int) -> np.ndarray:
    out = np.empty(elements, dtype=np.float32)
    oracle().oracle_dequantize_int8_blocks(p(np.ascontiguousarray(stored)), elements, p(out))
    return out


def ref_quantize(values: np.ndarray) -> np.ndarray:
    values = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
    out = np.zeros(int(ref().ref_int8_blocks_byte_count(values.size)), dtype=np.uint8)
    ref().ref_quantize_int8_blocks(p(values), 0, values.size, values.size, p(out))
    return out


def argmax(logits: np.ndarray, mask: np.ndarray | None = None) -> int:
    logits = np.ascontiguousarray(logits)
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.float32)
    if logits.dtype == np.float64:
        return int(oracle().oracle_argmax_double(p(logits), p(m), logits.size))
    logits = logits.astype(np.float32, copy=False)
    return int(oracle().oracle_argmax(p(logits), p(m), logits.size))


# ---- the BASELINE configs' seeded inputs, without the product's libraries ----

LINEAR_STDDEV = 0.02  # linear weights and the embedding
NORM_STDDEV = 0.1     # norm weights


def synthetic_normal(seed: int, tensor: int, layer: int, count: int, stddev: float) -> np.ndarray:
    out = np.empty(count, dtype=np.float32)
    lib = oracle()
    rc = lib.oracle_synthetic_normal(seed, lib.oracle_synthetic_stream(tensor, layer), 0, count, stddev, p(out), 0)
    assert rc == 0
    return out


def synthetic_tokens(seed: int, count: int, vocab: int) -> np.ndarray:
    out = np.empty(count, dtype=np.uint32)
    assert oracle().oracle_synthetic_tokens(seed, count, vocab, p(out)) == 0
    return out


def synthetic_model(shape, seed: int) -> dict:
    """Every tensor of the random-init model, {(tensor id, layer): Q8_0 bytes
    or fp32 norm}, as native.Context.load_synthetic(keep=True) returns them,
    built from oracle.c alone (generator and quantizer)."""
    from huggingfaceeacp_b200.native import model_tensors, NORM_TENSORS, FINAL_NORM

    out = {}
    for tensor, layer in model_tensors(shape):
        count = int(np.prod(shape.tensor_shape(tensor)))
        if tensor in NORM_TENSORS or tensor == FINAL_NORM:
            out[(tensor, layer)] = synthetic_normal(seed, tensor, layer, count, NORM_STDDEV)
        else:
            out[(tensor, layer)] = quantize_threaded(synthetic_normal(seed, tensor, layer, count, LINEAR_STDDEV))
    return out


def worst_error(actual: np.ndarray, expected: np.ndarray) -> float:
    """Tests/Decoder/Common.h:391-400: max |a - e| / (1 + |e|)."""
    a = np.asarray(actual, dtype=np.float64).reshape(-1)
    e = np.asarray(expected, dtype=np.float64).reshape(-1)
    return float(np.max(np.abs(a - e) / (1.0 + np.abs(e)))) if a.size else 0.0


def dot_product_tolerance(inner: int) -> float:
    """Tests/Kernels/TiledProduct.h:186-198."""
    return 1e-5 + 2.4e-7 * inner


# ---- the model -------------------------------------------------------------

class OracleModel:
    """The CPU forward over the same Q8 bytes the GPU was given.

    tensors: {(tensor_id, layer): uint8 Q8 bytes or float32 norm}, as
    huggingfaceeacp_b200.native.Context.load_synthetic(keep=True) returns.
    """

    def __init__(self, shape, tensors, precision="double", threads=0):
        self.shape = shape
        self.real = np.float64 if precision == "double" else np.float32
        s = OracleShape(shape.width, shape.heads, shape.kv_heads, shape.head_width, shape.layers,
                        shape.intermediate, shape.vocab, shape.max_positions, shape.rms_eps, shape.rope_theta,
                        shape.scale)
        self.lib = oracle()
        self.handle = self.lib.oracle_model_create(ctypes.byref(s), 0 if precision == "double" else 1, threads)
        self.tensors = {k: np.ascontiguousarray(v) for k, v in tensors.items()}  # kept alive: borrowed by C
        for (tensor, layer), data in self.tensors.items():
            if data.dtype == np.uint8:
                rc = self.lib.oracle_model_set_q8(self.handle, tensor, layer, p(data))
            else:
                rc = self.lib.oracle_model_set_f32(self.handle, tensor, layer, p(data))
            assert rc == 0, (tensor, layer)

    def close(self):
        if self.handle:
            self.lib.oracle_model_destroy(self.handle)
            self.handle = None

    def __del__(self):
        self.close()

    @property
    def threads(self) -> int:
        return int(self.lib.oracle_threads(self.handle))

    def begin_sequence(self):
        self.lib.oracle_begin_sequence(self.handle)

    @property
    def position(self) -> int:
        return int(self.lib.oracle_position(self.handle))

    def step(self, tokens, last_row_only=False, want_hidden=True):
        tokens = np.ascontiguousarray(tokens, dtype=np.uint32).reshape(-1)
        n = tokens.size
        hidden = np.empty((n, self.shape.width), dtype=self.real) if want_hidden else None
        logits = np.empty((1 if last_row_only else n, self.shape.vocab), dtype=self.real)
        rc = self.lib.oracle_step(self.handle, p(tokens), n, p(hidden), p(logits), 1 if last_row_only else 0)
        assert rc == 0, "oracle step refused (window)"
        return hidden, logits


def greedy_reference(shape, tensors, prompt, count, precision="double", eos=-1, with_margins=False):
    """The host-driven greedy loop (Tests/Generation/Common.h:248-300):
    prefill, then one step per token, argmax (Sampler.cpp:60-76) fed back."""
    model = OracleModel(shape, tensors, precision=precision)
    _, logits = model.step(prompt, last_row_only=True, want_hidden=False)
    tokens, margins = [], []
    for i in range(count):
        row = logits[-1]
        token = argmax(row)
        if with_margins:
            top = np.partition(row, -2)[-2:]
            margins.append(float(top[1] - top[0]))
        if token == eos:
            break
        tokens.append(token)
        if i + 1 < count and model.position < shape.max_positions:
            _, logits = model.step([token], want_hidden=False)
        elif i + 1 < count:
            break
    model.close()
    return (tokens, margins) if with_margins else tokens


# Raw (unquantized) fp32 tensors of one layer, in the order the reference's
# ReferenceLayer holds them (Tests/Decoder/ReferenceDecoder.h:18-29).
REFERENCE_LAYER_ORDER = ("input_norm", "query", "key", "value", "output", "gate", "up", "down", "post_norm")


def ref_decode(shape, raw, tokens, quantize=True):
    """The reference's own referenceDecode (Tests/Decoder/ReferenceDecoder.h:
    294-375), compiled from the reference tree into oracle/_ref: the whole
    sequence from position 0 in double. raw = {"embedding", "final_norm",
    "layers": [{name: fp32 array} per layer]} holds the unquantized weights;
    quantize takes them through the reference's Int8Blocks round trip first
    (quantizedReferenceModel, :79-103). Returns (hidden [n, width], logits
    [n, vocab]) in float64."""
    tokens = np.ascontiguousarray(tokens, dtype=np.int32).reshape(-1)
    extents = np.array([shape.width, shape.heads, shape.kv_heads, shape.head_width, shape.layers,
                        shape.intermediate, shape.vocab, shape.max_positions], dtype=np.int32)
    arrays = [np.ascontiguousarray(raw["embedding"], dtype=np.float32),
              np.ascontiguousarray(raw["final_norm"], dtype=np.float32)]
    for layer in raw["layers"]:
        arrays += [np.ascontiguousarray(layer[name], dtype=np.float32) for name in REFERENCE_LAYER_ORDER]
    pointers = (_vp * len(arrays))(*[a.ctypes.data for a in arrays])
    hidden = np.empty((tokens.size, shape.width), dtype=np.float64)
    logits = np.empty((tokens.size, shape.vocab), dtype=np.float64)
    rc = ref().ref_reference_decode(p(extents), shape.rms_eps, shape.rope_theta, shape.scale, pointers,
                                    1 if quantize else 0, p(tokens), tokens.size, p(hidden), p(logits))
    assert rc == 0, "the reference decode threw"
    return hidden, logits


def q8_model_tensors(raw):
    """The same raw weights as the engine and the oracle take them: every
    projection and the embedding quantized (oracle.c's quantizer, pinned to the
    reference's), gate and up stacked gate first (DecoderWeights.cpp:45-58),
    norms fp32. Keys are (tensor id, layer) as in native.model_tensors."""
    from huggingfaceeacp_b200 import native

    out = {(native.EMBEDDING, -1): quantize(raw["embedding"]), (native.FINAL_NORM, -1): raw["final_norm"]}
    for l, layer in enumerate(raw["layers"]):
        out[(native.INPUT_NORM, l)] = layer["input_norm"]
        out[(native.QUERY, l)] = quantize(layer["query"])
        out[(native.KEY, l)] = quantize(layer["key"])
        out[(native.VALUE, l)] = quantize(layer["value"])
        out[(native.OUTPUT, l)] = quantize(layer["output"])
        out[(native.GATE_UP, l)] = quantize(np.concatenate([layer["gate"], layer["up"]]))
        out[(native.DOWN, l)] = quantize(layer["down"])
        out[(native.POST_NORM, l)] = layer["post_norm"]
    return out


def reference_synthetic_raw(shape):
    """The reference's synthetic checkpoint values (Tests/Decoder/Common.h:
    179-237): every tensor from spreadValues with seeds counting up from 7100,
    embedding range 0.2, norms 0.1, projections 1/sqrtf(fan-in)."""
    seed = [7100]

    def spread(count, value_range):
        values = spread_values(count, seed[0], value_range)
        seed[0] += 1
        return values

    def fan_in(inner):
        return float(np.float32(1.0) / np.sqrt(np.float32(inner)))

    w, q, kv, f = shape.width, shape.query_width, shape.kv_width, shape.intermediate
    raw = {"embedding": spread(shape.vocab * w, 0.2), "layers": []}
    for _ in range(shape.layers):
        raw["layers"].append({
            "input_norm": spread(w, 0.1), "query": spread(q * w, fan_in(w)), "key": spread(kv * w, fan_in(w)),
            "value": spread(kv * w, fan_in(w)), "output": spread(w * q, fan_in(q)), "gate": spread(f * w, fan_in(w)),
            "up": spread(f * w, fan_in(w)), "down": spread(w * f, fan_in(f)), "post_norm": spread(w, 0.1)})
    raw["final_norm"] = spread(w, 0.1)
    return raw


def ref_sample(logits, mask, temperature, top_k, top_p, seed, draws):
    """The reference's own Sampler (Sampler.cpp:78-215): `draws` tokens from one row."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    mask = None if mask is None else np.ascontiguousarray(mask, dtype=np.float32)
    out = np.zeros(draws, dtype=np.int32)
    rc = ref().ref_sampler_sample(p(logits), p(mask) if mask is not None else None, logits.size, temperature, top_k,
                                  top_p, seed, draws, p(out))
    assert rc == 0, "the reference refused the sampling options"
    return out.astype(np.uint32)


def ref_sample_at(logits, temperature, top_k, top_p, seed, skip):
    """The reference Sampler's draw from `logits` after `skip` earlier draws."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    out = np.zeros(1, dtype=np.int32)
    rc = ref().ref_sampler_sample_at(p(logits), logits.size, temperature, top_k, top_p, seed, skip, p(out))
    assert rc == 0
    return int(out[0])
