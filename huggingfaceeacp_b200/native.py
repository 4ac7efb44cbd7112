"""ctypes bindings to the two native libraries of this package.

``libhf_cuda.so`` is the sm_100a engine (include/hf_cuda.h); ``libhf_host.so``
holds the Q8_0 quantizer and the seeded weight generator (include/hf_host.h).
Both are built in-tree by ``huggingfaceeacp_b200.build`` into
``huggingfaceeacp_b200/lib``. There is no fallback: a missing library is an
ImportError-grade failure, raised loudly.
"""
from __future__ import annotations

import ctypes
import math
import os
import re
from dataclasses import dataclass

import numpy as np

LIB_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib")

HF_OK = 0
HF_E_INVALID = -1
HF_E_SHAPE = -2
HF_E_CAPACITY = -3
HF_E_WINDOW = -4
HF_E_NOT_READY = -5
HF_E_CUDA = -6
HF_E_DEVICE = -7
HF_E_TOKEN = -8

# Failure-detection probes (hf_cuda.h HF_PROBE_*).
PROBE_STAGE_WAIT, PROBE_GRID_BARRIER = 0, 1

# Decode paths (hf_cuda.h HF_DECODE_*).
DECODE_AUTO, DECODE_GRAPH, DECODE_PERSISTENT = 0, 1, 2

# Stamp slots per CTA of hf_cuda_trace_decode: 0 start, 1 embed, 2 + 32 l + event.
TRACE_SLOTS = 1024
TRACE_LAYER_SLOTS = 32
TRACE_EVENTS = ("qkv.staged", "qkv.limbs", "qkv.done", "qkv.left", "attn.loaded", "attn.scored", "attn.done",
                "attn.left", "merge.done", "merge.left", "o.staged", "o.limbs", "o.done", "o.left", "gu.staged",
                "gu.limbs", "gu.done", "gu.left", "down.staged", "down.done", "down.left", "merge.ml", "merge.rows",
                "merge.folded", "attn.dots")
TRACE_LOGITS_EVENTS = ("logits.staged", "logits.limbs", "logits.done", "logits.left")

# Decode-step kernels the timing hook measures (hf_cuda.h HF_KERNEL_*).
KERNEL_QKV, KERNEL_ATTENTION, KERNEL_OUTPUT, KERNEL_GATE_UP, KERNEL_DOWN, KERNEL_LOGITS = range(6)
KERNEL_NAMES = ("qkv_rope", "attention", "o_proj_residual", "gate_up_geglu", "down_residual", "logits_argmax")

# Tensor ids (DecoderWeights.h:53-116).
EMBEDDING, FINAL_NORM, INPUT_NORM, QUERY, KEY, VALUE, OUTPUT, GATE_UP, DOWN, POST_NORM = range(10)
Q8_TENSORS = (QUERY, KEY, VALUE, OUTPUT, GATE_UP, DOWN)
NORM_TENSORS = (INPUT_NORM, POST_NORM)

_u8p = ctypes.POINTER(ctypes.c_uint8)
_f32p = ctypes.POINTER(ctypes.c_float)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_vp = ctypes.c_void_p


class HFError(RuntimeError):
    """A non-zero status from the C-ABI; ``code`` is the HF_E* value."""

    def __init__(self, code: int, text: str):
        super().__init__(f"[{code}] {text}")
        self.code = code


class ShapeStruct(ctypes.Structure):
    _fields_ = [
        ("width", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("kv_heads", ctypes.c_int32),
        ("head_width", ctypes.c_int32),
        ("layers", ctypes.c_int32),
        ("intermediate", ctypes.c_int32),
        ("vocab", ctypes.c_int32),
        ("max_positions", ctypes.c_int32),
        ("max_step_rows", ctypes.c_int32),
        ("rms_eps", ctypes.c_float),
        ("rope_theta", ctypes.c_double),
        ("embed_scale", ctypes.c_float),
    ]


@dataclass(frozen=True)
class DecoderShape:
    """HF::DecoderShape (Decoder/DecoderShape.h:42-110)."""

    width: int
    heads: int
    kv_heads: int
    head_width: int
    layers: int
    intermediate: int
    vocab: int
    max_positions: int
    max_step_rows: int = 0
    rms_eps: float = 1e-6
    rope_theta: float = 10000.0
    embed_scale: float | None = None  # sqrtf(width) (GemmaConfig.cpp:123-126)

    @property
    def scale(self) -> float:
        if self.embed_scale is not None:
            return float(np.float32(self.embed_scale))
        return float(np.sqrt(np.float32(self.width), dtype=np.float32))

    @property
    def query_width(self) -> int:
        return self.heads * self.head_width

    @property
    def kv_width(self) -> int:
        return self.kv_heads * self.head_width

    def struct(self) -> ShapeStruct:
        return ShapeStruct(self.width, self.heads, self.kv_heads, self.head_width, self.layers, self.intermediate,
                           self.vocab, self.max_positions, self.max_step_rows, self.rms_eps, self.rope_theta,
                           self.scale)

    def tensor_shape(self, tensor: int) -> tuple[int, ...]:
        return {
            EMBEDDING: (self.vocab, self.width),
            FINAL_NORM: (self.width,),
            INPUT_NORM: (self.width,),
            POST_NORM: (self.width,),
            QUERY: (self.query_width, self.width),
            KEY: (self.kv_width, self.width),
            VALUE: (self.kv_width, self.width),
            OUTPUT: (self.width, self.query_width),
            GATE_UP: (2 * self.intermediate, self.width),
            DOWN: (self.width, self.intermediate),
        }[tensor]

    def replace(self, **changes) -> "DecoderShape":
        values = {f: getattr(self, f) for f in self.__dataclass_fields__}
        values.update(changes)
        return DecoderShape(**values)


# google/gemma-2b (GemmaConfig.h:45-65).
GEMMA_2B = DecoderShape(width=2048, heads=8, kv_heads=1, head_width=256, layers=18, intermediate=16384,
                        vocab=256000, max_positions=8192)

# The reference's synthetic test decoder (Tests/Decoder/Common.h:38-72): the
# int8 variant has a 64-wide feed-forward.
SMALL_INT8 = DecoderShape(width=32, heads=2, kv_heads=1, head_width=16, layers=2, intermediate=64, vocab=64,
                          max_positions=16)


def _load(name: str) -> ctypes.CDLL:
    path = os.path.join(LIB_DIR, name)
    if not os.path.exists(path):
        raise ImportError(f"{path} is not built; run python -c 'import __graft_entry__ as g; g.build()'")
    return ctypes.CDLL(path)


_host = None
_cuda = None


def host() -> ctypes.CDLL:
    global _host
    if _host is None:
        lib = _load("libhf_host.so")
        lib.hf_int8_block_count.restype = ctypes.c_int64
        lib.hf_int8_block_count.argtypes = [ctypes.c_int64]
        lib.hf_int8_blocks_byte_count.restype = ctypes.c_int64
        lib.hf_int8_blocks_byte_count.argtypes = [ctypes.c_int64]
        lib.hf_quantizes_as_int8_blocks.argtypes = [ctypes.c_int64, ctypes.c_int64]
        lib.hf_quantize_int8_blocks.argtypes = [_vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _vp, ctypes.c_int]
        lib.hf_dequantize_int8_blocks.argtypes = [_vp, ctypes.c_int64, _vp]
        lib.hf_half_from_float.restype = ctypes.c_uint16
        lib.hf_half_from_float.argtypes = [ctypes.c_float]
        lib.hf_half_to_float.restype = ctypes.c_float
        lib.hf_half_to_float.argtypes = [ctypes.c_uint16]
        lib.hf_synthetic_stream.restype = ctypes.c_uint64
        lib.hf_synthetic_stream.argtypes = [ctypes.c_int, ctypes.c_int]
        lib.hf_synthetic_normal.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int64, ctypes.c_int64,
                                            ctypes.c_double, _vp, ctypes.c_int]
        lib.hf_synthetic_tokens.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.c_int, _vp]
        lib.hf_host_threads.restype = ctypes.c_int
        lib.hf_safetensors_describe.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_uint64]
        _host = lib
    return _host


class SamplingStruct(ctypes.Structure):
    """hf_sampling (include/hf_cuda.h): HF::SamplingOptions."""
    _fields_ = [("temperature", ctypes.c_float), ("top_k", ctypes.c_int32), ("top_p", ctypes.c_float),
                ("seed", ctypes.c_uint64)]


def cuda() -> ctypes.CDLL:
    global _cuda
    if _cuda is None:
        lib = _load("libhf_cuda.so")
        lib.hf_cuda_device_count.argtypes = [ctypes.POINTER(ctypes.c_int)]
        lib.hf_cuda_create.argtypes = [ctypes.c_int, ctypes.POINTER(ShapeStruct), ctypes.POINTER(_vp)]
        lib.hf_cuda_create_batch.argtypes = [ctypes.c_int, ctypes.POINTER(ShapeStruct), ctypes.c_int,
                                             ctypes.POINTER(_vp)]
        lib.hf_cuda_sequences.argtypes = [_vp]
        lib.hf_cuda_create_paged.argtypes = [ctypes.c_int, ctypes.POINTER(ShapeStruct), ctypes.c_int, ctypes.c_int,
                                             ctypes.POINTER(_vp)]
        lib.hf_cuda_admit_async.argtypes = [_vp, ctypes.c_int, _vp, ctypes.c_int]
        lib.hf_cuda_release.argtypes = [_vp, ctypes.c_int]
        lib.hf_cuda_sequence_position.argtypes = [_vp, ctypes.c_int]
        lib.hf_cuda_free_pages.argtypes = [_vp]
        lib.hf_cuda_prefill_batch_async.argtypes = [_vp, _vp, ctypes.c_int]
        lib.hf_cuda_decode_batch_async.argtypes = [_vp, ctypes.c_int]
        lib.hf_cuda_read_batch_slots.argtypes = [_vp, ctypes.c_int, ctypes.c_int, _vp]
        lib.hf_cuda_generate_batch.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp]
        lib.hf_cuda_sample.argtypes = [_vp, _vp, _vp, ctypes.c_int, ctypes.POINTER(SamplingStruct), ctypes.c_int, _vp]
        lib.hf_cuda_generate_sampled.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                 ctypes.POINTER(SamplingStruct), _vp, ctypes.POINTER(ctypes.c_int)]
        lib.hf_cuda_destroy.argtypes = [_vp]
        lib.hf_cuda_destroy.restype = None
        lib.hf_cuda_last_error.argtypes = [_vp]
        lib.hf_cuda_last_error.restype = ctypes.c_char_p
        lib.hf_cuda_upload_q8.argtypes = [_vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_uint64]
        lib.hf_cuda_upload_f32.argtypes = [_vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_uint64]
        lib.hf_cuda_load_safetensors.argtypes = [_vp, ctypes.POINTER(ctypes.c_char_p), ctypes.c_int]
        lib.hf_cuda_prepared.argtypes = [_vp]
        lib.hf_cuda_begin_sequence.argtypes = [_vp]
        lib.hf_cuda_position.argtypes = [_vp]
        lib.hf_cuda_step.argtypes = [_vp, _vp, ctypes.c_int, _vp, _vp]
        lib.hf_cuda_argmax.argtypes = [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, _vp]
        lib.hf_cuda_generate_greedy.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp,
                                                ctypes.POINTER(ctypes.c_int)]
        lib.hf_cuda_prefill_async.argtypes = [_vp, _vp, ctypes.c_int]
        lib.hf_cuda_decode_async.argtypes = [_vp, ctypes.c_int]
        lib.hf_cuda_read_slots.argtypes = [_vp, ctypes.c_int, ctypes.c_int, _vp]
        lib.hf_cuda_sync.argtypes = [_vp]
        lib.hf_cuda_stream.argtypes = [_vp]
        lib.hf_cuda_stream.restype = _vp
        lib.hf_cuda_decode_launches.argtypes = [_vp, ctypes.c_int]
        lib.hf_cuda_set_decode_path.argtypes = [_vp, ctypes.c_int]
        lib.hf_cuda_probe_wait_timeout.argtypes = [_vp, ctypes.c_int]
        lib.hf_cuda_nccl_unique_id.argtypes = [_vp]
        lib.hf_cuda_set_tensor_parallel.argtypes = [_vp, ctypes.c_int, ctypes.c_int, _vp]
        lib.hf_cuda_trace_decode.argtypes = [_vp, ctypes.c_int, _vp, ctypes.c_int, ctypes.POINTER(ctypes.c_int),
                                             ctypes.POINTER(ctypes.c_int)]
        lib.hf_cuda_decode_path.argtypes = [_vp]
        lib.hf_cuda_fast_path.argtypes = [_vp]
        lib.hf_cuda_linear_q8.argtypes = [_vp, _vp, _vp, _vp, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                          ctypes.c_int, ctypes.c_int, _vp]
        lib.hf_cuda_quantize_q8.argtypes = [_vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _vp, _vp]
        lib.hf_cuda_linear_create.argtypes = [ctypes.c_int, _vp, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                              ctypes.POINTER(_vp)]
        lib.hf_cuda_linear_run.argtypes = [_vp, _vp, _vp, _vp, ctypes.c_uint32, ctypes.c_int, ctypes.c_int, _vp]
        lib.hf_cuda_linear_path.argtypes = [_vp, ctypes.c_uint32]
        lib.hf_cuda_linear_destroy.argtypes = [_vp]
        lib.hf_cuda_linear_destroy.restype = None
        lib.hf_cuda_argmax_noalloc.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp, _vp]
        lib.hf_cuda_time_kernel.argtypes = [_vp, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_float),
                                            ctypes.POINTER(ctypes.c_double)]
        _cuda = lib
    return _cuda


def _ptr(array: np.ndarray | None):
    if array is None:
        return None
    assert array.flags["C_CONTIGUOUS"]
    return array.ctypes.data_as(_vp)


# ---------------------------------------------------------------------------
# Q8_0 blocks on the host (Kernels/Int8Blocks.h).

class SafeTensorsError(ValueError):
    """A safetensors file the reader refuses (hf_safetensors_describe)."""


def describe_safetensors(path: str, capacity: int = 1 << 20) -> dict:
    """The validated header of a safetensors file (hf_safetensors_describe):
    {"tensors": [(name, dtype, shape, begin, end), ...], "metadata": {...}}."""
    text = ctypes.create_string_buffer(capacity)
    rc = host().hf_safetensors_describe(os.fsencode(path), text, capacity)
    if rc < 0:
        raise SafeTensorsError(text.value.decode(errors="replace"))
    def unescape(field):
        return re.sub(r"\\(.)", lambda m: {"t": "\t", "n": "\n"}.get(m.group(1), m.group(1)), field)

    tensors, metadata = [], {}
    for line in text.value.decode().split("\n")[:-1]:
        parts = [unescape(f) for f in line.split("\t")]
        if parts[0] == "__metadata__":
            metadata[parts[1]] = parts[2]
        else:
            shape = tuple(int(d) for d in parts[2].split(",")) if parts[2] else ()
            tensors.append((parts[0], parts[1], shape, int(parts[3]), int(parts[4])))
    assert len(tensors) == rc
    return {"tensors": tensors, "metadata": metadata}


def int8_blocks_byte_count(elements: int) -> int:
    return int(host().hf_int8_blocks_byte_count(elements))


def quantizes_as_int8_blocks(contiguous: int, elements: int) -> bool:
    return bool(host().hf_quantizes_as_int8_blocks(contiguous, elements))


def quantize(values: np.ndarray, threads: int = 0) -> np.ndarray:
    values = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
    out = np.zeros(int8_blocks_byte_count(values.size), dtype=np.uint8)
    rc = host().hf_quantize_int8_blocks(_ptr(values), 0, values.size, values.size, _ptr(out), threads)
    if rc:
        raise HFError(rc, "quantize refused")
    return out


def dequantize(stored: np.ndarray, elements: int) -> np.ndarray:
    out = np.zeros(elements, dtype=np.float32)
    rc = host().hf_dequantize_int8_blocks(_ptr(np.ascontiguousarray(stored, dtype=np.uint8)), elements, _ptr(out))
    if rc:
        raise HFError(rc, "dequantize refused")
    return out


# ---------------------------------------------------------------------------
# Seeded synthetic weights (hf_host.h): linear weights and the embedding
# N(0, 0.02), norm weights N(0, 0.1).

LINEAR_STDDEV = 0.02
NORM_STDDEV = 0.1


def synthetic_normal(seed: int, tensor: int, layer: int, count: int, stddev: float, threads: int = 0,
                     first: int = 0) -> np.ndarray:
    out = np.empty(count, dtype=np.float32)
    stream = host().hf_synthetic_stream(tensor, layer)
    rc = host().hf_synthetic_normal(seed, stream, first, count, stddev, _ptr(out), threads)
    if rc:
        raise HFError(rc, "generator refused")
    return out


def synthetic_tokens(seed: int, count: int, vocab: int) -> np.ndarray:
    out = np.empty(count, dtype=np.uint32)
    rc = host().hf_synthetic_tokens(seed, count, vocab, _ptr(out))
    if rc:
        raise HFError(rc, "token generator refused")
    return out


def synthetic_tensor(shape: DecoderShape, tensor: int, layer: int, seed: int, threads: int = 0) -> np.ndarray:
    """One tensor of the random-init model: fp32 norms, or Q8_0 bytes."""
    dims = shape.tensor_shape(tensor)
    count = int(np.prod(dims))
    if tensor in (FINAL_NORM, INPUT_NORM, POST_NORM):
        return synthetic_normal(seed, tensor, layer, count, NORM_STDDEV, threads)
    values = synthetic_normal(seed, tensor, layer, count, LINEAR_STDDEV, threads)
    return quantize(values, threads)


def model_tensors(shape: DecoderShape):
    """(tensor, layer) pairs in load order."""
    yield EMBEDDING, -1
    yield FINAL_NORM, -1
    for layer in range(shape.layers):
        for tensor in (INPUT_NORM, QUERY, KEY, VALUE, OUTPUT, GATE_UP, DOWN, POST_NORM):
            yield tensor, layer


# ---------------------------------------------------------------------------

PAGE_ROWS = 64  # hf_cuda.h HF_PAGE_ROWS: positions per KV page of a batched sequence


class Context:
    """One hf_ctx: a prepared decoder on one device (HF::Decoder + DecoderWeights).

    sequences > 1 (or pages given) makes a batch context: that many independent
    sequences over a paged KV cache, decoded together by the *_batch methods
    and admitted / released one by one; `pages` sizes the page pool
    (hf_cuda_create_paged), None reserves every sequence's whole window
    (hf_cuda_create_batch). The other methods use the single-sequence window."""

    def __init__(self, shape: DecoderShape, device: int = 0, sequences: int = 1, pages: int | None = None):
        self.lib = cuda()
        self.shape = shape
        self.sequences = sequences
        handle = _vp()
        struct = shape.struct()
        if pages is not None:
            rc = self.lib.hf_cuda_create_paged(device, ctypes.byref(struct), sequences, pages, ctypes.byref(handle))
        elif sequences == 1:
            rc = self.lib.hf_cuda_create(device, ctypes.byref(struct), ctypes.byref(handle))
        else:
            rc = self.lib.hf_cuda_create_batch(device, ctypes.byref(struct), sequences, ctypes.byref(handle))
        if rc:
            raise HFError(rc, "the engine refused the shape, the sequence count or the device")
        self.handle = handle

    def close(self):
        if getattr(self, "handle", None):
            self.lib.hf_cuda_destroy(self.handle)
            self.handle = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def error(self) -> str:
        text = self.lib.hf_cuda_last_error(self.handle)
        return text.decode() if text else ""

    def check(self, rc: int):
        if rc:
            raise HFError(rc, self.error())

    def upload(self, tensor: int, layer: int, data: np.ndarray):
        data = np.ascontiguousarray(data)
        if data.dtype == np.uint8:
            self.check(self.lib.hf_cuda_upload_q8(self.handle, tensor, layer, _ptr(data), data.size))
        else:
            data = data.astype(np.float32, copy=False)
            self.check(self.lib.hf_cuda_upload_f32(self.handle, tensor, layer, _ptr(data), data.size))

    def load_synthetic(self, seed: int, keep: bool = False, threads: int = 0):
        """Generates, quantizes and uploads every tensor; returns them when keep."""
        kept = {}
        for tensor, layer in model_tensors(self.shape):
            data = synthetic_tensor(self.shape, tensor, layer, seed, threads)
            self.upload(tensor, layer, data)
            if keep:
                kept[(tensor, layer)] = data
        return kept

    def load_safetensors(self, paths):
        """Every Gemma tensor from a (sharded) safetensors checkpoint, the
        projection weights quantized on the device (hf_cuda_load_safetensors)."""
        paths = [paths] if isinstance(paths, (str, os.PathLike)) else list(paths)
        array = (ctypes.c_char_p * len(paths))(*[os.fsencode(p) for p in paths])
        self.check(self.lib.hf_cuda_load_safetensors(self.handle, array, len(paths)))

    @property
    def prepared(self) -> bool:
        return bool(self.lib.hf_cuda_prepared(self.handle))

    @property
    def fast_path(self) -> bool:
        return bool(self.lib.hf_cuda_fast_path(self.handle))

    def begin_sequence(self):
        self.check(self.lib.hf_cuda_begin_sequence(self.handle))

    @property
    def position(self) -> int:
        return int(self.lib.hf_cuda_position(self.handle))

    def step(self, tokens, want_logits=True, want_hidden=True):
        tokens = np.ascontiguousarray(tokens, dtype=np.uint32).reshape(-1)
        n = tokens.size
        logits = np.empty((n, self.shape.vocab), dtype=np.float32) if want_logits else None
        hidden = np.empty((n, self.shape.width), dtype=np.float32) if want_hidden else None
        self.check(self.lib.hf_cuda_step(self.handle, _ptr(tokens), n, _ptr(logits), _ptr(hidden)))
        return logits, hidden

    def argmax(self, logits: np.ndarray, mask: np.ndarray | None = None) -> np.ndarray:
        logits = np.ascontiguousarray(logits, dtype=np.float32)
        rows, length = (1, logits.size) if logits.ndim == 1 else logits.shape
        out = np.empty(rows, dtype=np.uint32)
        m = None if mask is None else np.ascontiguousarray(mask, dtype=np.float32)
        self.check(self.lib.hf_cuda_argmax(self.handle, _ptr(logits), _ptr(m), rows, length, _ptr(out)))
        return out

    def generate(self, prompt, max_tokens: int, eos: int = -1) -> np.ndarray:
        prompt = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.empty(max(max_tokens, 1), dtype=np.uint32)
        count = ctypes.c_int(0)
        self.check(self.lib.hf_cuda_generate_greedy(self.handle, _ptr(prompt), prompt.size, max_tokens, eos,
                                                    _ptr(out), ctypes.byref(count)))
        return out[: count.value].copy()

    def prefill_async(self, prompt):
        prompt = np.ascontiguousarray(prompt, dtype=np.uint32)
        self.check(self.lib.hf_cuda_prefill_async(self.handle, _ptr(prompt), prompt.size))

    def decode_async(self, steps: int):
        self.check(self.lib.hf_cuda_decode_async(self.handle, steps))

    def read_slots(self, first: int, count: int) -> np.ndarray:
        out = np.empty(count, dtype=np.uint32)
        self.check(self.lib.hf_cuda_read_slots(self.handle, first, count, _ptr(out)))
        return out

    def sync(self):
        self.check(self.lib.hf_cuda_sync(self.handle))

    # ---- sampling on the device (hf_cuda_sample, hf_cuda_generate_sampled) --
    def sample(self, logits, temperature: float, top_k: int = 0, top_p: float = 1.0, seed: int = 0, draws: int = 1,
               mask=None) -> np.ndarray:
        logits = np.ascontiguousarray(logits, dtype=np.float32)
        mask = None if mask is None else np.ascontiguousarray(mask, dtype=np.float32)
        out = np.empty(max(draws, 1), dtype=np.uint32)
        options = SamplingStruct(temperature, top_k, top_p, seed)
        self.check(self.lib.hf_cuda_sample(self.handle, _ptr(logits), _ptr(mask), logits.size, ctypes.byref(options),
                                           draws, _ptr(out)))
        return out[:draws].copy()

    def generate_sampled(self, prompt, max_tokens: int, temperature: float, top_k: int = 0, top_p: float = 1.0,
                         seed: int = 0, eos: int = -1) -> np.ndarray:
        prompt = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.empty(max(max_tokens, 1), dtype=np.uint32)
        count = ctypes.c_int(0)
        options = SamplingStruct(temperature, top_k, top_p, seed)
        self.check(self.lib.hf_cuda_generate_sampled(self.handle, _ptr(prompt), prompt.size, max_tokens, eos,
                                                     ctypes.byref(options), _ptr(out), ctypes.byref(count)))
        return out[: count.value].copy()

    # ---- batched decode (hf_cuda_*_batch) ----------------------------------
    def _prompts(self, prompts) -> np.ndarray:
        prompts = np.ascontiguousarray(prompts, dtype=np.uint32)
        if prompts.ndim != 2 or prompts.shape[0] != self.sequences:
            raise ValueError(f"prompts must be [{self.sequences}, length]")
        return prompts

    def prefill_batch_async(self, prompts):
        prompts = self._prompts(prompts)
        self.check(self.lib.hf_cuda_prefill_batch_async(self.handle, _ptr(prompts), prompts.shape[1]))

    def decode_batch_async(self, steps: int):
        self.check(self.lib.hf_cuda_decode_batch_async(self.handle, steps))

    def admit_async(self, sequence: int, prompt):
        """Admits one sequence of a batch with its prompt (hf_cuda_admit_async)."""
        prompt = np.ascontiguousarray(prompt, dtype=np.uint32)
        self.check(self.lib.hf_cuda_admit_async(self.handle, sequence, _ptr(prompt), prompt.size))

    def release(self, sequence: int):
        self.check(self.lib.hf_cuda_release(self.handle, sequence))

    def sequence_position(self, sequence: int) -> int:
        """Tokens in a batched sequence's cache, -1 when it is not active."""
        return int(self.lib.hf_cuda_sequence_position(self.handle, sequence))

    @property
    def free_pages(self) -> int:
        return int(self.lib.hf_cuda_free_pages(self.handle))

    def read_batch_slots(self, first: int, count: int) -> np.ndarray:
        out = np.empty((self.sequences, count), dtype=np.uint32)
        self.check(self.lib.hf_cuda_read_batch_slots(self.handle, first, count, _ptr(out)))
        return out

    def generate_batch(self, prompts, tokens: int) -> np.ndarray:
        """[sequences, tokens]: each sequence's first `tokens` greedy ids."""
        prompts = self._prompts(prompts)
        out = np.empty((self.sequences, max(tokens, 1)), dtype=np.uint32)
        self.check(self.lib.hf_cuda_generate_batch(self.handle, _ptr(prompts), prompts.shape[1], tokens, _ptr(out)))
        return out[:, :tokens].copy()

    @property
    def stream(self) -> int:
        return int(self.lib.hf_cuda_stream(self.handle) or 0)

    def decode_launches(self, steps: int) -> int:
        """Kernel launches that decode_async(steps) makes from the current position."""
        return int(self.lib.hf_cuda_decode_launches(self.handle, steps))

    def trace_decode(self, steps: int, max_ctas: int = 1024) -> np.ndarray:
        """[ctas, events] %globaltimer stamps (ns) of the first traced step (hf_cuda_trace_decode)."""
        stamps = np.zeros(max_ctas * TRACE_SLOTS, dtype=np.uint64)
        ctas, events = ctypes.c_int(0), ctypes.c_int(0)
        self.check(self.lib.hf_cuda_trace_decode(self.handle, steps, _ptr(stamps), stamps.size, ctypes.byref(ctas),
                                                 ctypes.byref(events)))
        return stamps[: ctas.value * events.value].reshape(ctas.value, events.value)

    def set_tensor_parallel(self, rank: int, world: int, nccl_id: bytes | None):
        """Tensor-parallel prefill on `world` GPUs (hf_cuda_set_tensor_parallel);
        every rank calls it at the same time with the id rank 0 made."""
        buf = None
        if nccl_id is not None:
            buf = (ctypes.c_uint8 * NCCL_ID_BYTES).from_buffer_copy(nccl_id)
        self.check(self.lib.hf_cuda_set_tensor_parallel(self.handle, rank, world, buf))

    def probe_wait_timeout(self, kind: int):
        """Enqueues one bounded wait that must give up (hf_cuda_probe_wait_timeout)."""
        self.check(self.lib.hf_cuda_probe_wait_timeout(self.handle, kind))

    def set_decode_path(self, path: int):
        self.check(self.lib.hf_cuda_set_decode_path(self.handle, path))

    @property
    def decode_path(self) -> int:
        return int(self.lib.hf_cuda_decode_path(self.handle))

    def time_kernel(self, kernel: int, reps: int) -> tuple[float, float]:
        """(mean microseconds, algorithmic bytes) of one decode-step kernel launch."""
        us = ctypes.c_float(0.0)
        nbytes = ctypes.c_double(0.0)
        self.check(self.lib.hf_cuda_time_kernel(self.handle, kernel, reps, ctypes.byref(us), ctypes.byref(nbytes)))
        return float(us.value), float(nbytes.value)


# Kernels a prepared linear runs (hf_cuda.h HF_LINEAR_*).
LINEAR_STREAM, LINEAR_ROWS_MMA, LINEAR_TENSOR_CORES, LINEAR_GENERIC = range(4)
LINEAR_PATH_NAMES = ("q8_gemv_stream", "q8_rows_mma", "q8_tc_gemm", "q8_rows_generic")


class Linear:
    """One Q8_0 weight prepared for the product kernels (hf_cuda_linear_*):
    LinearProductFor<Int8Blocks> bound to its stored weight. `weights` is the
    two-region bytes (host array, or a device address as an int); run() takes
    device addresses (ints) and enqueues on `stream`."""

    def __init__(self, weights, inner: int, outputs: int, max_rows: int, device: int = 0):
        self.lib = cuda()
        handle = _vp()
        pointer = weights if isinstance(weights, int) else _ptr(np.ascontiguousarray(weights, dtype=np.uint8))
        rc = self.lib.hf_cuda_linear_create(device, pointer, inner, outputs, max_rows, ctypes.byref(handle))
        if rc:
            raise HFError(rc, "the engine refused the linear weight")
        self.handle, self.inner, self.outputs, self.max_rows = handle, inner, outputs, max_rows

    def path(self, rows: int) -> int:
        return int(self.lib.hf_cuda_linear_path(self.handle, rows))

    def run(self, input_ptr: int, output_ptr: int, rows: int, bias_ptr: int | None = None, gelu: bool = False,
            residual: bool = False, stream: int | None = None):
        rc = self.lib.hf_cuda_linear_run(self.handle, input_ptr, bias_ptr, output_ptr, rows, int(gelu), int(residual),
                                         stream)
        if rc:
            raise HFError(rc, "linear run refused")

    def close(self):
        if getattr(self, "handle", None):
            self.lib.hf_cuda_linear_destroy(self.handle)
            self.handle = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


NCCL_ID_BYTES = 128  # hf_cuda.h HF_NCCL_ID_BYTES


def nccl_unique_id() -> bytes:
    """A new NCCL communicator id (hf_cuda_nccl_unique_id), made by rank 0."""
    buf = (ctypes.c_uint8 * NCCL_ID_BYTES)()
    rc = cuda().hf_cuda_nccl_unique_id(buf)
    if rc:
        raise HFError(rc, "libnccl.so.2 could not make a communicator id")
    return bytes(buf)


def broadcast_bytes(dist, payload: bytes | None, size: int, device="cpu") -> bytes:
    """rank 0's `size` bytes on every rank (torch.distributed broadcast)."""
    import torch

    t = torch.zeros(size, dtype=torch.uint8, device=device)
    if dist.get_rank() == 0:
        t.copy_(torch.frombuffer(bytearray(payload), dtype=torch.uint8))
    dist.broadcast(t, src=0)
    return bytes(t.cpu().numpy().tobytes())


def device_count() -> int:
    n = ctypes.c_int(0)
    cuda().hf_cuda_device_count(ctypes.byref(n))
    return n.value


def weight_bytes(shape: DecoderShape) -> int:
    """Algorithmic Q8_0 weight bytes one decode token streams (layers + tied logits)."""
    per_layer = sum(int8_blocks_byte_count(int(np.prod(shape.tensor_shape(t)))) for t in Q8_TENSORS)
    return per_layer * shape.layers + int8_blocks_byte_count(shape.vocab * shape.width)


def decode_bytes(shape: DecoderShape, keys: int) -> int:
    """Algorithmic bytes of one batch-1 decode token attending to `keys` positions."""
    norms = 4 * shape.width * (2 * shape.layers + 1)
    kv = 4 * 2 * shape.kv_width * shape.layers
    return weight_bytes(shape) + norms + kv * keys + kv + 4 * shape.vocab


def batched_decode_bytes(shape: DecoderShape, sequences: int, keys: int) -> int:
    """Algorithmic bytes of one batched decode step: the weights once, and per
    sequence its K/V rows read (`keys` positions) and written, and its logits."""
    per_sequence = decode_bytes(shape, keys) - weight_bytes(shape) - 4 * shape.width * (2 * shape.layers + 1)
    return decode_bytes(shape, keys) + (sequences - 1) * per_sequence
