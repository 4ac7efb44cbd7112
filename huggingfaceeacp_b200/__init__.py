"""B200-native (sm_100a) engine for HuggingFaceEACP's Gemma-2B Q8_0 token loop.

The product is two native libraries built in-tree (``huggingfaceeacp_b200/lib``):
``libhf_cuda.so`` (CUDA kernels + C-ABI, include/hf_cuda.h) and
``libhf_host.so`` (Q8_0 quantizer + seeded generator, include/hf_host.h), with
the C++ ``HF::`` surface (include/HF/) in ``libhf.so``. ``native`` binds them
through ctypes for the tests and the bench.
"""
from .native import (  # noqa: F401
    GEMMA_2B,
    SMALL_INT8,
    Context,
    DecoderShape,
    HFError,
    decode_bytes,
    device_count,
    weight_bytes,
)
