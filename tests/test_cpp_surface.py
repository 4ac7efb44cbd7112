"""The C++ HF surface (include/HF/*.h over libhf.so): HF::Decoder, HF::Gemma
(greedy, sampled and text generation), HF::Argmax, HF::Sampler,
HF::SamplingOptions and HF::DecoderWeights with the reference's names
(Decoder/Decoder.h:72-136, Generation/Gemma.h:65-251, Kernels/Argmax.h:206-257,
Sampling/Sampler.h:20-70, Decoder/DecoderWeights.h:53-116), driven by
tests/cpp/hf_surface_test.cpp and checked against the Python binding over the
same engine and the same seeded weights.
"""
import os
import subprocess

import numpy as np
import pytest

from huggingfaceeacp_b200 import build, native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SOURCE = os.path.join(ROOT, "tests", "cpp", "hf_surface_test.cpp")
SHAPE = native.DecoderShape(width=2048, heads=8, kv_heads=1, head_width=256, layers=2, intermediate=4096, vocab=8192,
                            max_positions=64, max_step_rows=16, embed_scale=1.0)
SEED = 31
PROMPT = [2, 5, 41, 3, 17, 28, 9, 60]
EOS = 1  # HF::Gemma::endOfSequence (GemmaConfig.h:62)


def byte_encode(text: str) -> list[int]:
    """The test program's stand-in tokenizer: BOS 2, then byte b as token 3 + b."""
    return [2] + [3 + b for b in text.encode()]


def byte_decode(tokens) -> bytes:
    out = b""
    for t in (int(v) for v in tokens):
        if 3 <= t < 259:
            out += bytes([t - 3])
        elif t >= 259:
            out += f"<{t}>".encode()
    return out


@pytest.fixture(scope="module")
def program(tmp_path_factory):
    lib = build.build_cpp_surface()
    assert lib and os.path.exists(lib)
    out = str(tmp_path_factory.mktemp("cpp") / "hf_surface_test")
    subprocess.run(["g++", "-std=c++20", "-O2", f"-I{os.path.join(ROOT, 'include')}", SOURCE,
                    f"-L{os.path.dirname(lib)}", "-lhf", f"-Wl,-rpath,{os.path.dirname(lib)}", "-o", out], check=True)
    return out


def test_surface_compiles_and_links(program):
    assert os.path.exists(program)


def test_host_side_refusals(tmp_path):
    """SamplingOptions refused as the reference's Sampler refuses them, and the
    text entry points refused without a tokenizer or a prepared decoder: no
    device is touched (tests/cpp/hf_host_refusals.cpp)."""
    lib = build.build_cpp_surface()
    out = str(tmp_path / "hf_host_refusals")
    subprocess.run(["g++", "-std=c++20", "-O1", f"-I{os.path.join(ROOT, 'include')}",
                    os.path.join(ROOT, "tests", "cpp", "hf_host_refusals.cpp"), f"-L{os.path.dirname(lib)}", "-lhf",
                    f"-Wl,-rpath,{os.path.dirname(lib)}", "-o", out], check=True)
    result = subprocess.run([out], capture_output=True, text=True)
    assert result.returncode == 0, result.stderr


@pytest.mark.gpu
def test_cpp_surface_matches_the_python_binding(program, tmp_path):
    out = str(tmp_path / "out.bin")
    s = SHAPE
    subprocess.run([program, out, str(s.width), str(s.heads), str(s.kv_heads), str(s.head_width), str(s.layers),
                    str(s.intermediate), str(s.vocab), str(s.max_positions), str(SEED)], check=True)
    raw = np.fromfile(out, dtype=np.uint8)
    at = 4
    rows = np.frombuffer(raw[at:at + 16 * s.vocab], np.float32).reshape(4, s.vocab)
    at += 16 * s.vocab
    hidden = np.frombuffer(raw[at:at + 4 * s.width], np.float32)
    at += 4 * s.width
    picks = np.frombuffer(raw[at:at + 16], np.uint32)
    host = np.frombuffer(raw[at + 16:at + 32], np.uint32)
    at += 32
    def section(dtype, size):
        nonlocal at
        n = int(np.frombuffer(raw[at:at + 4], np.int32)[0])
        values = np.frombuffer(raw[at + 4:at + 4 + size * n], dtype)
        at += 4 + size * n
        return values

    generated = section(np.uint32, 4)
    refusals = section(np.int32, 4)
    sampled = section(np.uint32, 4)
    text = section(np.uint8, 1).tobytes()
    sampling_refusals = section(np.int32, 4)
    assert at == raw.size

    with native.Context(s) as ctx:
        ctx.load_synthetic(seed=SEED)
        ctx.begin_sequence()
        lg, _ = ctx.step(PROMPT)
        expected = [lg[-1]]
        for t in (7, 11, 13):
            lg, hd = ctx.step([t])
            expected.append(lg[-1])
        np.testing.assert_array_equal(rows, np.stack(expected))
        np.testing.assert_array_equal(hidden, hd[-1])
        reference_tokens = ctx.generate(np.array(PROMPT, np.uint32), 12, eos=EOS)
        text_tokens = ctx.generate(np.array(byte_encode("hi"), np.uint32), 12, eos=EOS)
        sampled_tokens = ctx.generate_sampled(np.array(PROMPT, np.uint32), 12, 0.8, top_k=40, top_p=0.9, seed=7,
                                              eos=EOS)
    np.testing.assert_array_equal(picks, [int(np.argmax(r)) for r in rows])
    np.testing.assert_array_equal(host, picks)
    np.testing.assert_array_equal(generated, reference_tokens)
    assert list(refusals) == [1, 1, 1, 1, 1, 1]
    assert text == byte_decode(text_tokens)
    np.testing.assert_array_equal(sampled, sampled_tokens)
    assert list(sampling_refusals) == [1, 1, 1, 1, 1]
