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


def _compile(lib, source, out):
    subprocess.run(["g++", "-std=c++20", "-O1", f"-I{os.path.join(ROOT, 'include')}", source,
                    f"-L{os.path.dirname(lib)}", "-lhf", f"-Wl,-rpath,{os.path.dirname(lib)}", "-o", out], check=True)
    return out


def _config(shape, **fields):
    config = {"model_type": "gemma", "vocab_size": shape.vocab, "hidden_size": shape.width,
              "intermediate_size": shape.intermediate, "num_hidden_layers": shape.layers,
              "num_attention_heads": shape.heads, "num_key_value_heads": shape.kv_heads, "head_dim": shape.head_width,
              "max_position_embeddings": shape.max_positions, "rms_norm_eps": 1e-6, "rope_theta": 10000.0,
              "hidden_activation": "gelu_pytorch_tanh", "tie_word_embeddings": True}
    config.update(fields)
    return {k: v for k, v in config.items() if v is not None}


def test_config_and_directory_reading(tmp_path):
    """DecoderShape::fromConfigFile and ShardedTensors::fromDirectory (host
    only): the fields, google/gemma-2b's values for absent ones, and the
    refusals naming the file, the field or the directory."""
    import json

    lib = build.build_cpp_surface()
    program = _compile(lib, os.path.join(ROOT, "tests", "cpp", "hf_config_test.cpp"), str(tmp_path / "hf_config_test"))
    cases = {
        "full": (_config(SHAPE), ["model-00001-of-00002.safetensors", "model-00002-of-00002.safetensors"]),
        "defaults": ({"model_type": "gemma"}, ["model.safetensors", "extra.safetensors"]),
        "llama": (_config(SHAPE, model_type="llama"), ["model.safetensors"]),
        "zero_layers": (_config(SHAPE, num_hidden_layers=0), ["model.safetensors"]),
        "heads": (_config(SHAPE, num_key_value_heads=3), ["model.safetensors"]),  # 3 does not divide 8
        "no_weights": (_config(SHAPE), []),
        "no_config": (None, ["model.safetensors"]),
        "not_json": ("{\"vocab_size\": 12,", ["model.safetensors"]),
    }
    dirs = []
    for name, (config, files) in cases.items():
        d = tmp_path / name
        d.mkdir()
        if isinstance(config, dict):
            (d / "config.json").write_text(json.dumps(config))
        elif isinstance(config, str):
            (d / "config.json").write_text(config)
        for f in files:
            (d / f).write_bytes(b"")
        dirs.append(str(d))
    lines = subprocess.run([program, *dirs], capture_output=True, text=True, check=True).stdout.splitlines()
    got = dict(zip(cases, lines))
    s = SHAPE
    assert got["full"].split()[1:9] == [str(v) for v in (s.width, s.heads, s.kv_heads, s.head_width, s.layers,
                                                         s.intermediate, s.vocab, s.max_positions)]
    assert got["full"].split()[-1] == "2" and np.float32(got["full"].split()[11]) == np.sqrt(np.float32(2048))
    assert got["defaults"].split()[1:9] == ["2048", "8", "1", "256", "18", "16384", "256000", "8192"]
    assert got["defaults"].split()[-1] == "1"  # model.safetensors alone
    assert got["llama"].startswith("error") and "llama" in got["llama"]
    assert got["zero_layers"].startswith("error") and "num_hidden_layers" in got["zero_layers"]
    assert got["heads"].startswith("error") and "num_key_value_heads" in got["heads"]
    assert got["no_weights"].startswith("error") and "no .safetensors" in got["no_weights"]
    assert got["no_config"].startswith("error") and "config.json" in got["no_config"]
    assert got["not_json"].startswith("error") and "JSON" in got["not_json"]


@pytest.mark.gpu
def test_cpp_loads_a_model_directory_like_the_python_binding(tmp_path):
    """Gemma::load(directory) and DecoderWeights(ShardedTensors, shape) over a
    two-shard BF16 checkpoint with its config.json: the same tokens and
    bit-identical logits as the Python binding's hf_cuda_load_safetensors."""
    import json

    import safetensors_files as stf

    shape = SHAPE.replace(embed_scale=None)  # config.json's scale: sqrtf(hidden_size)
    tensors, _ = stf.gemma_checkpoint(shape, seed=SEED)
    names = sorted(tensors)
    paths = []
    for i in range(2):
        path = str(tmp_path / f"model-{i + 1:05d}-of-00002.safetensors")
        stf.write(path, {n: tensors[n] for n in names[i::2]}, metadata={"format": "pt"})
        paths.append(path)
    (tmp_path / "config.json").write_text(json.dumps(_config(shape)))
    lib = build.build_cpp_surface()
    program = _compile(lib, os.path.join(ROOT, "tests", "cpp", "hf_checkpoint_test.cpp"),
                       str(tmp_path / "hf_checkpoint_test"))
    out = str(tmp_path / "out.bin")
    subprocess.run([program, str(tmp_path), out], check=True)
    raw = np.fromfile(out, dtype=np.uint8)
    head = np.frombuffer(raw[:16], np.int32)
    assert list(head) == [shape.width, shape.layers, shape.vocab, shape.max_positions]
    count = int(np.frombuffer(raw[16:20], np.int32)[0])
    tokens = np.frombuffer(raw[20:20 + 4 * count], np.uint32)
    logits = np.frombuffer(raw[20 + 4 * count:20 + 4 * count + 4 * shape.vocab], np.float32)
    with native.Context(shape) as ctx:
        ctx.load_safetensors(paths)
        ctx.begin_sequence()
        ref_logits, _ = ctx.step(np.array(PROMPT, dtype=np.uint32))
        ref_tokens = ctx.generate(np.array(PROMPT, dtype=np.uint32), 6, eos=EOS)
    assert np.array_equal(logits, ref_logits[-1])
    assert list(tokens) == list(ref_tokens)
