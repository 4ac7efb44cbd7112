"""HF::Gemma's text entry points (include/HF/Gemma.h: generateFromText,
generateText, textForTokens; Gemma.cpp:596-615) driven by the reference's own
tokenizer: its Tokenizer/*.cpp compiled unchanged into oracle/_ref (pinned
against its own known answers in tests/test_reference_tokenizer.py), over a
synthetic SentencePiece-BPE tokenizer.json of 384 pieces and a synthetic model
of the same vocabulary (tests/cpp/hf_text_test.cpp). The text calls must equal
encodeWithBos -> generate -> decode done by hand, and the prompt's tokens must
equal the reference tokenizer's own encoding of it.
"""
import os
import subprocess

import pytest

import oracle_bindings as ob
from huggingfaceeacp_b200 import build

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not ob.ref_available(), reason="oracle/_ref not built (needs the reference tree)")]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SOURCE = os.path.join(ROOT, "tests", "cpp", "hf_text_test.cpp")
SHAPE = ["256", "4", "1", "64", "2", "512", "384", "64", "7"]  # width heads kv_heads head_width layers intermediate vocab positions seed


@pytest.mark.parametrize("prompt", ["the cat sat on the mat", "a dog in a hat", "héllo"])
def test_text_generation_through_the_reference_tokenizer(tmp_path, prompt):
    lib = build.build_cpp_surface()
    ref_dir = os.path.dirname(ob.REF_LIB)
    program = str(tmp_path / "hf_text_test")
    subprocess.run(["g++", "-std=c++20", "-O2", f"-I{os.path.join(ROOT, 'include')}", SOURCE,
                    f"-L{os.path.dirname(lib)}", "-lhf", f"-L{ref_dir}", "-lhf_ref",
                    f"-Wl,-rpath,{os.path.dirname(lib)}", f"-Wl,-rpath,{ref_dir}", "-o", program], check=True)
    text, vocab = ob.synthetic_tokenizer_json()
    json_path = tmp_path / "tokenizer.json"
    json_path.write_text(text, encoding="utf-8")
    out = tmp_path / "out.txt"
    subprocess.run([program, str(json_path), str(out), *SHAPE, prompt], check=True)
    lines = dict(line.split(" ", 1) if " " in line else (line, "") for line in out.read_text().splitlines())
    ids = lambda key: [int(t) for t in lines[key].split()]
    hexed = lambda key: bytes.fromhex(lines[key].strip())

    tok = ob.RefTokenizer(text.encode())
    assert ids("encoded") == tok.encode(prompt, bos=True)
    assert ids("encoded")[0] == vocab["<bos>"]
    generated = ids("generated")
    assert ids("from_text") == generated and 0 < len(generated) <= 12
    assert all(0 <= t < 384 for t in generated)
    assert hexed("text") == hexed("for_tokens") == hexed("decoded") == tok.decode(generated)
