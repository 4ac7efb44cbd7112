"""The reference's own tokenizer (Tokenizer/Tokenizer.cpp, ByteFallback.cpp,
Metaspace.cpp, SpecialTokens.cpp), compiled unchanged into oracle/_ref with
small stand-ins for Miro's JSON reader and UTF-8 decoder (oracle/ref_shim/Miro),
pinned on CPU against the reference's own known answers for its committed
fixture (Tests/Tokenizer/TokenizerTests.cpp:140-194 on
Tests/Tokenizer/Fixtures/MiniTokenizer.json, read where it lies), then checked
on this repository's synthetic tokenizer.json that the GPU text tests use.
"""
import os

import pytest

import oracle_bindings as ob
from huggingfaceeacp_b200 import build

pytestmark = pytest.mark.skipif(not ob.ref_available(), reason="oracle/_ref not built (needs the reference tree)")


def fixture_text():
    root = build.reference_root()
    path = os.path.join(root, "Tests", "Tokenizer", "Fixtures", "MiniTokenizer.json") if root else None
    if not path or not os.path.exists(path):
        pytest.skip("the reference tree's tokenizer fixture is not here")
    with open(path, "rb") as f:
        return f.read()


def test_reference_fixture_known_answers():
    tok = ob.RefTokenizer(fixture_text())
    assert tok.vocabulary() == 289
    # encodeWithBos puts the fixture's <bos> (2) in front of encode's tokens
    assert tok.encode("", bos=True) == [2]
    assert tok.encode("hello world") == [276, 282]
    assert tok.encode("the cat") == [284, 288]
    assert tok.encode("cat") == [287]
    assert tok.encode("the") == [284]
    assert tok.encode(" the") == [285]
    assert tok.encode("the  cat") == [284, 262, 288]
    for text in ("the  cat", " the cat "):
        assert tok.decode(tok.encode(text)) == text.encode()


def test_reference_tokenizer_on_the_synthetic_vocabulary():
    text, vocab = ob.synthetic_tokenizer_json()
    tok = ob.RefTokenizer(text.encode())
    assert tok.vocabulary() == len(vocab) == 384
    sp = ob.SPACE_PIECE
    assert tok.encode("the cat sat on the mat", bos=True) == [
        vocab["<bos>"], vocab["the"], vocab[sp + "cat"], vocab[sp + "sat"], vocab[sp + "on"], vocab[sp + "the"],
        vocab[sp + "mat"]]
    # a character with no piece of its own falls back to its bytes
    assert tok.encode("é") == [vocab["<0xC3>"], vocab["<0xA9>"]]
    for text_ in ("the cat sat on the mat", "a dog and a hat", "héllo  wor ld "):
        assert tok.decode(tok.encode(text_)) == text_.encode()
    # decode leaves the special tokens out
    assert tok.decode([vocab["<bos>"], vocab["the"], vocab["<eos>"]]) == b"the"
