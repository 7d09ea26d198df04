"""C++ byte-level BPE tokenizer, chat templates and streaming detokenizer.

The tokenizer is checked token-for-token against the HF `tokenizers` library on a small
byte-level BPE trained here with the Qwen2 pre-tokenizer split rule."""

import json
import os
import random

import pytest

from zstep_b200 import _master as M

QWEN2_SPLIT = (r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*|"
               r"\s*[\r\n]+|\s+(?!\S)|\s+")

CORPUS = ["The quick brown fox jumps over the lazy dog. " * 3, "Hello, world! 12345 it's we're they'll",
          "def f(x):\n    return x*2\n\n", "Καλημέρα κόσμε — 你好，世界！ こんにちは", "naïve café résumé 😀 🚀",
          "SELECT * FROM t WHERE a >= 10 AND b <> 'x';\n", "   indented\n\t\ttabs\r\nwindows"] * 40


def build_hf_tokenizer(path: str):
    tokenizers = pytest.importorskip("tokenizers")
    from tokenizers import Regex, decoders, models, pre_tokenizers, trainers

    tok = tokenizers.Tokenizer(models.BPE())
    tok.pre_tokenizer = pre_tokenizers.Sequence([
        pre_tokenizers.Split(Regex(QWEN2_SPLIT), behavior="isolated", invert=False),
        pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)])
    tok.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=700, special_tokens=["<|endoftext|>", "<|im_start|>", "<|im_end|>"],
                                  initial_alphabet=pre_tokenizers.ByteLevel.alphabet(), show_progress=False)
    tok.train_from_iterator(CORPUS, trainer)
    tok.add_tokens(["<think>", "</think>"])
    tok.save(os.path.join(path, "tokenizer.json"))
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump({"eos_token_id": [tok.token_to_id("<|im_end|>"), tok.token_to_id("<|endoftext|>")]}, f)
    return tok


@pytest.fixture(scope="module")
def toks(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("tok"))
    hf = build_hf_tokenizer(d)
    t = M.Tokenizer()
    t.load_dir(d)
    return hf, t, d


SAMPLES = ["Hello, world! it's 2024\n\n  ok", "def f(x):\n    return x*2\n\n", "Καλημέρα κόσμε — 你好，世界！",
           "naïve café 😀 🚀", "<|im_start|>user\nhi<|im_end|>\n", "   leading\t\ttabs\r\n crlf", "I'M HERE, YOU'RE",
           "a1b2c3 4567", "   ", "\n\n\n", "x  \n  y", "!!!???...", "<think>\nreason</think>\n\nanswer", ""]


def test_encode_matches_hf(toks):
    hf, t, _ = toks
    for s in SAMPLES:
        assert t.encode(s) == hf.encode(s).ids, s


def test_encode_fuzz_matches_hf(toks):
    hf, t, _ = toks
    rng = random.Random(0)
    alphabet = list("abcXYZ019 \t\n\r.,;:'\"!?-_()[]{}<>/\\") + ["é", "ß", "Ω", "ж", "你", "の", "😀", "—", " ", "²"]
    for _ in range(300):
        s = "".join(rng.choice(alphabet) for _ in range(rng.randint(1, 40)))
        assert t.encode(s) == hf.encode(s).ids, repr(s)


def test_decode_roundtrip_and_specials(toks):
    hf, t, _ = toks
    for s in SAMPLES:
        ids = t.encode(s)
        assert t.decode(ids, False) == s.encode()
    im_end = t.token_id("<|im_end|>")
    assert t.is_special(im_end)
    assert t.decode([im_end], True) == b""
    assert sorted(t.eos_ids()) == sorted([hf.token_to_id("<|im_end|>"), hf.token_to_id("<|endoftext|>")])


def test_chatml_template():
    p = M.render_chat([("system", "be brief", ""), ("user", "hi", ""), ("assistant", "hello", "thought"),
                       ("user", "again", "")])
    assert p == ("<|im_start|>system\nbe brief<|im_end|>\n<|im_start|>user\nhi<|im_end|>\n"
                 "<|im_start|>assistant\n<think>\nthought\n</think>\n\nhello<|im_end|>\n"
                 "<|im_start|>user\nagain<|im_end|>\n<|im_start|>assistant\n")
    assert M.render_chat([("user", "q", "")], thinking=True).endswith("<|im_start|>assistant\n<think>\n")
    with pytest.raises(ValueError):
        M.render_chat([("tool", "x", "")])


def test_deepseek_template():
    p = M.render_chat([("system", "sys", ""), ("user", "hi", "")], format="deepseek")
    assert p == "<｜begin▁of▁sentence｜>sys<｜User｜>hi<｜Assistant｜></think>"
    p = M.render_chat([("user", "hi", ""), ("assistant", "yo", ""), ("user", "more", "")], format="deepseek",
                      thinking=True)
    assert p == ("<｜begin▁of▁sentence｜><｜User｜>hi<｜Assistant｜></think>yo<｜end▁of▁sentence｜>"
                 "<｜User｜>more<｜Assistant｜><think>")


def test_stream_decoder_utf8_and_stop(toks):
    _, t, _ = toks
    text = "你好 world STOP here"
    ids = t.encode(text)
    # Without stop strings the concatenated deltas equal the full decode, every delta is valid UTF-8.
    d = M.StreamDecoder(t, [])
    out = b""
    for i in ids:
        piece = d.push(i)
        piece.decode("utf-8")
        out += piece
    out += d.finish()
    assert out == text.encode()
    # A stop string spanning several tokens cuts the text right before it.
    d = M.StreamDecoder(t, ["STOP"])
    out = b""
    for i in ids:
        out += d.push(i)
        if d.stopped():
            break
    assert d.stopped() and out == "你好 world ".encode()


def test_pre_split_rules():
    parts = [p.decode() for p in M.Tokenizer.pre_split("it's  Hello 123\n\n x")]
    assert parts == ["it", "'s", " ", " Hello", " ", "1", "2", "3", "\n\n", " x"]
