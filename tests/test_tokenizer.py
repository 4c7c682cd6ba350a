"""Tokenizer and chat template (script.js:175-200): the byte-level BPE of
tokenizer.py against the `tokenizers` library (the algorithm the reference's
@huggingface/transformers tokenizer runs) on a tokenizer.json in the Qwen2 layout
(tests/golden/tokenizer_toy.json, made by tests/golden/make_tokenizer.py)."""
import importlib
import os
import random

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
PATH = os.path.join(HERE, "golden", "tokenizer_toy.json")

CASES = [
    "", "hello", "Hello world!", "  leading and trailing  ", "tab\tseparated\tvalues", "line\nbreaks\n\n\nhere\r\n",
    "numbers 1234567 and 3.14159", "it's we'll they'd I'M YOU'RE", "données naïve Straße", "東京 数据 😀 emoji",
    "mixed-case CamelCaseWords and snake_case_words", "code: if (x == 1) { return y->z; }",
    "<|im_start|>user\nhi<|im_end|>", "text<|endoftext|>more", "<|im_end|><|im_start|>", "ñandú Ελλάδα москва",
    "   ", "\n", "a" * 50, "Ω ≈ ç √ ∫ ˜ µ ≤ ≥ ÷", "é (decomposed e-acute)",
]


@pytest.fixture(scope="module")
def pair(dllm):
    from tokenizers import Tokenizer
    tk = importlib.import_module("distributed-llm1_b200.tokenizer")
    return tk.Qwen2Tokenizer.from_file(PATH), Tokenizer.from_file(PATH), tk


@pytest.mark.parametrize("text", CASES)
def test_encode_matches_tokenizers_library(pair, text):
    mine, ref, _ = pair
    assert mine.encode(text) == ref.encode(text, add_special_tokens=False).ids


def test_encode_random_strings(pair):
    mine, ref, _ = pair
    rnd = random.Random(7)
    alphabet = "abcdeféèçñ東京 \n\t.,'!?0123456789😀<|>_-"
    for _ in range(300):
        s = "".join(rnd.choice(alphabet) for _ in range(rnd.randint(0, 40)))
        assert mine.encode(s) == ref.encode(s, add_special_tokens=False).ids, repr(s)


@pytest.mark.parametrize("text", CASES)
def test_decode_round_trip(pair, text):
    import unicodedata
    mine, ref, _ = pair
    ids = mine.encode(text)
    assert mine.decode(ids) == unicodedata.normalize("NFC", text)
    assert mine.decode(ids) == ref.decode(ids, skip_special_tokens=False)


def test_decode_skips_special_tokens_when_asked(pair):
    mine, ref, _ = pair
    ids = mine.encode("<|im_start|>assistant\nok<|im_end|>")
    assert mine.decode(ids, skip_special_tokens=True) == ref.decode(ids, skip_special_tokens=True) == "assistant\nok"


def test_decode_partial_utf8_is_replaced(pair):
    """A generated stream can stop inside a multi-byte character (script.js:188
    re-decodes the growing id list); the partial bytes decode as U+FFFD."""
    mine, _, _ = pair
    ids = mine.encode("東")
    assert len(ids) >= 2
    assert mine.decode(ids[:-1]).endswith("�")


def test_chat_template_matches_reference(pair):
    mine, ref, tk = pair
    s = tk.chat_template("What is 2+2?")
    assert s == ("<|im_start|>system\nYou are a helpful assistant.<|im_end|>\n<|im_start|>user\nWhat is 2+2?"
                 "<|im_end|>\n<|im_start|>assistant\n")  # script.js:198
    ids = mine.encode_chat("What is 2+2?")
    assert ids == ref.encode(s, add_special_tokens=False).ids
    assert ids[0] == 1001 and ids.count(1002) == 2  # <|im_start|> first, two <|im_end|>
