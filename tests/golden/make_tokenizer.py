"""Builds tests/golden/tokenizer_toy.json: a small byte-level BPE tokenizer in the
Hugging Face `tokenizer.json` layout of Qwen2 (NFC normaliser, the Qwen2
pre-tokenizer split regex + byte-level mapping, BPE without merges of special
tokens, byte-level decoder, <|endoftext|> <|im_start|> <|im_end|> as added special
tokens), trained with the `tokenizers` library on a seeded synthetic corpus. The
real Qwen2.5 tokenizer.json is not in this container; this file has the same
structure at 1/150 of the vocabulary, so tokenizer.py can be checked id for id
against the `tokenizers` library.

    python tests/golden/make_tokenizer.py
"""
import os
import random

from tokenizers import Regex, Tokenizer, decoders, models, normalizers, pre_tokenizers, trainers

HERE = os.path.dirname(os.path.abspath(__file__))
QWEN2_SPLIT = (r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+"
               r"|\s+(?!\S)|\s+")
SPECIAL = ["<|endoftext|>", "<|im_start|>", "<|im_end|>"]


def corpus(seed: int = 0, n: int = 4000):
    rnd = random.Random(seed)
    syll = ["ka", "lo", "mi", "ne", "ru", "ta", "shi", "qu", "ver", "ion", "ing", "the", "and", "of", "de", "la"]
    extra = ["données", "naïve", "Straße", "東京", "数据", "😀", "ñandú", "Ελλάδα", "москва"]
    punct = [".", ",", "!", "?", ":", ";", "(", ")", "\"", "'s", "'ll", "->", "==", "{", "}", "\n", "\n\n", "\t"]
    for _ in range(n):
        words = []
        for _ in range(rnd.randint(3, 14)):
            r = rnd.random()
            if r < 0.6:
                w = "".join(rnd.choice(syll) for _ in range(rnd.randint(1, 3)))
                words.append(w.capitalize() if rnd.random() < 0.2 else w)
            elif r < 0.75:
                words.append(str(rnd.randint(0, 99999)))
            elif r < 0.85:
                words.append(rnd.choice(extra))
            else:
                words.append(rnd.choice(punct))
        yield " ".join(words)


def main():
    tok = Tokenizer(models.BPE(unk_token=None, fuse_unk=False, byte_fallback=False))
    tok.normalizer = normalizers.NFC()
    tok.pre_tokenizer = pre_tokenizers.Sequence([
        pre_tokenizers.Split(Regex(QWEN2_SPLIT), behavior="isolated", invert=False),
        pre_tokenizers.ByteLevel(add_prefix_space=False, trim_offsets=False, use_regex=False)])
    tok.decoder = decoders.ByteLevel(add_prefix_space=False, trim_offsets=False, use_regex=False)
    trainer = trainers.BpeTrainer(vocab_size=1000, min_frequency=2, special_tokens=[],
                                  initial_alphabet=pre_tokenizers.ByteLevel.alphabet(), show_progress=False)
    tok.train_from_iterator(corpus(), trainer=trainer)
    tok.add_special_tokens(SPECIAL)
    tok.save(os.path.join(HERE, "tokenizer_toy.json"))


if __name__ == "__main__":
    main()
