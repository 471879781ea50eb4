"""Regenerates tests/golden/tokenizer-synthetic.json and
tests/golden/tokenizer-cases.json with HF `tokenizers` (the library the
reference pins, Cargo.toml: tokenizers 0.21.4; this image has 0.22.2).

    python tests/golden/make_tokenizer_golden.py

The real Qwen2 vocabulary is not in this image, so a small byte-level BPE
is trained here in the Qwen2 configuration: NFC normalizer, the Qwen2 split
pattern (Isolated) then ByteLevel without prefix space or regex, the
ByteLevel decoder, and <|endoftext|>, <|im_start|>, <|im_end|> as special
tokens after the vocabulary (Qwen's file has them there too: ids
151643-151645 after its 151,643 vocabulary entries).  The corpus is generated below (words
built from seeded syllables in several scripts); no dataset is used.  The
cases record HF's encode (no special tokens added), decode with and without
special tokens, and the DecodeStream chunks of every case.
"""
import json
import os
import random

from tokenizers import Regex, Tokenizer, decoders, models, normalizers, pre_tokenizers, trainers

HERE = os.path.dirname(os.path.abspath(__file__))
PATTERN = (r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*|"
           r"\s*[\r\n]+|\s+(?!\S)|\s+")
SPECIALS = [("<|endoftext|>", 151643), ("<|im_start|>", 151644), ("<|im_end|>", 151645)]


def corpus(seed=11, lines=4000):
    rng = random.Random(seed)
    syll = {
        "latin": ["ka", "to", "re", "ve", "an", "the", "in", "on", "ing", "er", "st", "qu", "ll", "ou", "é", "ü", "ñ"],
        "cyr": ["при", "вет", "ма", "ло", "ко", "ни", "ра", "ст"],
        "cjk": ["世", "界", "你", "好", "学", "生", "中", "文"],
        "greek": ["κα", "λη", "με", "ρα", "σο", "φι"],
    }
    punct = [".", ",", "!", "?", ";", ":", "'s", "'t", "'re", "'ll", "'ve", "'d", "'m", "(", ")", "-", "—", "…",
             "🙂", "🌍", "#", "$", "%"]
    out = []
    for _ in range(lines):
        words = []
        for _ in range(rng.randint(3, 14)):
            script = rng.choice(list(syll))
            w = "".join(rng.choice(syll[script]) for _ in range(rng.randint(1, 4)))
            if rng.random() < 0.2:
                w = w.capitalize()
            if rng.random() < 0.1:
                w = str(rng.randint(0, 99999))
            words.append(w)
            if rng.random() < 0.2:
                words.append(rng.choice(punct))
        sep = rng.choice([" ", " ", " ", "  ", "\t", "\n", " \n", "\r\n"])
        out.append(sep.join(words))
    return out


CASES = [
    "Hello!", "Rust is", "  a\t b\n", "Привет 🌍 café", "世界🙂", "", "It's THEY'RE we'LL you'Ve I'M he'D",
    "tab\there  two   spaces\n\n\nthree newlines \r\n crlf", "trailing spaces   ", "   leading", "x\n  \n  y",
    "numbers 12345 and 3.14159, ١٢٣ ½", "é vs é and 각 hangul jamo", "Å̊ ẋ̣",
    "<|im_start|>user\nx<|im_end|>\n", "a<|endoftext|>b<|im_end|><|im_start|>", "!!! ??? ... —— …",
    "emoji 👩‍💻 and flags 🇫🇷", "mixed καλημέρα and приветмир", "ǅemo Ǆ ǆ", "ſt 'ſ 'S", " nbsp　ideo",
    "line sep para\u0085nel", "#hashtag $dollar %percent @at", "trailing newline\n",
]


def main():
    tok = Tokenizer(models.BPE())
    tok.normalizer = normalizers.NFC()
    tok.pre_tokenizer = pre_tokenizers.Sequence([
        pre_tokenizers.Split(Regex(PATTERN), behavior="isolated", invert=False),
        pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)])
    tok.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=1400, initial_alphabet=pre_tokenizers.ByteLevel.alphabet(),
                                  show_progress=False)
    tok.train_from_iterator(corpus(), trainer)
    n = tok.get_vocab_size()
    tok.add_special_tokens([c for c, _ in SPECIALS])  # ids n, n + 1, n + 2
    text = tok.to_str()
    for k, (c, _) in enumerate(SPECIALS):
        assert tok.token_to_id(c) == n + k, c
    cases = []
    for t in CASES:
        ids = tok.encode(t, add_special_tokens=False).ids
        stream = decoders.DecodeStream(skip_special_tokens=True)
        chunks = []
        for i in ids:
            out = stream.step(tok, i)
            chunks.append(out)
        cases.append({"text": t, "ids": ids, "decoded": tok.decode(ids, skip_special_tokens=False),
                      "decoded_skip": tok.decode(ids, skip_special_tokens=True), "stream": chunks})
    # Byte-level tokens that split UTF-8 sequences, decoded alone and streamed.
    raw = [tok.token_to_id(c) for c in ("Ã", "©", "x") if tok.token_to_id(c) is not None]
    with open(os.path.join(HERE, "tokenizer-synthetic.json"), "w") as f:
        f.write(text)
    with open(os.path.join(HERE, "tokenizer-cases.json"), "w") as f:
        json.dump({"tokenizers_version": __import__("tokenizers").__version__, "cases": cases,
                   "split_ids": raw, "split_decoded": tok.decode(raw), "split_stream":
                   [decoders.DecodeStream(skip_special_tokens=True).step(tok, i) for i in raw[:1]]},
                  f, ensure_ascii=False, indent=1)


if __name__ == "__main__":
    main()
