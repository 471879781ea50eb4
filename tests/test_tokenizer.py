"""The host tokenizer and chat template (src/tokenizer.rs) on the CPU:

* golden vectors from HF `tokenizers` (the library the reference pins) on a
  synthetic byte-level BPE in the Qwen2 configuration
  (tests/golden/make_tokenizer_golden.py): encode, decode with and without
  special tokens, and the stream's chunks, for ASCII, whitespace runs,
  contractions in every case, numbers, combining marks (NFC), Hangul,
  Cyrillic, CJK, emoji and inline special tokens;
* the reference's own stream test (src/tokenizer.rs:215-246) restated on
  that tokenizer's byte tokens;
* render_chat against the reference's chat fixture (fixtures/t06, the
  texts; its ids need the Qwen vocabulary, which is not in this image);
* ChatTokenizer::load's checks of the three files."""
import json
import os

import pytest

from conftest import GOLDEN, golden
from helpers import chat_tokenizer_files

SYN = os.path.join(GOLDEN, "tokenizer-synthetic.json")


def _tok():
    import llm_inference_edu_b200 as qb
    return qb.Tokenizer.from_json(open(SYN, "rb").read())


def test_encode_decode_and_stream_match_hf_tokenizers():
    t = _tok()
    g = golden("tokenizer-cases.json")
    for case in g["cases"]:
        ids = t.encode(case["text"])
        assert ids == case["ids"], case["text"]
        assert t.decode(ids, False) == case["decoded"], case["text"]
        assert t.decode(ids, True) == case["decoded_skip"], case["text"]
        s = t.text_stream()
        assert [s.push(i) for i in ids] == case["stream"], case["text"]


def test_byte_tokens_stream_until_complete_and_specials_are_hidden():
    # src/tokenizer.rs:215-246 with the byte tokens of "é" split across two
    # ids ("Ã", "©"), then "x", an unknown id and a special token.
    import llm_inference_edu_b200 as qb
    t = _tok()
    g = golden("tokenizer-cases.json")
    a, b, x = g["split_ids"]
    stop = t.encode("<|endoftext|>")
    assert len(stop) == 1
    s = t.text_stream()
    assert s.push(a) is None and s.pending_tokens() == 1
    with pytest.raises(qb.TokenizerError) as e:
        s.push(999999)
    assert e.value.kind == "InvalidToken" and e.value.actual == 999999
    assert s.pending_tokens() == 1
    assert s.push(b) == "é" and s.pending_tokens() == 0
    assert s.push(x) == "x"
    assert s.push(stop[0]) is None and s.pending_tokens() == 0
    assert t.decode([a, b, x, stop[0]], True) == "éx" == g["split_decoded"]
    assert t.decode([a, b, x, stop[0]], False) == "éx<|endoftext|>"
    with pytest.raises(qb.TokenizerError) as e:
        t.decode([5, 4242424], False)
    assert e.value.kind == "InvalidToken"


def test_round_trip_of_the_reference_fixture_texts():
    # Byte-level BPE is lossless: every t06 text (non-Latin scripts, emoji,
    # tabs, special tokens) decodes back to itself.
    t = _tok()
    fx = golden("t06-tokenizer.json")
    for case in fx["cases"]:
        assert t.decode(t.encode(case["text"]), False) == case["text"]
    for chat in fx["chats"]:
        assert t.decode(t.encode(chat["text"]), False) == chat["text"]


def test_render_chat_matches_the_reference_fixture():
    # fixtures/t06-tokenizer.json "chats": the rendered text of each.
    import llm_inference_edu_b200 as qb
    roles = {"system": qb.Role.System, "user": qb.Role.User, "assistant": qb.Role.Assistant}
    fx = golden("t06-tokenizer.json")
    assert fx["chats"]
    for chat in fx["chats"]:
        msgs = [(roles[m["role"]], m["content"]) for m in chat["messages"]]
        assert qb.render_chat(msgs, chat["generation_prompt"]) == chat["text"]
    with pytest.raises(qb.TokenizerError) as e:
        qb.render_chat([], True)
    assert e.value.kind == "EmptyMessages"


def test_chat_tokenizer_load_checks(tmp_path):
    # src/tokenizer.rs:68-124
    import llm_inference_edu_b200 as qb
    ok = tmp_path / "ok"
    ok.mkdir()
    t = qb.Tokenizer.load(chat_tokenizer_files(ok))
    assert t.stop_tokens() == [151645, 151643]
    assert t.encode("<|im_start|>user\nx<|im_end|>\n")[0] == 151644
    assert t.encode("<|im_start|>user\nx<|im_end|>\n")[-2] == 151645
    for k, over in enumerate([{"cfg": {"tokenizer_class": "GPT2Tokenizer"}}, {"cfg": {"add_bos_token": True}},
                              {"cfg": {"bos_token": "<s>"}}, {"cfg": {"eos_token": "<|endoftext|>"}},
                              {"gen": {"eos_token_id": [151645]}}, {"gen": {"eos_token_id": 151645}}]):
        d = tmp_path / f"bad{k}"
        d.mkdir()
        with pytest.raises(qb.TokenizerError) as e:
            qb.Tokenizer.load(chat_tokenizer_files(d, **over))
        assert e.value.kind == "UnsupportedAssets", over
    d = tmp_path / "json"
    d.mkdir()
    chat_tokenizer_files(d)
    (d / "tokenizer.json").write_text("{not json")
    with pytest.raises(qb.TokenizerError) as e:
        qb.Tokenizer.load(d)
    assert e.value.kind == "Json"


def test_unsupported_configurations_and_bad_text():
    import llm_inference_edu_b200 as qb
    doc = json.loads(open(SYN, encoding="utf-8").read())
    for mutate in [lambda d: d["model"].update(byte_fallback=True),
                   lambda d: d.update(normalizer={"type": "NFKC"}),
                   lambda d: d["pre_tokenizer"]["pretokenizers"][0]["pattern"].update(Regex="\\s+"),
                   lambda d: d.update(decoder={"type": "Metaspace"}),
                   lambda d: d["added_tokens"][0].update(lstrip=True)]:
        bad = json.loads(json.dumps(doc))
        mutate(bad)
        with pytest.raises(qb.TokenizerError) as e:
            qb.Tokenizer.from_json(json.dumps(bad).encode())
        assert e.value.kind == "UnsupportedAssets"
    from llm_inference_edu_b200._lib import lib
    import ctypes as C
    t = _tok()
    n = C.c_size_t()
    assert lib().qb_tokenizer_encode(t.handle, b"\xff", 1, None, 0, C.byref(n)) == 46  # Encoding
    assert lib().qb_tokenizer_encode(t.handle, b"Hello!", 6, None, 0, C.byref(n)) == 20 and n.value == 5


def test_random_texts_match_hf_tokenizers():
    # Differential check against the library the reference wraps, on 600
    # seeded random strings drawn from every class the split pattern and NFC
    # distinguish: letters of several scripts (with case), digits and other
    # numbers, combining marks in both orders, Hangul jamo, spaces, tabs,
    # newlines and other Unicode whitespace, apostrophe contractions,
    # symbols, emoji and the special tokens.
    tokenizers = pytest.importorskip("tokenizers")
    import random
    hf = tokenizers.Tokenizer.from_file(SYN)
    t = _tok()
    pool = (list("abcXYZ") + list("éüñÅ") + list("приВЕТ") + list("世界中") + list("καλΩ") + list("0123")
            + ["٣", "½", "Ⅷ"] + ["́", "̈", "̣", "̇", "̊"]
            + ["ᄀ", "ᅡ", "ᆨ", "각"] + [" ", " ", "  ", "\t", "\n", "\r\n", " ", "　",
                                                          " ", "\u0085"]
            + ["'s", "'T", "'re", "'VE", "'m", "'LL", "'d", "'ſ", "'"] + list("!?.,;:-()#$%&*+/<=>@[]^_`{|}~")
            + ["🙂", "🌍", "👩‍💻", "‍"] + ["<|im_start|>", "<|im_end|>", "<|endoftext|>", "<|im_"])
    rng = random.Random(1234)
    for k in range(600):
        text = "".join(rng.choice(pool) for _ in range(rng.randint(0, 24)))
        want = hf.encode(text, add_special_tokens=False).ids
        got = t.encode(text)
        assert got == want, (k, text)
        assert t.decode(got, False) == hf.decode(want, skip_special_tokens=False), (k, text)
        assert t.decode(got, True) == hf.decode(want, skip_special_tokens=True), (k, text)
        ds, s = tokenizers.decoders.DecodeStream(skip_special_tokens=True), t.text_stream()
        assert [s.push(i) for i in got] == [ds.step(hf, i) for i in want], (k, text)


def test_long_word_matches_hf_tokenizers():
    # One 64,000-character word (the bridge admits 64 KiB of text): the merge
    # order over a long symbol list equals the library's, in linearithmic
    # time.
    tokenizers = pytest.importorskip("tokenizers")
    import random
    hf = tokenizers.Tokenizer.from_file(SYN)
    t = _tok()
    rng = random.Random(3)
    word = "".join(rng.choice("abcdefghijklmnopqrstuvwxyzéñ") for _ in range(64000))
    assert t.encode(word) == hf.encode(word, add_special_tokens=False).ids
