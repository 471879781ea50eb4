"""The poll bridge over the device token loop, as the reference's bridge
tests drive it (apple/cpu_bridge/src/tests.rs): the Tiny-R model file
through aie_open, the greedy known answer [41, 53, 41, 50] with a
cancellation and resume in the middle, stop, reset, admission rejections,
stale ids, the text poll, cancellation before admission, and a numerical
failure after the KV write.  A Qwen2 directory source decodes like the same
checkpoint loaded directly."""
import ctypes as C
import json

import numpy as np
import pytest

from helpers import bridge_event, bridge_open, bridge_wait, ev_tuple, small_qwen_checkpoint, tiny_model_json

pytestmark = pytest.mark.gpu

OK, PENDING, INVALID_INPUT, INVALID_HANDLE, BUSY, CANCELLED, MODEL_FAILED, EXECUTION_FAILED, PANIC, CLOSED = range(10)
READY, STARTED, TOKEN, STOPPED, CANCEL_EVENT, RESET_EVENT, ERROR = range(1, 8)
NONE = 0xFFFFFFFF


def _L():
    from llm_inference_edu_b200._lib import lib
    return lib()


def _ready(source=None, kind=0):
    st, h = bridge_open(source if source is not None else tiny_model_json(), kind)
    assert st == OK
    ev = bridge_wait(h)
    assert (ev.kind, ev.code) == (READY, OK), ev_tuple(ev)
    return h


def _ids(*v):
    return (C.c_uint32 * len(v))(*v)


def test_known_answer_cancel_resume_reset_and_stale_ids():
    # tests.rs:76-135
    L = _L()
    h = _ready()
    prompt = _ids(1, 5, 7)
    assert L.aie_begin_ids(h, prompt, 3, 4) == OK
    assert L.aie_next(h) == BUSY  # one command, one event
    ev = bridge_wait(h)
    assert (ev.kind, ev.processed, ev.history) == (STARTED, 3, 3)
    for index, expected in enumerate([41, 53, 41, 50]):
        if index == 1:
            assert L.aie_set_cancel(h, 1) == OK
            assert L.aie_next(h) == OK
            ev = bridge_wait(h)
            assert (ev.kind, ev.code, ev.processed, ev.history) == (CANCEL_EVENT, CANCELLED, 3, 4)
            assert L.aie_set_cancel(h, 0) == OK
        assert L.aie_next(h) == OK
        ev = bridge_wait(h)
        assert (ev.kind, ev.token) == (TOKEN, expected)
        assert (ev.processed, ev.history) == (3 + index, 4 + index)
    assert L.aie_next(h) == OK
    assert bridge_wait(h).kind == STOPPED
    assert L.aie_reset(h) == OK
    ev = bridge_wait(h)
    assert (ev.kind, ev.history, ev.processed) == (RESET_EVENT, 0, 0)
    assert L.aie_begin_ids(h, _ids(64), 1, 4) == OK  # out of the vocabulary: rejected on the worker
    ev = bridge_wait(h)
    assert (ev.kind, ev.code, ev.history, ev.processed) == (ERROR, INVALID_INPUT, 0, 0)
    assert L.aie_begin_ids(h, _ids(1, 2), 2, 31) == OK  # 2 + 31 > 32 positions
    assert bridge_wait(h).code == INVALID_INPUT
    assert L.aie_begin_text(h, b"hello", 5, 4) == OK  # no tokenizer: refused as for tiny models
    assert bridge_wait(h).code == INVALID_INPUT
    assert L.aie_begin_ids(h, prompt, 3, 4) == OK
    assert bridge_wait(h).kind == STARTED
    assert L.aie_begin_ids(h, prompt, 3, 4) == OK  # history not empty: reset first
    assert bridge_wait(h).code == INVALID_INPUT
    assert L.aie_close(h) == OK
    assert L.aie_next(h) == INVALID_HANDLE and L.aie_close(h) == INVALID_HANDLE
    fresh = _ready()
    assert fresh != h
    assert L.aie_close(fresh) == OK


def test_single_worker_and_bad_buffers_do_not_consume_events():
    # tests.rs:136-157
    L = _L()
    h = _ready()
    other = C.c_uint64(99)
    src = tiny_model_json()
    assert L.aie_open(0, src, len(src), C.byref(other)) == BUSY
    assert other.value == 99
    assert L.aie_begin_ids(h, None, 1, 4) == INVALID_INPUT
    assert L.aie_poll(h, None) == INVALID_INPUT
    assert L.aie_reset(h) == OK
    assert L.aie_poll(h, None) == INVALID_INPUT
    assert bridge_wait(h).kind == RESET_EVENT
    assert L.aie_close(h) == OK


def test_text_poll_is_atomic_and_bounded():
    # tests.rs:258-298
    L = _L()
    h = _ready()
    assert L.aie_begin_ids(h, _ids(1, 5, 7), 3, 4) == OK
    assert bridge_wait(h).kind == STARTED
    assert L.aie_next(h) == OK
    out, length = bridge_event(), C.c_size_t(99)
    text = (C.c_uint8 * 4096)(*([99] * 4096))
    assert L.aie_poll_text(h, C.byref(out), text, 4095, C.byref(length)) == INVALID_INPUT
    assert ev_tuple(out) == (99,) * 5 and length.value == 99
    import time
    deadline = time.monotonic() + 20
    while True:
        st = L.aie_poll_text(h, C.byref(out), text, 4096, C.byref(length))
        if st == OK:
            break
        assert st == PENDING and length.value == 99 and list(text) == [99] * 4096
        assert time.monotonic() < deadline
        time.sleep(0.001)
    assert out.token == 41
    assert bytes(text[:length.value]) == b"41 "
    assert all(b == 99 for b in text[length.value:])
    assert L.aie_close(h) == OK


def test_cancellation_before_admission_can_clear_and_retry():
    # tests.rs:299-319
    L = _L()
    h = _ready()
    assert L.aie_set_cancel(h, 1) == OK
    assert L.aie_begin_ids(h, _ids(1, 5, 7), 3, 4) == OK
    ev = bridge_wait(h)
    assert (ev.kind, ev.code, ev.processed, ev.history) == (CANCEL_EVENT, CANCELLED, 0, 0)
    assert L.aie_set_cancel(h, 0) == OK
    assert L.aie_begin_ids(h, _ids(1, 5, 7), 3, 4) == OK
    ev = bridge_wait(h)
    assert (ev.kind, ev.processed, ev.history) == (STARTED, 3, 3)
    assert L.aie_close(h) == OK


def test_failure_after_the_kv_write_leaves_no_valid_prefix():
    # tests.rs:222-257: Q and K zero, V the identity, down at the float
    # maximum so the FFN overflows after the KV write; the session
    # invalidates, the worker is terminal.
    L = _L()
    fmax = float(np.finfo(np.float32).max)
    src = json.dumps({
        "config": {"vocab_size": 2, "layers": 1, "hidden_dim": 2, "query_heads": 1, "kv_heads": 1,
                   "head_dim": 2, "ff_dim": 2, "max_tokens": 2, "rope_base": 10000.0, "norm_epsilon": 1e-5},
        "weights": {"embedding": [0.0, 0.0, 1.0, 1.0], "final_norm": [1.0, 1.0], "layers": [{
            "attention_norm": [1.0, 1.0], "query": [0.0] * 4, "key": [0.0] * 4, "value": [1.0, 0.0, 0.0, 1.0],
            "attention_output": [0.0] * 4, "ffn_norm": [1.0, 1.0], "gate": [1.0] * 4, "up": [1.0] * 4,
            "down": [fmax] * 4}]}}).encode()
    h = _ready(src)
    assert L.aie_begin_ids(h, _ids(1), 1, 1) == OK
    ev = bridge_wait(h)
    assert (ev.kind, ev.code, ev.processed, ev.history) == (ERROR, EXECUTION_FAILED, 0, 1)
    assert L.aie_next(h) == EXECUTION_FAILED and L.aie_reset(h) == EXECUTION_FAILED
    assert L.aie_close(h) == OK


def test_qwen_directory_source_with_tokenizer(tmp_path):
    # Source kind 1 (src/worker.rs:85-99): config.json and model.safetensors
    # of a small Qwen2 checkpoint with the vocabulary of its chat tokenizer
    # (151,646 ids), and the tokenizer's three files.  A text prompt is
    # encoded on the worker; the greedy ids equal those of the same file
    # loaded directly (token by token, as the worker evaluates a prompt it
    # may cancel); each token event carries the stream decoder's text.
    import llm_inference_edu_b200 as qb
    from helpers import chat_tokenizer_files
    L = _L()
    hf, _cfg, _w, data = small_qwen_checkpoint(seed=9, vocab=151646)
    (tmp_path / "config.json").write_text(json.dumps(hf))
    (tmp_path / "model.safetensors").write_bytes(data)
    chat_tokenizer_files(tmp_path)
    tok = qb.Tokenizer.load(tmp_path)
    prompt = tok.encode("Hello!")
    assert 0 < len(prompt) <= 5
    m = qb.Decoder.from_safetensors(data, hf)
    s = qb.CachedSession(m, 32)
    for t in prompt:
        lg = s.step(t)
    want = [int(np.argmax(lg))]
    for _ in range(2):
        want.append(int(np.argmax(s.step(want[-1]))))
    stream = tok.text_stream()
    texts = [stream.push(t) or "" for t in want]
    h = _ready(str(tmp_path).encode(), kind=1)
    assert L.aie_begin_text(h, b"Hello! Hello! Hello!", 20, 3) == OK  # more than 8 positions
    assert bridge_wait(h).code == INVALID_INPUT
    assert L.aie_begin_text(h, b"Hello!", 6, 3) == OK
    ev = bridge_wait(h)
    assert (ev.kind, ev.processed, ev.history) == (STARTED, len(prompt), len(prompt))
    out, length = bridge_event(), C.c_size_t()
    text = (C.c_uint8 * 4096)()
    import time
    for k in range(3):
        assert L.aie_next(h) == OK
        deadline = time.monotonic() + 20
        while (st := L.aie_poll_text(h, C.byref(out), text, 4096, C.byref(length))) == PENDING:
            assert time.monotonic() < deadline
            time.sleep(0.001)
        assert st == OK and out.kind == TOKEN and out.token == want[k]
        assert bytes(text[:length.value]).decode() == texts[k]
    assert L.aie_next(h) == OK
    assert bridge_wait(h).kind == STOPPED
    assert L.aie_close(h) == OK
    # Without the tokenizer's files the source does not load (the reference
    # loads its tokenizer with the weights).
    bare = tmp_path / "bare"
    bare.mkdir()
    (bare / "config.json").write_text(json.dumps(hf))
    (bare / "model.safetensors").write_bytes(data)
    st, bad = bridge_open(str(bare).encode(), kind=1)
    assert st == OK and bridge_wait(bad).code == MODEL_FAILED
    assert L.aie_close(bad) == OK
