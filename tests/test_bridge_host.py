"""The poll bridge's host side (apple/cpu_bridge/src/tests.rs), on the CPU:
ABI layout, admission that writes nothing on error, a model source that
fails on the worker, and single-worker admission.  Nothing here touches a
GPU: a source that is not a model fails while it is parsed."""
import ctypes as C

from helpers import bridge_event, bridge_open, bridge_wait, ev_tuple
from llm_inference_edu_b200._lib import AieEvent, lib

OK, PENDING, INVALID_INPUT, INVALID_HANDLE, BUSY, CANCELLED, MODEL_FAILED, EXECUTION_FAILED, PANIC, CLOSED = range(10)
READY, STARTED, TOKEN, STOPPED, CANCEL_EVENT, RESET_EVENT, ERROR = range(1, 8)


def test_abi_layout_and_pre_admission_outputs_are_preserved():
    # tests.rs:48-75
    L = lib()
    assert L.aie_abi_version() == 2
    assert C.sizeof(AieEvent) == 20 and C.alignment(AieEvent) == 4
    h = C.c_uint64(99)
    assert L.aie_open(0, None, 1, C.byref(h)) == INVALID_INPUT
    assert L.aie_open(0, b"{}", 2**64 - 1, C.byref(h)) == INVALID_INPUT
    assert L.aie_open(2, b"{}", 2, C.byref(h)) == INVALID_INPUT
    assert L.aie_open(0, b"{}", 0, C.byref(h)) == INVALID_INPUT
    assert L.aie_open(1, b"bad\x00path", 8, C.byref(h)) == INVALID_INPUT
    assert L.aie_open(1, b"\xff\xfe", 2, C.byref(h)) == INVALID_INPUT
    assert L.aie_open(0, b"{}", 2, None) == INVALID_INPUT
    assert h.value == 99
    out = bridge_event()
    assert L.aie_poll(0, C.byref(out)) == INVALID_HANDLE
    assert ev_tuple(out) == (99,) * 5
    assert L.aie_close(0) == INVALID_HANDLE
    assert L.aie_set_cancel(0, 1) == INVALID_HANDLE
    assert L.aie_set_cancel(0, 2) == INVALID_INPUT


def test_buffer_checks_come_before_the_handle():
    # aie_begin_ids / aie_begin_text check their buffers first (src/lib.rs:206-247).
    L = lib()
    ids = (C.c_uint32 * 3)(1, 5, 7)
    assert L.aie_begin_ids(12345, None, 1, 4) == INVALID_INPUT
    assert L.aie_begin_ids(12345, ids, 0, 4) == INVALID_INPUT
    assert L.aie_begin_ids(12345, ids, 33, 4) == INVALID_INPUT
    assert L.aie_begin_ids(12345, ids, 3, 0) == INVALID_INPUT
    assert L.aie_begin_ids(12345, ids, 3, 32) == INVALID_INPUT
    assert L.aie_begin_ids(12345, C.cast(C.addressof(ids) + 1, C.c_void_p), 1, 4) == INVALID_INPUT  # misaligned
    assert L.aie_begin_ids(12345, ids, 3, 4) == INVALID_HANDLE
    assert L.aie_begin_text(12345, b"\xc3\x28", 2, 4) == INVALID_INPUT  # not UTF-8
    assert L.aie_begin_text(12345, b"hi", 2, 4) == INVALID_HANDLE
    assert L.aie_next(12345) == INVALID_HANDLE and L.aie_reset(12345) == INVALID_HANDLE


def test_initialization_failure_is_terminal_and_admission_is_single_worker():
    # tests.rs:158-178 (first half) and 136-157: the worker's failure event,
    # then every command is EXECUTION_FAILED; while the handle is open no
    # second worker is admitted and the output is untouched.
    L = lib()
    st, h = bridge_open(b"not model JSON")
    assert st == OK
    ev = bridge_wait(h)
    assert (ev.kind, ev.code, ev.token, ev.processed, ev.history) == (ERROR, MODEL_FAILED, 0xFFFFFFFF, 0, 0)
    assert L.aie_next(h) == EXECUTION_FAILED and L.aie_reset(h) == EXECUTION_FAILED
    other = C.c_uint64(99)
    assert L.aie_open(0, b"{}", 2, C.byref(other)) == BUSY
    assert other.value == 99
    out = bridge_event()
    assert L.aie_poll(h, None) == INVALID_INPUT
    assert L.aie_poll(h, C.byref(out)) == CLOSED  # the worker is gone and its event was taken
    assert L.aie_close(h) == OK
    assert L.aie_close(h) == INVALID_HANDLE
    # A model file with an unknown field is refused as the reference's
    # deny_unknown_fields refuses it; ids are never reused.
    st, h2 = bridge_open(b'{"config": {}, "weights": {}, "extra": 1}')
    assert st == OK and h2 != h
    assert bridge_wait(h2).code == MODEL_FAILED
    assert L.aie_close(h2) == OK


def test_poll_text_checks_its_outputs_first():
    # tests.rs:258-298: a wrong capacity writes nothing and consumes no event.
    L = lib()
    st, h = bridge_open(b"[1, 2")
    assert st == OK
    out, length = bridge_event(), C.c_size_t(99)
    text = (C.c_uint8 * 4096)(*([99] * 4096))
    assert L.aie_poll_text(h, C.byref(out), text, 4095, C.byref(length)) == INVALID_INPUT
    assert L.aie_poll_text(h, C.byref(out), None, 4096, C.byref(length)) == INVALID_INPUT
    assert ev_tuple(out) == (99,) * 5 and length.value == 99 and list(text) == [99] * 4096
    ev = bridge_wait(h)  # the event is still there
    assert ev.code == MODEL_FAILED
    assert L.aie_close(h) == OK


def test_qwen_directory_without_files_fails_on_the_worker(tmp_path):
    # Source kind 1 reads config.json, model.safetensors and the tokenizer's
    # files on the worker; a directory without them is AIE_MODEL_FAILED
    # (src/worker.rs:85-104), decided before any device work.
    L = lib()
    st, h = bridge_open(str(tmp_path / "absent").encode(), kind=1)
    assert st == OK
    ev = bridge_wait(h)
    assert (ev.kind, ev.code) == (ERROR, MODEL_FAILED)
    assert L.aie_begin_text(h, b"hi", 2, 4) == EXECUTION_FAILED
    assert L.aie_close(h) == OK
    (tmp_path / "config.json").write_text('{"model_type": "qwen2"}')
    st, h = bridge_open(str(tmp_path).encode(), kind=1)
    assert st == OK and bridge_wait(h).code == MODEL_FAILED
    assert L.aie_close(h) == OK


def test_malformed_model_files_fail_on_the_worker():
    # Decoder::from_json's serde rules (src/model.rs:185-189): exact fields,
    # integer sizes, arrays of numbers, no trailing content.  Each of these
    # files is refused on the worker (AIE_MODEL_FAILED); all but the one with
    # non-numeric weights fail while the file is read, before any device work.
    import json
    good_cfg = {"vocab_size": 2, "layers": 1, "hidden_dim": 2, "query_heads": 1, "kv_heads": 1, "head_dim": 2,
                "ff_dim": 2, "max_tokens": 2, "rope_base": 10000.0, "norm_epsilon": 1e-5}
    bad = [
        b'{"config": {}, "config": {}, "weights": {}}',                          # duplicate key
        json.dumps({"config": dict(good_cfg, layers=-1), "weights": {}}).encode(),  # negative size
        json.dumps({"config": dict(good_cfg, layers=1.5), "weights": {}}).encode(),  # fractional size
        json.dumps({"config": dict(good_cfg, rope_base="x"), "weights": {}}).encode(),  # wrong type
        json.dumps({"config": good_cfg}).encode(),                                   # missing weights
        json.dumps({"config": good_cfg, "weights": {"embedding": [0.0], "layers": 3,
                                                    "final_norm": [1.0]}}).encode(),  # layers not a list
        json.dumps({"config": good_cfg, "weights": {"embedding": ["a"], "layers": [],
                                                    "final_norm": [1.0]}}).encode(),  # not numbers
        b'{"config": {}, "weights": {}} trailing',                                   # trailing content
        b"[" * 100 + b"]" * 100,                                                     # nesting too deep
    ]
    L = lib()
    for src in bad:
        st, h = bridge_open(src)
        assert st == OK, src
        ev = bridge_wait(h)
        assert (ev.kind, ev.code) == (ERROR, MODEL_FAILED), src
        assert L.aie_close(h) == OK
