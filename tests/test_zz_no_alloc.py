"""qb_rope_static, the RoPE entry point that allocates nothing: its results
must equal qb_rope's bit for bit on consecutive calls of different sizes
(the shared static scratch keeps nothing from one call to the next), and a
request beyond its fixed scratch is refused before any device work.

Named to be collected last, so it also runs after every other GPU test has
used the library's allocating paths."""
import ctypes as C
import os
import subprocess
import sys

import numpy as np
import pytest

from llm_inference_edu_b200._lib import Detail, lib

RESOURCE_BUDGET, NONFINITE = 19, 11
MAX_TABLE = 65472  # QB_ROPE_STATIC_MAX_TABLE


def test_rope_static_refuses_oversize_before_device_work():
    # 1024 tokens x head_dim 64 = 65536 floats of table > 65472: refused on
    # the host, so no GPU is needed and no pointer is touched.
    L = lib()
    tokens, heads, hd = 1024, 2, 64
    n = tokens * heads * hd
    assert L.qb_rope_static(None, n, None, n, tokens, heads, hd, 0, 1e6, None) == RESOURCE_BUDGET
    d = Detail()
    L.qb_last_detail(C.byref(d))
    assert (d.expected, d.actual) == (MAX_TABLE, tokens * hd)
    # Argument checks shared with qb_rope come first and agree with it.
    for args in [(None, 0, None, 0, 1, 1, 3, 0, 1e4, None), (None, 0, None, 0, 2, 1, 2, 1 << 24, 1e4, None),
                 (None, 0, None, 0, 0, 1, 2, 0, 1e4, None), (None, 4, None, 4, 2, 1, 2, 0, -1.0, None)]:
        assert L.qb_rope_static(*args) == L.qb_rope(*args)


@pytest.mark.gpu
def test_rope_static_matches_rope_on_consecutive_calls():
    import torch
    L = lib()
    torch.cuda.init()
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(7)

    def run(fn, x, tokens, heads, hd, start, base):
        y = torch.full_like(x, 37.0)
        st = fn(C.c_void_p(x.data_ptr()), x.numel(), C.c_void_p(y.data_ptr()), y.numel(),
                tokens, heads, hd, start, base, C.c_void_p(stream))
        torch.cuda.synchronize()
        return st, y.cpu().numpy()

    # Two consecutive calls: a large one near the limit, then a smaller one
    # at other positions, each compared with qb_rope on the same input.
    cases = [(1023, 14, 64, 5, 1e6), (37, 2, 128, 100000, 1e4)]
    for tokens, heads, hd, start, base in cases:
        assert tokens * hd <= MAX_TABLE
        x = torch.from_numpy(rng.standard_normal(tokens * heads * hd).astype(np.float32)).cuda()
        s_ref, y_ref = run(L.qb_rope, x, tokens, heads, hd, start, base)
        s_new, y_new = run(L.qb_rope_static, x, tokens, heads, hd, start, base)
        assert s_ref == 0 and s_new == 0
        assert np.array_equal(y_new.view(np.uint32), y_ref.view(np.uint32)), (tokens, heads, hd)

    # A non-finite input is reported with its index and leaves y unwritten.
    x = torch.ones(4 * 2 * 8, dtype=torch.float32, device="cuda")
    x[21] = float("nan")
    st, y = run(L.qb_rope_static, x, 4, 2, 8, 0, 1e4)
    d = Detail()
    L.qb_last_detail(C.byref(d))
    assert st == NONFINITE and d.index == 21
    assert np.all(y == 37.0)
    # The flag word is reset by each call: a clean input right after passes.
    x[21] = 0.5
    st, y = run(L.qb_rope_static, x, 4, 2, 8, 0, 1e4)
    s_ref, y_ref = run(L.qb_rope, x, 4, 2, 8, 0, 1e4)
    assert st == 0 and s_ref == 0 and np.array_equal(y.view(np.uint32), y_ref.view(np.uint32))


_NO_ALLOC_PROBE = r"""
import ctypes as C, sys
sys.path.insert(0, sys.argv[1])
import torch
from llm_inference_edu_b200._lib import lib
L = lib()
torch.cuda.init()
x = torch.randn(1023 * 14 * 64, device="cuda")
y = torch.empty_like(x)
stream = torch.cuda.current_stream().cuda_stream

def call(tokens, heads, hd, start):
    n = tokens * heads * hd
    st = L.qb_rope_static(C.c_void_p(x.data_ptr()), n, C.c_void_p(y.data_ptr()), n, tokens, heads, hd,
                          start, 1e6, C.c_void_p(stream))
    assert st == 0, st

call(16, 2, 64, 0)  # the first call loads the library's device code and its static array
torch.cuda.synchronize()
free0 = torch.cuda.mem_get_info()[0]
for args in [(1023, 14, 64, 5), (37, 2, 128, 100000), (1, 1, 2, 0), (1023, 14, 64, 7)]:
    call(*args)
torch.cuda.synchronize()
free1 = torch.cuda.mem_get_info()[0]
print(free0, free1)
assert free0 == free1, (free0, free1)
"""


@pytest.mark.gpu
def test_rope_static_allocates_no_device_memory():
    # In a fresh process (so nothing else of the library has run): once the
    # first call has loaded the device code, further calls of several sizes
    # leave the device's free memory unchanged -- no cudaMalloc, no pool.
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _NO_ALLOC_PROBE, root], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
