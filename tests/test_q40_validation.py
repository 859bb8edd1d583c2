"""MulQ40Into / MulQ40BatchInto argument checks through the C ABI, on a
host-only context (no compute call): every case of TestMulQ40Validation
(tests/testdata/forward/q40_stream_test.go:107-165) that has a counterpart
here, with q40Shape's and MulQ40BatchInto's error classes
(forward/q40.go:49-71, 105-130)."""
import dataclasses

import numpy as np
import pytest

import refdata

spt = refdata.spt


def _fixture():
    data = refdata.q40_fixture(64, 5, "stream")
    return spt.q40_tensor(data, 64, 5, name="test.weight", prefix=37)


def test_valid_call_reaches_the_device_check(host_ctx):
    reader, tensor = _fixture()
    with pytest.raises(spt.SptError) as e:
        host_ctx.mul_q40(reader, tensor, np.zeros(64, np.float32))
    assert e.value.status == spt.ERR_NO_DEVICE


@pytest.mark.parametrize("name,call,status", [
    ("input length", lambda c, r, t, x, y: c.mul_q40(r, t, x[1:], y), "ERR_DIMENSIONS"),
    ("output length", lambda c, r, t, x, y: c.mul_q40(r, t, x, y[1:]), "ERR_DIMENSIONS"),
    ("zero batch", lambda c, r, t, x, y: c.mul_q40_batch(r, t, x, 0, y), "ERR_DIMENSIONS"),
    ("negative batch", lambda c, r, t, x, y: c.mul_q40_batch(r, t, x, -1, y), "ERR_DIMENSIONS"),
    ("overflow batch", lambda c, r, t, x, y: c.mul_q40_batch(r, t, x, (1 << 63) - 1, y), "ERR_DIMENSIONS"),
    ("batch length", lambda c, r, t, x, y: c.mul_q40_batch(r, t, x, 2, y), "ERR_DIMENSIONS"),
])
def test_argument_errors(host_ctx, name, call, status):
    reader, tensor = _fixture()
    x, y = np.zeros(64, np.float32), np.zeros(5, np.float32)
    with pytest.raises(spt.SptError) as e:
        call(host_ctx, reader, tensor, x, y)
    assert e.value.status == getattr(spt, status), (name, e.value)


def test_overlap(host_ctx):
    reader, tensor = _fixture()
    backing = np.zeros(70, np.float32)
    for x, y in ((backing[:64], backing[3:8]), (backing[4:68], backing[:5]), (backing[:64], backing[63:68])):
        with pytest.raises(spt.SptError) as e:
            host_ctx.mul_q40(reader, tensor, x, y)
        assert e.value.status == spt.ERR_OVERLAP
    # adjacent is not overlapping: it gets as far as the device check
    with pytest.raises(spt.SptError) as e:
        host_ctx.mul_q40(reader, tensor, backing[:64], backing[64:69])
    assert e.value.status == spt.ERR_NO_DEVICE


@pytest.mark.parametrize("name,change,status", [
    ("type 1", dict(type=1), "ERR_DIMENSIONS"),
    ("one dimension", dict(shape=(64,)), "ERR_DIMENSIONS"),
    ("input 63", dict(shape=(63, 5)), "ERR_DIMENSIONS"),
    ("output 0", dict(shape=(64, 0)), "ERR_DIMENSIONS"),
    ("huge input", dict(shape=((1 << 64) - 1, 5)), "ERR_DIMENSIONS"),
    ("range end - 1", "end-1", "ERR_FILE_RANGE"),
    ("empty range", "start=end", "ERR_FILE_RANGE"),
    ("range past the file", "shift", "ERR_FILE_RANGE"),
])
def test_tensor_errors(host_ctx, name, change, status):
    reader, tensor = _fixture()
    if change == "end-1":
        bad = dataclasses.replace(tensor, end=tensor.end - 1)
    elif change == "start=end":
        bad = dataclasses.replace(tensor, start=tensor.end)
    elif change == "shift":
        bad = dataclasses.replace(tensor, start=tensor.start + 1, end=tensor.end + 1)
    else:
        bad = dataclasses.replace(tensor, **change)
    x, y = np.zeros(64, np.float32), np.zeros(5, np.float32)
    with pytest.raises(spt.SptError) as e:
        host_ctx.mul_q40(reader, bad, x, y)
    assert e.value.status == getattr(spt, status), (name, e.value)


def test_unsupported_width(host_ctx):
    """Rows wider than the one-input kernel's shared-memory ring."""
    reader, tensor = spt.q40_tensor(np.zeros(16384 // 32 * 18, np.uint8), 16384, 1)
    with pytest.raises(spt.SptError) as e:
        host_ctx.mul_q40(reader, tensor, np.zeros(16384, np.float32))
    assert e.value.status == spt.ERR_UNSUPPORTED


def test_pre_canceled(host_ctx):
    reader, tensor = _fixture()
    with pytest.raises(spt.CanceledError):
        host_ctx.mul_q40(reader, tensor, np.zeros(64, np.float32), cancel=np.ones(1, np.int32))
