"""MulQ80Into / MulQ80Argmax argument checks through the C ABI, on a
host-only context (no compute call): q80Shape's error classes
(forward/q80.go:150-170) for spt_mul_q80 and spt_q80_matrix_create, including
TestQuantOptimizationQ80ShapeOverflow
(tests/testdata/forward/quant_optimization_test.go:368-374).  A valid call gets
as far as the device check.  The length, window and cancellation checks of
TestMulQ80Into (tests/testdata/forward/sampling_test.go:179-209) sit in the
cgo shim, which checks x and y against the shape before calling the library
(stream-pt_b200/go/q80_cuda.go)."""
import ctypes

import numpy as np
import pytest

import refdata

spt = refdata.spt


def raw_mul(ctx, data, data_len, input_, output):
    """spt_mul_q80 with small x / y buffers: every case here fails before
    either is touched."""
    x = np.zeros(64, np.float32)
    y = np.zeros(64, np.float32)
    am, best = ctypes.c_int64(), ctypes.c_float()
    st = spt.lib().spt_mul_q80(ctx._h, None if data is None else spt._p(data), data_len, input_, output,
                               spt._p(x), spt._p(y), ctypes.byref(am), ctypes.byref(best))
    return st, spt.lib().spt_last_error(ctx._h).decode()


def raw_create(ctx, data, data_len, input_, output):
    m = ctypes.c_void_p()
    st = spt.lib().spt_q80_matrix_create(ctx._h, spt._p(data), data_len, input_, output, ctypes.byref(m))
    assert not m.value
    return st, spt.lib().spt_last_error(ctx._h).decode()


def fixture(input_=96, rows=17):
    data, x = refdata.q80_fixture(input_, rows, x_kind="into")
    return data, x


def test_valid_call_reaches_the_device_check(host_ctx):
    data, x = fixture()
    with pytest.raises(spt.SptError) as e:
        host_ctx.mul_q80(data, 96, 17, x)
    assert e.value.status == spt.ERR_NO_DEVICE
    st, _ = raw_create(host_ctx, data, data.size, 96, 17)
    assert st == spt.ERR_NO_DEVICE


@pytest.mark.parametrize("name,input_,output,status,text", [
    ("input 0", 0, 17, "ERR_DIMENSIONS", "invalid Q8_0 shape"),
    ("input -32", -32, 17, "ERR_DIMENSIONS", "invalid Q8_0 shape"),
    ("input 95", 95, 17, "ERR_DIMENSIONS", "invalid Q8_0 shape"),
    ("output 0", 96, 0, "ERR_DIMENSIONS", "invalid Q8_0 shape"),
    # TestQuantOptimizationQ80ShapeOverflow: output = MaxUint64 (-1 as int64)
    ("output MaxUint64", 32, -1, "ERR_DIMENSIONS", "invalid Q8_0 shape"),
    ("output 2^32", 32, 1 << 32, "ERR_DIMENSIONS", "exceed platform limits"),
    ("input 2^25", 1 << 25, 1, "ERR_DIMENSIONS", "exceed platform limits"),
])
def test_shape_errors(host_ctx, name, input_, output, status, text):
    data, _ = fixture()
    for call in (raw_mul, raw_create):
        st, msg = call(host_ctx, data, data.size, input_, output)
        assert st == getattr(spt, status), (name, call.__name__, msg)
        assert text in msg, (name, msg)


@pytest.mark.parametrize("delta", [-1, 1, -102])
def test_byte_range_errors(host_ctx, delta):
    data, _ = fixture()
    buf = np.zeros(data.size + 200, np.uint8)
    buf[:data.size] = data
    for call in (raw_mul, raw_create):
        st, msg = call(host_ctx, buf, data.size + delta, 96, 17)
        assert st == spt.ERR_FILE_RANGE and "invalid byte range" in msg, (call.__name__, msg)


def test_null_data(host_ctx):
    st, _ = raw_mul(host_ctx, None, 17 * 102, 96, 17)
    assert st == spt.ERR_NULL_ARG


def test_rows_too_long_for_the_ring(host_ctx):
    """A row of 2^20 elements (1.1 MB) does not fit the shared-memory ring:
    refused as unsupported, not attempted."""
    input_ = 1 << 20
    data = np.zeros(input_ // 32 * 34, np.uint8)
    for call in (raw_mul, raw_create):
        st, msg = call(host_ctx, data, data.size, input_, 1)
        assert st == spt.ERR_UNSUPPORTED, (call.__name__, msg)
