"""tvp_decode_projections, host side: the C-ABI entry point rejects every
argument it cannot run before it launches anything (no GPU needed)."""
import ctypes

import pytest

from vllm_b200 import _native as N


@pytest.fixture(scope="module")
def lib():
    return N.load()


def call(lib, x=0x1000, rows=4, k=2048, ws=(0x2000,), ns=(2048,), outs=(0x3000,), f32=0,
         count=None):
    cnt = len(ws) if count is None else count
    size = max(len(ws), 1)
    wp = (ctypes.c_void_p * size)(*ws)
    op = (ctypes.c_void_p * size)(*outs)
    nn = (ctypes.c_int * size)(*ns)
    return lib.tvp_decode_projections(None if x is None else ctypes.c_void_p(x), rows, k, cnt,
                                      wp, nn, op, f32, None)


def test_projection_entry_point_checks_arguments(lib):
    bad = N.TVP_ERR_INVALID_ARGUMENT
    assert call(lib, x=None) == bad
    assert call(lib, x=0x1008) == bad                       # x not 16-byte aligned
    assert call(lib, rows=0) == bad
    assert call(lib, rows=9) == bad                         # at most 8 rows (the MMA's N)
    assert call(lib, k=0) == bad
    assert call(lib, k=2048 + 128) == bad                   # k a multiple of 256
    assert call(lib, count=0) == bad
    assert call(lib, ws=(0x2000,) * 4, ns=(16,) * 4, outs=(0x3000,) * 4) == bad  # at most 3
    assert call(lib, ns=(8,)) == bad                        # n a multiple of 16
    assert call(lib, ns=(2048 + 8,)) == bad
    assert call(lib, ws=(0,)) == bad                        # null weight
    assert call(lib, ws=(0x2008,)) == bad                   # weight not 16-byte aligned
    assert call(lib, outs=(0,)) == bad
    assert call(lib, outs=(0x3001,)) == bad                 # BF16 output misaligned
    assert call(lib, outs=(0x3002,), f32=1) == bad          # FP32 output misaligned
    assert call(lib, f32=4) == bad                          # epilogue 0..3
    assert call(lib, f32=-1) == bad
    # SwiGLU: exactly two matrices of one shape
    assert call(lib, f32=3) == bad
    assert call(lib, ws=(0x2000, 0x4000), ns=(2048, 1024), outs=(0x3000, 0), f32=3) == bad
    assert call(lib, ws=(0x2000, 0x4000, 0x5000), ns=(16,) * 3, outs=(0x3000,) * 3, f32=3) == bad
    # an output overlapping the input rows
    assert call(lib, x=0x100000, outs=(0x100000 + 2 * 4 * 2048 - 16,)) == bad
    assert call(lib, x=0x100000, outs=(0x100000 - 2 * 4 * 2048 + 2,)) == bad
    assert call(lib, ws=(0x2000, 0x2008), ns=(16, 16), outs=(0x3000, 0x4000)) == bad


def test_projection_wrapper_checks_shapes():
    torch = pytest.importorskip("torch")
    from vllm_b200 import ops
    x = torch.zeros(4, 256, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        ops.decode_projections(x, [torch.zeros(16, 256, dtype=torch.bfloat16)])  # not CUDA
