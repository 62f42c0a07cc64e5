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


def test_fragment_mapping_covers_every_k_once():
    """Host model of K5's index arithmetic (tvp_project.cu): the lane loads
    (16 B of weight rows g and g + 8 and of input row g, at k = 8q .. 8q + 7 of
    a 32-column block), their placement in the two m16n8k16 MMAs, the MMA's
    fragment ownership (PTX ISA: a0/a2 rows g, a1/a3 rows g + 8, k pairs 2q and
    2q + 8; b0/b1 k pairs 2q and 2q + 8 of column g; c0..c3 rows g, g + 8,
    columns 2q, 2q + 1) and the epilogue's map from accumulator r of lane ln to
    (weight row, input row).  The emulated block product must equal W X^T."""
    import numpy as np
    rng = np.random.default_rng(0)
    W = rng.standard_normal((16, 32))
    X = rng.standard_normal((8, 32))
    acc = np.zeros((32, 4))  # per lane c0..c3
    for mma in range(2):
        A = np.full((16, 16), np.nan)
        B = np.full((16, 8), np.nan)
        for lane in range(32):
            g, q = lane >> 2, lane & 3
            wa, wb, xv = W[g, 8 * q:8 * q + 8], W[g + 8, 8 * q:8 * q + 8], X[g, 8 * q:8 * q + 8]
            lo, hi = slice(4 * mma, 4 * mma + 2), slice(4 * mma + 2, 4 * mma + 4)
            for regs, (row, kk) in ((wa[lo], (g, 2 * q)), (wb[lo], (g + 8, 2 * q)),
                                    (wa[hi], (g, 2 * q + 8)), (wb[hi], (g + 8, 2 * q + 8))):
                assert np.isnan(A[row, kk:kk + 2]).all()  # each slot written once
                A[row, kk:kk + 2] = regs
            for regs, kk in ((xv[lo], 2 * q), (xv[hi], 2 * q + 8)):
                assert np.isnan(B[kk:kk + 2, g]).all()
                B[kk:kk + 2, g] = regs
        assert not np.isnan(A).any() and not np.isnan(B).any()
        D = A @ B
        for lane in range(32):
            g, q = lane >> 2, lane & 3
            acc[lane] += [D[g, 2 * q], D[g, 2 * q + 1], D[g + 8, 2 * q], D[g + 8, 2 * q + 1]]
    expect = W @ X.T  # [weight row][input row]
    seen = np.zeros((16, 8), bool)
    for tid in range(128):  # the epilogue's threads
        r, ln = tid >> 5, tid & 31
        row = (ln >> 2) + (8 if r & 2 else 0)
        t = 2 * (ln & 3) + (r & 1)
        assert not seen[row, t]
        seen[row, t] = True
        assert abs(acc[ln, r] - expect[row, t]) < 1e-9
    assert seen.all()


def _reference_sum_of_squares(x):
    """rmsNormKernel's sum (src/model/rmsNorm.cu:6-14) in FP32: leaf t < 1024 is
    x[t]^2 + x[t + 1024]^2, then for i = 1, 2, ..., 512 leaf t += leaf t + i where
    t % 2i == 0.  x holds BF16 values, so each square is exact in FP32 and the
    leaf is one rounding (the kernel's FMA form gives the same)."""
    import numpy as np
    sq = (x.astype(np.float32) * x.astype(np.float32)).astype(np.float32)
    leaf = (sq[:1024] + sq[1024:]).astype(np.float32)
    i = 1
    while i < 1024:
        leaf[0::2 * i] = (leaf[0::2 * i] + leaf[i::2 * i]).astype(np.float32)
        i *= 2
    return leaf[0]


def _spread_sum_of_squares(x):
    """The spread norm's order: CTA a (of 128) owns features 8a..8a+7 and
    1024+8a..; it forms leaves 8a..8a+7 and sums them by shuffles of 4, 8 and
    16 lanes (the tree's levels 1, 2, 4); a warp then sums the 128 subtree
    values, four per lane as (p0 + p1) + (p2 + p3) (levels 8, 16), then by
    shuffles down 1, 2, 4, 8, 16 (levels 32 .. 512)."""
    import numpy as np
    f = np.float32
    sq = (x.astype(f) * x.astype(f)).astype(f)
    parts = []
    for a in range(128):
        v = [f(sq[8 * a + j] + sq[1024 + 8 * a + j]) for j in range(8)]
        for step in (1, 2, 4):                 # lanes j and j + step, j % 2step == 0
            for j in range(0, 8, 2 * step):
                v[j] = f(v[j] + v[j + step])
        parts.append(v[0])
    lanes = [f(f(parts[4 * l] + parts[4 * l + 1]) + f(parts[4 * l + 2] + parts[4 * l + 3]))
             for l in range(32)]
    off = 1
    while off < 32:
        for l in range(0, 32, 2 * off):
            lanes[l] = f(lanes[l] + lanes[l + off])
        off *= 2
    return lanes[0]


def test_spread_norm_sums_in_the_reference_tree_order():
    """The subtree decomposition of the spread RMSNorm is the reference's tree,
    so the FP32 sum is the same bits for any row (checked on rows of every
    magnitude, including ones where a different order would round differently)."""
    import numpy as np
    rng = np.random.default_rng(5)
    order_matters = 0
    for scale in (1e-3, 1.0, 3.0, 100.0, 3e4):
        for _ in range(20):
            x = (rng.standard_normal(2048) * scale).astype(np.float32)
            x = (x.view(np.uint32) & 0xFFFF0000).view(np.float32)  # BF16 values
            ref = np.float32(_reference_sum_of_squares(x))
            assert np.float32(_spread_sum_of_squares(x)).view(np.uint32) == ref.view(np.uint32)
            seq = np.float32(0)
            for v in (x * x).astype(np.float32):
                seq = np.float32(seq + v)
            order_matters += int(seq.view(np.uint32) != ref.view(np.uint32))
    assert order_matters > 50  # a sequential sum would differ on most rows
