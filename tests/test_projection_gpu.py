"""tvp_decode_projections (K5) on the GPU against an FP32 PyTorch reference of
the reference engine's projection GEMMs (cublasGemmEx, BF16 operands, FP32
accumulation, BF16 or FP32 result; src/model/attention.cu:194-323,
src/model/mlp.cu:8-102, src/model/lm_head.cu:8-36).

Tolerance: the exact sum rounded once, so the FP32 result may differ from
the FP32 reference by the accumulation error, bounded here by 1e-4 of the
sum of |products|, and a BF16 result additionally by one BF16 rounding
(2^-8 relative).  Results must be bitwise identical from call to call.

The fused epilogues must equal, bit for bit, the reference's own residualAdd
and silu kernels (src/model/resConnection.cu:6-17, src/model/SiLU.cu:5-16, run
from the reference engine compiled under oracle/_ref) applied to the
projection's BF16 result."""
import ctypes
from pathlib import Path

import pytest
import torch

from vllm_b200 import _native as N
from vllm_b200 import ops

ROOT = Path(__file__).resolve().parents[1]

pytestmark = pytest.mark.gpu


def make(rows, k, ns, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, k, generator=g, device="cuda").to(torch.bfloat16)
    ws = [(torch.randn(n, k, generator=g, device="cuda") * 0.02).to(torch.bfloat16) for n in ns]
    return x, ws


def check(x, w, out, f32):
    ref = x.float() @ w.float().t()
    mag = x.float().abs() @ w.float().abs().t()
    tol = 1e-4 * mag + (0.0 if f32 else 2.0 ** -8 * ref.abs()) + 1e-30
    err = (out.float() - ref).abs()
    assert out.dtype == (torch.float32 if f32 else torch.bfloat16)
    assert bool((err <= tol).all()), float((err / tol).max())


@pytest.mark.parametrize("rows", [1, 4, 8])
@pytest.mark.parametrize("k,ns", [(2048, [2048, 512, 512]),   # Q, K, V of one launch
                                  (2048, [8192, 8192]),        # gate, up
                                  (8192, [2048]),              # down (16-warp form)
                                  (256, [16]),                 # smallest shape
                                  (2304, [48, 32]),            # 8 warps of 9 blocks: a partial batch
                                  (4608, [32])])               # 16 warps of 9 blocks
def test_projection_matches_fp32_reference(rows, k, ns):
    x, ws = make(rows, k, ns, seed=rows * 131 + k + len(ns))
    outs = ops.decode_projections(x, ws)
    torch.cuda.synchronize()
    for w, o in zip(ws, outs):
        check(x, w, o, f32=False)


def test_lm_head_form_fp32_output_and_determinism():
    x, (w,) = make(4, 2048, [4096], seed=7)
    a = ops.decode_projections(x, [w], epilogue="f32")[0]
    b = ops.decode_projections(x, [w], epilogue="f32")[0]
    torch.cuda.synchronize()
    check(x, w, a, f32=True)
    assert torch.equal(a, b)


def test_rows_past_the_batch_are_left_alone():
    # out has exactly `rows` rows; the kernel must not write row `rows`
    x, (w,) = make(3, 2048, [512], seed=11)
    buf = torch.full((4, 512), 7.0, dtype=torch.bfloat16, device="cuda")
    ops.decode_projections(x, [w], outs=[buf[:3]])
    torch.cuda.synchronize()
    check(x, w, buf[:3], f32=False)
    assert bool((buf[3] == 7.0).all())


def test_matches_cublas_bf16_gemm_closely():
    x, ws = make(4, 2048, [2048], seed=5)
    ours = ops.decode_projections(x, ws)[0].float()
    lib = (x @ ws[0].t()).float()  # torch's cuBLAS BF16 GEMM, FP32 accumulation
    torch.cuda.synchronize()
    assert float((ours - lib).abs().max()) <= 2.0 ** -7 * float(lib.abs().max())


@pytest.fixture(scope="module")
def reference_engine():
    path = ROOT / "oracle" / "_ref" / "libtvp_e2e_ref.so"
    if not path.exists():
        pytest.skip("reference engine not built (make -C oracle e2e)")
    lib = ctypes.CDLL(str(path))
    for name in ("_Z4siluP13__nv_bfloat16S0_i", "_Z11residualAddP13__nv_bfloat16S0_i"):
        getattr(lib, name).argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
        getattr(lib, name).restype = None
    return lib


@pytest.mark.parametrize("rows", [1, 4, 8])
@pytest.mark.parametrize("k", [2048, 8192])  # O projection, down projection
def test_residual_epilogue_is_the_reference_residual_add(reference_engine, rows, k):
    x, (w,) = make(rows, k, [2048], seed=40 + rows + k)
    g = torch.Generator(device="cuda").manual_seed(rows)
    hidden = torch.randn(rows, 2048, generator=g, device="cuda").to(torch.bfloat16)
    y = ops.decode_projections(x, [w])[0]
    expect = hidden.clone()
    torch.cuda.synchronize()
    # residualAdd(hidden, y, rows) launches on the legacy default stream
    reference_engine._Z11residualAddP13__nv_bfloat16S0_i(expect.data_ptr(), y.data_ptr(), rows)
    torch.cuda.synchronize()
    got = hidden.clone()
    ops.decode_projections(x, [w], outs=[got], epilogue="residual")
    torch.cuda.synchronize()
    assert torch.equal(got, expect)
    assert not torch.equal(got, hidden)


@pytest.mark.parametrize("rows", [1, 4, 8])
def test_swiglu_epilogue_is_the_reference_silu(reference_engine, rows):
    x, (wg, wu) = make(rows, 2048, [8192, 8192], seed=60 + rows)
    gate, up = ops.decode_projections(x, [wg, wu])
    expect = gate.clone()
    torch.cuda.synchronize()
    reference_engine._Z4siluP13__nv_bfloat16S0_i(expect.data_ptr(), up.data_ptr(), rows)
    torch.cuda.synchronize()
    got = ops.decode_projections(x, [wg, wu], epilogue="swiglu")[0]
    again = ops.decode_projections(x, [wg, wu], epilogue="swiglu")[0]
    torch.cuda.synchronize()
    assert torch.equal(got, expect)
    assert torch.equal(got, again)


def test_back_to_back_launches_read_the_previous_output():
    """Each launch lets the next one start early and streams its weights before
    it waits for the previous grid; the input rows must still be the previous
    launch's finished output.  `act` is NaN before every chain, so a read ahead
    of the wait would leave NaNs in y."""
    x, (wg, wu) = make(4, 2048, [8192, 8192], seed=81)
    _, (wd,) = make(4, 8192, [2048], seed=82)
    act = torch.empty(4, 8192, dtype=torch.bfloat16, device="cuda")
    hidden = torch.empty(4, 2048, dtype=torch.bfloat16, device="cuda")
    h0 = torch.randn(4, 2048, device="cuda").to(torch.bfloat16)
    results = []
    for _ in range(4):
        act.fill_(float("nan"))
        hidden.copy_(h0)
        ops.decode_projections(x, [wg, wu], outs=[act], epilogue="swiglu")
        ops.decode_projections(act, [wd], outs=[hidden], epilogue="residual")
        results.append(hidden.clone())
    torch.cuda.synchronize()
    act_ref = ops.decode_projections(x, [wg, wu], epilogue="swiglu")[0]
    torch.cuda.synchronize()
    y_ref = ops.decode_projections(act_ref, [wd])[0]
    torch.cuda.synchronize()
    expect = h0 + y_ref
    for r in results:
        assert not bool(r.isnan().any())
        assert torch.equal(r, expect)


@pytest.mark.parametrize("rows", [1, 4, 8])
@pytest.mark.parametrize("k", [2048, 8192])  # O projection, down projection
def test_residual_rmsnorm_form_is_residual_add_then_the_reference_rmsnorm(reference_engine, rows, k):
    """tvp_decode_projection_residual_rmsnorm: the residual epilogue, then the
    reference's rmsNormKernel of the updated rows, bit for bit (each CTA sums
    its features' squares as a subtree of the reference's tree, and all CTAs
    normalise their own features once every subtree is in); three times in a
    row on one scratch."""
    reference_engine.e2e_ref_rmsnorm.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int]
    x, (w,) = make(rows, k, [2048], seed=90 + rows + k)
    g = torch.Generator(device="cuda").manual_seed(rows + 3)
    hidden0 = (torch.randn(rows, 2048, generator=g, device="cuda") * 3).to(torch.bfloat16)
    gain = (1 + 0.1 * torch.randn(2048, generator=g, device="cuda")).to(torch.bfloat16)
    scratch = ops.norm_scratch("cuda")
    # expected: K5 residual form, then the reference kernel on its output
    want_hidden = hidden0.clone()
    ops.decode_projections(x, [w], outs=[want_hidden], epilogue="residual")
    want_norm = torch.empty_like(want_hidden)
    torch.cuda.synchronize()
    assert reference_engine.e2e_ref_rmsnorm(want_hidden.data_ptr(), want_norm.data_ptr(),
                                            gain.data_ptr(), rows) == 0
    torch.cuda.synchronize()
    for _ in range(3):
        hidden = hidden0.clone()
        norm = torch.full_like(hidden, float("nan"))
        ops.decode_projection_residual_rmsnorm(x, w, hidden, gain, norm, scratch)
        torch.cuda.synchronize()
        assert torch.equal(hidden, want_hidden)
        assert torch.equal(norm, want_norm)
        assert int(scratch[1].item()) == 0


def test_residual_rmsnorm_wait_gives_up_and_reports():
    """The CTAs of the residual + RMSNorm launch wait for one another at an
    arrival counter, bounded by 2 s.  A counter that starts off a multiple of
    the grid (128) makes the last arrival wait for a count nothing reaches:
    it must give up, set TVP_DEVERR_TIMEOUT in the scratch's error word and
    leave its 16 norm outputs per row unwritten, while the residual update
    completes and the other CTAs write theirs (their values are unspecified:
    the counter no longer says that every subtree is in); the next launch on
    a good scratch is whole."""
    x, (w,) = make(4, 2048, [2048], seed=7)
    hidden0 = torch.randn(4, 2048, device="cuda").to(torch.bfloat16)
    gain = torch.ones(2048, dtype=torch.bfloat16, device="cuda")
    want_hidden = hidden0.clone()
    ops.decode_projections(x, [w], outs=[want_hidden], epilogue="residual")
    scratch = ops.norm_scratch("cuda")
    scratch[0] = 1
    hidden = hidden0.clone()
    norm = torch.full_like(hidden, float("nan"))
    ops.decode_projection_residual_rmsnorm(x, w, hidden, gain, norm, scratch)
    torch.cuda.synchronize()
    assert int(scratch[1].item()) & N.TVP_DEVERR_TIMEOUT
    assert torch.equal(hidden, want_hidden)
    assert int(torch.isnan(norm.float()).sum(dim=1).max()) == 16   # one CTA's features
    good = ops.norm_scratch("cuda")
    hidden = hidden0.clone()
    norm2 = torch.full_like(hidden, float("nan"))
    ops.decode_projection_residual_rmsnorm(x, w, hidden, gain, norm2, good)
    torch.cuda.synchronize()
    assert int(good[1].item()) == 0 and not bool(torch.isnan(norm2.float()).any())


def _pools_and_tables(rows, seed, num_pages=64, layers=3):
    g = torch.Generator(device="cuda").manual_seed(seed)
    kp = torch.randn(layers, num_pages, 16, 512, generator=g, device="cuda").to(torch.bfloat16)
    vp = torch.randn(layers, num_pages, 16, 512, generator=g, device="cuda").to(torch.bfloat16)
    perm = torch.randperm(num_pages, generator=torch.Generator().manual_seed(seed))
    tables = perm[:rows * 8].reshape(rows, 8).to(torch.int32).cuda()
    pos = torch.tensor([5, 127, 16, 0, 64, 100, 33, 77][:rows], dtype=torch.int32, device="cuda")
    return kp, vp, tables, pos


@pytest.mark.parametrize("rows", [1, 4, 8])
def test_qkv_rope_append_form_equals_projections_then_rope_append(rows):
    """tvp_decode_qkv_rope_append: the three projections, then K1
    (tvp_rope_append of q and k, v as is) into the same pools, bit for bit:
    q rows, and every page of every layer afterwards."""
    x, (wq, wk, wv) = make(rows, 2048, [2048, 512, 512], seed=120 + rows)
    kp, vp, tables, pos = _pools_and_tables(rows, 7 + rows)
    layer = 1
    q, k, v = ops.decode_projections(x, [wq, wk, wv])
    kp_want, vp_want = kp.clone(), vp.clone()
    err = ops.new_error_word("cuda")
    ops.rope_append(kp_want, vp_want, layer, tables, pos, k, v, q=q, error=err)
    q_got = torch.empty_like(q)
    ops.decode_qkv_rope_append(x, wq, wk, wv, q_got, kp, vp, layer, tables, pos, error=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(q_got, q)
    assert torch.equal(kp, kp_want)
    assert torch.equal(vp, vp_want)


@pytest.mark.parametrize("rows", [1, 4, 8])
def test_down_norm_qkv_is_the_two_launches_it_replaces(rows):
    """tvp_decode_down_norm_qkv: the down projection with its residual add and
    spread RMSNorm, then the next layer's Q/K/V with RoPE and the page append,
    in one launch: hidden, norm_out, q and every page equal, bit for bit, what
    decode_projection_residual_rmsnorm then decode_qkv_rope_append produce;
    twice on one scratch."""
    g = torch.Generator(device="cuda").manual_seed(300 + rows)
    x = torch.randn(rows, 8192, generator=g, device="cuda").to(torch.bfloat16)
    w_down = (torch.randn(2048, 8192, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    _, (wq, wk, wv) = make(rows, 2048, [2048, 512, 512], seed=310 + rows)
    hidden0 = (torch.randn(rows, 2048, generator=g, device="cuda") * 3).to(torch.bfloat16)
    gain = (1 + 0.1 * torch.randn(2048, generator=g, device="cuda")).to(torch.bfloat16)
    kp0, vp0, tables, pos = _pools_and_tables(rows, 17 + rows)
    layer = 2
    err = ops.new_error_word("cuda")
    # the two launches
    h_want = hidden0.clone()
    n_want = torch.empty_like(h_want)
    ops.decode_projection_residual_rmsnorm(x, w_down, h_want, gain, n_want, ops.norm_scratch("cuda"))
    kp_want, vp_want = kp0.clone(), vp0.clone()
    q_want = torch.empty(rows, 2048, dtype=torch.bfloat16, device="cuda")
    ops.decode_qkv_rope_append(n_want, wq, wk, wv, q_want, kp_want, vp_want, layer, tables, pos,
                               error=err)
    scratch = ops.norm_scratch("cuda")
    for _ in range(2):
        h_got = hidden0.clone()
        n_got = torch.full_like(h_got, float("nan"))
        kp, vp = kp0.clone(), vp0.clone()
        q_got = torch.full_like(q_want, float("nan"))
        ops.decode_down_norm_qkv(x, w_down, h_got, gain, n_got, scratch, wq, wk, wv, q_got, kp, vp,
                                 layer, tables, pos, error=err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0 and int(scratch[1].item()) == 0
        assert torch.equal(h_got, h_want)
        assert torch.equal(n_got, n_want)
        assert torch.equal(q_got, q_want)
        assert torch.equal(kp, kp_want)
        assert torch.equal(vp, vp_want)


def test_qkv_rope_append_reports_a_bad_page_and_skips_it():
    x, (wq, wk, wv) = make(2, 2048, [2048, 512, 512], seed=140)
    kp, vp, tables, pos = _pools_and_tables(2, 11)
    tables[1, pos[1] // 16] = 10_000  # outside the pool
    before_k, before_v = kp.clone(), vp.clone()
    err = ops.new_error_word("cuda")
    q = torch.empty(2, 2048, dtype=torch.bfloat16, device="cuda")
    ops.decode_qkv_rope_append(x, wq, wk, wv, q, kp, vp, 0, tables, pos, error=err)
    torch.cuda.synchronize()
    assert int(err.item()) & 1  # TVP_DEVERR_BAD_PAGE
    # row 0 was appended, row 1 touched nothing
    changed = (kp != before_k).any(dim=-1) | (vp != before_v).any(dim=-1)
    assert int(changed.sum()) == 1
