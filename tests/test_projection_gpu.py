"""tvp_decode_projections (K5) on the GPU against an FP32 PyTorch reference of
the reference engine's projection GEMMs (cublasGemmEx, BF16 operands, FP32
accumulation, BF16 or FP32 result; src/model/attention.cu:194-323,
src/model/mlp.cu:8-102, src/model/lm_head.cu:8-36).

Tolerance: the exact sum rounded once, so the FP32 result may differ from
the FP32 reference by the accumulation error, bounded here by 1e-4 of the
sum of |products|, and a BF16 result additionally by one BF16 rounding
(2^-8 relative).  Results must be bitwise identical from call to call."""
import pytest
import torch

from vllm_b200 import ops

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
    a = ops.decode_projections(x, [w], out_f32=True)[0]
    b = ops.decode_projections(x, [w], out_f32=True)[0]
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
