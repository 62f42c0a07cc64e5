"""Host <-> device helpers of the GPU tests (BF16 carried as raw uint16 on the host)."""
from __future__ import annotations

import numpy as np
import torch

from vllm_b200 import ops


def dev_bf16(a: np.ndarray, device="cuda") -> torch.Tensor:
    a = np.ascontiguousarray(a, dtype=np.uint16)
    return torch.from_numpy(a.view(np.int16)).to(device).view(torch.bfloat16)


def host_bf16(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def dev_i32(a, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(device)


def f32(a: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(a, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def run_decode(case, layer=0, mode=0, num_ctas=0, q=None, error=None, workspace=None):
    """Uploads a DecodeCase and runs the fused decode attention; returns (out bits, error bits)."""
    k = dev_bf16(case.k_pool)
    v = dev_bf16(case.v_pool)
    qd = dev_bf16(case.q if q is None else q)
    tables = dev_i32(case.tables)
    lens = dev_i32(case.lens)
    err = error if error is not None else ops.new_error_word("cuda")
    ws = workspace or ops.DecodeWorkspace(case.batch, "cuda", num_ctas=num_ctas,
                                          kv_heads=case.k_pool.shape[3] // 64)
    if mode == 0:
        ops.decode_plan(lens, case.tables.shape[1], ws, error=err)
    out = ops.paged_decode_attention(qd, k, v, layer, tables, lens, ws if mode == 0 else None,
                                     mode=mode, error=err)
    torch.cuda.synchronize()
    return host_bf16(out), int(err.item())


def assert_close_bf16(actual_bits, expected, atol, rtol, what=""):
    a = f32(actual_bits).astype(np.float64)
    e = np.asarray(expected, dtype=np.float64)
    assert np.isfinite(a).all(), f"{what}: non-finite output"
    err = np.abs(a - e)
    bad = err > atol + rtol * np.abs(e)
    assert not bad.any(), (f"{what}: {bad.sum()} of {bad.size} outside atol={atol} rtol={rtol}; "
                           f"max abs err {err.max():.3g}")
    return float(err.max())
