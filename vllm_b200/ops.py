"""Operator layer over the C-ABI: the paged-KV kernels on torch CUDA tensors.

torch is used only as plumbing (device memory and the current stream); every
operation here is one call into ``libtvp_paged.so``.

Shapes (reference geometry, src/model/paged_kvcache.cu:10-11):
  k_pool, v_pool : bf16 [num_layers, num_pages, 16, kv_heads * 64]
  block_tables   : int32 [batch, table_stride]   (-1 = no page)
  seq_lens       : int32 [batch]                 attended length L per row
  q, out         : bf16 [batch, 4 * kv_heads * 64]  head h at h * 64

kv_heads is the model's 8, or the 4, 2 or 1 heads one GPU holds when the KV
heads are sharded over 2, 4 or 8 GPUs (``vllm_b200.sharding``).
"""
from __future__ import annotations

import ctypes

import torch

from . import _native as N


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream):
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _need(t, name, dtype, device=None):
    if t is None:
        raise ValueError(f"{name} is required")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if device is not None and t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")


def _pool_geometry(k_pool, v_pool):
    _need(k_pool, "k_pool", torch.bfloat16)
    _need(v_pool, "v_pool", torch.bfloat16, k_pool.device)
    if k_pool.dim() != 4 or k_pool.shape != v_pool.shape or k_pool.shape[2] != N.PAGE_TOKENS \
            or k_pool.shape[3] % N.HEAD_DIM:
        raise ValueError("pools must be [num_layers, num_pages, 16, kv_heads*64] and equal")
    num_layers, num_pages, _, kv_dim = k_pool.shape
    return num_layers, num_pages, kv_dim // N.HEAD_DIM


def new_error_word(device) -> torch.Tensor:
    return torch.zeros(1, dtype=torch.int32, device=device)


def rope_append(k_pool, v_pool, layer, block_tables, token_pos, k, v, q=None, token_seq=None,
                rope_k=True, writeback_k=True, error=None, stream=None):
    """K1: RoPE (q optional, k) + append of k, v rows into their page slots.

    Token i goes to row ``token_seq[i]`` (default i) of ``block_tables`` at
    position ``token_pos[i]``.  k is rotated in place when ``writeback_k``.
    """
    lib = N.load()
    num_layers, num_pages, kv_heads = _pool_geometry(k_pool, v_pool)
    dev = k_pool.device
    _need(block_tables, "block_tables", torch.int32, dev)
    _need(token_pos, "token_pos", torch.int32, dev)
    _need(k, "k", torch.bfloat16, dev)
    _need(v, "v", torch.bfloat16, dev)
    n = token_pos.numel()
    if k.shape != (n, kv_heads * N.HEAD_DIM) or v.shape != k.shape:
        raise ValueError("k and v must be [num_tokens, kv_heads*64]")
    flags = 0
    if rope_k:
        flags |= N.TVP_APPEND_ROPE_K
    if writeback_k:
        flags |= N.TVP_APPEND_WRITEBACK_K
    q_heads = 0
    if q is not None:
        _need(q, "q", torch.bfloat16, dev)
        if q.dim() != 2 or q.shape[0] != n or q.shape[1] % N.HEAD_DIM:
            raise ValueError("q must be [num_tokens, q_heads*64]")
        q_heads = q.shape[1] // N.HEAD_DIM
        flags |= N.TVP_APPEND_ROPE_Q
    if token_seq is not None:
        _need(token_seq, "token_seq", torch.int32, dev)
        if token_seq.numel() != n:
            raise ValueError("token_seq must have one entry per token")
    if block_tables.dim() != 2:
        raise ValueError("block_tables must be [rows, table_stride]")
    rc = lib.tvp_rope_append(_ptr(k_pool), _ptr(v_pool), num_pages, num_layers, layer, kv_heads,
                             _ptr(block_tables), block_tables.shape[1], block_tables.shape[0],
                             _ptr(token_seq), _ptr(token_pos), n, _ptr(k), _ptr(v), _ptr(q),
                             q_heads, flags, _ptr(error), _stream(stream))
    N.check(rc, "tvp_rope_append")


class DecodeWorkspace:
    """Device workspace of the decode path for up to ``max_batch`` rows of a
    pool of ``kv_heads`` KV heads and a fixed grid (``num_ctas`` CTAs, 0 = one
    per SM)."""

    def __init__(self, max_batch: int, device=None, num_ctas: int = 0, kv_heads: int = N.KV_HEADS):
        lib = N.load()
        device = torch.device(device if device is not None else "cuda")
        with torch.cuda.device(device):
            sms = ctypes.c_int(0)
            N.check(lib.tvp_device_sm_count(ctypes.byref(sms)), "tvp_device_sm_count")
            self.num_ctas = num_ctas if num_ctas > 0 else sms.value
            self.nbytes = int(lib.tvp_decode_workspace_bytes(max_batch, kv_heads, self.num_ctas))
        if self.nbytes == 0:
            raise ValueError("invalid workspace request")
        self.max_batch = max_batch
        self.kv_heads = kv_heads
        self.buffer = torch.empty(self.nbytes, dtype=torch.uint8, device=device)
        self.batch = None


def decode_plan(seq_lens, table_stride, workspace: DecodeWorkspace, error=None, stream=None):
    """Plan of one decode step (page prefix sums, split-K counters)."""
    lib = N.load()
    _need(seq_lens, "seq_lens", torch.int32, workspace.buffer.device)
    batch = seq_lens.numel()
    if batch > workspace.max_batch:
        raise ValueError("batch larger than the workspace was sized for")
    workspace.nbytes_needed = int(lib.tvp_decode_workspace_bytes(batch, workspace.kv_heads,
                                                                 workspace.num_ctas))
    rc = lib.tvp_decode_plan(_ptr(seq_lens), batch, table_stride, workspace.kv_heads,
                             workspace.num_ctas,
                             _ptr(workspace.buffer), workspace.nbytes, _ptr(error), _stream(stream))
    N.check(rc, "tvp_decode_plan")
    workspace.batch = batch


def paged_decode_attention(q, k_pool, v_pool, layer, block_tables, seq_lens, workspace=None,
                           out=None, scale=0.125, mode=N.TVP_MODE_FAST, error=None, stream=None):
    """K2: out = softmax(scale q K^T) V over each row's pages, read in place.

    FAST mode needs ``workspace`` planned by :func:`decode_plan` for these lengths.
    """
    lib = N.load()
    num_layers, num_pages, kv_heads = _pool_geometry(k_pool, v_pool)
    dev = k_pool.device
    _need(q, "q", torch.bfloat16, dev)
    _need(block_tables, "block_tables", torch.int32, dev)
    _need(seq_lens, "seq_lens", torch.int32, dev)
    batch = seq_lens.numel()
    if q.shape != (batch, kv_heads * N.GQA_GROUP * N.HEAD_DIM):
        raise ValueError("q must be [batch, 4*kv_heads*64]")
    if block_tables.dim() != 2 or block_tables.shape[0] < batch:
        raise ValueError("block_tables must be [>=batch, table_stride]")
    if out is None:
        out = torch.empty_like(q)
    _need(out, "out", torch.bfloat16, dev)
    ws_ptr, ws_bytes, ctas = None, 0, 0
    if mode == N.TVP_MODE_FAST:
        if workspace is None or workspace.batch != batch:
            raise ValueError("FAST mode needs a workspace planned for this batch")
        if workspace.kv_heads != kv_heads:
            raise ValueError(f"workspace was sized for {workspace.kv_heads} KV heads, pools hold {kv_heads}")
        ws_ptr, ws_bytes, ctas = _ptr(workspace.buffer), workspace.nbytes, workspace.num_ctas
    rc = lib.tvp_paged_decode_attention(_ptr(q), _ptr(k_pool), _ptr(v_pool), num_pages, num_layers,
                                        layer, kv_heads, kv_heads * N.GQA_GROUP,
                                        _ptr(block_tables), block_tables.shape[1], _ptr(seq_lens),
                                        batch, float(scale), mode, ctas, ws_ptr, ws_bytes,
                                        _ptr(out), _ptr(error), _stream(stream))
    N.check(rc, "tvp_paged_decode_attention")
    return out


def paged_prefill_attention(q, k_pool, v_pool, layer, block_tables, cu_q, q_pos0, max_q_len,
                            out=None, scale=0.125, error=None, stream=None):
    """K3: causal prefill attention over the pages.  Sequence s (row s of
    ``block_tables``) owns query rows [cu_q[s], cu_q[s + 1]) of ``q`` at
    positions q_pos0[s], q_pos0[s] + 1, ...; each attends the keys 0..its
    position already in the sequence's pages.  ``max_q_len`` bounds the
    longest sequence's query count (host value, sizes the grid)."""
    lib = N.load()
    num_layers, num_pages, kv_heads = _pool_geometry(k_pool, v_pool)
    dev = k_pool.device
    _need(q, "q", torch.bfloat16, dev)
    _need(block_tables, "block_tables", torch.int32, dev)
    _need(cu_q, "cu_q", torch.int32, dev)
    _need(q_pos0, "q_pos0", torch.int32, dev)
    num_seqs = q_pos0.numel()
    if cu_q.numel() != num_seqs + 1:
        raise ValueError("cu_q must have num_seqs + 1 entries")
    if q.dim() != 2 or q.shape[1] != kv_heads * N.GQA_GROUP * N.HEAD_DIM:
        raise ValueError("q must be [num_tokens, 4*kv_heads*64]")
    if block_tables.dim() != 2 or block_tables.shape[0] < num_seqs:
        raise ValueError("block_tables must be [>=num_seqs, table_stride]")
    if out is None:
        out = torch.empty_like(q)
    _need(out, "out", torch.bfloat16, dev)
    rc = lib.tvp_paged_prefill_attention(_ptr(q), _ptr(k_pool), _ptr(v_pool), num_pages,
                                         num_layers, layer, kv_heads, kv_heads * N.GQA_GROUP,
                                         _ptr(block_tables), block_tables.shape[1], _ptr(cu_q),
                                         _ptr(q_pos0), num_seqs, int(max_q_len), float(scale),
                                         _ptr(out), _ptr(error), _stream(stream))
    N.check(rc, "tvp_paged_prefill_attention")
    return out


def greedy_argmax(logits, out=None, workspace=None, stream=None):
    """Greedy token per row of FP32 logits [rows, vocab] (rows may be strided:
    logits.stride(1) must be 1), with the reference engine's selection rule
    (BF16-rounded logits, NaNs skipped, ties to the lowest index, a NaN logit 0
    selects 0), one launch for all rows.  ``workspace``: a zeroed uint8 tensor
    of tvp_greedy_argmax_workspace_bytes(rows) bytes, reusable across calls
    (each call leaves it zeroed); allocated per call when omitted."""
    lib = N.load()
    if not (logits.is_cuda and logits.dtype == torch.float32):
        raise ValueError("logits must be a CUDA float32 tensor")
    if logits.dim() != 2 or logits.stride(1) != 1 or logits.stride(0) < logits.shape[1]:
        raise ValueError("logits must be [rows, vocab] with unit stride along vocab")
    rows, vocab = logits.shape
    dev = logits.device
    nbytes = lib.tvp_greedy_argmax_workspace_bytes(rows)
    if workspace is None:
        workspace = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    if out is None:
        out = torch.empty(rows, dtype=torch.int32, device=dev)
    _need(out, "out", torch.int32, dev)
    rc = lib.tvp_greedy_argmax(_ptr(logits), rows, vocab, logits.stride(0), _ptr(out),
                               _ptr(workspace), workspace.numel() * workspace.element_size(),
                               _stream(stream))
    N.check(rc, "tvp_greedy_argmax")
    return out


_EPILOGUES = {"bf16": 0, "f32": 1, "residual": 2, "swiglu": 3}


def decode_projections(x, weights, outs=None, epilogue="bf16", stream=None):
    """The decode step's projections of 1-8 rows by up to three weight matrices
    that share them, in one launch: y[i][t] = weights[i] @ x[t].

    x: BF16 [rows, k] (k a multiple of 256); weights[i]: BF16 [n_i, k] (n_i a
    multiple of 16), the reference's weight layout.  FP32 accumulation in a
    fixed order.  ``epilogue``:
      "bf16"      outs[i] = bf16(y[i])                    [rows, n_i] BF16
      "f32"       outs[i] = y[i] (the LM head)            [rows, n_i] FP32
      "residual"  outs[i] += bf16(y[i]) as one BF16 add (residualAdd fused;
                  ``outs`` required: the hidden rows)
      "swiglu"    two weights (gate, up) of one shape; outs = [out]:
                  out = bf16(g (1 / (1 + exp(-g))) u), g, u = bf16(y[0]), bf16(y[1])
    Returns the list of outputs."""
    lib = N.load()
    weights = list(weights)
    if epilogue not in _EPILOGUES:
        raise ValueError(f"epilogue must be one of {sorted(_EPILOGUES)}")
    dev = x.device
    _need(x, "x", torch.bfloat16, dev)
    if x.dim() != 2:
        raise ValueError("x must be [rows, k]")
    rows, k = x.shape
    if not 1 <= len(weights) <= 3:
        raise ValueError("one to three weight matrices")
    for i, w in enumerate(weights):
        _need(w, f"weights[{i}]", torch.bfloat16, dev)
        if w.dim() != 2 or w.shape[1] != k:
            raise ValueError(f"weights[{i}] must be [n, {k}]")
    swiglu = epilogue == "swiglu"
    if swiglu and (len(weights) != 2 or weights[0].shape != weights[1].shape):
        raise ValueError("swiglu takes two weights of one shape (gate, up)")
    shapes = [(rows, weights[0].shape[0])] if swiglu else [(rows, w.shape[0]) for w in weights]
    odt = torch.float32 if epilogue == "f32" else torch.bfloat16
    if outs is None:
        if epilogue == "residual":
            raise ValueError("the residual epilogue needs outs (the rows it adds to)")
        outs = [torch.empty(*sh, dtype=odt, device=dev) for sh in shapes]
    outs = list(outs)
    if len(outs) != len(shapes):
        raise ValueError(f"{len(shapes)} output(s) expected")
    for i, (o, sh) in enumerate(zip(outs, shapes)):
        _need(o, f"outs[{i}]", odt, dev)
        if tuple(o.shape) != sh:
            raise ValueError(f"outs[{i}] must be {list(sh)}")
    cnt = len(weights)
    ptrs = [o.data_ptr() for o in outs] + [None] * (cnt - len(outs))
    wp = (ctypes.c_void_p * cnt)(*[w.data_ptr() for w in weights])
    op = (ctypes.c_void_p * cnt)(*ptrs)
    ns = (ctypes.c_int * cnt)(*[w.shape[0] for w in weights])
    rc = lib.tvp_decode_projections(_ptr(x), rows, k, cnt, wp, ns, op, _EPILOGUES[epilogue],
                                    _stream(stream))
    N.check(rc, "tvp_decode_projections")
    return outs


NORM_SCRATCH_BYTES = 4352  # TVP_NORM_SCRATCH_BYTES


def norm_scratch(device):
    """Device scratch for decode_projection_residual_rmsnorm, zeroed: the
    launch's arrival counter, its error word and the rows' subtree sums."""
    return torch.zeros(NORM_SCRATCH_BYTES // 4, dtype=torch.int32, device=device)


def decode_projection_residual_rmsnorm(x, w, hidden, norm_gain, norm_out, scratch, stream=None):
    """hidden += bf16(w @ x) (the residual epilogue), then in the same launch
    norm_out = rmsnorm(hidden) * norm_gain with the reference kernel's
    arithmetic.  x: BF16 [rows, k]; w: BF16 [2048, k]; hidden, norm_out: BF16
    [rows, 2048]; norm_gain: BF16 [2048]; scratch: from norm_scratch(), reused
    by every call (its element 1 is the error word: TVP_DEVERR_TIMEOUT if the
    launch's CTAs gave up waiting for one another)."""
    lib = N.load()
    dev = x.device
    _need(x, "x", torch.bfloat16, dev)
    _need(w, "w", torch.bfloat16, dev)
    _need(hidden, "hidden", torch.bfloat16, dev)
    _need(norm_gain, "norm_gain", torch.bfloat16, dev)
    _need(norm_out, "norm_out", torch.bfloat16, dev)
    _need(scratch, "scratch", torch.int32, dev)
    if scratch.numel() * 4 < NORM_SCRATCH_BYTES:
        raise ValueError(f"scratch must hold {NORM_SCRATCH_BYTES} bytes (norm_scratch())")
    rows, k = x.shape
    if w.shape != (2048, k) or hidden.shape != (rows, 2048) or norm_out.shape != (rows, 2048) \
            or norm_gain.numel() != 2048:
        raise ValueError("shapes: x [rows, k], w [2048, k], hidden/norm_out [rows, 2048], gain [2048]")
    rc = lib.tvp_decode_projection_residual_rmsnorm(_ptr(x), rows, k, _ptr(w), _ptr(hidden),
                                                    _ptr(norm_gain), _ptr(norm_out), _ptr(scratch),
                                                    _stream(stream))
    N.check(rc, "tvp_decode_projection_residual_rmsnorm")
    return hidden, norm_out


def decode_qkv_rope_append(x, w_q, w_k, w_v, q_out, k_pool, v_pool, layer, block_tables,
                           positions, error=None, stream=None):
    """Q/K/V projections of one decode token per row with RoPE and the paged
    append in the epilogue: q_out = rope(w_q x); rope(w_k x) and w_v x go into
    each row's page slot at its position (tvp_rope_append's arithmetic).
    x: BF16 [rows, k]; w_q [2048, k]; w_k, w_v [512, k]; pools [layers, pages,
    16, 512]; block_tables int32 [rows, stride]; positions int32 [rows]."""
    lib = N.load()
    num_layers, num_pages, kv_heads = _pool_geometry(k_pool, v_pool)
    dev = x.device
    for t, name in ((x, "x"), (w_q, "w_q"), (w_k, "w_k"), (w_v, "w_v"), (q_out, "q_out")):
        _need(t, name, torch.bfloat16, dev)
    _need(block_tables, "block_tables", torch.int32, dev)
    _need(positions, "positions", torch.int32, dev)
    rows, k = x.shape
    if kv_heads != N.KV_HEADS or w_q.shape != (2048, k) or w_k.shape != (512, k) \
            or w_v.shape != (512, k) or q_out.shape != (rows, 2048) or positions.numel() != rows \
            or block_tables.dim() != 2 or block_tables.shape[0] < rows:
        raise ValueError("shapes: x [rows, k], w_q [2048, k], w_k/w_v [512, k], q_out [rows, 2048], "
                         "8-head pools, block_tables [>=rows, stride], positions [rows]")
    rc = lib.tvp_decode_qkv_rope_append(_ptr(x), rows, k, _ptr(w_q), _ptr(w_k), _ptr(w_v),
                                        _ptr(q_out), _ptr(k_pool), _ptr(v_pool), num_pages,
                                        num_layers, layer, _ptr(block_tables),
                                        block_tables.shape[1], _ptr(positions), _ptr(error),
                                        _stream(stream))
    N.check(rc, "tvp_decode_qkv_rope_append")
    return q_out


def decode_down_norm_qkv(x, w_down, hidden, norm_gain, norm_out, scratch, w_q, w_k, w_v, q_out,
                         k_pool, v_pool, layer, block_tables, positions, error=None, stream=None):
    """decode_projection_residual_rmsnorm(x, w_down, hidden, norm_gain, norm_out,
    scratch) followed by decode_qkv_rope_append(norm_out, w_q, w_k, w_v, q_out,
    k_pool, v_pool, layer, block_tables, positions, error), as one launch with
    the same outputs.  Raises RuntimeError (TVP_ERR_UNSUPPORTED) where the
    fused form does not apply; the two calls then do the same work."""
    lib = N.load()
    num_layers, num_pages, kv_heads = _pool_geometry(k_pool, v_pool)
    dev = x.device
    for t, name in ((x, "x"), (w_down, "w_down"), (hidden, "hidden"), (norm_gain, "norm_gain"),
                    (norm_out, "norm_out"), (w_q, "w_q"), (w_k, "w_k"), (w_v, "w_v"),
                    (q_out, "q_out")):
        _need(t, name, torch.bfloat16, dev)
    _need(scratch, "scratch", torch.int32, dev)
    _need(block_tables, "block_tables", torch.int32, dev)
    _need(positions, "positions", torch.int32, dev)
    if scratch.numel() * 4 < NORM_SCRATCH_BYTES:
        raise ValueError(f"scratch must hold {NORM_SCRATCH_BYTES} bytes (norm_scratch())")
    rows, k = x.shape
    if w_down.shape != (2048, k) or hidden.shape != (rows, 2048) or norm_out.shape != (rows, 2048) \
            or norm_gain.numel() != 2048 or kv_heads != N.KV_HEADS or w_q.shape != (2048, 2048) \
            or w_k.shape != (512, 2048) or w_v.shape != (512, 2048) or q_out.shape != (rows, 2048) \
            or positions.numel() != rows or block_tables.dim() != 2 or block_tables.shape[0] < rows:
        raise ValueError("shapes: see decode_projection_residual_rmsnorm and decode_qkv_rope_append")
    rc = lib.tvp_decode_down_norm_qkv(_ptr(x), rows, k, _ptr(w_down), _ptr(hidden), _ptr(norm_gain),
                                      _ptr(norm_out), _ptr(scratch), _ptr(w_q), _ptr(w_k),
                                      _ptr(w_v), _ptr(q_out), _ptr(k_pool), _ptr(v_pool), num_pages,
                                      num_layers, layer, _ptr(block_tables), block_tables.shape[1],
                                      _ptr(positions), _ptr(error), _stream(stream))
    N.check(rc, "tvp_decode_down_norm_qkv")
    return hidden, norm_out, q_out
