"""The C-ABI library: loads, exports every declared symbol, rejects bad
arguments on the host before touching the device (no GPU needed)."""
import ctypes

import pytest

from vllm_b200 import _native as N


def test_library_exports_every_declared_symbol(native):
    declared = N.declared_symbols()
    assert len(declared) >= 30
    missing = [name for name in declared if not hasattr(native, name)]
    assert not missing, f"declared in include/tvp_paged.h but not exported: {missing}"


def test_every_declared_symbol_has_a_binding():
    assert set(N.declared_symbols()) == set(N._SIGNATURES)


def test_strerror_and_version(native):
    assert native.tvp_version() == 1
    assert native.tvp_strerror(N.TVP_OK) == b"ok"
    assert b"invalid" in native.tvp_strerror(N.TVP_ERR_INVALID_ARGUMENT)
    assert b"free blocks" in native.tvp_strerror(N.TVP_ERR_NO_FREE_BLOCKS)


def test_rope_append_rejects_bad_arguments_on_host(native):
    # Null pools / tables: refused before any CUDA call.
    rc = native.tvp_rope_append(None, None, 8, 16, 0, 8, None, 4, 1, None, None, 1, None, None,
                                None, 32, 0, None, None)
    assert rc == N.TVP_ERR_INVALID_ARGUMENT
    fake = ctypes.c_void_p(0x10000)
    # layer out of range
    rc = native.tvp_rope_append(fake, fake, 8, 16, 16, 8, fake, 4, 1, None, fake, 1, fake, fake,
                                None, 32, 0, None, None)
    assert rc == N.TVP_ERR_INVALID_ARGUMENT
    # unknown flag bit
    rc = native.tvp_rope_append(fake, fake, 8, 16, 0, 8, fake, 4, 1, None, fake, 1, fake, fake,
                                None, 32, 64, None, None)
    assert rc == N.TVP_ERR_INVALID_ARGUMENT
    # q rope requested without q
    rc = native.tvp_rope_append(fake, fake, 8, 16, 0, 8, fake, 4, 1, None, fake, 1, fake, fake,
                                None, 32, N.TVP_APPEND_ROPE_Q, None, None)
    assert rc == N.TVP_ERR_INVALID_ARGUMENT
    # misaligned v
    rc = native.tvp_rope_append(fake, fake, 8, 16, 0, 8, fake, 4, 1, None, fake, 1, fake,
                                ctypes.c_void_p(0x10002), None, 32, 0, None, None)
    assert rc == N.TVP_ERR_INVALID_ARGUMENT
    # zero tokens is a no-op
    rc = native.tvp_rope_append(fake, fake, 8, 16, 0, 8, fake, 4, 1, None, fake, 0, fake, fake,
                                None, 32, 0, None, None)
    assert rc == N.TVP_OK


def test_decode_rejects_bad_arguments_on_host(native):
    fake = ctypes.c_void_p(0x10000)
    args = dict(q=fake, k=fake, v=fake, pages=8, layers=16, layer=0, kvh=8, qh=32, tables=fake,
                stride=4, lens=fake, batch=2, scale=0.125, mode=0, ctas=148, ws=fake, wsb=1 << 30,
                out=fake, err=None, stream=None)

    def call(**over):
        a = dict(args, **over)
        return native.tvp_paged_decode_attention(a["q"], a["k"], a["v"], a["pages"], a["layers"],
                                                 a["layer"], a["kvh"], a["qh"], a["tables"],
                                                 a["stride"], a["lens"], a["batch"], a["scale"],
                                                 a["mode"], a["ctas"], a["ws"], a["wsb"], a["out"],
                                                 a["err"], a["stream"])

    assert call(q=None) == N.TVP_ERR_INVALID_ARGUMENT
    assert call(layer=16) == N.TVP_ERR_INVALID_ARGUMENT
    assert call(batch=0) == N.TVP_ERR_INVALID_ARGUMENT
    assert call(scale=float("nan")) == N.TVP_ERR_INVALID_ARGUMENT
    assert call(kvh=3, qh=12) == N.TVP_ERR_UNSUPPORTED   # head shards are 1, 2, 4 or 8 heads
    assert call(kvh=16, qh=64) == N.TVP_ERR_UNSUPPORTED
    assert call(qh=16) == N.TVP_ERR_UNSUPPORTED          # q heads must be 4 per KV head
    assert call(kvh=4, qh=32) == N.TVP_ERR_UNSUPPORTED
    assert call(mode=7) == N.TVP_ERR_UNSUPPORTED
    assert call(ws=None) == N.TVP_ERR_WORKSPACE
    assert call(wsb=16) == N.TVP_ERR_WORKSPACE
    assert call(out=ctypes.c_void_p(0x10008)) == N.TVP_ERR_INVALID_ARGUMENT


def test_prefill_rejects_bad_arguments_on_host(native):
    fake = ctypes.c_void_p(0x10000)
    args = dict(q=fake, k=fake, v=fake, pages=8, layers=16, layer=0, kvh=8, qh=32, tables=fake,
                stride=4, cu=fake, pos0=fake, seqs=2, maxq=64, scale=0.125, out=fake, err=None,
                stream=None)

    def call(**over):
        a = dict(args, **over)
        return native.tvp_paged_prefill_attention(a["q"], a["k"], a["v"], a["pages"], a["layers"],
                                                  a["layer"], a["kvh"], a["qh"], a["tables"],
                                                  a["stride"], a["cu"], a["pos0"], a["seqs"],
                                                  a["maxq"], a["scale"], a["out"], a["err"],
                                                  a["stream"])

    assert call(q=None) == N.TVP_ERR_INVALID_ARGUMENT
    assert call(cu=None) == N.TVP_ERR_INVALID_ARGUMENT
    assert call(layer=16) == N.TVP_ERR_INVALID_ARGUMENT
    assert call(seqs=0) == N.TVP_ERR_INVALID_ARGUMENT
    assert call(seqs=65536) == N.TVP_ERR_INVALID_ARGUMENT    # one grid row per sequence
    assert call(maxq=-1) == N.TVP_ERR_INVALID_ARGUMENT
    assert call(maxq=65535 * 32 + 1) == N.TVP_ERR_UNSUPPORTED  # 32-token tiles beyond the grid
    assert call(scale=float("inf")) == N.TVP_ERR_INVALID_ARGUMENT
    assert call(kvh=3, qh=12) == N.TVP_ERR_UNSUPPORTED
    assert call(qh=16) == N.TVP_ERR_UNSUPPORTED
    # q and output rows move as 16-byte vectors
    assert call(q=ctypes.c_void_p(0x10004)) == N.TVP_ERR_INVALID_ARGUMENT
    assert call(out=ctypes.c_void_p(0x10008)) == N.TVP_ERR_INVALID_ARGUMENT
    assert call(k=ctypes.c_void_p(0x10008)) == N.TVP_ERR_INVALID_ARGUMENT
    assert call(maxq=0) == N.TVP_OK                         # nothing to attend: no launch


def test_workspace_size_grows_with_batch_and_grid(native):
    a = native.tvp_decode_workspace_bytes(4, 8, 148)
    b = native.tvp_decode_workspace_bytes(256, 8, 148)
    c = native.tvp_decode_workspace_bytes(256, 8, 296)
    assert 0 < a < b < c
    assert a % 256 == 0
    assert native.tvp_decode_workspace_bytes(0, 8, 148) == 0
    assert native.tvp_decode_workspace_bytes(4, 3, 148) == 0
    assert native.tvp_decode_workspace_bytes(4, 16, 148) == 0
    # per CTA: a 16-byte start record and 2 partial slots x 8 KV heads x (4 + 4 + 256) floats
    # (regions are rounded up to 256 bytes)
    assert c - b >= 148 * (16 + 2 * 8 * 264 * 4) - 256
    # a head shard's workspace holds counters and partials for its heads only
    sizes = [native.tvp_decode_workspace_bytes(256, h, 148) for h in (1, 2, 4, 8)]
    assert 0 < sizes[0] < sizes[1] < sizes[2] < sizes[3] == b


def test_python_layer_maps_codes_to_reference_exceptions():
    with pytest.raises(ValueError):
        N.check(N.TVP_ERR_INVALID_ARGUMENT)
    with pytest.raises(N.TvpNoFreeBlocks):
        N.check(N.TVP_ERR_NO_FREE_BLOCKS)
    with pytest.raises(N.TvpError):
        N.check(N.TVP_ERR_RUNTIME)
    assert N.check(3) == 3


def test_cxx_header_compiles_against_c_header(tmp_path):
    """include/tvp_paged.h is plain C (no C++ or torch types)."""
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    src = tmp_path / "t.c"
    src.write_text("#include \"tvp_paged.h\"\nint main(void){return tvp_version() == 0;}\n")
    subprocess.run([gcc, "-std=c99", "-Wall", "-Werror", "-I", str(N.HEADER_PATH.parent), "-c",
                    str(src), "-o", str(tmp_path / "t.o")], check=True)


def test_head_gather_rejects_bad_arguments_on_host(native):
    h = ctypes.c_void_p()
    assert native.tvp_head_gather_create(3, 0, 2, 16, ctypes.byref(h)) == N.TVP_ERR_UNSUPPORTED
    assert native.tvp_head_gather_create(2, 0, 2, 16, ctypes.byref(h)) == N.TVP_ERR_UNSUPPORTED
    assert native.tvp_head_gather_create(2, 2, 4, 16, ctypes.byref(h)) == N.TVP_ERR_INVALID_ARGUMENT
    assert native.tvp_head_gather_create(2, 0, 4, 0, ctypes.byref(h)) == N.TVP_ERR_INVALID_ARGUMENT
    assert native.tvp_head_gather_create(2, 0, 4, 16, None) == N.TVP_ERR_INVALID_ARGUMENT
    assert native.tvp_head_gather_destroy(None) == N.TVP_ERR_INVALID_ARGUMENT
    fake = ctypes.c_void_p(0x10000)
    assert native.tvp_paged_decode_attention_gather(
        fake, fake, fake, 8, 1, 0, 4, 16, fake, 4, fake, 2, 0.125, 148, fake, 1 << 20, None, 0,
        None, None) == N.TVP_ERR_INVALID_ARGUMENT


def test_noalloc_checks_every_argument_and_its_limit_on_host(native):
    """The no-allocation decode refuses bad arguments before it enqueues
    anything (so a rejected call leaves its shared device array untouched),
    and refuses a batch whose workspace exceeds its fixed 4 MiB array.  With
    148 CTAs the limit falls between 46,968 and 46,969 rows at 8 KV heads and
    between 147,056 and 147,057 rows at 4 KV heads.  Every case returns before
    any CUDA call (fake, never dereferenced pointers; no GPU needed)."""
    fake = ctypes.c_void_p(0x10000)
    args = dict(q=fake, k=fake, v=fake, pages=8, layers=16, layer=0, kvh=8, qh=32, tables=fake,
                stride=4, lens=fake, batch=2, scale=0.125, ctas=148, out=fake, err=None,
                stream=None)

    def call(**over):
        a = dict(args, **over)
        return native.tvp_paged_decode_attention_noalloc(
            a["q"], a["k"], a["v"], a["pages"], a["layers"], a["layer"], a["kvh"], a["qh"],
            a["tables"], a["stride"], a["lens"], a["batch"], a["scale"], a["ctas"], a["out"],
            a["err"], a["stream"])

    assert call(q=None) == N.TVP_ERR_INVALID_ARGUMENT
    assert call(out=None) == N.TVP_ERR_INVALID_ARGUMENT
    assert call(k=None) == N.TVP_ERR_INVALID_ARGUMENT
    assert call(layer=16) == N.TVP_ERR_INVALID_ARGUMENT
    assert call(batch=0) == N.TVP_ERR_INVALID_ARGUMENT
    assert call(ctas=-1) == N.TVP_ERR_INVALID_ARGUMENT
    assert call(scale=float("nan")) == N.TVP_ERR_INVALID_ARGUMENT
    assert call(qh=16) == N.TVP_ERR_UNSUPPORTED
    assert call(kvh=3, qh=12) == N.TVP_ERR_UNSUPPORTED
    assert call(out=ctypes.c_void_p(0x10008)) == N.TVP_ERR_INVALID_ARGUMENT
    assert call(k=ctypes.c_void_p(0x10008)) == N.TVP_ERR_INVALID_ARGUMENT

    limit = 4 << 20
    for heads, rows in ((8, 46_968), (4, 147_056)):
        assert native.tvp_decode_workspace_bytes(rows, heads, 148) <= limit
        assert native.tvp_decode_workspace_bytes(rows + 1, heads, 148) > limit
        assert call(kvh=heads, qh=4 * heads, batch=rows + 1) == N.TVP_ERR_WORKSPACE


def test_fused_projection_forms_reject_bad_arguments_on_host(native):
    fake = ctypes.c_void_p(0x10000)
    odd = ctypes.c_void_p(0x10008)
    f = native.tvp_decode_projection_residual_rmsnorm
    hid, out, scr = ctypes.c_void_p(0x20000), ctypes.c_void_p(0x30000), ctypes.c_void_p(0x50000)
    assert f(None, 4, 2048, fake, hid, fake, out, scr, None) == N.TVP_ERR_INVALID_ARGUMENT
    assert f(fake, 9, 2048, fake, hid, fake, out, scr, None) == N.TVP_ERR_INVALID_ARGUMENT  # rows 1..8
    assert f(fake, 4, 100, fake, hid, fake, out, scr, None) == N.TVP_ERR_INVALID_ARGUMENT   # k % 256
    assert f(fake, 4, 2048, fake, hid, fake, odd, scr, None) == N.TVP_ERR_INVALID_ARGUMENT  # alignment
    assert f(fake, 4, 2048, fake, hid, fake, hid, scr, None) == N.TVP_ERR_INVALID_ARGUMENT  # norm_out on hidden
    assert f(fake, 4, 2048, fake, hid, fake, out, None, None) == N.TVP_ERR_INVALID_ARGUMENT  # no scratch
    assert f(fake, 4, 2048, fake, hid, fake, out, ctypes.c_void_p(0x50008),
             None) == N.TVP_ERR_INVALID_ARGUMENT                                          # scratch alignment
    assert f(fake, 4, 2048, fake, hid, fake, out, ctypes.c_void_p(0x21000),
             None) == N.TVP_ERR_INVALID_ARGUMENT                                          # scratch on hidden
    g = native.tvp_decode_qkv_rope_append
    args = [fake, 4, 2048, fake, fake, fake, ctypes.c_void_p(0x40000), fake, fake, 8, 16, 0, fake, 4,
            fake, None, None]
    assert g(*args[:11], 16, *args[12:]) == N.TVP_ERR_INVALID_ARGUMENT  # layer out of range
    assert g(*args[:1], 0, *args[2:]) == N.TVP_ERR_INVALID_ARGUMENT     # no rows
    assert g(*args[:13], 0, *args[14:]) == N.TVP_ERR_INVALID_ARGUMENT   # table stride
    assert g(*args[:3], odd, *args[4:]) == N.TVP_ERR_INVALID_ARGUMENT   # weight alignment


def test_down_norm_qkv_rejects_bad_arguments_on_host(native):
    f = native.tvp_decode_down_norm_qkv
    v = ctypes.c_void_p
    x, wd, hid, gain, out, scr = v(0x100000), v(0x200000), v(0x300000), v(0x400000), v(0x500000), v(0x600000)
    wq, wk, wv, q, kp, vp, tab, pos = (v(0x700000), v(0x800000), v(0x900000), v(0xa00000),
                                       v(0xb00000), v(0xc00000), v(0xd00000), v(0xe00000))
    ok = [x, 4, 8192, wd, hid, gain, out, scr, wq, wk, wv, q, kp, vp, 8, 16, 0, tab, 64, pos, None, None]

    def call(**kw):
        args = list(ok)
        for i, val in kw.items():
            args[int(i[1:])] = val
        return f(*args)
    assert call(a0=None) == N.TVP_ERR_INVALID_ARGUMENT              # no x
    assert call(a1=9) == N.TVP_ERR_INVALID_ARGUMENT                 # rows 1..8
    assert call(a7=None) == N.TVP_ERR_INVALID_ARGUMENT              # no scratch
    assert call(a6=hid) == N.TVP_ERR_INVALID_ARGUMENT               # norm_out on hidden
    assert call(a11=None) == N.TVP_ERR_INVALID_ARGUMENT             # no q_out
    assert call(a16=16) == N.TVP_ERR_INVALID_ARGUMENT               # layer out of range
    assert call(a11=v(0x500000)) == N.TVP_ERR_INVALID_ARGUMENT      # q_out on norm_out
