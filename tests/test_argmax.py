"""The greedy-token oracle against the reference's own argmax checks
(tests/argmax_test.cu:20-70 of the reference: five BF16 rounding and tie
cases, then NaN / Inf / signed-zero / subnormal cases against its CPU scan),
and the C-ABI entry point's argument checks (no GPU needed)."""
import ctypes
import struct

import numpy as np
import pytest

import oracle
from vllm_b200 import _native as N

VOCAB = 128256
NAN, INF = np.float32(np.nan), np.float32(np.inf)


def f(bits):
    return struct.unpack("<f", struct.pack("<I", bits))[0]


def known_answer_cases():
    """(logits, token) pairs: the reference test's five fixed expectations, then
    its extended cases with the answers its CPU scan gives."""
    s = np.full(VOCAB, -100.0, np.float32)
    cases = [(s.copy(), 0)]
    s[469], s[9928] = 16.497030, 16.497549   # both round to the same BF16: lower index
    cases.append((s.copy(), 469))
    s[9928] = 16.6
    cases.append((s.copy(), 9928))
    s[:] = -100.0
    s[469], s[9928] = 16.5, 16.5625          # halfway: 16.5625 rounds to even, 16.5
    cases.append((s.copy(), 469))
    s[9928] = 16.5626
    cases.append((s.copy(), 9928))
    e = np.full(VOCAB, -INF, np.float32)
    cases.append((e.copy(), 0))                               # all -inf: token 0
    e[255] = e[256] = INF
    cases.append((e.copy(), 255))                             # +inf tie: lower index
    e[0] = NAN
    cases.append((e.copy(), 0))                               # NaN at 0 beats later +inf
    n = np.full(VOCAB, NAN, np.float32)
    cases.append((n.copy(), 0))                               # all NaN
    n[0] = -INF
    cases.append((n.copy(), 0))                               # -inf at 0, NaN elsewhere
    n[700] = n[900] = INF
    cases.append((n.copy(), 700))
    z = np.full(VOCAB, -INF, np.float32)
    z[0], z[1000] = -0.0, 0.0
    cases.append((z.copy(), 0))                               # -0 == +0: lower index
    m = np.zeros(VOCAB, np.float32)
    m[127000], m[128000] = np.finfo(np.float32).max, INF      # FLT_MAX rounds to +inf in BF16
    cases.append((m.copy(), 127000))
    t = np.full(VOCAB, -1.0, np.float32)
    t[0], t[42] = 0.0, f(0x00010000)                          # smallest BF16 subnormal > 0
    cases.append((t.copy(), 42))
    t[:] = -1.0
    t[0], t[42] = -f(0x00010000), -f(0x00000001)              # -denorm_min rounds to -0 > -tiny
    cases.append((t.copy(), 42))
    return cases


def test_oracle_matches_the_reference_known_answers():
    for i, (logits, token) in enumerate(known_answer_cases()):
        got = int(oracle.greedy_argmax(logits)[0])
        assert got == token, (i, got, token)


def test_oracle_matches_a_plain_scan_on_random_bit_patterns():
    """As the reference's 100 random-bit trials, on a shorter row."""
    rng = np.random.default_rng(20261015)
    for _ in range(20):
        x = rng.integers(0, 2**32, size=4096, dtype=np.uint64).astype(np.uint32).view(np.float32)
        b = oracle.bf16_to_f32(oracle.f32_to_bf16(x))
        best, sel = b[0], 0
        for i in range(1, b.size):  # the reference test's CPU scan
            if b[i] > best:
                best, sel = b[i], i
        assert int(oracle.greedy_argmax(x)[0]) == sel


def test_argmax_entry_point_checks_arguments():
    lib = N.load()
    assert lib.tvp_greedy_argmax_workspace_bytes(0) == 0
    need = lib.tvp_greedy_argmax_workspace_bytes(4)
    assert need >= 4 * 8
    p = ctypes.c_void_p(0x1000)
    assert lib.tvp_greedy_argmax(None, 4, VOCAB, VOCAB, p, p, need, None) == N.TVP_ERR_INVALID_ARGUMENT
    assert lib.tvp_greedy_argmax(p, 0, VOCAB, VOCAB, p, p, need, None) == N.TVP_ERR_INVALID_ARGUMENT
    assert lib.tvp_greedy_argmax(p, 4, VOCAB, VOCAB - 1, p, p, need, None) == N.TVP_ERR_INVALID_ARGUMENT
    assert lib.tvp_greedy_argmax(p, 4, VOCAB, VOCAB, p, None, need, None) == N.TVP_ERR_WORKSPACE
    assert lib.tvp_greedy_argmax(p, 4, VOCAB, VOCAB, p, p, need - 1, None) == N.TVP_ERR_WORKSPACE
