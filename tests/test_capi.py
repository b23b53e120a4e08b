"""The C ABI (CPU): the library loads, exports every entry point the header
declares, sizes workspaces and rejects bad problems before touching a GPU."""

import ctypes
import os
import re

import pytest

from flashslice_b200.kernels import _native as nat

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "flashslice_b200.h")


def declared():
    with open(HEADER) as f:
        src = f.read()
    return sorted(set(re.findall(r"FS_API\s+[\w\s\*]+?\b(fs_\w+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared()
    assert {"fs_slice_fwd", "fs_deslice_fwd", "fs_slice_bwd", "fs_deslice_bwd",
            "fs_compute_stats", "fs_workspace_bytes", "fs_last_error", "fs_version"} <= set(names)


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(nat.LIBPATH)
    for name in declared():
        assert hasattr(lib, name), name
    assert set(declared()) <= set(nat.SIGNATURES)
    assert nat.load().fs_version() == nat.ABI_VERSION


def test_struct_layout_matches_header():
    # int64 x6 + int32 x10 + the row_splits pointer
    assert ctypes.sizeof(nat.Problem) == 6 * 8 + 10 * 4 + 8
    assert nat.Problem.row_splits.offset == 6 * 8 + 10 * 4
    assert ctypes.sizeof(nat.Tensor4) == 8 + 4 * 8


def prob(**kw):
    d = dict(B=1, N=1000, H=2, D=32, DV=32, G=32, act_dtype=0, dot=0, family=0, stats_mode=0,
             w_batch=1, w_heads=1, b_batch=1, b_heads=1, flags=0, engine=0)
    d.update(kw)
    return nat.Problem(**d)


def test_workspace_sizes():
    lib = nat.load()
    ws = lambda op, p: lib.fs_workspace_bytes(op, ctypes.byref(p))  # noqa: E731
    assert ws(nat.OP_DESLICE_FWD, prob()) == 0            # fused deslice: no partials
    assert ws(nat.OP_SLICE_FWD, prob()) > 0
    assert ws(nat.OP_STATS, prob()) == 0
    # the blocked family without statistics in hand needs room for them
    blk = prob(family=1, G=256)
    with_stats = ws(nat.OP_SLICE_FWD, prob(family=1, G=256, flags=nat.FLAG_STATS_IN))
    assert ws(nat.OP_SLICE_FWD, blk) >= with_stats + 2 * 2 * 1000 * 4
    # deterministic: a pure function of the problem
    assert ws(nat.OP_SLICE_BWD, blk) == ws(nat.OP_SLICE_BWD, blk)
    assert ws(nat.OP_SLICE_FWD, prob(D=300)) == 0         # invalid problem
    # bf16 points in the bf16 dot mode, G a multiple of 128: room for the
    # tensor-core kernels' operand images, one per (b, h, 64 slots), each
    # 512 + 2 * 4096 + 2 * 64 * DV * 2 bytes
    tc = dict(family=1, G=1024, DV=64, act_dtype=1, dot=3, flags=nat.FLAG_STATS_IN)
    img = 2 * (1024 // 64) * (512 + 2 * 4096 + 2 * 64 * 64 * 2)
    for op in (nat.OP_SLICE_FWD, nat.OP_DESLICE_FWD, nat.OP_SLICE_BWD, nat.OP_DESLICE_BWD):
        assert ws(op, prob(**tc)) >= ws(op, prob(**dict(tc, dot=0))) + img, op


@pytest.mark.parametrize("kw,code", [
    (dict(D=0), nat.FS_ERR_UNSUPPORTED), (dict(D=257), nat.FS_ERR_UNSUPPORTED),
    (dict(DV=300), nat.FS_ERR_UNSUPPORTED), (dict(G=0), nat.FS_ERR_SHAPE),
    (dict(B=0), nat.FS_ERR_SHAPE), (dict(w_heads=3), nat.FS_ERR_SHAPE),
    (dict(b_batch=2), nat.FS_ERR_SHAPE), (dict(act_dtype=7), nat.FS_ERR_ARGUMENT),
    (dict(dot=9), nat.FS_ERR_ARGUMENT), (dict(family=3), nat.FS_ERR_ARGUMENT),
])
def test_bad_problem_rejected_without_gpu(kw, code):
    lib = nat.load()
    p = prob(**kw)
    t = nat.Tensor4(ctypes.c_void_p(16), (ctypes.c_int64 * 4)(0, 0, 0, 1))
    one = ctypes.c_void_p(16)
    rc = lib.fs_slice_fwd(ctypes.byref(p), ctypes.byref(t), ctypes.byref(t), one, one, one, None,
                          None, one, one, None, 0, None)
    assert rc == code
    assert lib.fs_last_error()
    with pytest.raises(ValueError):
        nat.check(rc)


def test_null_pointers_rejected():
    lib = nat.load()
    p = prob()
    t = nat.Tensor4(ctypes.c_void_p(16), (ctypes.c_int64 * 4)(0, 0, 0, 1))
    one = ctypes.c_void_p(16)
    rc = lib.fs_slice_fwd(ctypes.byref(p), ctypes.byref(t), None, one, one, one, None, None, one,
                          one, None, 0, None)
    assert rc == nat.FS_ERR_ARGUMENT and b"fx_mid" in lib.fs_last_error()
    # workspace too small
    rc = lib.fs_slice_fwd(ctypes.byref(p), ctypes.byref(t), ctypes.byref(t), one, one, one, None,
                          None, one, one, one, 8, None)
    assert rc == nat.FS_ERR_WORKSPACE
    # blocked backward without the forward's statistics
    pb = prob(family=1)
    rc = lib.fs_slice_bwd(ctypes.byref(pb), ctypes.byref(t), ctypes.byref(t), one, one, one, None,
                          one, one, ctypes.byref(t), ctypes.byref(t), one, one, one, None, 0, None)
    assert rc == nat.FS_ERR_ARGUMENT


def test_stats_flags_must_match_pointers():
    lib = nat.load()
    p = prob(family=1, flags=nat.FLAG_STATS_IN)
    t = nat.Tensor4(ctypes.c_void_p(16), (ctypes.c_int64 * 4)(0, 0, 0, 1))
    one = ctypes.c_void_p(16)
    rc = lib.fs_slice_fwd(ctypes.byref(p), ctypes.byref(t), ctypes.byref(t), one, one, one, None,
                          None, one, one, None, 0, None)
    assert rc == nat.FS_ERR_ARGUMENT


def test_row_splits_validated_without_gpu():
    """Row splits must run from 0 to N without decreasing; the check needs no
    GPU (fs_coupled_supported reports 0 for a problem that fails it)."""
    import ctypes
    lib = nat.load()
    for splits, ok in (([0, 40, 100], 1), ([0, 60, 40, 100], 0), ([0, 50, 99], 0),
                       ([1, 50, 100], 0)):
        arr = (ctypes.c_int64 * len(splits))(*splits)
        p = prob(B=len(splits) - 1, N=100)
        p.row_splits = ctypes.cast(arr, ctypes.c_void_p)
        assert lib.fs_coupled_supported(ctypes.byref(p)) == ok, splits


def test_wait_selftest_argument_checked_without_gpu():
    lib = nat.load()
    assert lib.fs_selftest_wait_timeout(0, None) == nat.FS_ERR_ARGUMENT
    assert lib.fs_selftest_wait_timeout(3_000_000_000, None) == nat.FS_ERR_ARGUMENT



@pytest.mark.parametrize("kw,codes", [
    (dict(flags=1), (nat.FS_ERR_ARGUMENT,)),                      # statistics handed in
    (dict(flags=2), (nat.FS_ERR_ARGUMENT,)),                      # statistics asked for
    (dict(family=1), (nat.FS_ERR_UNSUPPORTED, nat.FS_ERR_ARGUMENT)),  # blocked family, G <= 32
    (dict(G=64), (nat.FS_ERR_UNSUPPORTED,)),                      # beyond the single-tile family
])
def test_noalloc_refusals_without_gpu(kw, codes):
    """fs_slice_fwd_noalloc refuses, before any launch, what it does not
    serve: statistics in or out, the blocked family, G > 32, ragged rows."""
    lib = nat.load()
    t = nat.Tensor4(ctypes.c_void_p(16), (ctypes.c_int64 * 4)(0, 0, 0, 1))
    one = ctypes.c_void_p(16)
    p = prob(**kw)
    rc = lib.fs_slice_fwd_noalloc(ctypes.byref(p), ctypes.byref(t), ctypes.byref(t), one, one,
                                  one, one, one, None)
    assert rc in codes, (kw, rc)
    assert lib.fs_last_error()


def test_noalloc_refuses_row_splits_without_gpu():
    lib = nat.load()
    t = nat.Tensor4(ctypes.c_void_p(16), (ctypes.c_int64 * 4)(0, 0, 0, 1))
    one = ctypes.c_void_p(16)
    arr = (ctypes.c_int64 * 3)(0, 400, 1000)
    p = prob(B=2)
    p.row_splits = ctypes.cast(arr, ctypes.c_void_p)
    rc = lib.fs_slice_fwd_noalloc(ctypes.byref(p), ctypes.byref(t), ctypes.byref(t), one, one,
                                  one, one, one, None)
    assert rc == nat.FS_ERR_UNSUPPORTED


def test_wait_limit_argument_checked_without_gpu():
    lib = nat.load()
    assert lib.fs_set_wait_limit_ns(3_000_000_000) == nat.FS_ERR_ARGUMENT
    assert lib.fs_set_wait_limit_ns(0) == nat.FS_OK
