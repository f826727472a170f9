"""The allocation-free C entry point of the GQA decode kernel, called through its exported symbol.

Some callers cannot allocate device memory themselves (a pre-sized memory arena, a plugin handed raw pointers, a path
where cudaMalloc must not synchronize or fail), so `iob_gqa_decode_noalloc` keeps the split-K scratch in a fixed device
array inside the library.  This test loads the extension's shared object with ctypes, calls that symbol twice in a row
on a case that needs split-K scratch, and checks each result against the regular (caller-allocated workspace) entry
point.  It also checks that an oversized request is refused without launching.  The file sorts last so that a run
stopping at the first failure has run every other test first.
"""
import ctypes
import math

import pytest
import torch

from inference_optimizations_b200.ops import attention as A
from inference_optimizations_b200.ops import kvcache as K

pytestmark = pytest.mark.gpu


def _lib():
    from inference_optimizations_b200._ext import ext
    mod = ext()
    path = getattr(mod, "__file__", None) or getattr(getattr(mod, "_m", None), "__file__")
    lib = ctypes.CDLL(path)
    fn = lib.iob_gqa_decode_noalloc
    fn.restype = ctypes.c_int
    # q, pool, page_table | pt_stride | req_idx, kv_len, out | B, n_q, Hq, Hk, D, window, fmt, tiles_per_split,
    # num_splits | sm_scale, k_scale, v_scale | exact | stream
    fn.argtypes = ([ctypes.c_void_p] * 3 + [ctypes.c_int] + [ctypes.c_void_p] * 3 + [ctypes.c_int] * 9
                   + [ctypes.c_float] * 3 + [ctypes.c_int, ctypes.c_void_p])
    lib.iob_gqa_decode_noalloc_status.restype = ctypes.c_int
    lib.iob_gqa_decode_noalloc_status.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.c_void_p]
    lib.iob_gqa_decode_noalloc_strerror.restype = ctypes.c_char_p
    lib.iob_gqa_decode_noalloc_strerror.argtypes = [ctypes.c_int]
    return lib


def _pool(cuda, fmt, d, hk, lens, seed=11):
    g = torch.Generator().manual_seed(seed)
    per = max((n + 63) // 64 for n in lens)
    n_pages = len(lens) * per + 2
    pt = (torch.randperm(n_pages - 1, generator=g)[: len(lens) * per] + 1).reshape(len(lens), per).int()
    pool = torch.zeros(n_pages, hk, 2, K.part_bytes(fmt, d), dtype=torch.uint8)
    for i, n in enumerate(lens):
        k = torch.randn(n, hk, d, generator=g).to(torch.bfloat16).float()
        v = torch.randn(n, hk, d, generator=g).to(torch.bfloat16).float()
        pos = torch.arange(n)
        K.gqa_pool_write_ref(pool, pt[i][pos // 64].long() * 64 + pos % 64, k, v, fmt)
    return pool.to(cuda), pt.to(cuda), torch.tensor(lens, dtype=torch.int32, device=cuda)


@pytest.mark.parametrize("exact", [False, True])
def test_noalloc_entry_point_matches_allocating_one(cuda, exact):
    lib = _lib()
    hq, hk, d, n_q = 4, 2, 512, 1
    lens = [3000, 1900, 2500]
    fmt = K.FMT_NVFP4
    pool, pt, kv_len = _pool(cuda, fmt, d, hk, lens)
    q = torch.randn(len(lens) * n_q, hq, d, device=cuda).to(torch.bfloat16)
    sm = 1.0 / math.sqrt(d)
    splits = A.split_policy(len(lens) * hk, max(lens))
    assert splits[0] > 1, splits          # the case must exercise the split-K scratch
    ref = A.gqa_decode(q, pool, pt, kv_len, n_q, hk, fmt, sm, splits=splits, exact=exact)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):                     # two calls in a row share (and must reset) the same scratch
        out = torch.full_like(q, float("nan"))
        rc = lib.iob_gqa_decode_noalloc(q.data_ptr(), pool.data_ptr(), pt.data_ptr(), pt.shape[1], None,
                                        kv_len.data_ptr(), out.data_ptr(), len(lens), n_q, hq, hk, d, 0, fmt,
                                        splits[1], splits[0], sm, 1.0, 1.0, int(exact), stream)
        assert rc == 0, lib.iob_gqa_decode_noalloc_strerror(rc)
        status = ctypes.c_int(-7)
        rc = lib.iob_gqa_decode_noalloc_status(ctypes.byref(status), stream)
        assert rc == 0 and status.value == 0, (rc, status.value)
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        assert (out.float() - ref.float()).abs().max().item() < 2e-2


def test_noalloc_entry_point_rejects_oversized_workspace(cuda):
    lib = _lib()
    hq, hk, d = 4, 2, 512
    q = torch.zeros(1024, hq, d, device=cuda, dtype=torch.bfloat16)
    out = torch.zeros_like(q)
    kv_len = torch.full((1024,), 4096, dtype=torch.int32, device=cuda)
    pt = torch.zeros(1024, 64, dtype=torch.int32, device=cuda)
    pool = torch.zeros(1, hk, 2, K.part_bytes(K.FMT_NVFP4, d), dtype=torch.uint8, device=cuda)
    rc = lib.iob_gqa_decode_noalloc(q.data_ptr(), pool.data_ptr(), pt.data_ptr(), 64, None, kv_len.data_ptr(),
                                    out.data_ptr(), 1024, 1, hq, hk, d, 0, K.FMT_NVFP4, 1, 32, 0.05, 1.0, 1.0, 0,
                                    torch.cuda.current_stream().cuda_stream)
    assert rc == -1
    assert b"built-in scratch" in lib.iob_gqa_decode_noalloc_strerror(rc)
    torch.cuda.synchronize()
    assert (out == 0).all()                 # nothing was launched
