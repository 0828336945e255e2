"""The allocation-free KV commit (vc_kv_commit_noalloc) against vc_kv_commit.

It serves callers that cannot allocate device memory while committing, so
it keeps its scratch in a fixed array inside the library.  Checked here
through the C ABI: two calls in a row (the second reuses the scratch the
first left behind) must give the same kv_roots, bit for bit, as the
allocating entry point; sizes beyond the fixed maximum are refused with a
clear error.  This file is collected last, and passes alone in a fresh
process as well as after the other tests.
"""
import ctypes

import numpy as np
import pytest
import torch

from commitllm_b200 import _lib
from commitllm_b200 import commit as C
from tests import kvref

pytestmark = pytest.mark.gpu


def _noalloc(view, stream):
    d, keep = C._kv_desc(view)
    roots = torch.zeros(d.n_seqs, d.n_layers, 32, dtype=torch.uint8, device=view.k_layers[0].device)
    flag = torch.zeros(1, dtype=torch.int32, device=view.k_layers[0].device)
    _lib.check(_lib.lib().vc_kv_commit_noalloc(ctypes.byref(d), ctypes.c_void_p(roots.data_ptr()),
                                               ctypes.c_void_p(flag.data_ptr()), ctypes.c_void_p(stream.cuda_stream)))
    del keep
    return roots, flag


def test_noalloc_matches_kv_commit_two_calls(ctx):
    stream = torch.cuda.current_stream(ctx.device)
    cases = [kvref.paged(501, 3, [300, 1, 129, 4096], 8, 128, block_size=16),   # ragged paged batch
             kvref.contiguous(502, 4, [1000, 37], 2, 64)]                         # contiguous, another shape
    for tr in cases:
        view = tr.view(ctx.device)
        want, _ = C.kv_commit(ctx, view, keep_trees=False)
        r1, f1 = _noalloc(view, stream)
        r2, f2 = _noalloc(view, stream)
        torch.cuda.synchronize()
        assert torch.equal(r1, want)
        assert torch.equal(r2, want)
        assert int(f1.item()) == 0 and int(f2.item()) == 0


def test_noalloc_matches_oracle():
    tr = kvref.contiguous(503, 2, [77, 5], 1, 16)
    view = tr.view(0)
    r, _ = _noalloc(view, torch.cuda.current_stream(0))
    torch.cuda.synchronize()
    oroots, _ = tr.oracle(with_nodes=False)
    assert np.array_equal(r.cpu().numpy(), oroots)


def test_noalloc_rejects_sizes_beyond_its_maximum():
    # 65 sequences: one more than the fixed per-call maximum
    tr = kvref.contiguous(504, 1, [2] * 65, 1, 8)
    with pytest.raises(_lib.VcValueError, match="at most 64 sequences"):
        _noalloc(tr.view(0), torch.cuda.current_stream(0))
    # scratch: 64 sequences x 256 layers of 2^16 positions needs far more than 8 MiB
    tr2 = kvref.contiguous(505, 1, [1], 1, 8)
    view = tr2.view(0)
    d, keep = C._kv_desc(view)
    lens = (ctypes.c_int32 * 64)(*([1 << 16] * 64))
    d.n_seqs = 64
    d.seq_lens = ctypes.cast(lens, ctypes.POINTER(ctypes.c_int32))
    d.block_tables = None
    d.cache_elems = 1 << 40   # host-side row checks pass; the scratch limit must refuse first
    kp = (ctypes.c_void_p * 256)(*([view.k_layers[0].data_ptr()] * 256))
    d.n_layers = 256
    d.k_layers = ctypes.cast(kp, ctypes.POINTER(ctypes.c_void_p))
    d.v_layers = ctypes.cast(kp, ctypes.POINTER(ctypes.c_void_p))
    roots = torch.zeros(1, dtype=torch.uint8, device="cuda")
    st = _lib.lib().vc_kv_commit_noalloc(ctypes.byref(d), ctypes.c_void_p(roots.data_ptr()), None, None)
    assert st == _lib.VC_EINVAL
    assert "bytes of scratch" in _lib.last_error()


def test_noalloc_flags_bad_page_ids(ctx):
    """A block table holding -1 and a page past the cache: the kernel checks
    each page id before it reads the page, skips the row and sets the flag,
    so the caller learns that the roots of this call are void."""
    stream = torch.cuda.current_stream(ctx.device)
    tr = kvref.paged(506, 2, [40, 33], 2, 64, block_size=16)
    n_pages = tr.k.shape[1]
    bt = tr.block_tables.copy()
    bt[0, 1] = -1
    bt[1, 0] = n_pages + 5
    tr.block_tables = bt
    view = tr.view(ctx.device)
    _, flag = _noalloc(view, stream)
    torch.cuda.synchronize()
    assert int(flag.item()) == 1
    # the same table through the allocating entry point reports VC_ERANGE
    C.kv_commit(ctx, view, keep_trees=False)
    with pytest.raises(_lib.VcValueError):
        ctx.sync(timeout_ms=60000)


def test_noalloc_refuses_paged_layout_without_flag():
    tr = kvref.paged(507, 1, [20], 2, 64, block_size=16)
    view = tr.view(0)
    d, keep = C._kv_desc(view)
    roots = torch.zeros(1, 1, 32, dtype=torch.uint8, device="cuda:0")
    st = _lib.lib().vc_kv_commit_noalloc(ctypes.byref(d), ctypes.c_void_p(roots.data_ptr()), None, None)
    assert st == _lib.VC_EINVAL
    assert "err_flag_dev" in _lib.last_error()
    del keep
