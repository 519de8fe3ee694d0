"""dd_decode_paged_static, the decode entry point that allocates nothing.

It exists for callers that cannot allocate device scratch themselves (a plugin
given only input/output pointers by an engine that owns all device memory, or
a decode loop that must not call cudaMalloc). This file is collected last so
that a failure here comes after every other test has run. The test calls the
entry point through the C ABI twice in a row and compares each result with
dd_decode_paged's on the same inputs, within the bf16 tolerances used by the
other parity tests; it also checks that an oversized batch is rejected.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import dendrite_b200 as dd
from dendrite_b200 import _lib
from tests.helpers import assert_close

pytestmark = pytest.mark.gpu


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def _paged_batch(dev, seed, Hq=32, Hkv=8, D=128, P=512):
    rng = np.random.default_rng(seed)
    ntok = np.array([1, 16, 17, 300, 0, 1500, 64, 999], dtype=np.int32)
    perm = rng.permutation(P).astype(np.int32)
    tables, k = [], 0
    for n in ntok:
        nb = -(-int(n) // 16)
        tables.append(perm[k:k + nb])
        k += nb
    indptr = np.cumsum([0] + [len(t) for t in tables]).astype(np.int32)
    ids = np.concatenate(tables).astype(np.int32)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    pool = torch.randn(P, 2, Hkv, 16, D, generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn(len(ntok), Hq, D, generator=g, device=dev).to(torch.bfloat16)
    t = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    cfg = dd.make_config(Hq, Hkv, D, P)
    return cfg, q, pool, t(indptr), t(ids), t(ntok), int(max(len(x) for x in tables))


def _static_call(cfg, q, pool, indptr, ids, ntok, max_pages, out, lse):
    return _lib.lib.dd_decode_paged_static(C.byref(cfg), q.shape[0], max_pages, _ptr(q), _ptr(pool),
                                           None, _ptr(indptr), _ptr(ids), _ptr(ntok), _ptr(out),
                                           _ptr(lse), C.c_void_p(torch.cuda.current_stream().cuda_stream))


def test_static_scratch_matches_workspace_entry_point(cuda):
    for call, seed in enumerate((1, 2)):  # two calls in a row share the static scratch
        cfg, q, pool, indptr, ids, ntok, mp = _paged_batch(cuda, seed)
        ref, ref_lse = dd.decode_paged(cfg, q, pool, indptr, ids, ntok, mp)
        out = torch.full_like(q, float("nan"))
        lse = torch.full((q.shape[0], q.shape[1]), float("nan"), device=cuda)
        _lib.check(_static_call(cfg, q, pool, indptr, ids, ntok, mp, out, lse),
                   "dd_decode_paged_static")
        torch.cuda.synchronize()
        assert_close(out.float().cpu().numpy(), ref.float().cpu().numpy(), what=f"call {call}")
        r, l = ref_lse.cpu().numpy(), lse.cpu().numpy()
        fin = np.isfinite(r)
        assert np.array_equal(fin, np.isfinite(l))
        np.testing.assert_allclose(l[fin], r[fin], atol=1e-5)
        assert torch.all(out[4] == 0)  # the empty table gives zeros


def test_static_scratch_rejects_oversized_batch(cuda):
    Hq, Hkv, D, B = 64, 8, 128, 1024
    cfg = dd.make_config(Hq, Hkv, D, 4)
    z = torch.zeros(B + 1, dtype=torch.int32, device=cuda)
    q = torch.zeros(B, Hq, D, dtype=torch.bfloat16, device=cuda)
    pool = torch.zeros(4, 2, Hkv, 16, D, dtype=torch.bfloat16, device=cuda)
    lse = torch.empty(B, Hq, device=cuda)
    rc = _static_call(cfg, q, pool, z, z, z[:B], 1, q, lse)
    assert rc == _lib.DD_ERR_WORKSPACE
    assert "static scratch" in _lib.lib.dd_last_error().decode()
