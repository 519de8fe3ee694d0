"""GPU decode-step KV writes: dd_append_kv_batch (with FP8 quantization fused)
and dd_copy_pages (copy-on-write data copy), against the oracle, and a
fork + copy-on-write + append step decoded through the cascade."""
import numpy as np
import pytest
import torch

import dendrite_b200 as dd
import oracle
from dendrite_b200 import _lib
from tests.helpers import assert_close, bf16_bits, bits_to_f32, random_pool

pytestmark = pytest.mark.gpu

HKV, D, P = 4, 128, 64


def _targets(rng, n):
    flat = rng.choice(P * 16, size=n, replace=False)   # distinct (page, slot)
    return (flat // 16).astype(np.uint32), (flat % 16).astype(np.int32)


def _dev(x, cuda):
    return torch.from_numpy(np.ascontiguousarray(x)).to(cuda)


def _bf16_dev(bits, cuda):
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(cuda)


@pytest.mark.parametrize("pool_dtype", ["bf16", "f32", "e4m3", "mxfp8"])
@pytest.mark.parametrize("src", ["bf16", "f32"])
def test_append_batch_vs_oracle(cuda, pool_dtype, src):
    rng = np.random.default_rng(7)
    n = 200
    pages, slots = _targets(rng, n)
    kx = rng.standard_normal((n, HKV, D)).astype(np.float32) * 3
    vx = rng.standard_normal((n, HKV, D)).astype(np.float32) * 3
    kx[::17] *= 60.0                                   # outliers: saturation / large exponents
    if src == "bf16":
        kx, vx = bits_to_f32(bf16_bits(kx)), bits_to_f32(bf16_bits(vx))
        kd, vd = _bf16_dev(bf16_bits(kx), cuda), _bf16_dev(bf16_bits(vx), cuda)
    else:
        kd, vd = _dev(kx, cuda), _dev(vx, cuda)
    kvd = {"bf16": _lib.DTYPE_BF16, "f32": _lib.DTYPE_F32, "e4m3": _lib.DTYPE_E4M3,
           "mxfp8": _lib.DTYPE_MXFP8}[pool_dtype]
    cfg = dd.make_config(8, HKV, D, P, kv_dtype=kvd)
    shape = (P, 2, HKV, 16, D)
    if pool_dtype in ("bf16", "f32"):
        pool = torch.zeros(shape, dtype=torch.bfloat16 if pool_dtype == "bf16" else torch.float32, device=cuda)
        scales = None
    else:
        pool = torch.zeros(shape, dtype=torch.uint8, device=cuda)
        if pool_dtype == "e4m3":
            scales_np = (rng.random((2, HKV)).astype(np.float32) * 0.02 + 0.005)
            scales = _dev(scales_np, cuda)
        else:
            scales = torch.zeros((P, 2, HKV, 16, D // 32), dtype=torch.uint8, device=cuda)
    status = torch.zeros(2, dtype=torch.int32, device=cuda)
    dd.append_kv_batch(cfg, pool, scales, _dev(pages, cuda), _dev(slots, cuda), kd, vd, status=status)
    torch.cuda.synchronize()
    assert status.cpu().tolist() == [0, 0]
    got = pool.cpu()
    for which, x in ((0, kx), (1, vx)):
        rows = got[pages, which, :, slots]              # [n, HKV, D]
        if pool_dtype == "f32":
            assert np.array_equal(rows.numpy(), x)
        elif pool_dtype == "bf16":
            assert np.array_equal(rows.view(torch.int16).numpy().view(np.uint16), bf16_bits(x))
        elif pool_dtype == "e4m3":
            want = oracle.e4m3_encode(x / scales_np[which][None, :, None])
            assert np.array_equal(rows.numpy(), want)
        else:
            want_c, want_s = oracle.quantize_mx(x.reshape(n * HKV, 1, 1, 1, D))
            assert np.array_equal(rows.numpy(), want_c.reshape(n, HKV, D))
            got_s = scales.cpu()[pages, which, :, slots]
            assert np.array_equal(got_s.numpy(), want_s.reshape(n, HKV, D // 32))
    # untouched slots stay zero
    mask = np.ones((P, 16), bool)
    mask[pages, slots] = False
    assert not got.reshape(P, 2, HKV, 16, D).permute(0, 3, 1, 2, 4)[torch.from_numpy(mask)].any()


def test_append_reports_bad_targets(cuda):
    cfg = dd.make_config(8, HKV, D, P)
    pool = torch.zeros((P, 2, HKV, 16, D), dtype=torch.bfloat16, device=cuda)
    k = torch.ones((3, HKV, D), dtype=torch.bfloat16, device=cuda)
    pages = torch.tensor([1, P + 3, 2], dtype=torch.int32, device=cuda)
    slots = torch.tensor([0, 0, 16], dtype=torch.int32, device=cuda)
    status = torch.zeros(2, dtype=torch.int32, device=cuda)
    dd.append_kv_batch(cfg, pool, None, pages, slots, k, k, status=status)
    torch.cuda.synchronize()
    st = status.cpu().tolist()
    assert st[0] == 1 and st[1] in (1, 2)
    assert pool[1, :, :, 0].float().eq(1).all() and pool[2].float().eq(0).all()


@pytest.mark.parametrize("fmt", ["bf16", "mxfp8"])
def test_copy_pages(cuda, fmt):
    rng = np.random.default_rng(3)
    bits = bf16_bits(random_pool(rng, P, HKV, D))
    src_pool = _bf16_dev(bits, cuda)
    if fmt == "bf16":
        cfg = dd.make_config(8, HKV, D, P)
        pool, scales = src_pool.clone(), None
    else:
        cfg = dd.make_config(8, HKV, D, P, kv_dtype=_lib.DTYPE_MXFP8)
        pool, scales = dd.quantize_kv_pages(src_pool, "mxfp8")
    before = pool.clone()
    sb = scales.clone() if scales is not None else None
    src = torch.tensor([3, 5, 7, 7], dtype=torch.int32, device=cuda)
    dst = torch.tensor([10, 11, 12, 7], dtype=torch.int32, device=cuda)
    dd.copy_pages(cfg, pool, scales, src, dst)
    torch.cuda.synchronize()
    want = before.clone()
    want[[10, 11, 12]] = before[[3, 5, 7]]
    assert torch.equal(pool, want)
    if scales is not None:
        ws = sb.clone()
        ws[[10, 11, 12]] = sb[[3, 5, 7]]
        assert torch.equal(scales, ws)


def test_fork_copy_on_write_append_decode(cuda):
    """A branch forked from a sequence whose last page is partial: the shared
    partial page is copied (copy-on-write), both branches append a different
    token, and the cascade decode of both matches the oracle."""
    rng = np.random.default_rng(11)
    Hq = 8
    bits = bf16_bits(random_pool(rng, P, HKV, D))
    pool = _bf16_dev(bits, cuda)
    cfg = dd.make_config(Hq, HKV, D, P)
    # parent: pages 0..4, 70 tokens (last page 4 holds 6 tokens)
    parent = np.array([0, 1, 2, 3, 4], np.uint32)
    child = np.array([0, 1, 2, 3, 9], np.uint32)   # copy of page 4 -> page 9
    dd.copy_pages(cfg, pool, None, _dev(np.array([4], np.int32), cuda), _dev(np.array([9], np.int32), cuda))
    new_k = bf16_bits(rng.standard_normal((2, HKV, D)).astype(np.float32))
    new_v = bf16_bits(rng.standard_normal((2, HKV, D)).astype(np.float32))
    dd.append_kv_batch(cfg, pool, None, _dev(np.array([4, 9], np.int32), cuda),
                       _dev(np.array([6, 6], np.int32), cuda), _bf16_dev(new_k, cuda), _bf16_dev(new_v, cuda))
    torch.cuda.synchronize()
    # host copy of the same operations for the oracle
    ref_pool = bits.copy()
    ref_pool[9] = ref_pool[4]
    ref_pool[4, 0, :, 6], ref_pool[4, 1, :, 6] = new_k[0], new_v[0]
    ref_pool[9, 0, :, 6], ref_pool[9, 1, :, 6] = new_k[1], new_v[1]
    assert np.array_equal(pool.view(torch.int16).cpu().numpy().view(np.uint16), ref_pool)
    indptr = np.array([0, 5, 10], np.int32)
    ids = np.concatenate([parent, child])
    ntok = np.array([71, 71], np.int32)
    q = bf16_bits(rng.standard_normal((2, Hq, D)).astype(np.float32))
    plan = dd.CascadePlan(cfg, indptr, ids, ntok)
    assert plan.info().num_nodes == 3                 # shared pages 0-3, two private tails
    out, _ = dd.cascade_decode(cfg, plan, _bf16_dev(q, cuda), pool)
    ref, _ = oracle.decode_batch(bits_to_f32(q), ref_pool, indptr, ids, ntok, HKV)
    assert_close(out.float().cpu().numpy(), bits_to_f32(bf16_bits(ref)), what="fork+CoW+append")
