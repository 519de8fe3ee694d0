"""Decode with a plan advanced in place (dd_plan_advance) over 20 steps of
leaf growth, against the oracle on the grown block tables."""
import numpy as np
import pytest
import torch

import dendrite_b200 as dd
import oracle
from dendrite_b200 import workloads as wl
from tests.helpers import assert_close, bf16_bits, bits_to_f32, random_pool
from tests.test_plan_advance import _grow

pytestmark = pytest.mark.gpu


def test_decode_after_advance(cuda):
    tb = wl.small_tree(8, Hq=32, Hkv=8, D=128, prefix=512, levels=((4, 64, 256),),
                       leaves_per_node=4, suffix=(1, 60))
    steps = 20
    extra = tb.batch_size * (steps // 16 + 2)
    P = tb.num_pages + extra
    rng = np.random.default_rng(8)
    pool = bf16_bits(random_pool(rng, P, 8, 128))
    q = bf16_bits(rng.standard_normal((tb.batch_size, 32, 128)).astype(np.float32))
    cfg = dd.make_config(32, 8, 128, P)
    tables, ntok = tb.tables(), tb.num_tokens.copy()
    plan = dd.CascadePlan(cfg, tb.indptr, tb.block_ids, ntok)
    new_ids = iter(range(tb.num_pages, P))
    for _ in range(steps):
        assert plan.advance(*_grow(tables, ntok, new_ids))
    plan.upload(cuda)
    dev = lambda b: torch.from_numpy(b.view(np.int16).copy()).view(torch.bfloat16).to(cuda)  # noqa: E731
    out, _ = dd.cascade_decode(cfg, plan, dev(q), dev(pool))
    torch.cuda.synchronize()
    indptr = np.cumsum([0] + [len(t) for t in tables]).astype(np.int32)
    ref, _ = oracle.decode_batch(bits_to_f32(q), pool, indptr, np.concatenate(tables).astype(np.uint32),
                                 ntok, 8)
    assert_close(out.float().cpu().numpy(), bits_to_f32(bf16_bits(ref)), what="after advance")


def test_advance_forgets_the_upload(cuda):
    """An advance repacks the plan image (new offsets, possibly larger), so a
    decode before the next upload must be refused, not read the old image."""
    tb = wl.small_tree(9, Hq=8, Hkv=2, D=128, prefix=64, levels=((2, 16, 48),),
                       leaves_per_node=2, suffix=(1, 40))
    P = tb.num_pages + 2 * tb.batch_size
    cfg = dd.make_config(8, 2, 128, P)
    tables, ntok = tb.tables(), tb.num_tokens.copy()
    plan = dd.CascadePlan(cfg, tb.indptr, tb.block_ids, ntok)
    plan.upload(cuda)
    assert plan.advance(*_grow(tables, ntok, iter(range(tb.num_pages, P))))
    q = torch.zeros(tb.batch_size, 8, 128, dtype=torch.bfloat16, device=cuda)
    pool = torch.zeros(P, 2, 2, 16, 128, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(dd.InvalidArgument, match="not uploaded"):
        dd.cascade_decode(cfg, plan, q, pool)
    plan.upload(cuda)
    dd.cascade_decode(cfg, plan, q, pool)
    torch.cuda.synchronize()
