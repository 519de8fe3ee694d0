"""dd_plan_advance: one decode step in place (every leaf grows by a token,
some into a new block) gives the same plan as re-planning the grown block
tables from scratch; shared last pages fall back to re-planning."""
import numpy as np
import pytest

import dendrite_b200 as dd
from dendrite_b200 import workloads as wl


def _grow(tables, ntok, new_ids):
    """Host bookkeeping of one decode step: +1 token per query, a new block
    when the last one is full. Returns tokens_added, new_block."""
    added = np.ones(len(ntok), np.int32)
    nb = np.zeros(len(ntok), np.uint32)
    for b in range(len(ntok)):
        if ntok[b] % 16 == 0:
            nb[b] = next(new_ids)
            tables[b].append(int(nb[b]))
        ntok[b] += 1
    return added, nb


def _node_set(plan):
    n = plan.nodes()
    return sorted((int(n["num_q"][i]), int(n["num_tokens"][i]),
                   tuple(n["pages"][n["page_offset"][i]:n["page_offset"][i] + n["page_count"][i]]))
                  for i in range(len(n["num_q"])))


@pytest.mark.parametrize("steps", [1, 20])
def test_advance_matches_fresh_plan(steps):
    tb = wl.small_tree(3, Hq=8, Hkv=2, D=128, prefix=64, levels=((2, 16, 48),),
                       leaves_per_node=3, suffix=(1, 40))
    extra = tb.batch_size * (steps // 16 + 2)
    cfg = dd.make_config(8, 2, 128, tb.num_pages + extra)
    tables = tb.tables()
    ntok = tb.num_tokens.copy()
    plan = dd.CascadePlan(cfg, tb.indptr, tb.block_ids, ntok)
    new_ids = iter(range(tb.num_pages, tb.num_pages + extra))
    for _ in range(steps):
        added, nb = _grow(tables, ntok, new_ids)
        assert plan.advance(added, nb)
        indptr = np.cumsum([0] + [len(t) for t in tables]).astype(np.int32)
        fresh = dd.CascadePlan(cfg, indptr, np.concatenate(tables).astype(np.uint32), ntok)
        assert _node_set(plan) == _node_set(fresh)
        assert plan.info().kv_tokens == fresh.info().kv_tokens
        assert plan.info().kv_tokens_flat == fresh.info().kv_tokens_flat


def test_advance_falls_back_on_shared_pages():
    cfg = dd.make_config(8, 2, 128, 64)
    # two queries with the same table: their last page is shared
    plan = dd.CascadePlan(cfg, [0, 2, 4, 6], [0, 1, 0, 1, 2, 3], [20, 20, 30])
    before = _node_set(plan)
    assert not plan.advance([1, 0, 1], [0, 0, 0])
    assert _node_set(plan) == before
    # the unshared query alone can grow
    assert plan.advance([0, 0, 1], [0, 0, 0])


def test_advance_rejects_bad_input():
    cfg = dd.make_config(8, 2, 128, 64)
    plan = dd.CascadePlan(cfg, [0, 1], [0], [16])
    with pytest.raises(dd.InvalidArgument):
        plan.advance([2])
    with pytest.raises(dd.InvalidArgument):
        plan.advance([1], [99])          # block id >= num_pages
    pf = dd.CascadePlan.prefill(cfg, [0, 1], [0], [0], [5])
    assert not pf.advance([1] * 5, [0] * 5)


def test_advance_without_tokens_keeps_the_plan():
    tb = wl.small_tree(5, Hq=8, Hkv=2, D=128)
    cfg = dd.make_config(8, 2, 128, tb.num_pages)
    plan = dd.CascadePlan(cfg, tb.indptr, tb.block_ids, tb.num_tokens)
    before = (_node_set(plan), plan.info().kv_tokens)
    assert plan.advance(np.zeros(tb.batch_size, np.int32))
    assert (_node_set(plan), plan.info().kv_tokens) == before


def test_advance_refuses_flat_plans():
    cfg = dd.make_config(8, 2, 128, 64)
    plan = dd.CascadePlan(cfg, [0, 2, 4], [0, 1, 2, 3], [20, 30], share_prefixes=False)
    assert not plan.advance([1, 1], [5, 6])
