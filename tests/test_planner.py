"""Host-side cascade planner (C++ in libdendrite_b200.so), no GPU needed."""
import numpy as np
import pytest

import dendrite_b200 as dd
import oracle
from dendrite_b200 import workloads as wl
from tests.helpers import random_pool


def plan_for(tb, share=True, **kw):
    cfg = dd.make_config(tb.num_qo_heads, tb.num_kv_heads, tb.head_dim, tb.num_pages)
    return dd.CascadePlan(cfg, tb.indptr, tb.block_ids, tb.num_tokens, share_prefixes=share, **kw)


def query_paths(plan):
    """For each query: the concatenated pages of the nodes on its path."""
    n = plan.nodes()
    order = n["query_order"]
    pos = np.empty_like(order)
    pos[order] = np.arange(len(order))
    paths = []
    for q in range(plan.batch_size):
        p = pos[q]
        nodes = [i for i in range(len(n["parent"]))
                 if n["q_begin"][i] <= p < n["q_begin"][i] + n["num_q"][i]]
        nodes.sort(key=lambda i: n["page_offset"][i])
        # the nodes must form a parent chain
        for a, b in zip(nodes, nodes[1:]):
            assert n["parent"][b] == a
        pages, toks = [], 0
        for i in nodes:
            off, c = n["page_offset"][i], n["page_count"][i]
            pages += n["pages"][off:off + c].tolist()
            toks += n["num_tokens"][i]
        paths.append((pages, toks))
    return paths


def test_mcts_config_structure():
    tb = wl.mcts_llama3_8b()
    plan = plan_for(tb)
    info = plan.info()
    assert tb.batch_size == 512
    assert info.num_nodes == 1 + 8 + 32 + 128 + 512
    assert info.max_depth == 5
    assert info.kv_tokens == tb.unique_tokens
    assert info.kv_tokens_flat == int(tb.num_tokens.sum())
    n = plan.nodes()
    root = int(np.argmax(n["num_q"]))
    assert n["num_q"][root] == 512 and n["num_tokens"][root] == 8192 and n["parent"][root] == -1


@pytest.mark.parametrize("seed", range(6))
def test_paths_reconstruct_block_tables(seed):
    tb = wl.small_tree(seed, levels=((3, 16, 64), (2, 16, 32)), leaves_per_node=2, suffix=(1, 50))
    plan = plan_for(tb)
    for q, (pages, toks) in enumerate(query_paths(plan)):
        used = -(-int(tb.num_tokens[q]) // 16)
        assert pages == tb.block_ids[tb.indptr[q]:tb.indptr[q] + used].tolist()
        assert toks == tb.num_tokens[q]
    order = plan.nodes()["query_order"]
    assert sorted(order.tolist()) == list(range(tb.batch_size))


def test_flat_plan_has_one_node_per_query():
    tb = wl.small_tree(3)
    plan = plan_for(tb, share=False)
    info = plan.info()
    assert info.num_nodes == tb.batch_size
    assert info.kv_tokens == info.kv_tokens_flat == int(tb.num_tokens.sum())


def test_shared_partial_last_page_and_prefix_tables():
    # q0 and q1 share a partial last page (same id, same count); q2 is a prefix
    # of q3; q4 is empty; q5 uses the same page id as q0's last page but with a
    # different count (no sharing allowed).
    cfg = dd.make_config(4, 2, 64, 10)
    tables = [[0, 1, 2], [0, 1, 2], [0, 3], [0, 3, 4], [], [0, 1, 2]]
    ntok = [40, 40, 32, 33, 0, 35]
    indptr = np.cumsum([0] + [len(t) for t in tables]).astype(np.int32)
    ids = np.array([b for t in tables for b in t], dtype=np.uint32)
    plan = dd.CascadePlan(cfg, indptr, ids, np.array(ntok, dtype=np.int32))
    info = plan.info()
    # nodes: [0] shared by q0,q1,q2,q3,q5; [1] by q0,q1,q5; [2 (8 tok)] q0,q1;
    # [2 (3 tok)] q5; [3] q2,q3; [4] q3
    assert info.num_nodes == 6
    assert info.kv_tokens == 16 + 16 + 8 + 3 + 16 + 1
    paths = query_paths(plan)
    assert paths[4] == ([], 0)
    assert paths[0][0] == [0, 1, 2] and paths[5][0] == [0, 1, 2]


def test_tables_longer_than_num_tokens_use_first_pages():
    cfg = dd.make_config(4, 2, 64, 8)
    plan = dd.CascadePlan(cfg, np.array([0, 4], np.int32), np.array([5, 6, 7, 1], np.uint32),
                          np.array([17], np.int32))
    assert query_paths(plan)[0] == ([5, 6], 17)


def test_invalid_block_id_rejected():
    cfg = dd.make_config(4, 2, 64, 8)
    with pytest.raises(dd.InvalidArgument, match="invalid block id: 8"):
        dd.CascadePlan(cfg, np.array([0, 2], np.int32), np.array([1, 8], np.uint32),
                       np.array([20], np.int32))


def test_num_tokens_beyond_table_rejected():
    cfg = dd.make_config(4, 2, 64, 8)
    with pytest.raises(dd.InvalidArgument):
        dd.CascadePlan(cfg, np.array([0, 1], np.int32), np.array([1], np.uint32),
                       np.array([17], np.int32))


def test_chunking_splits_long_single_query_nodes():
    cfg = dd.make_config(8, 8, 128, 4096)
    ids = np.arange(4096, dtype=np.uint32)
    plan = dd.CascadePlan(cfg, np.array([0, 4096], np.int32), ids, np.array([65536], np.int32))
    info = plan.info()
    assert info.num_nodes == 1
    assert info.num_items >= 8 * 64  # split-K chunks x KV heads


def _np_partial(q, K, V, scale):
    """Partial attention state (o, natural lse) of q [R, D] over K, V [T, D]."""
    s = (q.astype(np.float64) @ K.T.astype(np.float64)) * scale
    m = s.max(axis=1, keepdims=True)
    p = np.exp(s - m)
    l = p.sum(axis=1, keepdims=True)
    return (p @ V) / l, (m + np.log(l))[:, 0]


@pytest.mark.parametrize("seed", [0, 1])
def test_cascade_decomposition_equals_flat_reference(seed):
    """Per-node partial states merged along each path with
    merge_attention_outputs reproduce ReferenceBackend::decode_batch."""
    tb = wl.small_tree(seed, Hq=8, Hkv=2, D=64, levels=((2, 16, 48), (2, 16, 32)),
                       leaves_per_node=2, suffix=(1, 40))
    rng = np.random.default_rng(seed)
    pool = random_pool(rng, tb.num_pages, 2, 64)
    q = rng.standard_normal((tb.batch_size, 8, 64)).astype(np.float32)
    ref, ref_lse = oracle.decode_batch(q, pool, tb.indptr, tb.block_ids, tb.num_tokens, 2)
    plan = plan_for(tb)
    n = plan.nodes()
    order = n["query_order"]
    scale = float(np.float32(1) / np.sqrt(np.float32(64)))
    acc_o = np.zeros((tb.batch_size, 8, 64), np.float32)
    acc_l = np.full((tb.batch_size, 8), -np.inf, np.float32)
    for i in range(len(n["parent"])):
        off, c, ntk = n["page_offset"][i], n["page_count"][i], n["num_tokens"][i]
        pages = n["pages"][off:off + c]
        for qq in order[n["q_begin"][i]:n["q_begin"][i] + n["num_q"][i]]:
            for h in range(8):
                kvh = h % 2
                K = np.concatenate([pool[p, 0, kvh] for p in pages])[:ntk]
                V = np.concatenate([pool[p, 1, kvh] for p in pages])[:ntk]
                o, l = _np_partial(q[qq, h][None], K, V, scale)
                if np.isneginf(acc_l[qq, h]):
                    acc_o[qq, h], acc_l[qq, h] = o[0], l[0]
                else:
                    mo, ml = oracle.merge_states(acc_o[qq, h][None], acc_l[qq, h][None],
                                                 o.astype(np.float32), l.astype(np.float32))
                    acc_o[qq, h], acc_l[qq, h] = mo[0], ml[0]
    np.testing.assert_allclose(acc_o, ref, atol=2e-5)
    np.testing.assert_allclose(acc_l, ref_lse, atol=2e-5)


def test_rebuild_matches_fresh_plan():
    """dd_plan_rebuild (re-planning into a live plan) gives the same plan as
    dd_plan_create, across batches of different shapes, and an invalid batch
    leaves an empty plan."""
    import dendrite_b200 as dd
    from dendrite_b200 import workloads as wl

    trees = [wl.small_tree(s, Hq=8, Hkv=2, D=64, prefix=200 + 16 * s, leaves_per_node=2 + s % 3)
             for s in range(4)]
    P = max(t.num_pages for t in trees)
    cfg = dd.make_config(8, 2, 64, P)
    live = dd.CascadePlan(cfg, trees[0].indptr, trees[0].block_ids, trees[0].num_tokens)
    for t in trees + trees[::-1]:
        live.rebuild(t.indptr, t.block_ids, t.num_tokens)
        fresh = dd.CascadePlan(cfg, t.indptr, t.block_ids, t.num_tokens)
        a, b = live.info(), fresh.info()
        for f in ("batch_size", "num_nodes", "num_items", "max_depth", "kv_tokens", "workspace_bytes",
                  "device_bytes", "tc_row_tokens"):
            assert getattr(a, f) == getattr(b, f), f
        assert list(a.kv_tokens_by_kernel) == list(b.kv_tokens_by_kernel)
        na, nb = live.nodes(), fresh.nodes()
        for k in nb:
            assert np.array_equal(na[k], nb[k]), k
    bad = trees[0].block_ids.copy()
    bad[0] = P + 5
    with pytest.raises(dd.InvalidArgument):
        live.rebuild(trees[0].indptr, bad, trees[0].num_tokens)
    assert live.info().batch_size == 0 and live.info().num_items == 0


def test_tcgen05_schedule_sizes():
    """The tcgen05 work items go onto one CTA per SM at most (or the CTAs the
    tc_sms option asks for); tc_sms = -1 keeps one CTA per item; the
    makespan-aware split keeps config 5a's 32768-token roots whole."""
    tb = wl.mcts_llama3_8b(0xD3D1)
    cfg = dd.make_config(32, 8, 128, tb.num_pages)
    auto = dd.CascadePlan(cfg, tb.indptr, tb.block_ids, tb.num_tokens).info()
    per_item = dd.CascadePlan(cfg, tb.indptr, tb.block_ids, tb.num_tokens, tc_sms=-1).info()
    fixed = dd.CascadePlan(cfg, tb.indptr, tb.block_ids, tb.num_tokens, tc_sms=60).info()
    assert auto.tc_ctas == 148
    assert fixed.tc_ctas == 60
    assert per_item.tc_ctas > 148  # one CTA per item, more items than SMs
    forest = wl.llama3_70b_forest(num_trees=8, seed=1)
    fcfg = dd.make_config(64, 8, 128, forest.num_pages)
    f_auto = dd.CascadePlan(fcfg, forest.indptr, forest.block_ids, forest.num_tokens).info()
    f_item = dd.CascadePlan(fcfg, forest.indptr, forest.block_ids, forest.num_tokens, tc_sms=-1).info()
    # 8 trees x 2 row tiles x 8 KV heads = 128 unsplit root items; the older
    # rule cut them further, the schedule keeps them whole.
    assert f_auto.workspace_bytes < f_item.workspace_bytes
