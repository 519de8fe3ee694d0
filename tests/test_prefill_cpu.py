"""Causal prefill on the CPU: the oracle's restatement of
ReferenceBackend::prefill (crates/dendrite-core/src/attention/backend.rs:
163-204) against an independent float64 computation, its equality with the
decode restatement over nested token counts (the form the GPU prefill plan
computes), and the structure of dd_plan_create_prefill plans."""
import numpy as np
import pytest

import dendrite_b200 as dd
import oracle


def _dense_causal_f64(q, k, v):
    Hq, S, D = q.shape
    Hkv = k.shape[0]
    out = np.zeros((Hq, S, D))
    for h in range(Hq):
        kh, vh = k[h % Hkv].astype(np.float64), v[h % Hkv].astype(np.float64)
        s = q[h].astype(np.float64) @ kh.T / np.sqrt(D)
        s[np.triu_indices(S, 1)] = -np.inf
        p = np.exp(s - s.max(axis=1, keepdims=True))
        out[h] = (p / p.sum(axis=1, keepdims=True)) @ vh
    return out


@pytest.mark.parametrize("S,Hq,Hkv,D", [(1, 4, 4, 64), (23, 8, 2, 64), (40, 32, 4, 128)])
def test_oracle_prefill_vs_float64(S, Hq, Hkv, D):
    rng = np.random.default_rng(S * 131 + Hq)
    q = rng.standard_normal((Hq, S, D)).astype(np.float32)
    k = rng.standard_normal((Hkv, S, D)).astype(np.float32)
    v = rng.standard_normal((Hkv, S, D)).astype(np.float32)
    got = oracle.prefill(q, k, v)
    want = _dense_causal_f64(q, k, v)
    assert np.abs(got - want).max() < 2e-5


def test_prefill_equals_decode_over_prefixes():
    """Token i of a dense causal prefill = a decode of query i over the first
    i + 1 tokens of the same pages."""
    rng = np.random.default_rng(5)
    S, Hq, Hkv, D = 37, 8, 2, 64
    q = rng.standard_normal((Hq, S, D)).astype(np.float32)
    k = rng.standard_normal((Hkv, S, D)).astype(np.float32)
    v = rng.standard_normal((Hkv, S, D)).astype(np.float32)
    pages = (S + 15) // 16
    ids = rng.permutation(8)[:pages].astype(np.uint32)
    pool = np.zeros((8, 2, Hkv, 16, D), np.float32)
    for t in range(S):
        pool[ids[t // 16], 0, :, t % 16] = k[:, t]
        pool[ids[t // 16], 1, :, t % 16] = v[:, t]
    indptr = np.arange(S + 1, dtype=np.int32) * pages
    dec, _ = oracle.decode_batch(q.transpose(1, 0, 2), pool, indptr, np.tile(ids, S),
                                 np.arange(1, S + 1, dtype=np.int32), Hkv)
    ref = oracle.prefill(q, k, v)
    assert np.abs(dec.transpose(1, 0, 2) - ref).max() < 1e-5


def test_prefill_plan_structure():
    cfg = dd.make_config(8, 2, 128, 64)
    # sequence 0: 30 prefix + 37 new tokens (5 pages); sequence 1: 50 new (4 pages)
    p = dd.CascadePlan.prefill(cfg, [0, 5, 9], np.arange(9), [30, 0], [37, 50])
    info = p.info()
    assert info.batch_size == 87 and info.max_depth == 2
    n = p.nodes()
    # the full prefix page of sequence 0, then a causal suffix per sequence
    # starting at the page holding its first new token (page 1 of sequence 0)
    assert sorted(zip(n["num_q"], n["num_tokens"], n["page_count"])) == [(37, 16, 1), (37, 51, 4), (50, 50, 4)]
    assert sorted(n["query_order"]) == list(range(87))
    # tokens each query sees: prefix + i + 1, summed
    assert info.kv_tokens_flat == sum(30 + i + 1 for i in range(37)) + sum(i + 1 for i in range(50))


def test_prefill_plan_shares_prefix_pages():
    """Branches over the same prefix pages: the shared full pages are one node
    read for every new token below it."""
    cfg = dd.make_config(8, 2, 128, 64)
    shared = [0, 1, 2]
    tables = [shared + [10 + 2 * b, 11 + 2 * b] for b in range(4)]
    indptr = np.arange(5) * 5
    p = dd.CascadePlan.prefill(cfg, indptr, np.concatenate(tables), [48] * 4, [20, 5, 30, 8])
    n = p.nodes()
    root = int(np.argmax(n["page_count"] * (n["parent"] < 0)))
    assert n["page_count"][root] == 3 and n["num_q"][root] == 63
    assert sorted(n["num_q"][n["parent"] == root]) == [5, 8, 20, 30]


def test_prefill_plan_rejects_bad_input():
    cfg = dd.make_config(8, 2, 128, 64)
    with pytest.raises(dd.InvalidArgument):
        dd.CascadePlan.prefill(cfg, [0, 2], [0, 1], [20], [20])   # 40 tokens > 2 pages
    with pytest.raises(dd.InvalidArgument):
        dd.CascadePlan.prefill(cfg, [0, 1], [99], [0], [5])       # block id >= num_pages
    with pytest.raises(dd.InvalidArgument):
        dd.CascadePlan.prefill(cfg, [0, 1], [0], [-1], [5])


def test_prefill_plan_skips_sequences_without_new_tokens():
    cfg = dd.make_config(8, 2, 128, 64)
    p = dd.CascadePlan.prefill(cfg, [0, 2, 4, 6], np.arange(6), [20, 17, 5], [0, 9, 0])
    info = p.info()
    assert info.batch_size == 9
    n = p.nodes()
    assert int(n["num_q"].max()) == 9 and sorted(n["query_order"]) == list(range(9))
    empty = dd.CascadePlan.prefill(cfg, [0, 1], [0], [10], [0])
    assert empty.info().batch_size == 0 and empty.info().num_items == 0
